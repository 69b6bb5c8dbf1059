"""GPU parity at the production gate setting and on a single 720p stream and on a shard of a 64-stream job.

* gate band: on normalised fp16 camera frames at SarbonVideo's threshold
  (tau = 8/255 * 255 / mean(STD), video.py:63-64) the engine's change mask is compared
  with the reference's own expression evaluated by torch on the same GPU,
  ``(frames - img).abs().view(n,hb,b,wb,b,3).sum((2,4,5), dtype=float32) > tau*b*b*3``
  (fused_engine.py:142-144), with ``img`` read from the engine's cache before each step.
  The kernel decides by the exact sum; the two can only disagree for a block whose exact
  sum lies inside the fp32 rounding band of a 3072-term sum around the threshold.  Every
  disagreement is reported with its distance from the threshold and must lie in the band.
* one 1280x720 stream padded to 1280x736 (920 blocks): change masks, dilated
  masks, block lists and the image cache bit-exact against the oracle over a sequence;
  every layer elementwise (1e-2 rel / 1e-3 abs) against the oracle's conv of the engine's
  own input caches.
* one shard of the 64-stream 1280x736 job (streams 16..31, the second of four
  GPUs) run as its own 16-stream engine equals the matching slice of one 64-stream engine
  bit for bit: caches, change masks, dilated masks and block lists.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import sparse_oracle as so

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False


def production_tau():
    """SarbonVideo(tau=8/255) converted to the engine's normalised units (video.py:63-64)."""
    from sarbon_b200 import scenes
    return (8 / 255) * 255 / float(scenes.STD.mean())


def padded_720p(src, pad_to=736):
    """Next 1280x720 frames of `src`, zero-padded at the bottom to the engine height."""
    u8 = src.next()
    return F.pad(u8, (0, 0, 0, 0, 0, pad_to - u8.shape[1]))


def oracle_engine(net, n, h, w, tau, refresh=0):
    nodes = []
    for nd in net.program()[0]:
        d = {"kind": nd.kind, "src": list(nd.src), "dst": nd.dst, "stride": nd.stride, "radius": nd.radius,
             "act": bool(nd.act)}
        if nd.kind == "conv":
            d["w"] = nd.conv.weight.detach().float().cpu().numpy()
            d["b"] = nd.conv.bias.detach().float().cpu().numpy()
            d["conv_stride"] = nd.conv.stride[0]
        nodes.append(d)
    return so.OracleEngine(so.fuse_program(nodes), n, h, w, dtype=np.float16, tau=tau, refresh=refresh)


# fp32 rounding band of the gate: a recursive fp32 sum of 3072 non-negative terms is within
# 3071 * 2^-24 (relative) of the exact sum in any order
BAND = 3 * 32 * 32 * 2.0 ** -24


@pytest.mark.parametrize("n,h,w,rects,steps", [(16, 1088, 1920, 15, 32), (1, 736, 1280, 7, 64)],
                         ids=["16x1080p", "1x736p"])
def test_gate_matches_torch_fp32_sum_at_production_tau(n, h, w, rects, steps):
    from sarbon_b200 import FusedSparseEngine, LocalBackbone, scenes
    torch.manual_seed(5)
    b = 32
    hb, wb = h // b, w // b
    tau = production_tau()
    thr32 = float(np.float32(tau * b * b * 3))
    eng = FusedSparseEngine(LocalBackbone().cuda().eval(), n, h, w, dtype=torch.float16, tau=tau)
    src = scenes.Streams(n, h, w, seed=31, n_rects=rects, device="cuda")
    eng.reset(scenes.normalise(src.next()))
    decisions, changed, mismatches = 0, 0, []
    for i in range(steps):
        f = scenes.normalise(src.next())
        img = eng.cache["img"].clone()
        ref = (f - img).abs().view(n, hb, b, wb, b, 3).sum((2, 4, 5), dtype=torch.float32) > tau * b * b * 3
        mode, k = eng.step(f)
        assert mode in ("skip", "sparse"), mode
        got = eng.changed.clone()
        decisions += got.numel()
        changed += int(ref.sum())
        bad = (got != ref).nonzero().tolist()
        if bad:
            exact = (f.float() - img.float()).half().abs().double().view(n, hb, b, wb, b, 3).sum((2, 4, 5))
            for c, y, x in bad:
                rel = (float(exact[c, y, x]) - thr32) / thr32
                mismatches.append((i, c, y, x, bool(got[c, y, x]), rel))
    print(f"\ngate vs torch fp32 sum at tau={tau:.6f}: {decisions} block decisions, {changed} changed "
          f"({changed / decisions:.2%}), {len(mismatches)} mismatches {mismatches[:8]}")
    assert changed > 0
    # every disagreement must be a block whose exact sum sits inside the fp32 band
    assert all(abs(m[-1]) <= BAND for m in mismatches), mismatches


def test_config2_720p_single_stream_vs_oracle():
    from sarbon_b200 import FusedSparseEngine, LocalBackbone, scenes
    torch.manual_seed(6)
    n, h, w = 1, 736, 1280
    tau = production_tau()
    net = LocalBackbone().eval()
    eng = FusedSparseEngine(net.cuda(), n, h, w, dtype=torch.float16, tau=tau, refresh=16)
    assert eng.n_blocks == 920
    ora = oracle_engine(net, n, h, w, tau, refresh=16)
    src = scenes.Streams(n, 720, w, seed=41, n_rects=7)
    f = scenes.normalise(padded_720p(src))
    eng.reset(f.cuda())
    ora.reset(f.numpy())
    seen = set()
    for i in range(10):
        f = scenes.normalise(padded_720p(src))
        if i == 4:
            extra = torch.zeros(n, h // 32, w // 32, dtype=torch.bool)
            extra[0, 22, 39] = extra[0, 0, 0] = True  # corner blocks, padded rows included
            eng.set_extra(extra.cuda())
            ora.extra = extra.numpy()
        elif i == 5:
            eng.set_extra(torch.zeros(n, h // 32, w // 32, dtype=torch.bool, device="cuda"))
            ora.extra = np.zeros_like(ora.extra)
        got = eng.step(f.cuda())
        exp = ora.step(f.numpy())
        assert got == exp, (i, got, exp)
        seen.add(got[0])
        np.testing.assert_array_equal(eng.changed.cpu().numpy(), ora.changed, f"step {i} changed")
        for d in eng.ds:
            np.testing.assert_array_equal(eng.masks[d].cpu().numpy(), ora.masks[d], f"step {i} mask {d}")
            if got[0] == "sparse":
                lst = np.stack([x.cpu().numpy() for x in eng.block_lists(d)])
                np.testing.assert_array_equal(lst, np.stack(so.block_lists(ora.masks[d])), f"step {i} list {d}")
        np.testing.assert_array_equal(eng.cache["img"].cpu().numpy(), ora.cache["img"], f"step {i} img")
    assert "sparse" in seen
    # every layer from the engine's own inputs: elementwise fp16 tolerance
    cache = {name: v.float().cpu().numpy() for name, v in eng.cache.items()}
    for l in ora.layers:
        ref = so.conv_dense(cache[l.src], l.w, l.bias, l.stride, l.act,
                            None if l.res is None else cache[l.res], np.float32)
        err = np.abs(cache[l.dst] - ref)
        bad = err > 1e-3 + 1e-2 * np.abs(ref)
        assert not bad.any(), (l.dst, int(bad.sum()), float(err.max()))


def test_config4_shard_equals_slice_of_64_stream_engine():
    from sarbon_b200 import FusedSparseEngine, LocalBackbone, scenes
    from sarbon_b200.multi import shard_streams
    torch.manual_seed(7)
    total, world, rank, h, w = 64, 4, 1, 736, 1280
    sh = shard_streams(total, world, rank)
    assert (sh.start, sh.stop) == (16, 32)
    sl = slice(sh.start, sh.stop)
    tau = production_tau()
    net = LocalBackbone().cuda().eval()
    full = FusedSparseEngine(net, total, h, w, dtype=torch.float16, tau=tau)
    part = FusedSparseEngine(net, sh.stop - sh.start, h, w, dtype=torch.float16, tau=tau)
    src = scenes.Streams(total, 720, w, seed=51, n_rects=7, device="cuda")
    f = scenes.normalise(padded_720p(src))
    full.reset(f)
    part.reset(f[sl].contiguous())
    for i in range(5):
        f = scenes.normalise(padded_720p(src))
        mf, kf = full.step(f)
        mp, kp = part.step(f[sl].contiguous())
        assert mf == mp == "sparse", (mf, mp)
        assert torch.equal(full.changed[sl], part.changed), i
        for d in full.ds:
            assert torch.equal(full.masks[d][sl], part.masks[d]), (i, d)
            cam, by, bx = full.block_lists(d)
            sel = (cam >= sh.start) & (cam < sh.stop)
            pc, pby, pbx = part.block_lists(d)
            assert torch.equal(cam[sel] - sh.start, pc) and torch.equal(by[sel], pby) and torch.equal(bx[sel], pbx)
        assert kp == int(part.masks[part.ds[-1]].sum())
    for name in full.cache:
        assert torch.equal(full.cache[name][sl], part.cache[name]), name
