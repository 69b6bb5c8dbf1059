"""GPU parity of the B200 engine (through the C ABI via the drop-in FusedSparseEngine).

* golden: the reference's own outputs (tests/golden) -- masks, modes, counts and block
  lists bit-exact; p4/p8 caches within the dtype tolerance;
* oracle: the CPU restatement on fresh seeded inputs;
* the reference test scenario (tests/test_fused_engine.py:24-79 of the reference):
  sparse == dense forward over chained frames, skip, dense replay, hysteresis.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from golden_io import CASES, OUTPUT_ULPS, assert_close, load
from oracle import sparse_oracle as so

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False


def net_from_nodes(nodes, dtype=torch.float32):
    from sarbon_b200 import LocalBackbone
    net = LocalBackbone()
    convs = [n.conv for n in net.program()[0] if n.kind == "conv"]
    ws = [(n["w"], n["b"]) for n in nodes if n["kind"] == "conv"]
    assert len(convs) == len(ws)
    with torch.no_grad():
        for c, (w, b) in zip(convs, ws):
            c.weight.copy_(torch.from_numpy(w))
            c.bias.copy_(torch.from_numpy(b))
    return net.eval()


def tdt(np_dtype):
    return torch.float16 if np_dtype == np.float16 else torch.float32


@pytest.mark.parametrize("name", CASES)
def test_golden_parity(name):
    from sarbon_b200 import FusedSparseEngine
    case = load(name)
    m = case["meta"]
    dt = tdt(case["dtype"])
    net = net_from_nodes(case["nodes"])
    eng = FusedSparseEngine(net, m["n_cams"], m["h"], m["w"], block=m["block"], dtype=dt, tau=m["tau"],
                            refresh=m["refresh"])
    assert eng.ds == m["ds"] and eng.buckets == m["buckets"]
    eng.reset(torch.from_numpy(case["frames0"]).cuda().to(dt))
    assert_close(eng.cache["t7"].float().cpu(), case["reset"]["t7"], case["dtype"], f"{name} reset t7", OUTPUT_ULPS["t7"])
    assert_close(eng.cache["t14"].float().cpu(), case["reset"]["t14"], case["dtype"], f"{name} reset t14", OUTPUT_ULPS["t14"])
    for i, st in enumerate(case["steps"]):
        eng.set_extra(torch.from_numpy(st["extra"]).cuda())
        mode, k = eng.step(torch.from_numpy(st["frames"]).cuda().to(dt))
        assert (mode, k) == (st["mode"], st["k"]), f"{name} step {i}"
        np.testing.assert_array_equal(eng.changed.cpu().numpy(), st["changed"], f"{name} step {i} changed")
        for d in eng.ds:
            np.testing.assert_array_equal(eng.masks[d].cpu().numpy(), st["masks"][d], f"{name} step {i} mask {d}")
            if mode == "sparse":
                got = np.stack([x.cpu().numpy() for x in eng.block_lists(d)])
                np.testing.assert_array_equal(got, st["lists"][d][:, :got.shape[1]], f"{name} step {i} list {d}")
                assert got.shape[1] == st["masks"][d].sum()
        assert_close(eng.cache["t7"].float().cpu(), st["t7"], case["dtype"], f"{name} step {i} t7", OUTPUT_ULPS["t7"])
        assert_close(eng.cache["t14"].float().cpu(), st["t14"], case["dtype"], f"{name} step {i} t14", OUTPUT_ULPS["t14"])


def rel_err(engine, net, frames):
    """max |engine - dense fp32| / max |dense| over p4 and p8 (the reference test's metric)."""
    with torch.no_grad():
        ref = net.float()(frames.float().permute(0, 3, 1, 2).contiguous())
    return max(((o.float() - r).abs().max() / r.abs().max()).item() for o, r in zip(engine.outputs_nchw(), ref))


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.float16, 1e-2)])
@pytest.mark.parametrize("block", [32, 64])
def test_reference_scenario(dtype, tol, block):
    """The reference's own engine test (tests/test_fused_engine.py:24-79), same steps."""
    from sarbon_b200 import FusedSparseEngine, LocalBackbone
    n_cams, h, w = 3, 256, 384
    torch.manual_seed(0)
    net = LocalBackbone().cuda().eval()
    eng = FusedSparseEngine(net, n_cams, h, w, block=block, dtype=dtype)
    frames = torch.rand(n_cams, h, w, 3, device="cuda", dtype=dtype)
    eng.reset(frames)
    errs = {"reset": rel_err(eng, net, frames)}
    for i in range(4):
        frames = frames.clone()
        cam = i % n_cams
        y, x = 40 * i + 7, 60 * i + 13
        frames[cam, y:y + 37, x:x + 51] = torch.rand(3, device="cuda", dtype=dtype)
        if i == 3:
            frames[:, :, -20:] = 0.5
        mode, k = eng.step(frames)
        assert mode == "sparse", mode
        errs[f"step{i}"] = rel_err(eng, net, frames)
    mode, k = eng.step(frames)
    assert mode == "skip" and k == 0
    eng.frames.copy_(torch.rand_like(frames))
    eng.dense_graph.replay()
    errs["dense"] = rel_err(eng, net, eng.frames)
    frames = eng.frames.clone()
    for i in range(2):
        frames[i, 100:140, 200:260] = 0.25 * (i + 1)
        mode, k = eng.step(frames)
        assert mode == "sparse", mode
        errs[f"after-dense{i}"] = rel_err(eng, net, frames)
    budget, eng.fallback = eng.fallback, 0
    seen = []
    for i in range(eng.dense_check_every + 1):
        frames[i % n_cams, 10 * i:10 * i + 30, 50:90] = 0.1 * i
        seen.append(eng.step(frames)[0])
    assert seen == ["dense"] * len(seen), seen
    eng.fallback = budget
    for i in range(eng.dense_check_every + 1):
        frames[0, 150:170, 20 * i:20 * i + 25] = 0.9
        mode, _ = eng.step(frames)
    assert mode == "sparse", mode
    errs["after-hysteresis"] = rel_err(eng, net, frames)
    assert max(errs.values()) < tol, errs
    st = eng.stats
    assert st["skip"] == 1 and st["dense"] >= eng.dense_check_every + 1


def _oracle_engine(net, n, h, w, block, dtype, tau, refresh=0):
    nodes = []
    for nd in net.program()[0]:
        d = {"kind": nd.kind, "src": list(nd.src), "dst": nd.dst, "stride": nd.stride, "radius": nd.radius,
             "act": bool(nd.act)}
        if nd.kind == "conv":
            d["w"] = nd.conv.weight.detach().float().cpu().numpy()
            d["b"] = nd.conv.bias.detach().float().cpu().numpy()
            d["conv_stride"] = nd.conv.stride[0]
        nodes.append(d)
    return so.OracleEngine(so.fuse_program(nodes), n, h, w, block=block, dtype=dtype, tau=tau, refresh=refresh)


def test_gate_and_lists_vs_oracle_normalised_stream():
    """Seeded synthetic camera streams, normalised fp16 input, tau = 8 grey levels:
    change masks, dilated masks and block lists bit-exact against the oracle; caches
    within fp16 tolerance.  Refresh and extra are exercised."""
    from sarbon_b200 import FusedSparseEngine, LocalBackbone, scenes
    torch.manual_seed(1)
    n, h, w = 3, 256, 448
    net = LocalBackbone().eval()
    tau = 8 / float(scenes.STD.mean())
    eng = FusedSparseEngine(net.cuda(), n, h, w, dtype=torch.float16, tau=tau, refresh=7)
    ora = _oracle_engine(net, n, h, w, 32, np.float16, tau, refresh=7)
    src = scenes.Streams(n, h, w, seed=5, n_rects=3)
    f = scenes.normalise(src.next())
    eng.reset(f.cuda())
    ora.reset(f.numpy())
    modes = set()
    for i in range(8):
        f = scenes.normalise(src.next())
        extra = torch.zeros(n, h // 32, w // 32, dtype=torch.bool)
        if i == 3:
            extra[1, 2, 5] = True
        eng.set_extra(extra.cuda())
        ora.extra = extra.numpy()
        got = eng.step(f.cuda())
        exp = ora.step(f.numpy())
        assert got == exp, (i, got, exp)
        modes.add(got[0])
        np.testing.assert_array_equal(eng.changed.cpu().numpy(), ora.changed)
        for d in eng.ds:
            np.testing.assert_array_equal(eng.masks[d].cpu().numpy(), ora.masks[d])
            if got[0] == "sparse":
                lst = np.stack([x.cpu().numpy() for x in eng.block_lists(d)])
                ref = np.stack(so.block_lists(ora.masks[d]))
                np.testing.assert_array_equal(lst, ref)
        np.testing.assert_array_equal(eng.cache["img"].cpu().numpy(), ora.cache["img"])
        for o in ("t7", "t14"):
            assert_close(eng.cache[o].float().cpu(), ora.cache[o].astype(np.float32), np.float16, f"{i} {o}",
                         OUTPUT_ULPS[o])
    assert "sparse" in modes


def test_uint8_fused_prep_matches_fp16_path():
    """sb_step_u8 (BGR uint8, normalisation fused into the gate) == sb_step on the frames
    SarbonVideo._prep would produce: same masks, same image cache bits, same features."""
    from sarbon_b200 import FusedSparseEngine, LocalBackbone, scenes
    n, h, w = 2, 192, 320
    torch.manual_seed(2)
    net = LocalBackbone().cuda().eval()
    tau = 8 / float(scenes.STD.mean())
    a = FusedSparseEngine(net, n, h, w, dtype=torch.float16, tau=tau)
    b = FusedSparseEngine(net, n, h, w, dtype=torch.float16, tau=tau)
    src = scenes.Streams(n, h, w, seed=9, n_rects=2)
    rgb = src.next()
    a.reset(scenes.normalise(rgb).cuda())
    b.reset(scenes.normalise(rgb).cuda())
    for _ in range(4):
        rgb = src.next()
        bgr = rgb.flip(-1).contiguous().cuda()
        ma = a.step(scenes.normalise(rgb).cuda())
        mb = b.step_u8(bgr, scenes.MEAN, scenes.STD)
        assert ma == mb
        assert torch.equal(a.changed, b.changed)
        assert torch.equal(a.cache["img"], b.cache["img"])
        assert torch.equal(a.cache["t14"], b.cache["t14"])


def test_lists_many_chunks_vs_oracle():
    """Block lists over many look-back chunks (8 streams x 1080p = 16320 blocks):
    random extra masks of several densities, tau = inf so only `extra` fires."""
    from sarbon_b200 import FusedSparseEngine, LocalBackbone
    n, h, w = 8, 1088, 1920
    net = LocalBackbone().cuda().eval()
    eng = FusedSparseEngine(net, n, h, w, dtype=torch.float16, tau=float("inf"))
    frames = torch.zeros(n, h, w, 3, device="cuda", dtype=torch.float16)
    eng.reset(frames)
    rng = np.random.default_rng(0)
    for p in (0.0, 0.001, 0.01, 0.05, 0.3, 1.0):
        ext = rng.random((n, h // 32, w // 32)) < p
        eng.set_extra(torch.from_numpy(ext).cuda())
        mode, k = eng.step(frames)
        for d in eng.ds:
            md = so.dilate(ext, d)
            np.testing.assert_array_equal(eng.masks[d].cpu().numpy(), md)
            if mode == "sparse":
                lst = np.stack([x.cpu().numpy() for x in eng.block_lists(d)])
                np.testing.assert_array_equal(lst, np.stack(so.block_lists(md)))
        assert k == int(so.dilate(ext, eng.ds[-1]).sum())
        assert mode == ("skip" if k == 0 else "sparse")


def test_multistream_equals_single_streams():
    """Batching streams changes nothing per stream: the 3-stream engine's caches are
    bit-identical to three 1-stream engines (each tile's arithmetic is the same)."""
    from sarbon_b200 import FusedSparseEngine, LocalBackbone, scenes
    n, h, w = 3, 128, 256
    net = LocalBackbone().cuda().eval()
    big = FusedSparseEngine(net, n, h, w, dtype=torch.float16)
    singles = [FusedSparseEngine(net, 1, h, w, dtype=torch.float16) for _ in range(n)]
    src = scenes.Streams(n, h, w, seed=11, n_rects=2)
    f = scenes.normalise(src.next()).cuda()
    big.reset(f)
    for i, e in enumerate(singles):
        e.reset(f[i:i + 1])
    for _ in range(3):
        f = scenes.normalise(src.next()).cuda()
        big.step(f)
        for i, e in enumerate(singles):
            e.step(f[i:i + 1])
    for i, e in enumerate(singles):
        for o in ("t7", "t14"):
            assert torch.equal(big.cache[o][i], e.cache[o][0]), (i, o)


def test_calibrate_restores_caches_and_sets_crossover():
    """calibrate() (fused_engine.py:242-275): times every budget bucket against the dense
    pass, sets `fallback` to the last bucket before two slower-than-dense buckets in a row,
    and leaves the caches exactly as they were."""
    from sarbon_b200 import FusedSparseEngine, LocalBackbone, scenes
    torch.manual_seed(3)
    net = LocalBackbone().eval()
    eng = FusedSparseEngine(net, 2, 256, 384, dtype=torch.float16, tau=0.05)
    src = scenes.Streams(2, 256, 384, seed=4, n_rects=2, device="cuda")
    eng.reset(scenes.normalise(src.next()))
    eng.step(scenes.normalise(src.next()))
    before = {k: v.clone() for k, v in eng.cache.items()}
    table = eng.calibrate(reps=3)
    buckets = [b for b, _, _ in table]
    assert buckets == sorted(buckets) and len(buckets) >= 1
    assert set(buckets) <= {eng._bucket(x) for x in eng.buckets}
    assert all(ms > 0 and ratio > 0 for _, ms, ratio in table)
    assert eng.fallback == 0 or eng.fallback in buckets
    for k, v in eng.cache.items():
        assert torch.equal(v, before[k]), k
    # the engine still steps normally with the calibrated crossover
    mode, k = eng.step(scenes.normalise(src.next()))
    assert mode in ("skip", "sparse", "dense")


def test_step_phases_times_the_same_step():
    """step_phases (events only between the step's phases) computes exactly what step does and
    returns a positive time for every phase."""
    from sarbon_b200 import FusedSparseEngine, LocalBackbone, scenes
    n, h, w = 2, 256, 384
    torch.manual_seed(12)
    net = LocalBackbone().cuda().eval()
    tau = 8 / float(scenes.STD.mean())
    a = FusedSparseEngine(net, n, h, w, dtype=torch.float16, tau=tau)
    b = FusedSparseEngine(net, n, h, w, dtype=torch.float16, tau=tau)
    src = scenes.Streams(n, h, w, seed=13, n_rects=2, device="cuda")
    f = scenes.normalise(src.next())
    a.reset(f)
    b.reset(f)
    for _ in range(3):
        f = scenes.normalise(src.next())
        ma = a.step(f.clone())
        mode, k, ph = b.step_phases(f.clone())
        assert ma == (mode, k)
        assert set(ph) == {"gate", "lists", "copy", "conv", "finalize"} and all(v > 0 for v in ph.values())
        for name in a.cache:
            assert torch.equal(a.cache[name], b.cache[name]), name
