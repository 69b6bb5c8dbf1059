"""B200Detector (the detector after the stem on this library's kernels) against the reference.

The reference is its own ``SarbonDetector`` (sarbon/models/sarbon_det.py, installed under
baseline/_ref), built as ``build("s", 6, halo_zero=False)`` with non-trivial BatchNorm
statistics and affine parameters, randomised heads and sampling offsets, run as
``SarbonVideo._run_det`` runs it: ``det(None, p8=p8)`` under ``torch.autocast(float16)``
(sarbon/inference/video.py:116-118).  Inputs: 640x384 frames (p8 48x80)
and two images; 300 queries.

* DenseCore's three output levels against ``det.core(p8)``;
* the encoder's query selection against the reference's top-K (fraction of equal rows);
* with the reference's selected rows forced (top-K ties may order differently, so the
  decoder is compared on the same selection), the final boxes and class logits elementwise
  within |a - b| <= 1e-3 + 1e-2 |b|, and the identity embedding;
* the CUDA-graph replay equals the eager run bit for bit.
"""
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")


@pytest.fixture(scope="module")
def ref_pkg():
    if not (REF / "sarbon").is_dir():
        pytest.skip("the reference package is not installed under baseline/_ref")
    import sys
    sys.path.insert(0, str(REF))
    import sarbon.models.sarbon_det as sd
    yield sd
    sys.path.remove(str(REF))


def make_det(sd, seed=0):
    torch.manual_seed(seed)
    det = sd.build("s", 6, halo_zero=False)
    gen = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        for m in det.modules():
            if isinstance(m, torch.nn.BatchNorm2d):
                c = m.num_features
                m.running_mean.copy_(torch.rand(c, generator=gen) * 0.4 - 0.2)
                m.running_var.copy_(torch.rand(c, generator=gen) * 1.5 + 0.5)
                m.weight.copy_(torch.rand(c, generator=gen) + 0.5)
                m.bias.copy_(torch.rand(c, generator=gen) * 0.4 - 0.2)
            elif isinstance(m, torch.nn.Linear) and not m.weight.any():
                # zero-initialised heads, sampling offsets and attention logits
                m.weight.copy_(torch.randn(m.weight.shape, generator=gen) * 0.02)
    return det.cuda().eval()


def ref_forward(sd, det, p8):
    with torch.no_grad(), torch.autocast("cuda", torch.float16):
        feats = det.core(p8)
        out = det(None, p8=p8)
        # the query selection of sarbon_det.py:306-314, for the forced-top-K comparison
        shapes = [f.shape[-2:] for f in feats]
        memory = torch.cat([f.flatten(2).transpose(1, 2) for f in feats], 1)
        _, valid = det.anchors(shapes, memory.device, memory.dtype)
        enc = det.enc_proj(memory * valid.to(memory.dtype))
        top = det.enc_cls(enc).max(-1).values.masked_fill(~valid[..., 0], float("-inf")).topk(det.cfg.queries, 1).indices
    return feats, out, top


def close_frac(got, ref, rtol=1e-2, atol=1e-3):
    got, ref = got.float(), ref.float()
    bad = (got - ref).abs() > atol + rtol * ref.abs()
    return bad.float().mean().item(), (got - ref).abs().max().item()


@pytest.fixture(scope="module")
def setup(ref_pkg):
    from sarbon_b200.detector import B200Detector
    det = make_det(ref_pkg)
    g = torch.Generator().manual_seed(7)
    p8 = torch.randn(2, 128, 48, 80, generator=g).relu().cuda().half()
    p8 = p8.permute(0, 2, 3, 1).contiguous().permute(0, 3, 1, 2)  # NCHW view of NHWC, as the engine gives
    feats, ref_out, ref_top = ref_forward(ref_pkg, det, p8)
    mine = B200Detector(det, 2, 48, 80)
    return det, p8, feats, ref_out, ref_top, mine


def test_dense_core_levels(setup):
    det, p8, feats, ref_out, ref_top, mine = setup
    mine.run(p8)
    torch.cuda.synchronize()
    for i, f in enumerate(feats):
        got = mine.level(i).permute(0, 3, 1, 2)
        frac, err = close_frac(got, f)
        rel = err / f.float().abs().max().item()
        print(f"\nDenseCore level {i}: max |diff| {err:.3e} ({rel:.2e} of max), outside 1e-3 + 1e-2|b|: {frac:.2e}")
        assert rel < 1e-2 and frac < 1e-3, (i, err, rel, frac)


def test_query_selection(setup):
    det, p8, feats, ref_out, ref_top, mine = setup
    mine.force_top = None
    mine.run(p8)
    torch.cuda.synchronize()
    got = mine.top.long()
    same = sum(len(set(got[b].tolist()) & set(ref_top[b].tolist())) for b in range(got.shape[0]))
    frac = same / got.numel()
    print(f"\ntop-{mine.K} rows shared with the reference's selection: {frac:.4f}")
    assert frac > 0.95


def test_outputs_with_reference_selection(setup):
    det, p8, feats, ref_out, ref_top, mine = setup
    mine.force_top = ref_top.to(torch.int32)
    out = mine.run(p8)
    torch.cuda.synchronize()
    report = {}
    for key in ("pred_boxes", "pred_logits", "enc_boxes"):
        frac, err = close_frac(out[key], ref_out[key])
        report[key] = (frac, err)
    fe, ee = close_frac(out["id_embed"], ref_out["id_embed"], rtol=1e-2, atol=1e-2)
    print(f"\ndetector outputs vs the reference (fraction outside 1e-3 + 1e-2|b|, max |diff|): {report}; "
          f"id_embed {fe:.2e} {ee:.2e}")
    for key, (frac, err) in report.items():
        assert frac == 0.0, (key, frac, err)
    assert fe == 0.0
    mine.force_top = None


def test_graph_replay_and_timing(setup):
    import time
    det, p8, feats, ref_out, ref_top, mine = setup
    eager = {k: v.clone() for k, v in mine.run(p8).items() if torch.is_tensor(v)}
    mine.capture(p8)
    out = mine.replay()
    torch.cuda.synchronize()
    for k in ("pred_boxes", "pred_logits", "id_embed"):
        assert torch.equal(out[k], eager[k]), k

    def timed(fn, n=20):
        fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(n):
            fn()
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) / n * 1e3

    ms_mine = timed(mine.replay)
    # the reference's own graph of the same call (SarbonVideo._detect, video.py:120-137)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), torch.no_grad(), torch.autocast("cuda", torch.float16):
        for _ in range(3):
            det(None, p8=p8)
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(g), torch.no_grad(), torch.autocast("cuda", torch.float16):
        det(None, p8=p8)
    ms_ref = timed(g.replay)
    print(f"\ndetector on 2 x p8 48x80 (300 queries): {ms_mine:.3f} ms per call (B200Detector graph) vs "
          f"{ms_ref:.3f} ms (the reference under autocast, CUDA graph)")
    from sarbon_b200.det_ops import kernels_error
    assert kernels_error() == 0
