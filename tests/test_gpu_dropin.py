"""The drop-in inside the reference's own video pipeline.

After the reference's own GPU pipeline test (tests/test_pipeline_gpu.py:20-48 of the
reference): `sarbon.inference.video.SarbonVideo` builds its engine with
`from ..sparse.fused_engine import FusedSparseEngine` (video.py:58-64); here that name is
pointed at `sarbon_b200.FusedSparseEngine` and nothing else of the reference changes.  Two
720p cameras run for 12 frames through the whole reference pipeline (its `_prep` with the
resize to 640x1152, stem_to_local, calibrate, the engine, the detector on p8, tracking and
track steering); after every frame the engine's p8 must match the reference's dense fp16
stem on the same prepared frames within the reference test's own bar (max |a - b| / max |b|
< 2e-2).  The reference is the package installed under baseline/_ref.

A second run also replaces the detector after the stem (``sarbon_b200.detector.install``:
SarbonVideo's own CUDA graph then captures B200Detector's kernels): the pipeline runs the
same frames with no reference compute left on the GPU path, and on the last frame's p8 the
installed detector, given the reference detector's query selection, matches the reference's
boxes and class logits within |a - b| <= 1e-3 + 1e-2 |b|.
"""
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")


def randomize_bn(m, gen):
    """Non-trivial BatchNorm statistics and affine parameters (the ranges of the reference's
    own pipeline test, tests/test_pipeline.py:20-27)."""
    with torch.no_grad():
        for b in m.modules():
            if isinstance(b, torch.nn.BatchNorm2d):
                c = b.num_features
                b.running_mean.copy_(torch.rand(c, generator=gen) * 0.4 - 0.2)
                b.running_var.copy_(torch.rand(c, generator=gen) * 1.5 + 0.5)
                b.weight.copy_(torch.rand(c, generator=gen) + 0.5)
                b.bias.copy_(torch.rand(c, generator=gen) * 0.4 - 0.2)


def test_sarbon_video_runs_on_the_b200_engine(monkeypatch):
    if not (REF / "sarbon").is_dir():
        pytest.skip("the reference package is not installed under baseline/_ref")
    monkeypatch.syspath_prepend(str(REF))
    import sarbon.sparse.fused_engine as fe
    from sarbon.inference.video import SarbonVideo
    from sarbon.models.sarbon_det import build

    import sarbon_b200
    from sarbon_b200 import scenes
    monkeypatch.setattr(fe, "FusedSparseEngine", sarbon_b200.FusedSparseEngine)
    torch.manual_seed(0)
    det = build("s", 6, halo_zero=False)
    randomize_bn(det, torch.Generator().manual_seed(1))
    video = SarbonVideo(det, n_cams=2, size=(640, 1152), device="cuda", keep_score=0.3)
    # moving objects over a static background without sensor noise: at the pipeline's
    # default tau = 0 (lossless) only the objects' blocks change
    src = scenes.Streams(2, 720, 1280, seed=71, n_rects=4, noise=0.0)
    worst, modes = 0.0, []
    for t in range(12):
        frames = [f.flip(-1).contiguous().numpy() for f in src.next()]  # uint8 BGR, HWC
        res = video.step(frames)
        assert isinstance(video.engine, sarbon_b200.FusedSparseEngine)
        assert len(res) == 2
        x = video._prep(frames).permute(0, 3, 1, 2).contiguous().half()
        with torch.no_grad():
            ref = det.stem.half().forward_blocks(x)[1].float()
            det.stem.float()
        got = video.engine.outputs_nchw()[1].float()
        worst = max(worst, ((got - ref).abs().max() / ref.abs().max()).item())
        modes.append(video.engine.stats)
    print(f"\nSarbonVideo on the B200 engine, 12 frames: max rel err of p8 vs the dense fp16 stem {worst:.1e}; "
          f"engine stats {modes[-1]}; active blocks {[round(a, 3) for a in video.stats['active_blocks']]}")
    assert worst < 2e-2
    assert modes[-1]["sparse"] >= 6, modes[-1]


def test_sarbon_video_with_the_b200_detector(monkeypatch):
    if not (REF / "sarbon").is_dir():
        pytest.skip("the reference package is not installed under baseline/_ref")
    monkeypatch.syspath_prepend(str(REF))
    import sarbon.sparse.fused_engine as fe
    from sarbon.inference.video import SarbonVideo
    from sarbon.models.sarbon_det import build

    import sarbon_b200
    from sarbon_b200 import scenes
    from sarbon_b200.detector import install
    monkeypatch.setattr(fe, "FusedSparseEngine", sarbon_b200.FusedSparseEngine)
    torch.manual_seed(0)
    det = build("s", 6, halo_zero=False)
    randomize_bn(det, torch.Generator().manual_seed(1))
    gen = torch.Generator().manual_seed(2)
    with torch.no_grad():
        for m in det.modules():  # zero-initialised heads and sampling offsets made non-trivial
            if isinstance(m, torch.nn.Linear) and not m.weight.any():
                m.weight.copy_(torch.randn(m.weight.shape, generator=gen) * 0.02)
    video = install(SarbonVideo(det, n_cams=2, size=(640, 1152), device="cuda", keep_score=0.0))
    src = scenes.Streams(2, 720, 1280, seed=73, n_rects=4, noise=0.0)
    for t in range(8):
        frames = [f.flip(-1).contiguous().numpy() for f in src.next()]
        res = video.step(frames)
        assert len(res) == 2
    mine = video.b200_detector["det"]
    # the video's own graph replays the B200 kernels: its outputs are B200Detector's buffers
    assert video._graph is not None and video._graph_out["pred_boxes"] is mine.box
    # the last frame's p8 through the installed detector vs the reference detector
    p8 = video.engine.outputs_nchw()[1]
    with torch.no_grad(), torch.autocast("cuda", torch.float16):
        ref = det(None, p8=p8)
        feats = det.core(p8)
        shapes = [f.shape[-2:] for f in feats]
        memory = torch.cat([f.flatten(2).transpose(1, 2) for f in feats], 1)
        _, valid = det.anchors(shapes, memory.device, memory.dtype)
        enc = det.enc_proj(memory * valid.to(memory.dtype))
        top = det.enc_cls(enc).max(-1).values.masked_fill(~valid[..., 0], float("-inf")).topk(det.cfg.queries, 1).indices
    mine.force_top = top.to(torch.int32)
    out = mine.run(p8)
    torch.cuda.synchronize()
    mine.force_top = None
    for key in ("pred_boxes", "pred_logits"):
        a, b = out[key].float(), ref[key].float()
        bad = ((a - b).abs() > 1e-3 + 1e-2 * b.abs()).float().mean().item()
        assert bad == 0.0, (key, bad, (a - b).abs().max().item())
