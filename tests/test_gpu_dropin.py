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
