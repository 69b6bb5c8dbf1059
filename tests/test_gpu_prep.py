"""The caller's frame preparation done by the engine for cameras of another size.

SarbonVideo._prep (sarbon/inference/video.py:95-99) turns uint8 BGR camera frames into the
engine input: BGR->RGB, float, F.interpolate(bilinear, align_corners=False) to the engine
size when the sizes differ, (x - MEAN) / STD, and the step's .half() (:105).
``FusedSparseEngine.step_u8`` on frames of another size runs all of it as one kernel of
the library (sb_step_u8_resized).  Compared here with PyTorch's own expression on the same
GPU: the image cache after a step in which every block changes must equal PyTorch's fp16
frames, bit for bit except where the fp32 bilinear value sits on an fp16 rounding boundary
(PyTorch's kernel may contract the products into fused multiply-adds differently); those
elements are counted, must be rare and may differ by one fp16 ulp at most.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")


def torch_prep(bgr, hw):
    """video.py:95-99 on the GPU, then the engine's fp16 cast (video.py:105)."""
    from sarbon_b200 import scenes
    x = bgr.flip(-1).permute(0, 3, 1, 2).float()
    if tuple(x.shape[-2:]) != tuple(hw):
        x = F.interpolate(x, hw, mode="bilinear", align_corners=False)
    mean = torch.from_numpy(scenes.MEAN).to(bgr.device)
    std = torch.from_numpy(scenes.STD).to(bgr.device)
    return ((x.permute(0, 2, 3, 1) - mean) / std).half()


@pytest.mark.parametrize("cam,hw", [((720, 1280), (736, 1280)), ((1080, 1920), (736, 1280)),
                                    ((480, 640), (512, 704))], ids=["720p->736", "1080p->736", "480p->512x704"])
def test_resize_prep_matches_torch(cam, hw):
    from sarbon_b200 import FusedSparseEngine, LocalBackbone, scenes
    torch.manual_seed(8)
    n = 2
    src = scenes.Streams(n, *cam, seed=61, n_rects=3, device="cuda")
    bgr = src.next().flip(-1).contiguous()
    ref = torch_prep(bgr, hw)
    # tau < 0: every block changes, so the step copies the whole prepared frame into the image cache
    eng = FusedSparseEngine(LocalBackbone().cuda().eval(), n, *hw, dtype=torch.float16, tau=-1.0)
    mode, k = eng.step_u8(bgr, scenes.MEAN, scenes.STD)
    assert mode == "sparse" and k == eng.n_blocks
    got = eng.cache["img"]
    diff = (got.float() - ref.float()).abs()
    ulp = torch.from_numpy(np.spacing(np.abs(ref.cpu().numpy())).astype(np.float32)).cuda()
    n_diff = int((got != ref).sum())
    print(f"\n{cam}->{hw}: {n_diff} of {ref.numel()} values differ from PyTorch's; "
          f"max |diff| / ulp {float((diff / ulp).max()):.2f}")
    assert bool((diff <= ulp).all())
    assert n_diff <= 1e-4 * ref.numel()


def test_resized_step_equals_fp16_step_on_the_same_frames():
    """Gating, lists and features of the resized uint8 step equal those of sb_step on the
    fp16 frames the prep kernel produced (read back from the image cache)."""
    from sarbon_b200 import FusedSparseEngine, LocalBackbone, scenes
    torch.manual_seed(9)
    n, cam, hw = 2, (720, 1280), (736, 1280)
    net = LocalBackbone().cuda().eval()
    tau = 8 / float(scenes.STD.mean())
    a = FusedSparseEngine(net, n, *hw, dtype=torch.float16, tau=tau)
    b = FusedSparseEngine(net, n, *hw, dtype=torch.float16, tau=-1.0)  # b's image cache = each prepared frame
    src = scenes.Streams(n, *cam, seed=62, n_rects=4, device="cuda")
    bgr = src.next().flip(-1).contiguous()
    b.step_u8(bgr, scenes.MEAN, scenes.STD)
    a.reset(b.cache["img"].clone())
    for _ in range(4):
        bgr = src.next().flip(-1).contiguous()
        b.step_u8(bgr, scenes.MEAN, scenes.STD)
        prepared = b.cache["img"].clone()
        c = FusedSparseEngine(net, n, *hw, dtype=torch.float16, tau=tau)
        c.reset(a.cache["img"].clone())
        for name in a.cache:
            c.cache[name].copy_(a.cache[name])
        ma = a.step_u8(bgr, scenes.MEAN, scenes.STD)
        mc = c.step(prepared)
        assert ma == mc
        assert torch.equal(a.changed, c.changed)
        for name in a.cache:
            assert torch.equal(a.cache[name], c.cache[name]), name
