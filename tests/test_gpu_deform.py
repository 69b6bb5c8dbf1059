"""The detector's deformable-attention core as one kernel (sb_ms_deform_attn).

Against the reference's own function (sarbon/models/deform_attn.py:14-28, from the reference
package installed under baseline/_ref): random values, sampling points inside and outside
the maps (zero padding), three levels of different sizes, fp32 and fp16 values.  Then the
reference's own detector (`build("s", 6, halo_zero=False)`, 300 queries) on a stride-8
feature map, with the kernel installed at the reference's documented replacement point:
boxes and class logits must equal the unpatched detector's (the encoder's top-K is computed
before the decoder, so both runs decode the same queries).
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


@pytest.fixture()
def ref_deform(monkeypatch):
    if not (REF / "sarbon").is_dir():
        pytest.skip("the reference package is not installed under baseline/_ref")
    monkeypatch.syspath_prepend(str(REF))
    import sarbon.models.deform_attn as da
    return da


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.float16, 2e-3)])
def test_core_matches_reference(ref_deform, dtype, tol):
    from sarbon_b200 import ms_deform_attn_core
    g = torch.Generator(device="cuda").manual_seed(3)
    shapes = [(48, 80), (24, 40), (12, 20)]
    b, q, nh, dh, npnt = 2, 300, 8, 32, 4
    s = sum(h * w for h, w in shapes)
    value = torch.randn(b, s, nh, dh, device="cuda", generator=g).to(dtype)
    # locations mostly inside [0, 1], some outside: zero padding at the map borders
    loc = torch.rand(b, q, nh, len(shapes), npnt, 2, device="cuda", generator=g) * 1.2 - 0.1
    loc = loc.to(dtype)  # under autocast the sampling locations come in the value's type too
    w = torch.rand(b, q, nh, len(shapes) * npnt, device="cuda", generator=g).softmax(-1)
    w = w.view(b, q, nh, len(shapes), npnt)
    ref = ref_deform.ms_deform_attn_core(value, shapes, loc, w)
    got = ms_deform_attn_core(value, shapes, loc, w)
    assert got.shape == ref.shape and got.dtype == ref.dtype
    err = ((got.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
    assert err < tol, err


def test_reference_detector_with_the_kernel(ref_deform, monkeypatch):
    import time
    from sarbon.models.sarbon_det import build

    from sarbon_b200 import ms_deform_attn_core
    torch.manual_seed(0)
    det = build("s", 6, halo_zero=False).cuda().eval()
    gen = torch.Generator().manual_seed(4)
    with torch.no_grad():
        for m in det.modules():  # BN statistics and the zero-initialised heads made non-trivial
            if isinstance(m, torch.nn.BatchNorm2d):
                m.running_mean.copy_(torch.rand(m.num_features, generator=gen) * 0.4 - 0.2)
                m.running_var.copy_(torch.rand(m.num_features, generator=gen) * 1.5 + 0.5)
            elif isinstance(m, torch.nn.Linear) and not m.weight.any():
                m.weight.copy_(torch.randn(m.weight.shape, generator=gen) * 0.02)
    p8 = torch.randn(1, 128, 48, 80, generator=gen).relu().cuda()  # a 384x640 frame's stride-8 map

    def run():
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        with torch.no_grad():
            out = det(None, p8=p8)
        torch.cuda.synchronize()
        return out, time.perf_counter() - t0

    ref, _ = run()
    ref_t = min(run()[1] for _ in range(5))
    monkeypatch.setattr(ref_deform, "ms_deform_attn_core", ms_deform_attn_core)
    got, _ = run()
    got_t = min(run()[1] for _ in range(5))
    assert ref["pred_boxes"].shape == (1, 300, 4)
    for key, atol in (("pred_boxes", 1e-4), ("pred_logits", 1e-3)):
        err = (got[key] - ref[key]).abs().max().item()
        assert err < atol, (key, err)
    print(f"\nreference detector on p8 (300 queries, 4 decoder layers): {1e3 * ref_t:.2f} ms with the "
          f"reference core, {1e3 * got_t:.2f} ms with the kernel")
