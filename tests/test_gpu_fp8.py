"""The e4m3 stride-8 stage (FusedSparseEngine(fp8=True), SB_CREATE_FP8_S8).

The reference has no e4m3 path (its tile weights are cast to the engine dtype,
fused_engine.py:114), so its kernels are pinned here by their own arithmetic:

* every e4m3 layer, computed from the engine's own input caches, equals the oracle's
  restatement (dequantise the e4m3 input and residual, weights quantised per output
  channel exactly as the engine quantises them, fp32 conv + bias + residual + ReLU,
  e4m3 of y / s_out): the codes are equal except where the fp32 sum sits on an e4m3
  rounding boundary, and there they differ by one code;
* a sparse step equals a dense pass of the same frames bit for bit (tau = 0);
* against the fp16 engine on the same frames the quantisation error of p8 is measured and
  bounded (it is the precision of e4m3, not a kernel error).
"""
import numpy as np
import pytest
import torch

from oracle import sparse_oracle as so

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")


STAGES = {True: ({"t8", "t9", "t11", "t12", "t14"}, [0, 0, 0, 0, 0, 0, 1, 2, 2, 2, 2]),
          "all": ({"t1", "t2", "t4", "t5", "t8", "t9", "t11", "t12", "t14"}, [0, 1, 2, 2, 2, 3, 1, 2, 2, 2, 2])}


def _engines(n=2, h=256, w=384, seed=0, tau=0.0, fp8=True):
    from sarbon_b200 import FusedSparseEngine, LocalBackbone, scenes
    torch.manual_seed(seed)
    net = LocalBackbone().cuda().eval()
    src = scenes.Streams(n, h, w, seed=seed + 1, n_rects=3, device="cuda")
    frames = [scenes.normalise(src.next()) for _ in range(4)]
    e8 = FusedSparseEngine(net, n, h, w, dtype=torch.float16, fp8=fp8, tau=tau)
    scales = e8.calibrate_fp8(frames[0])
    return net, e8, frames, scales


@pytest.mark.parametrize("fp8", [True, "all"], ids=["s8", "s4+s8"])
def test_fp8_layers_vs_oracle(fp8):
    net, eng, frames, scales = _engines(fp8=fp8)
    caches, qs = STAGES[fp8]
    assert eng.fp8_caches == caches
    modes = eng.layer_variants()
    assert [m >> 4 for m in modes] == qs, modes
    eng.reset(frames[1])
    deq = {name: eng.dequantized(name).float().cpu().numpy() for name in eng.cache}
    worst = {}
    for i, l in enumerate(eng.layers):
        if l.dst not in eng.fp8_caches and l.src not in eng.fp8_caches:
            continue
        w = l.w_tile.numpy()
        ws = eng.weight_scales(i) if l.src in eng.fp8_caches else None
        if ws is None:
            w = w.astype(np.float16).astype(np.float32)  # fp16 MMA: the weights in the engine dtype
        if l.dst not in eng.fp8_caches:  # e4m3 in, fp16 out (the stage's output)
            exp = so.conv_dense_e4m3(deq[l.src], w, l.bias.numpy(), l.stride, l.act,
                                     None if l.res is None else deq[l.res], None, ws)
            got = eng.cache[l.dst].float().cpu().numpy()
            bad = np.abs(got - exp) > 1e-3 + 1e-2 * np.abs(exp)
            assert not bad.any(), (l.dst, int(bad.sum()))
            continue
        exp = so.conv_dense_e4m3(deq[l.src], w, l.bias.numpy(), l.stride, l.act,
                                 None if l.res is None else deq[l.res], eng.act_scale(l.dst), ws)
        got = eng.cache[l.dst].view(torch.uint8).cpu().numpy()
        diff = got != exp
        # neighbouring codes of the same sign differ by one in the low seven bits
        step = np.abs((got.astype(np.int16) & 0x7F) - (exp.astype(np.int16) & 0x7F))
        same_sign = (got & 0x80) == (exp & 0x80)
        near_zero = ((got & 0x7F) <= 1) & ((exp & 0x7F) <= 1)
        assert np.all(~diff | (same_sign & (step <= 1)) | near_zero), (l.dst, int(diff.sum()))
        worst[l.dst] = float(diff.mean())
        assert diff.mean() < 1e-3, (l.dst, float(diff.mean()))
    print(f"\ne4m3 layers: fraction of codes one step from the oracle's {worst}; scales {scales}")


@pytest.mark.parametrize("fp8", [True, "all"], ids=["s8", "s4+s8"])
def test_fp8_sparse_step_equals_dense_pass(fp8):
    from sarbon_b200 import FusedSparseEngine, scenes
    net, sparse, frames, scales = _engines(seed=3, fp8=fp8)
    dense = FusedSparseEngine(net, sparse.n, sparse.h, sparse.w, dtype=torch.float16, fp8=fp8)
    for name, sc in scales.items():
        dense.set_act_scale(name, sc)
    sparse.reset(frames[0])
    for f in frames[1:]:
        mode, k = sparse.step(f)
        assert mode == "sparse"
    dense.reset(frames[-1])
    for name in sparse.cache:
        assert torch.equal(sparse.cache[name].view(torch.uint8) if name in sparse.fp8_caches else sparse.cache[name],
                           dense.cache[name].view(torch.uint8) if name in dense.fp8_caches else dense.cache[name]), name


@pytest.mark.parametrize("fp8", [True, "all"], ids=["s8", "s4+s8"])
def test_fp8_quantisation_error_vs_fp16_engine(fp8):
    from sarbon_b200 import FusedSparseEngine
    net, e8, frames, scales = _engines(n=2, h=512, w=768, seed=5, fp8=fp8)
    e16 = FusedSparseEngine(net, e8.n, e8.h, e8.w, dtype=torch.float16)
    e8.reset(frames[0])
    e16.reset(frames[0])
    p8_8 = e8.outputs_nchw()[1].float()
    p8_16 = e16.outputs_nchw()[1].float()
    rel_max = float((p8_8 - p8_16).abs().max() / p8_16.abs().max())
    rel_rms = float(((p8_8 - p8_16) ** 2).mean().sqrt() / (p8_16 ** 2).mean().sqrt())
    p4_8 = e8.outputs_nchw()[0].float()
    p4_16 = e16.outputs_nchw()[0].float()
    p4_rms = float(((p4_8 - p4_16) ** 2).mean().sqrt() / (p4_16 ** 2).mean().sqrt())
    if fp8 is True:
        assert torch.equal(e8.cache["t7"], e16.cache["t7"])  # the fp16 stages are untouched
    print(f"\n{fp8}: p8 e4m3 vs fp16 engine: max |diff| / max |p8| {rel_max:.4f}, rms ratio {rel_rms:.4f}; "
          f"p4 rms ratio {p4_rms:.4f}")
    assert rel_rms < 0.1 and rel_max < 0.25 and p4_rms < 0.1, (rel_rms, rel_max, p4_rms)
