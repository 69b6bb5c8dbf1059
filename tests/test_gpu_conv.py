"""Per-layer tile-conv numerics and the 1080p change-rate sweep (16 x 1080p streams, 1-30 % changed blocks).

* every layer of a dense pass equals a PyTorch fp32 conv (+bias, +residual, ReLU) of the
  engine's own input cache, within the fp16 tolerance (1e-2 rel / 1e-3 abs);
* the sweep forces 0/1/5/20/50/100% changed blocks at 1920x1088: the change mask equals
  the forced mask, dilated masks / block lists equal the oracle's bit for bit, and the
  sparse result equals a dense pass on the same frames bit for bit (with tau = 0 the
  engine is lossless and every tile is computed by the same kernel either way).
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


def _layer_refs(eng):
    """fp32 PyTorch recomputation of every layer from the engine's own input caches, with
    the weights in the engine dtype as the reference tile kernel has them
    (fused_engine.py:114: w_tile in the engine dtype, bias fp32)."""
    out = []
    for l in eng.layers:
        x = eng.cache[l.src].float().permute(0, 3, 1, 2)
        w = l.w_tile.to(eng.dtype).float().permute(3, 2, 0, 1).contiguous().cuda()
        y = F.conv2d(x, w, l.bias.cuda(), l.stride, 1)
        if l.res is not None:
            y = y + eng.cache[l.res].float().permute(0, 3, 1, 2)
        if l.act:
            y = F.relu(y)
        out.append((l.dst, y.permute(0, 2, 3, 1)))
    return out


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
@pytest.mark.parametrize("block", [32, 64])
def test_every_layer_dense_vs_torch(dtype, block):
    from sarbon_b200 import FusedSparseEngine, LocalBackbone
    torch.manual_seed(3)
    n, h, w = 2, 256, 384
    net = LocalBackbone().cuda().eval()
    eng = FusedSparseEngine(net, n, h, w, block=block, dtype=dtype)
    frames = (torch.rand(n, h, w, 3, device="cuda") * 4 - 2).to(dtype)
    eng.reset(frames)
    torch.cuda.synchronize()
    assert torch.equal(eng.cache["img"], frames)
    for dst, ref in _layer_refs(eng):
        got = eng.cache[dst].float()
        if dtype == torch.float16:
            bad = (got - ref).abs() > 1e-3 + 1e-2 * ref.abs()
            assert not bad.any(), (dst, bad.sum().item(), (got - ref).abs().max().item())
            # outputs are fp32 accumulations rounded once: at most ~1 fp16 ulp apart
            ulp = torch.finfo(torch.float16).eps * ref.abs().clamp(min=2 ** -14)
            assert ((got - ref).abs() <= 1.01 * ulp + 1e-7).float().mean() > 0.999, dst
        else:
            err = ((got - ref).abs().max() / ref.abs().max()).item()
            assert err < 1e-5, (dst, err)


@pytest.mark.parametrize("frac", [0.0, 0.01, 0.05, 0.20, 0.50, 1.0])
def test_change_rate_sweep_1080p(frac):
    from sarbon_b200 import FusedSparseEngine, LocalBackbone, scenes
    n, h, w, block = 1, 1088, 1920, 32
    torch.manual_seed(4)
    net = LocalBackbone().cuda().eval()
    sparse = FusedSparseEngine(net, n, h, w, dtype=torch.float16)
    dense = FusedSparseEngine(net, n, h, w, dtype=torch.float16)
    src = scenes.Streams(n, h, w, seed=21, n_rects=3, device="cuda")
    u0 = src.next()
    sparse.reset(scenes.normalise(u0))
    u1, forced = scenes.forced_change(u0.cpu(), frac, block, seed=int(frac * 1000) + 1)
    f1 = scenes.normalise(u1.cuda())
    mode, k = sparse.step(f1)
    np.testing.assert_array_equal(sparse.changed.cpu().numpy(), forced.numpy())
    for d in sparse.ds:
        md = so.dilate(forced.numpy(), d)
        np.testing.assert_array_equal(sparse.masks[d].cpu().numpy(), md)
        if mode == "sparse":
            lst = np.stack([x.cpu().numpy() for x in sparse.block_lists(d)])
            np.testing.assert_array_equal(lst, np.stack(so.block_lists(md)))
    k_exp = int(so.dilate(forced.numpy(), sparse.ds[-1]).sum())
    assert k == k_exp
    assert mode == ("skip" if k == 0 else "sparse")
    dense.reset(f1)
    for name in sparse.cache:
        assert torch.equal(sparse.cache[name], dense.cache[name]), name
