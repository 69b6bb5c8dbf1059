"""GPU tests of the M0 API (`BlockSparseEngine`, sarbon/sparse/block_sparse.py:122-326) on
the B200 engine, after the reference's own M0 bench (bench/bench_block_sparse.py:47-66):
lossless chained sparse steps against the dense forward pass, the overflow flag, and
`update` with a caller-given mask."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

H, W = 256, 384


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False


def moving(prev, frac, gen):
    """A frame whose changed area is about `frac` of the image: random squares of new
    content (uniform), as the reference bench's moving objects."""
    f = prev.clone()
    n = max(1, int(frac * H * W / 48 ** 2))
    for _ in range(n):
        y = int(torch.randint(0, H - 48, (1,), generator=gen))
        x = int(torch.randint(0, W - 48, (1,), generator=gen))
        f[:, y:y + 48, x:x + 48] = torch.rand(3, 48, 48, generator=gen).to(f)
    return f


@pytest.mark.parametrize("block", [32, 64])
def test_chained_steps_are_lossless_fp32(block):
    from sarbon_b200 import LocalBackbone
    from sarbon_b200.block_sparse import BlockSparseEngine
    torch.manual_seed(0)
    net = LocalBackbone().cuda().float().eval()
    eng = BlockSparseEngine(net, block)
    gen = torch.Generator().manual_seed(1)
    f0 = torch.rand(3, H, W, generator=gen).cuda()
    eng.full(f0)
    prev, worst = f0, 0.0
    cap = (H // block) * (W // block)  # budget = all blocks, so no overflow
    for frac in (0.01, 0.05, 0.2):  # consecutive frames: errors must not accumulate
        f1 = moving(prev, frac, gen)
        outs, over = eng.step(f1, cap)
        assert not bool(over)
        with torch.no_grad():
            ref = net(f1[None])
        for o, r in zip(outs, ref):
            worst = max(worst, ((o - r[0]).abs().max() / r.abs().max()).item())
        prev = f1
    assert worst < 1e-5, worst


def test_overflow_flag_and_capacity_fp16():
    """More active blocks than the capacity: the flag is raised and, as in M0
    (block_sparse.py:268-271), only the first `capacity` blocks of each dilation are
    recomputed -- the rest keep their old values until the caller's dense refresh; within
    the capacity a step is exact (sparse == dense bit for bit at tau = 0)."""
    from sarbon_b200 import LocalBackbone
    from sarbon_b200.block_sparse import BlockSparseEngine
    torch.manual_seed(2)
    net = LocalBackbone().cuda().half().eval()
    gen = torch.Generator().manual_seed(3)
    f0 = torch.rand(3, H, W, generator=gen).cuda().half()
    f1 = moving(f0, 0.3, gen)
    eng = BlockSparseEngine(net, 32)
    eng.full(f0)
    outs, over = eng.step(f1, 16)          # far more than 16 active blocks
    assert over.dim() == 0 and bool(over)
    ref = BlockSparseEngine(net, 32)
    ref_outs = ref.full(f1)
    assert any(not torch.equal(o, r) for o, r in zip(outs, ref_outs)), "blocks past the capacity were recomputed"
    # the dense refresh the flag asks for, then a small change within the budget: exact
    outs = eng.full(f1)
    for o, r in zip(outs, ref_outs):
        assert torch.equal(o, r)
    f2 = f1.clone()
    f2[:, 100:110, 200:210] += 0.5
    outs, over = eng.step(f2, (H // 32) * (W // 32))
    assert not bool(over)
    for o, r in zip(outs, ref.full(f2)):
        assert torch.equal(o, r)


def test_update_with_given_mask_and_helpers():
    from sarbon_b200 import LocalBackbone
    from sarbon_b200.block_sparse import BlockSparseEngine
    torch.manual_seed(4)
    net = LocalBackbone().cuda().half().eval()
    gen = torch.Generator().manual_seed(5)
    f0 = torch.rand(3, H, W, generator=gen).cuda().half()
    f1 = moving(f0, 0.05, gen)
    eng = BlockSparseEngine(net, 32)
    eng.full(f0)
    changed = eng.changed_blocks(f1, f0)
    assert changed.shape == (H // 32, W // 32) and bool(changed.any())
    outs = eng.update(f1, changed)
    for o, r in zip(outs, BlockSparseEngine(net, 32).full(f1)):
        assert torch.equal(o, r)
    # cache views are CHW
    assert eng.cache["img"].shape == (3, H, W)
    assert eng.cache["t14"].shape[1:] == (H // 8, W // 8)
