"""Cell-level gating inside the engine (``FusedSparseEngine.set_cell_gating``,
``sb_set_cell_gating``): the tighter estimate of the reference's gating.py:42-43 used for the
step's own masks.

* change mask, per-group block masks, block lists and active count equal the oracle
  (``gate_cells`` + ``cell_group_masks``) bit for bit, with tau > 0 on integer-valued frames
  (exact sums) and an ``extra`` mask, over several steps, and the image cache follows;
* at tau = 0 a cell-gated sparse step equals a dense pass of the same frames bit for bit
  (lossless) while activating fewer blocks than block-level gating;
* switching back (cell 0) gives block-level results again; argument errors.
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


def _engine(n, h, w, tau, block=32):
    from sarbon_b200 import FusedSparseEngine, LocalBackbone
    torch.manual_seed(3)
    net = LocalBackbone().cuda().eval()
    eng = FusedSparseEngine(net, n, h, w, block=block, dtype=torch.float16, tau=tau)
    eng.fallback = eng.n_blocks  # keep the sparse kernels running
    return net, eng


@pytest.mark.parametrize("cell", [8, 16])
def test_masks_lists_and_image_cache_vs_oracle(cell):
    n, h, w, block = 2, 256, 384, 32
    tau = 0.5
    _, eng = _engine(n, h, w, tau, block)
    eng.set_cell_gating(cell)
    k = block // cell
    rng = np.random.default_rng(cell)
    f = rng.integers(-4, 5, (n, h, w, 3)).astype(np.float16)
    eng.reset(torch.from_numpy(f).cuda())
    img = f.copy()
    for step in range(4):
        f = f.copy()
        for _ in range(3):  # small integer changes, some below the cell threshold
            cam, y, x = rng.integers(0, n), rng.integers(0, h - 20), rng.integers(0, w - 20)
            hh, ww = rng.integers(1, 20, 2)
            f[cam, y:y + hh, x:x + ww] += np.float16(rng.integers(1, 3))
        extra = np.zeros((n, h // block, w // block), bool)
        if step == 2:
            extra[1, 3, 7] = True
        eng.set_extra(torch.from_numpy(extra).cuda())
        mode, cnt = eng.step(torch.from_numpy(f).cuda())
        cells, changed = so.gate_cells(f, img, cell, block, tau, extra)
        masks = so.cell_group_masks(cells, eng.cell_radii, k)
        np.testing.assert_array_equal(eng.changed.cpu().numpy(), changed, err_msg=f"step {step}")
        for di, d in enumerate(eng.ds):
            np.testing.assert_array_equal(eng.masks[d].cpu().numpy(), masks[di], err_msg=f"step {step} d {d}")
        assert cnt == int(masks[-1].sum())
        assert mode == ("skip" if cnt == 0 else "sparse")
        if mode == "sparse":
            for di, d in enumerate(eng.ds):
                got = np.stack([x.cpu().numpy() for x in eng.block_lists(d)])
                np.testing.assert_array_equal(got, np.stack(so.block_lists(masks[di])))
        img = so.update_img(img, f, changed, block)
        np.testing.assert_array_equal(eng.cache["img"].cpu().numpy(), img, err_msg=f"step {step}")


def test_lossless_at_tau0_and_fewer_blocks():
    from sarbon_b200 import FusedSparseEngine, scenes
    n, h, w = 2, 384, 640
    net, eng = _engine(n, h, w, 0.0)
    blk = FusedSparseEngine(net, n, h, w, dtype=torch.float16, tau=0.0)
    blk.fallback = blk.n_blocks
    dense = FusedSparseEngine(net, n, h, w, dtype=torch.float16, tau=0.0)
    eng.set_cell_gating(8)
    src = scenes.Streams(n, h, w, seed=5, n_rects=2, noise=0.0)  # only the rectangles move
    frames = [scenes.normalise(src.next()).cuda() for _ in range(4)]
    for e in (eng, blk):
        e.reset(frames[0])
    fewer = 0
    for f in frames[1:]:
        mode, k = eng.step(f)
        _, kb = blk.step(f)
        assert k <= kb
        fewer += kb - k
        dense.reset(f)
        for name in eng.cache:
            assert torch.equal(eng.cache[name], dense.cache[name]), (name, mode)
    assert fewer > 0  # the moving rectangles activate fewer blocks at cell level
    # back to block level: the same counts as the block-level engine
    eng.set_cell_gating(0)
    f = frames[1]
    assert eng.step(f) == blk.step(f)


def test_errors():
    from sarbon_b200 import FusedSparseEngine, LocalBackbone, SarbonLibraryError, scenes
    net, eng = _engine(1, 64, 96, 0.0)
    with pytest.raises(SarbonLibraryError, match="multiple of 8"):
        eng.set_cell_gating(12)
    with pytest.raises(SarbonLibraryError, match="multiple of 8"):
        eng.set_cell_gating(64)  # larger than the block
    eng.set_cell_gating(8)
    u8 = torch.zeros(1, 64, 96, 3, dtype=torch.uint8, device="cuda")
    eng.reset(torch.zeros(1, 64, 96, 3, dtype=torch.float16, device="cuda"))
    with pytest.raises(SarbonLibraryError, match="fp16 frames"):
        eng.step_u8(u8, scenes.MEAN, scenes.STD, sync=True)
    f32 = FusedSparseEngine(LocalBackbone().cuda().eval(), 1, 64, 96, dtype=torch.float32)
    with pytest.raises(SarbonLibraryError, match="fp16 engines"):
        f32.set_cell_gating(8)
