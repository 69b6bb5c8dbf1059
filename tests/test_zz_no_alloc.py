"""GPU tests of sb_block_lists_static, the allocation-free list builder (C ABI).

It must reproduce, bit for bit, the dilated masks, block lists and counts that the
engine's own step (sb_step, read back through sb_gate_buffers / sb_debug_lists) builds
from the same change mask, on two calls in a row that share its static scratch, and it
must reject masks larger than SB_STATIC_LISTS_MAX_BLOCKS before touching the GPU.
The file name sorts last so that it also runs after every other GPU test.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_BLOCKS = 1 << 20  # SB_STATIC_LISTS_MAX_BLOCKS in include/sarbon_sparse.h


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")


def static_lists(changed, ds, stream=None):
    """Calls sb_block_lists_static on a [N, Hb, Wb] uint8/bool device mask."""
    from sarbon_b200._lib import lib
    n, hb, wb = changed.shape
    nb = n * hb * wb
    masks = torch.full((len(ds), nb), 7, dtype=torch.uint8, device=changed.device)
    lists = torch.full((len(ds), 3, nb), -5, dtype=torch.int32, device=changed.device)
    counts = torch.full((len(ds),), -9, dtype=torch.int32, device=changed.device)
    dil = (C.c_int * len(ds))(*ds)
    s = torch.cuda.current_stream().cuda_stream if stream is None else stream
    rc = lib().sb_block_lists_static(C.c_void_p(changed.data_ptr()), n, hb, wb, dil, len(ds),
                                     C.c_void_p(masks.data_ptr()), C.c_void_p(lists.data_ptr()),
                                     C.c_void_p(counts.data_ptr()), C.c_void_p(s))
    assert rc == 0, lib().sb_last_error().decode()
    torch.cuda.synchronize()
    return masks, lists, counts


def np_lists(changed, d):
    """max_pool2d(changed, 2d+1, 1, d) per camera, then nonzero in flat order."""
    c = changed.astype(bool)
    n, hb, wb = c.shape
    p = np.zeros((n, hb + 2 * d, wb + 2 * d), bool)
    p[:, d:d + hb, d:d + wb] = c
    m = np.zeros_like(c)
    for dy in range(2 * d + 1):
        for dx in range(2 * d + 1):
            m |= p[:, dy:dy + hb, dx:dx + wb]
    cam, by, bx = np.nonzero(m)
    return m.reshape(-1).astype(np.uint8), np.stack([cam, by, bx]).astype(np.int32)


def engine_and_frames(seed):
    from sarbon_b200 import FusedSparseEngine, LocalBackbone
    torch.manual_seed(seed)
    net = LocalBackbone().eval()
    n, h, w = 4, 1088, 1920
    eng = FusedSparseEngine(net, n, h, w, dtype=torch.float16, tau=0.05)
    g = torch.Generator(device="cuda").manual_seed(seed)
    base = torch.randn(n, h, w, 3, device="cuda", generator=g).half()
    return eng, base


def changed_frames(base, rects, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    f = base.clone()
    for cam, y0, x0, hh, ww in rects:
        f[cam, y0:y0 + hh, x0:x0 + ww] += torch.randn(hh, ww, 3, device="cuda", generator=g).half()
    return f


def check_against_engine(eng):
    changed = eng.changed.view(torch.uint8)
    m1, l1, c1 = static_lists(changed, eng.ds)
    m2, l2, c2 = static_lists(changed, eng.ds)   # second call reuses the shared scratch
    nb = eng.n_blocks
    for i, d in enumerate(eng.ds):
        em = eng.masks[d].reshape(-1).view(torch.uint8)
        cam, by, bx = eng.block_lists(d)
        k = cam.numel()
        for m, l, c in ((m1, l1, c1), (m2, l2, c2)):
            assert int(c[i]) == k, (d, int(c[i]), k)
            assert torch.equal(m[i, :nb], em), d
            assert torch.equal(l[i, 0, :k], cam) and torch.equal(l[i, 1, :k], by) and torch.equal(l[i, 2, :k], bx), d
            assert bool((l[i, :, k:] == -5).all()), "entries past the count are left untouched"


def test_static_lists_match_engine_step():
    eng, base = engine_and_frames(11)
    eng.reset(base)
    rects = [(0, 100, 200, 70, 300), (1, 900, 1500, 150, 400), (3, 0, 0, 40, 40), (3, 1050, 1880, 38, 40)]
    mode, k = eng.step(changed_frames(base, rects, 12))
    assert k > 0
    check_against_engine(eng)
    # a second, different step: the lists follow the new mask
    rects = [(2, 500, 960, 200, 200)] + [(c, 64 * c, 64 * c, 33, 33) for c in range(4)]
    eng.step(changed_frames(base, rects, 13))
    check_against_engine(eng)


def test_static_lists_empty_and_full_masks():
    ds = [0, 1, 3]
    for fill in (0, 1):
        changed = torch.full((3, 17, 29), fill, dtype=torch.uint8, device="cuda")
        for _ in range(2):
            m, l, c = static_lists(changed, ds)
            for i, d in enumerate(ds):
                em, el = np_lists(changed.cpu().numpy(), d)
                assert int(c[i]) == el.shape[1]
                assert np.array_equal(m[i].cpu().numpy(), em)
                assert np.array_equal(l[i, :, :el.shape[1]].cpu().numpy(), el)


def test_static_lists_at_the_size_limit():
    g = torch.Generator(device="cuda").manual_seed(5)
    changed = (torch.rand(256, 64, 64, device="cuda", generator=g) < 0.002).to(torch.uint8)
    assert changed.numel() == MAX_BLOCKS
    ds = [0, 2, 5, 7]
    ch = changed.cpu().numpy()
    for _ in range(2):
        m, l, c = static_lists(changed, ds)
        for i, d in enumerate(ds):
            em, el = np_lists(ch, d)
            assert int(c[i]) == el.shape[1], d
            assert np.array_equal(m[i].cpu().numpy(), em), d
            assert np.array_equal(l[i, :, :el.shape[1]].cpu().numpy(), el), d


def test_static_lists_reject_oversize_and_bad_args():
    from sarbon_b200._lib import lib
    dil = (C.c_int * 1)(1)
    one = C.c_void_p(16)  # never dereferenced: the size checks come first
    rc = lib().sb_block_lists_static(one, 257, 64, 64, dil, 1, one, one, None, None)
    assert rc == 1 and b"static scratch limit" in lib().sb_last_error()
    rc = lib().sb_block_lists_static(one, 1, 4, 4, dil, 0, one, one, None, None)
    assert rc == 1 and b"n_dil" in lib().sb_last_error()
    rc = lib().sb_block_lists_static(None, 1, 4, 4, dil, 1, one, one, None, None)
    assert rc == 1 and b"null pointer" in lib().sb_last_error()


def test_static_lists_huge_dilation_is_clamped():
    """A dilation far beyond the grid (up to INT_MAX) marks every block of a camera that has
    a change, exactly as a dilation of max(hb, wb) does."""
    changed = torch.zeros((3, 9, 13), dtype=torch.uint8, device="cuda")
    changed[0, 4, 6] = 1
    changed[2, 0, 12] = 1
    ds = [2 ** 31 - 1, 13, 1]
    ch = changed.cpu().numpy()
    for _ in range(2):
        m, l, c = static_lists(changed, ds)
        for i, d in enumerate(ds):
            em, el = np_lists(ch, min(d, 13))
            assert int(c[i]) == el.shape[1], d
            assert np.array_equal(m[i].cpu().numpy(), em), d
            assert np.array_equal(l[i, :, :el.shape[1]].cpu().numpy(), el), d
    assert int(c[0]) == 2 * 9 * 13  # cameras 0 and 2 entirely, camera 1 nothing
