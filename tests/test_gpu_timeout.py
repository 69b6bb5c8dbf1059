"""The bounded look-back wait of the list kernel runs out and is reported, without a fault.

A test hook (sb_debug_withhold_lookback) makes one list chunk keep its decoupled
look-back words unpublished and lowers the poll limit, so the next chunk's wait gives up
after a few microseconds.  Nothing faults, traps or hangs: the kernel sets its timeout
flag and finishes.  The host then sees it through the C ABI:

* an engine step returns SB_ETIMEOUT and sb_stats().error carries the look-back flag;
* sb_block_lists_static writes -1 into every count;
* with the hook cleared, a fresh engine and the next static call are valid again.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LOOKBACK_FLAG = 0x08  # SB_ERR_TIMEOUT_LOOKBK


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")


def _engine():
    from sarbon_b200 import FusedSparseEngine, LocalBackbone
    torch.manual_seed(2)
    # 8 x 1080p = 16,320 blocks = 16 list chunks of 1024
    eng = FusedSparseEngine(LocalBackbone().cuda().eval(), 8, 1088, 1920, dtype=torch.float16,
                            tau=float("inf"))
    frames = torch.zeros(8, 1088, 1920, 3, device="cuda", dtype=torch.float16)
    eng.reset(frames)
    rng = np.random.default_rng(1)
    eng.set_extra(torch.from_numpy(rng.random((8, 34, 60)) < 0.05).cuda())
    return eng, frames


def test_engine_step_reports_lookback_timeout():
    from sarbon_b200._lib import SB_ETIMEOUT, SarbonLibraryError, lib
    eng, frames = _engine()
    assert lib().sb_debug_withhold_lookback(eng._h.ptr, 5, 64) == 0
    try:
        with pytest.raises(SarbonLibraryError) as ei:
            eng.step(frames)
        assert ei.value.status == SB_ETIMEOUT, str(ei.value)
        assert eng.device_stats().error & LOOKBACK_FLAG
    finally:
        assert lib().sb_debug_withhold_lookback(eng._h.ptr, -1, 0) == 0
    # the context is intact: a fresh engine steps normally with exact lists
    fresh, frames = _engine()
    mode, k = fresh.step(frames)
    assert mode == "sparse" and k > 0
    assert fresh.device_stats().error == 0
    from oracle import sparse_oracle as so
    ext = fresh.extra.cpu().numpy()
    for d in fresh.ds:
        lst = np.stack([x.cpu().numpy() for x in fresh.block_lists(d)])
        np.testing.assert_array_equal(lst, np.stack(so.block_lists(so.dilate(ext, d))))


def test_static_lists_report_lookback_timeout():
    from sarbon_b200._lib import lib
    g = torch.Generator(device="cuda").manual_seed(3)
    changed = (torch.rand(8, 34, 60, device="cuda", generator=g) < 0.05).to(torch.uint8)
    nb, ds = changed.numel(), [1, 2]
    masks = torch.empty((2, nb), dtype=torch.uint8, device="cuda")
    lists = torch.empty((2, 3, nb), dtype=torch.int32, device="cuda")
    counts = torch.zeros(2, dtype=torch.int32, device="cuda")
    dil = (C.c_int * 2)(*ds)
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    def call():
        rc = lib().sb_block_lists_static(C.c_void_p(changed.data_ptr()), 8, 34, 60, dil, 2,
                                         C.c_void_p(masks.data_ptr()), C.c_void_p(lists.data_ptr()),
                                         C.c_void_p(counts.data_ptr()), s)
        assert rc == 0, lib().sb_last_error().decode()
        torch.cuda.synchronize()

    assert lib().sb_debug_withhold_lookback(None, 3, 64) == 0
    try:
        call()
        assert counts.tolist() == [-1, -1]
    finally:
        assert lib().sb_debug_withhold_lookback(None, -1, 0) == 0
    call()
    from oracle import sparse_oracle as so
    ch = changed.bool().cpu().numpy()
    for i, d in enumerate(ds):
        k = int(so.dilate(ch, d).sum())
        assert int(counts[i]) == k
        np.testing.assert_array_equal(lists[i, :, :k].cpu().numpy(), np.stack(so.block_lists(so.dilate(ch, d))))


def test_hook_rejects_bad_arguments():
    from sarbon_b200._lib import SB_EINVAL, lib
    assert lib().sb_debug_withhold_lookback(None, -2, 0) == SB_EINVAL
    assert lib().sb_debug_withhold_lookback(None, 0, -1) == SB_EINVAL
