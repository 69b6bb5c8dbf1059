"""Track-steered block masks on the GPU (``sb_boxes_to_block_mask``; video.py:26-34 and the
``_steer`` step at video.py:139-147 of the reference).

* through the C ABI, the kernel reproduces bit for bit the masks the reference's own
  ``boxes_to_block_mask`` produced for the golden cases (tests/golden/boxes), twice in a row
  over a dirty output buffer (the mask is overwritten, not ORed);
* on 16 cameras of 1080p blocks with up to 600 random boxes each and margins -1..2, it
  equals the oracle;
* ``FusedSparseEngine.steer`` writes the engine's ``extra`` mask, and the next step
  recomputes exactly the steered blocks, dilated per layer, as ``set_extra`` of the same mask
  does;
* argument errors come back as error codes with a message.
"""
import ctypes as C
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import sparse_oracle as so

pytestmark = pytest.mark.gpu

GOLDEN = np.load(Path(__file__).parent / "golden" / "boxes" / "boxes_mask.npz")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")


def _abi_call(boxes, offsets, n, hb, wb, block, margin, out):
    from sarbon_b200._lib import lib
    b = torch.from_numpy(np.ascontiguousarray(boxes, np.float64)).cuda()
    o = torch.from_numpy(np.ascontiguousarray(offsets, np.int32)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    return lib().sb_boxes_to_block_mask(C.c_void_p(b.data_ptr() if len(boxes) else None), C.c_void_p(o.data_ptr()),
                                        len(boxes), n, hb, wb, block, margin, C.c_void_p(out.data_ptr()),
                                        C.c_void_p(stream))


def test_abi_matches_reference_golden_twice():
    for i in range(int(GOLDEN["n_cases"])):
        hb, wb, block, margin = (int(v) for v in GOLDEN[f"c{i}_grid"])
        boxes, off = GOLDEN[f"c{i}_boxes"], GOLDEN[f"c{i}_offsets"]
        want = GOLDEN[f"c{i}_mask"]
        n = len(off) - 1
        out = torch.full((n, hb, wb), 7, dtype=torch.uint8, device="cuda")  # dirty: every byte is written
        for call in range(2):
            assert _abi_call(boxes, off, n, hb, wb, block, margin, out) == 0
            torch.cuda.synchronize()
            np.testing.assert_array_equal(out.cpu().numpy(), want, err_msg=f"case {i} call {call}")


def test_wrapper_matches_reference_golden():
    from sarbon_b200 import boxes_to_block_mask, boxes_to_block_masks
    for i in range(int(GOLDEN["n_cases"])):
        hb, wb, block, margin = (int(v) for v in GOLDEN[f"c{i}_grid"])
        boxes, off = GOLDEN[f"c{i}_boxes"], GOLDEN[f"c{i}_offsets"]
        per = [boxes[off[c]:off[c + 1]] for c in range(len(off) - 1)]
        got = boxes_to_block_masks(per, hb, wb, block, margin).cpu().numpy()
        np.testing.assert_array_equal(got, GOLDEN[f"c{i}_mask"].astype(bool), err_msg=f"case {i}")
        one = boxes_to_block_mask(per[0], hb, wb, block, margin).cpu().numpy()
        np.testing.assert_array_equal(one, GOLDEN[f"c{i}_mask"][0].astype(bool), err_msg=f"case {i} camera 0")


@pytest.mark.parametrize("margin", [-1, 0, 1, 2])
def test_1080p_streams_vs_oracle(margin):
    from sarbon_b200 import boxes_to_block_masks
    n, hb, wb, block = 16, 34, 60, 32
    rng = np.random.default_rng(100 + margin)
    per = []
    for c in range(n):
        k = int(rng.integers(0, 600)) if c else 0
        x = rng.uniform(-100, wb * block + 100, (k, 2))
        y = rng.uniform(-100, hb * block + 100, (k, 2))
        w = rng.uniform(0, 200, (k, 2))
        per.append(np.stack([x[:, 0], y[:, 0], x[:, 0] + w[:, 0], y[:, 0] + w[:, 1]], 1))
    got = boxes_to_block_masks(per, hb, wb, block, margin).cpu().numpy()
    for c in range(n):
        np.testing.assert_array_equal(got[c], so.boxes_to_block_mask(per[c], hb, wb, block, margin),
                                      err_msg=f"camera {c}")


def test_engine_steer_equals_set_extra():
    from sarbon_b200 import FusedSparseEngine, LocalBackbone
    n, h, w = 2, 256, 384
    net = LocalBackbone().cuda().eval()
    eng = FusedSparseEngine(net, n, h, w, dtype=torch.float16, tau=float("inf"))  # only `extra` fires
    frames = torch.zeros(n, h, w, 3, device="cuda", dtype=torch.float16)
    eng.reset(frames)
    boxes = [np.array([[40.0, 10.0, 90.5, 70.0], [300.0, 200.0, 420.0, 290.0]]), np.zeros((0, 4))]
    want = np.stack([so.boxes_to_block_mask(b, eng.hb, eng.wb, eng.block, 1) for b in boxes])
    eng.steer(boxes, margin=1)
    np.testing.assert_array_equal(eng.extra.cpu().numpy(), want)
    mode, k = eng.step(frames)
    assert mode == "sparse" and k == int(so.dilate(want, eng.ds[-1]).sum())
    for d in eng.ds:
        np.testing.assert_array_equal(eng.masks[d].cpu().numpy(), so.dilate(want, d))
    ref = FusedSparseEngine(net, n, h, w, dtype=torch.float16, tau=float("inf"))
    ref.reset(frames)
    ref.set_extra(torch.from_numpy(want).cuda())
    assert ref.step(frames) == (mode, k)
    for name in eng.cache:
        assert torch.equal(eng.cache[name], ref.cache[name]), name
    with pytest.raises(ValueError, match="one box list per camera"):
        eng.steer(boxes[:1])


def test_abi_errors():
    from sarbon_b200._lib import lib
    out = torch.zeros((1, 2, 2), dtype=torch.uint8, device="cuda")
    off = torch.zeros(2, dtype=torch.int32, device="cuda")
    p_out, p_off = C.c_void_p(out.data_ptr()), C.c_void_p(off.data_ptr())
    L = lib()
    cases = [
        ((None, p_off, 1, 1, 2, 2, 32, 0, p_out, None), "null pointer"),   # boxes null with n_boxes > 0
        ((None, p_off, -1, 1, 2, 2, 32, 0, p_out, None), "negative n_boxes"),
        ((None, p_off, 0, 0, 2, 2, 32, 0, p_out, None), "n_cams"),
        ((None, p_off, 0, 1, 0, 2, 32, 0, p_out, None), "hb and wb"),
        ((None, p_off, 0, 1, 2, 2, 0, 0, p_out, None), "block must be positive"),
    ]
    for args, msg in cases:
        assert L.sb_boxes_to_block_mask(*args) != 0
        assert msg in L.sb_last_error().decode(), (msg, L.sb_last_error())
    # no boxes at all: a valid call that clears the mask
    out.fill_(1)
    assert L.sb_boxes_to_block_mask(None, p_off, 0, 1, 2, 2, 32, 0, p_out, None) == 0
    torch.cuda.synchronize()
    assert not out.any()
