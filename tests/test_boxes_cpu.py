"""Track-steered block masks (video.py:26-34) on the CPU: the oracle reproduces, bit for bit,
the masks the reference's own ``boxes_to_block_mask`` produced for the golden cases
(tests/golden/boxes, made by ``make_boxes_golden.py``), and the Python wrapper rejects the
boxes the reference cannot convert before it touches a GPU."""
from pathlib import Path

import numpy as np
import pytest

from oracle import sparse_oracle as so

GOLDEN = np.load(Path(__file__).parent / "golden" / "boxes" / "boxes_mask.npz")


def golden_cases():
    for i in range(int(GOLDEN["n_cases"])):
        hb, wb, block, margin = (int(v) for v in GOLDEN[f"c{i}_grid"])
        off = GOLDEN[f"c{i}_offsets"]
        boxes = GOLDEN[f"c{i}_boxes"]
        per = [boxes[off[c]:off[c + 1]] for c in range(len(off) - 1)]
        yield i, per, hb, wb, block, margin, GOLDEN[f"c{i}_mask"].astype(bool)


def test_oracle_matches_reference_golden():
    seen = 0
    for i, per, hb, wb, block, margin, mask in golden_cases():
        for c, b in enumerate(per):
            np.testing.assert_array_equal(so.boxes_to_block_mask(b, hb, wb, block, margin), mask[c],
                                          err_msg=f"case {i} camera {c}")
        seen += 1
    assert seen == 7
    # the fixture covers empty cameras, all-clear and non-trivial masks, and > 256 boxes
    # (more than one shared-memory chunk of the kernel)
    assert any(len(b) == 0 for _, per, *_ in golden_cases() for b in per)
    assert max(len(b) for _, per, *_ in golden_cases() for b in per) > 256


def test_wrapper_rejects_what_the_reference_cannot_convert():
    from sarbon_b200 import boxes_to_block_masks
    with pytest.raises(ValueError, match="NaN"):
        boxes_to_block_masks([[[0.0, 0.0, np.nan, 5.0]]], 4, 4, 32)
    with pytest.raises(ValueError, match="finite"):
        boxes_to_block_masks([[[0.0, -np.inf, 1.0, 5.0]]], 4, 4, 32)
    with pytest.raises(ValueError, match=r"\[k, 4\]"):
        boxes_to_block_masks([[[0.0, 1.0, 2.0]]], 4, 4, 32)
    with pytest.raises(ValueError, match="block"):
        boxes_to_block_masks([[]], 4, 4, 0)
    with pytest.raises(ValueError, match="one box list per camera"):
        boxes_to_block_masks([], 4, 4, 32)
    # the reference raises on the same inputs
    with pytest.raises(ValueError):
        so.boxes_to_block_mask([[0.0, 0.0, np.nan, 5.0]], 4, 4, 32)
    with pytest.raises(ValueError):  # -inf // 32 is NaN
        so.boxes_to_block_mask([[0.0, -np.inf, 1.0, 5.0]], 4, 4, 32)
