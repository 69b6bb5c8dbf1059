"""Golden vectors for track-steered block masks, made by the reference's own code.

Runs ``boxes_to_block_mask`` of ``sarbon/inference/video.py`` (video.py:26-34) of the
reference checkout (its path is the first argument) on seeded random and
hand-picked boxes and writes ``boxes/boxes_mask.npz`` next to this script.  The tests only
read the ``.npz``; they never need the reference.

Each case holds N cameras' boxes (float64 ``[total, 4]`` xyxy in engine pixels, camera c
owning rows ``offsets[c]:offsets[c+1]``), the grid ``hb x wb``, ``block``, ``margin`` and
the reference's masks ``[N, hb, wb]``.  The boxes include the engine-pixel values the video
loop produces (float32 track boxes divided by a float64 scale, video.py:145), coordinates
on and next to block edges, outside the image, reversed, and huge.

Usage: python tests/golden/make_boxes_golden.py /path/to/reference
"""
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "boxes"
if len(sys.argv) < 2:
    sys.exit("usage: make_boxes_golden.py /path/to/reference")
REF = Path(sys.argv[1])
sys.path.insert(0, str(REF))
from sarbon.inference.video import boxes_to_block_mask  # noqa: E402


def random_boxes(rng, k, h, w, scale=None):
    """k boxes over (and a little past) an h x w image; a fifth of them reversed."""
    x = rng.uniform(-80, w + 80, (k, 2))
    y = rng.uniform(-80, h + 80, (k, 2))
    b = np.stack([x.min(1), y.min(1), x.max(1), y.max(1)], 1)
    flip = rng.random(k) < 0.2
    b[flip] = b[flip][:, [2, 3, 0, 1]]
    if scale is not None:  # video.py:145,167: float32 predictions / np.r_[scale, scale]
        s4 = np.r_[scale, scale]  # scale = (source w / engine w, source h / engine h)
        b = (b * s4).astype(np.float32) / s4
    return b.astype(np.float64)


def edge_boxes(block, h, w):
    """Coordinates on, just below and just above block edges, outside the image, huge."""
    e = float(block)
    dn, up = np.nextafter(e, 0.0), np.nextafter(e, np.inf)
    return np.array([
        [0.0, 0.0, 0.0, 0.0],
        [e, e, 2 * e, 2 * e],
        [dn, dn, np.nextafter(2 * e, 0.0), np.nextafter(2 * e, 0.0)],
        [up, up, up, up],
        [-0.5, -0.5, -1e-300, 3 * e - 1e-9],
        [-e, -e, -np.nextafter(e, 0.0), -0.0],
        [-e - 1e-9, 0.0, -e - 1e-9, 0.0],
        [w + 5.0, h + 5.0, w + 50.0, h + 50.0],
        [w - 0.25, h - 0.25, 1e30, 1e30],
        [-1e30, -1e300, 1e300, 1e30],
        [5 * e, 2 * e, 3 * e, 4 * e],
        [0.1 * 3 * e, 0.7 * e, 1.1 * e * 3, 0.3 * e * 7],
    ])


def main():
    rng = np.random.default_rng(11)
    cases = [  # (n cams, hb, wb, block, margin, boxes per camera (None = edge set), scale)
        (3, 6, 9, 32, 1, [5, 0, 12], np.array([1920 / 1152, 1080 / 640])),
        (2, 5, 7, 64, 0, [3, 8], None),
        (2, 8, 6, 48, 2, [None, 6], np.array([1.5, 1.5])),
        (1, 4, 4, 20, -1, [9], None),
        (2, 7, 11, 32, 1, [None, None], None),
        (4, 34, 60, 32, 1, [40, 1, 0, 300], np.array([3840 / 1920, 2160 / 1088])),  # 1080p blocks, many tracks
        (1, 3, 5, 32, 3, [2], None),
    ]
    out = {"n_cases": np.int32(len(cases))}
    for i, (n, hb, wb, block, margin, ks, scale) in enumerate(cases):
        h, w = hb * block, wb * block
        per = [edge_boxes(block, h, w) if k is None else random_boxes(rng, k, h, w, scale) for k in ks]
        masks = np.stack([boxes_to_block_mask(b, hb, wb, block, margin=margin) for b in per])
        offsets = np.zeros(n + 1, np.int32)
        np.cumsum([len(b) for b in per], out=offsets[1:])
        out[f"c{i}_boxes"] = np.concatenate(per).astype(np.float64).reshape(-1, 4)
        out[f"c{i}_offsets"] = offsets
        out[f"c{i}_grid"] = np.array([hb, wb, block, margin], np.int32)
        out[f"c{i}_mask"] = masks.astype(np.uint8)
    OUT.mkdir(exist_ok=True)
    np.savez_compressed(OUT / "boxes_mask.npz", **out)
    print("wrote", OUT / "boxes_mask.npz", {k: v.shape for k, v in out.items() if k.endswith("_mask")})


if __name__ == "__main__":
    main()
