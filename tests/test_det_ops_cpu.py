"""Host-side layout logic of the detector op wrappers (sarbon_b200/det_ops.py), on the CPU:
the (ld, image stride) read off NHWC views -- a channel slice of a wider map, one level of
the decoder's concatenated [B, S, C] memory, a [rows, C] matrix -- and the rejections that
keep a wrong view from reaching a kernel."""
import pytest
import torch

from sarbon_b200 import det_ops as ops


def test_geometry_of_views():
    x = torch.zeros(2, 5, 7, 64)
    assert ops._geometry(x, "x") == (64, 35)
    wide = torch.zeros(2, 5, 7, 384)
    assert ops._geometry(wide[..., 128:], "x") == (384, 35)  # channel slice: pixels 384 apart
    mem = torch.zeros(3, 35 + 20, 256)
    lvl = mem[:, 20:55].view(3, 5, 7, 256)  # one level of a concatenated memory
    assert ops._geometry(lvl, "lvl") == (256, 55)
    m = torch.zeros(300, 96)
    assert ops._geometry(ops.as_map(m), "m") == (96, 300)
    assert ops._rows(torch.zeros(4, 300, 768)[..., 256:512], "q")[1:] == (768, 300)


def test_rejections():
    with pytest.raises(ValueError):
        ops._geometry(torch.zeros(2, 5, 7, 64).transpose(2, 3), "x")  # channels not contiguous
    with pytest.raises(ValueError):
        ops._geometry(torch.zeros(2, 5, 9, 64)[:, :, :7], "x")  # rows not consecutive
    with pytest.raises(ValueError):
        ops.as_map(torch.zeros(3, 4, 5))
    with pytest.raises(ValueError):  # sources must be fp16 CUDA maps: nothing reaches the library
        ops.gemm_conv(torch.zeros(10, 64), torch.zeros(16, 64, dtype=torch.float16))
