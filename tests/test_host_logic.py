"""Host-side logic: stem program and layer fusion, dilations, budget buckets,
BatchNorm folding, and the synthetic stream generator."""
import math

import numpy as np
import pytest
import torch

from golden_io import CASES, load
from oracle import sparse_oracle as so
from sarbon_b200 import LocalBackbone, budget_buckets, fold, fuse_layers, stem_to_local
from sarbon_b200 import scenes


def test_budget_buckets_match_reference():
    for name in CASES:
        m = load(name)["meta"]
        n_blocks = m["n_cams"] * m["hb"] * m["wb"]
        assert budget_buckets(n_blocks) == m["buckets"] == so.budget_buckets(n_blocks)
    b = budget_buckets(920)
    assert b[0] == 16 and b[-1] == 928 and all(x % 16 == 0 for x in b)
    assert all(b[i + 1] >= b[i] + 16 for i in range(len(b) - 1))


def test_program_matches_reference_topology():
    """Node names, strides and receptive radii equal the reference program
    (block_sparse.py:78-113) recorded in the fixtures."""
    net = LocalBackbone()
    nodes, outs = net.program()
    ref = load(CASES[0])["meta"]
    assert list(outs) == ref["outputs"] == ["t7", "t14"]
    got = [(n.kind, list(n.src), n.dst, n.stride, n.radius) for n in nodes]
    exp = [(n["kind"], n["src"], n["dst"], n["stride"], n["radius"]) for n in ref["nodes"]]
    assert got == exp


def test_fused_layers_and_dilations():
    layers = fuse_layers(LocalBackbone())
    assert len(layers) == 11
    assert [l.dst for l in layers] == ["t0", "t1", "t2", "t4", "t5", "t7", "t8", "t9", "t11", "t12", "t14"]
    assert [l.res for l in layers] == [None, None, None, "t1", None, "t4", None, None, "t8", None, "t11"]
    assert [l.radius for l in layers] == [1, 3, 7, 11, 15, 19, 23, 31, 39, 47, 55]
    assert [math.ceil(l.radius / 32) for l in layers] == [1] * 8 + [2] * 3
    assert [math.ceil(l.radius / 64) for l in layers] == [1] * 11
    # MFLOP per 32x32 block: 42.91 in total (2*cin*cout*9*t^2 per layer)
    fl = sum(2 * l.w_tile.shape[2] * l.w_tile.shape[3] * 9 * (32 // l.out_stride) ** 2 for l in layers)
    assert abs(fl / 1e6 - 42.91) < 0.01


def test_fold_matches_conv_bn():
    torch.manual_seed(0)
    conv = torch.nn.Conv2d(8, 16, 3, 1, 1, bias=False)
    bn = torch.nn.BatchNorm2d(16)
    with torch.no_grad():
        bn.running_mean.uniform_(-0.2, 0.2)
        bn.running_var.uniform_(0.5, 2.0)
        bn.weight.uniform_(0.5, 1.5)
        bn.bias.uniform_(-0.2, 0.2)
    bn.eval()
    x = torch.randn(2, 8, 12, 12)
    w, b = fold(conv, bn)
    ref = bn(conv(x))
    got = torch.nn.functional.conv2d(x, w, b, 1, 1)
    assert (got - ref).abs().max() / ref.abs().max() < 1e-5


class _Res(torch.nn.Module):
    def __init__(self, c):
        super().__init__()
        mk = lambda act: torch.nn.Sequential(torch.nn.Conv2d(c, c, 3, 1, 1, bias=False), torch.nn.BatchNorm2d(c),
                                             *( [torch.nn.ReLU()] if act else []))
        self.body = torch.nn.Sequential(mk(True), mk(False))
        self.act = torch.nn.ReLU()

    def forward(self, x):
        return self.act(self.body(x) + x)


class _Stem(torch.nn.Module):
    """Same attribute layout as the reference BlockLocalStem (block_local.py:132-153)."""

    def __init__(self, w=(32, 64, 128)):
        super().__init__()
        cba = lambda ci, co, s: torch.nn.Sequential(torch.nn.Conv2d(ci, co, 3, s, 1, bias=False),
                                                    torch.nn.BatchNorm2d(co), torch.nn.ReLU())
        self.stem = torch.nn.Sequential(cba(3, w[0], 2), cba(w[0], w[1], 2))
        self.s4 = torch.nn.Sequential(_Res(w[1]), _Res(w[1]))
        self.down = cba(w[1], w[2], 2)
        self.s8 = torch.nn.Sequential(_Res(w[2]), _Res(w[2]))

    def forward(self, x):
        p4 = self.s4(self.stem(x))
        return p4, self.s8(self.down(p4))


def test_stem_to_local_is_exact():
    torch.manual_seed(0)
    stem = _Stem()
    for b in stem.modules():
        if isinstance(b, torch.nn.BatchNorm2d):
            with torch.no_grad():
                b.running_mean.uniform_(-0.2, 0.2)
                b.running_var.uniform_(0.5, 2.0)
                b.weight.uniform_(0.5, 1.5)
                b.bias.uniform_(-0.2, 0.2)
    stem.eval()
    x = torch.randn(2, 3, 64, 96)
    with torch.no_grad():
        ref = stem(x)[1]
        got = stem_to_local(stem)(x)[1]
    assert (got - ref).abs().max() / ref.abs().max() < 1e-5


def test_streams_statistics():
    s = scenes.Streams(2, 192, 256, seed=1, n_rects=3)
    f0 = s.next()
    f1 = s.next()
    assert f0.dtype == torch.uint8 and f0.shape == (2, 192, 256, 3)
    x = scenes.normalise(f1)
    assert x.dtype == torch.float16
    # noise-only blocks stay below a mean abs diff of 8; rectangles move
    d = (f1.float() - f0.float()).abs().view(2, 6, 32, 8, 32, 3).mean((2, 4, 5))
    assert (d < 8).float().mean() > 0.5 and (d > 8).any()
    g, mask = scenes.forced_change(f1, 0.25, 32, seed=3)
    assert mask.sum().item() == round(0.25 * 2 * 6 * 8)


def test_normalise_matches_prep_formula():
    """(x - MEAN) / STD in fp32 then fp16, MEAN/STD as float32 arrays (video.py:22-23,99)."""
    u = torch.arange(256, dtype=torch.uint8).view(1, 1, 256, 1).expand(1, 1, 256, 3).contiguous()
    got = scenes.normalise(u).float().numpy()
    mean = np.array([0.485, 0.456, 0.406], np.float32) * 255
    std = np.array([0.229, 0.224, 0.225], np.float32) * 255
    ref = ((u.numpy().astype(np.float32) - mean) / std).astype(np.float16).astype(np.float32)
    np.testing.assert_array_equal(got, ref)


def test_m0_helpers_on_cpu():
    """BlockSparseEngine's host helpers (block_sparse.py:115-119,181-192,323-326)."""
    import math
    import torch
    from sarbon_b200 import LocalBackbone
    from sarbon_b200.block_sparse import BlockSparseEngine, _bucket
    assert [_bucket(n) for n in (0, 1, 16, 17, 33, 100, 1024)] == [16, 16, 16, 32, 64, 128, 1024]
    eng = BlockSparseEngine(LocalBackbone(), 32)
    assert eng.dilation(1) == 1 and eng.dilation(32) == 1 and eng.dilation(33) == 2 and eng.dilation(0) == 0
    g = torch.Generator().manual_seed(0)
    prev = torch.rand(3, 64, 96, generator=g)
    cur = prev.clone()
    cur[:, 0:32, 32:64] += 0.25           # block (0, 1) changes by mean 0.25
    ch = eng.changed_blocks(cur, prev, tau=0.2)
    assert ch.tolist() == [[False, True, False], [False, False, False]]
    assert not eng.changed_blocks(cur, prev, tau=0.3).any()
    act = eng.active_blocks(ch, 33)       # d = 2: the whole 2x3 grid
    assert bool(act.all())
    act1 = eng.active_blocks(ch, 10)      # d = 1: 3x3 neighbourhood of (0, 1)
    assert act1.tolist() == [[True, True, True], [True, True, True]]
    act0 = eng.active_blocks(ch, 0)       # d = 0: the block itself
    assert act0.tolist() == ch.tolist()
