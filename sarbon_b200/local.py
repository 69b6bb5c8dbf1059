"""Stem topology the block-sparse engine executes, and BatchNorm folding.

Mirrors the reference interface so that networks built here and networks built by
the reference (``sarbon.sparse.LocalBackbone``, ``sarbon.sparse.convert.stem_to_local``)
are interchangeable inputs of :class:`sarbon_b200.FusedSparseEngine`:

* ``Node`` / ``LocalBackbone.program()``  -- sarbon/sparse/block_sparse.py:25-33, 78-113:
  a flat list of conv / add nodes with output names ``t0, t1, ...``, the output stride of
  each node and its cumulative receptive radius in image pixels
  (``radius = r_in + (k // 2) * s_in``; an add takes the max of its inputs).
* ``fold`` / ``stem_to_local``            -- sarbon/sparse/convert.py:14-44.

The engine only reads ``program()``; the module's ``forward`` is the dense fp32 PyTorch
reference used by the numerics tests.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass
class Node:
    kind: str             # "conv" or "add"
    src: tuple            # input cache names
    dst: str              # output cache name
    stride: int           # output feature stride w.r.t. the image
    radius: int           # cumulative receptive radius (image pixels)
    conv: nn.Conv2d = None
    act: bool = True


class ConvAct(nn.Module):
    """3x3 conv with bias (a folded Conv-BN) and optional ReLU."""

    def __init__(self, cin, cout, stride=1, act=True):
        super().__init__()
        self.conv = nn.Conv2d(cin, cout, 3, stride, 1, bias=True)
        nn.init.kaiming_normal_(self.conv.weight, nonlinearity="relu")
        nn.init.normal_(self.conv.bias, std=0.01)
        self.act = act

    def forward(self, x):
        y = self.conv(x)
        return F.relu(y) if self.act else y


class ResBlock(nn.Module):
    """relu(conv(relu(conv(x))) + x); the second conv is scaled down at init."""

    def __init__(self, c):
        super().__init__()
        self.c1 = ConvAct(c, c)
        self.c2 = ConvAct(c, c, act=False)
        with torch.no_grad():
            self.c2.conv.weight.mul_(0.5)

    def forward(self, x):
        return F.relu(self.c2(self.c1(x)) + x)


class LocalBackbone(nn.Module):
    """Stride-2 conv, stride-2 conv, Res x blocks[0] (stride 4, output p4), stride-2 conv,
    Res x blocks[1] (stride 8, output p8).  Sarbon-S widths are (32, 64, 128)."""

    def __init__(self, w=(32, 64, 128), blocks=(2, 2)):
        super().__init__()
        self.stem1 = ConvAct(3, w[0], 2)
        self.stem2 = ConvAct(w[0], w[1], 2)
        self.stage4 = nn.Sequential(*[ResBlock(w[1]) for _ in range(blocks[0])])
        self.down = ConvAct(w[1], w[2], 2)
        self.stage8 = nn.Sequential(*[ResBlock(w[2]) for _ in range(blocks[1])])

    def forward(self, x):
        p4 = self.stage4(self.stem2(self.stem1(x)))
        return p4, self.stage8(self.down(p4))

    def program(self):
        nodes = []
        cur = {"name": "img", "stride": 1, "radius": 0}
        counter = [0]

        def fresh():
            name = f"t{counter[0]}"
            counter[0] += 1
            return name

        def conv(unit):
            c = unit.conv
            radius = cur["radius"] + (c.kernel_size[0] // 2) * cur["stride"]
            stride = cur["stride"] * c.stride[0]
            dst = fresh()
            nodes.append(Node("conv", (cur["name"],), dst, stride, radius, c, unit.act))
            cur.update(name=dst, stride=stride, radius=radius)

        def res(block):
            skip = dict(cur)
            conv(block.c1)
            conv(block.c2)
            dst = fresh()
            radius = max(cur["radius"], skip["radius"])
            nodes.append(Node("add", (cur["name"], skip["name"]), dst, skip["stride"], radius))
            cur.update(name=dst, radius=radius)

        conv(self.stem1)
        conv(self.stem2)
        for b in self.stage4:
            res(b)
        p4 = cur["name"]
        conv(self.down)
        for b in self.stage8:
            res(b)
        return nodes, (p4, cur["name"])


@torch.no_grad()
def fold(conv, bn):
    """Conv followed by inference BatchNorm -> (weight, bias) of one conv."""
    scale = bn.weight / (bn.running_var + bn.eps).sqrt()
    w = conv.weight * scale.view(-1, 1, 1, 1)
    b = bn.bias - bn.running_mean * scale
    if conv.bias is not None:
        b = b + conv.bias * scale
    return w, b


@torch.no_grad()
def stem_to_local(stem) -> LocalBackbone:
    """Map a Sarbon ``BlockLocalStem`` (block_type='res', ReLU) onto a LocalBackbone with
    BatchNorm folded into every conv.  Duck-typed on the stem's attributes
    (``stem.stem[i][0|1]``, ``stem.s4``, ``stem.down``, ``stem.s8``, ``block.body[j]``)."""
    s4, s8 = list(stem.s4), list(stem.s8)
    for b in s4 + s8:
        if not hasattr(b, "body") or len(b.body) != 2:
            raise ValueError("only residual blocks (block_type='res') map onto LocalBackbone")
    if not isinstance(getattr(s4[0], "act", None), nn.ReLU):
        raise ValueError("only ReLU stems map onto LocalBackbone")
    widths = (stem.stem[0][0].out_channels, stem.stem[1][0].out_channels, stem.down[0].out_channels)
    net = LocalBackbone(widths, (len(s4), len(s8)))

    def put(dst, seq):
        w, b = fold(seq[0], seq[1])
        dst.conv.weight.copy_(w)
        dst.conv.bias.copy_(b)

    put(net.stem1, stem.stem[0])
    put(net.stem2, stem.stem[1])
    put(net.down, stem.down)
    for src, dst in zip(s4 + s8, list(net.stage4) + list(net.stage8)):
        put(dst.c1, src.body[0])
        put(dst.c2, src.body[1])
    return net.eval()
