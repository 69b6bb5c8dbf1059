"""Golden vectors of the reference's M0 engine (BlockSparseEngine, sarbon/sparse/block_sparse.py).

Run once in a container with the reference checkout (its path is the first, required
argument); the GPU tests read only the .npz written next to this script.

M0's `full` and `update(graph=False)` run on CPU as they are.  Its `step` captures a CUDA
graph around a body of the reference's own calls (block_sparse.py:264-275); here that
body runs eagerly with the same calls in the same order: `changed_blocks(frame, prev, tau)`,
per dilation `active_blocks` + `nonzero_static(size=capacity, fill_value=0)` and the
overflow test, the whole-frame image copy, `_run(lists)`, then prev <- frame.  Inputs:
fp32 unit frames with moving squares, tau > 0, a capacity small enough to overflow at some
steps.  Recorded per step: overflow, the change mask and the p4/p8 outputs.  Frames are
multiples of 1/256 (stored as uint8, exact in fp32); outputs are stored as bit-XOR deltas
against the previous step's (zero where nothing changed, so they compress).

Usage: python tests/golden/make_m0_golden.py /path/to/reference
"""
import json
import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent
if len(sys.argv) < 2:
    sys.exit("usage: make_m0_golden.py /path/to/reference")
sys.path.insert(0, sys.argv[1])
sys.path.insert(0, str(OUT.parent))
from golden_io import conv_specs, golden_weights, weights_digest  # noqa: E402

from sarbon.sparse import LocalBackbone  # noqa: E402
from sarbon.sparse.block_sparse import BlockSparseEngine  # noqa: E402


def step_body(eng, frame, prev, capacity, tau):
    """The body BlockSparseEngine.step captures (block_sparse.py:264-275), run eagerly."""
    hb, wb = (s // eng.block for s in eng._interior("img").shape[1:])
    ds = sorted({eng.dilation(n.radius) for n in eng.nodes})
    changed = eng.changed_blocks(frame, prev, tau)
    lists, over = {}, torch.zeros((), dtype=torch.bool)
    for d in ds:
        m = eng.active_blocks(changed, d * eng.block).flatten()
        flat = torch.nonzero_static(m, size=capacity, fill_value=0)[:, 0]
        lists[d] = (flat // wb, flat % wb, capacity)
        over = over | (m.sum() > capacity)
    eng._interior("img").copy_(frame)
    eng._run(lists)
    return changed, bool(over)


def main():
    seed, h, w, block, tau, capacity = 17, 192, 320, 32, 0.05, 30
    torch.manual_seed(seed)
    net = LocalBackbone().eval()
    topo = []
    for n in net.program()[0]:
        d = {"kind": n.kind, "src": list(n.src), "dst": n.dst, "stride": n.stride, "radius": n.radius,
             "act": bool(n.act)}
        if n.kind == "conv":
            d["cout"], d["cin"] = n.conv.out_channels, n.conv.in_channels
            d["conv_stride"] = n.conv.stride[0]
        topo.append(d)
    ws = golden_weights(conv_specs(topo), seed)
    with torch.no_grad():
        for c, (cw, cb) in zip([n.conv for n in net.program()[0] if n.kind == "conv"], ws):
            c.weight.copy_(torch.from_numpy(cw))
            c.bias.copy_(torch.from_numpy(cb))
    eng = BlockSparseEngine(net, block)
    g = torch.Generator().manual_seed(seed + 1)
    def q(x):  # multiples of 1/256 in [0, 1): exact in fp32, stored as uint8
        return (x * 256).floor().clamp(0, 255) / 256

    def u8(x):
        return (x * 256).round().to(torch.uint8).numpy()

    def bits(a):
        return np.ascontiguousarray(a).view(np.uint32)

    frame = q(torch.rand(3, h, w, generator=g))
    arrays = {"frame0": u8(frame)}
    with torch.no_grad():
        outs = eng.full(frame)
        arrays["full_t7"], arrays["full_t14"] = (o.numpy().copy() for o in outs)
        last = {"t7": arrays["full_t7"], "t14": arrays["full_t14"]}
        prev, steps = frame.clone(), []
        # moving squares: (y, x, side); small steps fit the capacity, large ones overflow;
        # the last one has tiny changes below tau
        plan = [[(40, 40, 20)], [(10, 10, 24), (150, 280, 30), (64, 128, 32)], [(100, 200, 20)], [], "noise",
                [(0, 0, 12)]]
        for i, sq in enumerate(plan):
            f = prev.clone()
            if sq == "noise":
                f = q((f + (torch.rand(f.shape, generator=g) - 0.5) * 0.04).clamp(0, 1))
            else:
                for y, x, s in sq:
                    f[:, y:y + s, x:x + s] = q(torch.rand(3, 1, 1, generator=g))
            changed, over = step_body(eng, f, prev, capacity, tau)
            prev = f.clone()
            arrays[f"step{i}_frame"] = u8(f)
            arrays[f"step{i}_changed"] = changed.numpy().copy()
            cur = {"t7": eng._interior("t7").numpy().copy(), "t14": eng._interior("t14").numpy().copy()}
            for k in ("t7", "t14"):
                arrays[f"step{i}_{k}_x"] = bits(cur[k]) ^ bits(last[k])
            last = cur
            steps.append({"over": over, "changed": int(changed.sum())})
            print(f"step {i}: changed {int(changed.sum())} over {over}", flush=True)
    meta = {"seed": seed, "h": h, "w": w, "block": block, "tau": tau, "capacity": capacity, "steps": steps,
            "weights_sha256": weights_digest(ws), "nodes": topo, "outputs": list(eng.outputs)}
    arrays["meta_json"] = np.frombuffer(json.dumps(meta).encode(), np.uint8)
    (OUT / "m0").mkdir(exist_ok=True)
    np.savez_compressed(OUT / "m0" / "m0_fp32.npz", **arrays)
    print("wrote m0/m0_fp32.npz")


if __name__ == "__main__":
    main()
