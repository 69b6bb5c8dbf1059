"""The M0 API (`sarbon_b200.block_sparse.BlockSparseEngine`) against the reference M0
engine's own outputs (tests/golden/m0/m0_fp32.npz, written by make_m0_golden.py from
sarbon/sparse/block_sparse.py).

fp32, tau > 0 and a capacity of 30 of 60 blocks: steps that fit, a step with more active
blocks than the capacity (overflow: only the first 30 blocks of each dilation are
recomputed, the rest keep their old values), steps with no change at all and with
sub-threshold noise (M0 then recomputes block 0 from its padding entries, with the new
frame already in the image cache).  Per step the overflow flag and the change mask must
equal the reference's, and p4/p8 the reference's within its own fp32 test metric
(max |a - b| / max |b| < 1e-5, tests/test_fused_engine.py:72 of the reference).
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from golden_io import conv_specs, golden_weights, weights_digest

pytestmark = pytest.mark.gpu

FIXTURE = Path(__file__).resolve().parent / "golden" / "m0" / "m0_fp32.npz"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA")


def _load():
    z = np.load(FIXTURE)
    meta = json.loads(bytes(z["meta_json"]).decode())
    ws = golden_weights(conv_specs(meta["nodes"]), meta["seed"])
    assert weights_digest(ws) == meta["weights_sha256"]
    return z, meta, ws


def _rel(a, b):
    b = np.asarray(b, np.float64)
    return float(np.abs(np.asarray(a, np.float64) - b).max() / np.abs(b).max())


def test_m0_step_matches_reference_m0():
    from sarbon_b200 import LocalBackbone
    from sarbon_b200.block_sparse import BlockSparseEngine
    z, meta, ws = _load()
    net = LocalBackbone()
    with torch.no_grad():
        for c, (w, b) in zip([n.conv for n in net.program()[0] if n.kind == "conv"], ws):
            c.weight.copy_(torch.from_numpy(w))
            c.bias.copy_(torch.from_numpy(b))
    eng = BlockSparseEngine(net.cuda().eval(), meta["block"])

    def frame(key):
        return torch.from_numpy(z[key].astype(np.float32) / 256).cuda()

    outs = eng.full(frame("frame0"))
    ref = {"t7": z["full_t7"], "t14": z["full_t14"]}
    for o, name in zip(outs, ("t7", "t14")):
        assert _rel(o.cpu().numpy(), ref[name]) < 1e-5, name
    worst = 0.0
    for i, st in enumerate(meta["steps"]):
        for name in ("t7", "t14"):
            ref[name] = (ref[name].view(np.uint32) ^ z[f"step{i}_{name}_x"]).view(np.float32)
        outs, over = eng.step(frame(f"step{i}_frame"), meta["capacity"], meta["tau"])
        assert bool(over) == st["over"], i
        np.testing.assert_array_equal(eng._eng.changed[0].cpu().numpy(), z[f"step{i}_changed"], f"step {i}")
        for o, name in zip(outs, ("t7", "t14")):
            err = _rel(o.cpu().numpy(), ref[name])
            worst = max(worst, err)
            assert err < 1e-5, (i, name, err)
    assert any(st["over"] for st in meta["steps"]) and not all(st["over"] for st in meta["steps"])
    print(f"\nM0 vs the reference M0: worst max-abs / max-ref {worst:.2e}")
