"""Readers for the golden fixtures written by ``tests/golden/make_golden.py``.

Each fixture holds what the reference engine (run on CPU) produced: the network
weights and topology, the frame sequence, and per step the mode, active count,
change mask, dilated masks, budget-padded block lists and the p4/p8 caches.
Frames and caches are stored as bit-XOR deltas against the previous step.
"""
import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("*.npz"))


def _unx(prev, x):
    dt = prev.dtype
    return (prev.view(x.dtype) ^ x).view(dt)


def load(name):
    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(bytes(z["meta_json"]).decode())
    fdt = np.float16 if meta["dtype"] == "float16" else np.float32
    nodes = [dict(n) for n in meta["nodes"]]
    ws = golden_weights(conv_specs(nodes), meta["weight_seed"])
    assert weights_digest(ws) == meta["weights_sha256"], "golden weights drifted"
    it = iter(ws)
    for n in nodes:
        if n["kind"] == "conv":
            n["w"], n["b"] = next(it)
    frames = z["frames0"].astype(fdt)
    t7, t14 = z["reset_t7"].astype(fdt), z["reset_t14"].astype(fdt)
    case = {"meta": meta, "nodes": nodes, "frames0": frames, "reset": {"t7": t7, "t14": t14},
            "dtype": fdt, "steps": []}
    for i, s in enumerate(meta["steps"]):
        p = f"step{i}_"
        frames = _unx(frames, z[p + "frames_x"])
        t7 = _unx(t7, z[p + "t7_x"])
        t14 = _unx(t14, z[p + "t14_x"])
        st = dict(s, frames=frames, t7=t7, t14=t14, extra=z[p + "extra"])
        if p + "changed" in z:
            st["changed"] = z[p + "changed"]
            st["masks"] = {d: z[p + f"mask{d}"] for d in meta["ds"]}
        if p + f"list{meta['ds'][0]}" in z:
            st["lists"] = {d: z[p + f"list{d}"] for d in meta["ds"]}
        case["steps"].append(st)
    for when in ("reset", "final"):
        pre = f"{when}_cache_"
        caches = {k[len(pre):]: z[k].astype(fdt) for k in z.files if k.startswith(pre)}
        if caches:
            case[when + "_caches"] = caches
    return case


def feature_tol(dtype):
    """(rtol, atol) of the parity checks: fp16 1e-2 relative / 1e-3 absolute (north
    star), fp32 1e-5 (the reference's own test, tests/test_fused_engine.py:72)."""
    return (1e-2, 1e-3) if dtype == np.float16 else (1e-5, 1e-6)


def fp16_ulp(x):
    """Spacing of fp16 numbers at |x| (one unit in the last place)."""
    return np.spacing(np.abs(np.asarray(x, np.float16))).astype(np.float64)


def assert_close(a, b, dtype, what="", extra_ulps=0):
    """fp16: every element within 1e-3 + 1e-2 * |b| (elementwise), widened by
    ``extra_ulps`` fp16 units of the map's largest value for outputs that went through
    several layers of independently rounded fp16 caches (each layer rounds its fp32
    accumulation once; two implementations that sum in different orders differ by an
    ulp here and there, and those differences travel through the later layers).
    fp32: max-abs / max-ref below 1e-5, exactly the reference test's check.
    Returns the largest error as a multiple of the bound."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    rtol, atol = feature_tol(dtype)
    if dtype == np.float16:
        bound = atol + rtol * np.abs(b) + extra_ulps * fp16_ulp(np.abs(b).max())
        err = np.abs(a - b)
        worst = float((err / bound).max()) if err.size else 0.0
        assert (err <= bound).all(), (f"{what}: {(err > bound).sum()} of {err.size} elements above "
                                      f"1e-3 + 1e-2|b| + {extra_ulps} ulp(max|b|); max abs err {err.max():.3g}, "
                                      f"worst err/bound {worst:.3g}")
        return worst
    else:
        err = np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)
        assert err < rtol, f"{what}: max rel err {err:.3g} >= {rtol}"
        return float(err / rtol)


# fp16 allowance of the end-to-end outputs checked against the reference's own caches:
# p4 (t7, 8 conv layers deep) and p8 (t14, 11 layers) are held to the elementwise
# 1e-2 / 1e-3 bar plus 2 and 4 fp16 ulps of the map's largest value.  Measured for the
# oracle against the reference over every fp16 fixture: at most 0.11 ulp (t7) and 0.78 ulp
# (t14) beyond the plain bar.  Every single layer, computed from the reference's own input
# caches, meets the plain elementwise bar with no allowance
# (tests/test_gpu_golden_layers.py, test_oracle_every_layer_from_reference_inputs).
OUTPUT_ULPS = {"t7": 2, "t14": 4}


def golden_weights(convs, seed):
    """Deterministic conv weights for the fixtures (numpy PCG64, platform-independent):
    kaiming-normal scale, bias N(0, 0.01), the second conv of each residual block
    halved, every value rounded to fp16 so fp16 and fp32 engines see the same numbers.
    ``convs`` is a list of (cout, cin, k, is_second_of_res)."""
    rng = np.random.default_rng(seed)
    out = []
    for cout, cin, k, second in convs:
        w = rng.standard_normal((cout, cin, k, k)) * np.sqrt(2.0 / (cin * k * k))
        if second:
            w *= 0.5
        b = rng.standard_normal(cout) * 0.01
        out.append((w.astype(np.float16).astype(np.float32), b.astype(np.float16).astype(np.float32)))
    return out


def weights_digest(ws):
    import hashlib
    h = hashlib.sha256()
    for w, b in ws:
        h.update(np.ascontiguousarray(w).tobytes())
        h.update(np.ascontiguousarray(b).tobytes())
    return h.hexdigest()


def conv_specs(nodes):
    """(cout, cin, k, is_second_of_res) for the conv nodes of a program, in order."""
    specs = []
    for i, n in enumerate(nodes):
        if n["kind"] != "conv":
            continue
        nxt = nodes[i + 1] if i + 1 < len(nodes) else None
        second = nxt is not None and nxt["kind"] == "add" and nxt["src"][0] == n["dst"]
        specs.append((n["cout"], n["cin"], 3, second))
    return specs
