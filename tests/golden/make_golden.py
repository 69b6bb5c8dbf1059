"""Generate golden vectors by running the reference engine itself on CPU.

Run once in a container that has the reference checkout (its path is the first,
required argument); the GPU tests only read the ``.npz`` files written next to this
script and never need the reference.

The reference ``FusedSparseEngine`` (sarbon/sparse/fused_engine.py) normally runs
on CUDA with CUDA graphs; here it runs on CPU with Triton's interpreter
(``TRITON_INTERPRET=1``) and four stubs: a no-op graph pool handle, a current
stream with ``synchronize()``, identity ``pin_memory`` and a ``_capture`` that
replays the body eagerly. Every number in the fixtures comes from the
reference's own code: its gate, its ``nonzero_static`` lists, its Triton tile
kernel (interpreted) and its dense ``F.conv2d`` path.

Usage: python tests/golden/make_golden.py /path/to/reference [case ...]
"""
import os
import sys
import time
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

OUT = Path(__file__).resolve().parent
if len(sys.argv) < 2:
    sys.exit("usage: make_golden.py /path/to/reference [case ...]")
REF = Path(sys.argv[1])
sys.path.insert(0, str(REF))
sys.path.insert(0, str(OUT.parent))
sys.path.insert(0, str(OUT.parent.parent))
from golden_io import conv_specs, golden_weights, weights_digest  # noqa: E402

from sarbon.sparse import LocalBackbone  # noqa: E402
from sarbon.sparse import fused_engine as fe  # noqa: E402


class _Graph:
    def __init__(self, body):
        self.body = body

    def replay(self):
        self.body()


class _Stream:
    def synchronize(self):
        pass


def _install_cpu_stubs():
    torch.cuda.graph_pool_handle = lambda: None
    torch.cuda.current_stream = lambda *a, **k: _Stream()
    torch.Tensor.pin_memory = lambda self, *a, **k: self

    def capture(self, body, pool=None):
        body()
        return _Graph(body)

    fe.FusedSparseEngine._capture = capture


def _net_arrays(net):
    """Conv weights/biases and program topology, in program order."""
    nodes, outs = net.program()
    rec = []
    for n in nodes:
        d = {"kind": n.kind, "src": list(n.src), "dst": n.dst, "stride": n.stride,
             "radius": n.radius, "act": bool(n.act)}
        if n.kind == "conv":
            d["cout"], d["cin"] = n.conv.out_channels, n.conv.in_channels
            d["conv_stride"] = n.conv.stride[0]
        rec.append(d)
    return rec, outs


def _rect(frames, cam, y, x, h, w, value):
    frames[cam, y:y + h, x:x + w] = value


def _all_caches(eng):
    return {k: v.float().numpy().copy() for k, v in eng.cache.items()}


def run_case(name, dtype, n_cams, h, w, block, tau, refresh, domain, seed, steps, all_caches=False):
    """Drive the reference engine through `steps` and record everything it produced.
    With ``all_caches`` every cache (image and all layers) is also kept after the reset
    and after the last step, for layer-by-layer checks from the reference's own inputs."""
    torch.manual_seed(seed)
    net = LocalBackbone().eval()
    # replace the random init by the seeded, fp16-representable weights of golden_io
    topo, _ = _net_arrays(net)
    ws = golden_weights(conv_specs(topo), seed)
    convs = [n.conv for n in net.program()[0] if n.kind == "conv"]
    with torch.no_grad():
        for c, (cw, cb) in zip(convs, ws):
            c.weight.copy_(torch.from_numpy(cw))
            c.bias.copy_(torch.from_numpy(cb))
    net = net.to(dtype)
    digest = weights_digest(ws)
    eng = fe.FusedSparseEngine(net, n_cams, h, w, block=block, dtype=dtype, tau=tau,
                               refresh=refresh, device="cpu")
    g = torch.Generator().manual_seed(seed + 1)
    scene = None
    if domain == "unit":
        frames = torch.rand(n_cams, h, w, 3, generator=g).to(dtype)
    elif domain == "norm":  # the bench's camera streams, normalised as SarbonVideo._prep does
        from sarbon_b200 import scenes
        scene = scenes.Streams(n_cams, h, w, seed=seed, n_rects=1)
        frames = scenes.normalise(scene.next(), dtype)
    else:  # integer-valued raw 0..255 frames
        frames = torch.randint(0, 256, (n_cams, h, w, 3), generator=g).to(dtype)
    rec = {"frames0": frames.float().numpy().astype(np.float16 if dtype == torch.float16 else np.float32, copy=True)}
    t0 = time.time()
    eng.reset(frames)
    rec["reset_t7"] = eng.cache["t7"].float().numpy().copy()
    rec["reset_t14"] = eng.cache["t14"].float().numpy().copy()
    if all_caches:
        rec["reset_caches"] = _all_caches(eng)
    log = []
    for i, ev in enumerate(steps):
        frames = frames.clone()
        kind = ev[0]
        if kind == "rect":
            _, cam, y, x, hh, ww = ev
            val = torch.rand(3, generator=g) if domain == "unit" else torch.randint(0, 256, (3,), generator=g).float()
            _rect(frames, cam, y, x, hh, ww, val.to(dtype))
        elif kind == "noise":  # small +-1 perturbation everywhere (below tau for raw frames)
            if domain == "unit":
                frames = (frames.float() + (torch.rand(frames.shape, generator=g) - 0.5) * 0.02).to(dtype)
            else:
                frames = (frames.float() + torch.randint(-1, 2, frames.shape, generator=g)).clamp(0, 255).to(dtype)
        elif kind == "extra":
            _, cam, by, bx = ev
            m = torch.zeros_like(eng.extra)
            m[cam, by, bx] = True
            eng.set_extra(m)
        elif kind == "clear_extra":
            eng.set_extra(torch.zeros_like(eng.extra))
        elif kind == "scene":  # next frame of the camera streams
            from sarbon_b200 import scenes
            frames = scenes.normalise(scene.next(), dtype)
        elif kind == "same":
            pass
        mode, k = eng.step(frames)
        step = {"mode": mode, "k": k, "frames": frames.float().numpy().copy(),
                "extra": eng.extra.numpy().copy()}
        if k >= 0:
            step["changed"] = eng.changed.numpy().copy()
            step["masks"] = {d: eng.masks[d].numpy().copy() for d in eng.ds}
            if mode == "sparse":
                cap = eng._bucket(k)
                step["cap"] = cap
                per = eng.hb * eng.wb
                lists = {}
                for d in eng.ds:
                    flat = torch.nonzero_static(eng.masks[d].flatten(), size=cap, fill_value=0)[:, 0]
                    r = flat % per
                    lists[d] = np.stack([(flat // per).numpy(), (r // eng.wb).numpy(),
                                         (r % eng.wb).numpy()]).astype(np.int32)
                step["lists"] = lists
        # copies: for fp32, .float().numpy() would alias the live cache that later steps update
        step["t7"] = eng.cache["t7"].float().numpy().copy()
        step["t14"] = eng.cache["t14"].float().numpy().copy()
        log.append(step)
        print(f"  {name} step {i}: {mode} k={k}", flush=True)
    rec["steps"] = log
    if all_caches:
        rec["final_caches"] = _all_caches(eng)
    print(f"{name}: {time.time() - t0:.1f}s", flush=True)
    nodes, outs = _net_arrays(net)
    rec["weight_seed"], rec["weights_sha256"] = seed, digest
    return rec, nodes, outs, eng


def _bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint16 if a.dtype == np.float16 else np.uint32)


def save(name, meta, rec, nodes, outs, eng):
    """Frames and caches are stored as bit-XOR deltas against the previous step: exactly
    invertible, and zero wherever nothing changed (so they compress)."""
    fdt = np.float16 if meta["dtype"] == "float16" else np.float32
    raw = meta["domain"] == "raw"
    arrays = {"frames0": rec["frames0"].astype(np.uint8) if raw else rec["frames0"].astype(fdt),
              "reset_t7": rec["reset_t7"].astype(fdt), "reset_t14": rec["reset_t14"].astype(fdt)}
    prev = {"frames": rec["frames0"].astype(fdt), "t7": rec["reset_t7"].astype(fdt),
            "t14": rec["reset_t14"].astype(fdt)}
    for i, s in enumerate(rec["steps"]):
        p = f"step{i}_"
        cur = {"frames": s["frames"].astype(fdt), "t7": s["t7"].astype(fdt), "t14": s["t14"].astype(fdt)}
        for key in ("frames", "t7", "t14"):
            arrays[p + key + "_x"] = _bits(cur[key]) ^ _bits(prev[key])
        prev = cur
        arrays[p + "extra"] = s["extra"]
        if "changed" in s:
            arrays[p + "changed"] = s["changed"]
            for d, m in s["masks"].items():
                arrays[p + f"mask{d}"] = m
        if "lists" in s:
            for d, l in s["lists"].items():
                arrays[p + f"list{d}"] = l
    for when in ("reset", "final"):
        if when + "_caches" in rec:
            for key, v in rec[when + "_caches"].items():
                arrays[f"{when}_cache_{key}"] = v.astype(fdt)
    steps = [{"mode": s["mode"], "k": int(s["k"]), "cap": int(s.get("cap", 0))} for s in rec["steps"]]
    topo = nodes
    import json
    arrays["meta_json"] = np.frombuffer(json.dumps({
        **{k: v for k, v in meta.items() if k != "all_caches"}, "all_caches": bool(meta.get("all_caches")),
        "weight_seed": rec["weight_seed"], "weights_sha256": rec["weights_sha256"], "steps": steps, "nodes": topo, "outputs": list(outs), "ds": list(eng.ds),
        "buckets": list(eng.buckets), "hb": eng.hb, "wb": eng.wb}).encode(), np.uint8)
    np.savez_compressed(OUT / f"{name}.npz", **arrays)
    print(f"wrote {name}.npz ({(OUT / f'{name}.npz').stat().st_size / 1e6:.2f} MB)", flush=True)


# SarbonVideo's engine threshold for its default-style tau of 8 grey levels, computed as
# video.py:63-64 computes it: tau * 255 / float(STD.mean()) with STD the float32 array
_STD = np.array([0.229, 0.224, 0.225], np.float32) * 255
TAU_8_GREY = (8 / 255) * 255 / float(_STD.mean())

CASES = {
    # the reference test's own scenario (tests/test_fused_engine.py:24-45), smaller frames
    "unit_fp32_b32": dict(dtype=torch.float32, n_cams=2, h=96, w=160, block=32, tau=0.0, refresh=0,
                          domain="unit", seed=0,
                          steps=[("rect", 0, 7, 13, 37, 51), ("rect", 1, 47, 73, 37, 51),
                                 ("rect", 0, 60, 120, 28, 40), ("same",)]),
    "unit_fp16_b32": dict(dtype=torch.float16, n_cams=2, h=128, w=192, block=32, tau=0.0, refresh=0,
                          domain="unit", seed=3,
                          steps=[("rect", 1, 40, 100, 37, 51), ("rect", 0, 0, 160, 30, 32),
                                 ("same",)]),
    # block 64: every layer has dilation 1
    "unit_fp32_b64": dict(dtype=torch.float32, n_cams=1, h=128, w=192, block=64, tau=0.0, refresh=0,
                          domain="unit", seed=5, steps=[("rect", 0, 70, 20, 30, 30)]),
    # raw 0..255 frames, tau > 0: noise below the threshold, extra mask, refresh phase
    "raw_tau_fp32": dict(dtype=torch.float32, n_cams=2, h=96, w=160, block=32, tau=8.0, refresh=4,
                         domain="raw", seed=7,
                         steps=[("noise",), ("rect", 0, 30, 40, 20, 50), ("extra", 1, 2, 3),
                                ("clear_extra",), ("noise",)]),
    # the production gate setting: normalised fp16 camera frames (SarbonVideo._prep) with
    # tau = 8 grey levels (SarbonVideo(tau=8/255), video.py:63-64), refresh and an extra
    # mask; every cache kept after the reset and after the last step
    "norm_tau_fp16": dict(dtype=torch.float16, n_cams=2, h=96, w=192, block=32,
                          tau=TAU_8_GREY, refresh=5,
                          domain="norm", seed=11, all_caches=True,
                          steps=[("scene",), ("scene",), ("extra", 1, 1, 4), ("scene",), ("clear_extra",),
                                 ("scene",)]),
}


def main():
    _install_cpu_stubs()
    torch.set_num_threads(os.cpu_count() or 1)
    only = set(sys.argv[2:])
    for name, cfg in CASES.items():
        if only and name not in only:
            continue
        meta = {k: (str(v).replace("torch.", "") if k == "dtype" else v)
                for k, v in cfg.items() if k != "steps"}
        rec, nodes, outs, eng = run_case(name, **cfg)
        save(name, meta, rec, nodes, outs, eng)


if __name__ == "__main__":
    main()
