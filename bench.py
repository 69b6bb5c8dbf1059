#!/usr/bin/env python
"""Benchmark: frames/s of the B200 temporal block-sparse stem engine at 1080p with ~5%
changed blocks, plus the tile-conv roofline fraction.

Workload (one "step" = one frame of every stream on the GPU): S independent 1920x1088
camera streams per GPU (default 16, the reference's own 16-camera M1 benchmark,
bench/bench_m1.py:148-151), seeded synthetic content (blurred-noise background, N(0,2)
sensor noise, moving filled rectangles tuned to ~5% changed 32 px blocks per frame),
Sarbon-S stem widths (32/64/128) with random-init weights, fp16 caches, change threshold
8 grey levels of mean abs diff.  Frames are pre-staged in HBM (normalised fp16, as the
engine input); every step reads S x 12.5 MB of new frames plus the image cache, far more
than the 126 MB L2, so no L2 flush is needed.

Arms:
  --impl b200 (default)  the CUDA engine; `value` is device-timed frames/s with inputs in
                         HBM; `e2e` runs the same steps through the public API from pinned
                         host uint8 BGR frames (H2D copy of every frame and a D2H read of
                         every step's {mode, count} inside the timed region).
  --impl reference       the reference's own CPU path for the stem features on the host
                         cores: with no CUDA device SarbonVideo runs the dense stem every
                         frame (sarbon/inference/video.py:101-104), i.e. the reference's
                         LocalBackbone forward in fp32 (installed under baseline/_ref); the
                         numpy oracle that restates the sparse engine when it is absent.

Multi-GPU (torchrun): streams are independent; each rank runs its own shard of the
streams with no collective inside the timed region; the time is the max over ranks.
Weak scaling (default): S streams per GPU.  Strong scaling (--total-streams T, e.g. a
fixed job of 64 streams of 1280x720 padded to 736 rows over 1/2/4/8 GPUs): the job's T
streams split contiguously over the ranks.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "frames/s/GPU at 1080p, 5% changed blocks; stem tile-conv % of tensor/HBM roofline"
UNIT = "frames/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=1000)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--streams", type=int, default=16, help="camera streams per GPU (weak scaling)")
    p.add_argument("--total-streams", type=int, default=0,
                   help="streams of the whole job split over the GPUs (strong scaling; 0 = weak)")
    p.add_argument("--height", type=int, default=1088)
    p.add_argument("--camera-height", type=int, default=0,
                   help="camera frame height, zero-padded at the bottom to --height (0 = --height)")
    p.add_argument("--width", type=int, default=1920)
    p.add_argument("--rects", type=int, default=0, help="moving rectangles per stream (0 = auto for ~5%%)")
    p.add_argument("--frames", type=int, default=16, help="distinct frames staged per stream")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--e2e-steps", type=int, default=200)
    p.add_argument("--profile-steps", type=int, default=24)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-stats", action="store_true", help="skip the untimed statistics cycle")
    p.add_argument("--no-masks", action="store_true", help="skip timing the mask utility kernels")
    p.add_argument("--cell", type=int, default=0,
                   help="gate at cell level with this cell size (px; 0 = block level, the reference's rule)")
    p.add_argument("--fp8", nargs="?", const="s8", default=None, choices=["s8", "all"],
                   help="e4m3 caches and per-output-channel e4m3 weights (the full-detection benchmark's weight "
                        "format): in the stride-8 stage "
                        "(s8, SB_CREATE_FP8_S8) or in the stride-4 stage too (all)")
    p.add_argument("--cpu-seconds", type=float, default=20.0)
    p.add_argument("--no-reference-gpu", action="store_true",
                   help="skip timing the reference's own Triton engine on the GPU (rank 0, N = 1)")
    p.add_argument("--reference-gpu-steps", type=int, default=60)
    p.add_argument("--no-detector", action="store_true",
                   help="skip timing the detector after the stem (B200Detector vs the reference's own)")
    p.add_argument("--detector-iters", type=int, default=20)
    p.add_argument("--dec-layers", type=int, default=4,
                   help="decoder layers of the detector (the 's' preset has 4; the full-detection benchmark uses 6)")
    return p.parse_args()


# ----------------------------------------------------------------------------- helpers
def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def auto_rects(h, w):
    """Rectangles per stream for ~5% changed 32 px blocks (calibrated on the generator at
    1080p: each moving 40-120 px rectangle changes ~7 blocks per frame at 8 grey levels)."""
    return max(1, round(0.05 * (h // 32) * (w // 32) / 7))


def pingpong(n):
    return list(range(n)) + list(range(n - 2, 0, -1))


# DRAM bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum) of one capture of
# the default workload (16 streams x 1920x1088, ~5 % changed blocks) per cache format (key:
# the --fp8 choice); they describe the kernels as they were at that capture, named in
# "capture".  None: not captured.
TRAFFIC = {
    None: {"conv": 71.9e6, "gate": 419.0e6,
           "capture": "ncu dram__bytes_read.sum + dram__bytes_write.sum per launch, 16 streams x "
                      "1920x1088 (--frames 4), two timed steps, commit fc1b017: conv = the mean over "
                      "its 22 launches, gate = the mean over 2"},
    "s8": {"conv": 68.4e6, "gate": 419.7e6,
           "capture": "ncu dram__bytes_read.sum + dram__bytes_write.sum per launch, 16 streams x "
                      "1920x1088 (--frames 4, --fp8 s8), one sparse step of the profile pass, commit "
                      "534d084: conv = the mean over its 11 launches, gate = the mean over 2"},
    "all": {"conv": 51.2e6, "gate": 419.7e6,
            "capture": "ncu dram__bytes_read.sum + dram__bytes_write.sum per launch, 16 streams x "
                       "1920x1088 (--frames 4, --fp8 all), one sparse step of the profile pass, commit "
                       "534d084: conv = the mean over its 11 launches, gate = the mean over 2"},
}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return d, "measured"
        except Exception:
            pass
    return FALLBACK_PEAKS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms in the background."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


def layer_flops(eng, counts, mode):
    """Algorithmic conv FLOPs of one step per layer: 2*cin*cout*9*t^2 per active tile,
    counted on the real active counts k_d (dense: every block)."""
    out = []
    for l in eng.layers:
        t = eng.block // l.out_stride
        k = eng.n_blocks if mode == "dense" else counts[eng.ds.index(eng.dilation(l.radius))]
        out.append(2 * l.w_tile.shape[2] * l.w_tile.shape[3] * 9 * t * t * k)
    return out


def gate_bytes(eng, n_changed):
    """Algorithmic bytes of the gate kernel: read the frames and the image cache (fp16),
    write the changed blocks into the image cache (block^2 * 3 fp16 each), read the extra
    mask and write the change mask (one byte per block each)."""
    px = eng.n * eng.h * eng.w * 3
    return 2 * px * 2 + n_changed * eng.block * eng.block * 3 * 2 + 2 * eng.n_blocks


def mma_flops(eng, mode):
    """FLOPs the tile-conv kernels issue on the tensor cores in one step, per layer:
    2 x 128-row M-tiles x 128 x C_out x issued K.  Above the algorithmic FLOPs because
    window layers compute whole regions (inactive blocks inside an active region too),
    the first layer pads its 27 taps to K = 32 and the 32-channel stride-2 layer issues
    6 K-blocks of 64 for its 9 x 32 taps."""
    import torch.nn.functional as F
    out = []
    for l, m in zip(eng.layers, eng.layer_variants()):
        t = eng.block // l.out_stride
        cin, cout = l.w_tile.shape[2], l.w_tile.shape[3]
        win = m & 7
        rw, rh = (8 // t, 16 // t if win == 3 else 1) if win else (1, 1)
        mask = eng.masks[eng.dilation(l.radius)]
        if mode == "dense":
            mask = torch.ones_like(mask)
        if rw * rh > 1:
            units = int(F.max_pool2d(mask.float()[:, None], (rh, rw), (rh, rw), ceil_mode=True).sum())
        else:
            units = int(mask.sum())
        upx = 8 * (16 if win == 3 else t) if win else t * t   # output pixels per unit
        mtiles = -(-units * upx // 128) if upx < 128 else units * (upx // 128)
        k = 32 if cin < 16 else (6 * 64 if (win == 2 and cin == 32) else 9 * cin)
        out.append(2 * mtiles * 128 * cout * k)
    return out


def build_net(seed):
    from sarbon_b200 import LocalBackbone
    torch.manual_seed(seed)
    return LocalBackbone().eval()


def job_streams(args, world):
    """Streams of the whole job: --total-streams (strong scaling) or S per GPU (weak)."""
    return args.total_streams if args.total_streams else world * args.streams


def make_frames(args, rank, dev, world=1):
    """This rank's shard of the job's streams (contiguous global stream ids), seeded by its
    first global stream id so that no two ranks share a camera.  Frames are generated at
    the camera height and zero-padded at the bottom to the engine height (720p -> 736)."""
    from sarbon_b200 import scenes
    from sarbon_b200.multi import shard_streams, stream_seed
    cam_h = args.camera_height or args.height
    rects = args.rects or auto_rects(cam_h, args.width)
    shard = shard_streams(job_streams(args, world), world, rank)
    src = scenes.Streams(len(shard), cam_h, args.width, seed=stream_seed(args.seed, shard.start),
                         n_rects=rects, device=dev)
    u8 = torch.stack([src.next() for _ in range(args.frames)])  # [F, S, h, W, 3] RGB
    if cam_h < args.height:
        u8 = torch.nn.functional.pad(u8, (0, 0, 0, 0, 0, args.height - cam_h))
    return u8, rects


def workload_name(args, world):
    cam_h = args.camera_height or args.height
    res = f"{args.width}x{cam_h}" + (f" padded to {args.width}x{args.height}" if cam_h < args.height else "")
    change = "~5% changed blocks" if not args.rects else f"{args.rects} moving rectangles per stream"
    if args.total_streams:
        return f"{res} x {args.total_streams} streams over {world} GPU(s), {change}"
    return f"{res} x {args.streams} streams/GPU, {change}"


# ----------------------------------------------------------------------------- CPU (reference algorithm)
def oracle_for(net, n, h, w, tau):
    from oracle import sparse_oracle as so
    nodes = []
    for nd in net.program()[0]:
        d = {"kind": nd.kind, "src": list(nd.src), "dst": nd.dst, "stride": nd.stride, "radius": nd.radius,
             "act": bool(nd.act)}
        if nd.kind == "conv":
            d["w"] = nd.conv.weight.detach().float().cpu().numpy()
            d["b"] = nd.conv.bias.detach().float().cpu().numpy()
            d["conv_stride"] = nd.conv.stride[0]
        nodes.append(d)
    return so.OracleEngine(so.fuse_program(nodes), n, h, w, dtype=np.float16, tau=tau)


def cpu_run(net, frames_seq, tau, max_steps, seconds, warmup=1, warmup_seconds=30.0):
    """Time the CPU oracle (the reference's algorithm) on 1 stream: reset, ``warmup``
    untimed steps (at least one, stopping early after ``warmup_seconds``), then one
    stream-frame per timed step.  Returns (frames/s, timed steps, threads, warm-up steps)."""
    h, w = frames_seq[0].shape[1:3]
    ora = oracle_for(net, 1, h, w, tau)
    ora.reset(frames_seq[0])
    nw, t0 = 0, time.perf_counter()
    while nw < max(1, warmup):  # BLAS threads, page faults
        ora.step(frames_seq[(1 + nw) % len(frames_seq)])
        nw += 1
        if time.perf_counter() - t0 > warmup_seconds:
            break
    t0 = time.perf_counter()
    n = 0
    while n < max_steps:
        ora.step(frames_seq[(1 + nw + n) % len(frames_seq)])
        n += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = time.perf_counter() - t0
    return n / dt, n, os.cpu_count(), nw


REF_DIR = ROOT / "baseline" / "_ref"


def import_reference():
    """The reference package installed under baseline/_ref (its block_sparse and
    fused_engine modules), or None when it is not installed."""
    if not (REF_DIR / "sarbon").is_dir():
        return None
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    try:
        import sarbon.sparse.block_sparse as bs
        import sarbon.sparse.fused_engine as fe
        return bs, fe
    except Exception:
        return None


def reference_net(ref, net):
    """The reference's own LocalBackbone (sarbon/sparse/block_sparse.py:62-76) holding the
    same weights as `net` (the module and parameter names are the same)."""
    bs, _ = ref
    rnet = bs.LocalBackbone().eval()
    rnet.load_state_dict({k: v.detach().cpu() for k, v in net.state_dict().items()})
    return rnet


def cpu_reference_run(rnet, frames_nchw, max_steps, seconds, warmup=1, warmup_seconds=30.0):
    """The reference's CPU path for the stem features: SarbonVideo without a CUDA device
    runs the dense stem on every frame (video.py:101-104), fp32, all host threads.  One
    stream-frame per step.  Returns (frames/s, timed steps, threads, warm-up steps)."""
    torch.set_num_threads(os.cpu_count() or 1)
    nw, t0 = 0, time.perf_counter()
    with torch.no_grad():
        while nw < max(1, warmup):
            rnet(frames_nchw[nw % len(frames_nchw)])
            nw += 1
            if time.perf_counter() - t0 > warmup_seconds:
                break
        n, t0 = 0, time.perf_counter()
        while n < max_steps:
            rnet(frames_nchw[(nw + n) % len(frames_nchw)])
            n += 1
            if time.perf_counter() - t0 > seconds:
                break
    return n / (time.perf_counter() - t0), n, torch.get_num_threads(), nw


def gpu_reference_run(ref, net, seq, tau, steps, dev):
    """The reference's own FusedSparseEngine (Triton tile kernel JIT-compiled for this GPU,
    CUDA graphs, one host sync per step; sarbon/sparse/fused_engine.py:54-240) on the same
    staged frames and weights: frames/s over `steps` steps after one warm-up pass over the
    sequence (which captures the budget buckets the sequence needs), CUDA events."""
    _, fe = ref
    rnet = reference_net(ref, net).to(dev)
    S, H, W = seq[0].shape[:3]
    eng = fe.FusedSparseEngine(rnet, S, H, W, dtype=torch.float16, tau=tau, device=str(dev))
    eng.reset(seq[0])
    modes = {}
    for f in seq[1:] + seq[:1]:
        m, _ = eng.step(f)
        modes[m] = modes.get(m, 0) + 1
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        eng.step(seq[1 + i % (len(seq) - 1)])
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    del eng
    return {"value": S * steps / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms / steps, "steps": steps,
            "modes_warmup": modes, "what": "the reference FusedSparseEngine (its Triton tile kernel, "
            "CUDA graphs and per-step host sync) on the same frames and weights, this GPU"}


def detector_run(eng, S, H, W, dev, iters, dec_layers=4, seed=0):
    """The detector after the stem on the engine's p8 (rank 0, N = 1): this library's
    B200Detector (one CUDA graph of sb_gemm_conv / sb_attention / ... launches) against the
    reference's own SarbonDetector under autocast, captured as a CUDA graph the way
    SarbonVideo._detect does (sarbon/inference/video.py:116-137), on the same p8 and weights
    (random-init Sarbon-S with non-trivial BatchNorm statistics and heads).  Both are timed
    with CUDA events over `iters` replays after 3 warm-up replays."""
    if not (REF_DIR / "sarbon").is_dir():
        return {"unavailable": "the reference is not installed under baseline/_ref"}
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import sarbon.models.sarbon_det as sd
    from sarbon_b200 import det_ops
    from sarbon_b200.detector import B200Detector
    torch.manual_seed(seed)
    det = sd.build("s", 6, halo_zero=False, dec_layers=dec_layers)
    gen = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        for m in det.modules():
            if isinstance(m, torch.nn.BatchNorm2d):
                c = m.num_features
                m.running_mean.copy_(torch.rand(c, generator=gen) * 0.4 - 0.2)
                m.running_var.copy_(torch.rand(c, generator=gen) * 1.5 + 0.5)
                m.weight.copy_(torch.rand(c, generator=gen) + 0.5)
                m.bias.copy_(torch.rand(c, generator=gen) * 0.4 - 0.2)
            elif isinstance(m, torch.nn.Linear) and not m.weight.any():
                m.weight.copy_(torch.randn(m.weight.shape, generator=gen) * 0.02)
    det = det.to(dev).eval()
    p8 = eng.outputs_nchw()[1]
    if p8.dtype != torch.float16:
        p8 = p8.half()
    h8, w8 = p8.shape[-2:]

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / iters

    mine = B200Detector(det, S, h8, w8, device=dev)
    det_ops.LAUNCHES[0] = 0
    mine.run(p8)
    launches = det_ops.LAUNCHES[0]
    mine.capture(p8)
    ms_mine = timed(mine.replay)
    out = {k: v.clone() for k, v in mine.outputs().items() if torch.is_tensor(v)}
    # the reference, graph-captured under autocast (SarbonVideo._detect)
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st), torch.no_grad(), torch.autocast("cuda", torch.float16):
        for _ in range(3):
            det(None, p8=p8)
    torch.cuda.current_stream().wait_stream(st)
    with torch.cuda.graph(g), torch.no_grad(), torch.autocast("cuda", torch.float16):
        ref_out = det(None, p8=p8)
    ms_ref = timed(g.replay)
    # agreement on these inputs: the selected queries, and the boxes / logits with the
    # reference's selection forced (top-K rows of equal scores may order differently)
    with torch.no_grad(), torch.autocast("cuda", torch.float16):
        feats = det.core(p8)
        shapes = [f.shape[-2:] for f in feats]
        memory = torch.cat([f.flatten(2).transpose(1, 2) for f in feats], 1)
        _, valid = det.anchors(shapes, memory.device, memory.dtype)
        enc = det.enc_proj(memory * valid.to(memory.dtype))
        top = det.enc_cls(enc).max(-1).values.masked_fill(~valid[..., 0], float("-inf")).topk(det.cfg.queries, 1).indices
    shared = sum(len(set(out["top"][b].tolist()) & set(top[b].tolist())) for b in range(S)) / top.numel()
    mine.force_top = top.to(torch.int32)
    forced = mine.run(p8)
    torch.cuda.synchronize()
    dbox = (forced["pred_boxes"].float() - ref_out["pred_boxes"].float()).abs().max().item()
    dlog = (forced["pred_logits"].float() - ref_out["pred_logits"].float()).abs().max().item()
    res = {"ms_per_batch": ms_mine, "frames_per_s": S / (ms_mine * 1e-3),
           "reference_ms_per_batch": ms_ref, "reference_frames_per_s": S / (ms_ref * 1e-3),
           "batch": S, "p8": [int(h8), int(w8)], "queries": det.cfg.queries, "gpu_launches_per_batch": launches,
           "top_k_rows_shared_with_reference": round(shared, 4),
           "pred_boxes_max_abs_diff_forced_top_k": dbox, "pred_logits_max_abs_diff_forced_top_k": dlog,
           "decoder_layers": dec_layers,
           "timing": f"CUDA events over {iters} graph replays after 3 warm-up replays, both arms",
           "reference": f"SarbonDetector (build('s', 6, halo_zero=False, dec_layers={dec_layers})) under "
                        "torch.autocast(float16), captured as one CUDA graph (SarbonVideo._detect)"}
    del mine, g, ref_out, det
    torch.cuda.empty_cache()
    return res


def time_mask_kernels(dev, S, H, W, block, seconds=2.0):
    """Per-call times of the two mask utilities beside the step, at the bench's grid:
    track-steered masks (100 predicted boxes a camera, margin 1; the reference's
    ``_steer``, video.py:139-147) and cell-level masks (8 px cells, 1 % changed, the 11
    receptive radii of the stem; gating.py:42-43).  ``kernel_us``: back-to-back launches
    through the C ABI on device-resident inputs (CUDA events); ``api_us``: the Python call
    a user makes, synchronised, including the box upload; ``cpu_us``: the host restatement
    of the reference's loop (one thread), the cost that the kernel replaces."""
    import ctypes as C
    from oracle import sparse_oracle as so
    from sarbon_b200 import boxes_to_block_masks, cell_active_blocks
    from sarbon_b200._lib import check, lib
    hb, wb = H // block, W // block
    rng = np.random.default_rng(3)
    per = []
    for _ in range(S):
        xy = rng.uniform(0, [W, H], (100, 2))
        wh = rng.uniform(8, 240, (100, 2))
        per.append(np.concatenate([xy, xy + wh], 1))
    out = torch.empty((S, hb, wb), dtype=torch.bool, device=dev)
    boxes = torch.from_numpy(np.concatenate(per)).to(dev)
    offsets = torch.arange(0, 100 * S + 1, 100, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    L = lib()

    def events(fn, n):
        for _ in range(3):
            fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        return 1e3 * e0.elapsed_time(e1) / n

    def wall(fn, budget):
        fn()
        torch.cuda.synchronize(dev)
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < budget:
            fn()
            n += 1
        torch.cuda.synchronize(dev)
        return 1e6 * (time.perf_counter() - t0) / n

    args_b = (C.c_void_p(boxes.data_ptr()), C.c_void_p(offsets.data_ptr()), 100 * S, S, hb, wb, block, 1,
              C.c_void_p(out.data_ptr()), C.c_void_p(stream.cuda_stream))
    k_box = events(lambda: check(L.sb_boxes_to_block_mask(*args_b), "sb_boxes_to_block_mask"), 500)
    a_box = wall(lambda: boxes_to_block_masks(per, hb, wb, block, 1, out=out), seconds / 4)
    c_box = wall(lambda: np.stack([so.boxes_to_block_mask(b, hb, wb, block, 1) for b in per]), seconds / 4)

    cell = 8
    radii = [1, 3, 7, 11, 15, 19, 23, 31, 39, 47, 55]
    g = torch.Generator(device=dev).manual_seed(4)
    cells = (torch.rand(S, H // cell, W // cell, device=dev, generator=g) < 0.01).view(torch.uint8)
    cout = torch.empty((len(radii), S, hb, wb), dtype=torch.uint8, device=dev)
    r_arr = (C.c_int * len(radii))(*radii)
    args_c = (C.c_void_p(cells.data_ptr()), S, H // cell, W // cell, cell, block, r_arr, len(radii),
              C.c_void_p(cout.data_ptr()), C.c_void_p(stream.cuda_stream))
    k_cell = events(lambda: check(L.sb_cell_active_blocks(*args_c), "sb_cell_active_blocks"), 500)
    a_cell = wall(lambda: cell_active_blocks(cells, radii, cell, block), seconds / 4)
    ch = cells.bool().cpu().numpy()
    c_cell = wall(lambda: [so.active_blocks_cell_level(ch, r, cell, block) for r in radii], seconds / 4)
    return {"boxes_to_block_mask": {"kernel_us": round(k_box, 2), "api_us": round(a_box, 1),
                                    "cpu_us": round(c_box, 1), "boxes": 100 * S, "cameras": S,
                                    "out_bytes": S * hb * wb},
            "cell_active_blocks": {"kernel_us": round(k_cell, 2), "api_us": round(a_cell, 1),
                                   "cpu_us": round(c_cell, 1), "cell": cell, "radii": len(radii),
                                   "in_bytes": int(cells.numel()), "out_bytes": int(cout.numel())},
            "note": "outside the timed step; kernel_us = CUDA-event time per call over back-to-back "
                    "ctypes launches (the box masks are bound by the host's call rate at this size); "
                    "cpu_us is the numpy restatement of the reference's loops on one host thread"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from sarbon_b200 import scenes
    net = build_net(args.seed)
    u8, rects = make_frames(args, 0, "cpu")
    order = pingpong(min(args.frames, 8))
    tau = 8 / float(scenes.STD.mean())
    budget = max(10.0, min(150.0, 0.5 * args.steps))
    from sarbon_b200.multi import shard_streams
    S = len(shard_streams(job_streams(args, world), world, 0))
    ref = import_reference()
    if ref is not None:
        rnet = reference_net(ref, net)
        frames = [scenes.normalise(u8[i, :1], torch.float32).permute(0, 3, 1, 2).contiguous() for i in order]
        fps, n, cores, nw = cpu_reference_run(rnet, frames, args.steps, budget, warmup=args.warmup)
        kind, dtype = "reference", "f32 (the reference's dense CPU path)"
        sample = (f"{n} steps of 1 stream x {args.width}x{args.height}: the reference's own LocalBackbone "
                  f"forward (sarbon/sparse/block_sparse.py:62-76, installed under baseline/_ref), the stem "
                  f"SarbonVideo runs per frame without CUDA (video.py:101-104); torch threads = host cores")
    else:
        seq = [scenes.normalise(u8[i, :1]).numpy() for i in order]
        fps, n, cores, nw = cpu_run(net, seq, tau, args.steps, budget, warmup=args.warmup)
        kind, dtype = "port", "f16 in / f32 accumulate (numpy fp32)"
        sample = (f"{n} steps of 1 stream x {args.width}x{args.height} after reset (numpy oracle restating "
                  f"sarbon/sparse, BLAS threads = host cores; the reference is not installed under baseline/_ref)")
    line = {"metric": METRIC, "value": fps, "unit": UNIT, "impl": "reference", "n_gpus": world, "steps": n,
            "warmup": nw, "ms_per_step": 1e3 / fps, "higher_is_better": True,
            "scaling": "strong" if args.total_streams else "weak",
            "vs_baseline": None, "dtype": dtype, "data": "synthetic",
            "config": {"workload": workload_name(args, world),
                       "height": args.height, "width": args.width, "streams_per_gpu": S,
                       "rects_per_stream": rects, "sample": "1 stream-frame per step"},
            "cpu_baseline": {"value": fps, "unit": UNIT, "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": fps, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- GPU
def run_b200(args):
    import torch.distributed as dist
    from sarbon_b200 import FusedSparseEngine, scenes
    from sarbon_b200.multi import job_rate, max_over_ranks
    rank, world, local = dist_env()
    if world > 1:
        # NCCL prints its version banner on stdout when a communicator starts; send it to
        # stderr so that rank 0's stdout stays the single JSON line
        sys.stdout.flush()
        saved = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                    device_id=torch.device("cuda", local))
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved, 1)
            os.close(saved)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    tau = 8 / float(scenes.STD.mean())
    net = build_net(args.seed).to(dev)
    from sarbon_b200.multi import shard_streams
    if args.total_streams and args.total_streams % world:
        raise SystemExit(f"--total-streams {args.total_streams} does not split evenly over {world} GPUs")
    S = len(shard_streams(job_streams(args, world), world, rank))
    H, W = args.height, args.width
    eng = FusedSparseEngine(net, S, H, W, dtype=torch.float16, tau=tau, device=dev,
                            fp8={None: False, "s8": True, "all": "all"}[args.fp8])
    if args.cell:
        eng.set_cell_gating(args.cell)  # the u8 end-to-end step gates per block only
        args.no_e2e = True
    u8, rects = make_frames(args, rank, dev, world)
    staged = torch.stack([scenes.normalise(u8[i]) for i in range(u8.shape[0])])  # [F,S,H,W,3] fp16
    fp8_scales = eng.calibrate_fp8(staged[0], net=net) if args.fp8 else None
    order = pingpong(args.frames)
    seq = [staged[i] for i in order]

    # --- statistics pass (untimed): modes, changed and active counts over one cycle
    eng.reset(seq[0])
    modes, changed, act = {"skip": 0, "sparse": 0, "dense": 0}, [0], [[0] * len(eng.ds)]
    for f in ([] if args.no_stats else seq[1:] + seq[:1]):
        mode, k = eng.step(f)
        modes[mode] += 1
        changed.append(int(eng.changed.sum().item()))
        act.append(list(eng.device_stats().counts)[:len(eng.ds)])
    if len(changed) > 1:
        changed, act = changed[1:], act[1:]
    nb = eng.n_blocks
    changed_frac = statistics.mean(changed) / nb
    act_frac = [statistics.mean(a[i] for a in act) / nb for i in range(len(eng.ds))]

    # --- timed region: K steps, no host sync, frames already in HBM
    eng.reset(seq[0])
    for i in range(args.warmup):
        eng.step_async(seq[(1 + i) % len(seq)])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    start.record()
    base = 1 + args.warmup
    for i in range(args.steps):
        eng.step_async(seq[(base + i) % len(seq)])
    end.record()
    torch.cuda.synchronize()
    clock_info = clocks.stop()
    launches = eng.launch_count() * args.steps
    ms = start.elapsed_time(end)
    if world > 1:
        dist.barrier()
    ms_max = max_over_ranks(ms, dev)
    st = eng.device_stats()
    if st.error:
        raise RuntimeError(f"device error flags {st.error} after the timed region")

    # --- per-kernel roofline pass (events around every launch; separate from the timing)
    prof = {"gate": 0.0, "lists": 0.0, "copy": 0.0, "conv": 0.0, "finalize": 0.0}
    per_layer = [0.0] * len(eng.layers)
    conv_flops, gbytes, nprof = 0, 0, 0
    flops_layer = [0] * len(eng.layers)
    mma_layer = [0] * len(eng.layers)
    eng.reset(seq[0])
    for i in range(args.profile_steps):
        f = seq[1 + i % (len(seq) - 1)]
        mode, k, kms = eng.step_profiled(f)
        counts = list(eng.device_stats().counts)[:len(eng.ds)]
        prof["gate"] += kms[0]
        prof["lists"] += kms[1]
        prof["copy"] += kms[2]
        prof["conv"] += sum(kms[3:3 + len(eng.layers)])
        for j in range(len(eng.layers)):
            per_layer[j] += kms[3 + j]
        prof["finalize"] += kms[3 + len(eng.layers)]
        if mode != "skip":
            fl = layer_flops(eng, counts, mode)
            conv_flops += sum(fl)
            flops_layer = [a + b for a, b in zip(flops_layer, fl)]
            mma_layer = [a + b for a, b in zip(mma_layer, mma_flops(eng, mode))]
        gbytes += gate_bytes(eng, int(eng.changed.sum().item()))
        nprof += 1
    # --- phase pass: events only between the step's phases; the 11 convs run back to back
    # with programmatic dependent launch exactly as in the timed region
    ph = {"gate": 0.0, "lists": 0.0, "copy": 0.0, "conv": 0.0, "finalize": 0.0}
    ph_flops, nph = 0, 0
    ph_ideal_s = 0.0  # the conv FLOPs at each layer's tensor peak (e4m3 layers: twice fp16)
    peaks0, _ = load_peaks()
    layer_peak = [peaks0["bf16_tflops"] * (2.0 if (m >> 4) >= 2 else 1.0) for m in eng.layer_variants()]
    eng.reset(seq[0])
    for i in range(args.profile_steps):
        f = seq[1 + i % (len(seq) - 1)]
        mode, k, pm = eng.step_phases(f)
        counts = list(eng.device_stats().counts)[:len(eng.ds)]
        for key in ph:
            ph[key] += pm[key]
        if mode != "skip":
            fl = layer_flops(eng, counts, mode)
            ph_flops += sum(fl)
            ph_ideal_s += sum(f / (p * 1e12) for f, p in zip(fl, layer_peak))
        nph += 1
    peaks, src = load_peaks()
    default_workload = (S, H, W) == (16, 1088, 1920) and not args.cell
    traffic = TRAFFIC[args.fp8] if default_workload else {"conv": None, "gate": None, "capture": None}
    n_conv = nprof * len(eng.layers)
    conv_tflops = conv_flops / (prof["conv"] * 1e-3) / 1e12
    pipe_tflops = ph_flops / (ph["conv"] * 1e-3) / 1e12
    gate_gbs = gbytes / (prof["gate"] * 1e-3) / 1e9
    # Denominator: the burst GEMM peak (kernels timed over a ~25-step pass, not a seconds-long
    # loop).  Headline: the conv launches as the step runs them (one CUDA-event interval
    # around the 11-layer sequence, programmatic dependent launch kept between layers), so a
    # launch's average duration is the sequence time / 11.  `isolated`: an event around every
    # launch, which serialises each layer's start-up (launch, barriers, weight copy, first
    # loads) with the previous layer's end; the step itself overlaps them.
    # e4m3 layers run at twice the fp16 tensor rate: the peak is then the FLOP-weighted one
    # of the sequence (FLOPs / the time they take at each layer's peak)
    peak_eff = ph_flops / ph_ideal_s / 1e12 if ph_ideal_s > 0 else peaks["bf16_tflops"]
    roof = {"bound": "tensor", "kernel": "sb::conv_tc_kernel (tile conv, all 11 layers)",
            "achieved": pipe_tflops, "peak": peak_eff, "unit": "TFLOP/s",
            "frac": pipe_tflops / peak_eff,
            "timing": "conv sequence of the pipelined step (events at the phase boundaries only)",
            "traffic": traffic["conv"], "traffic_source": traffic["capture"],
            "peak_source": f"{src} bf16_tflops (burst; fp16 dense runs at the bf16 rate)" + (
                "; e4m3 layers (kind::f8f6f4) at 2x that, the dense fp8:fp16 ratio of the tensor cores, "
                "FLOP-weighted over the sequence" if args.fp8 else ""),
            "flops_per_launch": ph_flops / (nph * len(eng.layers)),
            "mma_flops_per_launch": sum(mma_layer) / n_conv,
            "ms_per_launch": ph["conv"] / (nph * len(eng.layers)),
            "isolated": {"achieved": conv_tflops, "frac": conv_tflops / peaks["bf16_tflops"],
                         "ms_per_launch": prof["conv"] / n_conv,
                         "timing": "an event pair around every launch (start-up serialised)"}}
    roof_gate = {"bound": "hbm", "kernel": "sb::gate_kernel<0>", "achieved": gate_gbs, "peak": peaks["hbm_gbs"],
                 "unit": "GB/s", "frac": gate_gbs / peaks["hbm_gbs"], "bytes_per_launch": gbytes / nprof,
                 "traffic": traffic["gate"], "traffic_source": traffic["capture"],
                 "ms_per_launch": prof["gate"] / nprof}
    share = {k: v / sum(prof.values()) for k, v in prof.items()}
    phase_us = {k: round(1e3 * v / max(nph, 1), 1) for k, v in ph.items()}

    # --- e2e through the public API from pinned host uint8 BGR frames
    e2e = None
    if not args.no_e2e:
        ne = min(args.frames, 8)
        host = [u8[i].flip(-1).contiguous().cpu().pin_memory() for i in range(ne)]
        eorder = [host[i] for i in pingpong(ne)]
        dbuf = [torch.empty_like(host[0], device=dev) for _ in range(2)]
        res_dev = eng.result_view()
        ring = torch.zeros(args.e2e_steps, 2, dtype=torch.int64).pin_memory()
        copy_s = torch.cuda.Stream(dev)
        up = [torch.cuda.Event() for _ in range(2)]
        done = [torch.cuda.Event() for _ in range(2)]
        eng.reset(scenes.normalise(u8[0]))
        for i in range(3):
            eng.step_u8(dbuf[0].copy_(eorder[(1 + i) % len(eorder)]), scenes.MEAN, scenes.STD, sync=True)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        cur = torch.cuda.current_stream(dev)
        e0.record()
        for i in range(args.e2e_steps):
            b = i % 2
            with torch.cuda.stream(copy_s):
                if i >= 2:
                    copy_s.wait_event(done[b])
                dbuf[b].copy_(eorder[(4 + i) % len(eorder)], non_blocking=True)
                up[b].record(copy_s)
            cur.wait_event(up[b])
            eng.step_u8(dbuf[b], scenes.MEAN, scenes.STD, sync=False)
            done[b].record(cur)
            ring[i].copy_(res_dev, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        ems = e0.elapsed_time(e1)
        e2e = {"value": job_rate(world, S, args.e2e_steps, max_over_ranks(ems, dev)), "unit": UNIT,
               "h2d_bytes_per_step": int(host[0].numel()), "d2h_bytes_per_step": 16,
               "steps": args.e2e_steps, "input": "pinned host uint8 BGR, normalisation fused into the gate",
               "modes_seen": sorted({int(m) for m in ring[:, 0].tolist()})}

    # --- the mask utilities beside the step (rank 0; untimed by the step's clock)
    masks = None
    if rank == 0 and not args.no_masks:
        masks = time_mask_kernels(dev, S, H, W, eng.block)

    # --- CPU baseline (rank 0, N = 1 only)
    cpu = None
    ref = import_reference()
    ref_gpu = None
    if rank == 0 and world == 1 and not args.no_reference_gpu:
        if ref is None:
            ref_gpu = {"unavailable": "the reference is not installed under baseline/_ref"}
        else:
            try:
                ref_gpu = gpu_reference_run(ref, net, seq[:len(seq)], tau, args.reference_gpu_steps, dev)
            except Exception as ex:  # report, do not fail the bench
                ref_gpu = {"unavailable": f"{type(ex).__name__}: {str(ex)[:200]}"}
            torch.cuda.empty_cache()
    detector = None
    if rank == 0 and world == 1 and not args.no_detector:
        try:
            detector = detector_run(eng, S, H, W, dev, args.detector_iters, args.dec_layers)
            if ref_gpu and "ms_per_step" in ref_gpu and "ms_per_batch" in detector:
                # the stem step and the detector on its p8, per batch of S frames (device time)
                detector["stem_plus_detector_frames_per_s"] = S / ((ms_max / args.steps + detector["ms_per_batch"]) * 1e-3)
                detector["reference_stem_plus_detector_frames_per_s"] = S / (
                    (ref_gpu["ms_per_step"] + detector["reference_ms_per_batch"]) * 1e-3)
        except Exception as ex:  # report, do not fail the bench
            detector = {"unavailable": f"{type(ex).__name__}: {str(ex)[:200]}"}
        torch.cuda.empty_cache()
    if rank == 0 and world == 1 and not args.no_cpu:
        order = pingpong(min(args.frames, 8))
        if ref is not None:
            rnet = reference_net(ref, net)
            frames = [scenes.normalise(u8[i, :1].cpu(), torch.float32).permute(0, 3, 1, 2).contiguous()
                      for i in order]
            fps, n, cores, _ = cpu_reference_run(rnet, frames, 64, args.cpu_seconds)
            cpu = {"value": fps, "unit": UNIT, "cores": cores, "kind": "reference",
                   "sample": f"{n} steps of 1 stream x {W}x{H}: the reference's dense CPU stem "
                             f"(LocalBackbone forward, fp32; video.py:101-104); torch threads = host cores"}
        else:
            cseq = [scenes.normalise(u8[i, :1]).cpu().numpy() for i in order]
            fps, n, cores, _ = cpu_run(net.cpu(), cseq, tau, 64, args.cpu_seconds)
            cpu = {"value": fps, "unit": UNIT, "cores": cores, "kind": "port",
                   "sample": f"{n} steps of 1 stream x {W}x{H} (numpy oracle restating sarbon/sparse; "
                             f"BLAS threads = host cores)"}

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    value = job_rate(world, S, args.steps, ms_max)
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong" if args.total_streams else "weak", "vs_baseline": None,
            "dtype": {None: "f16 (fp32 accumulate)", "s8": "f16 + e4m3 stride-8 stage (fp32 accumulate)",
                      "all": "f16 + e4m3 stride-4 and stride-8 stages (fp32 accumulate)"}[args.fp8],
            "data": "synthetic (seeded moving-rectangle camera streams, random-init Sarbon-S stem)",
            "config": {"workload": workload_name(args, world), "job_streams": job_streams(args, world),
                       "height": H, "width": W, "block": 32, "streams_per_gpu": S, "rects_per_stream": rects,
                       "gating": f"cell level, {args.cell} px cells" if args.cell else "block level",
                       "fp8_act_scales": fp8_scales,
                       "tau_grey_levels": 8, "frames_staged": args.frames,
                       "changed_block_frac": changed_frac,
                       "active_block_frac": {f"d{d}": a for d, a in zip(eng.ds, act_frac)},
                       "modes_cycle": modes, "per_gpu_fps": S * args.steps / (ms_max * 1e-3),
                       "l2": f"no flush: each step reads {S * H * W * 6 / 1e6:.0f} MB of new frames + "
                             f"the image cache (> 126 MB L2)"},
            "roofline": roof, "roofline_gate": roof_gate, "kernel_time_share": share,
            "phase_us_per_step": phase_us,
            "conv_us_per_layer": {l.dst: round(1e3 * t / max(nprof, 1), 1) for l, t in zip(eng.layers, per_layer)},
            "conv_tflops_per_layer": {l.dst: round(f / (t * 1e-3) / 1e12, 1) if t > 0 else None
                                      for l, f, t in zip(eng.layers, flops_layer, per_layer)},
            # issued tensor-core work over algorithmic work per layer (window regions, K padding)
            "conv_mma_over_alg_per_layer": {l.dst: round(m / f, 3) if f else None
                                            for l, f, m in zip(eng.layers, flops_layer, mma_layer)},
            "cpu_baseline": cpu, "reference_gpu": ref_gpu, "e2e": e2e, "gpu_launches": launches,
            "mask_kernels": masks, "detector": detector, "clocks": clock_info}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
