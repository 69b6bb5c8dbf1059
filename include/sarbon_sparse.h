/*
 * sarbon_sparse.h -- C ABI of the B200 temporal block-sparse stem engine.
 *
 * One engine serves N camera streams of H x W pixels on one GPU.  Per step it
 *   1. gates every block x block tile of the new frames against the cached image
 *      (exact per-block sum of |fp16 diff|, threshold, OR extra mask, refresh phase),
 *   2. dilates the change mask per receptive-field dilation and compacts the active
 *      blocks into ordered (cam, by, bx) lists,
 *   3. recomputes only the active tiles of the 3x3 conv stem (tcgen05 tensor cores
 *      for fp16, CUDA cores for fp32), fused with bias, residual add and ReLU,
 *      writing straight into the NHWC feature caches,
 *   4. falls back to a dense pass above a calibrated active-block count.
 *
 * Conventions: plain C types only, an opaque engine handle, int status codes,
 * no exceptions.  Device pointers are raw CUDA device addresses on the engine's
 * GPU; `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 * Caches and block lists are engine-owned device memory, valid until
 * sb_destroy().  Calls on one engine are serial (one host thread at a time).
 *
 * Reference interface replaced (Bahrombekk/Sarbon, sarbon/sparse/fused_engine.py):
 * the functions below mirror FusedSparseEngine, see each declaration.
 */
#ifndef SARBON_SPARSE_H
#define SARBON_SPARSE_H

#include <stdint.h>

#if defined(__GNUC__)
#define SB_API __attribute__((visibility("default")))
#else
#define SB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define SB_OK         0
#define SB_EINVAL     1   /* bad argument (shape, id, dtype, topology) */
#define SB_EOVERFLOW  2   /* active count above capacity: dense refresh needed */
#define SB_ETIMEOUT   3   /* a bounded device-side wait gave up */
#define SB_ECUDA      4   /* a CUDA runtime/driver call failed */
#define SB_ENOMEM     5   /* device or pinned allocation failed */

/* cache element types (fused_engine.py:55-56 `dtype`); SB_F8: e4m3 codes with an
 * activation scale per cache (value = code * scale), see SB_CREATE_FP8_S8 */
#define SB_F16 0
#define SB_F32 1
#define SB_F8  2

/* step modes (fused_engine.py:230-237) */
#define SB_MODE_SKIP   0
#define SB_MODE_SPARSE 1
#define SB_MODE_DENSE  2

#define SB_MAX_LAYERS 32
#define SB_MAX_DILATIONS 4

typedef struct sb_engine sb_engine;

/* One fused conv(+add) of the stem (fused_engine.py:29-41, built by _fuse :99-119).
 * Cache ids: 0 is the image cache; cache id i+1 is the output of layer i. */
typedef struct sb_layer_desc {
    int32_t src;         /* input cache id */
    int32_t res;         /* residual cache id, or -1 */
    int32_t cin, cout;   /* channels */
    int32_t stride;      /* conv stride (1 or 2), kernel 3x3, padding 1 */
    int32_t out_stride;  /* output feature stride w.r.t. the image */
    int32_t radius;      /* receptive radius in image pixels (dilation = ceil(radius/block)) */
    int32_t act;         /* 1 = ReLU */
} sb_layer_desc;

typedef struct sb_stats_t {
    int64_t skip, sparse, dense;   /* fused_engine.py:92 `stats` */
    int64_t last_count;            /* k of the last step (-1: hysteresis dense) */
    int32_t last_mode;
    int32_t error;                 /* sticky device error flags (0 = none) */
    int32_t counts[SB_MAX_DILATIONS]; /* active blocks per dilation of the last gated step */
    int32_t n_dilations;
    int32_t dilations[SB_MAX_DILATIONS];
} sb_stats_t;

/* FusedSparseEngine.__init__ (fused_engine.py:55-92).  `tau` is in frame units
 * per pixel-channel (threshold = float32(tau*block*block*3), :144); `refresh` 0
 * disables the round-robin refresh (:145-147).  Allocates the NHWC caches
 * (zeroed), lists, masks and device state on the current CUDA device. */
SB_API int sb_create(const sb_layer_desc* layers, int n_layers, int n_streams, int height, int width,
              int block, int dtype, double tau, int refresh, int dense_check_every,
              sb_engine** out);

/* sb_create with creation flags.  SB_CREATE_BLOCK_UNITS: every layer runs over single
 * blocks (no multi-block window regions), which M0 mode needs; slower for the 4x4-pixel
 * layers.  sb_create(...) is sb_create_ex(..., 0, out). */
#define SB_CREATE_BLOCK_UNITS 1
/* SB_CREATE_FP8_S8 (fp16 engines): the caches of the stride-8 stage (every layer with
 * out_stride >= 8) hold e4m3 codes with one activation scale per cache (sb_set_act_scale,
 * default 1); the layer that enters the stage runs fp16 MMAs and writes e4m3, the layers
 * inside it run tcgen05 kind::f8f6f4 MMAs on e4m3 activations and e4m3 weights quantised
 * per output channel (scale = max |w| / 448 of the channel, sb_layer_wscale), dequantised
 * in the fp32 epilogue (bias, residual, ReLU), then quantised to e4m3 again.  No reference
 * counterpart (the reference casts its tile weights to the engine dtype,
 * fused_engine.py:114): this is the full-detection benchmark's weight format, applied where the layer's
 * input is an e4m3 cache (it halves the tensor-core work and the weights). */
#define SB_CREATE_FP8_S8 2
/* SB_CREATE_FP8_S4: the same for the stride-4 stage (layers with out_stride == 4), except its
 * last cache, the stage's output p4, which stays fp16 (that layer reads e4m3 and writes
 * fp16).  With both flags every layer whose input is an e4m3 cache runs kind::f8f6f4. */
#define SB_CREATE_FP8_S4 4
SB_API int sb_create_ex(const sb_layer_desc* layers, int n_layers, int n_streams, int height, int width,
                        int block, int dtype, double tau, int refresh, int dense_check_every, int flags,
                        sb_engine** out);

/* M0 semantics for the steps launched after this call (the reference's first engine,
 * BlockSparseEngine.step / update, block_sparse.py:196-295): every step copies the whole
 * frame into the image cache (so the gate compares a frame with the previous one), there is
 * no dense fallback, and with capacity > 0 every layer recomputes exactly `capacity` entries
 * of its dilation's block list: the first `capacity` active blocks, padded with block 0
 * (nonzero_static(size=capacity, fill_value=0), :268-271); more active blocks than that are
 * left as they were (the caller sees count > capacity, the reference's overflow flag).
 * capacity = 0 recomputes the active blocks (update, :211-218).  on = 0 returns to the fused
 * engine's behaviour.  Needs an engine created with SB_CREATE_BLOCK_UNITS (or fp32). */
SB_API int sb_set_m0(sb_engine* e, int on, int64_t capacity);

/* Layer weights from host memory: w float32 [3][3][cin][cout] (the Triton kernel's
 * w_tile layout, fused_engine.py:114) and bias float32 [cout] (:116). */
SB_API int sb_upload_weights(sb_engine* e, int layer, const float* w, const float* bias);

/* FusedSparseEngine.reset (fused_engine.py:207-212): dense pass from fp16/fp32
 * frames [N][H][W][3] (engine dtype, device memory); clears hysteresis. */
SB_API int sb_reset(sb_engine* e, const void* frames_dev, void* stream);

/* Dense pass without touching the hysteresis state (the reference's
 * `dense_graph.replay()`, fused_engine.py:88,172-185). */
SB_API int sb_dense(sb_engine* e, const void* frames_dev, void* stream);

/* FusedSparseEngine.step (fused_engine.py:214-240) on frames [N][H][W][3] in the
 * engine dtype.  Skip/sparse/dense and hysteresis are decided on the device, so
 * the call is asynchronous; when mode_out or count_out is non-NULL it synchronises
 * `stream` and returns the mode (SB_MODE_*) and the active count (-1 for a
 * hysteresis dense step). */
SB_API int sb_step(sb_engine* e, const void* frames_dev, void* stream, int* mode_out, int64_t* count_out);

/* Step graphs (on by default): sb_step, sb_step_u8 and sb_step_u8_resized capture their
 * launch sequence into a CUDA graph the first time they see an input (frames pointer,
 * input kind, camera size, normalisation) and replay it afterwards, so a step costs the
 * host one graph launch instead of ~15 kernel launches (the reference replays CUDA graphs
 * too, fused_engine.py:85-88,196-199).  Up to 64 inputs are kept (least recently used
 * dropped); sb_set_tau, sb_set_cell_gating and sb_upload_weights drop them all, since they
 * change kernel arguments.  on = 0 launches every kernel directly. */
SB_API int sb_set_step_graphs(sb_engine* e, int on);

/* The same step on uint8 BGR frames [N][H][W][3] with the caller's normalisation
 * fused into the gate (sarbon/inference/video.py:74-99, `_prep`: BGR->RGB,
 * (x - mean[c]) / std[c] in fp32, rounded to fp16).  fp16 engines only. */
SB_API int sb_step_u8(sb_engine* e, const uint8_t* frames_dev, const float mean[3], const float std_[3],
               void* stream, int* mode_out, int64_t* count_out);

/* The same step on uint8 BGR frames [N][cam_h][cam_w][3] of any camera size: the whole
 * `_prep` of the caller (video.py:95-99: BGR->RGB, the bilinear resize to the engine size
 * with align_corners=False when the sizes differ, (x - mean[c]) / std[c] in fp32) runs
 * as one kernel of this library writing fp16 frames into an engine-owned buffer (allocated
 * by the first call that resizes), which the step then gates.  Equal sizes take
 * sb_step_u8's path (no extra pass).  fp16 engines only. */
SB_API int sb_step_u8_resized(sb_engine* e, const uint8_t* frames_dev, int cam_h, int cam_w, const float mean[3],
                              const float std_[3], void* stream, int* mode_out, int64_t* count_out);

/* sb_step with a CUDA event before and after every kernel it launches (gate, lists,
 * dense copy, one conv per layer, finalize); synchronises `stream` and writes the
 * duration of each launch in ms to kernel_ms[0..*n_kernels).  Measurement aid with
 * no counterpart in the reference (which has no per-kernel timing). */
SB_API int sb_step_profiled(sb_engine* e, const void* frames_dev, void* stream, float* kernel_ms, int capacity,
                            int* n_kernels);

/* sb_step with CUDA events only at its phase boundaries: phase_ms[0] gate, [1] list
 * kernel, [2] dense image copy, [3] the whole conv sequence (all layers, launched back to
 * back with programmatic dependent launch as in sb_step, so each layer's start-up overlaps
 * the previous layer's tail), [4] finalize.  Synchronises `stream`.  Measurement aid with
 * no counterpart in the reference. */
SB_API int sb_step_phases(sb_engine* e, const void* frames_dev, void* stream, float phase_ms[5]);

/* Device address of two int64 {mode, count} the last step's finalize kernel wrote;
 * lets a caller copy each step's result to the host asynchronously.  No counterpart
 * in the reference (its step returns them after a host sync, fused_engine.py:228-240). */
SB_API int sb_result_ptr(sb_engine* e, const int64_t** dev_ptr);

/* Mode and count of the last step (synchronises `stream`). */
SB_API int sb_query(sb_engine* e, void* stream, int* mode_out, int64_t* count_out);

/* FusedSparseEngine.set_extra (fused_engine.py:201-205): uint8 [N][Hb][Wb] device
 * mask of blocks recomputed regardless of pixel change (copied on `stream`). */
SB_API int sb_set_extra(sb_engine* e, const uint8_t* mask_dev, void* stream);

/* Set the dense-fallback crossover (fused_engine.py:89, written by calibrate
 * :242-275) and the hysteresis period (:91). */
SB_API int sb_set_fallback(sb_engine* e, int64_t fallback, void* stream);
/* Change threshold `tau` (mean |diff| per block) for the steps launched after this call;
 * host-side only.  Replaces the per-call `tau` of the M0 engine's step
 * (block_sparse.py:253,323-326) and `update`'s given mask (tau = +inf, block_sparse.py:213). */
SB_API int sb_set_tau(sb_engine* e, double tau);
SB_API int sb_set_dense_check_every(sb_engine* e, int n, void* stream);

/* Cell-level gating for the steps launched after this call (the tighter active-set
 * estimate of the reference's gating.py:42-43, which the reference uses only in its
 * gating analysis; its engine gates per block).  A cell of cell x cell pixels changed
 * when its exact sum of |fp16 diff| exceeds float32(tau * cell^2 * 3), or its block is
 * forced by `extra` / the refresh phase; a block changed (image cache update) when any
 * of its cells did; the mask of dilation group i marks the blocks that the changed cells,
 * dilated by cell_radii[i] cells, reach.  Lossless at tau = 0 when cell_radii[i] is at
 * least ceil(R / cell) for every layer R of group i.  fp16 engines and sb_step only;
 * cell a multiple of 8 dividing the block; n_radii = the number of dilation groups.
 * cell = 0 returns to block-level gating.  Allocates the cell buffers on first use. */
SB_API int sb_set_cell_gating(sb_engine* e, int cell, const int* cell_radii, int n_radii);

/* Calibration support (fused_engine.py:261-264): run the conv sequence over
 * exactly `n_tiles` entries of the current block lists (entries past the active
 * count recompute block 0, like nonzero_static's fill_value=0), updating the
 * image cache from `frames_dev` where `changed` is set. */
SB_API int sb_run_sparse_forced(sb_engine* e, const void* frames_dev, int64_t n_tiles, void* stream);

/* Dense recompute of layers first..last only (the per-layer loop of the reference's
 * dense pass, fused_engine.py:176-185), every block, from the caches as they are: the
 * image cache is not touched and the gate is not run.  With caches loaded from another
 * implementation (sb_cache_ptr), one layer's output from that implementation's own inputs
 * can be compared layer by layer. */
SB_API int sb_dense_layers(sb_engine* e, int first, int last, void* stream);

/* Element type of cache `cache_id` (SB_F16, SB_F32 or SB_F8) and, for SB_F8, its activation
 * scale (value = code * scale; scale may be NULL).  No reference counterpart. */
SB_API int sb_cache_dtype(sb_engine* e, int cache_id, int* dtype, float* scale);

/* Activation scale of an e4m3 cache (SB_CREATE_FP8_S8) for the steps launched after this
 * call: the layer writing it stores e4m3(y / scale), the layers reading it multiply by it.
 * Drops the captured step graphs.  No reference counterpart. */
SB_API int sb_set_act_scale(sb_engine* e, int cache_id, float scale);

/* Per-output-channel scales of layer `layer`'s e4m3 weights (n >= cout floats): weight =
 * e4m3 code * scale[c], code = e4m3(w / scale[c]) rounded to nearest even.  No reference
 * counterpart. */
SB_API int sb_layer_wscale(sb_engine* e, int layer, float* out, int n);

/* Cache views (fused_engine.py:67-71,124-125): device pointer and NHWC shape of
 * cache id (0 = image, i+1 = layer i output). */
SB_API int sb_cache_ptr(sb_engine* e, int cache_id, void** ptr, int64_t shape[4]);

/* Cell-level gating (gating.py:42-43, `active_blocks_cell_level`): from a change mask of
 * cell x cell-pixel cells, `cells_dev` uint8 [n_cams][hc][wc] (nonzero = changed), write for
 * each receptive radius radii[i] (image pixels) the active blocks of block x block pixels:
 * out_dev uint8 [n_radii][n_cams][hc*cell/block][wc*cell/block], a block being active when
 * the cells dilated by ceil(radii[i] / cell) cells reach it.  block must be a multiple of
 * cell and hc, wc multiples of block / cell; 1 <= n_radii <= 16.  One kernel on `stream`,
 * no allocation. */
SB_API int sb_cell_active_blocks(const uint8_t* cells_dev, int n_cams, int hc, int wc, int cell, int block,
                                 const int* radii, int n_radii, uint8_t* out_dev, void* stream);

/* Track-steered block masks (video.py:26-34 `boxes_to_block_mask`, as `SarbonVideo._steer`
 * uses it at video.py:139-147): out_dev uint8 [n_cams][hb][wb] = 1 where a block of
 * block x block pixels lies in a box's block range, rows max(0, floor(y0/block) - margin) ..
 * min(hb-1, floor(y1/block) + margin) and likewise for columns; 0 elsewhere (the mask is
 * overwritten).  boxes_dev: float64 [n_boxes][4] xyxy in engine pixels; offsets_dev: int32
 * [n_cams + 1], camera c owning rows offsets[c] .. offsets[c+1]-1 (clamped to
 * [0, n_boxes]).  Boxes with a non-finite coordinate mark nothing (the reference raises on
 * them; the Python wrapper does too).  boxes_dev may be null when n_boxes == 0.  Writing
 * into the engine's `extra` mask (sb_gate_buffers) steers its next step.  One kernel on
 * `stream`, no allocation. */
SB_API int sb_boxes_to_block_mask(const double* boxes_dev, const int* offsets_dev, int n_boxes, int n_cams,
                                  int hb, int wb, int block, int margin, uint8_t* out_dev, void* stream);

/* Which tile-conv kernel variant layer `layer` runs: *mode = window mode (0 per-tap boxes or
 * first-layer gather, 1 row windows, 2 strided windows, 3 full windows) + 8 for CTA pairs;
 * -1 for an fp32 engine (CUDA-core kernel).  Introspection only; no reference counterpart
 * (the reference has a single Triton tile kernel, triton_conv.py:15-86). */
SB_API int sb_layer_variant(sb_engine* e, int layer, int* mode);

/* Gate buffers (uint8 device pointers, engine-owned): `changed` [N][Hb][Wb], masks
 * [n_dil][N][Hb][Wb] (fused_engine.py:74-77) and the `extra` mask [N][Hb][Wb] the
 * next step ORs into the change mask (writing it directly equals sb_set_extra). */
SB_API int sb_gate_buffers(sb_engine* e, uint8_t** changed, uint8_t** masks, uint8_t** extra, int* n_dilations,
                    int dilations[SB_MAX_DILATIONS]);

/* Per-dilation block lists of the last gated step (fused_engine.py:161-165): int32
 * device pointers to cam, by, bx (capacity N*Hb*Wb, ascending flat block order) and,
 * when `count` is non-NULL, the number of valid entries (synchronises `stream`). */
SB_API int sb_debug_lists(sb_engine* e, int d_index, int32_t** cam, int32_t** by, int32_t** bx,
                   int64_t* count, void* stream);

/* Allocation-free block lists for a caller-supplied change mask.  No counterpart in
 * the reference (it builds lists only inside FusedSparseEngine); this is for callers
 * that cannot allocate device memory while they run -- a serving process that has
 * planned all of its device memory up front, or code that must not stall other streams
 * with the device-wide synchronisation cudaMalloc/cudaFree can imply -- and have no
 * engine, e.g. a scheduler deciding which cameras' blocks to run.
 *
 * From `changed_dev` (uint8 [n_cams][hb][wb], nonzero = changed) it writes, on `stream`:
 *   masks_dev  uint8 [n_dil][n_cams*hb*wb]: max_pool2d(changed, 2d+1, 1, d) per camera
 *              for each d = dilations[i] (fused_engine.py:151)
 *   lists_dev  int32 [n_dil][3][n_cams*hb*wb]: cam, by, bx of the active blocks in
 *              ascending flat order (nonzero_static, fused_engine.py:161-165); entries
 *              past the count are left as they were
 *   counts_dev int32 [n_dil] (may be NULL): active blocks per dilation, or -1 in every
 *              slot if a bounded device wait gave up (the lists are then invalid).  It
 *              is the only failure signal of the device side: a caller that needs to know
 *              that its lists are valid must pass it.
 * Dilations larger than max(hb, wb) give the same masks as max(hb, wb) and are clamped.
 * Its scratch is one static device array sized for n_cams*hb*wb <= SB_STATIC_LISTS_MAX_BLOCKS;
 * larger masks are rejected with SB_EINVAL.  Every call on a device shares that array:
 * calls must be ordered (one stream, or events between streams); overlapping calls race.
 * The first call on each device looks the array up (cudaGetSymbolAddress) with that
 * device current and keeps the address for the life of the process; make that first
 * call before any stream capture on the device, and do not use the entry point across a
 * cudaDeviceReset (the kept address would be stale).  The array is 33,024 bytes. */
#define SB_STATIC_LISTS_MAX_BLOCKS (1 << 20)
SB_API int sb_block_lists_static(const uint8_t* changed_dev, int n_cams, int hb, int wb, const int* dilations,
                                 int n_dil, uint8_t* masks_dev, int32_t* lists_dev, int32_t* counts_dev,
                                 void* stream);

/* Test hook with no counterpart in the reference: in the steps of engine `e` (or, with
 * e == NULL, the sb_block_lists_static calls) launched after this call, list-kernel chunk
 * `withhold_chunk` (blocks withhold_chunk*1024 .. +1023; -1 = none) publishes no look-back
 * words, and every look-back wait gives up after `spin_limit` polls (0 = the default limit,
 * 2^24 polls).  The next chunk's bounded wait then runs out: the list kernel sets its
 * timeout flag and finishes, the step completes without a fault, and the host sees
 * SB_ETIMEOUT from sb_step (and the flag in sb_stats().error) or -1 counts from
 * sb_block_lists_static.  The lists and features of such a step are invalid.  Synchronous. */
SB_API int sb_debug_withhold_lookback(sb_engine* e, int withhold_chunk, int spin_limit);

/* Multi-scale deformable attention core of the detector on the cached p8
 * (sarbon/models/deform_attn.py:14-28, `ms_deform_attn_core`; its docstring names it as the
 * place for a fused kernel).  value [B][S][H][D] (SB_F32 or SB_F16, S = sum of the levels'
 * h*w, level l's rows starting after the earlier levels'), level_hw [L][2] (h, w; host
 * memory, L <= 8), loc [B][Q][H][L][P][2] fp32 (x, y in [0, 1]), weight [B][Q][H][L][P] fp32
 * -> out [B][Q][H*D] in the value's type: per (b, q, h) the sum over levels and points of
 * weight * bilinear sample, sampled as grid_sample(align_corners=False, padding_mode="zeros")
 * at grid = 2*loc - 1.  One kernel on `stream`, no allocation. */
SB_API int sb_ms_deform_attn(const void* value, int value_dtype, int B, int S, int H, int D, const int* level_hw,
                             int L, const float* loc, const float* weight, int Q, int P, void* out, void* stream);

/* ---------------------------------------------------------------- detector kernels
 * The detector after the stem (sarbon/models/sarbon_det.py:118-356) runs on these entry
 * points; each is one kernel on `stream`, allocates nothing and may be captured in a CUDA
 * graph (after a first call outside capture on the device). */

/* One NHWC fp16 source of sb_gemm_conv: element (b, y, x, c) at
 * ptr[((b * img_stride) + y * W + x) * ld + c], c < C. */
typedef struct {
  const void* ptr;       /* 16-byte aligned */
  int C;                 /* channels read, a multiple of 64 */
  long long ld;          /* elements between pixels (>= C, a multiple of 8) */
  long long img_stride;  /* pixels between images (>= H * W) */
} sb_gemm_src;

/* Every nn.Linear / nn.Conv2d of the detector as one tcgen05 implicit GEMM with its
 * epilogue (under the reference's autocast each is an fp16 product with fp32 accumulation;
 * sarbon_det.py:118-171,294-356, deform_attn.py:57-66):
 *   out[b, yo, xo, n] = act(sum_{tap, c} src[b, yo*stride + ky - pad, xo*stride + kx - pad, c]
 *                                     * weight[n][tap * Ctot + c] + bias[n] + res[b, yo, xo, n])
 * over nsrc (1 or 2) sources of B x H x W pixels whose channels are concatenated (Ctot =
 * sum of C; torch.cat([a, b], 1)), taps = 1 (stride 1, pad 0) or 9 (3x3, pad 1, stride 1
 * or 2; tap = ky * 3 + kx); out-of-map pixels read as zero.  weight: fp16 [N][taps * Ctot]
 * row-major (16-byte aligned).  bias: fp32 [N] or NULL.  act: 0 none, 1 ReLU, 2 GELU (erf).
 * res (NULL for none) and out: rows of res_dtype / out_dtype (SB_F16 or SB_F32), element
 * (b, yo, xo, n) at [(b * img + yo * Wo + xo) * ld + n] (ld >= N; rows of a multiple of 16
 * bytes on a 16-byte aligned base take vector accesses, others element accesses).  A linear
 * layer over a [rows][C] matrix is B = 1, H = 1, W = rows. */
SB_API int sb_gemm_conv(const sb_gemm_src* src, int nsrc, int B, int H, int W, int taps, int stride,
                        const void* weight, int N, const float* bias, int act, const void* res, int res_dtype,
                        long long res_ld, long long res_img, void* out, int out_dtype, long long out_ld,
                        long long out_img, void* stream);

/* Sticky error flags (SB_ERR_* bits of the bounded waits) of the detector kernels; clear != 0
 * resets them.  Synchronous. */
SB_API int sb_kernels_error(int clear, int* flags);

/* In the functions below a "row" argument is a matrix of rows `ld` elements apart; *_dtype
 * is SB_F16 or SB_F32. */

/* nn.LayerNorm (sarbon_det.py:150,171,317 under autocast: fp32 statistics and output) of
 * the rows of a (+ b if non-NULL), D channels (32 <= D <= 1024, D % 32 == 0), eps; writes
 * any of y32 (fp32), y16 (fp16) and yp16 = fp16(y + sign * pos[row % period]) (pos fp16:
 * the decoder's `tgt + pos` query :169-170, the encoder's `aifi(t + pos) - pos` :146).  The
 * sum a + b of two fp16 operands is rounded to fp16 first (it is an fp16 tensor there). */
SB_API int sb_layernorm(const void* a, int a_dtype, long long lda, const void* b, int b_dtype, long long ldb,
                        const float* gamma, const float* beta, float eps, int rows, int D, float* y32, long long ld32,
                        void* y16, long long ld16, const void* pos, long long ldpos, int period, float sign, void* yp16,
                        long long ldp, void* stream);

/* out (fp16 rows) = fp16(a + sign * b[row % period]) over rows x D. */
SB_API int sb_add_rows(const void* a, int a_dtype, long long lda, const void* b, int b_dtype, long long ldb, int period,
                       float sign, int rows, int D, void* out, long long ldo, void* stream);

/* Depthwise 3x3 conv, padding 1, + bias (BatchNorm folded into w [9][C] fp32 and bias [C])
 * + ReLU if relu, on NHWC fp16 maps (x: pixels ldx elements apart, images imgx pixels
 * apart; C and the lds multiples of 8) -- fuse()'s depthwise half, sarbon_det.py:73-77. */
SB_API int sb_dwconv3x3(const void* x, long long ldx, long long imgx, int B, int H, int W, int C, const float* w,
                        const float* bias, int relu, void* y, long long ldy, long long imgy, void* stream);

/* Nearest 2x upsampling of an NHWC fp16 map B x H x W x C into B x 2H x 2W x C
 * (F.interpolate(scale_factor=2.0), sarbon_det.py:147-148). */
SB_API int sb_upsample2x(const void* x, long long ldx, long long imgx, int B, int H, int W, int C, void* y,
                         long long ldy, long long imgy, void* stream);

/* Multi-head attention core softmax(q k^T / sqrt(dh)) v, H heads of dh = 32 channels (head h
 * = columns 32h..32h+31), Tq queries and Tk keys per image, fp16 rows (16-byte aligned,
 * rows apart by ld, images by img rows), fp32 softmax -- the attention of the encoder's
 * nn.TransformerEncoderLayer and the decoder's nn.MultiheadAttention (sarbon_det.py:129,160). */
SB_API int sb_attention(const void* q, long long ldq, long long imgq, const void* k, long long ldk, long long imgk,
                        const void* v, long long ldv, long long imgv, int B, int H, int dh, int Tq, int Tk, void* out,
                        long long ldo, long long imgo, void* stream);

/* Query selection (sarbon_det.py:314): per image, the K (<= 1024) rows of the S (<= 65536)
 * rows of fp16 logits [rows][C] (image b's rows start at b * img) with the largest
 * max-over-classes value, rows with valid[row] == 0 excluded (valid may be NULL); int32
 * row indices idx[b * ldi + i], ordered by value (descending), equal values by row. */
SB_API int sb_topk_rows(const void* logits, long long ld, long long img, int B, int S, int C, const void* valid, int K,
                        void* idx, long long ldi, void* stream);

/* out[b][i] = src[b][idx[b * ldi + i]] over D columns (sarbon_det.py:315-320) for the S rows
 * of each image (an index outside [0, S) gives a zero row); fp32 (o32) and/or fp16 (o16)
 * outputs. */
SB_API int sb_gather_rows(const void* src, int src_dtype, long long lds, long long imgs, int S, const void* idx, long long ldi,
                          int B, int K, int D, float* o32, long long ld32, long long img32, void* o16, long long ld16,
                          long long img16, void* stream);

/* MSDeformAttn after its three projections (deform_attn.py:57-66 and the core :14-28):
 * value fp16 [B][S][H*32] (L levels of level_hw[l] = (h, w), host memory), sampling offsets
 * fp16 [B][Q][H*L*P*2], attention logits fp16 [B][Q][H*L*P], reference boxes cxcywh [B][Q][4]
 * (ref_dtype: SB_F16 evaluates the location expression with fp16 roundings, as the
 * reference does for an fp16 box); writes fp16 [B][Q][H*32]. */
SB_API int sb_deform_sample(const void* value, long long ldv, long long imgv, const int* level_hw, int L, const void* off,
                            long long ldoff, long long imgoff, const void* att, long long ldatt, long long imgatt,
                            const void* ref, int ref_dtype, long long ldref, long long imgref, int B, int Q, int H, int P,
                            void* out, long long ldo, long long imgo, void* stream);

/* Encoder proposals of the selected rows (sarbon_det.py:316-321): ref16 [B*K][4] =
 * fp16(sigmoid(fp16(encbox + anchors[idx]))) (anchors fp16 [S][4]; an index outside [0, S)
 * takes a zero anchor); qin [B*K][ldq] gets the same 4 values (the query_pos input). */
SB_API int sb_box_enc(const void* encbox, long long ldb, const void* anchors, int S, const void* idx, int B, int K, void* ref16,
                      void* qin, long long ldq, void* stream);

/* Decoder box of one layer (sarbon_det.py:336-350, box_ops.py:78-106): first != 0 computes
 * ref_init = sigmoid(prebox + inverse_sigmoid(ref16)) and corners = head, else corners =
 * fp16(head + corners); then box [rows][4] = distance2bbox(ref_init, integral(corners),
 * reg_scale) with R1 bins per edge (project[R1] fp32), and qin = fp16(box) if non-NULL. */
SB_API int sb_box_dec(int first, const void* prebox, long long ldp, const void* ref16, const void* head, long long ldh,
                      void* corners, long long ldc, int R1, const float* project, float reg_scale, float* ref_init,
                      float* box, void* qin, long long ldq, int rows, void* stream);

/* F.normalize(x.float(), dim=-1) of fp16 rows into fp32 rows (sarbon_det.py:359-360). */
SB_API int sb_l2norm_rows(const void* x, long long ldx, int rows, int D, float* out, long long ldo, void* stream);

/* Counters (fused_engine.py:92,239) and sticky device errors (synchronises). */
SB_API int sb_stats(sb_engine* e, void* stream, sb_stats_t* out);

/* Number of CUDA kernels the last sb_step / sb_step_u8 / sb_reset launched. */
SB_API int sb_last_launch_count(sb_engine* e);

SB_API int sb_destroy(sb_engine* e);

/* Human-readable text of the last error on this thread (never NULL). */
SB_API const char* sb_last_error(void);

/* Library build tag, e.g. "sarbon_b200 sm_100a". */
SB_API const char* sb_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SARBON_SPARSE_H */
