// sb_internal.cuh -- device state, kernel arguments and launcher declarations shared by
// the engine (sb_engine.cu) and the kernels (sb_gate.cu, sb_conv_tc.cu, sb_conv_simt.cu).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/sarbon_sparse.h"

namespace sb {

// Region kinds: groups of rw x rh blocks a window-mode conv processes as one unit (the
// block itself is kind "blocks" and has its own lists).
#define SB_MAX_RKINDS 3

// Blocks per CTA of the list kernel (a multiple of 32); the look-back status arrays hold
// one word per chunk = ceil(n_blocks / SB_LIST_CHUNK) per compaction lane.
#define SB_LIST_CHUNK 1024

// Device-resident engine state.  Written only by the engine's own kernels (and by
// cudaMemcpyAsync for host-set knobs), so a whole step runs without a host sync.
struct State {
  int64_t tick;         // refresh phase counter (fused_engine.py:80,146-147)
  int64_t count_cur;    // active count of the widest dilation this step; -1 = hysteresis dense
  int64_t fallback;     // dense above this count (fused_engine.py:89,232)
  int64_t stats[3];     // skip / sparse / dense steps (fused_engine.py:92,239)
  int64_t last_count;
  int32_t counts[SB_MAX_DILATIONS];  // active blocks per dilation this step
  int32_t mode_cur;     // SB_MODE_* of this step (read by the conv kernels)
  int32_t hyst_unused;
  int32_t dense_run;    // fused_engine.py:91 `_dense_run`
  int32_t check_every;  // fused_engine.py:91 `dense_check_every`
  int32_t force_tiles;  // >0: conv kernels process exactly this many list entries
  uint32_t epoch;       // tag of the block-list look-back words (never 0)
  uint32_t ticket;      // chunk ticket of the list kernel
  int32_t error;        // sticky SB_ERR_* flags
  int32_t last_mode;
  int32_t pad_;
  int64_t result[2];    // {mode, count} of the last finished step
  int32_t rcounts[SB_MAX_RKINDS][SB_MAX_DILATIONS];  // active regions per region kind and dilation
  // test hook (sb_debug_withhold_lookback): list chunk lb_withhold - 1 publishes no look-back
  // words (0 = none); look-back waits give up after lb_spin_limit polls (0 = SB_SPIN_LIMIT)
  int32_t lb_withhold;
  uint32_t lb_spin_limit;
  // M0 mode (sb_set_m0, block_sparse.py:253-295): every step copies the whole frame into the
  // image cache; m0_cap > 0 runs every layer over exactly m0_cap list entries (padding
  // entries recompute block 0); m0_cap = 0 runs the listed blocks (and skips when none)
  int32_t m0_mode;
  int32_t m0_cap;
};

struct GateArgs {
  const void* frames;      // [N][H][W][3]: fp16, fp32 or uint8 BGR
  void* img;               // image cache [N][H][W][3] in the engine dtype
  const uint8_t* extra;    // [N][Hb][Wb]
  uint8_t* changed;        // [N][Hb][Wb]
  State* st;
  int n, h, w, hb, wb, block;
  int seg;                 // blocks per CTA along the block row (set by launch_gate)
  int64_t thr_fx;          // floor(threshold * 2^24) (fp16/u8 paths); -1: always; INT64_MAX: never
  double thr;              // threshold as a double (fp32 path)
  double band_lo, band_hi; // fp32 sums outside [band_lo, band_hi] decide `sum > thr` exactly
  int refresh;
  float mean[3], stdv[3];  // u8 path normalisation (RGB order)
};

struct ListArgs {
  const uint8_t* changed;  // [n_blocks]
  uint8_t* masks;          // [n_dil][n_blocks]
  int32_t* lists;          // [n_dil][3][n_blocks] (cam, by, bx)
  int n_rk;                // region kinds
  int rw[SB_MAX_RKINDS], rh[SB_MAX_RKINDS];   // region shape in blocks
  int32_t* rlists[SB_MAX_RKINDS];             // [n_dil][3][rcap] (cam, ry, rx)
  unsigned long long* status;  // [(1+n_rk)*n_dil][n_chunks] look-back words
  State* st;
  int n_blocks, hb, wb, n_dil;
  int ds[SB_MAX_DILATIONS];
  // per-dilation source mask, dilated by ds[i] (nullptr: `changed`).  Cell-level gating
  // passes the block masks it computed from cells, with ds[i] = 0.
  const uint8_t* src[SB_MAX_DILATIONS];
};

struct CellGateArgs {      // cell-level gate (fp16 frames)
  const void* frames;      // [N][H][W][3] fp16
  void* img;               // image cache [N][H][W][3] fp16
  const uint8_t* extra;    // [N][Hb][Wb]
  uint8_t* changed;        // [N][Hb][Wb]: any cell of the block changed (or forced)
  uint8_t* cells;          // [N][H/cell][W/cell]
  State* st;
  int n, h, w, hb, wb, block, cell, k, hc, wc;
  int64_t thr_fx;          // floor(float32(tau * cell^2 * 3) * 2^24); -1: always; INT64_MAX: never
  int refresh;
};

struct CopyArgs {          // dense img copy or masked update
  const void* frames;
  void* img;
  const uint8_t* changed;  // masked update when non-null
  State* st;
  int n, h, w, hb, wb, block, elem_bytes;
  int u8;                  // frames are uint8 BGR (normalise)
  float mean[3], stdv[3];
};

struct ConvArgs {
  const void* x;           // src cache (used directly by the gather producers)
  void* y;                 // dst cache
  const void* res;         // residual cache or nullptr
  const float* bias;       // [cout] fp32
  const void* wimg;        // fp16 path: pre-swizzled weight image; fp32 path: w [3][3][cin][cout]
  const int32_t* lcam;
  const int32_t* lby;
  const int32_t* lbx;
  State* st;
  int d_idx;
  int n, hx, wx, cin;
  int ho, wo, cout;
  int hb, wb, n_blocks;
  int t, s, act;
  int rkind;               // -1: units are blocks; else the region kind of rcam/rry/rrx
  int rw, rh;              // region shape in blocks (1, 1 for blocks)
  const int32_t* rcam;     // region lists of this layer's dilation
  const int32_t* rry;
  const int32_t* rrx;
  // bias by value (kernel parameter space): epilogue reads are warp-uniform and go through
  // the constant cache, off the shared-memory path the tensor pipe saturates
  alignas(16) float bias_v[128];
  // e4m3 caches (Q > 0 variants): per output channel s_in * s_w[c] (Q = 2), the residual
  // cache's activation scale and 1 / the output cache's activation scale
  alignas(16) float dq_v[128];
  float res_scale;
  float out_inv_scale;
};

// ---------------------------------------------------------------- launchers
cudaError_t launch_gate(const GateArgs& a, int kind /*0 f16, 1 f32, 2 u8*/, cudaStream_t s);
cudaError_t launch_lists(const ListArgs& a, int n_chunks, cudaStream_t s);
cudaError_t launch_copy(const CopyArgs& a, cudaStream_t s);
cudaError_t launch_finalize(State* st, int refresh, int32_t* host_out, cudaStream_t s);
cudaError_t launch_set_mode(State* st, int mode, int reset_hyst, int64_t force_tiles, cudaStream_t s);
cudaError_t launch_cell_gate(const CellGateArgs& a, cudaStream_t s);
// block masks [n_r][n][hc/k][wc/k] of cells [n][hc][wc] dilated by rc[i] cells (sb_cells.cu)
cudaError_t launch_cell_masks(const uint8_t* cells, int n, int hc, int wc, int k, const int* rc, int n_r,
                              uint8_t* out, cudaStream_t s);

// fp16 tcgen05 path.  Returns cudaErrorInvalidValue for shapes without an instantiation.
bool conv_tc_supported(int cin, int cout, int t, int s);  // some mode exists for the shape
// the e4m3 variant of a layer: q = 1 (fp16 input, e4m3 output) or 2 (e4m3 input, weights,
// residual and output); returns its mode, or -1 when the shape has none
int conv_tc_q_mode(int cin, int cout, int t, int s, int q);
// mode the engine runs a layer with: window mode 0 per-tap im2col (or first-layer gather),
// 1 per-ky row windows over (8/t)x1-block regions, 3 full windows over (8/t)x(16/t)
// regions; plus 8 when 2-CTA clusters run M=256 cta_group::2 MMAs
int conv_tc_pick_mode(int cin, int cout, int t, int s);
// a mode whose units are single blocks (window mode 0, or a window mode whose region is one
// block), CTA pairs preferred; -1 when the shape has none
int conv_tc_block_mode(int cin, int cout, int t, int s);
int conv_tc_nsplit(int cin, int cout, int t, int s, int mode, int q = 0);   // CTA splits of cout
size_t conv_tc_wimg_bytes(int cin, int cout, int t, int s, int mode, int q = 0);  // all splits
// weight image (fp16 bits, or e4m3 codes for q = 2 with wscale[c] = the scale of output
// channel c: w = code * wscale[c])
void conv_tc_build_wimg(int cin, int cout, int t, int s, int mode, const float* w /*[3][3][cin][cout]*/,
                        const float* bias /*[cout]*/, uint16_t* out, int q = 0, float* wscale = nullptr);
cudaError_t conv_tc_make_tmap(CUtensorMap* map, const void* src, int n, int hx, int wx, int cin, int t, int s,
                              int mode, int q = 0);
// the destination cache's map for the variants whose epilogue stages its output in shared
// memory and writes it with TMA tile stores (zero-filled and unused for the others)
cudaError_t conv_tc_make_tmap_out(CUtensorMap* map, void* dst, int n, int ho, int wo, int cin, int cout, int t, int s,
                                  int mode);
cudaError_t launch_conv_tc(const ConvArgs& a, int mode, const CUtensorMap* map, const CUtensorMap* map_y, int grid_x,
                           cudaStream_t s, int q = 0);
int conv_tc_max_ctas_per_sm(int cin, int cout, int t, int s, int mode);

// uint8 BGR frames at camera size -> bilinear resize (align_corners=False) -> RGB,
// (x - mean) / std, fp16 NHWC at engine size (sb_prep.cu)
cudaError_t launch_prep_resize(const uint8_t* src, int n, int hin, int win, __half* dst, int hout, int wout,
                               const float mean[3], const float stdv[3], int n_sms, cudaStream_t s);

// Look-back test hook of sb_block_lists_static's calls launched after this one
// (sb_debug_withhold_lookback with a NULL engine; sb_noalloc.cu).
void static_lists_debug(int withhold_chunk, unsigned spin_limit);

// Sets the message sb_last_error() returns on this thread; returns `code`.
int record_error(int code, const char* msg);

// fp32 CUDA-core path
cudaError_t launch_conv_simt(const ConvArgs& a, int grid_x, cudaStream_t s);

}  // namespace sb
