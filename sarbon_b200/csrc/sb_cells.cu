// sb_cells.cu -- cell-level gating: which blocks a change of c x c-pixel cells reaches.
//
// Reference: Bahrombekk/Sarbon sarbon/sparse/gating.py:42-43 (`active_blocks_cell_level`):
// the change mask of cells is dilated by ceil(R / c) cells (max_pool2d, stride 1, zero
// padding, gating.py:25-28) and any-pooled into blocks of (block / c)^2 cells
// (gating.py:31-34).  A change in the middle of a block then no longer activates the whole
// ring of neighbouring blocks that the block-level estimate (changed blocks dilated by
// ceil(R / block), gating.py:37-39) does.
//
// The two steps compose into one test per output block: it is active when any cell in the
// block's own cell range, widened by the cell radius on every side (and clipped to the
// image), changed.
//
// cell_bits_kernel: one CTA per (camera, block row).  Its warps pack the cell rows that the
// largest radius reaches into bit rows in shared memory (one __ballot_sync per 32 cells),
// then each thread answers one (radius, block) by ORing, over the window's rows, the one or
// two words that hold the window's columns, and masking the column range.  When the bit rows
// do not fit in 48 KB (very wide images with very large radii), cell_active_kernel ORs each
// window's bytes straight from global memory instead.  Both are exact.
#include <algorithm>
#include <cstdio>
#include <string>

#include "sb_internal.cuh"

namespace sb {
namespace {

constexpr int kMaxRadii = 16;

constexpr int kBitsSmemMax = 48 * 1024;

struct CellArgs {
  const uint8_t* cells;  // [n][hc][wc], nonzero = changed
  uint8_t* out;          // [n_r][n][hc / k][wc / k]
  int n, hc, wc, k, hb, wb, n_r;
  int r[kMaxRadii];      // dilation in cells per output mask
  int rmax, wpr;         // largest r; 32-bit words per bit row
};

__global__ void __launch_bounds__(256) cell_active_kernel(const CellArgs a) {
  const long long per = (long long)a.n * a.hb * a.wb;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= per * a.n_r) return;
  const int ri = (int)(idx / per);
  const long long f = idx - ri * per;
  const int cam = (int)(f / ((long long)a.hb * a.wb));
  const int q = (int)(f - (long long)cam * a.hb * a.wb);
  const int by = q / a.wb, bx = q - by * a.wb;
  const int r = a.r[ri];
  const int y0 = max(0, by * a.k - r), y1 = min(a.hc - 1, by * a.k + a.k - 1 + r);
  const int x0 = max(0, bx * a.k - r), x1 = min(a.wc - 1, bx * a.k + a.k - 1 + r);
  const uint8_t* base = a.cells + (size_t)cam * a.hc * a.wc;
  uint32_t acc = 0;
  for (int y = y0; y <= y1; ++y) {
    const uint8_t* row = base + (size_t)y * a.wc;
#pragma unroll 4
    for (int x = x0; x <= x1; ++x) acc |= __ldg(row + x);
  }
  a.out[idx] = acc != 0 ? 1 : 0;
}

__global__ void __launch_bounds__(256) cell_bits_kernel(const CellArgs a) {
  extern __shared__ uint32_t s_bits[];  // [rows][wpr], bit l of word w = cell column 32 w + l
  const int by = blockIdx.x, cam = blockIdx.y;
  const int ybase = max(0, by * a.k - a.rmax);
  const int yend = min(a.hc - 1, by * a.k + a.k - 1 + a.rmax);
  const int nwords = (yend - ybase + 1) * a.wpr;
  const uint8_t* base = a.cells + (size_t)cam * a.hc * a.wc;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  // warp-uniform loop (every lane votes); eight words per warp and pass, their byte loads
  // issued together
  constexpr int U = 8;
  for (int t0 = warp * U; t0 < nwords; t0 += nwarps * U) {
    bool on[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int t = t0 + j;
      const int y = t / a.wpr, w = t - y * a.wpr;
      const int x = w * 32 + lane;
      on[j] = t < nwords && x < a.wc && __ldg(base + (size_t)(ybase + y) * a.wc + x) != 0;
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const uint32_t word = __ballot_sync(0xffffffffu, on[j]);
      if (lane == 0 && t0 + j < nwords) s_bits[t0 + j] = word;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < a.n_r * a.wb; i += blockDim.x) {
    const int ri = i / a.wb, bx = i - ri * a.wb;
    const int r = a.r[ri];
    const int y0 = max(0, by * a.k - r) - ybase, y1 = min(a.hc - 1, by * a.k + a.k - 1 + r) - ybase;
    const int x0 = max(0, bx * a.k - r), x1 = min(a.wc - 1, bx * a.k + a.k - 1 + r);
    uint32_t hit = 0;
    for (int w = x0 >> 5; w <= (x1 >> 5); ++w) {
      const int lo = max(x0 - 32 * w, 0), hi = min(x1 - 32 * w, 31);
      const uint32_t m = (hi == 31 ? 0xffffffffu : (1u << (hi + 1)) - 1u) & (0xffffffffu << lo);
      uint32_t acc = 0;
      for (int y = y0; y <= y1; ++y) acc |= s_bits[y * a.wpr + w];
      hit |= acc & m;
    }
    a.out[(((size_t)ri * a.n + cam) * a.hb + by) * a.wb + bx] = hit ? 1 : 0;
  }
}

}  // namespace

// Shared by the entry point below and the engine's cell-level gating: radii rc[] in cells.
cudaError_t launch_cell_masks(const uint8_t* cells, int n, int hc, int wc, int k, const int* rc, int n_r,
                              uint8_t* out, cudaStream_t s) {
  if (n_r < 1 || n_r > kMaxRadii || k <= 0 || hc % k || wc % k) return cudaErrorInvalidValue;
  CellArgs a{};
  a.cells = cells;
  a.out = out;
  a.n = n;
  a.hc = hc;
  a.wc = wc;
  a.k = k;
  a.hb = hc / k;
  a.wb = wc / k;
  a.n_r = n_r;
  const int rcap = hc > wc ? hc : wc;  // a larger radius reaches no further cell
  for (int i = 0; i < n_r; ++i) {
    if (rc[i] < 0) return cudaErrorInvalidValue;
    a.r[i] = rc[i] < rcap ? rc[i] : rcap;
    a.rmax = a.r[i] > a.rmax ? a.r[i] : a.rmax;
  }
  const long long total = (long long)n_r * n * a.hb * a.wb;
  if (total > (1ll << 31) - 256) return cudaErrorInvalidValue;
  a.wpr = (wc + 31) / 32;
  const long long rows = std::min<long long>(hc, (long long)k + 2ll * a.rmax);
  const long long bits_smem = rows * a.wpr * 4;
  const int threads = 256;
  if (bits_smem <= kBitsSmemMax && n <= 65535) {
    cell_bits_kernel<<<dim3(a.hb, n), threads, (size_t)bits_smem, s>>>(a);
  } else {
    const int grid = (int)((total + threads - 1) / threads);
    cell_active_kernel<<<grid, threads, 0, s>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace sb

using namespace sb;

extern "C" int sb_cell_active_blocks(const uint8_t* cells_dev, int n_cams, int hc, int wc, int cell, int block,
                                     const int* radii, int n_radii, uint8_t* out_dev, void* stream) {
  if (!cells_dev || !out_dev || !radii) return record_error(SB_EINVAL, "sb_cell_active_blocks: null pointer argument");
  if (n_cams <= 0 || hc <= 0 || wc <= 0)
    return record_error(SB_EINVAL, "sb_cell_active_blocks: n_cams, hc and wc must be positive");
  if (cell <= 0 || block <= 0 || block % cell)
    return record_error(SB_EINVAL, "sb_cell_active_blocks: the block size must be a positive multiple of the cell size");
  const int k = block / cell;
  if (hc % k || wc % k)
    return record_error(SB_EINVAL, "sb_cell_active_blocks: hc and wc must be multiples of block / cell");
  if (n_radii < 1 || n_radii > kMaxRadii)
    return record_error(SB_EINVAL, "sb_cell_active_blocks: n_radii must be in [1, 16]");
  int rc_cells[kMaxRadii];
  for (int i = 0; i < n_radii; ++i) {
    if (radii[i] < 0) return record_error(SB_EINVAL, "sb_cell_active_blocks: negative radius");
    rc_cells[i] = radii[i] / cell + (radii[i] % cell != 0);  // ceil(R / cell) cells (gating.py:43)
  }
  if ((long long)n_radii * n_cams * (hc / k) * (wc / k) > (1ll << 31) - 256)
    return record_error(SB_EINVAL, "sb_cell_active_blocks: output too large");
  cudaError_t rc = launch_cell_masks(cells_dev, n_cams, hc, wc, k, rc_cells, n_radii, out_dev,
                                     static_cast<cudaStream_t>(stream));
  if (rc != cudaSuccess)
    return record_error(SB_ECUDA, (std::string("sb_cell_active_blocks: launch: ") + cudaGetErrorString(rc)).c_str());
  return SB_OK;
}
