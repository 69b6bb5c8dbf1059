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
// image), changed.  One thread per (radius, camera, block) ORs that window; masks are
// bytes, so the result is exact.
#include <cstdio>
#include <string>

#include "sb_internal.cuh"

namespace sb {
namespace {

constexpr int kMaxRadii = 16;

struct CellArgs {
  const uint8_t* cells;  // [n][hc][wc], nonzero = changed
  uint8_t* out;          // [n_r][n][hc / k][wc / k]
  int n, hc, wc, k, hb, wb, n_r;
  int r[kMaxRadii];      // dilation in cells per output mask
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

}  // namespace
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
  CellArgs a{};
  a.cells = cells_dev;
  a.out = out_dev;
  a.n = n_cams;
  a.hc = hc;
  a.wc = wc;
  a.k = k;
  a.hb = hc / k;
  a.wb = wc / k;
  a.n_r = n_radii;
  for (int i = 0; i < n_radii; ++i) {
    if (radii[i] < 0) return record_error(SB_EINVAL, "sb_cell_active_blocks: negative radius");
    a.r[i] = (radii[i] + cell - 1) / cell;  // ceil(R / cell) cells (gating.py:43)
  }
  const long long total = (long long)n_radii * n_cams * a.hb * a.wb;
  if (total > (1ll << 31) - 256) return record_error(SB_EINVAL, "sb_cell_active_blocks: output too large");
  const int threads = 256;
  const int grid = (int)((total + threads - 1) / threads);
  cell_active_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  cudaError_t rc = cudaGetLastError();
  if (rc != cudaSuccess)
    return record_error(SB_ECUDA, (std::string("sb_cell_active_blocks: launch: ") + cudaGetErrorString(rc)).c_str());
  return SB_OK;
}
