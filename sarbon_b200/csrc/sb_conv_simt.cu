// sb_conv_simt.cu -- fp32 tile convolution on CUDA cores (engines with dtype float32).
//
// Reference: Bahrombekk/Sarbon sarbon/sparse/triton_conv.py:15-61, which for fp32 caches
// uses an IEEE fp32 dot (`input_precision="ieee"`, :49-52).  Tensor cores would round
// operands (TF32), so the fp32 engine keeps exact fp32 FMAs: gather the input window
// (zero padding at the image border) into shared memory 16 channels at a time,
// accumulate in shared memory, then bias -> (+residual) -> ReLU -> store.
#include <cstdint>

#include "sb_internal.cuh"
#include "sb_ptx.cuh"

namespace sb {

#define SIMT_THREADS 256
#define SIMT_CCH 16
#define SIMT_ACC_MAX 4096  // floats of accumulator per work item

__global__ void __launch_bounds__(SIMT_THREADS) conv_simt_kernel(ConvArgs a) {
  extern __shared__ float ssm[];
  const int T = a.t, S = a.s, cout = a.cout, cin = a.cin;
  const int mode = a.st->mode_cur;
  const int listed = a.st->counts[a.d_idx];
  int n_tiles = 0;
  if (mode == SB_MODE_DENSE) n_tiles = a.n_blocks;
  else if (mode == SB_MODE_SPARSE) n_tiles = a.st->force_tiles > 0 ? a.st->force_tiles : listed;
  if (n_tiles > a.n_blocks) n_tiles = a.n_blocks;
  if (n_tiles == 0) return;
  int R = SIMT_ACC_MAX / (T * cout);
  if (R < 1) R = 1;
  if (R > T) R = T;
  const int groups = (T + R - 1) / R;
  const int Ww = (T - 1) * S + 3, Rw = (R - 1) * S + 3;
  float* acc = ssm;                              // [R][T][cout]
  float* win = ssm + SIMT_ACC_MAX;               // [Rw][Ww][SIMT_CCH]
  const float* x = static_cast<const float*>(a.x);
  const float* w = static_cast<const float*>(a.wimg);
  float* y = static_cast<float*>(a.y);
  const float* res = static_cast<const float*>(a.res);
  const int per = a.hb * a.wb;
  const long long n_items = (long long)n_tiles * groups;
  for (long long item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int ti = (int)(item / groups), gi = (int)(item % groups);
    int cam = 0, by = 0, bx = 0;
    if (mode == SB_MODE_DENSE) {
      cam = ti / per;
      const int q = ti - cam * per;
      by = q / a.wb;
      bx = q - by * a.wb;
    } else if (ti < listed) {
      cam = a.lcam[ti];
      by = a.lby[ti];
      bx = a.lbx[ti];
    }
    if (cam >= a.n || by >= a.hb || bx >= a.wb) {
      if (threadIdx.x == 0) atomicOr(&a.st->error, SB_ERR_BAD_TILE);
      continue;
    }
    const int r0 = gi * R;
    const int rows = min(R, T - r0);
    const int n_out = rows * T * cout;
    for (int o = threadIdx.x; o < n_out; o += blockDim.x) acc[o] = 0.f;
    const int iy0 = (by * T + r0) * S - 1, ix0 = bx * T * S - 1;
    for (int c0 = 0; c0 < cin; c0 += SIMT_CCH) {
      const int cc = min(SIMT_CCH, cin - c0);
      __syncthreads();
      const int nwin = Rw * Ww * SIMT_CCH;
      for (int i = threadIdx.x; i < nwin; i += blockDim.x) {
        const int c = i % SIMT_CCH, px = (i / SIMT_CCH) % Ww, ry = i / (SIMT_CCH * Ww);
        const int iy = iy0 + ry, ix = ix0 + px;
        float v = 0.f;
        if (c < cc && iy >= 0 && iy < a.hx && ix >= 0 && ix < a.wx)
          v = x[(((size_t)cam * a.hx + iy) * a.wx + ix) * cin + c0 + c];
        win[i] = v;
      }
      __syncthreads();
      for (int o = threadIdx.x; o < n_out; o += blockDim.x) {
        const int co = o % cout, px = (o / cout) % T, ry = o / (cout * T);
        float s = acc[o];
        for (int ky = 0; ky < 3; ++ky)
          for (int kx = 0; kx < 3; ++kx) {
            const float* wp = w + ((size_t)((ky * 3 + kx) * cin + c0)) * cout + co;
            const float* xp = win + ((ry * S + ky) * Ww + (px * S + kx)) * SIMT_CCH;
            for (int c = 0; c < cc; ++c) s = fmaf(xp[c], wp[(size_t)c * cout], s);
          }
        acc[o] = s;
      }
    }
    __syncthreads();
    for (int o = threadIdx.x; o < n_out; o += blockDim.x) {
      const int co = o % cout, px = (o / cout) % T, ry = o / (cout * T);
      const int gy = by * T + r0 + ry, gx = bx * T + px;
      const size_t idx = (((size_t)cam * a.ho + gy) * a.wo + gx) * cout + co;
      float v = acc[o] + a.bias[co];
      if (res) v += res[idx];
      if (a.act) v = fmaxf(v, 0.f);
      y[idx] = v;
    }
    __syncthreads();
  }
}

cudaError_t launch_conv_simt(const ConvArgs& a, int grid_x, cudaStream_t s) {
  int R = SIMT_ACC_MAX / (a.t * a.cout);
  if (R < 1) R = 1;
  if (R > a.t) R = a.t;
  const int Ww = (a.t - 1) * a.s + 3, Rw = (R - 1) * a.s + 3;
  const size_t smem = (size_t)(SIMT_ACC_MAX + Rw * Ww * SIMT_CCH) * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(conv_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  conv_simt_kernel<<<grid_x, SIMT_THREADS, smem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace sb
