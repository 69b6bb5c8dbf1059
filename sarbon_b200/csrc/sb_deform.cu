// sb_deform.cu -- fused multi-scale deformable attention core of the detector after the stem.
//
// Reference: Bahrombekk/Sarbon sarbon/models/deform_attn.py:14-28 (`ms_deform_attn_core`):
// for every (batch, query, head) the value maps of L levels are sampled at P points each
// with F.grid_sample(mode="bilinear", padding_mode="zeros", align_corners=False) and the
// samples are summed with the softmaxed attention weights.  PyTorch runs it as L
// grid_sample launches on permuted copies of the value, a stack, a product and a sum; the
// reference's docstring names this function as the place for a fused kernel.
//
// Here one warp handles one (batch, query, head): the sampling locations and weights are
// warp-uniform, the lanes cover the head's channels (value rows are [S][H][D], so a corner
// read is D contiguous elements), and the L*P weighted bilinear samples are accumulated in
// fp32 registers; the output row [H*D] of the query is written once.  Work per query is
// H * L * P * 4 corner reads of D elements: gather-bound, no tensor cores.
//
// Sampling rule (grid_sample, align_corners=False, zeros padding): grid = 2 * loc - 1, source
// coordinate ((grid + 1) * size - 1) / 2, the four neighbours weighted by the opposite areas,
// neighbours outside the map contribute zero.
#include <cuda_fp16.h>

#include "sb_internal.cuh"

namespace sb {
namespace {

constexpr int kMaxLevels = 8;

struct DeformArgs {
  const void* value;      // [B][S][H][D], fp32 or fp16
  const float* loc;       // [B][Q][H][L][P][2] in [0, 1] (x, y)
  const float* weight;    // [B][Q][H][L][P]
  void* out;              // [B][Q][H*D], the value's type
  int B, S, H, D, Q, L, P;
  int lh[kMaxLevels], lw[kMaxLevels], lstart[kMaxLevels];
};

template <typename T>
__device__ __forceinline__ float load_f(const T* p);
template <>
__device__ __forceinline__ float load_f<float>(const float* p) {
  return __ldg(p);
}
template <>
__device__ __forceinline__ float load_f<__half>(const __half* p) {
  return __half2float(__ldg(p));
}

template <typename T>
__global__ void __launch_bounds__(256) deform_kernel(DeformArgs a) {
  const int warp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  const int total = a.B * a.Q * a.H;
  if (warp >= total) return;
  const int h = warp % a.H, q = (warp / a.H) % a.Q, b = warp / (a.H * a.Q);
  const T* value = static_cast<const T*>(a.value);
  const size_t lp = (size_t)a.L * a.P;
  const float* locp = a.loc + ((size_t)(b * a.Q + q) * a.H + h) * lp * 2;
  const float* wp = a.weight + ((size_t)(b * a.Q + q) * a.H + h) * lp;
  for (int d0 = 0; d0 < a.D; d0 += 32) {
    const int d = d0 + lane;
    const bool on = d < a.D;
    float acc = 0.f;
    for (int l = 0; l < a.L; ++l) {
      const int H_ = a.lh[l], W_ = a.lw[l];
      const T* vl = value + ((size_t)b * a.S + a.lstart[l]) * a.H * a.D + (size_t)h * a.D + d;
      const size_t row = (size_t)a.H * a.D;  // stride between value positions
      for (int p = 0; p < a.P; ++p) {
        const size_t k = (size_t)l * a.P + p;
        const float gx = __fsub_rn(__fmul_rn(2.f, locp[2 * k]), 1.f);
        const float gy = __fsub_rn(__fmul_rn(2.f, locp[2 * k + 1]), 1.f);
        const float ix = __fdiv_rn(__fsub_rn(__fmul_rn(__fadd_rn(gx, 1.f), (float)W_), 1.f), 2.f);
        const float iy = __fdiv_rn(__fsub_rn(__fmul_rn(__fadd_rn(gy, 1.f), (float)H_), 1.f), 2.f);
        const float fx = floorf(ix), fy = floorf(iy);
        const int x0 = (int)fx, y0 = (int)fy;
        const float tx = __fsub_rn(ix, fx), ty = __fsub_rn(iy, fy);
        const float w_nw = __fmul_rn(__fsub_rn(__fadd_rn(fx, 1.f), ix), __fsub_rn(__fadd_rn(fy, 1.f), iy));
        const float w_ne = __fmul_rn(tx, __fsub_rn(__fadd_rn(fy, 1.f), iy));
        const float w_sw = __fmul_rn(__fsub_rn(__fadd_rn(fx, 1.f), ix), ty);
        const float w_se = __fmul_rn(tx, ty);
        float s = 0.f;
        if (on) {
          const bool x0in = x0 >= 0 && x0 < W_, x1in = x0 + 1 >= 0 && x0 + 1 < W_;
          const bool y0in = y0 >= 0 && y0 < H_, y1in = y0 + 1 >= 0 && y0 + 1 < H_;
          if (y0in && x0in) s = fmaf(load_f(vl + ((size_t)y0 * W_ + x0) * row), w_nw, s);
          if (y0in && x1in) s = fmaf(load_f(vl + ((size_t)y0 * W_ + x0 + 1) * row), w_ne, s);
          if (y1in && x0in) s = fmaf(load_f(vl + ((size_t)(y0 + 1) * W_ + x0) * row), w_sw, s);
          if (y1in && x1in) s = fmaf(load_f(vl + ((size_t)(y0 + 1) * W_ + x0 + 1) * row), w_se, s);
        }
        acc = fmaf(s, wp[k], acc);
      }
    }
    if (on) {
      const size_t o = ((size_t)(b * a.Q + q) * a.H + h) * a.D + d;
      if constexpr (sizeof(T) == 4) static_cast<float*>(a.out)[o] = acc;
      else static_cast<__half*>(a.out)[o] = __float2half_rn(acc);
    }
  }
}

}  // namespace
}  // namespace sb

using namespace sb;

extern "C" int sb_ms_deform_attn(const void* value, int value_dtype, int B, int S, int H, int D,
                                 const int* level_hw, int L, const float* loc, const float* weight, int Q, int P,
                                 void* out, void* stream) {
  if (!value || !level_hw || !loc || !weight || !out) return record_error(SB_EINVAL, "sb_ms_deform_attn: null argument");
  if (value_dtype != SB_F16 && value_dtype != SB_F32) return record_error(SB_EINVAL, "sb_ms_deform_attn: dtype");
  if (B < 1 || S < 1 || H < 1 || D < 1 || Q < 1 || P < 1 || L < 1 || L > kMaxLevels)
    return record_error(SB_EINVAL, "sb_ms_deform_attn: sizes out of range (1 <= L <= 8)");
  DeformArgs a{};
  a.value = value;
  a.loc = loc;
  a.weight = weight;
  a.out = out;
  a.B = B;
  a.S = S;
  a.H = H;
  a.D = D;
  a.Q = Q;
  a.L = L;
  a.P = P;
  long long start = 0;
  for (int l = 0; l < L; ++l) {
    if (level_hw[2 * l] < 1 || level_hw[2 * l + 1] < 1) return record_error(SB_EINVAL, "sb_ms_deform_attn: level size");
    a.lh[l] = level_hw[2 * l];
    a.lw[l] = level_hw[2 * l + 1];
    a.lstart[l] = (int)start;
    start += (long long)a.lh[l] * a.lw[l];
  }
  if (start != S) return record_error(SB_EINVAL, "sb_ms_deform_attn: the level sizes do not add up to S");
  const long long warps = (long long)B * Q * H;
  const unsigned blocks = (unsigned)((warps * 32 + 255) / 256);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (value_dtype == SB_F32) deform_kernel<float><<<blocks, 256, 0, s>>>(a);
  else deform_kernel<__half><<<blocks, 256, 0, s>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return record_error(SB_ECUDA, cudaGetErrorString(e));
  return SB_OK;
}
