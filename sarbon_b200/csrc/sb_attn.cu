// sb_attn.cu -- multi-head attention core of the detector (softmax(q k^T / sqrt(dh)) v).
//
// Reference: Bahrombekk/Sarbon sarbon/models/sarbon_det.py -- the encoder's
// nn.TransformerEncoderLayer on the stride-32 tokens (:129,146) and every decoder layer's
// nn.MultiheadAttention over the queries (:160,169); under the reference's autocast both
// run scaled_dot_product_attention on fp16 q / k / v with fp32 softmax.
//
// Flash-attention layout on the tensor cores (mma.sync m16n8k16, fp16 operands, fp32
// accumulation), dh = 32: a CTA of 4 warps takes 64 queries of one (image, head), each warp
// 16 of them with its Q fragments in registers; key / value tiles of 64 rows are staged in
// shared memory (V transposed, rows padded so that fragment loads hit 32 distinct banks).
// Per tile: S = Q K^T (8 x 2 MMAs), scaled to base 2, masked past Tk, online softmax in
// fp32 with one rescale of the running row sums and outputs, P rounded to fp16 and reused
// in registers as the A operand of O += P V (4 x 4 MMAs).
#include <cuda_fp16.h>

#include <cstdint>

#include "sb_internal.cuh"

namespace sb {
namespace {

constexpr int kQ = 64;      // queries per CTA
constexpr int kKT = 64;     // keys per tile
constexpr int kDH = 32;
constexpr int kKPad = 40;   // sK row: 32 dims + 8 pad (halves)
constexpr int kVPad = 72;   // sVt row: 64 keys + 8 pad (halves)

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__global__ void __launch_bounds__(128) flash_attention_kernel(const __half* q, long long ldq, long long imgq,
                                                              const __half* k, long long ldk, long long imgk,
                                                              const __half* v, long long ldv, long long imgv, int Tq,
                                                              int Tk, float scale_log2, __half* out, long long ldo,
                                                              long long imgo) {
  __shared__ __align__(16) __half sK[kKT][kKPad];
  __shared__ __align__(16) __half sVt[kDH][kVPad];
  const int h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int r0 = blockIdx.x * kQ + warp * 16 + g, r1 = r0 + 8;
  const __half* qb = q + (long long)b * imgq * ldq + h * kDH;
  const __half* kb = k + (long long)b * imgk * ldk + h * kDH;
  const __half* vb = v + (long long)b * imgv * ldv + h * kDH;

  // Q fragments of the two 16-dim k-steps
  uint32_t qa[2][4];
#pragma unroll
  for (int ks = 0; ks < 2; ++ks) {
    const int c0 = ks * 16 + 2 * tig;
    qa[ks][0] = r0 < Tq ? *reinterpret_cast<const uint32_t*>(qb + (long long)r0 * ldq + c0) : 0u;
    qa[ks][1] = r1 < Tq ? *reinterpret_cast<const uint32_t*>(qb + (long long)r1 * ldq + c0) : 0u;
    qa[ks][2] = r0 < Tq ? *reinterpret_cast<const uint32_t*>(qb + (long long)r0 * ldq + c0 + 8) : 0u;
    qa[ks][3] = r1 < Tq ? *reinterpret_cast<const uint32_t*>(qb + (long long)r1 * ldq + c0 + 8) : 0u;
  }
  float o[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) o[i][j] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  for (int t0 = 0; t0 < Tk; t0 += kKT) {
    __syncthreads();  // the previous tile's fragments have been read
    for (int pce = threadIdx.x; pce < kKT * 4; pce += 128) {
      const int r = pce >> 2, c = (pce & 3) * 8;
      uint4 kr = make_uint4(0, 0, 0, 0), vr = make_uint4(0, 0, 0, 0);
      if (t0 + r < Tk) {
        kr = *reinterpret_cast<const uint4*>(kb + (long long)(t0 + r) * ldk + c);
        vr = *reinterpret_cast<const uint4*>(vb + (long long)(t0 + r) * ldv + c);
      }
      *reinterpret_cast<uint4*>(&sK[r][c]) = kr;
      const __half* vh = reinterpret_cast<const __half*>(&vr);
#pragma unroll
      for (int u = 0; u < 8; ++u) sVt[c + u][r] = vh[u];
    }
    __syncthreads();
    // S = Q K^T for 8 groups of 8 keys
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&sK[nt * 8 + g][ks * 16 + 2 * tig]);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&sK[nt * 8 + g][ks * 16 + 8 + 2 * tig]);
        mma16816(s[nt], qa[ks], b0, b1);
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int key = t0 + nt * 8 + 2 * tig;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool ok = key + e < Tk;
        s[nt][e] = ok ? s[nt][e] * scale_log2 : -INFINITY;
        s[nt][2 + e] = ok ? s[nt][2 + e] * scale_log2 : -INFINITY;
        mx0 = fmaxf(mx0, s[nt][e]);
        mx1 = fmaxf(mx1, s[nt][2 + e]);
      }
    }
#pragma unroll
    for (int x = 1; x <= 2; x <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xFFFFFFFFu, mx0, x));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xFFFFFFFFu, mx1, x));
    }
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float c0 = exp2f(m0 - mn0), c1 = exp2f(m1 - mn1);  // 0 on the first tile
    l0 *= c0;
    l1 *= c1;
#pragma unroll
    for (int nd = 0; nd < 4; ++nd) {
      o[nd][0] *= c0;
      o[nd][1] *= c0;
      o[nd][2] *= c1;
      o[nd][3] *= c1;
    }
    uint32_t pa[8][2];  // P rounded to fp16: rows g (index 0) and g + 8 (index 1)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const float p0 = exp2f(s[nt][0] - mn0), p1 = exp2f(s[nt][1] - mn0);
      const float p2 = exp2f(s[nt][2] - mn1), p3 = exp2f(s[nt][3] - mn1);
      l0 += p0 + p1;
      l1 += p2 + p3;
      pa[nt][0] = pack_half2(p0, p1);
      pa[nt][1] = pack_half2(p2, p3);
    }
    m0 = mn0;
    m1 = mn1;
    // O += P V over 4 k-steps of 16 keys
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const uint32_t a[4] = {pa[2 * ks][0], pa[2 * ks][1], pa[2 * ks + 1][0], pa[2 * ks + 1][1]};
#pragma unroll
      for (int nd = 0; nd < 4; ++nd) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&sVt[nd * 8 + g][ks * 16 + 2 * tig]);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&sVt[nd * 8 + g][ks * 16 + 8 + 2 * tig]);
        mma16816(o[nd], a, b0, b1);
      }
    }
  }
#pragma unroll
  for (int x = 1; x <= 2; x <<= 1) {
    l0 += __shfl_xor_sync(0xFFFFFFFFu, l0, x);
    l1 += __shfl_xor_sync(0xFFFFFFFFu, l1, x);
  }
  const float i0 = 1.f / l0, i1 = 1.f / l1;
  __half* ob = out + (long long)b * imgo * ldo + h * kDH;
#pragma unroll
  for (int nd = 0; nd < 4; ++nd) {
    const int c = nd * 8 + 2 * tig;
    if (r0 < Tq) *reinterpret_cast<__half2*>(ob + (long long)r0 * ldo + c) = __floats2half2_rn(o[nd][0] * i0, o[nd][1] * i0);
    if (r1 < Tq) *reinterpret_cast<__half2*>(ob + (long long)r1 * ldo + c) = __floats2half2_rn(o[nd][2] * i1, o[nd][3] * i1);
  }
}

}  // namespace
}  // namespace sb

using namespace sb;

extern "C" int sb_attention(const void* q, long long ldq, long long imgq, const void* k, long long ldk, long long imgk,
                            const void* v, long long ldv, long long imgv, int B, int H, int dh, int Tq, int Tk,
                            void* out, long long ldo, long long imgo, void* stream) {
  if (!q || !k || !v || !out || dh != kDH || B < 1 || H < 1 || Tq < 1 || Tk < 1 || H > 65535 || B > 65535 ||
      ldq % 8 || ldk % 8 || ldv % 8 || ldo % 8 || (reinterpret_cast<uintptr_t>(q) & 15) ||
      (reinterpret_cast<uintptr_t>(k) & 15) || (reinterpret_cast<uintptr_t>(v) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 15))
    return record_error(SB_EINVAL, "sb_attention: arguments (dh = 32, 16-byte rows)");
  const float scale_log2 = 1.4426950408889634f / sqrtf((float)dh);
  flash_attention_kernel<<<dim3((unsigned)((Tq + kQ - 1) / kQ), H, B), 128, 0, (cudaStream_t)stream>>>(
      static_cast<const __half*>(q), ldq, imgq, static_cast<const __half*>(k), ldk, imgk,
      static_cast<const __half*>(v), ldv, imgv, Tq, Tk, scale_log2, static_cast<__half*>(out), ldo, imgo);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return record_error(SB_ECUDA, cudaGetErrorString(e));
  return SB_OK;
}
