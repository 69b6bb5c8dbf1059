// sb_attn.cu -- multi-head attention core of the detector (softmax(q k^T / sqrt(dh)) v).
//
// Reference: Bahrombekk/Sarbon sarbon/models/sarbon_det.py -- the encoder's
// nn.TransformerEncoderLayer on the stride-32 tokens (:129,146) and every decoder layer's
// nn.MultiheadAttention over the queries (:160,169); under the reference's autocast both
// run scaled_dot_product_attention on fp16 q / k / v with fp32 softmax.
//
// Flash-attention layout on the tensor cores (mma.sync m16n8k16, fp16 operands, fp32
// accumulation), dh = 32: a CTA of 4 warps takes 64 queries of one (image, head), each warp
// 16 of them with its Q fragments in registers.  Key / value tiles of 64 rows are
// double-buffered in shared memory by cp.async (rows past Tk zero-filled), so the next
// tile's copy overlaps this tile's math; K and V keep their row-major [key][dim] layout
// (rows padded to 80 bytes, so the eight 16-byte rows an ldmatrix phase reads fall in
// distinct banks) and the B fragments come from ldmatrix (K) and ldmatrix.trans (V).
// Per tile: S = Q K^T (8 x 2 MMAs), masked past Tk on the last tile, online softmax in fp32
// (p = 2^(s * scale * log2 e - m), one FFMA and one ex2 per score), P rounded to fp16 and
// reused in registers as the A operand of O += P V (4 x 4 MMAs).
#include <cuda_fp16.h>

#include <cstdint>

#include "sb_internal.cuh"

namespace sb {
namespace {

constexpr int kQ = 64;      // queries per CTA (4 warps)
constexpr int kKT = 64;     // keys per tile
constexpr int kDH = 32;
constexpr int kPad = 40;    // shared row: 32 dims + 8 pad (halves)

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

__device__ __forceinline__ uint32_t saddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte global -> shared copy; `bytes` = 0 writes zeros and reads nothing
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__global__ void __launch_bounds__(128) flash_attention_kernel(const __half* q, long long ldq, long long imgq,
                                                              const __half* k, long long ldk, long long imgk,
                                                              const __half* v, long long ldv, long long imgv, int Tq,
                                                              int Tk, float scale_log2, __half* out, long long ldo,
                                                              long long imgo) {
  __shared__ __align__(128) __half sK[2][kKT][kPad];
  __shared__ __align__(128) __half sV[2][kKT][kPad];
  const int h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int r0 = blockIdx.x * kQ + warp * 16 + g, r1 = r0 + 8;
  const __half* qb = q + (long long)b * imgq * ldq + h * kDH;
  const __half* kb = k + (long long)b * imgk * ldk + h * kDH;
  const __half* vb = v + (long long)b * imgv * ldv + h * kDH;

  // one tile: 64 rows x four 16-byte pieces of K and of V
  auto load_tile = [&](int t0, int buf) {
    for (int pce = threadIdx.x; pce < kKT * 4; pce += 128) {
      const int r = pce >> 2, c = (pce & 3) * 8;
      const bool ok = t0 + r < Tk;
      const long long row = ok ? t0 + r : 0;
      cp_async16(saddr(&sK[buf][r][c]), kb + row * ldk + c, ok ? 16 : 0);
      cp_async16(saddr(&sV[buf][r][c]), vb + row * ldv + c, ok ? 16 : 0);
    }
    cp_async_commit();
  };
  const int ntiles = (Tk + kKT - 1) / kKT;
  load_tile(0, 0);

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
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // running maxima of the raw scores
  // ldmatrix row addresses of this lane: K rows nt*8 + (lane & 7), dims (lane >> 3) * 8;
  // V rows ks*16 + ((lane >> 3) & 1) * 8 + (lane & 7), dims p*16 + (lane >> 4) * 8
  const int krow = lane & 7, kcol = (lane >> 3) * 8;
  const int vrow = ((lane >> 3) & 1) * 8 + (lane & 7), vcol = (lane >> 4) * 8;

  for (int t = 0; t < ntiles; ++t) {
    const int buf = t & 1, t0 = t * kKT;
    if (t + 1 < ntiles) {
      load_tile(t0 + kKT, buf ^ 1);  // that buffer was released by the barrier ending tile t - 1
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // tile t is in shared memory for every thread
    // S = Q K^T for 8 groups of 8 keys
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      uint32_t kf[4];
      ldsm_x4(saddr(&sK[buf][nt * 8 + krow][kcol]), kf);
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
      mma16816(s[nt], qa[0], kf[0], kf[1]);
      mma16816(s[nt], qa[1], kf[2], kf[3]);
    }
    if (t0 + kKT > Tk) {  // the last tile: keys past Tk do not take part
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int key = t0 + nt * 8 + 2 * tig;
#pragma unroll
        for (int e = 0; e < 2; ++e)
          if (key + e >= Tk) s[nt][e] = s[nt][2 + e] = -INFINITY;
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      mx0 = fmaxf(mx0, fmaxf(s[nt][0], s[nt][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nt][2], s[nt][3]));
    }
#pragma unroll
    for (int x = 1; x <= 2; x <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xFFFFFFFFu, mx0, x));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xFFFFFFFFu, mx1, x));
    }
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);  // finite: a tile holds a key < Tk
    const float ms0 = mn0 * scale_log2, ms1 = mn1 * scale_log2;
    const float c0 = exp2f(m0 * scale_log2 - ms0), c1 = exp2f(m1 * scale_log2 - ms1);  // 0 on the first tile
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
      const float p0 = exp2f(fmaf(s[nt][0], scale_log2, -ms0)), p1 = exp2f(fmaf(s[nt][1], scale_log2, -ms0));
      const float p2 = exp2f(fmaf(s[nt][2], scale_log2, -ms1)), p3 = exp2f(fmaf(s[nt][3], scale_log2, -ms1));
      l0 += p0 + p1;
      l1 += p2 + p3;
      pa[nt][0] = pack_half2(p0, p1);
      pa[nt][1] = pack_half2(p2, p3);
    }
    m0 = mn0;
    m1 = mn1;
    // O += P V over 4 k-steps of 16 keys, two 8-dim column groups per ldmatrix.trans
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const uint32_t a[4] = {pa[2 * ks][0], pa[2 * ks][1], pa[2 * ks + 1][0], pa[2 * ks + 1][1]};
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        uint32_t vf[4];
        ldsm_x4_t(saddr(&sV[buf][ks * 16 + vrow][p * 16 + vcol]), vf);
        mma16816(o[2 * p], a, vf[0], vf[1]);
        mma16816(o[2 * p + 1], a, vf[2], vf[3]);
      }
    }
    __syncthreads();  // every warp is done with this buffer before it is refilled
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
