// sb_gemm.cu -- dense implicit-GEMM on tcgen05 for the detector after the stem.
//
// Reference: Bahrombekk/Sarbon sarbon/models/sarbon_det.py (DenseCore :118-155, the encoder
// heads :309-319, DecoderLayer :158-171, the box heads :336-356) and deform_attn.py:30-66.
// Under the reference's autocast every nn.Linear and nn.Conv2d of the detector is an fp16
// matrix product with fp32 accumulation; here each one (with its folded BatchNorm, bias,
// activation and residual) is one launch of this kernel:
//
//   out[p][n] = act( sum_k A[p][k] * W[n][k] + bias[n] + res[p][n] ),
//
// where row p is an output pixel (b, yo, xo) of an NHWC map (a token of a [rows][C] matrix
// is a pixel of a 1 x rows map) and k runs over (tap, source, channel): 1x1 or 3x3 taps
// (zero padding 1, stride 1 or 2) over the channels of one or two NHWC sources (the second
// source continues the channel axis: a 1x1 conv over torch.cat([a, b], 1)).
//
// One CTA per SM, persistent over the output tiles (128 pixels x BN channels, BN <= 256 a
// multiple of 16):
//   warp 0     TMA producer: per K-block one strided 4-D box of the source (64 channels x
//              the tile's Wt columns x R rows, element stride = conv stride, start shifted
//              by the tap; out-of-map pixels arrive as zeros = the conv's zero padding) and
//              one 64 x BN box of the weights, both 128-byte swizzled, into a 4-stage ring;
//   warp 1     tcgen05.mma issuer (M = 128, N = BN, K = 16 per instruction) into one of two
//              TMEM accumulators (2 x 256 columns), so the epilogue of tile i overlaps the
//              MMAs of tile i + 1;
//   warps 2-17 epilogue: TMEM lane quadrant (warp % 4) = 32 tile rows, four warps per
//              quadrant on every fourth 16-column chunk (one tcgen05.ld each), bias /
//              residual / activation in fp32, fp16 or fp32 stores.
// A tile holds R rows of Wt output pixels (R * Wt <= 128) chosen on the host so that few
// of the 128 MMA rows idle; rows past R * Wt hold stale shared memory and are never stored.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "sb_internal.cuh"
#include "sb_ptx.cuh"

namespace sb {
namespace {

constexpr int kStages = 4;
constexpr int kMaxBN = 256;
constexpr int kAStage = 128 * 128;            // 128 rows x 64 fp16
constexpr int kBStage = kMaxBN * 128;         // BN rows x 64 fp16
constexpr int kStageBytes = kAStage + kBStage;
constexpr int kEpiWarps = 16;   // four per TMEM lane quadrant
constexpr int kThreads = 64 + 32 * kEpiWarps;  // producer, MMA issuer, epilogue warps
constexpr int kBarBytes = 256;
constexpr int kSmem = 1024 + kStages * kStageBytes + kBarBytes;
constexpr uint32_t kTmemCols = 512;           // two accumulators of up to 256 columns
// Weights-resident mode (KB * BN * 128 bytes <= kBResBytes, several tiles per CTA): the grid is
// a multiple of n_tiles so every CTA keeps one N tile; its whole B tile (all K-blocks) is
// loaded once into the upper part of the stage area and only A boxes stream through a
// ring of kStages 16 KB stages below it.
constexpr int kBResOff = kStages * kAStage;                   // 64 KB
constexpr int kBResBytes = kStages * kStageBytes - kBResOff;  // 128 KB

// sticky error word of the detector kernels (SB_ERR_* bits), read by sb_kernels_error
__device__ int g_kernel_error;

struct GemmArgs {
  int kch0, kch1;             // 64-channel chunks of source 0 and source 1 (0: one source)
  int taps, stride, pad;      // 1 tap (pad 0) or 3x3 taps (pad 1); stride 1 or 2
  int Ho, Wo, R, Wt, tiles_y, tiles_x;
  int N, BN, n_tiles, KB;     // KB = K-blocks per tile = taps * (kch0 + kch1)
  uint32_t idesc;
  uint32_t a_bytes;           // bytes one A box writes: R * Wt rows of 128 B
  long long total_tiles;
  const float* bias;          // [N] or null
  int bias_vec;               // bias 16-byte aligned (vector loads)
  const void* res;            // residual rows (fp16 or fp32) or null
  int res_f32, res_vec;       // res_vec: rows 16-byte aligned (vector loads)
  long long res_ld, res_img;  // elements between pixels; pixels between images
  void* out;
  int out_f32, out_vec;       // out_vec: rows 16-byte aligned (vector stores)
  int out_v8;                 // rows 32-byte aligned: a lane stores whole 32-byte sectors
  long long out_ld, out_img;
  int act;                    // 0 none, 1 ReLU, 2 GELU (erf form)
  int bres;                   // weights resident: the CTA's whole B tile loaded once (see below)
};

SB_DEV float act_of(float v, int act) {
  if (act == 1) return fmaxf(v, 0.f);
  if (act == 2) return 0.5f * v * (1.f + erff(v * 0.70710678118654752f));
  return v;
}

struct TileCoord {
  int b, ty, tx, nt;
};

SB_DEV TileCoord tile_coord(const GemmArgs& a, long long t) {
  TileCoord c;
  c.nt = (int)(t % a.n_tiles);
  const long long mt = t / a.n_tiles;
  c.tx = (int)(mt % a.tiles_x);
  const long long r = mt / a.tiles_x;
  c.ty = (int)(r % a.tiles_y);
  c.b = (int)(r / a.tiles_y);
  return c;
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ GemmArgs a, const __grid_constant__ CUtensorMap map0,
                   const __grid_constant__ CUtensorMap map1, const __grid_constant__ CUtensorMap mapw) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* accf = empty + kStages;  // [2] accumulator ready
  uint64_t* acce = accf + 2;         // [2] accumulator drained by the epilogue
  uint64_t* dbar = acce + 2;         // drain of the MMA issuer
  uint64_t* wfull = dbar + 1;        // weights-resident mode: the B tile has landed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(wfull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], kEpiWarps);  // one arrival per epilogue warp
    }
    mbar_init(dbar, 1);
    mbar_init(wfull, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&map0);
    if (a.kch1 > 0) prefetch_tmap(&map1);
    prefetch_tmap(&mapw);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int my_tiles =
      (long long)blockIdx.x < a.total_tiles ? (int)((a.total_tiles - 1 - blockIdx.x) / gridDim.x) + 1 : 0;
  const int kch = a.kch0 + a.kch1;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    grid_dep_wait();  // inputs written by the previous kernel of the stream are complete
    uint32_t g = 0;
    bool ok = true;
    const int stage_bytes = a.bres ? kAStage : kStageBytes;
    if (a.bres && my_tiles > 0) {
      if (lane == 0) {  // this CTA's N tile, every K-block, once
        const int nt = (int)(blockIdx.x % a.n_tiles);
        mbar_arrive_expect_tx(wfull, (uint32_t)(a.KB * a.BN * 128));
        for (int kb = 0; kb < a.KB; ++kb)
          tma_load_2d(smem + kBResOff + kb * a.BN * 128, &mapw, wfull, kb * 64, nt * a.BN);
      }
      __syncwarp();
    }
    for (int i = 0; ok && i < my_tiles; ++i) {
      const TileCoord c = tile_coord(a, (long long)blockIdx.x + (long long)i * gridDim.x);
      const int xs = c.tx * a.Wt * a.stride - a.pad, ys = c.ty * a.R * a.stride - a.pad;
      for (int kb = 0; kb < a.KB; ++kb, ++g) {
        const uint32_t s = g % kStages, ph = (g / kStages) & 1u;
        if (!warp_wait(&empty[s], ph ^ 1u, abort_flag)) {
          if (lane == 0) atomicOr(&g_kernel_error, SB_ERR_TIMEOUT_EMPTY);
          *abort_flag = 1;
          ok = false;
          break;
        }
        if (lane == 0) {
          const int tap = kb / kch, cc = kb - tap * kch;
          const int ky = a.taps == 9 ? tap / 3 : 0, kx = a.taps == 9 ? tap % 3 : 0;
          uint8_t* sa = smem + s * stage_bytes;
          mbar_arrive_expect_tx(&full[s], a.a_bytes + (a.bres ? 0u : (uint32_t)a.BN * 128u));
          if (cc < a.kch0) tma_load_4d(sa, &map0, &full[s], cc * 64, xs + kx, ys + ky, c.b);
          else tma_load_4d(sa, &map1, &full[s], (cc - a.kch0) * 64, xs + kx, ys + ky, c.b);
          if (!a.bres) tma_load_2d(sa + kAStage, &mapw, &full[s], kb * 64, c.nt * a.BN);
        }
        __syncwarp();
      }
    }
    // drain: every issued copy has landed before the CTA may exit
    volatile int never = 0;
    const uint32_t first = g > (uint32_t)kStages ? g - kStages : 0u;
    for (uint32_t q = first; q < g; ++q) warp_wait(&full[q % kStages], (q / kStages) & 1u, &never);
    if (a.bres && my_tiles > 0) warp_wait(wfull, 0, &never);
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint64_t a_desc0 = smem_desc(smem_u32(smem), 1024, 2);
      const uint64_t b_desc0 = smem_desc(smem_u32(smem + (a.bres ? kBResOff : kAStage)), 1024, 2);
      const uint32_t SSTEP = (uint32_t)(a.bres ? kAStage : kStageBytes) >> 4;
      const uint32_t BSTEP = a.bres ? (uint32_t)(a.BN * 128) >> 4 : 0u;  // resident B: per K-block
      uint32_t g = 0;
      bool ok = my_tiles == 0 || !a.bres || mbar_wait(wfull, 0, abort_flag);
      if (!ok) {
        atomicOr(&g_kernel_error, SB_ERR_TIMEOUT_WGT);
        *abort_flag = 1;
      }
      for (int i = 0; ok && i < my_tiles; ++i) {
        const int ab = i & 1;
        if (!mbar_wait(&acce[ab], ((i >> 1) & 1) ^ 1, abort_flag)) {
          atomicOr(&g_kernel_error, SB_ERR_TIMEOUT_ACC);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)ab * kMaxBN;
        for (int kb = 0; kb < a.KB; ++kb, ++g) {
          const uint32_t s = g % kStages, ph = (g / kStages) & 1u;
          if (!mbar_wait(&full[s], ph, abort_flag)) {
            atomicOr(&g_kernel_error, SB_ERR_TIMEOUT_FULL);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = a_desc0 + s * SSTEP, bd = a.bres ? b_desc0 + kb * BSTEP : b_desc0 + s * SSTEP;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)  // K = 16 per MMA: 32 bytes along the swizzled row
            mma_f16_ss(d_tmem, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), a.idesc, (kb | kk) != 0 ? 1u : 0u);
          mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
        }
        if (!ok) break;
        mma_commit(&accf[ab]);  // accumulator complete
      }
      // drain: all MMAs this thread issued complete before TMEM is released
      mma_commit(dbar);
      volatile int never = 0;
      mbar_wait(dbar, 0, &never);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..)
    grid_dep_wait();  // residual rows written by the previous kernel of the stream
    // warp w reads TMEM lane quadrant w % 4 (tile rows 32q..32q+31); the four warps of a
    // quadrant take every fourth 16-column chunk
    const int q = warp & 3, part = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const int r = row / a.Wt, j = row - r * a.Wt;
    for (int i = 0; i < my_tiles; ++i) {
      const TileCoord c = tile_coord(a, (long long)blockIdx.x + (long long)i * gridDim.x);
      const int ab = i & 1;
      if (!warp_wait(&accf[ab], (i >> 1) & 1, abort_flag)) {
        if (lane == 0) atomicOr(&g_kernel_error, SB_ERR_TIMEOUT_ACC);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int yo = c.ty * a.R + r, xo = c.tx * a.Wt + j;
      const bool valid = r < a.R && yo < a.Ho && xo < a.Wo;
      const long long pix = (long long)c.b * a.out_img + (long long)yo * a.Wo + xo;
      const long long rpix = (long long)c.b * a.res_img + (long long)yo * a.Wo + xo;
      const int nbase = c.nt * a.BN;
      const int nch = a.BN / 16;
      for (int cc = part; cc < nch; cc += kEpiWarps / 4) {
        uint32_t v[16];
        tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * kMaxBN + cc * 16), v);
        tmem_ld_wait();
        const int n0 = nbase + cc * 16;
        if (!valid || n0 >= a.N) continue;
        const int nv = a.N - n0 < 16 ? a.N - n0 : 16;
        float f[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) f[t] = __uint_as_float(v[t]);
        if (a.bias) {
          if (nv == 16 && a.bias_vec) {
#pragma unroll
            for (int t = 0; t < 16; t += 4) {
              const float4 bb = __ldg(reinterpret_cast<const float4*>(a.bias + n0 + t));
              f[t] += bb.x;
              f[t + 1] += bb.y;
              f[t + 2] += bb.z;
              f[t + 3] += bb.w;
            }
          } else {
#pragma unroll
            for (int t = 0; t < 16; ++t)
              if (t < nv) f[t] += __ldg(a.bias + n0 + t);
          }
        }
        if (a.res) {
          if (a.res_f32) {
            const float* rp = static_cast<const float*>(a.res) + rpix * a.res_ld + n0;
            if (nv == 16 && a.res_vec) {
#pragma unroll
              for (int t = 0; t < 16; t += 4) {
                const float4 x = *reinterpret_cast<const float4*>(rp + t);
                f[t] += x.x;
                f[t + 1] += x.y;
                f[t + 2] += x.z;
                f[t + 3] += x.w;
              }
            } else {
#pragma unroll
              for (int t = 0; t < 16; ++t)
                if (t < nv) f[t] += rp[t];
            }
          } else {
            const __half* rp = static_cast<const __half*>(a.res) + rpix * a.res_ld + n0;
            if (nv == 16 && a.res_vec) {
#pragma unroll
              for (int t = 0; t < 16; t += 8) {
                const uint4 x = *reinterpret_cast<const uint4*>(rp + t);
                const __half2* h = reinterpret_cast<const __half2*>(&x);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  const float2 p = __half22float2(h[u]);
                  f[t + 2 * u] += p.x;
                  f[t + 2 * u + 1] += p.y;
                }
              }
            } else {
#pragma unroll
              for (int t = 0; t < 16; ++t)
                if (t < nv) f[t] += __half2float(rp[t]);
            }
          }
        }
#pragma unroll
        for (int t = 0; t < 16; ++t) f[t] = act_of(f[t], a.act);
        if (a.out_f32) {
          float* op = static_cast<float*>(a.out) + pix * a.out_ld + n0;
          if (nv == 16 && a.out_v8) {
#pragma unroll
            for (int t = 0; t < 16; t += 8)
              st_global_v8(op + t,
                           make_uint4(__float_as_uint(f[t]), __float_as_uint(f[t + 1]), __float_as_uint(f[t + 2]),
                                      __float_as_uint(f[t + 3])),
                           make_uint4(__float_as_uint(f[t + 4]), __float_as_uint(f[t + 5]), __float_as_uint(f[t + 6]),
                                      __float_as_uint(f[t + 7])));
          } else if (nv == 16 && a.out_vec) {
#pragma unroll
            for (int t = 0; t < 16; t += 4) *reinterpret_cast<float4*>(op + t) = make_float4(f[t], f[t + 1], f[t + 2], f[t + 3]);
          } else {
#pragma unroll
            for (int t = 0; t < 16; ++t)
              if (t < nv) op[t] = f[t];
          }
        } else {
          __half* op = static_cast<__half*>(a.out) + pix * a.out_ld + n0;
          if (nv == 16 && a.out_v8) {  // the chunk's 16 channels: one 32-byte sector
            uint4 x[2];
            __half2* h = reinterpret_cast<__half2*>(x);
#pragma unroll
            for (int u = 0; u < 8; ++u) h[u] = __floats2half2_rn(f[2 * u], f[2 * u + 1]);
            st_global_v8(op, x[0], x[1]);
          } else if (nv == 16 && a.out_vec) {
#pragma unroll
            for (int t = 0; t < 16; t += 8) {
              uint4 x;
              __half2* h = reinterpret_cast<__half2*>(&x);
#pragma unroll
              for (int u = 0; u < 4; ++u) h[u] = __floats2half2_rn(f[t + 2 * u], f[t + 2 * u + 1]);
              *reinterpret_cast<uint4*>(op + t) = x;
            }
          } else {
#pragma unroll
            for (int t = 0; t < 16; ++t)
              if (t < nv) op[t] = __float2half_rn(f[t]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[ab]);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  });
  return fn;
}

// R rows x Wt columns per tile (R * Wt <= 128) with the fewest idle MMA rows over the map.
void pick_tile(int Ho, int Wo, int& R, int& Wt) {
  R = 1;
  Wt = std::min(Wo, 128);
  if (Ho == 1) return;  // a row of tokens: 128 per tile
  double best = -1.0;
  for (int w = std::min(Wo, 128); w >= 1; --w) {
    if (w < 8 && best > 0.0) break;
    const long long k = (Wo + w - 1) / w;          // column segments
    const int wt = (int)((Wo + k - 1) / k);        // their width when balanced
    const int r = std::min(128 / wt, Ho);
    const long long tiles = (long long)((Ho + r - 1) / r) * k;
    const double eff = (double)Ho * Wo / ((double)tiles * 128.0);
    if (eff > best + 1e-9) {
      best = eff;
      R = r;
      Wt = wt;
    }
  }
}

struct DeviceInfo {
  int sms = 0;
  bool attr = false;
};

}  // namespace
}  // namespace sb

using namespace sb;

extern "C" int sb_gemm_conv(const sb_gemm_src* src, int nsrc, int B, int H, int W, int taps, int stride,
                            const void* weight, int N, const float* bias, int act, const void* res, int res_dtype,
                            long long res_ld, long long res_img, void* out, int out_dtype, long long out_ld,
                            long long out_img, void* stream) {
  if (!src || !weight || !out) return record_error(SB_EINVAL, "sb_gemm_conv: null argument");
  if (nsrc < 1 || nsrc > 2) return record_error(SB_EINVAL, "sb_gemm_conv: one or two sources");
  if (B < 1 || H < 1 || W < 1 || N < 1) return record_error(SB_EINVAL, "sb_gemm_conv: sizes");
  if (!((taps == 1 && stride == 1) || (taps == 9 && (stride == 1 || stride == 2))))
    return record_error(SB_EINVAL, "sb_gemm_conv: 1x1 (stride 1) or 3x3 (stride 1 or 2)");
  if (act < 0 || act > 2) return record_error(SB_EINVAL, "sb_gemm_conv: act");
  if ((res && res_dtype != SB_F16 && res_dtype != SB_F32) || (out_dtype != SB_F16 && out_dtype != SB_F32))
    return record_error(SB_EINVAL, "sb_gemm_conv: dtype");
  int kch[2] = {0, 0};
  for (int i = 0; i < nsrc; ++i) {
    const sb_gemm_src& s = src[i];
    if (!s.ptr || s.C < 64 || s.C % 64 != 0 || s.ld < s.C || s.ld % 8 != 0 || s.img_stride < (long long)H * W ||
        (reinterpret_cast<uintptr_t>(s.ptr) & 15) != 0)
      return record_error(SB_EINVAL, "sb_gemm_conv: source (C a multiple of 64, ld a multiple of 8 >= C, "
                                     "16-byte aligned, img_stride >= H*W)");
    kch[i] = s.C / 64;
  }
  const long long esz_o = out_dtype == SB_F32 ? 4 : 2, esz_r = res_dtype == SB_F32 ? 4 : 2;
  if (out_ld < N || (res && res_ld < N) || (reinterpret_cast<uintptr_t>(out) % esz_o) != 0 ||
      (res && (reinterpret_cast<uintptr_t>(res) % esz_r) != 0))
    return record_error(SB_EINVAL, "sb_gemm_conv: out/res rows (ld >= N, element-aligned)");
  GemmArgs a{};
  a.kch0 = kch[0];
  a.kch1 = kch[1];
  a.taps = taps;
  a.stride = stride;
  a.pad = taps == 9 ? 1 : 0;
  a.Ho = taps == 9 ? (H + 2 - 3) / stride + 1 : H;
  a.Wo = taps == 9 ? (W + 2 - 3) / stride + 1 : W;
  if (out_img < (long long)a.Ho * a.Wo || (res && res_img < (long long)a.Ho * a.Wo))
    return record_error(SB_EINVAL, "sb_gemm_conv: out/res image stride < Ho*Wo");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return record_error(SB_ECUDA, "sb_gemm_conv: cudaGetDevice");
  static DeviceInfo info[64];
  static std::mutex mu;
  int sms;
  {
    std::lock_guard<std::mutex> lk(mu);
    DeviceInfo& d = info[dev & 63];
    if (!d.attr) {
      if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
          cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
        return record_error(SB_ECUDA, "sb_gemm_conv: device setup");
      d.attr = true;
    }
    sms = d.sms;
  }
  pick_tile(a.Ho, a.Wo, a.R, a.Wt);
  a.tiles_y = (a.Ho + a.R - 1) / a.R;
  a.tiles_x = (a.Wo + a.Wt - 1) / a.Wt;
  a.N = N;
  // N per tile: up to 256; when the M tiles alone cannot occupy the SMs, narrower N tiles (down
  // to 64 columns) spread the work over more CTAs, each with a shorter epilogue
  const long long m_tiles = (long long)B * a.tiles_y * a.tiles_x;
  a.n_tiles = (N + kMaxBN - 1) / kMaxBN;
  while (m_tiles * a.n_tiles < sms && (N + 2 * a.n_tiles - 1) / (2 * a.n_tiles) >= 64) a.n_tiles *= 2;
  a.BN = ((N + a.n_tiles - 1) / a.n_tiles + 15) / 16 * 16;
  a.n_tiles = (N + a.BN - 1) / a.BN;
  a.KB = taps * (kch[0] + kch[1]);
  a.idesc = idesc_f16(128, a.BN);
  a.a_bytes = (uint32_t)(a.R * a.Wt * 128);
  a.total_tiles = (long long)B * a.tiles_y * a.tiles_x * a.n_tiles;
  a.bias = bias;
  a.bias_vec = bias && (reinterpret_cast<uintptr_t>(bias) & 15) == 0;
  a.res = res;
  a.res_f32 = res_dtype == SB_F32;
  a.res_vec = res && (res_ld * esz_r) % 16 == 0 && (reinterpret_cast<uintptr_t>(res) & 15) == 0;
  a.out_vec = (out_ld * esz_o) % 16 == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  a.out_v8 = (out_ld * esz_o) % 32 == 0 && (reinterpret_cast<uintptr_t>(out) & 31) == 0;
  a.res_ld = res_ld;
  a.res_img = res_img;
  a.out = out;
  a.out_f32 = out_dtype == SB_F32;
  a.out_ld = out_ld;
  a.out_img = out_img;
  a.act = act;

  PFN_encodeTiled enc = encode_fn();
  if (!enc) return record_error(SB_ECUDA, "sb_gemm_conv: cuTensorMapEncodeTiled unavailable");
  CUtensorMap maps[2], mapw;
  std::memset(maps, 0, sizeof maps);
  for (int i = 0; i < nsrc; ++i) {
    const sb_gemm_src& s = src[i];
    cuuint64_t dims[4] = {(cuuint64_t)s.C, (cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)s.ld * 2, (cuuint64_t)W * s.ld * 2, (cuuint64_t)s.img_stride * s.ld * 2};
    cuuint32_t box[4] = {64u, (cuuint32_t)(a.Wt * stride), (cuuint32_t)(a.R * stride), 1u};
    cuuint32_t estr[4] = {1u, (cuuint32_t)stride, (cuuint32_t)stride, 1u};
    if (enc(&maps[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(s.ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return record_error(SB_EINVAL, "sb_gemm_conv: source tensor map");
  }
  if (nsrc == 1) maps[1] = maps[0];
  {
    const long long K = (long long)a.KB * 64;
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {64u, (cuuint32_t)a.BN};
    cuuint32_t estr[2] = {1u, 1u};
    // rows >= N of the last tile arrive as zeros
    if ((reinterpret_cast<uintptr_t>(weight) & 15) != 0 ||
        enc(&mapw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(weight), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return record_error(SB_EINVAL, "sb_gemm_conv: weight tensor map");
  }

  long long grid = std::min<long long>(a.total_tiles, sms);
  a.bres = 0;
  if ((long long)a.KB * a.BN * 128 <= kBResBytes && grid >= a.n_tiles) {
    const long long g2 = grid / a.n_tiles * a.n_tiles;  // every CTA keeps one N tile
    if (a.total_tiles >= 2 * g2) {                      // worth it with several tiles per CTA
      grid = g2;
      a.bres = 1;
    }
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_tc_kernel, a, maps[0], maps[1], mapw);
  if (e != cudaSuccess) return record_error(SB_ECUDA, cudaGetErrorString(e));
  return SB_OK;
}

extern "C" int sb_kernels_error(int clear, int* flags) {
  if (!flags) return record_error(SB_EINVAL, "sb_kernels_error: null argument");
  if (cudaMemcpyFromSymbol(flags, g_kernel_error, sizeof(int)) != cudaSuccess)
    return record_error(SB_ECUDA, "sb_kernels_error: read");
  if (clear) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_kernel_error, &zero, sizeof(int)) != cudaSuccess)
      return record_error(SB_ECUDA, "sb_kernels_error: clear");
  }
  return SB_OK;
}
