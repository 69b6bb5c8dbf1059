// sb_gate.cu -- per-frame gating, dilation + ordered block lists, image-cache updates and
// the device-side dispatch state machine of the temporal block-sparse engine.
//
// Reference (Bahrombekk/Sarbon, sarbon/sparse/fused_engine.py):
//   gate            _gate        :140-153
//   img update      _sparse      :155-160 (fused into the gate here)
//   block lists     _sparse      :161-165 (nonzero_static: ascending flat order)
//   dispatch        step         :214-240 (skip / sparse / dense + hysteresis)
#include <algorithm>
#include <cstdint>

#include "sb_internal.cuh"
#include "sb_ptx.cuh"

namespace sb {

// A step taken while 0 < dense_run < dense_check_every is dense without a gate look
// (fused_engine.py:222-226).  Only finalize_kernel / set_mode_kernel change dense_run,
// and they run after / outside the gate and list kernels of a step.
SB_DEV bool in_hysteresis(const State* st) {
  return st->dense_run > 0 && st->dense_run < st->check_every;
}

// ---------------------------------------------------------------- exact |fp16 diff| sums
// |d| for fp16 d, as an integer multiple of 2^-24 (exact: every finite fp16 is one).
SB_DEV uint64_t abs_h_fixed(uint16_t h) {
  const uint32_t e = (h >> 10) & 0x1F, m = h & 0x3FF;
  return e ? (uint64_t)(m | 0x400) << (e - 1) : (uint64_t)m;
}

// fp16(fp32(a) - fp32(b)) with IEEE round-to-nearest at both steps, as torch computes a
// half-precision subtraction (fused_engine.py:142).
SB_DEV uint16_t sub_h(uint16_t a, uint16_t b) {
  const float fa = __half2float(__ushort_as_half(a)), fb = __half2float(__ushort_as_half(b));
  return __half_as_ushort(__float2half_rn(__fsub_rn(fa, fb)));
}

// Flags for inf / NaN diffs: an fp32 sum with an inf term is inf (> any finite
// threshold); with a NaN term the comparison is false.
#define GATE_INF 1u
#define GATE_NAN 2u

SB_DEV void accum_h(uint16_t d, uint64_t& acc, uint32_t& flags) {
  const uint16_t a = d & 0x7FFF;
  if ((a >> 10) == 0x1F) {
    flags |= (a & 0x3FF) ? GATE_NAN : GATE_INF;
  } else {
    acc += abs_h_fixed(a);
  }
}

SB_DEV uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
SB_DEV __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Sum of |a - b| over the two fp16 lanes of a 32-bit word, widened to fp32.  __hsub2
// rounds the exact difference to fp16 once; for fp16 operands that equals torch's
// fp16(fp32(a) - fp32(b)) (the fp32 step is exact unless the exponent gap exceeds 13
// bits, and then both round back to the larger operand).
SB_DEV float absdiff2(uint32_t x, uint32_t y) {
  const uint32_t d = h2_bits(__hsub2(bits_h2(x), bits_h2(y))) & 0x7FFF7FFFu;
  const float2 f = __half22float2(bits_h2(d));
  return f.x + f.y;
}

// Per-block change statistic.  One CTA per (segment of a block row, camera): reads the
// segment of the new frames and of the image cache with 16-byte coalesced loads (about one
// 16-byte column per thread, all rows of the block) and sums |diff| per block in fp32.  The fp32 sum of n non-negative terms is within (n-1)*2^-24 relative of
// the exact sum, so it decides `sum > thr` exactly unless it falls inside that band
// around the threshold; only those (rare) blocks are re-summed exactly, in integer
// multiples of 2^-24.  The result equals an exact comparison (the reference sums in fp32
// in torch's order, fused_engine.py:142-144).  Then `| extra`, the refresh phase, and the
// changed blocks of the new frames are copied into the image cache.
template <int KIND>  // 0: fp16 frames, 1: fp32 frames, 2: uint8 BGR frames (fused prep)
__global__ void __launch_bounds__(256, 4) gate_kernel(GateArgs a) {
  grid_dep_wait();  // programmatic dependent launch: the previous kernel's writes are visible
  if (in_hysteresis(a.st)) return;  // hysteresis dense step: the gate is not looked at (:222-226)
  // CTA = blocks [bx0, bx0 + nblk) of block row `by` of camera `cam` (a segment of the row)
  const int by = blockIdx.x, cam = blockIdx.y, bx0 = blockIdx.z * a.seg;
  const int nblk = min(a.seg, a.wb - bx0);
  const int B = a.block;
  extern __shared__ __align__(16) uint8_t gsm[];
  unsigned long long* s_sx = reinterpret_cast<unsigned long long*>(gsm);  // [wb] exact sums (or double)
  float* s_sf = reinterpret_cast<float*>(s_sx + a.seg);                   // [seg] fp32 sums
  uint32_t* s_flag = reinterpret_cast<uint32_t*>(s_sf + a.seg);          // [seg]
  int* s_amb = reinterpret_cast<int*>(s_flag + a.seg);                   // [seg] ambiguous blocks
  __half* s_lut = reinterpret_cast<__half*>(s_amb + a.seg);              // [3][256] (u8 path)
  __shared__ int s_namb;
  for (int i = threadIdx.x; i < nblk; i += blockDim.x) {
    s_sx[i] = 0ull;
    s_sf[i] = 0.f;
    s_flag[i] = 0u;
  }
  if (threadIdx.x == 0) s_namb = 0;
  if (KIND == 2) {
    // normalised value of every uint8 level per RGB channel, with the reference's ops:
    // (x - mean[c]) / std[c] in fp32, then rounded to fp16 (video.py:99, :108)
    for (int i = threadIdx.x; i < 768; i += blockDim.x) {
      const int c = i >> 8, u = i & 255;
      s_lut[i] = __float2half_rn(__fdiv_rn(__fsub_rn((float)u, a.mean[c]), a.stdv[c]));
    }
  }
  __syncthreads();

  const size_t row_px = (size_t)a.w;
  // element index of the segment's first pixel; rows stay row_px * 3 elements apart
  const size_t img_row0 = (((size_t)cam * a.h + (size_t)by * B) * row_px + (size_t)bx0 * B) * 3;
  if (KIND == 0) {
    // 16 B = 8 halves; a block row-segment is B*3*2/16 vectors
    const int vpb = B * 3 / 8, vpr = vpb * a.wb;  // vectors per block, per image row
    const uint4* f = reinterpret_cast<const uint4*>(static_cast<const __half*>(a.frames) + img_row0);
    const uint4* g = reinterpret_cast<const uint4*>(static_cast<const __half*>(a.img) + img_row0);
    for (int v = threadIdx.x; v < vpb * nblk; v += blockDim.x) {
      float acc = 0.f;
      // eight rows of both images in flight per thread (the image cache is written only by
      // the copy below, after every read of this kernel, so it is read through the
      // non-coherent path too)
      for (int r0 = 0; r0 < B; r0 += 8) {
        uint4 xs[8], ys[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          xs[k] = __ldg(f + (size_t)(r0 + k) * vpr + v);
          ys[k] = __ldg(g + (size_t)(r0 + k) * vpr + v);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k)
          acc += (absdiff2(xs[k].x, ys[k].x) + absdiff2(xs[k].y, ys[k].y)) +
                 (absdiff2(xs[k].z, ys[k].z) + absdiff2(xs[k].w, ys[k].w));
      }
      atomicAdd(&s_sf[v / vpb], acc);
    }
  } else if (KIND == 1) {
    // fp32 frames: |f32 diff| summed in double (exact for frames within 2^29 of dynamic range)
    const int vpb = B * 3 / 4, vpr = vpb * a.wb;
    const float4* f = reinterpret_cast<const float4*>(static_cast<const float*>(a.frames) + img_row0);
    const float4* g = reinterpret_cast<const float4*>(static_cast<const float*>(a.img) + img_row0);
    double* s_d = reinterpret_cast<double*>(s_sx);
    for (int v = threadIdx.x; v < vpb * nblk; v += blockDim.x) {
      double acc = 0.0;
#pragma unroll 4
      for (int r = 0; r < B; ++r) {
        const float4 x = __ldg(f + (size_t)r * vpr + v);
        const float4 y = g[(size_t)r * vpr + v];
        acc += (double)fabsf(__fsub_rn(x.x, y.x)) + (double)fabsf(__fsub_rn(x.y, y.y)) +
               (double)fabsf(__fsub_rn(x.z, y.z)) + (double)fabsf(__fsub_rn(x.w, y.w));
      }
      atomicAdd(&s_d[v / vpb], acc);
    }
  } else {
    // uint8 BGR: units of 16 pixels = 48 bytes of frame, 96 bytes of fp16 cache
    const int upb = B / 16;
    const uint8_t* f = static_cast<const uint8_t*>(a.frames) + img_row0;
    const __half* g = static_cast<const __half*>(a.img) + img_row0;
    for (int u = threadIdx.x; u < upb * nblk; u += blockDim.x) {
      float acc = 0.f;
#pragma unroll 2
      for (int r = 0; r < B; ++r) {
        const uint4* fp = reinterpret_cast<const uint4*>(f + (size_t)r * row_px * 3 + (size_t)u * 48);
        const uint4* gp = reinterpret_cast<const uint4*>(g + (size_t)r * row_px * 3 + (size_t)u * 48);
        uint4 fx[3], gx[6];
#pragma unroll
        for (int k = 0; k < 3; ++k) fx[k] = __ldg(fp + k);
#pragma unroll
        for (int k = 0; k < 6; ++k) gx[k] = gp[k];
        const uint32_t* fw = reinterpret_cast<const uint32_t*>(fx);
        const uint32_t* gw = reinterpret_cast<const uint32_t*>(gx);
#pragma unroll
        for (int j = 0; j < 24; ++j) {  // cache elements 2j, 2j+1 = (pixel, RGB channel)
          uint32_t hv = 0;
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int el = 2 * j + e, px = el / 3, c = el % 3, byte = px * 3 + (2 - c);  // BGR -> RGB
            const uint32_t q = (fw[byte >> 2] >> ((byte & 3) * 8)) & 0xFFu;
            hv |= (uint32_t)__half_as_ushort(s_lut[c * 256 + q]) << (16 * e);
          }
          acc += absdiff2(hv, gw[j]);
        }
      }
      atomicAdd(&s_sf[u / upb], acc);
    }
  }
  __syncthreads();

  // classify with the fp32 sums; collect the blocks inside the rounding band
  for (int bx = threadIdx.x; bx < nblk; bx += blockDim.x) {
    uint32_t cls;  // 0 unchanged, 1 changed, 2 ambiguous
    if (KIND == 1) {
      cls = reinterpret_cast<double*>(s_sx)[bx] > a.thr ? 1u : 0u;
    } else {
      const float sf = s_sf[bx];
      if (isnan(sf)) cls = 0u;                         // NaN > thr is false
      else if (sf == 0.f) cls = a.thr_fx < 0 ? 1u : 0u;  // every term was 0: the sum is exactly 0
      else if ((double)sf > a.band_hi) cls = 1u;
      else if ((double)sf < a.band_lo) cls = 0u;
      else cls = 2u;
    }
    s_flag[bx] = cls;
    if (cls == 2u) s_amb[atomicAdd(&s_namb, 1)] = bx;
  }
  __syncthreads();

  // exact re-sum of the ambiguous blocks (integer multiples of 2^-24, order-free)
  if (KIND != 1) {
    const int namb = s_namb;
    for (int ai = 0; ai < namb; ++ai) {
      const int bx = s_amb[ai];
      uint64_t acc = 0;
      uint32_t flags = 0;
      if (KIND == 0) {
        const int vpb = B * 3 / 8, vpr = vpb * a.wb;
        const uint4* f = reinterpret_cast<const uint4*>(static_cast<const __half*>(a.frames) + img_row0);
        const uint4* g = reinterpret_cast<const uint4*>(static_cast<const __half*>(a.img) + img_row0);
        for (int it = threadIdx.x; it < B * vpb; it += blockDim.x) {
          const int r = it / vpb, v = bx * vpb + it % vpb;
          const uint4 x = __ldg(f + (size_t)r * vpr + v), y = g[(size_t)r * vpr + v];
          const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            accum_h(sub_h(xs[k] & 0xFFFF, ys[k] & 0xFFFF), acc, flags);
            accum_h(sub_h(xs[k] >> 16, ys[k] >> 16), acc, flags);
          }
        }
      } else {
        const int upb = B / 16;
        const uint8_t* f = static_cast<const uint8_t*>(a.frames) + img_row0;
        const __half* g = static_cast<const __half*>(a.img) + img_row0;
        for (int it = threadIdx.x; it < B * upb * 48; it += blockDim.x) {
          const int r = it / (upb * 48), rem = it % (upb * 48), u = bx * upb + rem / 48, el = rem % 48;
          const int px = el / 3, c = el % 3;
          const uint8_t q = __ldg(f + (size_t)r * row_px * 3 + (size_t)u * 48 + px * 3 + (2 - c));
          const uint16_t hv = __half_as_ushort(s_lut[c * 256 + q]);
          const uint16_t gv = __half_as_ushort(g[(size_t)r * row_px * 3 + (size_t)u * 48 + el]);
          accum_h(sub_h(hv, gv), acc, flags);
        }
      }
      atomicAdd(&s_sx[bx], (unsigned long long)acc);
      if (flags) atomicOr(&s_flag[bx], flags << 2);
    }
    __syncthreads();
    for (int ai = threadIdx.x; ai < namb; ai += blockDim.x) {
      const int bx = s_amb[ai];
      const uint32_t fl = s_flag[bx] >> 2;
      bool ch;
      if (fl & GATE_NAN) ch = false;
      else if (fl & GATE_INF) ch = a.thr_fx < INT64_MAX;  // inf > finite thr; inf > inf is false
      else ch = (int64_t)s_sx[bx] > a.thr_fx;
      s_flag[bx] = ch ? 1u : 0u;
    }
    __syncthreads();
  }

  // extra + refresh (fused_engine.py:144-148)
  const int64_t tick = a.st->tick;
  for (int bx = threadIdx.x; bx < nblk; bx += blockDim.x) {
    const int64_t lin = ((int64_t)cam * a.hb + by) * a.wb + bx0 + bx;
    bool ch = s_flag[bx] == 1u;
    ch = ch || a.extra[lin] != 0;
    if (a.refresh) ch = ch || (lin % a.refresh) == (tick % a.refresh);
    a.changed[lin] = ch ? 1 : 0;
    s_flag[bx] = ch ? 1u : 0u;  // the changed flag for the update below
  }
  __syncthreads();

  // image-cache update for changed blocks (fused_engine.py:157-160)
  if (KIND == 2) {
    const int upb = B / 16;
    const uint8_t* f = static_cast<const uint8_t*>(a.frames) + img_row0;
    __half* g = static_cast<__half*>(a.img) + img_row0;
    for (int u = threadIdx.x; u < upb * nblk; u += blockDim.x) {
      if (!s_flag[u / upb]) continue;
      for (int r = 0; r < B; ++r) {
        const uint4* fp = reinterpret_cast<const uint4*>(f + (size_t)r * row_px * 3 + (size_t)u * 48);
        uint4* gp = reinterpret_cast<uint4*>(g + (size_t)r * row_px * 3 + (size_t)u * 48);
        uint4 fx[3], gx[6];
#pragma unroll
        for (int k = 0; k < 3; ++k) fx[k] = __ldg(fp + k);
        const uint8_t* fb = reinterpret_cast<const uint8_t*>(fx);
        uint16_t* gh = reinterpret_cast<uint16_t*>(gx);
#pragma unroll
        for (int j = 0; j < 48; ++j) {
          const int px = j / 3, c = j % 3;
          gh[j] = __half_as_ushort(s_lut[c * 256 + fb[px * 3 + (2 - c)]]);
        }
#pragma unroll
        for (int k = 0; k < 6; ++k) gp[k] = gx[k];
      }
    }
  } else {
    const int esz = KIND == 0 ? 2 : 4;
    const int vpb = B * 3 * esz / 16, vpr = vpb * a.wb;
    const uint4* f = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.frames) + img_row0 * esz);
    uint4* g = reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.img) + img_row0 * esz);
    for (int v = threadIdx.x; v < vpb * nblk; v += blockDim.x) {
      if (!s_flag[v / vpb]) continue;
#pragma unroll 4
      for (int r = 0; r < B; ++r) g[(size_t)r * vpr + v] = __ldg(f + (size_t)r * vpr + v);
    }
  }
  grid_dep_launch();
}

// ---------------------------------------------------------------- dilation + ordered lists
// One thread per block (flat index over all cameras), SB_LIST_CHUNK per CTA.  For each
// dilation d the mask is max_pool2d(changed, 2d+1, 1, d) within the camera
// (fused_engine.py:151); active blocks are compacted in ascending flat order
// (nonzero_static, :163) with a warp ballot, a CTA prefix and a decoupled look-back across
// CTAs in which a whole warp inspects 32 predecessors at a time.  Chunks are taken by
// ticket, so a CTA only ever waits on CTAs that are already running.
#define LIST_THREADS SB_LIST_CHUNK
#define LIST_WARPS (LIST_THREADS / 32)
#define LB_FLAG_AGG 1ull
#define LB_FLAG_INC 2ull

SB_DEV unsigned long long lb_pack(uint32_t epoch, unsigned long long flag, uint32_t v) {
  return ((unsigned long long)epoch << 32) | (flag << 30) | (unsigned long long)(v & 0x3FFFFFFFu);
}
SB_DEV void lb_store(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
SB_DEV unsigned long long lb_load(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
SB_DEV uint32_t warp_sum(uint32_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// Exclusive prefix of chunk `chunk` in the look-back array `stat` (executed by a full warp;
// the result is returned on every lane).  Lane i reads predecessor p - i; a window is
// usable once every lane up to the nearest inclusive prefix has published.
SB_DEV uint32_t lookback(unsigned long long* stat, uint32_t chunk, uint32_t epoch, State* st, uint32_t limit) {
  const uint32_t lane = threadIdx.x & 31;
  uint32_t excl = 0;
  int p = (int)chunk - 1;
  uint32_t spins = 0;
  while (p >= 0) {
    const int q = p - (int)lane;
    unsigned long long w = q >= 0 ? lb_load(stat + q) : lb_pack(epoch, LB_FLAG_INC, 0);  // before chunk 0: 0
    const bool ready = (uint32_t)(w >> 32) == epoch && ((w >> 30) & 3ull) != 0;
    const bool inc = ready && ((w >> 30) & 3ull) == LB_FLAG_INC;
    const uint32_t notready = __ballot_sync(0xFFFFFFFFu, !ready);
    const uint32_t incm = __ballot_sync(0xFFFFFFFFu, inc);
    const uint32_t upto = incm ? (2u << (__ffs(incm) - 1)) - 1u : 0xFFFFFFFFu;  // lanes 0..first inclusive
    if (notready & upto) {
      if (++spins > limit) {
        if (lane == 0) atomicOr(&st->error, SB_ERR_TIMEOUT_LOOKBK);
        break;
      }
      __nanosleep(32);
      continue;
    }
    const uint32_t v = (upto >> lane) & 1u ? (uint32_t)(w & 0x3FFFFFFFull) : 0u;
    excl += warp_sum(v);
    if (incm) break;
    p -= 32;
  }
  return excl;
}

// Cell-level gate (fp16 frames).  A cell of c x c pixels changed when its exact
// sum(|fp16(fp32(a) - fp32(b))|) exceeds float32(tau * c^2 * 3) -- the block rule of the
// gate above, applied per cell (the reference's gating.py:18-22 estimates cells the same
// way, as a mean) -- or when its block is forced by `extra` or the refresh phase.  A block
// changed when any of its cells did; changed blocks are copied into the image cache as in
// the block-level gate.  One CTA per (block row, camera); one thread per (cell row of the
// block row, cell column), summing exactly in integer multiples of 2^-24.
__global__ void __launch_bounds__(256) cell_gate_kernel(CellGateArgs a) {
  grid_dep_wait();
  if (in_hysteresis(a.st)) return;
  extern __shared__ uint32_t s_blk[];  // [wb] changed flag per block of this block row
  const int by = blockIdx.x, cam = blockIdx.y;
  for (int i = threadIdx.x; i < a.wb; i += blockDim.x) s_blk[i] = 0u;
  __syncthreads();
  const int C = a.cell, k = a.k;
  const int vpc = C * 3 / 8;                    // 16-byte vectors per cell row (C % 8 == 0)
  const size_t row_v = (size_t)a.w * 3 / 8;     // 16-byte vectors per image row
  const size_t base = ((size_t)cam * a.h + (size_t)by * a.block) * row_v;
  const uint4* f = reinterpret_cast<const uint4*>(a.frames) + base;
  const uint4* g = reinterpret_cast<const uint4*>(a.img) + base;
  const int64_t tick = a.st->tick;
  for (int it = threadIdx.x; it < k * a.wc; it += blockDim.x) {
    const int j = it / a.wc, cx = it - j * a.wc, bx = cx / k;
    uint64_t acc = 0;
    uint32_t flags = 0;
    for (int r = 0; r < C; ++r) {
      const size_t off = (size_t)(j * C + r) * row_v + (size_t)cx * vpc;
      for (int v = 0; v < vpc; ++v) {
        const uint4 x = __ldg(f + off + v), y = __ldg(g + off + v);
        const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          accum_h(sub_h(xs[q] & 0xFFFF, ys[q] & 0xFFFF), acc, flags);
          accum_h(sub_h(xs[q] >> 16, ys[q] >> 16), acc, flags);
        }
      }
    }
    bool ch;
    if (flags & GATE_NAN) ch = false;
    else if (flags & GATE_INF) ch = a.thr_fx < INT64_MAX;  // inf > finite thr; inf > inf is false
    else ch = (int64_t)acc > a.thr_fx;
    const int64_t lin = ((int64_t)cam * a.hb + by) * a.wb + bx;
    ch = ch || a.extra[lin] != 0;
    if (a.refresh) ch = ch || (lin % a.refresh) == (tick % a.refresh);
    a.cells[((size_t)cam * a.hc + (size_t)by * k + j) * a.wc + cx] = ch ? 1 : 0;
    if (ch) s_blk[bx] = 1u;  // every writer stores the same value
  }
  __syncthreads();
  for (int bx = threadIdx.x; bx < a.wb; bx += blockDim.x)
    a.changed[((size_t)cam * a.hb + by) * a.wb + bx] = s_blk[bx] ? 1 : 0;
  // image-cache update for changed blocks (fused_engine.py:157-160); this CTA read its
  // block row of the cache above, and no other CTA reads it
  const int vpb = a.block * 3 / 8;
  uint4* gw = reinterpret_cast<uint4*>(a.img) + base;
  for (int v = threadIdx.x; v < vpb * a.wb; v += blockDim.x) {
    if (!s_blk[v / vpb]) continue;
#pragma unroll 4
    for (int r = 0; r < a.block; ++r) gw[(size_t)r * row_v + v] = __ldg(f + (size_t)r * row_v + v);
  }
  grid_dep_launch();
}

__global__ void __launch_bounds__(LIST_THREADS) lists_kernel(ListArgs a) {
  grid_dep_wait();
  State* st = a.st;
  if (in_hysteresis(st)) {  // hysteresis dense step: no gate, count -1 (fused_engine.py:222-226)
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      st->mode_cur = SB_MODE_DENSE;
      st->count_cur = -1;
    }
    return;
  }
  // compaction lanes: one per (unit kind, dilation); kind 0 = blocks, kind k >= 1 = regions
  // of rw[k-1] x rh[k-1] blocks (active when any of their blocks is active at that dilation)
  constexpr int NK = 1 + SB_MAX_RKINDS;
  constexpr int ML = NK * SB_MAX_DILATIONS;
  __shared__ uint32_t s_chunk;
  __shared__ uint32_t s_warp[ML][LIST_WARPS];
  __shared__ uint32_t s_excl[ML];
  const uint32_t epoch = st->epoch;
  const uint32_t spin_limit = st->lb_spin_limit ? st->lb_spin_limit : SB_SPIN_LIMIT;
  if (threadIdx.x == 0) s_chunk = atomicAdd(&st->ticket, 1u);
  __syncthreads();
  const uint32_t chunk = s_chunk;
  // test hook: this chunk keeps its look-back words unpublished, so its successor's bounded
  // wait runs out (sb_debug_withhold_lookback)
  const bool publish = st->lb_withhold != (int32_t)chunk + 1;
  const int nchunks = gridDim.x;
  const int f = (int)chunk * LIST_THREADS + threadIdx.x;
  const int per = a.hb * a.wb, ncam = a.n_blocks / per;
  const int nk = 1 + a.n_rk, nl = nk * a.n_dil;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t rank[ML];
  bool act[ML];
  int coord[NK][3];
  int caps[NK];
#pragma unroll
  for (int kind = 0; kind < NK; ++kind) {
    if (kind >= nk) break;
    const int rw = kind ? a.rw[kind - 1] : 1, rh = kind ? a.rh[kind - 1] : 1;
    const int gw = (a.wb + rw - 1) / rw, gh = (a.hb + rh - 1) / rh;
    caps[kind] = ncam * gh * gw;
    const bool valid = f < caps[kind];
    int cam = 0, ry = 0, rx = 0;
    if (valid) {
      cam = f / (gh * gw);
      const int r = f - cam * gh * gw;
      ry = r / gw;
      rx = r - ry * gw;
    }
    coord[kind][0] = cam;
    coord[kind][1] = ry;
    coord[kind][2] = rx;
    for (int di = 0; di < a.n_dil; ++di) {
      const uint8_t* cm = (a.src[di] ? a.src[di] : a.changed) + (size_t)cam * per;
      const int d = a.ds[di], L = kind * a.n_dil + di;
      bool on = false;
      if (valid) {
        // blocks: max_pool(2d+1) of `changed` (fused_engine.py:151); regions: any of their blocks
        const int y0 = max(0, ry * rh - d), y1 = min(a.hb - 1, ry * rh + rh - 1 + d);
        const int x0 = max(0, rx * rw - d), x1 = min(a.wb - 1, rx * rw + rw - 1 + d);
        // OR of the window's bytes, no early exit: the loads are independent and overlap
        uint32_t acc = 0;
        for (int y = y0; y <= y1; ++y) {
          const uint8_t* rowp = cm + y * a.wb;
#pragma unroll 4
          for (int x = x0; x <= x1; ++x) acc |= __ldg(rowp + x);
        }
        on = acc != 0;
        if (kind == 0) a.masks[(size_t)di * a.n_blocks + f] = on ? 1 : 0;
      }
      act[L] = on;
      const uint32_t bal = __ballot_sync(0xFFFFFFFFu, on);
      rank[L] = __popc(bal & ((1u << lane) - 1u));
      if (lane == 0) s_warp[L][warp] = __popc(bal);
    }
  }
  __syncthreads();
  // warp w handles compaction lanes w, w + LIST_WARPS, ...: CTA prefix, then the look-back
  for (int L = (int)warp; L < nl; L += LIST_WARPS) {
    const uint32_t v = lane < LIST_WARPS ? s_warp[L][lane] : 0u;
    uint32_t inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, o);
      if (lane >= (uint32_t)o) inc += t;
    }
    if (lane < LIST_WARPS) s_warp[L][lane] = inc - v;  // exclusive warp offsets
    const uint32_t agg = __shfl_sync(0xFFFFFFFFu, inc, 31);
    unsigned long long* stat = a.status + (size_t)L * nchunks;
    uint32_t excl = 0;
    if (chunk == 0) {
      if (lane == 0 && publish) lb_store(stat, lb_pack(epoch, LB_FLAG_INC, agg));
    } else {
      if (lane == 0 && publish) lb_store(stat + chunk, lb_pack(epoch, LB_FLAG_AGG, agg));
      excl = lookback(stat, chunk, epoch, st, spin_limit);
      if (lane == 0 && publish) lb_store(stat + chunk, lb_pack(epoch, LB_FLAG_INC, excl + agg));
    }
    if (lane == 0) {
      s_excl[L] = excl;
      if ((int)chunk == nchunks - 1) {
        const int kind = L / a.n_dil, di = L - kind * a.n_dil;
        if (kind == 0) st->counts[di] = (int32_t)(excl + agg);
        else st->rcounts[kind - 1][di] = (int32_t)(excl + agg);
      }
    }
  }
  __syncthreads();
  for (int L = 0; L < nl; ++L) {
    if (!act[L]) continue;
    const int kind = L / a.n_dil, di = L - kind * a.n_dil;
    const uint32_t pos = s_excl[L] + s_warp[L][warp] + rank[L];
    const int cap = caps[kind];
    if (pos < (uint32_t)cap) {
      int32_t* Lp = (kind ? a.rlists[kind - 1] : a.lists) + (size_t)di * 3 * cap;
      Lp[pos] = coord[kind][0];
      Lp[cap + pos] = coord[kind][1];
      Lp[2 * (size_t)cap + pos] = coord[kind][2];
    }
  }
  if ((int)chunk == nchunks - 1 && threadIdx.x == 0) {
    __threadfence();
    const int64_t k = st->counts[a.n_dil - 1];
    st->count_cur = k;
    if (st->m0_mode) {
      // M0 (block_sparse.py:264-275): no dense fallback; with a capacity every layer runs
      // exactly that many list entries (nonzero_static, size=capacity, fill_value=0)
      st->mode_cur = st->m0_cap > 0 ? SB_MODE_SPARSE : (k == 0 ? SB_MODE_SKIP : SB_MODE_SPARSE);
      st->force_tiles = st->m0_cap > 0 ? st->m0_cap : 0;
    } else {
      st->mode_cur = k == 0 ? SB_MODE_SKIP : (k <= st->fallback ? SB_MODE_SPARSE : SB_MODE_DENSE);
      st->force_tiles = 0;
    }
  }
  grid_dep_launch();
}

// ---------------------------------------------------------------- img copies
// Dense: img <- frames for every block when this step is dense (fused_engine.py:173).
// Masked (calibration replays): img <- frames where `changed` (:157-160).
__global__ void __launch_bounds__(256) copy_kernel(CopyArgs a) {
  grid_dep_wait();
  const int mode = a.st->mode_cur;
  // dense steps and M0-mode steps (the whole frame enters the image cache,
  // block_sparse.py:272) copy every block
  if (a.changed == nullptr && mode != SB_MODE_DENSE && !a.st->m0_mode) return;
  const int by = blockIdx.x, cam = blockIdx.y, B = a.block;
  __shared__ __half s_lut[768];
  if (a.u8) {
    for (int i = threadIdx.x; i < 768; i += blockDim.x) {
      const int c = i >> 8, u = i & 255;
      s_lut[i] = __float2half_rn(__fdiv_rn(__fsub_rn((float)u, a.mean[c]), a.stdv[c]));
    }
    __syncthreads();
  }
  const size_t row0 = ((size_t)cam * a.h + (size_t)by * B) * a.w * 3;
  const uint8_t* chg = a.changed ? a.changed + ((size_t)cam * a.hb + by) * a.wb : nullptr;
  if (a.u8) {
    const int upb = B / 16, upr = upb * a.wb;
    const uint8_t* f = static_cast<const uint8_t*>(a.frames) + row0;
    __half* g = static_cast<__half*>(a.img) + row0;
    for (int u = threadIdx.x; u < upr; u += blockDim.x) {
      if (chg && !chg[u / upb]) continue;
      for (int r = 0; r < B; ++r) {
        const uint4* fp = reinterpret_cast<const uint4*>(f + (size_t)r * a.w * 3 + (size_t)u * 48);
        uint4* gp = reinterpret_cast<uint4*>(g + (size_t)r * a.w * 3 + (size_t)u * 48);
        uint4 fx[3], gx[6];
        for (int k = 0; k < 3; ++k) fx[k] = __ldg(fp + k);
        const uint8_t* fb = reinterpret_cast<const uint8_t*>(fx);
        uint16_t* gh = reinterpret_cast<uint16_t*>(gx);
#pragma unroll
        for (int j = 0; j < 48; ++j) {
          const int px = j / 3, c = j % 3;
          gh[j] = __half_as_ushort(s_lut[c * 256 + fb[px * 3 + (2 - c)]]);
        }
        for (int k = 0; k < 6; ++k) gp[k] = gx[k];
      }
    }
  } else {
    const int vpb = B * 3 * a.elem_bytes / 16, vpr = vpb * a.wb;
    const uint4* f = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.frames) + row0 * a.elem_bytes);
    uint4* g = reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.img) + row0 * a.elem_bytes);
    for (int v = threadIdx.x; v < vpr; v += blockDim.x) {
      if (chg && !chg[v / vpb]) continue;
#pragma unroll 4
      for (int r = 0; r < B; ++r) g[(size_t)r * vpr + v] = __ldg(f + (size_t)r * vpr + v);
    }
  }
  grid_dep_launch();
}

// ---------------------------------------------------------------- state machine
// End of a step (fused_engine.py:222-240): tick, hysteresis, stats, result slot.
__global__ void finalize_kernel(State* st, int refresh, int32_t* host_out) {
  grid_dep_wait();
  if (threadIdx.x != 0) return;
  const int mode = st->mode_cur;
  if (in_hysteresis(st)) {
    st->dense_run += 1;
  } else {
    if (refresh) st->tick += 1;
    st->dense_run = mode == SB_MODE_DENSE ? 1 : 0;
  }
  st->stats[mode] += 1;
  st->last_mode = mode;
  st->last_count = st->count_cur;
  st->result[0] = mode;
  st->result[1] = st->count_cur;
  st->epoch = st->epoch + 1u == 0u ? 1u : st->epoch + 1u;
  st->ticket = 0u;
  if (host_out) {
    host_out[0] = mode;
    host_out[1] = (int32_t)st->count_cur;
    host_out[2] = st->error;
    host_out[3] = 1;  // written
  }
  grid_dep_launch();
}

// Reset / dense replay / calibration: force the mode of the conv sequence.
__global__ void set_mode_kernel(State* st, int mode, int reset_hyst, int64_t force_tiles) {
  if (threadIdx.x != 0) return;
  st->mode_cur = mode;
  st->force_tiles = (int32_t)force_tiles;
  if (reset_hyst) st->dense_run = 0;
}

// ---------------------------------------------------------------- launchers
namespace {
// Launch with programmatic stream serialisation: the kernel may be scheduled before the
// previous kernel of the stream completes and waits for it with griddepcontrol.wait.
template <typename... Args>
cudaError_t launch_pdl(void (*k)(Args...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, args...);
}
}  // namespace

cudaError_t launch_gate(const GateArgs& a_in, int kind, cudaStream_t s) {
  // row segments of about one 16-byte column per thread (fp16 / fp32 frames); the uint8
  // path keeps whole block rows (its 48-byte units give few threads per block)
  GateArgs a = a_in;
  const int per_block = kind == 0 ? a.block * 3 / 8 : kind == 1 ? a.block * 3 / 4 : a.wb * a.block;
  a.seg = kind == 2 ? a.wb : std::max(1, std::min(a.wb, 256 / std::max(1, per_block)));
  dim3 grid(a.hb, a.n, (a.wb + a.seg - 1) / a.seg);
  const size_t smem = (size_t)a.seg * (8 + 4 + 4 + 4) + 768 * 2 + 16;
  switch (kind) {
    case 0: return launch_pdl(gate_kernel<0>, grid, dim3(256), smem, s, a);
    case 1: return launch_pdl(gate_kernel<1>, grid, dim3(256), smem, s, a);
    default: return launch_pdl(gate_kernel<2>, grid, dim3(256), smem, s, a);
  }
}

cudaError_t launch_cell_gate(const CellGateArgs& a, cudaStream_t s) {
  return launch_pdl(cell_gate_kernel, dim3(a.hb, a.n), dim3(256), (size_t)a.wb * 4, s, a);
}

cudaError_t launch_lists(const ListArgs& a, int n_chunks, cudaStream_t s) {
  return launch_pdl(lists_kernel, dim3(n_chunks), dim3(LIST_THREADS), 0, s, a);
}

cudaError_t launch_copy(const CopyArgs& a, cudaStream_t s) {
  return launch_pdl(copy_kernel, dim3(a.hb, a.n), dim3(256), 0, s, a);
}

cudaError_t launch_finalize(State* st, int refresh, int32_t* host_out, cudaStream_t s) {
  return launch_pdl(finalize_kernel, dim3(1), dim3(32), 0, s, st, refresh, host_out);
}

cudaError_t launch_set_mode(State* st, int mode, int reset_hyst, int64_t force_tiles, cudaStream_t s) {
  set_mode_kernel<<<1, 32, 0, s>>>(st, mode, reset_hyst, force_tiles);
  return cudaGetLastError();
}

}  // namespace sb
