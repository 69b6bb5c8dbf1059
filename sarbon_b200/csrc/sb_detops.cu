// sb_detops.cu -- the detector's non-GEMM kernels (Bahrombekk/Sarbon sarbon/models/sarbon_det.py,
// deform_attn.py, box_ops.py), run under the reference's autocast dtype flow
// (sarbon/inference/video.py:116-118: fp16 linear / conv outputs, fp32 LayerNorm / softmax):
//
//   sb_layernorm      nn.LayerNorm over rows of D <= 1024 channels of (a + b), fp32 statistics;
//                     writes the fp32 rows and/or their fp16 copy and/or fp16(y + sign*pos)
//                     (the decoder's `tgt + pos` query, the encoder's `aifi(t + pos) - pos`)
//   sb_add_rows       out = fp16(a + sign * pos[row % period]) (fp32 or fp16 operands)
//   sb_dwconv3x3      depthwise 3x3 conv (padding 1) + folded BatchNorm + ReLU, NHWC fp16
//                     (fuse()'s second half, sarbon_det.py:73-77)
//   sb_upsample2x     nearest 2x upsampling of an NHWC fp16 map (F.interpolate, scale 2)
//   sb_topk_rows      top-K rows of max-over-classes logits, masked rows excluded
//                     (sarbon_det.py:314), ordered by value, ties by row index
//   sb_gather_rows    rows of a matrix by per-image indices (sarbon_det.py:315-320)
//   sb_deform_sample  MSDeformAttn after its projections (deform_attn.py:57-66 and :14-28):
//                     softmax of the attention logits, box-relative sampling locations,
//                     bilinear zero-padded sampling, weighted sum -> fp16
//   sb_box_*          the box heads of the encoder and decoder (sarbon_det.py:316-352,
//                     box_ops.py:78-106)
// Each kernel reads and writes caller memory on the caller's stream and allocates nothing.
// (The attention core is in sb_attn.cu.)
#include <cuda_fp16.h>

#include <cstdint>

#include "sb_internal.cuh"
#include "sb_ptx.cuh"

namespace sb {
namespace {

SB_DEV float ld_any(const void* p, int f32, long long i) {
  return f32 ? static_cast<const float*>(p)[i] : __half2float(static_cast<const __half*>(p)[i]);
}
SB_DEV float r16(float x) { return __half2float(__float2half_rn(x)); }  // one fp16 rounding

// ------------------------------------------------------------------ LayerNorm
// warp per row; D <= 1024, D % 32 == 0
__global__ void __launch_bounds__(256) layernorm_kernel(const void* a, int a_f32, long long lda, const void* b, int b_f32,
                                                        long long ldb, const float* gamma, const float* beta, float eps,
                                                        int rows, int D, float* y32, long long ld32, __half* y16,
                                                        long long ld16, const __half* pos, long long ldpos, int period,
                                                        float sign, __half* yp16, long long ldp) {
  const int row = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[32];
  const int per = D / 32;
  float s = 0.f;
#pragma unroll
  for (int t = 0; t < 32; ++t) {
    if (t < per) {
      const int c = lane + 32 * t;
      float x = ld_any(a, a_f32, (long long)row * lda + c);
      if (b) {
        x += ld_any(b, b_f32, (long long)row * ldb + c);
        if (!a_f32 && !b_f32) x = r16(x);  // an fp16 + fp16 sum is an fp16 tensor
      }
      v[t] = x;
      s += x;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  const float mean = s / (float)D;
  float q = 0.f;
#pragma unroll
  for (int t = 0; t < 32; ++t)
    if (t < per) {
      const float d = v[t] - mean;
      q += d * d;
    }
#pragma unroll
  for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xFFFFFFFFu, q, o);
  const float rstd = rsqrtf(q / (float)D + eps);
  const long long prow = pos ? (long long)(row % period) * ldpos : 0;
#pragma unroll
  for (int t = 0; t < 32; ++t) {
    if (t < per) {
      const int c = lane + 32 * t;
      const float y = (v[t] - mean) * rstd * gamma[c] + beta[c];
      if (y32) y32[(long long)row * ld32 + c] = y;
      if (y16) y16[(long long)row * ld16 + c] = __float2half_rn(y);
      if (yp16) yp16[(long long)row * ldp + c] = __float2half_rn(y + sign * __half2float(pos[prow + c]));
    }
  }
}

// D = 256 with 16-byte aligned rows: lane l holds channels 8l..8l+7 (one 16-byte fp16 or two
// 16-byte fp32 accesses per operand), otherwise the same arithmetic as layernorm_kernel
SB_DEV void load8(const void* p, int f32, long long off, float (&v)[8]) {
  if (f32) {
    const float4 x0 = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + off);
    const float4 x1 = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + off + 4);
    v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w; v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
  } else {
    const uint4 raw = *reinterpret_cast<const uint4*>(static_cast<const __half*>(p) + off);
    const __half2* hh = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 f = __half22float2(hh[u]);
      v[2 * u] = f.x;
      v[2 * u + 1] = f.y;
    }
  }
}
SB_DEV uint4 pack8(const float (&v)[8]) {
  uint4 o;
  __half2* hh = reinterpret_cast<__half2*>(&o);
#pragma unroll
  for (int u = 0; u < 4; ++u) hh[u] = __floats2half2_rn(v[2 * u], v[2 * u + 1]);
  return o;
}

__global__ void __launch_bounds__(256) layernorm256_kernel(const void* a, int a_f32, long long lda, const void* b,
                                                           int b_f32, long long ldb, const float* gamma,
                                                           const float* beta, float eps, int rows, float* y32,
                                                           long long ld32, __half* y16, long long ld16,
                                                           const __half* pos, long long ldpos, int period, float sign,
                                                           __half* yp16, long long ldp) {
  const int row = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int c = lane * 8;
  float v[8];
  load8(a, a_f32, (long long)row * lda + c, v);
  if (b) {
    float w[8];
    load8(b, b_f32, (long long)row * ldb + c, w);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      v[u] += w[u];
      if (!a_f32 && !b_f32) v[u] = r16(v[u]);  // an fp16 + fp16 sum is an fp16 tensor
    }
  }
  float s = 0.f;
#pragma unroll
  for (int u = 0; u < 8; ++u) s += v[u];
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  const float mean = s * (1.f / 256.f);
  float q = 0.f;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const float d = v[u] - mean;
    q += d * d;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xFFFFFFFFu, q, o);
  const float rstd = rsqrtf(q * (1.f / 256.f) + eps);
  float gm[8], bt[8], y[8];
  load8(gamma, 1, c, gm);
  load8(beta, 1, c, bt);
#pragma unroll
  for (int u = 0; u < 8; ++u) y[u] = (v[u] - mean) * rstd * gm[u] + bt[u];
  if (y32) {
    float* p = y32 + (long long)row * ld32 + c;
    *reinterpret_cast<float4*>(p) = make_float4(y[0], y[1], y[2], y[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(y[4], y[5], y[6], y[7]);
  }
  if (y16) *reinterpret_cast<uint4*>(y16 + (long long)row * ld16 + c) = pack8(y);
  if (yp16) {
    float pv[8];
    load8(pos, 0, (long long)(row % period) * ldpos + c, pv);
#pragma unroll
    for (int u = 0; u < 8; ++u) pv[u] = y[u] + sign * pv[u];
    *reinterpret_cast<uint4*>(yp16 + (long long)row * ldp + c) = pack8(pv);
  }
}

__global__ void add_rows_kernel(const void* a, int a_f32, long long lda, const void* pos, int p_f32, long long ldpos,
                                int period, float sign, int rows, int D, __half* out, long long ldo) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long long)rows * D) return;
  const int row = (int)(i / D), c = (int)(i - (long long)row * D);
  const float x = ld_any(a, a_f32, (long long)row * lda + c);
  out[(long long)row * ldo + c] = __float2half_rn(x + sign * ld_any(pos, p_f32, (long long)(row % period) * ldpos + c));
}

// ------------------------------------------------------------------ depthwise conv, upsample
// grid (x: groups of kDwCols pixels of a row x 8-channel groups, y: row, z: image); a thread
// computes kDwCols neighbouring output pixels of one row and 8 channels: per kernel row it
// loads the kDwCols + 2 input pixels once and each tap's 8 weights once for all of them;
// w [9][C] fp32 (BatchNorm folded), bias [C]
constexpr int kDwCols = 4;
__global__ void __launch_bounds__(256) dwconv3x3_kernel(const __half* x, long long ldx, long long imgx, int H, int W,
                                                        int C, const float* w, const float* bias, int relu, __half* y,
                                                        long long ldy, long long imgy) {
  const int cg = C >> 3, ng = (W + kDwCols - 1) / kDwCols;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= ng * cg) return;
  const int xg = i / cg, c0 = (i - xg * cg) * 8;
  const int x0 = xg * kDwCols, yo = blockIdx.y, b = blockIdx.z;
  float acc[kDwCols][8];
  {
    const float4 b0 = *reinterpret_cast<const float4*>(bias + c0), b1 = *reinterpret_cast<const float4*>(bias + c0 + 4);
#pragma unroll
    for (int o = 0; o < kDwCols; ++o) {
      acc[o][0] = b0.x; acc[o][1] = b0.y; acc[o][2] = b0.z; acc[o][3] = b0.w;
      acc[o][4] = b1.x; acc[o][5] = b1.y; acc[o][6] = b1.z; acc[o][7] = b1.w;
    }
  }
  const __half* xb = x + (long long)b * imgx * ldx;
#pragma unroll
  for (int ky = 0; ky < 3; ++ky) {
    const int yi = yo + ky - 1;
    if (yi < 0 || yi >= H) continue;
    __half2 col[kDwCols + 2][4];
#pragma unroll
    for (int cidx = 0; cidx < kDwCols + 2; ++cidx) {
      const int xx = x0 + cidx - 1;
      uint4 raw = make_uint4(0, 0, 0, 0);
      if (xx >= 0 && xx < W) raw = *reinterpret_cast<const uint4*>(xb + ((long long)yi * W + xx) * ldx + c0);
      const __half2* hh = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
      for (int u = 0; u < 4; ++u) col[cidx][u] = hh[u];
    }
#pragma unroll
    for (int kx = 0; kx < 3; ++kx) {
      const float* wt = w + (ky * 3 + kx) * C + c0;
      const float4 w0 = *reinterpret_cast<const float4*>(wt), w1 = *reinterpret_cast<const float4*>(wt + 4);
      const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int o = 0; o < kDwCols; ++o)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float2 f = __half22float2(col[o + kx][u]);
          acc[o][2 * u] = fmaf(f.x, wv[2 * u], acc[o][2 * u]);
          acc[o][2 * u + 1] = fmaf(f.y, wv[2 * u + 1], acc[o][2 * u + 1]);
        }
    }
  }
#pragma unroll
  for (int o = 0; o < kDwCols; ++o) {
    const int xo = x0 + o;
    if (xo >= W) break;
    uint4 ov;
    __half2* oh = reinterpret_cast<__half2*>(&ov);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float a0 = acc[o][2 * u], a1 = acc[o][2 * u + 1];
      if (relu) {
        a0 = fmaxf(a0, 0.f);
        a1 = fmaxf(a1, 0.f);
      }
      oh[u] = __floats2half2_rn(a0, a1);
    }
    *reinterpret_cast<uint4*>(y + ((long long)b * imgy + (long long)yo * W + xo) * ldy + c0) = ov;
  }
}

// grid (x: output pixels of a row x 8-channel groups, y: output row, z: image)
__global__ void upsample2x_kernel(const __half* x, long long ldx, long long imgx, int W, int C, __half* y, long long ldy,
                                  long long imgy) {
  const int cg = C >> 3, W2 = 2 * W;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= W2 * cg) return;
  const int xo = i / cg, c0 = (i - xo * cg) * 8;
  const int yo = blockIdx.y, b = blockIdx.z;
  *reinterpret_cast<uint4*>(y + ((long long)b * imgy + (long long)yo * W2 + xo) * ldy + c0) =
      *reinterpret_cast<const uint4*>(x + ((long long)b * imgx + (long long)(yo >> 1) * W + (xo >> 1)) * ldx + c0);
}

// ------------------------------------------------------------------ top-K
// One CTA of 1024 threads per image.  Keys: the fp16 bit pattern of max over classes mapped
// to an unsigned order (masked rows: -inf); a two-pass byte radix select finds the K-th key,
// an ordered compaction keeps every larger key and the first (in row order) equal ones, and
// a bitonic sort orders the K rows by (key descending, row ascending).
constexpr int kTopkThreads = 1024;
constexpr int kTopkMaxRows = 65536;
constexpr int kTopkMaxK = 1024;

SB_DEV uint32_t order_key(__half h) {
  const uint16_t b = __half_as_ushort(h);
  return (b & 0x8000u) ? (uint32_t)(~b & 0xFFFFu) : (uint32_t)(b | 0x8000u);
}

SB_DEV int block_exclusive_scan(int x, int* warp_sums, int& total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int inc = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += t;
  }
  if (lane == 31) warp_sums[w] = inc;
  __syncthreads();
  if (w == 0) {
    int s = warp_sums[lane];
    int si = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xFFFFFFFFu, si, o);
      if (lane >= o) si += t;
    }
    warp_sums[lane] = si - s;
    if (lane == 31) warp_sums[32] = si;
  }
  __syncthreads();
  const int r = inc - x + warp_sums[w];
  total = warp_sums[32];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kTopkThreads) topk_kernel(const __half* logits, long long ld, long long img, int S,
                                                            int C, const uint8_t* valid, int K, int32_t* idx_out,
                                                            long long ldi) {
  extern __shared__ uint8_t tsm[];
  uint16_t* keys = reinterpret_cast<uint16_t*>(tsm);                                  // [S]
  unsigned long long* cand = reinterpret_cast<unsigned long long*>(tsm + ((S * 2 + 15) & ~15));  // [kTopkMaxK]
  __shared__ int hist[256];
  __shared__ int warp_sums[33];
  __shared__ int sel[4];
  const int b = blockIdx.x;
  const __half* lg = logits + (long long)b * img * ld;
  for (int i = threadIdx.x; i < S; i += kTopkThreads) {
    uint32_t key = 0;  // -inf and masked rows sort last (the key of -inf is 0x03FF; 0 is below every value)
    if (!valid || valid[i]) {
      __half mx = lg[(long long)i * ld];
      for (int c = 1; c < C; ++c) {
        const __half x = lg[(long long)i * ld + c];
        if (__hgt(x, mx)) mx = x;
      }
      key = order_key(mx);
    }
    keys[i] = (uint16_t)key;
  }
  // pass 1: high byte
  for (int i = threadIdx.x; i < 256; i += kTopkThreads) hist[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < S; i += kTopkThreads) atomicAdd(&hist[keys[i] >> 8], 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    int above = 0, hb = 0;
    for (int bkt = 255; bkt >= 0; --bkt) {
      if (above + hist[bkt] >= K) { hb = bkt; break; }
      above += hist[bkt];
    }
    sel[0] = hb;
    sel[1] = above;  // keys with a larger high byte
  }
  __syncthreads();
  const int hb = sel[0], above_hi = sel[1];
  for (int i = threadIdx.x; i < 256; i += kTopkThreads) hist[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < S; i += kTopkThreads)
    if ((keys[i] >> 8) == hb) atomicAdd(&hist[keys[i] & 0xFF], 1);
  __syncthreads();
  if (threadIdx.x == 0) {
    int above = above_hi, lb = 0;
    for (int bkt = 255; bkt >= 0; --bkt) {
      if (above + hist[bkt] >= K) { lb = bkt; break; }
      above += hist[bkt];
    }
    sel[2] = (hb << 8) | lb;
    sel[3] = above;  // keys above the threshold key (< K)
  }
  __syncthreads();
  const uint32_t thr = (uint32_t)sel[2];
  const int n_gt = sel[3], need_eq = K - n_gt;
  int base_gt = 0, base_eq = 0;
  for (int c0 = 0; c0 < S; c0 += kTopkThreads) {
    const int i = c0 + threadIdx.x;
    const uint32_t key = i < S ? keys[i] : 0u;
    const int gt = i < S && key > thr, eq = i < S && key == thr;
    int tg, te;
    const int pg = block_exclusive_scan(gt, warp_sums, tg);
    const int pe = block_exclusive_scan(eq, warp_sums, te);
    const unsigned long long comp = ((unsigned long long)key << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)i);
    if (gt) cand[base_gt + pg] = comp;
    if (eq && base_eq + pe < need_eq) cand[n_gt + base_eq + pe] = comp;
    base_gt += tg;
    base_eq += te;
  }
  __syncthreads();
  // bitonic sort (descending) over the next power of two >= K
  int P = 1;
  while (P < K) P <<= 1;
  for (int i = K + threadIdx.x; i < P; i += kTopkThreads) cand[i] = 0ull;
  __syncthreads();
  for (int size = 2; size <= P; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < P; i += kTopkThreads) {
        const int j = i ^ stride;
        if (j > i) {
          const bool desc = (i & size) == 0;
          const unsigned long long x = cand[i], y = cand[j];
          if (desc ? (x < y) : (x > y)) {
            cand[i] = y;
            cand[j] = x;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < K; i += kTopkThreads)
    idx_out[(long long)b * ldi + i] = (int32_t)(0xFFFFFFFFu - (uint32_t)(cand[i] & 0xFFFFFFFFull));
}

// ------------------------------------------------------------------ gather
// out[b, i, :] = src[b, idx[b, i], :] for D columns (zeros for an index outside [0, S));
// fp32 and/or fp16 outputs
__global__ void gather_rows_kernel(const void* src, int s_f32, long long lds, long long imgs, int S,
                                   const int32_t* idx, long long ldi, int B, int K, int D, float* o32, long long ld32,
                                   long long img32, __half* o16, long long ld16, long long img16) {
  const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (long long)B * K * D) return;
  const int c = (int)(t % D);
  const long long r = t / D;
  const int i = (int)(r % K), b = (int)(r / K);
  const int row = idx[(long long)b * ldi + i];
  const float x = row >= 0 && row < S ? ld_any(src, s_f32, ((long long)b * imgs + row) * lds + c) : 0.f;
  if (o32) o32[((long long)b * img32 + i) * ld32 + c] = x;
  if (o16) o16[((long long)b * img16 + i) * ld16 + c] = __float2half_rn(x);
}

// ------------------------------------------------------------------ deformable sampling
// Warp per (b, q, h); lane = channel (dh = 32).  deform_attn.py:57-66: w = softmax(attn
// logits) in fp32; loc = ref_xy + off / P * ref_wh * 0.5 evaluated in the reference box's
// type (fp16 arithmetic for an fp16 box, each product and sum rounded); core :14-28:
// grid = 2 * loc - 1 in loc's type, then grid_sample(bilinear, zeros, align_corners=False).
constexpr int kMaxLevels = 8;
struct DeformSampleArgs {
  const __half* value;  // [B][S][H*32] rows (ld, img)
  long long ldv, imgv;
  const __half* off;    // [B][Q][H*L*P*2]
  long long ldoff, imgoff;
  const __half* att;    // [B][Q][H*L*P] logits
  long long ldatt, imgatt;
  const void* ref;      // [B][Q][4] cxcywh, fp16 or fp32
  int ref_f32;
  long long ldref, imgref;
  __half* out;          // [B][Q][H*32]
  long long ldo, imgo;
  int B, Q, H, L, P;
  int lh[kMaxLevels], lw[kMaxLevels], lstart[kMaxLevels];
};

// Lane k < L*P first works out sampling point k (its softmax weight, location, the value rows
// of its four bilinear corners and their weights, corners outside the map dropped); every
// lane then takes each point's corners by shuffle and reads its own channel of them, so the
// warp's corner loads are independent of one another.
__global__ void __launch_bounds__(256) deform_sample_kernel(DeformSampleArgs a) {
  const int gw = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (gw >= a.B * a.Q * a.H) return;  // warp-uniform
  const int h = gw % a.H, qi = (gw / a.H) % a.Q, b = gw / (a.H * a.Q);
  const int LP = a.L * a.P;
  const bool mine = lane < LP;
  const int k = mine ? lane : 0;
  // softmax over the L*P logits of this head (lane k holds logit k)
  const __half* lg = a.att + ((long long)b * a.imgatt + qi) * a.ldatt + (long long)h * LP;
  const float x = mine ? __half2float(lg[k]) : -INFINITY;
  float mx = x;
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
  const float ex = mine ? expf(x - mx) : 0.f;
  float den = ex;
#pragma unroll
  for (int o = 16; o; o >>= 1) den += __shfl_xor_sync(0xFFFFFFFFu, den, o);
  const float w = ex / den;
  // geometry of point k
  int row00 = -1, row01 = -1, row10 = -1, row11 = -1;
  float w00 = 0.f, w01 = 0.f, w10 = 0.f, w11 = 0.f;
  if (mine) {
    const int l = k / a.P;
    const int H_ = a.lh[l], W_ = a.lw[l];
    const long long ro = ((long long)b * a.imgref + qi) * a.ldref;
    const float rx = ld_any(a.ref, a.ref_f32, ro), ry = ld_any(a.ref, a.ref_f32, ro + 1);
    const float rw = ld_any(a.ref, a.ref_f32, ro + 2), rh = ld_any(a.ref, a.ref_f32, ro + 3);
    const __half* op = a.off + ((long long)b * a.imgoff + qi) * a.ldoff + (long long)h * LP * 2;
    const float ox = __half2float(op[2 * k]), oy = __half2float(op[2 * k + 1]);
    float gx, gy;
    if (a.ref_f32) {
      // off / P (fp16) * ref_wh (fp32) * 0.5 + ref_xy in fp32; grid in fp32
      const float tx = r16(ox / (float)a.P), ty = r16(oy / (float)a.P);
      const float lx = __fadd_rn(rx, __fmul_rn(__fmul_rn(tx, rw), 0.5f));
      const float ly = __fadd_rn(ry, __fmul_rn(__fmul_rn(ty, rh), 0.5f));
      gx = __fsub_rn(__fmul_rn(2.f, lx), 1.f);
      gy = __fsub_rn(__fmul_rn(2.f, ly), 1.f);
    } else {
      // every op of the fp16 expression rounded to fp16
      const float tx = r16(ox / (float)a.P), ty = r16(oy / (float)a.P);
      const float lx = r16(rx + r16(r16(tx * rw) * 0.5f));
      const float ly = r16(ry + r16(r16(ty * rh) * 0.5f));
      gx = r16(r16(2.f * lx) - 1.f);
      gy = r16(r16(2.f * ly) - 1.f);
    }
    const float ix = __fdiv_rn(__fsub_rn(__fmul_rn(__fadd_rn(gx, 1.f), (float)W_), 1.f), 2.f);
    const float iy = __fdiv_rn(__fsub_rn(__fmul_rn(__fadd_rn(gy, 1.f), (float)H_), 1.f), 2.f);
    const float fx = floorf(ix), fy = floorf(iy);
    // the sampling point may lie far outside the map: clamp before the int conversion
    const float cfx = fminf(fmaxf(fx, -2.f), (float)W_ + 1.f), cfy = fminf(fmaxf(fy, -2.f), (float)H_ + 1.f);
    const int x0 = (int)cfx, y0 = (int)cfy;
    const float tx1 = __fsub_rn(ix, fx), ty1 = __fsub_rn(iy, fy);
    const float tx0 = __fsub_rn(__fadd_rn(fx, 1.f), ix), ty0 = __fsub_rn(__fadd_rn(fy, 1.f), iy);
    const bool x0in = x0 >= 0 && x0 < W_, x1in = x0 + 1 >= 0 && x0 + 1 < W_;
    const bool y0in = y0 >= 0 && y0 < H_, y1in = y0 + 1 >= 0 && y0 + 1 < H_;
    const int base = a.lstart[l];
    if (y0in && x0in) { row00 = base + y0 * W_ + x0; w00 = __fmul_rn(tx0, ty0); }
    if (y0in && x1in) { row01 = base + y0 * W_ + x0 + 1; w01 = __fmul_rn(tx1, ty0); }
    if (y1in && x0in) { row10 = base + (y0 + 1) * W_ + x0; w10 = __fmul_rn(tx0, ty1); }
    if (y1in && x1in) { row11 = base + (y0 + 1) * W_ + x0 + 1; w11 = __fmul_rn(tx1, ty1); }
  }
  const __half* vb = a.value + (long long)b * a.imgv * a.ldv + h * 32 + lane;
  float acc = 0.f;
  for (int j = 0; j < LP; ++j) {
    const int i00 = __shfl_sync(0xFFFFFFFFu, row00, j), i01 = __shfl_sync(0xFFFFFFFFu, row01, j);
    const int i10 = __shfl_sync(0xFFFFFFFFu, row10, j), i11 = __shfl_sync(0xFFFFFFFFu, row11, j);
    const float c00 = __shfl_sync(0xFFFFFFFFu, w00, j), c01 = __shfl_sync(0xFFFFFFFFu, w01, j);
    const float c10 = __shfl_sync(0xFFFFFFFFu, w10, j), c11 = __shfl_sync(0xFFFFFFFFu, w11, j);
    const float wj = __shfl_sync(0xFFFFFFFFu, w, j);
    const float v00 = i00 >= 0 ? __half2float(vb[(long long)i00 * a.ldv]) : 0.f;
    const float v01 = i01 >= 0 ? __half2float(vb[(long long)i01 * a.ldv]) : 0.f;
    const float v10 = i10 >= 0 ? __half2float(vb[(long long)i10 * a.ldv]) : 0.f;
    const float v11 = i11 >= 0 ? __half2float(vb[(long long)i11 * a.ldv]) : 0.f;
    float sv = 0.f;
    sv = fmaf(v00, c00, sv);
    sv = fmaf(v01, c01, sv);
    sv = fmaf(v10, c10, sv);
    sv = fmaf(v11, c11, sv);
    acc = fmaf(sv, wj, acc);
  }
  a.out[((long long)b * a.imgo + qi) * a.ldo + h * 32 + lane] = __float2half_rn(acc);
}

// ------------------------------------------------------------------ box heads
// Encoder proposals (sarbon_det.py:316-321): ref_logit = fp16(enc_box(x) + anchor[row]);
// ref = fp16(sigmoid(ref_logit)); also the query_pos input (ref as fp16 in a 64-wide row).
// (an index outside [0, S) takes an anchor of 0)
__global__ void box_enc_kernel(const __half* encbox, long long ldb, const __half* anchors, int S, const int32_t* idx,
                               int B, int K, __half* ref16, __half* qin, long long ldq) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= B * K * 4) return;
  const int c = t & 3, r = t >> 2;
  const int row = idx[r];
  const float an = row >= 0 && row < S ? __half2float(anchors[(long long)row * 4 + c]) : 0.f;
  const float lg = r16(__half2float(encbox[(long long)r * ldb + c]) + an);
  const __half v = __float2half_rn(1.f / (1.f + expf(-lg)));
  ref16[(long long)r * 4 + c] = v;
  qin[(long long)r * ldq + c] = v;
}

// Decoder box of layer i (sarbon_det.py:336-350, box_ops.py:78-106):
//   layer 0: pre = sigmoid(prebox(x) + inverse_sigmoid(ref)), ref_init = pre;
//            corners = head(x)
//   layer i > 0: corners = fp16(head(x) + corners)
//   box = distance2bbox(ref_init, integral(corners), reg_scale)   [fp32 points]
// integral: softmax over the R+1 bins of each edge (fp32), then the fp16 product with the
// bin values (fp32 accumulation of fp16 operands).  Thread per (row, edge); with RC > 0 bins
// known at compile time the edge's bins stay in registers (independent loads, one exp each).
template <int RC>
__global__ void box_dec_kernel(int first, const __half* prebox, long long ldp, const __half* ref16,
                               const __half* head, long long ldh, __half* corners, long long ldc, int R1,
                               const float* project, float reg_scale, float* ref_init, float* box, __half* qin,
                               long long ldq, int rows) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const bool active = t < rows * 4;  // no early exit: the row's four threads exchange their edges
  const int r = active ? t >> 2 : 0, e = t & 3;
  float dist = 0.f;
  if (active) {
    const __half* hp = head + (long long)r * ldh + e * R1;
    __half* cp = corners + (long long)r * ldc + e * R1;
    if constexpr (RC > 0) {
      float c[RC];
#pragma unroll
      for (int j = 0; j < RC; ++j) c[j] = __half2float(hp[j]);
      if (!first) {
#pragma unroll
        for (int j = 0; j < RC; ++j) c[j] = r16(c[j] + __half2float(cp[j]));
      }
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < RC; ++j) {
        cp[j] = __float2half_rn(c[j]);
        c[j] = __half2float(__float2half_rn(c[j]));
        mx = fmaxf(mx, c[j]);
      }
      float den = 0.f;
#pragma unroll
      for (int j = 0; j < RC; ++j) {
        c[j] = expf(c[j] - mx);
        den += c[j];
      }
#pragma unroll
      for (int j = 0; j < RC; ++j) dist = fmaf(r16(c[j] / den), r16(project[j]), dist);
    } else {
      float mx = -INFINITY;
      for (int j = 0; j < R1; ++j) {
        float c = __half2float(hp[j]);
        if (!first) c = r16(c + __half2float(cp[j]));
        cp[j] = __float2half_rn(c);
        mx = fmaxf(mx, c);
      }
      float den = 0.f;
      for (int j = 0; j < R1; ++j) den += expf(__half2float(cp[j]) - mx);
      for (int j = 0; j < R1; ++j) {
        const float p = expf(__half2float(cp[j]) - mx) / den;
        dist = fmaf(r16(p), r16(project[j]), dist);
      }
    }
    dist = r16(dist);
    if (first) {
      // pre = sigmoid(prebox + inverse_sigmoid(ref)); inverse_sigmoid on the fp16 box:
      // clamp(1e-5, 1 - 1e-5) and x / (1 - x) in fp16, the log in fp32
      const float x = __half2float(ref16[(long long)r * 4 + e]);
      const float xc = r16(fminf(fmaxf(x, 1e-5f), 1.f - 1e-5f));
      const float inv = logf(r16(xc / r16(1.f - xc)));
      const float pre = 1.f / (1.f + expf(-(__half2float(prebox[(long long)r * ldp + e]) + inv)));
      ref_init[(long long)r * 4 + e] = pre;
    }
  }
  __syncwarp();
  // the four edges of the row are the four consecutive threads t = 4r + e
  const unsigned mask = 0xFFFFFFFFu;
  const float d0 = __shfl_sync(mask, dist, (threadIdx.x & ~3) + 0);
  const float d1 = __shfl_sync(mask, dist, (threadIdx.x & ~3) + 1);
  const float d2 = __shfl_sync(mask, dist, (threadIdx.x & ~3) + 2);
  const float d3 = __shfl_sync(mask, dist, (threadIdx.x & ~3) + 3);
  if (active && e == 0) {
    const float cx = ref_init[(long long)r * 4 + 0], cy = ref_init[(long long)r * 4 + 1];
    const float w = ref_init[(long long)r * 4 + 2], h = ref_init[(long long)r * 4 + 3];
    const float sw = w / reg_scale, sh = h / reg_scale;
    const float hr = 0.5f * reg_scale;
    const float x0 = cx - r16(hr + d0) * sw, y0 = cy - r16(hr + d1) * sh;
    const float x1 = cx + r16(hr + d2) * sw, y1 = cy + r16(hr + d3) * sh;
    const float bx[4] = {(x0 + x1) / 2.f, (y0 + y1) / 2.f, x1 - x0, y1 - y0};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      box[(long long)r * 4 + c] = bx[c];
      if (qin) qin[(long long)r * ldq + c] = __float2half_rn(bx[c]);
    }
  }
}

// F.normalize(x.float(), dim=-1): x / max(||x||_2, 1e-12); warp per row
__global__ void l2norm_rows_kernel(const __half* x, long long ldx, int rows, int D, float* out, long long ldo) {
  const int row = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  float s = 0.f;
  for (int c = lane; c < D; c += 32) {
    const float v = __half2float(x[(long long)row * ldx + c]);
    s += v * v;
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  const float inv = 1.f / fmaxf(sqrtf(s), 1e-12f);
  for (int c = lane; c < D; c += 32) out[(long long)row * ldo + c] = __half2float(x[(long long)row * ldx + c]) * inv;
}

cudaError_t last() { return cudaGetLastError(); }
unsigned blocks_for(long long n, int t) { return (unsigned)((n + t - 1) / t); }

}  // namespace
}  // namespace sb

using namespace sb;

#define SB_LAUNCH_CHECK(what)                                        \
  do {                                                               \
    const cudaError_t e_ = last();                                   \
    if (e_ != cudaSuccess) return record_error(SB_ECUDA, cudaGetErrorString(e_)); \
  } while (0)

extern "C" int sb_layernorm(const void* a, int a_dtype, long long lda, const void* b, int b_dtype, long long ldb,
                            const float* gamma, const float* beta, float eps, int rows, int D, float* y32,
                            long long ld32, void* y16, long long ld16, const void* pos, long long ldpos, int period,
                            float sign, void* yp16, long long ldp, void* stream) {
  if (!a || !gamma || !beta || rows < 1 || D < 32 || D > 1024 || D % 32 != 0 || (!y32 && !y16 && !yp16) ||
      (yp16 && (!pos || period < 1)))
    return record_error(SB_EINVAL, "sb_layernorm: arguments");
  auto al = [](const void* p, long long ld, int f32) {
    return p == nullptr || ((reinterpret_cast<uintptr_t>(p) & 15) == 0 && (ld * (f32 ? 4 : 2)) % 16 == 0);
  };
  if (D == 256 && al(a, lda, a_dtype == SB_F32) && al(b, ldb, b_dtype == SB_F32) && al(y32, ld32, 1) &&
      al(y16, ld16, 0) && al(pos, ldpos, 0) && al(yp16, ldp, 0) && al(gamma, 0, 1) && al(beta, 0, 1)) {
    layernorm256_kernel<<<blocks_for((long long)rows * 32, 256), 256, 0, (cudaStream_t)stream>>>(
        a, a_dtype == SB_F32, lda, b, b_dtype == SB_F32, ldb, gamma, beta, eps, rows, y32, ld32,
        static_cast<__half*>(y16), ld16, static_cast<const __half*>(pos), ldpos, period > 0 ? period : 1, sign,
        static_cast<__half*>(yp16), ldp);
    SB_LAUNCH_CHECK("sb_layernorm");
    return SB_OK;
  }
  layernorm_kernel<<<blocks_for((long long)rows * 32, 256), 256, 0, (cudaStream_t)stream>>>(
      a, a_dtype == SB_F32, lda, b, b_dtype == SB_F32, ldb, gamma, beta, eps, rows, D, y32, ld32,
      static_cast<__half*>(y16), ld16, static_cast<const __half*>(pos), ldpos, period > 0 ? period : 1, sign,
      static_cast<__half*>(yp16), ldp);
  SB_LAUNCH_CHECK("sb_layernorm");
  return SB_OK;
}

extern "C" int sb_add_rows(const void* a, int a_dtype, long long lda, const void* pos, int pos_dtype, long long ldpos,
                           int period, float sign, int rows, int D, void* out, long long ldo, void* stream) {
  if (!a || !pos || !out || rows < 1 || D < 1 || period < 1) return record_error(SB_EINVAL, "sb_add_rows: arguments");
  add_rows_kernel<<<blocks_for((long long)rows * D, 256), 256, 0, (cudaStream_t)stream>>>(
      a, a_dtype == SB_F32, lda, pos, pos_dtype == SB_F32, ldpos, period, sign, rows, D, static_cast<__half*>(out), ldo);
  SB_LAUNCH_CHECK("sb_add_rows");
  return SB_OK;
}

extern "C" int sb_dwconv3x3(const void* x, long long ldx, long long imgx, int B, int H, int W, int C, const float* w,
                            const float* bias, int relu, void* y, long long ldy, long long imgy, void* stream) {
  if (!x || !w || !bias || !y || B < 1 || H < 1 || W < 1 || C < 8 || C % 8 != 0 || ldx % 8 != 0 || ldy % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15))
    return record_error(SB_EINVAL, "sb_dwconv3x3: arguments (C, ld multiples of 8, 16-byte aligned)");
  if ((long long)W * (C / 8) > (1ll << 30) || H > 65535 || B > 65535 || (reinterpret_cast<uintptr_t>(w) & 15) ||
      (reinterpret_cast<uintptr_t>(bias) & 15))
    return record_error(SB_EINVAL, "sb_dwconv3x3: sizes (H, B <= 65535) or unaligned weights");
  dwconv3x3_kernel<<<dim3(blocks_for((long long)((W + kDwCols - 1) / kDwCols) * (C / 8), 256), H, B), 256, 0,
                     (cudaStream_t)stream>>>(
      static_cast<const __half*>(x), ldx, imgx, H, W, C, w, bias, relu, static_cast<__half*>(y), ldy, imgy);
  SB_LAUNCH_CHECK("sb_dwconv3x3");
  return SB_OK;
}

extern "C" int sb_upsample2x(const void* x, long long ldx, long long imgx, int B, int H, int W, int C, void* y,
                             long long ldy, long long imgy, void* stream) {
  if (!x || !y || B < 1 || H < 1 || W < 1 || C < 8 || C % 8 != 0 || ldx % 8 != 0 || ldy % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 15))
    return record_error(SB_EINVAL, "sb_upsample2x: arguments");
  if ((long long)2 * W * (C / 8) > (1ll << 30) || 2 * H > 65535 || B > 65535)
    return record_error(SB_EINVAL, "sb_upsample2x: sizes");
  upsample2x_kernel<<<dim3(blocks_for((long long)2 * W * (C / 8), 256), 2 * H, B), 256, 0, (cudaStream_t)stream>>>(
      static_cast<const __half*>(x), ldx, imgx, W, C, static_cast<__half*>(y), ldy, imgy);
  SB_LAUNCH_CHECK("sb_upsample2x");
  return SB_OK;
}

extern "C" int sb_topk_rows(const void* logits, long long ld, long long img, int B, int S, int C, const void* valid,
                            int K, void* idx, long long ldi, void* stream) {
  if (!logits || !idx || B < 1 || S < 1 || S > kTopkMaxRows || C < 1 || K < 1 || K > kTopkMaxK || K > S)
    return record_error(SB_EINVAL, "sb_topk_rows: arguments (S <= 65536, K <= 1024, K <= S)");
  const int smem = ((S * 2 + 15) & ~15) + kTopkMaxK * 8;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    if (cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024) != cudaSuccess)
      return record_error(SB_ECUDA, "sb_topk_rows: shared memory attribute");
    attr_set[dev & 63] = true;
  }
  topk_kernel<<<B, kTopkThreads, smem, (cudaStream_t)stream>>>(static_cast<const __half*>(logits), ld, img, S, C,
                                                              static_cast<const uint8_t*>(valid), K,
                                                              static_cast<int32_t*>(idx), ldi);
  SB_LAUNCH_CHECK("sb_topk_rows");
  return SB_OK;
}

extern "C" int sb_gather_rows(const void* src, int src_dtype, long long lds, long long imgs, int S, const void* idx,
                              long long ldi, int B, int K, int D, float* o32, long long ld32, long long img32, void* o16,
                              long long ld16, long long img16, void* stream) {
  if (!src || !idx || B < 1 || K < 1 || D < 1 || S < 1 || S > imgs || (!o32 && !o16))
    return record_error(SB_EINVAL, "sb_gather_rows: arguments");
  gather_rows_kernel<<<blocks_for((long long)B * K * D, 256), 256, 0, (cudaStream_t)stream>>>(
      src, src_dtype == SB_F32, lds, imgs, S, static_cast<const int32_t*>(idx), ldi, B, K, D, o32, ld32, img32,
      static_cast<__half*>(o16), ld16, img16);
  SB_LAUNCH_CHECK("sb_gather_rows");
  return SB_OK;
}

extern "C" int sb_deform_sample(const void* value, long long ldv, long long imgv, const int* level_hw, int L,
                                const void* off, long long ldoff, long long imgoff, const void* att, long long ldatt,
                                long long imgatt, const void* ref, int ref_dtype, long long ldref, long long imgref,
                                int B, int Q, int H, int P, void* out, long long ldo, long long imgo, void* stream) {
  if (!value || !level_hw || !off || !att || !ref || !out || L < 1 || L > kMaxLevels || B < 1 || Q < 1 || H < 1 ||
      P < 1 || L * P > 32)
    return record_error(SB_EINVAL, "sb_deform_sample: arguments (L * P <= 32)");
  DeformSampleArgs a{};
  a.value = static_cast<const __half*>(value);
  a.ldv = ldv;
  a.imgv = imgv;
  a.off = static_cast<const __half*>(off);
  a.ldoff = ldoff;
  a.imgoff = imgoff;
  a.att = static_cast<const __half*>(att);
  a.ldatt = ldatt;
  a.imgatt = imgatt;
  a.ref = ref;
  a.ref_f32 = ref_dtype == SB_F32;
  a.ldref = ldref;
  a.imgref = imgref;
  a.out = static_cast<__half*>(out);
  a.ldo = ldo;
  a.imgo = imgo;
  a.B = B;
  a.Q = Q;
  a.H = H;
  a.L = L;
  a.P = P;
  long long start = 0;
  for (int l = 0; l < L; ++l) {
    if (level_hw[2 * l] < 1 || level_hw[2 * l + 1] < 1) return record_error(SB_EINVAL, "sb_deform_sample: level size");
    a.lh[l] = level_hw[2 * l];
    a.lw[l] = level_hw[2 * l + 1];
    a.lstart[l] = (int)start;
    start += (long long)a.lh[l] * a.lw[l];
  }
  if (start > imgv) return record_error(SB_EINVAL, "sb_deform_sample: levels exceed the value rows of an image");
  deform_sample_kernel<<<blocks_for((long long)B * Q * H * 32, 256), 256, 0, (cudaStream_t)stream>>>(a);
  SB_LAUNCH_CHECK("sb_deform_sample");
  return SB_OK;
}

extern "C" int sb_box_enc(const void* encbox, long long ldb, const void* anchors, int S, const void* idx, int B, int K,
                          void* ref16, void* qin, long long ldq, void* stream) {
  if (!encbox || !anchors || !idx || !ref16 || !qin || B < 1 || K < 1 || S < 1)
    return record_error(SB_EINVAL, "sb_box_enc: arguments");
  box_enc_kernel<<<blocks_for((long long)B * K * 4, 256), 256, 0, (cudaStream_t)stream>>>(
      static_cast<const __half*>(encbox), ldb, static_cast<const __half*>(anchors), S,
      static_cast<const int32_t*>(idx), B, K, static_cast<__half*>(ref16), static_cast<__half*>(qin), ldq);
  SB_LAUNCH_CHECK("sb_box_enc");
  return SB_OK;
}

extern "C" int sb_box_dec(int first, const void* prebox, long long ldp, const void* ref16, const void* head,
                          long long ldh, void* corners, long long ldc, int R1, const float* project, float reg_scale,
                          float* ref_init, float* box, void* qin, long long ldq, int rows, void* stream) {
  if (!head || !corners || !project || !ref_init || !box || rows < 1 || R1 < 2 || (first && (!prebox || !ref16)))
    return record_error(SB_EINVAL, "sb_box_dec: arguments");
  // four threads per row, rows never straddle a warp (256 threads = 64 rows per block)
  auto kern = R1 == 33 ? box_dec_kernel<33> : box_dec_kernel<0>;  // 33 bins: reg_max = 32, the config default
  kern<<<blocks_for((long long)rows * 4, 256), 256, 0, (cudaStream_t)stream>>>(
      first, static_cast<const __half*>(prebox), ldp, static_cast<const __half*>(ref16),
      static_cast<const __half*>(head), ldh, static_cast<__half*>(corners), ldc, R1, project, reg_scale, ref_init, box,
      static_cast<__half*>(qin), ldq, rows);
  SB_LAUNCH_CHECK("sb_box_dec");
  return SB_OK;
}

extern "C" int sb_l2norm_rows(const void* x, long long ldx, int rows, int D, float* out, long long ldo, void* stream) {
  if (!x || !out || rows < 1 || D < 1) return record_error(SB_EINVAL, "sb_l2norm_rows: arguments");
  l2norm_rows_kernel<<<blocks_for((long long)rows * 32, 256), 256, 0, (cudaStream_t)stream>>>(
      static_cast<const __half*>(x), ldx, rows, D, out, ldo);
  SB_LAUNCH_CHECK("sb_l2norm_rows");
  return SB_OK;
}
