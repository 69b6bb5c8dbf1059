// sb_prep.cu -- the caller's frame preparation for cameras whose size differs from the
// engine's: uint8 BGR frames at camera size -> RGB, bilinear resize to the engine size,
// (x - mean) / std in fp32, fp16 NHWC.
//
// Reference: Bahrombekk/Sarbon sarbon/inference/video.py:95-99 (`_prep`): BGR->RGB,
// float, F.interpolate(mode="bilinear", align_corners=False) when the camera size is not
// the engine size, then (x - MEAN) / STD; the engine step rounds it to fp16 (:105).
// PyTorch runs that as four passes over the frame (flip copy, float conversion,
// interpolation, normalisation) plus the fp16 conversion; here it is one kernel whose
// output the engine's gate reads.
//
// Resampling rule (align_corners=False, the half-pixel-centre rule of cv2.INTER_LINEAR):
// for output row h2 the source coordinate is max(0, scale * (h2 + 0.5) - 0.5) with scale =
// float32(in / out); its integer part h1 and fraction l pick rows h1 and min(h1 + 1,
// in - 1) with weights 1 - l and l; columns likewise.  Each output channel is
//   v = (1 - lh) * ((1 - lw) * p00 + lw * p01) + lh * ((1 - lw) * p10 + lw * p11)
// in fp32.  The products are contracted into fused multiply-adds as a compiler contracts
// `a * b + c * d` (the left product fused onto the rounded right one); a different
// contraction can move v by one fp32 ulp, which changes the fp16 result only when v sits
// at an fp16 rounding boundary.  Where an axis is not resized its fraction is exactly 0
// and v is the source value itself.
#include <cuda_fp16.h>

#include "sb_internal.cuh"

namespace sb {
namespace {

struct PrepArgs {
  const uint8_t* src;  // [n][hin][win][3] BGR
  __half* dst;         // [n][hout][wout][3] RGB, normalised
  int n, hin, win, hout, wout;
  float sh, sw;        // float32(hin / hout), float32(win / wout)
  float mean[3], stdv[3];
};

__device__ __forceinline__ void source_index(float scale, int dst, int in, int& i0, int& i1, float& l) {
  float r = __fmaf_rn(scale, (float)dst + 0.5f, -0.5f);
  if (r < 0.f) r = 0.f;
  i0 = (int)r;
  i1 = i0 + (i0 < in - 1 ? 1 : 0);
  l = __fsub_rn(r, (float)i0);
}

// One thread per output pixel (its three channels).
__global__ void __launch_bounds__(256) prep_resize_kernel(PrepArgs a) {
  const long long total = (long long)a.n * a.hout * a.wout;
  for (long long p = blockIdx.x * (long long)blockDim.x + threadIdx.x; p < total;
       p += (long long)gridDim.x * blockDim.x) {
    const int w2 = (int)(p % a.wout);
    const int h2 = (int)((p / a.wout) % a.hout);
    const int n = (int)(p / ((long long)a.wout * a.hout));
    int h0, h1, w0, w1;
    float lh, lw;
    source_index(a.sh, h2, a.hin, h0, h1, lh);
    source_index(a.sw, w2, a.win, w0, w1, lw);
    const float mh = __fsub_rn(1.f, lh), mw = __fsub_rn(1.f, lw);
    const uint8_t* row0 = a.src + ((size_t)n * a.hin + h0) * a.win * 3;
    const uint8_t* row1 = a.src + ((size_t)n * a.hin + h1) * a.win * 3;
    __half* out = a.dst + (size_t)p * 3;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const int sc = 2 - c;  // BGR source channel of RGB channel c
      const float p00 = row0[w0 * 3 + sc], p01 = row0[w1 * 3 + sc];
      const float p10 = row1[w0 * 3 + sc], p11 = row1[w1 * 3 + sc];
      const float top = __fmaf_rn(mw, p00, __fmul_rn(lw, p01));
      const float bot = __fmaf_rn(mw, p10, __fmul_rn(lw, p11));
      const float v = __fmaf_rn(mh, top, __fmul_rn(lh, bot));
      out[c] = __float2half_rn(__fdiv_rn(__fsub_rn(v, a.mean[c]), a.stdv[c]));
    }
  }
}

}  // namespace

cudaError_t launch_prep_resize(const uint8_t* src, int n, int hin, int win, __half* dst, int hout, int wout,
                               const float mean[3], const float stdv[3], int n_sms, cudaStream_t s) {
  PrepArgs a{};
  a.src = src;
  a.dst = dst;
  a.n = n;
  a.hin = hin;
  a.win = win;
  a.hout = hout;
  a.wout = wout;
  a.sh = (float)hin / (float)hout;
  a.sw = (float)win / (float)wout;
  for (int c = 0; c < 3; ++c) {
    a.mean[c] = mean[c];
    a.stdv[c] = stdv[c];
  }
  const long long total = (long long)n * hout * wout;
  long long blocks = (total + 255) / 256;
  const long long cap = (long long)n_sms * 8;
  if (blocks > cap) blocks = cap;
  prep_resize_kernel<<<(unsigned)blocks, 256, 0, s>>>(a);
  return cudaGetLastError();
}

}  // namespace sb
