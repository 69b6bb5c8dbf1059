// sb_boxes.cu -- track-steered block masks: which blocks the predicted track boxes touch.
//
// Reference: Bahrombekk/Sarbon sarbon/inference/video.py:26-34 (`boxes_to_block_mask`) and
// its caller `SarbonVideo._steer` (video.py:139-147), which turns every camera's predicted
// track boxes into the `extra` mask of the next step.  A box (x0, y0, x1, y1), in engine
// pixels, marks the blocks
//     rows  max(0, floor(y0 / block) - margin) .. min(hb - 1, floor(y1 / block) + margin)
//     cols  max(0, floor(x0 / block) - margin) .. min(wb - 1, floor(x1 / block) + margin)
// when both ranges are non-empty.  The reference loops over boxes on the host and uploads
// the stacked mask; here the boxes (32 bytes each) go up and one launch writes the masks of
// all cameras, typically straight into the engine's `extra` mask.
//
// One CTA column per camera: each CTA stages its camera's boxes as integer block
// rectangles in shared memory, 256 at a time, and each thread ORs them for one block, so
// every output byte is written once.  floor(x / block) is exact (corrected after the
// division), as Python's and numpy's floor division of a float by an int are, so the masks
// equal the reference's bit for bit.
#include <string>

#include "sb_internal.cuh"

namespace sb {
namespace {

constexpr int kBoxChunk = 256;

struct BoxArgs {
  const double* boxes;  // [n_boxes][4] xyxy, engine pixels
  const int* offsets;   // [n + 1]: the boxes of camera c are rows offsets[c] .. offsets[c + 1] - 1
  uint8_t* out;         // [n][hb][wb]
  int n_boxes, hb, wb, block, margin;
};

// floor(x / b) for finite x and b > 0, exact: the rounded quotient is off by at most one,
// and q * b is exact while |q| < 2^53 / b; beyond that the caller clamps the result anyway.
__device__ __forceinline__ double floor_div(double x, int b) {
  const double bd = (double)b;
  double q = floor(x / bd);
  if (q * bd > x) q -= 1.0;
  else if ((q + 1.0) * bd <= x) q += 1.0;
  return q;
}

__global__ void __launch_bounds__(256) boxes_kernel(const BoxArgs a) {
  __shared__ int4 rect[kBoxChunk];  // (r0, r1, c0, c1), empty when r0 > r1 or c0 > c1
  const int cam = blockIdx.y;
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  const int begin = max(0, min(a.offsets[cam], a.n_boxes));
  const int end = max(begin, min(a.offsets[cam + 1], a.n_boxes));
  const int by = q / a.wb, bx = q - by * a.wb;
  uint32_t hit = 0;
  for (int c0 = begin; c0 < end; c0 += kBoxChunk) {
    const int nb = min(kBoxChunk, end - c0);
    if ((int)threadIdx.x < nb) {
      const double* b = a.boxes + 4 * (size_t)(c0 + threadIdx.x);
      const double x0 = b[0], y0 = b[1], x1 = b[2], y1 = b[3];
      int4 r = make_int4(1, 0, 1, 0);
      if (isfinite(x0) && isfinite(y0) && isfinite(x1) && isfinite(y1)) {
        // clamped in double first: a huge coordinate must not overflow the int conversion
        // and clamping to [0, wb] / [-1, wb - 1] keeps empty ranges empty
        const double m = (double)a.margin;
        r.x = (int)fmin(fmax(floor_div(y0, a.block) - m, 0.0), (double)a.hb);
        r.y = (int)fmax(fmin(floor_div(y1, a.block) + m, a.hb - 1.0), -1.0);
        r.z = (int)fmin(fmax(floor_div(x0, a.block) - m, 0.0), (double)a.wb);
        r.w = (int)fmax(fmin(floor_div(x1, a.block) + m, a.wb - 1.0), -1.0);
      }
      rect[threadIdx.x] = r;
    }
    __syncthreads();
    for (int i = 0; i < nb; ++i) {
      const int4 r = rect[i];
      hit |= (uint32_t)(by >= r.x && by <= r.y && bx >= r.z && bx <= r.w);
    }
    __syncthreads();
  }
  if (q < a.hb * a.wb) a.out[(size_t)cam * a.hb * a.wb + q] = hit ? 1 : 0;
}

}  // namespace
}  // namespace sb

using namespace sb;

extern "C" int sb_boxes_to_block_mask(const double* boxes_dev, const int* offsets_dev, int n_boxes, int n_cams,
                                      int hb, int wb, int block, int margin, uint8_t* out_dev, void* stream) {
  if (!offsets_dev || !out_dev || (n_boxes > 0 && !boxes_dev))
    return record_error(SB_EINVAL, "sb_boxes_to_block_mask: null pointer argument");
  if (n_boxes < 0) return record_error(SB_EINVAL, "sb_boxes_to_block_mask: negative n_boxes");
  if (n_cams <= 0 || n_cams > 65535)
    return record_error(SB_EINVAL, "sb_boxes_to_block_mask: n_cams must be in [1, 65535]");
  if (hb <= 0 || wb <= 0 || (long long)hb * wb > (1ll << 30))
    return record_error(SB_EINVAL, "sb_boxes_to_block_mask: hb and wb must be positive, hb * wb at most 2^30");
  if (block <= 0) return record_error(SB_EINVAL, "sb_boxes_to_block_mask: block must be positive");
  BoxArgs a{};
  a.boxes = boxes_dev;
  a.offsets = offsets_dev;
  a.out = out_dev;
  a.n_boxes = n_boxes;
  a.hb = hb;
  a.wb = wb;
  a.block = block;
  a.margin = margin;
  const int threads = 256;
  const dim3 grid((unsigned)(((long long)hb * wb + threads - 1) / threads), (unsigned)n_cams);
  boxes_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  cudaError_t rc = cudaGetLastError();
  if (rc != cudaSuccess)
    return record_error(SB_ECUDA, (std::string("sb_boxes_to_block_mask: launch: ") + cudaGetErrorString(rc)).c_str());
  return SB_OK;
}
