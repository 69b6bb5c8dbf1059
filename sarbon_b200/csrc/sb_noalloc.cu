// sb_noalloc.cu -- sb_block_lists_static: dilated block masks and ordered per-dilation
// block lists for a caller-supplied change mask, without an engine and without any
// device allocation.
//
// It runs the engine's list kernel (lists_kernel in sb_gate.cu: max-pool dilation as in
// fused_engine.py:151, ascending flat order as nonzero_static in :161-165) unchanged.
// Only the scratch that kernel needs -- the engine-state words it reads and writes
// (chunk ticket, look-back epoch, per-dilation counts, error flags) and the decoupled
// look-back status words -- comes from the file-scope __device__ array below instead
// of engine memory.  The array is sized for SB_STATIC_LISTS_MAX_BLOCKS blocks.
//
// Every call shares that one array, so calls must not overlap: two calls on different
// streams (or from different host threads) with no ordering between them race on it
// and corrupt each other's lists.  Each call clears the part it uses on its own stream
// before the list kernel runs.
#include <cstdio>
#include <mutex>
#include <string>

#include "sb_internal.cuh"

namespace sb {
namespace {

constexpr int kChunk = SB_LIST_CHUNK;  // blocks per list CTA
constexpr int kMaxBlocks = SB_STATIC_LISTS_MAX_BLOCKS;
constexpr int kMaxChunks = kMaxBlocks / kChunk;
constexpr size_t kStatusOffset = 256;
constexpr size_t kScratchBytes = kStatusOffset + (size_t)SB_MAX_DILATIONS * kMaxChunks * 8;
static_assert(kMaxBlocks % kChunk == 0, "the block limit is a whole number of list chunks");
static_assert(sizeof(State) <= kStatusOffset, "the State fits in front of the look-back words");
// 256 + 4 dilations x 1024 chunks x 8 bytes = 33,024 bytes (about 32 KB) on every device
static_assert(kScratchBytes == 33024, "static scratch size as documented");

// One State and the look-back words (SB_MAX_DILATIONS x SB_STATIC_LISTS_MAX_BLOCKS /
// SB_LIST_CHUNK x 8 bytes): [State | pad to 256 | status[n_dil][n_chunks]].
static __device__ __align__(256) unsigned char g_lists_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch[kMaxDevices] = {};
// look-back test hook (sb_debug_withhold_lookback with a NULL engine): 0 = none
int g_withhold = 0;          // list chunk + 1 that publishes no look-back words
unsigned g_spin_limit = 0;   // look-back polls before giving up (0 = SB_SPIN_LIMIT)

// Device address of g_lists_scratch on the current device, looked up once per device (the
// first call on it) and kept for the life of the process: after a cudaDeviceReset the
// cached address is stale, so the entry point must not be used across a device reset.
int scratch_ptr(unsigned char** out) {
  int dev = 0;
  cudaError_t rc = cudaGetDevice(&dev);
  if (rc != cudaSuccess)
    return record_error(SB_ECUDA, (std::string("sb_block_lists_static: cudaGetDevice: ") +
                                   cudaGetErrorString(rc)).c_str());
  if (dev < 0 || dev >= kMaxDevices) return record_error(SB_EINVAL, "sb_block_lists_static: device ordinal above 63");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch[dev]) {
    void* p = nullptr;
    rc = cudaGetSymbolAddress(&p, g_lists_scratch);
    if (rc != cudaSuccess || !p)
      return record_error(SB_ECUDA, (std::string("sb_block_lists_static: cudaGetSymbolAddress: ") +
                                     cudaGetErrorString(rc)).c_str());
    g_scratch[dev] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch[dev]);
  return SB_OK;
}

// Clears the State and the status words this call uses; epoch 1 tags this call's words.
__global__ void static_lists_clear_kernel(State* st, unsigned long long* status, int n_words, int withhold,
                                          unsigned spin_limit) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  for (int k = i; k < n_words; k += gridDim.x * blockDim.x) status[k] = 0ull;
  if (i == 0) {
    *st = State{};
    st->epoch = 1u;
    st->fallback = INT64_MAX;  // the list kernel's mode decision is not used here
    st->lb_withhold = withhold;
    st->lb_spin_limit = spin_limit;
  }
}

// counts_out[d] = active blocks at dilation d, or -1 for every d if a look-back wait gave up.
__global__ void static_lists_counts_kernel(const State* st, int32_t* counts_out, int n_dil) {
  const int d = threadIdx.x;
  if (d < n_dil) counts_out[d] = st->error ? -1 : st->counts[d];
}

}  // namespace

void static_lists_debug(int withhold_chunk, unsigned spin_limit) {
  std::lock_guard<std::mutex> lock(g_mu);
  g_withhold = withhold_chunk >= 0 ? withhold_chunk + 1 : 0;
  g_spin_limit = spin_limit;
}

}  // namespace sb

using namespace sb;

extern "C" int sb_block_lists_static(const uint8_t* changed_dev, int n_cams, int hb, int wb, const int* dilations,
                                     int n_dil, uint8_t* masks_dev, int32_t* lists_dev, int32_t* counts_dev,
                                     void* stream) {
  if (!changed_dev || !masks_dev || !lists_dev || !dilations)
    return record_error(SB_EINVAL, "sb_block_lists_static: null pointer argument");
  if (n_cams <= 0 || hb <= 0 || wb <= 0)
    return record_error(SB_EINVAL, "sb_block_lists_static: n_cams, hb and wb must be positive");
  if (n_dil < 1 || n_dil > SB_MAX_DILATIONS)
    return record_error(SB_EINVAL, "sb_block_lists_static: n_dil must be in [1, SB_MAX_DILATIONS]");
  for (int i = 0; i < n_dil; ++i)
    if (dilations[i] < 0) return record_error(SB_EINVAL, "sb_block_lists_static: negative dilation");
  const long long n_blocks = (long long)n_cams * hb * wb;
  if (n_blocks > kMaxBlocks) {
    char msg[200];
    std::snprintf(msg, sizeof msg,
                  "sb_block_lists_static: %lld blocks (n_cams*hb*wb) exceed the static scratch limit of %d "
                  "blocks (SB_STATIC_LISTS_MAX_BLOCKS)",
                  n_blocks, kMaxBlocks);
    return record_error(SB_EINVAL, msg);
  }
  // A dilation of max(hb, wb) already reaches every block of a camera; larger ones give the
  // same masks, so they are clamped (the kernel's window arithmetic stays far from overflow).
  int dil[SB_MAX_DILATIONS];
  for (int i = 0; i < n_dil; ++i) dil[i] = dilations[i] < (hb > wb ? hb : wb) ? dilations[i] : (hb > wb ? hb : wb);
  unsigned char* scratch = nullptr;
  if (int rc = scratch_ptr(&scratch)) return rc;
  int withhold;
  unsigned spin_limit;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    withhold = g_withhold;
    spin_limit = g_spin_limit;
  }
  State* st = reinterpret_cast<State*>(scratch);
  unsigned long long* status = reinterpret_cast<unsigned long long*>(scratch + kStatusOffset);
  const int n_chunks = (int)((n_blocks + kChunk - 1) / kChunk);
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  static_lists_clear_kernel<<<4, 1024, 0, s>>>(st, status, n_dil * n_chunks, withhold, spin_limit);
  ListArgs l{};
  l.changed = changed_dev;
  l.masks = masks_dev;
  l.lists = lists_dev;
  l.n_rk = 0;
  l.status = status;
  l.st = st;
  l.n_blocks = (int)n_blocks;
  l.hb = hb;
  l.wb = wb;
  l.n_dil = n_dil;
  for (int i = 0; i < n_dil; ++i) l.ds[i] = dil[i];
  cudaError_t rc = cudaGetLastError();
  if (rc == cudaSuccess) rc = launch_lists(l, n_chunks, s);
  if (rc == cudaSuccess && counts_dev) {
    static_lists_counts_kernel<<<1, 32, 0, s>>>(st, counts_dev, n_dil);
    rc = cudaGetLastError();
  }
  if (rc != cudaSuccess)
    return record_error(SB_ECUDA, (std::string("sb_block_lists_static: launch: ") + cudaGetErrorString(rc)).c_str());
  return SB_OK;
}
