// sb_engine.cu -- the C ABI (include/sarbon_sparse.h): engine object, device memory,
// tensor maps and the per-step launch sequence.
//
// Reference: Bahrombekk/Sarbon sarbon/sparse/fused_engine.py (FusedSparseEngine).  The
// reference captures a gate graph, syncs once per step to read the active count, then
// replays a sparse graph per budget bucket or a dense cuDNN graph.  Here the whole step
// is one stream-ordered sequence with the dispatch decided on the device:
//   gate -> lists (+ mode) -> dense img copy (no-op unless dense) -> conv x L -> finalize
// Every conv kernel reads the mode and its list length from device memory and runs a
// persistent grid, so there is no host sync inside a step.
#include <algorithm>
#include <cstddef>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <string>
#include <vector>

#include "sb_internal.cuh"
#include "sb_ptx.cuh"

using namespace sb;

namespace {

thread_local std::string g_err = "no error";

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

}  // namespace

// Error recording for entry points defined in other translation units.
int sb::record_error(int code, const char* msg) { return fail(code, msg); }

namespace {

#define SB_CUDA(call)                                                                  \
  do {                                                                                 \
    cudaError_t e_ = (call);                                                           \
    if (e_ != cudaSuccess)                                                             \
      return fail(SB_ECUDA, std::string(#call) + ": " + cudaGetErrorString(e_));       \
  } while (0)

std::vector<int> budget_buckets(int n_blocks, int unit = 16, double ratio = 1.15) {
  std::vector<int> out;
  int b = unit;
  while (b < n_blocks) {
    out.push_back(b);
    const int nb = (int)std::ceil(b * ratio / unit) * unit;
    b = std::max(b + unit, nb);
  }
  out.push_back((int)std::ceil((double)n_blocks / unit) * unit);
  return out;
}

__global__ void set_i64_kernel(int64_t* p, int64_t v) { *p = v; }
__global__ void set_i32_kernel(int32_t* p, int32_t v) { *p = v; }

}  // namespace

struct sb_engine {
  int dev = 0;
  int n = 0, h = 0, w = 0, block = 0, hb = 0, wb = 0, n_blocks = 0, dtype = SB_F16, esz = 2;
  double tau = 0.0;
  int refresh = 0;
  int64_t thr_fx = 0;
  double thr = 0.0;
  double band_lo = 0.0, band_hi = 0.0;
  int n_layers = 0;
  sb_layer_desc layers[SB_MAX_LAYERS];
  int nd = 0;
  int ds[SB_MAX_DILATIONS] = {};
  int layer_di[SB_MAX_LAYERS] = {};
  int layer_t[SB_MAX_LAYERS] = {};
  void* cache[SB_MAX_LAYERS + 1] = {};
  int64_t shape[SB_MAX_LAYERS + 1][4] = {};
  // e4m3 caches (SB_CREATE_FP8_S8): element bytes and activation scale of each cache
  // (value = code * scale), and per layer its e4m3 variant (0 fp16, 1 fp16 in / e4m3 out,
  // 2 e4m3 in and out) and the per-output-channel scales of its e4m3 weights
  int cache_esz[SB_MAX_LAYERS + 1] = {};
  bool cache_f8[SB_MAX_LAYERS + 1] = {};
  float act_scale[SB_MAX_LAYERS + 1] = {};
  int layer_q[SB_MAX_LAYERS] = {};
  std::vector<float> wscale[SB_MAX_LAYERS];
  uint8_t* changed = nullptr;
  uint8_t* extra = nullptr;
  uint8_t* masks = nullptr;
  int32_t* lists = nullptr;
  // region kinds (rw x rh blocks) of the window-mode layers and their ordered lists
  int n_rk = 0;
  int rk_w[SB_MAX_RKINDS] = {}, rk_h[SB_MAX_RKINDS] = {}, rk_cap[SB_MAX_RKINDS] = {};
  int32_t* rlists[SB_MAX_RKINDS] = {};
  int layer_mode[SB_MAX_LAYERS] = {};   // 0 im2col / gather, 1 row windows, 3 full windows; +8 CTA pairs
  int layer_rk[SB_MAX_LAYERS] = {};     // region kind of a window-mode layer (-1: blocks)
  unsigned long long* status = nullptr;
  int n_chunks = 0;
  State* st = nullptr;
  float* bias[SB_MAX_LAYERS] = {};
  float bias_h[SB_MAX_LAYERS][128] = {};  // host copy, passed by value to the fp16 conv kernels
  void* wdev[SB_MAX_LAYERS] = {};
  bool wok[SB_MAX_LAYERS] = {};
  CUtensorMap tmap[SB_MAX_LAYERS];
  CUtensorMap tmap_y[SB_MAX_LAYERS];  // destination cache (staged-output variants)
  bool has_tmap[SB_MAX_LAYERS] = {};
  int32_t* host_out = nullptr;      // mapped pinned: mode, count, error, written
  int32_t* host_out_dev = nullptr;
  int n_sms = 148;
  int last_launches = 0;
  // cell-level gating (0: block level): cell size, cell radius per dilation group, buffers
  int cell = 0;
  int cell_r[SB_MAX_DILATIONS] = {};
  int64_t cell_thr_fx = 0;
  uint8_t* cells = nullptr;   // [N][H/cell][W/cell], allocated by the first sb_set_cell_gating
  int cells_cell = 0;         // the cell size `cells` was allocated for
  uint8_t* cmasks = nullptr;  // [nd][N][Hb][Wb] block masks from the cells
  void* prep = nullptr;       // [N][H][W][3] fp16 frames resized from the camera size (first use)
  std::vector<void*> allocs;
  // CUDA graphs of the step's launch sequence, one per input (frames pointer, input kind,
  // camera size, normalisation): a step is then one graph launch instead of ~15 kernel
  // launches from the host.  Dropped when a host-side value baked into kernel arguments
  // changes (threshold, gating mode, weights).
  struct StepGraph {
    const void* frames;
    int kind, cam_h, cam_w;
    float mean[3], stdv[3];
    cudaGraphExec_t exec;
    int launches;
    uint64_t used;
  };
  bool graphs_on = true;
  std::vector<StepGraph> graphs;
  cudaStream_t cap_stream = nullptr;
  uint64_t graph_clock = 0;
  // optional timing: an event after every launch (sb_step_profiled) or only at the phase
  // boundaries gate | lists | copy | conv sequence | finalize (sb_step_phases)
  bool profiling = false;
  bool phases = false;
  std::vector<cudaEvent_t> events;
  int n_events = 0;
};

namespace {

// Record a timing event on `s` when profiling (one before the first launch and one
// after every launch of the step).
void mark(sb_engine* e, cudaStream_t s) {
  if (!e->profiling) return;
  if (e->n_events >= (int)e->events.size()) {
    cudaEvent_t ev;
    if (cudaEventCreate(&ev) != cudaSuccess) return;
    e->events.push_back(ev);
  }
  cudaEventRecord(e->events[e->n_events++], s);
}

void drop_graphs(sb_engine* e) {
  for (auto& g : e->graphs) cudaGraphExecDestroy(g.exec);
  e->graphs.clear();
}

constexpr size_t kMaxStepGraphs = 64;

// Runs a step's launch sequence `launch` on `s`: through the step graph of this input
// (captured on first use on the engine's capture stream and instantiated), or directly when
// graphs are off or a step is being timed launch by launch.
int run_step(sb_engine* e, const void* frames, int kind, int cam_h, int cam_w, const float* mean, const float* stdv,
             const std::function<int(cudaStream_t)>& launch, cudaStream_t s) {
  if (!e->graphs_on || e->profiling) return launch(s);
  float mv[3], sv[3];
  for (int c = 0; c < 3; ++c) {
    mv[c] = mean ? mean[c] : 0.f;
    sv[c] = stdv ? stdv[c] : 1.f;
  }
  sb_engine::StepGraph* hit = nullptr;
  for (auto& g : e->graphs)
    if (g.frames == frames && g.kind == kind && g.cam_h == cam_h && g.cam_w == cam_w &&
        std::memcmp(g.mean, mv, sizeof mv) == 0 && std::memcmp(g.stdv, sv, sizeof sv) == 0)
      hit = &g;
  if (!hit) {
    if (!e->cap_stream) SB_CUDA(cudaStreamCreateWithFlags(&e->cap_stream, cudaStreamNonBlocking));
    SB_CUDA(cudaStreamBeginCapture(e->cap_stream, cudaStreamCaptureModeRelaxed));
    const int rc = launch(e->cap_stream);
    cudaGraph_t graph = nullptr;
    const cudaError_t ce = cudaStreamEndCapture(e->cap_stream, &graph);
    if (rc) {
      if (graph) cudaGraphDestroy(graph);
      return rc;
    }
    if (ce != cudaSuccess || !graph)
      return fail(SB_ECUDA, std::string("step graph capture: ") + cudaGetErrorString(ce));
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) return fail(SB_ECUDA, std::string("step graph instantiate: ") + cudaGetErrorString(ie));
    if (e->graphs.size() >= kMaxStepGraphs) {  // the least recently used input goes
      size_t lru = 0;
      for (size_t i = 1; i < e->graphs.size(); ++i)
        if (e->graphs[i].used < e->graphs[lru].used) lru = i;
      cudaGraphExecDestroy(e->graphs[lru].exec);
      e->graphs.erase(e->graphs.begin() + (long)lru);
    }
    sb_engine::StepGraph g{};
    g.frames = frames;
    g.kind = kind;
    g.cam_h = cam_h;
    g.cam_w = cam_w;
    std::memcpy(g.mean, mv, sizeof mv);
    std::memcpy(g.stdv, sv, sizeof sv);
    g.exec = exec;
    g.launches = e->last_launches;
    e->graphs.push_back(g);
    hit = &e->graphs.back();
  }
  hit->used = ++e->graph_clock;
  SB_CUDA(cudaGraphLaunch(hit->exec, s));
  e->last_launches = hit->launches;
  return SB_OK;
}

int alloc_dev(sb_engine* e, void** p, size_t bytes) {
  if (cudaMalloc(p, bytes) != cudaSuccess) return fail(SB_ENOMEM, "cudaMalloc failed");
  e->allocs.push_back(*p);
  if (cudaMemset(*p, 0, bytes) != cudaSuccess) return fail(SB_ECUDA, "cudaMemset failed");
  return SB_OK;
}

// floor(float32(tau * side^2 * 3) * 2^24): the gate threshold of a side x side area as an
// exact fixed-point value (-1: every area changes, INT64_MAX: none does)
int64_t threshold_fx(double tau, int side) {
  const float thr32 = (float)(tau * side * side * 3);
  if (std::isnan(thr32)) return INT64_MAX;
  if (thr32 < 0.f) return -1;
  if (std::isinf(thr32) || (double)thr32 * 16777216.0 >= 9.0e18) return INT64_MAX;
  return (int64_t)std::floor((double)thr32 * 16777216.0);
}

// Gate threshold from tau: float32(tau * block * block * 3), compared as torch does
// (fused_engine.py:144), as an exact fixed-point value and as the fp32 rounding band.
void set_threshold(sb_engine* e, double tau) {
  e->tau = tau;
  const float thr32 = (float)(tau * e->block * e->block * 3);
  e->thr = (double)thr32;
  e->thr_fx = threshold_fx(tau, e->block);
  if (e->cell) e->cell_thr_fx = threshold_fx(tau, e->cell);
  if (std::isnan(thr32)) e->thr = INFINITY;  // sum > NaN is false for every block
  // A recursive fp32 sum of n non-negative fp16 terms is within (n-1)*2^-24 relative of the
  // exact sum (any order); twice that margin decides the comparison from the fp32 sum.
  const double gam = 2.0 * 3.0 * e->block * e->block * std::ldexp(1.0, -24);
  if (std::isnan(thr32) || std::isinf(thr32) && thr32 > 0) {
    e->band_lo = e->band_hi = INFINITY;                // only inf / NaN sums reach the exact path
  } else if (thr32 < 0.f) {
    e->band_lo = e->band_hi = -1.0;                    // every block changes
  } else {
    e->band_lo = (double)thr32 * (1.0 - gam);
    e->band_hi = (double)thr32 * (1.0 + gam);
  }
}

int launch_convs(sb_engine* e, cudaStream_t s, int first = 0, int last = -1) {
  if (last < 0) last = e->n_layers - 1;
  for (int i = first; i <= last; ++i) {
    const sb_layer_desc& L = e->layers[i];
    if (!e->wok[i]) return fail(SB_EINVAL, "weights of layer " + std::to_string(i) + " not uploaded");
    ConvArgs a{};
    a.x = e->cache[L.src];
    a.y = e->cache[i + 1];
    a.res = L.res >= 0 ? e->cache[L.res] : nullptr;
    a.bias = e->bias[i];
    std::memcpy(a.bias_v, e->bias_h[i], sizeof(a.bias_v));
    const int q = e->layer_q[i];
    for (int c = 0; c < 128; ++c)
      a.dq_v[c] = q >= 2 && c < L.cout ? e->act_scale[L.src] * e->wscale[i][c] : 1.f;
    a.res_scale = L.res >= 0 && e->cache_f8[L.res] ? e->act_scale[L.res] : 1.f;
    a.out_inv_scale = e->cache_f8[i + 1] ? 1.f / e->act_scale[i + 1] : 1.f;
    a.wimg = e->wdev[i];
    const int di = e->layer_di[i];
    a.lcam = e->lists + (size_t)di * 3 * e->n_blocks;
    a.lby = a.lcam + e->n_blocks;
    a.lbx = a.lby + e->n_blocks;
    a.st = e->st;
    a.d_idx = di;
    a.n = e->n;
    a.hx = (int)e->shape[L.src][1];
    a.wx = (int)e->shape[L.src][2];
    a.cin = L.cin;
    a.ho = (int)e->shape[i + 1][1];
    a.wo = (int)e->shape[i + 1][2];
    a.cout = L.cout;
    a.hb = e->hb;
    a.wb = e->wb;
    a.n_blocks = e->n_blocks;
    a.t = e->layer_t[i];
    a.s = L.stride;
    a.act = L.act;
    const int rk = e->layer_rk[i];
    a.rkind = rk;
    a.rw = rk >= 0 ? e->rk_w[rk] : 1;
    a.rh = rk >= 0 ? e->rk_h[rk] : 1;
    if (rk >= 0) {
      a.rcam = e->rlists[rk] + (size_t)di * 3 * e->rk_cap[rk];
      a.rry = a.rcam + e->rk_cap[rk];
      a.rrx = a.rry + e->rk_cap[rk];
    } else {  // window layers with one-block regions iterate over the block lists
      a.rcam = a.lcam;
      a.rry = a.lby;
      a.rrx = a.lbx;
    }
    cudaError_t err;
    if (e->dtype == SB_F16) {
      err = launch_conv_tc(a, e->layer_mode[i], e->has_tmap[i] ? &e->tmap[i] : nullptr,
                           e->has_tmap[i] ? &e->tmap_y[i] : nullptr, e->n_sms, s, q);
    } else {
      err = launch_conv_simt(a, e->n_sms * 4, s);
    }
    if (err != cudaSuccess)
      return fail(SB_ECUDA, "conv launch (layer " + std::to_string(i) + "): " + cudaGetErrorString(err));
    e->last_launches += 1;
    if (!e->phases) mark(e, s);
  }
  if (e->phases) mark(e, s);  // the conv sequence as one interval: PDL stays on between layers
  return SB_OK;
}

int check_frames(sb_engine* e, const void* p) {
  if (!p) return fail(SB_EINVAL, "frames pointer is NULL");
  if (reinterpret_cast<uintptr_t>(p) % 16) return fail(SB_EINVAL, "frames must be 16-byte aligned");
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess || attr.type != cudaMemoryTypeDevice)
    return fail(SB_EINVAL, "frames must be device memory");
  return SB_OK;
}

// Every launch of one step on `s` (no host sync).
int launch_step(sb_engine* e, const void* frames, int kind, const float* mean, const float* stdv, cudaStream_t s) {
  int rc;
  e->last_launches = 0;
  GateArgs g{};
  g.frames = frames;
  g.img = e->cache[0];
  g.extra = e->extra;
  g.changed = e->changed;
  g.st = e->st;
  g.n = e->n;
  g.h = e->h;
  g.w = e->w;
  g.hb = e->hb;
  g.wb = e->wb;
  g.block = e->block;
  g.thr_fx = e->thr_fx;
  g.thr = e->thr;
  g.band_lo = e->band_lo;
  g.band_hi = e->band_hi;
  g.refresh = e->refresh;
  for (int c = 0; c < 3; ++c) {
    g.mean[c] = mean ? mean[c] : 0.f;
    g.stdv[c] = stdv ? stdv[c] : 1.f;
  }
  mark(e, s);
  if (e->cell) {
    if (kind != 0) return fail(SB_EINVAL, "cell-level gating needs fp16 frames (sb_step on an fp16 engine)");
    CellGateArgs cg{};
    cg.frames = frames;
    cg.img = e->cache[0];
    cg.extra = e->extra;
    cg.changed = e->changed;
    cg.cells = e->cells;
    cg.st = e->st;
    cg.n = e->n;
    cg.h = e->h;
    cg.w = e->w;
    cg.hb = e->hb;
    cg.wb = e->wb;
    cg.block = e->block;
    cg.cell = e->cell;
    cg.k = e->block / e->cell;
    cg.hc = e->h / e->cell;
    cg.wc = e->w / e->cell;
    cg.thr_fx = e->cell_thr_fx;
    cg.refresh = e->refresh;
    SB_CUDA(launch_cell_gate(cg, s));
    // the block masks of every dilation group from the cells; the lists kernel then takes
    // them as they are (dilation 0).  Timed with the gate when profiling.
    SB_CUDA(launch_cell_masks(e->cells, e->n, cg.hc, cg.wc, cg.k, e->cell_r, e->nd, e->cmasks, s));
  } else {
    SB_CUDA(launch_gate(g, kind, s));
  }
  mark(e, s);
  ListArgs l{};
  l.changed = e->changed;
  l.masks = e->masks;
  l.lists = e->lists;
  l.n_rk = e->n_rk;
  for (int k = 0; k < e->n_rk; ++k) {
    l.rw[k] = e->rk_w[k];
    l.rh[k] = e->rk_h[k];
    l.rlists[k] = e->rlists[k];
  }
  l.status = e->status;
  l.st = e->st;
  l.n_blocks = e->n_blocks;
  l.hb = e->hb;
  l.wb = e->wb;
  l.n_dil = e->nd;
  for (int i = 0; i < e->nd; ++i) {
    l.ds[i] = e->cell ? 0 : e->ds[i];
    l.src[i] = e->cell ? e->cmasks + (size_t)i * e->n_blocks : nullptr;
  }
  SB_CUDA(launch_lists(l, e->n_chunks, s));
  mark(e, s);
  CopyArgs c{};
  c.frames = frames;
  c.img = e->cache[0];
  c.changed = nullptr;
  c.st = e->st;
  c.n = e->n;
  c.h = e->h;
  c.w = e->w;
  c.hb = e->hb;
  c.wb = e->wb;
  c.block = e->block;
  c.elem_bytes = e->esz;
  c.u8 = kind == 2;
  for (int k = 0; k < 3; ++k) {
    c.mean[k] = g.mean[k];
    c.stdv[k] = g.stdv[k];
  }
  SB_CUDA(launch_copy(c, s));
  mark(e, s);
  e->last_launches = e->cell ? 4 : 3;
  rc = launch_convs(e, s);
  if (rc) return rc;
  SB_CUDA(launch_finalize(e->st, e->refresh, e->host_out_dev, s));
  mark(e, s);
  e->last_launches += 1;
  return SB_OK;
}

// Reads the step's {mode, count} after a stream sync when the caller asked for them.
int finish_step(sb_engine* e, cudaStream_t s, int* mode_out, int64_t* count_out) {
  if (mode_out || count_out) {
    SB_CUDA(cudaStreamSynchronize(s));
    volatile int32_t* ho = e->host_out;
    if (mode_out) *mode_out = ho[0];
    if (count_out) *count_out = ho[1];
    if (ho[2] & (SB_ERR_TIMEOUT_FULL | SB_ERR_TIMEOUT_EMPTY | SB_ERR_TIMEOUT_ACC | SB_ERR_TIMEOUT_LOOKBK |
                 SB_ERR_TIMEOUT_WGT))
      return fail(SB_ETIMEOUT, "a bounded device wait gave up (error flags " + std::to_string(ho[2]) + ")");
    if (ho[2]) return fail(SB_ECUDA, "device error flags " + std::to_string(ho[2]));
  }
  return SB_OK;
}

int step_impl(sb_engine* e, const void* frames, int kind, const float* mean, const float* stdv,
              cudaStream_t s, int* mode_out, int64_t* count_out) {
  int rc = check_frames(e, frames);
  if (rc) return rc;
  SB_CUDA(cudaSetDevice(e->dev));
  rc = run_step(e, frames, kind, e->h, e->w, mean, stdv,
                [&](cudaStream_t st) { return launch_step(e, frames, kind, mean, stdv, st); }, s);
  if (rc) return rc;
  return finish_step(e, s, mode_out, count_out);
}

int dense_impl(sb_engine* e, const void* frames, int reset, cudaStream_t s) {
  int rc = check_frames(e, frames);
  if (rc) return rc;
  SB_CUDA(cudaSetDevice(e->dev));
  SB_CUDA(launch_set_mode(e->st, SB_MODE_DENSE, reset, 0, s));
  CopyArgs c{};
  c.frames = frames;
  c.img = e->cache[0];
  c.st = e->st;
  c.n = e->n;
  c.h = e->h;
  c.w = e->w;
  c.hb = e->hb;
  c.wb = e->wb;
  c.block = e->block;
  c.elem_bytes = e->esz;
  SB_CUDA(launch_copy(c, s));
  e->last_launches = 2;
  return launch_convs(e, s);
}

}  // namespace

extern "C" {

const char* sb_last_error(void) { return g_err.c_str(); }

const char* sb_version(void) { return "sarbon_b200 0.1 sm_100a (tcgen05 fp16 tile conv, fp32 simt)"; }

int sb_create(const sb_layer_desc* layers, int n_layers, int n_streams, int height, int width, int block,
              int dtype, double tau, int refresh, int dense_check_every, sb_engine** out) {
  return sb_create_ex(layers, n_layers, n_streams, height, width, block, dtype, tau, refresh, dense_check_every, 0,
                      out);
}

int sb_create_ex(const sb_layer_desc* layers, int n_layers, int n_streams, int height, int width, int block,
                 int dtype, double tau, int refresh, int dense_check_every, int flags, sb_engine** out) {
  if (!out || !layers) return fail(SB_EINVAL, "null argument");
  if (flags & ~(SB_CREATE_BLOCK_UNITS | SB_CREATE_FP8_S8 | SB_CREATE_FP8_S4))
    return fail(SB_EINVAL, "unknown creation flags");
  if ((flags & (SB_CREATE_FP8_S8 | SB_CREATE_FP8_S4)) && (dtype != SB_F16 || (flags & SB_CREATE_BLOCK_UNITS)))
    return fail(SB_EINVAL, "e4m3 caches need an fp16 engine without block units");
  *out = nullptr;
  if (n_layers < 1 || n_layers > SB_MAX_LAYERS) return fail(SB_EINVAL, "n_layers out of range");
  if (n_streams < 1 || height < 1 || width < 1) return fail(SB_EINVAL, "bad frame geometry");
  if (block < 16 || block % 16) return fail(SB_EINVAL, "block must be a multiple of 16");
  if (height % block || width % block) return fail(SB_EINVAL, "height and width must be divisible by block");
  if (dtype != SB_F16 && dtype != SB_F32) return fail(SB_EINVAL, "dtype must be SB_F16 or SB_F32");
  if (refresh < 0) return fail(SB_EINVAL, "refresh must be >= 0");
  sb_engine* e = new sb_engine();
  auto bail = [&](int code) {
    sb_destroy(e);
    return code;
  };
  if (cudaGetDevice(&e->dev) != cudaSuccess) {
    delete e;
    return fail(SB_ECUDA, "no CUDA device");
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, e->dev) != cudaSuccess) return bail(fail(SB_ECUDA, "device query failed"));
  e->n_sms = prop.multiProcessorCount;
  e->n = n_streams;
  e->h = height;
  e->w = width;
  e->block = block;
  e->hb = height / block;
  e->wb = width / block;
  e->n_blocks = n_streams * e->hb * e->wb;
  e->dtype = dtype;
  e->esz = dtype == SB_F16 ? 2 : 4;
  e->tau = tau;
  e->refresh = refresh;
  e->n_layers = n_layers;
  set_threshold(e, tau);
  // caches: id 0 = image, id i+1 = layer i output
  e->shape[0][0] = n_streams;
  e->shape[0][1] = height;
  e->shape[0][2] = width;
  e->shape[0][3] = 3;
  std::vector<int> dl;
  for (int i = 0; i < n_layers; ++i) {
    const sb_layer_desc& L = layers[i];
    e->layers[i] = L;
    if (L.src < 0 || L.src > i) return bail(fail(SB_EINVAL, "layer " + std::to_string(i) + ": bad src id"));
    if (L.res >= i + 1 || L.res < -1) return bail(fail(SB_EINVAL, "layer " + std::to_string(i) + ": bad res id"));
    if (L.stride != 1 && L.stride != 2) return bail(fail(SB_EINVAL, "conv stride must be 1 or 2"));
    if (L.out_stride < 1 || block % L.out_stride || height % L.out_stride || width % L.out_stride)
      return bail(fail(SB_EINVAL, "out_stride must divide block, height and width"));
    if (e->shape[L.src][3] != L.cin) return bail(fail(SB_EINVAL, "layer " + std::to_string(i) + ": cin mismatch"));
    const int in_stride = L.src == 0 ? 1 : layers[L.src - 1].out_stride;
    if (in_stride * L.stride != L.out_stride)
      return bail(fail(SB_EINVAL, "layer " + std::to_string(i) + ": stride chain mismatch"));
    e->shape[i + 1][0] = n_streams;
    e->shape[i + 1][1] = height / L.out_stride;
    e->shape[i + 1][2] = width / L.out_stride;
    e->shape[i + 1][3] = L.cout;
    if (L.res >= 0 && (e->shape[L.res][3] != L.cout || e->shape[L.res][1] != e->shape[i + 1][1]))
      return bail(fail(SB_EINVAL, "layer " + std::to_string(i) + ": residual shape mismatch"));
    e->layer_t[i] = block / L.out_stride;
    if (dtype == SB_F16 && !conv_tc_supported(L.cin, L.cout, e->layer_t[i], L.stride))
      return bail(fail(SB_EINVAL, "layer " + std::to_string(i) + ": no tcgen05 kernel for cin=" +
                                      std::to_string(L.cin) + " cout=" + std::to_string(L.cout) +
                                      " tile=" + std::to_string(e->layer_t[i]) + " stride=" +
                                      std::to_string(L.stride)));
    const int d = (L.radius + block - 1) / block;
    bool seen = false;
    for (int x : dl) seen |= x == d;
    if (!seen) dl.push_back(d);
  }
  std::sort(dl.begin(), dl.end());
  if ((int)dl.size() > SB_MAX_DILATIONS) return bail(fail(SB_EINVAL, "too many distinct dilations"));
  e->nd = (int)dl.size();
  for (int i = 0; i < e->nd; ++i) e->ds[i] = dl[i];
  for (int i = 0; i < n_layers; ++i) {
    const int d = (layers[i].radius + block - 1) / block;
    for (int j = 0; j < e->nd; ++j)
      if (e->ds[j] == d) e->layer_di[i] = j;
  }
  // element type of every cache: e4m3 for the outputs of the stride-8 stage when asked
  // the stride-4 stage's last cache (its output, p4) stays fp16
  int last_s4 = -1;
  for (int i = 0; i < n_layers; ++i)
    if (layers[i].out_stride == 4) last_s4 = i;
  for (int i = 0; i <= n_layers; ++i) {
    const int os = i > 0 ? layers[i - 1].out_stride : 1;
    e->cache_f8[i] = i > 0 && (((flags & SB_CREATE_FP8_S8) && os >= 8) ||
                               ((flags & SB_CREATE_FP8_S4) && os == 4 && i - 1 != last_s4));
    e->cache_esz[i] = e->cache_f8[i] ? 1 : e->esz;
    e->act_scale[i] = 1.f;
  }
  for (int i = 0; i < n_layers; ++i) {
    const sb_layer_desc& L = layers[i];
    const bool in8 = e->cache_f8[L.src], out8 = e->cache_f8[i + 1];
    e->layer_q[i] = in8 ? (out8 ? 2 : 3) : (out8 ? 1 : 0);
    if (L.res >= 0 && e->cache_f8[L.res] != in8)
      return bail(fail(SB_EINVAL, "layer " + std::to_string(i) + ": the residual's type differs from the input's"));
  }
  // device memory
  int rc;
  for (int i = 0; i <= n_layers; ++i) {
    const size_t bytes =
        (size_t)e->shape[i][0] * e->shape[i][1] * e->shape[i][2] * e->shape[i][3] * e->cache_esz[i];
    if ((rc = alloc_dev(e, &e->cache[i], bytes))) return bail(rc);
  }
  e->n_chunks = (e->n_blocks + SB_LIST_CHUNK - 1) / SB_LIST_CHUNK;
  if ((rc = alloc_dev(e, (void**)&e->changed, e->n_blocks))) return bail(rc);
  if ((rc = alloc_dev(e, (void**)&e->extra, e->n_blocks))) return bail(rc);
  if ((rc = alloc_dev(e, (void**)&e->masks, (size_t)e->nd * e->n_blocks))) return bail(rc);
  if ((rc = alloc_dev(e, (void**)&e->lists, (size_t)e->nd * 3 * e->n_blocks * 4))) return bail(rc);
  // window-mode layers: the region kind each one iterates over
  for (int i = 0; i < n_layers; ++i) {
    e->layer_rk[i] = -1;
    e->layer_mode[i] = dtype == SB_F16 ? conv_tc_pick_mode(layers[i].cin, layers[i].cout, e->layer_t[i],
                                                           layers[i].stride)
                                       : 0;
    if (dtype == SB_F16 && (flags & SB_CREATE_BLOCK_UNITS)) {
      const int t = e->layer_t[i], win = e->layer_mode[i] & 7;
      const bool one_block = win == 0 || (8 / t == 1 && (win != 3 || 16 / t == 1));
      if (!one_block) {
        const int m = conv_tc_block_mode(layers[i].cin, layers[i].cout, t, layers[i].stride);
        if (m < 0) return bail(fail(SB_EINVAL, "layer " + std::to_string(i) + ": no block-unit tile conv"));
        e->layer_mode[i] = m;
      }
    }
    if (e->layer_q[i]) {
      const int m = conv_tc_q_mode(layers[i].cin, layers[i].cout, e->layer_t[i], layers[i].stride, e->layer_q[i]);
      if (m < 0) return bail(fail(SB_EINVAL, "layer " + std::to_string(i) + ": no e4m3 tile conv for its shape"));
      e->layer_mode[i] = m;
    }
    const int win = e->layer_mode[i] & 7;  // bit 3: CTA pairs
    if (win == 0) continue;
    const int t = e->layer_t[i];
    const int rw = 8 / t, rh = win == 3 ? 16 / t : 1;
    if (rw == 1 && rh == 1) continue;  // a one-block region is a block: the layer uses the block lists
    int k = 0;
    while (k < e->n_rk && !(e->rk_w[k] == rw && e->rk_h[k] == rh)) ++k;
    if (k == e->n_rk) {
      if (k == SB_MAX_RKINDS) return bail(fail(SB_EINVAL, "too many region kinds"));
      e->rk_w[k] = rw;
      e->rk_h[k] = rh;
      e->rk_cap[k] = n_streams * ((e->hb + rh - 1) / rh) * ((e->wb + rw - 1) / rw);
      ++e->n_rk;
    }
    e->layer_rk[i] = k;
  }
  for (int k = 0; k < e->n_rk; ++k)
    if ((rc = alloc_dev(e, (void**)&e->rlists[k], (size_t)e->nd * 3 * e->rk_cap[k] * 4))) return bail(rc);
  if ((rc = alloc_dev(e, (void**)&e->status, (size_t)(1 + e->n_rk) * e->nd * e->n_chunks * 8))) return bail(rc);
  if ((rc = alloc_dev(e, (void**)&e->st, sizeof(State)))) return bail(rc);
  State init{};
  init.epoch = 1;
  // The reference warms its gate graph up once at construction (fused_engine.py:85,130-132),
  // which executes `tick += 1` (:147): its first gated step sees tick == 1.
  init.tick = 1;
  init.fallback = budget_buckets(e->n_blocks).back();
  init.check_every = dense_check_every;
  init.mode_cur = SB_MODE_SKIP;
  if (cudaMemcpy(e->st, &init, sizeof(State), cudaMemcpyHostToDevice) != cudaSuccess)
    return bail(fail(SB_ECUDA, "state upload failed"));
  if (cudaHostAlloc((void**)&e->host_out, 16, cudaHostAllocMapped) != cudaSuccess)
    return bail(fail(SB_ENOMEM, "pinned allocation failed"));
  std::memset(e->host_out, 0, 16);
  if (cudaHostGetDevicePointer((void**)&e->host_out_dev, e->host_out, 0) != cudaSuccess)
    return bail(fail(SB_ECUDA, "mapped pointer failed"));
  for (int i = 0; i < n_layers; ++i) {
    const sb_layer_desc& L = layers[i];
    if ((rc = alloc_dev(e, (void**)&e->bias[i], (size_t)L.cout * 4))) return bail(rc);
    const size_t wbytes = dtype == SB_F16 ? conv_tc_wimg_bytes(L.cin, L.cout, e->layer_t[i], L.stride, e->layer_mode[i],
                                                               e->layer_q[i])
                                          : (size_t)9 * L.cin * L.cout * 4;
    if ((rc = alloc_dev(e, &e->wdev[i], wbytes))) return bail(rc);
    if (dtype == SB_F16) {  // every fp16 layer loads its input by TMA (the first layer: window boxes)
      cudaError_t err = conv_tc_make_tmap(&e->tmap[i], e->cache[L.src], n_streams, (int)e->shape[L.src][1],
                                          (int)e->shape[L.src][2], L.cin, e->layer_t[i], L.stride,
                                          e->layer_mode[i], e->layer_q[i] >= 2 ? 2 : 0);
      if (err == cudaSuccess)
        err = conv_tc_make_tmap_out(&e->tmap_y[i], e->cache[i + 1], n_streams, (int)e->shape[i + 1][1],
                                    (int)e->shape[i + 1][2], L.cin, L.cout, e->layer_t[i], L.stride,
                                    e->layer_mode[i]);
      if (err != cudaSuccess) return bail(fail(SB_ECUDA, std::string("tensor map: ") + cudaGetErrorString(err)));
      e->has_tmap[i] = true;
    }
  }
  *out = e;
  return SB_OK;
}

int sb_upload_weights(sb_engine* e, int layer, const float* w, const float* bias) {
  if (!e || !w || !bias) return fail(SB_EINVAL, "null argument");
  if (layer < 0 || layer >= e->n_layers) return fail(SB_EINVAL, "layer out of range");
  const sb_layer_desc& L = e->layers[layer];
  SB_CUDA(cudaSetDevice(e->dev));
  drop_graphs(e);  // the conv kernels take the bias by value
  SB_CUDA(cudaMemcpy(e->bias[layer], bias, (size_t)L.cout * 4, cudaMemcpyHostToDevice));
  for (int c = 0; c < L.cout && c < 128; ++c) e->bias_h[layer][c] = bias[c];
  if (e->dtype == SB_F16) {
    const int q = e->layer_q[layer];
    const size_t bytes = conv_tc_wimg_bytes(L.cin, L.cout, e->layer_t[layer], L.stride, e->layer_mode[layer], q);
    std::vector<uint16_t> img((bytes + 1) / 2);
    e->wscale[layer].assign(L.cout, 1.f);
    conv_tc_build_wimg(L.cin, L.cout, e->layer_t[layer], L.stride, e->layer_mode[layer], w, bias, img.data(), q,
                       e->wscale[layer].data());
    SB_CUDA(cudaMemcpy(e->wdev[layer], img.data(), bytes, cudaMemcpyHostToDevice));
  } else {
    SB_CUDA(cudaMemcpy(e->wdev[layer], w, (size_t)9 * L.cin * L.cout * 4, cudaMemcpyHostToDevice));
  }
  e->wok[layer] = true;
  return SB_OK;
}

int sb_reset(sb_engine* e, const void* frames_dev, void* stream) {
  if (!e) return fail(SB_EINVAL, "null engine");
  return dense_impl(e, frames_dev, 1, (cudaStream_t)stream);
}

int sb_dense(sb_engine* e, const void* frames_dev, void* stream) {
  if (!e) return fail(SB_EINVAL, "null engine");
  return dense_impl(e, frames_dev, 0, (cudaStream_t)stream);
}

int sb_step(sb_engine* e, const void* frames_dev, void* stream, int* mode_out, int64_t* count_out) {
  if (!e) return fail(SB_EINVAL, "null engine");
  return step_impl(e, frames_dev, e->dtype == SB_F16 ? 0 : 1, nullptr, nullptr, (cudaStream_t)stream, mode_out,
                   count_out);
}

int sb_step_u8(sb_engine* e, const uint8_t* frames_dev, const float mean[3], const float std_[3], void* stream,
               int* mode_out, int64_t* count_out) {
  if (!e || !mean || !std_) return fail(SB_EINVAL, "null argument");
  if (e->dtype != SB_F16) return fail(SB_EINVAL, "uint8 frames need an fp16 engine");
  return step_impl(e, frames_dev, 2, mean, std_, (cudaStream_t)stream, mode_out, count_out);
}

int sb_step_u8_resized(sb_engine* e, const uint8_t* frames_dev, int cam_h, int cam_w, const float mean[3],
                       const float std_[3], void* stream, int* mode_out, int64_t* count_out) {
  if (!e || !mean || !std_ || !frames_dev) return fail(SB_EINVAL, "null argument");
  if (e->dtype != SB_F16) return fail(SB_EINVAL, "uint8 frames need an fp16 engine");
  if (cam_h < 1 || cam_w < 1) return fail(SB_EINVAL, "camera size must be positive");
  if (cam_h == e->h && cam_w == e->w)  // no resize: the uint8 path fused into the gate
    return step_impl(e, frames_dev, 2, mean, std_, (cudaStream_t)stream, mode_out, count_out);
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, frames_dev) != cudaSuccess || attr.type != cudaMemoryTypeDevice)
    return fail(SB_EINVAL, "frames must be device memory");
  SB_CUDA(cudaSetDevice(e->dev));
  if (!e->prep) {
    int rc = alloc_dev(e, &e->prep, (size_t)e->n * e->h * e->w * 3 * 2);
    if (rc) return rc;
  }
  cudaStream_t s = (cudaStream_t)stream;
  int rc = run_step(e, frames_dev, 3, cam_h, cam_w, mean, std_, [&](cudaStream_t st) {
    SB_CUDA(launch_prep_resize(frames_dev, e->n, cam_h, cam_w, static_cast<__half*>(e->prep), e->h, e->w, mean,
                               std_, e->n_sms, st));
    const int r = launch_step(e, e->prep, 0, nullptr, nullptr, st);
    e->last_launches += 1;
    return r;
  }, s);
  if (rc) return rc;
  return finish_step(e, s, mode_out, count_out);
}

int sb_step_profiled(sb_engine* e, const void* frames_dev, void* stream, float* kernel_ms, int capacity,
                     int* n_kernels) {
  if (!e || !kernel_ms || !n_kernels) return fail(SB_EINVAL, "null argument");
  e->profiling = true;
  e->n_events = 0;
  int mode;
  int64_t count;
  const int rc = step_impl(e, frames_dev, e->dtype == SB_F16 ? 0 : 1, nullptr, nullptr, (cudaStream_t)stream,
                           &mode, &count);
  e->profiling = false;
  if (rc) return rc;
  const int n = e->n_events - 1;
  *n_kernels = n;
  for (int i = 0; i < n && i < capacity; ++i) {
    float ms = 0.f;
    SB_CUDA(cudaEventElapsedTime(&ms, e->events[i], e->events[i + 1]));
    kernel_ms[i] = ms;
  }
  return SB_OK;
}

int sb_step_phases(sb_engine* e, const void* frames_dev, void* stream, float phase_ms[5]) {
  if (!e || !phase_ms) return fail(SB_EINVAL, "null argument");
  e->profiling = true;
  e->phases = true;
  e->n_events = 0;
  int mode;
  int64_t count;
  const int rc = step_impl(e, frames_dev, e->dtype == SB_F16 ? 0 : 1, nullptr, nullptr, (cudaStream_t)stream,
                           &mode, &count);
  e->profiling = false;
  e->phases = false;
  if (rc) return rc;
  if (e->n_events != 6) return fail(SB_ECUDA, "phase timing: unexpected event count");
  for (int i = 0; i < 5; ++i) SB_CUDA(cudaEventElapsedTime(&phase_ms[i], e->events[i], e->events[i + 1]));
  return SB_OK;
}

int sb_result_ptr(sb_engine* e, const int64_t** dev_ptr) {
  if (!e || !dev_ptr) return fail(SB_EINVAL, "null argument");
  *dev_ptr = e->st->result;
  return SB_OK;
}

int sb_query(sb_engine* e, void* stream, int* mode_out, int64_t* count_out) {
  if (!e) return fail(SB_EINVAL, "null engine");
  SB_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  State st;
  SB_CUDA(cudaMemcpy(&st, e->st, sizeof(State), cudaMemcpyDeviceToHost));
  if (mode_out) *mode_out = st.last_mode;
  if (count_out) *count_out = st.last_count;
  return SB_OK;
}

int sb_set_extra(sb_engine* e, const uint8_t* mask_dev, void* stream) {
  if (!e || !mask_dev) return fail(SB_EINVAL, "null argument");
  SB_CUDA(cudaMemcpyAsync(e->extra, mask_dev, e->n_blocks, cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
  return SB_OK;
}

int sb_set_fallback(sb_engine* e, int64_t fallback, void* stream) {
  if (!e) return fail(SB_EINVAL, "null engine");
  set_i64_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(&e->st->fallback, fallback);
  SB_CUDA(cudaGetLastError());
  return SB_OK;
}

int sb_set_tau(sb_engine* e, double tau) {
  if (!e) return fail(SB_EINVAL, "null engine");
  drop_graphs(e);  // the threshold is a kernel argument of the captured steps
  set_threshold(e, tau);
  return SB_OK;
}

int sb_set_cell_gating(sb_engine* e, int cell, const int* cell_radii, int n_radii) {
  if (!e) return fail(SB_EINVAL, "null engine");
  drop_graphs(e);  // the gating mode decides which kernels a step launches
  if (cell == 0) {
    e->cell = 0;
    return SB_OK;
  }
  if (e->dtype != SB_F16) return fail(SB_EINVAL, "cell-level gating: fp16 engines only");
  if (cell < 8 || cell % 8 || e->block % cell)
    return fail(SB_EINVAL, "cell-level gating: the cell must be a multiple of 8 px dividing the block");
  if (!cell_radii || n_radii != e->nd)
    return fail(SB_EINVAL, "cell-level gating: one cell radius per dilation group (" + std::to_string(e->nd) + ")");
  for (int i = 0; i < n_radii; ++i)
    if (cell_radii[i] < 0) return fail(SB_EINVAL, "cell-level gating: negative cell radius");
  SB_CUDA(cudaSetDevice(e->dev));
  if (!e->cmasks) {
    void* p = nullptr;
    int rc = alloc_dev(e, &p, (size_t)e->nd * e->n_blocks);
    if (rc) return rc;
    e->cmasks = static_cast<uint8_t*>(p);
  }
  if (e->cells_cell != cell) {  // cells of another size: the old buffer is freed, a new one made
    if (e->cells) {
      SB_CUDA(cudaDeviceSynchronize());  // no launched step may still write the old buffer
      e->allocs.erase(std::remove(e->allocs.begin(), e->allocs.end(), static_cast<void*>(e->cells)),
                      e->allocs.end());
      SB_CUDA(cudaFree(e->cells));
      e->cells = nullptr;
      e->cells_cell = 0;
    }
    void* p = nullptr;
    int rc = alloc_dev(e, &p, (size_t)e->n * (e->h / cell) * (e->w / cell));
    if (rc) return rc;
    e->cells = static_cast<uint8_t*>(p);
    e->cells_cell = cell;
  }
  for (int i = 0; i < n_radii; ++i) e->cell_r[i] = cell_radii[i];
  e->cell = cell;
  e->cell_thr_fx = threshold_fx(e->tau, cell);
  return SB_OK;
}

int sb_set_dense_check_every(sb_engine* e, int n, void* stream) {
  if (!e) return fail(SB_EINVAL, "null engine");
  set_i32_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(&e->st->check_every, n);
  SB_CUDA(cudaGetLastError());
  return SB_OK;
}

int sb_run_sparse_forced(sb_engine* e, const void* frames_dev, int64_t n_tiles, void* stream) {
  if (!e) return fail(SB_EINVAL, "null engine");
  if (n_tiles < 1 || n_tiles > e->n_blocks) return fail(SB_EINVAL, "n_tiles out of range");
  int rc = check_frames(e, frames_dev);
  if (rc) return rc;
  cudaStream_t s = (cudaStream_t)stream;
  SB_CUDA(launch_set_mode(e->st, SB_MODE_SPARSE, 0, n_tiles, s));
  CopyArgs c{};
  c.frames = frames_dev;
  c.img = e->cache[0];
  c.changed = e->changed;
  c.st = e->st;
  c.n = e->n;
  c.h = e->h;
  c.w = e->w;
  c.hb = e->hb;
  c.wb = e->wb;
  c.block = e->block;
  c.elem_bytes = e->esz;
  SB_CUDA(launch_copy(c, s));
  rc = launch_convs(e, s);
  if (rc) return rc;
  SB_CUDA(launch_set_mode(e->st, SB_MODE_SPARSE, 0, 0, s));
  return SB_OK;
}

int sb_dense_layers(sb_engine* e, int first, int last, void* stream) {
  if (!e) return fail(SB_EINVAL, "null engine");
  if (first < 0 || last < first || last >= e->n_layers) return fail(SB_EINVAL, "layer range out of range");
  SB_CUDA(cudaSetDevice(e->dev));
  cudaStream_t s = (cudaStream_t)stream;
  SB_CUDA(launch_set_mode(e->st, SB_MODE_DENSE, 0, 0, s));
  e->last_launches = 1;
  return launch_convs(e, s, first, last);
}

int sb_set_m0(sb_engine* e, int on, int64_t capacity) {
  if (!e) return fail(SB_EINVAL, "null engine");
  if (capacity < 0 || capacity > e->n_blocks) return fail(SB_EINVAL, "capacity must be in [0, n_blocks]");
  if (on)
    for (int i = 0; i < e->n_layers; ++i)
      if (e->layer_rk[i] >= 0)
        return fail(SB_EINVAL, "M0 mode needs an engine whose layers run over single blocks (SB_CREATE_BLOCK_UNITS)");
  SB_CUDA(cudaSetDevice(e->dev));
  const int32_t v[2] = {on ? 1 : 0, on ? (int32_t)capacity : 0};
  SB_CUDA(cudaMemcpy(reinterpret_cast<uint8_t*>(e->st) + offsetof(State, m0_mode), v, 8, cudaMemcpyHostToDevice));
  return SB_OK;
}

int sb_set_step_graphs(sb_engine* e, int on) {
  if (!e) return fail(SB_EINVAL, "null engine");
  if (!on) drop_graphs(e);
  e->graphs_on = on != 0;
  return SB_OK;
}

int sb_debug_withhold_lookback(sb_engine* e, int withhold_chunk, int spin_limit) {
  if (withhold_chunk < -1 || spin_limit < 0) return fail(SB_EINVAL, "withhold_chunk >= -1 and spin_limit >= 0");
  if (!e) {
    static_lists_debug(withhold_chunk, (unsigned)spin_limit);
    return SB_OK;
  }
  SB_CUDA(cudaSetDevice(e->dev));
  const int32_t w = withhold_chunk >= 0 ? withhold_chunk + 1 : 0;
  const uint32_t lim = (uint32_t)spin_limit;
  // synchronous copies: ordered after every step launched so far on any stream
  SB_CUDA(cudaMemcpy(reinterpret_cast<uint8_t*>(e->st) + offsetof(State, lb_withhold), &w, 4,
                     cudaMemcpyHostToDevice));
  SB_CUDA(cudaMemcpy(reinterpret_cast<uint8_t*>(e->st) + offsetof(State, lb_spin_limit), &lim, 4,
                     cudaMemcpyHostToDevice));
  return SB_OK;
}

int sb_cache_dtype(sb_engine* e, int cache_id, int* dtype, float* scale) {
  if (!e || !dtype) return fail(SB_EINVAL, "null argument");
  if (cache_id < 0 || cache_id > e->n_layers) return fail(SB_EINVAL, "cache id out of range");
  *dtype = e->cache_f8[cache_id] ? SB_F8 : e->dtype;
  if (scale) *scale = e->act_scale[cache_id];
  return SB_OK;
}

int sb_set_act_scale(sb_engine* e, int cache_id, float scale) {
  if (!e) return fail(SB_EINVAL, "null engine");
  if (cache_id < 0 || cache_id > e->n_layers || !e->cache_f8[cache_id])
    return fail(SB_EINVAL, "not an e4m3 cache");
  if (!(scale > 0.f) || !std::isfinite(scale)) return fail(SB_EINVAL, "scale must be positive and finite");
  drop_graphs(e);  // the scales are kernel arguments
  e->act_scale[cache_id] = scale;
  return SB_OK;
}

int sb_layer_wscale(sb_engine* e, int layer, float* out, int n) {
  if (!e || !out) return fail(SB_EINVAL, "null argument");
  if (layer < 0 || layer >= e->n_layers) return fail(SB_EINVAL, "layer out of range");
  if (e->layer_q[layer] < 2) return fail(SB_EINVAL, "layer has no e4m3 weights");
  if (n < (int)e->wscale[layer].size()) return fail(SB_EINVAL, "output too small");
  std::memcpy(out, e->wscale[layer].data(), e->wscale[layer].size() * 4);
  return SB_OK;
}

int sb_cache_ptr(sb_engine* e, int cache_id, void** ptr, int64_t shape[4]) {
  if (!e || !ptr) return fail(SB_EINVAL, "null argument");
  if (cache_id < 0 || cache_id > e->n_layers) return fail(SB_EINVAL, "cache id out of range");
  *ptr = e->cache[cache_id];
  if (shape)
    for (int k = 0; k < 4; ++k) shape[k] = e->shape[cache_id][k];
  return SB_OK;
}

int sb_layer_variant(sb_engine* e, int layer, int* mode) {
  if (!e || !mode) return fail(SB_EINVAL, "null argument");
  if (layer < 0 || layer >= e->n_layers) return fail(SB_EINVAL, "layer out of range");
  *mode = e->dtype == SB_F16 ? e->layer_mode[layer] | (e->layer_q[layer] << 4) : -1;
  return SB_OK;
}

int sb_gate_buffers(sb_engine* e, uint8_t** changed, uint8_t** masks, uint8_t** extra, int* n_dilations,
                    int dilations[SB_MAX_DILATIONS]) {
  if (!e) return fail(SB_EINVAL, "null engine");
  if (changed) *changed = e->changed;
  if (masks) *masks = e->masks;
  if (extra) *extra = e->extra;
  if (n_dilations) *n_dilations = e->nd;
  if (dilations)
    for (int i = 0; i < SB_MAX_DILATIONS; ++i) dilations[i] = i < e->nd ? e->ds[i] : 0;
  return SB_OK;
}

int sb_debug_lists(sb_engine* e, int d_index, int32_t** cam, int32_t** by, int32_t** bx, int64_t* count,
                   void* stream) {
  if (!e) return fail(SB_EINVAL, "null engine");
  if (d_index < 0 || d_index >= e->nd) return fail(SB_EINVAL, "dilation index out of range");
  int32_t* base = e->lists + (size_t)d_index * 3 * e->n_blocks;
  if (cam) *cam = base;
  if (by) *by = base + e->n_blocks;
  if (bx) *bx = base + 2 * (size_t)e->n_blocks;
  if (count) {
    SB_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    State st;
    SB_CUDA(cudaMemcpy(&st, e->st, sizeof(State), cudaMemcpyDeviceToHost));
    *count = st.counts[d_index];
  }
  return SB_OK;
}

int sb_stats(sb_engine* e, void* stream, sb_stats_t* out) {
  if (!e || !out) return fail(SB_EINVAL, "null argument");
  SB_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  State st;
  SB_CUDA(cudaMemcpy(&st, e->st, sizeof(State), cudaMemcpyDeviceToHost));
  std::memset(out, 0, sizeof(*out));
  out->skip = st.stats[SB_MODE_SKIP];
  out->sparse = st.stats[SB_MODE_SPARSE];
  out->dense = st.stats[SB_MODE_DENSE];
  out->last_count = st.last_count;
  out->last_mode = st.last_mode;
  out->error = st.error;
  out->n_dilations = e->nd;
  for (int i = 0; i < e->nd; ++i) {
    out->counts[i] = st.counts[i];
    out->dilations[i] = e->ds[i];
  }
  return SB_OK;
}

int sb_last_launch_count(sb_engine* e) { return e ? e->last_launches : 0; }

int sb_destroy(sb_engine* e) {
  if (!e) return SB_OK;
  cudaSetDevice(e->dev);
  cudaDeviceSynchronize();
  drop_graphs(e);
  if (e->cap_stream) cudaStreamDestroy(e->cap_stream);
  for (void* p : e->allocs) cudaFree(p);
  for (cudaEvent_t ev : e->events) cudaEventDestroy(ev);
  if (e->host_out) cudaFreeHost(e->host_out);
  delete e;
  return SB_OK;
}

}  // extern "C"
