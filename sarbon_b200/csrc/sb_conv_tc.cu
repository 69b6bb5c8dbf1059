// sb_conv_tc.cu -- fused gather -> 3x3 conv -> bias -> (+residual) -> ReLU -> scatter on
// the sm_100a tensor cores (tcgen05.mma, fp16 inputs, fp32 accumulators in TMEM).
//
// Reference: Bahrombekk/Sarbon sarbon/sparse/triton_conv.py:15-86 (`_tile_conv_kernel`,
// `tile_conv`): one implicit GEMM per active tile list, M = tiles * t^2 output pixels,
// N = C_out, K = 9 * C_in, input windows read straight from the NHWC cache with zero
// padding only at the image border, epilogue writing straight into the output cache.
//
// B200 design (not a translation of the Triton kernel):
//   * persistent CTAs (one per SM, or one 2-CTA cluster per SM pair) loop over 128-pixel
//     M-tiles of the step's unit list; the list length and the skip/sparse/dense mode are
//     read from device memory, so the launch needs no host sync;
//   * the weights of the CTA's output channels stay resident in shared memory (one bulk
//     copy of a pre-swizzled image, started before the programmatic-launch wait);
//   * A tiles come by TMA from the NHWC cache: row windows (one box per ky feeds the three
//     kx taps through shifted descriptors), strided windows for stride 2, full windows or
//     per-tap im2col boxes as selectable variants; out-of-image coordinates zero-fill;
//   * one TMA producer warp and one MMA issuer thread per stage sub-ring (two of each when
//     the ring holds enough stages) keep tcgen05.mma fed; CTA pairs run cta_group::2 M=256
//     MMAs with each CTA holding half the output channels;
//   * epilogue warps read the TMEM accumulator, add bias and residual, apply ReLU, round
//     once to fp16 and write the destination cache: CTA pairs read 16x256b fragments of a
//     permuted channel order (whole-line stores), window layers stage each warp's pixels
//     for one TMA tile store, the first layer stores 32-byte sectors per pixel;
//   * the 3-channel first layer cannot be fetched by TMA (6-byte pixels); its A rows
//     (27 taps x channels, zero-padded to K=32) are gathered by producer warps from a
//     TMA-loaded input window.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "sb_internal.cuh"
#include "sb_ptx.cuh"

namespace sb {

constexpr int kMaxSmem = 232448;  // 227 KB opt-in shared memory per CTA on sm_100
constexpr int kMaxCout = 128;     // widest layer of the stem (ConvArgs::bias_v holds its bias)

// WIN = 0: per-tap im2col boxes over blocks (or the first layer's gather);
// WIN = 1: row windows -- regions of 8/T x 1 blocks (8 px x T rows), one box per (ky, chunk)
//          feeds the three kx taps;
// WIN = 3: full windows -- regions of 8/T x 16/T blocks (8 px x 16 rows), one 10 x 18 px box
//          per chunk feeds all nine taps.  Both window modes are for stride-1 layers.
// WIN = 2: strided windows for stride-2 layers; regions as WIN = 1 (8 output px x T rows).
//          32 input channels: the input is viewed as pixel pairs (2 px x 32 ch = one 128-byte
//          row); per ky one box of 10 pairs x T rows (row element stride 2) feeds two pair
//          taps: pair offset -1 carries kx = 0 (odd pixel of the pair), offset 0 carries kx = 1
//          (even) and kx = 2 (odd); the unused half of the offset -1 tap has zero weights.
//          64 input channels: per ky two boxes of 10 px x T rows with element stride 2 in x
//          and y, starting at the odd (2*x0 - 1) and even (2*x0 - 2) input column: the odd box
//          feeds kx = 0 (offset 0) and kx = 2 (offset 1), the even box kx = 1 (offset 1).
// PAIR = 1: a 2-CTA cluster runs M=256 cta_group::2 MMAs; each CTA holds NCTA of the
//           2*NCTA output channels as its half of B and all 2*NCTA accumulator columns of
//           its own 128 pixels.
// Q = 0: fp16 input, weights and output caches (kind::f16 MMAs).
// Q = 1: fp16 input and weights, the output cache in e4m3 (scaled by 1 / its activation scale).
// Q = 2: e4m3 input cache, weights (per output channel scale), residual and output caches;
//        kind::f8f6f4 MMAs (K = 32 per instruction) and the dequantisation in the fp32 epilogue:
//        y = acc * (s_in * s_w[c]) + bias[c] + s_res * res, ReLU, e4m3(y / s_out).
// Q = 3: as Q = 2 with an fp16 output cache (the last layer of an e4m3 stage, whose output
//        leaves the stage).
template <int CIN, int NCTA, int T, int S, int WIN, int PAIR = 0, int Q = 0>
struct TcCfg {
  static constexpr bool F8IN = Q >= 2;                 // e4m3 A / B and kind::f8f6f4 MMAs
  static constexpr int AE = F8IN ? 1 : 2;              // bytes per A / B element
  static constexpr int OE = (Q == 1 || Q == 2) ? 1 : 2;  // bytes per output element
  static constexpr int RE = F8IN ? 1 : 2;              // bytes per residual element
  static constexpr bool MANUAL = CIN < 16;            // gathered by threads (first layer)
  static constexpr int KPAD = MANUAL ? ((9 * CIN + 15) / 16) * 16 : 0;
  // first layer: K slots per ky (its 3*CIN (kx, c) elements rounded up to even, so that each
  // ky run starts on a 32-bit word of the A row); when two slots remain after the three runs
  // they hold the bias: A = 1.0 there and B = the bias split into fp16 high and low parts,
  // so the MMA adds it and the epilogue does not
  static constexpr int KRUN = MANUAL ? ((3 * CIN + 1) / 2) * 2 : 0;
  static constexpr bool BIAS_IN_K = MANUAL && 3 * KRUN + 2 <= KPAD;
  // K elements per K-block (WIN = 2: a pair of input pixels x channels)
  static constexpr int CH = MANUAL ? KPAD
                           : WIN == 2 ? 64
                           : AE == 1 ? (CIN % 128 == 0 ? 128 : 64)
                                     : (CIN % 64 == 0 ? 64 : 32);
  static constexpr int NCH = (MANUAL || WIN == 2) ? 1 : CIN / CH;
  // WIN = 2 with 64 channels: two boxes per K-block (odd and even input columns)
  static constexpr int NBOX = (WIN == 2 && CIN == 64) ? 2 : 1;
  static constexpr int NKB = MANUAL ? 1 : (WIN == 3 ? 1 : (WIN == 1 || WIN == 2) ? 3 : 9) * NCH;  // per M-tile
  static constexpr int NWKB = MANUAL ? 1 : WIN == 2 ? (CIN == 32 ? 6 : 9) : 9 * NCH;  // weight K-blocks
  static constexpr int ROWB = CH * AE;                // bytes per operand row
  static constexpr int KSTEPS = ROWB / 32;            // MMAs per row: 32 bytes of K each
  static constexpr int SWZ = ROWB == 128 ? 2 : 4;     // 128B / 64B swizzle
  static constexpr int SBO = 8 * ROWB;
  static constexpr int TT = T * T;
  // window modes: a region is 8 output px wide and RROWS tall; its input window row is 10 px
  static constexpr int RROWS = WIN == 3 ? 16 : T;
  static constexpr int RW = WIN ? 8 / T : 1, RH = WIN == 3 ? 16 / T : 1;  // region in blocks
  static constexpr int RPX = 8 * RROWS;                 // output pixels per region
  static constexpr int TPM = WIN ? 128 / RPX : (TT >= 128 ? 1 : 128 / TT);  // tiles / regions per M-tile
  static constexpr int MPT = WIN ? 1 : (TT >= 128 ? TT / 128 : 1);          // M-tiles per tile
  static constexpr int BOX_ROWS = WIN == 3 ? 18 : WIN ? T : (TT >= 128 ? 128 / T : T);
  static constexpr int BOX_BYTES = WIN ? 10 * BOX_ROWS * ROWB : T * BOX_ROWS * ROWB;
  static constexpr int WSBO = 10 * ROWB;                // window modes: stride between output rows
  static constexpr int A_BYTES = WIN ? NBOX * TPM * BOX_BYTES : 128 * ROWB;  // bytes a stage's boxes deliver
  static constexpr int A_STAGE = ((A_BYTES + 1023) / 1024) * 1024;     // stage stride (1024-aligned)
  static constexpr int B_KB = NCTA * ROWB;
  static constexpr int W_BYTES = NWKB * B_KB;
  static constexpr int NMMA = PAIR ? 2 * NCTA : NCTA;  // MMA N = accumulator columns per CTA
  // narrow layers: two epilogue groups of four warps take alternate items (each warp all
  // NMMA columns of its 32 rows); wide layers: all eight warps on every item (half the
  // columns each).  Accumulator buffers: see NACC below.
  static constexpr int EPG = NMMA <= 64 ? 2 : 1;
  // roles: warps 0-7 epilogue (two per TMEM lane quadrant, half the columns each),
  // warp 8 TMA producer, warps 9-10 MMA issuers (warp 9 owns TMEM), warps 11-14 first-layer
  // gather, or warp 11 the second TMA producer (see NPROD)
  static constexpr int NCOL = EPG == 2 ? NMMA : NMMA / 2;  // accumulator columns per epilogue warp
  static constexpr int EPI_WARPS_PER_ITEM = 8 / EPG;
  static constexpr int PROD_WARP = 8, MMA_WARP = 9, GATHER0 = 352, PROD_WARP2 = 11;  // MMA issuers: warps 9, 10
  static constexpr int W_OFF = 0;
  // bias: CTA pairs stage it in shared memory; the other layers read it from the kernel
  // parameters (ConvArgs::bias_v, warp-uniform constant-cache reads) -- measured faster there
  static constexpr bool BIAS_SMEM = PAIR != 0;
  // pairs: the bias, and for Q = 2 the per-channel dequantisation scales after it
  static constexpr int BIAS_BYTES = BIAS_SMEM ? kMaxCout * 4 * (F8IN ? 2 : 1) : 0;
  static constexpr int A_OFF = ((W_BYTES + 1023) / 1024) * 1024;
  // Epilogue output through shared memory: each epilogue warp writes its 32 output pixels
  // (NCOL channels each) into its own staging buffer and stores them with one TMA tile
  // store, a box of OBW px x 32/OBW rows of one unit.  Written directly, every 16-byte
  // store instruction of a warp touches 32 different lines; the tile store writes whole
  // lines.  Used where a warp's pixels form such a box of one unit (window modes); CTA
  // pairs store directly (their shared memory holds the weights and the stages), and so
  // does the first layer, whose per-item epilogue latency the staging would lengthen.
  static constexpr bool TSTORE = !PAIR && WIN != 0;
  static constexpr int OBW = 8;                                    // staged box width (px)
  static constexpr int EPI_WARP_BYTES = TSTORE ? 32 * NCOL * 2 : 0;  // one warp's buffer
  static constexpr int EPI_BYTES = 8 * EPI_WARP_BYTES;
  static constexpr int CRING = MANUAL ? 32 : 8;       // item-coordinate ring (producer -> epilogue)
  static constexpr int CRING_BYTES = CRING * 8 * 4 * 4; // <= 8 units x (cam, row, col, pad) per item
  // first layer: the input window of one M-tile (BOX_ROWS output rows of one tile), loaded
  // by one 3-D TMA box from the image cache viewed as [N][H][W*CIN]; the box starts 8
  // elements (16 B) before the window's first element... rounded so x stays 16-byte aligned
  static constexpr int WIN_ROWS = (BOX_ROWS - 1) * S + 3;
  static constexpr int WIN_ELEMS = ((T - 1) * S + 3) * CIN;
  static constexpr int WIN_COLS = ((8 + WIN_ELEMS + 7) / 8) * 8;     // box inner extent (elements)
  static constexpr int WIN_LEAD = 8 - CIN;                            // elements before the first used one
  static constexpr int WIN_BUF = ((WIN_ROWS * WIN_COLS * 2 + 127) / 128) * 128;
  static constexpr int NWB = 16;                                      // window ring depth
  static constexpr int NGW = 4;                                       // first layer: gather warps
  static constexpr int WIN_BYTES = MANUAL ? NWB * WIN_BUF : 0;
  // mbarriers (sized for the most stages that could fit) + TMEM address + abort flag
  static constexpr int STAGES_UB = (kMaxSmem - A_OFF) / A_STAGE > 24 ? 24 : (kMaxSmem - A_OFF) / A_STAGE;
  static constexpr int N_BARS = 2 * STAGES_UB + 2 * 4 /*NACC <= 4*/ + 4 + (MANUAL ? 2 * NWB : 0) + 2 * CRING;
  static constexpr int BAR_BYTES = ((N_BARS * 8 + 8) + 127) / 128 * 128;
  static constexpr int FIXED = 1024 /*align slack*/ + BIAS_BYTES + BAR_BYTES + WIN_BYTES + CRING_BYTES + EPI_BYTES;
  static constexpr int STAGES_FIT = (kMaxSmem - FIXED - A_OFF) / A_STAGE;
  // first layer: a multiple of 8 stages, so that each stage (and each window slot) is
  // always filled by the same one of the NGW gather warps (see the gather loop)
  static constexpr int STAGES = STAGES_FIT > 24 ? 24 : MANUAL ? (STAGES_FIT / 8) * 8 : STAGES_FIT;
  // MMA issuers: two (alternate items) when the ring holds two items' K-blocks, or for CTA
  // pairs whenever it holds four stages; each issuer owns a sub-ring of SUB stages used in
  // the order of its K-blocks, so every stage has one in-order consumer and the phase
  // parities stay exact.  An issuer's mbarrier wait costs ~200 cycles in which the tensor
  // pipe would run dry; with two, one keeps it fed while the other waits.
  static constexpr int NISS = (STAGES >= 2 * NKB || (PAIR && STAGES >= 4)) ? 2 : 1;
  static constexpr int SUB = STAGES / NISS;
  // TMA producers: with two issuers (TMA-loaded layers) each sub-ring has its own producer
  // warp filling its issuer's items, so neither issuer waits behind the other's loads when
  // a sub-ring holds less than an item
  static constexpr int NPROD = (!MANUAL && NISS == 2) ? 2 : 1;
  static constexpr int THREADS = MANUAL ? 480 : NPROD == 2 ? 384 : 352;
  // accumulator buffers: four for narrow layers (two epilogue groups) and for two issuers,
  // so the MMAs can run ahead of the epilogue
  static constexpr int NACC = (EPG == 2 || NISS == 2) ? 4 : 2;
  static constexpr int TMEM_COLS = (NACC * NMMA) <= 32 ? 32 : (NACC * NMMA) <= 64 ? 64 : (NACC * NMMA) <= 128 ? 128 : (NACC * NMMA) <= 256 ? 256 : 512;
  static constexpr int SMEM = FIXED + A_OFF + STAGES * A_STAGE;
  static constexpr uint32_t IDESC = idesc_f16(PAIR ? 256 : 128, NMMA);
  static_assert(STAGES >= 2, "shared memory too small for two stages");
  static_assert(TPM <= 8, "coordinate ring holds up to 8 units per item");
  static_assert(!PAIR || NCOL == 64, "pair epilogue: 16x256b fragments of 64 columns per warp");
  static_assert(NACC * NMMA <= 512, "accumulators exceed TMEM");
  static_assert(NPROD == 1 || (CRING % 2 == 0 && SUB >= 1), "two producers: ring slots alternate between them");
  static_assert(!TSTORE || (EPG == 2 && (NCOL == 32 || NCOL == 64) && RPX % 32 == 0),
                "staged output: a warp's 32 pixels are one box of one unit");
  static_assert(NCTA % 32 == 0 && NCTA >= 32 && NMMA <= 256, "UMMA N / epilogue split");
  static_assert(!PAIR || !MANUAL, "CTA pairs need TMA-loaded A stages");
  static_assert(!MANUAL || KPAD <= 64, "first-layer K too large");
  static_assert(Q == 0 || (PAIR && !MANUAL), "e4m3 caches: CTA-pair layers only");
  static_assert(!F8IN || (WIN == 1 && (ROWB == 128 || ROWB == 64)), "e4m3 inputs: row windows over 64/128-byte rows");
  static_assert(!MANUAL || ((NISS * SUB) % NGW == 0 && NWB % NGW == 0), "gather warp per stage / window slot");
  static_assert(!MANUAL || TT >= 128, "first layer: an M-tile must lie within one tile");
  static_assert(!MANUAL || (S == 2 && CIN <= 8 && WIN_COLS <= 256 && WIN_COLS % 2 == 0), "first-layer window box");
  static_assert(!WIN || ((((WIN == 1 || WIN == 3) && S == 1) || (WIN == 2 && S == 2 && (CIN == 32 || CIN == 64))) &&
                         8 % T == 0 && T <= 8 && (ROWB == 128 || (F8IN && ROWB == 64)) && !MANUAL),
                "window mode geometry");
};

struct TileXY {
  int cam, by, bx;
};

// Active-tile i of this layer: dense -> every block in flat order; sparse -> the
// block list (entries past the listed count are block 0, as nonzero_static pads).
// Unit i of this layer (a block, or for window modes a region of a.rw x a.rh blocks):
// dense -> every unit in flat order; sparse -> the ordered list (entries past the listed
// count are unit 0, as nonzero_static pads).  Returns (cam, unit row, unit column).
template <int WIN>
SB_DEV TileXY tile_at(const ConvArgs& a, int mode, int listed, int i) {
  TileXY r{0, 0, 0};
  if (mode == SB_MODE_DENSE) {
    const int gw = WIN ? (a.wb + a.rw - 1) / a.rw : a.wb;
    const int gh = WIN ? (a.hb + a.rh - 1) / a.rh : a.hb;
    const int per = gh * gw;
    r.cam = i / per;
    const int q = i - r.cam * per;
    r.by = q / gw;
    r.bx = q - r.by * gw;
  } else if (i < listed) {
    const int32_t* lc = WIN ? a.rcam : a.lcam;
    const int32_t* ly = WIN ? a.rry : a.lby;
    const int32_t* lx = WIN ? a.rrx : a.lbx;
    r.cam = __ldg(lc + i);
    r.by = __ldg(ly + i);
    r.bx = __ldg(lx + i);
  }
  return r;
}

// Work item -> (C_out slice, M-tile).  A CTA keeps one C_out slice for the whole launch
// (slice = CTA index mod nsplit; the grid is a multiple of nsplit), so its weights are
// loaded once, and strides over the M-tiles with the gridDim/nsplit CTAs of its slice.
struct Item {
  int split, m;
};
SB_DEV Item item_at(int it, int nsplit) {
  return Item{(int)blockIdx.x % nsplit, (int)blockIdx.x / nsplit + it * ((int)gridDim.x / nsplit)};
}

// Stage and phase of K-block kb of item it: item it belongs to issuer it % NISS, whose
// sub-ring holds stages [u*SUB, (u+1)*SUB) used in the order of that issuer's K-blocks.
template <class C>
SB_DEV void stage_of(int it, int kb, uint32_t& s, uint32_t& ph) {
  const uint32_t u = C::NISS == 2 ? (uint32_t)(it & 1) : 0u;
  const uint32_t gu = (uint32_t)(C::NISS == 2 ? (it >> 1) : it) * C::NKB + (uint32_t)kb;
  s = u * C::SUB + gu % C::SUB;
  ph = (gu / C::SUB) & 1u;
}

template <int CIN, int NCTA, int T, int S, int WIN, int PAIR, int Q>
__global__ void __launch_bounds__(TcCfg<CIN, NCTA, T, S, WIN, PAIR, Q>::THREADS, 1)
    conv_tc_kernel(const __grid_constant__ ConvArgs a, const __grid_constant__ CUtensorMap tmap,
                   const __grid_constant__ CUtensorMap tmap_y) {
  using C = TcCfg<CIN, NCTA, T, S, WIN, PAIR, Q>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem + C::W_OFF;
  uint8_t* sA = smem + C::A_OFF;
  uint8_t* sEpi = sA + C::STAGES * C::A_STAGE;  // [8 epilogue warps][EPI_WARP_BYTES], 1024-aligned
  float* sBias = reinterpret_cast<float*>(sEpi + C::EPI_BYTES);  // BIAS_SMEM only
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sBias) + C::BIAS_BYTES);
  uint64_t* full = bars;
  uint64_t* empty = bars + C::STAGES;
  uint64_t* accf = bars + 2 * C::STAGES;  // [NACC] accumulator full / empty
  uint64_t* acce = accf + C::NACC;
  uint64_t* wfull = acce + C::NACC;
  uint64_t* dbar = wfull + 1;            // [2]: drain of each MMA issuer
  uint64_t* wpeer = dbar + 2;            // pairs: the odd CTA's weights have landed
  uint64_t* winfull = dbar + 3;          // first-layer window ring (MANUAL only)
  uint64_t* winempty = winfull + C::NWB;
  uint64_t* cfull = C::MANUAL ? winempty + C::NWB : winfull;  // item-coordinate ring
  uint64_t* cempty = cfull + C::CRING;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(cempty + C::CRING);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  __half* win = reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(bars) + C::BAR_BYTES);
  int4* sCoord = reinterpret_cast<int4*>(reinterpret_cast<uint8_t*>(win) + C::WIN_BYTES);  // [CRING][8]

  const int warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < C::NACC; ++i) {
      mbar_init(&accf[i], 1);
      // one arrival per epilogue warp on the item (of both CTAs of a pair)
      mbar_init(&acce[i], C::EPI_WARPS_PER_ITEM * (PAIR ? 2 : 1));
    }
    mbar_init(wfull, 1);
    mbar_init(&dbar[0], 1);
    mbar_init(&dbar[1], 1);
    mbar_init(wpeer, 1);
    if (C::MANUAL) {
      for (int i = 0; i < C::NWB; ++i) {
        mbar_init(&winfull[i], 1);
        mbar_init(&winempty[i], 1);
      }
    }
    for (int i = 0; i < C::CRING; ++i) {
      mbar_init(&cfull[i], 1);
      mbar_init(&cempty[i], C::EPI_WARPS_PER_ITEM);  // one arrival per epilogue warp on the item
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == C::MMA_WARP) {
    if (PAIR) {
      tmem_alloc2(tmem_holder, C::TMEM_COLS);  // the same columns on both SMs of the pair
      tmem_relinquish2();
    } else {
      tmem_alloc(tmem_holder, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  if (C::BIAS_SMEM)
    for (int i = threadIdx.x; i < a.cout; i += blockDim.x) {
      sBias[i] = a.bias_v[i];
      if (C::F8IN) sBias[kMaxCout + i] = a.dq_v[i];
    }
  if (!C::MANUAL && warp == C::PROD_WARP && lane == 0) prefetch_tmap(&tmap);
  if (C::TSTORE && warp == 0 && lane == 0) prefetch_tmap(&tmap_y);
  tc_fence_before();
  if (PAIR) cluster_sync();  // the leader's barriers are initialised before the odd CTA uses them
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;

  // Programmatic dependent launch: this kernel may start while the previous kernel of the
  // stream (the previous layer, or the frame copy) still runs.  That kernel triggered this
  // launch only after its item loop, which began after the kernel before it had completed,
  // and it writes nothing but its output cache and error flags; so the step's
  // device state and unit lists (written by the gate / list / mode kernels, two or more
  // launches back) and this CTA's weight slice are read before griddepcontrol.wait.  Only the threads that read caches written by
  // earlier layers wait: the producer before its first input copy, the epilogue before its
  // first residual read.
  // work of this launch, decided on the device (no host sync)
  const int mode = a.st->mode_cur;
  const int listed = (WIN && a.rkind >= 0) ? a.st->rcounts[a.rkind][a.d_idx] : a.st->counts[a.d_idx];
  const int n_units =
      WIN ? a.n_blocks / (a.hb * a.wb) * ((a.hb + a.rh - 1) / a.rh) * ((a.wb + a.rw - 1) / a.rw) : a.n_blocks;
  int n_tiles = 0;
  if (mode == SB_MODE_DENSE) n_tiles = n_units;
  else if (mode == SB_MODE_SPARSE) n_tiles = a.st->force_tiles > 0 ? a.st->force_tiles : listed;
  if (n_tiles > n_units) n_tiles = n_units;
  const int n_mtiles = (!WIN && C::TT >= 128) ? n_tiles * C::MPT : (n_tiles + C::TPM - 1) / C::TPM;
  const int nsplit = PAIR ? 1 : a.cout / NCTA;
  // pairs: cluster p runs M-tiles 2q, 2q+1 (q = p, p + npairs, ...); CTA rank r takes 2q+r
  const int npairs = (int)gridDim.x / 2, pair = (int)blockIdx.x / 2;
  int my_items;
  if (PAIR) {
    const int pm = (n_mtiles + 1) / 2;
    my_items = pair < pm ? (pm - 1 - pair) / npairs + 1 : 0;
  } else {
    const int m_first = (int)blockIdx.x / nsplit, m_stride = (int)gridDim.x / nsplit;
    my_items = m_first < n_mtiles ? (n_mtiles - 1 - m_first) / m_stride + 1 : 0;
  }
  auto item_of = [&](int it) -> Item {
    if (PAIR) return Item{(int)rank, 2 * (pair + it * npairs) + (int)rank};
    return item_at(it, nsplit);
  };
  // the CTA's weight slice, copied only when it has items this launch (both CTAs of a pair
  // have the same item count)
  if (my_items > 0 && warp == C::PROD_WARP && lane == 0) {
    const int wsplit = PAIR ? (int)rank : (int)blockIdx.x % (a.cout / NCTA);
    const uint8_t* wsrc = static_cast<const uint8_t*>(a.wimg) + (size_t)wsplit * C::W_BYTES;
    mbar_arrive_expect_tx(wfull, C::W_BYTES);
    for (int off = 0; off < C::W_BYTES; off += 32768) {
      const int len = C::W_BYTES - off < 32768 ? C::W_BYTES - off : 32768;
      bulk_load(sW + off, wsrc + off, len, wfull);
    }
  }

  if (my_items > 0) {
    if (warp == C::PROD_WARP || (C::NPROD == 2 && warp == C::PROD_WARP2)) {
      // ------------------------------------------------ producer: the slice's weights, A stages
      // The whole warp runs the loop (warp-uniform control flow); lane 0 issues the copies.
      // With two producers, producer pu fills the items pu, pu + 2, ... (issuer pu's sub-ring).
      const bool leader = lane == 0;
      const int pu = warp == C::PROD_WARP ? 0 : 1;
      const int n_loc = (my_items - pu + C::NPROD - 1) / C::NPROD;  // this producer's items
      uint32_t g = 0, nload = 0;
      struct Coords {
        int cam[C::TPM], y0[C::TPM], x0[C::TPM], uy[C::TPM], ux[C::TPM];
      };
      auto fetch = [&](int it, Coords& o) {
        const Item w = item_of(it);
#pragma unroll
        for (int j = 0; j < C::TPM; ++j) {
          int ti, sub;
          if (!WIN && C::TT >= 128) { ti = w.m / C::MPT; sub = w.m % C::MPT; }
          else { ti = w.m * C::TPM + j; sub = 0; }
          const TileXY p = tile_at<WIN>(a, mode, listed, ti < n_tiles ? ti : 0);
          o.uy[j] = p.by;
          o.ux[j] = p.bx;
          o.cam[j] = p.cam;
          o.y0[j] = (WIN ? p.by * C::RROWS * S : (p.by * T + sub * C::BOX_ROWS) * S) - 1;
          o.x0[j] = (WIN ? p.bx * 8 : p.bx * T * S) - 1;
        }
      };
      // returns false when the pipeline was aborted
      auto issue = [&](int it, const Coords& cc) -> bool {
        const Item w = item_of(it);
        // publish this item's unit coordinates for the epilogue
        {
          const int slot = it % C::CRING;
          if (!warp_wait(&cempty[slot], ((it / C::CRING) & 1) ^ 1, abort_flag)) {
            atomicOr(&a.st->error, SB_ERR_TIMEOUT_EMPTY);
            *abort_flag = 1;
            return false;
          }
          if (leader) {
#pragma unroll
            for (int j = 0; j < C::TPM; ++j) sCoord[slot * 8 + j] = make_int4(cc.cam[j], cc.uy[j], cc.ux[j], 0);
            mbar_arrive(&cfull[slot]);
          }
          __syncwarp();
        }
        if (nload == 0) {  // the weights were issued in the prologue
          ++nload;
          if (PAIR && rank == 1 && pu == 0) {  // tell the leader that this CTA's half of B is resident
            if (!warp_wait(wfull, 0, abort_flag)) {
              atomicOr(&a.st->error, SB_ERR_TIMEOUT_WGT);
              *abort_flag = 1;
              return false;
            }
            if (leader) mbar_arrive_cluster(mapa_shared(smem_u32(wpeer), 0));
            __syncwarp();
          }
        }
        if (C::MANUAL) {
          // first layer: one window box per item into the ring
          const int b = it % C::NWB;
          if (!warp_wait(&winempty[b], ((it / C::NWB) & 1) ^ 1, abort_flag)) {
            atomicOr(&a.st->error, SB_ERR_TIMEOUT_EMPTY);
            *abort_flag = 1;
            return false;
          }
          if (leader) {
            mbar_arrive_expect_tx(&winfull[b], C::WIN_ROWS * C::WIN_COLS * 2);
            tma_load_3d(reinterpret_cast<uint8_t*>(win) + b * C::WIN_BUF, &tmap, &winfull[b],
                        (cc.x0[0] + 1) * CIN - CIN - C::WIN_LEAD, cc.y0[0], cc.cam[0]);
          }
          __syncwarp();
          ++g;
          return true;
        }
        for (int kb = 0; kb < C::NKB; ++kb, ++g) {
          // im2col: K-block = (tap, chunk); window: K-block = (ky, chunk), the 3 kx taps read
          // the same window rows at offsets of kx pixels
          // full window: K-block = chunk, the box covers all taps
          const int tap = WIN == 3 ? 0 : WIN ? (kb / C::NCH) * 3 : kb / C::NCH, ch = kb % C::NCH;
          const int ky = tap / 3, kx = WIN ? 0 : tap % 3;
          uint32_t s, ph;
          stage_of<C>(it, kb, s, ph);
          if (!warp_wait(&empty[s], ph ^ 1u, abort_flag)) {
            atomicOr(&a.st->error, SB_ERR_TIMEOUT_EMPTY);
            *abort_flag = 1;
            return false;
          }
          if (leader) {
            uint8_t* dst = sA + s * C::A_STAGE;
            if (PAIR) {
              // both CTAs' boxes complete on the leader's barrier; the leader expects both
              const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
              if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * C::A_BYTES);
#pragma unroll
              for (int bs = 0; bs < C::NBOX; ++bs)
#pragma unroll
                for (int j = 0; j < C::TPM; ++j)
                  tma_load_4d_pair(dst + (bs * C::TPM + j) * C::BOX_BYTES, &tmap, fb, ch * C::CH,
                                   C::NBOX == 2 ? 2 * cc.x0[j] + 1 - bs : cc.x0[j] + kx, cc.y0[j] + ky, cc.cam[j]);
            } else {
              mbar_arrive_expect_tx(&full[s], C::A_BYTES);
#pragma unroll
              for (int bs = 0; bs < C::NBOX; ++bs)
#pragma unroll
                for (int j = 0; j < C::TPM; ++j)
                  tma_load_4d(dst + (bs * C::TPM + j) * C::BOX_BYTES, &tmap, &full[s], ch * C::CH,
                              C::NBOX == 2 ? 2 * cc.x0[j] + 1 - bs : cc.x0[j] + kx, cc.y0[j] + ky, cc.cam[j]);
            }
          }
          __syncwarp();
        }
        return true;
      };
      // Lane l loads the unit coordinates of this producer's item base + l, one batch of 32
      // items ahead of their use (two batches alternate between the register sets ca and cb),
      // so the list reads' latency is paid once per 32 items; items take theirs by shuffle.
      auto fetch_lane = [&](int base, Coords& o) {
        if (base + (int)lane < n_loc) fetch(pu + (base + (int)lane) * C::NPROD, o);
      };
      auto run_batch = [&](int base, const Coords& cur) -> bool {
        for (int i = 0; i < 32 && base + i < n_loc; ++i) {
          if (*abort_flag) return false;
          Coords cc;
#pragma unroll
          for (int j = 0; j < C::TPM; ++j) {
            cc.cam[j] = __shfl_sync(0xFFFFFFFFu, cur.cam[j], i);
            cc.y0[j] = __shfl_sync(0xFFFFFFFFu, cur.y0[j], i);
            cc.x0[j] = __shfl_sync(0xFFFFFFFFu, cur.x0[j], i);
            cc.uy[j] = __shfl_sync(0xFFFFFFFFu, cur.uy[j], i);
            cc.ux[j] = __shfl_sync(0xFFFFFFFFu, cur.ux[j], i);
          }
          if (!issue(pu + (base + i) * C::NPROD, cc)) return false;
        }
        return true;
      };
      Coords ca, cb;
      fetch_lane(0, ca);
      grid_dep_wait();  // the input cache (previous layer / frame copy) is complete
      for (int base = 0; base < n_loc; base += 64) {
        if (base + 32 < n_loc) fetch_lane(base + 32, cb);
        if (!run_batch(base, ca) || base + 32 >= n_loc) break;
        if (base + 64 < n_loc) fetch_lane(base + 64, ca);
        if (!run_batch(base + 32, cb)) break;
      }
      // drain: every issued copy has landed before the CTA may exit
      volatile int never = 0;
      if (C::MANUAL) {
        const uint32_t first = g > (uint32_t)C::NWB ? g - C::NWB : 0u;
        for (uint32_t q = first; q < g; ++q) warp_wait(&winfull[q % C::NWB], (q / C::NWB) & 1u, &never);
      } else {
        // the last fill of every stage of each sub-ring (earlier fills were consumed); the
        // odd CTA of a pair has no full barriers of its own: it waits until the leader's
        // MMAs have released its last stages (no copy or commit into it is then pending)
        for (int u = 0; u < C::NISS; ++u) {
          if (C::NPROD == 2 && u != pu) continue;  // the other producer drains its own sub-ring
          const uint32_t uses = (uint32_t)((my_items - u + C::NISS - 1) / C::NISS) * C::NKB;
          const uint32_t first = uses > (uint32_t)C::SUB ? uses - C::SUB : 0u;
          for (uint32_t q = first; q < uses; ++q) {
            uint64_t* b = (PAIR && rank == 1) ? &empty[u * C::SUB + q % C::SUB] : &full[u * C::SUB + q % C::SUB];
            warp_wait(b, (q / C::SUB) & 1u, &never);
          }
        }
      }
      if (nload > 0) warp_wait(wfull, 0, &never);
    } else if (C::MANUAL && (int)threadIdx.x >= C::GATHER0) {
      // ------------------------------------------------ gather producers (first layer)
      // Gather warp gw builds all 128 A rows (one output pixel each: 3x3 taps x channels,
      // zero-padded to KPAD) of items gw, gw + NGW, ... from the TMA-loaded input window of
      // the item, four rows per lane, so NGW items are in flight.  Item it uses window slot
      // it % NWB and stage stage_of(it): both are always filled by this same warp.
      const int gw = ((int)threadIdx.x - C::GATHER0) >> 5;
      for (int it = gw; it < my_items && !*abort_flag; it += C::NGW) {
        const int b = it % C::NWB;
        if (!warp_wait(&winfull[b], (it / C::NWB) & 1u, abort_flag)) {
          atomicOr(&a.st->error, SB_ERR_TIMEOUT_FULL);
          *abort_flag = 1;
          break;
        }
        uint32_t s, ph;
        stage_of<C>(it, 0, s, ph);
        if (!warp_wait(&empty[s], ph ^ 1u, abort_flag)) {
          atomicOr(&a.st->error, SB_ERR_TIMEOUT_EMPTY);
          *abort_flag = 1;
          break;
        }
        const uint16_t* wbase =
            reinterpret_cast<const uint16_t*>(reinterpret_cast<const uint8_t*>(win) + b * C::WIN_BUF) + C::WIN_LEAD;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int r = lane + 32 * j;  // A row = output pixel slot, 0..127
          const int lr = r / T, lc = r % T;
          // element (ky, kx, c) of output (lr, lc): window row S*lr+ky, column
          // lead + (S*lc + kx)*CIN + c  (the window starts one input pixel left of the tile)
          // The 3*CIN elements (kx, c) of one ky are contiguous in the window row; in the A
          // row they fill K slots ky*KRUN .. (a run padded to even length), so each ky is
          // read as 32-bit words (S = 2 puts every pixel's run at the same parity: it starts
          // at an odd element when WIN_LEAD is odd) and realigned by funnel shifts.
          constexpr int RUN = 3 * CIN, KRUN = C::KRUN, NW = KRUN / 2;
          constexpr int ODD = C::WIN_LEAD & 1;
          constexpr int NWD = (RUN + ODD + 1) / 2;
          const uint32_t* wrow32 =
              reinterpret_cast<const uint32_t*>(wbase + (S * lr) * C::WIN_COLS + (S * lc) * CIN - ODD);
          uint32_t o[C::KPAD > 0 ? C::KPAD / 2 : 8];
#pragma unroll
          for (int k = 0; k < C::KPAD / 2; ++k) o[k] = 0u;
#pragma unroll
          for (int ky = 0; ky < 3; ++ky) {
            uint32_t w[NWD + 1];
#pragma unroll
            for (int i = 0; i < NWD; ++i) w[i] = wrow32[ky * (C::WIN_COLS / 2) + i];
            w[NWD] = 0u;
#pragma unroll
            for (int j = 0; j < NW; ++j) {
              uint32_t v = ODD ? __funnelshift_r(w[j], w[j + 1], 16) : w[j];
              if (2 * j + 1 >= RUN) v &= 0xFFFFu;  // the run's padding slot
              if (2 * j >= RUN) v = 0u;
              o[ky * NW + j] = v;
            }
          }
          if (C::BIAS_IN_K) o[3 * NW] = 0x3C003C00u;  // 1.0, 1.0: the bias's high and low parts
          uint8_t* row = sA + s * C::A_STAGE + r * C::ROWB;
          constexpr int NQ = C::ROWB / 16;
#pragma unroll
          for (int q = 0; q < NQ; ++q) {
            const int pq = C::SWZ == 2 ? (q ^ (r & 7)) : (q ^ ((r >> 1) & 3));
            *reinterpret_cast<uint4*>(row + pq * 16) = make_uint4(o[4 * q], o[4 * q + 1], o[4 * q + 2], o[4 * q + 3]);
          }
        }
        fence_proxy_async_smem();  // these generic-proxy writes feed the MMA (async proxy)
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&full[s]);
          mbar_arrive(&winempty[b]);
        }
        __syncwarp();
      }
    } else if (warp == C::MMA_WARP || warp == C::MMA_WARP + 1) {
      // ------------------------------------------------ MMA issuers
      // With NISS = 2, lane 0 of warp 9 issues the MMAs of the even items into accumulator
      // 0 and lane 0 of warp 10 those of the odd items into accumulator 1 (NISS = 1: warp 9
      // issues every item, alternating accumulators).  tcgen05.mma issue is
      // back-pressured by the tensor pipe and an N <= 96 MMA takes ~48 cycles, so the
      // instruction queue holds little work; an mbarrier wait of the issuing thread (its
      // shared-memory access queues behind the MMAs' operand reads) would let the pipe run
      // dry.  With two issuers one keeps the pipe fed while the other waits.  The K-block
      // loop is unrolled and both descriptors advance by compile-time offsets (which cannot
      // carry out of the 14-bit start-address field: shared memory < 256 KB).
      const int u = warp - C::MMA_WARP;
      if (lane == 0 && u < C::NISS && rank == 0) {  // pairs: only the even CTA issues
        const uint64_t a_desc0 = smem_desc(smem_u32(sA), WIN ? C::WSBO : C::SBO, C::SWZ);
        const uint64_t b_desc0 = smem_desc(smem_u32(sW), C::SBO, C::SWZ);
        constexpr uint32_t ASTEP = C::A_STAGE >> 4;
        bool ok = true;
        if (u < my_items && (!mbar_wait(wfull, 0, abort_flag) ||        // this CTA's C_out slice
                             (PAIR && !mbar_wait(wpeer, 0, abort_flag)))) {  // and the odd CTA's
          atomicOr(&a.st->error, SB_ERR_TIMEOUT_WGT);
          *abort_flag = 1;
          ok = false;
        }
        for (int it = u; ok && it < my_items; it += C::NISS) {
          const int ab = it % C::NACC;
          if (!mbar_wait(&acce[ab], ((it / C::NACC) & 1) ^ 1, abort_flag)) {
            atomicOr(&a.st->error, SB_ERR_TIMEOUT_ACC);
            *abort_flag = 1;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + ab * C::NMMA;
          uint32_t s, ph;
          stage_of<C>(it, 0, s, ph);
          const uint32_t s_end = (uint32_t)u * C::SUB + C::SUB;  // one past this sub-ring
#pragma unroll
          for (int kb = 0; kb < C::NKB; ++kb) {
            if (!mbar_wait(&full[s], ph, abort_flag)) {
              atomicOr(&a.st->error, SB_ERR_TIMEOUT_FULL);
              *abort_flag = 1;
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t a_desc = a_desc0 + s * ASTEP;
            if (WIN) {
              // window taps: A = the window shifted by (ky*10 + kx) pixels (128 B rows; the
              // hardware swizzle follows absolute smem addresses), B = that tap's weights.
              // Row windows hold one ky per K-block, full windows all three.
              // Pair windows: two pair taps per ky (weight blocks ky*2 + tap).
              // 64-channel strided windows: taps t = 0, 1, 2 are (odd box, offset 0) kx = 0,
              // (odd box, offset 1) kx = 2 and (even box, offset 1) kx = 1.
              constexpr int NKY = WIN == 3 ? 3 : 1, NTX = WIN == 2 ? (C::NBOX == 2 ? 3 : 2) : 3;
              const int ch = kb % C::NCH, ky0 = WIN == 3 ? 0 : kb / C::NCH;
#pragma unroll
              for (int dy = 0; dy < NKY; ++dy)
#pragma unroll
                for (int kx = 0; kx < NTX; ++kx)
#pragma unroll
                  for (int kk = 0; kk < C::KSTEPS; ++kk) {
                    constexpr int SLOT = C::TPM * C::BOX_BYTES;
                    const uint32_t a_off = C::NBOX == 2
                                               ? (kx == 2 ? SLOT : 0) + (kx == 0 ? 0 : 1) * C::ROWB + kk * 32
                                               : ((WIN == 3 ? dy * 10 : 0) + kx) * C::ROWB + kk * 32;
                    const int wk = C::NBOX == 2 ? kb * 3 + (kx == 0 ? 0 : kx == 1 ? 2 : 1)
                                   : WIN == 2 ? kb * 2 + kx : ((ky0 + dy) * 3 + kx) * C::NCH + ch;
                    const uint32_t b_off = wk * C::B_KB + kk * 32;
                    if (PAIR && C::F8IN)
                      mma_f8_ss2(d_tmem, a_desc + (a_off >> 4), b_desc0 + (b_off >> 4), C::IDESC,
                                 (kb | dy | kx | kk) != 0 ? 1u : 0u);
                    else if (PAIR)
                      mma_f16_ss2(d_tmem, a_desc + (a_off >> 4), b_desc0 + (b_off >> 4), C::IDESC,
                                  (kb | dy | kx | kk) != 0 ? 1u : 0u);
                    else
                      mma_f16_ss(d_tmem, a_desc + (a_off >> 4), b_desc0 + (b_off >> 4), C::IDESC,
                                 (kb | dy | kx | kk) != 0 ? 1u : 0u);
                  }
            } else {
#pragma unroll
              for (int kk = 0; kk < C::KSTEPS; ++kk) {
                if (PAIR)
                  mma_f16_ss2(d_tmem, a_desc + ((kk * 32) >> 4), b_desc0 + ((kb * C::B_KB + kk * 32) >> 4),
                              C::IDESC, (kb | kk) != 0 ? 1u : 0u);
                else
                  mma_f16_ss(d_tmem, a_desc + ((kk * 32) >> 4), b_desc0 + ((kb * C::B_KB + kk * 32) >> 4),
                             C::IDESC, (kb | kk) != 0 ? 1u : 0u);
              }
            }
            if (PAIR) {
              mma_commit2_both(&empty[s]);  // the stage is free in both CTAs once read
            } else {
              mma_commit(&empty[s]);  // stage free once these MMAs have read it
            }
            if (++s == s_end) {
              s = s_end - C::SUB;
              ph ^= 1u;
            }
          }
          if (!ok) break;
          if (PAIR) {
            mma_commit2_both(&accf[ab]);  // both CTAs' accumulators are ready
          } else {
            mma_commit(&accf[ab]);  // accumulator ready for the epilogue
          }
        }
        // drain: all MMAs this thread issued complete before TMEM is released
        if (PAIR) mma_commit2(smem_u32(&dbar[u]));
        else mma_commit(&dbar[u]);
        volatile int never = 0;
        mbar_wait(&dbar[u], 0, &never);
      }
      __syncwarp();
    } else if (PAIR && warp < 8) {
      grid_dep_wait();  // residual caches of earlier layers are complete
      // ------------------------------------------------ epilogue of CTA pairs: TMEM fragments -> cache
      // Warp w reads TMEM lane quadrant q = w % 4 (32 accumulator rows = pixels); with two
      // groups (EPG = 2) warps 0-3 take the even and warps 4-7 the odd items with all
      // NCOL = NMMA columns, else every warp takes every item with columns (w / 4) * NCOL...
      // The accumulator is read as 16x256b fragments (two loads, lanes 32q and 32q + 16):
      // thread t (k = t / 4, m = t % 4) gets, for the pixels k, k + 8, k + 16, k + 24 of the
      // quadrant, the columns 8j + 2m + b.  The weight image orders the output channels so
      // that column 8j + 2m + b of a group of NCOL columns holds channel CPT * m + 2j + b
      // (CPT = NCOL / 4): each thread then owns CPT consecutive channels of four pixels and
      // the four threads of a pixel store its NCOL channels as whole 32-byte sectors that
      // together fill complete lines.  The residual is read the same way one item ahead;
      // the TMEM buffer is released as soon as it sits in registers.
      constexpr int G = C::NCOL, CPT = G / 4, REP = G / 8;  // CPT channels per thread and pixel
      const int q = warp & 3, eg = C::EPG == 2 ? (warp >> 2) : 0;  // lane quadrant, group
      const int col0 = C::EPG == 2 ? 0 : (warp >> 2) * C::NCOL;
      const int k = lane >> 2, m = lane & 3;
      // output and residual caches: fp16, or e4m3 codes (C::OE bytes per element)
      uint8_t* y = static_cast<uint8_t*>(a.y);
      const uint8_t* res = static_cast<const uint8_t*>(a.res);
      // this thread's output channels are the same for every item of the launch
      const int n0 = (PAIR ? 0 : ((int)blockIdx.x % (a.cout / NCTA)) * NCTA) + col0 + CPT * m;
      float bias[CPT];
      float dq[C::F8IN ? CPT : 1];  // e4m3 inputs: s_in * s_w[c] of each channel
#pragma unroll
      for (int t = 0; t < CPT; ++t) {
        bias[t] = C::BIAS_SMEM ? sBias[n0 + t] : a.bias_v[n0 + t];
        if constexpr (C::F8IN) dq[t] = sBias[kMaxCout + n0 + t];
      }
      const float res_scale = a.res_scale, out_inv = a.out_inv_scale;
      // Pixel sr (0..3) of this thread is accumulator row q*32 + k + 8*sr.  When a warp's 32
      // rows lie in one unit (ONEUNIT) its pixels sit at fixed offsets from the first one.
      constexpr int UPX = WIN ? C::RPX : (C::TT >= 128 ? 128 : C::TT);  // rows of one unit in an M-tile
      constexpr bool ONEUNIT = UPX >= 32;
      constexpr int UW = WIN ? 8 : T;                                    // unit width (px)
      // destinations and residual of one item (this thread's four pixels), fetched one item ahead
      struct Row {
        size_t pix[ONEUNIT ? 1 : 4];  // element of channel n0: pixel 0 (ONEUNIT) or each pixel
        int p;                        // pixel 0's index within its unit (ONEUNIT)
        unsigned okm;                 // bit sr: pixel sr is stored
        uint4 rr[4][CPT * C::RE / 16];  // residual: CPT channels of each pixel
      };
      const size_t rowstride = (size_t)a.wo * a.cout;
      // offset of pixel sr from pixel 0 (ONEUNIT): unit pixel p + 8 sr, UW pixels per row
      auto pix_of = [&](const Row& o, int sr) -> size_t {
        if constexpr (ONEUNIT) {
          const int p1 = o.p + 8 * sr;
          return o.pix[0] + (size_t)(p1 / UW - o.p / UW) * rowstride + (ptrdiff_t)(p1 % UW - o.p % UW) * a.cout;
        } else {
          return o.pix[sr];
        }
      };
      // unit coordinates come from the producer through the shared-memory ring, so the
      // residual prefetch below depends on no global load
      auto fetch = [&](int it, Row& o) -> bool {
        const Item w = item_of(it);
        const int slot = it % C::CRING;
        if (!mbar_wait(&cfull[slot], (it / C::CRING) & 1, abort_flag)) return false;
        int4 u[4];
        int ti[4], pp[4];
#pragma unroll
        for (int sr = 0; sr < 4; ++sr) {
          const int r = q * 32 + k + 8 * sr;  // accumulator row of pixel sr
          int j;
          if (WIN) { j = r / C::RPX; ti[sr] = w.m * C::TPM + j; pp[sr] = r % C::RPX; }
          else if (C::TT >= 128) { j = 0; ti[sr] = w.m / C::MPT; pp[sr] = (w.m % C::MPT) * 128 + r; }
          else { j = r / C::TT; ti[sr] = w.m * C::TPM + j; pp[sr] = r % C::TT; }
          if (!ONEUNIT || sr == 0) u[sr] = sCoord[slot * 8 + j];
          else u[sr] = u[0];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&cempty[slot]);
        o.okm = 0u;
        o.p = pp[0];
#pragma unroll
        for (int sr = 0; sr < 4; ++sr) {
          const int p = pp[sr];
          const bool valid = ti[sr] < n_tiles;
          const TileXY tc{u[sr].x, u[sr].y, u[sr].z};
          const int gy = WIN ? tc.by * C::RROWS + p / 8 : tc.by * T + p / T;
          const int gx = WIN ? tc.bx * 8 + p % 8 : tc.bx * T + p % T;
          const bool inb = tc.cam < a.n && gy < a.ho && gx < a.wo;
          // a region may overhang the image's right / bottom edge (those pixels are skipped);
          // only a unit whose origin lies outside the image is a corrupt list entry
          if (sr == 0 || !ONEUNIT) {
            const bool origin_ok = tc.cam < a.n && (WIN ? tc.by * C::RROWS : tc.by * T) < a.ho &&
                                   (WIN ? tc.bx * 8 : tc.bx * T) < a.wo;
            if (valid && !origin_ok) atomicOr(&a.st->error, SB_ERR_BAD_TILE);
            o.pix[ONEUNIT ? 0 : sr] = (((size_t)tc.cam * a.ho + gy) * a.wo + gx) * a.cout + n0;
          }
          const bool st = valid && inb;
          if (st) o.okm |= 1u << sr;
          if (res != nullptr) {
            const uint8_t* rp = res + pix_of(o, sr) * C::RE;
            if constexpr (CPT * C::RE == 32) {
              if (st) ld_global_nc_v8(rp, o.rr[sr][0], o.rr[sr][1]);
              else o.rr[sr][0] = o.rr[sr][1] = make_uint4(0, 0, 0, 0);
            } else {
              o.rr[sr][0] = st ? __ldg(reinterpret_cast<const uint4*>(rp)) : make_uint4(0, 0, 0, 0);
            }
          }
        }
        return true;
      };
      // bias / residual / ReLU / store of pixel sr from its fragment registers f
      // (registers 4j + b hold channels CPT*m + 2j + b)
      auto out_pixel = [&](const Row& cu, int sr, const uint32_t* f) {
        if (!((cu.okm >> sr) & 1u)) return;
        const uint32_t* rw = reinterpret_cast<const uint32_t*>(&cu.rr[sr][0]);
        const uint16_t* rw8 = reinterpret_cast<const uint16_t*>(&cu.rr[sr][0]);
        uint32_t o[CPT / 2];
#pragma unroll
        for (int jj = 0; jj < REP; ++jj) {
          float f0, f1;
          if constexpr (C::F8IN) {  // dequantise the e4m3 x e4m3 accumulation per channel
            f0 = fmaf(__uint_as_float(f[4 * jj]), dq[2 * jj], bias[2 * jj]);
            f1 = fmaf(__uint_as_float(f[4 * jj + 1]), dq[2 * jj + 1], bias[2 * jj + 1]);
          } else {
            f0 = __uint_as_float(f[4 * jj]) + bias[2 * jj];
            f1 = __uint_as_float(f[4 * jj + 1]) + bias[2 * jj + 1];
          }
          if (res != nullptr) {
            if constexpr (C::RE == 1) {
              const float2 t2 = float2_of_e4m3x2(rw8[jj]);
              f0 = fmaf(t2.x, res_scale, f0);
              f1 = fmaf(t2.y, res_scale, f1);
            } else {
              const float2 t2 = __half22float2(*reinterpret_cast<const __half2*>(&rw[jj]));
              f0 += t2.x;
              f1 += t2.y;
            }
          }
          if (a.act) {
            f0 = fmaxf(f0, 0.0f);
            f1 = fmaxf(f1, 0.0f);
          }
          if constexpr (C::OE == 1) {  // two e4m3 codes per jj: 16 channels = 16 bytes
            const uint32_t q = e4m3x2_of(f0 * out_inv, f1 * out_inv);
            if (jj & 1) o[jj >> 1] |= q << 16;
            else o[jj >> 1] = q;
          } else {
            __half2 h2 = __floats2half2_rn(f0, f1);
            o[jj] = *reinterpret_cast<uint32_t*>(&h2);
          }
        }
        uint8_t* dst = y + pix_of(cu, sr) * C::OE;
        if constexpr (C::OE == 1)
          *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
        else if constexpr (CPT == 16)
          st_global_v8(dst, make_uint4(o[0], o[1], o[2], o[3]), make_uint4(o[4], o[5], o[6], o[7]));
        else
          *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
      };
      // one item: wait for the accumulator, move its fragments to registers, release TMEM and
      // prefetch the next item into `nx`, bias / residual / ReLU / store the four pixels
      auto step = [&](int it, const Row& cu, Row& nx) -> bool {
        const int ab = it % C::NACC;
        const bool got = mbar_wait(&accf[ab], (it / C::NACC) & 1, abort_flag);
        if (!got) {
          atomicOr(&a.st->error, SB_ERR_TIMEOUT_ACC);
          *abort_flag = 1;
        }
        // warp-uniform exit: tcgen05.ld below is .sync.aligned
        if (__any_sync(0xFFFFFFFFu, !got || *abort_flag != 0)) return false;
        tc_fence_after();
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + ab * C::NMMA + col0;
        auto ld_frag = [&](int hh, uint32_t* v) {
          if constexpr (REP == 8)
            tmem_ld16x256b8(taddr + ((uint32_t)(16 * hh) << 16), *reinterpret_cast<uint32_t(*)[32]>(v));
          else
            tmem_ld16x256b4(taddr + ((uint32_t)(16 * hh) << 16), *reinterpret_cast<uint32_t(*)[16]>(v));
        };
        auto release = [&]() {
          tc_fence_before();
          // one arrival per warp (on the pair leader's barrier): the MMA may overwrite it now
          __syncwarp();
          if (lane == 0) {
            if (PAIR) mbar_arrive_cluster(mapa_shared(smem_u32(&acce[ab]), 0));
            else mbar_arrive(&acce[ab]);
          }
          if (it + C::EPG < my_items && !fetch(it + C::EPG, nx)) {
            atomicOr(&a.st->error, SB_ERR_TIMEOUT_FULL);
            *abort_flag = 1;
          }
        };
        if constexpr (!PAIR) {
          // both fragments to registers, release the buffer at once, then the four pixels
          uint32_t v[2][4 * REP];
          ld_frag(0, v[0]);
          ld_frag(1, v[1]);
          tmem_ld_wait();
          release();
#pragma unroll
          for (int sr = 0; sr < 4; ++sr) out_pixel(cu, sr, &v[sr >> 1][2 * (sr & 1)]);
        } else {
          // CTA pairs (fewer registers to spare): lanes 32q.. -> pixels 0, 1 first, then
          // lanes 32q + 16.., release, pixels 2, 3
          uint32_t v[4 * REP];
          ld_frag(0, v);
          tmem_ld_wait();
          out_pixel(cu, 0, &v[0]);
          out_pixel(cu, 1, &v[2]);
          ld_frag(1, v);
          tmem_ld_wait();
          release();
          out_pixel(cu, 2, &v[0]);
          out_pixel(cu, 3, &v[2]);
        }
        return true;
      };
      // this group's items: eg, eg + EPG, ...
      Row ra, rb;
      if (eg < my_items && !fetch(eg, ra)) {
        atomicOr(&a.st->error, SB_ERR_TIMEOUT_FULL);
        *abort_flag = 1;
      }
      for (int it = eg; it < my_items; it += 2 * C::EPG) {
        if (!step(it, ra, rb) || it + C::EPG >= my_items) break;
        if (!step(it + C::EPG, rb, ra)) break;
      }
    } else if (warp < 8) {
      grid_dep_wait();  // residual caches of earlier layers are complete
      // ------------------------------------------------ epilogue: TMEM -> bias/res/ReLU -> cache
      // Warp w reads TMEM lanes 32*(w%4).. (its accumulator rows); with two groups (EPG = 2)
      // warps 0-3 take the even and warps 4-7 the odd items with all NCOL = NMMA columns,
      // else every warp takes every item with columns (w/4)*NCOL...  The residual is fetched
      // one item ahead and the TMEM buffer is released as soon as it sits in registers.
      const int q = warp & 3, eg = C::EPG == 2 ? (warp >> 2) : 0;  // lane quadrant, group
      const int col0 = C::EPG == 2 ? 0 : (warp >> 2) * C::NCOL;
      const int r = q * 32 + lane;  // accumulator row = TMEM lane
      __half* y = static_cast<__half*>(a.y);
      const __half* res = static_cast<const __half*>(a.res);
      // per-row destination and residual of one item, fetched one item ahead
      struct Row {
        size_t pix;
        int n0;
        bool st;
        bool ovalid;     // staged output: the warp's box belongs to a listed unit
        int ox, oy, oc;  // staged output: box origin (pixel column, row, camera)
        uint4 rr[C::NCOL / 8];
      };
      // unit coordinates come from the producer through the shared-memory ring, so the
      // residual prefetch below depends on no global load
      auto fetch = [&](int it, Row& o) -> bool {
        const Item w = item_of(it);
        o.n0 = PAIR ? col0 : w.split * NCTA + col0;
        int ti, p, j;
        if (WIN) { j = r / C::RPX; ti = w.m * C::TPM + j; p = r % C::RPX; }
        else if (C::TT >= 128) { j = 0; ti = w.m / C::MPT; p = (w.m % C::MPT) * 128 + r; }
        else { j = r / C::TT; ti = w.m * C::TPM + j; p = r % C::TT; }
        const int slot = it % C::CRING;
        if (!mbar_wait(&cfull[slot], (it / C::CRING) & 1, abort_flag)) return false;
        const int4 u = sCoord[slot * 8 + j];
        __syncwarp();
        if (lane == 0) mbar_arrive(&cempty[slot]);
        const bool valid = ti < n_tiles;
        TileXY tc{u.x, u.y, u.z};
        const int gy = WIN ? tc.by * C::RROWS + p / 8 : tc.by * T + p / T;
        const int gx = WIN ? tc.bx * 8 + p % 8 : tc.bx * T + p % T;
        const bool inb = tc.cam < a.n && gy < a.ho && gx < a.wo;
        // a region may overhang the image's right / bottom edge (those pixels are skipped);
        // only a unit whose origin lies outside the image is a corrupt list entry
        const bool origin_ok = tc.cam < a.n && (WIN ? tc.by * C::RROWS : tc.by * T) < a.ho &&
                               (WIN ? tc.bx * 8 : tc.bx * T) < a.wo;
        if (valid && !origin_ok) atomicOr(&a.st->error, SB_ERR_BAD_TILE);
        o.st = valid && inb;
        o.pix = (((size_t)tc.cam * a.ho + gy) * a.wo + gx) * a.cout + o.n0;
        if (C::TSTORE) {
          // the warp's 32 pixels: rows p0/OBW .. of the unit (p0 = this warp's first pixel)
          const int p0 = p - lane;
          o.ovalid = valid && origin_ok;
          o.ox = tc.bx * 8;
          o.oy = tc.by * C::RROWS + p0 / C::OBW;
          o.oc = tc.cam;
        }
        if (res != nullptr) {
#pragma unroll
          for (int q2 = 0; q2 < C::NCOL / 16; ++q2) {  // 32-byte loads: one sector per lane
            if (o.st) {
              ld_global_nc_v8(res + o.pix + q2 * 16, o.rr[2 * q2], o.rr[2 * q2 + 1]);
            } else {
              o.rr[2 * q2] = make_uint4(0, 0, 0, 0);
              o.rr[2 * q2 + 1] = make_uint4(0, 0, 0, 0);
            }
          }
        }
        return true;
      };
      // one item: wait for the accumulator, move it to registers, release TMEM, prefetch the
      // next item into `nx`, then bias / residual / ReLU / store item `it` from `cu`
      auto step = [&](int it, const Row& cu, Row& nx) -> bool {
        const int ab = it % C::NACC;
        const bool got = mbar_wait(&accf[ab], (it / C::NACC) & 1, abort_flag);
        if (!got) {
          atomicOr(&a.st->error, SB_ERR_TIMEOUT_ACC);
          *abort_flag = 1;
        }
        // warp-uniform exit: tcgen05.ld below is .sync.aligned
        if (__any_sync(0xFFFFFFFFu, !got || *abort_flag != 0)) return false;
        tc_fence_after();
        uint32_t v[C::NCOL];
        const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + ab * C::NMMA + col0;
#pragma unroll
        for (int j = 0; j < C::NCOL / 16; ++j)
          tmem_ld16(taddr + j * 16, *reinterpret_cast<uint32_t(*)[16]>(&v[j * 16]));
        tmem_ld_wait();
        tc_fence_before();
        // one arrival per warp (on the pair leader's barrier): the MMA may overwrite it now
        __syncwarp();
        if (lane == 0) {
          if (PAIR) mbar_arrive_cluster(mapa_shared(smem_u32(&acce[ab]), 0));
          else mbar_arrive(&acce[ab]);
        }
        if (it + C::EPG < my_items && !fetch(it + C::EPG, nx)) {
          atomicOr(&a.st->error, SB_ERR_TIMEOUT_FULL);
          *abort_flag = 1;
        }
        uint8_t* ebuf = sEpi + warp * C::EPI_WARP_BYTES;
        if (C::TSTORE) {
          if (lane == 0) bulk_wait_read0();  // the previous item's store has read the buffer
          __syncwarp();
        }
        if (C::TSTORE || cu.st) {
          uint4 prev = make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int j = 0; j < C::NCOL / 8; ++j) {
            float f[8];
            if constexpr (C::BIAS_IN_K) {  // the MMA added the bias (its K slots)
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(v[j * 8 + e]);
            } else {
              const float* bsrc = C::BIAS_SMEM ? sBias : a.bias_v;  // warp-uniform index either way
              const float4 b0 = *reinterpret_cast<const float4*>(bsrc + cu.n0 + j * 8);
              const float4 b1 = *reinterpret_cast<const float4*>(bsrc + cu.n0 + j * 8 + 4);
              const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(v[j * 8 + e]) + bb[e];
            }
            if (res != nullptr) {
              const __half2* h = reinterpret_cast<const __half2*>(&cu.rr[j]);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 t2 = __half22float2(h[e]);
                f[2 * e] += t2.x;
                f[2 * e + 1] += t2.y;
              }
            }
            if (a.act) {
#pragma unroll
              for (int e = 0; e < 8; ++e) f[e] = fmaxf(f[e], 0.0f);
            }
            uint4 o;
            __half2* ph = reinterpret_cast<__half2*>(&o);
#pragma unroll
            for (int e = 0; e < 4; ++e) ph[e] = __floats2half2_rn(f[2 * e], f[2 * e + 1]);
            if (C::TSTORE) {
              // box layout [pixel][NCOL channels] with the tensor map's swizzle (128-byte rows:
              // 16-byte chunk j at j ^ (pixel & 7); 64-byte rows: j ^ ((pixel >> 1) & 3)), so
              // the 32 lanes' writes spread over all banks
              const int pj = C::NCOL == 64 ? (j ^ (lane & 7)) : (j ^ ((lane >> 1) & 3));
              *reinterpret_cast<uint4*>(ebuf + lane * (C::NCOL * 2) + pj * 16) = o;
            } else if (j & 1) {
              st_global_v8(y + cu.pix + (j - 1) * 8, prev, o);  // 32-byte stores: one sector per lane
            } else {
              prev = o;
            }
          }
        }
        if (C::TSTORE) {
          fence_proxy_async_smem();  // generic-proxy writes -> the TMA store (async proxy)
          __syncwarp();
          if (lane == 0 && cu.ovalid) {  // pixels outside the image are clipped by the store
            tma_store_4d(&tmap_y, ebuf, cu.n0, cu.ox, cu.oy, cu.oc);
            bulk_commit_group();
          }
        }
        return true;
      };
      // this group's items: eg, eg + EPG, ...
      Row ra, rb;
      if (eg < my_items && !fetch(eg, ra)) {
        atomicOr(&a.st->error, SB_ERR_TIMEOUT_FULL);
        *abort_flag = 1;
      }
      for (int it = eg; it < my_items; it += 2 * C::EPG) {
        if (!step(it, ra, rb) || it + C::EPG >= my_items) break;
        if (!step(it + C::EPG, rb, ra)) break;
      }
      // the staged stores are complete (global writes performed) before the CTA signals
      // its dependents or exits
      if (C::TSTORE && lane == 0) bulk_wait0();
      __syncwarp();
    }
  }
  // the weight copy (issued when the CTA had items) has landed before the CTA may exit
  if (warp == C::PROD_WARP && my_items > 0) {
    volatile int never = 0;
    warp_wait(wfull, 0, &never);
  }
  // the next kernel of the stream may start its prologue on free SMs (triggering right after
  // the wait instead measured about 2 % slower per step: the early CTAs' weight copies compete
  // with this kernel's loads)
  grid_dep_launch();
  tc_fence_before();
  __syncthreads();
  if (PAIR) cluster_sync();  // both CTAs are done with TMEM and with each other's barriers
  if (warp == C::MMA_WARP) {
    tc_fence_after();
    if (PAIR) tmem_dealloc2(tmem_base, C::TMEM_COLS);
    else tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if (PAIR) cluster_sync();  // neither CTA exits while the other may still address it
}

// ---------------------------------------------------------------- host side
namespace {

struct Variant {
  int cin, cout, t, s, win, ncta, pair, q;
  void (*fn)(const ConvArgs, const CUtensorMap, const CUtensorMap);
  int smem, threads, w_bytes, ch, box_rows, win_cols, win_rows;
  int tstore, ncol, obw;  // staged output stores: flag, channels and width of a warp's box
  int mode() const { return win | (pair << 3); }
};

template <int CIN, int NCTA, int T, int S, int WIN = 0, int PAIR = 0, int Q = 0>
Variant make_variant(int cout) {
  using C = TcCfg<CIN, NCTA, T, S, WIN, PAIR, Q>;
  Variant v{CIN,       cout,       T,         S,         WIN,       NCTA,      PAIR,      Q,
                 conv_tc_kernel<CIN, NCTA, T, S, WIN, PAIR, Q>,  C::SMEM,   C::THREADS, C::W_BYTES,
                 C::CH,     C::BOX_ROWS, C::WIN_COLS, C::WIN_ROWS, C::TSTORE ? 1 : 0, C::NCOL, C::OBW};
  return v;
}

// Sarbon stem shapes (widths 32/64/128, Res blocks) at block 32 and block 64.  The first
// variant of a shape is its default.
const std::vector<Variant>& variants() {
  static const std::vector<Variant> v = {
      // block 32
      make_variant<3, 32, 16, 2>(32),
      make_variant<32, 32, 8, 2, 2, 1>(64),    // CTA pairs (M=256, N=64), pair windows over blocks
      make_variant<32, 64, 8, 2, 2>(64),       // pair windows over blocks
      make_variant<32, 64, 8, 2>(64),
      make_variant<64, 32, 8, 1, 1, 1>(64),    // CTA pairs (M=256, N=64), row windows over blocks
      make_variant<64, 64, 8, 1, 1>(64),       // row windows over blocks
      make_variant<64, 64, 8, 1, 3>(64),       // full windows over 1x2-block regions
      make_variant<64, 64, 4, 2, 2, 1>(128),   // CTA pairs, strided windows over 2x1-block regions
      make_variant<64, 64, 4, 2, 0, 1>(128),   // CTA pairs: M=256, N=128
      make_variant<64, 128, 4, 2>(128),
      make_variant<128, 64, 4, 1, 1, 1>(128),  // CTA pairs, row windows over horizontal block pairs
      make_variant<128, 64, 4, 1, 1>(128),     // row windows, two C_out slices
      make_variant<128, 64, 4, 1, 3, 1>(128),  // CTA pairs, full windows over 2x4-block regions
      make_variant<128, 64, 4, 1, 3>(128),     // full windows, two C_out slices
      make_variant<128, 64, 4, 1, 0, 1>(128),  // CTA pairs, per-tap boxes over blocks (block units)
      // e4m3 caches of the stride-8 stage: fp16 in / e4m3 out, then e4m3 in and out
      make_variant<64, 64, 4, 2, 2, 1, 1>(128),
      make_variant<128, 64, 4, 1, 1, 1, 2>(128),
      // e4m3 caches of the stride-4 stage: t1 fp16 in / e4m3 out, the 64->64 layers e4m3 in
      // and out (64-byte rows), the stage's last layer e4m3 in / fp16 out
      make_variant<32, 32, 8, 2, 2, 1, 1>(64),
      make_variant<64, 32, 8, 1, 1, 1, 2>(64),
      make_variant<64, 32, 8, 1, 1, 1, 3>(64),
      // block 64
      make_variant<3, 32, 32, 2>(32),
      make_variant<32, 64, 16, 2>(64),
      make_variant<64, 64, 16, 1>(64),
      make_variant<64, 64, 8, 2, 2, 1>(128),
      make_variant<64, 64, 8, 2, 0, 1>(128),
      make_variant<64, 128, 8, 2>(128),
      make_variant<128, 64, 8, 1, 3, 1>(128),  // CTA pairs, full windows over 1x2-block regions
      make_variant<128, 64, 8, 1, 3>(128),
      make_variant<128, 64, 8, 1, 1, 1>(128),
      make_variant<128, 64, 8, 1, 1>(128),
  };
  return v;
}

// SARBON_NO_PAIR=1 skips the CTA-pair variants (measurement aid).
bool pairs_disabled() {
  const char* env = std::getenv("SARBON_NO_PAIR");
  return env && std::atoi(env) != 0;
}

// mode < 0: the default variant of the shape; else the variant with that mode
// (window mode | pair << 3).  q selects the e4m3 variants (0: fp16 caches).
const Variant* find_variant(int cin, int cout, int t, int s, int mode = -1, int q = 0) {
  const bool no_pair = pairs_disabled();
  for (const auto& v : variants()) {
    if (v.cin != cin || v.cout != cout || v.t != t || v.s != s || v.q != q) continue;
    if (q) {
      if (mode < 0 || v.mode() == mode) return &v;
      continue;
    }
    if (mode < 0 ? (no_pair && v.pair) : v.mode() != mode) continue;
    return &v;
  }
  return nullptr;
}

}  // namespace

// The mode the engine runs a layer with: the default variant's, or with
// SARBON_WINDOW_MODE=0|1|3 (measurement aid) that window mode where the shape has it.
int conv_tc_pick_mode(int cin, int cout, int t, int s) {
  const Variant* v = find_variant(cin, cout, t, s);
  if (!v) return -1;
  const char* env = std::getenv("SARBON_WINDOW_MODE");
  if (env && v->win != 0) {
    const int want = std::atoi(env);
    if (find_variant(cin, cout, t, s, want | (v->pair << 3))) return want | (v->pair << 3);
    if (find_variant(cin, cout, t, s, want)) return want;
  }
  return v->mode();
}

int conv_tc_block_mode(int cin, int cout, int t, int s) {
  const bool no_pair = pairs_disabled();
  const Variant* best = nullptr;
  for (const auto& v : variants()) {
    if (v.cin != cin || v.cout != cout || v.t != t || v.s != s) continue;
    if (no_pair && v.pair) continue;
    const bool one_block = v.win == 0 || (8 / t == 1 && (v.win != 3 || 16 / t == 1));
    if (!one_block) continue;
    if (!best || (v.pair && !best->pair)) best = &v;
  }
  return best ? best->mode() : -1;
}

int conv_tc_q_mode(int cin, int cout, int t, int s, int q) {
  const Variant* v = find_variant(cin, cout, t, s, -1, q);
  return v ? v->mode() : -1;
}

namespace {
// The variant the engine runs (and whose weight image it builds) for a layer of mode `mode`.
const Variant* picked(int cin, int cout, int t, int s, int mode, int q = 0) {
  return mode < 0 ? nullptr : find_variant(cin, cout, t, s, mode, q);
}
}  // namespace

bool conv_tc_supported(int cin, int cout, int t, int s) { return find_variant(cin, cout, t, s) != nullptr; }

int conv_tc_nsplit(int cin, int cout, int t, int s, int mode, int q) {
  const Variant* v = picked(cin, cout, t, s, mode, q);
  return v ? v->cout / v->ncta : 0;
}

size_t conv_tc_wimg_bytes(int cin, int cout, int t, int s, int mode, int q) {
  const Variant* v = picked(cin, cout, t, s, mode, q);
  return v ? (size_t)v->w_bytes * (v->cout / v->ncta) : 0;
}

int conv_tc_max_ctas_per_sm(int cin, int cout, int t, int s, int mode) {
  const Variant* v = picked(cin, cout, t, s, mode);
  if (!v) return 0;
  return 1;
}

// Output-channel order of the weight image of CTA-pair variants (B rows = accumulator
// columns of the pair, both CTAs' halves together): within each group of g = 64 columns
// (one epilogue warp's), column 8j + 2m + b holds channel (g / 4) * m + 2j + b, so that a
// 16x256b TMEM fragment gives each thread g / 4 consecutive channels of its pixels (see the
// pair epilogue).  Other variants keep the natural order.
int out_channel_of_column(int n, int g) {
  const int c = n % g, j = c / 8, m = (c % 8) / 2, b = c % 2;
  return (n / g) * g + (g / 4) * m + 2 * j + b;
}

// Weight image for the tcgen05 B operand: per C_out slice, per K-block (tap-major,
// then channel chunk), NCTA rows of ROWB bytes, K-major, with the 128B/64B swizzle
// applied exactly as the MMA reads it from a 1024-byte-aligned shared buffer.
void conv_tc_build_wimg(int cin, int cout, int t, int s, int mode, const float* w, const float* bias,
                        uint16_t* out, int q, float* wscale) {
  const Variant* v = picked(cin, cout, t, s, mode, q);
  if (!v) return;
  if (q >= 2) {
    // e4m3 codes, one scale per output channel: wscale[c] = max |w[., ., ., c]| / 448 (the
    // largest e4m3 magnitude), code = e4m3(w / wscale[c]) rounded to nearest even.  Layout
    // as the fp16 image (tap-major K-blocks of ch input channels, one 128-byte row per
    // output channel, 16-byte chunks swizzled), one byte per element.
    const int ch = v->ch, rowb = ch, ncta = v->ncta, nsplit = cout / ncta, nch = cin / ch, nkb = 9 * nch;
    std::vector<float> sc(cout);
    for (int c = 0; c < cout; ++c) {
      float amax = 0.f;
      for (int k = 0; k < 9 * cin; ++k) amax = std::max(amax, std::fabs(w[(size_t)k * cout + c]));
      sc[c] = amax > 0.f ? amax / 448.f : 1.f;
      if (wscale) wscale[c] = sc[c];
    }
    uint8_t* bytes = reinterpret_cast<uint8_t*>(out);
    const size_t split_bytes = (size_t)v->w_bytes;
    for (int sp = 0; sp < nsplit; ++sp) {
      uint8_t* img = bytes + sp * split_bytes;
      std::memset(img, 0, split_bytes);
      for (int kb = 0; kb < nkb; ++kb)
        for (int n = 0; n < ncta; ++n) {
          const int co = v->pair ? out_channel_of_column(sp * ncta + n, v->ncol) : sp * ncta + n;
          for (int k = 0; k < ch; ++k) {
            const int tap = kb / nch, ci = (kb % nch) * ch + k;
            const float val = w[((size_t)tap * cin + ci) * cout + co] / sc[co];
            const int qq = k / 16, within = k % 16;
            const int pq = rowb == 128 ? (qq ^ (n & 7)) : (qq ^ ((n >> 1) & 3));
            img[(size_t)kb * ncta * rowb + (size_t)n * rowb + pq * 16 + within] =
                (uint8_t)__nv_cvt_float_to_fp8(val, __NV_SATFINITE, __NV_E4M3);
          }
        }
    }
    return;
  }
  if (v->win == 2 && cin == 32) {
    // pair windows: block ky*2 + tap; K element k = (dx, c) of a pixel pair; tap 0 (pair
    // offset -1) holds kx = 0 in its odd half, tap 1 (offset 0) kx = 1 / kx = 2 in its halves
    const int ncta = v->ncta, nsplit = cout / ncta, rowb = v->ch * 2;
    const size_t split_elems = (size_t)v->w_bytes / 2;
    for (int sp = 0; sp < nsplit; ++sp) {
      uint16_t* img = out + sp * split_elems;
      std::memset(img, 0, (size_t)v->w_bytes);
      for (int kb = 0; kb < 6; ++kb) {
        const int ky = kb / 2, tap = kb % 2;
        for (int n = 0; n < ncta; ++n) {
          const int co = v->pair ? out_channel_of_column(sp * ncta + n, v->ncol) : sp * ncta + n;
          for (int k = 0; k < v->ch; ++k) {
            const int dx = k / cin, c = k % cin;
            const int kx = tap == 0 ? (dx == 1 ? 0 : -1) : 1 + dx;
            const float val = kx < 0 ? 0.f : w[((size_t)(ky * 3 + kx) * cin + c) * cout + co];
            const int q = (k * 2) / 16, within = (k * 2) % 16;
            const int pq = q ^ (n & 7);
            const size_t byte = (size_t)kb * ncta * rowb + (size_t)n * rowb + pq * 16 + within;
            __half h = __float2half_rn(val);
            img[byte / 2] = *reinterpret_cast<uint16_t*>(&h);
          }
        }
      }
    }
    return;
  }
  const bool manual = cin < 16;
  const int ch = v->ch, rowb = ch * 2, ncta = v->ncta, nsplit = cout / ncta;
  const int nch = manual ? 1 : cin / ch, nkb = manual ? 1 : 9 * nch;
  const size_t split_elems = (size_t)v->w_bytes / 2;
  for (int sp = 0; sp < nsplit; ++sp) {
    uint16_t* img = out + sp * split_elems;
    std::memset(img, 0, (size_t)v->w_bytes);
    for (int kb = 0; kb < nkb; ++kb) {
      for (int n = 0; n < ncta; ++n) {
        const int co = v->pair ? out_channel_of_column(sp * ncta + n, v->ncol) : sp * ncta + n;
        for (int k = 0; k < ch; ++k) {
          float val = 0.f;
          if (manual) {
            // K slot k: ky = k / krun, element t = k % krun = kx * cin + c of that ky's run;
            // slots 3*krun and 3*krun + 1 carry the bias as fp16 high and low parts
            const int krun = ((3 * cin + 1) / 2) * 2;
            if (k < 3 * krun) {
              const int ky = k / krun, tt = k % krun;
              if (tt < 3 * cin) val = w[((size_t)(ky * 3 + tt / cin) * cin + tt % cin) * cout + co];
            } else if (3 * krun + 2 <= ch && k < 3 * krun + 2) {
              const float hi = __half2float(__float2half_rn(bias[co]));
              val = k == 3 * krun ? hi : bias[co] - hi;
            }
          } else {
            const int tap = kb / nch, ci = (kb % nch) * ch + k;
            val = w[((size_t)tap * cin + ci) * cout + co];
          }
          const int q = (k * 2) / 16, within = (k * 2) % 16;
          const int pq = rowb == 128 ? (q ^ (n & 7)) : (q ^ ((n >> 1) & 3));
          const size_t byte = (size_t)kb * ncta * rowb + (size_t)n * rowb + pq * 16 + within;
          __half h = __float2half_rn(val);
          img[byte / 2] = *reinterpret_cast<uint16_t*>(&h);
        }
      }
    }
  }
}

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode() {
  static PFN_encodeTiled fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  }
  return fn;
}

// 4-D tiled map over an NHWC fp16 cache: dims {C, W, H, N}; box {CH, T*S, rows*S, 1}
// with element strides {1, S, S, 1} so that one box is the strided im2col slice of one
// tap for one tile.
cudaError_t conv_tc_make_tmap(CUtensorMap* map, const void* src, int n, int hx, int wx, int cin, int t, int s,
                              int mode, int q) {
  const Variant* v = nullptr;
  for (const auto& c : variants())
    if (c.cin == cin && c.t == t && c.s == s && c.win == (mode & 7) && (q >= 2) == (c.q >= 2)) { v = &c; break; }
  if (!v) return cudaErrorInvalidValue;
  if (q >= 2) {
    // e4m3 cache [n][hx][wx][cin] bytes, row windows: 10 px x t rows of ch channels per box
    PFN_encodeTiled enc = get_encode();
    if (!enc) return cudaErrorNotSupported;
    cuuint64_t dims[4] = {(cuuint64_t)cin, (cuuint64_t)wx, (cuuint64_t)hx, (cuuint64_t)n};
    cuuint64_t strides[3] = {(cuuint64_t)cin, (cuuint64_t)wx * cin, (cuuint64_t)hx * wx * cin};
    cuuint32_t box[4] = {(cuuint32_t)v->ch, 10u, (cuuint32_t)v->box_rows, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(src), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     v->ch == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
  }
  const bool win = v->win != 0;
  if (cin < 16) {
    // first layer: the image cache as [N][H][W*cin] fp16, one box = one M-tile's window
    PFN_encodeTiled enc = get_encode();
    if (!enc) return cudaErrorNotSupported;
    cuuint64_t dims[3] = {(cuuint64_t)wx * cin, (cuuint64_t)hx, (cuuint64_t)n};
    cuuint64_t strides[2] = {(cuuint64_t)wx * cin * 2, (cuuint64_t)hx * wx * cin * 2};
    cuuint32_t box[3] = {(cuuint32_t)v->win_cols, (cuuint32_t)v->win_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(src), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
  }
  PFN_encodeTiled enc = get_encode();
  if (!enc) return cudaErrorNotSupported;
  if (v->win == 2 && cin == 64) {
    // strided windows: plain pixels, element stride 2 in x and y, 10 px x box_rows per box
    cuuint64_t pd[4] = {(cuuint64_t)cin, (cuuint64_t)wx, (cuuint64_t)hx, (cuuint64_t)n};
    cuuint64_t ps[3] = {(cuuint64_t)cin * 2, (cuuint64_t)wx * cin * 2, (cuuint64_t)hx * wx * cin * 2};
    cuuint32_t pb[4] = {(cuuint32_t)v->ch, 20u, (cuuint32_t)(v->box_rows * 2), 1};
    cuuint32_t pe[4] = {1, 2, 2, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(src), pd, ps, pb, pe,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
  }
  if (v->win == 2) {
    // pixel pairs: [pair = 2 px x cin][wx/2][hx][n]; rows taken with element stride 2
    if (wx % 2 != 0 || 2 * cin != v->ch) return cudaErrorInvalidValue;
    cuuint64_t pd[4] = {(cuuint64_t)2 * cin, (cuuint64_t)wx / 2, (cuuint64_t)hx, (cuuint64_t)n};
    cuuint64_t ps[3] = {(cuuint64_t)cin * 4, (cuuint64_t)wx * cin * 2, (cuuint64_t)hx * wx * cin * 2};
    cuuint32_t pb[4] = {(cuuint32_t)v->ch, 10u, (cuuint32_t)(v->box_rows * 2), 1};
    cuuint32_t pe[4] = {1, 1, 2, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(src), pd, ps, pb, pe,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
  }
  cuuint64_t dims[4] = {(cuuint64_t)cin, (cuuint64_t)wx, (cuuint64_t)hx, (cuuint64_t)n};
  cuuint64_t strides[3] = {(cuuint64_t)cin * 2, (cuuint64_t)wx * cin * 2, (cuuint64_t)hx * wx * cin * 2};
  // window mode: 10 input px (8 output px + halo) x T rows; im2col: the strided tile itself
  cuuint32_t box[4] = {(cuuint32_t)v->ch, win ? 10u : (cuuint32_t)(t * s), (cuuint32_t)(v->box_rows * s), 1};
  cuuint32_t estr[4] = {1, (cuuint32_t)s, (cuuint32_t)s, 1};
  const CUtensorMapSwizzle swz = v->ch * 2 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(src), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t conv_tc_make_tmap_out(CUtensorMap* map, void* dst, int n, int ho, int wo, int cin, int cout, int t, int s,
                                  int mode) {
  const Variant* v = find_variant(cin, cout, t, s, mode);
  if (!v) return cudaErrorInvalidValue;
  std::memset(map, 0, sizeof(*map));
  if (!v->tstore) return cudaSuccess;  // this variant stores directly; the map is not read
  PFN_encodeTiled enc = get_encode();
  if (!enc) return cudaErrorNotSupported;
  // the destination cache [n][ho][wo][cout]; one box = one epilogue warp's 32 pixels
  cuuint64_t dims[4] = {(cuuint64_t)cout, (cuuint64_t)wo, (cuuint64_t)ho, (cuuint64_t)n};
  cuuint64_t strides[3] = {(cuuint64_t)cout * 2, (cuuint64_t)wo * cout * 2, (cuuint64_t)ho * wo * cout * 2};
  cuuint32_t box[4] = {(cuuint32_t)v->ncol, (cuuint32_t)v->obw, (cuuint32_t)(32 / v->obw), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapSwizzle swz = v->ncol * 2 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, dst, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_conv_tc(const ConvArgs& a, int mode, const CUtensorMap* map, const CUtensorMap* map_y, int grid_x,
                           cudaStream_t st, int q) {
  const Variant* v = find_variant(a.cin, a.cout, a.t, a.s, mode, q);
  // every variant loads through TMA; staged-output variants also store through map_y
  if (!v || map == nullptr || map_y == nullptr || a.cout > kMaxCout) return cudaErrorInvalidValue;
  static bool attr_done[64] = {};
  const int idx = (int)(v - variants().data());
  if (!attr_done[idx]) {
    cudaError_t e = cudaFuncSetAttribute(v->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, v->smem);
    if (e != cudaSuccess) return e;
    attr_done[idx] = true;
  }
  static int occ[64] = {};
  if (occ[idx] == 0) {
    int o = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, v->fn, v->threads, v->smem) != cudaSuccess || o < 1) o = 1;
    occ[idx] = o;
  }
  if (v->pair) {
    // 2-CTA clusters, as many as can be resident at once (the loop over M-tile pairs is
    // persistent, so every cluster must be running)
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(v->threads, 1, 1);
    cfg.dynamicSmemBytes = v->smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;  // occupancy query with the cluster shape only
    static int max_clusters[64] = {};
    if (max_clusters[idx] == 0) {
      cfg.gridDim = dim3(2 * (grid_x / 2 > 0 ? grid_x / 2 : 1), 1, 1);
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, v->fn, &cfg) != cudaSuccess || n < 1) n = 1;
      max_clusters[idx] = n;
    }
    int pairs = grid_x / 2;
    if (pairs > max_clusters[idx]) pairs = max_clusters[idx];
    if (pairs < 1) pairs = 1;
    cfg.gridDim = dim3(2 * pairs, 1, 1);
    cfg.numAttrs = 2;  // + programmatic dependent launch
    return cudaLaunchKernelEx(&cfg, v->fn, a, *map, *map_y);
  }
  // each CTA keeps one C_out slice: the grid is a multiple of the number of slices
  const int nsplit = a.cout / v->ncta;
  int gx = grid_x * occ[idx];
  gx -= gx % nsplit;
  if (gx < nsplit) gx = nsplit;
  // programmatic dependent launch: the kernel's prologue and weight copy overlap the tail of
  // the previous kernel of the stream (the kernel waits for it before reading its outputs)
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(gx, 1, 1);
  cfg.blockDim = dim3(v->threads, 1, 1);
  cfg.dynamicSmemBytes = v->smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, v->fn, a, *map, *map_y);
}

}  // namespace sb
