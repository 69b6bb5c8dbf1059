// sb_ptx.cuh -- thin inline-PTX wrappers for sm_100a: mbarriers with bounded waits,
// TMA tile loads, bulk copies and tcgen05 (TMEM alloc, MMA, commit, loads).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#define SB_DEV __device__ __forceinline__

// Sticky device error flags (OR-ed into the engine state's `error` word).
#define SB_ERR_TIMEOUT_FULL   0x01
#define SB_ERR_TIMEOUT_EMPTY  0x02
#define SB_ERR_TIMEOUT_ACC    0x04
#define SB_ERR_TIMEOUT_LOOKBK 0x08
#define SB_ERR_TIMEOUT_WGT    0x10
#define SB_ERR_BAD_TILE       0x20

// Limits of every spin-wait: 2 s of waiting on an mbarrier (SB_WAIT_NS), 2^24 polls with
// a short back-off on a global flag (SB_SPIN_LIMIT); both are orders of magnitude above
// any legitimate wait inside one kernel.
#define SB_WAIT_NS 2000000000ull
#define SB_SPIN_LIMIT (1u << 24)

namespace sb {

SB_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

SB_DEV uint32_t lane_id() { return threadIdx.x & 31; }
SB_DEV uint32_t warp_id() { return threadIdx.x >> 5; }

// ---------------------------------------------------------------- mbarrier
SB_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
SB_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
SB_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
SB_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
SB_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
SB_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for the phase with the given parity.  mbarrier.try_wait suspends the
// thread in hardware until the phase completes or a short system time limit passes, so
// the loop needs no extra back-off.  Returns false after SB_WAIT_NS of waiting (far above
// any legitimate wait inside one kernel) or as soon as *abort is set by another thread.
SB_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 15u) == 0) {
      if (*abort) return false;
      if (global_ns() - t0 > SB_WAIT_NS) return false;
    }
  }
}

// mbar_wait executed by a full warp with a warp-uniform result.
SB_DEV bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, abort);
  return __all_sync(0xFFFFFFFFu, ok);
}

// ---------------------------------------------------------------- proxies / fences
SB_DEV void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMA / bulk copies
SB_DEV void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                        int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
SB_DEV void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
SB_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
SB_DEV void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Tile store shared -> global through a tensor map (bulk async-group of the issuing thread).
// Elements of the box outside the tensor's extent are not written.
SB_DEV void tma_store_4d(const CUtensorMap* map, const void* smem_src, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
SB_DEV void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The issuing thread's bulk groups have finished reading their shared-memory sources.
SB_DEV void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// The issuing thread's bulk groups are complete (their global writes performed).
SB_DEV void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// 32-byte global accesses (sm_100): one full sector per lane.  p must be 32-byte aligned.
SB_DEV void st_global_v8(void* p, uint4 lo, uint4 hi) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(lo.x), "r"(lo.y),
               "r"(lo.z), "r"(lo.w), "r"(hi.x), "r"(hi.y), "r"(hi.z), "r"(hi.w)
               : "memory");
}
SB_DEV void ld_global_nc_v8(const void* p, uint4& lo, uint4& hi) {
  asm volatile("ld.global.nc.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(lo.x), "=r"(lo.y), "=r"(lo.z), "=r"(lo.w), "=r"(hi.x), "=r"(hi.y), "=r"(hi.z), "=r"(hi.w)
               : "l"(p));
}
SB_DEV void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- tcgen05
// Allocate `ncols` TMEM columns (power of two >= 32); the base address lands in *dst (smem).
// Executed by one full warp.
SB_DEV void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
SB_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
SB_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
SB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
SB_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (fp16 inputs, fp32 accumulate).
SB_DEV void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}
// Arrive once on `bar` when all prior tcgen05 async ops of this thread have completed.
SB_DEV void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// 32 lanes x 32 bit, 16 consecutive columns: thread i of the warp gets lane (base_lane + i).
SB_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
SB_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 16 lanes x 256 bits, four (eight) repetitions along the columns.  Thread t (k = t / 4,
// m = t % 4) holds, for repetition j: r[4j], r[4j+1] = lane base+k, columns 8j+2m, 8j+2m+1
// and r[4j+2], r[4j+3] = lane base+8+k, the same columns (checked on a B200 by a probe).
SB_DEV void tmem_ld16x256b4(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
SB_DEV void tmem_ld16x256b8(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Shared-memory matrix descriptor for tcgen05 (K-major operand, swizzled rows).
//   swz_mode: 2 = 128B swizzle (rows of 128 B), 4 = 64B swizzle (rows of 64 B).
//   sbo: byte distance between consecutive 8-row groups.
SB_DEV uint64_t smem_desc(uint32_t saddr, uint32_t sbo, uint32_t swz_mode) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);        // start address  [0,14)
  d |= (uint64_t)(16u >> 4) << 16;                 // leading byte offset (unused when swizzled)
  d |= (uint64_t)((sbo & 0x3FFFFu) >> 4) << 32;    // stride byte offset [32,46)
  d |= (uint64_t)1 << 46;                          // descriptor version (sm100)
  d |= (uint64_t)(swz_mode & 7u) << 61;            // layout / swizzle [61,64)
  return d;
}

// Instruction descriptor for kind::f16 with fp16 A/B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4)                       // D format: f32
         | (0u << 7) | (0u << 10)         // A, B format: f16
         | (0u << 15) | (0u << 16)        // A, B K-major
         | ((uint32_t)(N >> 3) << 17)     // N >> 3
         | ((uint32_t)(M >> 4) << 24);    // M >> 4
}

// ---------------------------------------------------------------- CTA pairs (cta_group::2)
// A 2-CTA cluster runs one M=256 tcgen05.mma: each CTA supplies 128 rows of A and half of
// the N rows of B from its own shared memory (same offsets), and holds its 128 rows of D
// in its own TMEM.  Only the even CTA (rank 0) issues MMAs and commits.
SB_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// All threads of both CTAs: release prior memory operations, wait for the other CTA.
SB_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the variable at shared::cta address `a` in CTA `rank`.
SB_DEV uint32_t mapa_shared(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
// Arrive on an mbarrier given by its shared::cluster address (default semantics: release
// at CTA scope).  A cluster-scope release would first wait until this thread's earlier
// global stores are visible device-wide; the callers only need their tcgen05 accesses
// ordered, which tcgen05.fence::before_thread_sync does, or earlier mbarrier completions.
SB_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
SB_DEV void tmem_alloc2(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
SB_DEV void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
SB_DEV void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
SB_DEV void mma_f16_ss2(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}
// The same with e4m3 A and B (kind::f8f6f4; format code 0 of the instruction descriptor is
// E4M3 there), fp32 accumulate; one instruction covers K = 32 (32 bytes of each row).
SB_DEV void mma_f8_ss2(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accum)
      : "memory");
}
// Two floats -> two e4m3 codes (round to nearest even, saturated to +-448), x in the low byte.
SB_DEV uint16_t e4m3x2_of(float x, float y) {
  return (uint16_t)__nv_cvt_float2_to_fp8x2(make_float2(x, y), __NV_SATFINITE, __NV_E4M3);
}
// Two e4m3 codes (low byte first) -> two floats (exact: e4m3 values are fp16 values).
SB_DEV float2 float2_of_e4m3x2(uint16_t v) {
  const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)v, __NV_E4M3);
  return __half22float2(*reinterpret_cast<const __half2*>(&h));
}

// Arrive once on the mbarrier at shared::cluster address `bar` (this CTA's or the peer's)
// when all prior cta_group::2 tcgen05 ops of this thread have completed.
SB_DEV void mma_commit2(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
// Arrive once on the mbarrier at the same shared-memory offset as `bar` in both CTAs of
// the pair when all prior cta_group::2 tcgen05 ops of this thread have completed.
SB_DEV void mma_commit2_both(const uint64_t* bar) {
  const uint16_t mask = 3;
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "h"(mask)
               : "memory");
}
// Tile load into this CTA's shared memory whose completed bytes are counted on the mbarrier
// at shared::cluster address `bar` (the pair leader's), for cta_group::2 MMAs.
SB_DEV void tma_load_4d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// ---------------------------------------------------------------- misc
SB_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
SB_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace sb
