// Shared device helpers for the quantfun2-b200 kernels (sm_100a only).
//
// Thin inline-PTX wrappers around the Blackwell primitives the attention and
// GEMM kernels use: mbarriers with bounded waits, bulk async copies
// (cp.async.bulk / cp.async.bulk.tensor), and the tcgen05 tensor-core family
// (TMEM alloc, mma, commit, ld/st, fences).  Descriptor bit layouts follow the
// public PTX ISA (tcgen05 "shared memory descriptor" and "instruction
// descriptor" tables).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "../../include/qf2b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "quantfun2-b200 kernels are written for sm_100a only"
#endif

#define QF2_DEV __device__ __forceinline__
#define QF2_DEV_HOST_INLINE __host__ __device__ __forceinline__

namespace qf2 {

// ----------------------------------------------------------------------------
// Error flag written by bounded waits.  Kernels that spin on an mbarrier take a
// pointer to a device status word; on timeout they store a code there and
// unwind instead of spinning forever.
// ----------------------------------------------------------------------------
enum : int {
  kDevOk = 0,
  kDevTimeoutProducer = 1,
  kDevTimeoutMma = 2,
  kDevTimeoutSoftmax = 3,
  kDevTimeoutEpilogue = 4,
  kDevBadLaunch = 5,
  kDevBadIndex = 6,   // an index argument outside its range (the access was skipped)
  kDevTimeoutConvert = 7,
};

// ~2 s at 1.9 GHz; each wait gives up after this many SM clocks.
constexpr long long kWaitClocks = 4000000000LL;

QF2_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

QF2_DEV uint32_t lane_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(r));
  return r;
}

QF2_DEV bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------- mbarrier --
QF2_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

QF2_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

QF2_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

QF2_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

QF2_DEV bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on the phase with the given parity: gives up after `limit` SM clocks.
// Returns false on timeout.
QF2_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, long long limit = kWaitClocks) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(a, parity)) return true;
    if (clock64() - t0 > limit) return false;
  }
}

// ------------------------------------------------------- CTA pairs (2-SM) --
// Rank of this CTA in its cluster.
QF2_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared::cluster address of the object at local shared address `addr` in CTA `rank`.
QF2_DEV uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Arrive (release, cluster scope) on an mbarrier given by a shared::cluster address.
QF2_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// All threads of all CTAs of the cluster.
QF2_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The two halves of cluster_sync, for threads that have work to do in between (every
// thread of every CTA of the cluster arrives once per phase, warp-convergent).
QF2_DEV void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
QF2_DEV void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Loads from another CTA's shared memory (shared::cluster address from mapa_shared).
QF2_DEV double ld_dsmem_f64(uint32_t cluster_addr) {
  double v;
  asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(cluster_addr) : "memory");
  return v;
}
QF2_DEV float ld_dsmem_f32(uint32_t cluster_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
  return v;
}

// 2-D tiled TMA load into this CTA's shared memory whose completion is counted on an
// mbarrier of either CTA of the pair (shared::cluster address).  No multicast.
QF2_DEV void tma_load_2d_pair(void* smem_dst, const void* tmap, int32_t x, int32_t y, uint32_t bar_cluster_addr) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(bar_cluster_addr)
      : "memory");
}

QF2_DEV void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
QF2_DEV void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
QF2_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Arrive on the mbarrier at a shared::cluster address once every tcgen05 operation of
// the pair issued so far by this thread has completed.
QF2_DEV void tc_commit_pair(uint32_t bar_cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster_addr)
               : "memory");
}

// M256 pair MMAs: A rows 0-127 / B rows (N half 0) from the issuing CTA's shared memory,
// A rows 128-255 / B N half 1 from the peer's at the same offsets; D split across the
// two CTAs' TMEM (128 lanes each).
QF2_DEV void mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
QF2_DEV void mma_f8f6f4_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// ------------------------------------------------------------- bulk copies --
// 1-D bulk copy global -> shared, completion counted on an mbarrier (tx bytes).
QF2_DEV void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2-D tiled TMA load (no multicast).
QF2_DEV void tma_load_2d(void* smem_dst, const void* tmap, int32_t x, int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled TMA load (no multicast).
QF2_DEV void tma_load_3d(void* smem_dst, const void* tmap, int32_t x, int32_t y, int32_t z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(smem_dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// 4-D tiled TMA load (no multicast).
QF2_DEV void tma_load_4d(void* smem_dst, const void* tmap, int32_t x, int32_t y, int32_t z, int32_t w, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}

// L2 eviction-priority policies for the cache-hinted loads below (the whole access
// range gets the priority).
QF2_DEV uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
QF2_DEV uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 4-D tiled TMA load (no multicast) with an L2 eviction-priority hint.
QF2_DEV void tma_load_4d_hint(void* smem_dst, const void* tmap, int32_t x, int32_t y, int32_t z, int32_t w,
                              uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// 2-D tiled TMA store shared -> global (bulk group completion); out-of-bounds parts of
// the box are not written.
QF2_DEV void tma_store_2d(const void* tmap, const void* smem_src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
// 1-D bulk copy shared -> global (bulk group completion); both addresses 16-byte
// aligned, size a multiple of 16.
QF2_DEV void bulk_s2g(void* gmem_dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst), "r"(smem_u32(smem_src)),
               "r"(bytes)
               : "memory");
}
QF2_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's bulk groups still read their shared-memory source.
template <int N>
QF2_DEV void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until all of this thread's bulk groups have completed.
QF2_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

QF2_DEV void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy
// (tcgen05.mma operands written by threads).
QF2_DEV void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}


// ----------------------------------------------------------------- tcgen05 --
QF2_DEV void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}

QF2_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

QF2_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

QF2_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
QF2_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive on an mbarrier once every tcgen05 op previously issued by this
// thread has completed.
QF2_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle
// canonical layout: rows of 128 bytes, 8-row atoms of 1024 bytes (SBO), tile
// base 1024-byte aligned.  Advancing along K inside the atom is done by adding
// the byte offset to the start address.
QF2_DEV uint64_t sdesc_sw128_kmajor(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);      // start address
  d |= (uint64_t)(1) << 16;                          // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;                  // SBO: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                            // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                            // SWIZZLE_128B
  return d;
}

// Shared-memory matrix descriptor, MN-major operand in the 128-byte swizzle
// canonical layout: 128-byte rows along MN (64 x 16-bit elements), 8-row (K)
// atoms of 1024 bytes.  LBO = byte distance between successive 128-byte MN
// column blocks, SBO = byte distance between successive 8-row K groups.
QF2_DEV uint64_t sdesc_sw128_mnmajor(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor fields (kind::f16 / kind::f8f6f4 / kind::i8).
// c_fmt: 0=f16 1=f32 2=s32.  a/b_fmt: f16 kind 0=f16 1=bf16; f8f6f4 kind
// 0=e4m3 1=e5m2; i8 kind 0=u8 1=s8.  a/b_major: 0=K-major 1=MN-major.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t c_fmt, uint32_t a_fmt, uint32_t b_fmt, uint32_t a_major,
                                                  uint32_t b_major, uint32_t M, uint32_t N) {
  return (c_fmt << 4) | (a_fmt << 7) | (b_fmt << 10) | (a_major << 15) | (b_major << 16) | ((N >> 3) << 17) |
         ((M >> 4) << 24);
}

QF2_DEV void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

QF2_DEV void mma_f8f6f4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

QF2_DEV void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same with the A operand in tensor memory (M rows = TMEM lanes, K along the columns,
// two 16-bit elements per 32-bit column, the lower half holding the even K index).
QF2_DEV void mma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// TMEM -> registers: 32 lanes x 32 bits, 32 consecutive columns per thread.
QF2_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

QF2_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Registers -> TMEM: every one of 32 lanes x 8 consecutive columns set to v (the store's
// eight source registers are one aligned block, so wider forms would tie up more of them).
QF2_DEV void tmem_fill8(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr), "r"(v)
               : "memory");
}


QF2_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
QF2_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------ conversions --
// Two fp32 -> packed e4m3x2 (round to nearest even, saturate to +-448).
// Low byte holds `lo`.
QF2_DEV uint16_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(r) : "f"(lo), "f"(hi));
  return r;
}

// Packed two-lane fp32 arithmetic (sm_100 f32x2 instructions) and a three-way max.
QF2_DEV float2 fadd2(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}

// fma on two packed fp32 lanes (sm_100 f32x2 instruction)
QF2_DEV float2 ffma2(float2 a, float2 b, float2 c) {
  float2 r;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
}

QF2_DEV float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// ex2.approx: 2^x on the SFU.
QF2_DEV float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// e4m3 codes of four non-negative fp32 values already scaled by 2^-120, without the
// conversion unit: after the scaling the fp32 exponent field equals the e4m3 exponent
// (fp32 subnormals reproduce e4m3 subnormals), so the code is bits [27:20] of the fp32
// pattern rounded at bit 20 (half up).  Valid for scaled values below 464 * 2^-120.
// Shifting left by 4 puts each code in byte 3; three byte permutes gather them (first
// value in the lowest byte, like cvt.rn.satfinite.e4m3x2).
QF2_DEV uint32_t e4m3x4_from_scaled(float a, float b, float c, float d) {
  const uint32_t ua = (__float_as_uint(a) << 4) + 0x800000u, ub = (__float_as_uint(b) << 4) + 0x800000u;
  const uint32_t uc = (__float_as_uint(c) << 4) + 0x800000u, ud = (__float_as_uint(d) << 4) + 0x800000u;
  return __byte_perm(__byte_perm(ua, ub, 0x0073), __byte_perm(uc, ud, 0x0073), 0x5410);
}

template <typename T>
QF2_DEV float to_f32(T v);
template <>
QF2_DEV float to_f32<float>(float v) { return v; }
template <>
QF2_DEV float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
QF2_DEV float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T>
QF2_DEV T from_f32(float v);
template <>
QF2_DEV float from_f32<float>(float v) { return v; }
template <>
QF2_DEV __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
QF2_DEV __half from_f32<__half>(float v) { return __float2half_rn(v); }

}  // namespace qf2

// -------------------------------------------------- host: per-device setup --
#include <atomic>

// Raises `kernel`'s dynamic shared memory limit the first time it is launched on the
// current device (the attribute is per device; later calls cost one cudaGetDevice).
template <typename K>
inline cudaError_t qf2_set_smem_once(K* kernel, int bytes, std::atomic<uint64_t>* done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done->load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done->fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

// SM count of the current device, cached per device.
inline cudaError_t qf2_sm_count(int* out) {
  static std::atomic<int> cache[64];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int v = cache[dev & 63].load(std::memory_order_relaxed);
  if (v == 0) {
    e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    cache[dev & 63].store(v, std::memory_order_relaxed);
  }
  *out = v;
  return cudaSuccess;
}

// ------------------------------------------------------------- host: TMA --
#include <cudaTypedefs.h>

// Encodes a 4-D tiled tensor map (dims innermost first, byte strides of dims 1..3)
// with 128-byte swizzle; out-of-bounds elements read as zero.  Returns false when
// the driver entry point is unavailable or the encoder rejects the layout.
bool qf2_make_tmap_4d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[4],
                      const uint64_t strides_bytes[3], const uint32_t box[4]);
// Same without swizzle (rows land in shared memory as they are in global memory).
bool qf2_make_tmap_4d_noswizzle(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[4],
                                const uint64_t strides_bytes[3], const uint32_t box[4]);
// Same, 2-D (dims innermost first, byte stride of dim 1).
bool qf2_make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[2],
                      uint64_t stride_bytes, const uint32_t box[2]);

// Same, 2-D with 64-byte swizzle (output staging tiles of 64-byte rows).
bool qf2_make_tmap_2d_noswizzle(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[2],
                                uint64_t stride_bytes, const uint32_t box[2]);
bool qf2_make_tmap_2d_sw64(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t dims[2],
                           uint64_t stride_bytes, const uint32_t box[2]);

// Records the CUDA error behind a QF2_ERR_LAUNCH for qf2_last_error().
void qf2_record_cuda_error(cudaError_t e, const char* where);

// Host-side launch check shared by every entry point.
#define QF2_LAUNCH_CHECK()                                          \
  do {                                                              \
    cudaError_t _e = cudaGetLastError();                            \
    if (_e != cudaSuccess) {                                        \
      qf2_record_cuda_error(_e, __FILE__ ":" QF2_STR(__LINE__));    \
      return QF2_ERR_LAUNCH;                                        \
    }                                                               \
  } while (0)
#define QF2_STR2(x) #x
#define QF2_STR(x) QF2_STR2(x)
// Same, for a runtime call that returns cudaError_t.
#define QF2_CUDA_CHECK(call)                                        \
  do {                                                              \
    cudaError_t _e = (call);                                        \
    if (_e != cudaSuccess) {                                        \
      qf2_record_cuda_error(_e, __FILE__ ":" QF2_STR(__LINE__));    \
      return QF2_ERR_LAUNCH;                                        \
    }                                                               \
  } while (0)
