// Shared device helpers for the sm_100a kernels: mbarriers, TMA, tcgen05 (UMMA + TMEM),
// programmatic dependent launch, and small numeric utilities. Inline PTX only; no library.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define TTS_DEV __device__ __forceinline__

namespace tts {

// ------------------------------------------------------------------ smem addressing
TTS_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier
TTS_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
TTS_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
TTS_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
TTS_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Generic-proxy shared-memory writes made visible to the async proxy (tcgen05.mma operands).
TTS_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// The same for global memory: generic stores that a TMA load (async proxy) reads later.
TTS_DEV void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
// Named barrier over `n` threads (whole warps) that also ANDs a predicate across them, so a
// group of warps takes one uniform branch after a bounded wait.
TTS_DEV bool bar_and(uint32_t id, uint32_t n, bool p) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.and.pred po, %2, %3, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(r)
      : "r"(uint32_t(p)), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}
TTS_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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
TTS_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Per-CTA timeline records, compiled only with -DTTS_TIMELINE (the library variant built by
// `build.py --timeline`; the product library has no trace code). A record is (kind, phase time,
// record time, SM id); kinds are kTl* | phase.
constexpr int kTlGemm = 0x100;   // | epilogue << 4 | phase
constexpr int kTlAttn = 0x200;   // | phase
constexpr int kTlNorm = 0x300;   // | phase (rms_norm; 0x310 | phase: the deferred norm's input)
// conv_nlc: | warp << 4 | field; fields 1..3 are per-role sums of wait (or busy) time
constexpr int kTlConv = 0x400;
constexpr int kTlEntry = 0, kTlReleased = 1, kTlMainDone = 2, kTlReduced = 3, kTlCta = 4,
              kTlMerged = 5, kTlEnd = 15;  // kTlCta: the phase time field holds blockIdx.x
// GEMM epilogue (warp 0): its first batch of rows reduced, every batch done
constexpr int kTlEpiFirst = 6, kTlEpiLoop = 7;
// attention: first score MMAs issued, first and last P handed to the output MMA
constexpr int kTlAttnFirstS = 6, kTlAttnFirstP = 7, kTlAttnLastP = 8;
// attention: the softmax warps past the dependency wait, and q staged for the first scores
constexpr int kTlAttnQWait = 9, kTlAttnQReady = 10;
#ifdef TTS_TIMELINE
constexpr unsigned kTimelineCap = 1u << 21;  // 64 MB of records (tracing build only)
extern __device__ unsigned long long g_timeline[kTimelineCap * 4];
extern __device__ unsigned g_timeline_n;
// A CTA's records go in one contiguous run (one atomic), so they pair up exactly; callers take
// their end time before calling, so the log's own cost is outside every phase.
template <int N>
TTS_DEV void timeline_recs(const int (&kind)[N], const uint64_t (&t)[N]) {
  const unsigned i = atomicAdd(&g_timeline_n, unsigned(N));
  unsigned sm;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
  const uint64_t now = global_ns();
#pragma unroll
  for (int k = 0; k < N; ++k) {
    if (i + k < kTimelineCap) {
      g_timeline[(i + k) * 4] = unsigned(kind[k]);
      g_timeline[(i + k) * 4 + 1] = t[k];
      g_timeline[(i + k) * 4 + 2] = now;
      g_timeline[(i + k) * 4 + 3] = sm;
    }
  }
}
#define TTS_TL_NOW() ::tts::global_ns()
#else
#define TTS_TL_NOW() 0ull
#endif

// Bounded wait: gives up after ~`limit_ns` of wall time (default 2 s) and reports false, so no
// kernel can spin forever; the caller records an error flag the host reads.
TTS_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > limit_ns) return false;
  }
}

// One lane of a converged warp (elect.sync). Asynchronous tcgen05/TMA/bulk-copy issue belongs
// to a converged warp with one elected lane: issued from a lone diverged lane, tcgen05.mma ran
// several times slower on B200 (measured ~220 ns vs ~65 ns per 128x48x16 MMA).
TTS_DEV bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\t"
      "elect.sync rx|px, %1;\n\t"
      "@px mov.s32 %0, 1;\n\t}"
      : "+r"(pred)
      : "r"(0xffffffffu));
  return pred != 0;
}
// Bounded wait by every lane of a warp with a warp-uniform result.
TTS_DEV bool mbar_wait_warp(uint64_t* bar, uint32_t parity);

TTS_DEV bool mbar_wait_warp(uint64_t* bar, uint32_t parity) {
  const bool ok = mbar_wait(bar, parity);
  return __all_sync(0xffffffffu, ok);
}

// ------------------------------------------------------------------ TMA
TTS_DEV void tma_prefetch_desc(const void* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(desc)) : "memory");
}
TTS_DEV void tma_load_2d(void* smem_dst, const void* desc, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
TTS_DEV void tma_load_2d_hint(void* smem_dst, const void* desc, uint64_t* bar, int c0, int c1,
                              uint64_t hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(hint)
      : "memory");
}
TTS_DEV void tma_load_4d(void* smem_dst, const void* desc, uint64_t* bar, int c0, int c1, int c2,
                         int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}
TTS_DEV void tma_load_3d(void* smem_dst, const void* desc, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// Shared -> global tile store (elements outside the tensor map's extents are not written);
// tracked by the issuing thread's bulk async-groups.
TTS_DEV void tma_store_3d(const void* desc, const void* smem_src, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(desc)),
      "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
TTS_DEV void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// This thread's committed bulk stores have finished reading their shared-memory sources.
TTS_DEV void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// This thread's committed bulk stores are complete (written to global memory).
TTS_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Prefetch `bytes` (a multiple of 16, from a 16-byte aligned address) into L2; no completion
// to wait for.
// One contiguous global -> shared copy by the bulk-copy engine (no multicast): both addresses
// 16-byte aligned, `bytes` a multiple of 16; completes on `bar`'s transaction count.
TTS_DEV void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(smem_dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
TTS_DEV void l2_prefetch_bulk(const void* src, uint32_t bytes, uint64_t policy) {
  asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(
                   reinterpret_cast<uint64_t>(src)),
               "r"(bytes), "l"(policy)
               : "memory");
}
// L2 eviction-priority policies for streamed (read once) and reused operands.
TTS_DEV uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
TTS_DEV uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ------------------------------------------------------------------ PDL
TTS_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
TTS_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// A load with acquire semantics at GPU scope (pairs with a writer's fence + atomic).
TTS_DEV unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// ------------------------------------------------------------------ thread-block clusters
TTS_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// All threads of all CTAs in the cluster; release/acquire orders shared-memory writes.
TTS_DEV void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Reads 16 bytes at the same shared-memory offset in CTA `rank` of the cluster (DSMEM).
TTS_DEV float4 ld_dsmem_f4(const void* local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote)
               : "memory");
  return v;
}

// ------------------------------------------------------------------ tcgen05
// TMEM allocation is warp-collective; the allocated base address is written to smem.
TTS_DEV void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
TTS_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
TTS_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
TTS_DEV void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
TTS_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (f16 inputs, f32 accumulate).
TTS_DEV void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                      uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every previously issued tcgen05.mma of this thread has completed.
TTS_DEV void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// ---- CTA pairs (cta_group::2): the even CTA of a 2-CTA cluster issues M = 256 MMAs whose A
// rows and B rows are split between the two CTAs' shared memory (128 A rows and N/2 B rows
// each, at the same offsets) and whose accumulators land in both CTAs' TMEM (each its own 128
// lanes, all N columns). Allocation is collective: one warp with the same warp index in each
// CTA of the pair allocates, relinquishes and frees.
TTS_DEV void tmem_alloc_pair(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
TTS_DEV void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
TTS_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
TTS_DEV void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` (same offset) in every CTA of `cta_mask` once the pair MMAs issued so far
// have completed.
TTS_DEV void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}
// The shared::cluster address of `local` (an address in this CTA's shared memory) in CTA
// `rank` of the cluster.
TTS_DEV uint32_t cluster_addr(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}
// Arrive on an mbarrier of any CTA of the cluster, releasing this thread's prior writes at
// cluster scope.
TTS_DEV void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                   bar_cluster_addr)
               : "memory");
}
// 2D tile load into this CTA's shared memory whose completion is counted on an mbarrier in
// either CTA of the pair (`bar_cluster_addr`, a shared::cluster address).
TTS_DEV void tma_load_2d_pair(void* smem_dst, const void* desc, uint32_t bar_cluster_addr, int c0,
                              int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(bar_cluster_addr), "r"(c0), "r"(c1)
      : "memory");
}

// Instruction descriptor for kind::f16 with f16 A and B, f32 D, both K-major.
// Bits: [4,6) D format (1 = f32); [7,10) A fmt (0 = f16); [10,13) B fmt; bit 15/16 major
// (0 = K); [17,23) N >> 3; [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

// Shared-memory matrix descriptor (tcgen05 form, version 1 at bit 46).
// layout: 0 = no swizzle (core matrices 8 rows x 16 B), 2 = 128-byte swizzle.
TTS_DEV uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                           uint32_t layout) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3FFF);
  d |= uint64_t((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= uint64_t((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(layout & 7) << 61;
  return d;
}
// K-major operand tile written by TMA with 128-byte swizzle: rows of 64 f16 (128 B),
// 8-row groups 1024 B apart.
TTS_DEV uint64_t desc_k_sw128(uint32_t saddr) { return smem_desc(saddr, 16, 1024, 2); }
// K-major operand without swizzle where row r of an 8-channel slab sits at r * 16 bytes
// (8-row core matrices contiguous, SBO = 128 B) and consecutive 8-channel slabs are
// `slab_bytes` apart (LBO). Any row offset is a plain 16-byte shift of the start address.
TTS_DEV uint64_t desc_k_interleave(uint32_t saddr, uint32_t slab_bytes) {
  return smem_desc(saddr, slab_bytes, 128, 0);
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
TTS_DEV void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Four 32x32b.x16 loads (e.g. the same columns of four accumulators) behind one wait, so their
// latencies overlap: v[i][c] = column c of address a_i.
TTS_DEV void tmem_ld16x4(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, float (*v)[16]) {
  uint32_t r[4][16];
#define TTS_LD16(I, A)                                                                        \
  asm volatile(                                                                               \
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"                                                \
      " {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"                      \
      : "=r"(r[I][0]), "=r"(r[I][1]), "=r"(r[I][2]), "=r"(r[I][3]), "=r"(r[I][4]),            \
        "=r"(r[I][5]), "=r"(r[I][6]), "=r"(r[I][7]), "=r"(r[I][8]), "=r"(r[I][9]),            \
        "=r"(r[I][10]), "=r"(r[I][11]), "=r"(r[I][12]), "=r"(r[I][13]), "=r"(r[I][14]),       \
        "=r"(r[I][15])                                                                        \
      : "r"(A))
  TTS_LD16(0, a0);
  TTS_LD16(1, a1);
  TTS_LD16(2, a2);
  TTS_LD16(3, a3);
#undef TTS_LD16
  // the wait names every destination register, so no use of them moves above it
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0][0]), "+r"(r[0][1]), "+r"(r[0][2]), "+r"(r[0][3]), "+r"(r[0][4]),
                 "+r"(r[0][5]), "+r"(r[0][6]), "+r"(r[0][7]), "+r"(r[0][8]), "+r"(r[0][9]),
                 "+r"(r[0][10]), "+r"(r[0][11]), "+r"(r[0][12]), "+r"(r[0][13]),
                 "+r"(r[0][14]), "+r"(r[0][15]), "+r"(r[1][0]), "+r"(r[1][1]), "+r"(r[1][2]),
                 "+r"(r[1][3]), "+r"(r[1][4]), "+r"(r[1][5]), "+r"(r[1][6]), "+r"(r[1][7]),
                 "+r"(r[1][8]), "+r"(r[1][9]), "+r"(r[1][10]), "+r"(r[1][11]),
                 "+r"(r[1][12]), "+r"(r[1][13]), "+r"(r[1][14]), "+r"(r[1][15]),
                 "+r"(r[2][0]), "+r"(r[2][1]), "+r"(r[2][2]), "+r"(r[2][3]), "+r"(r[2][4]),
                 "+r"(r[2][5]), "+r"(r[2][6]), "+r"(r[2][7]), "+r"(r[2][8]), "+r"(r[2][9]),
                 "+r"(r[2][10]), "+r"(r[2][11]), "+r"(r[2][12]), "+r"(r[2][13]),
                 "+r"(r[2][14]), "+r"(r[2][15]), "+r"(r[3][0]), "+r"(r[3][1]), "+r"(r[3][2]),
                 "+r"(r[3][3]), "+r"(r[3][4]), "+r"(r[3][5]), "+r"(r[3][6]), "+r"(r[3][7]),
                 "+r"(r[3][8]), "+r"(r[3][9]), "+r"(r[3][10]), "+r"(r[3][11]),
                 "+r"(r[3][12]), "+r"(r[3][13]), "+r"(r[3][14]), "+r"(r[3][15])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < 16; ++c) v[i][c] = __uint_as_float(r[i][c]);
}

// ------------------------------------------------------------------ numerics
// Monotone map of a float onto u32 so that an unsigned max picks the larger float.
TTS_DEV uint32_t float_order_key(float f) {
  uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
TTS_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
TTS_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace tts
