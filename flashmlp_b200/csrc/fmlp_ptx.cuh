// Thin inline-PTX layer for sm_100a: mbarriers with bounded waits, TMA tile loads,
// tcgen05 (TMEM alloc, MMA, commit, ld/st, fences) and UMMA descriptor builders.
//
// Every wait in this file is bounded: after FMLP_WAIT_LIMIT_NS of wall time on the
// GPU's global timer the wait gives up, raises the CTA-wide abort flag and records an
// error code in the caller-visible status word, so a broken pipeline ends the kernel
// instead of hanging the GPU.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#ifndef FMLP_WAIT_LIMIT_NS
#define FMLP_WAIT_LIMIT_NS 2000000000ull  // 2 s
#endif

namespace fmlp {

// Status codes a kernel can leave in the device status word (bit flags).
enum : uint32_t {
  kDevOk = 0,
  kDevTimeout = 1u,  // a bounded wait ran out
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ----------------------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
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

// Shared abort flag and the kernel's status word, used by every bounded wait.
struct WaitCtx {
  volatile uint32_t* abort_flag;  // in shared memory
  uint32_t* status;               // in global memory (may be null)
};

// Waits until the phase with the given parity of `bar` has completed. Returns false
// (and raises the abort flag) when the time limit passes or another thread aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const WaitCtx& ctx) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  uint64_t t0 = global_timer_ns();
  uint32_t n = 0;
  while (true) {
    if (mbar_try_wait(a, parity)) return true;
    if ((++n & 255u) == 0) {
      if (*ctx.abort_flag) return false;
      if (global_timer_ns() - t0 > FMLP_WAIT_LIMIT_NS) {
        *ctx.abort_flag = 1u;
        if (ctx.status) atomicOr(ctx.status, kDevTimeout);
        return false;
      }
    }
  }
}

// Warp-uniform wait: every lane polls and a vote makes the verdict uniform, so the warp
// leaves converged (needed before elect.sync). The fast path (phase already complete)
// is one try_wait and one vote: measured ~110 cycles, against ~255 for lane-0 polling
// plus a shuffle broadcast.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, const WaitCtx& ctx) {
  if (__all_sync(0xffffffffu, mbar_try_wait(smem_u32(bar), parity))) return true;
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, ctx));
}

// One lane of a converged warp returns true.
__device__ __forceinline__ bool elect_one() {
  uint32_t p;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "elect.sync _|P1, 0xffffffff;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}"
      : "=r"(p));
  return p != 0;
}

// ----------------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 3-D tiled load of one box into shared memory; completion is signalled on `bar`
// as transaction bytes. Coordinates are element indices, innermost first.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0,
                                            int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Untiled bulk copy of `bytes` contiguous bytes from global to shared memory (both
// addresses 16-byte aligned, size a multiple of 16); completion as transaction bytes.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Makes generic-proxy shared-memory writes visible to the async proxy (tensor core).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 8-bit forms (kind::f8f6f4, here e4m3 x e4m3 with fp32 accumulation): one K-step is 32
// elements (32 bytes of a 128-byte row, or 8 TMEM columns of 4 packed values).
__device__ __forceinline__ void mma_ss_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_ts_f8(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// TF32 forms (kind::tf32): fp32 operands used at TF32 precision (10-bit mantissa),
// fp32 accumulation; one K-step is 8 elements (32 bytes of a 128-byte row, or 8 TMEM
// columns for an A operand in TMEM).
__device__ __forceinline__ void mma_ss_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_ts_tf32(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05 async op issued so far by this thread is done.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Warp-wide: 32 lanes x 32 consecutive 32-bit columns -> 32 registers per thread.
// The wait is inside the same asm statement so no use of the registers can be
// scheduled before the load has landed.
__device__ __forceinline__ void tmem_ld32_sync(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// 16-column variant of tmem_ld32_sync.
__device__ __forceinline__ void tmem_ld16_sync(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Two 32-column loads (columns taddr0.. and taddr1..) completed by one wait.
__device__ __forceinline__ void tmem_ld32x2_sync(uint32_t taddr0, uint32_t taddr1, uint32_t (&r)[32],
                                                 uint32_t (&s)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
      "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(s[0]), "=r"(s[1]), "=r"(s[2]), "=r"(s[3]), "=r"(s[4]), "=r"(s[5]), "=r"(s[6]),
        "=r"(s[7]), "=r"(s[8]), "=r"(s[9]), "=r"(s[10]), "=r"(s[11]), "=r"(s[12]), "=r"(s[13]),
        "=r"(s[14]), "=r"(s[15]), "=r"(s[16]), "=r"(s[17]), "=r"(s[18]), "=r"(s[19]),
        "=r"(s[20]), "=r"(s[21]), "=r"(s[22]), "=r"(s[23]), "=r"(s[24]), "=r"(s[25]),
        "=r"(s[26]), "=r"(s[27]), "=r"(s[28]), "=r"(s[29]), "=r"(s[30]), "=r"(s[31])
      : "r"(taddr0), "r"(taddr1)
      : "memory");
}

// Asynchronous 16-column load: the registers are valid only after tmem_wait_ld_dep(r).
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Waits for every outstanding tcgen05.ld of this thread. The registers of the last
// asynchronous load are in/out operands, so no use of them can move above the wait.
__device__ __forceinline__ void tmem_wait_ld_dep(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]),
                 "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

// Waits for every outstanding tcgen05.ld of this thread; both register sets of two
// asynchronous loads are in/out operands, so no use of either can move above the wait.
__device__ __forceinline__ void tmem_wait_ld_dep2(uint32_t (&r)[16], uint32_t (&s)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]),
                 "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(s[0]), "+r"(s[1]), "+r"(s[2]), "+r"(s[3]),
                 "+r"(s[4]), "+r"(s[5]), "+r"(s[6]), "+r"(s[7]), "+r"(s[8]), "+r"(s[9]), "+r"(s[10]),
                 "+r"(s[11]), "+r"(s[12]), "+r"(s[13]), "+r"(s[14]), "+r"(s[15])
               :
               : "memory");
}

// Warp-wide: 8 registers per thread -> 32 lanes x 8 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}

// Warp-wide: 16 registers per thread -> 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ----------------------------------------------------------------------------- CTA pairs
// A cluster of two CTAs on two SMs runs one tcgen05.mma with M = 256 (cta_group::2): the
// MMA is issued by one thread of CTA rank 0, each CTA holds half of A (its 128 rows) and
// half of B (N/2 columns) at the same shared-memory offsets, and each CTA's TMEM receives
// its 128 rows of D. Barriers that the issuing thread waits on live in CTA 0 and collect
// arrivals and TMA transaction bytes from both CTAs; commits reach both CTAs' barriers.

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_index() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}

// Every thread of every CTA of the cluster (release / acquire at cluster scope).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The shared::cluster address of the same shared-memory location in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

// Arrive on a barrier of any CTA of the cluster. The handoffs through such barriers here
// are of TMEM contents, whose tcgen05.st / tcgen05.ld the arriving thread has waited for
// (tcgen05.wait) and ordered with tcgen05.fence::before_thread_sync; so the default
// semantics (release at CTA scope) suffice, and a cluster-scope release, which costs a
// memory barrier per arrival, is not used. Waits on such barriers are the plain ones.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// TMA load into this CTA's shared memory whose transaction bytes are counted on a barrier
// of either CTA of the pair (`bar_cluster_addr`, from mapa_shared). No multicast.
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* m, uint32_t bar_cluster_addr, int c0,
                                                 int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster_addr), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// TMEM allocation mirrored on both SMs of the pair: issued by the warp with the same
// index in both CTAs, which receive the same column address.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem, both CTAs] (+)= A[smem, 128 rows per CTA] * B[smem, N/2 columns per CTA]
__device__ __forceinline__ void mma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem, both CTAs] (+)= A[tmem, 128 lanes per CTA] * B[smem, N/2 columns per CTA]
__device__ __forceinline__ void mma_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on the barrier at this shared-memory offset in every CTA of `cta_mask`
// when the pair MMAs issued so far by this thread are done.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// ----------------------------------------------------------------------------- descriptors
// Instruction descriptor for tcgen05.mma kind::f16 with fp32 accumulation.
//   bits [4,6) D format (1 = f32); [7,10) A format, [10,13) B format (0 = f16, 1 = bf16);
//   bit 15 A major, bit 16 B major (0 = K-major, 1 = MN-major); [17,23) N>>3; [24,29) M>>4.
__host__ __device__ constexpr uint32_t make_idesc_f16(bool bf16, int M, int N, bool a_mn_major,
                                                      bool b_mn_major) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t(N) >> 3) << 17) | ((uint32_t(M) >> 4) << 24);
}

// Instruction descriptor for tcgen05.mma kind::tf32 (A and B format 2 = TF32), fp32
// accumulation; fields as in make_idesc_f16.
__host__ __device__ constexpr uint32_t make_idesc_tf32(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t(N) >> 3) << 17) | ((uint32_t(M) >> 4) << 24);
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), sm_100 version bit.
//   [0,14) start>>4, [16,30) LBO>>4, [32,46) SBO>>4, bit 46 version, [61,64) layout type.
// Tiles are laid out the way TMA writes a box whose inner extent is 128 bytes with
// CU_TENSOR_MAP_SWIZZLE_128B: rows of 128 B, 8-row (1024 B) swizzle atoms.
//  * K-major operand (rows = M or N, 64 K-elements per row): SBO = 1024 (next 8 rows);
//    LBO unused (1). A K-step of 16 elements inside a row is a +32 B start offset.
//  * MN-major operand (rows = K, 64 MN-elements per row): SBO = 1024 (next 8 K rows);
//    LBO = byte distance to the next 64-wide MN group.
__device__ __forceinline__ uint64_t make_sdesc_sw128(uint32_t smem_addr, uint32_t lbo_bytes,
                                                     uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= uint64_t((smem_addr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

// Shared-memory matrix descriptor without swizzle (layout type 0): the operand is tiled
// in 8 x 16-byte core matrices of 128 contiguous bytes. For an MN-major 16-bit operand a
// core matrix holds 8 MN elements (16 B) in each of 8 consecutive K rows; LBO is the byte
// distance between core matrices adjacent in K, SBO between those adjacent in MN.
__device__ __forceinline__ uint64_t make_sdesc_noswz(uint32_t smem_addr, uint32_t lbo_bytes,
                                                     uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= uint64_t((smem_addr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;
  return d;
}

// Shared-memory matrix descriptor for an MN-major 32-bit (TF32) operand: layout type 1
// (128-byte swizzle span with 32-byte atoms, what TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B), the only MN-major layout TF32 operands support.
// Rows of 128 bytes (32 MN elements); atoms of 4 K-rows, SBO = 512 bytes between them;
// LBO = byte distance to the next group of 32 MN elements. A K-step of 8 rows is +1024 B.
__device__ __forceinline__ uint64_t make_sdesc_mn32(uint32_t smem_addr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= uint64_t((smem_addr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((512u >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(1) << 61;
  return d;
}

// Warp-wide 8-column TMEM load (32 lanes x 8 consecutive 32-bit columns), waited.
__device__ __forceinline__ void tmem_ld8_sync(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr)
      : "memory");
}

// The same descriptor with its start address moved by `bytes` (a multiple of 16; shared
// addresses are below 2^18, so the 14-bit field never carries).
__host__ __device__ constexpr uint64_t sdesc_add(uint64_t desc, uint32_t bytes) {
  return desc + uint64_t(bytes >> 4);
}

// MMA issue rate: a tcgen05.mma inside a loop whose trip count or operands are only known
// at run time issues far below the tensor pipe's rate (measured: about 240 cycles per
// instruction on B200, whatever the tile), while a fully unrolled burst with descriptors
// formed by constant offsets from one base issues back to back (about 65 cycles for
// M=128,N=128,K=16 — 98% of peak). Every MMA sequence below is such a burst.

// ----------------------------------------------------------------------------- numerics
template <typename T>
struct Pack;
template <>
struct Pack<__nv_bfloat16> {
  static constexpr bool kBF16 = true;
  // Rounds (lo, hi) to bf16 (round-to-nearest-even) and packs lo in the low half.
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ __forceinline__ static float round(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
  }
  // The two values of a packed pair, widened back to fp32 (exact; integer ops only).
  __device__ __forceinline__ static float lo(uint32_t p) { return __uint_as_float(p << 16); }
  __device__ __forceinline__ static float hi(uint32_t p) { return __uint_as_float(p & 0xFFFF0000u); }
};
template <>
struct Pack<__half> {
  static constexpr bool kBF16 = false;
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ __forceinline__ static float round(float x) { return __half2float(__float2half_rn(x)); }
  __device__ __forceinline__ static float lo(uint32_t p) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(p & 0xFFFFu)));
  }
  __device__ __forceinline__ static float hi(uint32_t p) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(p >> 16)));
  }
};

template <>
struct Pack<float> {  // fp32 inputs (TF32 products): nothing is rounded between the products
  static constexpr bool kBF16 = false;
  __device__ __forceinline__ static float round(float x) { return x; }
};

// tanh on the SFU (one MUFU op), max relative error about 2^-11.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Logistic sigmoid via the identity sigma(z) = 0.5 * tanh(z / 2) + 0.5.
__device__ __forceinline__ float sigmoid_fast(float z) {
  return fmaf(0.5f, tanh_approx(0.5f * z), 0.5f);
}

// Two fp32 values in one 64-bit register (lo = first element) for sm_100's packed fp32
// instructions: one instruction performs the two IEEE round-to-nearest operations of the
// scalar forms, so results are bit-identical to them with half the issue slots.
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float f2_lo(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  (void)hi;
  return lo;
}
__device__ __forceinline__ float f2_hi(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  (void)lo;
  return hi;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {  // a * b + c
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {  // a - b
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Logistic sigmoid of a pair on the FMA/ALU pipes only (no SFU op), for activation warps
// whose MUFU unit is the bottleneck: sigma(z) = 1 / (1 + 2^x), x = -z log2(e).
//  * 2^x: x clamped to [-126, 126], split as x = n + f with n = round(x) by the
//    1.5 * 2^23 addition (n lands in the low mantissa bits of t), f in [-0.5, 0.5];
//    2^f by a degree-3 polynomial whose coefficients minimise the maximum relative error
//    on that interval (Remez exchange, max relative error 7.5e-5), and 2^n added to its
//    exponent field (bits(p) + (bits(t) << 23): the high bits of t's exponent shift out).
//  * 1 / d, d = 1 + 2^x in [1, 2^126]: first estimate from the bit pattern,
//    bits(r0) = 0x7EF311C2 - bits(d) (constant chosen to minimise the maximum relative
//    error of r0 over a binade, 5.1 %), then two Newton steps r <- r (2 - d r).
// Overall max relative error of sigma 8.1e-5 for z > -80 (tanh.approx-based: about 5e-4);
// below -87 the clamp keeps sigma at about 2^-126 instead of smaller.
__device__ __forceinline__ uint64_t sigmoid2_fma(uint64_t z) {
  const uint64_t x0 = mul2(z, f2(-1.4426950408889634f, -1.4426950408889634f));
  const uint64_t x = f2(fminf(fmaxf(f2_lo(x0), -126.f), 126.f), fminf(fmaxf(f2_hi(x0), -126.f), 126.f));
  const uint64_t magic = f2(12582912.f, 12582912.f);
  const uint64_t t = add2(x, magic);
  const uint64_t f = sub2(x, sub2(t, magic));
  uint64_t p = fma2(f2(0.0551716685295105f, 0.0551716685295105f), f, f2(0.2426111251115799f, 0.2426111251115799f));
  p = fma2(p, f, f2(0.6932609677314758f, 0.6932609677314758f));
  p = fma2(p, f, f2(0.9999280571937561f, 0.9999280571937561f));
  const uint32_t e0 = __float_as_uint(f2_lo(p)) + (__float_as_uint(f2_lo(t)) << 23);
  const uint32_t e1 = __float_as_uint(f2_hi(p)) + (__float_as_uint(f2_hi(t)) << 23);
  const uint64_t d = add2(f2(__uint_as_float(e0), __uint_as_float(e1)), f2(1.f, 1.f));
  const uint64_t nd = sub2(f2(0.f, 0.f), d);
  uint64_t r = f2(__uint_as_float(0x7EF311C2u - __float_as_uint(f2_lo(d))),
                  __uint_as_float(0x7EF311C2u - __float_as_uint(f2_hi(d))));
  const uint64_t two = f2(2.f, 2.f);
  r = mul2(r, fma2(nd, r, two));
  r = mul2(r, fma2(nd, r, two));
  return r;
}

// Activation codes shared with the host (see include/flashmlp_b200.h).
enum Act : int { kLinear = 0, kLeakyRelu = 1, kSilu = 2, kSigmoid = 3 };

}  // namespace fmlp
