// Thin inline-PTX wrappers for the sm_100a features the W8A8 kernels use:
// mbarriers with bounded waits, TMA tile loads/stores, and tcgen05 (TMEM
// allocation, MMA issue, commit, TMEM->register loads).
//
// Every spin on an mbarrier is bounded: after kSpinLimitNs of wall time the
// waiter records an error code in a device word supplied by the host, raises a
// CTA-local abort flag, and returns false so that every role of the CTA can
// fall through to teardown (TMEM is always freed).  No path traps.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace w8a8 {

// Wall-clock bound on any single wait (ns).  A healthy wait in these kernels
// lasts microseconds; two seconds means a protocol bug.
constexpr uint64_t kSpinLimitNs = 2000000000ull;

// Error codes written to the device error word.
enum DeviceError : int {
  kDevOk = 0,
  kDevTimeoutFull = 1,      // MMA issuer waited too long for a TMA stage
  kDevTimeoutEmpty = 2,     // producer waited too long for a free stage
  kDevTimeoutTmemFull = 3,  // epilogue waited too long for an accumulator
  kDevTimeoutTmemEmpty = 4, // MMA issuer waited too long for a free accumulator
  kDevBadScaleBlock = 5,    // an MXFP8 scale block outside the caller's buffers
  kDevTimeoutPeer = 6,      // a peer GPU's flag did not arrive (fused all-gather)
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- dependent launch
// A kernel that produces a GEMM's operands (the quantisers) lets the GEMM
// grid launch early; the GEMM waits for the producer's completion (and its
// memory) before reading them.  Without a producer that triggers, the wait
// returns once the previous kernel on the stream has finished, as usual.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------------- peers
// Flags between GPUs: release / acquire at system scope.
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Barrier among the first n threads of the CTA (id 0 is __syncthreads').
__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity.  Returns false (and makes
// sure the CTA abort flag is raised) if the CTA is aborting or the wait ran
// past kSpinLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* err_word, int code) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(addr, parity)) return true;
    if ((i & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kSpinLimitNs) {
        *abort_flag = 1;
        if (err_word) atomicCAS(err_word, 0, code);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- clusters
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// ---------------------------------------------------------------- TMA
// Fetch the 128-byte line holding `p` into L2 (no register result).
__device__ __forceinline__ void prefetch_l2_line(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, uint64_t* bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 2-SM form: the data lands in this CTA's shared memory, the transaction
// bytes are counted on the barrier at `bar_cluster` (the pair leader's).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const void* tmap,
                                                 uint32_t bar_cluster, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}

// Untiled bulk copy global -> shared (both 16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* smem_src, int32_t x,
                                             int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y)
      : "memory");
}

// Untiled bulk copy shared -> global (16-byte aligned addresses, size a
// multiple of 16), in the thread's current bulk group.
__device__ __forceinline__ void bulk_store(void* gdst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst),
               "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void tma_store_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N bulk groups are still reading shared memory.
template <int N>
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void tma_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Element-wise add of a shared-memory tile into global memory (TMA
// reduction; s32 adds for an INT32 tensor map).  Tile elements outside the
// map's extent are not touched.
__device__ __forceinline__ void tma_reduce_add_2d(const void* tmap, const void* smem_src, int32_t x,
                                                  int32_t y) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          tmap),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y)
      : "memory");
}

// Make generic-proxy shared-memory writes visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Order this thread's completed async-proxy global writes with its later
// generic-proxy operations.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
template <uint32_t kCols, int CG = 1>
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem) {
  static_assert(kCols >= 32 && (kCols & (kCols - 1)) == 0 && kCols <= 512, "bad TMEM size");
  if constexpr (CG == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "n"(kCols)
                 : "memory");
  } else {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "n"(kCols)
                 : "memory");
  }
}

template <uint32_t kCols, int CG = 1>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr) {
  if constexpr (CG == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "n"(kCols)
                 : "memory");
  } else {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "n"(kCols)
                 : "memory");
  }
}

template <int CG = 1>
__device__ __forceinline__ void tmem_relinquish() {
  if constexpr (CG == 1) {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  } else {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T for one 128 x N x 32 step.
// kKind: 0 = kind::i8 (s32 accumulate), 1 = kind::f8f6f4 (f32 accumulate).
template <int kKind>
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  if constexpr (kKind == 0) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// 2-SM MMA (issued by the pair leader): M = 256 rows, half from each CTA's
// shared memory at the same offsets; D lands in both CTAs' TMEM.
template <int kKind>
__device__ __forceinline__ void umma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  if constexpr (kKind == 0) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// Block-scaled MMA, kind::mxf8f6f4 (e4m3 x e4m3, one e8m0 scale per 32 K
// elements per row), scale factors read from TMEM.  CG = 2: the pair's MMA,
// issued by the leader; each CTA's TMEM holds the scales of its own 128 rows
// of A and of all N columns of B at the same addresses.
template <int CG = 1>
__device__ __forceinline__ void umma_mx(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                       uint32_t accumulate) {
  if constexpr (CG == 1) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
            d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
            d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
        : "memory");
  }
}

// Shared -> TMEM copy of a 32 x 16 B block, replicated into the four 32-lane
// quadrants (the scale-factor layout of a 128-row block).  CG = 2 (issued by
// the pair's leader): each CTA's block, at the same shared-memory offset, into
// its own TMEM at the same address.
template <int CG = 1>
__device__ __forceinline__ void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  if constexpr (CG == 1) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
                 : "memory");
  } else {
    asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
                 : "memory");
  }
}

// Descriptor of a 32-row x 16-byte shared-memory block with no swizzle: 8-row
// core matrices of 128 contiguous bytes, 128 B apart (stride byte offset).
__device__ __forceinline__ uint64_t smem_desc_sf(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(128u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  return d;
}

// Instruction descriptor of the block-scaled MMA: E4M3 x E4M3, UE8M0 scales,
// both operands K-major, sf_id selects the byte (K sub-block) of each scale
// word for A and B.
__host__ __device__ constexpr uint32_t make_idesc_mx(int m, int n, uint32_t sf_id) {
  return (sf_id << 4)                                  // B scale factor id
         | (static_cast<uint32_t>(n >> 3) << 17)        // N >> 3
         | (1u << 23)                                   // scale format: UE8M0
         | (static_cast<uint32_t>(m >> 4) << 24)        // M >> 4
         | (sf_id << 29);                               // A scale factor id
}

// Arrive on the barrier at shared::cluster address `bar_cluster` (this CTA's
// or the peer's) once all prior 2-SM MMAs of this thread have completed.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          bar_cluster)
      : "memory");
}

// Arrive on an mbarrier once every tcgen05.mma issued so far by this thread
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzling: rows of 128 bytes, 8-row (1024 B) swizzle atoms
// stacked along M/N.  Fields (sm100 layout): start address >> 4 in [0,14),
// leading byte offset >> 4 in [16,30) (unused for swizzled K-major, set to 1),
// stride byte offset >> 4 in [32,46) = 1024 B between 8-row groups,
// descriptor version 1 in [46,48), layout type 2 (128B swizzle) in [61,64).
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor for a dense 128 x N MMA with both operands K-major.
// kKind 0: s8 x s8 -> s32; kKind 1: e4m3 x e4m3 -> f32.
template <int kKind>
__host__ __device__ constexpr uint32_t make_idesc(int m, int n) {
  return (kKind == 0 ? (2u << 4) : (1u << 4))           // D format: s32 / f32
         | (kKind == 0 ? (1u << 7) : 0u)                 // A: signed int8 / e4m3
         | (kKind == 0 ? (1u << 10) : 0u)                // B: signed int8 / e4m3
         | (static_cast<uint32_t>(n >> 3) << 17)         // N >> 3
         | (static_cast<uint32_t>(m >> 4) << 24);        // M >> 4
}

}  // namespace w8a8
