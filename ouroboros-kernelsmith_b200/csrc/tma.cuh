// Bulk-copy (TMA) and mbarrier primitives for the row pipelines (sm_90+ PTX,
// used here on sm_100a).  Only the untiled global->shared bulk copy is used,
// always from this GPU's own memory and never with .multicast::cluster.
//
// Every wait is bounded: after kTimeoutNs of global time without progress the
// wait gives up, the kernel bumps its translation unit's timeout counter
// (read on the host with b2k_pipeline_timeouts) and leaves the loop.
#pragma once

#include <stdlib.h>

#include "common.cuh"

namespace b2k {

constexpr unsigned long long kTimeoutNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Makes barrier initialisation (generic proxy) visible to the async proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Orders this thread's earlier shared-memory accesses before its later
// async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// barrier over the first `nthreads` threads of the block (named barrier id)
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// global -> shared bulk copy of `bytes` (multiple of 16, both addresses
// 16-byte aligned) completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 prefetch hint for `bytes` (multiple of 16) at a 16-byte aligned address
// of this GPU's global memory: no data reaches the block and nothing
// completes on a barrier.  L2 is the GPU's point of coherence, so a line
// prefetched before another kernel writes it holds the written data
// afterwards; the hint never makes a later read stale.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// L2 eviction-priority policies for bulk copies (createpolicy, sm_80+)
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// bulk_g2s with an L2 eviction policy for the source lines
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait for the phase with `parity` to complete.  Returns false
// after `limit_ns` of global time without completion.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          unsigned long long limit_ns = kTimeoutNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && globaltimer() - t0 > limit_ns) return false;
  }
}

// ---------------------------------------------------------------------------
// Thread-block cluster primitives (distributed shared memory between the
// CTAs of one cluster on this GPU; no multicast).
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
// all threads of every CTA of the cluster (release / acquire at cluster scope)
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire;" ::: "memory");
}
// shared::cluster address of the same variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32x4(uint32_t addr, float a, float b, float c,
                                                 float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}
// arrive on an mbarrier of another CTA of the cluster; release at cluster
// scope orders this thread's earlier st.shared::cluster before the arrival
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_acq_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// bounded wait on a local mbarrier whose arrivals come from other CTAs of the
// cluster (acquire at cluster scope: their stores before the arrival are seen)
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity,
                                                  unsigned long long limit_ns = kTimeoutNs) {
  if (mbar_try_wait_acq_cluster(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_acq_cluster(bar, parity)) return true;
    if ((i & 255u) == 0 && globaltimer() - t0 > limit_ns) return false;
  }
}

// Programmatic dependent launch: the kernel may start while the previous
// kernel in the stream is still finishing; every input read must come after
// griddep_wait(), which returns once the preceding grid has completed and its
// writes are visible.  griddep_launch_dependents() lets the next kernel in
// the stream begin its own launch (its blocks still wait for resources and,
// before reading, for this grid to finish).
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Prologue of a non-persistent row kernel launched with launch_pdl, whose
// block handles rows [row0, row0 + nrows) of up to two inputs (x, r; r may be
// null): lets the next kernel of the stream launch, hints the block's rows
// into L2 when `hint` (rows 16-byte aligned, a multiple of 16 bytes long) and
// waits for the previous kernel, before which nothing may be read or written.
__device__ __forceinline__ void pdl_rows_prologue(const void* x, int64_t ldx_bytes,
                                                  const void* r, int64_t ldr_bytes,
                                                  int64_t row0, int64_t nrows,
                                                  uint32_t row_bytes, bool hint) {
  griddep_launch_dependents();
  if (hint && row_bytes > 0 && threadIdx.x == 0 && threadIdx.y == 0) {
    for (int64_t i = 0; i < nrows; ++i) {
      bulk_prefetch_l2(static_cast<const unsigned char*>(x) + (row0 + i) * ldx_bytes, row_bytes);
      if (r)
        bulk_prefetch_l2(static_cast<const unsigned char*>(r) + (row0 + i) * ldr_bytes,
                         row_bytes);
    }
  }
  griddep_wait();
}

// Launch with programmatic dependent launch enabled (B2K_PDL=0 disables it):
// the kernel's blocks may be scheduled while the previous kernel of the
// stream drains; the kernel itself calls griddep_wait() before its first
// global read.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* s = getenv("B2K_PDL");
    return !(s && s[0] == '0');
  }();
  return on;
}

template <typename Kernel, typename... Args>
inline void launch_pdl(Kernel kern, dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kern, args...);
}

// Host-side registry of per-translation-unit timeout counters.
using TimeoutReader = unsigned (*)(bool reset);
void register_timeout_reader(TimeoutReader f);

}  // namespace b2k

// Defines this translation unit's device timeout counter `b2k_tu_timeouts`
// and registers its host reader.  Use once per .cu file that launches a
// pipelined kernel (before the kernels).
#define B2K_DEFINE_TIMEOUT_COUNTER()                                                     \
  static __device__ unsigned b2k_tu_timeouts;                                          \
  static unsigned b2k_read_tu_timeouts(bool reset) {                                     \
    unsigned v = 0;                                                                      \
    if (cudaMemcpyFromSymbol(&v, b2k_tu_timeouts, sizeof(v)) != cudaSuccess) return 0;   \
    if (reset && v) {                                                                    \
      const unsigned z = 0;                                                              \
      cudaMemcpyToSymbol(b2k_tu_timeouts, &z, sizeof(z));                                \
    }                                                                                    \
    return v;                                                                            \
  }                                                                                      \
  static const int b2k_tu_timeouts_registered =                                          \
      (::b2k::register_timeout_reader(&b2k_read_tu_timeouts), 0);
