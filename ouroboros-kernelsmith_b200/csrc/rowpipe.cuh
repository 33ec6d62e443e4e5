// Persistent row pipeline: a block walks rows first, first+stride, ... and
// keeps the next S-1 of them streaming into an S-stage shared-memory ring
// with bulk copies while it computes on the current one.
//
// Protocol per row k (stage s = k % S, parity (k / S) & 1):
//   wait_next()    all threads wait (bounded) for the stage to be full
//   ...            threads read their slice of the stage, then reach a block
//                  barrier (every row op here has one in its reduction)
//   refill()       thread 0 re-arms the stage with row k + S
// after the loop: drain(k) waits (bounded) for copies still in flight when a
// wait timed out, so nothing lands in shared memory after the block exits.
// Inputs are NIN row-major matrices with their own row strides; each row is
// copied as one bulk transfer of N * sizeof(T) bytes (16-byte multiple).
#pragma once

#include <mutex>
#include <stdlib.h>

#include "tma.cuh"

namespace b2k {

template <int NIN>
struct RowPipe {
  unsigned char* dsm;
  uint64_t* full;
  int S;
  uint32_t row_bytes, stage_bytes;
  int64_t first, stride, nrows, issued;
  int istage;        // stage of the next issue (issuing thread)
  int cstage;        // stage of the next row to consume
  uint32_t cphase;   // its barrier phase parity
  const unsigned char* src[NIN];
  int64_t ld_bytes[NIN];

  // dynamic shared memory needed for S stages
  static size_t smem_bytes(int S, int64_t row_bytes) {
    return (size_t)S * NIN * (size_t)row_bytes + (size_t)S * sizeof(uint64_t);
  }

  __device__ __forceinline__ void issue(int64_t k) {
    const int s = istage;
    if (++istage == S) istage = 0;
    const int64_t row = first + k * stride;
    unsigned char* st = dsm + (size_t)s * stage_bytes;
    mbar_arrive_expect_tx(&full[s], stage_bytes);
#pragma unroll
    for (int i = 0; i < NIN; ++i)
      bulk_g2s(st + (size_t)i * row_bytes, src[i] + row * ld_bytes[i], row_bytes, &full[s]);
  }

  // Called by every thread; contains a __syncthreads.
  __device__ __forceinline__ void init(unsigned char* smem, int stages, int64_t M,
                                       uint32_t rbytes, const void* const* srcs,
                                       const int64_t* ld_elems, int elem_bytes) {
    dsm = smem;
    S = stages;
    row_bytes = rbytes;
    stage_bytes = NIN * rbytes;
    full = reinterpret_cast<uint64_t*>(dsm + (size_t)S * stage_bytes);
    first = blockIdx.x;
    stride = gridDim.x;
    nrows = first < M ? (M - 1 - first) / stride + 1 : 0;
#pragma unroll
    for (int i = 0; i < NIN; ++i) {
      src[i] = static_cast<const unsigned char*>(srcs[i]);
      ld_bytes[i] = ld_elems[i] * elem_bytes;
    }
    if (threadIdx.x == 0 && threadIdx.y == 0) {
      for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
      fence_barrier_init();
    }
    __syncthreads();
    issued = 0;
    istage = 0;
    cstage = 0;
    cphase = 0;
    if (threadIdx.x == 0 && threadIdx.y == 0)
      for (; issued < nrows && issued < S; ++issued) issue(issued);
  }

  __device__ __forceinline__ int64_t row_of(int64_t k) const { return first + k * stride; }

  // Thread 0: L2 prefetch hints for the first `rows` rows of this block.
  // Needs no barrier or shared memory, so a kernel calls it before
  // griddep_wait(): the DRAM reads of its first rows then overlap the tail of
  // the previous kernel in the stream, and their bulk copies find them in L2.
  // One row per block measured best (4096 x 4096 fp16 rmsnorm 13.9 -> 12.8
  // us, a 2048 x 8192 residual LayerNorm shard 26.0 -> 23.8 us); more rows
  // queue ahead of the other blocks' first rows and lose again.
  __device__ static void prefetch_l2(const void* const* srcs, const int64_t* ld_elems,
                                     int elem_bytes, uint32_t rbytes, int64_t M, int rows) {
    if (rows <= 0 || threadIdx.x != 0 || threadIdx.y != 0) return;
    const int64_t b = blockIdx.x, g = gridDim.x;
    const int64_t mine = b < M ? (M - 1 - b) / g + 1 : 0;
    const int64_t n = rows < mine ? rows : mine;
    for (int64_t k = 0; k < n; ++k)
#pragma unroll
      for (int i = 0; i < NIN; ++i)
        bulk_prefetch_l2(static_cast<const unsigned char*>(srcs[i]) +
                             (b + k * g) * ld_elems[i] * elem_bytes,
                         rbytes);
  }

  // Bounded wait for the next row (rows are consumed in order 0, 1, ...);
  // returns the stage base, ok=false on timeout.
  __device__ __forceinline__ const unsigned char* wait_next(bool& ok) {
    const int s = cstage;
    ok = mbar_wait(&full[s], cphase);
    if (++cstage == S) { cstage = 0; cphase ^= 1u; }
    return dsm + (size_t)s * stage_bytes;
  }

  // Thread 0, after a block barrier that follows every thread's reads of the
  // stage of the row just consumed.
  __device__ __forceinline__ void refill() {
    if (threadIdx.x == 0 && threadIdx.y == 0 && issued < nrows) {
      fence_proxy_async();
      issue(issued);
      ++issued;
    }
  }

  __device__ __forceinline__ void drain(int64_t k) {
    if (threadIdx.x == 0 && threadIdx.y == 0)
      for (int64_t j = k; j < issued; ++j)
        mbar_wait(&full[(int)(j % S)], (uint32_t)((j / S) & 1));
  }
};

// Host: pipeline shape for rows of `stage_bytes` (all inputs of one row).
// More resident blocks per SM hide the per-row reduction latency better than
// a deeper ring, so the shape takes as many blocks as registers, threads and
// shared memory allow (up to 16) and then as many stages (2..4) as fit the
// shared-memory budget.  Explicit want_cps / want_stages override.  Returns
// false when the rows do not fit (the caller uses another kernel).
struct PipeShape {
  int cps, S;
};

// B2K_L2PF_ROWS: rows per block that the bulk-copy row pipelines hint into L2
// before waiting for the previous kernel (default 1, 0 = off, at most 8).
inline int l2_prefetch_rows_knob() {
  static const int v = [] {
    const char* s = getenv("B2K_L2PF_ROWS");
    const int r = s ? atoi(s) : 1;
    return r >= 0 && r <= 8 ? r : 1;
  }();
  return v;
}

// Raises the kernel's dynamic shared-memory cap once per device (to the whole
// per-block maximum); the launch itself asks for what it needs.  The
// attribute belongs to the current device's context, so a process that
// launches on several GPUs sets it on each.
template <typename Kernel>
inline void allow_max_dynamic_smem(Kernel kern) {
  static std::mutex mu;
  static const void* done[512];
  static int done_dev[512];
  static int ndone = 0;
  int dev = 0, optin = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < ndone; ++i)
    if (done[i] == (const void*)kern && done_dev[i] == dev) return;
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaFuncAttributes fa;
  cudaFuncGetAttributes(&fa, kern);
  const int cap = optin - (int)fa.sharedSizeBytes;
  if (cap > 0) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, cap);
  cudaGetLastError();
  if (ndone < 512) {
    done[ndone] = (const void*)kern;
    done_dev[ndone++] = dev;
  }
}

template <typename Kernel>
inline bool choose_pipe_shape_uncached(Kernel kern, int threads, int64_t stage_bytes,
                                       int want_cps, int want_stages, PipeShape* ps) {
  const int64_t budget = 200 << 10;  // dynamic shared memory per SM
  if (want_cps > 0) {
    int cps = want_cps;
    int S = want_stages > 0 ? want_stages : 4;
    while (S > 2 && (int64_t)cps * S * stage_bytes > budget) --S;
    while (cps > 1 && (int64_t)cps * S * stage_bytes > budget) --cps;
    if ((int64_t)cps * S * stage_bytes > budget) return false;
    ps->cps = cps;
    ps->S = S;
    return true;
  }
  // blocks per SM: as many as are resident (up to B2K_PIPE_MAXCPS, default
  // 16), each with want_stages (else 4).  The cap matters for 64-thread
  // blocks (rows of 256 vectors): 16 instead of 8 of them per SM took
  // cumsum over 16384 x 2048 fp16 from 42.1 to 26.1 us and entropy from 29.7
  // to 20.2 us; 32 measured the same as 16.
  static const int max_cps = [] {
    const char* s = getenv("B2K_PIPE_MAXCPS");
    const int v = s ? atoi(s) : 16;
    return v >= 1 && v <= 32 ? v : 16;
  }();
  for (int cps = max_cps; cps >= 1; --cps) {
    int S = want_stages > 0 ? want_stages : 4;
    while (S > 2 && (int64_t)cps * S * stage_bytes > budget) --S;
    if ((int64_t)cps * S * stage_bytes > budget) continue;
    const size_t smem = (size_t)S * (size_t)stage_bytes + (size_t)S * sizeof(uint64_t);
    int resident = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, kern, threads, smem) !=
        cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    if (resident >= cps) {
      ps->cps = cps;
      ps->S = S;
      return true;
    }
  }
  return false;
}

// Cached per (device, kernel, threads, stage bytes, overrides): the occupancy
// query runs once, later launches pay a table lookup.
template <typename Kernel>
inline bool choose_pipe_shape(Kernel kern, int threads, int64_t stage_bytes, int want_cps,
                              int want_stages, PipeShape* ps) {
  struct Entry {
    const void* k;
    int dev, threads, cps, stages;
    int64_t stage;
    PipeShape ps;
    bool ok;
  };
  static std::mutex mu;
  static Entry cache[512];
  static int n = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  allow_max_dynamic_smem(kern);
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < n; ++i) {
      const Entry& e = cache[i];
      if (e.k == (const void*)kern && e.dev == dev && e.threads == threads &&
          e.stage == stage_bytes && e.cps == want_cps && e.stages == want_stages) {
        *ps = e.ps;
        return e.ok;
      }
    }
  }
  PipeShape r{1, 2};
  const bool ok = choose_pipe_shape_uncached(kern, threads, stage_bytes, want_cps, want_stages, &r);
  std::lock_guard<std::mutex> lock(mu);
  if (n < 512)
    cache[n++] = Entry{(const void*)kern, dev, threads, want_cps, want_stages, stage_bytes, r, ok};
  *ps = r;
  return ok;
}

}  // namespace b2k
