// Mean cross-entropy over the rows of all ranks with the exchange fused into
// the reducing kernel.  Replaces b2k_ce_reduce -> NCCL all-reduce of the
// [loss sum, valid count] pair -> b2k_ce_mean when the ranks' exchange
// buffers are mapped into every rank's process (CUDA IPC, peer access over
// NVLink; plain loads and stores, no multicast): one
// block reduces this rank's per-row losses in fp64 in a fixed order (as
// b2k_ce_reduce), stores the pair into the slot of this rank in EVERY rank's
// buffer, publishes it with a system-scope release store of the epoch, waits
// (bounded) until every rank's flag in its own buffer carries the epoch,
// and adds the pairs in rank order (the same order on every rank, so every
// rank gets the same bits).
//
// Buffer of one rank (b2k_ce_exchange_bytes(world) bytes, zeroed once before
// the first call, identical layout on every rank):
//   pairs[2][world]  (fp64 sum, fp64 count)   16 B each, by epoch parity
//   flags[2][world]  (u64 epoch)              8 B each
//   epoch            (u64, this rank's call counter; never read remotely)
// Slots alternate by epoch parity: a rank overwrites the slot of epoch e in a
// peer only during call e + 2, after its own wait of call e + 1, which needs
// the peer's flag of e + 1, which the peer publishes only after it finished
// reading the pairs of call e (stream order on the peer).
//
// That argument holds while no wait gives up.  A rank whose wait ran out may
// step on and reach call e + 2 while a slow peer is still in call e, so:
//  * a flag ABOVE the waiting rank's epoch can only come from such a rank;
//    it is an error (status 2), never accepted as "arrived";
//  * the status word is sticky: once nonzero (1 = wait ran out, 2 = a peer
//    ran ahead) every later call of that rank returns NaN without writing
//    into any peer's buffer, so its peers time out in turn and every rank
//    ends in the failed state instead of mixing epochs.  The host reads the
//    word (b200k raises) and the exchange has to be set up again.
#include <string.h>

#include "tma.cuh"

B2K_DEFINE_TIMEOUT_COUNTER()

namespace b2k {

__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__host__ __device__ constexpr size_t xchg_pair_off(int par, int world, int r) {
  return ((size_t)par * world + r) * 16;
}
__host__ __device__ constexpr size_t xchg_flag_off(int par, int world, int r) {
  return (size_t)2 * world * 16 + ((size_t)par * world + r) * 8;
}
__host__ __device__ constexpr size_t xchg_epoch_off(int world) {
  return (size_t)2 * world * 16 + (size_t)2 * world * 8;
}
__host__ __device__ constexpr size_t xchg_bytes(int world) { return xchg_epoch_off(world) + 8; }

// The exchange of one [sum, count] pair: every rank stores (ts, tc) into its
// slot in every rank's buffer and publishes it; each rank then waits
// (bounded) for all flags of the epoch in its own buffer and adds the pairs in
// rank order.  Called by every thread of the block (barriers inside); thread
// 0 holds (ts, tc) on entry and (S, C) on a true return.  False when a wait ran
// out or a peer ran ahead: *status is then set (sticky) and nothing more is
// read.
struct XchgShared {
  int timed_out, ran_ahead;
  unsigned long long epoch;
};

__device__ __forceinline__ bool exchange_pair(double ts, double tc, unsigned char* const* peers,
                                              int rank, int world,
                                              unsigned long long limit_ns, int* status,
                                              XchgShared& sh, double& S, double& C) {
  unsigned char* mine = peers[rank];
  if (threadIdx.x == 0) {
    sh.timed_out = 0;
    sh.ran_ahead = 0;
    unsigned long long* ep = reinterpret_cast<unsigned long long*>(mine + xchg_epoch_off(world));
    const unsigned long long epoch = *ep + 1;
    *ep = epoch;
    sh.epoch = epoch;
    const int par = (int)(epoch & 1);
    for (int r = 0; r < world; ++r) {
      unsigned char* base = peers[r];
      double* pair = reinterpret_cast<double*>(base + xchg_pair_off(par, world, rank));
      pair[0] = ts;
      pair[1] = tc;
      // release: the pair is visible to whoever acquires the flag
      st_release_sys_u64(reinterpret_cast<unsigned long long*>(base + xchg_flag_off(par, world, rank)),
                         epoch);
    }
  }
  __syncthreads();
  const unsigned long long epoch = sh.epoch;
  const int par = (int)(epoch & 1);
  // thread r watches rank r's flag in this rank's own buffer, bounded
  if (threadIdx.x < world) {
    const unsigned long long* flag =
        reinterpret_cast<const unsigned long long*>(mine + xchg_flag_off(par, world, threadIdx.x));
    unsigned long long f = ld_acquire_sys_u64(flag);
    if (f < epoch) {
      const unsigned long long t0 = globaltimer();
      for (uint32_t i = 1;; ++i) {
        f = ld_acquire_sys_u64(flag);
        if (f >= epoch) break;
        if ((i & 63u) == 0 && globaltimer() - t0 > limit_ns) {
          atomicExch(&sh.timed_out, 1);
          break;
        }
      }
    }
    if (f > epoch) atomicExch(&sh.ran_ahead, 1);  // a peer two calls ahead: see above
  }
  __syncthreads();
  if (threadIdx.x != 0) return true;
  if (sh.timed_out || sh.ran_ahead) {
    atomicAdd(&b2k_tu_timeouts, 1u);
    *status = sh.ran_ahead ? 2 : 1;
    return false;
  }
  S = 0.0;
  C = 0.0;
  for (int r = 0; r < world; ++r) {
    // acquire again in this thread, then read past the L1 (cache-volatile)
    (void)ld_acquire_sys_u64(
        reinterpret_cast<const unsigned long long*>(mine + xchg_flag_off(par, world, r)));
    const double* pair = reinterpret_cast<const double*>(mine + xchg_pair_off(par, world, r));
    S += __ldcv(pair);
    C += __ldcv(pair + 1);
  }
  return true;
}

__device__ __forceinline__ bool exchange_failed_before(const int* status) {
  return *reinterpret_cast<const volatile int*>(status) != 0;
}

__global__ void __launch_bounds__(1024) ce_reduce_exchange_mean_kernel(
    const float* loss, const int64_t* tgt, int64_t M, int64_t ignore,
    unsigned char* const* peers, int rank, int world, unsigned long long limit_ns,
    double* sumcount, float* out, int* status) {
  __shared__ double rs[32], rc[32];
  __shared__ XchgShared sh;
  const double qnan = __longlong_as_double(0x7ff8000000000000ll);
  // a failed exchange stays failed (sticky status): no pair is published
  if (exchange_failed_before(status)) {
    if (threadIdx.x == 0) {
      sumcount[0] = qnan;
      sumcount[1] = 0.0;
      out[0] = __int_as_float(0x7fc00000);
    }
    return;
  }
  double s = 0.0, c = 0.0;
  for (int64_t i = threadIdx.x; i < M; i += blockDim.x) {
    if (tgt[i] != ignore) { s += (double)loss[i]; c += 1.0; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    c += __shfl_xor_sync(0xffffffffu, c, o);
  }
  if ((threadIdx.x & 31) == 0) { rs[threadIdx.x >> 5] = s; rc[threadIdx.x >> 5] = c; }
  __syncthreads();
  double ts = 0.0, tc = 0.0;
  if (threadIdx.x == 0)
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) { ts += rs[i]; tc += rc[i]; }
  double S = 0.0, C = 0.0;
  const bool ok = exchange_pair(ts, tc, peers, rank, world, limit_ns, status, sh, S, C);
  if (threadIdx.x == 0) {
    sumcount[0] = ok ? S : qnan;
    sumcount[1] = ok ? C : 0.0;
    out[0] = ok ? (float)(S / C) : __int_as_float(0x7fc00000);  // 0/0 -> NaN: no valid row
  }
}

// The pair exchange alone: global = the sum over all ranks of local (two
// doubles in device memory).  NaN on a failure (sticky, as above).
__global__ void __launch_bounds__(32) exchange_pair_kernel(const double* local,
                                                           unsigned char* const* peers, int rank,
                                                           int world, unsigned long long limit_ns,
                                                           double* global, int* status) {
  __shared__ XchgShared sh;
  const double qnan = __longlong_as_double(0x7ff8000000000000ll);
  if (exchange_failed_before(status)) {
    if (threadIdx.x == 0) { global[0] = qnan; global[1] = qnan; }
    return;
  }
  const double ts = threadIdx.x == 0 ? local[0] : 0.0, tc = threadIdx.x == 0 ? local[1] : 0.0;
  double S = 0.0, C = 0.0;
  const bool ok = exchange_pair(ts, tc, peers, rank, world, limit_ns, status, sh, S, C);
  if (threadIdx.x == 0) {
    global[0] = ok ? S : qnan;
    global[1] = ok ? C : qnan;
  }
}

}  // namespace b2k

extern "C" int64_t b2k_ce_exchange_bytes(int world) {
  if (world < 1 || world > 32) {
    b2k::set_error("b2k_ce_exchange_bytes: world %d outside 1..32", world);
    return -1;
  }
  return (int64_t)b2k::xchg_bytes(world);
}

extern "C" int b2k_ce_reduce_exchange_mean(const float* row_loss, const int64_t* tgt, int64_t M,
                                           int64_t ignore_index, void* const* peers, int rank,
                                           int world, unsigned long long limit_ns,
                                           double* sumcount, float* out, int* status,
                                           void* stream) {
  B2K_REQUIRE(world >= 1 && world <= 32 && rank >= 0 && rank < world,
              "b2k_ce_reduce_exchange_mean: rank %d of world %d", rank, world);
  B2K_REQUIRE(M >= 0 && (M == 0 || (row_loss != nullptr && tgt != nullptr)),
              "b2k_ce_reduce_exchange_mean: bad rows");
  B2K_REQUIRE(peers != nullptr && sumcount != nullptr && out != nullptr && status != nullptr,
              "b2k_ce_reduce_exchange_mean: null pointer");
  B2K_REQUIRE(limit_ns > 0 && limit_ns <= 10000000000ull,
              "b2k_ce_reduce_exchange_mean: wait limit outside (0, 10 s]");
  b2k::ce_reduce_exchange_mean_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(
      row_loss, tgt, M, ignore_index, reinterpret_cast<unsigned char* const*>(peers), rank, world,
      limit_ns, sumcount, out, status);
  return b2k::check_launch("b2k_ce_reduce_exchange_mean");
}

extern "C" int b2k_exchange_pair(const double* local, void* const* peers, int rank, int world,
                                 unsigned long long limit_ns, double* global, int* status,
                                 void* stream) {
  B2K_REQUIRE(world >= 1 && world <= 32 && rank >= 0 && rank < world,
              "b2k_exchange_pair: rank %d of world %d", rank, world);
  B2K_REQUIRE(local != nullptr && peers != nullptr && global != nullptr && status != nullptr,
              "b2k_exchange_pair: null pointer");
  B2K_REQUIRE(limit_ns > 0 && limit_ns <= 10000000000ull,
              "b2k_exchange_pair: wait limit outside (0, 10 s]");
  b2k::exchange_pair_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      local, reinterpret_cast<unsigned char* const*>(peers), rank, world, limit_ns, global, status);
  return b2k::check_launch("b2k_exchange_pair");
}

// ---------------------------------------------------------------------------
// Plumbing for the exchange buffers: plain device allocations shared between
// the ranks' processes with CUDA IPC (a peer mapping, no multicast object).
extern "C" int b2k_ce_exchange_alloc(int world, void** buf) {
  B2K_REQUIRE(world >= 1 && world <= 32 && buf != nullptr, "b2k_ce_exchange_alloc: bad arguments");
  void* p = nullptr;
  const size_t n = b2k::xchg_bytes(world);
  cudaError_t e = cudaMalloc(&p, n);
  if (e == cudaSuccess) e = cudaMemset(p, 0, n);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    b2k::set_error("b2k_ce_exchange_alloc: %s", cudaGetErrorString(e));
    return B2K_ELAUNCH;
  }
  *buf = p;
  return B2K_OK;
}

extern "C" int b2k_ce_exchange_free(void* buf) {
  if (buf == nullptr) return B2K_OK;
  const cudaError_t e = cudaFree(buf);
  if (e != cudaSuccess) {
    b2k::set_error("b2k_ce_exchange_free: %s", cudaGetErrorString(e));
    return B2K_ELAUNCH;
  }
  return B2K_OK;
}

extern "C" int b2k_ipc_handle(void* buf, void* handle64) {
  B2K_REQUIRE(buf != nullptr && handle64 != nullptr, "b2k_ipc_handle: null pointer");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, buf);
  if (e != cudaSuccess) {
    b2k::set_error("b2k_ipc_handle: %s", cudaGetErrorString(e));
    return B2K_ELAUNCH;
  }
  memcpy(handle64, &h, sizeof(h));
  return B2K_OK;
}

extern "C" int b2k_ipc_open(const void* handle64, void** ptr) {
  B2K_REQUIRE(handle64 != nullptr && ptr != nullptr, "b2k_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    b2k::set_error("b2k_ipc_open: %s", cudaGetErrorString(e));
    return B2K_ELAUNCH;
  }
  *ptr = p;
  return B2K_OK;
}

extern "C" int b2k_ipc_close(void* ptr) {
  if (ptr == nullptr) return B2K_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    b2k::set_error("b2k_ipc_close: %s", cudaGetErrorString(e));
    return B2K_ELAUNCH;
  }
  return B2K_OK;
}
