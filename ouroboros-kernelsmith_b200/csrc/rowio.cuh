// Row slice load/store used by every row kernel.
//
// Layout of a row held by a thread group of G threads with V vector slots per
// thread: slot v of thread tx covers elements [(v*G + tx)*E, +E) where E is
// the number of elements in 16 bytes.  Consecutive threads touch consecutive
// 16-byte vectors, so every warp-wide access is a fully coalesced 512-byte
// transaction.  `aligned` (uniform per launch) says that every row base is
// 16-byte aligned and N % E == 0; otherwise the same slots are filled with
// bounds-checked scalar accesses (odd N such as 4097, misaligned views).
#pragma once

#include "common.cuh"

namespace b2k {

template <typename T, bool STREAM>
__device__ __forceinline__ void load_vec(float* f, const T* row, int64_t c, int64_t N,
                                         bool aligned) {
  constexpr int E = Traits<T>::E;
  if (aligned) {
    if (c < N) {
      unpack<T>(STREAM ? ld_stream(row + c) : ld_keep(row + c), f);
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) f[e] = 0.0f;
    }
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) f[e] = (c + e < N) ? ld1(row + c + e) : 0.0f;
  }
}

// Same as load_vec but fills out-of-range elements with `fill`.
template <typename T, bool STREAM>
__device__ __forceinline__ void load_vec_fill(float* f, const T* row, int64_t c, int64_t N,
                                              bool aligned, float fill) {
  constexpr int E = Traits<T>::E;
  if (aligned) {
    if (c < N) {
      unpack<T>(STREAM ? ld_stream(row + c) : ld_keep(row + c), f);
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) f[e] = fill;
    }
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) f[e] = (c + e < N) ? ld1(row + c + e) : fill;
  }
}

template <typename T>
__device__ __forceinline__ void store_vec(T* row, int64_t c, int64_t N, bool aligned,
                                          const float* f) {
  constexpr int E = Traits<T>::E;
  if (aligned) {
    if (c < N) st_stream(row + c, pack<T>(f));
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e)
      if (c + e < N) st1(row + c + e, f[e]);
  }
}

// Host-side choice of (G, V, R) for a register-resident row of N elements.
// V (vector slots per thread) doubles until the row fits G_target threads;
// G is the next power of two covering the row; R rows share a 256-thread
// block when G < 256.  Returns false when the row exceeds gmax threads x vmax
// slots (the caller then streams the row).
struct RowCfg {
  int G, V, R;
};

inline int next_pow2(int64_t v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

inline bool choose_row_cfg(int64_t N, int E, int g_target, RowCfg* cfg, int vmax = 8,
                           int gmax = 1024) {
  const int64_t nvec = (N + E - 1) / E;
  int V = 1;
  while (V < vmax && nvec > (int64_t)V * g_target) V <<= 1;
  int64_t need = (nvec + V - 1) / V;
  if (need > gmax) return false;
  int G = next_pow2(need < 1 ? 1 : need);
  int R = G >= 256 ? 1 : 256 / G;
  cfg->G = G; cfg->V = V; cfg->R = R;
  return true;
}

}  // namespace b2k
