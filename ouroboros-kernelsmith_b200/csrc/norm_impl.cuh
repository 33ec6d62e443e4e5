// Row normalisation family: [x + r] -> {RMS, L2, LayerNorm} -> affine ->
// epilogue.  Covers rmsnorm, add_rmsnorm, layernorm, add_layernorm, l2norm,
// layernorm_gelu, rmsnorm_gemma, rmsnorm_wide and the 76 chains
// (ouroboros/specs.py:75-120,171-190,216-220; ouroboros/chains.py:69-87).
//
// One thread group per row.  The row is read from HBM exactly once into
// registers (16-byte coalesced loads, evict-first), the statistics are group
// reductions over registers (LayerNorm: two-pass mean then centred variance,
// the reference's order), and the output is written once.  Rows longer than
// 512 threads x 8 vector slots take the streaming kernel, which re-reads the
// row from L2 for its later passes.
//
// The epilogue is a template parameter (one kernel per activation) so each
// kernel stays small; instances are spread over the norm_inst_*.cu files so
// they compile in parallel.
#pragma once

#include "rowio.cuh"

namespace b2k {

struct NormArgs {
  const void* x;
  const void* r;
  const void* w;
  const void* b;
  void* y;
  void* h;
  int64_t ldx, ldr, ldy, ldh;
  int64_t M, N;
  float eps;
  int norm;     // b2k_norm_kind
  int affine;   // b2k_affine
  int aligned;  // all row bases 16-byte aligned and N % E == 0
  int g_target; // threads-per-row target of the register path
};

constexpr int kNormMaxThreads = 512;

template <typename T, int ACT>
int norm_launch(const NormArgs& a, cudaStream_t st);

#ifdef B2K_NORM_DEFINE_KERNELS

// Affine as uniform selects rather than a branch per element:
//   n = ((h - mu) * rs) * (w + w_off) + b, optionally rounded through T twice
//   (rmsnorm/add_rmsnorm compute T(T(h*rs) * w), specs.py:78,93).
struct AffineSel {
  bool has_w, has_b, rounded;
  float w_off;
  __device__ __forceinline__ explicit AffineSel(int affine)
      : has_w(affine != B2K_AFF_NONE),
        has_b(affine == B2K_AFF_WB),
        rounded(affine == B2K_AFF_W_ROUNDED),
        w_off(affine == B2K_AFF_ONE_PLUS_W ? 1.0f : 0.0f) {}
};

template <typename T, int ACT>
__device__ __forceinline__ void norm_emit(const NormArgs& a, const AffineSel& s, T* yrow,
                                          int64_t c, const float* hv, float mu, float rs) {
  constexpr int E = Traits<T>::E;
  constexpr bool P = std::is_same<T, float>::value;
  const bool aligned = a.aligned;
  float wv[E], bv[E], out[E];
  if (s.has_w) {
    load_vec<T, false>(wv, static_cast<const T*>(a.w), c, a.N, aligned);
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) wv[e] = 1.0f;
  }
  if (s.has_b) {
    load_vec<T, false>(bv, static_cast<const T*>(a.b), c, a.N, aligned);
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) bv[e] = 0.0f;
  }
#pragma unroll
  for (int e = 0; e < E; ++e) {
    float t = (hv[e] - mu) * rs;
    if (s.rounded) t = round_to<T>(t);
    float n = t * (wv[e] + s.w_off);
    if (s.has_b) n += bv[e];
    if (s.rounded) n = round_to<T>(n);
    out[e] = act_apply<ACT, P>(n);
  }
  store_vec<T>(yrow, c, a.N, aligned, out);
}

template <typename T, int V, bool RESID, int ACT>
__global__ void __launch_bounds__(kNormMaxThreads) norm_rows_kernel(const NormArgs a) {
  constexpr int E = Traits<T>::E;
  __shared__ float red[1024];
  const Group g;
  const int64_t row = (int64_t)blockIdx.x * blockDim.y + g.ty;
  const bool valid = row < a.M;
  const int64_t N = a.N;
  const bool aligned = a.aligned;
  const T* xr = static_cast<const T*>(a.x) + (valid ? row * a.ldx : 0);
  const T* rr = RESID ? static_cast<const T*>(a.r) + (valid ? row * a.ldr : 0) : nullptr;

  // ---- one read of the row (x and r), h = x + r in fp32 -------------------
  float hv[V][E];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int64_t c = (int64_t)(v * g.G + g.tx) * E;
    if (valid) {
      load_vec<T, true>(hv[v], xr, c, N, aligned);
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) hv[v][e] = 0.0f;
    }
  }
  if (RESID && valid) {
#pragma unroll
    for (int v = 0; v < V; ++v) {
      float t[E];
      load_vec<T, true>(t, rr, (int64_t)(v * g.G + g.tx) * E, N, aligned);
#pragma unroll
      for (int e = 0; e < E; ++e) hv[v][e] += t[e];
    }
  }
  // residual stream output T(x + r), issued before the reductions
  if (a.h != nullptr && valid) {
    T* hrow = static_cast<T*>(a.h) + row * a.ldh;
#pragma unroll
    for (int v = 0; v < V; ++v) store_vec<T>(hrow, (int64_t)(v * g.G + g.tx) * E, N, aligned, hv[v]);
  }

  // ---- statistics --------------------------------------------------------
  float mu = 0.0f, rs;
  if (a.norm == B2K_NORM_LN) {
    float s = 0.0f;
#pragma unroll
    for (int v = 0; v < V; ++v)
#pragma unroll
      for (int e = 0; e < E; ++e) s += hv[v][e];
    s = group_sum(s, g, red);
    mu = s / (float)N;
    float q = 0.0f;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int64_t c = (int64_t)(v * g.G + g.tx) * E;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float d = (c + e < N) ? hv[v][e] - mu : 0.0f;
        q += d * d;
      }
    }
    q = group_sum(q, g, red);
    rs = rsqrtf(q / (float)N + a.eps);
  } else {
    float s = 0.0f;
#pragma unroll
    for (int v = 0; v < V; ++v)
#pragma unroll
      for (int e = 0; e < E; ++e) s += hv[v][e] * hv[v][e];
    s = group_sum(s, g, red);
    rs = rsqrtf((a.norm == B2K_NORM_L2 ? s : s / (float)N) + a.eps);
  }
  if (!valid) return;

  // ---- affine + epilogue + one write ---------------------------------------
  const AffineSel sel(a.affine);
  T* yrow = static_cast<T*>(a.y) + row * a.ldy;
#pragma unroll
  for (int v = 0; v < V; ++v)
    norm_emit<T, ACT>(a, sel, yrow, (int64_t)(v * g.G + g.tx) * E, hv[v], mu, rs);
}

// Rows too long for registers: one row per block; the statistics pass(es)
// read with the default L2 policy so the final pass re-reads the row from L2.
template <typename T, bool RESID, int ACT>
__global__ void __launch_bounds__(kNormMaxThreads) norm_rows_stream_kernel(const NormArgs a) {
  constexpr int E = Traits<T>::E;
  __shared__ float red[1024];
  const Group g;
  const int64_t row = blockIdx.x;
  const int64_t N = a.N;
  const bool aligned = a.aligned;
  const T* xr = static_cast<const T*>(a.x) + row * a.ldx;
  const T* rr = RESID ? static_cast<const T*>(a.r) + row * a.ldr : nullptr;
  T* hrow = a.h ? static_cast<T*>(a.h) + row * a.ldh : nullptr;
  const int64_t step = (int64_t)g.G * E;
  const bool ln = a.norm == B2K_NORM_LN;

  auto load_h = [&](float* hv, int64_t c) {
    load_vec<T, false>(hv, xr, c, N, aligned);
    if (RESID) {
      float t[E];
      load_vec<T, false>(t, rr, c, N, aligned);
#pragma unroll
      for (int e = 0; e < E; ++e) hv[e] += t[e];
    }
  };

  float mu = 0.0f, rs;
  float s = 0.0f;
  for (int64_t c = (int64_t)g.tx * E; c < N; c += step) {
    float hv[E];
    load_h(hv, c);
    if (hrow) store_vec<T>(hrow, c, N, aligned, hv);
#pragma unroll
    for (int e = 0; e < E; ++e) s += ln ? hv[e] : hv[e] * hv[e];
  }
  s = group_sum(s, g, red);
  if (ln) {
    mu = s / (float)N;
    float q = 0.0f;
    for (int64_t c = (int64_t)g.tx * E; c < N; c += step) {
      float hv[E];
      load_h(hv, c);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float d = (c + e < N) ? hv[e] - mu : 0.0f;
        q += d * d;
      }
    }
    q = group_sum(q, g, red);
    rs = rsqrtf(q / (float)N + a.eps);
  } else {
    rs = rsqrtf((a.norm == B2K_NORM_L2 ? s : s / (float)N) + a.eps);
  }
  const AffineSel sel(a.affine);
  T* yrow = static_cast<T*>(a.y) + row * a.ldy;
  for (int64_t c = (int64_t)g.tx * E; c < N; c += step) {
    float hv[E];
    load_h(hv, c);
    norm_emit<T, ACT>(a, sel, yrow, c, hv, mu, rs);
  }
}

template <typename T, bool RESID, int ACT>
static int norm_launch_resid(const NormArgs& a, cudaStream_t st) {
  constexpr int E = Traits<T>::E;
  RowCfg cfg;
  if (choose_row_cfg(a.N, E, a.g_target, &cfg, 8, kNormMaxThreads)) {
    const dim3 block(cfg.G, cfg.R);
    const int64_t grid = (a.M + cfg.R - 1) / cfg.R;
    switch (cfg.V) {
      case 1: norm_rows_kernel<T, 1, RESID, ACT><<<grid, block, 0, st>>>(a); break;
      case 2: norm_rows_kernel<T, 2, RESID, ACT><<<grid, block, 0, st>>>(a); break;
      case 4: norm_rows_kernel<T, 4, RESID, ACT><<<grid, block, 0, st>>>(a); break;
      default: norm_rows_kernel<T, 8, RESID, ACT><<<grid, block, 0, st>>>(a); break;
    }
  } else {
    norm_rows_stream_kernel<T, RESID, ACT><<<a.M, dim3(kNormMaxThreads, 1), 0, st>>>(a);
  }
  return check_launch("b2k_norm");
}

template <typename T, int ACT>
int norm_launch(const NormArgs& a, cudaStream_t st) {
  return a.r ? norm_launch_resid<T, true, ACT>(a, st) : norm_launch_resid<T, false, ACT>(a, st);
}

#define B2K_NORM_INSTANTIATE(T, ACT) template int norm_launch<T, ACT>(const NormArgs&, cudaStream_t);

#endif  // B2K_NORM_DEFINE_KERNELS

}  // namespace b2k
