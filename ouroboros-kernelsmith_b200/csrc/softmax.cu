// Row softmax family: softmax, softcap_softmax (cap 30), log_softmax and
// softmax_scale (ouroboros/specs.py:81-82,176-181,207-213).
//
// One read, one write per element.  Each thread keeps its slice of the row
// in registers as t = transform(x), takes its local max m_t and local sum
// s_t = sum exp(t - m_t), and the block merges the (max, sum) pairs in ONE
// reduction (online logsumexp).  Softmax output is then e * exp(m_t - M) / S
// with the exponentials already in registers; log-softmax is t - M - log S.
// Paths as in the norm family: bulk-copy pipeline for aligned rows of
// 4..64 KB, register kernel (several rows per block) for short or odd rows,
// and a two-pass streaming kernel for rows beyond the register budget.
#include <stdlib.h>

#include "rowio.cuh"
#include "rowpipe.cuh"

B2K_DEFINE_TIMEOUT_COUNTER()

namespace b2k {

constexpr int kSmMaxThreads = 512;

struct SoftmaxArgs {
  const void* x;
  void* y;
  int64_t ldx, ldy, M;
  int N;
  const void* scale;
  int scale_dtype;
  int aligned;
  int l2pf_rows;  // bulk-copy path: rows per block hinted into L2 before the wait
};

__device__ __forceinline__ float load_scalar(const void* p, int dtype) {
  switch (dtype) {
    case B2K_F16: return __half2float(*static_cast<const __half*>(p));
    case B2K_BF16: return __bfloat162float(*static_cast<const __nv_bfloat16*>(p));
    default: return *static_cast<const float*>(p);
  }
}

// t = transform(x) for one pair
template <int KIND, bool P>
__device__ __forceinline__ float2 sm_transform(float2 x, float scale) {
  if constexpr (KIND == B2K_SOFTCAP) {
    // 30 * tanh(x / 30) with an absolute-error tanh (the cap feeds exp)
    return f2(30.0f * f_tanh_abs<P>(x.x * (1.0f / 30.0f)), 30.0f * f_tanh_abs<P>(x.y * (1.0f / 30.0f)));
  } else if constexpr (KIND == B2K_SOFTMAX_SCALE) {
    return mul2(x, f2s(scale));
  } else {
    return x;
  }
}

// Slice of a row in registers -> outputs.  hv holds x on entry.  `valid`
// tells per element whether it is inside the row.  Called by every thread
// of the block (reductions inside).
template <typename T, int KIND, int V>
struct SoftmaxSlice {
  static constexpr int E = Traits<T>::E;
  static constexpr int H = E / 2;
  static constexpr bool P = std::is_same<T, float>::value;

  // transform + local (max, sum-exp); leaves e = exp(t - m) in hv for
  // softmax kinds, t for log-softmax.  m is the thread's maximum, or with WM
  // the warp's (every lane of the warp calls this; see group_lse_wmax).
  template <bool WM = false>
  __device__ __forceinline__ static void local(float2 (&hv)[V][H], int N, bool whole,
                                               const Group& g, float scale, float& m,
                                               float& s) {
    m = -INFINITY;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (v * g.G + g.tx) * E;
#pragma unroll
      for (int j = 0; j < H; ++j) {
        float2 t = sm_transform<KIND, P>(hv[v][j], scale);
        if (!(whole ? c < N : c + 2 * j < N)) t.x = -INFINITY;
        if (!(whole ? c < N : c + 2 * j + 1 < N)) t.y = -INFINITY;
        hv[v][j] = t;
        m = fmaxf(m, fmaxf(t.x, t.y));
      }
    }
    if constexpr (WM) m = warp_allmax(m);
    s = 0.0f;
    if (m == -INFINITY) return;
    if constexpr (P) {
#pragma unroll
      for (int v = 0; v < V; ++v)
#pragma unroll
        for (int j = 0; j < H; ++j) {
          const float2 e = f2(expf(hv[v][j].x - m), expf(hv[v][j].y - m));
          s += e.x + e.y;
          if (KIND != B2K_LOG_SOFTMAX) hv[v][j] = e;
        }
    } else {
      const float2 nm = f2s(-m * kLog2e);
      float2 s2 = f2s(0.0f);
#pragma unroll
      for (int v = 0; v < V; ++v)
#pragma unroll
        for (int j = 0; j < H; ++j) {
          const float2 z = fma2(hv[v][j], f2s(kLog2e), nm);
          const float2 e = f2(ex2_approx(z.x), ex2_approx(z.y));
          s2 = add2(s2, e);
          if (KIND != B2K_LOG_SOFTMAX) hv[v][j] = e;
        }
      s = s2.x + s2.y;
    }
  }

  // per-thread output transform after the block-wide (M, S)
  __device__ __forceinline__ static void finish(float2 (&hv)[V][H], float m_local, float M,
                                                float S) {
    if constexpr (KIND == B2K_LOG_SOFTMAX) {
      const float c = -(M + (P ? logf(S) : f_log<false>(S)));
#pragma unroll
      for (int v = 0; v < V; ++v)
#pragma unroll
        for (int j = 0; j < H; ++j) hv[v][j] = add2(hv[v][j], f2s(c));
    } else {
      float c;
      if (m_local == -INFINITY) c = 0.0f;
      else if constexpr (P) c = expf(m_local - M) / S;
      else c = ex2_approx((m_local - M) * kLog2e) * rcp_approx(S);
#pragma unroll
      for (int v = 0; v < V; ++v)
#pragma unroll
        for (int j = 0; j < H; ++j) hv[v][j] = mul2(hv[v][j], f2s(c));
    }
  }
};

// ---------------------------------------------------------------- register path
template <typename T, int KIND, int V>
__global__ void __launch_bounds__(kSmMaxThreads) softmax_rows_kernel(const SoftmaxArgs a) {
  constexpr int E = Traits<T>::E;
  constexpr int H = E / 2;
  using Slice = SoftmaxSlice<T, KIND, V>;
  __shared__ float red[1024];
  const Group g;
  const int64_t row = (int64_t)blockIdx.x * blockDim.y + g.ty;
  const bool valid = row < a.M;
  const int N = a.N;
  const bool aligned = a.aligned;
  {
    const int64_t row0 = (int64_t)blockIdx.x * blockDim.y;
    const int64_t nr = a.M - row0 < (int64_t)blockDim.y ? a.M - row0 : (int64_t)blockDim.y;
    pdl_rows_prologue(a.x, a.ldx * (int64_t)sizeof(T), nullptr, 0, row0, nr,
                      (uint32_t)N * (uint32_t)sizeof(T), aligned && a.l2pf_rows > 0);
  }
  const float scale = (KIND == B2K_SOFTMAX_SCALE) ? load_scalar(a.scale, a.scale_dtype) : 1.0f;
  const T* xr = static_cast<const T*>(a.x) + (valid ? row * a.ldx : 0);
  float2 hv[V][H];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * g.G + g.tx) * E;
    if (valid) load_vec<T, true>(reinterpret_cast<float*>(hv[v]), xr, c, N, aligned);
    else
#pragma unroll
      for (int j = 0; j < H; ++j) hv[v][j] = f2s(0.0f);
  }
  float m, s;
  Slice::local(hv, valid ? N : 0, aligned, g, scale, m, s);
  float M = m, S = s;
  group_lse(M, S, g, red);
  if (!valid) return;
  Slice::finish(hv, m, M, S);
  T* yr = static_cast<T*>(a.y) + row * a.ldy;
#pragma unroll
  for (int v = 0; v < V; ++v)
    store_vec<T>(yr, (v * g.G + g.tx) * E, N, aligned, reinterpret_cast<const float*>(hv[v]));
}

// ---------------------------------------------------------------- pipelined path
template <typename T, int KIND, int V>
__global__ void __launch_bounds__(kSmMaxThreads) softmax_tma_kernel(const SoftmaxArgs a,
                                                                    const int S_) {
  constexpr int E = Traits<T>::E;
  constexpr int H = E / 2;
  using Slice = SoftmaxSlice<T, KIND, V>;
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ float red[1024];
  __shared__ volatile int abort_flag;
  const Group g;
  const int N = a.N;
  if (g.tx == 0) abort_flag = 0;
  // programmatic dependent launch: first row hinted into L2, then wait for
  // the previous kernel before any read
  griddep_launch_dependents();
  const void* srcs[1] = {a.x};
  const int64_t lds[1] = {a.ldx};
  RowPipe<1>::prefetch_l2(srcs, lds, (int)sizeof(T), (uint32_t)N * (uint32_t)sizeof(T), a.M,
                          a.l2pf_rows);
  griddep_wait();
  const float scale = (KIND == B2K_SOFTMAX_SCALE) ? load_scalar(a.scale, a.scale_dtype) : 1.0f;
  RowPipe<1> pipe;
  pipe.init(dsm, S_, a.M, (uint32_t)N * (uint32_t)sizeof(T), srcs, lds, (int)sizeof(T));
  int64_t k = 0;
  for (; k < pipe.nrows; ++k) {
    bool ok;
    const T* xs = reinterpret_cast<const T*>(pipe.wait_next(ok));
    if (!ok) { abort_flag = 1; atomicAdd(&b2k_tu_timeouts, 1u); }
    float2 hv[V][H];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (v * g.G + g.tx) * E;
      if (c < N) unpack2<T>(*reinterpret_cast<const uint4*>(xs + c), hv[v]);
      else
#pragma unroll
        for (int j = 0; j < H; ++j) hv[v][j] = f2s(0.0f);
    }
    // the warp's maximum before the exponentials: the warp stage of the
    // merge is then a plain sum (group_lse_wmax)
    float m, s;
    Slice::template local<true>(hv, N, true, g, scale, m, s);
    float M = m, S = s;
    group_lse_wmax(M, S, g, red);
    if (abort_flag) break;
    pipe.refill();
    Slice::finish(hv, m, M, S);
    T* yr = static_cast<T*>(a.y) + pipe.row_of(k) * a.ldy;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (v * g.G + g.tx) * E;
      if (c < N) st_stream(yr + c, pack2<T>(hv[v]));
    }
  }
  pipe.drain(k);
}

// ---------------------------------------------------------------- long rows
template <typename T, int KIND>
__global__ void __launch_bounds__(kSmMaxThreads) softmax_stream_kernel(const SoftmaxArgs a) {
  constexpr int E = Traits<T>::E;
  constexpr bool P = std::is_same<T, float>::value;
  __shared__ float red[1024];
  const Group g;
  const int64_t row = blockIdx.x;
  const int N = a.N;
  const bool aligned = a.aligned;
  const float scale = (KIND == B2K_SOFTMAX_SCALE) ? load_scalar(a.scale, a.scale_dtype) : 1.0f;
  const T* xr = static_cast<const T*>(a.x) + row * a.ldx;
  auto tr = [&](float x) {
    if constexpr (KIND == B2K_SOFTCAP) return 30.0f * f_tanh_abs<P>(x * (1.0f / 30.0f));
    else if constexpr (KIND == B2K_SOFTMAX_SCALE) return x * scale;
    else return x;
  };
  float m = -INFINITY, s = 0.0f;
  for (int c = g.tx * E; c < N; c += g.G * E) {
    float f[E];
    load_vec<T, false>(f, xr, c, N, aligned);
    float bm = -INFINITY;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      f[e] = (c + e < N) ? tr(f[e]) : -INFINITY;
      bm = fmaxf(bm, f[e]);
    }
    const float nm = fmaxf(m, bm);
    float acc = (m == -INFINITY) ? 0.0f : s * f_exp<P>(m - nm);
#pragma unroll
    for (int e = 0; e < E; ++e) acc += f_exp<P>(f[e] - nm);
    s = acc;
    m = nm;
  }
  float M = m, S = s;
  group_lse(M, S, g, red);
  const float lS = P ? logf(S) : f_log<false>(S);
  const float rS = P ? 1.0f / S : rcp_approx(S);
  T* yr = static_cast<T*>(a.y) + row * a.ldy;
  for (int c = g.tx * E; c < N; c += g.G * E) {
    float f[E];
    load_vec<T, false>(f, xr, c, N, aligned);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float t = tr(f[e]);
      f[e] = (KIND == B2K_LOG_SOFTMAX) ? t - M - lS : f_exp<P>(t - M) * rS;
    }
    store_vec<T>(yr, c, N, aligned, f);
  }
}

static int env_int(const char* name, int dflt) {
  const char* s = getenv(name);
  return s ? atoi(s) : dflt;
}

template <typename T, int KIND>
static int softmax_launch(const SoftmaxArgs& a, cudaStream_t st) {
  constexpr int E = Traits<T>::E;
  static const int use_tma = env_int("B2K_TMA", 1);
  const int64_t nvec = (a.N + E - 1) / E;
  const int64_t row_bytes = (int64_t)a.N * sizeof(T);
  // rows of at most B2K_SM_TMA_MINVEC - 1 vectors (default 128: 2 KB of
  // 16-bit values) go to the rows kernel.  Rows of 256 vectors run 64-thread
  // blocks, up to 16 per SM: 16384 x 2048 fp16 softmax 23.3 us against 29.6
  // us in the rows kernel, softcap 29.1 against 31.1 us.
  static const int min_vec = env_int("B2K_SM_TMA_MINVEC", 129);
  if (use_tma && a.aligned && nvec >= min_vec && row_bytes <= (64 << 10)) {
    static const int want_g = env_int("B2K_TMA_THREADS", 0);
    int G = want_g > 0 ? want_g : next_pow2((nvec + 3) / 4);
    G = G < 64 ? 64 : (G > kSmMaxThreads ? kSmMaxThreads : G);
    const int64_t vneed = (nvec + G - 1) / G;
    PipeShape ps;
    if (vneed <= 4) {
      auto kern = vneed <= 2 ? softmax_tma_kernel<T, KIND, 2> : softmax_tma_kernel<T, KIND, 4>;
      static const int want_cps = env_int("B2K_TMA_CPS", 0);
      static const int want_st = env_int("B2K_TMA_STAGES", 0);
      // 2-stage ring unless set: measured equal or faster on the spec grid
      if (choose_pipe_shape(kern, G, row_bytes, want_cps, want_st > 0 ? want_st : 2, &ps)) {
        const size_t smem = RowPipe<1>::smem_bytes(ps.S, row_bytes);
        int64_t grid = (int64_t)sm_count() * ps.cps;
        if (grid > a.M) grid = a.M;
        launch_pdl(kern, dim3((unsigned)grid), dim3(G), smem, st, a, ps.S);
        return check_launch("b2k_softmax(tma)");
      }
    }
  }
  RowCfg cfg;
  if (choose_row_cfg(a.N, E, 128, &cfg, 4, kSmMaxThreads)) {
    const dim3 block(cfg.G, cfg.R);
    const int64_t grid = (a.M + cfg.R - 1) / cfg.R;
    switch (cfg.V) {
      case 1: launch_pdl(softmax_rows_kernel<T, KIND, 1>, dim3((unsigned)grid), block, 0, st, a); break;
      case 2: launch_pdl(softmax_rows_kernel<T, KIND, 2>, dim3((unsigned)grid), block, 0, st, a); break;
      default: launch_pdl(softmax_rows_kernel<T, KIND, 4>, dim3((unsigned)grid), block, 0, st, a); break;
    }
  } else {
    softmax_stream_kernel<T, KIND><<<a.M, kSmMaxThreads, 0, st>>>(a);
  }
  return check_launch("b2k_softmax");
}

}  // namespace b2k

using namespace b2k;

extern "C" int b2k_softmax(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t M, int64_t N,
                           int dtype, int kind, const void* scale, int scale_dtype, void* stream) {
  B2K_REQUIRE(M >= 0 && N >= 0, "b2k_softmax: negative shape");
  B2K_REQUIRE(kind >= B2K_SOFTMAX && kind <= B2K_SOFTMAX_SCALE, "b2k_softmax: bad kind %d", kind);
  B2K_REQUIRE(kind != B2K_SOFTMAX_SCALE || scale != nullptr, "b2k_softmax: scale required");
  B2K_REQUIRE(kind != B2K_SOFTMAX_SCALE ||
                  (scale_dtype == B2K_F32 || scale_dtype == B2K_F16 || scale_dtype == B2K_BF16),
              "b2k_softmax: bad scale dtype %d", scale_dtype);
  B2K_REQUIRE(M <= 1 || (ldx >= N && ldy >= N), "b2k_softmax: row stride smaller than N");
  B2K_REQUIRE(N < ((int64_t)1 << 30) && M <= 0x7fffffffLL, "b2k_softmax: shape too large");
  if (M == 0 || N == 0) return B2K_OK;
  SoftmaxArgs a;
  a.x = x; a.y = y; a.ldx = ldx; a.ldy = ldy; a.M = M; a.N = (int)N;
  a.scale = scale; a.scale_dtype = scale_dtype;
  a.l2pf_rows = l2_prefetch_rows_knob();
  const int es = dtype_size(dtype);
  const int E = es ? 16 / es : 1;
  a.aligned = (N % E == 0) && aligned16(x) && aligned16(y) && ((ldx * es) % 16 == 0) &&
              ((ldy * es) % 16 == 0);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  B2K_DISPATCH_FLOAT(dtype, {
    switch (kind) {
      case B2K_SOFTMAX: return softmax_launch<T, B2K_SOFTMAX>(a, st);
      case B2K_SOFTCAP: return softmax_launch<T, B2K_SOFTCAP>(a, st);
      case B2K_LOG_SOFTMAX: return softmax_launch<T, B2K_LOG_SOFTMAX>(a, st);
      default: return softmax_launch<T, B2K_SOFTMAX_SCALE>(a, st);
    }
  });
  return B2K_OK;
}
