// Row normalisation family: [x + r] -> {RMS, L2, LayerNorm} -> affine ->
// epilogue.  Covers rmsnorm, add_rmsnorm, layernorm, add_layernorm, l2norm,
// layernorm_gelu, rmsnorm_gemma, rmsnorm_wide and the 76 chains
// (ouroboros/specs.py:75-120,171-190,216-220; ouroboros/chains.py:69-87).
//
// Two kernels:
//  * norm_tma_kernel — aligned rows of 4..64 KB (per input).  Persistent CTAs
//    (a few per SM) walk their rows through an S-stage shared-memory ring
//    filled by bulk copies (cp.async.bulk, mbarrier completion): while one
//    row is normalised, the next S-1 rows are already streaming in.  Weights
//    live in registers for the whole kernel.  Every element is read from HBM
//    once and written once.
//  * norm_rows_kernel — everything else (short rows, several rows per block;
//    odd N / misaligned views with scalar accesses), row in registers, one
//    read, one write; rows beyond 512 threads x 4 slots stream through L2
//    (norm_rows_stream_kernel).
//
// LayerNorm statistics use per-thread two-pass moments merged across the
// block with Chan et al.'s pairwise update (one block reduction per row);
// the result equals the reference's mean-then-centred-variance up to fp32
// rounding.  The (norm, affine) mode and the epilogue are template
// parameters; instances are spread over norm_inst_*.cu.
#pragma once

#include "rowio.cuh"
#include <cooperative_groups.h>

#include "rowpipe.cuh"

namespace b2k {

// supported (norm, affine) combinations
enum NormMode {
  NM_LN = 0,        // LayerNorm, n = (h-mu)*rs*w + b        (+ any epilogue)
  NM_RMS_W = 1,     // n = h*rs*w                            (+ any epilogue)
  NM_RMS_WROUND = 2,// n = T(T(h*rs)*w)                      rmsnorm, add_rmsnorm
  NM_RMS_1PW = 3,   // n = h*rs*(1+w)                        rmsnorm_gemma
  NM_L2 = 4         // n = h*rsqrt(sum(h^2)+eps)             l2norm
};

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
  int aligned;     // all row bases 16-byte aligned and N % E == 0
  int g_target;    // threads-per-row target of the register path
  int tma_threads; // 0 = automatic
  int tma_cps;     // CTAs per SM of the bulk-copy path (0 = automatic)
  int tma_stages;  // pipeline depth (0 = automatic)
  int use_tma;     // 0 disables the bulk-copy path
  int l2_prefetch_rows;  // bulk-copy path: rows per block hinted into L2 before the wait
  int ln_shift;          // bulk-copy path: LayerNorm statistics from shifted sums (else Chan)
};

constexpr int kNormMaxThreads = 512;

template <typename T, int MODE, int ACT>
int norm_launch(const NormArgs& a, cudaStream_t st);

#ifdef B2K_NORM_DEFINE_KERNELS

B2K_DEFINE_TIMEOUT_COUNTER()

// ---------------------------------------------------------------------------
// Affine + epilogue of one pair of elements (f32x2 arithmetic; each lane is
// rounded exactly like the scalar reference expression).
//   nmu2 = (-mu, -mu), rs2 = (rs, rs)
template <typename T, int MODE, int ACT>
__device__ __forceinline__ float2 norm_pair(float2 h, float2 nmu2, float2 rs2, float2 w,
                                            float2 b) {
  constexpr bool P = std::is_same<T, float>::value;
  float2 n;
  if constexpr (MODE == NM_LN) {
    n = fma2(mul2(add2(h, nmu2), rs2), w, b);
  } else if constexpr (MODE == NM_RMS_W) {
    n = mul2(mul2(h, rs2), w);
  } else if constexpr (MODE == NM_RMS_WROUND) {
    // T(T(h*rs) * w): the outer rounding is the store's own conversion to T
    n = mul2(round2<T>(mul2(h, rs2)), w);
  } else if constexpr (MODE == NM_RMS_1PW) {
    n = mul2(mul2(h, rs2), add2(w, f2s(1.0f)));
  } else {
    n = mul2(h, rs2);
  }
  return act_apply2<ACT, P>(n);
}

// ---------------------------------------------------------------------------
// Chan et al. merge of (count, mean, M2) moments
__device__ __forceinline__ void chan_merge(float& n, float& m, float& q, float nb, float mb,
                                           float qb) {
  const float nt = n + nb;
  if (nt == 0.0f) return;
  const float f = __fdividef(nb, nt);
  const float d = mb - m;
  m = fmaf(d, f, m);
  q = q + qb + d * d * n * f;
  n = nt;
}

// Warp stage of the moments: bf16 kernels take plain shuffle sums (SUMS),
// the others Chan's pairwise merge.  The sums (count, n*mean, then
// q + n (mean - warp mean)^2) drop the division per level: the residual
// LayerNorm at 16384 x 8192 bf16 0.1681 -> 0.1676 ms; in the fp16 and fp32
// LayerNorm kernels, already at the 128-register cap, they made ptxas spill
// and those kernels 5-7 % slower, so there the pairwise merge stays.
template <typename T>
constexpr bool kMomentSums = std::is_same<T, __nv_bfloat16>::value;

// group-wide moments; `red` holds 1536 floats ([3][R<=16][32])
template <bool SUMS>
__device__ __forceinline__ void group_moments(float& n, float& m, float& q, const Group& g,
                                              float* red) {
  const int width = g.G < 32 ? g.G : 32;
  if constexpr (SUMS) {
    float nt = n, st = n * m;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      if (o < width) {
        nt += __shfl_xor_sync(0xffffffffu, nt, o);
        st += __shfl_xor_sync(0xffffffffu, st, o);
      }
    const float mt = nt > 0.0f ? st / nt : 0.0f;
    const float d = m - mt;
    float qt = fmaf(n * d, d, q);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      if (o < width) qt += __shfl_xor_sync(0xffffffffu, qt, o);
    n = nt;
    m = mt;
    q = qt;
  } else {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      if (o < width) {
        const float nb = __shfl_xor_sync(0xffffffffu, n, o);
        const float mb = __shfl_xor_sync(0xffffffffu, m, o);
        const float qb = __shfl_xor_sync(0xffffffffu, q, o);
        chan_merge(n, m, q, nb, mb, qb);
      }
  }
  if (g.G > 32) {
    // warp partials -> the group's first warp merges them with shuffles
    const int nw = g.G >> 5, w = g.tx >> 5, lane = g.tx & 31;
    float* rn = red + g.ty * 32;
    float* rm = red + 512 + g.ty * 32;
    float* rq = red + 1024 + g.ty * 32;
    if (lane == 0) { rn[w] = n; rm[w] = m; rq[w] = q; }
    __syncthreads();
    if (w == 0) {
      float a = lane < nw ? rn[lane] : 0.0f;
      float b = lane < nw ? rm[lane] : 0.0f;
      float c = lane < nw ? rq[lane] : 0.0f;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
        if (o < nw) {
          const float nb = __shfl_xor_sync(0xffffffffu, a, o);
          const float mb = __shfl_xor_sync(0xffffffffu, b, o);
          const float qb = __shfl_xor_sync(0xffffffffu, c, o);
          chan_merge(a, b, c, nb, mb, qb);
        }
      if (lane == 0) { rn[0] = a; rm[0] = b; rq[0] = c; }
    }
    __syncthreads();
    n = rn[0]; m = rm[0]; q = rq[0];
    __syncthreads();
  }
}

// LayerNorm statistics of a staged row from sums shifted by K, the row's
// first value (the same in every thread): S = sum (h - K), Q = sum (h - K)^2,
// mean = K + S/N, var = Q/N - (S/N)^2.  Two plain sums in one block reduction:
// no division per merge step and about half the dependent instructions of
// the Chan merge, which bounds these kernels on rows of a few KB.  K is an
// element of the row, so |K - mean| is at most the row's largest deviation
// and the cancellation in Q/N - (S/N)^2 costs at most log2((largest
// deviation / std)^2) bits (a single 1e4 outlier in a unit row of 4096: a
// relative error of ~2e-4 in the variance).  Slots are whole (aligned rows).
template <int V, int H>
__device__ __forceinline__ void ln_stats_shift(const float2 (&hv)[V][H], int N, const Group& g,
                                               float* red, float eps, float K, float& mu,
                                               float& rs) {
  constexpr int E = 2 * H;
  float2 s2 = f2s(0.0f), q2 = f2s(0.0f);
  const float2 nk = f2s(-K);
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * g.G + g.tx) * E;
    if (c < N) {
#pragma unroll
      for (int j = 0; j < H; ++j) {
        const float2 d = add2(hv[v][j], nk);
        s2 = add2(s2, d);
        q2 = fma2(d, d, q2);
      }
    }
  }
  float s = s2.x + s2.y, q = q2.x + q2.y;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    q += __shfl_xor_sync(0xffffffffu, q, o);
  }
  if (g.G > 32) {
    // every warp sums the warp partials itself (two barriers instead of the
    // three of a merge in warp 0 plus a broadcast: 8192 x 4096 fp16 24.7
    // against 26.0 us; the redundant merges cost more than the barrier they
    // save in the exponential-merging and Chan reductions).  Lane 0's sums
    // are taken, so every thread holds the same bits.
    const int nw = g.G >> 5, w = g.tx >> 5, lane = g.tx & 31;
    if (lane == 0) { red[w] = s; red[512 + w] = q; }
    __syncthreads();
    float a = lane < nw ? red[lane] : 0.0f;
    float b = lane < nw ? red[512 + lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      if (o < nw) {
        a += __shfl_xor_sync(0xffffffffu, a, o);
        b += __shfl_xor_sync(0xffffffffu, b, o);
      }
    s = __shfl_sync(0xffffffffu, a, 0);
    q = __shfl_sync(0xffffffffu, b, 0);
    __syncthreads();  // red is written again by the next row
  }
  const float inv = 1.0f / (float)N;
  const float ms = s * inv;
  mu = K + ms;
  rs = rsqrtf(fmaxf(fmaf(q, inv, -ms * ms), 0.0f) + eps);
}

// Statistics of a row slice held as pairs hv[V][H] (slot v covers elements
// [(v*G+tx)*E, +E)); out-of-range elements hold 0.  `whole` = every slot is
// either entirely inside or entirely outside the row (aligned rows).
template <int MODE, int V, int H, bool SUMS>
__device__ __forceinline__ void row_stats(const float2 (&hv)[V][H], int N, bool whole,
                                          const Group& g, float* red, float eps, float& mu,
                                          float& rs) {
  constexpr int E = 2 * H;
  if constexpr (MODE == NM_LN) {
    float2 s2 = f2s(0.0f);
    float cnt = 0.0f;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (v * g.G + g.tx) * E;
      if (whole || c + E <= N) {
        if (c < N) {
#pragma unroll
          for (int j = 0; j < H; ++j) s2 = add2(s2, hv[v][j]);
          cnt += (float)E;
        }
      } else {
        const float* hf = reinterpret_cast<const float*>(hv[v]);
#pragma unroll
        for (int e = 0; e < E; ++e)
          if (c + e < N) { s2.x += hf[e]; cnt += 1.0f; }
      }
    }
    float m = cnt > 0.0f ? (s2.x + s2.y) / cnt : 0.0f;
    const float2 nm2 = f2s(-m);
    float2 q2 = f2s(0.0f);
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (v * g.G + g.tx) * E;
      if (whole || c + E <= N) {
        if (c < N) {
#pragma unroll
          for (int j = 0; j < H; ++j) {
            const float2 d = add2(hv[v][j], nm2);
            q2 = fma2(d, d, q2);
          }
        }
      } else {
        const float* hf = reinterpret_cast<const float*>(hv[v]);
#pragma unroll
        for (int e = 0; e < E; ++e)
          if (c + e < N) { const float d = hf[e] - m; q2.x = fmaf(d, d, q2.x); }
      }
    }
    float q = q2.x + q2.y;
    group_moments<SUMS>(cnt, m, q, g, red);
    mu = m;
    rs = rsqrtf(q / (float)N + eps);
  } else {
    float2 q2 = f2s(0.0f);
#pragma unroll
    for (int v = 0; v < V; ++v)
#pragma unroll
      for (int j = 0; j < H; ++j) q2 = fma2(hv[v][j], hv[v][j], q2);
    const float s = group_sum(q2.x + q2.y, g, red);
    mu = 0.0f;
    rs = rsqrtf((MODE == NM_L2 ? s : s / (float)N) + eps);
  }
}

// pairs of one 16-byte slot from global memory (aligned: one vector load;
// otherwise bounds-checked scalars); out-of-range elements read as 0
template <typename T, bool STREAM>
__device__ __forceinline__ void load_pairs(float2* f, const T* row, int c, int N, bool aligned) {
  load_vec<T, STREAM>(reinterpret_cast<float*>(f), row, c, N, aligned);
}
template <typename T>
__device__ __forceinline__ void store_pairs(T* row, int c, int N, bool aligned, const float2* f) {
  store_vec<T>(row, c, N, aligned, reinterpret_cast<const float*>(f));
}

// ---------------------------------------------------------------------------
// register path
template <typename T, int V, bool RESID, int MODE, int ACT>
__global__ void __launch_bounds__(kNormMaxThreads) norm_rows_kernel(const NormArgs a) {
  constexpr int E = Traits<T>::E;
  constexpr int H = E / 2;
  constexpr bool HAS_W = MODE != NM_L2;
  __shared__ float red[1536];
  const Group g;
  const int64_t row = (int64_t)blockIdx.x * blockDim.y + g.ty;
  const bool valid = row < a.M;
  const int N = (int)a.N;
  const bool aligned = a.aligned;
  {
    const int64_t row0 = (int64_t)blockIdx.x * blockDim.y;
    const int64_t nr = a.M - row0 < (int64_t)blockDim.y ? a.M - row0 : (int64_t)blockDim.y;
    pdl_rows_prologue(a.x, a.ldx * (int64_t)sizeof(T), RESID ? a.r : nullptr,
                      a.ldr * (int64_t)sizeof(T), row0, nr, (uint32_t)N * (uint32_t)sizeof(T),
                      aligned && a.l2_prefetch_rows > 0);
  }
  const T* xr = static_cast<const T*>(a.x) + (valid ? row * a.ldx : 0);
  const T* rr = RESID ? static_cast<const T*>(a.r) + (valid ? row * a.ldr : 0) : nullptr;

  float2 hv[V][H];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * g.G + g.tx) * E;
    if (valid) {
      load_pairs<T, true>(hv[v], xr, c, N, aligned);
    } else {
#pragma unroll
      for (int j = 0; j < H; ++j) hv[v][j] = f2s(0.0f);
    }
  }
  if (RESID && valid) {
#pragma unroll
    for (int v = 0; v < V; ++v) {
      float2 t[H];
      load_pairs<T, true>(t, rr, (v * g.G + g.tx) * E, N, aligned);
#pragma unroll
      for (int j = 0; j < H; ++j) hv[v][j] = add2(hv[v][j], t[j]);
    }
  }
  if (a.h != nullptr && valid) {
    T* hrow = static_cast<T*>(a.h) + row * a.ldh;
#pragma unroll
    for (int v = 0; v < V; ++v) store_pairs<T>(hrow, (v * g.G + g.tx) * E, N, aligned, hv[v]);
  }

  float mu, rs;
  row_stats<MODE, V, H, kMomentSums<T>>(hv, N, aligned, g, red, a.eps, mu, rs);
  if (!valid) return;

  const float2 nmu2 = f2s(-mu), rs2 = f2s(rs);
  T* yrow = static_cast<T*>(a.y) + row * a.ldy;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * g.G + g.tx) * E;
    float2 wv[H], bv[H], out[H];
    if constexpr (HAS_W) load_pairs<T, false>(wv, static_cast<const T*>(a.w), c, N, aligned);
    if constexpr (MODE == NM_LN) load_pairs<T, false>(bv, static_cast<const T*>(a.b), c, N, aligned);
#pragma unroll
    for (int j = 0; j < H; ++j)
      out[j] = norm_pair<T, MODE, ACT>(hv[v][j], nmu2, rs2, HAS_W ? wv[j] : f2s(1.0f),
                                       MODE == NM_LN ? bv[j] : f2s(0.0f));
    store_pairs<T>(yrow, c, N, aligned, out);
  }
}

// rows longer than the register budget: one row per block, statistics from
// L2-friendly re-reads (LayerNorm: mean pass, centred-variance pass)
template <typename T, bool RESID, int MODE, int ACT>
__global__ void __launch_bounds__(kNormMaxThreads) norm_rows_stream_kernel(const NormArgs a) {
  constexpr int E = Traits<T>::E;
  constexpr int H = E / 2;
  constexpr bool HAS_W = MODE != NM_L2;
  __shared__ float red[1536];
  const Group g;
  const int64_t row = blockIdx.x;
  const int N = (int)a.N;
  const bool aligned = a.aligned;
  const T* xr = static_cast<const T*>(a.x) + row * a.ldx;
  const T* rr = RESID ? static_cast<const T*>(a.r) + row * a.ldr : nullptr;
  T* hrow = a.h ? static_cast<T*>(a.h) + row * a.ldh : nullptr;
  const int step = g.G * E;

  auto load_h = [&](float2* hv, int c) {
    load_pairs<T, false>(hv, xr, c, N, aligned);
    if (RESID) {
      float2 t[H];
      load_pairs<T, false>(t, rr, c, N, aligned);
#pragma unroll
      for (int j = 0; j < H; ++j) hv[j] = add2(hv[j], t[j]);
    }
  };

  float mu = 0.0f, rs;
  float2 s2 = f2s(0.0f);
  for (int c = g.tx * E; c < N; c += step) {
    float2 hv[H];
    load_h(hv, c);
    if (hrow) store_pairs<T>(hrow, c, N, aligned, hv);
#pragma unroll
    for (int j = 0; j < H; ++j) s2 = (MODE == NM_LN) ? add2(s2, hv[j]) : fma2(hv[j], hv[j], s2);
  }
  const float s = group_sum(s2.x + s2.y, g, red);
  if constexpr (MODE == NM_LN) {
    mu = s / (float)N;
    float q = 0.0f;
    for (int c = g.tx * E; c < N; c += step) {
      float2 hv[H];
      load_h(hv, c);
      const float* hf = reinterpret_cast<const float*>(hv);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float d = (c + e < N) ? hf[e] - mu : 0.0f;
        q = fmaf(d, d, q);
      }
    }
    q = group_sum(q, g, red);
    rs = rsqrtf(q / (float)N + a.eps);
  } else {
    rs = rsqrtf((MODE == NM_L2 ? s : s / (float)N) + a.eps);
  }
  const float2 nmu2 = f2s(-mu), rs2 = f2s(rs);
  T* yrow = static_cast<T*>(a.y) + row * a.ldy;
  for (int c = g.tx * E; c < N; c += step) {
    float2 hv[H], wv[H], bv[H], out[H];
    load_h(hv, c);
    if constexpr (HAS_W) load_pairs<T, false>(wv, static_cast<const T*>(a.w), c, N, aligned);
    if constexpr (MODE == NM_LN) load_pairs<T, false>(bv, static_cast<const T*>(a.b), c, N, aligned);
#pragma unroll
    for (int j = 0; j < H; ++j)
      out[j] = norm_pair<T, MODE, ACT>(hv[j], nmu2, rs2, HAS_W ? wv[j] : f2s(1.0f),
                                       MODE == NM_LN ? bv[j] : f2s(0.0f));
    store_pairs<T>(yrow, c, N, aligned, out);
  }
}

// ---------------------------------------------------------------------------
// bulk-copy pipelined path (aligned rows only)
template <typename T, int V, bool RESID, int MODE, int ACT>
__global__ void __launch_bounds__(kNormMaxThreads) norm_tma_kernel(const NormArgs a, const int S) {
  constexpr int E = Traits<T>::E;
  constexpr int H = E / 2;
  constexpr bool HAS_W = MODE != NM_L2;
  constexpr int NIN = RESID ? 2 : 1;
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ float red[1536];
  __shared__ volatile int abort_flag;
  const Group g;  // G = blockDim.x, one row at a time
  const int N = (int)a.N;
  if (g.tx == 0) abort_flag = 0;
  griddep_launch_dependents();
  const void* srcs[2] = {a.x, a.r};
  const int64_t lds[2] = {a.ldx, a.ldr};
  RowPipe<NIN>::prefetch_l2(srcs, lds, (int)sizeof(T), (uint32_t)N * (uint32_t)sizeof(T), a.M,
                            a.l2_prefetch_rows);
  griddep_wait();  // inputs may come from the previous kernel in the stream
  RowPipe<NIN> pipe;
  pipe.init(dsm, S, a.M, (uint32_t)N * (uint32_t)sizeof(T), srcs, lds, (int)sizeof(T));

  // weight slices stay in registers (raw 16-byte vectors) for every row
  uint4 wraw[V], braw[V];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * g.G + g.tx) * E;
    wraw[v] = (HAS_W && c < N) ? ld_keep(static_cast<const T*>(a.w) + c) : zero4();
    braw[v] = (MODE == NM_LN && c < N) ? ld_keep(static_cast<const T*>(a.b) + c) : zero4();
  }

  int64_t k = 0;
  for (; k < pipe.nrows; ++k) {
    bool ok;
    const T* xs = reinterpret_cast<const T*>(pipe.wait_next(ok));
    if (!ok) {
      abort_flag = 1;  // garbage row; every thread leaves after the reduction
      atomicAdd(&b2k_tu_timeouts, 1u);
    }
    const T* rsm = xs + N;
    const int64_t row = pipe.row_of(k);
    float2 hv[V][H];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (v * g.G + g.tx) * E;
      if (c < N) {
        unpack2<T>(*reinterpret_cast<const uint4*>(xs + c), hv[v]);
        if (RESID) {
          float2 t[H];
          unpack2<T>(*reinterpret_cast<const uint4*>(rsm + c), t);
#pragma unroll
          for (int j = 0; j < H; ++j) hv[v][j] = add2(hv[v][j], t[j]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < H; ++j) hv[v][j] = f2s(0.0f);
      }
    }
    // the shift of the LayerNorm sums: the row's first value (x + r as the
    // threads formed it), read from the stage
    float K = 0.0f;
    if (MODE == NM_LN && a.ln_shift) {
      K = to_f<T>(xs[0]);
      if constexpr (RESID) K += to_f<T>(rsm[0]);
    }
    if (a.h != nullptr) {
      T* hrow = static_cast<T*>(a.h) + row * a.ldh;
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const int c = (v * g.G + g.tx) * E;
        if (c < N) st_stream(hrow + c, pack2<T>(hv[v]));
      }
    }
    float mu, rs;
    if (MODE == NM_LN && a.ln_shift) {
      ln_stats_shift<V, H>(hv, N, g, red, a.eps, K, mu, rs);
    } else {
      row_stats<MODE, V, H, kMomentSums<T>>(hv, N, true, g, red, a.eps, mu, rs);
    }
    // the reduction's barriers order every thread's reads of the stage
    // before the refill
    if (abort_flag) break;
    pipe.refill();
    const float2 nmu2 = f2s(-mu), rs2 = f2s(rs);
    T* yrow = static_cast<T*>(a.y) + row * a.ldy;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (v * g.G + g.tx) * E;
      if (c < N) {
        float2 wv[H], bv[H], out[H];
        if constexpr (HAS_W) unpack2<T>(wraw[v], wv);
        if constexpr (MODE == NM_LN) unpack2<T>(braw[v], bv);
#pragma unroll
        for (int j = 0; j < H; ++j)
          out[j] = norm_pair<T, MODE, ACT>(hv[v][j], nmu2, rs2, HAS_W ? wv[j] : f2s(1.0f),
                                           MODE == NM_LN ? bv[j] : f2s(0.0f));
        st_stream(yrow + c, pack2<T>(out));
      }
    }
  }
  pipe.drain(k);
}

// ---------------------------------------------------------------------------
// Few long rows (rmsnorm_wide, specs.py:866-871: M <= 32, N up to 131072):
// a thread-block cluster of C CTAs splits each row into C contiguous
// segments held in registers; every CTA reduces its segment, the partials are
// exchanged through distributed shared memory, and each CTA normalises its
// own segment.  One read and one write per element, M*C CTAs in flight
// instead of M.
template <typename T, bool RESID, int MODE>
__global__ void __launch_bounds__(kNormMaxThreads) norm_cluster_kernel(const NormArgs a,
                                                                       const int seg) {
  namespace cg = cooperative_groups;
  constexpr int E = Traits<T>::E;
  constexpr int H = E / 2;
  constexpr int V = 4;
  constexpr bool HAS_W = MODE != NM_L2;
  __shared__ float red[1536];
  __shared__ float part[3];
  __shared__ float fin[2];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int C = (int)cluster.num_blocks();
  const Group g;
  const int64_t row = blockIdx.y;
  const int N = (int)a.N;
  const int c0 = rank * seg;
  const int nh = N - c0 < seg ? (N - c0 > 0 ? N - c0 : 0) : seg;  // elements of this segment
  const T* xr = static_cast<const T*>(a.x) + row * a.ldx + c0;
  const T* rr = RESID ? static_cast<const T*>(a.r) + row * a.ldr + c0 : nullptr;

  float2 hv[V][H];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * g.G + g.tx) * E;
    load_pairs<T, true>(hv[v], xr, c, nh, true);
    if (RESID) {
      float2 t[H];
      load_pairs<T, true>(t, rr, c, nh, true);
#pragma unroll
      for (int j = 0; j < H; ++j) hv[v][j] = add2(hv[v][j], t[j]);
    }
  }
  if (a.h != nullptr) {
    T* hrow = static_cast<T*>(a.h) + row * a.ldh + c0;
#pragma unroll
    for (int v = 0; v < V; ++v) store_pairs<T>(hrow, (v * g.G + g.tx) * E, nh, true, hv[v]);
  }
  // partial statistics of the segment
  if constexpr (MODE == NM_LN) {
    float2 s2 = f2s(0.0f);
    float cnt = 0.0f;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (v * g.G + g.tx) * E;
      if (c < nh) {
#pragma unroll
        for (int j = 0; j < H; ++j) s2 = add2(s2, hv[v][j]);
        cnt += (float)E;
      }
    }
    float m = cnt > 0.0f ? (s2.x + s2.y) / cnt : 0.0f, q = 0.0f;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (v * g.G + g.tx) * E;
      if (c < nh) {
#pragma unroll
        for (int j = 0; j < H; ++j) {
          const float2 d = add2(hv[v][j], f2s(-m));
          q = fmaf(d.x, d.x, fmaf(d.y, d.y, q));
        }
      }
    }
    group_moments<kMomentSums<T>>(cnt, m, q, g, red);
    if (g.tx == 0) { part[0] = cnt; part[1] = m; part[2] = q; }
  } else {
    float2 q2 = f2s(0.0f);
#pragma unroll
    for (int v = 0; v < V; ++v)
#pragma unroll
      for (int j = 0; j < H; ++j) q2 = fma2(hv[v][j], hv[v][j], q2);
    const float s = group_sum(q2.x + q2.y, g, red);
    if (g.tx == 0) part[0] = s;
  }
  cluster.sync();  // partials of every segment visible cluster-wide
  if (g.tx == 0) {
    float mu = 0.0f, rs;
    if constexpr (MODE == NM_LN) {
      float n = 0.0f, m = 0.0f, q = 0.0f;
      for (int r = 0; r < C; ++r) {
        const float* pr = cluster.map_shared_rank(part, r);
        chan_merge(n, m, q, pr[0], pr[1], pr[2]);
      }
      mu = m;
      rs = rsqrtf(q / (float)N + a.eps);
    } else {
      float s = 0.0f;
      for (int r = 0; r < C; ++r) s += *cluster.map_shared_rank(part, r);
      rs = rsqrtf((MODE == NM_L2 ? s : s / (float)N) + a.eps);
    }
    fin[0] = mu;
    fin[1] = rs;
  }
  __syncthreads();
  const float2 nmu2 = f2s(-fin[0]), rs2 = f2s(fin[1]);
  T* yrow = static_cast<T*>(a.y) + row * a.ldy + c0;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * g.G + g.tx) * E;
    if (c < nh) {
      float2 wv[H], bv[H], out[H];
      if constexpr (HAS_W) load_pairs<T, false>(wv, static_cast<const T*>(a.w) + c0, c, nh, true);
      if constexpr (MODE == NM_LN) load_pairs<T, false>(bv, static_cast<const T*>(a.b) + c0, c, nh, true);
#pragma unroll
      for (int j = 0; j < H; ++j)
        out[j] = norm_pair<T, MODE, 0>(hv[v][j], nmu2, rs2, HAS_W ? wv[j] : f2s(1.0f),
                                       MODE == NM_LN ? bv[j] : f2s(0.0f));
      store_pairs<T>(yrow, c, nh, true, out);
    }
  }
  cluster.sync();  // no block leaves while another may still read its partial
}

template <typename T, bool RESID, int MODE>
static bool norm_try_cluster(const NormArgs& a, cudaStream_t st, int* status) {
  constexpr int E = Traits<T>::E;
  if (!a.aligned || a.M > 64 || a.N / E < 2048) return false;
  const int sms = sm_count();
  // cluster size: enough blocks to cover the SMs about twice, within 2..16,
  // and large enough that a segment fits 512 threads x 4 vectors
  int C = next_pow2((2 * sms + a.M - 1) / a.M);
  C = C < 2 ? 2 : (C > 16 ? 16 : C);
  int64_t seg = 0;
  for (;; C <<= 1) {
    if (C > 16) return false;
    seg = ((a.N + C - 1) / C + E - 1) / E * E;
    if (seg / E <= (int64_t)kNormMaxThreads * 4) break;
  }
  int G = next_pow2((seg / E + 3) / 4);
  G = G < 64 ? 64 : (G > kNormMaxThreads ? kNormMaxThreads : G);
  auto kern = norm_cluster_kernel<T, RESID, MODE>;
  if (C > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) !=
                   cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)C, (unsigned)a.M, 1);
  cfg.blockDim = dim3((unsigned)G, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kern, a, (int)seg) != cudaSuccess) {
    cudaGetLastError();  // cluster shape not available: use another kernel
    return false;
  }
  *status = check_launch("b2k_norm(cluster)");
  return true;
}

// ---------------------------------------------------------------------------
// launch
template <typename T, bool RESID, int MODE, int ACT>
static bool norm_try_tma(const NormArgs& a, cudaStream_t st, int* status) {
  constexpr int E = Traits<T>::E;
  if (!a.use_tma || !a.aligned) return false;
  const int64_t nvec = a.N / E;
  if (nvec < 256) return false;  // short rows: register path packs several rows per block
  const int64_t stage = (RESID ? 2 : 1) * a.N * (int64_t)sizeof(T);
  if (stage > (64 << 10)) return false;
  int G = a.tma_threads;
  if (G <= 0) {
    // RMS / L2: two vectors per thread while that fits 256 threads (rows of
    // <= 512 vectors: more warps per row, fewer registers), else four.
    // LayerNorm (a costlier block reduction per row): four.
    G = MODE == NM_LN ? 1 << 30 : next_pow2((nvec + 1) / 2);
    if (G > 256) G = next_pow2((nvec + 3) / 4);
    G = G < 64 ? 64 : (G > kNormMaxThreads ? kNormMaxThreads : G);
  }
  const int64_t vneed = (nvec + G - 1) / G;
  if (vneed > 4) return false;  // longer rows: register / streaming kernels
  const int sms = sm_count();
  auto kern = (vneed <= 2) ? norm_tma_kernel<T, 2, RESID, MODE, ACT> : norm_tma_kernel<T, 4, RESID, MODE, ACT>;
  // a 2-stage ring with as many blocks per SM as are resident: measured equal
  // or faster than deeper rings for every norm shape of the spec grid and for
  // add -> LayerNorm -> GELU at 16384 x 8192 (167.8 against 170.2 us with 3
  // stages): more blocks in flight beat a deeper ring per block
  int want_stages = a.tma_stages;
  if (want_stages <= 0) want_stages = 2;
  PipeShape ps;
  if (!choose_pipe_shape(kern, G, stage, a.tma_cps, want_stages, &ps)) return false;
  const int cps = ps.cps, S = ps.S;
  const size_t smem = RowPipe<RESID ? 2 : 1>::smem_bytes(S, a.N * (int64_t)sizeof(T));
  int64_t grid = (int64_t)sms * cps;
  if (grid > a.M) grid = a.M;
  // LayerNorm statistics (B2K_LN_SHIFT: 0 Chan's merge, 2 shifted sums, 1 =
  // by shape): shifted sums, except when the residual stream is written and
  // each block walks 8 rows or more, where Chan's merge measured faster
  // (x + r -> LayerNorm -> GELU, 8192-wide bf16 rows with h, fractions of the
  // copy peak, Chan against shifted: 16384 rows 0.977 / 0.87, 4096 rows
  // 0.914 / 0.845, 3072 rows (10.4 per block) 0.881 / 0.871, 2048 rows (6.9
  // per block) 0.854 / 0.926; without h the shifted sums win at every shape,
  // LayerNorm 8192 x 4096 bf16 0.81 against 0.64)
  NormArgs b = a;
  if (MODE == NM_LN && a.ln_shift == 1)
    b.ln_shift = (a.h == nullptr || a.M < 8 * grid) ? 1 : 0;
  launch_pdl(kern, (unsigned)grid, (unsigned)G, smem, st, b, S);
  *status = check_launch("b2k_norm(tma)");
  return true;
}

template <typename T, bool RESID, int MODE, int ACT>
static int norm_launch_resid(const NormArgs& a, cudaStream_t st) {
  constexpr int E = Traits<T>::E;
  int status;
  if (norm_try_tma<T, RESID, MODE, ACT>(a, st, &status)) return status;
  if constexpr (ACT == 0) {
    if (a.use_tma && norm_try_cluster<T, RESID, MODE>(a, st, &status)) return status;
  }
  RowCfg cfg;
  if (choose_row_cfg(a.N, E, a.g_target, &cfg, 4, kNormMaxThreads)) {
    const dim3 block(cfg.G, cfg.R);
    const int64_t grid = (a.M + cfg.R - 1) / cfg.R;
    switch (cfg.V) {
      case 1: launch_pdl(norm_rows_kernel<T, 1, RESID, MODE, ACT>, dim3((unsigned)grid), block, 0, st, a); break;
      case 2: launch_pdl(norm_rows_kernel<T, 2, RESID, MODE, ACT>, dim3((unsigned)grid), block, 0, st, a); break;
      default: launch_pdl(norm_rows_kernel<T, 4, RESID, MODE, ACT>, dim3((unsigned)grid), block, 0, st, a); break;
    }
  } else {
    norm_rows_stream_kernel<T, RESID, MODE, ACT><<<a.M, dim3(kNormMaxThreads, 1), 0, st>>>(a);
  }
  return check_launch("b2k_norm");
}

template <typename T, int MODE, int ACT>
int norm_launch(const NormArgs& a, cudaStream_t st) {
  return a.r ? norm_launch_resid<T, true, MODE, ACT>(a, st)
             : norm_launch_resid<T, false, MODE, ACT>(a, st);
}

#define B2K_NORM_INSTANTIATE(T, MODE, ACT) \
  template int norm_launch<T, MODE, ACT>(const NormArgs&, cudaStream_t);

#endif  // B2K_NORM_DEFINE_KERNELS

}  // namespace b2k
