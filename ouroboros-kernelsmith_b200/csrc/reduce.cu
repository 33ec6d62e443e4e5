// Double reductions and the scan of the op suite: entropy of softmax(x)
// (ouroboros/specs.py:251-256), KL(softmax(x) || softmax(y)) from logit pairs
// (specs.py:259-265) and the row-wise inclusive prefix sum (specs.py:245-248).
//
// entropy / kl_div: one row per thread group, the row(s) read once into
// registers; the passes of the reference (max, logsumexp, weighted sum) run
// over registers with one group reduction each.  Rows beyond the register
// budget re-read the row from L2 per pass.
// cumsum: chunks of G*E elements in row order; per chunk a thread scans its
// E contiguous elements, the group scans the thread totals, and a running
// carry joins the chunks.  Accumulation is in fp64 (torch's CPU cumsum of
// float accumulates in double), output rounded once to fp32 and then to T.
#include "rowio.cuh"

namespace b2k {

constexpr int kRedMaxThreads = 512;

struct RowRedArgs {
  const void* x;
  const void* y;
  void* out;
  int64_t ldx, ldy, ldo, M;
  int N;
  int aligned;
};

// ---------------------------------------------------------------- entropy
template <typename T, int V>
__global__ void __launch_bounds__(kRedMaxThreads) entropy_rows_kernel(const RowRedArgs a) {
  constexpr int E = Traits<T>::E;
  constexpr bool P = std::is_same<T, float>::value;
  __shared__ float red[1024];
  const Group g;
  const int64_t row = (int64_t)blockIdx.x * blockDim.y + g.ty;
  const bool valid = row < a.M;
  const int N = valid ? a.N : 0;
  const T* xr = static_cast<const T*>(a.x) + (valid ? row * a.ldx : 0);
  float xv[V][E];
  float m = -INFINITY;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * g.G + g.tx) * E;
    load_vec_fill<T, true>(xv[v], xr, c, N, a.aligned, -INFINITY);
#pragma unroll
    for (int e = 0; e < E; ++e) m = fmaxf(m, xv[v][e]);
  }
  const float M = group_max(m, g, red);
  float s = 0.0f;
#pragma unroll
  for (int v = 0; v < V; ++v)
#pragma unroll
    for (int e = 0; e < E; ++e)
      if (xv[v][e] != -INFINITY) s += f_exp<P>(xv[v][e] - M);
  s = group_sum(s, g, red);
  // the reference's order (specs.py:253-256): lse, p = exp(x - lse), then
  // lse - sum(x * p).  For peaked rows the two terms nearly cancel and the
  // fp32 rounding of lse dominates the result, so the same order is used.
  const float lse = M + (P ? logf(s) : f_log<false>(s));
  float q = 0.0f;
#pragma unroll
  for (int v = 0; v < V; ++v)
#pragma unroll
    for (int e = 0; e < E; ++e)
      if (xv[v][e] != -INFINITY) q = fmaf(xv[v][e], f_exp<P>(xv[v][e] - lse), q);
  q = group_sum(q, g, red);
  if (valid && g.tx == 0) static_cast<T*>(a.out)[row * a.ldo] = from_f<T>(lse - q);
}

// ---------------------------------------------------------------- kl
template <typename T, int V>
__global__ void __launch_bounds__(kRedMaxThreads) kl_rows_kernel(const RowRedArgs a) {
  constexpr int E = Traits<T>::E;
  constexpr bool P = std::is_same<T, float>::value;
  __shared__ float red[1024];
  const Group g;
  const int64_t row = (int64_t)blockIdx.x * blockDim.y + g.ty;
  const bool valid = row < a.M;
  const int N = valid ? a.N : 0;
  const T* xr = static_cast<const T*>(a.x) + (valid ? row * a.ldx : 0);
  const T* yr = static_cast<const T*>(a.y) + (valid ? row * a.ldy : 0);
  float xv[V][E], yv[V][E];
  float mx = -INFINITY, my = -INFINITY;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * g.G + g.tx) * E;
    load_vec_fill<T, true>(xv[v], xr, c, N, a.aligned, -INFINITY);
    load_vec_fill<T, true>(yv[v], yr, c, N, a.aligned, -INFINITY);
#pragma unroll
    for (int e = 0; e < E; ++e) { mx = fmaxf(mx, xv[v][e]); my = fmaxf(my, yv[v][e]); }
  }
  mx = group_max(mx, g, red);
  my = group_max(my, g, red);
  float sx = 0.0f, sy = 0.0f;
#pragma unroll
  for (int v = 0; v < V; ++v)
#pragma unroll
    for (int e = 0; e < E; ++e) {
      if (xv[v][e] == -INFINITY) continue;
      sx += f_exp<P>(xv[v][e] - mx);
      sy += f_exp<P>(yv[v][e] - my);
    }
  sx = group_sum(sx, g, red);
  sy = group_sum(sy, g, red);
  // lx = x - lse(x), ly = y - lse(y); out = sum exp(lx) * (lx - ly)
  const float lsex = mx + (P ? logf(sx) : f_log<false>(sx));
  const float lsey = my + (P ? logf(sy) : f_log<false>(sy));
  float acc = 0.0f;
#pragma unroll
  for (int v = 0; v < V; ++v)
#pragma unroll
    for (int e = 0; e < E; ++e) {
      if (xv[v][e] == -INFINITY) continue;
      const float lx = xv[v][e] - lsex, ly = yv[v][e] - lsey;
      acc = fmaf(f_exp<P>(lx), lx - ly, acc);
    }
  acc = group_sum(acc, g, red);
  if (valid && g.tx == 0) static_cast<T*>(a.out)[row * a.ldo] = from_f<T>(acc);
}

// rows beyond the register budget: the same passes, re-reading the row
template <typename T, bool KL>
__global__ void __launch_bounds__(kRedMaxThreads) rowred_stream_kernel(const RowRedArgs a) {
  constexpr int E = Traits<T>::E;
  constexpr bool P = std::is_same<T, float>::value;
  __shared__ float red[1024];
  const Group g;
  const int64_t row = blockIdx.x;
  const int N = a.N;
  const T* xr = static_cast<const T*>(a.x) + row * a.ldx;
  const T* yr = KL ? static_cast<const T*>(a.y) + row * a.ldy : nullptr;
  const int step = g.G * E;
  float mx = -INFINITY, my = -INFINITY;
  for (int c = g.tx * E; c < N; c += step) {
    float f[E];
    load_vec_fill<T, false>(f, xr, c, N, a.aligned, -INFINITY);
#pragma unroll
    for (int e = 0; e < E; ++e) mx = fmaxf(mx, f[e]);
    if (KL) {
      load_vec_fill<T, false>(f, yr, c, N, a.aligned, -INFINITY);
#pragma unroll
      for (int e = 0; e < E; ++e) my = fmaxf(my, f[e]);
    }
  }
  mx = group_max(mx, g, red);
  if (KL) my = group_max(my, g, red);
  float s = 0.0f, q = 0.0f;
  for (int c = g.tx * E; c < N; c += step) {
    float f[E], h[E];
    load_vec_fill<T, false>(f, xr, c, N, a.aligned, -INFINITY);
    if (KL) load_vec_fill<T, false>(h, yr, c, N, a.aligned, -INFINITY);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      if (f[e] == -INFINITY) continue;
      s += f_exp<P>(f[e] - mx);
      if (KL) q += f_exp<P>(h[e] - my);
    }
  }
  s = group_sum(s, g, red);
  if (KL) q = group_sum(q, g, red);
  float res;
  if (!KL) {
    // reference order: lse, then lse - sum(x * exp(x - lse))
    const float lse = mx + (P ? logf(s) : f_log<false>(s));
    float acc = 0.0f;
    for (int c = g.tx * E; c < N; c += step) {
      float f[E];
      load_vec_fill<T, false>(f, xr, c, N, a.aligned, -INFINITY);
#pragma unroll
      for (int e = 0; e < E; ++e)
        if (f[e] != -INFINITY) acc = fmaf(f[e], f_exp<P>(f[e] - lse), acc);
    }
    res = lse - group_sum(acc, g, red);
  } else {
    const float lsex = mx + (P ? logf(s) : f_log<false>(s));
    const float lsey = my + (P ? logf(q) : f_log<false>(q));
    float acc = 0.0f;
    for (int c = g.tx * E; c < N; c += step) {
      float f[E], h[E];
      load_vec_fill<T, false>(f, xr, c, N, a.aligned, -INFINITY);
      load_vec_fill<T, false>(h, yr, c, N, a.aligned, -INFINITY);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        if (f[e] == -INFINITY) continue;
        const float lx = f[e] - lsex, ly = h[e] - lsey;
        acc = fmaf(f_exp<P>(lx), lx - ly, acc);
      }
    }
    res = group_sum(acc, g, red);
  }
  if (g.tx == 0) static_cast<T*>(a.out)[row * a.ldo] = from_f<T>(res);
}

// ---------------------------------------------------------------- cumsum
// inclusive scan of a double across the G threads of the group
__device__ __forceinline__ double group_scan_incl(double v, const Group& g, double* sred) {
  const int lane = g.tx & 31;
  const int width = g.G < 32 ? g.G : 32;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    if (o < width) {
      const double u = __shfl_up_sync(0xffffffffu, v, o, width);
      if ((lane % width) >= o) v += u;
    }
  }
  if (g.G > 32) {
    const int w = g.tx >> 5, nw = g.G >> 5;
    if (lane == 31) sred[g.ty * 32 + w] = v;
    __syncthreads();
    double off = 0.0;
    for (int i = 0; i < w; ++i) off += sred[g.ty * 32 + i];
    __syncthreads();
    (void)nw;
    v += off;
  }
  return v;
}

__device__ __forceinline__ double group_bcast_last(double v, const Group& g, double* sred) {
  // value of the group's last thread, to every thread of the group
  if (g.G <= 32) return __shfl_sync(0xffffffffu, v, g.G - 1, g.G < 32 ? g.G : 32);
  if (g.tx == g.G - 1) sred[512 + g.ty] = v;
  __syncthreads();
  const double r = sred[512 + g.ty];
  __syncthreads();
  return r;
}

template <typename T>
__global__ void __launch_bounds__(kRedMaxThreads) cumsum_kernel(const RowRedArgs a) {
  constexpr int E = Traits<T>::E;
  __shared__ double sred[512 + 32];
  const Group g;
  const int64_t row = (int64_t)blockIdx.x * blockDim.y + g.ty;
  const bool valid = row < a.M;
  const int N = valid ? a.N : 0;
  const int nN = a.N;
  const T* xr = static_cast<const T*>(a.x) + (valid ? row * a.ldx : 0);
  T* yr = static_cast<T*>(a.out) + (valid ? row * a.ldo : 0);
  double carry = 0.0;
  for (int c0 = 0; c0 < nN; c0 += g.G * E) {
    const int c = c0 + g.tx * E;
    float f[E];
    load_vec<T, false>(f, xr, c, N, a.aligned);
    double loc[E];
    double run = 0.0;
#pragma unroll
    for (int e = 0; e < E; ++e) { run += (double)f[e]; loc[e] = run; }
    const double incl = group_scan_incl(run, g, sred);
    const double excl = incl - run;
    const double total = group_bcast_last(incl, g, sred);
    float o[E];
#pragma unroll
    for (int e = 0; e < E; ++e) o[e] = (float)(carry + excl + loc[e]);
    store_vec<T>(yr, c, N, a.aligned, o);
    carry += total;
  }
}

template <typename T>
static int rowred_launch(const RowRedArgs& a, bool kl, cudaStream_t st) {
  constexpr int E = Traits<T>::E;
  RowCfg cfg;
  if (choose_row_cfg(a.N, E, 128, &cfg, 4, kRedMaxThreads)) {
    const dim3 block(cfg.G, cfg.R);
    const int64_t grid = (a.M + cfg.R - 1) / cfg.R;
    auto go = [&](auto kern) { kern<<<(unsigned)grid, block, 0, st>>>(a); };
    if (kl) {
      switch (cfg.V) {
        case 1: go(kl_rows_kernel<T, 1>); break;
        case 2: go(kl_rows_kernel<T, 2>); break;
        default: go(kl_rows_kernel<T, 4>); break;
      }
    } else {
      switch (cfg.V) {
        case 1: go(entropy_rows_kernel<T, 1>); break;
        case 2: go(entropy_rows_kernel<T, 2>); break;
        default: go(entropy_rows_kernel<T, 4>); break;
      }
    }
  } else {
    if (kl) rowred_stream_kernel<T, true><<<(unsigned)a.M, kRedMaxThreads, 0, st>>>(a);
    else rowred_stream_kernel<T, false><<<(unsigned)a.M, kRedMaxThreads, 0, st>>>(a);
  }
  return check_launch(kl ? "b2k_kl_div" : "b2k_entropy");
}

template <typename T>
static int cumsum_launch(const RowRedArgs& a, cudaStream_t st) {
  constexpr int E = Traits<T>::E;
  const int64_t nvec = (a.N + E - 1) / E;
  int G = next_pow2(nvec);
  G = G < 1 ? 1 : (G > 256 ? 256 : G);
  const int R = G >= 256 ? 1 : 256 / G;
  const int64_t grid = (a.M + R - 1) / R;
  cumsum_kernel<T><<<(unsigned)grid, dim3(G, R), 0, st>>>(a);
  return check_launch("b2k_cumsum");
}

static bool rows_aligned(const void* x, int64_t ldx, const void* y, int64_t ldy, int64_t N,
                         int es) {
  const int E = es ? 16 / es : 1;
  bool al = (N % E == 0) && aligned16(x) && ((ldx * es) % 16 == 0);
  if (y) al = al && aligned16(y) && ((ldy * es) % 16 == 0);
  return al;
}

}  // namespace b2k

using namespace b2k;

extern "C" int b2k_entropy(const void* x, int64_t ldx, void* out, int64_t M, int64_t N, int dtype,
                           void* stream) {
  B2K_REQUIRE(M >= 0 && N >= 1, "b2k_entropy: need M >= 0 and N >= 1");
  B2K_REQUIRE(M <= 1 || ldx >= N, "b2k_entropy: row stride smaller than N");
  B2K_REQUIRE(N < ((int64_t)1 << 30) && M <= 0x7fffffffLL, "b2k_entropy: shape too large");
  if (M == 0) return B2K_OK;
  RowRedArgs a;
  a.x = x; a.y = nullptr; a.out = out; a.ldx = ldx; a.ldy = 0; a.ldo = 1; a.M = M; a.N = (int)N;
  a.aligned = rows_aligned(x, ldx, nullptr, 0, N, dtype_size(dtype));
  B2K_DISPATCH_FLOAT(dtype, { return rowred_launch<T>(a, false, (cudaStream_t)stream); });
  return B2K_OK;
}

extern "C" int b2k_kl_div(const void* x, int64_t ldx, const void* y, int64_t ldy, void* out,
                          int64_t M, int64_t N, int dtype, void* stream) {
  B2K_REQUIRE(M >= 0 && N >= 1, "b2k_kl_div: need M >= 0 and N >= 1");
  B2K_REQUIRE(M <= 1 || (ldx >= N && ldy >= N), "b2k_kl_div: row stride smaller than N");
  B2K_REQUIRE(N < ((int64_t)1 << 30) && M <= 0x7fffffffLL, "b2k_kl_div: shape too large");
  if (M == 0) return B2K_OK;
  RowRedArgs a;
  a.x = x; a.y = y; a.out = out; a.ldx = ldx; a.ldy = ldy; a.ldo = 1; a.M = M; a.N = (int)N;
  a.aligned = rows_aligned(x, ldx, y, ldy, N, dtype_size(dtype));
  B2K_DISPATCH_FLOAT(dtype, { return rowred_launch<T>(a, true, (cudaStream_t)stream); });
  return B2K_OK;
}

extern "C" int b2k_cumsum(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t M, int64_t N,
                          int dtype, void* stream) {
  B2K_REQUIRE(M >= 0 && N >= 0, "b2k_cumsum: negative shape");
  B2K_REQUIRE(M <= 1 || (ldx >= N && ldy >= N), "b2k_cumsum: row stride smaller than N");
  B2K_REQUIRE(N < ((int64_t)1 << 30) && M <= 0x7fffffffLL, "b2k_cumsum: shape too large");
  if (M == 0 || N == 0) return B2K_OK;
  RowRedArgs a;
  a.x = x; a.y = nullptr; a.out = y; a.ldx = ldx; a.ldy = 0; a.ldo = ldy; a.M = M; a.N = (int)N;
  a.aligned = rows_aligned(x, ldx, y, ldy, N, dtype_size(dtype));
  B2K_DISPATCH_FLOAT(dtype, { return cumsum_launch<T>(a, (cudaStream_t)stream); });
  return B2K_OK;
}
