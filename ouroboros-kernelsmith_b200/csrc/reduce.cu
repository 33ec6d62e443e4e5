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
#include <stdlib.h>

#include "rowio.cuh"
#include "rowpipe.cuh"

B2K_DEFINE_TIMEOUT_COUNTER()

namespace b2k {

constexpr int kRedMaxThreads = 512;

struct RowRedArgs {
  const void* x;
  const void* y;
  void* out;
  int64_t ldx, ldy, ldo, M;
  int N;
  int aligned;
  int l2pf_rows;  // pipelined path: rows per block hinted into L2 before the wait
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
  {
    const int64_t row0 = (int64_t)blockIdx.x * blockDim.y;
    const int64_t nr = a.M - row0 < (int64_t)blockDim.y ? a.M - row0 : (int64_t)blockDim.y;
    pdl_rows_prologue(a.x, a.ldx * (int64_t)sizeof(T), nullptr,
                      a.ldy * (int64_t)sizeof(T), row0, nr, (uint32_t)a.N * (uint32_t)sizeof(T),
                      a.aligned && a.l2pf_rows > 0);
  }
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
  {
    const int64_t row0 = (int64_t)blockIdx.x * blockDim.y;
    const int64_t nr = a.M - row0 < (int64_t)blockDim.y ? a.M - row0 : (int64_t)blockDim.y;
    pdl_rows_prologue(a.x, a.ldx * (int64_t)sizeof(T), a.y,
                      a.ldy * (int64_t)sizeof(T), row0, nr, (uint32_t)a.N * (uint32_t)sizeof(T),
                      a.aligned && a.l2pf_rows > 0);
  }
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
  {
    const int64_t row0 = (int64_t)blockIdx.x * blockDim.y;
    const int64_t nr = a.M - row0 < (int64_t)blockDim.y ? a.M - row0 : (int64_t)blockDim.y;
    pdl_rows_prologue(a.x, a.ldx * (int64_t)sizeof(T), nullptr, 0, row0, nr,
                      (uint32_t)a.N * (uint32_t)sizeof(T), a.aligned && a.l2pf_rows > 0);
  }
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

// ---------------------------------------------------------------- pipelined path
// Aligned rows whose inputs fit a ring stage (<= 64 KB): persistent blocks
// walk their rows through the bulk-copy row pipeline (rowpipe.cuh), one row
// per block at a time, the next one streaming in while the current one is
// reduced.  The row is read once; every pass of the reference runs over
// registers, and each row costs ONE block-wide merge:
//  * entropy: per thread (m, s, t) = (max, sum e^(x-m), sum x e^(x-m)) over its
//    slice, merged across the block like a logsumexp.  Then lse = M + log S
//    and sum x exp(x - lse) = T * exp(M - lse): the reference's p = exp(x -
//    lse) factored through the same rounded lse, so the cancellation of lse
//    against the weighted sum that decides peaked rows is the reference's,
//    with one exponential per element instead of two.
//  * kl_div: (mx, sx, u) with u = sum e^(x-mx) (x - y), and (my, sy).  With
//    w = exp(Mx - lse_x): sum exp(lx)(lx - ly) = w U - (lse_x - lse_y) Sx w,
//    two exponentials per element instead of three.
//  * cumsum: each thread takes a contiguous run of the row, prefix-sums it in
//    fp32, and the block scans the per-thread totals in fp64; an output is
//    the thread's fp64 offset (rounded once to fp32) plus its local prefix.

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// merge of K floats across the warps of the block when every lane of a warp
// already holds its warp's value (one row per block); every thread gets the
// result; red holds K * 32 floats
template <int K, typename Merge>
__device__ __forceinline__ void xwarp_merge(float (&v)[K], const float (&ident)[K], float* red,
                                            Merge merge) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (nw == 1) return;
  if (lane == 0)
#pragma unroll
    for (int k = 0; k < K; ++k) red[k * 32 + w] = v[k];
  __syncthreads();
  if (w == 0) {
#pragma unroll
    for (int k = 0; k < K; ++k) v[k] = lane < nw ? red[k * 32 + lane] : ident[k];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      if (o >= nw) continue;
      float u[K];
#pragma unroll
      for (int k = 0; k < K; ++k) u[k] = __shfl_xor_sync(0xffffffffu, v[k], o);
      merge(v, u);
    }
    if (lane == 0)
#pragma unroll
      for (int k = 0; k < K; ++k) red[k * 32] = v[k];
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < K; ++k) v[k] = red[k * 32];
  __syncthreads();  // red is reused by the next row
}

template <bool P>
__device__ __forceinline__ float exp_of(float x) {
  if constexpr (P) return expf(x);
  else return ex2_approx(x * kLog2e);
}

// (m, s, t...) logsumexp-style merge: the values after the max are sums
// scaled by e^(x - m)
template <bool P, int K>
__device__ __forceinline__ void lse_merge_k(float (&a)[K], const float (&b)[K]) {
  const float M = fmaxf(a[0], b[0]);
  if (M == -INFINITY) return;
  const float fa = exp_of<P>(a[0] - M), fb = exp_of<P>(b[0] - M);
#pragma unroll
  for (int k = 1; k < K; ++k) a[k] = a[k] * fa + b[k] * fb;
  a[0] = M;
}

// sum of e^(x - m) (and of x e^(x - m) / e^(x - m) (x - y)) over a slice, one
// exponential per element; f32x2 + ex2.approx for 16-bit inputs
template <typename T, int V>
struct RedSlice {
  static constexpr int E = Traits<T>::E;
  static constexpr int H = E / 2;
  static constexpr bool P = std::is_same<T, float>::value;

  __device__ __forceinline__ static float vmax(const float2 (&x)[V][H], const bool (&in)[V]) {
    float m = -INFINITY;
#pragma unroll
    for (int v = 0; v < V; ++v)
      if (in[v])
#pragma unroll
        for (int j = 0; j < H; ++j) m = fmaxf(m, fmaxf(x[v][j].x, x[v][j].y));
    return m;
  }
  // s += e^(x-m); t += x e^(x-m) (y == nullptr) or e^(x-m) (x - y)
  __device__ __forceinline__ static void sums(const float2 (&x)[V][H], const float2 (*y)[H],
                                              const bool (&in)[V], float m, float& s, float& t) {
    s = 0.0f;
    t = 0.0f;
    if (m == -INFINITY) return;
    float2 s2 = f2s(0.0f), t2 = f2s(0.0f);
#pragma unroll
    for (int v = 0; v < V; ++v)
      if (in[v])
#pragma unroll
        for (int j = 0; j < H; ++j) {
          float2 e;
          if constexpr (P) {
            e = f2(expf(x[v][j].x - m), expf(x[v][j].y - m));
          } else {
            // x - m first (exact for the terms near the max), then the scale
            // to base 2: fma(x, log2e, -m log2e) would carry an absolute
            // error of |x| 2^-24 into every exponent, and the x-weighted sums
            // here (x up to +-256 at the spec's stress scale) turn that into
            // 1e-3-level errors of entropy / kl
            const float2 z = mul2(sub2(x[v][j], f2s(m)), f2s(kLog2e));
            e = f2(ex2_approx(z.x), ex2_approx(z.y));
          }
          s2 = add2(s2, e);
          const float2 wgt = y ? sub2(x[v][j], y[v][j]) : x[v][j];
          t2 = fma2(wgt, e, t2);
        }
    s = s2.x + s2.y;
    t = t2.x + t2.y;
  }
};

template <typename T, int V>
__global__ void __launch_bounds__(kRedMaxThreads) entropy_tma_kernel(const RowRedArgs a,
                                                                    const int S_) {
  constexpr int E = Traits<T>::E;
  constexpr int H = E / 2;
  constexpr bool P = std::is_same<T, float>::value;
  using Sl = RedSlice<T, V>;
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ float red[3 * 32];
  __shared__ volatile int abort_flag;
  const int G = blockDim.x, tx = threadIdx.x;
  const int N = a.N;
  if (tx == 0) abort_flag = 0;
  griddep_launch_dependents();
  const void* srcs[1] = {a.x};
  const int64_t lds[1] = {a.ldx};
  RowPipe<1>::prefetch_l2(srcs, lds, (int)sizeof(T), (uint32_t)N * (uint32_t)sizeof(T), a.M,
                          a.l2pf_rows);
  griddep_wait();
  RowPipe<1> pipe;
  pipe.init(dsm, S_, a.M, (uint32_t)N * (uint32_t)sizeof(T), srcs, lds, (int)sizeof(T));
  const float ident[3] = {-INFINITY, 0.0f, 0.0f};
  int64_t k = 0;
  for (; k < pipe.nrows; ++k) {
    bool ok;
    const T* xs = reinterpret_cast<const T*>(pipe.wait_next(ok));
    if (!ok) { abort_flag = 1; atomicAdd(&b2k_tu_timeouts, 1u); }
    float2 xv[V][H];
    bool in[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (v * G + tx) * E;
      in[v] = c < N;
      if (in[v]) unpack2<T>(*reinterpret_cast<const uint4*>(xs + c), xv[v]);
      else
#pragma unroll
        for (int j = 0; j < H; ++j) xv[v][j] = f2s(0.0f);
    }
    // the warp's max first (no exponentials in the shuffle stages), the sums
    // against it, warp sums, then one merge of the warps' triples
    float r[3];
    r[0] = warp_max(Sl::vmax(xv, in));
    Sl::sums(xv, nullptr, in, r[0], r[1], r[2]);
    r[1] = warp_sum(r[1]);
    r[2] = warp_sum(r[2]);
    xwarp_merge<3>(r, ident, red, [](float (&p)[3], const float (&q)[3]) {
      lse_merge_k<P, 3>(p, q);
    });  // barriers inside: every thread has read the stage
    if (abort_flag) break;
    pipe.refill();
    if (tx == 0) {
      const float lse = r[0] + (P ? logf(r[1]) : f_log<false>(r[1]));
      const float q = r[2] * exp_of<P>(r[0] - lse);
      static_cast<T*>(a.out)[pipe.row_of(k) * a.ldo] = from_f<T>(lse - q);
    }
  }
  pipe.drain(k);
}

template <typename T, int V>
__global__ void __launch_bounds__(kRedMaxThreads) kl_tma_kernel(const RowRedArgs a, const int S_) {
  constexpr int E = Traits<T>::E;
  constexpr int H = E / 2;
  constexpr bool P = std::is_same<T, float>::value;
  using Sl = RedSlice<T, V>;
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ float red[5 * 32];
  __shared__ volatile int abort_flag;
  const int G = blockDim.x, tx = threadIdx.x;
  const int N = a.N;
  if (tx == 0) abort_flag = 0;
  griddep_launch_dependents();
  const void* srcs[2] = {a.x, a.y};
  const int64_t lds[2] = {a.ldx, a.ldy};
  RowPipe<2>::prefetch_l2(srcs, lds, (int)sizeof(T), (uint32_t)N * (uint32_t)sizeof(T), a.M,
                          a.l2pf_rows);
  griddep_wait();
  RowPipe<2> pipe;
  pipe.init(dsm, S_, a.M, (uint32_t)N * (uint32_t)sizeof(T), srcs, lds, (int)sizeof(T));
  const float ident[5] = {-INFINITY, 0.0f, 0.0f, -INFINITY, 0.0f};
  auto merge5 = [](float (&p)[5], const float (&q)[5]) {
    float a3[3] = {p[0], p[1], p[2]}, b3[3] = {q[0], q[1], q[2]};
    lse_merge_k<P, 3>(a3, b3);
    float a2[2] = {p[3], p[4]}, b2[2] = {q[3], q[4]};
    lse_merge_k<P, 2>(a2, b2);
    p[0] = a3[0]; p[1] = a3[1]; p[2] = a3[2]; p[3] = a2[0]; p[4] = a2[1];
  };
  int64_t k = 0;
  for (; k < pipe.nrows; ++k) {
    bool ok;
    const T* xs = reinterpret_cast<const T*>(pipe.wait_next(ok));
    if (!ok) { abort_flag = 1; atomicAdd(&b2k_tu_timeouts, 1u); }
    const T* ys = xs + N;
    float2 xv[V][H], yv[V][H];
    bool in[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (v * G + tx) * E;
      in[v] = c < N;
      if (in[v]) {
        unpack2<T>(*reinterpret_cast<const uint4*>(xs + c), xv[v]);
        unpack2<T>(*reinterpret_cast<const uint4*>(ys + c), yv[v]);
      } else {
#pragma unroll
        for (int j = 0; j < H; ++j) { xv[v][j] = f2s(0.0f); yv[v][j] = f2s(0.0f); }
      }
    }
    float r[5];
    r[0] = warp_max(Sl::vmax(xv, in));
    Sl::sums(xv, yv, in, r[0], r[1], r[2]);
    r[3] = warp_max(Sl::vmax(yv, in));
    float unused;
    Sl::sums(yv, nullptr, in, r[3], r[4], unused);
    r[1] = warp_sum(r[1]);
    r[2] = warp_sum(r[2]);
    r[4] = warp_sum(r[4]);
    xwarp_merge<5>(r, ident, red, merge5);
    if (abort_flag) break;
    pipe.refill();
    if (tx == 0) {
      const float lsex = r[0] + (P ? logf(r[1]) : f_log<false>(r[1]));
      const float lsey = r[3] + (P ? logf(r[4]) : f_log<false>(r[4]));
      const float w = exp_of<P>(r[0] - lsex);
      static_cast<T*>(a.out)[pipe.row_of(k) * a.ldo] =
          from_f<T>(w * r[2] - (lsex - lsey) * (r[1] * w));
    }
  }
  pipe.drain(k);
}

// inclusive scan of one double per thread across the block (one row per
// block); sred holds 32 doubles
__device__ __forceinline__ double block_scan_incl(double v, double* sred) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  if (nw > 1) {
    if (lane == 31) sred[w] = v;
    __syncthreads();
    if (w == 0) {
      double t = lane < nw ? sred[lane] : 0.0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double u = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += u;
      }
      if (lane < nw) sred[lane] = t;  // inclusive totals of warps 0..lane
    }
    __syncthreads();
    if (w > 0) v += sred[w - 1];
    __syncthreads();  // sred is reused by the next row
  }
  return v;
}

template <typename T, int V>
__global__ void __launch_bounds__(kRedMaxThreads) cumsum_tma_kernel(const RowRedArgs a,
                                                                   const int S_) {
  constexpr int E = Traits<T>::E;
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ double sred[32];
  __shared__ volatile int abort_flag;
  const int tx = threadIdx.x;
  const int N = a.N;
  if (tx == 0) abort_flag = 0;
  griddep_launch_dependents();
  const void* srcs[1] = {a.x};
  const int64_t lds[1] = {a.ldx};
  RowPipe<1>::prefetch_l2(srcs, lds, (int)sizeof(T), (uint32_t)N * (uint32_t)sizeof(T), a.M,
                          a.l2pf_rows);
  griddep_wait();
  RowPipe<1> pipe;
  pipe.init(dsm, S_, a.M, (uint32_t)N * (uint32_t)sizeof(T), srcs, lds, (int)sizeof(T));
  int64_t k = 0;
  for (; k < pipe.nrows; ++k) {
    bool ok;
    const T* xs = reinterpret_cast<const T*>(pipe.wait_next(ok));
    if (!ok) { abort_flag = 1; atomicAdd(&b2k_tu_timeouts, 1u); }
    // this thread's contiguous run: vectors tx*V .. tx*V + V - 1
    float f[V][E];
    float run = 0.0f;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (tx * V + v) * E;
      if (c < N) unpack<T>(*reinterpret_cast<const uint4*>(xs + c), f[v]);
      else
#pragma unroll
        for (int e = 0; e < E; ++e) f[v][e] = 0.0f;
#pragma unroll
      for (int e = 0; e < E; ++e) { run += f[v][e]; f[v][e] = run; }
    }
    const double incl = block_scan_incl((double)run, sred);  // barriers: the stage was read
    if (abort_flag) break;
    pipe.refill();
    const float base = (float)(incl - (double)run);
    T* yr = static_cast<T*>(a.out) + pipe.row_of(k) * a.ldo;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (tx * V + v) * E;
      if (c < N) {
        float o[E];
#pragma unroll
        for (int e = 0; e < E; ++e) o[e] = base + f[v][e];
        st_stream(yr + c, pack<T>(o));
      }
    }
  }
  pipe.drain(k);
}

// The pipelined kernels, when the rows are aligned and a ring stage (all
// inputs of one row) is at most 64 KB: kind 0 entropy, 1 kl_div, 2 cumsum.
// Threads per row: B2K_RED_VPT 16-byte vectors each (2 or 4; default 4 for
// entropy and cumsum, 2 for kl_div, whose two inputs double the registers)
// while that fits 64..512 threads.
template <typename T>
static bool rowred_try_tma(const RowRedArgs& a, int kind, cudaStream_t st) {
  constexpr int E = Traits<T>::E;
  static const int use_tma = [] {
    const char* s = getenv("B2K_TMA");
    return s ? atoi(s) : 1;
  }();
  static const int vpt_knob = [] {
    const char* s = getenv("B2K_RED_VPT");
    const int v = s ? atoi(s) : 0;
    return v == 2 || v == 4 ? v : 0;
  }();
  if (!use_tma || !a.aligned) return false;
  const int64_t nvec = a.N / E;
  const int nin = kind == 1 ? 2 : 1;
  const int64_t row_bytes = (int64_t)a.N * (int64_t)sizeof(T);
  if (nvec < 64 || nin * row_bytes > (64 << 10)) return false;
  const int vpt = vpt_knob ? vpt_knob : (kind == 1 ? 2 : 4);
  int G = next_pow2((nvec + vpt - 1) / vpt);
  G = G < 64 ? 64 : (G > kRedMaxThreads ? kRedMaxThreads : G);
  const int64_t vneed = (nvec + G - 1) / G;
  if (vneed > 4) return false;
  const bool v2 = vneed <= 2;
  static const int stages_knob = [] {
    const char* s = getenv("B2K_TMA_STAGES");
    const int v = s ? atoi(s) : 0;
    return v >= 2 && v <= 8 ? v : 2;
  }();
  const int want_stages = stages_knob;
  auto go = [&](auto kern, int n_in) -> bool {
    PipeShape ps;
    if (!choose_pipe_shape(kern, G, n_in * row_bytes, 0, want_stages, &ps)) return false;
    const size_t smem = (size_t)ps.S * n_in * (size_t)row_bytes + (size_t)ps.S * sizeof(uint64_t);
    int64_t grid = (int64_t)sm_count() * ps.cps;
    if (grid > a.M) grid = a.M;
    const int64_t per = (a.M + grid - 1) / grid;  // every block walks the same number of rows
    grid = (a.M + per - 1) / per;
    launch_pdl(kern, dim3((unsigned)grid), dim3(G), smem, st, a, ps.S);
    return true;
  };
  if (kind == 0) return go(v2 ? entropy_tma_kernel<T, 2> : entropy_tma_kernel<T, 4>, 1);
  if (kind == 1) return go(v2 ? kl_tma_kernel<T, 2> : kl_tma_kernel<T, 4>, 2);
  return go(v2 ? cumsum_tma_kernel<T, 2> : cumsum_tma_kernel<T, 4>, 1);
}

template <typename T>
static int rowred_launch(const RowRedArgs& a, bool kl, cudaStream_t st) {
  constexpr int E = Traits<T>::E;
  if (rowred_try_tma<T>(a, kl ? 1 : 0, st))
    return check_launch(kl ? "b2k_kl_div(tma)" : "b2k_entropy(tma)");
  RowCfg cfg;
  if (choose_row_cfg(a.N, E, 128, &cfg, 4, kRedMaxThreads)) {
    const dim3 block(cfg.G, cfg.R);
    const int64_t grid = (a.M + cfg.R - 1) / cfg.R;
    auto go = [&](auto kern) { launch_pdl(kern, dim3((unsigned)grid), block, 0, st, a); };
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
  if (rowred_try_tma<T>(a, 2, st)) return check_launch("b2k_cumsum(tma)");
  const int64_t nvec = (a.N + E - 1) / E;
  int G = next_pow2(nvec);
  G = G < 1 ? 1 : (G > 256 ? 256 : G);
  const int R = G >= 256 ? 1 : 256 / G;
  const int64_t grid = (a.M + R - 1) / R;
  launch_pdl(cumsum_kernel<T>, dim3((unsigned)grid), dim3(G, R), 0, st, a);
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
  a.l2pf_rows = l2_prefetch_rows_knob();
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
  a.l2pf_rows = l2_prefetch_rows_knob();
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
  a.l2pf_rows = l2_prefetch_rows_knob();
  B2K_DISPATCH_FLOAT(dtype, { return cumsum_launch<T>(a, (cudaStream_t)stream); });
  return B2K_OK;
}
