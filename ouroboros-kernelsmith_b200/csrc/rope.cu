// Rotary embeddings (ouroboros/specs.py:96-102 rotate_half, :228-236
// interleaved pairs, :133-143 and :193-198 RMSNorm + RoPE).
//
// b2k_rope (spec layout, per-row tables): one work item = one 16-byte vector
// of x together with its partner (the vector D/2 away for the half-split
// form, or the E/2 table entries of its pairs for the interleaved form).
// b2k_rope_qk (attention layout): one block per 4 consecutive (batch,
// position) pairs; its threads cover every head of q and k for those
// positions, so a position's table row is read from HBM once and served from
// L1 for all heads; q and k are rotated in the same launch.
// b2k_norm_rope: RMSNorm over the head dim in registers, the normalised row
// staged in shared memory so each element can read its rotation partner.
#include "rowio.cuh"
#include "tma.cuh"

namespace b2k {

constexpr int kRopeThreads = 256;

// ---------------------------------------------------------------- spec layout
struct RopeArgs {
  const void* x;
  const void* cos;
  const void* sin;
  void* y;
  int64_t ldx, ldc, lds, ldy, M;
  int D;
};

// half-split, vector path: item = (row, j), j-th vector of the first half
template <typename T>
__global__ void __launch_bounds__(kRopeThreads) rope_half_vec_kernel(const RopeArgs a,
                                                                     int64_t items, int vph) {
  constexpr int E = Traits<T>::E;
  const int h = a.D / 2;
  for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < items;
       it += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = it / vph;
    const int c = (int)(it - row * vph) * E;
    const T* xr = static_cast<const T*>(a.x) + row * a.ldx;
    const T* cr = static_cast<const T*>(a.cos) + row * a.ldc;
    const T* sr = static_cast<const T*>(a.sin) + row * a.lds;
    float x1[E], x2[E], c1[E], c2[E], s1[E], s2[E], o1[E], o2[E];
    unpack<T>(ld_stream(xr + c), x1);
    unpack<T>(ld_stream(xr + c + h), x2);
    unpack<T>(ld_stream(cr + c), c1);
    unpack<T>(ld_stream(cr + c + h), c2);
    unpack<T>(ld_stream(sr + c), s1);
    unpack<T>(ld_stream(sr + c + h), s2);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      o1[e] = x1[e] * c1[e] - x2[e] * s1[e];
      o2[e] = x2[e] * c2[e] + x1[e] * s2[e];
    }
    T* yr = static_cast<T*>(a.y) + row * a.ldy;
    st_stream(yr + c, pack<T>(o1));
    st_stream(yr + c + h, pack<T>(o2));
  }
}

// interleaved, vector path: item = (row, j), j-th vector of x (E/2 pairs)
template <typename T>
__global__ void __launch_bounds__(kRopeThreads) rope_inter_vec_kernel(const RopeArgs a,
                                                                      int64_t items, int vpr) {
  constexpr int E = Traits<T>::E;
  constexpr int H = E / 2;
  for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < items;
       it += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = it / vpr;
    const int c = (int)(it - row * vpr) * E;
    const T* xr = static_cast<const T*>(a.x) + row * a.ldx;
    const T* cr = static_cast<const T*>(a.cos) + row * a.ldc + c / 2;
    const T* sr = static_cast<const T*>(a.sin) + row * a.lds + c / 2;
    float xv[E], cv[H], sv[H], o[E];
    unpack<T>(ld_stream(xr + c), xv);
    // E/2 table entries = 8 bytes
    const uint2 cw = __ldcs(reinterpret_cast<const uint2*>(cr));
    const uint2 sw = __ldcs(reinterpret_cast<const uint2*>(sr));
    {
      float tmp[2 * H];
      unpack<T>(make_uint4(cw.x, cw.y, sw.x, sw.y), tmp);
#pragma unroll
      for (int i = 0; i < H; ++i) { cv[i] = tmp[i]; sv[i] = tmp[H + i]; }
    }
#pragma unroll
    for (int i = 0; i < H; ++i) {
      o[2 * i] = xv[2 * i] * cv[i] - xv[2 * i + 1] * sv[i];
      o[2 * i + 1] = xv[2 * i + 1] * cv[i] + xv[2 * i] * sv[i];
    }
    st_stream(static_cast<T*>(a.y) + row * a.ldy + c, pack<T>(o));
  }
}

// any shape: item = (row, i) for i < D/2, one rotation pair per item
template <typename T, bool INTER>
__global__ void __launch_bounds__(kRopeThreads) rope_scalar_kernel(const RopeArgs a) {
  const int h = a.D / 2;
  const int64_t items = a.M * h;
  for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < items;
       it += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = it / h;
    const int i = (int)(it - row * h);
    const T* xr = static_cast<const T*>(a.x) + row * a.ldx;
    const T* cr = static_cast<const T*>(a.cos) + row * a.ldc;
    const T* sr = static_cast<const T*>(a.sin) + row * a.lds;
    T* yr = static_cast<T*>(a.y) + row * a.ldy;
    if (INTER) {
      const float x1 = ld1(xr + 2 * i), x2 = ld1(xr + 2 * i + 1);
      const float c = ld1(cr + i), s = ld1(sr + i);
      st1(yr + 2 * i, x1 * c - x2 * s);
      st1(yr + 2 * i + 1, x2 * c + x1 * s);
    } else {
      const float x1 = ld1(xr + i), x2 = ld1(xr + i + h);
      st1(yr + i, x1 * ld1(cr + i) - x2 * ld1(sr + i));
      st1(yr + i + h, x2 * ld1(cr + i + h) + x1 * ld1(sr + i + h));
    }
  }
}

// ---------------------------------------------------------------- attention layout
struct RopeQkArgs {
  const void* q;
  const void* k;
  const void* cos;
  const void* sin;
  void* qo;
  void* ko;
  int64_t B, S, H, Hk;
  int D;
};

// block (per_head, heads_per_pass) over kRopePos consecutive positions:
// threadIdx.x = vector slot within a head, threadIdx.y walks the heads.
// Every thread moves two 16-byte vectors of a head: the half-split form pairs
// element i with i + D/2, the interleaved form takes vectors c and c + D/2
// (both whole pairs) so each thread keeps 32 B of q/k in flight.  (Measured
// on B200: one position per block beats 2 or 4 per block.)
constexpr int kRopePos = 1;

// INTER: 0 half-split (neox), 1 interleaved pairs with the thread's vectors
// c and c + D/2 (8-byte table loads), 2 interleaved pairs with two adjacent
// vectors per thread, whose E table entries are one 16-byte load of cos and
// one of sin (16-byte aligned tables)
template <typename T, int INTER>
__global__ void __launch_bounds__(1024) rope_qk_kernel(const RopeQkArgs a) {
  constexpr int E = Traits<T>::E;
  constexpr int HP = E / 2;
  const int64_t npos = a.B * a.S;
  const int64_t p0 = (int64_t)blockIdx.x * kRopePos;
  const int D = a.D, half = D / 2;
  const int heads = (int)(a.H + a.Hk);
  const int c = threadIdx.x * E;
  // programmatic dependent launch: the next kernel may begin launching; L2
  // prefetch hints for this block's q and k rows (contiguous per position)
  // while the previous kernel drains; then wait for it before reading
  griddep_launch_dependents();
  if (threadIdx.x == 0 && threadIdx.y == 0) {
#pragma unroll
    for (int u = 0; u < kRopePos; ++u) {
      const int64_t p = p0 + u;
      if (p < npos) {
        if (a.H) bulk_prefetch_l2(static_cast<const T*>(a.q) + p * a.H * D,
                                  (uint32_t)(a.H * D * (int64_t)sizeof(T)));
        if (a.Hk) bulk_prefetch_l2(static_cast<const T*>(a.k) + p * a.Hk * D,
                                   (uint32_t)(a.Hk * D * (int64_t)sizeof(T)));
      }
    }
  }
  griddep_wait();
  for (int hh = threadIdx.y; hh < heads; hh += blockDim.y) {
    const bool isq = hh < a.H;
    const int64_t hstride = isq ? a.H * D : a.Hk * D;  // elements per position
    const int64_t hoff = (int64_t)(isq ? hh : hh - (int)a.H) * D;
    const T* src = (isq ? static_cast<const T*>(a.q) : static_cast<const T*>(a.k)) + hoff;
    T* dst = (isq ? static_cast<T*>(a.qo) : static_cast<T*>(a.ko)) + hoff;
    if constexpr (INTER == 2) {
      const int c2 = threadIdx.x * 2 * E;
      uint4 rx[kRopePos][2], rc[kRopePos], rs[kRopePos];
#pragma unroll
      for (int u = 0; u < kRopePos; ++u) {
        const int64_t p = p0 + u;
        if (p < npos) {
          const int64_t s = p % a.S;
          rx[u][0] = ld_stream(src + p * hstride + c2);
          rx[u][1] = ld_stream(src + p * hstride + c2 + E);
          rc[u] = ld_keep(static_cast<const T*>(a.cos) + s * half + c2 / 2);
          rs[u] = ld_keep(static_cast<const T*>(a.sin) + s * half + c2 / 2);
        }
      }
#pragma unroll
      for (int u = 0; u < kRopePos; ++u) {
        const int64_t p = p0 + u;
        if (p < npos) {
          float cs[E], sn[E];
          unpack<T>(rc[u], cs);
          unpack<T>(rs[u], sn);
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            float xv[E], o[E];
            unpack<T>(rx[u][h2], xv);
#pragma unroll
            for (int i = 0; i < HP; ++i) {
              const float cc = cs[h2 * HP + i], ss = sn[h2 * HP + i];
              o[2 * i] = xv[2 * i] * cc - xv[2 * i + 1] * ss;
              o[2 * i + 1] = xv[2 * i + 1] * cc + xv[2 * i] * ss;
            }
            st_stream(dst + p * hstride + c2 + h2 * E, pack<T>(o));
          }
        }
      }
    } else if constexpr (INTER == 0) {
      uint4 r1[kRopePos], r2[kRopePos], rc[kRopePos], rs[kRopePos];
#pragma unroll
      for (int u = 0; u < kRopePos; ++u) {
        const int64_t p = p0 + u;
        if (p < npos) {
          const int64_t s = p % a.S;
          r1[u] = ld_stream(src + p * hstride + c);
          r2[u] = ld_stream(src + p * hstride + c + half);
          rc[u] = ld_keep(static_cast<const T*>(a.cos) + s * half + c);
          rs[u] = ld_keep(static_cast<const T*>(a.sin) + s * half + c);
        }
      }
#pragma unroll
      for (int u = 0; u < kRopePos; ++u) {
        const int64_t p = p0 + u;
        if (p < npos) {
          float x1[E], x2[E], cv[E], sv[E], o1[E], o2[E];
          unpack<T>(r1[u], x1);
          unpack<T>(r2[u], x2);
          unpack<T>(rc[u], cv);
          unpack<T>(rs[u], sv);
#pragma unroll
          for (int e = 0; e < E; ++e) {
            o1[e] = x1[e] * cv[e] - x2[e] * sv[e];
            o2[e] = x2[e] * cv[e] + x1[e] * sv[e];
          }
          st_stream(dst + p * hstride + c, pack<T>(o1));
          st_stream(dst + p * hstride + c + half, pack<T>(o2));
        }
      }
    } else {
      uint4 rx[kRopePos][2];
      uint2 rc[kRopePos][2], rs[kRopePos][2];
#pragma unroll
      for (int u = 0; u < kRopePos; ++u) {
        const int64_t p = p0 + u;
        if (p < npos) {
          const int64_t s = p % a.S;
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            const int cc = c + h2 * half;
            rx[u][h2] = ld_stream(src + p * hstride + cc);
            rc[u][h2] = __ldg(reinterpret_cast<const uint2*>(static_cast<const T*>(a.cos) + s * half + cc / 2));
            rs[u][h2] = __ldg(reinterpret_cast<const uint2*>(static_cast<const T*>(a.sin) + s * half + cc / 2));
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kRopePos; ++u) {
        const int64_t p = p0 + u;
        if (p < npos) {
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            float xv[E], cs[E], o[E];
            unpack<T>(rx[u][h2], xv);
            unpack<T>(make_uint4(rc[u][h2].x, rc[u][h2].y, rs[u][h2].x, rs[u][h2].y), cs);
#pragma unroll
            for (int i = 0; i < HP; ++i) {
              const float cc = cs[i], ss = cs[HP + i];
              o[2 * i] = xv[2 * i] * cc - xv[2 * i + 1] * ss;
              o[2 * i + 1] = xv[2 * i + 1] * cc + xv[2 * i] * ss;
            }
            st_stream(dst + p * hstride + c + h2 * half, pack<T>(o));
          }
        }
      }
    }
  }
}

template <typename T, bool INTER>
__global__ void __launch_bounds__(kRopeThreads) rope_qk_scalar_kernel(const RopeQkArgs a) {
  const int D = a.D, half = D / 2;
  const int64_t heads = a.H + a.Hk;
  const int64_t items = a.B * a.S * heads * half;
  for (int64_t it = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; it < items;
       it += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(it % half);
    const int64_t t = it / half;
    const int64_t hh = t % heads;
    const int64_t p = t / heads;
    const int64_t s = p % a.S;
    const bool isq = hh < a.H;
    const int64_t base = isq ? (p * a.H + hh) * D : (p * a.Hk + (hh - a.H)) * D;
    const T* src = (isq ? static_cast<const T*>(a.q) : static_cast<const T*>(a.k)) + base;
    T* dst = (isq ? static_cast<T*>(a.qo) : static_cast<T*>(a.ko)) + base;
    const float c = ld1(static_cast<const T*>(a.cos) + s * half + i);
    const float sn = ld1(static_cast<const T*>(a.sin) + s * half + i);
    if (INTER) {
      const float x1 = ld1(src + 2 * i), x2 = ld1(src + 2 * i + 1);
      st1(dst + 2 * i, x1 * c - x2 * sn);
      st1(dst + 2 * i + 1, x2 * c + x1 * sn);
    } else {
      const float x1 = ld1(src + i), x2 = ld1(src + i + half);
      st1(dst + i, x1 * c - x2 * sn);
      st1(dst + i + half, x2 * c + x1 * sn);
    }
  }
}

// ---------------------------------------------------------------- norm + rope
struct NormRopeArgs {
  const void* x;
  const void* r;
  const void* w;
  const void* cos;
  const void* sin;
  void* y;
  int64_t ldx, ldr, ldc, lds, ldy, M;
  int D;
  float eps;
  int aligned;
};

template <typename T, int V, bool RESID>
__global__ void __launch_bounds__(256) norm_rope_kernel(const NormRopeArgs a) {
  constexpr int E = Traits<T>::E;
  extern __shared__ float nrow[];  // [R][D]
  __shared__ float red[1024];
  const Group g;
  const int64_t row = (int64_t)blockIdx.x * blockDim.y + g.ty;
  const bool valid = row < a.M;
  const int D = a.D, half = D / 2;
  const int N = valid ? D : 0;
  const T* xr = static_cast<const T*>(a.x) + (valid ? row * a.ldx : 0);
  float hv[V][E];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * g.G + g.tx) * E;
    load_vec<T, true>(hv[v], xr, c, N, a.aligned);
    if (RESID) {
      float t[E];
      load_vec<T, true>(t, static_cast<const T*>(a.r) + (valid ? row * a.ldr : 0), c, N, a.aligned);
#pragma unroll
      for (int e = 0; e < E; ++e) hv[v][e] += t[e];
    }
  }
  float s = 0.0f;
#pragma unroll
  for (int v = 0; v < V; ++v)
#pragma unroll
    for (int e = 0; e < E; ++e) s = fmaf(hv[v][e], hv[v][e], s);
  s = group_sum(s, g, red);
  const float rs = rsqrtf(s / (float)D + a.eps);
  float* nr = nrow + (size_t)g.ty * D;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * g.G + g.tx) * E;
    float wv[E];
    load_vec<T, false>(wv, static_cast<const T*>(a.w), c, N, a.aligned);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      hv[v][e] = hv[v][e] * rs * wv[e];
      if (c + e < N) nr[c + e] = hv[v][e];
    }
  }
  __syncthreads();
  if (!valid) return;
  const T* cr = static_cast<const T*>(a.cos) + row * a.ldc;
  const T* sr = static_cast<const T*>(a.sin) + row * a.lds;
  T* yr = static_cast<T*>(a.y) + row * a.ldy;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * g.G + g.tx) * E;
    float cv[E], sv[E], o[E];
    load_vec<T, true>(cv, cr, c, N, a.aligned);
    load_vec<T, true>(sv, sr, c, N, a.aligned);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int i = c + e;
      if (i < N) {
        const float rot = i < half ? -nr[i + half] : nr[i - half];
        o[e] = hv[v][e] * cv[e] + rot * sv[e];
      } else {
        o[e] = 0.0f;
      }
    }
    store_vec<T>(yr, c, N, a.aligned, o);
  }
}

// Rows whose half (D/2) is P vectors, P a power of two <= 32 (D = 128 at 16
// bits: P = 8), 16-byte aligned: a group of P lanes per row inside one warp;
// lane j holds vector j of BOTH halves of x, w, cos and sin.  RoPE pairs
// element i with i + D/2, so every lane owns both partners of its rotations:
// no shared-memory exchange and no block barrier, the row's sum of squares is
// a log2(P)-step shuffle reduction, and all eight loads of a lane are in
// flight together.
template <typename T, bool RESID>
__global__ void __launch_bounds__(256) norm_rope_half_kernel(const NormRopeArgs a, const int P) {
  constexpr int E = Traits<T>::E;
  const int h = a.D / 2;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t row = gid / P;
  const int c = (int)(gid - row * P) * E;  // offset in the first half
  const bool valid = row < a.M;
  // raw 16-byte vectors: the operands used after the reduction stay packed
  uint4 xv1 = zero4(), xv2 = zero4(), wv1, wv2, cv1, cv2, sv1, sv2;
  if (valid) {
    const T* xr = static_cast<const T*>(a.x) + row * a.ldx;
    const T* cr = static_cast<const T*>(a.cos) + row * a.ldc;
    const T* sr = static_cast<const T*>(a.sin) + row * a.lds;
    const T* w = static_cast<const T*>(a.w);
    xv1 = ld_stream(xr + c);
    xv2 = ld_stream(xr + c + h);
    wv1 = ld_keep(w + c);
    wv2 = ld_keep(w + c + h);
    cv1 = ld_stream(cr + c);
    cv2 = ld_stream(cr + c + h);
    sv1 = ld_stream(sr + c);
    sv2 = ld_stream(sr + c + h);
  }
  float x1[E], x2[E];
  unpack<T>(xv1, x1);
  unpack<T>(xv2, x2);
  if constexpr (RESID) {
    if (valid) {
      const T* rr = static_cast<const T*>(a.r) + row * a.ldr;
      float r1[E], r2[E];
      unpack<T>(ld_stream(rr + c), r1);
      unpack<T>(ld_stream(rr + c + h), r2);
#pragma unroll
      for (int e = 0; e < E; ++e) { x1[e] += r1[e]; x2[e] += r2[e]; }
    }
  }
  float ss = 0.0f;
#pragma unroll
  for (int e = 0; e < E; ++e) ss = fmaf(x2[e], x2[e], fmaf(x1[e], x1[e], ss));
  // the row's P lanes are aligned within the warp: xor offsets < P stay inside
  for (int o = P >> 1; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (!valid) return;
  const float rs = rsqrtf(ss / (float)a.D + a.eps);
  float w1[E], w2[E], c1[E], c2[E], s1[E], s2[E], o1[E], o2[E];
  unpack<T>(wv1, w1);
  unpack<T>(wv2, w2);
  unpack<T>(cv1, c1);
  unpack<T>(cv2, c2);
  unpack<T>(sv1, s1);
  unpack<T>(sv2, s2);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float n1 = x1[e] * rs * w1[e], n2 = x2[e] * rs * w2[e];
    o1[e] = n1 * c1[e] + (-n2) * s1[e];
    o2[e] = n2 * c2[e] + n1 * s2[e];
  }
  T* yr = static_cast<T*>(a.y) + row * a.ldy;
  st_stream(yr + c, pack<T>(o1));
  st_stream(yr + c + h, pack<T>(o2));
}

static unsigned grid_for(int64_t items) {
  const int64_t want = (items + kRopeThreads - 1) / kRopeThreads;
  const int64_t cap = (int64_t)sm_count() * 32;
  return (unsigned)(want < 1 ? 1 : (want < cap ? want : cap));
}

}  // namespace b2k

using namespace b2k;

extern "C" int b2k_rope(const void* x, int64_t ldx, const void* cos, int64_t ldc, const void* sin,
                        int64_t lds, void* y, int64_t ldy, int64_t M, int64_t D, int dtype,
                        int interleaved, void* stream) {
  B2K_REQUIRE(M >= 0 && D >= 0 && D % 2 == 0, "b2k_rope: need M >= 0 and even D");
  const int64_t tw = interleaved ? D / 2 : D;
  B2K_REQUIRE(M <= 1 || (ldx >= D && ldy >= D && ldc >= tw && lds >= tw),
              "b2k_rope: row stride too small");
  B2K_REQUIRE(D < (1 << 30), "b2k_rope: D too large");
  if (M == 0 || D == 0) return B2K_OK;
  RopeArgs a;
  a.x = x; a.cos = cos; a.sin = sin; a.y = y;
  a.ldx = ldx; a.ldc = ldc; a.lds = lds; a.ldy = ldy; a.M = M; a.D = (int)D;
  const int es = dtype_size(dtype);
  const int E = es ? 16 / es : 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool rows16 = aligned16(x) && aligned16(y) && (ldx * es) % 16 == 0 && (ldy * es) % 16 == 0;
  B2K_DISPATCH_FLOAT(dtype, {
    if (!interleaved) {
      const bool vec = rows16 && (D / 2) % E == 0 && aligned16(cos) && aligned16(sin) &&
                       (ldc * es) % 16 == 0 && (lds * es) % 16 == 0;
      if (vec) {
        const int vph = (int)(D / 2 / E);
        const int64_t items = M * vph;
        rope_half_vec_kernel<T><<<grid_for(items), kRopeThreads, 0, st>>>(a, items, vph);
      } else {
        rope_scalar_kernel<T, false><<<grid_for(M * (D / 2)), kRopeThreads, 0, st>>>(a);
      }
    } else {
      const bool vec = rows16 && D % E == 0 && ((uintptr_t)cos % 8 == 0) &&
                       ((uintptr_t)sin % 8 == 0) && (ldc * es) % 8 == 0 && (lds * es) % 8 == 0;
      if (vec) {
        const int vpr = (int)(D / E);
        const int64_t items = M * vpr;
        rope_inter_vec_kernel<T><<<grid_for(items), kRopeThreads, 0, st>>>(a, items, vpr);
      } else {
        rope_scalar_kernel<T, true><<<grid_for(M * (D / 2)), kRopeThreads, 0, st>>>(a);
      }
    }
    return check_launch("b2k_rope");
  });
  return B2K_OK;
}

extern "C" int b2k_rope_qk(const void* q, const void* k, const void* cos, const void* sin,
                           void* q_out, void* k_out, int64_t B, int64_t S, int64_t H, int64_t Hk,
                           int64_t D, int dtype, int interleaved, void* stream) {
  B2K_REQUIRE(B >= 0 && S >= 0 && H >= 0 && Hk >= 0 && D >= 0 && D % 2 == 0,
              "b2k_rope_qk: bad shape");
  B2K_REQUIRE(D < (1 << 20) && H + Hk < (1 << 20), "b2k_rope_qk: shape too large");
  if (B == 0 || S == 0 || D == 0 || H + Hk == 0) return B2K_OK;
  RopeQkArgs a;
  a.q = q; a.k = k; a.cos = cos; a.sin = sin; a.qo = q_out; a.ko = k_out;
  a.B = B; a.S = S; a.H = H; a.Hk = Hk; a.D = (int)D;
  const int es = dtype_size(dtype);
  const int E = es ? 16 / es : 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool base16 = aligned16(q_out) && aligned16(k_out) && (H == 0 || aligned16(q)) &&
                      (Hk == 0 || aligned16(k)) && (D * es) % 16 == 0;
  B2K_DISPATCH_FLOAT(dtype, {
    bool vec;
    int per_head;
    if (!interleaved) {
      vec = base16 && (D / 2) % E == 0 && aligned16(cos) && aligned16(sin) &&
            ((D / 2) * es) % 16 == 0;
      per_head = (int)(D / 2 / E);
    } else {
      vec = base16 && (D / 2) % E == 0 && ((uintptr_t)cos % 8 == 0) &&
            ((uintptr_t)sin % 8 == 0) && ((D / 2) * es) % 8 == 0;
      per_head = (int)(D / 2 / E);
    }
    if (vec) {
      B2K_REQUIRE(per_head <= 1024, "b2k_rope_qk: head dim too large");
      int hpp = 1024 / per_head;
      const int64_t heads = H + Hk;
      if (hpp > heads) hpp = (int)heads;
      const dim3 block(per_head, hpp);
      const int64_t grid = (B * S + kRopePos - 1) / kRopePos;
      B2K_REQUIRE(grid <= 0x7fffffffLL, "b2k_rope_qk: too many positions");
      static const int use_adj = [] {
        const char* s = getenv("B2K_ROPE_ADJ");
        return s ? atoi(s) : 1;
      }();
      const bool adj = use_adj && aligned16(cos) && aligned16(sin) && ((D / 2) * es) % 16 == 0;
      auto kern = interleaved ? (adj ? rope_qk_kernel<T, 2> : rope_qk_kernel<T, 1>)
                              : rope_qk_kernel<T, 0>;
      launch_pdl(kern, dim3((unsigned)grid), block, 0, st, a);
    } else {
      const int64_t items = B * S * (H + Hk) * (D / 2);
      if (interleaved)
        rope_qk_scalar_kernel<T, true><<<grid_for(items), kRopeThreads, 0, st>>>(a);
      else
        rope_qk_scalar_kernel<T, false><<<grid_for(items), kRopeThreads, 0, st>>>(a);
    }
    return check_launch("b2k_rope_qk");
  });
  return B2K_OK;
}

extern "C" int b2k_norm_rope(const void* x, int64_t ldx, const void* r, int64_t ldr, const void* w,
                             const void* cos, int64_t ldc, const void* sin, int64_t lds, void* y,
                             int64_t ldy, int64_t M, int64_t D, int dtype, float eps,
                             void* stream) {
  B2K_REQUIRE(M >= 0 && D >= 0 && D % 2 == 0, "b2k_norm_rope: need M >= 0 and even D");
  B2K_REQUIRE(M <= 1 || (ldx >= D && ldy >= D && ldc >= D && lds >= D && (!r || ldr >= D)),
              "b2k_norm_rope: row stride too small");
  B2K_REQUIRE(D <= 8192, "b2k_norm_rope: head dim above 8192 is not supported");
  B2K_REQUIRE(w != nullptr, "b2k_norm_rope: weight required");
  if (M == 0 || D == 0) return B2K_OK;
  NormRopeArgs a;
  a.x = x; a.r = r; a.w = w; a.cos = cos; a.sin = sin; a.y = y;
  a.ldx = ldx; a.ldr = ldr; a.ldc = ldc; a.lds = lds; a.ldy = ldy; a.M = M; a.D = (int)D;
  a.eps = eps;
  const int es = dtype_size(dtype);
  const int E = es ? 16 / es : 1;
  bool al = D % E == 0 && aligned16(x) && aligned16(y) && aligned16(w) && aligned16(cos) &&
            aligned16(sin) && (ldx * es) % 16 == 0 && (ldy * es) % 16 == 0 &&
            (ldc * es) % 16 == 0 && (lds * es) % 16 == 0;
  if (r) al = al && aligned16(r) && (ldr * es) % 16 == 0;
  a.aligned = al ? 1 : 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  static const int use_half = [] {
    const char* s = getenv("B2K_NORM_ROPE_HALF");
    return s ? atoi(s) : 1;
  }();
  B2K_DISPATCH_FLOAT(dtype, {
    const int P = (int)(D / 2 / Traits<T>::E);
    if (use_half && al && (D / 2) % Traits<T>::E == 0 && P >= 1 && P <= 32 && (P & (P - 1)) == 0) {
      const int64_t threads = M * P;
      const int64_t grid = (threads + 255) / 256;
      if (r) norm_rope_half_kernel<T, true><<<(unsigned)grid, 256, 0, st>>>(a, P);
      else norm_rope_half_kernel<T, false><<<(unsigned)grid, 256, 0, st>>>(a, P);
      return check_launch("b2k_norm_rope(half)");
    }
    RowCfg cfg;
    if (!choose_row_cfg(D, Traits<T>::E, 32, &cfg, 4, 256)) {
      set_error("b2k_norm_rope: head dim %lld does not fit", (long long)D);
      return B2K_EUNSUPPORTED;
    }
    const size_t smem = (size_t)cfg.R * D * sizeof(float);
    const dim3 block(cfg.G, cfg.R);
    const int64_t grid = (M + cfg.R - 1) / cfg.R;
    auto go = [&](auto kern) {
      if (smem > 48 * 1024)
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      kern<<<(unsigned)grid, block, smem, st>>>(a);
    };
    if (r) {
      switch (cfg.V) {
        case 1: go(norm_rope_kernel<T, 1, true>); break;
        case 2: go(norm_rope_kernel<T, 2, true>); break;
        default: go(norm_rope_kernel<T, 4, true>); break;
      }
    } else {
      switch (cfg.V) {
        case 1: go(norm_rope_kernel<T, 1, false>); break;
        case 2: go(norm_rope_kernel<T, 2, false>); break;
        default: go(norm_rope_kernel<T, 4, false>); break;
      }
    }
    return check_launch("b2k_norm_rope");
  });
  return B2K_OK;
}
