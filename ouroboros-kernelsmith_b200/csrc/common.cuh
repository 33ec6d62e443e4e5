// Shared device helpers for the b200k kernels: element traits, 16-byte vector
// load/store with cache hints, group reductions and the epilogue functions of
// the chain grammar (ouroboros/chains.py:13-53).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <math.h>
#include <type_traits>

#include "b200k.h"

namespace b2k {

constexpr float kLog2e = 1.4426950408889634f;   // log2(e)
constexpr float kLn2 = 0.6931471805599453f;     // ln(2)
constexpr float kGeluC = 0.7978845608028654f;   // sqrt(2/pi), chains.py:10

// ---------------------------------------------------------------------------
// element traits: E = elements per 16-byte vector
template <typename T> struct Traits;
template <> struct Traits<float> { static constexpr int E = 4; };
template <> struct Traits<__half> { static constexpr int E = 8; };
template <> struct Traits<__nv_bfloat16> { static constexpr int E = 8; };

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// value after a round trip through T (models a `.to(dtype)` in the reference)
template <typename T> __device__ __forceinline__ float round_to(float v) {
  return to_f<T>(from_f<T>(v));
}

// 16-byte vector -> E floats
template <typename T> __device__ __forceinline__ void unpack(const uint4& v, float* f);
template <> __device__ __forceinline__ void unpack<float>(const uint4& v, float* f) {
  f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
  f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
}
template <> __device__ __forceinline__ void unpack<__nv_bfloat16>(const uint4& v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
template <> __device__ __forceinline__ void unpack<__half>(const uint4& v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h2 = *reinterpret_cast<const __half2*>(&w[i]);
    float2 t = __half22float2(h2);
    f[2 * i] = t.x; f[2 * i + 1] = t.y;
  }
}

// E floats -> 16-byte vector (round to nearest even)
template <typename T> __device__ __forceinline__ uint4 pack(const float* f);
template <> __device__ __forceinline__ uint4 pack<float>(const float* f) {
  return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                    __float_as_uint(f[3]));
}
template <> __device__ __forceinline__ uint4 pack<__nv_bfloat16>(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 p = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&p);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
template <> __device__ __forceinline__ uint4 pack<__half>(const float* f) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 p = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&p);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// ---------------------------------------------------------------------------
// global memory access.  Streaming operands (read or written once) use the
// evict-first (.cs) forms so they do not push reused data (weights, tables,
// rows re-read in a later pass) out of L2.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  return __ldcs(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ uint4 ld_keep(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void st_stream(void* p, const uint4& v) {
  __stcs(reinterpret_cast<uint4*>(p), v);
}
__device__ __forceinline__ uint4 zero4() { return make_uint4(0u, 0u, 0u, 0u); }

template <typename T> __device__ __forceinline__ float ld1(const T* p) { return to_f<T>(p[0]); }
template <typename T> __device__ __forceinline__ void st1(T* p, float v) { p[0] = from_f<T>(v); }

// ---------------------------------------------------------------------------
// PTX approximations (hardware MUFU ops), used only where the output is a
// 16-bit float.  ex2/rcp/lg2.approx have relative errors near 2^-22.
// tanh.approx.f32 on B200 (sm_100a) was measured against tanhf on 2^24
// points of [-40, 40]: max absolute error 7.8e-6, max relative 9.9e-6, and
// exactly +-1 for |x| > 9.02 — far below half an fp16 ulp, and exact in the
// saturated tails where tanh-based sigmoid / GELU would otherwise cancel.
__device__ __forceinline__ float ex2_approx(float x) {
  float y; asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x)); return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y; asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x)); return y;
}
__device__ __forceinline__ float lg2_approx(float x) {
  float y; asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x)); return y;
}
__device__ __forceinline__ float tanh_approx(float x) {
  float y; asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x)); return y;
}

// exp / log / sigmoid / tanh in two precisions.  P (precise) = fp32 output,
// library functions; !P = 16-bit output, MUFU forms.
template <bool P> __device__ __forceinline__ float f_exp(float x) {
  if constexpr (P) return expf(x); else return ex2_approx(x * kLog2e);
}
template <bool P> __device__ __forceinline__ float f_log(float x) {
  if constexpr (P) return logf(x); else return lg2_approx(x) * kLn2;
}
template <bool P> __device__ __forceinline__ float f_rcp(float x) {
  if constexpr (P) return 1.0f / x; else return rcp_approx(x);
}
// sigmoid(x) = 0.5 + 0.5 tanh(x/2): one MUFU op instead of ex2 + rcp in the
// 16-bit form (absolute error <= 3.9e-6, exact 0 / 1 in the tails)
template <bool P> __device__ __forceinline__ float f_sigmoid(float x) {
  if constexpr (P) return 1.0f / (1.0f + expf(-x));
  else return fmaf(0.5f, tanh_approx(0.5f * x), 0.5f);
}
// tanh feeding an exponential (softcap): its absolute error is what matters;
// tanh.approx's 7.8e-6 times the cap of 30 moves exp() by ~2.3e-4 relative.
template <bool P> __device__ __forceinline__ float f_tanh_abs(float x) {
  if constexpr (P) return tanhf(x);
  else return tanh_approx(x);
}
template <bool P> __device__ __forceinline__ float f_tanh(float x) {
  if constexpr (P) return tanhf(x); else return tanh_approx(x);
}

// ---------------------------------------------------------------------------
// Epilogues, chains.py:13-53.  The gelu/tanh identity 0.5*(1+tanh(u)) =
// sigmoid(2u) is used in the MUFU form (no cancellation for large negative
// inputs); the precise form is the reference formula itself.
template <int ACT, bool P> __device__ __forceinline__ float act_apply(float t) {
  if constexpr (ACT == B2K_ACT_NONE) {
    return t;
  } else if constexpr (ACT == B2K_ACT_GELU) {
    const float u = kGeluC * (t + 0.044715f * t * t * t);
    if constexpr (P) return 0.5f * t * (1.0f + tanhf(u));
    else { const float ht = 0.5f * t; return fmaf(ht, tanh_approx(u), ht); }
  } else if constexpr (ACT == B2K_ACT_SILU) {
    return t * f_sigmoid<P>(t);
  } else if constexpr (ACT == B2K_ACT_RELU2) {
    const float r = fmaxf(t, 0.0f); return r * r;
  } else if constexpr (ACT == B2K_ACT_TANH) {
    return f_tanh<P>(t);
  } else if constexpr (ACT == B2K_ACT_SIGMOID) {
    return f_sigmoid<P>(t);
  } else if constexpr (ACT == B2K_ACT_RELU) {
    return fmaxf(t, 0.0f);
  } else if constexpr (ACT == B2K_ACT_SQUARE) {
    return t * t;
  } else if constexpr (ACT == B2K_ACT_ABS) {
    return fabsf(t);
  } else if constexpr (ACT == B2K_ACT_SOFTSIGN) {
    if constexpr (P) return t / (1.0f + fabsf(t));
    else return t * rcp_approx(1.0f + fabsf(t));
  } else if constexpr (ACT == B2K_ACT_HARDSIGMOID) {
    const float c = fminf(fmaxf(t + 3.0f, 0.0f), 6.0f);
    if constexpr (P) return c / 6.0f; else return c * (1.0f / 6.0f);
  } else if constexpr (ACT == B2K_ACT_HARDSWISH) {
    const float c = t * fminf(fmaxf(t + 3.0f, 0.0f), 6.0f);
    if constexpr (P) return c / 6.0f; else return c * (1.0f / 6.0f);
  } else if constexpr (ACT == B2K_ACT_LEAKY_RELU) {
    return t > 0.0f ? t : 0.01f * t;
  } else if constexpr (ACT == B2K_ACT_RELU6) {
    return fminf(fmaxf(t, 0.0f), 6.0f);
  } else if constexpr (ACT == B2K_ACT_HARDTANH) {
    return fminf(fmaxf(t, -1.0f), 1.0f);
  } else if constexpr (ACT == B2K_ACT_ELU) {
    return t > 0.0f ? t : f_exp<P>(fminf(t, 0.0f)) - 1.0f;
  } else if constexpr (ACT == B2K_ACT_SELU) {
    return 1.0507009873554805f *
           (t > 0.0f ? t : 1.6732632423543772f * (f_exp<P>(fminf(t, 0.0f)) - 1.0f));
  } else if constexpr (ACT == B2K_ACT_SOFTPLUS) {
    return t > 20.0f ? t : f_log<P>(1.0f + f_exp<P>(fminf(t, 20.0f)));
  } else if constexpr (ACT == B2K_ACT_MISH) {
    const float sp = t > 20.0f ? t : f_log<P>(1.0f + f_exp<P>(fminf(t, 20.0f)));
    return t * f_tanh<P>(sp);
  } else if constexpr (ACT == B2K_ACT_GELU_ERF) {
    return 0.5f * t * (1.0f + erff(t * 0.7071067811865476f));
  } else {
    static_assert(ACT >= 0 && ACT < B2K_ACT_COUNT, "unknown epilogue");
    return t;
  }
}

// Expands F(std::integral_constant<int, ACT>) for a runtime `act` value.
template <typename F> __device__ __forceinline__ void dispatch_act(int act, F&& f) {
#define B2K_ACT_CASE(k) case k: f(std::integral_constant<int, k>{}); break;
  switch (act) {
    B2K_ACT_CASE(0) B2K_ACT_CASE(1) B2K_ACT_CASE(2) B2K_ACT_CASE(3) B2K_ACT_CASE(4)
    B2K_ACT_CASE(5) B2K_ACT_CASE(6) B2K_ACT_CASE(7) B2K_ACT_CASE(8) B2K_ACT_CASE(9)
    B2K_ACT_CASE(10) B2K_ACT_CASE(11) B2K_ACT_CASE(12) B2K_ACT_CASE(13) B2K_ACT_CASE(14)
    B2K_ACT_CASE(15) B2K_ACT_CASE(16) B2K_ACT_CASE(17) B2K_ACT_CASE(18) B2K_ACT_CASE(19)
    default: break;
  }
#undef B2K_ACT_CASE
}

// ---------------------------------------------------------------------------
// Group reductions.  A thread block is (G, R): G threads (threadIdx.x) share
// one row, R rows (threadIdx.y) per block, G*R a multiple of 32, G a power of
// two.  Every thread of the block must call these (they may __syncthreads).
// `red` is shared scratch of 1024 floats.  The result is returned to
// every thread of the group, summed in a fixed order (deterministic).
struct Group {
  int G, tx, ty;
  __device__ __forceinline__ Group() : G(blockDim.x), tx(threadIdx.x), ty(threadIdx.y) {}
};

template <typename Op>
__device__ __forceinline__ float group_reduce(float v, const Group& g, float* red, Op op,
                                             float identity) {
  const int width = g.G < 32 ? g.G : 32;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    if (o < width) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (g.G > 32) {
    // warp partials -> the group's first warp combines them with shuffles
    // (log depth) -> broadcast through shared memory
    const int nw = g.G >> 5, w = g.tx >> 5, lane = g.tx & 31;
    float* slot = red + g.ty * 32;
    if (lane == 0) slot[w] = v;
    __syncthreads();
    if (w == 0) {
      float t = lane < nw ? slot[lane] : identity;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
        if (o < nw) t = op(t, __shfl_xor_sync(0xffffffffu, t, o));
      if (lane == 0) slot[0] = t;
    }
    __syncthreads();
    v = slot[0];
    __syncthreads();
  }
  return v;
}

struct OpSum { __device__ __forceinline__ float operator()(float a, float b) const { return a + b; } };
struct OpMax { __device__ __forceinline__ float operator()(float a, float b) const { return fmaxf(a, b); } };

__device__ __forceinline__ float group_sum(float v, const Group& g, float* red) {
  return group_reduce(v, g, red, OpSum{}, 0.0f);
}
__device__ __forceinline__ float group_max(float v, const Group& g, float* red) {
  return group_reduce(v, g, red, OpMax{}, -INFINITY);
}

// (max, sum-of-exp) pair merge for online logsumexp.  s is relative to m.
__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  const float M = fmaxf(m, m2);
  if (M == -INFINITY) return;  // both empty
  s = s * ex2_approx((m - M) * kLog2e) + s2 * ex2_approx((m2 - M) * kLog2e);
  m = M;
}

// cross-warp stage of the group (max, sum-exp) merge (G > 32): warp 0 merges
// the warps' pairs, every thread gets the result
__device__ __forceinline__ void group_lse_xwarp(float& m, float& s, const Group& g, float* red) {
  const int nw = g.G >> 5, w = g.tx >> 5, lane = g.tx & 31;
  float* rm = red + g.ty * 32;        // [R <= 16][32]
  float* rs = red + 512 + g.ty * 32;  // (red must hold 1024 floats)
  if (lane == 0) { rm[w] = m; rs[w] = s; }
  __syncthreads();
  if (w == 0) {
    float M = lane < nw ? rm[lane] : -INFINITY;
    float S = lane < nw ? rs[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
      if (o < nw) {
        const float m2 = __shfl_xor_sync(0xffffffffu, M, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, S, o);
        lse_merge(M, S, m2, s2);
      }
    if (lane == 0) { rm[0] = M; rs[0] = S; }
  }
  __syncthreads();
  m = rm[0];
  s = rs[0];
  __syncthreads();
}

// Within a warp (or a G < 32 group): the maximum by shuffles, each thread's
// sum rescaled to it once, then a plain sum; one exponential per thread
// instead of two per level of a pairwise merge.  Across warps: group_lse_xwarp.
__device__ __forceinline__ void group_lse(float& m, float& s, const Group& g, float* red) {
  const int width = g.G < 32 ? g.G : 32;
  float M = m;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    if (o < width) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
  if (M != -INFINITY) s *= ex2_approx((m - M) * kLog2e);  // m = -inf: s is 0 and stays 0
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    if (o < width) s += __shfl_xor_sync(0xffffffffu, s, o);
  m = M;
  if (g.G > 32) group_lse_xwarp(m, s, g, red);
}

// maximum over the warp, in every lane
__device__ __forceinline__ float warp_allmax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// group_lse for G >= 32 when m is already the same in every lane of a warp
// (the warp's maximum, taken before the exponentials): the warp stage is a
// plain sum of s with no exponentials (group_lse's spends two per level),
// the warps' pairs are merged as in group_lse
__device__ __forceinline__ void group_lse_wmax(float& m, float& s, const Group& g, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (g.G > 32) group_lse_xwarp(m, s, g, red);
}

// ---------------------------------------------------------------------------
// host side helpers (defined in api.cu)
void set_error(const char* fmt, ...);
int sm_count();
int check_launch(const char* what);
bool aligned16(const void* p);
int dtype_size(int dtype);

}  // namespace b2k

#define B2K_REQUIRE(cond, ...)                 \
  do {                                         \
    if (!(cond)) {                             \
      ::b2k::set_error(__VA_ARGS__);           \
      return B2K_EINVAL;                       \
    }                                          \
  } while (0)

// Runs BODY with `T` bound to the element type of a floating dtype.
#define B2K_DISPATCH_FLOAT(dtype, ...)                                          \
  switch (dtype) {                                                              \
    case B2K_F32: { using T = float; __VA_ARGS__; break; }                      \
    case B2K_F16: { using T = __half; __VA_ARGS__; break; }                     \
    case B2K_BF16: { using T = __nv_bfloat16; __VA_ARGS__; break; }             \
    default: ::b2k::set_error("unsupported dtype %d", (int)(dtype)); return B2K_EINVAL; \
  }

// ---------------------------------------------------------------------------
// Packed fp32 pairs (sm_100 f32x2 FMA/ADD/MUL: one instruction per pair).
namespace b2k {

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 f2s(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
  return __fadd2_rn(a, make_float2(-b.x, -b.y));
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// E floats <-> E/2 pairs views of a 16-byte vector
template <typename T> __device__ __forceinline__ void unpack2(const uint4& v, float2* f) {
  unpack<T>(v, reinterpret_cast<float*>(f));
}
template <typename T> __device__ __forceinline__ uint4 pack2(const float2* f) {
  return pack<T>(reinterpret_cast<const float*>(f));
}

// value of a pair after a round trip through T (one packed conversion)
template <typename T> __device__ __forceinline__ float2 round2(float2 v) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return __bfloat1622float2(__floats2bfloat162_rn(v.x, v.y));
  } else if constexpr (std::is_same<T, __half>::value) {
    return __half22float2(__floats2half2_rn(v.x, v.y));
  } else {
    return v;
  }
}

// Pairwise epilogue.  Transcendental-free epilogues and the precise (fp32
// output) forms apply the scalar act_apply per lane; the MUFU forms of the
// sigmoid-based epilogues do their polynomial/affine parts as f32x2 ops.
template <int ACT, bool P> __device__ __forceinline__ float2 act_apply2(float2 t) {
  if constexpr (!P && ACT == B2K_ACT_GELU) {
    // 0.5 x (1 + tanh(u)), u = sqrt(2/pi) (x + 0.044715 x^3)
    constexpr float k0 = kGeluC;
    constexpr float k1 = kGeluC * 0.044715f;
    const float2 u = mul2(t, fma2(mul2(t, t), f2s(k1), f2s(k0)));
    const float2 ht = mul2(t, f2s(0.5f));
    return fma2(ht, f2(tanh_approx(u.x), tanh_approx(u.y)), ht);
  } else if constexpr (!P && (ACT == B2K_ACT_SILU || ACT == B2K_ACT_SIGMOID)) {
    const float2 z = mul2(t, f2s(0.5f));
    const float2 s = fma2(f2(tanh_approx(z.x), tanh_approx(z.y)), f2s(0.5f), f2s(0.5f));
    return ACT == B2K_ACT_SILU ? mul2(t, s) : s;
  } else {
    return f2(act_apply<ACT, P>(t.x), act_apply<ACT, P>(t.y));
  }
}

}  // namespace b2k
