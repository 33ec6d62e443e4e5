// Pointwise family: gated units act(gate)*up (swiglu, glu, geglu, reglu),
// pointwise activations with optional bias (gelu, silu, relu2, bias_gelu) and
// per-row int8 dequantisation (ouroboros/specs.py:85-87,126-130,147-168,
// 201-203,223-225).
//
// Fast path: every operand contiguous and 16-byte aligned -> a flat stream of
// 16-byte vectors, U vectors per thread issued back to back (U*16 B of every
// input in flight per thread), evict-first loads and stores, the arithmetic
// as f32x2 pairs.  Bias / per-row scales need the column / row of a vector,
// which costs one 32-bit division per vector (rows never straddle a vector
// because N % E == 0 on this path).  Anything else (odd N, strided rows)
// takes a scalar grid-stride kernel.
#include "tma.cuh"

namespace b2k {

constexpr int kEwThreads = 256;
constexpr int kEwUnroll = 4;

// ---------------------------------------------------------------- gated
// Programmatic dependent launch prologue of the flat vector kernels: let the
// next kernel of the stream begin launching, give L2 a prefetch hint for this
// block's 16-byte vectors of each input (they may load while the previous
// kernel drains), then wait for the previous kernel before reading.
__device__ __forceinline__ void pdl_prologue_flat(int64_t nvec, int U, const void* a,
                                                  const void* b) {
  griddep_launch_dependents();
  if (threadIdx.x == 0) {
    const int64_t v0 = (int64_t)blockIdx.x * kEwThreads * U;
    const int64_t n = nvec - v0 < (int64_t)kEwThreads * U ? nvec - v0 : (int64_t)kEwThreads * U;
    if (n > 0) {
      if (a) bulk_prefetch_l2(static_cast<const unsigned char*>(a) + v0 * 16, (uint32_t)(n * 16));
      if (b) bulk_prefetch_l2(static_cast<const unsigned char*>(b) + v0 * 16, (uint32_t)(n * 16));
    }
  }
  griddep_wait();
}

template <typename T, int ACT, int U>
__global__ void __launch_bounds__(kEwThreads) glu_vec_kernel(const T* __restrict__ g,
                                                             const T* __restrict__ u,
                                                             T* __restrict__ y, int64_t nvec) {
  constexpr int E = Traits<T>::E;
  constexpr bool P = std::is_same<T, float>::value;
  const int64_t base = (int64_t)blockIdx.x * (kEwThreads * U) + threadIdx.x;
  pdl_prologue_flat(nvec, U, g, u);
  uint4 gv[U], uv[U];
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const int64_t i = base + (int64_t)k * kEwThreads;
    if (i < nvec) { gv[k] = ld_stream(g + i * E); uv[k] = ld_stream(u + i * E); }
  }
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const int64_t i = base + (int64_t)k * kEwThreads;
    if (i < nvec) {
      float2 a[E / 2], b[E / 2];
      unpack2<T>(gv[k], a);
      unpack2<T>(uv[k], b);
#pragma unroll
      for (int j = 0; j < E / 2; ++j) a[j] = mul2(act_apply2<ACT, P>(a[j]), b[j]);
      st_stream(y + i * E, pack2<T>(a));
    }
  }
}

template <typename T, int ACT>
__global__ void __launch_bounds__(kEwThreads) glu_scalar_kernel(const T* g, int64_t ldg,
                                                                const T* u, int64_t ldu, T* y,
                                                                int64_t ldy, int64_t M,
                                                                int64_t N) {
  constexpr bool P = std::is_same<T, float>::value;
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / N, c = i - r * N;
    const float a = ld1(g + r * ldg + c), b = ld1(u + r * ldu + c);
    st1(y + r * ldy + c, act_apply<ACT, P>(a) * b);
  }
}

// ---------------------------------------------------------------- pointwise
template <typename T, int ACT, bool BIAS, int U>
__global__ void __launch_bounds__(kEwThreads) act_vec_kernel(const T* __restrict__ x,
                                                             const T* __restrict__ bias,
                                                             T* __restrict__ y, int64_t nvec,
                                                             uint32_t nvr) {
  constexpr int E = Traits<T>::E;
  constexpr bool P = std::is_same<T, float>::value;
  const int64_t base = (int64_t)blockIdx.x * (kEwThreads * U) + threadIdx.x;
  pdl_prologue_flat(nvec, U, x, nullptr);
  uint4 xv[U];
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const int64_t i = base + (int64_t)k * kEwThreads;
    if (i < nvec) xv[k] = ld_stream(x + i * E);
  }
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const int64_t i = base + (int64_t)k * kEwThreads;
    if (i < nvec) {
      float2 a[E / 2];
      unpack2<T>(xv[k], a);
      if constexpr (BIAS) {
        const uint32_t col = (uint32_t)(i % nvr);
        float2 b[E / 2];
        unpack2<T>(ld_keep(bias + (int64_t)col * E), b);
#pragma unroll
        for (int j = 0; j < E / 2; ++j) a[j] = add2(a[j], b[j]);
      }
#pragma unroll
      for (int j = 0; j < E / 2; ++j) a[j] = act_apply2<ACT, P>(a[j]);
      st_stream(y + i * E, pack2<T>(a));
    }
  }
}

template <typename T, int ACT>
__global__ void __launch_bounds__(kEwThreads) act_scalar_kernel(const T* x, int64_t ldx,
                                                                const T* bias, T* y, int64_t ldy,
                                                                int64_t M, int64_t N) {
  constexpr bool P = std::is_same<T, float>::value;
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / N, c = i - r * N;
    float a = ld1(x + r * ldx + c);
    if (bias) a += ld1(bias + c);
    st1(y + r * ldy + c, act_apply<ACT, P>(a));
  }
}

// ---------------------------------------------------------------- dequant
// 16 int8 per input vector -> two 16-byte fp16 vectors.  q*scale is exact in
// fp32 (8-bit x 11-bit significands), so the single rounding to fp16 matches
// (q.float() * scale.float()).to(float16) bit for bit.
template <typename S, int U>
__global__ void __launch_bounds__(kEwThreads) dequant_vec_kernel(const int8_t* __restrict__ q,
                                                                 const S* __restrict__ scale,
                                                                 int64_t lds,
                                                                 __half* __restrict__ y,
                                                                 int64_t nvec, uint32_t nvr) {
  const int64_t base = (int64_t)blockIdx.x * (kEwThreads * U) + threadIdx.x;
  pdl_prologue_flat(nvec, U, q, nullptr);
  uint4 qv[U];
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const int64_t i = base + (int64_t)k * kEwThreads;
    if (i < nvec) qv[k] = ld_stream(q + i * 16);
  }
#pragma unroll
  for (int k = 0; k < U; ++k) {
    const int64_t i = base + (int64_t)k * kEwThreads;
    if (i < nvec) {
      const int64_t row = i / nvr;
      const float s = to_f<S>(scale[row * lds]);
      const uint32_t w[4] = {qv[k].x, qv[k].y, qv[k].z, qv[k].w};
      float f[16];
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int b = 0; b < 4; ++b) f[4 * j + b] = (float)(int8_t)(w[j] >> (8 * b)) * s;
      st_stream(y + i * 16, pack<__half>(f));
      st_stream(y + i * 16 + 8, pack<__half>(f + 8));
    }
  }
}

template <typename S>
__global__ void __launch_bounds__(kEwThreads) dequant_scalar_kernel(const int8_t* q, int64_t ldq,
                                                                    const S* scale, int64_t lds,
                                                                    __half* y, int64_t ldy,
                                                                    int64_t M, int64_t N) {
  const int64_t total = M * N;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / N, c = i - r * N;
    y[r * ldy + c] = __float2half_rn((float)q[r * ldq + c] * to_f<S>(scale[r * lds]));
  }
}

static unsigned scalar_grid(int64_t total) {
  const int64_t want = (total + kEwThreads - 1) / kEwThreads;
  const int64_t cap = (int64_t)sm_count() * 16;
  return (unsigned)(want < cap ? (want < 1 ? 1 : want) : cap);
}

template <typename T, int ACT>
static int glu_launch(const void* g, int64_t ldg, const void* u, int64_t ldu, void* y,
                      int64_t ldy, int64_t M, int64_t N, bool vec, cudaStream_t st) {
  constexpr int E = Traits<T>::E;
  if (vec) {
    const int64_t nvec = M * N / E;
    const int64_t grid = (nvec + kEwThreads * kEwUnroll - 1) / (kEwThreads * kEwUnroll);
    launch_pdl(glu_vec_kernel<T, ACT, kEwUnroll>, dim3((unsigned)grid), dim3(kEwThreads), 0, st,
               (const T*)g, (const T*)u, (T*)y, nvec);
  } else {
    glu_scalar_kernel<T, ACT><<<scalar_grid(M * N), kEwThreads, 0, st>>>(
        (const T*)g, ldg, (const T*)u, ldu, (T*)y, ldy, M, N);
  }
  return check_launch("b2k_glu");
}

template <typename T, int ACT>
static int act_launch(const void* x, int64_t ldx, const void* bias, void* y, int64_t ldy,
                      int64_t M, int64_t N, bool vec, cudaStream_t st) {
  constexpr int E = Traits<T>::E;
  if (vec) {
    const int64_t nvec = M * N / E;
    const int64_t grid = (nvec + kEwThreads * kEwUnroll - 1) / (kEwThreads * kEwUnroll);
    if (bias)
      launch_pdl(act_vec_kernel<T, ACT, true, kEwUnroll>, dim3((unsigned)grid), dim3(kEwThreads),
                 0, st, (const T*)x, (const T*)bias, (T*)y, nvec, (uint32_t)(N / E));
    else
      launch_pdl(act_vec_kernel<T, ACT, false, kEwUnroll>, dim3((unsigned)grid),
                 dim3(kEwThreads), 0, st, (const T*)x, (const T*)nullptr, (T*)y, nvec,
                 (uint32_t)(N / E));
  } else {
    act_scalar_kernel<T, ACT><<<scalar_grid(M * N), kEwThreads, 0, st>>>(
        (const T*)x, ldx, (const T*)bias, (T*)y, ldy, M, N);
  }
  return check_launch("b2k_act");
}

}  // namespace b2k

using namespace b2k;

extern "C" int b2k_glu(const void* gate, int64_t ldg, const void* up, int64_t ldu, void* y,
                       int64_t ldy, int64_t M, int64_t N, int dtype, int act, void* stream) {
  B2K_REQUIRE(M >= 0 && N >= 0, "b2k_glu: negative shape");
  B2K_REQUIRE(M <= 1 || (ldg >= N && ldu >= N && ldy >= N), "b2k_glu: row stride smaller than N");
  B2K_REQUIRE(act == B2K_ACT_SILU || act == B2K_ACT_SIGMOID || act == B2K_ACT_GELU ||
                  act == B2K_ACT_RELU,
              "b2k_glu: act must be SILU, SIGMOID, GELU or RELU (got %d)", act);
  if (M == 0 || N == 0) return B2K_OK;
  const int es = dtype_size(dtype);
  B2K_REQUIRE(es == 2 || es == 4, "b2k_glu: bad dtype %d", dtype);
  const int E = 16 / es;
  // contiguous (or single-row) operands of a whole number of vectors
  const bool contig = (M == 1 || (ldg == N && ldu == N && ldy == N));
  const bool vec = contig && ((M * N) % E == 0) && aligned16(gate) && aligned16(up) &&
                   aligned16(y) && (M * N / E) < ((int64_t)1 << 40);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  B2K_DISPATCH_FLOAT(dtype, {
    switch (act) {
      case B2K_ACT_SILU: return glu_launch<T, B2K_ACT_SILU>(gate, ldg, up, ldu, y, ldy, M, N, vec, st);
      case B2K_ACT_SIGMOID: return glu_launch<T, B2K_ACT_SIGMOID>(gate, ldg, up, ldu, y, ldy, M, N, vec, st);
      case B2K_ACT_GELU: return glu_launch<T, B2K_ACT_GELU>(gate, ldg, up, ldu, y, ldy, M, N, vec, st);
      default: return glu_launch<T, B2K_ACT_RELU>(gate, ldg, up, ldu, y, ldy, M, N, vec, st);
    }
  });
  return B2K_OK;
}

extern "C" int b2k_act(const void* x, int64_t ldx, const void* bias, void* y, int64_t ldy,
                       int64_t M, int64_t N, int dtype, int act, void* stream) {
  B2K_REQUIRE(M >= 0 && N >= 0, "b2k_act: negative shape");
  B2K_REQUIRE(M <= 1 || (ldx >= N && ldy >= N), "b2k_act: row stride smaller than N");
  B2K_REQUIRE(act == B2K_ACT_GELU || act == B2K_ACT_SILU || act == B2K_ACT_RELU2,
              "b2k_act: act must be GELU, SILU or RELU2 (got %d)", act);
  if (M == 0 || N == 0) return B2K_OK;
  const int es = dtype_size(dtype);
  B2K_REQUIRE(es == 2 || es == 4, "b2k_act: bad dtype %d", dtype);
  const int E = 16 / es;
  const bool contig = (M == 1 || (ldx == N && ldy == N));
  bool vec = contig && aligned16(x) && aligned16(y);
  if (bias) vec = vec && (N % E == 0) && aligned16(bias) && (N / E) < ((int64_t)1 << 32);
  else vec = vec && ((M * N) % E == 0);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  B2K_DISPATCH_FLOAT(dtype, {
    switch (act) {
      case B2K_ACT_GELU: return act_launch<T, B2K_ACT_GELU>(x, ldx, bias, y, ldy, M, N, vec, st);
      case B2K_ACT_SILU: return act_launch<T, B2K_ACT_SILU>(x, ldx, bias, y, ldy, M, N, vec, st);
      default: return act_launch<T, B2K_ACT_RELU2>(x, ldx, bias, y, ldy, M, N, vec, st);
    }
  });
  return B2K_OK;
}

extern "C" int b2k_dequant_i8(const void* q, int64_t ldq, const void* scale, int64_t lds,
                              int scale_dtype, void* y, int64_t ldy, int64_t M, int64_t N,
                              void* stream) {
  B2K_REQUIRE(M >= 0 && N >= 0, "b2k_dequant_i8: negative shape");
  B2K_REQUIRE(M <= 1 || (ldq >= N && ldy >= N), "b2k_dequant_i8: row stride smaller than N");
  if (M == 0 || N == 0) return B2K_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool contig = (M == 1 || (ldq == N && ldy == N));
  const bool vec = contig && (N % 16 == 0) && aligned16(q) && aligned16(y) &&
                   (N / 16) < ((int64_t)1 << 32);
  auto go = [&](auto tag) -> int {
    using S = decltype(tag);
    if (vec) {
      const int64_t nvec = M * N / 16;
      const int64_t grid = (nvec + kEwThreads * kEwUnroll - 1) / (kEwThreads * kEwUnroll);
      launch_pdl(dequant_vec_kernel<S, kEwUnroll>, dim3((unsigned)grid), dim3(kEwThreads), 0, st,
                 (const int8_t*)q, (const S*)scale, lds, (__half*)y, nvec, (uint32_t)(N / 16));
    } else {
      dequant_scalar_kernel<S><<<scalar_grid(M * N), kEwThreads, 0, st>>>(
          (const int8_t*)q, ldq, (const S*)scale, lds, (__half*)y, ldy, M, N);
    }
    return check_launch("b2k_dequant_i8");
  };
  switch (scale_dtype) {
    case B2K_F32: return go(float{});
    case B2K_F16: return go(__half{});
    case B2K_BF16: return go(__nv_bfloat16{});
    default: set_error("b2k_dequant_i8: bad scale dtype %d", scale_dtype); return B2K_EINVAL;
  }
}
