// b2k_norm: argument checks and dispatch to the norm-family instances
// (kernels in norm_impl.cuh, instances in norm_inst_*.cu).
#include <stdlib.h>

#include "norm_impl.cuh"

namespace b2k {

// Threads-per-row target of the register path; B2K_NORM_TPR overrides it
// (power of two, 1..512) for launch-shape sweeps.
static int norm_g_target() {
  static const int v = [] {
    const char* s = getenv("B2K_NORM_TPR");
    const int t = s ? atoi(s) : 0;
    return (t >= 1 && t <= kNormMaxThreads && (t & (t - 1)) == 0) ? t : 128;
  }();
  return v;
}

template <typename T>
static int norm_dispatch(const NormArgs& a, int act, cudaStream_t st) {
#define B2K_CASE(k) case k: return norm_launch<T, k>(a, st);
  switch (act) {
    B2K_CASE(0) B2K_CASE(1) B2K_CASE(2) B2K_CASE(3) B2K_CASE(4) B2K_CASE(5) B2K_CASE(6)
    B2K_CASE(7) B2K_CASE(8) B2K_CASE(9) B2K_CASE(10) B2K_CASE(11) B2K_CASE(12) B2K_CASE(13)
    B2K_CASE(14) B2K_CASE(15) B2K_CASE(16) B2K_CASE(17) B2K_CASE(18) B2K_CASE(19)
    default: set_error("b2k_norm: bad act %d", act); return B2K_EINVAL;
  }
#undef B2K_CASE
}

}  // namespace b2k

using namespace b2k;

extern "C" int b2k_norm(const void* x, int64_t ldx, const void* r, int64_t ldr, const void* w,
                        const void* b, void* y, int64_t ldy, void* h, int64_t ldh, int64_t M,
                        int64_t N, int dtype, int norm_kind, int affine, int act, float eps,
                        void* stream) {
  B2K_REQUIRE(M >= 0 && N >= 0, "b2k_norm: negative shape M=%lld N=%lld", (long long)M,
              (long long)N);
  B2K_REQUIRE(norm_kind >= B2K_NORM_RMS && norm_kind <= B2K_NORM_LN, "b2k_norm: bad norm_kind %d",
              norm_kind);
  B2K_REQUIRE(affine >= B2K_AFF_NONE && affine <= B2K_AFF_WB, "b2k_norm: bad affine %d", affine);
  B2K_REQUIRE(act >= 0 && act < B2K_ACT_COUNT, "b2k_norm: bad act %d", act);
  B2K_REQUIRE((affine == B2K_AFF_WB) == (norm_kind == B2K_NORM_LN),
              "b2k_norm: affine WB goes with LayerNorm only");
  B2K_REQUIRE(affine == B2K_AFF_NONE || w != nullptr, "b2k_norm: weight required");
  B2K_REQUIRE(affine != B2K_AFF_WB || b != nullptr, "b2k_norm: bias required");
  B2K_REQUIRE(M == 0 || N == 0 || (x != nullptr && y != nullptr), "b2k_norm: null x or y");
  B2K_REQUIRE(M <= 1 || (ldx >= N && ldy >= N && (!r || ldr >= N) && (!h || ldh >= N)),
              "b2k_norm: row stride smaller than N");
  B2K_REQUIRE(N <= ((int64_t)1 << 30), "b2k_norm: N too large");
  B2K_REQUIRE(M <= 0x7fffffffLL, "b2k_norm: M too large");
  if (M == 0 || N == 0) return B2K_OK;

  NormArgs a;
  a.x = x; a.r = r; a.w = w; a.b = b; a.y = y; a.h = h;
  a.ldx = ldx; a.ldr = ldr; a.ldy = ldy; a.ldh = ldh;
  a.M = M; a.N = N; a.eps = eps;
  a.norm = norm_kind; a.affine = affine;
  a.g_target = norm_g_target();
  const int es = dtype_size(dtype);
  const int E = es ? 16 / es : 1;
  bool al = (N % E == 0) && aligned16(x) && aligned16(y) && ((ldx * es) % 16 == 0) &&
            ((ldy * es) % 16 == 0);
  if (r) al = al && aligned16(r) && ((ldr * es) % 16 == 0);
  if (h) al = al && aligned16(h) && ((ldh * es) % 16 == 0);
  if (affine != B2K_AFF_NONE) al = al && aligned16(w);
  if (affine == B2K_AFF_WB) al = al && aligned16(b);
  a.aligned = al ? 1 : 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  B2K_DISPATCH_FLOAT(dtype, { return norm_dispatch<T>(a, act, st); });
  return B2K_OK;
}
