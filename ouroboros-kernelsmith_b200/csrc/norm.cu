// b2k_norm: argument checks and dispatch to the norm-family instances
// (kernels in norm_impl.cuh, instances in norm_inst_*.cu).
#include <stdlib.h>

#include "norm_impl.cuh"

namespace b2k {

static int env_int(const char* name, int dflt) {
  const char* s = getenv(name);
  return s ? atoi(s) : dflt;
}

// Launch-shape knobs, read once: B2K_NORM_TPR (threads-per-row target of the
// register path, power of two <= 512), B2K_TMA (0 disables the bulk-copy
// path), B2K_TMA_THREADS, B2K_TMA_CPS (blocks per SM), B2K_TMA_STAGES,
// B2K_L2PF_ROWS (rows per block of the bulk-copy path hinted into L2 before
// the kernel waits for its predecessor; 0 = off), B2K_LN_SHIFT (LayerNorm
// statistics of the bulk-copy path: 0 Chan's merge, 2 shifted sums, 1 by
// shape).
struct NormKnobs {
  int g_target, use_tma, tma_threads, tma_cps, tma_stages, l2pf, ln_shift;
  NormKnobs() {
    const int t = env_int("B2K_NORM_TPR", 0);
    g_target = (t >= 1 && t <= kNormMaxThreads && (t & (t - 1)) == 0) ? t : 128;
    use_tma = env_int("B2K_TMA", 1);
    const int th = env_int("B2K_TMA_THREADS", 0);
    tma_threads = (th >= 32 && th <= kNormMaxThreads && (th & (th - 1)) == 0) ? th : 0;
    const int c = env_int("B2K_TMA_CPS", 0);
    tma_cps = (c >= 1 && c <= 8) ? c : 0;
    const int st = env_int("B2K_TMA_STAGES", 0);
    tma_stages = (st >= 2 && st <= 8) ? st : 0;
    l2pf = l2_prefetch_rows_knob();
    const int sh = env_int("B2K_LN_SHIFT", 1);
    ln_shift = sh >= 0 && sh <= 2 ? sh : 1;
  }
};

static const NormKnobs& knobs() {
  static const NormKnobs k;
  return k;
}

template <typename T, int MODE>
static int norm_dispatch_act(const NormArgs& a, int act, cudaStream_t st) {
#define B2K_CASE(k) case k: return norm_launch<T, MODE, k>(a, st);
  switch (act) {
    B2K_CASE(0) B2K_CASE(1) B2K_CASE(2) B2K_CASE(3) B2K_CASE(4) B2K_CASE(5) B2K_CASE(6)
    B2K_CASE(7) B2K_CASE(8) B2K_CASE(9) B2K_CASE(10) B2K_CASE(11) B2K_CASE(12) B2K_CASE(13)
    B2K_CASE(14) B2K_CASE(15) B2K_CASE(16) B2K_CASE(17) B2K_CASE(18) B2K_CASE(19)
    default: set_error("b2k_norm: bad act %d", act); return B2K_EINVAL;
  }
#undef B2K_CASE
}

template <typename T>
static int norm_dispatch(const NormArgs& a, int mode, int act, cudaStream_t st) {
  switch (mode) {
    case NM_LN: return norm_dispatch_act<T, NM_LN>(a, act, st);
    case NM_RMS_W: return norm_dispatch_act<T, NM_RMS_W>(a, act, st);
    case NM_RMS_WROUND: return norm_launch<T, NM_RMS_WROUND, 0>(a, st);
    case NM_RMS_1PW: return norm_launch<T, NM_RMS_1PW, 0>(a, st);
    default: return norm_launch<T, NM_L2, 0>(a, st);
  }
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
  int mode = -1;
  if (norm_kind == B2K_NORM_LN && affine == B2K_AFF_WB) mode = NM_LN;
  if (norm_kind == B2K_NORM_RMS && affine == B2K_AFF_W) mode = NM_RMS_W;
  if (norm_kind == B2K_NORM_RMS && affine == B2K_AFF_W_ROUNDED) mode = NM_RMS_WROUND;
  if (norm_kind == B2K_NORM_RMS && affine == B2K_AFF_ONE_PLUS_W) mode = NM_RMS_1PW;
  if (norm_kind == B2K_NORM_L2 && affine == B2K_AFF_NONE) mode = NM_L2;
  if (mode < 0) {
    set_error("b2k_norm: unsupported (norm_kind %d, affine %d) combination", norm_kind, affine);
    return B2K_EUNSUPPORTED;
  }
  if (act != B2K_ACT_NONE && mode != NM_LN && mode != NM_RMS_W) {
    set_error("b2k_norm: epilogues are built for LayerNorm+WB and RMS+W only");
    return B2K_EUNSUPPORTED;
  }
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
  const NormKnobs& kn = knobs();
  a.g_target = kn.g_target;
  a.use_tma = kn.use_tma;
  a.tma_threads = kn.tma_threads;
  a.tma_cps = kn.tma_cps;
  a.tma_stages = kn.tma_stages;
  a.l2_prefetch_rows = kn.l2pf;
  a.ln_shift = kn.ln_shift;
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

  B2K_DISPATCH_FLOAT(dtype, { return norm_dispatch<T>(a, mode, act, st); });
  return B2K_OK;
}
