// Forward cross-entropy (ouroboros/specs.py:239-241): per row
// loss = logsumexp(x) - x[tgt], 0 for tgt == ignore_index (torch's -100).
//
// Rows up to vocabulary size (128256 at the Llama-3 config) are far larger
// than a block's registers, so each row is streamed once with an online
// (max, sum-of-exp) pair per thread, merged across the block in one
// reduction at the end of the row.
//  * ce_tma_kernel (aligned rows): warp-specialised persistent blocks.  One
//    producer warp streams the block's rows as 16 KB chunks through an
//    S-stage shared-memory ring with bulk copies (full/empty mbarriers); the
//    consumer warps fold each chunk into their running pairs and release the
//    stage.  Loads never wait for the exponentials and vice versa.
//  * ce_pipe_kernel (aligned rows of 4..64 KB, at most 8 rows per SM): whole
//    rows through the block-wide row pipeline.
//  * ce_rows_kernel (any layout): each thread walks its 16-byte vectors U at
//    a time straight from global memory.
// The target logit is a single scalar read; rows whose target is
// ignore_index are not read at all.  b2k_ce_reduce sums per-row losses of a
// shard in fp64 in a fixed order (deterministic) and counts valid rows;
// b2k_ce_mean turns the (possibly all-reduced) pair into the mean.
#include <stdlib.h>

#include "rowio.cuh"
#include "rowpipe.cuh"
#include "tma.cuh"

B2K_DEFINE_TIMEOUT_COUNTER()

namespace b2k {

constexpr int kCeU = 4;

struct CeArgs {
  const void* x;
  const int64_t* tgt;
  void* loss;
  int64_t ldx, M, N, ignore;
  int aligned;
  // backward (fused forward + gradient): dx = (softmax(x) - onehot(t)) *
  // grad_scale / *valid_count for valid rows, 0 for ignored rows
  void* dx;
  int64_t ldd;
  const double* valid_count;
  float grad_scale;
  int l2pf_rows;  // row pipeline: rows per block hinted into L2 before the wait
};

template <typename T, typename OutT>
__global__ void __launch_bounds__(1024) ce_rows_kernel(const CeArgs a) {
  constexpr int E = Traits<T>::E;
  constexpr int H = E / 2;
  constexpr bool P = std::is_same<T, float>::value;
  __shared__ float red[1024];
  const Group g;
  const int64_t row = (int64_t)blockIdx.x * blockDim.y + g.ty;
  const bool valid = row < a.M;
  const int64_t N = a.N;
  // programmatic dependent launch; no L2 hint, since rows whose target is
  // ignore_index are not to be read at all
  griddep_launch_dependents();
  griddep_wait();
  const int64_t t = valid ? a.tgt[row] : a.ignore;
  const bool ignore = (t == a.ignore);
  const bool bad = !ignore && (t < 0 || t >= N);
  const T* xr = static_cast<const T*>(a.x) + (valid ? row * a.ldx : 0);

  // the target logit, loaded now so that its latency overlaps the row
  const float xt = (valid && !ignore && !bad && g.tx == 0) ? to_f<T>(xr[t]) : 0.0f;
  float m = -INFINITY, s = 0.0f;
  if (valid && !ignore && !bad) {
    const int64_t step = (int64_t)g.G * E;
    for (int64_t c0 = (int64_t)g.tx * E; c0 < N; c0 += step * kCeU) {
      float2 v[kCeU][H];
      if (a.aligned && c0 + (kCeU - 1) * step + E <= N) {  // whole group: no bounds checks
#pragma unroll
        for (int u = 0; u < kCeU; ++u) unpack2<T>(ld_stream(xr + c0 + u * step), v[u]);
      } else {
#pragma unroll
        for (int u = 0; u < kCeU; ++u)
          load_vec_fill<T, true>(reinterpret_cast<float*>(v[u]), xr, c0 + u * step, N,
                                 a.aligned, -INFINITY);
      }
      if constexpr (!P) {
        // lazy rescale, as in ce_tma_kernel: keep the running maximum while
        // the group's partial sum against it stays below 2^64
        if (m != -INFINITY) {
          const float2 nz = f2s(-m * kLog2e);
          float2 acc = f2s(0.0f);
#pragma unroll
          for (int u = 0; u < kCeU; ++u)
#pragma unroll
            for (int j = 0; j < H; ++j) {
              const float2 z = fma2(v[u][j], f2s(kLog2e), nz);
              acc = add2(acc, f2(ex2_approx(z.x), ex2_approx(z.y)));
            }
          const float part = acc.x + acc.y;
          if (part < 0x1p64f) {
            s += part;
            continue;
          }
        }
      }
      float bm = -INFINITY;
#pragma unroll
      for (int u = 0; u < kCeU; ++u)
#pragma unroll
        for (int j = 0; j < H; ++j) bm = fmaxf(bm, fmaxf(v[u][j].x, v[u][j].y));
      const float nm = fmaxf(m, bm);
      if (nm == -INFINITY) continue;
      if constexpr (P) {
        float acc = s * expf(m - nm);
#pragma unroll
        for (int u = 0; u < kCeU; ++u)
#pragma unroll
          for (int j = 0; j < H; ++j) acc += expf(v[u][j].x - nm) + expf(v[u][j].y - nm);
        s = acc;
      } else {
        const float2 nz = f2s(-nm * kLog2e);
        float2 acc = f2(s * ex2_approx((m - nm) * kLog2e), 0.0f);
#pragma unroll
        for (int u = 0; u < kCeU; ++u)
#pragma unroll
          for (int j = 0; j < H; ++j) {
            const float2 z = fma2(v[u][j], f2s(kLog2e), nz);
            acc = add2(acc, f2(ex2_approx(z.x), ex2_approx(z.y)));
          }
        s = acc.x + acc.y;
      }
      m = nm;
    }
  }
  group_lse(m, s, g, red);
  if (valid && g.tx == 0) {
    float loss;
    if (ignore) loss = 0.0f;
    else if (bad) loss = __int_as_float(0x7fc00000);  // NaN: target outside [0, N)
    else loss = (m + (P ? logf(s) : f_log<false>(s))) - xt;
    static_cast<OutT*>(a.loss)[row] = from_f<OutT>(loss);
  }
}

#ifndef B2K_CE_CHUNK_BYTES
#define B2K_CE_CHUNK_BYTES 16384
#endif
#ifndef B2K_CE_CONSUMER_WARPS
#define B2K_CE_CONSUMER_WARPS 8
#endif
constexpr int kCeChunkBytes = B2K_CE_CHUNK_BYTES;
constexpr int kCeConsumerWarps = B2K_CE_CONSUMER_WARPS;
constexpr int kCeThreads = 32 * (kCeConsumerWarps + 1);

template <typename T, typename OutT, bool BWD>
__global__ void __launch_bounds__(kCeThreads) ce_tma_kernel(const CeArgs a, const int S) {
  constexpr int E = Traits<T>::E;
  constexpr int H = E / 2;
  constexpr bool P = std::is_same<T, float>::value;
  constexpr int NC = 32 * kCeConsumerWarps;           // consumer threads
  constexpr int CE = kCeChunkBytes / (int)sizeof(T);  // elements per chunk
  constexpr int VPT = CE / E / NC;                    // vectors per consumer per chunk
  static_assert(VPT * E * NC == CE, "chunk must split evenly over the consumers");
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ float red_m[kCeConsumerWarps], red_s[kCeConsumerWarps];
  __shared__ volatile int abort_flag;
  __shared__ int stop;
  __shared__ float row_lse;
  __shared__ float xt_s;
  __shared__ int64_t consumed;
  uint64_t* full = reinterpret_cast<uint64_t*>(dsm + (size_t)S * kCeChunkBytes);
  uint64_t* empty = full + S;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t first = blockIdx.x, stride = gridDim.x;
  const int64_t nrows = first < a.M ? (a.M - 1 - first) / stride + 1 : 0;
  const int64_t N = a.N;
  const int64_t nchunks = (N + CE - 1) / CE;
  const T* xg = static_cast<const T*>(a.x);

  // programmatic dependent launch: wait for the previous kernel before any
  // read (an L2 hint of the first ring's chunks measured 0.9 % slower at
  // 4096 x 128256 bf16, so there is none)
  griddep_launch_dependents();
  griddep_wait();
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCeConsumerWarps);
    }
    fence_barrier_init();
    abort_flag = 0;
    stop = 0;
    consumed = 0;
  }
  __syncthreads();

  int64_t issued = 0;
  // ring position as (stage, phase) counters: no 64-bit division per chunk
  int p_stage = 0;
  uint32_t p_phase = 0;  // phase of the current lap; the empty wait is for the previous lap
  if (warp == 0) {
    const uint64_t pol_keep = policy_evict_last(), pol_drop = policy_evict_first();
    (void)pol_keep;
    (void)pol_drop;
    // ---- producer warp: the whole warp walks the loop (warp-uniform
    // control flow), lane 0 issues the bulk copies
    for (int64_t i = 0; i < nrows; ++i) {
      if (__any_sync(0xffffffffu, abort_flag != 0)) break;
      const int64_t row = first + i * stride;
      const int64_t t = a.tgt[row];
      if (t == a.ignore || t < 0 || t >= N) continue;
      const T* xr = xg + row * a.ldx;
      bool ok = true;
      // forward: one pass; with the gradient a second pass over the same
      // row (served from L2: the row was read a moment ago)
      for (int64_t cc = 0; cc < (BWD ? 2 : 1) * nchunks; ++cc) {
        // the second pass walks the row back to front: its first chunks are
        // the ones the first pass brought into L2 last
        const int64_t c = cc < nchunks ? cc : 2 * nchunks - 1 - cc;
        const int s = p_stage;
        if (issued >= S) {
          ok = __all_sync(0xffffffffu, mbar_wait(&empty[s], p_phase ^ 1u));
          if (!ok) {
            if (lane == 0) { abort_flag = 1; atomicAdd(&b2k_tu_timeouts, 1u); }
            break;
          }
        }
        if (lane == 0) {
          const int64_t n = (N - c * CE) < CE ? (N - c * CE) : CE;
          const uint32_t bytes = (uint32_t)(n * (int64_t)sizeof(T));
          mbar_arrive_expect_tx(&full[s], bytes);
          if constexpr (BWD) {
            // first pass keeps the row in L2 for the second, which drops it
            bulk_g2s_hint(dsm + (size_t)s * kCeChunkBytes, xr + c * CE, bytes, &full[s],
                          cc < nchunks ? pol_keep : pol_drop);
          } else {
            bulk_g2s(dsm + (size_t)s * kCeChunkBytes, xr + c * CE, bytes, &full[s]);
          }
        }
        ++issued;
        if (++p_stage == S) { p_stage = 0; p_phase ^= 1u; }
      }
      __syncwarp();
      if (!ok) break;
    }
  } else {
    // ---- consumers
    const int ct = threadIdx.x - 32;
    const int cw = warp - 1;
    int64_t u = 0;
    int c_stage = 0;
    uint32_t c_phase = 0;
    int64_t t_next = nrows > 0 ? a.tgt[first] : 0;
    // gradient scale, one load per kernel (the count is written before launch)
    float scale = 0.0f;
    if constexpr (BWD) scale = a.grad_scale / (float)(*a.valid_count);
    (void)scale;
    // a positive finite scale is folded into the exponent of the 16-bit path
    const bool fold = !P && scale > 0.0f && scale < INFINITY;
    const float log2_scale = fold ? log2f(scale) : 0.0f;
    (void)fold;
    (void)log2_scale;
    for (int64_t i = 0; i < nrows; ++i) {
      const int64_t row = first + i * stride;
      const int64_t t = t_next;  // loaded one row ahead
      if (i + 1 < nrows) t_next = a.tgt[row + stride];
      const bool ignore = (t == a.ignore);
      if (ignore || t < 0 || t >= N) {
        if (ct == 0)
          static_cast<OutT*>(a.loss)[row] =
              from_f<OutT>(ignore ? 0.0f : __int_as_float(0x7fc00000));
        if constexpr (BWD) {  // no gradient through ignored rows (NaN for bad targets)
          const float fill = ignore ? 0.0f : __int_as_float(0x7fc00000);
          float z[E];
#pragma unroll
          for (int e = 0; e < E; ++e) z[e] = fill;
          const uint4 zv = pack<T>(z);
          T* dr = static_cast<T*>(a.dx) + row * a.ldd;
          for (int64_t c = (int64_t)ct * E; c < N; c += (int64_t)NC * E) st_stream(dr + c, zv);
        }
        continue;
      }
      // where the target logit sits: chunk, offset, and (second pass) the
      // consumer thread and vector slot that hold it
      const int64_t t_chunk = t / CE;
      const int t_in = (int)(t - t_chunk * CE);
      const int t_owner = (t_in / E) % NC;
      (void)t_owner;
      float m = -INFINITY, s = 0.0f;
      int n_left = (int)(N < (int64_t)0x7fffffff ? N : 0x7fffffff);
      for (int64_t c = 0; c < nchunks; ++c, ++u, n_left -= CE) {
        const int st = c_stage;
        bool ok = false;
        if (!abort_flag) {
          ok = mbar_wait(&full[st], c_phase);
          if (!ok) { abort_flag = 1; atomicAdd(&b2k_tu_timeouts, 1u); }
        }
        if (ok) {
          const T* cs = reinterpret_cast<const T*>(dsm + (size_t)st * kCeChunkBytes);
          const int n = n_left < CE ? n_left : CE;
          if (ct == 0 && c == t_chunk) xt_s = to_f<T>(cs[t_in]);  // the target logit
          float2 v[VPT][H];
          if (n == CE) {  // every chunk but a row's last: no bounds checks
#pragma unroll
            for (int k = 0; k < VPT; ++k)
              unpack2<T>(*reinterpret_cast<const uint4*>(cs + (k * NC + ct) * E), v[k]);
          } else {
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
              const int idx = (k * NC + ct) * E;
              if (idx < n) {
                unpack2<T>(*reinterpret_cast<const uint4*>(cs + idx), v[k]);
              } else {
#pragma unroll
                for (int j = 0; j < H; ++j) v[k][j] = f2s(-INFINITY);
              }
            }
          }
          // sum of 2^(x log2e - nz) over the chunk, f32x2 FMA + ex2.approx
          auto sum_exp = [&](const float2 nz) {
            float2 acc[VPT];
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
              acc[k] = f2s(0.0f);
#pragma unroll
              for (int j = 0; j < H; ++j) {
                const float2 z = fma2(v[k][j], f2s(kLog2e), nz);
                acc[k] = add2(acc[k], f2(ex2_approx(z.x), ex2_approx(z.y)));
              }
            }
#pragma unroll
            for (int k = 1; k < VPT; ++k) acc[0] = add2(acc[0], acc[k]);
            return acc[0].x + acc[0].y;
          };
          bool done = false;
          if constexpr (!P) {
            // Lazy rescale: sum against the running maximum without taking
            // the chunk's maximum.  A partial sum below 2^64 proves every
            // term finite and below 2^64 (no rescale needed: the pair stays
            // exact up to fp32 rounding); otherwise (a new maximum far above
            // the old one, inf or NaN) the chunk is redone below against its
            // own maximum.
            if (m != -INFINITY) {
              const float part = sum_exp(f2s(-m * kLog2e));
              if (part < 0x1p64f) { s += part; done = true; }
            }
          }
          if (!done) {
            // tree max (short dependency chains)
            float bmk[VPT];
#pragma unroll
            for (int k = 0; k < VPT; ++k) {
              float t0 = fmaxf(v[k][0].x, v[k][0].y);
#pragma unroll
              for (int j = 1; j < H; ++j) t0 = fmaxf(t0, fmaxf(v[k][j].x, v[k][j].y));
              bmk[k] = t0;
            }
            float bm = bmk[0];
#pragma unroll
            for (int k = 1; k < VPT; ++k) bm = fmaxf(bm, bmk[k]);
            const float nm = fmaxf(m, bm);
            if (nm != -INFINITY) {
              if constexpr (P) {
                float acc = s * expf(m - nm);
#pragma unroll
                for (int k = 0; k < VPT; ++k)
#pragma unroll
                  for (int j = 0; j < H; ++j) acc += expf(v[k][j].x - nm) + expf(v[k][j].y - nm);
                s = acc;
              } else {
                s = fmaf(s, ex2_approx((m - nm) * kLog2e), sum_exp(f2s(-nm * kLog2e)));
              }
              m = nm;
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        if (++c_stage == S) { c_stage = 0; c_phase ^= 1u; }
      }
      // merge the consumers' pairs: warp shuffles, then across warps
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
        lse_merge(m, s, m2, s2);
      }
      if (lane == 0) { red_m[cw] = m; red_s[cw] = s; }
      named_bar_sync(1, NC);
      if (ct == 0) {
        float M = red_m[0], Ssum = red_s[0];
        for (int w = 1; w < kCeConsumerWarps; ++w) lse_merge(M, Ssum, red_m[w], red_s[w]);
        const float lse = M + (P ? logf(Ssum) : f_log<false>(Ssum));
        static_cast<OutT*>(a.loss)[row] = from_f<OutT>(lse - xt_s);
        row_lse = lse;
        stop = abort_flag;
      }
      named_bar_sync(1, NC);
      if (stop) break;
      if constexpr (BWD) {
        // second pass: dx = exp(x - lse) * scale - scale * [j == t]
        const float lse = row_lse;
        // 16-bit path: exp(x - lse) * scale = 2^(x log2e - lse log2e + log2 scale),
        // the scale folded into the exponent (one multiply less per pair)
        const float2 nl = f2s(-lse * kLog2e + (fold ? log2_scale : 0.0f));
        T* dr = static_cast<T*>(a.dx) + row * a.ldd;
        for (int64_t c = nchunks - 1; c >= 0; --c, ++u) {  // back to front
          const int st = c_stage;
          bool ok = false;
          if (!abort_flag) {
            ok = mbar_wait(&full[st], c_phase);
            if (!ok) { abort_flag = 1; atomicAdd(&b2k_tu_timeouts, 1u); }
          }
          if (ok) {
            const T* cs = reinterpret_cast<const T*>(dsm + (size_t)st * kCeChunkBytes);
            const int n = (int)((N - c * CE) < CE ? (N - c * CE) : CE);
            auto grad_vec = [&](const int idx, auto folded) {
              float2 v[H];
              unpack2<T>(*reinterpret_cast<const uint4*>(cs + idx), v);
#pragma unroll
              for (int j = 0; j < H; ++j) {
                if constexpr (P) {
                  v[j] = f2(expf(v[j].x - lse) * scale, expf(v[j].y - lse) * scale);
                } else {
                  const float2 z = fma2(v[j], f2s(kLog2e), nl);
                  v[j] = f2(ex2_approx(z.x), ex2_approx(z.y));
                  if constexpr (!decltype(folded)::value) v[j] = mul2(v[j], f2s(scale));
                }
              }
              st_stream(dr + c * CE + idx, pack2<T>(v));
            };
            auto grad_chunk = [&](auto folded) {
              if (n == CE) {  // full chunk: no bounds checks
#pragma unroll
                for (int k = 0; k < VPT; ++k) grad_vec((k * NC + ct) * E, folded);
              } else {
#pragma unroll
                for (int k = 0; k < VPT; ++k)
                  if ((k * NC + ct) * E < n) grad_vec((k * NC + ct) * E, folded);
              }
            };
            if (fold) grad_chunk(std::true_type{});
            else grad_chunk(std::false_type{});
            if (c == t_chunk && ct == t_owner) {
              // the target's entry, p*scale - scale, stored over the vector
              // that this same thread wrote above (program order: this wins)
              const float xt = to_f<T>(cs[t_in]);
              float ps;  // p * scale
              if constexpr (P) ps = expf(xt - lse) * scale;
              else ps = fold ? ex2_approx(fmaf(xt, kLog2e, nl.x))
                             : ex2_approx(fmaf(xt, kLog2e, nl.x)) * scale;
              dr[t] = from_f<T>(ps - scale);
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[st]);
          if (++c_stage == S) { c_stage = 0; c_phase ^= 1u; }
        }
      }
    }
    if (ct == 0) consumed = u;
  }
  __syncthreads();
  // after an abort, wait (bounded) for copies still in flight
  if (threadIdx.x == 0)
    for (int64_t j = consumed; j < issued; ++j)
      mbar_wait(&full[(int)(j % S)], (uint32_t)((j / S) & 1));
}

// Rows of 4..64 KB (the spec shapes, V up to 32768 at 2 bytes): whole rows
// through the persistent bulk-copy row pipeline; each thread takes a local
// (max, sum-exp) over its slice, one block reduction per row, the target
// logit read from the staged row.
template <typename T, typename OutT, int V>
__global__ void __launch_bounds__(512) ce_pipe_kernel(const CeArgs a, const int S_) {
  constexpr int E = Traits<T>::E;
  constexpr int H = E / 2;
  constexpr bool P = std::is_same<T, float>::value;
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ float red[1024];
  __shared__ volatile int abort_flag;
  __shared__ float xt_s;
  const Group g;
  const int N = (int)a.N;
  if (g.tx == 0) abort_flag = 0;
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
    const int64_t row = pipe.row_of(k);
    const int64_t t = a.tgt[row];
    const bool ignore = (t == a.ignore), bad = !ignore && (t < 0 || t >= N);
    float m = -INFINITY, s = 0.0f;
    if (!ignore && !bad) {
      float2 v[V][H];
      float bm = -INFINITY;
#pragma unroll
      for (int q = 0; q < V; ++q) {
        const int c = (q * g.G + g.tx) * E;
        if (c < N) {
          unpack2<T>(*reinterpret_cast<const uint4*>(xs + c), v[q]);
        } else {
#pragma unroll
          for (int j = 0; j < H; ++j) v[q][j] = f2s(-INFINITY);
        }
#pragma unroll
        for (int j = 0; j < H; ++j) bm = fmaxf(bm, fmaxf(v[q][j].x, v[q][j].y));
      }
      // the warp's maximum (the row's branch is the same in the whole block):
      // the warp stage of the merge is then a plain sum
      bm = warp_allmax(bm);
      if (bm != -INFINITY) {
        m = bm;
        if constexpr (P) {
#pragma unroll
          for (int q = 0; q < V; ++q)
#pragma unroll
            for (int j = 0; j < H; ++j) s += expf(v[q][j].x - m) + expf(v[q][j].y - m);
        } else {
          const float2 nz = f2s(-m * kLog2e);
          float2 acc = f2s(0.0f);
#pragma unroll
          for (int q = 0; q < V; ++q)
#pragma unroll
            for (int j = 0; j < H; ++j) {
              const float2 z = fma2(v[q][j], f2s(kLog2e), nz);
              acc = add2(acc, f2(ex2_approx(z.x), ex2_approx(z.y)));
            }
          s = acc.x + acc.y;
        }
      }
      if (g.tx == 0) xt_s = to_f<T>(xs[t]);
    }
    group_lse_wmax(m, s, g, red);  // barriers: every read of the stage is done
    if (abort_flag) break;
    pipe.refill();
    if (g.tx == 0) {
      float loss;
      if (ignore) loss = 0.0f;
      else if (bad) loss = __int_as_float(0x7fc00000);
      else loss = (m + (P ? logf(s) : f_log<false>(s))) - xt_s;
      static_cast<OutT*>(a.loss)[row] = from_f<OutT>(loss);
    }
  }
  pipe.drain(k);
}

static int ce_env(const char* name, int dflt) {
  const char* s = getenv(name);
  return s ? atoi(s) : dflt;
}

// Launches the row-loss kernel; with a.dx set, the pipelined kernel also
// writes the gradient (*bwd_done = true), the rows kernel does not.
template <typename T, typename OutT>
static int ce_launch(const CeArgs& a, cudaStream_t st, bool* bwd_done = nullptr) {
  constexpr int E = Traits<T>::E;
  static const int use_tma = ce_env("B2K_TMA", 1);
  if (bwd_done) *bwd_done = false;
  if (use_tma && a.aligned && a.N * (int64_t)sizeof(T) >= 4 * kCeChunkBytes) {
    // ring shape measured at 32768 x 128256 bf16: the forward runs best with
    // 3 CTAs per SM x 4 stages, forward + gradient (twice the stores, the
    // second pass served from L2, whose capacity bounds the rows in flight)
    // with 2 CTAs per SM x 4 stages
    static const int S_fwd = [] {
      const int v = ce_env("B2K_CE_STAGES", 4);
      return v >= 2 && v <= 12 ? v : 4;
    }();
    static const int cps_fwd = [] {
      const int v = ce_env("B2K_CE_CPS", 3);
      return v >= 1 && v <= 4 ? v : 3;
    }();
    static const int S_bwd = [] {
      const int v = ce_env("B2K_CE_BWD_STAGES", 4);
      return v >= 2 && v <= 12 ? v : 4;
    }();
    static const int cps_bwd = [] {
      const int v = ce_env("B2K_CE_BWD_CPS", 2);
      return v >= 1 && v <= 4 ? v : 2;
    }();
    const int S = a.dx ? S_bwd : S_fwd;
    const int cps = a.dx ? cps_bwd : cps_fwd;
    const size_t smem = (size_t)S * kCeChunkBytes + 2 * (size_t)S * sizeof(uint64_t);
    // every resident slot gets a block: the kernel is bound by the SMs'
    // exponential throughput as much as by HBM, so what must be even is the
    // rows per SM (27-28 at 4096 rows), not per block.  A grid trimmed so
    // that every block walks the same number of rows (410 blocks of 10 at
    // 4096 rows) left 114 SMs with 30 rows and measured 0.190 against 0.176
    // ms.
    int64_t grid = (int64_t)sm_count() * cps;
    if (grid > a.M) grid = a.M;
    auto kern = a.dx ? ce_tma_kernel<T, OutT, true> : ce_tma_kernel<T, OutT, false>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    launch_pdl(kern, dim3((unsigned)grid), dim3(kCeThreads), smem, st, a, S);
    if (bwd_done) *bwd_done = a.dx != nullptr;
    return check_launch("b2k_cross_entropy(tma)");
  }
  const int64_t nvec = (a.N + E - 1) / E;
  // few rows (<= 8 per SM) of 256 vectors .. 64 KB: whole rows through the
  // persistent row pipeline, whose staged loads hide the latency a handful of
  // row blocks cannot (forward only; a gradient is added by the rows kernel).
  // With more rows the rows kernel below keeps more loads in flight and is
  // faster (measured on the spec shape grid: 1024 x 4096 5.0 vs 7.2 us,
  // 8192 x 4096 21.2 vs 18.3 us).
  static const int use_pipe = ce_env("B2K_CE_PIPE", 1);
  // B2K_CE_PIPE_RPS: most rows per SM that take the pipeline (default 8)
  static const int pipe_rps = [] {
    const int v = ce_env("B2K_CE_PIPE_RPS", 8);
    return v >= 1 && v <= 1 << 20 ? v : 8;
  }();
  const int64_t row_bytes = a.N * (int64_t)sizeof(T);
  if (use_tma && use_pipe && a.aligned && nvec >= 256 && row_bytes <= (64 << 10) &&
      a.M <= (int64_t)pipe_rps * sm_count()) {
    int G = next_pow2((nvec + 3) / 4);
    G = G < 64 ? 64 : (G > 512 ? 512 : G);
    const int64_t vneed = (nvec + G - 1) / G;
    if (vneed <= 4) {
      auto kern = vneed <= 2 ? ce_pipe_kernel<T, OutT, 2> : ce_pipe_kernel<T, OutT, 4>;
      PipeShape ps;
      if (choose_pipe_shape(kern, G, row_bytes, 0, 0, &ps)) {
        const size_t smem = RowPipe<1>::smem_bytes(ps.S, row_bytes);
        int64_t grid = (int64_t)sm_count() * ps.cps;
        if (grid > a.M) grid = a.M;
        launch_pdl(kern, dim3((unsigned)grid), dim3(G), smem, st, a, ps.S);
        return check_launch("b2k_cross_entropy(pipe)");
      }
    }
  }
  // threads per row: enough that each walks ~32 vectors, 32..1024
  int G = next_pow2((nvec + 31) / 32);
  G = G < 32 ? 32 : (G > 1024 ? 1024 : G);
  static const int override_g = [] {
    const char* s = getenv("B2K_CE_THREADS");
    const int v = s ? atoi(s) : 0;
    return (v >= 32 && v <= 1024 && (v & (v - 1)) == 0) ? v : 0;
  }();
  if (override_g) G = override_g;
  const int R = G >= 256 ? 1 : 256 / G;
  const int64_t grid = (a.M + R - 1) / R;
  launch_pdl(ce_rows_kernel<T, OutT>, dim3((unsigned)grid), dim3(G, R), 0, st, a);
  return check_launch("b2k_cross_entropy");
}

// one block, fixed summation order
__global__ void __launch_bounds__(1024) ce_reduce_kernel(const float* loss, const int64_t* tgt,
                                                         int64_t M, int64_t ignore,
                                                         double* sumcount) {
  __shared__ double rs[32], rc[32];
  double s = 0.0, c = 0.0;
  for (int64_t i = threadIdx.x; i < M; i += blockDim.x) {
    if (tgt[i] != ignore) { s += (double)loss[i]; c += 1.0; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    c += __shfl_xor_sync(0xffffffffu, c, o);
  }
  if ((threadIdx.x & 31) == 0) { rs[threadIdx.x >> 5] = s; rc[threadIdx.x >> 5] = c; }
  __syncthreads();
  if (threadIdx.x == 0) {
    double ts = 0.0, tc = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) { ts += rs[i]; tc += rc[i]; }
    sumcount[0] = ts;
    sumcount[1] = tc;
  }
}

__global__ void ce_mean_kernel(const double* sumcount, float* out) {
  out[0] = (float)(sumcount[0] / sumcount[1]);  // 0/0 -> NaN (no valid row)
}

// Gradient of the mean loss for layouts the pipelined kernel does not take
// (short or misaligned rows): lse recovered from the fp32 row loss
// (loss = lse - x[t]), then dx = (exp(x - lse) - [j == t]) * scale.
template <typename T>
__global__ void __launch_bounds__(256) ce_bwd_rows_kernel(const CeArgs a) {
  constexpr bool P = std::is_same<T, float>::value;
  const int64_t row = blockIdx.x;
  const int64_t t = a.tgt[row];
  const bool ignore = (t == a.ignore), bad = !ignore && (t < 0 || t >= a.N);
  const T* xr = static_cast<const T*>(a.x) + row * a.ldx;
  T* dr = static_cast<T*>(a.dx) + row * a.ldd;
  if (ignore || bad) {
    const float fill = ignore ? 0.0f : __int_as_float(0x7fc00000);
    for (int64_t j = threadIdx.x; j < a.N; j += blockDim.x) dr[j] = from_f<T>(fill);
    return;
  }
  const float lse = static_cast<const float*>(a.loss)[row] + to_f<T>(xr[t]);
  const float scale = a.grad_scale / (float)(*a.valid_count);
  for (int64_t j = threadIdx.x; j < a.N; j += blockDim.x) {
    float d = f_exp<P>(to_f<T>(xr[j]) - lse) * scale;
    if (j == t) d -= scale;
    dr[j] = from_f<T>(d);
  }
}

__global__ void __launch_bounds__(1024) ce_count_kernel(const int64_t* tgt, int64_t M,
                                                        int64_t ignore, double* count) {
  __shared__ double rc[32];
  double c = 0.0;
  for (int64_t i = threadIdx.x; i < M; i += blockDim.x) c += (tgt[i] != ignore) ? 1.0 : 0.0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) rc[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    double tc = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tc += rc[i];
    *count = tc;
  }
}

}  // namespace b2k

using namespace b2k;

extern "C" int b2k_cross_entropy(const void* x, int64_t ldx, const int64_t* tgt, void* loss,
                                 int64_t M, int64_t N, int dtype, int out_dtype,
                                 int64_t ignore_index, void* stream) {
  B2K_REQUIRE(M >= 0 && N >= 0, "b2k_cross_entropy: negative shape");
  B2K_REQUIRE(M <= 1 || ldx >= N, "b2k_cross_entropy: row stride smaller than N");
  B2K_REQUIRE(M <= 0x7fffffffLL * 8LL, "b2k_cross_entropy: too many rows");
  B2K_REQUIRE(out_dtype == dtype || out_dtype == B2K_F32,
              "b2k_cross_entropy: out_dtype must be the input dtype or F32");
  if (M == 0) return B2K_OK;
  B2K_REQUIRE(x != nullptr || N == 0, "b2k_cross_entropy: null x");
  B2K_REQUIRE(tgt != nullptr && loss != nullptr, "b2k_cross_entropy: null tgt/loss");
  CeArgs a = {};
  a.x = x; a.tgt = tgt; a.loss = loss; a.ldx = ldx; a.M = M; a.N = N; a.ignore = ignore_index;
  a.l2pf_rows = l2_prefetch_rows_knob();
  const int es = dtype_size(dtype);
  const int E = es ? 16 / es : 1;
  a.aligned = (N % E == 0) && aligned16(x) && ((ldx * es) % 16 == 0);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  B2K_DISPATCH_FLOAT(dtype, {
    if (out_dtype == B2K_F32) return ce_launch<T, float>(a, st);
    return ce_launch<T, T>(a, st);
  });
  return B2K_OK;
}

extern "C" int b2k_ce_reduce(const float* row_loss, const int64_t* tgt, int64_t M,
                             int64_t ignore_index, double* sumcount, void* stream) {
  B2K_REQUIRE(M >= 0, "b2k_ce_reduce: negative M");
  B2K_REQUIRE(sumcount != nullptr, "b2k_ce_reduce: null output");
  B2K_REQUIRE(M == 0 || (row_loss != nullptr && tgt != nullptr), "b2k_ce_reduce: null input");
  ce_reduce_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(row_loss, tgt, M,
                                                                    ignore_index, sumcount);
  return check_launch("b2k_ce_reduce");
}

extern "C" int b2k_ce_mean(const double* sumcount, float* out, void* stream) {
  B2K_REQUIRE(sumcount != nullptr && out != nullptr, "b2k_ce_mean: null pointer");
  ce_mean_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(sumcount, out);
  return check_launch("b2k_ce_mean");
}

extern "C" int b2k_ce_valid_count(const int64_t* tgt, int64_t M, int64_t ignore_index,
                                  double* count, void* stream) {
  B2K_REQUIRE(M >= 0 && count != nullptr && (M == 0 || tgt != nullptr),
              "b2k_ce_valid_count: bad arguments");
  ce_count_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(tgt, M, ignore_index, count);
  return check_launch("b2k_ce_valid_count");
}

extern "C" int b2k_cross_entropy_fwd_bwd(const void* x, int64_t ldx, const int64_t* tgt,
                                         int64_t M, int64_t N, int dtype, int64_t ignore_index,
                                         const double* valid_count, float grad_scale,
                                         float* row_loss, void* dx, int64_t ldd, void* stream) {
  B2K_REQUIRE(M >= 0 && N >= 1, "b2k_cross_entropy_fwd_bwd: need M >= 0 and N >= 1");
  B2K_REQUIRE(M <= 1 || (ldx >= N && ldd >= N), "b2k_cross_entropy_fwd_bwd: row stride < N");
  B2K_REQUIRE(valid_count != nullptr && row_loss != nullptr && dx != nullptr,
              "b2k_cross_entropy_fwd_bwd: null valid_count / row_loss / dx");
  B2K_REQUIRE(M <= 0x7fffffffLL, "b2k_cross_entropy_fwd_bwd: too many rows");
  if (M == 0) return B2K_OK;
  CeArgs a = {};
  a.x = x; a.tgt = tgt; a.loss = row_loss; a.ldx = ldx; a.M = M; a.N = N; a.ignore = ignore_index;
  a.dx = dx; a.ldd = ldd; a.valid_count = valid_count; a.grad_scale = grad_scale;
  a.l2pf_rows = l2_prefetch_rows_knob();
  const int es = dtype_size(dtype);
  const int E = es ? 16 / es : 1;
  a.aligned = (N % E == 0) && aligned16(x) && aligned16(dx) && ((ldx * es) % 16 == 0) &&
              ((ldd * es) % 16 == 0);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  B2K_DISPATCH_FLOAT(dtype, {
    bool done = false;
    const int rc = ce_launch<T, float>(a, st, &done);
    if (rc != B2K_OK || done) return rc;
    // the rows kernel wrote the row losses; now the gradient from them
    ce_bwd_rows_kernel<T><<<(unsigned)M, 256, 0, st>>>(a);
    return check_launch("b2k_cross_entropy_fwd_bwd");
  });
  return B2K_OK;
}
