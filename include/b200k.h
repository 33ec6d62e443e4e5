/*
 * b200k.h — C ABI of libb200k.so, the sm_100a (B200) kernels for the
 * ouroboros-kernelsmith op suite (ouroboros/specs.py, ouroboros/chains.py).
 *
 * In the reference every op is a Python source string defining
 * `run(*inputs) -> Tensor`, evaluated by ouroboros/harness.py (_worker calls
 * `run(*clones)` at harness.py:176 and times it at harness.py:253).  Each
 * entry point below is the native body behind one family of those `run`
 * functions; the Python package `b200k` keeps the spec signatures and calls
 * these through ctypes.
 *
 * Conventions shared by every entry point:
 *   - tensors are device pointers; 2-D operands are row-major with a row
 *     stride `ld*` counted in ELEMENTS and a unit inner stride;
 *   - `dtype` is a b2k_dtype; floating operands of one call share it unless
 *     the argument list names a separate dtype;
 *   - inputs are never written (harness.py:184-188 rejects mutation); outputs
 *     are written completely;
 *   - launches go on `stream` (a cudaStream_t, NULL = legacy default stream),
 *     nothing synchronises the host;
 *   - the return value is a b2k_status; on failure b2k_last_error() returns a
 *     thread-local message.  No compute entry point allocates device memory;
 *     the one allocating call is b2k_ce_exchange_alloc, the set-up of the
 *     multi-GPU cross-entropy exchange buffer (freed by b2k_ce_exchange_free).
 */
#ifndef B200K_H
#define B200K_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types (torch.float32 / float16 / bfloat16 / int8 / int64). */
enum b2k_dtype { B2K_F32 = 0, B2K_F16 = 1, B2K_BF16 = 2, B2K_I8 = 3, B2K_I64 = 4 };

enum b2k_status {
  B2K_OK = 0,
  B2K_EINVAL = 1,       /* bad shape / stride / dtype / enum argument        */
  B2K_EALIGN = 2,       /* reserved: misaligned operand where one is required */
  B2K_ELAUNCH = 3,      /* a CUDA launch or runtime call failed               */
  B2K_EUNSUPPORTED = 4  /* combination not built into this library            */
};

/* Epilogues of the chain grammar, in the order of chains.py:56-58 (ACTNAMES),
 * with the functions of chains.py:13-53 (ACTS).  0 = identity. */
enum b2k_act {
  B2K_ACT_NONE = 0, B2K_ACT_GELU = 1, B2K_ACT_SILU = 2, B2K_ACT_RELU2 = 3,
  B2K_ACT_TANH = 4, B2K_ACT_SIGMOID = 5, B2K_ACT_RELU = 6, B2K_ACT_SQUARE = 7,
  B2K_ACT_ABS = 8, B2K_ACT_SOFTSIGN = 9, B2K_ACT_HARDSIGMOID = 10,
  B2K_ACT_HARDSWISH = 11, B2K_ACT_LEAKY_RELU = 12, B2K_ACT_RELU6 = 13,
  B2K_ACT_HARDTANH = 14, B2K_ACT_ELU = 15, B2K_ACT_SELU = 16,
  B2K_ACT_SOFTPLUS = 17, B2K_ACT_MISH = 18, B2K_ACT_GELU_ERF = 19,
  B2K_ACT_COUNT = 20
};

/* Row statistic of b2k_norm. */
enum b2k_norm_kind {
  B2K_NORM_RMS = 0,   /* rs = rsqrt(mean(h^2) + eps)                       */
  B2K_NORM_L2 = 1,    /* rs = rsqrt(sum(h^2) + eps)        (specs.py:171)  */
  B2K_NORM_LN = 2     /* mu = mean(h), rs = rsqrt(mean((h-mu)^2) + eps)    */
};

/* How the normalised row meets the weights (before the epilogue). */
enum b2k_affine {
  B2K_AFF_NONE = 0,      /* n = h*rs                              l2norm     */
  B2K_AFF_W_ROUNDED = 1, /* n = T(T(h*rs) * w)   rmsnorm/add_rmsnorm (specs.py:78,93) */
  B2K_AFF_W = 2,         /* n = h*rs*w           RMS chains (chains.py:80)    */
  B2K_AFF_ONE_PLUS_W = 3,/* n = h*rs*(1+w)       rmsnorm_gemma (specs.py:220) */
  B2K_AFF_WB = 4         /* n = (h-mu)*rs*w + b  LayerNorm (specs.py:112)     */
};

/* Softmax-family variants. */
enum b2k_softmax_kind {
  B2K_SOFTMAX = 0,       /* specs.py:81-82   */
  B2K_SOFTCAP = 1,       /* specs.py:210-213 (cap 30) */
  B2K_LOG_SOFTMAX = 2,   /* specs.py:176-177 */
  B2K_SOFTMAX_SCALE = 3  /* specs.py:180-181, scale read from device memory */
};

/* Library version (major*10000 + minor*100 + patch). */
int b2k_version(void);

/* Message of the last failed call on this host thread ("" if none). */
const char* b2k_last_error(void);

/* Number of bounded pipeline waits that gave up (each is a failed kernel
 * whose outputs are incomplete) since the last reset, summed over all kernel
 * families; reset != 0 clears the counters.  Synchronous: call after the
 * work of interest has completed.  No reference counterpart (the Triton
 * kernels have no device-side waits). */
unsigned b2k_pipeline_timeouts(int reset);

/* Exercises the bounded device wait of the pipelines: one block waits on a
 * barrier that nothing completes, gives up after limit_ns (<= 10 s), adds one
 * to the timeout counter and writes *status = 1 (device int) — the context
 * stays usable.  No reference counterpart (failure-path self-test). */
int b2k_selftest_bounded_wait(unsigned long long limit_ns, int* status, void* stream);

/* Residual -> {RMSNorm, L2, LayerNorm} -> affine -> epilogue, one row per
 * thread group, row held in registers (rows longer than the register budget
 * stream through L2 in two or three passes).
 * Replaces the `run` of: rmsnorm (specs.py:667-678), add_rmsnorm (:701-712),
 * layernorm (:725-736), add_layernorm (:737-748), l2norm (:788-790),
 * layernorm_gelu (:798-801), rmsnorm_gemma (:818-823), rmsnorm_wide
 * (:866-871), the 76 chains of chains.py:69-87 registered at specs.py:1001-1017,
 * and the *_short variants (specs.py:983-997).
 *   r  : residual (NULL = none)          ldr : its row stride
 *   w,b: (N,) weights / bias (NULL where the affine mode does not use them)
 *   y  : (M,N) output                     h   : optional (M,N) output of
 *        T(x + r) (the residual stream; NULL = not written)
 *   eps: added inside the rsqrt. */
int b2k_norm(const void* x, int64_t ldx, const void* r, int64_t ldr,
             const void* w, const void* b, void* y, int64_t ldy,
             void* h, int64_t ldh, int64_t M, int64_t N, int dtype,
             int norm_kind, int affine, int act, float eps, void* stream);

/* Row softmax family (see b2k_softmax_kind).  `scale` points to one element
 * of `scale_dtype` in device memory (B2K_SOFTMAX_SCALE only, else NULL).
 * Replaces softmax (specs.py:679-689), softcap_softmax (:813-817),
 * log_softmax (:791-793), softmax_scale (:794-797). */
int b2k_softmax(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t M,
                int64_t N, int dtype, int kind, const void* scale,
                int scale_dtype, void* stream);

/* Gated units y = act(gate) * up over (M,N), act in {SILU (swiglu),
 * SIGMOID (glu), GELU (geglu), RELU (reglu)}.
 * Replaces swiglu (specs.py:690-700), glu (:824-826), geglu (:749-759),
 * reglu (:785-787). */
int b2k_glu(const void* gate, int64_t ldg, const void* up, int64_t ldu,
            void* y, int64_t ldy, int64_t M, int64_t N, int dtype, int act,
            void* stream);

/* Pointwise y = act(x + bias) over (M,N); bias is (N,) or NULL.
 * act = GELU (gelu, bias_gelu), SILU (silu), RELU2 (relu2).
 * Replaces gelu (specs.py:775), silu (:778), relu2 (:780), bias_gelu (:782). */
int b2k_act(const void* x, int64_t ldx, const void* bias, void* y,
            int64_t ldy, int64_t M, int64_t N, int dtype, int act,
            void* stream);

/* Per-row int8 dequantisation y = fp16(float(q) * float(scale[row])).
 * q: (M,N) int8, scale: (M,1) of scale_dtype with row stride lds, y: fp16.
 * Replaces dequant_int8 (specs.py:808-811). */
int b2k_dequant_i8(const void* q, int64_t ldq, const void* scale, int64_t lds,
                   int scale_dtype, void* y, int64_t ldy, int64_t M, int64_t N,
                   void* stream);

/* Rotary embedding with per-row tables (the spec layout).
 *   interleaved = 0: x, cos, sin are (M,D); out = x*cos + rotate_half(x)*sin
 *                    (rope, specs.py:713-724, reference specs.py:96-102)
 *   interleaved = 1: cos, sin are (M,D/2); pairs (x[2i],x[2i+1]) rotate by
 *                    (cos[i],sin[i])  (rope_interleaved, specs.py:827-832) */
int b2k_rope(const void* x, int64_t ldx, const void* cos, int64_t ldc,
             const void* sin, int64_t lds, void* y, int64_t ldy, int64_t M,
             int64_t D, int dtype, int interleaved, void* stream);

/* Rotary embedding of q [B,S,H,D] and k [B,S,Hk,D] (contiguous) in ONE
 * launch, from position tables cos, sin [S, D/2] (position s uses row s).
 * Writes q_out, k_out (same shapes).  interleaved as in b2k_rope; for the
 * half-split form, element i and i+D/2 both use table column i.
 * No reference counterpart: the attention-layout form of the rope /
 * rope_interleaved math above (specs.py:96-102, :228-236). */
int b2k_rope_qk(const void* q, const void* k, const void* cos, const void* sin,
                void* q_out, void* k_out, int64_t B, int64_t S, int64_t H,
                int64_t Hk, int64_t D, int dtype, int interleaved,
                void* stream);

/* Residual -> RMSNorm over D -> *w -> half-split RoPE with (M,D) tables.
 * r = NULL: qknorm_rope (specs.py:760-773, reference :133-143);
 * r given : add_rmsnorm_rope (specs.py:802-807, reference :193-198). */
int b2k_norm_rope(const void* x, int64_t ldx, const void* r, int64_t ldr,
                  const void* w, const void* cos, int64_t ldc, const void* sin,
                  int64_t lds, void* y, int64_t ldy, int64_t M, int64_t D,
                  int dtype, float eps, void* stream);

/* Per-row cross-entropy loss[i] = logsumexp(x[i]) - x[i, tgt[i]] (single
 * streaming pass, online max/sum), 0 where tgt[i] == ignore_index, NaN where
 * tgt[i] is out of [0,N) otherwise.  loss is (M,) of `out_dtype` (the spec
 * returns x.dtype).  Replaces cross_entropy (specs.py:833-838, reference
 * :239-241). */
int b2k_cross_entropy(const void* x, int64_t ldx, const int64_t* tgt,
                      void* loss, int64_t M, int64_t N, int dtype,
                      int out_dtype, int64_t ignore_index, void* stream);

/* Sum of per-row losses and count of valid rows of one shard:
 * sumcount[0] = sum(loss[i] for tgt[i] != ignore_index) (fp64),
 * sumcount[1] = number of such rows.  One CTA, fixed order (deterministic).
 * With b2k_cross_entropy (out_dtype F32) it forms the reduced loss; the two
 * doubles are what the multi-GPU path all-reduces. */
int b2k_ce_reduce(const float* row_loss, const int64_t* tgt, int64_t M,
                  int64_t ignore_index, double* sumcount, void* stream);

/* out[0] = (float)(sumcount[0] / sumcount[1]) (NaN when the count is 0). */
int b2k_ce_mean(const double* sumcount, float* out, void* stream);

/* count[0] = number of rows with tgt != ignore_index (fp64, one block). */
int b2k_ce_valid_count(const int64_t* tgt, int64_t M, int64_t ignore_index,
                       double* count, void* stream);

/* Bytes of one rank's exchange buffer for b2k_ce_reduce_exchange_mean with
 * `world` ranks (1..32; -1 otherwise). */
int64_t b2k_ce_exchange_bytes(int world);

/* b2k_ce_reduce, the all-reduce of its [sum, count] pair across `world` ranks
 * and b2k_ce_mean in ONE kernel, the exchange over peer memory instead of a
 * collective library: peers is a DEVICE array of `world` pointers, peers[r]
 * = rank r's exchange buffer as mapped in this process (b2k_ce_exchange_alloc
 * on each rank, mapped with b2k_ipc_handle / b2k_ipc_open; zeroed before the
 * first call).  Every rank calls it once per step, in the same order.  The block
 * stores this rank's pair into every rank's buffer, publishes it with a
 * system-scope release, waits until all ranks' pairs are in its own buffer
 * (at most limit_ns of global time), and adds them in rank order (the same
 * bits on every rank).  On success sumcount = global [sum, count] and out[0]
 * = sum / count.  *status (zeroed once at set-up) is sticky: a wait that
 * runs out sets 1, a peer flag above this rank's epoch (a peer that gave up
 * waiting and stepped on) sets 2, out[0] is then NaN, and every later call
 * with a nonzero status returns NaN at once without writing to any peer.
 * Replaces ouroboros/specs.py's per-row cross-entropy (:239-241) reduced to
 * the mean over valid rows with the rows sharded across GPUs; the reference
 * has no multi-GPU path. */
int b2k_ce_reduce_exchange_mean(const float* row_loss, const int64_t* tgt, int64_t M,
                                int64_t ignore_index, void* const* peers, int rank, int world,
                                unsigned long long limit_ns, double* sumcount, float* out,
                                int* status, void* stream);

/* The exchange of b2k_ce_reduce_exchange_mean alone: global[0..1] = the sum
 * over all ranks of local[0..1] (two device doubles per rank), added in rank
 * order, through the same buffers and epoch sequence (every rank makes the
 * same sequence of exchange calls).  NaN and a sticky *status on a failure,
 * as above.  Used for the global valid count that scales the fused
 * cross-entropy gradient when the rows are sharded; no reference
 * counterpart (the reference has no multi-GPU path). */
int b2k_exchange_pair(const double* local, void* const* peers, int rank, int world,
                      unsigned long long limit_ns, double* global, int* status, void* stream);

/* Exchange-buffer plumbing (no reference counterpart): a zeroed device
 * allocation of b2k_ce_exchange_bytes(world) bytes on the current device, its
 * 64-byte CUDA IPC handle, and the mapping of a peer process's buffer from
 * its handle (plain peer access; no multicast object), each with its
 * release. */
int b2k_ce_exchange_alloc(int world, void** buf);
int b2k_ce_exchange_free(void* buf);
int b2k_ipc_handle(void* buf, void* handle64);
int b2k_ipc_open(const void* handle64, void** ptr);
int b2k_ipc_close(void* ptr);

/* Forward and backward of the reduced cross-entropy in one kernel: per-row
 * fp32 losses as b2k_cross_entropy, and the gradient of
 * grad_scale * mean-over-valid-rows(loss) w.r.t. the logits,
 *   dx[i, j] = (softmax(x[i])[j] - [j == tgt[i]]) * grad_scale / *valid_count,
 * 0 for rows with tgt == ignore_index (NaN for other out-of-range targets),
 * written in dtype with row stride ldd (dx may alias x).  The logits are read
 * from HBM once: the second pass over a row is served from L2.
 * valid_count is a device fp64 (b2k_ce_valid_count, all-reduced when rows are
 * sharded).  The gradient the reference pays for in a separate backward
 * (ouroboros/README.md:56-58 on the fused Liger kernel). */
int b2k_cross_entropy_fwd_bwd(const void* x, int64_t ldx, const int64_t* tgt, int64_t M,
                              int64_t N, int dtype, int64_t ignore_index,
                              const double* valid_count, float grad_scale, float* row_loss,
                              void* dx, int64_t ldd, void* stream);

/* Largest M accepted by b2k_cross_entropy_mean_noalloc. */
#define B2K_NOALLOC_MAX_ROWS 262144

/* Mean cross-entropy over rows whose target is not ignore_index, written to
 * out[0] (fp32, device memory), for callers that cannot allocate device
 * memory: the same result as b2k_cross_entropy(out_dtype F32) ->
 * b2k_ce_reduce -> b2k_ce_mean, but the per-row losses and the [sum, count]
 * pair live in a fixed buffer inside the library (1 MiB + 256 B on every GPU
 * that loads it), so the caller passes only inputs and the output and
 * nothing is allocated.  M above B2K_NOALLOC_MAX_ROWS is rejected with
 * B2K_EINVAL.  The first call on a device looks up the buffer's device
 * address (make it before any stream capture) and keeps it: after a
 * cudaDeviceReset of that device the cached address is stale, so do not call
 * this entry point there again.  Calls whose GPU work overlaps share the
 * buffer and race.  No counterpart in the reference: its kernels allocate
 * their outputs through PyTorch. */
int b2k_cross_entropy_mean_noalloc(const void* x, int64_t ldx, const int64_t* tgt,
                                   int64_t M, int64_t N, int dtype,
                                   int64_t ignore_index, float* out, void* stream);

/* Row-wise inclusive prefix sum, fp64 carry, output in dtype.
 * Replaces cumsum (specs.py:840-849, reference :245-248). */
int b2k_cumsum(const void* x, int64_t ldx, void* y, int64_t ldy, int64_t M,
               int64_t N, int dtype, void* stream);

/* Per-row Shannon entropy of softmax(x), (M,) in dtype.
 * Replaces entropy (specs.py:850-859, reference :251-256). */
int b2k_entropy(const void* x, int64_t ldx, void* out, int64_t M, int64_t N,
                int dtype, void* stream);

/* Per-row KL(softmax(x) || softmax(y)), (M,) in dtype.
 * Replaces kl_div (specs.py:860-864, reference :259-265). */
int b2k_kl_div(const void* x, int64_t ldx, const void* y, int64_t ldy,
               void* out, int64_t M, int64_t N, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200K_H */
