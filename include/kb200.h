/*
 * kb200.h -- C ABI of the B200 (sm_100a) implementation of the Kairos
 * hybrid-attention hot path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches asynchronously on that stream, never
 * synchronises the host, and returns 0 on success or a KB200_ERR_* code.
 * kb200_last_error() returns a human-readable message for the last failure
 * on the calling thread.  No entry point allocates device memory: callers
 * pass any scratch they need as a workspace pointer sized by the matching
 * *_workspace_size() query.
 *
 * Layouts follow the reference's PyTorch operators ("head-last", contiguous):
 *   q, k  [B*T, H, K]  bf16        v  [B*T, H, V] bf16
 *   g     [B*T, H]     fp32 (log-space decay)   beta [B*T, H] bf16
 *   states [N, H, K, V] fp32
 */
#ifndef KB200_H
#define KB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  KB200_OK = 0,
  KB200_ERR_INVALID = 1,     /* bad shape / null pointer / unsupported dims   */
  KB200_ERR_ALIGN = 2,       /* pointer not 16-byte aligned                   */
  KB200_ERR_WORKSPACE = 3,   /* workspace missing or too small                */
  KB200_ERR_LAUNCH = 4,      /* CUDA launch error                             */
  KB200_ERR_TIMEOUT = 5      /* a bounded device-side wait gave up            */
};

/* ABI version; bumped on any signature change. */
int kb200_abi_version(void);
/* Message for the last error returned on this thread ("" if none). */
const char* kb200_last_error(void);

/* ---------------------------------------------------------------------
 * Gated delta rule, chunked forward (chunk size 64).
 * Replaces chunk_gated_delta_rule / chunk_gated_delta_rule_fwd:
 *   kairos/third_party/fla/ops/gated_delta_rule/chunk.py:216-323 (public op)
 *   kairos/third_party/fla/ops/gated_delta_rule/chunk.py:16-67  (pipeline)
 * with use_qk_l2norm_in_kernel handled in-kernel (chunk.py:166-168).
 * --------------------------------------------------------------------- */
typedef struct KB200GdnArgs {
  const void* q;            /* [B*T, H, K] bf16                                 */
  const void* k;            /* [B*T, H, K] bf16                                 */
  const void* v;            /* [B*T, H, V] bf16                                 */
  const float* g;           /* [B*T, H] fp32 log decay                          */
  const void* beta;         /* [B*T, H] bf16                                    */
  const float* initial_state; /* [N, H, K, V] fp32 or NULL                      */
  void* o;                  /* out [B*T, H, V] bf16                             */
  float* final_state;       /* out [N, H, K, V] fp32 or NULL                    */
  const int32_t* cu_seqlens;  /* device [N+1] or NULL (then N = B, length T)    */
  const int32_t* chunk_indices; /* device [num_chunks, 2] (seq, chunk) or NULL  */
  const int32_t* chunk_offsets; /* device [N+1] first chunk of each seq or NULL */
  int64_t B, T, H, K, V;    /* T = tokens per sequence (B*T = total tokens)     */
  int64_t N;                /* number of sequences (B, or len(cu_seqlens)-1)    */
  int64_t num_chunks;       /* total 64-token chunks over all sequences         */
  float scale;              /* output scale (reference default K^-1/2)          */
  int use_qk_l2norm;        /* 1: L2-normalise q and k inside the op            */
} KB200GdnArgs;

/* Bytes of workspace kb200_gdn_chunk_fwd needs for these arguments. */
size_t kb200_gdn_workspace_size(const KB200GdnArgs* a);

/* Kernel launches kb200_gdn_chunk_fwd makes for these arguments (3, or 5 when the
 * state pass is split into concurrent segments), -1 for invalid arguments.  A
 * query for launch accounting; no counterpart in the reference. */
int kb200_gdn_launch_count(const KB200GdnArgs* a);
/* Launch the forward.  `workspace` must be 256-byte aligned. */
int kb200_gdn_chunk_fwd(const KB200GdnArgs* a, void* workspace, size_t workspace_bytes,
                        void* stream);
/* Sliding-window attention: query i attends keys i - window_left .. i + window_right
 * (a negative bound means unbounded), the window_size = (left, right) of the
 * reference's flash_attention call (kairos/modules/dits/kairos_dit.py:232-277, used by
 * SelfAttention with window_size / dilated_length, :423-507).  Key tiles entirely
 * outside the window of a 256-query block are skipped.  Same other arguments as
 * kb200_attn_fp8_fwd / _attend; _attend_window follows a _quantize. */
int kb200_attn_fp8_fwd_window(const void* q, const void* k, const void* v, void* o, int64_t B,
                              int64_t S, int64_t H, int64_t D, int64_t row_stride, float softmax_scale,
                              void* workspace, size_t workspace_bytes, void* stream, int64_t window_left,
                              int64_t window_right);
int kb200_attn_fp8_attend_window(const void* q, const void* k, const void* v, void* o, int64_t B,
                                 int64_t S, int64_t H, int64_t D, int64_t row_stride, float softmax_scale,
                                 void* workspace, size_t workspace_bytes, void* stream, int64_t window_left,
                                 int64_t window_right);
/* Synchronises `stream` and reports KB200_ERR_TIMEOUT if a bounded device-side
 * wait of the last kb200_gdn_chunk_fwd on `workspace` gave up (the kernels then
 * record the site, let their copies in flight land and stop instead of hanging;
 * later chunks' outputs are left unwritten).  No counterpart in the reference. */
int kb200_gdn_status(const void* workspace, void* stream);

/* Allocation-free variant of kb200_gdn_chunk_fwd (no counterpart in the
 * reference).  For callers that cannot allocate device memory when they run
 * the operator (a plugin host that owns all device memory, code in a host
 * callback): the scratch comes from a 64 MiB array compiled into this
 * library, which every GPU that loads the library keeps until process exit.
 * Problems needing more scratch than kb200_gdn_noalloc_scratch_bytes()
 * are rejected with KB200_ERR_WORKSPACE.  Every call looks up the array's
 * device address (cudaGetSymbolAddress) on the current device; make the first
 * call on a device before any stream capture (it may initialise the module).  All calls share
 * the one array: calls that overlap on the GPU (different streams, or
 * different threads on one device) race and must be serialised by the caller.
 * The array's device address is looked up on every call, so the entry point
 * stays valid after cudaDeviceReset (the array's contents do not survive it).
 * Nothing in the array needs to start at zero, so stale contents from an
 * earlier call do not matter.  Makes no cudaMalloc/cudaFree call. */
size_t kb200_gdn_noalloc_scratch_bytes(void);
int kb200_gdn_chunk_fwd_noalloc(const KB200GdnArgs* a, void* stream);

/* ---------------------------------------------------------------------
 * Attention prologue: y = RoPE(bf16(RMSNorm(x) * weight)) for each token row.
 * Replaces SelfAttention.forward's q/k path (kairos/modules/dits/kairos_dit.py:452-456):
 * FusedRMSNorm over the full `dim` channels (eps, weight [dim] fp32 or NULL)
 * then rope_apply (kairos_dit.py:324-329): per head of `head_dim` channels, pair
 * (2j, 2j+1) -> complex product with (cos, sin) = cos_sin[row][j] ([rows,
 * head_dim/2, 2] fp32).  Channel c of a row lives at
 *   base + (h / heads_per_block) * block_stride + row * ld + (h % heads_per_block) * head_dim + c % head_dim,
 * h = c / head_dim (heads_per_block = dim / head_dim for a plain [rows, ld] matrix),
 * so q/k can be normalised in place inside a destination-grouped projection.
 * x == y is allowed.  cos_sin == NULL skips the rotation (plain FusedRMSNorm, as
 * CrossAttention.forward's norm_q / norm_k, kairos_dit.py:687-688).
 * --------------------------------------------------------------------- */
int kb200_rmsnorm_rope(const void* x, void* y, int64_t rows, int64_t dim, int64_t head_dim, int64_t ld,
                       int64_t heads_per_block, int64_t block_stride, const float* weight,
                       const float* cos_sin, float eps, void* stream);

/* ---------------------------------------------------------------------
 * Softmax attention with FP8-e4m3 Q/K (per-(batch, head) amax scaling,
 * scale = amax/448), fp32 scores and softmax, bf16 probabilities times the
 * bf16 V for the P.V product (fp32 accumulation), bf16 output.
 * Replaces the attention core called by AttentionModule.forward
 *   kairos/modules/dits/kairos_dit.py:367-373 (module)
 *   kairos/modules/dits/kairos_dit.py:232-277 (flash_attention dispatcher;
 *   non-causal, no mask, softmax scale D^-1/2 as in F.scaled_dot_product_attention)
 * q, k, v: [B, S, H*D] bf16 rows, `row_stride` elements apart (0 = H*D, i.e.
 * contiguous; larger when q/k/v are column slices of one fused projection);
 * o: [B, S, H*D] bf16 contiguous; D = 128.
 * Cosine similarity to the bf16 reference ~0.9992 on N(0,1) inputs (e4m3 P
 * and V as well would bound it near 0.9986).
 * --------------------------------------------------------------------- */
size_t kb200_attn_fp8_workspace_size(int64_t B, int64_t S, int64_t H, int64_t D);
int kb200_attn_fp8_fwd(const void* q, const void* k, const void* v, void* o, int64_t B, int64_t S,
                       int64_t H, int64_t D, int64_t row_stride, float softmax_scale,
                       void* workspace, size_t workspace_bytes, void* stream);
/* The two halves of kb200_attn_fp8_fwd, for callers that time or overlap them
 * separately: _quantize fills the workspace (amax, e4m3 q/k, bf16 v^T, row
 * norms), _attend reads it and writes o.  Same arguments; _attend must follow a
 * _quantize of the same inputs into the same workspace on the same stream. */
int kb200_attn_fp8_quantize(const void* q, const void* k, const void* v, void* o, int64_t B,
                            int64_t S, int64_t H, int64_t D, int64_t row_stride,
                            float softmax_scale, void* workspace, size_t workspace_bytes, void* stream);
int kb200_attn_fp8_attend(const void* q, const void* k, const void* v, void* o, int64_t B,
                          int64_t S, int64_t H, int64_t D, int64_t row_stride, float softmax_scale,
                          void* workspace, size_t workspace_bytes, void* stream);
/* Synchronises `stream` and reports KB200_ERR_TIMEOUT if a bounded device-side
 * wait of the last attention launch on `workspace` gave up (the kernel then
 * skipped its remaining work instead of hanging). */
int kb200_attn_fp8_status(const void* workspace, int64_t B, int64_t S, int64_t H, void* stream);

/* ---------------------------------------------------------------------
 * GatedDeltaNet prologue in one launch: short causal depthwise convolutions
 * + SiLU for q, k, v and the beta / g gates.
 * Replaces (kairos/third_party/fla/layers/gated_deltanet.py):
 *   :238-255  ShortConvolution q/k/v (causal_conv1d_fwd, fla/modules/convolution.py:410)
 *   :267-271  beta = sigmoid(b_proj(x)) (x2 if allow_neg_eigval);
 *             g = -exp(A_log) * softplus(a_proj(x) + dt_bias), fp32
 * Inputs are the projection outputs (rows of B*T tokens, row strides ld* in
 * elements, so q/k/v may be column slices of one fused projection).
 * --------------------------------------------------------------------- */
typedef struct KB200GdnPrologueArgs {
  const void* xq; const void* xk; const void* xv;   /* bf16 [B*T, C] rows, stride ld*       */
  int64_t ldq, ldk, ldv;
  const float* wq; const float* wk; const float* wv; /* conv weights [C, W] fp32            */
  const float* bq; const float* bk; const float* bv; /* conv bias [C] or NULL               */
  void* q; void* k; void* v;                         /* out bf16 [B*T, C] contiguous         */
  const void* a; const void* b;                      /* bf16 [B*T, H] rows, strides lda/ldb  */
  int64_t lda, ldb;
  const float* A_log; const float* dt_bias;          /* [H] fp32                             */
  float* g;                                          /* out [B*T, H] fp32                    */
  void* beta;                                        /* out [B*T, H] bf16                    */
  int64_t B, T, H, Cqk, Cv;
  int W;                                             /* conv width, 1..4                     */
  int allow_neg_eigval;
  /* Conv states carried from the previous piece of the sequence (ShortConvolution's
   * `cache`, fla/modules/convolution.py:801-853): bf16 [B, C, W], column W-1 the
   * input just before token 0, column W-1-j the one j tokens earlier; NULL = zeros
   * (sequence start).  The new state (the last W inputs) is the caller's to form. */
  const void* cache_q; const void* cache_k; const void* cache_v;
} KB200GdnPrologueArgs;
int kb200_gdn_prologue(const KB200GdnPrologueArgs* a, void* stream);

/* ---------------------------------------------------------------------
 * Gated RMSNorm epilogue: y = x * rsqrt(mean(x^2) + eps) * weight * silu(gate)
 * per row of D channels.  Replaces FusedRMSNormGated.forward with
 * activation 'swish' (kairos/third_party/fla/modules/fused_norm_gate.py:1024-1085,
 * kernel :60-110) as called at gated_deltanet.py:309-311.
 * x, y: [rows, D] bf16 with rows = tokens * heads; gate: bf16, row (token) stride
 * ld_gate elements, head h at column h*D; weight: [D] fp32.
 * --------------------------------------------------------------------- */
int kb200_rmsnorm_gated(const void* x, const void* gate, const float* weight, void* y,
                        int64_t rows, int64_t heads, int64_t D, int64_t ld_gate, float eps,
                        void* stream);

/* ---------------------------------------------------------------------
 * DiT norm sites: residual add, LayerNorm, modulation in one pass.
 *   x <- bf16(x + gate * r)         when r != NULL (gate [dim] fp32, NULL = 1):
 *                                   GateModule.forward / x.add_ (kairos_dit.py:700-701, 929-931, 968)
 *   y  = bf16(LN(x) * m + a)        LayerNorm without affine, eps, then
 *                                   m = mul_plus_one ? 1 + mul : mul (NULL: 1), a = add (NULL: 0):
 *                                   modulate(norm(x), shift, scale) (kairos_dit.py:306-309, 873-874, 955-957),
 *                                   the affine cross_attn_norm (mul = weight, add = bias, :797, 931)
 *                                   and Head.forward (:1047-1052)
 * x, y: [rows, dim] bf16 contiguous (y must not alias x); r: row stride ld_r.
 * --------------------------------------------------------------------- */
int kb200_residual_ln_mod(void* x, const void* r, int64_t rows, int64_t dim, int64_t ld_r,
                          const float* gate, const float* mul, const float* add, int mul_plus_one,
                          float eps, void* y, void* stream);

/* ---------------------------------------------------------------------
 * Failure-path test hooks (no counterpart in the reference).
 * kb200_wait_probe: one CTA waits on an mbarrier nothing arrives on, with the
 * bounded wait every kernel here uses and a budget of `budget_cycles` SM
 * clocks (<= 4e9), then records site 99 in the device int `err_word` (zeroed
 * first) -- the error path of a wait that runs out, with nothing in flight.
 * kb200_read_error_word: synchronises `stream`, returns KB200_ERR_TIMEOUT if
 * `err_word` holds a site code, KB200_OK if it is 0.
 * --------------------------------------------------------------------- */
int kb200_wait_probe(void* err_word, int64_t budget_cycles, void* stream);
int kb200_read_error_word(const void* err_word, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* KB200_H */
