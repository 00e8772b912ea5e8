/*
 * specb200.h - C ABI of the B200 speculative-decoding engine (libspecb200.so).
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream passed as
 * `void*` (a cudaStream_t; NULL is the legacy default stream). Calls are asynchronous
 * and stream-ordered; they allocate no device memory. Scratch memory ("workspace") is
 * passed in by the caller, sized by the matching *_workspace_bytes() query, and must be
 * zero-filled once before its first use: the kernels return every counter in it to zero
 * before they finish, so a workspace can be reused (and captured in a CUDA graph) without
 * another memset. Two calls that run at the same time on the GPU must not share a
 * workspace.
 *
 * Return value: SPECB200_OK or one of the error codes below, for errors found on the host
 * before launch. Errors found by a kernel (a drafted token with zero draft probability, a
 * token id out of range, a wait that gave up) are written to the caller's device status
 * word and read back by the caller after the stream has reached that point.
 *
 * Each function names the reference code it replaces (beriltatli/speculative-decoder,
 * paths relative to that project's root).
 */
#ifndef SPECB200_H
#define SPECB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------------------- */
#define SPECB200_OK 0
#define SPECB200_ERR_ARG 1          /* bad shape, size, null pointer or alignment        */
#define SPECB200_ERR_RANGE 2        /* token id or slot out of range                     */
#define SPECB200_ERR_ZERO_Q 3       /* drafted token has zero draft probability          */
#define SPECB200_ERR_CUDA 4         /* a CUDA runtime call failed                        */
#define SPECB200_ERR_TIMEOUT 5      /* a bounded device-side wait gave up                */
#define SPECB200_ERR_UNSUPPORTED 6  /* model shape or dtype the kernels do not handle    */
#define SPECB200_ERR_WORKSPACE 7    /* workspace smaller than the *_workspace_bytes size, or (accept) not zero-filled */

/* ---- element types ------------------------------------------------------------------ */
#define SPECB200_F32 0
#define SPECB200_BF16 1

/* Library version (major*10000 + minor*100 + patch) and the text of the last host-side
 * error raised on the calling thread. */
int specb200_version(void);
const char* specb200_last_error(void);

/* Failure-path check of the bounded device waits (no reference counterpart; the reference has
 * no device code): one kernel thread waits, with the helper every pipeline uses for its
 * mbarrier waits, on a barrier phase that never completes. After the spin limit (~2 s) it
 * records SPECB200_ERR_TIMEOUT in *status and writes 1 to *gave_up (2 if the wait gave up
 * without raising the abort flag, 0 if it returned). Both are device int32 words; nothing else
 * is in flight, so the context stays usable. Stream-ordered. */
int specb200_wait_probe(int32_t* status, int32_t* gave_up, void* stream);

/* ======================================================================================
 * K8/K10: fused accept-reject and sampling
 *   replaces spec/accept.py:44-79 (accept_reject), spec/accept.py:18-26
 *   (residual_distribution), spec/accept.py:29-35 (sample_inverse_cdf) and
 *   lm/sampling.py:13-18 (probabilities), fused into one launch.
 * ====================================================================================== */

/* p: [B, k+1, V] fp32 target rows. q: [B, k, V] fp32 draft rows, or NULL with
 * SPECB200_ACCEPT_Q_ONEHOT (q is the one-hot of the drafted token, as NGramDraft's is).
 * With SPECB200_ACCEPT_LOGITS both are logits and are turned into softmax(x / temperature)
 * on the fly; temperature 0 is greedy (one-hot of the first maximum). Without it they are
 * probabilities and `temperature` is ignored.
 * draft: [B, k] int64. u_accept: [B, k] fp32, u_residual: [B] fp32, uniforms in [0, 1).
 * Outputs n_accepted [B] and next_token [B], int64. k = 0 samples one token per row from
 * p[:, 0] (the first-token / plain-decode sampler). With SPECB200_ACCEPT_DECIDE_ONLY only
 * n_accepted is written. status: device int32, set to a SPECB200_ERR_* code by the kernel
 * (zero draft mass, draft id out of range); the call clears it first.
 * workspace: specb200_accept_workspace_bytes(B, k) bytes, zero-filled before its first use
 * (the kernel's work queue and tickets start at zero and every call leaves them at zero), and
 * used by one call at a time. */
#define SPECB200_ACCEPT_LOGITS 1
#define SPECB200_ACCEPT_Q_ONEHOT 2
#define SPECB200_ACCEPT_DECIDE_ONLY 4
#define SPECB200_ACCEPT_Q_STEP_MAJOR 8   /* q is laid out [k, B, V] (one draft step per block) */
size_t specb200_accept_workspace_bytes(int B, int k);
int specb200_accept(const float* p, const float* q, const int64_t* draft, const float* u_accept,
                    const float* u_residual, int B, int k, int V, int flags, float temperature,
                    int64_t* n_accepted, int64_t* next_token, int32_t* status, void* workspace,
                    size_t workspace_bytes, void* stream);

/* Allocation-free variant of specb200_accept (no counterpart in the reference): same
 * arguments and results, minus the workspace. For callers that cannot allocate device memory
 * or hold a scratch buffer for this library (a runtime that reserves all HBM up front and
 * forbids later cudaMalloc, or an operator interface that passes only inputs and outputs).
 * Its scratch is a fixed device array inside the library (about 600 KB per GPU, held until
 * exit), so B is limited to specb200_accept_noalloc_max_rows() (512) and k to 15; larger
 * calls return SPECB200_ERR_ARG. The first call on each device looks up the array's device
 * address with that device current: make it before any stream capture. Every call shares the
 * array: calls that overlap on the GPU race, so serialise them (one stream per process). */
size_t specb200_accept_noalloc_max_rows(void);
int specb200_accept_noalloc(const float* p, const float* q, const int64_t* draft, const float* u_accept,
                            const float* u_residual, int B, int k, int V, int flags, float temperature,
                            int64_t* n_accepted, int64_t* next_token, int32_t* status, void* stream);

/* probabilities() of lm/sampling.py:13-18 written out as rows: out[r] = one-hot of the first
 * maximum of logits[r] at temperature 0, else softmax(logits[r] / temperature). [rows, V]. */
int specb200_probabilities(const float* logits, int rows, int V, float temperature, float* out, void* stream);

/* ======================================================================================
 * K9: n-gram prompt lookup
 *   replaces spec/ngram.py:32-45 (lookup) and the draft half of spec/ngram.py:19-23.
 * ====================================================================================== */

/* ctx: [B, ctx_stride] int32 token ids, row b holding ctx_len[b] (>= 1) tokens.
 * draft: [B, k] int64 out. For n = min(max_n, len-1) .. 1 the most recent earlier
 * occurrence of the last n tokens wins; its continuation is copied forward, reading its
 * own output past the end of the context; with no match the last token repeats. max_n
 * must be in [1, 8]. status: as for specb200_accept (a row of length 0 sets RANGE). */
int specb200_ngram(const int32_t* ctx, int64_t ctx_stride, const int32_t* ctx_len, int B, int k,
                   int max_n, int64_t* draft, int32_t* status, void* stream);

/* ======================================================================================
 * Device-resident context bookkeeping for the round driver
 *   replaces the context/output list updates of spec/loop.py:79-88.
 * ====================================================================================== */

/* After an accept: ctx[b, len[b] + j] = draft[b, j] for j < n_accepted[b], then
 * ctx[b, len[b] + n] = next_token[b], len[b] += n + 1 (rows with active[b] == 0 are left
 * alone; active may be NULL). Writes never pass ctx_stride. */
int specb200_commit_tokens(int32_t* ctx, int64_t ctx_stride, int32_t* ctx_len, const int64_t* draft,
                           const int64_t* n_accepted, const int64_t* next_token, const int32_t* active,
                           int B, int k, void* stream);

/* ids[b, 0] = ctx[b, len[b]-1], ids[b, 1+j] = draft[b, j]: the (k+1)-token verify input of
 * spec/verify.py:26-27, built on the device. When given, past[b] = len[b] - 1 (the cache
 * invariant spec/verify.py:23-25 asserts) and n_new[b] = k + 1, or 0 for rows whose active
 * flag is 0 (active may be NULL: all rows active). */
int specb200_verify_ids(const int32_t* ctx, int64_t ctx_stride, const int32_t* ctx_len,
                        const int64_t* draft, const int32_t* active, int B, int k, int32_t* ids,
                        int32_t* past, int32_t* n_new, void* stream);

/* draft[b, j] = tokens[b] (draft [B, k], may be NULL) and ids[b] = tokens[b] as int32 (may be
 * NULL): hands one draft step's sampled token to the next draft step and to the verify input
 * (the token loop of spec/draft.py:50-55). */
int specb200_scatter_tokens(const int64_t* tokens, int B, int k, int j, int64_t* draft, int32_t* ids,
                            void* stream);

/* ======================================================================================
 * Seeded logit noise for the noisy-copy drafter (BASELINE config 2's second variant: the
 * target itself as the draft with N(0, sigma^2) added to its final logits). No counterpart
 * in the reference, which has no such drafter.
 * ====================================================================================== */

/* logits[b, v] += sigma * z(seed, row_id[b], past[b] + n_new[b], v) for every row with
 * n_new[b] > 0 (n_new NULL: every row, as if 1; past NULL: 0; row_id NULL: b). z is a
 * standard normal by Box-Muller from Philox4x32-10 at counter (v, position, row id, 0) and key
 * (seed low, seed high 32 bits); the position is that of the token the logits predict.
 * logits: [B, ld] fp32 device rows, ld >= V. */
int specb200_logit_noise(float* logits, int B, int V, int64_t ld, const int32_t* past, const int32_t* n_new,
                         const int32_t* row_id, uint64_t seed, float sigma, void* stream);

/* ======================================================================================
 * Llama verify / decode / prefill forward
 *   replaces lm/forward.py:21-68 (forward) and lm/forward.py:71-84 (logits), with
 *   cache/kv.py:79-112 (append's slot maps, write, gather) done inside the kernels:
 *   K1 embed gather, K2 RMSNorm, K3 QKV GEMM + RoPE + paged KV write, K4 paged
 *   attention, K5 O-proj + residual, K6 gate/up + SiLU*mul and down + residual,
 *   K7 fp32-accumulated LM head.
 * ====================================================================================== */

typedef struct specb200_model_config {
  int n_layers;
  int hidden;         /* H                                                       */
  int n_heads;        /* query heads Hq                                          */
  int n_kv_heads;     /* key/value heads Hkv (Hq % Hkv == 0)                      */
  int head_dim;       /* d: 16, 32 or 64                                         */
  int intermediate;   /* I (multiple of 64)                                      */
  int vocab;          /* V                                                       */
  float rms_eps;
  int dtype;          /* SPECB200_F32 or SPECB200_BF16: weights, activations, KV */
  int max_positions;  /* rows of the RoPE tables                                 */
} specb200_model_config;

typedef struct specb200_layer_weights {
  const void* attn_norm;  /* [H]                                                    */
  const void* w_qkv;      /* [(Hq + 2 Hkv) d, H]: q_proj, k_proj, v_proj rows       */
  const void* w_o;        /* [H, Hq d]                                              */
  const void* mlp_norm;   /* [H]                                                    */
  const void* w_gate_up;  /* [2 I, H]: 64-row groups, gate rows 64g.. then up rows  */
  const void* w_down;     /* [H, I]                                                 */
} specb200_layer_weights;

typedef struct specb200_model_weights {
  const void* embed;        /* [V, H]                                            */
  const void* final_norm;   /* [H]                                               */
  const void* lm_head;      /* [V, H] (the embedding when tied)                  */
  const float* rope_cos;    /* [max_positions, d/2] fp32, cos(pos * inv_freq)    */
  const float* rope_sin;    /* [max_positions, d/2] fp32                         */
  const specb200_layer_weights* layers; /* host array of n_layers entries          */
} specb200_model_weights;

/* Builds the host-side model handle: shapes, the weight pointers and one TMA descriptor
 * per weight matrix. Holds no device memory; the weights must outlive it. */
int specb200_model_create(const specb200_model_config* config, const specb200_model_weights* weights,
                          void** handle);
int specb200_model_destroy(void* handle);

typedef struct specb200_batch {
  int B;                        /* rows (sequences)                                       */
  int T;                        /* padded tokens per row                                  */
  const int32_t* input_ids;     /* [B, T] device                                          */
  const int32_t* n_new;         /* [B] device: real tokens in row b, 1..T                 */
  const int32_t* past_len;      /* [B] device: cached positions before this call          */
  const int32_t* block_table;   /* [B, table_stride] device: pool block of each position  */
  int table_stride;
  int block_size;
  int num_slots;                /* pool entries: num_blocks * block_size                  */
  void* k_pool;                 /* [n_layers, num_slots, Hkv, d], model dtype             */
  void* v_pool;
  int last_only;                /* 1: logits of each row's last real token, [B, V]         */
  float* logits;                /* fp32 [B*T, V] or [B, V]                                */
  int max_kv_len;               /* >= past_len[b] + n_new[b] for every row                */
  int32_t* status;              /* device int32 status word (cleared by the call)         */
  uint64_t* trace;              /* NULL, or globaltimer stamps (profiling only): the        */
                                /* GEMV schedule writes                                     */
                                /* [4 n_layers + 1 launches][296 CTAs][8]: entry,           */
                                /* wait return, inputs staged, weights landed, end; the    */
                                /* per-layer schedule [4 n_layers + 1 GEMMs][512][8]; both */
                                /* followed by the attention launches [n_layers][512][8]   */
                                /* (zeroed first)                                          */
} specb200_batch;

size_t specb200_forward_workspace_bytes(void* model, int B, int T, int max_kv_len);
/* Which schedule a call with B rows of T tokens runs: 3 = decode steps of at most 4 token rows
 * of a model whose layer weights fit on chip, on the GEMV kernels with the norms folded in
 * (2 + 5 n_layers launches, 3 + 5 n_layers with a tensor-core LM head), 0 = one kernel per
 * layer op (3 + 7 n_layers launches). No reference counterpart. */
int specb200_forward_schedule(void* model, int B, int T);

/* Kernel launches one forward call with B rows of T tokens makes (no reference counterpart;
 * used to count launches). */
int specb200_forward_launches(void* model, int B, int T);
int specb200_forward(void* model, const specb200_batch* batch, void* workspace, size_t workspace_bytes,
                     void* stream);

/* ---- single kernels, exported for layer-by-layer parity tests ------------------------ */

/* y = weight * round(x * rsqrt(mean(x^2) + eps)) per row (LlamaRMSNorm,
 * transformers/models/llama/modeling_llama.py:62-67). x, y: [M, H]; dtype per config. */
int specb200_rmsnorm(int dtype, const void* x, const void* weight, int M, int H, float eps, void* y,
                     void* stream);

/* Y = X W^T: W [N, K], X [M, K] row-major, Y [M, N]. dtype SPECB200_BF16 runs the tcgen05
 * tensor-core kernel (fp32 accumulation), SPECB200_F32 the FFMA kernel. out_f32 selects fp32
 * or model-dtype output. Replaces nn.Linear at lm/forward.py:57-59,64 and lm/forward.py:84. */
size_t specb200_linear_workspace_bytes(int M, int N, int K);
int specb200_linear(int dtype, const void* w, const void* x, int M, int N, int K, int out_f32, void* y,
                    void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/* Paged causal attention over block tables (cache/kv.py:108-112 + the SDPA call at
 * lm/forward.py:62-63). q, out: [B*T, Hq, d]; pools for one layer: [num_slots, Hkv, d]. */
size_t specb200_attention_workspace_bytes(int B, int T, int n_heads, int n_kv_heads, int head_dim,
                                          int max_kv_len);
int specb200_attention(int dtype, const void* q, const void* k_pool, const void* v_pool,
                       const int32_t* block_table, int table_stride, int block_size,
                       const int32_t* past_len, const int32_t* n_new, int B, int T, int n_heads,
                       int n_kv_heads, int head_dim, int max_kv_len, float scale, void* out,
                       void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SPECB200_H */
