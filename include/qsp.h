/*
 * qsp.h — C ABI of the B200 (sm_100a) qwen3_5 MTP speculative-decoding step.
 *
 * Every entry point takes plain device pointers, explicit sizes/leading dimensions, a dtype
 * enum and a CUDA stream (as void*), launches asynchronously on that stream, allocates
 * nothing, and returns a status (QSP_OK == 0). On failure `qsp_last_error()` (thread-local)
 * describes the problem. Reference citations name the giapnguyen74/lollm function each entry
 * point replaces (paths relative to the project root).
 *
 * Row-major everywhere. "dtype" is the model dtype of activations and weights (QSP_F32 or
 * QSP_BF16); recurrent GDN state, softmax statistics and accumulators are always fp32.
 */
#ifndef QSP_H_
#define QSP_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QSP_OK 0
#define QSP_ERR_INVALID 1     /* bad argument: shape, pointer, alignment, range        */
#define QSP_ERR_CUDA 2        /* a CUDA runtime call or kernel launch failed            */
#define QSP_ERR_UNSUPPORTED 3 /* valid request this build does not implement            */

#define QSP_F32 0
#define QSP_BF16 1

#define QSP_ABI_VERSION 1

/* Thread-local description of the last failure on this thread. */
const char* qsp_last_error(void);
int qsp_abi_version(void);

/* ---------------------------------------------------------------- elementwise / norms */

/* out[r,:] = table[ids[r·ids_stride],:]. Replaces `embed_tokens(input_ids)`
 * (src/qwen3_5/modeling_qwen3_5.py:86). ids outside [0,vocab) are rejected on the device
 * by writing zeros and setting *bad_ids (optional, may be NULL) to 1. */
int qsp_embed(const int64_t* ids, int64_t ids_stride, int64_t rows, const void* table,
              int64_t vocab, int64_t dim, void* out, int64_t ld_out, int32_t* bad_ids,
              int dtype, void* stream);

/* y = x̂·(1+w), statistics in fp32 — RMSNorm (src/qwen3_5/blocks.py:23-35). */
int qsp_rmsnorm(const void* x, int64_t ld_x, const void* w, void* y, int64_t ld_y,
                int64_t rows, int64_t dim, float eps, int dtype, void* stream);

/* x := x + h (rounded to dtype), then y = RMSNorm(x): the residual add followed by the next
 * pre-norm (src/qwen3_5/modeling_qwen3_5.py:59-60). */
int qsp_add_rmsnorm(void* x, const void* h, const void* w, void* y, int64_t rows,
                    int64_t dim, float eps, int dtype, void* stream);

/* y = silu(gu[:, :inter]) · gu[:, inter:] — the SwiGLU middle of MLP
 * (src/qwen3_5/blocks.py:341-342) on a fused [gate | up] projection. */
int qsp_swiglu(const void* gu, int64_t ld_gu, void* y, int64_t ld_y, int64_t rows,
               int64_t inter, int dtype, void* stream);

/* ---------------------------------------------------------------- projections */

#define QSP_GEMM_ACCUMULATE 1 /* c := c + round(a·wᵀ) (residual add in the epilogue) */

/* c[m,n] = a[m,k] · w[n,k]ᵀ with fp32 accumulation: every nn.Linear of the step
 * (blocks.py:202-205, 251-260, 337-339, modeling_qwen3_5.py:73, mtp.py:52). bf16 runs on
 * tcgen05 tensor cores (TMA-fed, TMEM accumulators); fp32 (parity configs) on CUDA cores.
 * `workspace` (may be NULL, 16-byte aligned) holds split-K partials; it must not be shared by
 * two GEMMs running concurrently. With too little workspace the GEMM runs unsplit. */
int qsp_gemm(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc,
             int64_t m, int64_t n, int64_t k, int dtype, int flags, void* workspace,
             size_t workspace_bytes, void* stream);

/* x := x + round(a·wᵀ) (the residual add after o_proj / out_proj / down_proj), then
 * y = RMSNorm(x)·(1+norm_w) (the next input_layernorm / post_attention_layernorm / final
 * norm) — modeling_qwen3_5.py:59-60 + blocks.py:23-35. Split-K merges, the residual add and
 * the norm run in one pass when the GEMM splits. */
int qsp_gemm_residual_rmsnorm(const void* a, int64_t lda, const void* w, int64_t ldw, void* x,
                              int64_t ldx, const void* norm_w, void* y, int64_t ldy, int64_t m,
                              int64_t n, int64_t k, float eps, int dtype, void* workspace,
                              size_t workspace_bytes, void* stream);

/* act = silu(a·w_gateᵀ) ⊙ (a·w_upᵀ) with w_gu = [gate; up] (2·inter rows) — MLP
 * (blocks.py:341-342). gu_tmp [m, 2·inter] holds the projection when the GEMM does not split. */
int qsp_gemm_swiglu(const void* a, int64_t lda, const void* w_gu, int64_t ldw, void* act,
                    int64_t ld_act, void* gu_tmp, int64_t ld_gu, int64_t m, int64_t inter,
                    int64_t k, int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes qsp_gemm uses for this shape (0 when it never splits). */
size_t qsp_gemm_workspace_bytes(int64_t m, int64_t n, int64_t k, int dtype);

/* Device status codes (qsp_device_status). 1xx-3xx: a kernel's bounded mbarrier wait ran out
 * (GEMM, GDN, attention, MoE, cluster GEMM) and the kernel returned instead of hanging. */
#define QSP_DEV_BAD_ACCEPT 401  /* qsp_cache_accept got an accepted count outside [0, T-1]
                                   (clamped into range)                                      */
#define QSP_DEV_NAN_LOGITS 501  /* a sampler or argmax row held a NaN logit (argmax then
                                   picks the first NaN, as torch.argmax does)                */
#define QSP_DEV_WAIT_PROBE 901  /* qsp_wait_probe's wait ran out (its expected outcome)      */

/* Device status: the first nonzero code recorded by any kernel since the last reset, else 0.
 * Synchronous; `reset` clears it. The "hard-fail, never guess" checks of the reference
 * (src/qwen3_5/weights.py:57-62) have no device side; this is where device-side failures
 * surface for the host to raise. */
int qsp_device_status(int32_t* code, int32_t reset);

/* Failure-detection probe (test support, no reference counterpart): one CTA waits on an
 * mbarrier that is never signalled, through the same bounded wait as the tensor-core kernels
 * but with a limit of `polls` polls (the kernels use 2^24, about a second). When it runs out
 * the kernel records QSP_DEV_WAIT_PROBE and returns; `waited_ns` (device, may be NULL)
 * receives how long it waited. polls in [1, 2^24]. */
int qsp_wait_probe(uint32_t polls, uint32_t* waited_ns, void* stream);

/* ---------------------------------------------------------------- Gated DeltaNet */

/*
 * One GDN layer's token mixer core over T tokens per sequence, fused: causal depthwise
 * conv + SiLU over cat(q,k,v) (GatedDeltaNet._conv, blocks.py:268-286), head split and
 * v_per_k expansion, β = σ(b), g = −exp(A_log)·softplus(a+dt_bias) (blocks.py:297-314),
 * l2-normalised q,k and the recurrent gated delta rule (blocks.py:116-144), then
 * RMSNormGated(core, z) (blocks.py:38-51, 324). Output feeds out_proj.
 *
 * Deferred commit (rollback by index): in speculative mode the kernel does NOT write the
 * state after the T tokens. It stores each token's prepared q̂, k̂, v, g, β and Gram products
 * in the token ring `pending` and the raw conv inputs in `conv_hist`; the NEXT call first
 * replays the `replay_n[b]` kept tokens onto the stored state (same arithmetic, so the
 * result is bit-identical to having run only those tokens) and reads its conv window at row
 * `conv_off[b]`. Commit-all mode (speculative == 0, any T) writes the final state and window
 * directly.
 *
 * Buffers (per layer):
 *   proj       [B*T, ld_proj]           cols [0,C): raw qkv, [C,C+Vd): z, then b [Hv], a [Hv]
 *   state      [B, Hv, dk, dv] fp32     (same layout as the reference's recurrent_state)
 *   conv_hist  [2, B, K-1+Ts, C] dtype  ping-pong on *parity
 *   pending    token ring, qsp_gdn_pending_bytes(...) bytes (two parity halves of
 *              [B, Ts] rows; the layout is private to the library)
 *   out        [B*T, ld_out]            cols [0, Vd)
 * with C = 2·Hk·dk + Hv·dv (conv_dim), Vd = Hv·dv, Ts = max_spec_tokens ≤ 8, conv kernel ≤ 4;
 * proj, state, pending, conv_hist and conv_w 16-byte aligned, ld_proj a multiple of 16 bytes.
 */
typedef struct qsp_gdn_layer {
  int32_t batch, tokens;
  int32_t n_k_heads, n_v_heads, head_k, head_v, conv_kernel;
  int32_t max_spec_tokens;
  int32_t speculative;
  int32_t dtype;
  float eps;
  const void* proj;
  int64_t ld_proj;
  const void* conv_w;     /* [C, K]   (conv1d.weight squeezed) */
  const void* a_log;      /* [Hv]     */
  const void* dt_bias;    /* [Hv]     */
  const void* norm_w;     /* [dv]     */
  float* state;
  void* conv_hist;
  void* pending;
  const int32_t* replay_n; /* [B] */
  const int32_t* conv_off; /* [B] */
  const int32_t* parity;   /* [1] */
  void* out;
  int64_t ld_out;
} qsp_gdn_layer;

int qsp_gdn_verify(const qsp_gdn_layer* layer, void* stream);

/* Bytes of the `pending` token ring of one GDN layer (0 for invalid sizes). It replaces the
 * reference's cache clone + recompute on rejection (mtp.py:141,156-162), which keeps no
 * per-token buffer. */
size_t qsp_gdn_pending_bytes(int32_t batch, int32_t n_k_heads, int32_t n_v_heads, int32_t head_k,
                             int32_t head_v, int32_t max_spec_tokens, int32_t dtype);

/* ---------------------------------------------------------------- gated attention */

/*
 * Paged KV cache: k_pages/v_pages [num_pages, n_kv, page_size, head_dim] (dtype);
 * page_table [B, max_pages] int32; seq_lens [B] = committed tokens before this call. The
 * T new tokens of sequence b sit at positions seq_lens[b] + t.
 *
 * qkv row layout (one row per token, b-major): per q head h: [q (hd) | gate (hd)], then
 * k (n_kv·hd), then v (n_kv·hd) — q_proj / k_proj / v_proj stacked (blocks.py:202-205,
 * 214-220).
 */
typedef struct qsp_attn_layer {
  int32_t batch, tokens;
  int32_t n_heads, n_kv_heads, head_dim, rotary_dim;
  int32_t page_size, max_pages, num_pages;
  int32_t dtype;
  float eps, scale;
  const void* qkv;
  int64_t ld_qkv;
  const void* q_norm_w;   /* [hd] */
  const void* k_norm_w;   /* [hd] */
  const void* rope_cos;   /* [rope_rows, rotary_dim] dtype (RoPE.cos_sin table) */
  const void* rope_sin;
  int32_t rope_rows;
  void* k_pages;
  void* v_pages;
  const int32_t* page_table;
  const int32_t* seq_lens;
  void* q_buf;            /* [B*T, n_heads, hd] workspace: normed + rotated q */
  void* out;              /* [B*T, ld_out] gated attention output (o_proj input) */
  int64_t ld_out;
  float* partial;         /* split-KV workspace (qsp_attn_workspace_bytes) */
  int32_t num_splits;     /* key splits per (sequence, kv head); 0 = choose */
  int32_t* bad_index;     /* optional [1]: set to 1 if a page index was out of range */
} qsp_attn_layer;

/* QK-norm + partial RoPE on q and k, append k,v into the pages
 * (blocks.py:218-227, kv.py:26-33 append_kv). */
int qsp_attn_prep(const qsp_attn_layer* layer, void* stream);

/* Offset-causal GQA attention of the T new queries over seq_lens[b]+T keys, split over
 * the key axis and merged, times σ(gate) (attention.py:43-51, 84-91; _triton_attn.py
 * kv_fwd_kernel; blocks.py:229-235). */
int qsp_attn_verify(const qsp_attn_layer* layer, void* stream);

/* Bytes of `partial` workspace needed by qsp_attn_verify for this shape and split count. */
size_t qsp_attn_workspace_bytes(int32_t batch, int32_t tokens, int32_t n_heads,
                                int32_t head_dim, int32_t num_splits);

/* qsp_attn_verify with the split-KV partials placed in a scratch region that the library
 * reserves statically on each device (QSP_ATTN_STATIC_SCRATCH_BYTES), so the call itself
 * allocates no device memory; layer->partial is ignored and may be NULL. It has no
 * counterpart in the reference, whose attention allocates its temporaries through torch.
 *
 * - Limit: the shape's qsp_attn_workspace_bytes(...) must not exceed
 *   QSP_ATTN_STATIC_SCRATCH_BYTES; larger requests return QSP_ERR_INVALID and launch nothing.
 * - Set-up: the first call on a device looks up the region's address on the current device
 *   (which may load the library's device code); make that first call outside any CUDA stream
 *   capture. Later calls only launch kernels.
 * - One region per device: calls that overlap in time on one device (two streams, two host
 *   threads) race on it and must be serialised by the caller.
 * - The address is looked up once per device ordinal and kept for the life of the process,
 *   which assumes every call runs in that device's primary context (the CUDA runtime's
 *   default) and that nothing calls cudaDeviceReset on the device in between; after a reset,
 *   or from another driver context on the same device, the kept address is not valid.
 * - Nothing in the region has to start at zero: every partial the merge reads is written
 *   earlier in the same call (a key split past the end of its sequence either writes an
 *   all-masked partial or is not read by the merge). */
#define QSP_ATTN_STATIC_SCRATCH_BYTES ((size_t)16 << 20)
int qsp_attn_verify_static(const qsp_attn_layer* layer, void* stream);

/* MTP attention with no cache over a single position: softmax over one key is 1, so the
 * output is the GQA-expanded v times σ(gate) (mtp.py:71-72 via blocks.py:226-235).
 * gate of head h at gate[r·ld_gate + h·gate_head_stride + d] (2·hd for the q_proj
 * [q|gate] layout, hd for a gate-only projection); v rows: n_kv·hd. */
int qsp_mtp_single_token_attn(const void* gate, int64_t ld_gate, int64_t gate_head_stride,
                              const void* v, int64_t ld_v, void* out, int64_t ld_out,
                              int64_t rows, int32_t n_heads, int32_t n_kv_heads,
                              int32_t head_dim, int dtype, void* stream);

/* dst[b,:] = src[(b·tokens + index[b]),:] — the pre-norm hidden at each sequence's last
 * kept position, handed to the MTP head (mtp.py:155 `hidden_last = hidden2[:, 1:2]`). */
int qsp_select_rows(const void* src, int64_t ld_src, int32_t batch, int32_t tokens,
                    const int32_t* index, void* dst, int64_t ld_dst, int64_t dim, int dtype,
                    void* stream);

/* ---------------------------------------------------------------- token selection */

/* Row-wise argmax (first index of the maximum, like torch.argmax) over `vocab` logits. */
int qsp_argmax_rows(const void* logits, int64_t ld, int64_t rows, int64_t vocab,
                    int64_t* out, int64_t out_stride, int dtype, void* stream);

/*
 * Greedy verification (temperature 0): row i of sequence b scores the token after input i.
 * accept_n[b] = number of leading drafts equal to argmax of their row; next_tok[b] = argmax
 * of row accept_n[b]; draft i of sequence b is drafts[b·drafts_ld + i]. The exact-match rule of generate_mtp (src/qwen3_5/mtp.py:144-162)
 * generalised to k = tokens-1 drafts. argmax_out [B*T] optional.
 */
int qsp_greedy_verify(const void* logits, int64_t ld, int32_t batch, int32_t tokens,
                      int64_t vocab, const int64_t* drafts, int64_t drafts_ld, int32_t* accept_n,
                      int64_t* next_tok, int64_t* argmax_out, float* workspace, int dtype,
                      void* stream);

/*
 * Lossless speculative sampling (new behaviour; the reference has none): with
 * p_i = softmax(target_logits[b,i]/temperature), q_i = softmax(draft_logits[b,i]/temperature),
 * draft i is accepted iff u_accept[b,i]·q_i(d_i) < p_i(d_i); at the first rejection the token
 * is drawn by inverse CDF at u_resample[b] from max(0, p_i − q_i); after k acceptances a
 * bonus token is drawn from p_k. Writes accept_n[b], next_tok[b].
 */
int qsp_spec_sample(const void* target_logits, int64_t ld_t, const void* draft_logits,
                    int64_t ld_d, int32_t batch, int32_t k, int64_t vocab, float temperature,
                    const int64_t* drafts, int64_t drafts_ld, const float* u_accept,
                    const float* u_resample, int32_t* accept_n, int64_t* next_tok,
                    float* workspace, int dtype, void* stream);

/* Categorical draw by inverse CDF of softmax(logits/temperature) at u[r] (temperature > 0),
 * or argmax (temperature <= 0): the draw of sample_next (src/generate.py:25-37). */
int qsp_sample_rows(const void* logits, int64_t ld, int64_t rows, int64_t vocab,
                    float temperature, const float* u, int64_t* out, int64_t out_stride,
                    float* workspace, int dtype, void* stream);

/* Bytes of fp32 workspace the selection kernels need for `rows` rows of `vocab`. */
size_t qsp_select_workspace_bytes(int64_t rows, int64_t vocab);

/* Sampling filters of sample_next (src/generate.py:17-37): repetition penalty over a
 * context, temperature, top-k, top-p. Row r of a call belongs to sequence b = r / rows_per_seq
 * and scores position t = r % rows_per_seq; its penalty context is
 *   hist[b, 0 : hist_n[b]]  ∪  step_ids[b, 0 : step_base + t]
 * (either part may be NULL; lengths are clamped to hist_ld and step_ld). Duplicates in the
 * context are penalised once. */
typedef struct qsp_sample_params {
  float temperature;         /* <= 0: greedy (argmax of the penalised logits) */
  int32_t top_k;             /* <= 0 or >= vocab: off */
  float top_p;               /* outside (0, 1): off */
  float repetition_penalty;  /* 1: off; else x/p for x > 0, x·p for x <= 0 on context tokens */
  const int64_t* hist;       /* [B, hist_ld] token history (prompt + committed tokens) */
  int64_t hist_ld;
  const int32_t* hist_n;     /* [B] */
  const int64_t* step_ids;   /* [B, step_ld] tokens of the step being scored */
  int64_t step_ld;
  int32_t step_base;
} qsp_sample_params;

/* Bytes of workspace qsp_sample_filtered / qsp_spec_sample_filtered need for `rows` scored
 * rows of `vocab` (the penalised, scaled rows in fp32 plus per-row statistics). */
size_t qsp_filter_workspace_bytes(int64_t rows, int64_t vocab);

/* sample_next for every row (src/generate.py:17-37): penalty → argmax when
 * temperature <= 0; else /temperature → top-k → top-p → categorical draw by inverse CDF at
 * u[r] over the kept tokens (the reference draws with torch.multinomial from the same
 * distribution). Ties at the top-p boundary value are all kept. */
int qsp_sample_filtered(const void* logits, int64_t ld, int64_t rows, int32_t rows_per_seq,
                        int64_t vocab, const qsp_sample_params* params, const float* u,
                        int64_t* out, int64_t out_stride, void* workspace, size_t workspace_bytes,
                        int dtype, void* stream);

/* qsp_spec_sample / qsp_greedy_verify with the filters: p and q are the filtered target
 * (B·(k+1) rows) and draft (B·k rows) distributions, each row's penalty context being the
 * history plus the step's tokens up to the scored position (step_ids = the step's
 * [pending, d1..dk], step_base = 1). temperature <= 0: greedy verification of the
 * penalised argmax, as generate_mtp does (mtp.py:139-148). */
int qsp_spec_sample_filtered(const void* target_logits, int64_t ld_t, const void* draft_logits,
                             int64_t ld_d, int32_t batch, int32_t k, int64_t vocab,
                             const qsp_sample_params* params, const int64_t* drafts,
                             int64_t drafts_ld, const float* u_accept, const float* u_resample,
                             int32_t* accept_n, int64_t* next_tok, void* workspace,
                             size_t workspace_bytes, int dtype, void* stream);

/* ---------------------------------------------------------------- sparse MoE FFN */

/*
 * The qwen3_5_moe FFN block followed by the residual add and the next RMSNorm
 * (SparseMoeBlock.forward, src/qwen3_5_moe/blocks.py:399-421, inside DecoderLayer.forward,
 * src/qwen3_5_moe/modeling_qwen3_5_moe.py:57-59):
 *   p = softmax(xn·gateᵀ) in fp32; top_k experts (largest p; equal values → lower index);
 *   renormalised to sum 1 when norm_topk_prob; rounded to dtype;
 *   out = Σ_e p_e·SwiGLU_e(xn) accumulated in ascending expert order with a rounding to dtype
 *   after each add (index_add_ into a dtype buffer) + σ(shared_gate·xn)·SwiGLU_s(xn);
 *   x := x + out; y = RMSNorm(x)·(1 + norm_w) (skipped when norm_w is NULL).
 *
 * Weights (dtype, row-major, 16-byte aligned):
 *   w_in        [n_route + 2·shared_inter, hidden] — rows [0, n_experts): router
 *               (mlp.gate.weight); row n_experts: mlp.shared_expert_gate.weight (when
 *               shared_inter > 0); zero rows up to n_route = qsp_moe_router_rows(...); then
 *               mlp.shared_expert.gate_proj.weight and .up_proj.weight. One GEMM reads xn once
 *               for all of them.
 *   gate_up     [n_experts, 2·inter, hidden]   mlp.experts.gate_up_proj (gate rows first)
 *   down        [n_experts, hidden, inter]     mlp.experts.down_proj
 *   shared_down [hidden, shared_inter]         mlp.shared_expert.down_proj.weight
 * Limits: n_experts ≤ 1024, top_k ≤ 16 (and ≤ n_experts), hidden ≤ 8192.
 * y may alias xn (xn is last read before y is written).
 */
typedef struct qsp_moe_layer {
  int32_t tokens;          /* rows of this call (batch · tokens per sequence) */
  int32_t hidden, n_experts, top_k, inter, shared_inter;
  int32_t norm_topk_prob;
  int32_t dtype;
  float eps;
  const void* xn;          /* [tokens, ld_xn] post_attention_layernorm(x) */
  int64_t ld_xn;
  const void* w_in;
  const void* gate_up;
  const void* down;
  const void* shared_down; /* may be NULL when shared_inter == 0 */
  void* x;                 /* [tokens, ld_x] residual stream, updated in place */
  int64_t ld_x;
  const void* norm_w;      /* [hidden] next RMSNorm weight, or NULL */
  void* y;                 /* [tokens, ld_y] RMSNorm output */
  int64_t ld_y;
  void* workspace;         /* qsp_moe_workspace_bytes(...) bytes, 256-byte aligned */
  size_t workspace_bytes;
  int32_t* expert_counts;  /* optional [n_experts]: tokens routed to each expert */
} qsp_moe_layer;

int qsp_moe_ffn(const qsp_moe_layer* layer, void* stream);

/* Rows of w_in before the shared expert's gate|up block (router + shared gate, padded to 8). */
int64_t qsp_moe_router_rows(int32_t n_experts, int32_t shared_inter);

/* Workspace bytes qsp_moe_ffn needs for `tokens` rows (0 for invalid sizes). */
size_t qsp_moe_workspace_bytes(int32_t tokens, int32_t hidden, int32_t n_experts, int32_t top_k,
                               int32_t inter, int32_t shared_inter, int32_t dtype);

/* ---------------------------------------------------------------- cache bookkeeping */

/* After a forward of T tokens: seq_lens[b] += T; parity ^= 1; speculative → replay_n =
 * conv_off = T (keep all unless qsp_cache_accept trims), commit-all → both 0. This is the
 * reference's `advance(n)` (kv.py:46-47) for per-sequence lengths. */
int qsp_cache_finalize(int32_t batch, int32_t tokens, int32_t speculative, int32_t* seq_lens,
                       int32_t* replay_n, int32_t* conv_off, int32_t* parity, void* stream);

/* Keep only keep[b] = accept_n[b] + 1 of the last speculative call's T tokens: the
 * index rollback that replaces `past.clone()` + restore + recompute (mtp.py:141,156-162). */
int qsp_cache_accept(int32_t batch, int32_t tokens, const int32_t* accept_n,
                     int32_t* seq_lens, int32_t* replay_n, int32_t* conv_off, void* stream);

/* Copy committed step tokens into per-sequence output streams: out[b, n_out[b] + j] =
 * ids[b, j] for j <= accept_n[b] (capacity-checked), n_out[b] += accept_n[b]+1; then
 * ids[b,0] := next_tok[b] (the next pending token). */
int qsp_commit_tokens(int32_t batch, int32_t tokens, int64_t* ids, const int32_t* accept_n,
                      const int64_t* next_tok, int64_t* out, int64_t out_cap, int32_t* n_out,
                      void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QSP_H_ */
