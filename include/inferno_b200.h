/*
 * inferno_b200 — C ABI of the B200 (sm_100a) speculative-decoding verify path
 * for Inferno.jl.  Plain pointers and sizes only; no CUDA or torch types.
 *
 * Conventions
 *   - Every native entry point returns int: IFR_OK (0) or an IFR_ERR_* code;
 *     ifr_last_error() gives this thread's message for the last failure.
 *   - Sizes are validated before any launch; invalid ones return IFR_ERR_ARG.
 *   - "dev" pointers are CUDA device pointers on the context's device; all
 *     work is enqueued on the context's stream (asynchronous unless stated).
 *   - Token ids are 0-based (the Julia side adds 1).
 *   - Weight types are GGML type ids (src/GGUF.jl:25-60 of the reference).
 *   - Activations X are column-major by token: X[n*cols + k] is element k of
 *     verify column (token) n; outputs Y[n*rows + r].
 */
#ifndef INFERNO_B200_H
#define INFERNO_B200_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* the library is built with hidden visibility; only these symbols export */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define IFR_OK 0
#define IFR_ERR_ARG 1          /* invalid argument / size / type            */
#define IFR_ERR_CUDA 2         /* CUDA runtime error (message has details)  */
#define IFR_ERR_NOMEM 3        /* device allocation failed                  */
#define IFR_ERR_TIMEOUT 4      /* a bounded device-side wait ran out        */
#define IFR_ERR_UNSUPPORTED 5  /* not built for this device / type          */

#define IFR_TYPE_F32 0
#define IFR_TYPE_F16 1
#define IFR_TYPE_Q8_0 8
#define IFR_TYPE_Q4_K 12
#define IFR_TYPE_Q5_K 13
#define IFR_TYPE_Q6_K 14

#define IFR_MAX_VERIFY_COLS 8  /* columns per pass of the small-N kernel */
#define IFR_MAX_BATCH 256      /* requests per batched state */
#define IFR_DENSE_MIN_COLS_DEFAULT 24  /* engine GEMMs of >= this many columns use ifr_qgemm_dense's path */

typedef struct ifr_ctx ifr_ctx;
typedef struct ifr_tensor ifr_tensor;

/* thread-local message of the last failing call on this thread ("" if none) */
const char *ifr_last_error(void);
/* library version, major*10000 + minor*100 + patch */
int ifr_version(void);

/* --- context: one device + one stream, one host thread at a time ---------
 * Replaces the reference's process-global library handle and Q8_K buffer
 * pool (src/QuantizedKernels.jl:22-72). */
int ifr_ctx_create(int device, ifr_ctx **out);
int ifr_ctx_destroy(ifr_ctx *ctx);
/* enqueue on an external cudaStream_t (passed as void*; NULL = the CUDA
 * default stream).  A new context starts on its own non-blocking stream. */
int ifr_ctx_set_stream(ifr_ctx *ctx, void *cuda_stream);
int ifr_ctx_get_stream(ifr_ctx *ctx, void **cuda_stream);
/* pre-size the context's scratch for ifr_accept / ifr_accept_greedy up to
 * (batch, gamma, vocab) so later calls allocate nothing (e.g. before CUDA
 * graph capture).  ifr_qgemm needs no scratch. */
int ifr_ctx_reserve_accept(ifr_ctx *ctx, int batch, int gamma, int vocab);
/* Activations of the K-quant (Q4_K/Q5_K/Q6_K) GEMVs:
 *   IFR_ACT_EXACT (default)  f32 activations, split exactly into fp16 hi + lo
 *                            on the fp16 tensor cores: the exact product with
 *                            the dequantized weights, up to f32 summation;
 *   IFR_ACT_Q8K              each 256-block of a column quantized as the
 *                            reference's quantize_row_q8_K (src/kernels/
 *                            quant_kernels.c:166-194; d = amax/127, roundf(x/d))
 *                            and multiplied exactly on the integer tensor
 *                            cores: the results of the reference's q4_k_gemv
 *                            .. q6_k_gemv up to f32 summation order.
 * Q8_0 GEMVs always use exact f32 activations (the reference's q8_0_gemv).
 * The mode applies to ifr_qgemm and to the model engine of this context. */
#define IFR_ACT_EXACT 0
#define IFR_ACT_Q8K 1
int ifr_ctx_set_activation(ifr_ctx *ctx, int mode);
/* The model engine computes a projection over n columns (requests x verify
 * tokens) with the exact small-N kernel in passes of 8 columns while
 * n < ncols, and with the dense tensor-core path of ifr_qgemm_dense (fp16
 * operands, f32 accumulation) from ncols columns on.  Default
 * IFR_DENSE_MIN_COLS_DEFAULT; a state of one request reaches it only in the
 * prefill chunks that ifr_ctx_set_prefill_dense allows. */
int ifr_ctx_set_dense_min_cols(ifr_ctx *ctx, int ncols);
/* one-request prefill (forward_cpu! over the prompt, src/ModelCPU.jl:1325)
 * runs in chunks of 64 tokens; enable = 1 lets a chunk's projections take
 * the dense tensor-core path (fp16 operands: logits within 1e-2 of the exact
 * product instead of 1e-4), 0 (default) keeps them exact.  No counterpart in
 * the reference (its prefill is the f32 token loop). */
int ifr_ctx_set_prefill_dense(ifr_ctx *ctx, int enable);
/* enable = 1 runs the decoder layers of a one-request verify (<= 8 columns,
 * exact activations, one rank) as one persistent cooperative launch - every
 * projection, GatedDeltaNet step and attention step of the layer stack as a
 * phase separated by grid barriers - instead of ~5 launches per layer
 * (forward_cpu!, src/ModelCPU.jl:976-1020, same arithmetic and tolerance).
 * Models it does not cover (Gemma4 blocks, other head dims, formats other
 * than Q4_K/Q6_K) keep the separate launches.  Default 0. */
int ifr_ctx_set_fused_layers(ifr_ctx *ctx, int enable);
/* failure detection of the fused launch, for tests: runs a two-phase fused
 * launch in which one CTA never arrives at the grid barrier; the other CTAs'
 * bounded waits (~2 s) run out and the call returns IFR_ERR_TIMEOUT, with the
 * context still usable afterwards.  No counterpart in the reference. */
int ifr_test_fused_timeout(ifr_ctx *ctx);
/* enable = 1 (default): a batched state (ifr_state_create_batch, batch > 1)
 * gives every projection of its model an fp16 copy of the dequantized weights
 * in the dense GEMM's operand layout (~3.6 x the Q4_K bytes of HBM), which the
 * dense path (ifr_qgemm_dense's kernel) then copies instead of dequantizing.
 * Results are identical either way: each weight is rounded to fp16 once in
 * both.  Takes effect for states created afterwards. */
int ifr_ctx_set_dense_f16_weights(ifr_ctx *ctx, int enable);
/* enable = 1: states created afterwards that take the split-KV attention
 * (batches, or one request with a long cache) keep their attention caches,
 * the target's and the MTP layer's, in bf16: each key and value row is
 * rounded to nearest even as it is written, half the bytes of the f32 cache
 * for the attention to read.  Scores and outputs stay f32 sums of the stored
 * values (the oracle's or_model_set_kv_bf16).  Default 0 (f32 caches, the
 * reference's Float32 KV of src/ModelCPU.jl).  No counterpart in the
 * reference. */
int ifr_ctx_set_kv_bf16(ifr_ctx *ctx, int enable);
/* wait for the context's stream; IFR_ERR_TIMEOUT if a bounded device-side
 * wait of a kernel ran out since the last ifr_sync */
int ifr_sync(ifr_ctx *ctx);

/* --- weights: device-resident quantized matrices -------------------------
 * rows = outer (output) dim, cols = inner dim; bytes are GGUF blocks, row by
 * row (src/LoaderCPU.jl:123-161 keeps the same bytes as Q*_Matrix).  The
 * library owns the device copy (it may re-lay out blocks for the kernels;
 * values are unchanged, see ifr_dequant).  Synchronous. */
int ifr_weights_upload(ifr_ctx *ctx, int type, const void *host_bytes,
                       int64_t rows, int64_t cols, ifr_tensor **out);
int ifr_weights_from_device(ifr_ctx *ctx, int type, const void *dev_bytes,
                            int64_t rows, int64_t cols, ifr_tensor **out);
int ifr_tensor_free(ifr_tensor *t);
/* the fp16 operand stages of t for ifr_qgemm_dense (see
 * ifr_ctx_set_dense_f16_weights); ifr_tensor_free releases them.  No
 * counterpart in the reference. */
int ifr_tensor_prepare_dense(ifr_ctx *ctx, ifr_tensor *t);
int ifr_tensor_info(const ifr_tensor *t, int *type, int64_t *rows, int64_t *cols,
                    int64_t *device_bytes);

/* bit-exact dequantization to f32 [rows][cols] (dev_out), the values of
 * src/Dequant.jl:304-601 (dequantize_q8_0/q4_k/q5_k/q6_k) */
int ifr_dequant(ifr_ctx *ctx, const ifr_tensor *t, float *dev_out);

/* Y = W * X for ncols verify columns (any ncols >= 1; passes of 8).
 * X [ncols][cols] and Y [ncols][rows] f32 on the device, X 16-byte aligned.
 * K-quants use the context's activation mode (ifr_ctx_set_activation): exact
 * f32 products by default, or the reference's Q8_K quantized activations;
 * Q8_0 always exact.  f32 accumulation.  Replaces q4_k_gemv/q5_k_gemv/
 * q6_k_gemv/q8_0_gemv (src/kernels/quant_kernels.c:602-697), which the
 * reference calls once per column (src/ModelCPU.jl:285-379). */
int ifr_qgemm(ifr_ctx *ctx, const ifr_tensor *W, const float *X_dev, int ncols,
              float *Y_dev);

/* Y = W * RMSNorm(X) for ncols columns: each column x normalised as
 * x * (1 / sqrt(mean(x^2) + eps)) * norm_w (rmsnorm_cpu!, src/ModelCPU.jl:
 * 111-123) and multiplied by W, in one launch per 8 columns.  With exact
 * activations the norm is folded into the epilogue: W (x * norm_w) times the
 * column's 1/rms, the sums of squares formed from the loads that feed the
 * tensor cores.  norm_w [cols] f32 on the device, 16-byte aligned; other
 * arguments as ifr_qgemm.  Replaces the reference's rmsnorm_cpu! followed by
 * the per-column GEMV of src/ModelCPU.jl:285-379. */
int ifr_qgemm_rmsnorm(ifr_ctx *ctx, const ifr_tensor *W, const float *X_dev, int ncols,
                      const float *norm_w_dev, float eps, float *Y_dev);

/* Y = W * X for many columns at once (batched verify across requests, prompt
 * chunks) on the tcgen05 tensor cores: every weight is its exact dequantized
 * value rounded to fp16, every activation column is scaled by a power of two
 * and rounded to fp16, products are summed in f32 (relative error of each
 * product <= 2^-10).  Same arguments as ifr_qgemm; uses the context's scratch
 * (allocated on first use, or by ifr_ctx_reserve_dense).  Replaces the same
 * per-column calls as ifr_qgemm, once ncols makes the contraction dense. */
int ifr_qgemm_dense(ifr_ctx *ctx, const ifr_tensor *W, const float *X_dev, int ncols,
                    float *Y_dev);
/* pre-size the scratch of ifr_qgemm_dense for W and up to ncols columns */
int ifr_ctx_reserve_dense(ifr_ctx *ctx, const ifr_tensor *W, int ncols);

/* host-side quantizer (f32 rows -> GGUF blocks of `type`), the library's own
 * encoder (the reference has none); multithreaded, no device needed */
int ifr_quantize(int type, const float *x, int64_t rows, int64_t cols, uint8_t *out);

/* --- acceptance ------------------------------------------------------------
 * Sampled verification (fixed semantics of src/SpeculativeDecoding.jl:37-104):
 *   target  [batch][gamma+1][vocab] f32 logits (dev)
 *   draft   [batch][gamma][vocab]   f32 logits (dev)
 *   draft_tokens [batch][gamma] (dev) or NULL: drafts are then drawn from
 *           softmax(draft/T) with u_d
 *   uniforms [batch][2*gamma+1] (dev): u_d[gamma], u_a[gamma], u_rb
 *   accept_count [batch], out_tokens [batch][gamma+1] (-1 past the emitted
 *   tokens), draft_out [batch][gamma] or NULL.  Bit-exact with the oracle.
 *   batch * (2 * gamma + 1) <= 65535, else IFR_ERR_ARG. */
int ifr_accept(ifr_ctx *ctx, const float *target, const float *draft,
               const int32_t *draft_tokens, const float *uniforms, int batch,
               int gamma, int vocab, float temperature, int32_t *accept_count,
               int32_t *out_tokens, int32_t *draft_out);
/* ifr_accept without any device allocation (no counterpart in the reference):
 * same arguments and bit-identical results, with the scratch in a fixed
 * 1 MiB array per device inside the library instead of the context's
 * cudaMalloc'd buffer.  For callers that must not allocate device memory at
 * call time: a host whose own pool (e.g. CUDA.jl's) already holds the free
 * HBM, or a serving loop that cannot take the device-wide synchronization
 * cudaMalloc/cudaFree may cause.  Sizes whose scratch
 * (2 * batch * (2 * gamma + 1) * ceil(vocab / 2048) floats plus small terms)
 * exceeds 1 MiB fail with IFR_ERR_ARG.  The first call on a device does a
 * one-time set-up (module load, symbol lookup): make it once before stream
 * capture or timed work.  The array is shared by all callers on the device:
 * calls that can overlap (other streams or contexts on that device) race and
 * must be ordered by the caller.  The set-up is cached for the life of the
 * process: after a device reset (cudaDeviceReset, or a host runtime that
 * resets the device's primary context) do not call it on that device again. */
int ifr_accept_noalloc(ifr_ctx *ctx, const float *target, const float *draft,
                       const int32_t *draft_tokens, const float *uniforms, int batch,
                       int gamma, int vocab, float temperature, int32_t *accept_count,
                       int32_t *out_tokens, int32_t *draft_out);
/* sampled verification with the sampler's filters (replaces the filtered
 * draws of src/SpeculativeDecoding.jl:57,102, which call
 * CommonOps.softmax_sample_scratch!, src/CommonOps.jl:196-318): top_k,
 * top_p and min_p (as in ifr_sample: 0 / 1 / 0 turn them off) and the
 * temperature applied to every target and draft row; drafts drawn from the
 * filtered draft rows with u_d, the ratio test and the residual
 * max(p_t - p_d, 0) over the filtered distributions, the bonus token from
 * the filtered last target row.  Same layouts as ifr_accept (drafts are
 * always drawn here); finite logits; vocab <= 524288; parameter errors as in
 * ifr_sample.  Bit-exact with the oracle (or_accept_filtered). */
int ifr_accept_filtered(ifr_ctx *ctx, const float *target, const float *draft, const float *uniforms,
                        int batch, int gamma, int vocab, float temperature, int top_k, float top_p,
                        float min_p, int32_t *accept_count, int32_t *out_tokens, int32_t *draft_out);
/* greedy verification (src/ModelCPU.jl:2099-2115): accept while
 * argmax(target[i]) == draft[i], then emit the target argmax */
int ifr_accept_greedy(ifr_ctx *ctx, const float *target, const int32_t *draft_tokens,
                      int batch, int gamma, int vocab, int32_t *accept_count,
                      int32_t *out_tokens);
/* filtered sampling, one token per row: CommonOps.softmax_sample_scratch!
 * (src/CommonOps.jl:196-318) with uniforms[row] in [0, 1) in place of
 * rand().  logits [rows][vocab] and uniforms [rows] on the device;
 * out_tokens [rows] (device, 0-based).  temperature >= 0 (0 = argmax),
 * top_k >= 0 (0 or >= vocab: off), top_p in [0, 1] (1: off), min_p in
 * [0, 1] (0: off); values the reference rejects with ArgumentError
 * (:126-139), vocab < 1 and vocab > 524288 give IFR_ERR_ARG.  A row holding
 * NaN or +Inf (which the reference also rejects) gets token -1; a row of
 * -Inf only gets token 0.  Ties at the top-k and top-p cuts go to the lower
 * token id, and the top-p running sum is exact (integer weights). */
int ifr_sample(ifr_ctx *ctx, const float *logits, int rows, int vocab, float temperature, int top_k,
               float top_p, float min_p, const float *uniforms, int32_t *out_tokens);
/* in place on logits [rows][vocab] (device): for every distinct token t of
 * seen[row][0 .. n_seen) with 0 <= t < vocab (others, e.g. -1 padding, are
 * skipped), the presence penalty l -= presence, then the repetition penalty
 * l = l > 0 ? l / repetition : l * repetition (src/ModelCPU.jl:1202-1211,
 * 1237-1238; src/CommonOps.jl:63-76).  presence 0 and repetition 1 are
 * no-ops as there; repetition must be finite and > 0, vocab <= 1048576. */
int ifr_apply_penalties(ifr_ctx *ctx, float *logits, int rows, int vocab, const int32_t *seen, int n_seen,
                        float presence, float repetition);

/* --- model and speculative-decoding state ---------------------------------
 * A Qwen3.5-hybrid GGUF (general.architecture "qwen35": GatedDeltaNet layers
 * where blk.N.ssm_a exists, full-attention layers elsewhere, SwiGLU MLPs,
 * tied or separate lm_head; src/LoaderCPU.jl:265-694 of the reference) plus
 * an optional MTP draft head (mtp.fc.weight, mtp.pre_fc_norm_embedding.weight,
 * mtp.pre_fc_norm_hidden.weight, mtp.norm.weight, mtp.blk.0.* attention layer). */
typedef struct ifr_model ifr_model;
typedef struct ifr_state ifr_state;
typedef struct {
    int32_t hidden, n_layers, n_head, n_kv_head, head_dim, rotary_dim, ffn, vocab;
    int32_t ssm_heads, ssm_head_dim, conv_kernel, context_length, n_attention_layers, has_mtp;
    float rope_theta, rms_eps;
    int64_t weight_bytes;   /* quantized bytes of the decoder layers + lm_head */
} ifr_model_info;

/* load all weights to the context's device (synchronous) */
int ifr_model_load_gguf(ifr_ctx *ctx, const char *path, ifr_model **out);

/* --- tensor parallelism (config 5): one process or thread per GPU ---------
 * A communicator (NCCL over NVLink, bound at run time) for `world` ranks;
 * rank 0 creates the unique id and the host hands it to every rank.  The
 * reference has no multi-GPU path; this replaces its single-process
 * forward_cpu! for models too large or too slow for one GPU. */
#define IFR_COMM_ID_BYTES 128
typedef struct ifr_comm ifr_comm;
int ifr_comm_available(void);                 /* 1 if libnccl.so.2 could be bound */
int ifr_comm_unique_id(uint8_t *id_out);      /* IFR_COMM_ID_BYTES bytes */
int ifr_comm_create(ifr_ctx *ctx, int rank, int world, const uint8_t *id, ifr_comm **out);
int ifr_comm_destroy(ifr_comm *comm);
/* load this rank's shard of an attention-only model: query/key/value heads,
 * gate/up rows (256-column units) and lm_head vocabulary rows split across the
 * ranks (column parallel), attention-output and down projections split along
 * their inner dimension (row parallel, one sum all-reduce of the residual
 * after each); norms and the embedding are replicated.  Greedy acceptance
 * takes the argmax over all ranks' vocabulary shards.  comm == NULL is
 * ifr_model_load_gguf.  The communicator must outlive the model. */
int ifr_model_load_gguf_tp(ifr_ctx *ctx, const char *path, ifr_comm *comm, ifr_model **out);
/* this rank's share: shard[8] = {rank, world, query heads, KV heads, FFN
 * columns, FFN offset, lm_head vocabulary rows, vocabulary offset}.  The
 * logits of ifr_state_last_verify are the rank's vocabulary rows. */
int ifr_model_get_shard(const ifr_model *m, int32_t *shard);
int ifr_model_free(ifr_model *m);
int ifr_model_get_info(const ifr_model *m, ifr_model_info *info);

/* KV caches, SSM/conv states and rollback buffers for max_ctx positions */
int ifr_state_create(ifr_model *m, int max_ctx, ifr_state **out);
/* the same for `batch` independent requests that advance together: every
 * call below then works on all of them at once (prompts, drafts and reads
 * per request as documented).  No counterpart in the reference, which
 * serves one sequence at a time (src/SpeculativeDecoding.jl:106-172). */
int ifr_state_create_batch(ifr_model *m, int max_ctx, int batch, ifr_state **out);
int ifr_state_free(ifr_state *s);
int ifr_state_reset(ifr_state *s);
/* prefill a prompt (host tokens), emit the first greedy token (synchronous);
 * forward_cpu!(prompt) then softmax_sample at temperature 0
 * (src/ModelCPU.jl:1325-1336) */
int ifr_prefill(ifr_state *s, const int32_t *tokens, int n, int32_t *first_token);
/* batched state: tokens [batch][n] (every request's prompt has n tokens),
 * first_tokens [batch] (may be NULL) */
int ifr_prefill_batch(ifr_state *s, const int32_t *tokens, int n, int32_t *first_tokens);
/* one greedy speculative step, asynchronous on the context stream:
 * draft gamma tokens with the MTP head (or take `drafts`, gamma host tokens),
 * verify [last, drafts] in one gamma+1-column forward, accept the longest
 * prefix matching the target argmax (src/ModelCPU.jl:2099-2115), emit the
 * accepted drafts plus the target's next token, and roll the SSM/conv/KV
 * state back to the accepted prefix.  gamma = 0 is plain greedy decoding. */
int ifr_spec_step(ifr_state *s, int gamma, const int32_t *drafts);
/* (batched state: drafts [batch][gamma]) */
/* capture `steps` consecutive MTP spec steps (gamma drafts each) into one
 * CUDA graph on the context stream (which must not be the legacy default
 * stream); ifr_spec_graph_launch replays it asynchronously.  Run one eager
 * ifr_spec_step first so that every kernel is initialised before capture. */
int ifr_spec_graph(ifr_state *s, int gamma, int steps);
int ifr_spec_graph_launch(ifr_state *s);
/* one greedy speculative step with a separate draft model (the draft ->
 * verify -> accept loop of src/SpeculativeDecoding.jl:106-172 with the draft
 * model's greedy tokens; the reference drafts with the same call shape):
 * `draft` (an attention-only, unsharded model on the same context, prefilled
 * with the same prompt) decodes gamma tokens, the target verifies them as in
 * ifr_spec_step, and the draft follows the target's accepted prefix.
 * Asynchronous; batch sizes must match.  ifr_spec_graph_draft captures
 * `steps` such steps into the target state's graph (ifr_spec_graph_launch). */
int ifr_spec_step_draft(ifr_state *target, ifr_state *draft, int gamma);
int ifr_spec_graph_draft(ifr_state *target, ifr_state *draft, int gamma, int steps);
/* The step in parts, for acceptance decided by the caller (e.g. sampled with
 * ifr_accept): speculate_and_verify (src/SpeculativeDecoding.jl:37-104) as
 * draft, verify, accept, commit.
 * ifr_draft_mtp: gamma (1..7) greedy MTP draft tokens per request into the
 * state (the input of the next ifr_verify_step with drafts == NULL); copied
 * to drafts_out [batch][gamma] (host) when given (synchronizes).
 * ifr_verify_step: the target forward over [last token, drafts] (drafts host
 * [batch][gamma], or NULL for the state's MTP drafts) at the state's position
 * (ModelCPU.jl:2099-2115); logits [batch][gamma+1][vocab] (device) copied to
 * logits_out when given.  Nothing is committed: KV entries of the columns are
 * written, the GatedDeltaNet state is not advanced.
 * ifr_rollback: commits accept_count[b] (0..gamma) drafts and the emitted
 * token of request b: tokens [batch][gamma+1] (host), tokens[b][0..a] with
 * a = accept_count[b] the accepted drafts then the correction or bonus token.
 * The rest of the verify is rolled back (the SSM state replays only the
 * accepted columns; later KV entries are overwritten).  Each verify needs its
 * rollback before the next draft, verify or spec step (IFR_ERR_ARG). */
int ifr_draft_mtp(ifr_state *s, int gamma, int32_t *drafts_out);
int ifr_verify_step(ifr_state *s, int gamma, const int32_t *drafts, float *logits_out);
int ifr_rollback(ifr_state *s, const int32_t *accept_count, const int32_t *tokens);
/* per-launch CUDA-event timing of the state's work (0 = off, default), and
 * its totals per category since enabling: 0 verify lm_head, 1 draft lm_head,
 * 2 decoder-layer GEMVs, 3 draft GEMVs, 4 SSM steps, 5 attention steps
 * (ms[8], algorithmic weight bytes[8], timed launches[8]); launches = kernel
 * launches enqueued by the state so far */
int ifr_state_profile(ifr_state *s, int enable);
int ifr_state_profile_read(ifr_state *s, double *ms, int64_t *bytes, int *count, int64_t *launches);
/* with profiling on (ifr_state_profile): the phases of the last fused
 * layer-stack launch (ifr_ctx_set_fused_layers) - kinds[i] (1 projection,
 * 2 GatedDeltaNet state update, 3 attention slices, 4 attention combine,
 * 5 GatedDeltaNet norm, gate and commits) and
 * us[6 i .. 6 i + 5] in microseconds: the phase from CTA 0's start to the
 * next phase's start; the slowest CTA's parts (fragments, tiles, epilogue -
 * projections only, other kinds report the whole phase as the third part -
 * and its barrier wait to the next phase's start) and its whole phase; when max_phases >= 2 * the phase count, us[6 n + 4 i ..] also
 * holds phase i's grid barrier: CTA 0's arrival to the last CTA's, the last
 * arrival to CTA 0 seeing it, CTA 0's acquire fence, and on to the next
 * phase's start; *n_phases = 0 when none was traced */
int ifr_state_fused_trace(ifr_state *s, int max_phases, int *kinds, double *us, int *n_phases);
/* enqueue only the dequant-GEMV launches of one verify forward (every
 * decoder-layer projection + the lm_head) on ncols columns of scratch
 * activations, back to back (capturable): a measurement of the verify GEMVs
 * alone.  Scratch buffers only; the committed state is not touched. */
int ifr_gemv_pass(ifr_state *s, int ncols);
/* synchronous read of the emitted tokens and of
 * scalars[4] = {position, last accept count, steps, last token} */
int ifr_state_read(ifr_state *s, int32_t *tokens, int max_tokens, int *n_tokens, int32_t *scalars);
/* the same for request b of a batched state (ifr_state_read reads request 0) */
int ifr_state_read_request(ifr_state *s, int b, int32_t *tokens, int max_tokens, int *n_tokens,
                           int32_t *scalars);
/* synchronous read of the last forward: logits [batch * n][vocab] (verify
 * columns, request-major), final-normed hidden [batch * n][hidden], the
 * tokens fed [batch][n]; any pointer may be NULL */
int ifr_state_last_verify(ifr_state *s, float *logits, float *hidden, int32_t *tokens, int *n_cols);

/* --- legacy shims: the reference's C symbols, identical signatures --------
 * src/kernels/quant_kernels.c:602-697, bound by src/QuantizedKernels.jl:90-145.
 * HOST pointers; each call uploads W and x, runs ifr_qgemm on device 0 and
 * copies out back (parity / drop-in, not speed).  q8_scratch is ignored: the
 * activations stay f32.  On failure `out` is filled with NaN and the message
 * is printed to stderr and kept in ifr_last_error(). */
void q4_k_gemv(const uint8_t *weight, const float *x, float *out, void *q8_scratch,
               int inner_dim, int outer_dim);
void q5_k_gemv(const uint8_t *weight, const float *x, float *out, void *q8_scratch,
               int inner_dim, int outer_dim);
void q6_k_gemv(const uint8_t *weight, const float *x, float *out, void *q8_scratch,
               int inner_dim, int outer_dim);
void q8_0_gemv(const uint8_t *weight, const float *x, float *out, int inner_dim,
               int outer_dim);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif
