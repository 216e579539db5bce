/*
 * CPU oracle for the speculative-decoding verify path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library links, loads or
 * calls this code; only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg use it, and only as the checker or the timed CPU baseline.
 *
 * It restates, in plain C compiled with -ffp-contract=off, the reference's CPU
 * arithmetic for the path (Inferno.jl, paths relative to that project):
 *   - dequantizers   src/Dequant.jl:304-321 (Q8_0), :325-375 (Q4_K),
 *                    :379-441 (Q5_K), :558-601 (Q6_K)
 *   - block layouts  src/kernels/quant_kernels.c:25-62
 *   - GEMV           src/QuantsCPU.jl / src/ModelCPU.jl:285-379 (dequant, then dot)
 *   - acceptance     src/SpeculativeDecoding.jl:20-104, src/CommonOps.jl:172-318
 *                    (bug-fixed semantics, see accept.c)
 *   - model forward  src/ModelCPU.jl:95-1020, src/FlashAttention.jl:19-84 (model.c)
 * The K-quant encoders are this project's own (the reference has none).
 */
#ifndef INFERNO_ORACLE_H
#define INFERNO_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGML type ids, src/GGUF.jl:25-60 */
enum { OR_F32 = 0, OR_F16 = 1, OR_Q8_0 = 8, OR_Q4_K = 12, OR_Q5_K = 13, OR_Q6_K = 14 };

float    or_f16_to_f32(uint16_t h);
uint16_t or_f32_to_f16(float f);              /* round to nearest even */

/* bytes for one row of `cols` elements, 0 if cols is not a multiple of the block */
int64_t  or_row_bytes(int type, int64_t cols);

/* quantize rows x cols f32 (row-major) into GGUF blocks, own encoder */
int or_quantize(int type, const float *x, int64_t rows, int64_t cols, uint8_t *out);

/* dequantize n elements of GGUF blocks to f32, bit-exact with src/Dequant.jl */
int or_dequantize(int type, const uint8_t *blocks, int64_t n, float *out);

/* Y[n][r] = sum_k W[r][k] * X[n][k]; W quantized rows x cols, X ncols x cols.
 * or_gemm_q8k quantizes each activation column to Q8_K first (the reference's
 * quantized kernels, K-quant weights only) and then accumulates in double,
 * or_gemm_f64 accumulates the dequantized f32 weights in double ("truth"),
 * or_gemm_f32 accumulates in float, index order (the reference's fallback). */
void or_quantize_q8k(const float *x, int64_t k, float *d, int8_t *q);
int or_gemm_q8k(int type, const uint8_t *W, int64_t rows, int64_t cols,
                const float *X, int ncols, double *Y);
int or_gemm_f64(int type, const uint8_t *W, int64_t rows, int64_t cols,
                const float *X, int ncols, double *Y);
int or_gemm_f32(int type, const uint8_t *W, int64_t rows, int64_t cols,
                const float *X, int ncols, float *Y);

/* ---- acceptance (accept.c) ---- */
float or_exp(float x);                          /* shared Cody-Waite exp */
int   or_sample_from_probs(const float *probs, int n, float r);   /* 1-based, SpeculativeDecoding.jl:20-30 */
void  or_chunk_stats(const float *row, int V, float inv_temp, float *cmax, float *csum);
void  or_row_stats(const float *cmax, const float *csum, int nchunk, float inv_temp,
                   float *rmax, float *rsum);
int   or_accept(const float *target, const float *draft, const int32_t *draft_tokens,
                const float *uniforms, int batch, int gamma, int vocab, float temperature,
                int32_t *accept_count, int32_t *out_tokens, int32_t *draft_out);
int   or_accept_greedy(const float *target, const int32_t *draft_tokens, int batch,
                       int gamma, int vocab, int32_t *accept_count, int32_t *out_tokens);
int   or_argmax(const float *row, int n);
/* filtered sampling (CommonOps.jl:196-318) and penalties (ModelCPU.jl:1202-1238) */
int   or_sample_filtered(const float *logits, int vocab, float temperature, int top_k, float top_p,
                         float min_p, float u);                 /* 0-based; -1 on NaN/+Inf */
int   or_sample_rows(const float *logits, int rows, int vocab, float temperature, int top_k,
                     float top_p, float min_p, const float *uniforms, int32_t *out_tokens);
void  or_apply_penalties(float *logits, int rows, int vocab, const int32_t *seen, int n_seen,
                         float presence, float repetition);
/* or_accept on the filtered target and draft distributions (accept.c) */
int   or_accept_filtered(const float *target, const float *draft, const float *uniforms, int batch,
                         int gamma, int vocab, float temperature, int top_k, float top_p, float min_p,
                         int32_t *accept_count, int32_t *out_tokens, int32_t *draft_out);

/* ---- model forward (model.c) ---- */
typedef struct {
    int32_t hidden, n_layers, n_head, n_kv_head, head_dim, rotary_dim, ffn, vocab;
    int32_t ssm_heads, ssm_head_dim, conv_kernel, max_ctx;
    float rope_theta, rms_eps;
} or_model_config;
typedef struct or_model or_model;
typedef struct or_snapshot or_snapshot;
enum {
    OR_T_EMBED = 0, OR_T_FINAL_NORM, OR_T_MTP_FC, OR_T_MTP_NORM_E, OR_T_MTP_NORM_H, OR_T_MTP_NORM,
    OR_T_ATTN_NORM = 10, OR_T_POST_NORM, OR_T_IN_PROJ, OR_T_GATE_PROJ, OR_T_SSM_OUT, OR_T_CONV,
    OR_T_ALPHA, OR_T_BETA, OR_T_SSM_A, OR_T_DT_BIAS, OR_T_SSM_NORM, OR_T_WQ, OR_T_WK, OR_T_WV,
    OR_T_WO, OR_T_Q_NORM, OR_T_K_NORM, OR_T_FFN_GATE, OR_T_FFN_UP, OR_T_FFN_DOWN,
    /* Gemma4 blocks: pre-MLP norm, post-MLP norm, layer scalar (1 element) */
    OR_T_FFN_NORM, OR_T_POST_FFW_NORM, OR_T_LAYER_SCALAR,
    /* Gemma4 per-layer inputs: per layer gate (pli x d), projection (d x pli),
       post norm (d); global token table (vocab x L pli), model projection
       (L pli x d, pre-scaled by d^-1/2) and its norm (pli) */
    OR_T_PLI_GATE = 40, OR_T_PLI_PROJ, OR_T_PLI_POST_NORM,
    OR_T_PLI_TOKEN_EMBD = 50, OR_T_PLI_MODEL_PROJ, OR_T_PLI_PROJ_NORM
};
/* Gemma4 block semantics (src/Gemma4.jl:253-688, src/CommonOps.jl:326-333),
 * switched on by or_model_set_gemma: layer i is a full-attention layer iff
 * (i + 1) % sliding_pattern == 0, else a sliding one (window keys) */
typedef struct {
    int32_t window, sliding_pattern;
    float attn_softcap, final_softcap;   /* 0: off */
    float rope_theta_swa, rope_theta_full, partial_rotary_factor;
    float embed_scale;
    int32_t pli;                         /* per-layer input size (0: none) */
} or_gemma_config;
void or_model_set_gemma(or_model *m, const or_gemma_config *g);
or_model *or_model_new(const or_model_config *c);
void or_model_free(or_model *m);
/* layer >= 0: decoder layer; -1: global tensors; -2: the MTP decoder layer */
int  or_model_set(or_model *m, int layer, int kind, int type, const void *data, int64_t n);
void or_model_set_activation(or_model *m, int mode);  /* 0 exact f32 (default), 1 Q8_K */
/* 1: every key and value row is rounded to bf16 (round to nearest even) as it
 * is written to the attention caches, the target's and the MTP layer's; the
 * engine's bf16 KV cache (ifr_ctx_set_kv_bf16) stores exactly these values */
void or_model_set_kv_bf16(or_model *m, int on);
void or_model_reset(or_model *m);
int  or_forward_token(or_model *m, int token, int pos, float *logits, float *hidden);
int  or_mtp_step(or_model *m, int token, const float *hidden, int pos, float *logits, float *hidden_out);
or_snapshot *or_snapshot_take(or_model *m);
void or_snapshot_restore(or_model *m, const or_snapshot *s);
void or_snapshot_free(or_snapshot *s);

#define OR_ACCEPT_CHUNK 2048   /* elements per statistics chunk */
#define OR_ACCEPT_THREADS 256  /* lanes per chunk in the canonical reduction */

#ifdef __cplusplus
}
#endif
#endif
