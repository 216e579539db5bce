/*
 * Qwen3.5-hybrid forward pass, token by token, on dequantized f32 weights.
 * TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Restates the reference's CPU path (Inferno.jl, src/ModelCPU.jl):
 *   rmsnorm_cpu!            :111-123  out = x * (1/sqrt(ss/n + eps)) * w
 *   rmsnorm_rotary!         :188-232  per-head RMSNorm, then half-split RoPE
 *                                     on the first rotary_dim dims (pairs i, i+half)
 *   RotaryEmbeddingCPU      :136-154  inv_freq = 1/theta^(2(i-1)/rd) in f64 -> f32,
 *                                     angle = inv_freq * pos (f32), 0-based pos
 *   GatedDeltaNetCPU        :566-731  conv ring + SiLU, L2-normalised q (x 1/sqrt(dk))
 *                                     and k, f64 gates, delta rule, per-head norm,
 *                                     y * silu(z), ssm_out
 *   FullAttentionCPU        :787-887  per-head interleaved [q; gate], Q/K norm + RoPE,
 *                                     KV cache, GQA flash attention (FlashAttention.jl
 *                                     :19-84, 64-key blocks, online softmax), sigmoid gate
 *   mlp_forward             :482-508  down(silu(gate x) * up x)
 *   DecoderLayerCPU         :901-922  x += op(norm(x)); x += mlp(norm(x))
 *   forward_cpu!            :976-1020 embedding column, layers, final norm, lm_head
 * The embedding is tied (lm_head = token_embd rows, LoaderCPU.jl:411-417).
 * The MTP draft head (mtp_forward!, :2031-2048) gains one attention decoder
 * layer between fc and the final norm; its input hidden is the final-normed
 * hidden of the last verified token for the first draft, then the layer
 * output of the previous draft.
 * Gemma4 mode (or_model_set_gemma; src/Gemma4.jl): attention-only blocks
 *   forward!                :604-676  embedding x embed_scale; per layer
 *                                     x = x + norm_pa(attn(norm_in(x)));
 *                                     x = (x + norm_pf(mlp(norm_ff(x)))) * layer_scalar
 *   attention_forward!      :296-456  q / k RMSNorm with weights, v RMSNorm without,
 *                                     RoPE on pairs (k, k + hd/2) (sliding layers: every
 *                                     pair, theta_swa; full layers: the first
 *                                     partial * hd / 2 pairs, frequencies over hd,
 *                                     theta_full), scores q.k (scale 1) capped by
 *                                     tanh(s / cap) cap, sliding window of `window`
 *                                     keys, softmax, no output gate
 *   mlp_forward!            :556-581  down(gelu_tanh(gate x) * up x)
 *   get_logits              :678-693  tied lm_head, then logit_softcap!
 *                                     (CommonOps.jl:326-333)
 *   compute_per_layer_inputs! / per_layer_input_forward! (:459-533, :626-634):
 *                                     per-layer inputs when the config's pli > 0
 *                                     (config 5 has none): per token, per layer
 *                                     (RMSNorm(proj_i) + table_i sqrt(pli)) 2^-1/2;
 *                                     after each MLP block
 *                                     x += RMSNorm(proj(gelu_tanh(gate x) * pli_i)),
 *                                     before the layer scalar
 * Matrix-vector products accumulate in f32 in index order (activation mode
 * 0, default: the GPU engine's exact f32 activations).  In mode 1 those with
 * K-quant weights (Q4_K/Q5_K/Q6_K) follow the reference's quantized kernels:
 * the activation vector is quantized to Q8_K first (quantize_row_q8_K,
 * src/kernels/quant_kernels.c:166-194, then q4_k_gemv .. q6_k_gemv :602-650)
 * and the products are summed per 256 block in double.
 */
#define _GNU_SOURCE
#include "oracle.h"
#include <math.h>
#include <stdint.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

typedef struct {
    int ssm;
    float *attn_norm, *post_norm;
    float *ffn_norm, *post_ffw_norm, *layer_scalar;   /* Gemma4 */
    float *pli_gate, *pli_proj, *pli_post_norm;       /* Gemma4 per-layer inputs */
    /* ssm */
    float *in_proj, *gate_proj, *ssm_out, *conv_w, *alpha_w, *beta_w, *ssm_a, *dt_bias, *ssm_norm;
    float *conv_state, *h;                  /* [C][K], [heads][vd][kd] */
    /* attention */
    float *wq, *wk, *wv, *wo, *q_norm, *k_norm;
    float *kc, *vc;                         /* [max_ctx][n_kv][hd] */
    /* mlp */
    float *ffn_gate, *ffn_up, *ffn_down;
} or_layer;

struct or_model {
    or_model_config c;
    or_layer *layers;
    or_layer mtp_layer;
    float *embed;        /* [vocab][d] dequantized */
    float *final_norm;
    float *mtp_fc, *mtp_norm_e, *mtp_norm_h, *mtp_norm;
    float *cos_cache, *sin_cache;   /* [max_ctx][half] */
    int conv_channels, inner, qk;
    const float *kq[1024];          /* weight slots holding K-quant matrices */
    int nkq;
    int act;                        /* K-quant activation mode: 0 exact f32, 1 Q8_K */
    int kv_bf16;                    /* cached keys / values rounded to bf16 */
    int gemma;                      /* Gemma4 block semantics */
    or_gemma_config g;
    float *cos_swa, *sin_swa, *cos_full, *sin_full;   /* [max_ctx][hd/2] */
    float *pli_token_embd, *pli_model_proj, *pli_proj_norm;  /* Gemma4 per-layer inputs */
    float *pli_in;                                   /* [n_layers][pli] of the current token */
};

static void *xcalloc(size_t n, size_t s) { void *p = calloc(n, s); if (!p) abort(); return p; }

or_model *or_model_new(const or_model_config *c) {
    or_model *m = (or_model *)xcalloc(1, sizeof(or_model));
    m->c = *c;
    m->inner = c->ssm_heads * c->ssm_head_dim;
    m->qk = c->ssm_heads * c->ssm_head_dim;
    m->conv_channels = m->inner + 2 * m->qk;
    m->layers = (or_layer *)xcalloc(c->n_layers, sizeof(or_layer));
    m->act = 0;
    int half = c->rotary_dim / 2;
    m->cos_cache = (float *)xcalloc((size_t)c->max_ctx * half, 4);
    m->sin_cache = (float *)xcalloc((size_t)c->max_ctx * half, 4);
    for (int i = 0; i < half; i++) {
        /* 1.0 / (theta ^ (2(i-1)/rd)) in Float64, stored as Float32 (ModelCPU.jl:139) */
        float inv = (float)(1.0 / pow((double)c->rope_theta, (double)(2 * i) / (double)c->rotary_dim));
        for (int p = 0; p < c->max_ctx; p++) {
            float ang = inv * (float)p;
            m->cos_cache[(size_t)p * half + i] = cosf(ang);
            m->sin_cache[(size_t)p * half + i] = sinf(ang);
        }
    }
    return m;
}

static void free_layer(or_layer *L) {
    float **f[] = {&L->attn_norm, &L->post_norm, &L->in_proj, &L->gate_proj, &L->ssm_out, &L->conv_w,
                   &L->alpha_w, &L->beta_w, &L->ssm_a, &L->dt_bias, &L->ssm_norm, &L->conv_state, &L->h,
                   &L->wq, &L->wk, &L->wv, &L->wo, &L->q_norm, &L->k_norm, &L->kc, &L->vc,
                   &L->ffn_gate, &L->ffn_up, &L->ffn_down, &L->ffn_norm, &L->post_ffw_norm, &L->layer_scalar,
                   &L->pli_gate, &L->pli_proj, &L->pli_post_norm};
    for (size_t i = 0; i < sizeof f / sizeof f[0]; i++) { free(*f[i]); *f[i] = NULL; }
}

void or_model_free(or_model *m) {
    if (!m) return;
    for (int i = 0; i < m->c.n_layers; i++) free_layer(&m->layers[i]);
    free_layer(&m->mtp_layer);
    free(m->layers);
    free(m->embed); free(m->final_norm); free(m->mtp_fc); free(m->mtp_norm_e); free(m->mtp_norm_h);
    free(m->mtp_norm); free(m->cos_cache); free(m->sin_cache);
    free(m->cos_swa); free(m->sin_swa); free(m->cos_full); free(m->sin_full);
    free(m->pli_token_embd); free(m->pli_model_proj); free(m->pli_proj_norm); free(m->pli_in);
    free(m);
}

/* tensor slots, addressed by (layer, kind); layer -1 = global, -2 = MTP layer */
static float **slot(or_model *m, int layer, int kind) {
    or_layer *L = layer >= 0 ? &m->layers[layer] : (layer == -2 ? &m->mtp_layer : NULL);
    if (!L) {
        switch (kind) {
        case OR_T_EMBED: return &m->embed;
        case OR_T_FINAL_NORM: return &m->final_norm;
        case OR_T_MTP_FC: return &m->mtp_fc;
        case OR_T_MTP_NORM_E: return &m->mtp_norm_e;
        case OR_T_MTP_NORM_H: return &m->mtp_norm_h;
        case OR_T_MTP_NORM: return &m->mtp_norm;
        case OR_T_PLI_TOKEN_EMBD: return &m->pli_token_embd;
        case OR_T_PLI_MODEL_PROJ: return &m->pli_model_proj;
        case OR_T_PLI_PROJ_NORM: return &m->pli_proj_norm;
        }
        return NULL;
    }
    switch (kind) {
    case OR_T_ATTN_NORM: return &L->attn_norm;
    case OR_T_POST_NORM: return &L->post_norm;
    case OR_T_IN_PROJ: return &L->in_proj;
    case OR_T_GATE_PROJ: return &L->gate_proj;
    case OR_T_SSM_OUT: return &L->ssm_out;
    case OR_T_CONV: return &L->conv_w;
    case OR_T_ALPHA: return &L->alpha_w;
    case OR_T_BETA: return &L->beta_w;
    case OR_T_SSM_A: return &L->ssm_a;
    case OR_T_DT_BIAS: return &L->dt_bias;
    case OR_T_SSM_NORM: return &L->ssm_norm;
    case OR_T_WQ: return &L->wq;
    case OR_T_WK: return &L->wk;
    case OR_T_WV: return &L->wv;
    case OR_T_WO: return &L->wo;
    case OR_T_Q_NORM: return &L->q_norm;
    case OR_T_K_NORM: return &L->k_norm;
    case OR_T_FFN_GATE: return &L->ffn_gate;
    case OR_T_FFN_UP: return &L->ffn_up;
    case OR_T_FFN_DOWN: return &L->ffn_down;
    case OR_T_FFN_NORM: return &L->ffn_norm;
    case OR_T_POST_FFW_NORM: return &L->post_ffw_norm;
    case OR_T_LAYER_SCALAR: return &L->layer_scalar;
    case OR_T_PLI_GATE: return &L->pli_gate;
    case OR_T_PLI_PROJ: return &L->pli_proj;
    case OR_T_PLI_POST_NORM: return &L->pli_post_norm;
    }
    return NULL;
}

/* raw GGUF bytes of `type` with n elements -> f32 slot (dequantized) */
int or_model_set(or_model *m, int layer, int kind, int type, const void *data, int64_t n) {
    float **s = slot(m, layer, kind);
    if (!s) return -1;
    for (int i = 0; i < m->nkq; i++)
        if (m->kq[i] == *s) m->kq[i] = m->kq[--m->nkq];
    free(*s);
    *s = (float *)malloc((size_t)n * 4);
    if (!*s) return -2;
    if (or_dequantize(type, (const uint8_t *)data, n, *s)) return -1;
    if ((type == OR_Q4_K || type == OR_Q5_K || type == OR_Q6_K) && m->nkq < 1024) m->kq[m->nkq++] = *s;
    if (layer != -1 && kind == OR_T_SSM_A) {
        or_layer *L = layer >= 0 ? &m->layers[layer] : &m->mtp_layer;
        L->ssm = 1;
    }
    return 0;
}

static void alloc_state(or_model *m, or_layer *L) {
    const or_model_config *c = &m->c;
    if (L->ssm) {
        if (!L->conv_state) L->conv_state = (float *)xcalloc((size_t)m->conv_channels * c->conv_kernel, 4);
        if (!L->h) L->h = (float *)xcalloc((size_t)c->ssm_heads * c->ssm_head_dim * c->ssm_head_dim, 4);
    } else {
        size_t kv = (size_t)c->max_ctx * c->n_kv_head * c->head_dim;
        if (!L->kc) L->kc = (float *)xcalloc(kv, 4);
        if (!L->vc) L->vc = (float *)xcalloc(kv, 4);
    }
}

void or_model_reset(or_model *m) {
    for (int i = 0; i < m->c.n_layers; i++) {
        or_layer *L = &m->layers[i];
        alloc_state(m, L);
        if (L->ssm) {
            memset(L->conv_state, 0, (size_t)m->conv_channels * m->c.conv_kernel * 4);
            memset(L->h, 0, (size_t)m->c.ssm_heads * m->c.ssm_head_dim * m->c.ssm_head_dim * 4);
        }
    }
    if (m->mtp_fc) {
        /* the MTP layer attends over positions that only its drafts write:
           zeros until then, as after allocation */
        or_layer *L = &m->mtp_layer;
        alloc_state(m, L);
        const size_t kv = (size_t)m->c.max_ctx * m->c.n_kv_head * m->c.head_dim * 4;
        memset(L->kc, 0, kv);
        memset(L->vc, 0, kv);
    }
}

/* ---------------- building blocks ---------------- */

static void rmsnorm(float *out, const float *x, const float *w, int n, float eps) {
    float ss = 0.f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    float scale = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; i++) out[i] = x[i] * scale * w[i];
}

/* rows split over threads; every row keeps its own index-order sum */
typedef struct { float *y; const float *W, *x; int r0, r1, cols; } mv_job;
static void *mv_run(void *p) {
    mv_job *j = (mv_job *)p;
    for (int r = j->r0; r < j->r1; r++) {
        const float *w = j->W + (size_t)r * j->cols;
        float acc = 0.f;
        for (int k = 0; k < j->cols; k++) acc += w[k] * j->x[k];
        j->y[r] = acc;
    }
    return NULL;
}
static void matvec(float *y, const float *W, const float *x, int rows, int cols) {
    int nt = (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (nt > 32) nt = 32;
    if (nt < 1 || (size_t)rows * cols < (1u << 18)) nt = 1;
    mv_job jobs[32];
    pthread_t th[32];
    for (int i = 0; i < nt; i++) {
        jobs[i] = (mv_job){y, W, x, (int)((int64_t)rows * i / nt), (int)((int64_t)rows * (i + 1) / nt), cols};
        if (nt > 1) pthread_create(&th[i], NULL, mv_run, &jobs[i]);
        else mv_run(&jobs[i]);
    }
    if (nt > 1)
        for (int i = 0; i < nt; i++) pthread_join(th[i], NULL);
}

/* K-quant weights with Q8_K activations, per-block sums in double */
typedef struct { float *y; const float *W; const float *d1; const int8_t *q1; int r0, r1, cols; } mq_job;
static void *mq_run(void *p) {
    mq_job *j = (mq_job *)p;
    const int nb = j->cols / 256;
    for (int r = j->r0; r < j->r1; r++) {
        const float *w = j->W + (size_t)r * j->cols;
        double acc = 0.0;
        for (int b = 0; b < nb; b++) {
            double s1 = 0.0;
            for (int k = 0; k < 256; k++) s1 += (double)w[256 * b + k] * (double)j->q1[256 * b + k];
            acc += (double)j->d1[b] * s1;
        }
        j->y[r] = (float)acc;
    }
    return NULL;
}
static void matvec_w(or_model *m, float *y, const float *W, const float *x, int rows, int cols) {
    int kq = 0;
    for (int i = 0; i < m->nkq; i++) kq |= m->kq[i] == W;
    if (!kq || cols % 256 || m->act == 0) {
        matvec(y, W, x, rows, cols);
        return;
    }
    float *d1 = (float *)xcalloc((size_t)cols / 256, 4);
    int8_t *q1 = (int8_t *)xcalloc((size_t)cols, 1);
    or_quantize_q8k(x, cols, d1, q1);
    int nt = (int)sysconf(_SC_NPROCESSORS_ONLN);
    if (nt > 32) nt = 32;
    if (nt < 1 || (size_t)rows * cols < (1u << 18)) nt = 1;
    mq_job jobs[32];
    pthread_t th[32];
    for (int i = 0; i < nt; i++) {
        jobs[i] = (mq_job){y, W, d1, q1, (int)((int64_t)rows * i / nt), (int)((int64_t)rows * (i + 1) / nt), cols};
        if (nt > 1) pthread_create(&th[i], NULL, mq_run, &jobs[i]);
        else mq_run(&jobs[i]);
    }
    if (nt > 1)
        for (int i = 0; i < nt; i++) pthread_join(th[i], NULL);
    free(d1);
    free(q1);
}

void or_model_set_activation(or_model *m, int mode) { m->act = mode; }
void or_model_set_kv_bf16(or_model *m, int on) { m->kv_bf16 = on != 0; }

/* f32 -> bf16 -> f32, round to nearest even on the upper 16 bits (NaN kept quiet) */
static float bf16_round(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) {
        if (u & 0x007fffffu) u |= 0x00400000u;
        u &= 0xffff0000u;
    } else {
        u += 0x7fffu + ((u >> 16) & 1u);
        u &= 0xffff0000u;
    }
    memcpy(&x, &u, 4);
    return x;
}
/* the n cached key and value elements of one position, as the cache stores them */
static void kv_store(const or_model *m, float *kc, float *vc, const float *k, const float *v, size_t n) {
    for (size_t i = 0; i < n; i++) {
        kc[i] = m->kv_bf16 ? bf16_round(k[i]) : k[i];
        vc[i] = m->kv_bf16 ? bf16_round(v[i]) : v[i];
    }
}

static inline float silu(float g) { return g / (1.0f + expf(-g)); }

/* GatedDeltaNetCPU (ModelCPU.jl:566-731) */
static void ssm_forward(or_model *m, or_layer *L, const float *x, float *out) {
    const or_model_config *c = &m->c;
    const int C = m->conv_channels, K = c->conv_kernel, H = c->ssm_heads, dk = c->ssm_head_dim,
              dv = c->ssm_head_dim, inner = m->inner, d = c->hidden;
    float *qkv = (float *)malloc(C * 4), *z = (float *)malloc(inner * 4), *xc = (float *)malloc(C * 4);
    float *al = (float *)malloc(H * 4), *be = (float *)malloc(H * 4), *y = (float *)malloc(inner * 4);
    float *qn = (float *)malloc(dk * 4), *kn = (float *)malloc(dk * 4), *sk = (float *)malloc(dv * 4);
    matvec_w(m, qkv, L->in_proj, x, C, d);
    matvec_w(m, z, L->gate_proj, x, inner, d);
    for (int j = 0; j < K - 1; j++)
        for (int i = 0; i < C; i++) L->conv_state[(size_t)i * K + j] = L->conv_state[(size_t)i * K + j + 1];
    for (int i = 0; i < C; i++) L->conv_state[(size_t)i * K + K - 1] = qkv[i];
    for (int ch = 0; ch < C; ch++) {
        float v = 0.f;
        for (int k = 0; k < K; k++) v += L->conv_state[(size_t)ch * K + k] * L->conv_w[(size_t)ch * K + k];
        xc[ch] = v / (1.0f + expf(-v));
    }
    matvec_w(m, al, L->alpha_w, x, H, d);
    matvec_w(m, be, L->beta_w, x, H, d);
    const float eps = 1e-6f, scale = 1.0f / sqrtf((float)dk);
    for (int h = 0; h < H; h++) {
        int g = h % H;  /* num_k_heads == num_v_heads */
        const float *qg = xc + g * dk, *kg = xc + m->qk + g * dk, *vg = xc + 2 * m->qk + h * dv;
        float qs = 0.f, ks = 0.f;
        for (int i = 0; i < dk; i++) { qs += qg[i] * qg[i]; ks += kg[i] * kg[i]; }
        float qnv = 1.0f / (sqrtf(qs) + eps) * scale, knv = 1.0f / (sqrtf(ks) + eps);
        for (int i = 0; i < dk; i++) { qn[i] = qg[i] * qnv; kn[i] = kg[i] * knv; }
        double av = (double)al[h] + (double)L->dt_bias[h];
        av = av < -20.0 ? -20.0 : (av > 20.0 ? 20.0 : av);
        double sp = log(1.0 + exp(av));
        float decay = (float)((double)L->ssm_a[h] * sp);
        float dta = expf(decay);
        double bv = (double)be[h];
        bv = bv < -20.0 ? -20.0 : (bv > 20.0 ? 20.0 : bv);
        float bg = (float)(1.0 / (1.0 + exp(-bv)));
        float *S = L->h + (size_t)h * dv * dk;    /* S[i][j], i = v index */
        for (int i = 0; i < dv * dk; i++) S[i] *= dta;
        for (int i = 0; i < dv; i++) {
            float s = 0.f;
            for (int j = 0; j < dk; j++) s += S[(size_t)i * dk + j] * kn[j];
            sk[i] = s;
        }
        for (int i = 0; i < dv; i++) {
            float di = bg * (vg[i] - sk[i]);
            for (int j = 0; j < dk; j++) S[(size_t)i * dk + j] += di * kn[j];
        }
        for (int i = 0; i < dv; i++) {
            float s = 0.f;
            for (int j = 0; j < dk; j++) s += S[(size_t)i * dk + j] * qn[j];
            y[h * dv + i] = s;
        }
    }
    for (int h = 0; h < H; h++) rmsnorm(y + h * dv, y + h * dv, L->ssm_norm, dv, c->rms_eps);
    for (int i = 0; i < inner; i++) y[i] = y[i] * z[i] * (1.0f / (1.0f + expf(-z[i])));
    matvec_w(m, out, L->ssm_out, y, d, inner);
    free(qkv); free(z); free(xc); free(al); free(be); free(y); free(qn); free(kn); free(sk);
}

static void rmsnorm_rope(or_model *m, float *x, int nheads, int hd, const float *w, int pos) {
    int half = m->c.rotary_dim / 2;
    const float *cs = m->cos_cache + (size_t)pos * half, *sn = m->sin_cache + (size_t)pos * half;
    for (int h = 0; h < nheads; h++) {
        float *v = x + h * hd;
        float ss = 0.f;
        for (int i = 0; i < hd; i++) ss += v[i] * v[i];
        float inv = 1.0f / sqrtf(ss / (float)hd + m->c.rms_eps);
        for (int i = 0; i < hd; i++) v[i] = v[i] * inv * w[i];
        for (int i = 0; i < half; i++) {
            float x1 = v[i], x2 = v[i + half];
            v[i] = x1 * cs[i] - x2 * sn[i];
            v[i + half] = x1 * sn[i] + x2 * cs[i];
        }
    }
}

/* flash_attention_cpu! (FlashAttention.jl:19-84) for one query */
static void flash_attn(float *out, const float *q, const float *kc, const float *vc, int kvh, int nkv,
                       int seq, float scale, int hd) {
    float scores[64];
    float mx = -INFINITY, l = 0.f;
    for (int d = 0; d < hd; d++) out[d] = 0.f;
    for (int j = 0; j < seq; j += 64) {
        int je = j + 64 < seq ? j + 64 : seq, bl = je - j;
        float mn = mx;
        for (int n = 0; n < bl; n++) {
            const float *k = kc + ((size_t)(j + n) * nkv + kvh) * hd;
            float s = 0.f;
            for (int d = 0; d < hd; d++) s += q[d] * k[d];
            float sc = s * scale;
            scores[n] = sc;
            if (sc > mn) mn = sc;
        }
        float sf = expf(mx - mn);
        if (mn > mx) {
            for (int d = 0; d < hd; d++) out[d] *= sf;
            l *= sf;
        }
        for (int n = 0; n < bl; n++) {
            const float *v = vc + ((size_t)(j + n) * nkv + kvh) * hd;
            float p = expf(scores[n] - mn);
            l += p;
            for (int d = 0; d < hd; d++) out[d] += p * v[d];
        }
        mx = mn;
    }
    float il = 1.0f / l;
    for (int d = 0; d < hd; d++) out[d] *= il;
}

/* FullAttentionCPU (ModelCPU.jl:787-887) */
static void attn_forward(or_model *m, or_layer *L, const float *x, int pos, float *out) {
    const or_model_config *c = &m->c;
    const int nh = c->n_head, nkv = c->n_kv_head, hd = c->head_dim, d = c->hidden;
    float *qg = (float *)malloc((size_t)2 * nh * hd * 4), *k = (float *)malloc((size_t)nkv * hd * 4);
    float *v = (float *)malloc((size_t)nkv * hd * 4), *q = (float *)malloc((size_t)nh * hd * 4);
    float *gate = (float *)malloc((size_t)nh * hd * 4), *o = (float *)malloc((size_t)nh * hd * 4);
    matvec_w(m, qg, L->wq, x, 2 * nh * hd, d);
    matvec_w(m, k, L->wk, x, nkv * hd, d);
    matvec_w(m, v, L->wv, x, nkv * hd, d);
    for (int h = 0; h < nh; h++)
        for (int i = 0; i < hd; i++) {
            q[h * hd + i] = qg[(size_t)h * 2 * hd + i];
            gate[h * hd + i] = qg[(size_t)h * 2 * hd + hd + i];
        }
    rmsnorm_rope(m, q, nh, hd, L->q_norm, pos);
    rmsnorm_rope(m, k, nkv, hd, L->k_norm, pos);
    kv_store(m, L->kc + (size_t)pos * nkv * hd, L->vc + (size_t)pos * nkv * hd, k, v, (size_t)nkv * hd);
    const int ratio = nh / nkv;
    const float scale = 1.0f / sqrtf((float)hd);
    for (int h = 0; h < nh; h++) flash_attn(o + h * hd, q + h * hd, L->kc, L->vc, h / ratio, nkv, pos + 1, scale, hd);
    for (int i = 0; i < nh * hd; i++) o[i] *= 1.0f / (1.0f + expf(-gate[i]));
    matvec_w(m, out, L->wo, o, d, nh * hd);
    free(qg); free(k); free(v); free(q); free(gate); free(o);
}

static void mlp_forward(or_model *m, or_layer *L, const float *x, float *out) {
    const int f = m->c.ffn, d = m->c.hidden;
    float *g = (float *)malloc(f * 4), *u = (float *)malloc(f * 4);
    matvec_w(m, g, L->ffn_gate, x, f, d);
    for (int i = 0; i < f; i++) g[i] = g[i] / (1.0f + expf(-g[i]));
    matvec_w(m, u, L->ffn_up, x, f, d);
    for (int i = 0; i < f; i++) g[i] = g[i] * u[i];
    matvec_w(m, out, L->ffn_down, g, d, f);
    free(g); free(u);
}

static void decoder_layer(or_model *m, or_layer *L, float *x, int pos) {
    const int d = m->c.hidden;
    float *xn = (float *)malloc(d * 4), *r = (float *)malloc(d * 4);
    rmsnorm(xn, x, L->attn_norm, d, m->c.rms_eps);
    if (L->ssm) ssm_forward(m, L, xn, r);
    else attn_forward(m, L, xn, pos, r);
    for (int i = 0; i < d; i++) x[i] += r[i];
    rmsnorm(xn, x, L->post_norm, d, m->c.rms_eps);
    mlp_forward(m, L, xn, r);
    for (int i = 0; i < d; i++) x[i] += r[i];
    free(xn); free(r);
}

/* ---------------- Gemma4 blocks (src/Gemma4.jl) ---------------- */

/* precompute_rope (:205-249): inverse frequencies and angles in Float64,
   cos / sin stored as Float32; pair k rotates dims (k, k + hd/2) */
void or_model_set_gemma(or_model *m, const or_gemma_config *g) {
    m->gemma = 1;
    m->g = *g;
    free(m->pli_in);
    m->pli_in = g->pli > 0 ? (float *)xcalloc((size_t)m->c.n_layers * g->pli, 4) : NULL;
    const int hd = m->c.head_dim, half = hd / 2, T = m->c.max_ctx;
    const int angles = (int)(g->partial_rotary_factor * (float)hd) / 2;  /* Int(partial * hd / 2) */
    free(m->cos_swa); free(m->sin_swa); free(m->cos_full); free(m->sin_full);
    m->cos_swa = (float *)xcalloc((size_t)T * half, 4);
    m->sin_swa = (float *)xcalloc((size_t)T * half, 4);
    m->cos_full = (float *)xcalloc((size_t)T * half, 4);
    m->sin_full = (float *)xcalloc((size_t)T * half, 4);
    for (int k = 0; k < half; k++) {
        const double fs = 1.0 / pow((double)g->rope_theta_swa, 2.0 * k / (double)hd);
        const double ff = k < angles ? 1.0 / pow((double)g->rope_theta_full, 2.0 * k / (double)hd) : 0.0;
        for (int p = 0; p < T; p++) {
            m->cos_swa[(size_t)p * half + k] = (float)cos(p * fs);
            m->sin_swa[(size_t)p * half + k] = (float)sin(p * fs);
            m->cos_full[(size_t)p * half + k] = (float)cos(p * ff);
            m->sin_full[(size_t)p * half + k] = (float)sin(p * ff);
        }
    }
}

static int gemma_sliding(const or_model *m, int layer) {
    return m->g.sliding_pattern <= 0 || (layer + 1) % m->g.sliding_pattern != 0;
}

/* gelu_tanh (:253-257) */
static inline float gelu_tanh(float x) {
    const float c = sqrtf(2.0f / (float)M_PI);
    return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
}

/* apply_rope! (:263-293) on nheads heads with the layer's table */
static void gemma_rope(float *x, int nheads, int hd, const float *cs, const float *sn) {
    const int half = hd / 2;
    for (int h = 0; h < nheads; h++) {
        float *v = x + (size_t)h * hd;
        for (int k = 0; k < half; k++) {
            const float q0 = v[k], q1 = v[k + half];
            v[k] = q0 * cs[k] - q1 * sn[k];
            v[k + half] = q0 * sn[k] + q1 * cs[k];
        }
    }
}

/* attention_forward! (:296-456) for one token at pos */
static void gemma_attn(or_model *m, or_layer *L, int layer, const float *x, int pos, float *out) {
    const or_model_config *c = &m->c;
    const int nh = c->n_head, nkv = c->n_kv_head, hd = c->head_dim, d = c->hidden, half = hd / 2;
    const int sliding = gemma_sliding(m, layer);
    const float *cs = (sliding ? m->cos_swa : m->cos_full) + (size_t)pos * half;
    const float *sn = (sliding ? m->sin_swa : m->sin_full) + (size_t)pos * half;
    float *q = (float *)malloc((size_t)nh * hd * 4), *k = (float *)malloc((size_t)nkv * hd * 4);
    float *v = (float *)malloc((size_t)nkv * hd * 4), *o = (float *)malloc((size_t)nh * hd * 4);
    float *sc = (float *)malloc((size_t)(pos + 1) * 4);
    matvec_w(m, q, L->wq, x, nh * hd, d);
    for (int h = 0; h < nh; h++) rmsnorm(q + (size_t)h * hd, q + (size_t)h * hd, L->q_norm, hd, c->rms_eps);
    gemma_rope(q, nh, hd, cs, sn);
    matvec_w(m, k, L->wk, x, nkv * hd, d);
    matvec_w(m, v, L->wv, x, nkv * hd, d);
    for (int h = 0; h < nkv; h++) {  /* rmsnorm_no_scale! (CommonOps.jl:43-53) */
        float *vh = v + (size_t)h * hd, ss = 0.f;
        for (int i = 0; i < hd; i++) ss += vh[i] * vh[i];
        const float inv = 1.0f / sqrtf(ss / (float)hd + c->rms_eps);
        for (int i = 0; i < hd; i++) vh[i] = vh[i] * inv;
    }
    for (int h = 0; h < nkv; h++) rmsnorm(k + (size_t)h * hd, k + (size_t)h * hd, L->k_norm, hd, c->rms_eps);
    gemma_rope(k, nkv, hd, cs, sn);
    kv_store(m, L->kc + (size_t)pos * nkv * hd, L->vc + (size_t)pos * nkv * hd, k, v, (size_t)nkv * hd);
    const int start = sliding && m->g.window > 0 ? (pos + 1 - m->g.window > 0 ? pos + 1 - m->g.window : 0) : 0;
    const int ratio = nh / nkv;
    const float cap = m->g.attn_softcap;
    for (int h = 0; h < nh; h++) {
        const int kvh = h / ratio;
        const float *qh = q + (size_t)h * hd;
        float mx = -INFINITY;
        for (int t = start; t <= pos; t++) {
            const float *kt = L->kc + ((size_t)t * nkv + kvh) * hd;
            float s = 0.f;
            for (int i = 0; i < hd; i++) s += qh[i] * kt[i];
            if (cap > 0.f) s = tanhf(s / cap) * cap;
            sc[t - start] = s;
            if (s > mx) mx = s;
        }
        float sum = 0.f;
        for (int t = start; t <= pos; t++) {
            sc[t - start] = expf(sc[t - start] - mx);
            sum += sc[t - start];
        }
        const float inv = 1.0f / sum;
        float *oh = o + (size_t)h * hd;
        for (int i = 0; i < hd; i++) oh[i] = 0.f;
        for (int t = start; t <= pos; t++) {
            const float w = sc[t - start] * inv;
            const float *vt = L->vc + ((size_t)t * nkv + kvh) * hd;
            for (int i = 0; i < hd; i++) oh[i] += w * vt[i];
        }
    }
    matvec_w(m, out, L->wo, o, d, nh * hd);
    free(q); free(k); free(v); free(o); free(sc);
}

/* mlp_forward! (:556-581) */
static void gemma_mlp(or_model *m, or_layer *L, const float *x, float *out) {
    const int f = m->c.ffn, d = m->c.hidden;
    float *g = (float *)malloc(f * 4), *u = (float *)malloc(f * 4);
    matvec_w(m, g, L->ffn_gate, x, f, d);
    for (int i = 0; i < f; i++) g[i] = gelu_tanh(g[i]);
    matvec_w(m, u, L->ffn_up, x, f, d);
    for (int i = 0; i < f; i++) g[i] = g[i] * u[i];
    matvec_w(m, out, L->ffn_down, g, d, f);
    free(g); free(u);
}

/* compute_per_layer_inputs! (:459-503) for the token: per layer i,
   (RMSNorm(proj_i, w) + table_row_i * sqrt(pli)) * 2^-1/2, proj = the model
   projection (pre-scaled) of the scaled embedding x */
static void gemma_pli_inputs(or_model *m, int token, const float *x) {
    const int P = m->g.pli, n = m->c.n_layers, d = m->c.hidden;
    float *proj = (float *)malloc((size_t)n * P * 4);
    matvec_w(m, proj, m->pli_model_proj, x, n * P, d);
    const float scale = sqrtf((float)P), in_scale = (float)pow(2.0, -0.5);
    const float *row = m->pli_token_embd + (size_t)token * n * P;
    for (int i = 0; i < n; i++) {
        float *o = m->pli_in + (size_t)i * P;
        rmsnorm(o, proj + (size_t)i * P, m->pli_proj_norm, P, m->c.rms_eps);
        for (int j = 0; j < P; j++) o[j] = (o[j] + row[(size_t)i * P + j] * scale) * in_scale;
    }
    free(proj);
}

/* per_layer_input_forward! (:505-533): x += RMSNorm(proj(gelu_tanh(gate x) * pli_i)) */
static void gemma_pli_block(or_model *m, or_layer *L, int layer, float *x) {
    const int P = m->g.pli, d = m->c.hidden;
    float *g = (float *)malloc((size_t)P * 4), *o = (float *)malloc((size_t)d * 4);
    matvec_w(m, g, L->pli_gate, x, P, d);
    const float *pl = m->pli_in + (size_t)layer * P;
    for (int j = 0; j < P; j++) g[j] = gelu_tanh(g[j]);
    for (int j = 0; j < P; j++) g[j] *= pl[j];
    matvec_w(m, o, L->pli_proj, g, d, P);
    rmsnorm(o, o, L->pli_post_norm, d, m->c.rms_eps);
    for (int i = 0; i < d; i++) x[i] = x[i] + o[i];
    free(g); free(o);
}

/* the layer body of forward! (:622-650) */
static void gemma_layer(or_model *m, or_layer *L, int layer, float *x, int pos) {
    const int d = m->c.hidden;
    const float eps = m->c.rms_eps;
    float *xn = (float *)malloc(d * 4), *r = (float *)malloc(d * 4);
    rmsnorm(xn, x, L->attn_norm, d, eps);
    gemma_attn(m, L, layer, xn, pos, r);
    rmsnorm(r, r, L->post_norm, d, eps);
    for (int i = 0; i < d; i++) x[i] = r[i] + x[i];
    rmsnorm(xn, x, L->ffn_norm, d, eps);
    gemma_mlp(m, L, xn, r);
    rmsnorm(r, r, L->post_ffw_norm, d, eps);
    for (int i = 0; i < d; i++) x[i] = x[i] + r[i];
    if (m->g.pli > 0 && L->pli_gate) gemma_pli_block(m, L, layer, x);
    const float s = L->layer_scalar ? L->layer_scalar[0] : 1.0f;
    for (int i = 0; i < d; i++) x[i] *= s;
    free(xn); free(r);
}

static int gemma_forward_token(or_model *m, int token, int pos, float *logits, float *hidden) {
    const or_model_config *c = &m->c;
    const int d = c->hidden;
    float *x = (float *)malloc(d * 4), *xn = (float *)malloc(d * 4);
    for (int i = 0; i < d; i++) x[i] = m->embed[(size_t)token * d + i] * m->g.embed_scale;
    if (m->g.pli > 0) gemma_pli_inputs(m, token, x);
    for (int i = 0; i < c->n_layers; i++) gemma_layer(m, &m->layers[i], i, x, pos);
    rmsnorm(xn, x, m->final_norm, d, c->rms_eps);
    if (hidden) memcpy(hidden, xn, d * 4);
    if (logits) {
        matvec_w(m, logits, m->embed, xn, c->vocab, d);
        const float cap = m->g.final_softcap;
        if (cap > 0.f)
            for (int i = 0; i < c->vocab; i++) logits[i] = tanhf(logits[i] / cap) * cap;
    }
    free(x); free(xn);
    return 0;
}

/* one token of forward_cpu!: logits (vocab) and the final-normed hidden (d) */
int or_forward_token(or_model *m, int token, int pos, float *logits, float *hidden) {
    const or_model_config *c = &m->c;
    if (token < 0 || token >= c->vocab || pos < 0 || pos >= c->max_ctx) return -1;
    if (m->gemma) return gemma_forward_token(m, token, pos, logits, hidden);
    const int d = c->hidden;
    float *x = (float *)malloc(d * 4), *xn = (float *)malloc(d * 4);
    memcpy(x, m->embed + (size_t)token * d, d * 4);
    for (int i = 0; i < c->n_layers; i++) decoder_layer(m, &m->layers[i], x, pos);
    rmsnorm(xn, x, m->final_norm, d, c->rms_eps);
    if (hidden) memcpy(hidden, xn, d * 4);
    if (logits) matvec_w(m, logits, m->embed, xn, c->vocab, d);
    free(x); free(xn);
    return 0;
}

/* one MTP draft step: token embedding + hidden -> logits (vocab), next hidden (d) */
int or_mtp_step(or_model *m, int token, const float *hidden, int pos, float *logits, float *hidden_out) {
    const or_model_config *c = &m->c;
    if (!m->mtp_fc || token < 0 || token >= c->vocab || pos < 0 || pos >= c->max_ctx) return -1;
    const int d = c->hidden;
    float *cat = (float *)malloc(2 * d * 4), *x = (float *)malloc(d * 4), *xn = (float *)malloc(d * 4);
    rmsnorm(cat, m->embed + (size_t)token * d, m->mtp_norm_e, d, c->rms_eps);
    rmsnorm(cat + d, hidden, m->mtp_norm_h, d, c->rms_eps);
    matvec_w(m, x, m->mtp_fc, cat, d, 2 * d);
    decoder_layer(m, &m->mtp_layer, x, pos);
    if (hidden_out) memcpy(hidden_out, x, d * 4);
    rmsnorm(xn, x, m->mtp_norm, d, c->rms_eps);
    if (logits) matvec_w(m, logits, m->embed, xn, c->vocab, d);
    free(cat); free(x); free(xn);
    return 0;
}

/* state snapshot: SSM/conv states and the KV caches of all layers (incl. MTP) */
struct or_snapshot { float **bufs; size_t *sizes; int n; };

static int collect(or_model *m, float ***ptrs, size_t **sizes) {
    const or_model_config *c = &m->c;
    int n = 0, cap = 2 * (c->n_layers + 1);
    *ptrs = (float **)xcalloc(cap, sizeof(float *));
    *sizes = (size_t *)xcalloc(cap, sizeof(size_t));
    for (int i = -1; i < c->n_layers; i++) {
        or_layer *L = i < 0 ? &m->mtp_layer : &m->layers[i];
        if (i < 0 && !m->mtp_fc) continue;
        if (L->ssm) {
            (*ptrs)[n] = L->conv_state; (*sizes)[n++] = (size_t)m->conv_channels * c->conv_kernel;
            (*ptrs)[n] = L->h; (*sizes)[n++] = (size_t)c->ssm_heads * c->ssm_head_dim * c->ssm_head_dim;
        } else {
            size_t kv = (size_t)c->max_ctx * c->n_kv_head * c->head_dim;
            (*ptrs)[n] = L->kc; (*sizes)[n++] = kv;
            (*ptrs)[n] = L->vc; (*sizes)[n++] = kv;
        }
    }
    return n;
}

or_snapshot *or_snapshot_take(or_model *m) {
    or_snapshot *s = (or_snapshot *)xcalloc(1, sizeof(or_snapshot));
    float **p;
    s->n = collect(m, &p, &s->sizes);
    s->bufs = (float **)xcalloc(s->n, sizeof(float *));
    for (int i = 0; i < s->n; i++) {
        s->bufs[i] = (float *)malloc(s->sizes[i] * 4);
        memcpy(s->bufs[i], p[i], s->sizes[i] * 4);
    }
    free(p);
    return s;
}

void or_snapshot_restore(or_model *m, const or_snapshot *s) {
    float **p;
    size_t *sz;
    int n = collect(m, &p, &sz);
    for (int i = 0; i < n && i < s->n; i++) memcpy(p[i], s->bufs[i], s->sizes[i] * 4);
    free(p);
    free(sz);
}

void or_snapshot_free(or_snapshot *s) {
    if (!s) return;
    for (int i = 0; i < s->n; i++) free(s->bufs[i]);
    free(s->bufs);
    free(s->sizes);
    free(s);
}
