// Internal interface of the layer kernels (model.cu) used by the engine.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace ifr {

// device-resident scalars of one generation state (read by kernels, so a
// verify step needs no host round trip)
struct EngineScalars {
    int32_t pos;          // committed tokens in the caches = position of the next token
    int32_t a_prev;       // accepted drafts of the last call (-1: nothing to replay)
    int32_t last_token;   // emitted, not yet fed to the target
    int32_t last_accept;  // accept count of the last verify
    int32_t n_log;        // tokens in the emitted-token log
    int32_t steps;        // verify steps committed
    int32_t pad[2];
};

// Batched calls: blockIdx.z = request b; per-request data is offset by b
// times the b_* strides (elements), and a request's N columns of proj, xn and
// y start at column b * N.
struct SsmArgs {
    const float *proj;   // [N][ldp]: conv inputs q|k|v (C) then z (inner)
    int64_t ldp;
    const float *xn;     // [N][d] normalised layer input (alpha/beta projections), or
                         // the raw input when in_norm is set
    int d;
    const float *in_norm = nullptr;  // RMSNorm weights [d]: alpha/beta = rms(x)^-1 (ab_w . (x w))
    const float *conv_w; // [C][K]
    const float *ab_w;   // [2H][d]: alpha rows then beta rows
    const float *ssm_a, *dt_bias, *norm_w;
    float *S;            // [H][HD][HD] committed state
    float *hist;         // [K-1][C] committed conv inputs
    float *rq;           // [8][C] conv inputs of the last call's tokens
    float *rkv;          // [H][8][2HD+2] k, v, decay, beta of the last call's tokens
    const int32_t *a_prev;
    float *y;            // [N][ldy]
    int64_t ldy;
    int N, H, C, K;
    float eps;
    int64_t b_S = 0, b_hist = 0, b_rq = 0, b_rkv = 0;  // per-request strides
    int b_prev = 0;                                    // stride of a_prev (int32)
};

struct AttnArgs {
    const float *qkv;    // [N][ldq]: per head [q; gate] (2 nh hd; gated 0: q only, nh hd), then k (nkv hd), then v
    int64_t ldq;
    const float *q_norm, *k_norm;
    float *kc, *vc;      // [max_ctx][nkv][hd]
    const int32_t *pos;
    const float *rope_cos, *rope_sin;  // [max_ctx][rotary_dim/2]
    float *out;          // [N][ldo]
    int64_t ldo;
    int N, nh, nkv, hd, rotary_dim;
    float eps;
    int64_t b_kv = 0;    // per-request stride of kc / vc
    int b_pos = 0;       // stride of pos (int32)
    // split-KV path (attn_splits > 0): key slices per row group and the
    // scratch of their partial softmax states (attn_part_floats floats)
    int splits = 0;
    float *part = nullptr;
    // Gemma4 attention (src/Gemma4.jl:296-456); the defaults are the Qwen3.5
    // attention.  gated 0: q rows nh x hd (no per-head gate, no output gate);
    // vnorm 1: RMSNorm of v without weights; scale: score scale (0: 1/sqrt(hd));
    // softcap: scores become tanh(s / cap) cap (0: off); window: a query at
    // position p sees keys p - window + 1 .. p (0: all); RoPE pair i < rope_pairs
    // rotates dims (i, i + rope_off) with table entries [pos * rope_ld + i]
    // (0: rotary_dim / 2 for each)
    int gated = 1, vnorm = 0;
    float scale = 0.f, softcap = 0.f;
    int window = 0, rope_pairs = 0, rope_off = 0, rope_ld = 0;
    // 1: kc / vc hold bf16 rows (round to nearest even of the f32 rows); the
    // split-KV path only (attn_part_bf16_kernel)
    int kv16 = 0;
};

void rmsnorm(const float *x, const float *w, float *out, int rows, int n, float eps, int64_t ldx, int64_t ldo,
             cudaStream_t s);
void swiglu(const float *gu, float *h, int n, int ffn, cudaStream_t s);
// Gemma4 sub-block tail on `cols` columns of width n: x = (x + RMSNorm(y) w) * (*scalar or 1)
void norm_add(const float *y, const float *w, float *x, int cols, int n, float eps, const float *scalar,
              cudaStream_t s);
// l = tanh(l / cap) cap in place (final logit softcap)
void softcap(float *l, int64_t n, float cap, cudaStream_t s);
// Gemma4 per-layer inputs (compute_per_layer_inputs!, Gemma4.jl:459-503), nc
// columns: out[c][i P + j] = (RMSNorm(proj[c][i P ..], w)_j + emb[c][i P + j]
// sqrt(P)) 2^-1/2 for each of the L layers
cudaError_t pli_inputs(const float *proj, const float *emb, const float *w, int P, int L, int nc, float eps,
                       float *out, cudaStream_t s);
// per_layer_input_forward! (:514-524): g[c][j] = gelu_tanh(g[c][j]) pli[c][layer P + j]
cudaError_t pli_gate(float *g, const float *pli, int P, int64_t lp, int layer, int nc, cudaStream_t s);
cudaError_t ssm_step(const SsmArgs &a, int head_dim, int batch, cudaStream_t s);
// a prefill chunk of a.N <= 64 tokens of one request, committed at once (no
// replay record; the caller's commit must leave nothing to replay)
cudaError_t ssm_chunk(const SsmArgs &a, int head_dim, cudaStream_t s);
constexpr int kPrefillChunk = 64;
cudaError_t attn_step(const AttnArgs &a, int batch, cudaStream_t s);
// key slices of a split-KV call of N tokens per request, and the scratch
// (floats) that every call on a state of `batch` requests and max_ctx fits in
int attn_splits(int nh, int nkv, int N, int batch, int max_ctx);
int64_t attn_part_floats(int nh, int nkv, int hd, int batch, int max_ctx);
// per request b (grid of `batch` CTAs): sc + b, acc + b, out_tok + b * n,
// hid + b * n * d, mtp_h + b * d, log + b * log_cap.  all: 0 commit acc + 1
// verify tokens; 1 commit all n (prefill; the SSM layers replay them next
// call); 2 commit all n that the layers already committed (prefill chunks)
void commit(EngineScalars *sc, const int32_t *acc, const int32_t *out_tok, int n, int all, const float *hid,
            float *mtp_h, int d, int32_t *log, int log_cap, int batch, cudaStream_t s);
// dst[i] = sc->pos + step * i for i < count (<= 32)
void chunk_positions(int32_t *dst, const EngineScalars *sc, int count, int step, cudaStream_t s);
void set_token(int32_t *dst, const int32_t *src, cudaStream_t s);

}  // namespace ifr
