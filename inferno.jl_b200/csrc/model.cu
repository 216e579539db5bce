// Layer kernels of the Qwen3.5-hybrid verify step (N <= 8 tokens per call).
//
// Reference semantics: src/ModelCPU.jl of Inferno.jl (line numbers below).
// All arithmetic is f32 except the SSM gates, which the reference evaluates in
// f64 (:654-667) and so do we.
#include "common.cuh"
#include "model.cuh"

#include <math_constants.h>

namespace ifr {

constexpr int kMaxN = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// block-wide sum for 256 threads; `red` has >= 8 floats; all threads get it
__device__ __forceinline__ float block_sum256(float v, float *red) {
    v = warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; w++) s += red[w];
    return s;
}

// ------------------------------------------------------------- RMSNorm ------
// rmsnorm_cpu! (ModelCPU.jl:111-123): out = x * (1/sqrt(ss/n + eps)) * w
// one CTA per row; `out` may alias `x`
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                                      float *out, int n, float eps, int64_t ldx, int64_t ldo) {
    __shared__ float red[8];
    const float *xr = x + blockIdx.x * ldx;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += 256) ss += xr[i] * xr[i];
    ss = block_sum256(ss, red);
    const float scale = 1.0f / sqrtf(ss / (float)n + eps);
    float *orow = out + blockIdx.x * ldo;
    for (int i = threadIdx.x; i < n; i += 256) orow[i] = xr[i] * scale * w[i];
}

void rmsnorm(const float *x, const float *w, float *out, int rows, int n, float eps, int64_t ldx, int64_t ldo,
             cudaStream_t s) {
    rmsnorm_kernel<<<rows, 256, 0, s>>>(x, w, out, n, eps, ldx, ldo);
}

// ------------------------------------------------------------- SwiGLU -------
// mlp_forward (ModelCPU.jl:482-508): h = silu(g) * u with g, u from one GEMV
// whose output rows are [gate (ffn) | up (ffn)]
__global__ void swiglu_kernel(const float *__restrict__ gu, float *__restrict__ h, int n, int ffn) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= (int64_t)n * ffn) return;
    const int64_t t = i / ffn, j = i % ffn;
    float g = gu[t * 2 * ffn + j];
    g = g / (1.0f + expf(-g));
    h[i] = g * gu[t * 2 * ffn + ffn + j];
}

void swiglu(const float *gu, float *h, int n, int ffn, cudaStream_t s) {
    const int64_t tot = (int64_t)n * ffn;
    swiglu_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(gu, h, n, ffn);
}

// -------------------------------------------------------- GatedDeltaNet -----
// One CTA per head.  GatedDeltaNetCPU (ModelCPU.jl:566-731) for the N new
// tokens, preceded by the replay of the previous call's committed tokens:
//   * conv ring (:576-599): window = committed history (K-1 tokens) + new tokens
//   * q, k L2-normalised with 1/(sqrt(ss) + 1e-6), q also x 1/sqrt(dk) (:638-651)
//   * decay = exp(f32(ssm_a * softplus(clamp(alpha + dt_bias, +-20)))),
//     beta = f32(sigmoid(clamp(beta, +-20))) in f64 (:654-667)
//   * S *= decay; sk = S k; d = beta (v - sk); S += d k^T; y = S q (:674-702)
//   * per-head RMSNorm with ssm_norm, then y * z * sigmoid(z) (:713-723)
// Rollback: the state in memory is the committed one.  Each call saves the
// new tokens' conv inputs and (k, v, decay, beta); the next call first
// replays the first a_prev+1 of them (a_prev = accepted drafts of the last
// verify) and writes that committed state back before computing new outputs.
template <int HD>
__global__ void __launch_bounds__(256) ssm_step_kernel(SsmArgs a) {
    constexpr int TPR = 256 / HD;   // threads per state row
    constexpr int CPT = HD / TPR;   // state columns per thread
    const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int N = a.N, K = a.K, C = a.C, qk = a.H * HD;
    __shared__ float xc[3][kMaxN][HD];        // conv outputs q, k, v of the new tokens
    __shared__ float rk[kMaxN][HD], rv[kMaxN][HD];
    __shared__ float rdec[kMaxN], rbeta[kMaxN], ndec[kMaxN], nbeta[kMaxN];
    __shared__ float ab[2][kMaxN];
    __shared__ float ys[kMaxN][HD];
    __shared__ float red[8];
    const int r = min(max(*a.a_prev + 1, 0), kMaxN);  // tokens to replay

    // 1. conv window: committed history and new tokens, per owned channel
    for (int lc = tid; lc < 3 * HD; lc += 256) {
        const int part = lc / HD, ch = part * qk + h * HD + lc % HD;
        float seq[3 + kMaxN + kMaxN];  // old history (K-1) + replayed + new
        int n = 0;
        for (int j = 0; j < K - 1; j++) seq[n++] = a.hist[(int64_t)j * C + ch];
        for (int j = 0; j < r; j++) seq[n++] = a.rq[(int64_t)j * C + ch];
        // new committed history = last K-1 of (history + replayed)
        for (int j = 0; j < K - 1; j++) a.hist[(int64_t)j * C + ch] = seq[n - (K - 1) + j];
        const int base = n - (K - 1);
        for (int t = 0; t < N; t++) {
            const float v = a.proj[(int64_t)t * a.ldp + ch];
            seq[n + t] = v;
            a.rq[(int64_t)t * C + ch] = v;  // saved for the next call's replay
        }
        const float *w = a.conv_w + (int64_t)ch * K;
        for (int t = 0; t < N; t++) {
            float acc = 0.f;
            for (int k = 0; k < K; k++) acc += seq[base + t + k] * w[k];
            xc[part][t][lc % HD] = acc / (1.0f + expf(-acc));
        }
    }
    // 2. alpha / beta projections of the new tokens (ssm_alpha/beta . x)
    for (int item = warp; item < 2 * N; item += 8) {
        const int which = item / N, t = item % N;
        const float *w = a.ab_w + (int64_t)(which * a.H + h) * a.d;
        const float *x = a.xn + (int64_t)t * a.d;
        float s = 0.f;
        for (int i = lane; i < a.d; i += 32) s += w[i] * x[i];
        s = warp_sum(s);
        if (lane == 0) ab[which][t] = s;
    }
    // saved replay data of the previous call (read before it is overwritten)
    float *rkv = a.rkv + (int64_t)h * kMaxN * (2 * HD + 2);
    for (int i = tid; i < r * (2 * HD + 2); i += 256) {
        const int j = i / (2 * HD + 2), c = i % (2 * HD + 2);
        const float v = rkv[i];
        if (c < HD) rk[j][c] = v;
        else if (c < 2 * HD) rv[j][c - HD] = v;
        else if (c == 2 * HD) rdec[j] = v;
        else rbeta[j] = v;
    }
    __syncthreads();
    // 3. L2 norms of q, k per new token (warp t), gates in f64
    if (warp < N) {
        const int t = warp;
        float qs = 0.f, ks = 0.f;
        for (int i = lane; i < HD; i += 32) {
            qs += xc[0][t][i] * xc[0][t][i];
            ks += xc[1][t][i] * xc[1][t][i];
        }
        qs = warp_sum(qs);
        ks = warp_sum(ks);
        const float scale = 1.0f / sqrtf((float)HD);
        const float qn = 1.0f / (sqrtf(qs) + 1e-6f) * scale, kn = 1.0f / (sqrtf(ks) + 1e-6f);
        for (int i = lane; i < HD; i += 32) {
            xc[0][t][i] *= qn;
            xc[1][t][i] *= kn;
        }
        if (lane == 0) {
            double av = (double)ab[0][t] + (double)a.dt_bias[h];
            av = av < -20.0 ? -20.0 : (av > 20.0 ? 20.0 : av);
            const double sp = log(1.0 + exp(av));
            const float dec = (float)((double)a.ssm_a[h] * sp);
            ndec[t] = expf(dec);
            double bv = (double)ab[1][t];
            bv = bv < -20.0 ? -20.0 : (bv > 20.0 ? 20.0 : bv);
            nbeta[t] = (float)(1.0 / (1.0 + exp(-bv)));
        }
    }
    __syncthreads();
    // save this call's replay data
    for (int i = tid; i < N * (2 * HD + 2); i += 256) {
        const int t = i / (2 * HD + 2), c = i % (2 * HD + 2);
        rkv[i] = c < HD ? xc[1][t][c] : (c < 2 * HD ? xc[2][t][c - HD] : (c == 2 * HD ? ndec[t] : nbeta[t]));
    }
    // 4. the state: row = tid / TPR, columns c0 .. c0 + CPT
    const int row = tid / TPR, c0 = (tid % TPR) * CPT;
    float *Sp = a.S + ((int64_t)h * HD + row) * HD + c0;
    float s[CPT];
#pragma unroll
    for (int c = 0; c < CPT; c += 4) {
        const float4 v = *reinterpret_cast<const float4 *>(Sp + c);
        s[c] = v.x; s[c + 1] = v.y; s[c + 2] = v.z; s[c + 3] = v.w;
    }
    auto update = [&](const float *kv, float dec, float beta, float vrow) {
        float sk = 0.f;
#pragma unroll
        for (int c = 0; c < CPT; c++) {
            s[c] *= dec;
            sk += s[c] * kv[c0 + c];
        }
#pragma unroll
        for (int o = 1; o < TPR; o <<= 1) sk += __shfl_xor_sync(0xffffffffu, sk, o);
        const float dd = beta * (vrow - sk);
#pragma unroll
        for (int c = 0; c < CPT; c++) s[c] += dd * kv[c0 + c];
    };
    for (int j = 0; j < r; j++) update(rk[j], rdec[j], rbeta[j], rv[j][row]);
#pragma unroll
    for (int c = 0; c < CPT; c += 4) *reinterpret_cast<float4 *>(Sp + c) = make_float4(s[c], s[c + 1], s[c + 2], s[c + 3]);
    for (int t = 0; t < N; t++) {
        update(xc[1][t], ndec[t], nbeta[t], xc[2][t][row]);
        float y = 0.f;
#pragma unroll
        for (int c = 0; c < CPT; c++) y += s[c] * xc[0][t][c0 + c];
#pragma unroll
        for (int o = 1; o < TPR; o <<= 1) y += __shfl_xor_sync(0xffffffffu, y, o);
        if (tid % TPR == 0) ys[t][row] = y;
    }
    __syncthreads();
    // 5. per-head RMSNorm, gate with silu(z)
    for (int t = 0; t < N; t++) {
        float ss = 0.f;
        for (int i = tid; i < HD; i += 256) ss += ys[t][i] * ys[t][i];
        ss = block_sum256(ss, red);
        const float scale = 1.0f / sqrtf(ss / (float)HD + a.eps);
        for (int i = tid; i < HD; i += 256) {
            const float z = a.proj[(int64_t)t * a.ldp + C + h * HD + i];
            const float yn = ys[t][i] * scale * a.norm_w[i];
            a.y[(int64_t)t * a.ldy + h * HD + i] = yn * z * (1.0f / (1.0f + expf(-z)));
        }
    }
}

cudaError_t ssm_step(const SsmArgs &a, int head_dim, cudaStream_t s) {
    if (a.N < 1 || a.N > kMaxN || a.K < 1 || a.K > 4) return cudaErrorInvalidValue;
    if (head_dim == 128) ssm_step_kernel<128><<<a.H, 256, 0, s>>>(a);
    else if (head_dim == 64) ssm_step_kernel<64><<<a.H, 256, 0, s>>>(a);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

// ----------------------------------------------------------- attention ------
// One CTA per query head.  FullAttentionCPU (ModelCPU.jl:787-887): per-head
// [q; gate] rows, RMSNorm + half-split partial RoPE of q and k
// (rmsnorm_rotary!, :188-232), K/V written at the token positions, GQA
// attention with scale 1/sqrt(hd) over keys 0..pos+t (online softmax in
// chunks of 64 keys), output x sigmoid(gate).  Every CTA of a KV group
// normalises the group's new keys itself; the first one writes the cache.
template <int HD>
__global__ void __launch_bounds__(256) attn_step_kernel(AttnArgs a) {
    constexpr int DPT = (HD + 255) / 256;  // dims per thread
    const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int N = a.N, ratio = a.nh / a.nkv, kvh = h / ratio;
    const int p0 = *a.pos;
    __shared__ float q[kMaxN][HD], kn[kMaxN][HD], vn[kMaxN][HD], gt[kMaxN][HD];
    __shared__ float sc[kMaxN][64];
    __shared__ float red[8];
    const int half = a.rotary_dim / 2;
    // load
    for (int i = tid; i < N * HD; i += 256) {
        const int t = i / HD, d = i % HD;
        const float *row = a.qkv + (int64_t)t * a.ldq;
        q[t][d] = row[(int64_t)h * 2 * HD + d];
        gt[t][d] = row[(int64_t)h * 2 * HD + HD + d];
        kn[t][d] = row[(int64_t)a.nh * 2 * HD + kvh * HD + d];
        vn[t][d] = row[(int64_t)a.nh * 2 * HD + a.nkv * HD + kvh * HD + d];
    }
    __syncthreads();
    // RMSNorm + RoPE of q and k, token by token
    for (int t = 0; t < N; t++) {
        float sq = 0.f, sk = 0.f;
        for (int d = tid; d < HD; d += 256) {
            sq += q[t][d] * q[t][d];
            sk += kn[t][d] * kn[t][d];
        }
        sq = block_sum256(sq, red);
        sk = block_sum256(sk, red);
        const float iq = 1.0f / sqrtf(sq / (float)HD + a.eps), ik = 1.0f / sqrtf(sk / (float)HD + a.eps);
        __syncthreads();
        for (int d = tid; d < HD; d += 256) {
            q[t][d] = q[t][d] * iq * a.q_norm[d];
            kn[t][d] = kn[t][d] * ik * a.k_norm[d];
        }
        __syncthreads();
        const float *cs = a.rope_cos + (int64_t)(p0 + t) * half, *sn = a.rope_sin + (int64_t)(p0 + t) * half;
        for (int i = tid; i < half; i += 256) {
            const float c = cs[i], s_ = sn[i];
            float x1 = q[t][i], x2 = q[t][i + half];
            q[t][i] = x1 * c - x2 * s_;
            q[t][i + half] = x1 * s_ + x2 * c;
            x1 = kn[t][i];
            x2 = kn[t][i + half];
            kn[t][i] = x1 * c - x2 * s_;
            kn[t][i + half] = x1 * s_ + x2 * c;
        }
        __syncthreads();
    }
    if (h % ratio == 0) {
        for (int i = tid; i < N * HD; i += 256) {
            const int t = i / HD, d = i % HD;
            const int64_t o = ((int64_t)(p0 + t) * a.nkv + kvh) * HD + d;
            a.kc[o] = kn[t][d];
            a.vc[o] = vn[t][d];
        }
    }
    // attention, online softmax over chunks of 64 keys
    const float scale = 1.0f / sqrtf((float)HD);
    float o_[kMaxN][DPT];
    float m[kMaxN], l[kMaxN];
#pragma unroll
    for (int t = 0; t < kMaxN; t++) {
        m[t] = -CUDART_INF_F;
        l[t] = 0.f;
#pragma unroll
        for (int e = 0; e < DPT; e++) o_[t][e] = 0.f;
    }
    const int nkeys = p0 + N;
    for (int j0 = 0; j0 < nkeys; j0 += 64) {
        const int nj = min(64, nkeys - j0);
        __syncthreads();
        for (int jj = warp; jj < nj; jj += 8) {
            const int j = j0 + jj;
            const float *kp = j < p0 ? a.kc + ((int64_t)j * a.nkv + kvh) * HD : kn[j - p0];
            float part[kMaxN];
#pragma unroll
            for (int t = 0; t < kMaxN; t++) part[t] = 0.f;
            for (int d = lane; d < HD; d += 32) {
                const float kd = kp[d];
#pragma unroll
                for (int t = 0; t < kMaxN; t++)
                    if (t < N) part[t] += q[t][d] * kd;
            }
#pragma unroll
            for (int t = 0; t < kMaxN; t++) {
                if (t < N) {
                    const float v = warp_sum(part[t]);
                    if (lane == 0) sc[t][jj] = (j <= p0 + t) ? v * scale : -CUDART_INF_F;
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int t = 0; t < kMaxN; t++) {
            if (t >= N) break;
            float cm = -CUDART_INF_F;
            for (int jj = 0; jj < nj; jj++) cm = fmaxf(cm, sc[t][jj]);
            const float mn = fmaxf(m[t], cm);
            if (mn == -CUDART_INF_F) continue;
            const float f = expf(m[t] - mn);
            l[t] *= f;
#pragma unroll
            for (int e = 0; e < DPT; e++) o_[t][e] *= f;
            for (int jj = 0; jj < nj; jj++) {
                const float p = expf(sc[t][jj] - mn);
                l[t] += p;
                const int j = j0 + jj;
                const float *vp = j < p0 ? a.vc + ((int64_t)j * a.nkv + kvh) * HD : vn[j - p0];
#pragma unroll
                for (int e = 0; e < DPT; e++) {
                    const int d = tid + 256 * e;
                    if (d < HD) o_[t][e] += p * vp[d];
                }
            }
            m[t] = mn;
        }
    }
#pragma unroll
    for (int t = 0; t < kMaxN; t++) {
        if (t >= N) break;
#pragma unroll
        for (int e = 0; e < DPT; e++) {
            const int d = tid + 256 * e;
            if (d < HD) {
                const float g = 1.0f / (1.0f + expf(-gt[t][d]));
                a.out[(int64_t)t * a.ldo + (int64_t)h * HD + d] = o_[t][e] / l[t] * g;
            }
        }
    }
}

cudaError_t attn_step(const AttnArgs &a, cudaStream_t s) {
    if (a.N < 1 || a.N > kMaxN || a.nh % a.nkv) return cudaErrorInvalidValue;
    if (a.hd == 256) attn_step_kernel<256><<<a.nh, 256, 0, s>>>(a);
    else if (a.hd == 128) attn_step_kernel<128><<<a.nh, 256, 0, s>>>(a);
    else if (a.hd == 64) attn_step_kernel<64><<<a.nh, 256, 0, s>>>(a);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

// ------------------------------------------------------------- commit -------
// After greedy acceptance (accept count acc, tokens out[0..acc]): the target
// committed acc+1 verify tokens.  Advance pos, remember acc for the SSM
// replay, log the emitted tokens, set the next verify's first token, and keep
// the final hidden of column acc for the MTP draft.  `all` commits every one
// of `n` tokens (prefill chunks) with no emitted tokens.
__global__ void commit_kernel(EngineScalars *sc, const int32_t *acc_dev, const int32_t *out_tok, int n,
                              int all, const float *hid, float *mtp_h, int d, int32_t *log, int log_cap) {
    __shared__ int acc_s;
    if (threadIdx.x == 0) {
        const int acc = all ? n - 1 : *acc_dev;
        acc_s = acc;
        sc->a_prev = acc;
        sc->pos += acc + 1;
        if (!all) {
            for (int i = 0; i <= acc; i++)
                if (sc->n_log < log_cap) log[sc->n_log++] = out_tok[i];
            sc->last_token = out_tok[acc];
            sc->last_accept = acc;
            sc->steps += 1;
        }
    }
    __syncthreads();
    if (!all && hid)
        for (int i = threadIdx.x; i < d; i += blockDim.x) mtp_h[i] = hid[(int64_t)acc_s * d + i];
}

void commit(EngineScalars *sc, const int32_t *acc, const int32_t *out_tok, int n, bool all, const float *hid,
            float *mtp_h, int d, int32_t *log, int log_cap, cudaStream_t s) {
    commit_kernel<<<1, 256, 0, s>>>(sc, acc, out_tok, n, all ? 1 : 0, hid, mtp_h, d, log, log_cap);
}

// copy a device scalar token into a slot of the verify token vector
__global__ void set_token_kernel(int32_t *dst, const int32_t *src) { *dst = *src; }
void set_token(int32_t *dst, const int32_t *src, cudaStream_t s) { set_token_kernel<<<1, 1, 0, s>>>(dst, src); }

}  // namespace ifr
