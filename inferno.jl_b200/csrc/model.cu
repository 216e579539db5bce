// Layer kernels of the Qwen3.5-hybrid verify step (N <= 8 tokens per request
// and call; batched calls put the requests on blockIdx.z).
//
// Reference semantics: src/ModelCPU.jl of Inferno.jl (line numbers below).
// All arithmetic is f32 except the SSM gates, which the reference evaluates in
// f64 (:654-667) and so do we.
#include "common.cuh"
#include "model.cuh"
#include "qgemv_kernels.cuh"  // the M-tile code of the fused verify (fused_step.cuh)

#include <algorithm>
#include <cuda_bf16.h>
#include <cooperative_groups.h>
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

// a barrier over the 256 threads of a (virtual) block: BAR 0 = the whole CTA
// (__syncthreads), BAR > 0 = named barrier BAR of 256 threads, so that two
// 256-thread virtual blocks can share one 512-thread CTA (fused.cu)
template <int BAR>
__device__ __forceinline__ void bar256() {
    if constexpr (BAR == 0) __syncthreads();
    else asm volatile("bar.sync %0, 256;" ::"n"(BAR) : "memory");
}
template <int BAR>
__device__ __forceinline__ float block_sum256_b(float v, float *red, int tid) {
    v = warp_sum(v);
    bar256<BAR>();
    if ((tid & 31) == 0) red[tid >> 5] = v;
    bar256<BAR>();
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
    pdl_trigger();
    pdl_wait();
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
    launch_k(rmsnorm_kernel, dim3(rows), dim3(256), 0, s, x, w, out, n, eps, ldx, ldo);
}

// ------------------------------------------------- Gemma4 block tails -------
// forward! (Gemma4.jl:622-650) after a sub-block: x = (x + RMSNorm(y) w) * s -
// the post-attention (s = 1) and post-feed-forward (s = layer scalar) norms
// added to the residual; one CTA per column
__global__ void __launch_bounds__(256) norm_add_kernel(const float *__restrict__ y, const float *__restrict__ w,
                                                       float *x, int n, float eps, const float *scalar) {
    __shared__ float red[8];
    pdl_trigger();
    pdl_wait();
    const float *yr = y + (int64_t)blockIdx.x * n;
    float *xr = x + (int64_t)blockIdx.x * n;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += 256) ss += yr[i] * yr[i];
    ss = block_sum256(ss, red);
    const float inv = 1.0f / sqrtf(ss / (float)n + eps);
    const float sc = scalar ? *scalar : 1.0f;
    for (int i = threadIdx.x; i < n; i += 256) {
        const float v = __fadd_rn(xr[i], yr[i] * inv * w[i]);
        xr[i] = scalar ? __fmul_rn(v, sc) : v;
    }
}

void norm_add(const float *y, const float *w, float *x, int cols, int n, float eps, const float *scalar,
              cudaStream_t s) {
    launch_k(norm_add_kernel, dim3(cols), dim3(256), 0, s, y, w, x, n, eps, scalar);
}

// logit_softcap! (CommonOps.jl:326-333) in place: l = tanh(l / cap) cap
__global__ void softcap_kernel(float *l, int64_t n, float cap) {
    pdl_trigger();
    pdl_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        l[i] = tanhf(l[i] / cap) * cap;
}

void softcap(float *l, int64_t n, float cap, cudaStream_t s) {
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, 148 * 8);
    launch_k(softcap_kernel, dim3((unsigned)std::max<int64_t>(blocks, 1)), dim3(256), 0, s, l, n, cap);
}

// Gemma4 per-layer inputs (compute_per_layer_inputs!, Gemma4.jl:459-503):
// block (layer i, column c), 256 threads: RMSNorm of the projection slice
// (CommonOps.rmsnorm!), plus the table row slice times sqrt(P), times 2^-1/2
__global__ void __launch_bounds__(256) pli_inputs_kernel(const float *__restrict__ proj, const float *__restrict__ emb,
                                                         const float *__restrict__ w, int P, int L, float eps,
                                                         float *__restrict__ out) {
    __shared__ float red[8];
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x, c = blockIdx.y, tid = threadIdx.x;
    const int64_t base = (int64_t)c * L * P + (int64_t)i * P;
    float ss = 0.f;
    for (int j = tid; j < P; j += 256) ss += proj[base + j] * proj[base + j];
    ss = block_sum256_b<0>(ss, red, tid);
    const float inv = 1.0f / sqrtf(ss / (float)P + eps);
    const float scale = sqrtf((float)P), in_scale = 0.707106781186547524f;  // Float32(2^-1/2)
    for (int j = tid; j < P; j += 256) {
        const float o = proj[base + j] * inv * w[j];
        out[base + j] = (o + emb[base + j] * scale) * in_scale;
    }
}

cudaError_t pli_inputs(const float *proj, const float *emb, const float *w, int P, int L, int nc, float eps,
                       float *out, cudaStream_t s) {
    if (P < 1 || L < 1 || nc < 1) return cudaErrorInvalidValue;
    return launch_k(pli_inputs_kernel, dim3(L, nc), dim3(256), 0, s, proj, emb, w, P, L, eps, out);
}

// per_layer_input_forward! (Gemma4.jl:514-524): g = gelu_tanh(g) * pli slice
__global__ void pli_gate_kernel(float *__restrict__ g, const float *__restrict__ pli, int P, int64_t lp, int layer,
                                int64_t n) {
    pdl_trigger();
    pdl_wait();
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t c = i / P;
    const int j = (int)(i % P);
    const float v = gelu_tanh(g[i]);
    g[i] = v * pli[c * lp + (int64_t)layer * P + j];
}

cudaError_t pli_gate(float *g, const float *pli, int P, int64_t lp, int layer, int nc, cudaStream_t s) {
    const int64_t n = (int64_t)nc * P;
    return launch_k(pli_gate_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, g, pli, P, lp, layer, n);
}

// ------------------------------------------------------------- SwiGLU -------
// mlp_forward (ModelCPU.jl:482-508): h = silu(g) * u with g, u from one GEMV
// whose output rows are [gate (ffn) | up (ffn)]
__global__ void swiglu_kernel(const float *__restrict__ gu, float *__restrict__ h, int n, int ffn) {
    pdl_trigger();
    pdl_wait();
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= (int64_t)n * ffn) return;
    const int64_t t = i / ffn, j = i % ffn;
    float g = gu[t * 2 * ffn + j];
    g = g / (1.0f + expf(-g));
    h[i] = g * gu[t * 2 * ffn + ffn + j];
}

void swiglu(const float *gu, float *h, int n, int ffn, cudaStream_t s) {
    const int64_t tot = (int64_t)n * ffn;
    launch_k(swiglu_kernel, dim3((unsigned)((tot + 255) / 256)), dim3(256), 0, s, gu, h, n, ffn);
}

// -------------------------------------------------------- GatedDeltaNet -----
// GatedDeltaNetCPU (ModelCPU.jl:566-731) for the N new tokens, preceded by
// the replay of the previous call's committed tokens:
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
//
// Grid (kSsmSplit, H), one cluster of kSsmSplit CTAs per head.  The rows of S
// (value dims) are independent given k and q, so CTA `rank` owns rows
// r0 .. r0 + RPC of S, the conv channels of v rows r0.. and of q, k dims r0..;
// the head's q and k are gathered from the cluster's shared memory, and the
// per-head RMSNorm sums the CTAs' partial sums of squares in rank order.
// Each conv channel's history is read and written by its owner only; the
// replay record is read by every CTA before the first cluster barrier and
// rewritten after it.
constexpr int kSsmSplit = 8;

template <int HD>
__global__ void __cluster_dims__(kSsmSplit, 1, 1) __launch_bounds__(256) ssm_step_kernel(SsmArgs a) {
    // (a is a by-value copy: the per-request offsets below are local)
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    constexpr int RPC = HD / kSsmSplit;  // state rows (and q, k dims) per CTA
    constexpr int TPR = 256 / RPC;       // threads per state row
    constexpr int CPT = HD / TPR;        // state columns per thread (interleaved by TPR)
    constexpr int REC = 2 * HD + 2;      // replay record floats per token
    const int rank = (int)cluster.block_rank();
    const int h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int N = a.N, K = a.K, C = a.C, qk = a.H * HD;
    const int r0 = rank * RPC;
    __shared__ float cq[kMaxN][RPC], ck[kMaxN][RPC], cv[kMaxN][RPC];  // own conv outputs
    __shared__ __align__(16) float xq[kMaxN][HD];
    __shared__ __align__(16) float xk[kMaxN][HD];
    __shared__ __align__(16) float rk[kMaxN][HD];
    __shared__ float rv[kMaxN][RPC];
    __shared__ float rdec[kMaxN], rbeta[kMaxN], ndec[kMaxN], nbeta[kMaxN];
    __shared__ float ab[3][kMaxN], ab_part[3][kMaxN];
    __shared__ float ys[kMaxN][RPC];
    __shared__ float ssq[kMaxN];
    __shared__ float red_n[8][3 * kMaxN];
    pdl_trigger();
    pdl_wait();
    {  // request blockIdx.z of a batched call
        const int64_t b = blockIdx.z;
        a.proj += b * a.N * a.ldp;
        a.xn += b * a.N * a.d;
        a.y += b * a.N * a.ldy;
        a.S += b * a.b_S;
        a.hist += b * a.b_hist;
        a.rq += b * a.b_rq;
        a.rkv += b * a.b_rkv;
        a.a_prev += b * a.b_prev;
    }
    const int r = min(max(*a.a_prev + 1, 0), kMaxN);  // tokens to replay
    // this thread's state row slice, loaded first so that its memory latency
    // overlaps the conv, the projections and the cluster exchange below
    const int row = tid / TPR, lc = tid % TPR;
    float *Sp = a.S + ((int64_t)h * HD + r0 + row) * HD + lc;
    float s[CPT];
#pragma unroll
    for (int e = 0; e < CPT; e++) s[e] = Sp[TPR * e];

    // 1. conv of the owned channels over the window: committed history (K-1),
    //    replayed tokens (r), new tokens (N).  Element i of the window is read
    //    straight from where it lives, so all loads are independent.
    auto win = [&](int i, int ch) -> const float * {
        if (i < K - 1) return a.hist + (int64_t)i * C + ch;
        if (i < K - 1 + r) return a.rq + (int64_t)(i - K + 1) * C + ch;
        return a.proj + (int64_t)(i - K + 1 - r) * a.ldp + ch;
    };
    for (int lc = tid; lc < 3 * RPC; lc += 256) {
        const int part = lc / RPC, i = lc % RPC;
        const int ch = part * qk + h * HD + r0 + i;
        float w[4], tap[kMaxN][4], nh[3], pv[kMaxN];
#pragma unroll
        for (int k = 0; k < 4; k++) w[k] = k < K ? a.conv_w[(int64_t)ch * K + k] : 0.f;
#pragma unroll
        for (int t = 0; t < kMaxN; t++) {
            pv[t] = t < N ? a.proj[(int64_t)t * a.ldp + ch] : 0.f;
#pragma unroll
            for (int k = 0; k < 4; k++) tap[t][k] = (t < N && k < K) ? *win(r + t + k, ch) : 0.f;
        }
        // new committed history = last K-1 of (history + replayed)
#pragma unroll
        for (int j = 0; j < 3; j++) nh[j] = j < K - 1 ? *win(r + j, ch) : 0.f;
#pragma unroll
        for (int j = 0; j < 3; j++)
            if (j < K - 1) a.hist[(int64_t)j * C + ch] = nh[j];
#pragma unroll
        for (int t = 0; t < kMaxN; t++) {
            if (t < N) {
                a.rq[(int64_t)t * C + ch] = pv[t];  // saved for the next call's replay
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < 4; k++)
                    if (k < K) acc += tap[t][k] * w[k];
                const float o = acc / (1.0f + expf(-acc));
                if (part == 0) cq[t][i] = o;
                else if (part == 1) ck[t][i] = o;
                else cv[t][i] = o;
            }
        }
    }
    // 2. alpha / beta projections of the new tokens (ssm_alpha/beta . xn): CTA
    //    `rank` sums its d / kSsmSplit slice, the partials are added across the
    //    cluster in rank order after the next cluster barrier (step 5)
    {
        float pa[kMaxN], pb[kMaxN], ps[kMaxN];
#pragma unroll
        for (int t = 0; t < kMaxN; t++) pa[t] = pb[t] = ps[t] = 0.f;
        const float *wa = a.ab_w + (int64_t)h * a.d, *wb = a.ab_w + (int64_t)(a.H + h) * a.d;
        const int per = (a.d + kSsmSplit - 1) / kSsmSplit;
        const int i0 = rank * per, i1 = min(a.d, i0 + per);
        for (int i = i0 + tid; i < i1; i += 256) {
            const float al = wa[i], be = wb[i], nw = a.in_norm ? a.in_norm[i] : 1.f;
#pragma unroll
            for (int t = 0; t < kMaxN; t++)
                if (t < N) {
                    const float xv = a.xn[(int64_t)t * a.d + i], xn = xv * nw;
                    pa[t] += al * xn;
                    pb[t] += be * xn;
                    ps[t] += xv * xv;
                }
        }
#pragma unroll
        for (int t = 0; t < kMaxN; t++) {
            const float va = warp_sum(pa[t]), vb = warp_sum(pb[t]), vs = warp_sum(ps[t]);
            if (lane == 0) {
                red_n[warp][t] = va;
                red_n[warp][kMaxN + t] = vb;
                red_n[warp][2 * kMaxN + t] = vs;
            }
        }
        __syncthreads();
        if (tid < 3 * N) {
            const int which = tid / N, t = tid % N;
            float v = 0.f;
            for (int w8 = 0; w8 < 8; w8++) v += red_n[w8][which * kMaxN + t];
            ab_part[which][t] = v;
        }
    }
    // 3. the previous call's replay record: k (all dims), own v rows, decay,
    //    beta (a thread's loads issued before its shared stores)
    float *rec = a.rkv + (int64_t)h * kMaxN * REC;
    {
        constexpr int LPT = (kMaxN * HD + 255) / 256;
        float kr[LPT];
#pragma unroll
        for (int k = 0; k < LPT; k++) {
            const int i = tid + 256 * k;
            kr[k] = i < r * HD ? rec[(i / HD) * REC + i % HD] : 0.f;
        }
#pragma unroll
        for (int k = 0; k < LPT; k++) {
            const int i = tid + 256 * k;
            if (i < r * HD) rk[i / HD][i % HD] = kr[k];
        }
    }
    for (int i = tid; i < r * RPC; i += 256) rv[i / RPC][i % RPC] = rec[(i / RPC) * REC + HD + r0 + i % RPC];
    if (tid < r) {
        rdec[tid] = rec[tid * REC + 2 * HD];
        rbeta[tid] = rec[tid * REC + 2 * HD + 1];
    }
    cluster.sync();  // conv slices visible to the cluster; old record read by all
    // 4. the head's q and k, gathered from the owners; alpha / beta summed over
    //    the cluster's slices
    {
        constexpr int LPT = (kMaxN * HD + 255) / 256;
        float gq[LPT], gk[LPT];
#pragma unroll
        for (int k = 0; k < LPT; k++) {
            const int i = tid + 256 * k, t = i / HD, c = i % HD, src = c / RPC, ci = c % RPC;
            gq[k] = i < N * HD ? cluster.map_shared_rank(&cq[0][0], src)[t * RPC + ci] : 0.f;
            gk[k] = i < N * HD ? cluster.map_shared_rank(&ck[0][0], src)[t * RPC + ci] : 0.f;
        }
#pragma unroll
        for (int k = 0; k < LPT; k++) {
            const int i = tid + 256 * k, t = i / HD, c = i % HD;
            if (i < N * HD) {
                xq[t][c] = gq[k];
                xk[t][c] = gk[k];
            }
        }
    }
    if (tid < 3 * N) {
        const int which = tid / N, t = tid % N;
        float v = 0.f;
        for (int q = 0; q < kSsmSplit; q++) v += cluster.map_shared_rank(&ab_part[0][0], q)[which * kMaxN + t];
        ab[which][t] = v;
    }
    __syncthreads();
    if (a.in_norm && tid < N) {  // RMSNorm folded: the projections of x w, scaled by rms(x)^-1
        const float iv = 1.0f / sqrtf(ab[2][tid] / (float)a.d + a.eps);
        ab[0][tid] *= iv;
        ab[1][tid] *= iv;
    }
    __syncthreads();
    // 5. L2 norms of q, k per new token (warp t), gates in f64
    if (warp < N) {
        const int t = warp;
        float qs = 0.f, ks = 0.f;
        for (int i = lane; i < HD; i += 32) {
            qs += xq[t][i] * xq[t][i];
            ks += xk[t][i] * xk[t][i];
        }
        qs = warp_sum(qs);
        ks = warp_sum(ks);
        const float scale = 1.0f / sqrtf((float)HD);
        const float qn = 1.0f / (sqrtf(qs) + 1e-6f) * scale, kn = 1.0f / (sqrtf(ks) + 1e-6f);
        __syncwarp();
        for (int i = lane; i < HD; i += 32) {
            xq[t][i] *= qn;
            xk[t][i] *= kn;
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
    // 6. this call's replay record (rank 0: k, decay, beta; every CTA: its v rows)
    if (rank == 0) {
        for (int i = tid; i < N * HD; i += 256) rec[(i / HD) * REC + i % HD] = xk[i / HD][i % HD];
        if (tid < N) {
            rec[tid * REC + 2 * HD] = ndec[tid];
            rec[tid * REC + 2 * HD + 1] = nbeta[tid];
        }
    }
    for (int i = tid; i < N * RPC; i += 256) rec[(i / RPC) * REC + HD + r0 + i % RPC] = cv[i / RPC][i % RPC];
    // 7. the state rows (loaded at the start): row r0 + tid / TPR, columns lc + TPR * e
    auto update = [&](const float *kv, float dec, float beta, float vrow) {
        float sk = 0.f;
#pragma unroll
        for (int e = 0; e < CPT; e++) {
            s[e] *= dec;
            sk += s[e] * kv[lc + TPR * e];
        }
#pragma unroll
        for (int o = 1; o < TPR; o <<= 1) sk += __shfl_xor_sync(0xffffffffu, sk, o);
        const float dd = beta * (vrow - sk);
#pragma unroll
        for (int e = 0; e < CPT; e++) s[e] += dd * kv[lc + TPR * e];
    };
    for (int j = 0; j < r; j++) update(rk[j], rdec[j], rbeta[j], rv[j][row]);
#pragma unroll
    for (int e = 0; e < CPT; e++) Sp[TPR * e] = s[e];
    for (int t = 0; t < N; t++) {
        update(xk[t], ndec[t], nbeta[t], cv[t][row]);
        float y = 0.f;
#pragma unroll
        for (int e = 0; e < CPT; e++) y += s[e] * xq[t][lc + TPR * e];
#pragma unroll
        for (int o = 1; o < TPR; o <<= 1) y += __shfl_xor_sync(0xffffffffu, y, o);
        if (lc == 0) ys[t][row] = y;
    }
    __syncthreads();
    // 8. per-head RMSNorm (partial sums of squares, summed over the cluster in
    //    rank order), gate with silu(z)
    if (warp < N) {
        const float v = lane < RPC ? ys[warp][lane] * ys[warp][lane] : 0.f;
        const float t2 = warp_sum(v);
        if (lane == 0) ssq[warp] = t2;
    }
    cluster.sync();
    for (int i = tid; i < N * RPC; i += 256) {
        const int t = i / RPC, c = i % RPC;
        float ss = 0.f;
        for (int q = 0; q < kSsmSplit; q++) ss += cluster.map_shared_rank(&ssq[0], q)[t];
        const float scale = 1.0f / sqrtf(ss / (float)HD + a.eps);
        const float z = a.proj[(int64_t)t * a.ldp + C + h * HD + r0 + c];
        const float yn = ys[t][c] * scale * a.norm_w[r0 + c];
        a.y[(int64_t)t * a.ldy + h * HD + r0 + c] = yn * z * (1.0f / (1.0f + expf(-z)));
    }
    cluster.sync();  // peers may still read this CTA's shared memory
}

// Batched variant: one CTA of 4 HD threads per (head, request), no cluster.
// Same arithmetic as ssm_step_kernel: thread (row = tid / 4, lc = tid % 4) owns
// columns lc + 4 e of state row `row`; thread c < 3 HD owns conv channel c of
// the head (q, k, v); the alpha/beta projections are summed block-wide.
// one (head h, request b) block of 4 HD threads (the whole CTA)
template <int HD>
__device__ __forceinline__ void ssm_batch_body(SsmArgs a, int h, int64_t b) {
    constexpr int NT = 4 * HD;
    constexpr int CPT = HD / 4;        // state columns per thread
    constexpr int REC = 2 * HD + 2;
    constexpr int NW = NT / 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int N = a.N, K = a.K, C = a.C, qk = a.H * HD;
    __shared__ __align__(16) float xq[kMaxN][HD];
    __shared__ __align__(16) float xk[kMaxN][HD];
    __shared__ __align__(16) float cv[kMaxN][HD];
    __shared__ __align__(16) float rk[kMaxN][HD];
    __shared__ float rv[kMaxN][HD];
    __shared__ float ys[kMaxN][HD];
    __shared__ float rdec[kMaxN], rbeta[kMaxN], ndec[kMaxN], nbeta[kMaxN];
    __shared__ float ab[3][kMaxN], ssq[kMaxN];
    __shared__ float red_n[NW][3 * kMaxN];
    {  // request b
        a.proj += b * a.N * a.ldp;
        a.xn += b * a.N * a.d;
        a.y += b * a.N * a.ldy;
        a.S += b * a.b_S;
        a.hist += b * a.b_hist;
        a.rq += b * a.b_rq;
        a.rkv += b * a.b_rkv;
        a.a_prev += b * a.b_prev;
    }
    const int r = min(max(*a.a_prev + 1, 0), kMaxN);  // tokens to replay
    // thread (row = tid / 4, lc = tid % 4) owns columns 16 e + 4 lc + v of
    // state row `row`, read as 16-byte vectors (a warp reads 64 contiguous
    // bytes per row) once steps 1-5 are done: two CTAs share an SM, so one's
    // state traffic overlaps the other's arithmetic
    const int row = tid >> 2, lc = tid & 3;
    float4 *Sp = reinterpret_cast<float4 *>(a.S + ((int64_t)h * HD + row) * HD + 4 * lc);
    // 1. conv of the head's channels (ssm_step_kernel step 1): the window
    //    (committed history K-1, replayed r, new N) read once into registers;
    //    element r + j of it is the new committed history j, element K-1+r+t
    //    the new token t's input
    auto win = [&](int i, int ch) -> const float * {
        if (i < K - 1) return a.hist + (int64_t)i * C + ch;
        if (i < K - 1 + r) return a.rq + (int64_t)(i - K + 1) * C + ch;
        return a.proj + (int64_t)(i - K + 1 - r) * a.ldp + ch;
    };
    if (tid < 3 * HD) {
        const int part = tid / HD, i = tid % HD;
        const int ch = part * qk + h * HD + i;
        float w[4], wv[kMaxN + 3];
#pragma unroll
        for (int k = 0; k < 4; k++) w[k] = k < K ? a.conv_w[(int64_t)ch * K + k] : 0.f;
#pragma unroll
        for (int j = 0; j < kMaxN + 3; j++) wv[j] = j < N + K - 1 ? *win(r + j, ch) : 0.f;
#pragma unroll
        for (int j = 0; j < 3; j++)
            if (j < K - 1) a.hist[(int64_t)j * C + ch] = wv[j];
#pragma unroll
        for (int t = 0; t < kMaxN; t++) {
            if (t < N) {
                a.rq[(int64_t)t * C + ch] = wv[K - 1 + t];
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < 4; k++)
                    if (k < K) acc += wv[t + k] * w[k];
                const float o = acc / (1.0f + expf(-acc));
                if (part == 0) xq[t][i] = o;
                else if (part == 1) xk[t][i] = o;
                else cv[t][i] = o;
            }
        }
    }
    // 2. alpha / beta projections of the new tokens, block-wide
    {
        float pa[kMaxN], pb[kMaxN], ps[kMaxN];
#pragma unroll
        for (int t = 0; t < kMaxN; t++) pa[t] = pb[t] = ps[t] = 0.f;
        const float *wa = a.ab_w + (int64_t)h * a.d, *wb = a.ab_w + (int64_t)(a.H + h) * a.d;
        if ((a.d & 3) == 0) {
            // 16-byte loads, every load of an iteration (weights, norm weights,
            // the N token rows) issued before the first use: d / (4 NT)
            // memory round trips instead of d / NT
            for (int i = 4 * tid; i < a.d; i += 4 * NT) {
                const float4 al = *reinterpret_cast<const float4 *>(wa + i);
                const float4 be = *reinterpret_cast<const float4 *>(wb + i);
                const float4 nw = a.in_norm ? *reinterpret_cast<const float4 *>(a.in_norm + i)
                                            : make_float4(1.f, 1.f, 1.f, 1.f);
                float4 xv[kMaxN];
#pragma unroll
                for (int t = 0; t < kMaxN; t++)
                    xv[t] = t < N ? *reinterpret_cast<const float4 *>(a.xn + (int64_t)t * a.d + i)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int t = 0; t < kMaxN; t++) {
                    const float4 x = xv[t];
                    pa[t] += al.x * (x.x * nw.x) + al.y * (x.y * nw.y) + al.z * (x.z * nw.z) + al.w * (x.w * nw.w);
                    pb[t] += be.x * (x.x * nw.x) + be.y * (x.y * nw.y) + be.z * (x.z * nw.z) + be.w * (x.w * nw.w);
                    ps[t] += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
                }
            }
        } else {
            for (int i = tid; i < a.d; i += NT) {
                const float al = wa[i], be = wb[i], nw = a.in_norm ? a.in_norm[i] : 1.f;
#pragma unroll
                for (int t = 0; t < kMaxN; t++)
                    if (t < N) {
                        const float xv = a.xn[(int64_t)t * a.d + i], xn = xv * nw;
                        pa[t] += al * xn;
                        pb[t] += be * xn;
                        ps[t] += xv * xv;
                    }
            }
        }
#pragma unroll
        for (int t = 0; t < kMaxN; t++) {
            if (t < N) {  // uniform: only the present tokens' sums
                const float va = warp_sum(pa[t]), vb = warp_sum(pb[t]), vs = warp_sum(ps[t]);
                if (lane == 0) {
                    red_n[warp][t] = va;
                    red_n[warp][kMaxN + t] = vb;
                    red_n[warp][2 * kMaxN + t] = vs;
                }
            }
        }
    }
    // 3. the previous call's replay record
    float *rec = a.rkv + (int64_t)h * kMaxN * REC;
    for (int i = tid; i < r * HD; i += NT) {
        rk[i / HD][i % HD] = rec[(i / HD) * REC + i % HD];
        rv[i / HD][i % HD] = rec[(i / HD) * REC + HD + i % HD];
    }
    if (tid < r) {
        rdec[tid] = rec[tid * REC + 2 * HD];
        rbeta[tid] = rec[tid * REC + 2 * HD + 1];
    }
    __syncthreads();
    if (tid < 3 * N) {
        const int which = tid / N, t = tid % N;
        float v = 0.f;
        for (int w8 = 0; w8 < NW; w8++) v += red_n[w8][which * kMaxN + t];
        ab[which][t] = v;
    }
    __syncthreads();
    if (a.in_norm && tid < N) {  // RMSNorm folded: the projections of x w, scaled by rms(x)^-1
        const float iv = 1.0f / sqrtf(ab[2][tid] / (float)a.d + a.eps);
        ab[0][tid] *= iv;
        ab[1][tid] *= iv;
    }
    __syncthreads();
    // 4. L2 norms of q, k (warp t), gates in f64
    if (warp < N) {
        const int t = warp;
        float qs = 0.f, ks = 0.f;
        for (int i = lane; i < HD; i += 32) {
            qs += xq[t][i] * xq[t][i];
            ks += xk[t][i] * xk[t][i];
        }
        qs = warp_sum(qs);
        ks = warp_sum(ks);
        const float scale = 1.0f / sqrtf((float)HD);
        const float qn = 1.0f / (sqrtf(qs) + 1e-6f) * scale, kn = 1.0f / (sqrtf(ks) + 1e-6f);
        __syncwarp();
        for (int i = lane; i < HD; i += 32) {
            xq[t][i] *= qn;
            xk[t][i] *= kn;
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
    // 5. this call's replay record (the old one was read in step 3)
    for (int i = tid; i < N * HD; i += NT) {
        rec[(i / HD) * REC + i % HD] = xk[i / HD][i % HD];
        rec[(i / HD) * REC + HD + i % HD] = cv[i / HD][i % HD];
    }
    if (tid < N) {
        rec[tid * REC + 2 * HD] = ndec[tid];
        rec[tid * REC + 2 * HD + 1] = nbeta[tid];
    }
    // 6. the state rows through the replayed and new tokens
    float4 sv[CPT / 4];
#pragma unroll
    for (int e = 0; e < CPT / 4; e++) sv[e] = Sp[4 * e];
    auto update = [&](const float *kv, float dec, float beta, float vrow) {
        float sk = 0.f;
#pragma unroll
        for (int e = 0; e < CPT / 4; e++) {
            const float4 k4 = *reinterpret_cast<const float4 *>(kv + 16 * e + 4 * lc);
            sv[e].x *= dec;
            sv[e].y *= dec;
            sv[e].z *= dec;
            sv[e].w *= dec;
            sk += sv[e].x * k4.x;
            sk += sv[e].y * k4.y;
            sk += sv[e].z * k4.z;
            sk += sv[e].w * k4.w;
        }
        sk += __shfl_xor_sync(0xffffffffu, sk, 1);
        sk += __shfl_xor_sync(0xffffffffu, sk, 2);
        const float dd = beta * (vrow - sk);
#pragma unroll
        for (int e = 0; e < CPT / 4; e++) {
            const float4 k4 = *reinterpret_cast<const float4 *>(kv + 16 * e + 4 * lc);
            sv[e].x += dd * k4.x;
            sv[e].y += dd * k4.y;
            sv[e].z += dd * k4.z;
            sv[e].w += dd * k4.w;
        }
    };
    for (int j = 0; j < r; j++) update(rk[j], rdec[j], rbeta[j], rv[j][row]);
#pragma unroll
    for (int e = 0; e < CPT / 4; e++) Sp[4 * e] = sv[e];
    for (int t = 0; t < N; t++) {
        update(xk[t], ndec[t], nbeta[t], cv[t][row]);
        float yv = 0.f;
#pragma unroll
        for (int e = 0; e < CPT / 4; e++) {
            const float4 q4 = *reinterpret_cast<const float4 *>(&xq[t][16 * e + 4 * lc]);
            yv += sv[e].x * q4.x;
            yv += sv[e].y * q4.y;
            yv += sv[e].z * q4.z;
            yv += sv[e].w * q4.w;
        }
        yv += __shfl_xor_sync(0xffffffffu, yv, 1);
        yv += __shfl_xor_sync(0xffffffffu, yv, 2);
        if (lc == 0) ys[t][row] = yv;
    }
    __syncthreads();
    // 7. per-head RMSNorm and the silu(z) gate
    if (warp < N) {
        float v = 0.f;
        for (int i = lane; i < HD; i += 32) v += ys[warp][i] * ys[warp][i];
        v = warp_sum(v);
        if (lane == 0) ssq[warp] = v;
    }
    __syncthreads();
    for (int i = tid; i < N * HD; i += NT) {
        const int t = i / HD, c = i % HD;
        const float scale = 1.0f / sqrtf(ssq[t] / (float)HD + a.eps);
        const float z = a.proj[(int64_t)t * a.ldp + C + h * HD + c];
        const float yn = ys[t][c] * scale * a.norm_w[c];
        a.y[(int64_t)t * a.ldy + h * HD + c] = yn * z * (1.0f / (1.0f + expf(-z)));
    }
}

template <int HD>
__global__ void __launch_bounds__(4 * HD, 2) ssm_batch_kernel(SsmArgs a) {
    pdl_trigger();
    pdl_wait();
    ssm_batch_body<HD>(a, blockIdx.x, blockIdx.y);
}

// Prefill chunk of up to kChunkMax tokens of one request (GatedDeltaNetCPU,
// ModelCPU.jl:566-731, over the chunk's tokens in order, as forward_cpu! feeds
// a prompt): the scan of the chunk runs inside one launch with each CTA's
// state rows in registers, and the result is committed at once - S holds the
// state after the last token, the conv history the chunk's last K-1 inputs,
// and no replay record is written (the caller's commit leaves nothing to
// replay).  A pending replay of the previous call's tokens is applied first,
// as in ssm_step_kernel.  Grid (kSsmSplit, H), one cluster per head; the
// per-token arrays live in dynamic shared memory (ChunkSmem).
constexpr int kChunkMax = 64;

template <int HD>
struct ChunkSmem {
    static constexpr int RPC = HD / kSsmSplit;
    float cq[kChunkMax][RPC], ck[kChunkMax][RPC], cv[kChunkMax][RPC];
    float xq[kChunkMax][HD], xk[kChunkMax][HD];
    float rk[kMaxN][HD], rv[kMaxN][RPC];
    float rdec[kMaxN], rbeta[kMaxN], ndec[kChunkMax], nbeta[kChunkMax];
    float ab[3][kChunkMax], ab_part[3][kChunkMax];
    float ys[kChunkMax][RPC];
    float ssq[kChunkMax];
    float red_n[8][3 * kChunkMax];
};

template <int HD>
__global__ void __cluster_dims__(kSsmSplit, 1, 1) __launch_bounds__(256) ssm_chunk_kernel(SsmArgs a) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    constexpr int RPC = HD / kSsmSplit, TPR = 256 / RPC, CPT = HD / TPR, REC = 2 * HD + 2;
    extern __shared__ __align__(16) unsigned char chunk_smem[];
    ChunkSmem<HD> &m = *reinterpret_cast<ChunkSmem<HD> *>(chunk_smem);
    const int rank = (int)cluster.block_rank();
    const int h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int N = a.N, K = a.K, C = a.C, qk = a.H * HD;
    const int r0 = rank * RPC;
    pdl_trigger();
    pdl_wait();
    const int r = min(max(*a.a_prev + 1, 0), kMaxN);  // tokens to replay

    // 1. conv of the owned channels over committed history, replayed and new tokens
    auto win = [&](int i, int ch) -> const float * {
        if (i < K - 1) return a.hist + (int64_t)i * C + ch;
        if (i < K - 1 + r) return a.rq + (int64_t)(i - K + 1) * C + ch;
        return a.proj + (int64_t)(i - K + 1 - r) * a.ldp + ch;
    };
    for (int lc = tid; lc < 3 * RPC; lc += 256) {
        const int part = lc / RPC, i = lc % RPC;
        const int ch = part * qk + h * HD + r0 + i;
        float w[4];
#pragma unroll
        for (int k = 0; k < 4; k++) w[k] = k < K ? a.conv_w[(int64_t)ch * K + k] : 0.f;
        for (int t = 0; t < N; t++) {
            float acc = 0.f;
#pragma unroll
            for (int k = 0; k < 4; k++)
                if (k < K) acc += *win(r + t + k, ch) * w[k];
            const float o = acc / (1.0f + expf(-acc));
            if (part == 0) m.cq[t][i] = o;
            else if (part == 1) m.ck[t][i] = o;
            else m.cv[t][i] = o;
        }
    }
    // 2. alpha / beta projections of the new tokens, this CTA's d slice
    {
        const float *wa = a.ab_w + (int64_t)h * a.d, *wb = a.ab_w + (int64_t)(a.H + h) * a.d;
        const int per = (a.d + kSsmSplit - 1) / kSsmSplit;
        const int i0 = rank * per, i1 = min(a.d, i0 + per);
        for (int t0 = 0; t0 < N; t0 += kMaxN) {
            float pa[kMaxN], pb[kMaxN], ps[kMaxN];
#pragma unroll
            for (int t = 0; t < kMaxN; t++) pa[t] = pb[t] = ps[t] = 0.f;
            for (int i = i0 + tid; i < i1; i += 256) {
                const float al = wa[i], be = wb[i], nw = a.in_norm ? a.in_norm[i] : 1.f;
#pragma unroll
                for (int t = 0; t < kMaxN; t++)
                    if (t0 + t < N) {
                        const float xv = a.xn[(int64_t)(t0 + t) * a.d + i], xn = xv * nw;
                        pa[t] += al * xn;
                        pb[t] += be * xn;
                        ps[t] += xv * xv;
                    }
            }
#pragma unroll
            for (int t = 0; t < kMaxN; t++) {
                const float va = warp_sum(pa[t]), vb = warp_sum(pb[t]), vs = warp_sum(ps[t]);
                if (lane == 0 && t0 + t < N) {
                    m.red_n[warp][t0 + t] = va;
                    m.red_n[warp][kChunkMax + t0 + t] = vb;
                    m.red_n[warp][2 * kChunkMax + t0 + t] = vs;
                }
            }
        }
        __syncthreads();
        for (int i = tid; i < 3 * N; i += 256) {
            const int which = i / N, t = i % N;
            float v = 0.f;
            for (int w8 = 0; w8 < 8; w8++) v += m.red_n[w8][which * kChunkMax + t];
            m.ab_part[which][t] = v;
        }
    }
    // 3. the previous call's replay record
    float *rec = a.rkv + (int64_t)h * kMaxN * REC;
    for (int i = tid; i < r * HD; i += 256) m.rk[i / HD][i % HD] = rec[(i / HD) * REC + i % HD];
    for (int i = tid; i < r * RPC; i += 256) m.rv[i / RPC][i % RPC] = rec[(i / RPC) * REC + HD + r0 + i % RPC];
    if (tid < r) {
        m.rdec[tid] = rec[tid * REC + 2 * HD];
        m.rbeta[tid] = rec[tid * REC + 2 * HD + 1];
    }
    cluster.sync();  // conv slices and alpha/beta partials visible to the cluster
    // 4. the head's q and k from their owners; alpha / beta over the slices in rank order
    for (int i = tid; i < N * HD; i += 256) {
        const int t = i / HD, c = i % HD, src = c / RPC, ci = c % RPC;
        ChunkSmem<HD> &o = *cluster.map_shared_rank(&m, src);
        m.xq[t][c] = o.cq[t][ci];
        m.xk[t][c] = o.ck[t][ci];
    }
    for (int i = tid; i < 3 * N; i += 256) {
        const int which = i / N, t = i % N;
        float v = 0.f;
        for (int q = 0; q < kSsmSplit; q++) v += cluster.map_shared_rank(&m, q)->ab_part[which][t];
        m.ab[which][t] = v;
    }
    __syncthreads();
    if (a.in_norm)
        for (int t = tid; t < N; t += 256) {
            const float iv = 1.0f / sqrtf(m.ab[2][t] / (float)a.d + a.eps);
            m.ab[0][t] *= iv;
            m.ab[1][t] *= iv;
        }
    __syncthreads();
    // 5. L2 norms of q, k and the f64 gates, one warp per token
    for (int t = warp; t < N; t += 8) {
        float qs = 0.f, ks = 0.f;
        for (int i = lane; i < HD; i += 32) {
            qs += m.xq[t][i] * m.xq[t][i];
            ks += m.xk[t][i] * m.xk[t][i];
        }
        qs = warp_sum(qs);
        ks = warp_sum(ks);
        const float scale = 1.0f / sqrtf((float)HD);
        const float qn = 1.0f / (sqrtf(qs) + 1e-6f) * scale, kn = 1.0f / (sqrtf(ks) + 1e-6f);
        __syncwarp();
        for (int i = lane; i < HD; i += 32) {
            m.xq[t][i] *= qn;
            m.xk[t][i] *= kn;
        }
        if (lane == 0) {
            double av = (double)m.ab[0][t] + (double)a.dt_bias[h];
            av = av < -20.0 ? -20.0 : (av > 20.0 ? 20.0 : av);
            const double sp = log(1.0 + exp(av));
            const float dec = (float)((double)a.ssm_a[h] * sp);
            m.ndec[t] = expf(dec);
            double bv = (double)m.ab[1][t];
            bv = bv < -20.0 ? -20.0 : (bv > 20.0 ? 20.0 : bv);
            m.nbeta[t] = (float)(1.0 / (1.0 + exp(-bv)));
        }
    }
    __syncthreads();
    // 6. committed conv history: the last K-1 inputs of history + replayed + new tokens
    //    (every owned channel's window was read in step 1, before the cluster barrier)
    for (int lc = tid; lc < 3 * RPC; lc += 256) {
        const int part = lc / RPC, i = lc % RPC;
        const int ch = part * qk + h * HD + r0 + i;
        float nh[3];
#pragma unroll
        for (int j = 0; j < 3; j++) nh[j] = j < K - 1 ? *win(r + N + j, ch) : 0.f;
#pragma unroll
        for (int j = 0; j < 3; j++)
            if (j < K - 1) a.hist[(int64_t)j * C + ch] = nh[j];
    }
    // 7. the state rows through the replayed and the new tokens, committed at the end
    const int row = tid / TPR, lc = tid % TPR;
    float *Sp = a.S + ((int64_t)h * HD + r0 + row) * HD + lc;
    float st[CPT];
#pragma unroll
    for (int e = 0; e < CPT; e++) st[e] = Sp[TPR * e];
    auto update = [&](const float *kv, float dec, float beta, float vrow) {
        float sk = 0.f;
#pragma unroll
        for (int e = 0; e < CPT; e++) {
            st[e] *= dec;
            sk += st[e] * kv[lc + TPR * e];
        }
#pragma unroll
        for (int o = 1; o < TPR; o <<= 1) sk += __shfl_xor_sync(0xffffffffu, sk, o);
        const float dd = beta * (vrow - sk);
#pragma unroll
        for (int e = 0; e < CPT; e++) st[e] += dd * kv[lc + TPR * e];
    };
    for (int j = 0; j < r; j++) update(m.rk[j], m.rdec[j], m.rbeta[j], m.rv[j][row]);
    for (int t = 0; t < N; t++) {
        update(m.xk[t], m.ndec[t], m.nbeta[t], m.cv[t][row]);
        float y = 0.f;
#pragma unroll
        for (int e = 0; e < CPT; e++) y += st[e] * m.xq[t][lc + TPR * e];
#pragma unroll
        for (int o = 1; o < TPR; o <<= 1) y += __shfl_xor_sync(0xffffffffu, y, o);
        if (lc == 0) m.ys[t][row] = y;
    }
#pragma unroll
    for (int e = 0; e < CPT; e++) Sp[TPR * e] = st[e];
    __syncthreads();
    // 8. per-head RMSNorm (partial sums of squares over the cluster in rank order), gate
    for (int t = warp; t < N; t += 8) {
        const float v = lane < RPC ? m.ys[t][lane] * m.ys[t][lane] : 0.f;
        const float t2 = warp_sum(v);
        if (lane == 0) m.ssq[t] = t2;
    }
    cluster.sync();
    for (int i = tid; i < N * RPC; i += 256) {
        const int t = i / RPC, c = i % RPC;
        float ss = 0.f;
        for (int q = 0; q < kSsmSplit; q++) ss += cluster.map_shared_rank(&m, q)->ssq[t];
        const float scale = 1.0f / sqrtf(ss / (float)HD + a.eps);
        const float z = a.proj[(int64_t)t * a.ldp + C + h * HD + r0 + c];
        const float yn = m.ys[t][c] * scale * a.norm_w[r0 + c];
        a.y[(int64_t)t * a.ldy + h * HD + r0 + c] = yn * z * (1.0f / (1.0f + expf(-z)));
    }
    cluster.sync();  // peers may still read this CTA's shared memory
}

cudaError_t ssm_chunk(const SsmArgs &a, int head_dim, cudaStream_t s) {
    if (a.N < 1 || a.N > kChunkMax || a.K < 1 || a.K > 4) return cudaErrorInvalidValue;
    const dim3 grid(kSsmSplit, a.H, 1);
    if (head_dim == 128) {
        static DeviceFlags attr;
        if (!attr.test()) {
            cudaError_t e = cudaFuncSetAttribute(ssm_chunk_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)sizeof(ChunkSmem<128>));
            if (e != cudaSuccess) return e;
            attr.set();
        }
        return launch_k(ssm_chunk_kernel<128>, grid, dim3(256), sizeof(ChunkSmem<128>), s, a);
    }
    if (head_dim == 64) {
        static DeviceFlags attr;
        if (!attr.test()) {
            cudaError_t e = cudaFuncSetAttribute(ssm_chunk_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)sizeof(ChunkSmem<64>));
            if (e != cudaSuccess) return e;
            attr.set();
        }
        return launch_k(ssm_chunk_kernel<64>, grid, dim3(256), sizeof(ChunkSmem<64>), s, a);
    }
    return cudaErrorInvalidValue;
}

cudaError_t ssm_step(const SsmArgs &a, int head_dim, int batch, cudaStream_t s) {
    if (a.N < 1 || a.N > kMaxN || a.K < 1 || a.K > 4 || batch < 1) return cudaErrorInvalidValue;
    // batches: one CTA per (head, request), two per SM (the cluster kernel with
    // kSsmSplit CTAs per head and request measured 42.9 against 31.7 ms per
    // config-4 step)
    if (batch > 1) {
        const dim3 grid(a.H, batch);
        if (head_dim == 128) return launch_k(ssm_batch_kernel<128>, grid, dim3(512), 0, s, a);
        if (head_dim == 64) return launch_k(ssm_batch_kernel<64>, grid, dim3(256), 0, s, a);
        return cudaErrorInvalidValue;
    }
    const dim3 grid(kSsmSplit, a.H, batch);
    if (head_dim == 128) return launch_k(ssm_step_kernel<128>, grid, dim3(256), 0, s, a);
    if (head_dim == 64) return launch_k(ssm_step_kernel<64>, grid, dim3(256), 0, s, a);
    return cudaErrorInvalidValue;
}

// ----------------------------------------------------------- attention ------
// FullAttentionCPU (ModelCPU.jl:787-887) for N new tokens of one sequence:
// per-head [q; gate] rows, RMSNorm + half-split partial RoPE of q and k
// (rmsnorm_rotary!, :188-232), K/V written at the token positions, GQA
// attention with scale 1/sqrt(hd) over keys 0..pos+t, output x sigmoid(gate).
//
// Grid (kAttnSplit, n_head), one cluster of kAttnSplit CTAs per query head:
// CTA `rank` takes a contiguous slice of the keys (flash-decoding split) and
// runs an online softmax over it in chunks of 64 keys (FlashAttention.jl:19-84
// uses the same chunking over all keys); the partial (max, sum, P.V) of the
// slices are combined through distributed shared memory, each CTA finishing
// HD / kAttnSplit output dims.  Every CTA normalises the new keys itself and
// reads them from shared memory; one CTA per KV head writes them to the cache
// (no CTA reads the new positions from the cache, so there is no race).
constexpr int kAttnSplit = 8;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// the RoPE pairs of an attention call: pair i < pairs rotates dims
// (i, i + off) with table entries [pos * ld + i]
struct RopeSpec { int pairs, off, ld; };
__host__ __device__ inline RopeSpec rope_spec(const AttnArgs &a) {
    const int h = a.rotary_dim / 2;
    return {a.rope_pairs > 0 ? a.rope_pairs : h, a.rope_off > 0 ? a.rope_off : h, a.rope_ld > 0 ? a.rope_ld : h};
}
// causal, and within the sliding window when there is one
__device__ __forceinline__ bool key_visible(const AttnArgs &a, int j, int qpos) {
    return j <= qpos && (a.window <= 0 || j > qpos - a.window);
}
// attention logit softcap (Gemma4.jl:420-423): tanh(s / cap) cap
__device__ __forceinline__ float score_cap(const AttnArgs &a, float s) {
    return a.softcap > 0.f ? tanhf(s / a.softcap) * a.softcap : s;
}

template <int HD>
__global__ void __cluster_dims__(kAttnSplit, 1, 1) __launch_bounds__(256) attn_step_kernel(AttnArgs a) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    constexpr int G = 256 / HD;   // key groups of the P.V product
    constexpr int DL = HD / 32;   // dims per lane in the score dot products
    constexpr int DS = HD / kAttnSplit;
    const int rank = (int)cluster.block_rank();
    const int h = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int N = a.N, ratio = a.nh / a.nkv, kvh = h / ratio;
    pdl_trigger();
    pdl_wait();
    {  // request blockIdx.z of a batched call
        const int64_t b = blockIdx.z;
        a.qkv += b * a.N * a.ldq;
        a.out += b * a.N * a.ldo;
        a.kc += b * a.b_kv;
        a.vc += b * a.b_kv;
        a.pos += b * a.b_pos;
    }
    const int p0 = *a.pos;
    const int nkeys = p0 + N;
    const int per = (nkeys + kAttnSplit - 1) / kAttnSplit;
    const int lo = min(nkeys, rank * per), hi = min(nkeys, lo + per);
    {  // the slice's cached K and V rows toward L2 while q, k, v are normalised
        const int hic = min(hi, p0), lines = HD * 4 / 128;
        for (int i = tid; i < (hic > lo ? hic - lo : 0) * lines; i += 256) {
            const int64_t o = ((int64_t)(lo + i / lines) * a.nkv + kvh) * HD + (i % lines) * 32;
            asm volatile("prefetch.global.L2 [%0];" ::"l"(a.kc + o));
            asm volatile("prefetch.global.L2 [%0];" ::"l"(a.vc + o));
        }
    }
    __shared__ __align__(16) float q[kMaxN][HD];
    __shared__ __align__(16) float kn[kMaxN][HD];
    __shared__ __align__(16) float vn[kMaxN][HD];
    __shared__ __align__(16) float po[kMaxN][HD];  // this slice's P.V (unnormalised)
    __shared__ float sc[kMaxN][64];
    __shared__ float ms[kMaxN], ls[kMaxN], fs[kMaxN];
    const RopeSpec rs = rope_spec(a);
    const int qs = a.gated ? 2 : 1;  // q rows per head: [q; gate] or q

    // 1. q of this head, new k and v of its KV head; RMSNorm + RoPE (warp t =
    //    token t).  A thread's loads are all issued before its shared stores,
    //    and the norm weights are held in registers.
    {
        constexpr int LPT = (kMaxN * HD + 255) / 256;
        float qv[LPT], kv[LPT], vv[LPT];
#pragma unroll
        for (int k = 0; k < LPT; k++) {
            const int i = tid + 256 * k, t = i / HD, d = i % HD;
            const float *row = a.qkv + (int64_t)t * a.ldq;
            const bool in = i < N * HD;
            qv[k] = in ? row[(int64_t)h * qs * HD + d] : 0.f;
            kv[k] = in ? row[(int64_t)a.nh * qs * HD + kvh * HD + d] : 0.f;
            vv[k] = in ? row[(int64_t)a.nh * qs * HD + a.nkv * HD + kvh * HD + d] : 0.f;
        }
#pragma unroll
        for (int k = 0; k < LPT; k++) {
            const int i = tid + 256 * k, t = i / HD, d = i % HD;
            if (i < N * HD) {
                q[t][d] = qv[k];
                kn[t][d] = kv[k];
                vn[t][d] = vv[k];
            }
        }
    }
    float qw[HD / 32], kw[HD / 32];
#pragma unroll
    for (int e = 0; e < HD / 32; e++) {
        qw[e] = a.q_norm[lane + 32 * e];
        kw[e] = a.k_norm[lane + 32 * e];
    }
    if (tid < kMaxN) {
        ms[tid] = -CUDART_INF_F;
        ls[tid] = 0.f;
    }
    __syncthreads();
    if (warp < N) {
        const int t = warp;
        float sq = 0.f, sk = 0.f;
        for (int d = lane; d < HD; d += 32) {
            sq += q[t][d] * q[t][d];
            sk += kn[t][d] * kn[t][d];
        }
        sq = warp_sum(sq);
        sk = warp_sum(sk);
        const float iq = 1.0f / sqrtf(sq / (float)HD + a.eps), ik = 1.0f / sqrtf(sk / (float)HD + a.eps);
#pragma unroll
        for (int e = 0; e < HD / 32; e++) {
            const int d = lane + 32 * e;
            q[t][d] = q[t][d] * iq * qw[e];
            kn[t][d] = kn[t][d] * ik * kw[e];
        }
        if (a.vnorm) {  // rmsnorm_no_scale! (CommonOps.jl:43-53)
            float sv = 0.f;
            for (int d = lane; d < HD; d += 32) sv += vn[t][d] * vn[t][d];
            sv = warp_sum(sv);
            const float iv = 1.0f / sqrtf(sv / (float)HD + a.eps);
            for (int d = lane; d < HD; d += 32) vn[t][d] = vn[t][d] * iv;
        }
        __syncwarp();
        const float *cs = a.rope_cos + (int64_t)(p0 + t) * rs.ld, *sn = a.rope_sin + (int64_t)(p0 + t) * rs.ld;
        for (int i = lane; i < rs.pairs; i += 32) {
            const float c = cs[i], s_ = sn[i];
            float x1 = q[t][i], x2 = q[t][i + rs.off];
            q[t][i] = x1 * c - x2 * s_;
            q[t][i + rs.off] = x1 * s_ + x2 * c;
            x1 = kn[t][i];
            x2 = kn[t][i + rs.off];
            kn[t][i] = x1 * c - x2 * s_;
            kn[t][i + rs.off] = x1 * s_ + x2 * c;
        }
    }
    __syncthreads();
    if (rank == 0 && h % ratio == 0) {
        for (int i = tid; i < N * HD; i += 256) {
            const int t = i / HD, d = i % HD;
            const int64_t o = ((int64_t)(p0 + t) * a.nkv + kvh) * HD + d;
            a.kc[o] = kn[t][d];
            a.vc[o] = vn[t][d];
        }
    }

    // 2. keys lo..hi: scores, online softmax, P.V, in chunks of 64
    const float scale = a.scale > 0.f ? a.scale : 1.0f / sqrtf((float)HD);
    const int d = tid % HD, g = tid / HD;
    float o[kMaxN];
#pragma unroll
    for (int t = 0; t < kMaxN; t++) o[t] = 0.f;
    for (int j0 = lo; j0 < hi; j0 += 64) {
        const int nj = min(64, hi - j0);
        for (int jj = warp; jj < nj; jj += 8) {
            const int j = j0 + jj;
            const float *kp = j < p0 ? a.kc + ((int64_t)j * a.nkv + kvh) * HD : kn[j - p0];
            float kd[DL];
#pragma unroll
            for (int e = 0; e < DL; e++) kd[e] = kp[lane + 32 * e];
#pragma unroll
            for (int t = 0; t < kMaxN; t++) {
                if (t < N) {
                    float part = 0.f;
#pragma unroll
                    for (int e = 0; e < DL; e++) part += q[t][lane + 32 * e] * kd[e];
                    part = warp_sum(part);
                    if (lane == 0) sc[t][jj] = key_visible(a, j, p0 + t) ? score_cap(a, part * scale) : -CUDART_INF_F;
                }
            }
        }
        __syncthreads();
        if (warp < N) {
            const int t = warp;
            const float s0 = lane < nj ? sc[t][lane] : -CUDART_INF_F;
            const float s1 = lane + 32 < nj ? sc[t][lane + 32] : -CUDART_INF_F;
            const float mo = ms[t], mn = fmaxf(mo, warp_max(fmaxf(s0, s1)));
            float f = 1.f, e0 = 0.f, e1 = 0.f;
            if (mn != -CUDART_INF_F) {
                f = expf(mo - mn);
                e0 = expf(s0 - mn);
                e1 = expf(s1 - mn);
            }
            if (lane < nj) sc[t][lane] = e0;
            if (lane + 32 < nj) sc[t][lane + 32] = e1;
            const float ps = warp_sum(e0 + e1);
            if (lane == 0) {
                ls[t] = ls[t] * f + ps;
                ms[t] = mn;
                fs[t] = f;
            }
        }
        __syncthreads();
#pragma unroll
        for (int t = 0; t < kMaxN; t++)
            if (t < N) o[t] *= fs[t];
#pragma unroll 4
        for (int jj = g; jj < nj; jj += G) {
            const int j = j0 + jj;
            const float vd = j < p0 ? a.vc[((int64_t)j * a.nkv + kvh) * HD + d] : vn[j - p0][d];
#pragma unroll
            for (int t = 0; t < kMaxN; t++)
                if (t < N) o[t] += sc[t][jj] * vd;
        }
        __syncthreads();  // sc and fs are rewritten by the next chunk
    }
    // the key groups' partials, summed in group order
    for (int gg = 0; gg < G; gg++) {
        if (g == gg) {
#pragma unroll
            for (int t = 0; t < kMaxN; t++)
                if (t < N) po[t][d] = gg == 0 ? o[t] : po[t][d] + o[t];
        }
        __syncthreads();
    }

    // 3. combine the slices (distributed shared memory); this CTA: dims rank*DS ..
    cluster.sync();
    for (int i = tid; i < N * DS; i += 256) {
        const int t = i / DS, dd = rank * DS + i % DS;
        float M = -CUDART_INF_F;
        for (int r = 0; r < kAttnSplit; r++) M = fmaxf(M, cluster.map_shared_rank(&ms[0], r)[t]);
        float L = 0.f, O = 0.f;
        for (int r = 0; r < kAttnSplit; r++) {
            const float mr = cluster.map_shared_rank(&ms[0], r)[t];
            if (mr == -CUDART_INF_F) continue;
            const float w = expf(mr - M);
            L += cluster.map_shared_rank(&ls[0], r)[t] * w;
            O += cluster.map_shared_rank(&po[0][0], r)[t * HD + dd] * w;
        }
        float y = O / L;
        if (a.gated) {
            const float gv = a.qkv[(int64_t)t * a.ldq + (int64_t)h * 2 * HD + HD + dd];
            y *= 1.0f / (1.0f + expf(-gv));
        }
        a.out[(int64_t)t * a.ldo + (int64_t)h * HD + dd] = y;
    }
    cluster.sync();  // peers may still read this CTA's shared memory
}

// Split-KV (flash-decoding) attention, for batches and long caches: grid
// (S, n_kv x row groups, B), no cluster.  CTA (s, y, b) takes keys
// [s kps, (s + 1) kps) of request b - kps = attn_kps(nkeys, S), a multiple of
// kGrpKeys sized from that request's own key count, so the live keys are
// always spread evenly over the slices - for up to hg query heads of one KV
// group (rows r = hh N + t, at most kGrpRows), so each row group reads every
// cached key and value once, and the slice count grows with the cache length
// (few KV heads or requests still fill the GPU).  Keys are staged in chunks of
// kGrpKeys in shared memory (K rows padded by four floats: 16-byte loads
// without bank conflicts); thread (key jj, row group w) scores rows w, w + 8,
// ..., one warp per row updates the online softmax, and thread d accumulates
// P.V for dims d (+ 256) of every row.  The slice's unnormalised (max, sum,
// P.V) per row goes to scratch; attn_combine_kernel merges the slices with the
// online-softmax rescaling and applies the output gate.
//
// Scratch per slice s (rows = B nh N, row id (b nh + h) N + t):
// [max rows][sum rows][P.V rows x HD] at part + s rows (HD + 2).
constexpr int kGrpKeys = 32;
constexpr int kGrpRows = 32;      // hg * N
constexpr int kSplitCtas = 8 * 148;  // target CTAs of one split launch
constexpr int kMaxSplits = 256;

__host__ __device__ __forceinline__ int attn_kps(int nkeys, int S) {
    const int per = (nkeys + S - 1) / S;
    return max(kGrpKeys, (per + kGrpKeys - 1) / kGrpKeys * kGrpKeys);
}

template <int HD>
struct GrpSmem {
    static constexpr int KS = HD + 4;  // 16-byte rows; key jj starts 4 jj banks further
    // floats: q[R][HD] | kn[N][HD] | vn[N][HD] | Ks[kGrpKeys][KS] | Vs[kGrpKeys][HD] | sc[R][kGrpKeys] | ms, ls, fs [R]
    static __host__ __device__ int bytes(int R, int N) {
        return 4 * (R * HD + 2 * N * HD + kGrpKeys * KS + kGrpKeys * HD + R * kGrpKeys + 3 * R);
    }
};

// Step 1 of the split-KV attention of a row group (both split kernels): its
// R = heads x N q rows and the N new k, v rows into shared memory (q [R][HD],
// kn / vn [N][HD]), then per row (warp per row) RMSNorm with its weights, RoPE
// for q and k, the weightless RMSNorm of v when vnorm (CommonOps.jl:43-53).
// Every global load of a thread is issued before its shared stores (the
// stores cannot be ordered past loads through a generic pointer otherwise),
// the norm weights sit in registers and the N positions' RoPE tables are
// staged in rope_s (2 N pairs floats) first.  BAR as in bar256.
template <int HD, int BAR, int NTH = 256>
__device__ __forceinline__ void attn_rows_in(const AttnArgs &a, float *q, float *kn, float *vn, float *rope_s, int R,
                                             int h0, int g, int p0, int tid) {
    static_assert(BAR == 0 || NTH == 256, "named barriers cover 256 threads");
    constexpr int LB = 8;  // loads in flight per thread per batch
    const int N = a.N, lane = tid & 31, warp = tid >> 5, qs = a.gated ? 2 : 1;
    const RopeSpec rs = rope_spec(a);
    for (int i0 = tid; i0 < R * HD; i0 += NTH * LB) {
        float v[LB];
#pragma unroll
        for (int k = 0; k < LB; k++) {
            const int i = i0 + NTH * k, r = i / HD, d = i % HD, hh = r / N, t = r % N;
            v[k] = i < R * HD ? a.qkv[(int64_t)t * a.ldq + (int64_t)(h0 + hh) * qs * HD + d] : 0.f;
        }
#pragma unroll
        for (int k = 0; k < LB; k++)
            if (i0 + NTH * k < R * HD) q[i0 + NTH * k] = v[k];
    }
    for (int i0 = tid; i0 < N * HD; i0 += NTH * LB) {
        float kv[LB], vv[LB];
#pragma unroll
        for (int k = 0; k < LB; k++) {
            const int i = i0 + NTH * k, t = i / HD, d = i % HD;
            const float *row = a.qkv + (int64_t)t * a.ldq + (int64_t)a.nh * qs * HD;
            kv[k] = i < N * HD ? row[g * HD + d] : 0.f;
            vv[k] = i < N * HD ? row[a.nkv * HD + g * HD + d] : 0.f;
        }
#pragma unroll
        for (int k = 0; k < LB; k++)
            if (i0 + NTH * k < N * HD) {
                kn[i0 + NTH * k] = kv[k];
                vn[i0 + NTH * k] = vv[k];
            }
    }
    for (int i0 = tid; i0 < N * rs.pairs; i0 += NTH * LB) {
        float c[LB], sn[LB];
#pragma unroll
        for (int k = 0; k < LB; k++) {
            const int i = i0 + NTH * k, t = i / rs.pairs, pi = i % rs.pairs;
            const int64_t o = (int64_t)(p0 + t) * rs.ld + pi;
            c[k] = i < N * rs.pairs ? a.rope_cos[o] : 0.f;
            sn[k] = i < N * rs.pairs ? a.rope_sin[o] : 0.f;
        }
#pragma unroll
        for (int k = 0; k < LB; k++)
            if (i0 + NTH * k < N * rs.pairs) {
                rope_s[i0 + NTH * k] = c[k];
                rope_s[N * rs.pairs + i0 + NTH * k] = sn[k];
            }
    }
    float qw[HD / 32], kw[HD / 32];
#pragma unroll
    for (int j = 0; j < HD / 32; j++) {
        qw[j] = a.q_norm[lane + 32 * j];
        kw[j] = a.k_norm[lane + 32 * j];
    }
    bar256<BAR>();
    for (int rr = warp; rr < R + N + (a.vnorm ? N : 0); rr += NTH / 32) {
        if (rr >= R + N) {
            float *x = vn + (rr - R - N) * HD;
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < HD / 32; j++) ss += x[lane + 32 * j] * x[lane + 32 * j];
            ss = warp_sum(ss);
            const float iv = 1.0f / sqrtf(ss / (float)HD + a.eps);
#pragma unroll
            for (int j = 0; j < HD / 32; j++) x[lane + 32 * j] = x[lane + 32 * j] * iv;
            continue;
        }
        const bool isq = rr < R;
        float *x = isq ? q + rr * HD : kn + (rr - R) * HD;
        const int t = isq ? rr % N : rr - R;
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < HD / 32; j++) ss += x[lane + 32 * j] * x[lane + 32 * j];
        ss = warp_sum(ss);
        const float iv = 1.0f / sqrtf(ss / (float)HD + a.eps);
#pragma unroll
        for (int j = 0; j < HD / 32; j++) x[lane + 32 * j] = x[lane + 32 * j] * iv * (isq ? qw[j] : kw[j]);
        __syncwarp();
        const float *cs = rope_s + t * rs.pairs, *sn = rope_s + (N + t) * rs.pairs;
        for (int i = lane; i < rs.pairs; i += 32) {
            const float c = cs[i], s_ = sn[i];
            const float x1 = x[i], x2 = x[i + rs.off];
            x[i] = x1 * c - x2 * s_;
            x[i + rs.off] = x1 * s_ + x2 * c;
        }
    }
}

// virtual block (bx, by, bz) of a grid with gz requests; tid < 256; gs its
// shared memory (GrpSmem<HD>::bytes); BAR as in bar256
template <int HD, int BAR>
__device__ __forceinline__ void attn_part_body(AttnArgs a, int hg, int S, int bx, int by, int bz, int gz, int tid,
                                               float *gs) {
    constexpr int KS = GrpSmem<HD>::KS;
    constexpr int RPT = (kGrpRows * HD + 255) / 256;  // P.V outputs per thread (upper bound)
    const int lane = tid & 31, warp = tid >> 5;
    const int N = a.N, ratio = a.nh / a.nkv, nrg = (ratio + hg - 1) / hg;
    const int g = by / nrg, hb = by % nrg, h0 = g * ratio + hb * hg;
    const int R = min(hg, ratio - hb * hg) * N;
    const int sl = bx, b = bz;
    float *q = gs, *kn = q + R * HD, *vn = kn + N * HD, *Ks = vn + N * HD, *Vs = Ks + kGrpKeys * KS;
    float *sc = Vs + kGrpKeys * HD, *ms = sc + R * kGrpKeys, *ls = ms + R, *fs = ls + R;
    a.qkv += (int64_t)b * N * a.ldq;
    a.kc += b * a.b_kv;
    a.vc += b * a.b_kv;
    const int p0 = a.pos[(int64_t)b * a.b_pos];
    const int nkeys = p0 + N, kps = attn_kps(nkeys, S);
    const int lo = sl * kps, hi = min(nkeys, lo + kps);
    if (lo >= nkeys) return;  // the combine reads only the slices below nkeys
    const RopeSpec rs = rope_spec(a);
    const int64_t rows_all = (int64_t)gz * a.nh * N, rid_base = ((int64_t)b * a.nh + h0) * N;
    if (a.window > 0 && sl > 0 && hi + a.window <= p0 + 1) {
        // every key of this slice is outside every query's window (this
        // request's new keys are written by slice 0): an empty partial state
        float *pm = a.part + (int64_t)sl * rows_all * (HD + 2), *pl = pm + rows_all, *po = pl + rows_all;
        for (int i = tid; i < R * HD; i += 256) po[(rid_base + i / HD) * HD + i % HD] = 0.f;
        if (tid < R) {
            pm[rid_base + tid] = -CUDART_INF_F;
            pl[rid_base + tid] = 0.f;
        }
        return;
    }

    // 1. the row group's q rows, the new k and v; RMSNorm + RoPE (warp per row);
    //    the RoPE tables staged in the K chunk buffer (free until step 2)
    if (tid < R) {
        ms[tid] = -CUDART_INF_F;
        ls[tid] = 0.f;
    }
    attn_rows_in<HD, BAR>(a, q, kn, vn, Ks, R, h0, g, p0, tid);
    bar256<BAR>();
    // one CTA per (KV head, request) writes the new keys; no CTA reads them from the cache
    if (sl == 0 && hb == 0) {
        for (int i = tid; i < N * HD; i += 256) {
            const int t = i / HD, d = i % HD;
            const int64_t o = ((int64_t)(p0 + t) * a.nkv + g) * HD + d;
            a.kc[o] = kn[i];
            a.vc[o] = vn[i];
        }
    }

    // 2. keys lo..hi in chunks: scores, online softmax, P.V
    const float scale = a.scale > 0.f ? a.scale : 1.0f / sqrtf((float)HD);
    float o[RPT];
#pragma unroll
    for (int k = 0; k < RPT; k++) o[k] = 0.f;
    for (int j0 = lo; j0 < hi; j0 += kGrpKeys) {
        const int nj = min(kGrpKeys, hi - j0);
        {
            // the chunk's K and V rows, 16 bytes per load, every load of a thread in flight at once
            constexpr int NL = kGrpKeys * HD / 4 / 256;
            float4 kv[NL], vv[NL];
#pragma unroll
            for (int l = 0; l < NL; l++) {
                const int i = tid + 256 * l, jj = i / (HD / 4), d = 4 * (i % (HD / 4)), j = j0 + jj;
                kv[l] = vv[l] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (jj < nj && j < p0) {
                    const int64_t o = ((int64_t)j * a.nkv + g) * HD + d;
                    kv[l] = *reinterpret_cast<const float4 *>(a.kc + o);
                    vv[l] = *reinterpret_cast<const float4 *>(a.vc + o);
                } else if (jj < nj) {
                    kv[l] = *reinterpret_cast<const float4 *>(kn + (j - p0) * HD + d);
                    vv[l] = *reinterpret_cast<const float4 *>(vn + (j - p0) * HD + d);
                }
            }
#pragma unroll
            for (int l = 0; l < NL; l++) {
                const int i = tid + 256 * l, jj = i / (HD / 4), d = 4 * (i % (HD / 4));
                *reinterpret_cast<float4 *>(Ks + jj * KS + d) = kv[l];
                *reinterpret_cast<float4 *>(Vs + jj * HD + d) = vv[l];
            }
        }
        bar256<BAR>();
        {
            // thread (jj = lane, row group = warp): K row jj read once, q rows broadcast
            const int jj = lane, j = j0 + jj;
            constexpr int RG = kGrpRows / 8;
            float acc[RG];
#pragma unroll
            for (int k = 0; k < RG; k++) acc[k] = 0.f;
            const float4 *kr = reinterpret_cast<const float4 *>(Ks + jj * KS);
#pragma unroll 4
            for (int d4 = 0; d4 < HD / 4; d4++) {
                const float4 kv = kr[d4];
#pragma unroll
                for (int k = 0; k < RG; k++) {
                    const int r = warp + 8 * k;
                    if (r < R) {
                        const float4 qv = reinterpret_cast<const float4 *>(q + r * HD)[d4];
                        acc[k] += qv.x * kv.x + qv.y * kv.y + qv.z * kv.z + qv.w * kv.w;
                    }
                }
            }
#pragma unroll
            for (int k = 0; k < RG; k++) {
                const int r = warp + 8 * k;
                if (r < R)
                    sc[r * kGrpKeys + jj] = (jj < nj && key_visible(a, j, p0 + r % N)) ? score_cap(a, acc[k] * scale)
                                                                                      : -CUDART_INF_F;
            }
        }
        bar256<BAR>();
        for (int r = warp; r < R; r += 8) {
            const float sv = lane < kGrpKeys ? sc[r * kGrpKeys + lane] : -CUDART_INF_F;
            const float mo = ms[r], mn = fmaxf(mo, warp_max(sv));
            float f = 1.f, e = 0.f;
            if (mn != -CUDART_INF_F) {
                f = expf(mo - mn);
                e = expf(sv - mn);
            }
            if (lane < kGrpKeys) sc[r * kGrpKeys + lane] = e;
            const float ps = warp_sum(e);
            if (lane == 0) {
                ls[r] = ls[r] * f + ps;
                ms[r] = mn;
                fs[r] = f;
            }
        }
        bar256<BAR>();
        // thread: dim d = (tid + 256 k) % HD of row (tid + 256 k) / HD; V loaded once per key
#pragma unroll
        for (int k = 0; k < RPT; k++) {
            const int i = tid + 256 * k;
            if (i < R * HD) o[k] *= fs[i / HD];
        }
        // four keys per step: the rows' probabilities as one 16-byte load each (the
        // chunk's tail keys have probability 0 and zeroed V rows)
        for (int jj = 0; jj < nj; jj += 4) {
            const int d = tid % HD;
            const float v0 = Vs[jj * HD + d], v1 = Vs[(jj + 1) * HD + d];
            const float v2 = Vs[(jj + 2) * HD + d], v3 = Vs[(jj + 3) * HD + d];
#pragma unroll
            for (int k = 0; k < RPT; k++) {
                const int i = tid + 256 * k;
                if (i < R * HD) {
                    const float4 p = *reinterpret_cast<const float4 *>(sc + (i / HD) * kGrpKeys + jj);
                    o[k] += p.x * v0 + p.y * v1 + p.z * v2 + p.w * v3;
                }
            }
        }
        bar256<BAR>();  // Ks, Vs, sc and fs are rewritten by the next chunk
    }

    // 3. the slice's partial state
    const int64_t rows = (int64_t)gz * a.nh * N;
    float *pm = a.part + (int64_t)sl * rows * (HD + 2), *pl = pm + rows, *po = pl + rows;
    const int64_t rid0 = ((int64_t)b * a.nh + h0) * N;  // row r of this CTA is row id rid0 + r
#pragma unroll
    for (int k = 0; k < RPT; k++) {
        const int i = tid + 256 * k;
        if (i < R * HD) po[(rid0 + i / HD) * HD + i % HD] = o[k];
    }
    if (tid < R) {
        pm[rid0 + tid] = ms[tid];
        pl[rid0 + tid] = ls[tid];
    }
}

template <int HD>
__global__ void __launch_bounds__(256) attn_part_kernel(AttnArgs a, int hg, int S) {
    extern __shared__ __align__(16) float gs[];
    pdl_trigger();
    pdl_wait();
    attn_part_body<HD, 0>(a, hg, S, blockIdx.x, blockIdx.y, blockIdx.z, gridDim.z, threadIdx.x, gs);
}

// ---- split-KV attention on the tensor cores ----------------------------------
// attn_part_kernel's work (same slices, rows, masks, online softmax and
// partial states) with the two products on mma.sync m16n8k8 tf32: scores
// S = Q K^T over a chunk of kGrpKeys keys (2 x 4 tiles of 16 x 8, one per
// warp) and O += P V (2 x HD / 8 tiles, HD / 64 per warp, accumulators in
// registers across chunks).  Each operand is split into tf32 hi + lo and
// every product is formed as hi hi + hi lo + lo hi ("3xTF32"), which keeps
// the f32 accuracy of the CUDA-core kernel (relative error ~2^-21 per
// product).  The chunks of cached keys stream global -> shared with
// cp.async into two buffers, the next chunk's copies in flight while the
// current chunk is computed.  One CTA per SM (the two K/V buffers and the
// split q take up to ~220 KB of shared memory).
__device__ __forceinline__ uint32_t tf32_of(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ void split_tf32(float x, uint32_t &hi, uint32_t &lo) {
    hi = tf32_of(x);
    lo = tf32_of(x - __uint_as_float(hi));
}
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// hi hi + hi lo + lo hi
__device__ __forceinline__ void mma_3xtf32(float (&d)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4],
                                           uint32_t bh0, uint32_t bh1, uint32_t bl0, uint32_t bl1) {
    mma_tf32(d, ah, bh0, bh1);
    mma_tf32(d, ah, bl0, bl1);
    mma_tf32(d, al, bh0, bh1);
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int NPEND>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(NPEND) : "memory"); }

constexpr int kMmaThreads = 512;  // 16 warps: the scores' two K halves, the P.V n-tiles

template <int HD>
struct MmaSmem {
    static constexpr int QS = HD + 4, KS = HD + 4, VS = HD + 8, SS = kGrpKeys + 4;
    // uint32/float words: qh[R][QS] | ql[R][QS] | Ks[2][kGrpKeys][KS] | Vs[2][kGrpKeys][VS] |
    // kn[N][HD] | vn[N][HD] | sc[R][SS] | sc2[R][SS] | ms, ls, fs [R]; the f32 q rows are
    // staged in Vs[1]
    static __host__ __device__ int words(int R, int N) {
        return 2 * R * QS + 2 * kGrpKeys * KS + 2 * kGrpKeys * VS + 2 * N * HD + 2 * R * SS + 3 * R;
    }
    static __host__ __device__ int bytes(int R, int N) { return 4 * words(R, N); }
};

template <int HD>
__global__ void __launch_bounds__(kMmaThreads, 1) attn_part_mma_kernel(AttnArgs a, int hg, int S) {
    using M = MmaSmem<HD>;
    constexpr int QS = M::QS, KS = M::KS, VS = M::VS, SS = M::SS;
    constexpr int NTH = kMmaThreads, NWP = NTH / 32;
    // P.V: HD >= 128: every warp both m-tiles and NTW n-tiles (warp + 16 u);
    // HD 64: warp w the m-tile w / 8 and the n-tile w % 8
    constexpr int MT = HD >= 128 ? 2 : 1, NTW = HD >= 128 ? HD / 128 : 1;
    extern __shared__ __align__(16) float ms_buf[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g8 = lane >> 2, t4 = lane & 3;
    const int N = a.N, ratio = a.nh / a.nkv, nrg = (ratio + hg - 1) / hg;
    const int g = blockIdx.y / nrg, hb = blockIdx.y % nrg, h0 = g * ratio + hb * hg;
    const int R = min(hg, ratio - hb * hg) * N;
    const int sl = blockIdx.x, b = blockIdx.z;
    uint32_t *qh = reinterpret_cast<uint32_t *>(ms_buf), *ql = qh + R * QS;
    float *Ks = reinterpret_cast<float *>(ql + R * QS), *Vs = Ks + 2 * kGrpKeys * KS;
    float *kn = Vs + 2 * kGrpKeys * VS, *vn = kn + N * HD, *sc = vn + N * HD;
    float *sc2 = sc + R * SS, *ms = sc2 + R * SS, *ls = ms + R, *fs = ls + R;
    float *q = Vs + kGrpKeys * VS;  // f32 q rows [R][HD], staged in the second V buffer
    pdl_trigger();
    pdl_wait();
    a.qkv += (int64_t)b * N * a.ldq;
    a.kc += b * a.b_kv;
    a.vc += b * a.b_kv;
    const int p0 = a.pos[(int64_t)b * a.b_pos];
    const int nkeys = p0 + N, kps = attn_kps(nkeys, S);
    const int lo = sl * kps, hi = min(nkeys, lo + kps);
    if (lo >= nkeys) return;  // the combine reads only the slices below nkeys
    const RopeSpec rs = rope_spec(a);
    const int64_t rows_all = (int64_t)gridDim.z * a.nh * N, rid0 = ((int64_t)b * a.nh + h0) * N;
    if (a.window > 0 && sl > 0 && hi + a.window <= p0 + 1) {
        float *pm = a.part + (int64_t)sl * rows_all * (HD + 2), *pl = pm + rows_all, *po = pl + rows_all;
        for (int i = tid; i < R * HD; i += NTH) po[(rid0 + i / HD) * HD + i % HD] = 0.f;
        if (tid < R) {
            pm[rid0 + tid] = -CUDART_INF_F;
            pl[rid0 + tid] = 0.f;
        }
        return;
    }
    // the cached keys of chunk c (j < p0) into buffer bf with cp.async; the new
    // keys (j >= p0) and the zero V rows past the slice by plain stores
    auto stage = [&](int c, int bf) {
        const int j0 = lo + c * kGrpKeys, nj = min(kGrpKeys, hi - j0);
        float *kb = Ks + bf * kGrpKeys * KS, *vb = Vs + bf * kGrpKeys * VS;
        for (int i = tid; i < kGrpKeys * (HD / 4); i += NTH) {
            const int jj = i / (HD / 4), d = 4 * (i % (HD / 4)), j = j0 + jj;
            if (jj < nj && j < p0) {
                const int64_t o = ((int64_t)j * a.nkv + g) * HD + d;
                cp_async16(kb + jj * KS + d, a.kc + o);
                cp_async16(vb + jj * VS + d, a.vc + o);
            } else if (jj < nj) {
                *reinterpret_cast<float4 *>(kb + jj * KS + d) = *reinterpret_cast<const float4 *>(kn + (j - p0) * HD + d);
                *reinterpret_cast<float4 *>(vb + jj * VS + d) = *reinterpret_cast<const float4 *>(vn + (j - p0) * HD + d);
            } else {
                *reinterpret_cast<float4 *>(kb + jj * KS + d) = make_float4(0.f, 0.f, 0.f, 0.f);
                *reinterpret_cast<float4 *>(vb + jj * VS + d) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        cp_async_commit();
    };
    const int nch = (hi - lo + kGrpKeys - 1) / kGrpKeys;

    // 1. the new k and v rows and the row group's q rows; RMSNorm + RoPE (the
    //    RoPE tables staged in the second K buffer, free until chunk 1)
    if (tid < R) {
        ms[tid] = -CUDART_INF_F;
        ls[tid] = 0.f;
    }
    attn_rows_in<HD, 0, NTH>(a, q, kn, vn, Ks + kGrpKeys * KS, R, h0, g, p0, tid);
    __syncthreads();
    // the first chunk's copies start now; the new keys are in kn / vn for it
    stage(0, 0);
    // one CTA per (KV head, request) writes the new keys; no CTA reads them from the cache
    if (sl == 0 && hb == 0) {
        for (int i = tid; i < N * HD; i += NTH) {
            const int t = i / HD, d = i % HD;
            const int64_t o = ((int64_t)(p0 + t) * a.nkv + g) * HD + d;
            a.kc[o] = kn[i];
            a.vc[o] = vn[i];
        }
    }
    for (int i = tid; i < R * HD; i += NTH) {
        uint32_t h_, l_;
        split_tf32(q[i], h_, l_);
        qh[(i / HD) * QS + i % HD] = h_;
        ql[(i / HD) * QS + i % HD] = l_;
    }
    __syncthreads();  // q split (the staging buffer is free for chunk 1)

    const float scale = a.scale > 0.f ? a.scale : 1.0f / sqrtf((float)HD);
    float oacc[MT][NTW][4];
#pragma unroll
    for (int m = 0; m < MT; m++)
#pragma unroll
        for (int u = 0; u < NTW; u++)
#pragma unroll
            for (int i = 0; i < 4; i++) oacc[m][u][i] = 0.f;
    for (int c = 0; c < nch; c++) {
        const int bf = c & 1, j0 = lo + c * kGrpKeys, nj = min(kGrpKeys, hi - j0);
        cp_async_wait<0>();
        __syncthreads();  // chunk c complete; every warp is past chunk c - 1
        if (c + 1 < nch) stage(c + 1, bf ^ 1);  // into the buffer of chunk c - 1
        const float *kb = Ks + bf * kGrpKeys * KS, *vb = Vs + bf * kGrpKeys * VS;
        {   // scores: warp (k half = warp / 8, m = warp / 4 % 2, key tile nb = warp % 4);
            //   each half sums its HD / 2 dims into its own buffer (sc, sc2)
            const int kh = warp >> 3, m = (warp >> 2) & 1, nb = warp & 3, r0 = 16 * m + g8;
            if (16 * m < R) {
                // independent accumulators per k-step parity and product term:
                // six short MMA dependency chains instead of one long one
                float ac[2][3][4];
#pragma unroll
                for (int p2 = 0; p2 < 2; p2++)
#pragma unroll
                    for (int q3 = 0; q3 < 3; q3++)
#pragma unroll
                        for (int i = 0; i < 4; i++) ac[p2][q3][i] = 0.f;
                const float *kr = kb + (8 * nb + g8) * KS;
#pragma unroll 4
                for (int kk = kh * (HD / 16); kk < (kh + 1) * (HD / 16); kk++) {
                    const int k0 = 8 * kk + t4;
                    uint32_t ah[4], al[4];
                    ah[0] = r0 < R ? qh[r0 * QS + k0] : 0u;
                    ah[1] = r0 + 8 < R ? qh[(r0 + 8) * QS + k0] : 0u;
                    ah[2] = r0 < R ? qh[r0 * QS + k0 + 4] : 0u;
                    ah[3] = r0 + 8 < R ? qh[(r0 + 8) * QS + k0 + 4] : 0u;
                    al[0] = r0 < R ? ql[r0 * QS + k0] : 0u;
                    al[1] = r0 + 8 < R ? ql[(r0 + 8) * QS + k0] : 0u;
                    al[2] = r0 < R ? ql[r0 * QS + k0 + 4] : 0u;
                    al[3] = r0 + 8 < R ? ql[(r0 + 8) * QS + k0 + 4] : 0u;
                    uint32_t bh0, bl0, bh1, bl1;
                    split_tf32(kr[k0], bh0, bl0);
                    split_tf32(kr[k0 + 4], bh1, bl1);
                    const int p2 = kk & 1;
                    mma_tf32(ac[p2][0], ah, bh0, bh1);
                    mma_tf32(ac[p2][1], ah, bl0, bl1);
                    mma_tf32(ac[p2][2], al, bh0, bh1);
                }
                float acc[4];
#pragma unroll
                for (int i = 0; i < 4; i++)
                    acc[i] = (ac[0][0][i] + ac[1][0][i]) + ((ac[0][1][i] + ac[1][1][i]) + (ac[0][2][i] + ac[1][2][i]));
                float *dst = kh ? sc2 : sc;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int r = r0 + 8 * (i >> 1), jj = 8 * nb + 2 * t4 + (i & 1);
                    if (r < R) dst[r * SS + jj] = acc[i];
                }
            }
        }
        __syncthreads();
        {   // online softmax, one half-warp per row (keys l16 and l16 + 16): all rows in one
            // round; the two halves' dot products, scaled, capped and masked
            const int r = 2 * warp + (lane >> 4), l16 = lane & 15;
            const bool rv = r < R;
            float sv[2] = {-CUDART_INF_F, -CUDART_INF_F};
            if (rv) {
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int jj = l16 + 16 * h;
                    if (jj < nj && key_visible(a, j0 + jj, p0 + r % N))
                        sv[h] = score_cap(a, (sc[r * SS + jj] + sc2[r * SS + jj]) * scale);
                }
            }
            float mx = fmaxf(sv[0], sv[1]);
#pragma unroll
            for (int o = 8; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float mo = rv ? ms[r] : -CUDART_INF_F, mn = fmaxf(mo, mx);
            float f = 1.f, e[2] = {0.f, 0.f};
            if (mn != -CUDART_INF_F) {
                f = expf(mo - mn);
                e[0] = expf(sv[0] - mn);
                e[1] = expf(sv[1] - mn);
            }
            float ps = e[0] + e[1];
#pragma unroll
            for (int o = 8; o; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            if (rv) {
                sc[r * SS + l16] = e[0];
                sc[r * SS + l16 + 16] = e[1];
                if (l16 == 0) {
                    ls[r] = ls[r] * f + ps;
                    ms[r] = mn;
                    fs[r] = f;
                }
            }
        }
        __syncthreads();
        // P.V: the warp's m-tiles and n-tiles (see MT, NTW)
#pragma unroll
        for (int mi = 0; mi < MT; mi++) {
            const int m = MT == 2 ? mi : warp >> 3;
            if (16 * m >= R) continue;
            const int r0 = 16 * m + g8;
            const float f0 = r0 < R ? fs[r0] : 1.f, f1 = r0 + 8 < R ? fs[r0 + 8] : 1.f;
#pragma unroll
            for (int u = 0; u < NTW; u++) {
                oacc[mi][u][0] *= f0;
                oacc[mi][u][1] *= f0;
                oacc[mi][u][2] *= f1;
                oacc[mi][u][3] *= f1;
            }
#pragma unroll
            for (int kk = 0; kk < kGrpKeys / 8; kk++) {
                const int k0 = 8 * kk + t4;
                uint32_t ah[4], al[4];
                split_tf32(r0 < R ? sc[r0 * SS + k0] : 0.f, ah[0], al[0]);
                split_tf32(r0 + 8 < R ? sc[(r0 + 8) * SS + k0] : 0.f, ah[1], al[1]);
                split_tf32(r0 < R ? sc[r0 * SS + k0 + 4] : 0.f, ah[2], al[2]);
                split_tf32(r0 + 8 < R ? sc[(r0 + 8) * SS + k0 + 4] : 0.f, ah[3], al[3]);
#pragma unroll
                for (int u = 0; u < NTW; u++) {
                    const int nt = MT == 2 ? warp + NWP * u : (warp & 7);
                    const int n0 = 8 * nt + g8;
                    uint32_t bh0, bl0, bh1, bl1;
                    split_tf32(vb[k0 * VS + n0], bh0, bl0);
                    split_tf32(vb[(k0 + 4) * VS + n0], bh1, bl1);
                    mma_3xtf32(oacc[mi][u], ah, al, bh0, bh1, bl0, bl1);
                }
            }
        }
        // no barrier here: the next chunk's first barrier comes before anything
        // this chunk read (its buffer, sc, fs) is rewritten
    }

    // 3. the slice's partial state
    float *pm = a.part + (int64_t)sl * rows_all * (HD + 2), *pl = pm + rows_all, *po = pl + rows_all;
#pragma unroll
    for (int mi = 0; mi < MT; mi++)
#pragma unroll
        for (int u = 0; u < NTW; u++)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int m = MT == 2 ? mi : warp >> 3, nt = MT == 2 ? warp + NWP * u : (warp & 7);
                const int r = 16 * m + g8 + 8 * (i >> 1), d = 8 * nt + 2 * t4 + (i & 1);
                if (r < R) po[(rid0 + r) * HD + d] = oacc[mi][u][i];
            }
    if (tid < R) {
        pm[rid0 + tid] = ms[tid];
        pl[rid0 + tid] = ls[tid];
    }
}

// ---- split-KV attention over a bf16 KV cache (AttnArgs::kv16) ---------------
// attn_part_mma_kernel's slices, masks, online softmax and partial states
// with the cache rows in bf16 (as the cache stores them: round to nearest
// even of the f32 rows) on mma.sync m16n8k16 bf16.  K and V enter the MMAs
// exactly; q and the probabilities P are split into three bf16 pieces
// (hi + mid + lo, ~24 bits), so every product is the f32 one of the stored
// operands: S = sum_p q_p K^T, O += sum_p P_p V.  Fragments come from shared
// memory by ldmatrix (V transposed on the fly), rows padded to an odd number
// of 16-byte units (conflict-free).  Cached rows stream in by cp.async into
// a ring of four chunk buffers (three chunks in flight), the first two
// issued before the prologue; the new rows of this step are rounded to bf16
// on their way into the staged chunk and into the cache.
template <int HD>
struct Bf16Smem {
    static constexpr int kStages = 4;          // K/V chunk buffers: chunks c+1 .. c+3 in flight
    static constexpr int kRows = 32;           // two m-tiles (R <= kGrpRows)
    static constexpr int QP = HD + 8;          // bf16 pitch: q pieces, K and V rows
    static constexpr int PP = kGrpKeys + 8;    // bf16 pitch of the P pieces
    static constexpr int SS = kGrpKeys + 4;    // f32 pitch of the scores
    // bytes: qp[3][kRows][QP] | buffer[kStages] {K[kGrpKeys][QP], V[kGrpKeys][QP]} |
    // kn[N][HD], vn[N][HD] f32 | sc, sc2 [kRows][SS] f32 | pp[3][kRows][PP] | ms, ls, fs [kRows];
    // the f32 q rows are staged in buffer 3, the RoPE tables in buffer 2
    static __host__ __device__ int buf_elems() { return 2 * kGrpKeys * QP; }
    static __host__ __device__ int bytes(int N) {
        return 2 * (3 * kRows * QP + kStages * buf_elems()) + 4 * (2 * N * HD + 2 * kRows * SS) +
               2 * 3 * kRows * PP + 4 * 3 * kRows;
    }
};
static_assert(Bf16Smem<256>::kStages == 4, "the prologue stages buffers 0-2 and loads q / RoPE into 3 / 2");
static_assert(kGrpRows <= Bf16Smem<64>::kRows, "row groups fit two m-tiles");

__device__ __forceinline__ uint16_t bf16_bits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
__device__ __forceinline__ float bf16_val(uint16_t h) { return __bfloat162float(__ushort_as_bfloat16(h)); }
// x = hi + mid + lo (each the bf16 rounding of what is left)
__device__ __forceinline__ void split_bf16x3(float x, uint16_t &h, uint16_t &m, uint16_t &l) {
    h = bf16_bits(x);
    const float r1 = x - bf16_val(h);
    m = bf16_bits(r1);
    l = bf16_bits(r1 - bf16_val(m));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    return (uint32_t)bf16_bits(lo) | ((uint32_t)bf16_bits(hi) << 16);
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t &r0, uint32_t &r1, const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r0), "=r"(r1)
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int HD>
__global__ void __launch_bounds__(kMmaThreads, 1) attn_part_bf16_kernel(AttnArgs a, int hg, int S) {
    using M = Bf16Smem<HD>;
    constexpr int QP = M::QP, PP = M::PP, SS = M::SS, NR = M::kRows;
    constexpr int NTH = kMmaThreads;
    // P.V: HD >= 128: every warp both m-tiles and NTW adjacent n-tiles;
    // HD 64: warp w the m-tile w / 8 and the n-tile w % 8
    constexpr int MT = HD >= 128 ? 2 : 1, NTW = HD >= 128 ? HD / 128 : 1;
    extern __shared__ __align__(16) uint8_t b16_buf[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g8 = lane >> 2, t4 = lane & 3;
    const int N = a.N, ratio = a.nh / a.nkv, nrg = (ratio + hg - 1) / hg;
    const int g = blockIdx.y / nrg, hb = blockIdx.y % nrg, h0 = g * ratio + hb * hg;
    const int R = min(hg, ratio - hb * hg) * N;
    const int sl = blockIdx.x, b = blockIdx.z;
    uint16_t *qp = reinterpret_cast<uint16_t *>(b16_buf);
    uint16_t *kvb = qp + 3 * NR * QP;  // [2][K | V][kGrpKeys][QP]
    float *kn = reinterpret_cast<float *>(kvb + M::kStages * M::buf_elems()), *vn = kn + N * HD;
    float *sc = vn + N * HD, *sc2 = sc + NR * SS;
    uint16_t *pp = reinterpret_cast<uint16_t *>(sc2 + NR * SS);
    float *ms = reinterpret_cast<float *>(pp + 3 * NR * PP), *ls = ms + NR, *fs = ls + NR;
    constexpr int NST = M::kStages;
    float *q = reinterpret_cast<float *>(kvb + 3 * M::buf_elems());       // f32 q rows [R][HD] in buffer 3
    float *rope_s = reinterpret_cast<float *>(kvb + 2 * M::buf_elems());  // RoPE tables in buffer 2
    pdl_trigger();
    pdl_wait();
    a.qkv += (int64_t)b * N * a.ldq;
    uint16_t *kc = reinterpret_cast<uint16_t *>(a.kc) + b * a.b_kv;
    uint16_t *vc = reinterpret_cast<uint16_t *>(a.vc) + b * a.b_kv;
    const int p0 = a.pos[(int64_t)b * a.b_pos];
    const int nkeys = p0 + N, kps = attn_kps(nkeys, S);
    const int lo = sl * kps, hi = min(nkeys, lo + kps);
    if (lo >= nkeys) return;  // the combine reads only the slices below nkeys
    const int64_t rows_all = (int64_t)gridDim.z * a.nh * N, rid0 = ((int64_t)b * a.nh + h0) * N;
    if (a.window > 0 && sl > 0 && hi + a.window <= p0 + 1) {
        float *pm = a.part + (int64_t)sl * rows_all * (HD + 2), *pl = pm + rows_all, *po = pl + rows_all;
        for (int i = tid; i < R * HD; i += NTH) po[(rid0 + i / HD) * HD + i % HD] = 0.f;
        if (tid < R) {
            pm[rid0 + tid] = -CUDART_INF_F;
            pl[rid0 + tid] = 0.f;
        }
        return;
    }
    const int nch = (hi - lo + kGrpKeys - 1) / kGrpKeys;
    // chunk c into buffer c % NST.  Cached rows (j < p0) by cp.async, one
    // commit group per chunk (empty past the slice, so that group c is the
    // (c+1)-th of every thread); the buffer's earlier reads ended at a block barrier
    auto stage_async = [&](int c) {
        if (c < nch) {
            const int bf = c % NST, j0 = lo + c * kGrpKeys, nj = min(kGrpKeys, hi - j0);
            const int jc = max(0, min(nj, p0 - j0));
            uint16_t *kb = kvb + bf * M::buf_elems(), *vb = kb + kGrpKeys * QP;
            for (int i = tid; i < jc * (HD / 8); i += NTH) {
                const int jj = i / (HD / 8), d = 8 * (i % (HD / 8));
                const int64_t o = ((int64_t)(j0 + jj) * a.nkv + g) * HD + d;
                cp_async16(kb + jj * QP + d, kc + o);
                cp_async16(vb + jj * QP + d, vc + o);
            }
        }
        cp_async_commit();
    };
    // the rest of chunk c: the new rows (j >= p0) rounded from kn / vn, zero
    // rows past the slice (all threads, plain stores)
    auto stage_plain = [&](int c) {
        if (c >= nch) return;
        const int bf = c % NST, j0 = lo + c * kGrpKeys, nj = min(kGrpKeys, hi - j0);
        const int jc = max(0, min(nj, p0 - j0));  // rows [0, jc) come by bulk copy
        uint16_t *kb = kvb + bf * M::buf_elems(), *vb = kb + kGrpKeys * QP;
        for (int i = tid; i < (kGrpKeys - jc) * (HD / 8); i += NTH) {
            const int jj = jc + i / (HD / 8), d = 8 * (i % (HD / 8)), j = j0 + jj;
            uint4 kw = make_uint4(0u, 0u, 0u, 0u), vw = kw;
            if (jj < nj) {
                const float *kr = kn + (j - p0) * HD + d, *vr = vn + (j - p0) * HD + d;
                kw = make_uint4(pack_bf16x2(kr[0], kr[1]), pack_bf16x2(kr[2], kr[3]), pack_bf16x2(kr[4], kr[5]),
                                pack_bf16x2(kr[6], kr[7]));
                vw = make_uint4(pack_bf16x2(vr[0], vr[1]), pack_bf16x2(vr[2], vr[3]), pack_bf16x2(vr[4], vr[5]),
                                pack_bf16x2(vr[6], vr[7]));
            }
            *reinterpret_cast<uint4 *>(kb + jj * QP + d) = kw;
            *reinterpret_cast<uint4 *>(vb + jj * QP + d) = vw;
        }
    };
    stage_async(0);  // the cached rows stream in during the prologue
    stage_async(1);

    // 1. softmax state, zero P pieces (rows >= R stay zero), the new k / v rows
    //    and the q rows with RMSNorm + RoPE
    if (tid < NR) {
        ms[tid] = -CUDART_INF_F;
        ls[tid] = 0.f;
    }
    for (int i = tid; i < 3 * NR * PP / 2; i += NTH) reinterpret_cast<uint32_t *>(pp)[i] = 0u;
    attn_rows_in<HD, 0, NTH>(a, q, kn, vn, rope_s, R, h0, g, p0, tid);
    __syncthreads();
    stage_plain(0);
    stage_plain(1);
    stage_async(2);  // buffer 2 held the RoPE tables
    stage_plain(2);
    // one CTA per (KV head, request) writes the new rows; no CTA reads them from the cache
    if (sl == 0 && hb == 0) {
        for (int i = tid; i < N * HD; i += NTH) {
            const int t = i / HD, d = i % HD;
            const int64_t o = ((int64_t)(p0 + t) * a.nkv + g) * HD + d;
            kc[o] = bf16_bits(kn[i]);
            vc[o] = bf16_bits(vn[i]);
        }
    }
    for (int i = tid; i < NR * HD; i += NTH) {
        const int r = i / HD, d = i % HD;
        uint16_t h_, m_, l_;
        split_bf16x3(r < R ? q[r * HD + d] : 0.f, h_, m_, l_);
        qp[r * QP + d] = h_;
        qp[NR * QP + r * QP + d] = m_;
        qp[2 * NR * QP + r * QP + d] = l_;
    }
    __syncthreads();  // q pieces (buffer 3 is free for chunk 3)

    const float scale = a.scale > 0.f ? a.scale : 1.0f / sqrtf((float)HD);
    // ldmatrix row addresses of this lane: A tiles (16 x 16) and K tiles (8 keys x 16)
    const int arow = (lane & 7) + 8 * ((lane >> 3) & 1), acol = 8 * (lane >> 4);
    float oacc[MT][NTW][4];
#pragma unroll
    for (int m = 0; m < MT; m++)
#pragma unroll
        for (int u = 0; u < NTW; u++)
#pragma unroll
            for (int i = 0; i < 4; i++) oacc[m][u][i] = 0.f;
    for (int c = 0; c < nch; c++) {
        const int bf = c % NST, j0 = lo + c * kGrpKeys, nj = min(kGrpKeys, hi - j0);
        cp_async_wait<NST - 2>();  // this thread's copies of chunk c (c + 1, c + 2 may be in flight)
        __syncthreads();           // chunk c complete; every warp is past chunk c - 1
        // chunk c + 3 into the buffer of chunk c - 1
        stage_async(c + NST - 1);
        stage_plain(c + NST - 1);
        const uint16_t *kb = kvb + bf * M::buf_elems(), *vb = kb + kGrpKeys * QP;
        {   // scores: warp (k half kh = warp / 8, m-tile m = warp / 4 % 2, key n-tile nb = warp % 4)
            const int kh = warp >> 3, m = (warp >> 2) & 1, nb = warp & 3;
            if (16 * m < R) {
                float ac[3][4];
#pragma unroll
                for (int p3 = 0; p3 < 3; p3++)
#pragma unroll
                    for (int i = 0; i < 4; i++) ac[p3][i] = 0.f;
                // K rows 8 nb + (lane & 7); matrices j = lane / 8 at dims k0 + 8 j
                const uint16_t *kr = kb + (8 * nb + (lane & 7)) * QP + 8 * (lane >> 3);
                const uint16_t *qa = qp + (16 * m + arow) * QP + acol;
#pragma unroll 2
                for (int k2 = kh * (HD / 64); k2 < (kh + 1) * (HD / 64); k2++) {  // two k16 steps
                    uint32_t bk[4];
                    ldsm_x4(bk, kr + 32 * k2);
#pragma unroll
                    for (int s2 = 0; s2 < 2; s2++) {
                        const int k0 = 32 * k2 + 16 * s2;
#pragma unroll
                        for (int p3 = 0; p3 < 3; p3++) {
                            uint32_t af[4];
                            ldsm_x4(af, qa + p3 * NR * QP + k0);
                            mma_bf16(ac[p3], af, bk[2 * s2], bk[2 * s2 + 1]);
                        }
                    }
                }
                float *dst = kh ? sc2 : sc;
                const int r0 = 16 * m + g8;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int r = r0 + 8 * (i >> 1), jj = 8 * nb + 2 * t4 + (i & 1);
                    if (r < R) dst[r * SS + jj] = ac[0][i] + (ac[1][i] + ac[2][i]);
                }
            }
        }
        __syncthreads();
        {   // online softmax, one half-warp per row (keys l16 and l16 + 16): all rows in one round
            const int r = 2 * warp + (lane >> 4), l16 = lane & 15;
            const bool rv = r < R;
            float sv[2] = {-CUDART_INF_F, -CUDART_INF_F};
            if (rv) {
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int jj = l16 + 16 * h;
                    if (jj < nj && key_visible(a, j0 + jj, p0 + r % N))
                        sv[h] = score_cap(a, (sc[r * SS + jj] + sc2[r * SS + jj]) * scale);
                }
            }
            float mx = fmaxf(sv[0], sv[1]);
#pragma unroll
            for (int o = 8; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float mo = rv ? ms[r] : -CUDART_INF_F, mn = fmaxf(mo, mx);
            float f = 1.f, e[2] = {0.f, 0.f};
            if (mn != -CUDART_INF_F) {
                f = expf(mo - mn);
                e[0] = expf(sv[0] - mn);
                e[1] = expf(sv[1] - mn);
            }
            float ps = e[0] + e[1];
#pragma unroll
            for (int o = 8; o; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            if (rv) {
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const int jj = l16 + 16 * h;
                    uint16_t h_, m_, l_;
                    split_bf16x3(e[h], h_, m_, l_);
                    pp[r * PP + jj] = h_;
                    pp[NR * PP + r * PP + jj] = m_;
                    pp[2 * NR * PP + r * PP + jj] = l_;
                }
                if (l16 == 0) {
                    ls[r] = ls[r] * f + ps;
                    ms[r] = mn;
                    fs[r] = f;
                }
            }
        }
        __syncthreads();
        // P.V: the warp's m-tiles and n-tiles (see MT, NTW)
#pragma unroll
        for (int mi = 0; mi < MT; mi++) {
            const int m = MT == 2 ? mi : warp >> 3;
            if (16 * m >= R) continue;
            const int r0 = 16 * m + g8;
            const float f0 = r0 < R ? fs[r0] : 1.f, f1 = r0 + 8 < R ? fs[r0 + 8] : 1.f;
#pragma unroll
            for (int u = 0; u < NTW; u++) {
                oacc[mi][u][0] *= f0;
                oacc[mi][u][1] *= f0;
                oacc[mi][u][2] *= f1;
                oacc[mi][u][3] *= f1;
            }
#pragma unroll
            for (int kk = 0; kk < kGrpKeys / 16; kk++) {
                uint32_t af[3][4];
#pragma unroll
                for (int p3 = 0; p3 < 3; p3++) ldsm_x4(af[p3], pp + p3 * NR * PP + (16 * m + arow) * PP + 16 * kk + acol);
                // V rows (keys) 16 kk + arow; matrices (lane / 16) at dims n0 + 8 (lane / 16)
                const uint16_t *vr = vb + (16 * kk + arow) * QP;
                if constexpr (NTW == 2) {
                    const int n0 = 8 * (NTW * warp);
                    uint32_t bv[4];
                    ldsm_x4_t(bv, vr + n0 + acol);
#pragma unroll
                    for (int u = 0; u < 2; u++)
#pragma unroll
                        for (int p3 = 0; p3 < 3; p3++) mma_bf16(oacc[mi][u], af[p3], bv[2 * u], bv[2 * u + 1]);
                } else {
                    const int nt = MT == 2 ? NTW * warp : (warp & 7);
                    uint32_t b0, b1;
                    ldsm_x2_t(b0, b1, vr + 8 * nt);
#pragma unroll
                    for (int p3 = 0; p3 < 3; p3++) mma_bf16(oacc[mi][0], af[p3], b0, b1);
                }
            }
        }
        // no barrier here: the next chunk's first barrier comes before anything
        // this chunk read (its buffer, the scores, P, fs) is rewritten
    }

    // 3. the slice's partial state
    float *pm = a.part + (int64_t)sl * rows_all * (HD + 2), *pl = pm + rows_all, *po = pl + rows_all;
#pragma unroll
    for (int mi = 0; mi < MT; mi++)
#pragma unroll
        for (int u = 0; u < NTW; u++)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int m = MT == 2 ? mi : warp >> 3, nt = MT == 2 ? NTW * warp + u : (warp & 7);
                const int r = 16 * m + g8 + 8 * (i >> 1), d = 8 * nt + 2 * t4 + (i & 1);
                if (r < R) po[(rid0 + r) * HD + d] = oacc[mi][u][i];
            }
    if (tid < R) {
        pm[rid0 + tid] = ms[tid];
        pl[rid0 + tid] = ls[tid];
    }
}

// Merges the key slices of one row (b, h, t) per CTA: M = max_s m_s,
// L = sum_s l_s e^(m_s - M), O = sum_s o_s e^(m_s - M) (slice order), and
// writes O / L x sigmoid(gate).  The slices' (m, l) and weights are formed in
// parallel in shared memory; thread group q (256 / HD groups) sums P.V over
// slices q, q + 256 / HD, ... with independent loads in flight, and the groups'
// sums are added in group order.
// shared memory of one virtual block of the combine
template <int HD>
struct CombineSmem {
    float w[kMaxSplits], red[8], og[256 / HD][HD];
};
template <int HD, int BAR>
__device__ __forceinline__ void attn_combine_body(AttnArgs a, int batch, int S, int64_t rid, int tid,
                                                  CombineSmem<HD> &cs) {
    constexpr int NG = 256 / HD;
    float *w = cs.w, *red = cs.red;
    auto &og = cs.og;
    const int N = a.N, d = tid % HD, q = tid / HD;
    const int64_t rows = (int64_t)batch * a.nh * N;
    const int t = (int)(rid % N), h = (int)((rid / N) % a.nh), b = (int)(rid / ((int64_t)N * a.nh));
    const int nkeys = a.pos[(int64_t)b * a.b_pos] + N, kps = attn_kps(nkeys, S);
    const int ns = (nkeys + kps - 1) / kps;
    const int64_t stride = rows * (HD + 2);
    float mv = -CUDART_INF_F, lv = 0.f;
    if (tid < ns) {
        mv = a.part[tid * stride + rid];
        lv = a.part[tid * stride + rows + rid];
    }
    // block max of m (ns <= kMaxSplits <= 256)
    float M = warp_max(mv);
    if ((tid & 31) == 0) red[tid >> 5] = M;
    bar256<BAR>();
    M = red[0];
#pragma unroll
    for (int i = 1; i < 8; i++) M = fmaxf(M, red[i]);
    const float wv = mv == -CUDART_INF_F ? 0.f : expf(mv - M);
    if (tid < ns) w[tid] = wv;
    const float L = block_sum256_b<BAR>(lv * wv, red, tid);  // synchronises: w visible
    const float *po = a.part + 2 * rows + rid * HD + d;
    float O = 0.f;
    int sl = q;
    for (; sl + 3 * NG < ns; sl += 4 * NG) {
        const float o0 = po[sl * stride], o1 = po[(sl + NG) * stride];
        const float o2 = po[(sl + 2 * NG) * stride], o3 = po[(sl + 3 * NG) * stride];
        O += w[sl] * o0;
        O += w[sl + NG] * o1;
        O += w[sl + 2 * NG] * o2;
        O += w[sl + 3 * NG] * o3;
    }
    for (; sl < ns; sl += NG) O += w[sl] * po[sl * stride];
    if (NG > 1) {
        og[q][d] = O;
        bar256<BAR>();
        if (q) return;
        O = og[0][d];
#pragma unroll
        for (int g2 = 1; g2 < NG; g2++) O += og[g2][d];
    }
    const int64_t tok = (int64_t)b * N + t;
    float y = O / L;
    if (a.gated) {
        const float gv = a.qkv[tok * a.ldq + (int64_t)h * 2 * HD + HD + d];
        y *= 1.0f / (1.0f + expf(-gv));
    }
    a.out[tok * a.ldo + (int64_t)h * HD + d] = y;
}

template <int HD>
__global__ void __launch_bounds__(256) attn_combine_kernel(AttnArgs a, int batch, int S) {
    __shared__ CombineSmem<HD> cs;
    pdl_trigger();
    pdl_wait();
    attn_combine_body<HD, 0>(a, batch, S, blockIdx.x, threadIdx.x, cs);
}

static int split_heads(int ratio, int N) { return std::max(1, std::min(ratio, kGrpRows / N)); }

static bool attn_mma_enabled() {
    static const bool on = [] {
        const char *v = getenv("IFR_ATTN_MMA");
        return !(v && v[0] == '0');
    }();
    return on;
}

int attn_splits(int nh, int nkv, int N, int batch, int max_ctx) {
    const int ratio = nh / nkv, hg = split_heads(ratio, N), nrg = (ratio + hg - 1) / hg;
    const int64_t ctas = (int64_t)nkv * nrg * batch;
    int64_t S = (kSplitCtas + ctas - 1) / ctas;
    S = std::min<int64_t>(S, (max_ctx + kGrpKeys - 1) / kGrpKeys);
    S = std::min<int64_t>(S, kMaxSplits);
    return (int)std::max<int64_t>(S, 1);
}

int64_t attn_part_floats(int nh, int nkv, int hd, int batch, int max_ctx) {
    int S = 1;
    for (int N = 1; N <= kMaxN; N++) S = std::max(S, attn_splits(nh, nkv, N, batch, max_ctx));
    return (int64_t)S * batch * nh * kMaxN * (hd + 2);
}

template <int HD>
static cudaError_t launch_split(const AttnArgs &a, int batch, cudaStream_t s) {
    static DeviceFlags attr;
    if (!attr.test()) {
        cudaError_t e = cudaFuncSetAttribute(attn_part_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             GrpSmem<HD>::bytes(kGrpRows, kMaxN));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(attn_part_mma_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     MmaSmem<HD>::bytes(kGrpRows, kMaxN));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(attn_part_bf16_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Bf16Smem<HD>::bytes(kMaxN));
        if (e != cudaSuccess) return e;
        attr.set();
    }
    const int ratio = a.nh / a.nkv, hg = split_heads(ratio, a.N), nrg = (ratio + hg - 1) / hg;
    const int R = std::min(hg, ratio) * a.N;
    // a bf16 cache: its own kernel; else the tensor-core kernel (IFR_ATTN_MMA=0
    // in the environment selects the CUDA-core one)
    cudaError_t e = a.kv16 ? launch_k(attn_part_bf16_kernel<HD>, dim3(a.splits, a.nkv * nrg, batch),
                                      dim3(kMmaThreads), (size_t)Bf16Smem<HD>::bytes(a.N), s, a, hg, a.splits)
                  : attn_mma_enabled()
                        ? launch_k(attn_part_mma_kernel<HD>, dim3(a.splits, a.nkv * nrg, batch), dim3(kMmaThreads),
                                   (size_t)MmaSmem<HD>::bytes(R, a.N), s, a, hg, a.splits)
                        : launch_k(attn_part_kernel<HD>, dim3(a.splits, a.nkv * nrg, batch), dim3(256),
                                   (size_t)GrpSmem<HD>::bytes(R, a.N), s, a, hg, a.splits);
    if (e != cudaSuccess) return e;
    return launch_k(attn_combine_kernel<HD>, dim3((unsigned)(batch * a.nh * a.N)), dim3(256), 0, s, a, batch,
                    a.splits);
}

cudaError_t attn_step(const AttnArgs &a, int batch, cudaStream_t s) {
    if (a.N < 1 || a.N > kMaxN || a.nh % a.nkv || batch < 1) return cudaErrorInvalidValue;
    if (a.splits > 0) {
        if (!a.part || a.splits > kMaxSplits) return cudaErrorInvalidValue;
        if (a.hd == 256) return launch_split<256>(a, batch, s);
        if (a.hd == 128) return launch_split<128>(a, batch, s);
        if (a.hd == 64) return launch_split<64>(a, batch, s);
        return cudaErrorInvalidValue;
    }
    if (a.kv16) return cudaErrorNotSupported;  // bf16 caches take the split path
    const dim3 grid(kAttnSplit, a.nh, batch);
    if (a.hd == 256) return launch_k(attn_step_kernel<256>, grid, dim3(256), 0, s, a);
    if (a.hd == 128) return launch_k(attn_step_kernel<128>, grid, dim3(256), 0, s, a);
    if (a.hd == 64) return launch_k(attn_step_kernel<64>, grid, dim3(256), 0, s, a);
    return cudaErrorInvalidValue;
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
    pdl_trigger();
    pdl_wait();
    {  // request blockIdx.x
        const int b = blockIdx.x;
        sc += b;
        acc_dev += b;
        out_tok += (int64_t)b * n;
        if (hid) hid += (int64_t)b * n * d;
        if (mtp_h) mtp_h += (int64_t)b * d;
        log += (int64_t)b * log_cap;
    }
    if (threadIdx.x == 0) {
        const int acc = all ? n - 1 : *acc_dev;
        acc_s = acc;
        sc->a_prev = all == 2 ? -1 : acc;  // 2: committed by the layers themselves (prefill chunks)
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

void commit(EngineScalars *sc, const int32_t *acc, const int32_t *out_tok, int n, int all, const float *hid,
            float *mtp_h, int d, int32_t *log, int log_cap, int batch, cudaStream_t s) {
    launch_k(commit_kernel, dim3(batch), dim3(256), 0, s, sc, acc, out_tok, n, all, hid, mtp_h, d, log, log_cap);
}

// positions of the sub-chunks of a prefill chunk: dst[i] = pos + step * i
__global__ void chunk_pos_kernel(int32_t *dst, const EngineScalars *sc, int count, int step) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x < count) dst[threadIdx.x] = sc->pos + step * (int)threadIdx.x;
}
void chunk_positions(int32_t *dst, const EngineScalars *sc, int count, int step, cudaStream_t s) {
    launch_k(chunk_pos_kernel, dim3(1), dim3(32), 0, s, dst, sc, count, step);
}

// copy a device scalar token into a slot of the verify token vector
__global__ void set_token_kernel(int32_t *dst, const int32_t *src) {
    pdl_trigger();
    pdl_wait();
    *dst = *src;
}
void set_token(int32_t *dst, const int32_t *src, cudaStream_t s) {
    launch_k(set_token_kernel, dim3(1), dim3(1), 0, s, dst, src);
}

}  // namespace ifr

#include "fused_step.cuh"
