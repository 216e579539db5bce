// Speculative-decoding acceptance on the device.
//
// Fixed semantics of the reference's src/SpeculativeDecoding.jl:37-104
// (temperature on both distributions, vector residual max(p_t - p_d, 0),
// all target rows), sampled by inverse CDF "first i with r <= cumsum"
// (:20-30).  The floating-point evaluation order is fully specified so that
// the CPU oracle reproduces accept counts and tokens bit for bit:
//   chunks of 2048 elements; per chunk m_c = max, e_i = exp((l_i - m_c)/T),
//   256 lanes x 8 consecutive elements summed in order, a 32-lane xor
//   butterfly (16,8,4,2,1) per warp, warp sums left to right -> s_c;
//   per row M = max m_c, f_c = exp((m_c - M)/T), S = sum_c s_c f_c left to right.
// Every float operation uses the _rn intrinsics so nothing is contracted into
// an FMA behind our back; exp is ifr_exp below (the oracle's or_exp).
//
// Launches: chunk_stats (one CTA per row chunk, the only full pass over the
// logits), row_decide (per sequence and row: row stats, draft draw, ratio
// test), finish (per sequence: residual or bonus sample).
#include "common.cuh"
#include <math_constants.h>
#include <climits>

namespace ifr {

constexpr int kCH = 2048, kNL = 256, kPER = 8;

// Cody-Waite exp, identical operation sequence to the oracle's or_exp.
__device__ __forceinline__ float ifr_exp(float x) {
    if (x != x) return x;
    if (x > 88.5f) return CUDART_INF_F;
    if (x < -87.0f) return 0.0f;
    const float log2e = 1.44269502162933349609375f;
    const float ln2_hi = 0.693145751953125f;
    const float ln2_lo = 1.42860677e-06f;
    float n = rintf(__fmul_rn(x, log2e));
    float r = __fmaf_rn(-n, ln2_hi, x);
    r = __fmaf_rn(-n, ln2_lo, r);
    float p = 1.98412698e-04f;
    p = __fmaf_rn(p, r, 1.38888889e-03f);
    p = __fmaf_rn(p, r, 8.33333377e-03f);
    p = __fmaf_rn(p, r, 4.16666679e-02f);
    p = __fmaf_rn(p, r, 1.66666672e-01f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    int ni = (int)n;
    if (ni > 127) { p = __fmul_rn(p, 2.0f); ni -= 1; }
    return __fmul_rn(p, __int_as_float((ni + 127) << 23));
}

__device__ __forceinline__ float elem_e(float l, float m, float T) {
    return ifr_exp(__fdiv_rn(__fsub_rn(l, m), T));
}

// 256-lane canonical sum; all threads get the result.
__device__ float canon_sum(float t, float *wsum /* smem [8] */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, off));
    __syncthreads();
    if (lane == 0) wsum[warp] = t;
    __syncthreads();
    float s = wsum[0];
    for (int w = 1; w < kNL / 32; w++) s = __fadd_rn(s, wsum[w]);
    return s;
}

__device__ float block_max(float m, float *wbuf) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    __syncthreads();
    if (lane == 0) wbuf[warp] = m;
    __syncthreads();
    float r = wbuf[0];
    for (int w = 1; w < kNL / 32; w++) r = fmaxf(r, wbuf[w]);
    return r;
}

__device__ __forceinline__ const float *row_ptr(const float *target, const float *draft, int r,
                                                int B, int G, int V) {
    const int nt = B * (G + 1);
    return r < nt ? target + (int64_t)r * V : draft + (int64_t)(r - nt) * V;
}

// load the 8 elements of lane tid in chunk c (missing ones = -inf, flagged)
__device__ __forceinline__ int load8(const float *row, int V, int c, float (&x)[8]) {
    const int64_t b = (int64_t)c * kCH + kPER * threadIdx.x;
    int n = 0;
    if (b + kPER <= V && (V & 3) == 0) {
        const float4 *p = reinterpret_cast<const float4 *>(row + b);
        float4 a = __ldg(p), d = __ldg(p + 1);
        x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
        x[4] = d.x; x[5] = d.y; x[6] = d.z; x[7] = d.w;
        n = kPER;
    } else {
#pragma unroll
        for (int q = 0; q < kPER; q++) {
            if (b + q < V) { x[q] = __ldg(row + b + q); n = q + 1; }
            else x[q] = -CUDART_INF_F;
        }
    }
    return n;
}

__global__ void __launch_bounds__(kNL) chunk_stats_kernel(const float *__restrict__ target,
                                                          const float *__restrict__ draft, int B,
                                                          int G, int V, float T, int nch,
                                                          float *__restrict__ cmax,
                                                          float *__restrict__ csum) {
    __shared__ float wbuf[8];
    const int c = blockIdx.x, r = blockIdx.y;
    const float *row = row_ptr(target, draft, r, B, G, V);
    float x[8];
    const int n = load8(row, V, c, x);
    float m = -CUDART_INF_F;
#pragma unroll
    for (int q = 0; q < kPER; q++) if (q < n) m = fmaxf(m, x[q]);
    m = block_max(m, wbuf);
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < kPER; q++) if (q < n) t = __fadd_rn(t, elem_e(x[q], m, T));
    const float s = canon_sum(t, wbuf);
    if (threadIdx.x == 0) {
        cmax[(int64_t)r * nch + c] = m;
        csum[(int64_t)r * nch + c] = s;
    }
}

struct RowStat { float M, S; };

__device__ RowStat row_stat(const float *cm, const float *cs, int nch, float T) {
    float M = -CUDART_INF_F;
    for (int c = 0; c < nch; c++) M = fmaxf(M, cm[c]);
    float S = 0.f;
    for (int c = 0; c < nch; c++) S = __fadd_rn(S, __fmul_rn(cs[c], ifr_exp(__fdiv_rn(__fsub_rn(cm[c], M), T))));
    return {M, S};
}

// Blocked in-chunk search (all threads): first element with tau <= cumsum of
// vals; else the last element with val > 0; else the last element.
__device__ int chunk_search(const float (&v)[8], int n, int64_t base, float tau, float *lsum,
                            int *res) {
    const int tid = threadIdx.x;
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < kPER; q++) if (q < n) t = __fadd_rn(t, v[q]);
    __syncthreads();
    lsum[tid] = t;
    if (tid == 0) { res[0] = INT_MAX; res[1] = -1; res[2] = -1; }
    __syncthreads();
    if (tid == 0) {  // exclusive prefix, sequential
        float pre = 0.f;
        for (int j = 0; j < kNL; j++) { float tj = lsum[j]; lsum[j] = pre; pre = __fadd_rn(pre, tj); }
    }
    __syncthreads();
    float cum = lsum[tid];
    int hit = -1, lastpos = -1, lastany = -1;
#pragma unroll
    for (int q = 0; q < kPER; q++) {
        if (q < n) {
            cum = __fadd_rn(cum, v[q]);
            if (hit < 0 && tau <= cum) hit = kPER * tid + q;
            if (v[q] > 0.f) lastpos = kPER * tid + q;
            lastany = kPER * tid + q;
        }
    }
    if (hit >= 0) atomicMin(&res[0], hit);
    if (lastpos >= 0) atomicMax(&res[1], lastpos);
    if (lastany >= 0) atomicMax(&res[2], lastany);
    __syncthreads();
    int out = res[0] != INT_MAX ? res[0] : (res[1] >= 0 ? res[1] : res[2]);
    __syncthreads();
    return (int)(base + out);
}

struct SampleSmem {
    float lsum[kNL];
    int res[3];
    float bc[4];
    int ibc[2];
    float wsum[8];
};

// sample from softmax(row/T) with uniform u; row stats (M,S) and chunk stats given
__device__ int sample_row(const float *row, int V, const float *cm, const float *cs, int nch,
                          float T, RowStat st, float u, SampleSmem &sm) {
    if (threadIdx.x == 0) {
        float tau = __fmul_rn(u, st.S), P = 0.f;
        int csel = -1;
        for (int c = 0; c < nch; c++) {
            float nP = __fadd_rn(P, __fmul_rn(cs[c], ifr_exp(__fdiv_rn(__fsub_rn(cm[c], st.M), T))));
            if (tau <= nP) { csel = c; break; }
            P = nP;
        }
        if (csel < 0) {
            for (int c = nch - 1; c >= 0; c--) if (cs[c] > 0.f) { csel = c; break; }
            if (csel < 0) csel = nch - 1;
            P = 0.f;
            for (int c = 0; c < csel; c++)
                P = __fadd_rn(P, __fmul_rn(cs[c], ifr_exp(__fdiv_rn(__fsub_rn(cm[c], st.M), T))));
            tau = __fadd_rn(P, __fmul_rn(cs[csel], ifr_exp(__fdiv_rn(__fsub_rn(cm[csel], st.M), T))));
        }
        float fc = ifr_exp(__fdiv_rn(__fsub_rn(cm[csel], st.M), T));
        sm.bc[0] = __fdiv_rn(__fsub_rn(tau, P), fc);
        sm.ibc[0] = csel;
    }
    __syncthreads();
    const float taup = sm.bc[0];
    const int csel = sm.ibc[0];
    float x[8], v[8];
    const int n = load8(row, V, csel, x);
    const float mc = cm[csel];
#pragma unroll
    for (int q = 0; q < kPER; q++) v[q] = q < n ? elem_e(x[q], mc, T) : 0.f;
    return chunk_search(v, n, (int64_t)csel * kCH, taup, sm.lsum, sm.res);
}

__device__ __forceinline__ float weight_of(const float *row, int i, const float *cm, RowStat st, float T) {
    const int c = i / kCH;
    return __fmul_rn(elem_e(__ldg(row + i), cm[c], T), ifr_exp(__fdiv_rn(__fsub_rn(cm[c], st.M), T)));
}

// grid (B, G+1): row stats of target row i (and draft row i < G), draft token, ratio test
__global__ void __launch_bounds__(kNL) row_decide_kernel(
    const float *__restrict__ target, const float *__restrict__ draft,
    const int32_t *__restrict__ draft_tokens, const float *__restrict__ uniforms, int B, int G, int V,
    float T, int nch, const float *__restrict__ cmax, const float *__restrict__ csum,
    float *__restrict__ rstat, int32_t *__restrict__ xdraft, int32_t *__restrict__ okflag) {
    __shared__ SampleSmem sm;
    __shared__ RowStat st_s[2];
    const int b = blockIdx.x, i = blockIdx.y;
    const int tr = b * (G + 1) + i;
    const float *trow = target + (int64_t)tr * V;
    if (threadIdx.x == 0) {
        st_s[0] = row_stat(cmax + (int64_t)tr * nch, csum + (int64_t)tr * nch, nch, T);
        rstat[2 * tr] = st_s[0].M;
        rstat[2 * tr + 1] = st_s[0].S;
    }
    if (i == G) return;
    const int dr = B * (G + 1) + b * G + i;
    const float *drow = draft + (int64_t)(b * G + i) * V;
    if (threadIdx.x == 0) {
        st_s[1] = row_stat(cmax + (int64_t)dr * nch, csum + (int64_t)dr * nch, nch, T);
        rstat[2 * dr] = st_s[1].M;
        rstat[2 * dr + 1] = st_s[1].S;
    }
    __syncthreads();
    const float *u = uniforms + (int64_t)b * (2 * G + 1);
    int x;
    if (draft_tokens) {
        x = draft_tokens[b * G + i];
    } else {
        x = sample_row(drow, V, cmax + (int64_t)dr * nch, csum + (int64_t)dr * nch, nch, T, st_s[1],
                       u[i], sm);
    }
    if (threadIdx.x == 0) {
        int ok;
        if (x < 0 || x >= V) {
            ok = 0;  // invalid supplied draft token: reject
        } else {
            float pt = __fdiv_rn(weight_of(trow, x, cmax + (int64_t)tr * nch, st_s[0], T), st_s[0].S);
            float pd = __fdiv_rn(weight_of(drow, x, cmax + (int64_t)dr * nch, st_s[1], T), st_s[1].S);
            ok = pd > 0.f ? (u[G + i] < __fdiv_rn(pt, pd)) : (pt > 0.f);
        }
        xdraft[b * G + i] = x;
        okflag[b * G + i] = ok;
    }
}

// grid (B): accept count, emitted tokens, residual or bonus sample
__global__ void __launch_bounds__(kNL) finish_kernel(
    const float *__restrict__ target, const float *__restrict__ draft,
    const float *__restrict__ uniforms, int B, int G, int V, float T, int nch,
    const float *__restrict__ cmax, const float *__restrict__ csum, const float *__restrict__ rstat,
    const int32_t *__restrict__ xdraft, const int32_t *__restrict__ okflag,
    int32_t *__restrict__ accept_count, int32_t *__restrict__ out_tokens,
    int32_t *__restrict__ draft_out, float *__restrict__ rchunk /* [B][nch] */) {
    __shared__ SampleSmem sm;
    const int b = blockIdx.x, tid = threadIdx.x;
    int acc = 0;
    while (acc < G && okflag[b * G + acc]) acc++;
    int32_t *ot = out_tokens + (int64_t)b * (G + 1);
    if (tid == 0) {
        accept_count[b] = acc;
        for (int i = 0; i <= G; i++) ot[i] = i < acc ? xdraft[b * G + i] : -1;
    }
    if (draft_out && tid < G) draft_out[b * G + tid] = xdraft[b * G + tid];
    const float ub = uniforms[(int64_t)b * (2 * G + 1) + 2 * G];
    int y;
    if (acc == G) {
        const int tr = b * (G + 1) + G;
        RowStat st{rstat[2 * tr], rstat[2 * tr + 1]};
        y = sample_row(target + (int64_t)tr * V, V, cmax + (int64_t)tr * nch, csum + (int64_t)tr * nch,
                       nch, T, st, ub, sm);
    } else {
        const int tr = b * (G + 1) + acc, dr = B * (G + 1) + b * G + acc;
        const float *trow = target + (int64_t)tr * V, *drow = draft + (int64_t)(b * G + acc) * V;
        const float *tcm = cmax + (int64_t)tr * nch, *dcm = cmax + (int64_t)dr * nch;
        const RowStat ts{rstat[2 * tr], rstat[2 * tr + 1]}, ds{rstat[2 * dr], rstat[2 * dr + 1]};
        float *rc = rchunk + (int64_t)b * nch;
        // residual chunk sums
        for (int c = 0; c < nch; c++) {
            float xt[8], xd[8];
            const int n = load8(trow, V, c, xt);
            load8(drow, V, c, xd);
            const float ft = ifr_exp(__fdiv_rn(__fsub_rn(tcm[c], ts.M), T));
            const float fd = ifr_exp(__fdiv_rn(__fsub_rn(dcm[c], ds.M), T));
            float t = 0.f;
#pragma unroll
            for (int q = 0; q < kPER; q++) {
                if (q < n) {
                    float pt = __fdiv_rn(__fmul_rn(elem_e(xt[q], tcm[c], T), ft), ts.S);
                    float pd = __fdiv_rn(__fmul_rn(elem_e(xd[q], dcm[c], T), fd), ds.S);
                    float r = __fsub_rn(pt, pd);
                    t = __fadd_rn(t, r > 0.f ? r : 0.f);
                }
            }
            float s = canon_sum(t, sm.wsum);
            if (tid == 0) rc[c] = s;
        }
        __syncthreads();
        if (tid == 0) {
            float R = 0.f;
            for (int c = 0; c < nch; c++) R = __fadd_rn(R, rc[c]);
            int csel = -2;
            float P = 0.f, tau = 0.f;
            if (R > 0.f) {
                tau = __fmul_rn(ub, R);
                csel = -1;
                for (int c = 0; c < nch; c++) {
                    float nP = __fadd_rn(P, rc[c]);
                    if (tau <= nP) { csel = c; break; }
                    P = nP;
                }
                if (csel < 0) {
                    for (int c = nch - 1; c >= 0; c--) if (rc[c] > 0.f) { csel = c; break; }
                    P = 0.f;
                    for (int c = 0; c < csel; c++) P = __fadd_rn(P, rc[c]);
                    tau = __fadd_rn(P, rc[csel]);
                }
            }
            sm.ibc[1] = csel;
            sm.bc[1] = __fsub_rn(tau, P);
        }
        __syncthreads();
        const int csel = sm.ibc[1];
        if (csel == -2) {
            y = sample_row(trow, V, tcm, csum + (int64_t)tr * nch, nch, T, ts, ub, sm);
        } else {
            float xt[8], xd[8], v[8];
            const int n = load8(trow, V, csel, xt);
            load8(drow, V, csel, xd);
            const float ft = ifr_exp(__fdiv_rn(__fsub_rn(tcm[csel], ts.M), T));
            const float fd = ifr_exp(__fdiv_rn(__fsub_rn(dcm[csel], ds.M), T));
#pragma unroll
            for (int q = 0; q < kPER; q++) {
                if (q < n) {
                    float pt = __fdiv_rn(__fmul_rn(elem_e(xt[q], tcm[csel], T), ft), ts.S);
                    float pd = __fdiv_rn(__fmul_rn(elem_e(xd[q], dcm[csel], T), fd), ds.S);
                    float r = __fsub_rn(pt, pd);
                    v[q] = r > 0.f ? r : 0.f;
                } else {
                    v[q] = 0.f;
                }
            }
            y = chunk_search(v, n, (int64_t)csel * kCH, sm.bc[1], sm.lsum, sm.res);
        }
    }
    if (tid == 0) ot[acc] = y;
}

int64_t accept_scratch_bytes(int B, int G, int V) {
    const int64_t nch = (V + kCH - 1) / kCH, rows = (int64_t)B * (2 * G + 1);
    return 2 * rows * nch * 4 + 2 * rows * 4 + 2 * (int64_t)B * G * 4 + (int64_t)B * nch * 4 + 1024;
}

cudaError_t accept_sampled(const float *target, const float *draft, const int32_t *draft_tokens,
                           const float *uniforms, int B, int G, int V, float T, int32_t *accept_count,
                           int32_t *out_tokens, int32_t *draft_out, void *scratch, cudaStream_t s) {
    const int nch = (V + kCH - 1) / kCH;
    const int64_t rows = (int64_t)B * (2 * G + 1);
    char *p = (char *)scratch;
    float *cmax = (float *)p; p += rows * nch * 4;
    float *csum = (float *)p; p += rows * nch * 4;
    float *rstat = (float *)p; p += 2 * rows * 4;
    int32_t *xdraft = (int32_t *)p; p += (int64_t)B * G * 4;
    int32_t *okflag = (int32_t *)p; p += (int64_t)B * G * 4;
    float *rchunk = (float *)p;
    chunk_stats_kernel<<<dim3(nch, (unsigned)rows), kNL, 0, s>>>(target, draft, B, G, V, T, nch, cmax, csum);
    row_decide_kernel<<<dim3(B, G + 1), kNL, 0, s>>>(target, draft, draft_tokens, uniforms, B, G, V, T,
                                                     nch, cmax, csum, rstat, xdraft, okflag);
    finish_kernel<<<B, kNL, 0, s>>>(target, draft, uniforms, B, G, V, T, nch, cmax, csum, rstat, xdraft,
                                    okflag, accept_count, out_tokens, draft_out, rchunk);
    return cudaGetLastError();
}

// ------------------------------------------------------------- greedy -------

__global__ void __launch_bounds__(kNL) chunk_argmax_kernel(const float *__restrict__ target, int V,
                                                           int nch, float *__restrict__ vmax,
                                                           int32_t *__restrict__ imax) {
    __shared__ float sv[kNL];
    __shared__ int si[kNL];
    const int c = blockIdx.x, r = blockIdx.y;
    pdl_trigger();
    pdl_wait();
    const float *row = target + (int64_t)r * V;
    float x[8];
    const int n = load8(row, V, c, x);
    float bv = -CUDART_INF_F;
    int bi = INT_MAX;
#pragma unroll
    for (int q = 0; q < kPER; q++)
        if (q < n && (x[q] > bv || bi == INT_MAX)) { bv = x[q]; bi = c * kCH + kPER * threadIdx.x + q; }
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int off = kNL / 2; off; off >>= 1) {
        if (threadIdx.x < off) {
            float ov = sv[threadIdx.x + off];
            int oi = si[threadIdx.x + off];
            if (oi != INT_MAX && (si[threadIdx.x] == INT_MAX || ov > sv[threadIdx.x] ||
                                  (ov == sv[threadIdx.x] && oi < si[threadIdx.x]))) {
                sv[threadIdx.x] = ov;
                si[threadIdx.x] = oi;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        vmax[(int64_t)r * nch + c] = sv[0];
        imax[(int64_t)r * nch + c] = si[0];
    }
}

__global__ void greedy_finish_kernel(const float *__restrict__ vmax, const int32_t *__restrict__ imax,
                                     const int32_t *__restrict__ draft_tokens, int G, int nch,
                                     int32_t *__restrict__ accept_count, int32_t *__restrict__ out_tokens) {
    const int b = blockIdx.x;
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x != 0) return;
    int32_t *ot = out_tokens + (int64_t)b * (G + 1);
    for (int i = 0; i <= G; i++) ot[i] = -1;
    int acc = 0;
    for (int i = 0; i <= G; i++) {
        const int64_t r = (int64_t)b * (G + 1) + i;
        float bv = vmax[r * nch];
        int bi = imax[r * nch];
        for (int c = 1; c < nch; c++) {
            float v = vmax[r * nch + c];
            if (v > bv) { bv = v; bi = imax[r * nch + c]; }
        }
        ot[i] = bi;
        if (i == G || bi != draft_tokens[b * G + i]) break;
        acc++;
    }
    accept_count[b] = acc;
}

// One launch for both steps: every CTA writes its chunk's (max, argmax),
// then counts itself done on its sequence's counter; the CTA that finishes
// last (the classic fenced-counter reduction, nothing waits) reads all
// chunks in chunk order, decides, and returns the counter to zero for the
// next launch.
__global__ void __launch_bounds__(kNL) greedy_fused_kernel(const float *__restrict__ target, int V, int nch, int G,
                                                           const int32_t *__restrict__ draft_tokens, int draft_ld,
                                                           float *vmax, int32_t *imax, unsigned *counter,
                                                           int32_t *__restrict__ accept_count,
                                                           int32_t *__restrict__ out_tokens, int out_ld) {
    __shared__ float sv[kNL];
    __shared__ int si[kNL];
    __shared__ bool last;
    const int c = blockIdx.x, r = blockIdx.y, b = r / (G + 1);
    pdl_trigger();
    pdl_wait();
    const float *row = target + (int64_t)r * V;
    float x[8];
    const int n = load8(row, V, c, x);
    float bv = -CUDART_INF_F;
    int bi = INT_MAX;
#pragma unroll
    for (int q = 0; q < kPER; q++)
        if (q < n && (x[q] > bv || bi == INT_MAX)) { bv = x[q]; bi = c * kCH + kPER * threadIdx.x + q; }
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int off = kNL / 2; off; off >>= 1) {
        if (threadIdx.x < off) {
            float ov = sv[threadIdx.x + off];
            int oi = si[threadIdx.x + off];
            if (oi != INT_MAX && (si[threadIdx.x] == INT_MAX || ov > sv[threadIdx.x] ||
                                  (ov == sv[threadIdx.x] && oi < si[threadIdx.x]))) {
                sv[threadIdx.x] = ov;
                si[threadIdx.x] = oi;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        vmax[(int64_t)r * nch + c] = sv[0];
        imax[(int64_t)r * nch + c] = si[0];
        __threadfence();
        const unsigned done = atomicAdd(counter + b, 1u);
        last = done == (unsigned)(nch * (G + 1) - 1);
    }
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    __threadfence();
    int32_t *ot = out_tokens + (int64_t)b * out_ld;
    for (int i = 0; i <= G; i++) ot[i] = -1;
    int acc = 0;
    for (int i = 0; i <= G; i++) {
        const int64_t rr = (int64_t)b * (G + 1) + i;
        float best = __ldcg(vmax + rr * nch);
        int arg = __ldcg(imax + rr * nch);
        for (int cc = 1; cc < nch; cc++) {
            const float v = __ldcg(vmax + rr * nch + cc);
            if (v > best) { best = v; arg = __ldcg(imax + rr * nch + cc); }
        }
        ot[i] = arg;
        if (i == G || arg != draft_tokens[(int64_t)b * draft_ld + i]) break;
        acc++;
    }
    accept_count[b] = acc;
    counter[b] = 0u;
}

cudaError_t accept_greedy_fused(const float *target, const int32_t *draft_tokens, int B, int G, int V,
                                int32_t *accept_count, int32_t *out_tokens, void *scratch, unsigned *counter,
                                cudaStream_t s, int draft_ld, int out_ld) {
    const int nch = (V + kCH - 1) / kCH;
    float *vmax = (float *)scratch;
    int32_t *imax = (int32_t *)((char *)scratch + (int64_t)B * (G + 1) * nch * 4);
    return launch_k(greedy_fused_kernel, dim3(nch, B * (G + 1)), dim3(kNL), 0, s, target, V, nch, G, draft_tokens,
                    draft_ld > 0 ? draft_ld : G, vmax, imax, counter, accept_count, out_tokens,
                    out_ld > 0 ? out_ld : G + 1);
}

int64_t accept_greedy_scratch_bytes(int B, int G, int V) {
    const int64_t nch = (V + kCH - 1) / kCH;
    return (int64_t)B * (G + 1) * nch * 8 + 256;
}

cudaError_t accept_greedy(const float *target, const int32_t *draft_tokens, int B, int G, int V,
                          int32_t *accept_count, int32_t *out_tokens, void *scratch, cudaStream_t s) {
    const int nch = (V + kCH - 1) / kCH;
    float *vmax = (float *)scratch;
    int32_t *imax = (int32_t *)((char *)scratch + (int64_t)B * (G + 1) * nch * 4);
    cudaError_t e = launch_k(chunk_argmax_kernel, dim3(nch, B * (G + 1)), dim3(kNL), 0, s, target, V, nch, vmax, imax);
    if (e != cudaSuccess) return e;
    return launch_k(greedy_finish_kernel, dim3(B), dim3(32), 0, s, (const float *)vmax, (const int32_t *)imax,
                    draft_tokens, G, nch, accept_count, out_tokens);
}

}  // namespace ifr

// ------------------------------------------------ allocation-free entry ------
// ifr_accept_noalloc: the sampled verification of ifr_accept with its scratch
// in a file-scope device array instead of the context's cudaMalloc'd buffer.
// Every scratch word is written by an earlier launch of the same call before
// it is read (chunk_stats -> cmax/csum, row_decide -> rstat/xdraft/okflag,
// finish -> rchunk), so nothing has to start at zero.  The one array per
// device is shared by every caller on that device: calls whose launches can
// overlap (different streams or contexts on one device) race on it and must
// be ordered by the caller.
#include "../../include/inferno_b200.h"

#include <mutex>

int ifr_fail(int code, const char *fmt, ...);
int ifr_cuda_fail(cudaError_t e, const char *what);
int ifr_ctx_device(const ifr_ctx *c);
cudaStream_t ifr_ctx_stream_of(const ifr_ctx *c);

namespace {

constexpr int64_t kNoAllocScratch = (int64_t)1 << 20;  // 1 MiB per device
static __device__ __align__(256) unsigned char g_accept_scratch[kNoAllocScratch];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kMaxDevices];

// set-up, once per device, with that device current: the array's address
int noalloc_scratch(int dev, void **out) {
    if (dev < 0 || dev >= kMaxDevices) return ifr_fail(IFR_ERR_ARG, "device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        int prev = -1;
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_accept_scratch);
        if (prev >= 0 && prev != dev) cudaSetDevice(prev);
        if (e != cudaSuccess) return ifr_cuda_fail(e, "cudaGetSymbolAddress(accept scratch)");
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return IFR_OK;
}

}  // namespace

extern "C" int ifr_accept_noalloc(ifr_ctx *c, const float *target, const float *draft,
                                  const int32_t *draft_tokens, const float *uniforms, int batch,
                                  int gamma, int vocab, float temperature, int32_t *accept_count,
                                  int32_t *out_tokens, int32_t *draft_out) {
    if (!c || !target || !draft || !uniforms || !accept_count || !out_tokens)
        return ifr_fail(IFR_ERR_ARG, "NULL argument");
    if (batch < 1 || gamma < 1 || gamma > 64 || vocab < 1)
        return ifr_fail(IFR_ERR_ARG, "invalid sizes batch=%d gamma=%d vocab=%d", batch, gamma, vocab);
    if (!(temperature > 0.f) || !(temperature < 1e30f))
        return ifr_fail(IFR_ERR_ARG, "temperature must be finite and > 0 (got %g)", (double)temperature);
    const int64_t need = ifr::accept_scratch_bytes(batch, gamma, vocab);
    if (need > kNoAllocScratch)
        return ifr_fail(IFR_ERR_ARG,
                        "ifr_accept_noalloc: batch=%d gamma=%d vocab=%d needs %lld scratch bytes, above its "
                        "fixed %lld (use ifr_accept)",
                        batch, gamma, vocab, (long long)need, (long long)kNoAllocScratch);
    const int dev = ifr_ctx_device(c);
    void *scratch = nullptr;
    int rc = noalloc_scratch(dev, &scratch);
    if (rc) return rc;
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
    cudaError_t e = ifr::accept_sampled(target, draft, draft_tokens, uniforms, batch, gamma, vocab,
                                        temperature, accept_count, out_tokens, draft_out, scratch,
                                        ifr_ctx_stream_of(c));
    if (prev >= 0 && prev != dev) cudaSetDevice(prev);
    if (e != cudaSuccess) return ifr_cuda_fail(e, "accept_noalloc launch");
    return IFR_OK;
}

// ---- greedy acceptance over a vocabulary split across tensor-parallel ranks ----
namespace ifr {

// per row: (max, off + argmax) over V logits, the lowest index among equal
// maxima (the rule of greedy_fused_kernel); cand[row] = {value, index bits}
__global__ void __launch_bounds__(256) row_argmax_kernel(const float *__restrict__ x, int64_t V, int off,
                                                         float2 *__restrict__ cand) {
    __shared__ float sv[256];
    __shared__ int si[256];
    pdl_trigger();
    pdl_wait();
    const float *row = x + (int64_t)blockIdx.x * V;
    float bv = -CUDART_INF_F;
    int bi = INT_MAX;
    for (int64_t j = threadIdx.x; j < V; j += 256) {
        const float v = row[j];
        if (v > bv || bi == INT_MAX) {
            bv = v;
            bi = (int)j;
        }
    }
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int o = 128; o; o >>= 1) {
        if (threadIdx.x < o) {
            const float ov = sv[threadIdx.x + o];
            const int oi = si[threadIdx.x + o];
            if (oi != INT_MAX && (si[threadIdx.x] == INT_MAX || ov > sv[threadIdx.x] ||
                                  (ov == sv[threadIdx.x] && oi < si[threadIdx.x]))) {
                sv[threadIdx.x] = ov;
                si[threadIdx.x] = oi;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) cand[blockIdx.x] = make_float2(sv[0], __int_as_float(si[0] + off));
}

// one thread per sequence: the rows' argmax over the W ranks' candidates
// ([W][rows], ranks in vocabulary order), then the longest matching draft
// prefix (mtp_verify_step!, src/ModelCPU.jl:2099-2115)
__global__ void tp_accept_kernel(const float2 *__restrict__ cand, int W, int rows, const int32_t *drafts,
                                 int draft_ld, int B, int G, int32_t *acc, int32_t *out, int out_ld) {
    pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    int32_t *ot = out + (int64_t)b * out_ld;
    for (int i = 0; i <= G; i++) ot[i] = -1;
    int a = 0;
    for (int i = 0; i <= G; i++) {
        const int r = b * (G + 1) + i;
        float best = cand[r].x;
        int arg = __float_as_int(cand[r].y);
        for (int w = 1; w < W; w++) {
            const float2 c = cand[(int64_t)w * rows + r];
            if (c.x > best) {
                best = c.x;
                arg = __float_as_int(c.y);
            }
        }
        ot[i] = arg;
        if (i == G || arg != drafts[(int64_t)b * draft_ld + i]) break;
        a++;
    }
    acc[b] = a;
}

cudaError_t row_argmax(const float *x, int rows, int64_t V, int off, float *cand, cudaStream_t s) {
    return launch_k(row_argmax_kernel, dim3(rows), dim3(256), 0, s, x, V, off, reinterpret_cast<float2 *>(cand));
}

cudaError_t tp_accept(const float *cand, int W, int rows, const int32_t *drafts, int draft_ld, int B, int G,
                      int32_t *acc, int32_t *out, int out_ld, cudaStream_t s) {
    return launch_k(tp_accept_kernel, dim3((B + 127) / 128), dim3(128), 0, s, reinterpret_cast<const float2 *>(cand),
                    W, rows, drafts, draft_ld, B, G, acc, out, out_ld);
}

}  // namespace ifr
