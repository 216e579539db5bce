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
// test), resid_chunks (one CTA per chunk of each sequence's rejected row:
// residual chunk sums), finish (per sequence: residual or bonus sample).
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

__device__ __forceinline__ uint32_t f_key(float x) {
    const uint32_t u = __float_as_uint(x);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ unsigned long long e_fixed(float e) {
    return (unsigned long long)__fmul_rn(e, 1073741824.0f);
}

// the filters' state; w(i, l) = the final weight of element i with logit l
struct SampleFilter {
    float M, T, min_p;
    bool topk, topp;
    uint32_t key_k, key_p;
    int cut_k, cut_p;
    __device__ float ek(int i, float l) const {
        if (topk) {
            const uint32_t k = f_key(l);
            if (!(k > key_k || (k == key_k && i <= cut_k))) return 0.f;
        }
        return elem_e(l, M, T);
    }
    __device__ float w(int i, float l) const {
        float e = ek(i, l);
        if (topp && e > 0.f) {
            const uint32_t k = __float_as_uint(e);
            if (!(k > key_p || (k == key_p && i <= cut_p))) e = 0.f;
        }
        if (min_p > 0.f && e < min_p) e = 0.f;
        return e;
    }
};

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

// FILT (filtered acceptance, accept_filtered below): element i of row r
// counts only when the row's filters keep it (filt[r].w(i, l) > 0); the chunk
// max stays over every element; draws take the first element with a
// positive weight and tau <= cumsum, and chunks with a positive mass only.
template <bool FILT>
__global__ void __launch_bounds__(kNL) chunk_stats_kernel(const float *__restrict__ target,
                                                          const float *__restrict__ draft, int B,
                                                          int G, int V, float T, int nch,
                                                          const SampleFilter *__restrict__ filt,
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
    SampleFilter F;
    if constexpr (FILT) F = filt[r];
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < kPER; q++) {
        if (q < n) {
            if constexpr (FILT) {
                if (!(F.w(c * kCH + kPER * threadIdx.x + q, x[q]) > 0.f)) continue;
            }
            t = __fadd_rn(t, elem_e(x[q], m, T));
        }
    }
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
// vals (POS: and val > 0); else the last element with val > 0; else the last
// element.
template <bool POS = false>
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
            if (hit < 0 && tau <= cum && (!POS || v[q] > 0.f)) hit = kPER * tid + q;
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

// row_stat with every thread of the block: the chunk maxima and the chunk
// masses cs[c] e^((cm[c] - M) / T) formed in parallel (the loads of a serial
// loop would each wait a memory round trip), then summed left to right by
// thread 0 - the same operations in the same order as row_stat.  All threads
// get the result.
__device__ RowStat row_stat_blk(const float *cm, const float *cs, int nch, float T, SampleSmem &sm) {
    if (nch > kNL) {  // more chunks than threads (vocabularies above 512K): the serial form
        if (threadIdx.x == 0) {
            const RowStat r = row_stat(cm, cs, nch, T);
            sm.bc[2] = r.M;
            sm.bc[3] = r.S;
        }
        __syncthreads();
        const RowStat r{sm.bc[2], sm.bc[3]};
        __syncthreads();
        return r;
    }
    const int tid = threadIdx.x;
    const float mv = tid < nch ? cm[tid] : -CUDART_INF_F;
    const float csv = tid < nch ? cs[tid] : 0.f;
    const float M = block_max(mv, sm.wsum);
    if (tid < nch) sm.lsum[tid] = __fmul_rn(csv, ifr_exp(__fdiv_rn(__fsub_rn(mv, M), T)));
    __syncthreads();
    if (tid == 0) {
        float S = 0.f;
        for (int c = 0; c < nch; c++) S = __fadd_rn(S, sm.lsum[c]);
        sm.bc[2] = S;
    }
    __syncthreads();
    const RowStat r{M, sm.bc[2]};
    __syncthreads();  // lsum and bc are reused by the caller
    return r;
}

// sample from softmax(row/T) with uniform u; row stats (M,S) and chunk stats
// given; FILT: over the elements F keeps (F non-null), positive masses only
template <bool FILT = false>
__device__ int sample_row(const float *row, int V, const float *cm, const float *cs, int nch,
                          float T, RowStat st, float u, SampleSmem &sm, const SampleFilter *F = nullptr) {
    // the chunk masses in parallel first (thread 0's scan then reads shared memory)
    const bool pre = nch <= kNL;
    if (pre && (int)threadIdx.x < nch)
        sm.lsum[threadIdx.x] = __fmul_rn(cs[threadIdx.x], ifr_exp(__fdiv_rn(__fsub_rn(cm[threadIdx.x], st.M), T)));
    __syncthreads();
    if (threadIdx.x == 0) {
        float tau = __fmul_rn(u, st.S), P = 0.f;
        int csel = -1;
        for (int c = 0; c < nch; c++) {
            const float mc = pre ? sm.lsum[c] : __fmul_rn(cs[c], ifr_exp(__fdiv_rn(__fsub_rn(cm[c], st.M), T)));
            float nP = __fadd_rn(P, mc);
            if ((!FILT || mc > 0.f) && tau <= nP) { csel = c; break; }
            P = nP;
        }
        if (csel < 0) {
            for (int c = nch - 1; c >= 0; c--) {
                const float mc = FILT ? __fmul_rn(cs[c], ifr_exp(__fdiv_rn(__fsub_rn(cm[c], st.M), T))) : cs[c];
                if (mc > 0.f) { csel = c; break; }
            }
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
    for (int q = 0; q < kPER; q++) {
        v[q] = q < n ? elem_e(x[q], mc, T) : 0.f;
        if constexpr (FILT) {
            if (q < n && !(F->w(csel * kCH + kPER * threadIdx.x + q, x[q]) > 0.f)) v[q] = 0.f;
        }
    }
    return chunk_search<FILT>(v, n, (int64_t)csel * kCH, taup, sm.lsum, sm.res);
}

__device__ __forceinline__ float weight_of(const float *row, int i, const float *cm, RowStat st, float T) {
    const int c = i / kCH;
    return __fmul_rn(elem_e(__ldg(row + i), cm[c], T), ifr_exp(__fdiv_rn(__fsub_rn(cm[c], st.M), T)));
}
// the weight of element i under the row's filters (0 where they drop it)
template <bool FILT>
__device__ __forceinline__ float kept_weight_of(const float *row, int i, const float *cm, RowStat st, float T,
                                                const SampleFilter *F) {
    if constexpr (FILT) {
        if (!(F->w(i, __ldg(row + i)) > 0.f)) return 0.f;
    }
    return weight_of(row, i, cm, st, T);
}

// grid (B, G+1): row stats of target row i (and draft row i < G), draft token, ratio test
template <bool FILT>
__global__ void __launch_bounds__(kNL) row_decide_kernel(
    const float *__restrict__ target, const float *__restrict__ draft,
    const int32_t *__restrict__ draft_tokens, const float *__restrict__ uniforms, int B, int G, int V,
    float T, int nch, const SampleFilter *__restrict__ filt, const float *__restrict__ cmax,
    const float *__restrict__ csum, float *__restrict__ rstat, int32_t *__restrict__ xdraft,
    int32_t *__restrict__ okflag) {
    __shared__ SampleSmem sm;
    __shared__ RowStat st_s[2];
    const int b = blockIdx.x, i = blockIdx.y;
    const int tr = b * (G + 1) + i;
    const float *trow = target + (int64_t)tr * V;
    {
        const RowStat st = row_stat_blk(cmax + (int64_t)tr * nch, csum + (int64_t)tr * nch, nch, T, sm);
        if (threadIdx.x == 0) {
            st_s[0] = st;
            rstat[2 * tr] = st.M;
            rstat[2 * tr + 1] = st.S;
        }
    }
    if (i == G) return;
    const int dr = B * (G + 1) + b * G + i;
    const float *drow = draft + (int64_t)(b * G + i) * V;
    {
        const RowStat st = row_stat_blk(cmax + (int64_t)dr * nch, csum + (int64_t)dr * nch, nch, T, sm);
        if (threadIdx.x == 0) {
            st_s[1] = st;
            rstat[2 * dr] = st.M;
            rstat[2 * dr + 1] = st.S;
        }
    }
    __syncthreads();
    SampleFilter Ft, Fd;
    if constexpr (FILT) {
        Ft = filt[tr];
        Fd = filt[dr];
    }
    const float *u = uniforms + (int64_t)b * (2 * G + 1);
    int x;
    if (draft_tokens) {
        x = draft_tokens[b * G + i];
    } else {
        x = sample_row<FILT>(drow, V, cmax + (int64_t)dr * nch, csum + (int64_t)dr * nch, nch, T, st_s[1],
                             u[i], sm, &Fd);
    }
    if (threadIdx.x == 0) {
        int ok;
        if (x < 0 || x >= V) {
            ok = 0;  // invalid supplied draft token: reject
        } else {
            float pt = __fdiv_rn(kept_weight_of<FILT>(trow, x, cmax + (int64_t)tr * nch, st_s[0], T, &Ft), st_s[0].S);
            float pd = __fdiv_rn(kept_weight_of<FILT>(drow, x, cmax + (int64_t)dr * nch, st_s[1], T, &Fd), st_s[1].S);
            ok = pd > 0.f ? (u[G + i] < __fdiv_rn(pt, pd)) : (pt > 0.f);
        }
        xdraft[b * G + i] = x;
        okflag[b * G + i] = ok;
    }
}

// the residual weight max(p_t - p_d, 0) of one element (FILT: 0 for either
// side where its filters drop the element)
template <bool FILT>
__device__ __forceinline__ float resid_w(float lt, float ld, int i, float tcm, float ft, RowStat ts, float dcm,
                                         float fd, RowStat ds, float T, const SampleFilter &Ft,
                                         const SampleFilter &Fd) {
    float pt = __fdiv_rn(__fmul_rn(elem_e(lt, tcm, T), ft), ts.S);
    float pd = __fdiv_rn(__fmul_rn(elem_e(ld, dcm, T), fd), ds.S);
    if constexpr (FILT) {
        if (!(Ft.w(i, lt) > 0.f)) pt = 0.f;
        if (!(Fd.w(i, ld) > 0.f)) pd = 0.f;
    }
    const float r = __fsub_rn(pt, pd);
    return r > 0.f ? r : 0.f;
}

// grid (nch, B): chunk c of the residual max(p_t - p_d, 0) of sequence b's
// rejected row (none when every draft was accepted), canonical sum into
// rchunk[b][c]; one CTA per chunk, so the pass runs at full width
template <bool FILT>
__global__ void __launch_bounds__(kNL) resid_chunks_kernel(
    const float *__restrict__ target, const float *__restrict__ draft, int B, int G, int V, float T, int nch,
    const SampleFilter *__restrict__ filt, const float *__restrict__ cmax, const float *__restrict__ rstat,
    const int32_t *__restrict__ okflag, float *__restrict__ rchunk) {
    __shared__ float wsum[8];
    const int c = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    int acc = 0;
    while (acc < G && okflag[b * G + acc]) acc++;
    if (acc == G) return;
    const int tr = b * (G + 1) + acc, dr = B * (G + 1) + b * G + acc;
    const float *trow = target + (int64_t)tr * V, *drow = draft + (int64_t)(b * G + acc) * V;
    const float tcm = cmax[(int64_t)tr * nch + c], dcm = cmax[(int64_t)dr * nch + c];
    const RowStat ts{rstat[2 * tr], rstat[2 * tr + 1]}, ds{rstat[2 * dr], rstat[2 * dr + 1]};
    SampleFilter Ft, Fd;
    if constexpr (FILT) {
        Ft = filt[tr];
        Fd = filt[dr];
    }
    float xt[8], xd[8];
    const int n = load8(trow, V, c, xt);
    load8(drow, V, c, xd);
    const float ft = ifr_exp(__fdiv_rn(__fsub_rn(tcm, ts.M), T));
    const float fd = ifr_exp(__fdiv_rn(__fsub_rn(dcm, ds.M), T));
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < kPER; q++)
        if (q < n)
            t = __fadd_rn(t, resid_w<FILT>(xt[q], xd[q], c * kCH + kPER * tid + q, tcm, ft, ts, dcm, fd, ds, T, Ft,
                                           Fd));
    const float sum = canon_sum(t, wsum);
    if (tid == 0) rchunk[(int64_t)b * nch + c] = sum;
}

// grid (B): accept count, emitted tokens, residual or bonus sample
template <bool FILT>
__global__ void __launch_bounds__(kNL) finish_kernel(
    const float *__restrict__ target, const float *__restrict__ draft,
    const float *__restrict__ uniforms, int B, int G, int V, float T, int nch,
    const SampleFilter *__restrict__ filt, const float *__restrict__ cmax, const float *__restrict__ csum,
    const float *__restrict__ rstat, const int32_t *__restrict__ xdraft, const int32_t *__restrict__ okflag,
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
        SampleFilter Ft;
        if constexpr (FILT) Ft = filt[tr];
        y = sample_row<FILT>(target + (int64_t)tr * V, V, cmax + (int64_t)tr * nch, csum + (int64_t)tr * nch,
                             nch, T, st, ub, sm, &Ft);
    } else {
        const int tr = b * (G + 1) + acc, dr = B * (G + 1) + b * G + acc;
        const float *trow = target + (int64_t)tr * V, *drow = draft + (int64_t)(b * G + acc) * V;
        const float *tcm = cmax + (int64_t)tr * nch, *dcm = cmax + (int64_t)dr * nch;
        const RowStat ts{rstat[2 * tr], rstat[2 * tr + 1]}, ds{rstat[2 * dr], rstat[2 * dr + 1]};
        SampleFilter Ft, Fd;
        if constexpr (FILT) {
            Ft = filt[tr];
            Fd = filt[dr];
        }
        const float *rcg = rchunk + (int64_t)b * nch;  // residual chunk sums (resid_chunks_kernel)
        const bool pre = nch <= kNL;
        if (pre && tid < nch) sm.lsum[tid] = rcg[tid];
        __syncthreads();
        const float *rc = pre ? sm.lsum : rcg;
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
                    if ((!FILT || rc[c] > 0.f) && tau <= nP) { csel = c; break; }
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
            y = sample_row<FILT>(trow, V, tcm, csum + (int64_t)tr * nch, nch, T, ts, ub, sm, &Ft);
        } else {
            float xt[8], xd[8], v[8];
            const int n = load8(trow, V, csel, xt);
            load8(drow, V, csel, xd);
            const float ft = ifr_exp(__fdiv_rn(__fsub_rn(tcm[csel], ts.M), T));
            const float fd = ifr_exp(__fdiv_rn(__fsub_rn(dcm[csel], ds.M), T));
#pragma unroll
            for (int q = 0; q < kPER; q++)
                v[q] = q < n ? resid_w<FILT>(xt[q], xd[q], csel * kCH + kPER * tid + q, tcm[csel], ft, ts,
                                             dcm[csel], fd, ds, T, Ft, Fd)
                             : 0.f;
            y = chunk_search<FILT>(v, n, (int64_t)csel * kCH, sm.bc[1], sm.lsum, sm.res);
        }
    }
    if (tid == 0) ot[acc] = y;
}

int64_t accept_scratch_bytes(int B, int G, int V) {
    const int64_t nch = (V + kCH - 1) / kCH, rows = (int64_t)B * (2 * G + 1);
    return 2 * rows * nch * 4 + 2 * rows * 4 + 2 * (int64_t)B * G * 4 + (int64_t)B * nch * 4 + 1024;
}

namespace {
// the three acceptance launches over the scratch layout of accept_scratch_bytes
template <bool FILT>
cudaError_t accept_launch(const float *target, const float *draft, const int32_t *draft_tokens,
                          const float *uniforms, int B, int G, int V, float T, const SampleFilter *filt,
                          int32_t *accept_count, int32_t *out_tokens, int32_t *draft_out, void *scratch,
                          cudaStream_t s) {
    const int nch = (V + kCH - 1) / kCH;
    const int64_t rows = (int64_t)B * (2 * G + 1);
    char *p = (char *)scratch;
    float *cmax = (float *)p; p += rows * nch * 4;
    float *csum = (float *)p; p += rows * nch * 4;
    float *rstat = (float *)p; p += 2 * rows * 4;
    int32_t *xdraft = (int32_t *)p; p += (int64_t)B * G * 4;
    int32_t *okflag = (int32_t *)p; p += (int64_t)B * G * 4;
    float *rchunk = (float *)p;
    chunk_stats_kernel<FILT><<<dim3(nch, (unsigned)rows), kNL, 0, s>>>(target, draft, B, G, V, T, nch, filt, cmax,
                                                                       csum);
    row_decide_kernel<FILT><<<dim3(B, G + 1), kNL, 0, s>>>(target, draft, draft_tokens, uniforms, B, G, V, T,
                                                           nch, filt, cmax, csum, rstat, xdraft, okflag);
    resid_chunks_kernel<FILT><<<dim3(nch, B), kNL, 0, s>>>(target, draft, B, G, V, T, nch, filt, cmax, rstat,
                                                           okflag, rchunk);
    finish_kernel<FILT><<<B, kNL, 0, s>>>(target, draft, uniforms, B, G, V, T, nch, filt, cmax, csum, rstat,
                                          xdraft, okflag, accept_count, out_tokens, draft_out, rchunk);
    return cudaGetLastError();
}
}  // namespace

cudaError_t accept_sampled(const float *target, const float *draft, const int32_t *draft_tokens,
                           const float *uniforms, int B, int G, int V, float T, int32_t *accept_count,
                           int32_t *out_tokens, int32_t *draft_out, void *scratch, cudaStream_t s) {
    return accept_launch<false>(target, draft, draft_tokens, uniforms, B, G, V, T, nullptr, accept_count,
                                out_tokens, draft_out, scratch, s);
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

// ------------------------------------------------------ filtered sampling ---
// CommonOps.softmax_sample_scratch! (src/CommonOps.jl:196-318), one CTA per
// row, with the supplied uniform u in place of rand().  Fixed evaluation,
// shared with the oracle (oracle/accept.c, or_sample_filtered):
//   validation: NaN or +Inf -> token -1 (the reference throws, :145-160);
//     M = max finite logit and g its first index; all -Inf -> 0; T == 0 or
//     V == 1 -> g (:207-210)
//   top_k, 0 < k < V (:217-230): the k largest logits, ties at the k-th value
//     to the lower index; found by a 4 x 8-bit radix select on order-preserving
//     keys (counts per digit bin), the tie cut by an index-ordered count
//   e_i = ifr_exp((l_i - M) / T) for kept i, else 0 (:234-243); the
//     renormalisations scale all weights alike and fold into the draw's sum
//   top_p < 1 (:249-278): integer weights E_i = trunc(e_i 2^30), target =
//     top_p * sum E (double); keep the first m elements in (e desc, index asc)
//     order, m minimal with E_(1) + ... + E_(m) >= target - a radix select on
//     the keys of e with exact 64-bit sums per digit bin, then the smallest
//     count of the crossing value's elements, taken by index
//   min_p > 0 (:280-299): keep e_i >= min_p (max_p sits at e = 1)
//   draw (:301-317): w_i = kept ? e_i : 0; chunk sums in the canonical order
//     above; tau = u W; first i with w_i > 0 and tau <= cumsum, else the last
//     i with w_i > 0
constexpr int kSampleMaxChunks = 256;  // vocab <= 256 x 2048

struct SampleFSmem {
    unsigned cnt[256];
    unsigned long long sum[256];
    float cs[kSampleMaxChunks];
    float lsum[kNL];
    unsigned lcnt[kNL];
    float wsum[8];
    float bv[8];
    int bi[8];
    int res[2];
    unsigned long long S, above;
    unsigned prefix, need, eq, before, total;
    int sel, found, idx;
    float tau;
    int csel;
};

// Radix select, descending, over 32-bit keys key(i, l) of every element, with
// 64-bit weights weight(i, l) when BY_SUM.  BY_SUM: the largest key value v
// with sum_{key >= v} weight >= target; else the value of the rank-th largest
// key.  Leaves in sm: prefix (that key), eq (elements holding it), above (the
// weight above it), need (its rank among the equal ones, count select); sel <
// 0 if no bin reaches the target (BY_SUM only).
template <bool BY_SUM, class KeyF, class WF>
__device__ void radix_desc(const float *row, int V, int nch, KeyF key, WF weight, unsigned rank, double target,
                           SampleFSmem &sm) {
    const int tid = threadIdx.x;
    __syncthreads();
    if (tid == 0) { sm.prefix = 0u; sm.above = 0ull; sm.need = rank; sm.sel = 0; sm.eq = 0u; }
    uint32_t mask = 0u;
    for (int d = 3; d >= 0; d--) {
        const int shift = 8 * d;
        __syncthreads();
        sm.cnt[tid] = 0u;
        sm.sum[tid] = 0ull;
        __syncthreads();
        const uint32_t prefix = sm.prefix;
        if (sm.sel >= 0) {
            for (int c = 0; c < nch; c++) {
                float x[8];
                const int n = load8(row, V, c, x);
                for (int q = 0; q < n; q++) {
                    const int i = c * kCH + kPER * tid + q;
                    const uint32_t k = key(i, x[q]);
                    if (((k ^ prefix) & mask) == 0u) {
                        const int b = (int)((k >> shift) & 255u);
                        atomicAdd(&sm.cnt[b], 1u);
                        if (BY_SUM) atomicAdd(&sm.sum[b], weight(i, x[q]));
                    }
                }
            }
        }
        __syncthreads();
        if (tid == 0 && sm.sel >= 0) {
            int sel = -1;
            unsigned cum = 0u;
            unsigned long long cs = 0ull;
            for (int b = 255; b >= 0; b--) {
                if (sm.cnt[b] == 0u) continue;
                if (BY_SUM ? ((double)(sm.above + cs + sm.sum[b]) >= target) : (cum + sm.cnt[b] >= sm.need)) {
                    sel = b;
                    break;
                }
                cum += sm.cnt[b];
                cs += sm.sum[b];
            }
            if (sel >= 0) {
                sm.prefix = prefix | ((uint32_t)sel << shift);
                sm.above += cs;
                if (!BY_SUM) sm.need -= cum;
                sm.eq = sm.cnt[sel];
            }
            sm.sel = sel;
        }
        mask |= 255u << shift;
    }
    __syncthreads();
}

// index of the n-th element (1-based, index order) with pred(i, l); INT_MAX
// if there are fewer
template <class Pred>
__device__ int nth_index(const float *row, int V, int nch, Pred pred, unsigned n, SampleFSmem &sm) {
    const int tid = threadIdx.x;
    __syncthreads();
    if (tid == 0) { sm.before = 0u; sm.idx = INT_MAX; }
    for (int c = 0; c < nch; c++) {
        float x[8];
        const int nv = load8(row, V, c, x);
        unsigned m = 0u;
        for (int q = 0; q < nv; q++) m += pred(c * kCH + kPER * tid + q, x[q]) ? 1u : 0u;
        __syncthreads();
        sm.lcnt[tid] = m;
        __syncthreads();
        if (tid == 0) {
            unsigned cum = sm.before;
            int found = -1;
            for (int j = 0; j < kNL; j++) {
                if (cum + sm.lcnt[j] >= n) { found = j; break; }
                cum += sm.lcnt[j];
            }
            sm.found = found;
            sm.total = cum;  // matches before lane `found` (or in all lanes, when none)
        }
        __syncthreads();
        const int found = sm.found;
        if (found >= 0) {
            if (tid == found) {
                unsigned k = sm.total;
                for (int q = 0; q < nv; q++) {
                    const int i = c * kCH + kPER * tid + q;
                    if (pred(i, x[q]) && ++k == n) { sm.idx = i; break; }
                }
            }
            __syncthreads();
            return sm.idx;
        }
        if (tid == 0) sm.before = sm.total;
    }
    __syncthreads();
    return INT_MAX;
}

// smallest n >= 1 with above + n unit >= target (unit > 0)
__device__ unsigned long long cut_count(unsigned long long above, unsigned long long unit, double target) {
    const double q = ceil((target - (double)above) / (double)unit);
    unsigned long long n = q < 1.0 ? 1ull : (unsigned long long)q;
    while (n > 1ull && (double)(above + (n - 1ull) * unit) >= target) n--;
    while ((double)(above + n * unit) < target) n++;
    return n;
}

// the filters of one row (all threads; M = the row's max finite logit):
// top-k by radix select on the logits' keys, the exact top-p cut on the
// integer weights, min-p as a threshold (the rules above)
__device__ SampleFilter build_filter(const float *row, int V, int nch, float M, float T, int top_k, float top_p,
                                     float min_p, SampleFSmem &sm) {
    const int tid = threadIdx.x;
    SampleFilter F;
    F.M = M;
    F.T = T;
    F.min_p = min_p;
    F.topk = top_k > 0 && top_k < V;
    F.topp = false;
    F.key_k = 0u;
    F.cut_k = INT_MAX;
    F.key_p = 0u;
    F.cut_p = INT_MAX;
    auto none = [](int, float) { return 0ull; };
    if (F.topk) {
        radix_desc<false>(row, V, nch, [](int, float l) { return f_key(l); }, none, (unsigned)top_k, 0.0, sm);
        F.key_k = sm.prefix;
        const unsigned need = sm.need, eq = sm.eq;
        if (need < eq) {
            const uint32_t kk = F.key_k;
            F.cut_k = nth_index(row, V, nch, [kk](int, float l) { return f_key(l) == kk; }, need, sm);
        }
    }
    if (top_p < 1.0f) {
        // exact integer total of the top-k weights
        unsigned long long part = 0ull;
        for (int c = 0; c < nch; c++) {
            float x[8];
            const int n = load8(row, V, c, x);
            for (int q = 0; q < n; q++) part += e_fixed(F.ek(c * kCH + kPER * tid + q, x[q]));
        }
        __syncthreads();
        if (tid == 0) sm.S = 0ull;
        __syncthreads();
        atomicAdd(&sm.S, part);
        __syncthreads();
        const double target = (double)top_p * (double)sm.S;
        const SampleFilter Fk = F;
        radix_desc<true>(row, V, nch, [Fk](int i, float l) { return __float_as_uint(Fk.ek(i, l)); },
                         [Fk](int i, float l) { return e_fixed(Fk.ek(i, l)); }, 0u, target, sm);
        if (sm.sel >= 0) {
            F.topp = true;
            F.key_p = sm.prefix;
            const unsigned long long unit = e_fixed(__uint_as_float(F.key_p));
            const unsigned long long need =
                unit > 0ull ? cut_count(sm.above, unit, target) : (unsigned long long)sm.eq;
            if (need < (unsigned long long)sm.eq) {
                const uint32_t kp = F.key_p;
                F.cut_p = nth_index(row, V, nch, [Fk, kp](int i, float l) { return __float_as_uint(Fk.ek(i, l)) == kp; },
                                    (unsigned)need, sm);
            }
        }
    }
    return F;
}

__global__ void __launch_bounds__(kNL) sample_kernel(const float *__restrict__ logits, int V, float T, int top_k,
                                                     float top_p, float min_p, const float *__restrict__ uniforms,
                                                     int32_t *__restrict__ out) {
    __shared__ SampleFSmem sm;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, r = blockIdx.x;
    const float *row = logits + (int64_t)r * V;
    const int nch = (V + kCH - 1) / kCH;
    pdl_trigger();
    pdl_wait();
    // validation, max and its first index
    float bv = -CUDART_INF_F;
    int bi = INT_MAX, bad = 0;
    for (int c = 0; c < nch; c++) {
        float x[8];
        const int n = load8(row, V, c, x);
        for (int q = 0; q < n; q++) {
            const float v = x[q];
            if (v != v || v == CUDART_INF_F) bad = 1;
            else if (v != -CUDART_INF_F && v > bv) { bv = v; bi = c * kCH + kPER * tid + q; }
        }
    }
    bad = __syncthreads_or(bad);
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (oi != INT_MAX && (bi == INT_MAX || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
    }
    if (lane == 0) { sm.bv[warp] = bv; sm.bi[warp] = bi; }
    __syncthreads();
    float M = sm.bv[0];
    int g = sm.bi[0];
    for (int w = 1; w < kNL / 32; w++)
        if (sm.bi[w] != INT_MAX && (g == INT_MAX || sm.bv[w] > M || (sm.bv[w] == M && sm.bi[w] < g))) {
            M = sm.bv[w];
            g = sm.bi[w];
        }
    if (bad || g == INT_MAX || T == 0.f || V == 1) {
        if (tid == 0) out[r] = bad ? -1 : (g == INT_MAX ? 0 : g);
        return;
    }
    const SampleFilter F = build_filter(row, V, nch, M, T, top_k, top_p, min_p, sm);
    // draw: chunk sums of the final weights in the canonical order
    for (int c = 0; c < nch; c++) {
        float x[8];
        const int n = load8(row, V, c, x);
        float t = 0.f;
        for (int q = 0; q < n; q++) t = __fadd_rn(t, F.w(c * kCH + kPER * tid + q, x[q]));
        const float sc = canon_sum(t, sm.wsum);
        if (tid == 0) sm.cs[c] = sc;
    }
    __syncthreads();
    if (tid == 0) {
        float W = 0.f;
        for (int c = 0; c < nch; c++) W = __fadd_rn(W, sm.cs[c]);
        float tau = __fmul_rn(uniforms[r], W), P = 0.f;
        int csel = -1;
        for (int c = 0; c < nch; c++) {
            const float nP = __fadd_rn(P, sm.cs[c]);
            if (sm.cs[c] > 0.f && tau <= nP) { csel = c; break; }
            P = nP;
        }
        if (csel < 0) {
            for (int c = nch - 1; c >= 0; c--) if (sm.cs[c] > 0.f) { csel = c; break; }
            if (csel < 0) csel = nch - 1;
            P = 0.f;
            for (int c = 0; c < csel; c++) P = __fadd_rn(P, sm.cs[c]);
            tau = __fadd_rn(P, sm.cs[csel]);
        }
        sm.csel = csel;
        sm.tau = __fsub_rn(tau, P);
        sm.res[0] = INT_MAX;
        sm.res[1] = -1;
    }
    __syncthreads();
    const int csel = sm.csel;
    const float taup = sm.tau;
    float x[8], v[8];
    const int n = load8(row, V, csel, x);
    float t = 0.f;
    for (int q = 0; q < kPER; q++) {
        v[q] = q < n ? F.w(csel * kCH + kPER * tid + q, x[q]) : 0.f;
        if (q < n) t = __fadd_rn(t, v[q]);
    }
    sm.lsum[tid] = t;
    __syncthreads();
    if (tid == 0) {  // exclusive prefix, sequential
        float pre = 0.f;
        for (int j = 0; j < kNL; j++) { const float tj = sm.lsum[j]; sm.lsum[j] = pre; pre = __fadd_rn(pre, tj); }
    }
    __syncthreads();
    float cum = sm.lsum[tid];
    int hit = -1, lastpos = -1;
    for (int q = 0; q < n; q++) {
        cum = __fadd_rn(cum, v[q]);
        if (v[q] > 0.f) {
            if (hit < 0 && taup <= cum) hit = kPER * tid + q;
            lastpos = kPER * tid + q;
        }
    }
    if (hit >= 0) atomicMin(&sm.res[0], hit);
    if (lastpos >= 0) atomicMax(&sm.res[1], lastpos);
    __syncthreads();
    if (tid == 0) {
        const int base = csel * kCH;
        const int last = min(V, base + kCH) - 1;
        out[r] = sm.res[0] != INT_MAX ? base + sm.res[0] : (sm.res[1] >= 0 ? base + sm.res[1] : last);
    }
}

cudaError_t sample_filtered(const float *logits, int rows, int V, float T, int top_k, float top_p, float min_p,
                            const float *uniforms, int32_t *out, cudaStream_t s) {
    if ((V + kCH - 1) / kCH > kSampleMaxChunks) return cudaErrorInvalidValue;
    return launch_k(sample_kernel, dim3(rows), dim3(kNL), 0, s, logits, V, T, top_k, top_p, min_p, uniforms, out);
}

// ------------------------------------------------ filtered acceptance ------
// The sampled verification on the distributions the sampler's filters leave:
// top-k, top-p and min-p (the rules of sample_kernel) applied with the same
// temperature to every target and draft row.  The reference draws its drafts
// and the bonus token from filtered distributions
// (src/SpeculativeDecoding.jl:57,102 via CommonOps.softmax_sample_scratch!);
// filtering the target and draft rows of the ratio test and the residual as
// well keeps every emitted token distributed as the filtered target.  One
// filter pass per row (filter_rows_kernel: a CTA per row, the filter's few
// scalars into scratch), then the three acceptance launches with FILT.
// Restated on the CPU by oracle/accept.c (or_accept_filtered).
__global__ void __launch_bounds__(kNL) filter_rows_kernel(const float *__restrict__ target,
                                                          const float *__restrict__ draft, int B, int G, int V,
                                                          float T, int top_k, float top_p, float min_p,
                                                          SampleFilter *__restrict__ filt) {
    __shared__ SampleFSmem sm;
    __shared__ float wbuf[8];
    const int r = blockIdx.x;
    const float *row = row_ptr(target, draft, r, B, G, V);
    const int nch = (V + kCH - 1) / kCH;
    float m = -CUDART_INF_F;
    for (int c = 0; c < nch; c++) {
        float x[8];
        const int n = load8(row, V, c, x);
        for (int q = 0; q < n; q++) m = fmaxf(m, x[q]);
    }
    const float M = block_max(m, wbuf);
    const SampleFilter F = build_filter(row, V, nch, M, T, top_k, top_p, min_p, sm);
    if (threadIdx.x == 0) filt[r] = F;
}

int64_t accept_filtered_scratch_bytes(int B, int G, int V) {
    return accept_scratch_bytes(B, G, V) + (int64_t)B * (2 * G + 1) * (int64_t)sizeof(SampleFilter) + 256;
}

cudaError_t accept_filtered(const float *target, const float *draft, const float *uniforms, int B, int G, int V,
                            float T, int top_k, float top_p, float min_p, int32_t *accept_count,
                            int32_t *out_tokens, int32_t *draft_out, void *scratch, cudaStream_t s) {
    if ((V + kCH - 1) / kCH > kSampleMaxChunks) return cudaErrorInvalidValue;
    const int64_t rows = (int64_t)B * (2 * G + 1);
    const int64_t base = (accept_scratch_bytes(B, G, V) + 255) / 256 * 256;
    SampleFilter *filt = reinterpret_cast<SampleFilter *>((char *)scratch + base);
    filter_rows_kernel<<<(unsigned)rows, kNL, 0, s>>>(target, draft, B, G, V, T, top_k, top_p, min_p, filt);
    return accept_launch<true>(target, draft, nullptr, uniforms, B, G, V, T, filt, accept_count, out_tokens,
                               draft_out, scratch, s);
}

// presence then repetition penalty (src/ModelCPU.jl:1202-1211,1237-1238;
// src/CommonOps.jl:63-76) on each row's distinct seen tokens: a shared bitmap
// of the vocabulary lets exactly one thread apply each distinct token
__global__ void __launch_bounds__(256) penalty_kernel(float *__restrict__ logits, int V,
                                                      const int32_t *__restrict__ seen, int n_seen,
                                                      float presence, float repetition) {
    extern __shared__ unsigned bitmap[];
    const int r = blockIdx.x, words = (V + 31) >> 5;
    pdl_trigger();
    pdl_wait();
    for (int i = threadIdx.x; i < words; i += blockDim.x) bitmap[i] = 0u;
    __syncthreads();
    float *l = logits + (int64_t)r * V;
    const int32_t *sn = seen + (int64_t)r * n_seen;
    for (int j = threadIdx.x; j < n_seen; j += blockDim.x) {
        const int t = sn[j];
        if (t < 0 || t >= V) continue;
        const unsigned bit = 1u << (t & 31);
        if (atomicOr(&bitmap[t >> 5], bit) & bit) continue;
        float x = l[t];
        if (presence != 0.f) x = __fsub_rn(x, presence);
        if (repetition != 1.f) x = x > 0.f ? __fdiv_rn(x, repetition) : __fmul_rn(x, repetition);
        l[t] = x;
    }
}

cudaError_t apply_penalties(float *logits, int rows, int V, const int32_t *seen, int n_seen, float presence,
                            float repetition, cudaStream_t s) {
    const size_t smem = (size_t)((V + 31) / 32) * 4;
    static DeviceFlags attr;
    if (!attr.test()) {
        cudaError_t e = cudaFuncSetAttribute(penalty_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 128 * 1024);
        if (e != cudaSuccess) return e;
        attr.set();
    }
    return launch_k(penalty_kernel, dim3(rows), dim3(256), smem, s, logits, V, seen, n_seen, presence, repetition);
}

}  // namespace ifr

// ------------------------------------------------ allocation-free entry ------
// ifr_accept_noalloc: the sampled verification of ifr_accept with its scratch
// in a file-scope device array instead of the context's cudaMalloc'd buffer.
// The array's device address is looked up once per device and cached for the
// life of the process; a device reset (cudaDeviceReset, or a host runtime
// resetting the device's primary context) reloads the module at another
// address, so the cached set-up is then stale and this entry point must not
// be used on that device again.
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
    if ((int64_t)batch * (2 * gamma + 1) > ifr::kAcceptMaxRows)
        return ifr_fail(IFR_ERR_ARG, "batch=%d gamma=%d: batch * (2 gamma + 1) logits rows exceed %d", batch, gamma,
                        ifr::kAcceptMaxRows);
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
