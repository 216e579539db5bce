/*
 * Speculative-decoding acceptance, CPU oracle.  TEST INFRASTRUCTURE ONLY.
 *
 * Restates src/SpeculativeDecoding.jl:20-104 with the fixes listed below and
 * a fully specified floating-point evaluation order, so that the device
 * kernel (csrc/accept.cu) reproduces accept counts and tokens bit for bit
 * from the same supplied uniforms.
 *
 * Fixes relative to the reference (src/SpeculativeDecoding.jl):
 *   - draft probabilities use the same temperature as the target (:61-63
 *     ignored it);
 *   - the residual is max(p_t - p_d, 0) with the draft *distribution* p_d
 *     (:91-94 subtracted a scalar);
 *   - all rows of target logits are used (:70 requested only the last one).
 * Kept: accept iff u < min(1, p_t[x]/p_d[x]) (:85-87); inverse-CDF sampling
 * "first i with r <= cumsum" (:20-30, CommonOps.jl:303-314); bonus token from
 * the last target row after gamma accepts (:101-104).
 *
 * Canonical evaluation order (shared with the device code):
 *   row split into chunks of OR_ACCEPT_CHUNK elements; in chunk c
 *     m_c  = max(l)
 *     e_i  = or_exp((l_i - m_c) / T)
 *     lane j (0..255) sums e over elements 8j..8j+7 of the chunk, in order;
 *     the 256 lane sums are combined by a 32-lane xor butterfly
 *     (offsets 16,8,4,2,1) per warp, then warp sums 0..7 left to right -> s_c
 *   row: M = max_c m_c, f_c = or_exp((m_c - M)/T),
 *        S = sum_c s_c*f_c left to right, element weight w_i = e_i*f_c
 *   sampling with uniform u: tau = u*S; chunk c* = first c with
 *     tau <= P_{c+1} (P = running left-to-right sum of s_c*f_c);
 *     tau' = (tau - P_{c*}) / f_{c*}; inside the chunk the cumulative sum is
 *     blocked: sequential prefix of the lane sums, then sequential inside the
 *     lane; token = first element with tau' <= cumsum, else the last element
 *     of the chunk with e > 0.
 */
#include "oracle.h"
#include <math.h>
#include <string.h>
#include <stdlib.h>

/*
 * exp(x) by Cody & Waite range reduction (W. J. Cody, W. Waite, "Software
 * Manual for the Elementary Functions", 1980): x = n*ln2 + r, |r| <= ln2/2,
 * ln2 split into a head with 8 trailing zero bits and a tail so n*ln2_hi is
 * exact; e^r by its Taylor series to degree 7 (Horner, fused multiply-add);
 * result scaled by 2^n built from exponent bits.  Only IEEE-754 single
 * operations with round-to-nearest are used, so CPU and GPU agree bit for bit.
 */
float or_exp(float x) {
    if (x != x) return x;
    if (x > 88.5f) return INFINITY;
    if (x < -87.0f) return 0.0f;
    const float log2e = 1.44269502162933349609375f;     /* nearest float to 1/ln 2 */
    const float ln2_hi = 0.693145751953125f;             /* 0x3f317200 */
    const float ln2_lo = 1.42860677e-06f;                /* ln2 - ln2_hi */
    float n = rintf(x * log2e);
    float r = fmaf(-n, ln2_hi, x);
    r = fmaf(-n, ln2_lo, r);
    /* 1/k! for k = 7..2, rounded to float */
    float p = 1.98412698e-04f;            /* 1/5040 */
    p = fmaf(p, r, 1.38888889e-03f);      /* 1/720 */
    p = fmaf(p, r, 8.33333377e-03f);      /* 1/120 */
    p = fmaf(p, r, 4.16666679e-02f);      /* 1/24 */
    p = fmaf(p, r, 1.66666672e-01f);      /* 1/6 */
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;                      /* in [-126, 128] here */
    if (ni > 127) { p = p * 2.0f; ni -= 1; }
    uint32_t bits = (uint32_t)(ni + 127) << 23;
    float s; memcpy(&s, &bits, 4);
    return p * s;
}

/* src/SpeculativeDecoding.jl:20-30 with the random draw passed in; 1-based */
int or_sample_from_probs(const float *probs, int n, float r) {
    float cum = 0.f;
    for (int i = 0; i < n; i++) {
        cum += probs[i];
        if (r <= cum) return i + 1;
    }
    return n;
}

/* first maximal element, like Julia's argmax; 0-based */
int or_argmax(const float *row, int n) {
    int best = 0;
    for (int i = 1; i < n; i++) if (row[i] > row[best]) best = i;
    return best;
}

#define CH OR_ACCEPT_CHUNK
#define NL OR_ACCEPT_THREADS
#define PER (CH / NL)

static float butterfly_sum(float *v /* NL lanes, destroyed */) {
    float w[NL / 32];
    for (int wp = 0; wp < NL / 32; wp++) {
        float *x = v + 32 * wp;
        for (int off = 16; off >= 1; off >>= 1) {
            float y[32];
            for (int i = 0; i < 32; i++) y[i] = x[i] + x[i ^ off];
            memcpy(x, y, sizeof y);
        }
        w[wp] = x[0];
    }
    float s = w[0];
    for (int wp = 1; wp < NL / 32; wp++) s = s + w[wp];
    return s;
}

static inline float elem_e(float l, float m, float T) { return or_exp((l - m) / T); }

/* per chunk (max, canonical exp-sum) */
void or_chunk_stats(const float *row, int V, float T, float *cmax, float *csum) {
    int nch = (V + CH - 1) / CH;
    float lanes[NL];
    for (int c = 0; c < nch; c++) {
        int b = c * CH, e = b + CH < V ? b + CH : V;
        float m = -INFINITY;
        for (int i = b; i < e; i++) if (row[i] > m) m = row[i];
        for (int j = 0; j < NL; j++) {
            float t = 0.f;
            for (int q = 0; q < PER; q++) {
                int i = b + PER * j + q;
                if (i < e) t = t + elem_e(row[i], m, T);
            }
            lanes[j] = t;
        }
        cmax[c] = m;
        csum[c] = butterfly_sum(lanes);
    }
}

void or_row_stats(const float *cmax, const float *csum, int nch, float T,
                  float *rmax, float *rsum) {
    float M = -INFINITY;
    for (int c = 0; c < nch; c++) if (cmax[c] > M) M = cmax[c];
    float S = 0.f;
    for (int c = 0; c < nch; c++) S = S + csum[c] * or_exp((cmax[c] - M) / T);
    *rmax = M;
    *rsum = S;
}

typedef struct {
    int V, nch;
    float T, M, S;
    float *cmax, *csum;
} rowstat;

static void rowstat_init(rowstat *rs, const float *row, int V, float T) {
    rs->V = V; rs->T = T;
    rs->nch = (V + CH - 1) / CH;
    rs->cmax = (float *)malloc(sizeof(float) * rs->nch);
    rs->csum = (float *)malloc(sizeof(float) * rs->nch);
    or_chunk_stats(row, V, T, rs->cmax, rs->csum);
    or_row_stats(rs->cmax, rs->csum, rs->nch, T, &rs->M, &rs->S);
}
static void rowstat_free(rowstat *rs) { free(rs->cmax); free(rs->csum); }

static inline float rs_f(const rowstat *rs, int c) { return or_exp((rs->cmax[c] - rs->M) / rs->T); }

/* weight of element i: e_i * f_c */
static inline float rs_w(const rowstat *rs, const float *row, int i) {
    int c = i / CH;
    return elem_e(row[i], rs->cmax[c], rs->T) * rs_f(rs, c);
}

/* blocked in-chunk search: first element with tau' <= cumsum of vals */
static int chunk_search(const float *vals /* CH entries, 0 past the end */, int b, int e, float tau) {
    float lanes[NL];
    for (int j = 0; j < NL; j++) {
        float t = 0.f;
        for (int q = 0; q < PER; q++) { int i = b + PER * j + q; if (i < e) t = t + vals[i - b]; }
        lanes[j] = t;
    }
    float pre = 0.f;
    for (int j = 0; j < NL; j++) {
        float cum = pre;
        for (int q = 0; q < PER; q++) {
            int i = b + PER * j + q;
            if (i >= e) break;
            cum = cum + vals[i - b];
            if (tau <= cum) return i;
        }
        pre = pre + lanes[j];
    }
    for (int i = e - 1; i >= b; i--) if (vals[i - b] > 0.f) return i;
    return e - 1;
}

/* sample from the softmax of `row` with uniform u (0-based token) */
static int sample_row(const rowstat *rs, const float *row, float u) {
    float tau = u * rs->S, P = 0.f;
    int cs = -1;
    for (int c = 0; c < rs->nch; c++) {
        float nP = P + rs->csum[c] * rs_f(rs, c);
        if (tau <= nP) { cs = c; break; }
        P = nP;
    }
    if (cs < 0) {            /* tau beyond the total: last chunk with mass */
        for (int c = rs->nch - 1; c >= 0; c--) if (rs->csum[c] > 0.f) { cs = c; break; }
        if (cs < 0) cs = rs->nch - 1;
        P = 0.f;
        for (int c = 0; c < cs; c++) P = P + rs->csum[c] * rs_f(rs, c);
        tau = P + rs->csum[cs] * rs_f(rs, cs);
    }
    float fc = rs_f(rs, cs);
    float taup = (tau - P) / fc;
    int b = cs * CH, e = b + CH < rs->V ? b + CH : rs->V;
    float vals[CH];
    for (int i = b; i < e; i++) vals[i - b] = elem_e(row[i], rs->cmax[cs], rs->T);
    return chunk_search(vals, b, e, taup);
}

/* residual max(p_t - p_d, 0) sampling with uniform u; -1 if it has no mass */
static int sample_residual(const rowstat *ts, const float *trow, const rowstat *ds,
                           const float *drow, float u) {
    int V = ts->V, nch = ts->nch;
    float *rc = (float *)malloc(sizeof(float) * nch);
    float lanes[NL];
    for (int c = 0; c < nch; c++) {
        int b = c * CH, e = b + CH < V ? b + CH : V;
        for (int j = 0; j < NL; j++) {
            float t = 0.f;
            for (int q = 0; q < PER; q++) {
                int i = b + PER * j + q;
                if (i < e) {
                    float r = rs_w(ts, trow, i) / ts->S - rs_w(ds, drow, i) / ds->S;
                    t = t + (r > 0.f ? r : 0.f);
                }
            }
            lanes[j] = t;
        }
        rc[c] = butterfly_sum(lanes);
    }
    float R = 0.f;
    for (int c = 0; c < nch; c++) R = R + rc[c];
    if (!(R > 0.f)) { free(rc); return -1; }
    float tau = u * R, P = 0.f;
    int cs = -1;
    for (int c = 0; c < nch; c++) {
        float nP = P + rc[c];
        if (tau <= nP) { cs = c; break; }
        P = nP;
    }
    if (cs < 0) {
        for (int c = nch - 1; c >= 0; c--) if (rc[c] > 0.f) { cs = c; break; }
        P = 0.f;
        for (int c = 0; c < cs; c++) P = P + rc[c];
        tau = P + rc[cs];
    }
    float taup = tau - P;
    int b = cs * CH, e = b + CH < V ? b + CH : V;
    float vals[CH];
    for (int i = b; i < e; i++) {
        float r = rs_w(ts, trow, i) / ts->S - rs_w(ds, drow, i) / ds->S;
        vals[i - b] = r > 0.f ? r : 0.f;
    }
    free(rc);
    return chunk_search(vals, b, e, taup);
}

/*
 * target [batch][gamma+1][vocab], draft [batch][gamma][vocab];
 * draft_tokens [batch][gamma] or NULL (then drawn from p_d with u_d);
 * uniforms [batch][2*gamma+1] = u_d[gamma], u_a[gamma], u_rb.
 * accept_count [batch]; out_tokens [batch][gamma+1] (-1 past the emitted
 * ones); draft_out [batch][gamma] (may be NULL).
 */
int or_accept(const float *target, const float *draft, const int32_t *draft_tokens,
              const float *uniforms, int batch, int gamma, int vocab, float T,
              int32_t *accept_count, int32_t *out_tokens, int32_t *draft_out) {
    if (batch < 0 || gamma < 1 || gamma > 64 || vocab < 1 || !(T > 0.f)) return -1;
    for (int b = 0; b < batch; b++) {
        const float *tb = target + (int64_t)b * (gamma + 1) * vocab;
        const float *db = draft + (int64_t)b * gamma * vocab;
        const float *u = uniforms + (int64_t)b * (2 * gamma + 1);
        int32_t *ot = out_tokens + (int64_t)b * (gamma + 1);
        for (int i = 0; i <= gamma; i++) ot[i] = -1;
        int32_t x[64];
        rowstat ds[64];
        for (int i = 0; i < gamma; i++) {
            rowstat_init(&ds[i], db + (int64_t)i * vocab, vocab, T);
            x[i] = draft_tokens ? draft_tokens[(int64_t)b * gamma + i]
                                : sample_row(&ds[i], db + (int64_t)i * vocab, u[i]);
            if (draft_out) draft_out[(int64_t)b * gamma + i] = x[i];
        }
        int acc = 0, done = 0;
        for (int i = 0; i < gamma && !done; i++) {
            const float *trow = tb + (int64_t)i * vocab, *drow = db + (int64_t)i * vocab;
            rowstat ts;
            rowstat_init(&ts, trow, vocab, T);
            float pt = rs_w(&ts, trow, x[i]) / ts.S;
            float pd = rs_w(&ds[i], drow, x[i]) / ds[i].S;
            int ok = pd > 0.f ? (u[gamma + i] < pt / pd) : (pt > 0.f);
            if (ok) {
                ot[i] = x[i];
                acc++;
            } else {
                int y = sample_residual(&ts, trow, &ds[i], drow, u[2 * gamma]);
                if (y < 0) y = sample_row(&ts, trow, u[2 * gamma]);
                ot[i] = y;
                done = 1;
            }
            rowstat_free(&ts);
        }
        if (!done) {
            const float *trow = tb + (int64_t)gamma * vocab;
            rowstat ts;
            rowstat_init(&ts, trow, vocab, T);
            ot[gamma] = sample_row(&ts, trow, u[2 * gamma]);
            rowstat_free(&ts);
        }
        accept_count[b] = acc;
        for (int i = 0; i < gamma; i++) rowstat_free(&ds[i]);
    }
    return 0;
}

/* greedy verification (src/ModelCPU.jl:2099-2115 with the final norm applied
   upstream): accept while argmax(target[i]) == draft[i]; then emit the target
   argmax at the first mismatch, or the bonus argmax after gamma accepts */
int or_accept_greedy(const float *target, const int32_t *draft_tokens, int batch,
                     int gamma, int vocab, int32_t *accept_count, int32_t *out_tokens) {
    if (batch < 0 || gamma < 0 || vocab < 1) return -1;
    for (int b = 0; b < batch; b++) {
        const float *tb = target + (int64_t)b * (gamma + 1) * vocab;
        int32_t *ot = out_tokens + (int64_t)b * (gamma + 1);
        for (int i = 0; i <= gamma; i++) ot[i] = -1;
        int acc = 0;
        for (int i = 0; i <= gamma; i++) {
            int a = or_argmax(tb + (int64_t)i * vocab, vocab);
            ot[i] = a;
            if (i == gamma || a != draft_tokens[(int64_t)b * gamma + i]) break;
            acc++;
        }
        accept_count[b] = acc;
    }
    return 0;
}

/* ===================================================================== *
 * Filtered sampling: CommonOps.softmax_sample_scratch!
 * (src/CommonOps.jl:196-318) with a supplied uniform u in place of rand(),
 * and the presence / repetition penalties that precede it
 * (src/ModelCPU.jl:1202-1211,1237-1238; src/CommonOps.jl:63-76).
 * Shared with the device code (csrc/accept.cu, sample_kernel):
 *   validation (:145-160): NaN or +Inf anywhere -> -1 (the reference throws);
 *     M = max finite logit, g = its first index; every logit -Inf -> 0;
 *     T == 0 or V == 1 -> g (:207-210)
 *   top_k, 0 < k < V (:217-230): the k largest logits; ties at the k-th value
 *     go to the lower index (the reference's heap order leaves them open)
 *   e_i = or_exp((l_i - M) / T) for kept i, else 0 (:234-243).  The
 *     renormalisations (:244-247, :269-277, :292-298) scale every weight
 *     alike; they are folded into the sampling sum
 *   top_p < 1 (:249-278): weights as integers E_i = trunc(e_i * 2^30);
 *     target = (double)top_p * sum E; keep the first m elements in
 *     (e desc, index asc) order, m minimal with E_(1) + ... + E_(m) >= target
 *     (the reference's running cumsum, summed exactly)
 *   min_p > 0 (:280-299): keep e_i >= min_p (p >= max_p * min_p, max_p at e = 1)
 *   draw (:301-317): w_i = kept ? e_i : 0; chunk sums in the acceptance's
 *     canonical order; tau = u * W; first i with w_i > 0 and tau <= cumsum,
 *     else the last i with w_i > 0 (the reference's r <= cumsum alone would
 *     return a filtered-out first token when rand() gives exactly 0)
 * ===================================================================== */

static inline uint32_t f_key(float x) {     /* order-preserving key of a float */
    uint32_t u;
    memcpy(&u, &x, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
static inline uint64_t e_fixed(float e) { return (uint64_t)(e * 1073741824.0f); }

typedef struct { uint32_t key; int idx; } kidx;
static int kidx_desc(const void *a, const void *b) {
    const kidx *x = (const kidx *)a, *y = (const kidx *)b;
    if (x->key != y->key) return x->key > y->key ? -1 : 1;
    return x->idx - y->idx;
}

/* smallest n >= 1 with above + n * unit >= target (unit > 0) */
static uint64_t or_cut_count(uint64_t above, uint64_t unit, double target) {
    double q = ceil((target - (double)above) / (double)unit);
    uint64_t n = q < 1.0 ? 1 : (uint64_t)q;
    while (n > 1 && (double)(above + (n - 1) * unit) >= target) n--;
    while ((double)(above + n * unit) < target) n++;
    return n;
}

/* the filters' weights of one row: w_i = e_i = or_exp((l_i - M) / T) for the
   tokens top-k, top-p and min-p keep, else 0 (M = the row's max finite logit) */
static void filter_weights(const float *l, int V, float M, float T, int top_k, float top_p, float min_p,
                           float *w) {
    char *keep = (char *)malloc(V);
    kidx *ord = (kidx *)malloc(sizeof(kidx) * V);
    for (int i = 0; i < V; i++) keep[i] = 1;
    if (top_k > 0 && top_k < V) {
        for (int i = 0; i < V; i++) { ord[i].key = f_key(l[i]); ord[i].idx = i; }
        qsort(ord, V, sizeof(kidx), kidx_desc);
        for (int i = 0; i < V; i++) keep[i] = 0;
        for (int j = 0; j < top_k; j++) keep[ord[j].idx] = 1;
    }
    for (int i = 0; i < V; i++) w[i] = keep[i] ? or_exp((l[i] - M) / T) : 0.0f;
    if (top_p < 1.0f) {
        uint64_t S = 0;
        int n = 0;
        for (int i = 0; i < V; i++) {
            S += e_fixed(w[i]);
            if (keep[i]) { uint32_t k; memcpy(&k, &w[i], 4); ord[n].key = k; ord[n].idx = i; n++; }
        }
        const double target = (double)top_p * (double)S;
        qsort(ord, n, sizeof(kidx), kidx_desc);
        /* whole groups of equal e first, then the lowest indices of the
           group where the running sum reaches the target */
        uint64_t cum = 0;
        int j = 0, m = n;
        while (j < n) {
            int j2 = j;
            while (j2 < n && ord[j2].key == ord[j].key) j2++;
            float ev;
            memcpy(&ev, &ord[j].key, 4);
            const uint64_t unit = e_fixed(ev), grp = (uint64_t)(j2 - j) * unit;
            if ((double)(cum + grp) >= target) {
                uint64_t need = unit > 0 ? or_cut_count(cum, unit, target) : (uint64_t)(j2 - j);
                if (need > (uint64_t)(j2 - j)) need = (uint64_t)(j2 - j);
                m = j + (int)need;
                break;
            }
            cum += grp;
            j = j2;
        }
        for (int i = 0; i < V; i++) keep[i] = 0;
        for (int q = 0; q < m; q++) keep[ord[q].idx] = 1;
        for (int i = 0; i < V; i++) if (!keep[i]) w[i] = 0.0f;
    }
    if (min_p > 0.0f)
        for (int i = 0; i < V; i++) if (w[i] < min_p) w[i] = 0.0f;
    free(ord);
    free(keep);
}

int or_sample_filtered(const float *l, int V, float T, int top_k, float top_p, float min_p, float u) {
    if (V < 1) return -1;
    float M = -INFINITY;
    int g = 0, finite = 0;
    for (int i = 0; i < V; i++) {
        float x = l[i];
        if (isnan(x) || x == INFINITY) return -1;
        if (x != -INFINITY) {
            if (!finite || x > M) { M = x; g = i; }
            finite = 1;
        }
    }
    if (!finite) return 0;
    if (T == 0.0f || V == 1) return g;
    float *w = (float *)malloc(sizeof(float) * V);
    filter_weights(l, V, M, T, top_k, top_p, min_p, w);
    /* canonical chunked draw */
    const int nch = (V + CH - 1) / CH;
    float *cs = (float *)malloc(sizeof(float) * nch);
    float lanes[NL];
    for (int c = 0; c < nch; c++) {
        int b = c * CH, e = b + CH < V ? b + CH : V;
        for (int jn = 0; jn < NL; jn++) {
            float t = 0.f;
            for (int q = 0; q < PER; q++) { int i = b + PER * jn + q; if (i < e) t = t + w[i]; }
            lanes[jn] = t;
        }
        cs[c] = butterfly_sum(lanes);
    }
    float W = 0.f;
    for (int c = 0; c < nch; c++) W = W + cs[c];
    float tau = u * W, P = 0.f;
    int csel = -1;
    for (int c = 0; c < nch; c++) {
        float nP = P + cs[c];
        if (cs[c] > 0.f && tau <= nP) { csel = c; break; }
        P = nP;
    }
    if (csel < 0) {
        for (int c = nch - 1; c >= 0; c--) if (cs[c] > 0.f) { csel = c; break; }
        if (csel < 0) csel = nch - 1;
        P = 0.f;
        for (int c = 0; c < csel; c++) P = P + cs[c];
        tau = P + cs[csel];
    }
    int b = csel * CH, e = b + CH < V ? b + CH : V;
    /* blocked in-chunk search over positive weights */
    const float taup = tau - P;
    float pre = 0.f;
    int tok = -1;
    for (int jn = 0; jn < NL && tok < 0; jn++) {
        float cum = pre, t = 0.f;
        for (int q = 0; q < PER; q++) {
            int i = b + PER * jn + q;
            if (i >= e) break;
            t = t + w[i];
            cum = cum + w[i];
            if (w[i] > 0.f && taup <= cum) { tok = i; break; }
        }
        pre = pre + t;
    }
    if (tok < 0) {
        tok = e - 1;
        for (int i = e - 1; i >= b; i--) if (w[i] > 0.f) { tok = i; break; }
    }
    free(cs); free(w);
    return tok;
}

int or_sample_rows(const float *logits, int rows, int V, float T, int top_k, float top_p, float min_p,
                   const float *uniforms, int32_t *out) {
    for (int r = 0; r < rows; r++)
        out[r] = or_sample_filtered(logits + (int64_t)r * V, V, T, top_k, top_p, min_p, uniforms[r]);
    return 0;
}

/* presence then repetition penalty on every distinct seen token (0 <= t < V) */
void or_apply_penalties(float *logits, int rows, int V, const int32_t *seen, int n_seen, float presence,
                        float repetition) {
    char *mark = (char *)malloc(V > 0 ? V : 1);
    for (int r = 0; r < rows; r++) {
        float *l = logits + (int64_t)r * V;
        memset(mark, 0, V);
        for (int j = 0; j < n_seen; j++) {
            int t = seen[(int64_t)r * n_seen + j];
            if (t < 0 || t >= V || mark[t]) continue;
            mark[t] = 1;
            float x = l[t];
            if (presence != 0.0f) x = x - presence;
            if (repetition != 1.0f) x = x > 0.0f ? x / repetition : x * repetition;
            l[t] = x;
        }
    }
    free(mark);
}


/* ===================================================================== *
 * Filtered speculative acceptance: the verification of or_accept on the
 * distributions that the filters of or_sample_filtered leave (top-k, top-p,
 * min-p applied to every target and draft row with the same temperature).
 * The reference's speculate_and_verify (src/SpeculativeDecoding.jl:37-104)
 * filters only its draft draws and bonus token; filtering both distributions
 * keeps the emitted tokens distributed as the filtered target.  Per row: the
 * kept set K = {i : filter_weights(row)_i > 0}; chunk statistics as in
 * or_chunk_stats with the sums over K only (the chunk max over every
 * element); weights rs_w are 0 outside K; every draw (draft, residual, bonus)
 * takes the first i with a positive weight and tau <= cumsum.
 * TEST INFRASTRUCTURE: the restatement a device kernel is checked against.
 * ===================================================================== */

typedef struct {
    rowstat rs;
    char *keep;
} mrow;

static void mrow_init(mrow *m, const float *row, int V, float T, int top_k, float top_p, float min_p) {
    float M = -INFINITY;
    for (int i = 0; i < V; i++) if (row[i] > M) M = row[i];
    float *w = (float *)malloc(sizeof(float) * V);
    filter_weights(row, V, M, T, top_k, top_p, min_p, w);
    m->keep = (char *)malloc(V);
    for (int i = 0; i < V; i++) m->keep[i] = w[i] > 0.f;
    free(w);
    rowstat *rs = &m->rs;
    rs->V = V; rs->T = T;
    rs->nch = (V + CH - 1) / CH;
    rs->cmax = (float *)malloc(sizeof(float) * rs->nch);
    rs->csum = (float *)malloc(sizeof(float) * rs->nch);
    float lanes[NL];
    for (int c = 0; c < rs->nch; c++) {
        int b = c * CH, e = b + CH < V ? b + CH : V;
        float mc = -INFINITY;
        for (int i = b; i < e; i++) if (row[i] > mc) mc = row[i];
        for (int j = 0; j < NL; j++) {
            float t = 0.f;
            for (int q = 0; q < PER; q++) {
                int i = b + PER * j + q;
                if (i < e && m->keep[i]) t = t + elem_e(row[i], mc, T);
            }
            lanes[j] = t;
        }
        rs->cmax[c] = mc;
        rs->csum[c] = butterfly_sum(lanes);
    }
    or_row_stats(rs->cmax, rs->csum, rs->nch, T, &rs->M, &rs->S);
}
static void mrow_free(mrow *m) { rowstat_free(&m->rs); free(m->keep); }
static inline float mrow_w(const mrow *m, const float *row, int i) {
    return m->keep[i] ? rs_w(&m->rs, row, i) : 0.0f;
}

/* first element with a positive value and tau <= cumsum (blocked order), else
   the last positive one, else the last element */
static int chunk_search_pos(const float *vals, int b, int e, float tau) {
    float pre = 0.f;
    for (int j = 0; j < NL; j++) {
        float cum = pre, t = 0.f;
        for (int q = 0; q < PER; q++) {
            int i = b + PER * j + q;
            if (i >= e) break;
            t = t + vals[i - b];
            cum = cum + vals[i - b];
            if (vals[i - b] > 0.f && tau <= cum) return i;
        }
        pre = pre + t;
    }
    for (int i = e - 1; i >= b; i--) if (vals[i - b] > 0.f) return i;
    return e - 1;
}

/* draw from per-chunk masses cm[c] (and element values by vfun) with u */
typedef float (*vfun)(const void *ctx, int i);
static int draw_chunked(const float *cm, int nch, int V, float total, float u, vfun f, const void *ctx) {
    float tau = u * total, P = 0.f;
    int cs = -1;
    for (int c = 0; c < nch; c++) {
        float nP = P + cm[c];
        if (cm[c] > 0.f && tau <= nP) { cs = c; break; }
        P = nP;
    }
    if (cs < 0) {
        for (int c = nch - 1; c >= 0; c--) if (cm[c] > 0.f) { cs = c; break; }
        if (cs < 0) cs = nch - 1;
        P = 0.f;
        for (int c = 0; c < cs; c++) P = P + cm[c];
        tau = P + cm[cs];
    }
    int b = cs * CH, e = b + CH < V ? b + CH : V;
    float vals[CH];
    for (int i = b; i < e; i++) vals[i - b] = f(ctx, i);
    return chunk_search_pos(vals, b, e, tau - P);
}

typedef struct { const mrow *m; const float *row; int c; } mctx;
static float m_elem(const void *x, int i) {   /* element weight inside chunk c, relative to its max */
    const mctx *k = (const mctx *)x;
    return k->m->keep[i] ? elem_e(k->row[i], k->m->rs.cmax[k->c], k->m->rs.T) : 0.0f;
}

static int sample_mrow(const mrow *m, const float *row, float u) {
    const rowstat *rs = &m->rs;
    float *cm = (float *)malloc(sizeof(float) * rs->nch);
    for (int c = 0; c < rs->nch; c++) cm[c] = rs->csum[c] * rs_f(rs, c);
    /* chunk choice on the row-scaled masses, then the element search on the
       chunk's own weights with tau rescaled by the chunk factor */
    float tau = u * rs->S, P = 0.f;
    int cs = -1;
    for (int c = 0; c < rs->nch; c++) {
        float nP = P + cm[c];
        if (cm[c] > 0.f && tau <= nP) { cs = c; break; }
        P = nP;
    }
    if (cs < 0) {
        for (int c = rs->nch - 1; c >= 0; c--) if (cm[c] > 0.f) { cs = c; break; }
        if (cs < 0) cs = rs->nch - 1;
        P = 0.f;
        for (int c = 0; c < cs; c++) P = P + cm[c];
        tau = P + cm[cs];
    }
    float taup = (tau - P) / rs_f(rs, cs);
    int b = cs * CH, e = b + CH < rs->V ? b + CH : rs->V;
    float vals[CH];
    mctx k = {m, row, cs};
    for (int i = b; i < e; i++) vals[i - b] = m_elem(&k, i);
    free(cm);
    return chunk_search_pos(vals, b, e, taup);
}

typedef struct { const mrow *t; const float *trow; const mrow *d; const float *drow; } rctx;
static float r_elem(const void *x, int i) {
    const rctx *k = (const rctx *)x;
    float r = mrow_w(k->t, k->trow, i) / k->t->rs.S - mrow_w(k->d, k->drow, i) / k->d->rs.S;
    return r > 0.f ? r : 0.f;
}

static int sample_mresidual(const mrow *t, const float *trow, const mrow *d, const float *drow, float u) {
    int V = t->rs.V, nch = t->rs.nch;
    float *rc = (float *)malloc(sizeof(float) * nch);
    float lanes[NL];
    rctx k = {t, trow, d, drow};
    for (int c = 0; c < nch; c++) {
        int b = c * CH, e = b + CH < V ? b + CH : V;
        for (int j = 0; j < NL; j++) {
            float s2 = 0.f;
            for (int q = 0; q < PER; q++) { int i = b + PER * j + q; if (i < e) s2 = s2 + r_elem(&k, i); }
            lanes[j] = s2;
        }
        rc[c] = butterfly_sum(lanes);
    }
    float R = 0.f;
    for (int c = 0; c < nch; c++) R = R + rc[c];
    int y = R > 0.f ? draw_chunked(rc, nch, V, R, u, r_elem, &k) : -1;
    free(rc);
    return y;
}

int or_accept_filtered(const float *target, const float *draft, const float *uniforms, int batch, int gamma,
                       int vocab, float T, int top_k, float top_p, float min_p, int32_t *accept_count,
                       int32_t *out_tokens, int32_t *draft_out) {
    if (batch < 0 || gamma < 1 || gamma > 64 || vocab < 1 || !(T > 0.f)) return -1;
    for (int b = 0; b < batch; b++) {
        const float *tb = target + (int64_t)b * (gamma + 1) * vocab;
        const float *db = draft + (int64_t)b * gamma * vocab;
        const float *u = uniforms + (int64_t)b * (2 * gamma + 1);
        int32_t *ot = out_tokens + (int64_t)b * (gamma + 1);
        for (int i = 0; i <= gamma; i++) ot[i] = -1;
        int32_t x[64];
        mrow ds[64];
        for (int i = 0; i < gamma; i++) {
            mrow_init(&ds[i], db + (int64_t)i * vocab, vocab, T, top_k, top_p, min_p);
            x[i] = sample_mrow(&ds[i], db + (int64_t)i * vocab, u[i]);
            if (draft_out) draft_out[(int64_t)b * gamma + i] = x[i];
        }
        int acc = 0, done = 0;
        for (int i = 0; i < gamma && !done; i++) {
            const float *trow = tb + (int64_t)i * vocab, *drow = db + (int64_t)i * vocab;
            mrow ts;
            mrow_init(&ts, trow, vocab, T, top_k, top_p, min_p);
            float pt = mrow_w(&ts, trow, x[i]) / ts.rs.S;
            float pd = mrow_w(&ds[i], drow, x[i]) / ds[i].rs.S;
            int ok = pd > 0.f ? (u[gamma + i] < pt / pd) : (pt > 0.f);
            if (ok) {
                ot[i] = x[i];
                acc++;
            } else {
                int y = sample_mresidual(&ts, trow, &ds[i], drow, u[2 * gamma]);
                if (y < 0) y = sample_mrow(&ts, trow, u[2 * gamma]);
                ot[i] = y;
                done = 1;
            }
            mrow_free(&ts);
        }
        if (!done) {
            const float *trow = tb + (int64_t)gamma * vocab;
            mrow ts;
            mrow_init(&ts, trow, vocab, T, top_k, top_p, min_p);
            ot[gamma] = sample_mrow(&ts, trow, u[2 * gamma]);
            mrow_free(&ts);
        }
        accept_count[b] = acc;
        for (int i = 0; i < gamma; i++) mrow_free(&ds[i]);
    }
    return 0;
}
