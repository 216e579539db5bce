// Small-N quantized GEMM ("verify GEMV"): Y[n][r] = sum_k W[r][k] X[n][k]
// for N <= 8 verify columns, W in Q4_K / Q5_K / Q6_K / Q8_0.
//
// Replaces q4_k_gemv .. q8_0_gemv (reference src/kernels/quant_kernels.c:602-697),
// which the reference calls once per token; here the N tokens of one verify
// step share a single pass over the weights.
//
// Arithmetic (exact up to f32 accumulation):
//   * weights are unpacked in registers to fp16 *integers* (magic-number
//     trick, no conversions) and, for Q4_K/Q5_K, multiplied by their 6-bit
//     sub-block scale with one fp16 FMA - the product sc*q <= 63*31 < 2048 is
//     exact in fp16;
//   * each f32 activation is scaled by a power of two per 256-element unit
//     and split exactly into hi + lo fp16 halves, which become two B columns;
//   * mma.sync m16n8k16 (fp16 x fp16 -> f32) forms sum_k A*B over a unit;
//     the super-block scales d / dmin and the unit's power of two are applied
//     to the f32 accumulators; the Q4_K/Q5_K "min" term is one more m16n8k8
//     against per-sub-block activation sums.
// The MMA k-order is a permutation of the elements chosen so that each lane's
// loaded bytes feed its A fragment directly; pack_x writes B in the same order.
//
// Work split: 16-row tiles; the 8 warps of a CTA split the K units of WR
// tiles (WR x WK = 8) and reduce through shared memory.
#include "common.cuh"

namespace ifr {

constexpr int kThreads = 256;

// ---- MMA k-slot -> element index inside a 256-element chunk ----------------
// slot 0..3 = kcol 2t, 2t+1, 2t+8, 2t+9 of the lane quad t = lane % 4.
__host__ __device__ inline int elem_qk(int s, int t, int slot) {  // Q4_K / Q5_K
    int c = s >> 3, w = (s >> 1) & 3, h = s & 1, p = t >> 1;
    int j4 = 2 * c + p;
    int l = 16 * (t & 1) + 4 * w + h + ((slot & 1) ? 2 : 0);
    return 64 * j4 + ((slot & 2) ? 32 : 0) + l;
}
// sub-block fed to k-row (2t + kr) of the Q4_K/Q5_K min MMA
__host__ __device__ inline int minsub_qk(int t, int kr) {
    int p = t >> 1;
    return (t & 1) ? (4 + 2 * p + kr) : (2 * p + kr);
}
__host__ __device__ inline int jmap(int slot) { return slot == 0 ? 0 : slot == 1 ? 2 : slot == 2 ? 1 : 3; }
__host__ __device__ inline int elem_q6k(int s, int t, int slot) {
    int n = s >> 3, qq = (s >> 1) & 3, b = s & 1;
    return 128 * n + 32 * qq + 16 * b + 4 * t + jmap(slot);
}
__host__ __device__ inline int elem_q80(int s, int t, int slot) {  // s = step in the chunk
    return 32 * (s >> 1) + 8 * t + 4 * (s & 1) + jmap(slot);
}

// ---- scratch layout -----------------------------------------------------------
struct XPack {
    uint4 *xp;     // [chunk][8 step pairs][NT][32 lanes]  (B fragments, 2 steps each)
    uint32_t *xm;  // [chunk][NT][32 lanes]                (min-MMA B fragment)
    float *es;     // [unit][8 cols]                        (2^-e of each unit)
};

static inline int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }

int64_t qgemm_scratch_bytes(int type, int64_t cols) {
    int64_t nch = (cols + 255) / 256;
    int64_t nunits = type == 8 ? (cols + 31) / 32 : nch;
    return align256(nch * 8 * 2 * 32 * 16) + align256(nch * 2 * 32 * 4) + align256(nunits * 8 * 4);
}

static XPack carve(void *scratch, int type, int64_t cols) {
    int64_t nch = (cols + 255) / 256;
    char *p = (char *)scratch;
    XPack x;
    x.xp = (uint4 *)p;
    p += align256(nch * 8 * 2 * 32 * 16);
    x.xm = (uint32_t *)p;
    p += align256(nch * 2 * 32 * 4);
    x.es = (float *)p;
    (void)type;
    return x;
}

IFR_DEV uint32_t pack_h2(__half lo, __half hi) {
    return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
}

// 2^k for integer k in [-126, 127]
IFR_DEV float pow2i(int k) { return __int_as_float((k + 127) << 23); }

// scale exponent so that max|x| * 2^e < 2^14 (fp16-safe with headroom)
IFR_DEV int unit_exp(float m) {
    if (!(m > 0.f) || isinf(m)) return 0;
    int ex;
    frexpf(m, &ex);  // m = f * 2^ex, f in [0.5, 1)
    int e = 14 - ex;
    return e < -100 ? -100 : (e > 100 ? 100 : e);
}

// One CTA per 256-element chunk of K.  FMT: 12/13 (K-quants with mins), 14, 8.
template <int FMT>
__global__ void __launch_bounds__(kThreads) pack_x_kernel(const float *__restrict__ X, int ncols,
                                                          int64_t K, int NT, XPack P) {
    __shared__ __half xh[8][256], xl[8][256];
    __shared__ float sc_s[8][8];  // [unit in chunk][col] scale 2^e
    __shared__ float xsum[8][8];  // [col][sub-block] scaled sums (K-quants)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t chunk = blockIdx.x;
    const int64_t base = chunk * 256;
    const int64_t k = base + tid;
    float v[8];
#pragma unroll
    for (int c = 0; c < 8; c++) v[c] = (c < ncols && k < K) ? X[(int64_t)c * K + k] : 0.f;

    // unit maxima -> power-of-two scales
    if (FMT == 8) {
        // unit = 32 elements = one warp
#pragma unroll
        for (int c = 0; c < 8; c++) {
            float m = fabsf(v[c]);
            for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) sc_s[warp][c] = pow2i(unit_exp(m));
        }
    } else {
        __shared__ float wmax[8][8];
#pragma unroll
        for (int c = 0; c < 8; c++) {
            float m = fabsf(v[c]);
            for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            if (lane == 0) wmax[warp][c] = m;
        }
        __syncthreads();
        if (tid < 8) {
            float m = 0.f;
            for (int w = 0; w < 8; w++) m = fmaxf(m, wmax[w][tid]);
            sc_s[0][tid] = pow2i(unit_exp(m));
        }
    }
    __syncthreads();
    const int unit_in_chunk = (FMT == 8) ? warp : 0;
#pragma unroll
    for (int c = 0; c < 8; c++) {
        float sv = v[c] * sc_s[unit_in_chunk][c];  // exact (power of two)
        __half h = __float2half_rn(sv);
        __half l = __float2half_rn(sv - __half2float(h));
        xh[c][tid] = h;
        xl[c][tid] = l;
        v[c] = sv;
    }
    // unit scales out: es = 2^-e
    if (FMT == 8) {
        if (lane < 8) {
            int64_t unit = chunk * 8 + warp;
            if (unit * 32 < K) P.es[unit * 8 + lane] = 1.0f / sc_s[warp][lane];
        }
    } else {
        if (tid < 8) P.es[chunk * 8 + tid] = 1.0f / sc_s[0][tid];
        // per-sub-block sums of the scaled values, x 2^-5 for fp16 range
        // thread layout: col = warp, sub-block = lane/4, quarter = lane%4
        {
            int c = warp, j = lane >> 2, q = lane & 3;
            float s = 0.f;
            for (int e = 0; e < 8; e++) s += __half2float(xh[c][32 * j + 8 * q + e]) +
                                            __half2float(xl[c][32 * j + 8 * q + e]);
            s += __shfl_xor_sync(0xffffffffu, s, 1);
            s += __shfl_xor_sync(0xffffffffu, s, 2);
            if (q == 0) xsum[c][j] = s * 0.03125f;
        }
    }
    __syncthreads();

    // B fragments: item = (step pair sp, lane) ; 8 x 32 = 256 items per nt
    {
        const int sp = tid >> 5, g = lane >> 2, t = lane & 3;
        for (int nt = 0; nt < NT; nt++) {
            const int col = 4 * nt + (g >> 1), part = g & 1;
            uint32_t r[4];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int s = 2 * sp + h;
                __half e4[4];
#pragma unroll
                for (int slot = 0; slot < 4; slot++) {
                    int e = (FMT == 14) ? elem_q6k(s, t, slot)
                          : (FMT == 8)  ? elem_q80(s, t, slot)
                                        : elem_qk(s, t, slot);
                    e4[slot] = part ? xl[col][e] : xh[col][e];
                }
                r[2 * h] = pack_h2(e4[0], e4[1]);
                r[2 * h + 1] = pack_h2(e4[2], e4[3]);
            }
            P.xp[((chunk * 8 + sp) * NT + nt) * 32 + lane] = make_uint4(r[0], r[1], r[2], r[3]);
        }
    }
    if (FMT == 12 || FMT == 13) {
        if (tid < 32 * NT) {
            const int nt = tid >> 5, g = lane >> 2, t = lane & 3;
            const int col = 4 * nt + (g >> 1), part = g & 1;
            __half hv[2];
#pragma unroll
            for (int kr = 0; kr < 2; kr++) {
                float s = xsum[col][minsub_qk(t, kr)];
                __half h = __float2half_rn(s);
                hv[kr] = part ? __float2half_rn(s - __half2float(h)) : h;
            }
            P.xm[(chunk * NT + nt) * 32 + lane] = pack_h2(hv[0], hv[1]);
        }
    }
}

// ---- fp16 constants from a byte ---------------------------------------------
// (v, v) as f16x2 for an integer byte v < 1024
IFR_DEV uint32_t bcast_byte_h2(uint32_t word, int byte) {
    // place the byte in the low byte of both halves, add the 1024 magic, subtract it
    uint32_t sel = (uint32_t)byte | (4u << 4) | ((uint32_t)byte << 8) | (4u << 12);
    uint32_t x = __byte_perm(word, 0u, sel) | 0x64006400u;
    return hsub2_u(x, 0x64006400u);
}
// (b0, b1) as f16x2 from the two low bytes of `word`
IFR_DEV uint32_t bytes01_h2(uint32_t word) {
    uint32_t x = __byte_perm(word, 0u, 0x4140u) | 0x64006400u;
    return hsub2_u(x, 0x64006400u);
}

constexpr uint32_t kNegH1024 = 0xE400E400u;  // (-1024, -1024)
constexpr uint32_t kH1_16 = 0x2C002C00u;     // (1/16, 1/16)
constexpr uint32_t kNegH64 = 0xD400D400u;    // (-64, -64)

// Per row of a Q4_K/Q5_K super-block, everything lane (g,t) needs.
struct QKRow {
    uint32_t klo[2], nlo[2], khi[2], nhi[2];  // per chunk c: low-nibble and high-nibble FMA constants
    uint32_t mA;                              // min-MMA A fragment (2 mins)
    float d, dm32;
};

IFR_DEV void qk_row_consts(const uint4 &h, int t, QKRow &R) {
    const int p = t >> 1;
    const uint32_t A = h.y >> (16 * p), B = h.z >> (16 * p), C = h.w >> (16 * p);
    const uint32_t sc_a = A & 0x3F3Fu;
    const uint32_t m_a = B & 0x3F3Fu;
    const uint32_t sc_b = (C & 0x0F0Fu) | ((A >> 2) & 0x3030u);
    const uint32_t m_b = ((C >> 4) & 0x0F0Fu) | ((B >> 2) & 0x3030u);
#pragma unroll
    for (int c = 0; c < 2; c++) {
        const uint32_t scw = c ? sc_b : sc_a;
        const uint32_t s_lo = bcast_byte_h2(scw, 0), s_hi = bcast_byte_h2(scw, 1);
        R.klo[c] = s_lo;
        R.nlo[c] = hmul2_u(s_lo, kNegH1024);
        R.khi[c] = hmul2_u(s_hi, kH1_16);
        R.nhi[c] = hmul2_u(s_hi, kNegH64);
    }
    R.mA = bytes01_h2((t & 1) ? m_b : m_a);
    R.d = h2f((uint16_t)(h.x & 0xffffu));
    R.dm32 = h2f((uint16_t)(h.x >> 16)) * 32.0f;
}

IFR_DEV uint32_t u4w(const uint4 &v, int w) { return w == 0 ? v.x : w == 1 ? v.y : w == 2 ? v.z : v.w; }

// Q4_K / Q5_K kernel.  W raw blocks; nb super-blocks per row.
template <bool Q5, int NT>
__global__ void __launch_bounds__(kThreads) qgemv_qk_kernel(const uint8_t *__restrict__ W, int64_t M,
                                                            int nb, XPack P, float *__restrict__ Y,
                                                            int ncols, int WK) {
    constexpr int BLK = Q5 ? 176 : 144;
    constexpr int QS = Q5 ? 48 : 16;
    __shared__ float red[8][NT * 4][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int WR = 8 / WK, wr = warp / WK, wk = warp % WK;
    const int64_t nrb = (M + 15) / 16;
    const int64_t rowbytes = (int64_t)nb * BLK;

    for (int64_t rb0 = (int64_t)blockIdx.x * WR; rb0 < nrb; rb0 += (int64_t)gridDim.x * WR) {
        const int64_t rb = rb0 + wr;
        float tot[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) tot[nt][i] = 0.f;
        if (rb < nrb) {
            const int64_t r0 = rb * 16 + g, r1 = r0 + 8;
            const uint8_t *w0 = W + (r0 < M ? r0 : M - 1) * rowbytes;
            const uint8_t *w1 = W + (r1 < M ? r1 : M - 1) * rowbytes;
            for (int u = wk; u < nb; u += WK) {
                const uint8_t *b0 = w0 + (int64_t)u * BLK, *b1 = w1 + (int64_t)u * BLK;
                const uint4 h0 = ldg_nc4(b0), h1 = ldg_nc4(b1);
                uint4 q0[2], q1[2], qh0, qh1;
                q0[0] = ldg_nc4(b0 + QS + 16 * t);
                q0[1] = ldg_nc4(b0 + QS + 64 + 16 * t);
                q1[0] = ldg_nc4(b1 + QS + 16 * t);
                q1[1] = ldg_nc4(b1 + QS + 64 + 16 * t);
                if (Q5) {
                    qh0 = ldg_nc4(b0 + 16 + 16 * (t & 1));
                    qh1 = ldg_nc4(b1 + 16 + 16 * (t & 1));
                }
                const uint4 *xpu = P.xp + (int64_t)u * 8 * NT * 32 + lane;
                uint32_t xmv[NT];
                float esv[NT];
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    xmv[nt] = P.xm[((int64_t)u * NT + nt) * 32 + lane];
                    esv[nt] = P.es[(int64_t)u * 8 + 4 * nt + t];
                }
                QKRow R0, R1;
                qk_row_consts(h0, t, R0);
                qk_row_consts(h1, t, R1);

                float csc[NT][4], cm[NT][4];
#pragma unroll
                for (int nt = 0; nt < NT; nt++)
#pragma unroll
                    for (int i = 0; i < 4; i++) csc[nt][i] = cm[nt][i] = 0.f;

#pragma unroll
                for (int c = 0; c < 2; c++) {
                    const int j4 = 2 * c + (t >> 1);
#pragma unroll
                    for (int w = 0; w < 4; w++) {
                        const uint32_t W0 = u4w(q0[c], w), W1 = u4w(q1[c], w);
                        uint4 bb[NT];
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) bb[nt] = xpu[(4 * c + w) * NT * 32 + nt * 32];
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const uint32_t s0 = h ? (W0 >> 8) : W0, s1 = h ? (W1 >> 8) : W1;
                            uint32_t lo0 = lop_and_or(s0, 0x000F000Fu, 0x64006400u);
                            uint32_t hi0 = lop_and_or(s0, 0x00F000F0u, 0x64006400u);
                            uint32_t lo1 = lop_and_or(s1, 0x000F000Fu, 0x64006400u);
                            uint32_t hi1 = lop_and_or(s1, 0x00F000F0u, 0x64006400u);
                            if (Q5) {
                                // fifth bit: qh[l] bit 2*j4 (low nibble) / 2*j4+1 (high nibble)
                                const uint32_t H0 = (u4w(qh0, w) >> (8 * h + 2 * j4));
                                const uint32_t H1 = (u4w(qh1, w) >> (8 * h + 2 * j4));
                                lo0 |= (H0 << 4) & 0x00100010u;
                                hi0 |= (H0 << 7) & 0x01000100u;
                                lo1 |= (H1 << 4) & 0x00100010u;
                                hi1 |= (H1 << 7) & 0x01000100u;
                            }
                            const uint32_t a0 = hfma2_u(lo0, R0.klo[c], R0.nlo[c]);
                            const uint32_t a1 = hfma2_u(lo1, R1.klo[c], R1.nlo[c]);
                            const uint32_t a2 = hfma2_u(hi0, R0.khi[c], R0.nhi[c]);
                            const uint32_t a3 = hfma2_u(hi1, R1.khi[c], R1.nhi[c]);
#pragma unroll
                            for (int nt = 0; nt < NT; nt++) {
                                const uint32_t bx = h ? bb[nt].z : bb[nt].x;
                                const uint32_t by = h ? bb[nt].w : bb[nt].y;
                                mma16816(csc[nt], a0, a1, a2, a3, bx, by);
                            }
                        }
                    }
                }
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    mma1688(cm[nt], R0.mA, R1.mA, xmv[nt]);
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float d = (i < 2) ? R0.d : R1.d, dm = (i < 2) ? R0.dm32 : R1.dm32;
                        tot[nt][i] = fmaf(esv[nt], d * csc[nt][i] - dm * cm[nt][i], tot[nt][i]);
                    }
                }
            }
        }
        if (WK > 1) {
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int i = 0; i < 4; i++) red[warp][nt * 4 + i][lane] = tot[nt][i];
            __syncthreads();
            if (wk == 0 && rb < nrb) {
                for (int q = 1; q < WK; q++)
#pragma unroll
                    for (int nt = 0; nt < NT; nt++)
#pragma unroll
                        for (int i = 0; i < 4; i++) tot[nt][i] += red[warp + q][nt * 4 + i][lane];
            }
            __syncthreads();
        }
        if (wk == 0 && rb < nrb) {
            const int64_t r0 = rb * 16 + g, r1 = r0 + 8;
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const int col = 4 * nt + t;
                if (col < ncols) {
                    if (r0 < M) Y[(int64_t)col * M + r0] = tot[nt][0] + tot[nt][1];
                    if (r1 < M) Y[(int64_t)col * M + r1] = tot[nt][2] + tot[nt][3];
                }
            }
        }
    }
}

// Q6_K kernel (planar, lane-permuted layout; see QTensor)
template <int NT>
__global__ void __launch_bounds__(kThreads) qgemv_q6k_kernel(const uint8_t *__restrict__ QL,
                                                             const uint8_t *__restrict__ QH,
                                                             const int8_t *__restrict__ SC,
                                                             const uint16_t *__restrict__ DD,
                                                             int64_t M, int nb, XPack P,
                                                             float *__restrict__ Y, int ncols, int WK) {
    __shared__ float red[8][NT * 4][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int WR = 8 / WK, wr = warp / WK, wk = warp % WK;
    const int64_t nrb = (M + 15) / 16;

    for (int64_t rb0 = (int64_t)blockIdx.x * WR; rb0 < nrb; rb0 += (int64_t)gridDim.x * WR) {
        const int64_t rb = rb0 + wr;
        float tot[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) tot[nt][i] = 0.f;
        if (rb < nrb) {
            const int64_t r0 = rb * 16 + g, r1 = r0 + 8;
            const int64_t i0 = (r0 < M ? r0 : M - 1) * nb, i1 = (r1 < M ? r1 : M - 1) * nb;
            for (int u = wk; u < nb; u += WK) {
                const int64_t blk0 = i0 + u, blk1 = i1 + u;
                uint4 l0[2], l1[2];
                l0[0] = ldg_nc4(QL + blk0 * 128 + 32 * t);
                l0[1] = ldg_nc4(QL + blk0 * 128 + 32 * t + 16);
                l1[0] = ldg_nc4(QL + blk1 * 128 + 32 * t);
                l1[1] = ldg_nc4(QL + blk1 * 128 + 32 * t + 16);
                const uint4 hq0 = ldg_nc4(QH + blk0 * 64 + 16 * t);
                const uint4 hq1 = ldg_nc4(QH + blk1 * 64 + 16 * t);
                const uint4 sc0 = ldg_nc4(SC + blk0 * 16), sc1 = ldg_nc4(SC + blk1 * 16);
                const float d0 = h2f(__ldg(DD + blk0)), d1 = h2f(__ldg(DD + blk1));
                const uint4 *xpu = P.xp + (int64_t)u * 8 * NT * 32 + lane;
                float esv[NT];
#pragma unroll
                for (int nt = 0; nt < NT; nt++) esv[nt] = P.es[(int64_t)u * 8 + 4 * nt + t];
                float acc[NT][4];
#pragma unroll
                for (int nt = 0; nt < NT; nt++)
#pragma unroll
                    for (int i = 0; i < 4; i++) acc[nt][i] = 0.f;
#pragma unroll
                for (int s = 0; s < 16; s++) {
                    const int n = s >> 3, qq = (s >> 1) & 3, b = s & 1;
                    const int kw = 4 * n + 2 * (qq & 1) + b;  // ql word (of 8)
                    const int kh = 2 * n + b;                 // qh word (of 4)
                    const uint32_t WA0 = u4w(l0[kw >> 2], kw & 3), WA1 = u4w(l1[kw >> 2], kw & 3);
                    const uint32_t H0 = u4w(hq0, kh), H1 = u4w(hq1, kh);
                    const int ns = (qq >= 2) ? 4 : 0;      // nibble shift
                    const int hs = 2 * qq;                  // qh bit shift
                    // bytes 0,2 -> kcols 2t,2t+1 ; bytes 1,3 -> kcols 2t+8,2t+9
                    uint32_t x02_0 = ((WA0 >> ns) & 0x000F000Fu) | (((H0 >> hs) << 4) & 0x00300030u);
                    uint32_t x13_0 = ((WA0 >> (ns + 8)) & 0x000F000Fu) | (((H0 >> (hs + 8)) << 4) & 0x00300030u);
                    uint32_t x02_1 = ((WA1 >> ns) & 0x000F000Fu) | (((H1 >> hs) << 4) & 0x00300030u);
                    uint32_t x13_1 = ((WA1 >> (ns + 8)) & 0x000F000Fu) | (((H1 >> (hs + 8)) << 4) & 0x00300030u);
                    const uint32_t a0 = hsub2_u(x02_0 | 0x64006400u, 0x64206420u);
                    const uint32_t a1 = hsub2_u(x02_1 | 0x64006400u, 0x64206420u);
                    const uint32_t a2 = hsub2_u(x13_0 | 0x64006400u, 0x64206420u);
                    const uint32_t a3 = hsub2_u(x13_1 | 0x64006400u, 0x64206420u);
                    const float f0 = (float)(int8_t)(u4w(sc0, s >> 2) >> (8 * (s & 3)));
                    const float f1 = (float)(int8_t)(u4w(sc1, s >> 2) >> (8 * (s & 3)));
#pragma unroll
                    for (int nt = 0; nt < NT; nt++) {
                        const uint4 bb = xpu[(s >> 1) * NT * 32 + nt * 32];
                        const uint32_t bx = (s & 1) ? bb.z : bb.x, by = (s & 1) ? bb.w : bb.y;
                        float c[4] = {0.f, 0.f, 0.f, 0.f};
                        mma16816(c, a0, a1, a2, a3, bx, by);
                        acc[nt][0] = fmaf(f0, c[0], acc[nt][0]);
                        acc[nt][1] = fmaf(f0, c[1], acc[nt][1]);
                        acc[nt][2] = fmaf(f1, c[2], acc[nt][2]);
                        acc[nt][3] = fmaf(f1, c[3], acc[nt][3]);
                    }
                }
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    tot[nt][0] = fmaf(esv[nt] * d0, acc[nt][0], tot[nt][0]);
                    tot[nt][1] = fmaf(esv[nt] * d0, acc[nt][1], tot[nt][1]);
                    tot[nt][2] = fmaf(esv[nt] * d1, acc[nt][2], tot[nt][2]);
                    tot[nt][3] = fmaf(esv[nt] * d1, acc[nt][3], tot[nt][3]);
                }
            }
        }
        if (WK > 1) {
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int i = 0; i < 4; i++) red[warp][nt * 4 + i][lane] = tot[nt][i];
            __syncthreads();
            if (wk == 0 && rb < nrb) {
                for (int q = 1; q < WK; q++)
#pragma unroll
                    for (int nt = 0; nt < NT; nt++)
#pragma unroll
                        for (int i = 0; i < 4; i++) tot[nt][i] += red[warp + q][nt * 4 + i][lane];
            }
            __syncthreads();
        }
        if (wk == 0 && rb < nrb) {
            const int64_t r0 = rb * 16 + g, r1 = r0 + 8;
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const int col = 4 * nt + t;
                if (col < ncols) {
                    if (r0 < M) Y[(int64_t)col * M + r0] = tot[nt][0] + tot[nt][1];
                    if (r1 < M) Y[(int64_t)col * M + r1] = tot[nt][2] + tot[nt][3];
                }
            }
        }
    }
}

// Q8_0 kernel (planar).  Iterates 256-element chunks (8 blocks) of K; a tail
// chunk may hold fewer blocks.
template <int NT>
__global__ void __launch_bounds__(kThreads) qgemv_q80_kernel(const int8_t *__restrict__ QS,
                                                             const uint16_t *__restrict__ DD,
                                                             int64_t M, int nb, XPack P,
                                                             float *__restrict__ Y, int ncols, int WK) {
    __shared__ float red[8][NT * 4][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int WR = 8 / WK, wr = warp / WK, wk = warp % WK;
    const int64_t nrb = (M + 15) / 16;
    const int nch = (nb + 7) / 8;

    for (int64_t rb0 = (int64_t)blockIdx.x * WR; rb0 < nrb; rb0 += (int64_t)gridDim.x * WR) {
        const int64_t rb = rb0 + wr;
        float tot[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) tot[nt][i] = 0.f;
        if (rb < nrb) {
            const int64_t r0 = rb * 16 + g, r1 = r0 + 8;
            const int64_t i0 = (r0 < M ? r0 : M - 1) * nb, i1 = (r1 < M ? r1 : M - 1) * nb;
            for (int ch = wk; ch < nch; ch += WK) {
                const int nblk = min(8, nb - 8 * ch);
                uint2 q0[8], q1[8];
                float d0[8], d1[8];
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    if (j < nblk) {
                        const int64_t bi0 = i0 + 8 * ch + j, bi1 = i1 + 8 * ch + j;
                        q0[j] = ldg_nc2(QS + bi0 * 32 + 8 * t);
                        q1[j] = ldg_nc2(QS + bi1 * 32 + 8 * t);
                        d0[j] = h2f(__ldg(DD + bi0));
                        d1[j] = h2f(__ldg(DD + bi1));
                    }
                }
                const uint4 *xpu = P.xp + (int64_t)ch * 8 * NT * 32 + lane;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    if (j < nblk) {
                        float c[NT][4];
#pragma unroll
                        for (int nt = 0; nt < NT; nt++)
#pragma unroll
                            for (int i = 0; i < 4; i++) c[nt][i] = 0.f;
                        uint4 bb[NT];
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) bb[nt] = xpu[j * NT * 32 + nt * 32];
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            const uint32_t W0 = h ? q0[j].y : q0[j].x, W1 = h ? q1[j].y : q1[j].x;
                            // int8 -> f16: (b ^ 0x80) | 0x6400 = 1152 + q, minus 1152
                            const uint32_t a0 = hsub2_u(((W0 & 0x00FF00FFu) ^ 0x00800080u) | 0x64006400u, 0x64806480u);
                            const uint32_t a1 = hsub2_u(((W1 & 0x00FF00FFu) ^ 0x00800080u) | 0x64006400u, 0x64806480u);
                            const uint32_t a2 = hsub2_u((((W0 >> 8) & 0x00FF00FFu) ^ 0x00800080u) | 0x64006400u, 0x64806480u);
                            const uint32_t a3 = hsub2_u((((W1 >> 8) & 0x00FF00FFu) ^ 0x00800080u) | 0x64006400u, 0x64806480u);
#pragma unroll
                            for (int nt = 0; nt < NT; nt++) {
                                const uint32_t bx = h ? bb[nt].z : bb[nt].x, by = h ? bb[nt].w : bb[nt].y;
                                mma16816(c[nt], a0, a1, a2, a3, bx, by);
                            }
                        }
                        const int64_t unit = 8 * (int64_t)ch + j;
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) {
                            const float es = P.es[unit * 8 + 4 * nt + t];
                            tot[nt][0] = fmaf(es * d0[j], c[nt][0], tot[nt][0]);
                            tot[nt][1] = fmaf(es * d0[j], c[nt][1], tot[nt][1]);
                            tot[nt][2] = fmaf(es * d1[j], c[nt][2], tot[nt][2]);
                            tot[nt][3] = fmaf(es * d1[j], c[nt][3], tot[nt][3]);
                        }
                    }
                }
            }
        }
        if (WK > 1) {
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int i = 0; i < 4; i++) red[warp][nt * 4 + i][lane] = tot[nt][i];
            __syncthreads();
            if (wk == 0 && rb < nrb) {
                for (int q = 1; q < WK; q++)
#pragma unroll
                    for (int nt = 0; nt < NT; nt++)
#pragma unroll
                        for (int i = 0; i < 4; i++) tot[nt][i] += red[warp + q][nt * 4 + i][lane];
            }
            __syncthreads();
        }
        if (wk == 0 && rb < nrb) {
            const int64_t r0 = rb * 16 + g, r1 = r0 + 8;
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const int col = 4 * nt + t;
                if (col < ncols) {
                    if (r0 < M) Y[(int64_t)col * M + r0] = tot[nt][0] + tot[nt][1];
                    if (r1 < M) Y[(int64_t)col * M + r1] = tot[nt][2] + tot[nt][3];
                }
            }
        }
    }
}

static int num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

static int pick_wk(int units) {
    int wk = 1;
    while (wk < 8 && wk * 2 <= units) wk *= 2;
    return wk;
}

cudaError_t qgemm_small(const QTensor &T, const float *X, int ncols, float *Y, void *scratch,
                        cudaStream_t s) {
    if (ncols < 1 || ncols > 8) return cudaErrorInvalidValue;
    const int NT = ncols <= 4 ? 1 : 2;
    const int64_t K = T.cols, M = T.rows;
    const int64_t nch = (K + 255) / 256;
    XPack P = carve(scratch, T.type, K);
    switch (T.type) {
    case 12: pack_x_kernel<12><<<(unsigned)nch, kThreads, 0, s>>>(X, ncols, K, NT, P); break;
    case 13: pack_x_kernel<13><<<(unsigned)nch, kThreads, 0, s>>>(X, ncols, K, NT, P); break;
    case 14: pack_x_kernel<14><<<(unsigned)nch, kThreads, 0, s>>>(X, ncols, K, NT, P); break;
    case 8: pack_x_kernel<8><<<(unsigned)nch, kThreads, 0, s>>>(X, ncols, K, NT, P); break;
    default: return cudaErrorInvalidValue;
    }
    const int units = T.type == 8 ? (int)nch : (int)T.nb;
    const int WK = pick_wk(units), WR = 8 / WK;
    const int64_t nrb = (M + 15) / 16;
    int64_t want = (nrb + WR - 1) / WR;
    int64_t cap = (int64_t)num_sms() * 4;
    const unsigned grid = (unsigned)(want < cap ? want : cap);
    const int nb = (int)T.nb;
#define IFR_LAUNCH_NT(KER, ...)                                                  \
    do {                                                                         \
        if (NT == 1) KER<1><<<grid, kThreads, 0, s>>>(__VA_ARGS__);              \
        else KER<2><<<grid, kThreads, 0, s>>>(__VA_ARGS__);                      \
    } while (0)
    if (T.type == 12) {
        if (NT == 1) qgemv_qk_kernel<false, 1><<<grid, kThreads, 0, s>>>(T.data, M, nb, P, Y, ncols, WK);
        else qgemv_qk_kernel<false, 2><<<grid, kThreads, 0, s>>>(T.data, M, nb, P, Y, ncols, WK);
    } else if (T.type == 13) {
        if (NT == 1) qgemv_qk_kernel<true, 1><<<grid, kThreads, 0, s>>>(T.data, M, nb, P, Y, ncols, WK);
        else qgemv_qk_kernel<true, 2><<<grid, kThreads, 0, s>>>(T.data, M, nb, P, Y, ncols, WK);
    } else if (T.type == 14) {
        IFR_LAUNCH_NT(qgemv_q6k_kernel, T.data + T.off_ql, T.data + T.off_qh,
                      (const int8_t *)(T.data + T.off_sc), (const uint16_t *)(T.data + T.off_d), M,
                      nb, P, Y, ncols, WK);
    } else {
        IFR_LAUNCH_NT(qgemv_q80_kernel, (const int8_t *)(T.data + T.off_ql),
                      (const uint16_t *)(T.data + T.off_d), M, nb, P, Y, ncols, WK);
    }
#undef IFR_LAUNCH_NT
    return cudaGetLastError();
}

}  // namespace ifr
