// Small-N quantized GEMM ("verify GEMV"): Y[n][r] = sum_k W[r][k] X[n][k]
// for N <= 8 verify columns, W in Q4_K / Q5_K / Q6_K / Q8_0 (M-tile layout,
// tiles.cuh).
//
// Replaces q4_k_gemv .. q8_0_gemv (reference src/kernels/quant_kernels.c:602-697),
// which the reference calls once per token; here the N tokens of one verify
// step share a single pass over the weights.
//
// Arithmetic (exact up to f32 accumulation):
//   * weights are unpacked in registers to fp16 *integers* (magic-number
//     trick) and, for Q4_K/Q5_K, multiplied by their 6-bit sub-block scale
//     with one fp16 FMA - sc*q <= 63*31 < 2048 is exact in fp16;
//   * each f32 activation is scaled by a power of two per 256-column unit and
//     split exactly into hi + lo fp16 halves, which become two B columns;
//   * mma.sync m16n8k16 (fp16 x fp16 -> f32) forms sum_k A*B over a unit; the
//     super-block scales and the unit's power of two are applied to the f32
//     accumulators; the Q4_K/Q5_K "min" term is one m16n8k8 against
//     per-sub-block activation sums.
//
// Data movement (one persistent CTA per SM, 8 warps):
//   * thread 0 streams weight stages (16 M-tiles = one row group x the
//     units of one K pass) global -> shared with cp.async.bulk into a ring of
//     S stages guarded by mbarriers, keeping ~S x 37..70 KB in flight per SM;
//   * consumer warp w owns one unit of the pass (w % UW) and two M-tiles of
//     the row group; its B fragments for that unit stay in registers for the
//     whole pass, built straight from X (no separate packing launch);
//   * the UW unit-warps of an M-tile pair reduce through shared memory; K
//     passes accumulate into Y (read-modify-write by the same thread).
// Every mbarrier wait is bounded (~2 s); on expiry the kernel records an
// error flag, stops waiting and drains, and the host reports IFR_ERR_TIMEOUT.
#include "common.cuh"
#include "tiles.cuh"

namespace ifr {

__device__ int g_dev_error = 0;

constexpr int kConsumers = 8;
constexpr int kThreads = 32 * kConsumers;
constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at 1.9 GHz

IFR_DEV uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

IFR_DEV void mbar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
IFR_DEV void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
                 : "memory");
}
IFR_DEV void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
IFR_DEV bool mbar_try_wait(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait: false (and the device error flag set) after ~2 s
IFR_DEV bool mbar_wait(uint64_t *b, uint32_t parity) {
    if (mbar_try_wait(b, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(b, parity)) {
        if (clock64() - t0 > kWaitCycles) {
            atomicExch(&g_dev_error, 1);
            return false;
        }
    }
    return true;
}
IFR_DEV void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
IFR_DEV void consumer_bar() { __syncthreads(); }
IFR_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

IFR_DEV uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
IFR_DEV uint32_t u4w(const uint4 &v, int w) { return w == 0 ? v.x : w == 1 ? v.y : w == 2 ? v.z : v.w; }

IFR_DEV float pow2i(int k) { return __int_as_float((k + 127) << 23); }
// exponent e so that max|x| * 2^e < 2^14 (fp16-safe with headroom)
IFR_DEV int unit_exp(float m) {
    if (!(m > 0.f) || isinf(m)) return 0;
    int ex;
    frexpf(m, &ex);
    const int e = 14 - ex;
    return e < -100 ? -100 : (e > 100 ? 100 : e);
}
IFR_DEV uint32_t hi_lo_h2(float v) {  // (hi, lo) with v = hi + lo exactly up to f32 rounding of lo
    const __half h = __float2half_rn(v);
    const __half l = __float2half_rn(v - __half2float(h));
    return (uint32_t)__half_as_ushort(h) | ((uint32_t)__half_as_ushort(l) << 16);
}

// ---- B fragments of one unit, built in registers ------------------------------
// Lane L holds column 4*nt + L/8 as holder j = L%8 (tiles.cuh holder maps):
// 32 scaled values as (hi, lo) pairs; fragments are gathered by shuffles.
template <int FMT, int NT>
struct BFrag {
    uint32_t b[16][NT][2];  // per step: (k 2t,2t+1), (k 2t+8,2t+9) halves for B column g
    uint32_t m[NT];         // min-MMA B fragment (Q4_K/Q5_K)
    float es[NT];           // 2^-e of the unit for C column 4*nt + t
};

template <int FMT, int NT>
IFR_DEV void build_b(const float *__restrict__ X, int64_t K, int ncols, int64_t u, int lane,
                     BFrag<FMT, NT> &F) {
    const int g = lane >> 2, t = lane & 3, j = lane & 7;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const int col = 4 * nt + (lane >> 3);
        float v[32];
        const float *xc = X + (int64_t)col * K + u * 256;
        const bool has = col < ncols;
#pragma unroll
        for (int r4 = 0; r4 < 8; r4++) {
            const int e = elem_of_holder(FMT, j, 4 * r4);
            const int64_t k = u * 256 + e;
            if (has && k + 3 < K) {
                const float4 q = __ldg(reinterpret_cast<const float4 *>(xc + e));
                v[4 * r4] = q.x; v[4 * r4 + 1] = q.y; v[4 * r4 + 2] = q.z; v[4 * r4 + 3] = q.w;
            } else {
#pragma unroll
                for (int i = 0; i < 4; i++) v[4 * r4 + i] = (has && k + i < K) ? __ldg(xc + e + i) : 0.f;
            }
        }
        float m = 0.f;
#pragma unroll
        for (int r = 0; r < 32; r++) m = fmaxf(m, fabsf(v[r]));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
        const int ex = unit_exp(m);
        const float scl = pow2i(ex);
        F.es[nt] = __shfl_sync(0xffffffffu, pow2i(-ex), 8 * t);
        uint32_t H[32];
#pragma unroll
        for (int r = 0; r < 32; r++) {
            v[r] *= scl;  // exact
            H[r] = hi_lo_h2(v[r]);
        }
        const int src_base = 8 * (g >> 1), part = g & 1;
#pragma unroll
        for (int s = 0; s < 16; s++) {
            uint32_t hv[4];
#pragma unroll
            for (int slot = 0; slot < 4; slot++) {
                const int src = src_base + holder_of(FMT, elem_of(FMT, s, t, slot));
                const uint32_t w = __shfl_sync(0xffffffffu, H[slot_reg(FMT, s, slot)], src);
                hv[slot] = part ? (w >> 16) : (w & 0xffffu);
            }
            F.b[s][nt][0] = hv[0] | (hv[1] << 16);
            F.b[s][nt][1] = hv[2] | (hv[3] << 16);
        }
        if (FMT == 12 || FMT == 13) {
            // sub-block sums: holder j has elements of sub-blocks j/2 (r < 16) and 4 + j/2
            float p0 = 0.f, p1 = 0.f;
#pragma unroll
            for (int r = 0; r < 16; r++) { p0 += v[r]; p1 += v[16 + r]; }
            p0 += __shfl_xor_sync(0xffffffffu, p0, 1);
            p1 += __shfl_xor_sync(0xffffffffu, p1, 1);
            uint32_t hm[2];
#pragma unroll
            for (int kr = 0; kr < 2; kr++) {
                const int src = src_base + 4 * (t >> 1) + 2 * kr;
                const float a = __shfl_sync(0xffffffffu, p0, src);
                const float b = __shfl_sync(0xffffffffu, p1, src);
                const uint32_t w = hi_lo_h2(((t & 1) ? b : a) * 0.03125f);
                hm[kr] = part ? (w >> 16) : (w & 0xffffu);
            }
            F.m[nt] = hm[0] | (hm[1] << 16);
        }
    }
}

// ---- fp16 constants from a byte ---------------------------------------------
IFR_DEV uint32_t bcast_byte_h2(uint32_t word, int byte) {
    const uint32_t sel = (uint32_t)byte | (4u << 4) | ((uint32_t)byte << 8) | (4u << 12);
    return hsub2_u(__byte_perm(word, 0u, sel) | 0x64006400u, 0x64006400u);
}
IFR_DEV uint32_t bytes01_h2(uint32_t word) {
    return hsub2_u(__byte_perm(word, 0u, 0x4140u) | 0x64006400u, 0x64006400u);
}
constexpr uint32_t kNegH1024 = 0xE400E400u;  // (-1024, -1024)
constexpr uint32_t kH1_16 = 0x2C002C00u;     // (1/16, 1/16)
constexpr uint32_t kNegH64 = 0xD400D400u;    // (-64, -64)

struct QKRow {
    uint32_t klo[2], nlo[2], khi[2], nhi[2];
    uint32_t mA;
    float d, dm32;
};

// scales of the four sub-blocks lane quad t reads (2p, 2p+1, 4+2p, 5+2p)
IFR_DEV void qk_row_consts(const uint4 &h, int t, QKRow &R) {
    const int p = t >> 1;
    const uint32_t A = h.y >> (16 * p), B = h.z >> (16 * p), C = h.w >> (16 * p);
    const uint32_t sc_a = A & 0x3F3Fu, m_a = B & 0x3F3Fu;
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

// ---- one M-tile (16 rows x 256 columns) from shared memory --------------------
template <int FMT, int NT>
IFR_DEV void mtile_qk(const uint8_t *tile, int lane, const BFrag<FMT, NT> &F, float (&tot)[NT][4]) {
    constexpr bool Q5 = FMT == 13;
    const int g = lane >> 2, t = lane & 3;
    const uint4 h0 = lds128(tile + qk_hdr(g)), h1 = lds128(tile + qk_hdr(g + 8));
    uint4 q0[2], q1[2], qh0 = {}, qh1 = {};
#pragma unroll
    for (int c = 0; c < 2; c++) {
        q0[c] = lds128(tile + qk_qs(Q5, c, g, t));
        q1[c] = lds128(tile + qk_qs(Q5, c, g + 8, t));
    }
    if (Q5) {
        qh0 = lds128(tile + q5_qh(g, t & 1));
        qh1 = lds128(tile + q5_qh(g + 8, t & 1));
    }
    QKRow R0, R1;
    qk_row_consts(h0, t, R0);
    qk_row_consts(h1, t, R1);
    // two accumulator sets (even / odd words) halve the MMA dependency chains
    float csc[2][NT][4], cm[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) csc[0][nt][i] = csc[1][nt][i] = cm[nt][i] = 0.f;
#pragma unroll
    for (int c = 0; c < 2; c++) {
        const int j4 = 2 * c + (t >> 1);
#pragma unroll
        for (int w = 0; w < 4; w++) {
            const uint32_t W0 = u4w(q0[c], w), W1 = u4w(q1[c], w);
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t s0 = h ? (W0 >> 8) : W0, s1 = h ? (W1 >> 8) : W1;
                uint32_t lo0 = lop_and_or(s0, 0x000F000Fu, 0x64006400u);
                uint32_t hi0 = lop_and_or(s0, 0x00F000F0u, 0x64006400u);
                uint32_t lo1 = lop_and_or(s1, 0x000F000Fu, 0x64006400u);
                uint32_t hi1 = lop_and_or(s1, 0x00F000F0u, 0x64006400u);
                if (Q5) {
                    const uint32_t H0 = u4w(qh0, w) >> (8 * h + 2 * j4);
                    const uint32_t H1 = u4w(qh1, w) >> (8 * h + 2 * j4);
                    lo0 |= (H0 << 4) & 0x00100010u;
                    hi0 |= (H0 << 7) & 0x01000100u;
                    lo1 |= (H1 << 4) & 0x00100010u;
                    hi1 |= (H1 << 7) & 0x01000100u;
                }
                const uint32_t a0 = hfma2_u(lo0, R0.klo[c], R0.nlo[c]);
                const uint32_t a1 = hfma2_u(lo1, R1.klo[c], R1.nlo[c]);
                const uint32_t a2 = hfma2_u(hi0, R0.khi[c], R0.nhi[c]);
                const uint32_t a3 = hfma2_u(hi1, R1.khi[c], R1.nhi[c]);
                const int s = 8 * c + 2 * w + h;
#pragma unroll
                for (int nt = 0; nt < NT; nt++)
                    mma16816(csc[w & 1][nt], a0, a1, a2, a3, F.b[s][nt][0], F.b[s][nt][1]);
            }
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        mma1688(cm[nt], R0.mA, R1.mA, F.m[nt]);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float d = i < 2 ? R0.d : R1.d, dm = i < 2 ? R0.dm32 : R1.dm32;
            tot[nt][i] = fmaf(F.es[nt], d * (csc[0][nt][i] + csc[1][nt][i]) - dm * cm[nt][i], tot[nt][i]);
        }
    }
}

template <int NT>
IFR_DEV void mtile_q6k(const uint8_t *tile, int lane, const BFrag<14, NT> &F, float (&tot)[NT][4]) {
    const int g = lane >> 2, t = lane & 3;
    const float d0 = h2f(*reinterpret_cast<const uint16_t *>(tile + q6_d(g)));
    const float d1 = h2f(*reinterpret_cast<const uint16_t *>(tile + q6_d(g + 8)));
    const uint4 sc0 = lds128(tile + q6_sc(g)), sc1 = lds128(tile + q6_sc(g + 8));
    uint4 l0[2], l1[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        l0[h] = lds128(tile + q6_ql(h, g, t));
        l1[h] = lds128(tile + q6_ql(h, g + 8, t));
    }
    const uint4 hq0 = lds128(tile + q6_qh(g, t)), hq1 = lds128(tile + q6_qh(g + 8, t));
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[nt][i] = 0.f;
#pragma unroll
    for (int s = 0; s < 16; s++) {
        const int n = s >> 3, qq = (s >> 1) & 3, b = s & 1;
        const int kw = 4 * n + 2 * (qq & 1) + b, kh = 2 * n + b;
        const uint32_t WA0 = u4w(l0[kw >> 2], kw & 3), WA1 = u4w(l1[kw >> 2], kw & 3);
        const uint32_t H0 = u4w(hq0, kh), H1 = u4w(hq1, kh);
        const int ns = qq >= 2 ? 4 : 0, hs = 2 * qq;
        const uint32_t x02_0 = ((WA0 >> ns) & 0x000F000Fu) | (((H0 >> hs) << 4) & 0x00300030u);
        const uint32_t x13_0 = ((WA0 >> (ns + 8)) & 0x000F000Fu) | (((H0 >> (hs + 8)) << 4) & 0x00300030u);
        const uint32_t x02_1 = ((WA1 >> ns) & 0x000F000Fu) | (((H1 >> hs) << 4) & 0x00300030u);
        const uint32_t x13_1 = ((WA1 >> (ns + 8)) & 0x000F000Fu) | (((H1 >> (hs + 8)) << 4) & 0x00300030u);
        const uint32_t a0 = hsub2_u(x02_0 | 0x64006400u, 0x64206420u);
        const uint32_t a1 = hsub2_u(x02_1 | 0x64006400u, 0x64206420u);
        const uint32_t a2 = hsub2_u(x13_0 | 0x64006400u, 0x64206420u);
        const uint32_t a3 = hsub2_u(x13_1 | 0x64006400u, 0x64206420u);
        const float f0 = (float)(int8_t)(u4w(sc0, s >> 2) >> (8 * (s & 3)));
        const float f1 = (float)(int8_t)(u4w(sc1, s >> 2) >> (8 * (s & 3)));
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            float c[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(c, a0, a1, a2, a3, F.b[s][nt][0], F.b[s][nt][1]);
            acc[nt][0] = fmaf(f0, c[0], acc[nt][0]);
            acc[nt][1] = fmaf(f0, c[1], acc[nt][1]);
            acc[nt][2] = fmaf(f1, c[2], acc[nt][2]);
            acc[nt][3] = fmaf(f1, c[3], acc[nt][3]);
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        tot[nt][0] = fmaf(F.es[nt] * d0, acc[nt][0], tot[nt][0]);
        tot[nt][1] = fmaf(F.es[nt] * d0, acc[nt][1], tot[nt][1]);
        tot[nt][2] = fmaf(F.es[nt] * d1, acc[nt][2], tot[nt][2]);
        tot[nt][3] = fmaf(F.es[nt] * d1, acc[nt][3], tot[nt][3]);
    }
}

template <int NT>
IFR_DEV void mtile_q80(const uint8_t *tile, int lane, const BFrag<8, NT> &F, float (&tot)[NT][4]) {
    const int g = lane >> 2, t = lane & 3;
    const uint4 dd0 = lds128(tile + q8_d(g)), dd1 = lds128(tile + q8_d(g + 8));
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[nt][i] = 0.f;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const uint4 p0 = lds128(tile + q8_qs(q, g, t)), p1 = lds128(tile + q8_qs(q, g + 8, t));
#pragma unroll
        for (int bb = 0; bb < 2; bb++) {
            const int bl = 2 * q + bb;
            const float db0 = h2f((uint16_t)(u4w(dd0, bl >> 1) >> (16 * (bl & 1))));
            const float db1 = h2f((uint16_t)(u4w(dd1, bl >> 1) >> (16 * (bl & 1))));
            float c[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int i = 0; i < 4; i++) c[nt][i] = 0.f;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t W0 = bb ? (h ? p0.w : p0.z) : (h ? p0.y : p0.x);
                const uint32_t W1 = bb ? (h ? p1.w : p1.z) : (h ? p1.y : p1.x);
                // int8 -> f16: (b ^ 0x80) | 0x6400 = 1152 + q, minus 1152
                const uint32_t a0 = hsub2_u(((W0 & 0x00FF00FFu) ^ 0x00800080u) | 0x64006400u, 0x64806480u);
                const uint32_t a1 = hsub2_u(((W1 & 0x00FF00FFu) ^ 0x00800080u) | 0x64006400u, 0x64806480u);
                const uint32_t a2 = hsub2_u((((W0 >> 8) & 0x00FF00FFu) ^ 0x00800080u) | 0x64006400u, 0x64806480u);
                const uint32_t a3 = hsub2_u((((W1 >> 8) & 0x00FF00FFu) ^ 0x00800080u) | 0x64006400u, 0x64806480u);
                const int s = 2 * bl + h;
#pragma unroll
                for (int nt = 0; nt < NT; nt++) mma16816(c[nt], a0, a1, a2, a3, F.b[s][nt][0], F.b[s][nt][1]);
            }
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                acc[nt][0] = fmaf(db0, c[nt][0], acc[nt][0]);
                acc[nt][1] = fmaf(db0, c[nt][1], acc[nt][1]);
                acc[nt][2] = fmaf(db1, c[nt][2], acc[nt][2]);
                acc[nt][3] = fmaf(db1, c[nt][3], acc[nt][3]);
            }
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) tot[nt][i] = fmaf(F.es[nt], acc[nt][i], tot[nt][i]);
}

struct GemvArgs {
    const uint8_t *W;  // M-tiles
    int64_t M, K;
    int nrb, nu;       // row blocks of 16, units of 256
    const float *X;    // [ncols][K]
    int ncols;
    float *Y;          // [ncols][M]
    int UW, S;         // unit-warps per pass, ring stages
    int sweep_rg;      // row groups per sweep (their sums fit the shared accumulator)
    int accumulate;    // 1: Y += W X (residual), 0: Y = W X
    int64_t ldy;       // Y[col * ldy + row]
};

// Work order of one CTA: its contiguous range of row groups, cut into sweeps;
// per sweep all K passes; per pass the sweep's row groups (one stage each).
// Partial sums of a sweep live in shared memory, so no K pass touches global
// memory until the sweep's rows are final.
struct Order {
    int rg_lo, rg_hi, sweep_rg, passes;
    IFR_DEV int total() const {
        int n = 0;
        for (int sw = rg_lo; sw < rg_hi; sw += sweep_rg) n += passes * min(sweep_rg, rg_hi - sw);
        return n;
    }
    // stage q -> (pass, row group)
    IFR_DEV void at(int q, int &p, int &rg) const {
        const int full = passes * sweep_rg;
        const int sw = q / full, r = q % full;
        const int sw_lo = rg_lo + sw * sweep_rg;
        const int n = min(sweep_rg, rg_hi - sw_lo);
        p = r / n;
        rg = sw_lo + r % n;
    }
};

// Issue the bulk copies of stage q into its ring slot (one thread).
template <int MTB>
IFR_DEV void issue_stage(const GemvArgs &a, const Order &o, int q, uint8_t *ring, uint64_t *full) {
    constexpr int STAGE = 16 * MTB;
    const int UW = a.UW, MTG = 16 / UW;
    int p, rg;
    o.at(q, p, rg);
    const int s = q % a.S;
    const int u0 = p * UW, nuh = min(UW, a.nu - u0);
    const int nmt = min(MTG, a.nrb - rg * MTG);
    fence_proxy_async();  // earlier generic reads of this slot before the async writes
    mbar_expect_tx(full + s, (uint32_t)(nmt * nuh * MTB));
    for (int m = 0; m < nmt; m++) {
        const uint8_t *src = a.W + ((int64_t)(rg * MTG + m) * a.nu + u0) * MTB;
        bulk_g2s(ring + (size_t)s * STAGE + (size_t)m * UW * MTB, src, (uint32_t)(nuh * MTB), full + s);
    }
}

template <int FMT, int NT>
__global__ void __launch_bounds__(kThreads, 1) qgemv_kernel(GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int MTB = mtile_bytes(FMT);
    constexpr int STAGE = 16 * MTB;   // MTG * UW M-tiles
    constexpr int NRED = 2 * NT * 4;  // floats per lane per warp in the reduction
    const int UW = a.UW, MTG = 16 / UW;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint8_t *ring = smem + 128;
    float *red = reinterpret_cast<float *>(ring + (size_t)a.S * STAGE);
    float *acc = red + kConsumers * NRED * 32;  // [sweep_rg * MTG * 16 rows][8 cols]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nrg = (a.nrb + MTG - 1) / MTG;
    Order o;
    o.rg_lo = (int)((int64_t)blockIdx.x * nrg / gridDim.x);
    o.rg_hi = (int)((int64_t)(blockIdx.x + 1) * nrg / gridDim.x);
    o.sweep_rg = a.sweep_rg;
    o.passes = (a.nu + UW - 1) / UW;
    const int total = o.total();

    pdl_trigger();
    // the weights are constant: their first stages stream in before the
    // previous kernel (producer of X, reader/writer of Y) has finished
    if (tid == 0) {
        for (int s = 0; s < a.S; s++) mbar_init(full + s, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int q = 0; q < min(a.S, total); q++) issue_stage<MTB>(a, o, q, ring, full);
    }
    pdl_wait();
    __syncthreads();

    const int ui = warp % UW, mp = warp / UW;
    BFrag<FMT, NT> F;
    int it = 0;
    bool dead = false;
    for (int sw = o.rg_lo; sw < o.rg_hi; sw += o.sweep_rg) {
        const int sw_hi = min(o.rg_hi, sw + o.sweep_rg);
        const int sw_rows = (sw_hi - sw) * MTG * 16;
        for (int i = tid; i < sw_rows * 8; i += kThreads) acc[i] = 0.f;
        for (int p = 0; p < o.passes; p++) {
            const int64_t u = (int64_t)p * UW + ui;
            const bool active = u < a.nu;
            if (active) build_b<FMT, NT>(a.X, a.K, a.ncols, u, lane, F);
            for (int rg = sw; rg < sw_hi; rg++, it++) {
                const int s = it % a.S;
                if (!dead && !mbar_wait(full + s, (uint32_t)(it / a.S) & 1)) dead = true;
                float tot[2][NT][4];
#pragma unroll
                for (int mm = 0; mm < 2; mm++)
#pragma unroll
                    for (int nt = 0; nt < NT; nt++)
#pragma unroll
                        for (int i = 0; i < 4; i++) tot[mm][nt][i] = 0.f;
                if (active && !dead) {
                    const uint8_t *st = ring + (size_t)s * STAGE;
#pragma unroll
                    for (int mm = 0; mm < 2; mm++) {
                        const int m = 2 * mp + mm;
                        if (rg * MTG + m < a.nrb) {
                            const uint8_t *tile = st + (size_t)(m * UW + ui) * MTB;
                            if constexpr (FMT == 14) mtile_q6k<NT>(tile, lane, F, tot[mm]);
                            else if constexpr (FMT == 8) mtile_q80<NT>(tile, lane, F, tot[mm]);
                            else mtile_qk<FMT, NT>(tile, lane, F, tot[mm]);
                        }
                    }
                }
#pragma unroll
                for (int mm = 0; mm < 2; mm++)
#pragma unroll
                    for (int nt = 0; nt < NT; nt++)
#pragma unroll
                        for (int i = 0; i < 4; i++)
                            red[((warp * 2 + mm) * NT * 4 + nt * 4 + i) * 32 + lane] = tot[mm][nt][i];
                consumer_bar();  // slot s fully read; partials visible
                if (tid == 0 && !dead && it + a.S < total) issue_stage<MTB>(a, o, it + a.S, ring, full);
                // each thread owns outputs (m, row, col) = o, o + 256, ... in every pass
                const int base = (rg - sw) * MTG * 16;
                for (int oi = tid; oi < MTG * 128; oi += kThreads) {
                    const int col = oi & 7, r16 = (oi >> 3) & 15, m = oi >> 7;
                    const int nt = col >> 2;
                    if (nt >= NT) continue;
                    const int mmp = m >> 1, mm = m & 1, half = r16 >> 3;
                    const int ln = 4 * (r16 & 7) + (col & 3);
                    float v = 0.f;
                    for (int q = 0; q < UW; q++) {
                        const float *pp = red + (((mmp * UW + q) * 2 + mm) * NT * 4 + nt * 4 + 2 * half) * 32 + ln;
                        v += pp[0] + pp[32];
                    }
                    acc[(base + m * 16 + r16) * 8 + col] += v;
                }
                consumer_bar();  // red reused by the next stage
            }
        }
        // the sweep's rows are final: write Y (coalesced over rows)
        const int64_t row0 = (int64_t)sw * MTG * 16;
        for (int i = tid; i < sw_rows * a.ncols; i += kThreads) {
            const int col = i / sw_rows, r = i % sw_rows;
            if (row0 + r < a.M && !dead) {
                float *y = a.Y + (int64_t)col * a.ldy + row0 + r;
                *y = a.accumulate ? *y + acc[r * 8 + col] : acc[r * 8 + col];
            }
        }
        consumer_bar();
    }
    // stages issued but not consumed (only after a timeout) must land before exit
    if (tid == 0 && dead)
        for (int q = it; q < min(it + a.S, total); q++) mbar_wait(full + (q % a.S), (uint32_t)(q / a.S) & 1);
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

template <int FMT, int NT>
static cudaError_t launch(const QTensor &T, const float *X, int ncols, float *Y, bool accumulate, int64_t ldy,
                          cudaStream_t s) {
    constexpr int MTB = mtile_bytes(FMT);
    constexpr int STAGE = 16 * MTB;
    constexpr int kSmemMax = 227 * 1024;
    int UW = 1;
    while (UW < 8 && UW * 2 <= T.nu) UW *= 2;
    const int MTG = 16 / UW;
    const int red = kConsumers * (2 * NT * 4) * 32 * 4;
    const int64_t nrg = (T.nrb + MTG - 1) / MTG;
    const int grid = (int)(nrg < num_sms() ? nrg : num_sms());
    // ring stages first (2..5), then the shared accumulator gets the rest
    int S = (kSmemMax - 128 - red - 16 * 1024) / STAGE;
    S = S < 2 ? 2 : (S > 5 ? 5 : S);
    const int acc_bytes_avail = kSmemMax - 128 - S * STAGE - red;
    const int rg_bytes = MTG * 16 * 8 * 4;
    const int64_t per_cta = (nrg + grid - 1) / grid;
    int sweep_rg = acc_bytes_avail / rg_bytes;
    if (sweep_rg < 1) return cudaErrorInvalidConfiguration;
    if (sweep_rg > per_cta) sweep_rg = (int)per_cta;
    const int smem = 128 + S * STAGE + red + sweep_rg * rg_bytes;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(qgemv_kernel<FMT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    GemvArgs a{T.data, T.rows, T.cols, (int)T.nrb, (int)T.nu, X, ncols, Y, UW, S, sweep_rg, accumulate ? 1 : 0, ldy};
    return launch_k(qgemv_kernel<FMT, NT>, dim3(grid), dim3(kThreads), (size_t)smem, s, a);
}

cudaError_t qgemm_small(const QTensor &T, const float *X, int ncols, float *Y, bool accumulate, int64_t ldy,
                        cudaStream_t s) {
    if (ncols < 1 || ncols > 8) return cudaErrorInvalidValue;
    const bool two = ncols > 4;
    switch (T.type) {
    case 12: return two ? launch<12, 2>(T, X, ncols, Y, accumulate, ldy, s) : launch<12, 1>(T, X, ncols, Y, accumulate, ldy, s);
    case 13: return two ? launch<13, 2>(T, X, ncols, Y, accumulate, ldy, s) : launch<13, 1>(T, X, ncols, Y, accumulate, ldy, s);
    case 14: return two ? launch<14, 2>(T, X, ncols, Y, accumulate, ldy, s) : launch<14, 1>(T, X, ncols, Y, accumulate, ldy, s);
    case 8: return two ? launch<8, 2>(T, X, ncols, Y, accumulate, ldy, s) : launch<8, 1>(T, X, ncols, Y, accumulate, ldy, s);
    }
    return cudaErrorInvalidValue;
}

cudaError_t read_device_error(int *flag, cudaStream_t s) {
    int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(flag, g_dev_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(g_dev_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e;
}

}  // namespace ifr
