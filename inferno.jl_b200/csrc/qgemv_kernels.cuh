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
// Data movement, unit-split kernel (qgemv_kernel; one persistent CTA per SM,
// 16 warps):
//   * thread 0 streams weight stages (16 M-tiles = one row group x the
//     units of one K pass) global -> shared with cp.async.bulk into a ring of
//     S stages guarded by mbarriers, keeping ~S x 37..70 KB in flight per SM;
//   * consumer warp w owns one unit of the pass (w % UW) and one M-tile of the
//     row group (two with Q8_K activations); exact activations: the pass's B
//     fragments are built once into shared memory by the unit's warps, Q8_K:
//     each warp builds its unit's fragments in registers; both straight from
//     X (no separate packing launch);
//   * the UW unit-warps of a row block reduce through shared memory; K passes
//     accumulate in shared memory until the rows are final.
// Tall matrices (qgemv_rows_kernel, below) keep a whole row block per warp.
// Every mbarrier wait is bounded (~2 s); on expiry the kernel records an
// error flag, stops waiting and drains, and the host reports IFR_ERR_TIMEOUT.
#pragma once
#include "common.cuh"
#include "tiles.cuh"

#include <type_traits>

namespace ifr {

// set by a bounded wait that ran out; one flag per translation unit (the
// kernels of each weight format are compiled separately), read and cleared
// by read_device_error
static __device__ int g_dev_error = 0;

// consumer warps per CTA: 16 in both modes (<= 128 registers per thread).  With
// exact activations the B fragments live in shared memory (built once per pass
// by the warps of each unit), so a thread holds only one M-tile's operands.
template <int ACT>
__host__ __device__ constexpr int consumers() { return 16; }
constexpr int kMaxFoldUnits = 512;  // folded RMSNorm: K up to 131072
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

struct GemvArgs {
    const uint8_t *W;  // M-tiles
    int64_t M, K;
    int nrb, nu;       // row blocks of 16, units of 256
    const float *X;    // column c at X + c * ldx
    int64_t ldx;
    int ncols;
    float *Y;          // [ncols][M]
    int UW, S;         // unit-warps per pass, ring stages
    int sweep_rg;      // row groups per sweep (their sums fit the shared accumulator)
    int accumulate;    // 1: Y += W X (residual), 0: Y = W X
    int64_t ldy;       // Y[col * ldy + row]
    int xf;            // activation transform: 0 none, 1 RMSNorm(xw, eps), 2 SwiGLU
    const float *xw;   // RMSNorm weights [K]
    float eps;
    int ep;            // 1: SwiGLU epilogue over interleaved gate/up 16-row blocks
    int rev;           // qgemv_rows_kernel: row groups last to first (XForm::rev)
    int khalves;       // qgemv_rows_kernel: 2 = CTA 2b + h takes K half h of pair b's row groups
    float *kpart;      // khalves 2: the second half's partials [ncols][M]
};
// the greedy decision's arguments, a kernel parameter of the AM variants only
template <bool AM> struct AmArg { GemvArgmax am; };
template <> struct AmArg<false> {};

// order-preserving key of (value, row) for a 64-bit max: larger value first,
// then the lower row
IFR_DEV unsigned long long argmax_key(float v, int64_t row) {
    const uint32_t u = __float_as_uint(v);
    const uint32_t k = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)k << 32) | (0xFFFFFFFFu - (uint32_t)row);
}

// ---- exact f32 activations on the fp16 tensor cores ----------------------------
// Lane (g, t) feeds B column g of every step: activation column 4 nt + g/2,
// its fp16 high part (g even) or low part (g odd), for the elements
// 16 s + 4t + {0..3} of step s (tiles.cuh), slots (0, 1) = elements (0, 2) and
// slots (2, 3) = elements (1, 3).  The two lanes of a pair (g, g^1) load half
// the steps each, split them into (hi, lo) and swap halves by one shuffle per
// register.  Activations are scaled by a power of two per unit (exact) so that
// hi + lo carries ~22 bits; es undoes it on the f32 sums.
// One unit's fragments in shared memory, 32-bit words:
//   b  [step 16][n-tile NT][lane 32] x 2  slots (0,1), (2,3) of each step
//   m  [n-tile][lane]  Q4_K/Q5_K min MMA: sums of sub-blocks 2t, 2t+1 (x 2^-5)
//   es [n-tile][lane]  2^-e of the unit for C column 4*nt + t
__host__ __device__ constexpr int bunit_words(int NT) { return 16 * NT * 32 * 2 + 2 * NT * 32; }
template <int NT>
struct BView {
    const uint2 *b;     // this lane's entries: b[(s * NT + nt) * 32]
    const uint32_t *m;  // m[nt * 32]
    const float *es;    // es[nt * 32]
    IFR_DEV void at(const uint32_t *unit, int lane) {
        b = reinterpret_cast<const uint2 *>(unit) + lane;
        m = unit + 16 * NT * 32 * 2 + lane;
        es = reinterpret_cast<const float *>(unit + 16 * NT * 32 * 2 + NT * 32) + lane;
    }
    IFR_DEV uint2 ld(int s, int nt) const { return b[(s * NT + nt) * 32]; }
};

IFR_DEV uint32_t cvt_h2(float hi_half, float lo_half) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi_half), "f"(lo_half));
    return r;
}
IFR_DEV float h2_lo(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v & 0xffffu))); }
IFR_DEV float h2_hi(uint32_t v) { return __half2float(__ushort_as_half((unsigned short)(v >> 16))); }

// 8 runs of 4 floats at p + k0 + i * step (0 beyond K or when !has).  No
// value is used here, so every load of the 8 runs is in flight at once.
// NC: through the read-only path (data no thread of the launch writes);
// false for activations that earlier phases of the same launch produced
template <bool NC = true>
IFR_DEV void ld_runs(const float *p, int64_t K, int64_t k0, int step, bool has, float4 (&r)[8]) {
    auto ld4 = [](const float *q) { return NC ? __ldg(reinterpret_cast<const float4 *>(q)) : *reinterpret_cast<const float4 *>(q); };
    auto ld1 = [](const float *q) { return NC ? __ldg(q) : *q; };
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int64_t k = k0 + (int64_t)step * i;
        r[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (has && k + 3 < K) {
            r[i] = ld4(p + k);
        } else if (has) {  // ragged K: the rare scalar path
            if (k < K) r[i].x = ld1(p + k);
            if (k + 1 < K) r[i].y = ld1(p + k + 1);
            if (k + 2 < K) r[i].z = ld1(p + k + 2);
        }
    }
}

// 8 runs of 4 activations of column col at k0 + i * step (transform XF
// applied; 0 beyond K or for absent columns): all loads first, then the
// arithmetic.  XF 3 (RMSNorm folded into the epilogue): x * w, and ss
// accumulates the raw x^2
template <int XF>
IFR_DEV void xform_runs(const float4 (&xr)[8], const float4 (&wr)[8], float iv, float *v, float *ss) {
    float s2 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float4 q = xr[i];
        if (XF == 1) {
            q.x = q.x * iv * wr[i].x;
            q.y = q.y * iv * wr[i].y;
            q.z = q.z * iv * wr[i].z;
            q.w = q.w * iv * wr[i].w;
        } else if (XF == 3) {
            s2 += q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w;
            q.x *= wr[i].x;
            q.y *= wr[i].y;
            q.z *= wr[i].z;
            q.w *= wr[i].w;
        } else if (XF == 2) {
            q.x = q.x / (1.0f + expf(-q.x)) * wr[i].x;
            q.y = q.y / (1.0f + expf(-q.y)) * wr[i].y;
            q.z = q.z / (1.0f + expf(-q.z)) * wr[i].z;
            q.w = q.w / (1.0f + expf(-q.w)) * wr[i].w;
        }
        v[4 * i] = q.x;
        v[4 * i + 1] = q.y;
        v[4 * i + 2] = q.z;
        v[4 * i + 3] = q.w;
    }
    if (XF == 3) *ss += s2;
}

template <int XF>
IFR_DEV void load_x32(const GemvArgs &a, const float *inv, int col, int64_t k0, int step, bool has, float *v,
                      float *ss = nullptr) {
    const float *xc = a.X + (int64_t)col * a.ldx;
    float4 xr[8], wr[8];
    ld_runs(xc, a.K, k0, step, has, xr);
    if (XF == 1 || XF == 3) ld_runs(a.xw, a.K, k0, step, has, wr);
    if (XF == 2) ld_runs(xc + a.K, a.K, k0, step, has, wr);  // up half of [gate | up]
    xform_runs<XF>(xr, wr, XF == 1 && has ? inv[col] : 0.f, v, ss);
}

// Builds n-tile nt of unit u's fragments into `unit` (bunit_words(NT) words).
// ssq (XF 3, may be null): [unit][8] sums of x^2 of the unit's activations.
// COH: the activations are read with coherent loads (the fused launch, whose
// earlier phases wrote them)
template <int FMT, int NT, int XF, bool COH = false>
IFR_DEV void build_b(const GemvArgs &a, const float *inv, int64_t u, int lane, int nt, uint32_t *unit, float *ssq) {
    const int g = lane >> 2, t = lane & 3, part = g & 1;
    // this lane's steps 8 part .. 8 part + 7 (elem_s() of tiles.cuh): every load
    // (and the norm weights) in flight before the first is used
    const int64_t k0 = u * 256 + 128 * part + 4 * t;
    const int col = 4 * nt + (g >> 1);
    float v[32];
    float ss = 0.f;
    if (XF == 2) {
        load_x32<XF>(a, inv, col, k0, 16, col < a.ncols, v, &ss);
    } else {
        float4 xr[8], wr[8];
        ld_runs<!COH>(a.X + (int64_t)col * a.ldx, a.K, k0, 16, col < a.ncols, xr);
        if (XF == 1 || XF == 3) ld_runs(a.xw, a.K, k0, 16, true, wr);
        xform_runs<XF>(xr, wr, XF == 1 && col < a.ncols ? inv[col] : 0.f, v, &ss);
    }
    if (XF == 3) {
        // the unit's 256 elements of column col are spread over lanes 8c .. 8c + 7
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        ss += __shfl_xor_sync(0xffffffffu, ss, 4);
        if (ssq && (lane & 7) == 0) ssq[u * 8 + col] = ss;
    }
    float mx = 0.f;
#pragma unroll
    for (int r = 0; r < 32; r++) mx = fmaxf(mx, fabsf(v[r]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    const int ex = unit_exp(mx);
    const float scl = pow2i(ex);
    uint2 *ub = reinterpret_cast<uint2 *>(unit) + lane;
    reinterpret_cast<float *>(unit + 16 * NT * 32 * 2 + NT * 32)[nt * 32 + lane] =
        __shfl_sync(0xffffffffu, pow2i(-ex), 8 * t);
    uint32_t keep[8][2], send[8][2];
    float cs[4] = {0.f, 0.f, 0.f, 0.f};  // this lane's part of chunks 4 part .. 4 part + 3
#pragma unroll
    for (int i = 0; i < 8; i++) {
        float x[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            x[j] = v[4 * i + j] * scl;  // exact
            cs[i >> 1] += x[j];
        }
        const uint32_t h02 = cvt_h2(x[2], x[0]), h13 = cvt_h2(x[3], x[1]);
        const uint32_t l02 = cvt_h2(x[2] - h2_hi(h02), x[0] - h2_lo(h02));
        const uint32_t l13 = cvt_h2(x[3] - h2_hi(h13), x[1] - h2_lo(h13));
        keep[i][0] = part ? l02 : h02;
        keep[i][1] = part ? l13 : h13;
        send[i][0] = part ? h02 : l02;
        send[i][1] = part ? h13 : l13;
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        uint32_t lo[2], hi[2];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t r = __shfl_xor_sync(0xffffffffu, send[i][h], 4);
            lo[h] = part ? r : keep[i][h];
            hi[h] = part ? keep[i][h] : r;
        }
        ub[(i * NT + nt) * 32] = make_uint2(lo[0], lo[1]);
        ub[((8 + i) * NT + nt) * 32] = make_uint2(hi[0], hi[1]);
    }
    if (FMT == 12 || FMT == 13) {
        // sub-block (= chunk) sums of column col: over the lane quad, then the partner
        // lane's four chunks; lane (g, t) takes chunks 2t, 2t+1, its hi or lo part
        float S[8];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            float v2 = cs[k];
            v2 += __shfl_xor_sync(0xffffffffu, v2, 1);
            v2 += __shfl_xor_sync(0xffffffffu, v2, 2);
            const float o = __shfl_xor_sync(0xffffffffu, v2, 4);
            S[k] = part ? o : v2;
            S[4 + k] = part ? v2 : o;
        }
        float sa = S[0], sb = S[1];
#pragma unroll
        for (int k = 1; k < 4; k++)
            if (t == k) {
                sa = S[2 * k];
                sb = S[2 * k + 1];
            }
        sa *= 0.03125f;  // x 2^-5 keeps the sums in fp16 range
        sb *= 0.03125f;
        const uint32_t hs = cvt_h2(sb, sa);
        const uint32_t ls = cvt_h2(sb - h2_hi(hs), sa - h2_lo(hs));
        unit[16 * NT * 32 * 2 + nt * 32 + lane] = part ? ls : hs;
    }
}

constexpr uint32_t kMagic = 0x64006400u;  // (1024, 1024)

// fp16 constants from a byte
IFR_DEV uint32_t bcast_byte_h2(uint32_t word, int byte) {
    const uint32_t sel = (uint32_t)byte | (4u << 4) | ((uint32_t)byte << 8) | (4u << 12);
    return hsub2_u(__byte_perm(word, 0u, sel) | kMagic, kMagic);
}
IFR_DEV uint32_t bytes01_h2(uint32_t word) {
    return hsub2_u(__byte_perm(word, 0u, 0x4140u) | kMagic, kMagic);
}
constexpr uint32_t kNegH1024 = 0xE400E400u;  // (-1024, -1024)
constexpr uint32_t kH1_16 = 0x2C002C00u;     // (1/16, 1/16)
constexpr uint32_t kNegH64 = 0xD400D400u;    // (-64, -64)

// 6-bit scales and mins of the 8 sub-blocks of a Q4_K/Q5_K header
// (src/Dequant.jl:345-362), one byte each: words [0] = sub-blocks 0-3, [1] = 4-7
IFR_DEV void qk_scales(const uint4 &h, uint32_t (&sc)[2], uint32_t (&mn)[2]) {
    sc[0] = h.y & 0x3f3f3f3fu;
    mn[0] = h.z & 0x3f3f3f3fu;
    sc[1] = (h.w & 0x0f0f0f0fu) | (((h.y >> 6) & 0x03030303u) << 4);
    mn[1] = ((h.w >> 4) & 0x0f0f0f0fu) | (((h.z >> 6) & 0x03030303u) << 4);
}

// Q4_K / Q5_K with exact activations: A = q * sc in fp16 (exact: sc*q <= 63*31 <
// 2048), low-nibble chunks as fma(1024+q, sc, -1024 sc), high-nibble chunks as
// fma(1024+16q, sc/16, -64 sc); one qs word serves the steps of chunks 2p, 2p+1
template <bool Q5, int NT>
IFR_DEV void mtile_qk_h(const uint8_t *tile, int lane, const BView<NT> &F, float (&tot)[NT][4]) {
    const int g = lane >> 2, t = lane & 3;
    const uint4 h0 = lds128(tile + qk_hdr(g)), h1 = lds128(tile + qk_hdr(g + 8));
    const uint4 q00 = lds128(tile + qk_qs(Q5, 0, g, t)), q01 = lds128(tile + qk_qs(Q5, 1, g, t));
    const uint4 q10 = lds128(tile + qk_qs(Q5, 0, g + 8, t)), q11 = lds128(tile + qk_qs(Q5, 1, g + 8, t));
    uint4 hb = {};
    if (Q5) hb = lds128(tile + q5_qh(g, t));
    uint32_t sc0[2], mn0[2], sc1[2], mn1[2];
    qk_scales(h0, sc0, mn0);
    qk_scales(h1, sc1, mn1);
    // min MMA A fragment: (m_2t, m_2t+1) of rows g and g+8
    const uint32_t mA0 = bytes01_h2(mn0[t >> 1] >> (16 * (t & 1)));
    const uint32_t mA1 = bytes01_h2(mn1[t >> 1] >> (16 * (t & 1)));
    float c[2][NT][4], cm[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) c[0][nt][i] = c[1][nt][i] = cm[nt][i] = 0.f;
#pragma unroll
    for (int p = 0; p < 4; p++) {
        const int cl = 2 * p, chh = 2 * p + 1;
        const uint32_t kl0 = bcast_byte_h2(sc0[cl >> 2], cl & 3), kl1 = bcast_byte_h2(sc1[cl >> 2], cl & 3);
        const uint32_t nl0 = hmul2_u(kl0, kNegH1024), nl1 = hmul2_u(kl1, kNegH1024);
        const uint32_t sh0 = bcast_byte_h2(sc0[chh >> 2], chh & 3), sh1 = bcast_byte_h2(sc1[chh >> 2], chh & 3);
        const uint32_t kh0 = hmul2_u(sh0, kH1_16), kh1 = hmul2_u(sh1, kH1_16);
        const uint32_t nh0 = hmul2_u(sh0, kNegH64), nh1 = hmul2_u(sh1, kNegH64);
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint4 Q0 = (p >> 1) ? q01 : q00, Q1 = (p >> 1) ? q11 : q10;
            const uint32_t W0 = u4w(Q0, 2 * (p & 1) + h), W1 = u4w(Q1, 2 * (p & 1) + h);
            const uint32_t W0s = W0 >> 8, W1s = W1 >> 8;
            uint32_t lo02_0 = lop_and_or(W0, 0x000F000Fu, kMagic), lo13_0 = lop_and_or(W0s, 0x000F000Fu, kMagic);
            uint32_t hi02_0 = lop_and_or(W0, 0x00F000F0u, kMagic), hi13_0 = lop_and_or(W0s, 0x00F000F0u, kMagic);
            uint32_t lo02_1 = lop_and_or(W1, 0x000F000Fu, kMagic), lo13_1 = lop_and_or(W1s, 0x000F000Fu, kMagic);
            uint32_t hi02_1 = lop_and_or(W1, 0x00F000F0u, kMagic), hi13_1 = lop_and_or(W1s, 0x00F000F0u, kMagic);
            if (Q5) {
                // fifth bit: bit c of qh byte j; low nibble -> +16 (bit 4), high nibble -> +256 (bit 8)
                const uint32_t H0 = h ? hb.y : hb.x, H1 = h ? hb.w : hb.z;
                lo02_0 |= ((H0 >> cl) & 0x00010001u) << 4;
                lo13_0 |= ((H0 >> (8 + cl)) & 0x00010001u) << 4;
                lo02_1 |= ((H1 >> cl) & 0x00010001u) << 4;
                lo13_1 |= ((H1 >> (8 + cl)) & 0x00010001u) << 4;
                hi02_0 |= ((H0 >> chh) & 0x00010001u) << 8;
                hi13_0 |= ((H0 >> (8 + chh)) & 0x00010001u) << 8;
                hi02_1 |= ((H1 >> chh) & 0x00010001u) << 8;
                hi13_1 |= ((H1 >> (8 + chh)) & 0x00010001u) << 8;
            }
            const uint32_t a0 = hfma2_u(lo02_0, kl0, nl0), a1 = hfma2_u(lo02_1, kl1, nl1);
            const uint32_t a2 = hfma2_u(lo13_0, kl0, nl0), a3 = hfma2_u(lo13_1, kl1, nl1);
            const uint32_t b0 = hfma2_u(hi02_0, kh0, nh0), b1 = hfma2_u(hi02_1, kh1, nh1);
            const uint32_t b2 = hfma2_u(hi13_0, kh0, nh0), b3 = hfma2_u(hi13_1, kh1, nh1);
            const int sl = 2 * cl + h, shs = 2 * chh + h;
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const uint2 bl = F.ld(sl, nt), bh = F.ld(shs, nt);
                mma16816(c[0][nt], a0, a1, a2, a3, bl.x, bl.y);
                mma16816(c[1][nt], b0, b1, b2, b3, bh.x, bh.y);
            }
        }
    }
    const float d0 = h2f((uint16_t)(h0.x & 0xffffu)), dm0 = h2f((uint16_t)(h0.x >> 16)) * 32.0f;
    const float d1 = h2f((uint16_t)(h1.x & 0xffffu)), dm1 = h2f((uint16_t)(h1.x >> 16)) * 32.0f;
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        mma1688(cm[nt], mA0, mA1, F.m[nt * 32]);
        const float es = F.es[nt * 32];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float d = i < 2 ? d0 : d1, dm = i < 2 ? dm0 : dm1;
            tot[nt][i] = fmaf(es, d * (c[0][nt][i] + c[1][nt][i]) - dm * cm[nt][i], tot[nt][i]);
        }
    }
}

// Q6_K with exact activations: step s = scale group s; A = q - 32 as
// (1024 + q) - 1056 (low nibbles) or (1024 + 16 q) / 16 - 96 (high nibbles); the
// int8 group scale multiplies each step's f32 MMA result
template <int NT>
IFR_DEV void mtile_q6_h(const uint8_t *tile, int lane, const BView<NT> &F, float (&tot)[NT][4]) {
    const int g = lane >> 2, t = lane & 3;
    const float d0 = h2f(*reinterpret_cast<const uint16_t *>(tile + q6_d(g)));
    const float d1 = h2f(*reinterpret_cast<const uint16_t *>(tile + q6_d(g + 8)));
    const uint4 sc0 = lds128(tile + q6_sc(g)), sc1 = lds128(tile + q6_sc(g + 8));
    const uint4 l00 = lds128(tile + q6_ql(0, g, t)), l01 = lds128(tile + q6_ql(1, g, t));
    const uint4 l10 = lds128(tile + q6_ql(0, g + 8, t)), l11 = lds128(tile + q6_ql(1, g + 8, t));
    const uint4 hq0 = lds128(tile + q6_qh(g, t)), hq1 = lds128(tile + q6_qh(g + 8, t));
    constexpr uint32_t k1056 = 0x64206420u;   // (1056, 1056)
    constexpr uint32_t kNeg96 = 0xD600D600u;  // (-96, -96)
    float acc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[nt][i] = 0.f;
#pragma unroll
    for (int c = 0; c < 8; c++) {
        const int n = c >> 2, qq = c & 3;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int s = 2 * c + h;
            const uint32_t W0 = u4w(n ? l01 : l00, 2 * (qq & 1) + h), W1 = u4w(n ? l11 : l10, 2 * (qq & 1) + h);
            const uint32_t H0 = u4w(hq0, 2 * n + h) >> (2 * qq), H1 = u4w(hq1, 2 * n + h) >> (2 * qq);
            uint32_t a0, a1, a2, a3;
            if ((qq >> 1) == 0) {
                a0 = hsub2_u(lop_and_or(W0, 0x000F000Fu, kMagic) | ((H0 << 4) & 0x00300030u), k1056);
                a1 = hsub2_u(lop_and_or(W1, 0x000F000Fu, kMagic) | ((H1 << 4) & 0x00300030u), k1056);
                a2 = hsub2_u(lop_and_or(W0 >> 8, 0x000F000Fu, kMagic) | ((H0 >> 4) & 0x00300030u), k1056);
                a3 = hsub2_u(lop_and_or(W1 >> 8, 0x000F000Fu, kMagic) | ((H1 >> 4) & 0x00300030u), k1056);
            } else {
                a0 = hfma2_u(lop_and_or(W0, 0x00F000F0u, kMagic) | ((H0 << 8) & 0x03000300u), kH1_16, kNeg96);
                a1 = hfma2_u(lop_and_or(W1, 0x00F000F0u, kMagic) | ((H1 << 8) & 0x03000300u), kH1_16, kNeg96);
                a2 = hfma2_u(lop_and_or(W0 >> 8, 0x00F000F0u, kMagic) | (H0 & 0x03000300u), kH1_16, kNeg96);
                a3 = hfma2_u(lop_and_or(W1 >> 8, 0x00F000F0u, kMagic) | (H1 & 0x03000300u), kH1_16, kNeg96);
            }
            const float f0 = (float)(int8_t)(u4w(sc0, s >> 2) >> (8 * (s & 3)));
            const float f1 = (float)(int8_t)(u4w(sc1, s >> 2) >> (8 * (s & 3)));
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                float cc[4];
                const uint2 bb = F.ld(s, nt);
                mma16816_z(cc, a0, a1, a2, a3, bb.x, bb.y);
                acc[nt][0] = fmaf(f0, cc[0], acc[nt][0]);
                acc[nt][1] = fmaf(f0, cc[1], acc[nt][1]);
                acc[nt][2] = fmaf(f1, cc[2], acc[nt][2]);
                acc[nt][3] = fmaf(f1, cc[3], acc[nt][3]);
            }
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
        const float es = F.es[nt * 32];
        tot[nt][0] = fmaf(es * d0, acc[nt][0], tot[nt][0]);
        tot[nt][1] = fmaf(es * d0, acc[nt][1], tot[nt][1]);
        tot[nt][2] = fmaf(es * d1, acc[nt][2], tot[nt][2]);
        tot[nt][3] = fmaf(es * d1, acc[nt][3], tot[nt][3]);
    }
}

// Q8_0: steps 2b, 2b+1 = block b; int8 -> fp16 as ((x ^ 0x80) | 0x6400) - 1152,
// the block scale multiplies the f32 MMA result of its two steps
template <int NT>
IFR_DEV void mtile_q80(const uint8_t *tile, int lane, const BView<NT> &F, float (&tot)[NT][4]) {
    const int g = lane >> 2, t = lane & 3;
    const uint4 dd0 = lds128(tile + q8_d(g)), dd1 = lds128(tile + q8_d(g + 8));
    constexpr uint32_t k1152 = 0x64806480u;
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
            const int blk = 2 * q + bb;
            float c[NT][4];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int s = 2 * blk + h;
                const uint32_t W0 = u4w(p0, 2 * bb + h) ^ 0x80808080u, W1 = u4w(p1, 2 * bb + h) ^ 0x80808080u;
                const uint32_t a0 = hsub2_u(lop_and_or(W0, 0x00FF00FFu, kMagic), k1152);
                const uint32_t a1 = hsub2_u(lop_and_or(W1, 0x00FF00FFu, kMagic), k1152);
                const uint32_t a2 = hsub2_u(lop_and_or(W0 >> 8, 0x00FF00FFu, kMagic), k1152);
                const uint32_t a3 = hsub2_u(lop_and_or(W1 >> 8, 0x00FF00FFu, kMagic), k1152);
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    const uint2 bb = F.ld(s, nt);
                    if (h == 0) mma16816_z(c[nt], a0, a1, a2, a3, bb.x, bb.y);
                    else mma16816(c[nt], a0, a1, a2, a3, bb.x, bb.y);
                }
            }
            const float db0 = h2f((uint16_t)(u4w(dd0, blk >> 1) >> (16 * (blk & 1))));
            const float db1 = h2f((uint16_t)(u4w(dd1, blk >> 1) >> (16 * (blk & 1))));
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
        for (int i = 0; i < 4; i++) tot[nt][i] = fmaf(F.es[nt * 32], acc[nt][i], tot[nt][i]);
}

// ---- K-quants with Q8_K activations on the integer tensor cores ---------------
// quantize_row_q8_K (src/kernels/quant_kernels.c:166-194) per 256-element unit
// of each column: d = amax / 127, q = roundf(x * (1/d)), in correctly rounded
// f32, then exact integer sub-block sums: the reference's own kernels.
// Lane (g, t) builds the B fragments of column g (the C fragment's lanes
// (g', t) read columns 2t, 2t+1, whose scales and sub-block sums are fetched
// by shuffles).
IFR_DEV uint32_t pack4_s8(int q0, int q1, int q2, int q3) {
    return (uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8) | ((uint32_t)(q2 & 0xff) << 16) |
           ((uint32_t)(q3 & 0xff) << 24);
}

struct __align__(16) BFragI8 {
    uint32_t b[8][2];  // chunk c: int8 of k-slots 4t..4t+3 and 16+4t..16+4t+3, column g
    // B of the correction MMA (k16): the block sums of column g as 7-bit limbs,
    // [0] = sum & 127, [1] = sum >> 7 (k-slots 4t..4t+3); Q4_K/Q5_K: the 8
    // chunk sums (mins term, lanes t < 2), Q6_K: the 16 group sums (the -32 offset)
    uint32_t bc[2];
    float d8[2];       // Q8_K scales of columns 2t and 2t+1
};

// byte k of w, zero- or sign-extended (one PRMT)
IFR_DEV int ubyte(uint32_t w, int k) { return (int)__byte_perm(w, 0u, 0x4440u | (uint32_t)k); }
IFR_DEV int sbyte(uint32_t w, int k) {
    // selector nibbles: byte k, then three copies of its sign (msb of the nibble set)
    const uint32_t x = 8u | (uint32_t)k, sel = (uint32_t)k | (x << 4) | (x << 8) | (x << 12);
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(w), "r"(0u), "r"(sel));
    return (int)r;
}
// 4 sums as 7-bit limbs: lo bytes (v & 127) and hi bytes (v >> 7), v in [-2^14, 2^14)
IFR_DEV void limbs4(int v0, int v1, int v2, int v3, uint32_t &lo, uint32_t &hi) {
    lo = pack4_s8(v0 & 127, v1 & 127, v2 & 127, v3 & 127);
    hi = pack4_s8(v0 >> 7, v1 >> 7, v2 >> 7, v3 >> 7);
}

template <int FMT, int XF>
IFR_DEV void build_b_i8(const GemvArgs &a, const float *inv, int64_t u, int lane, BFragI8 &F) {
    const int g = lane >> 2, t = lane & 3;
    const bool has = g < a.ncols;
    // elements 32c + 16h + 4t + {0..3} for run i = 2c + h: k0 + 16 i
    float v[64];
    float *v0 = v, *v1 = v + 32;
    load_x32<XF>(a, inv, g, u * 256 + 4 * t, 16, has, v0);
    load_x32<XF>(a, inv, g, u * 256 + 128 + 4 * t, 16, has, v1);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 64; i++) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
    int hsum[16];  // this lane's 4 elements of each 16-element group 2c + h
#pragma unroll
    for (int c = 0; c < 8; c++) {
        int q[8];
#pragma unroll
        for (int j = 0; j < 8; j++) q[j] = (int)roundf(__fmul_rn(v[8 * c + j], id));
        F.b[c][0] = pack4_s8(q[0], q[1], q[2], q[3]);
        F.b[c][1] = pack4_s8(q[4], q[5], q[6], q[7]);
        hsum[2 * c] = q[0] + q[1] + q[2] + q[3];
        hsum[2 * c + 1] = q[4] + q[5] + q[6] + q[7];
    }
    F.d8[0] = __shfl_sync(0xffffffffu, d, 8 * t);
    F.d8[1] = __shfl_sync(0xffffffffu, d, 8 * t + 4);
    F.bc[0] = F.bc[1] = 0u;
    if (FMT == 12 || FMT == 13) {
        // chunk sums of column g (over the quad); lane t < 2 holds chunks 4t .. 4t + 3
        int cs[8];
#pragma unroll
        for (int c = 0; c < 8; c++) {
            int v2 = hsum[2 * c] + hsum[2 * c + 1];
            v2 += __shfl_xor_sync(0xffffffffu, v2, 1);
            v2 += __shfl_xor_sync(0xffffffffu, v2, 2);
            cs[c] = v2;
        }
        if (t < 2) {
            const bool hi = t == 1;
            limbs4(hi ? cs[4] : cs[0], hi ? cs[5] : cs[1], hi ? cs[6] : cs[2], hi ? cs[7] : cs[3], F.bc[0], F.bc[1]);
        }
    } else if (FMT == 14) {
        // group sums of column g (over the quad); lane t holds groups 4t .. 4t + 3
        int gs[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            int v2 = hsum[j];
            v2 += __shfl_xor_sync(0xffffffffu, v2, 1);
            v2 += __shfl_xor_sync(0xffffffffu, v2, 2);
            gs[j] = v2;
        }
        int w4[4];
#pragma unroll
        for (int i = 0; i < 4; i++) w4[i] = t == 0 ? gs[i] : t == 1 ? gs[4 + i] : t == 2 ? gs[8 + i] : gs[12 + i];
        limbs4(w4[0], w4[1], w4[2], w4[3], F.bc[0], F.bc[1]);
    }
}

// Q4_K / Q5_K x Q8_K (vec_dot_q4_K_q8_K / q5_K, quant_kernels.c:204-435): per
// unit and output, the exact integer sums S = sum_c sc_c (q . q8)_c and
// M = sum_c m_c bsum_c, then d8 * d * S - d8 * dmin * M in f32
template <bool Q5>
IFR_DEV void mtile_qk_i8(const uint8_t *tile, int lane, const BFragI8 &F, float (&tot)[4]) {
    const int g = lane >> 2, t = lane & 3;
    const uint4 h0 = lds128(tile + qk_hdr(g)), h1 = lds128(tile + qk_hdr(g + 8));
    const uint4 q00 = lds128(tile + qk_qs(Q5, 0, g, t)), q01 = lds128(tile + qk_qs(Q5, 1, g, t));
    const uint4 q10 = lds128(tile + qk_qs(Q5, 0, g + 8, t)), q11 = lds128(tile + qk_qs(Q5, 1, g + 8, t));
    uint4 hb = {};
    if (Q5) hb = lds128(tile + q5_qh(g, t));
    uint32_t sc[2][2], mn[2][2];
    qk_scales(h0, sc[0], mn[0]);
    qk_scales(h1, sc[1], mn[1]);
    int S[4] = {0, 0, 0, 0};
#pragma unroll
    for (int c = 0; c < 8; c++) {
        const int p = c >> 1, sh = 4 * (c & 1), wi = 2 * (p & 1);
        const uint4 Q0 = (p >> 1) ? q01 : q00, Q1 = (p >> 1) ? q11 : q10;
        uint32_t a0 = (u4w(Q0, wi) >> sh) & 0x0f0f0f0fu, a2 = (u4w(Q0, wi + 1) >> sh) & 0x0f0f0f0fu;
        uint32_t a1 = (u4w(Q1, wi) >> sh) & 0x0f0f0f0fu, a3 = (u4w(Q1, wi + 1) >> sh) & 0x0f0f0f0fu;
        if (Q5) {
            a0 |= ((hb.x >> c) & 0x01010101u) << 4;
            a2 |= ((hb.y >> c) & 0x01010101u) << 4;
            a1 |= ((hb.z >> c) & 0x01010101u) << 4;
            a3 |= ((hb.w >> c) & 0x01010101u) << 4;
        }
        int cc[4];
        imma16832_z(cc, a0, a1, a2, a3, F.b[c][0], F.b[c][1]);
        const int s0 = ubyte(sc[0][c >> 2], c & 3), s1 = ubyte(sc[1][c >> 2], c & 3);
        S[0] += s0 * cc[0];
        S[1] += s0 * cc[1];
        S[2] += s1 * cc[2];
        S[3] += s1 * cc[3];
    }
    // mins M = sum_c m_c bsum_c on the integer tensor cores: A = the 6-bit mins
    // (k-slot = chunk; lanes t < 2), B = the chunk sums' 7-bit limbs
    const uint32_t ma0 = t == 0 ? mn[0][0] : (t == 1 ? mn[0][1] : 0u);
    const uint32_t ma1 = t == 0 ? mn[1][0] : (t == 1 ? mn[1][1] : 0u);
    int ml[4], mh[4], M[4];
    imma16816_z(ml, ma0, ma1, F.bc[0]);
    imma16816_z(mh, ma0, ma1, F.bc[1]);
#pragma unroll
    for (int i = 0; i < 4; i++) M[i] = ml[i] + mh[i] * 128;
    const float d0 = h2f((uint16_t)(h0.x & 0xffffu)), dm0 = h2f((uint16_t)(h0.x >> 16));
    const float d1 = h2f((uint16_t)(h1.x & 0xffffu)), dm1 = h2f((uint16_t)(h1.x >> 16));
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float d8 = F.d8[i & 1];
        tot[i] += (d8 * (i < 2 ? d0 : d1)) * (float)S[i] - (d8 * (i < 2 ? dm0 : dm1)) * (float)M[i];
    }
}

// Q6_K x Q8_K (vec_dot_q6_K_q8_K, quant_kernels.c:440-...): S = sum_j sc_j
// ((q6 - 32) . q8)_j over the 16 groups, then d8 * d * S; one k16 MMA per group
IFR_DEV void mtile_q6_i8(const uint8_t *tile, int lane, const BFragI8 &F, float (&tot)[4]) {
    const int g = lane >> 2, t = lane & 3;
    const float d0 = h2f(*reinterpret_cast<const uint16_t *>(tile + q6_d(g)));
    const float d1 = h2f(*reinterpret_cast<const uint16_t *>(tile + q6_d(g + 8)));
    const uint4 sc0 = lds128(tile + q6_sc(g)), sc1 = lds128(tile + q6_sc(g + 8));
    const uint4 l00 = lds128(tile + q6_ql(0, g, t)), l01 = lds128(tile + q6_ql(1, g, t));
    const uint4 l10 = lds128(tile + q6_ql(0, g + 8, t)), l11 = lds128(tile + q6_ql(1, g + 8, t));
    const uint4 hq0 = lds128(tile + q6_qh(g, t)), hq1 = lds128(tile + q6_qh(g + 8, t));
    int S[4] = {0, 0, 0, 0};
#pragma unroll
    for (int c = 0; c < 8; c++) {
        const int n = c >> 2, qq = c & 3;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t w0 = u4w(n ? l01 : l00, 2 * (qq & 1) + h), w1 = u4w(n ? l11 : l10, 2 * (qq & 1) + h);
            // unsigned 6-bit q (0..63); the -32 is applied once per unit below
            const uint32_t x0 = ((w0 >> (4 * (qq >> 1))) & 0x0f0f0f0fu) |
                                (((u4w(hq0, 2 * n + h) >> (2 * qq)) & 0x03030303u) << 4);
            const uint32_t x1 = ((w1 >> (4 * (qq >> 1))) & 0x0f0f0f0fu) |
                                (((u4w(hq1, 2 * n + h) >> (2 * qq)) & 0x03030303u) << 4);
            int cc[4];
            imma16816_z(cc, x0, x1, F.b[c][h]);
            const int j = 2 * c + h;
            const int f0 = sbyte(u4w(sc0, j >> 2), j & 3);
            const int f1 = sbyte(u4w(sc1, j >> 2), j & 3);
            S[0] += f0 * cc[0];
            S[1] += f0 * cc[1];
            S[2] += f1 * cc[2];
            S[3] += f1 * cc[3];
        }
    }
    // sum_j sc_j ((q - 32) . q8)_j = sum_j sc_j (q . q8)_j - 32 sum_j sc_j bsum_j; the
    // second sum on the integer tensor cores: A = the int8 group scales (k-slot =
    // group), B = the group sums' 7-bit limbs
    const uint32_t sa0 = t == 0 ? sc0.x : t == 1 ? sc0.y : t == 2 ? sc0.z : sc0.w;
    const uint32_t sa1 = t == 0 ? sc1.x : t == 1 ? sc1.y : t == 2 ? sc1.z : sc1.w;
    int cl[4], ch[4];
    imma16816_z(cl, sa0, sa1, F.bc[0]);
    imma16816_z(ch, sa0, sa1, F.bc[1]);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        S[i] -= 32 * (cl[i] + ch[i] * 128);
        tot[i] += (F.d8[i & 1] * (i < 2 ? d0 : d1)) * (float)S[i];
    }
}

// ---- exact f32 activations on the integer tensor cores (Q4_K / Q5_K, tall) ----
// Each 256-element unit of a column is written as three int8 limbs over one
// scale d = amax / 127: x / d = l1 + l2 / 254 + l3 / 254^2 + r, |r| <= 0.5 /
// 254^2, so x is carried to ~6e-8 of the unit's amax (plus the f32 rounding
// of x / d) - the precision of the fp16 (hi, lo) split, with int8 weights
// taken from the nibbles directly (no fp16 conversion per weight).  The
// weight side is the Q8_K path's (exact integer sums per sub-block, scaled
// per sub-block); each limb level has its own sums, combined in f32 at the end.
// One unit's fragments in shared memory, uint2 entries [.][lane 32]:
//   [3 c + l]   chunk c, level l: int8 of k-slots 4t..4t+3 | 16+4t..16+4t+3, column g
//   [24 + l]    level l's chunk sums as 7-bit limbs (lo, hi), lanes t < 2: chunks 4t..4t+3
//   [27]        d of C columns 2t, 2t+1 (f32 bits)
constexpr int kL8Entries = 28;
constexpr int kL8Words = kL8Entries * 32 * 2;
constexpr float kL8Step = 254.0f;
constexpr float kL8Inv1 = 1.0f / 254.0f, kL8Inv2 = 1.0f / 64516.0f;

IFR_DEV int l8_limb(float v) { return (int)fminf(fmaxf(rintf(v), -127.f), 127.f); }

template <int FMT, int XF>
IFR_DEV void build_b_l8(const GemvArgs &a, const float *inv, int64_t u, int lane, uint32_t *unit, float *ssq) {
    const int g = lane >> 2, t = lane & 3;
    const bool has = g < a.ncols;
    // elements 32c + 16h + 4t + {0..3} of run i = 2c + h: v[8c + 4h + j]
    float v[64];
    float ss = 0.f;
    load_x32<XF>(a, inv, g, u * 256 + 4 * t, 16, has, v, &ss);
    load_x32<XF>(a, inv, g, u * 256 + 128 + 4 * t, 16, has, v + 32, &ss);
    if (XF == 3) {  // the unit's 256 elements of column g are spread over the quad
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        if (ssq && t == 0) ssq[u * 8 + g] = ss;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 64; i++) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
    uint2 *ub = reinterpret_cast<uint2 *>(unit) + lane;
    int keep[3][4];  // level l's sums of chunks 4t .. 4t + 3 (lanes t < 2)
#pragma unroll
    for (int c = 0; c < 8; c++) {
        int l[3][8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float x = v[8 * c + j];
            l[0][j] = l8_limb(__fmul_rn(x, id));
            const float r1 = fmaf(x, id, -(float)l[0][j]);
            l[1][j] = l8_limb(r1 * kL8Step);
            const float r2 = fmaf(r1, kL8Step, -(float)l[1][j]);
            l[2][j] = l8_limb(r2 * kL8Step);
        }
#pragma unroll
        for (int lv = 0; lv < 3; lv++) {
            ub[(3 * c + lv) * 32] = make_uint2(pack4_s8(l[lv][0], l[lv][1], l[lv][2], l[lv][3]),
                                               pack4_s8(l[lv][4], l[lv][5], l[lv][6], l[lv][7]));
            int cs = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) cs += l[lv][j];
            cs += __shfl_xor_sync(0xffffffffu, cs, 1);
            cs += __shfl_xor_sync(0xffffffffu, cs, 2);
            if ((c >> 2) == t) keep[lv][c & 3] = cs;
        }
    }
#pragma unroll
    for (int lv = 0; lv < 3; lv++) {
        uint32_t lo = 0u, hi = 0u;
        if (t < 2) limbs4(keep[lv][0], keep[lv][1], keep[lv][2], keep[lv][3], lo, hi);
        ub[(24 + lv) * 32] = make_uint2(lo, hi);
    }
    ub[27 * 32] = make_uint2(__float_as_uint(__shfl_sync(0xffffffffu, d, 8 * t)),
                             __float_as_uint(__shfl_sync(0xffffffffu, d, 8 * t + 4)));
}

// Q4_K / Q5_K with limb activations: per level l and output, the exact
// integer sums S_l = sum_c sc_c (q . l)_c and M_l = sum_c m_c bsum_c; then
// d * dq * sum_l S_l / 254^l - d * dmin * sum_l M_l / 254^l in f32
template <bool Q5>
IFR_DEV void mtile_qk_l8(const uint8_t *tile, int lane, const uint2 *fb, float (&tot)[4]) {
    const int g = lane >> 2, t = lane & 3;
    const uint4 h0 = lds128(tile + qk_hdr(g)), h1 = lds128(tile + qk_hdr(g + 8));
    const uint4 q00 = lds128(tile + qk_qs(Q5, 0, g, t)), q01 = lds128(tile + qk_qs(Q5, 1, g, t));
    const uint4 q10 = lds128(tile + qk_qs(Q5, 0, g + 8, t)), q11 = lds128(tile + qk_qs(Q5, 1, g + 8, t));
    uint4 hb = {};
    if (Q5) hb = lds128(tile + q5_qh(g, t));
    uint32_t sc[2][2], mn[2][2];
    qk_scales(h0, sc[0], mn[0]);
    qk_scales(h1, sc[1], mn[1]);
    int S[3][4];
#pragma unroll
    for (int lv = 0; lv < 3; lv++)
#pragma unroll
        for (int i = 0; i < 4; i++) S[lv][i] = 0;
#pragma unroll
    for (int c = 0; c < 8; c++) {
        const int p = c >> 1, sh = 4 * (c & 1), wi = 2 * (p & 1);
        const uint4 Q0 = (p >> 1) ? q01 : q00, Q1 = (p >> 1) ? q11 : q10;
        uint32_t a0 = (u4w(Q0, wi) >> sh) & 0x0f0f0f0fu, a2 = (u4w(Q0, wi + 1) >> sh) & 0x0f0f0f0fu;
        uint32_t a1 = (u4w(Q1, wi) >> sh) & 0x0f0f0f0fu, a3 = (u4w(Q1, wi + 1) >> sh) & 0x0f0f0f0fu;
        if (Q5) {
            a0 |= ((hb.x >> c) & 0x01010101u) << 4;
            a2 |= ((hb.y >> c) & 0x01010101u) << 4;
            a1 |= ((hb.z >> c) & 0x01010101u) << 4;
            a3 |= ((hb.w >> c) & 0x01010101u) << 4;
        }
        const int s0 = ubyte(sc[0][c >> 2], c & 3), s1 = ubyte(sc[1][c >> 2], c & 3);
#pragma unroll
        for (int lv = 0; lv < 3; lv++) {
            const uint2 b = fb[(3 * c + lv) * 32];
            int cc[4];
            imma16832_z(cc, a0, a1, a2, a3, b.x, b.y);
            S[lv][0] += s0 * cc[0];
            S[lv][1] += s0 * cc[1];
            S[lv][2] += s1 * cc[2];
            S[lv][3] += s1 * cc[3];
        }
    }
    // mins: A = the 6-bit mins (k-slot = chunk; lanes t < 2), B = each level's
    // chunk sums as 7-bit limbs
    const uint32_t ma0 = t == 0 ? mn[0][0] : (t == 1 ? mn[0][1] : 0u);
    const uint32_t ma1 = t == 0 ? mn[1][0] : (t == 1 ? mn[1][1] : 0u);
    int M[3][4];
#pragma unroll
    for (int lv = 0; lv < 3; lv++) {
        const uint2 bc = fb[(24 + lv) * 32];
        int ml[4], mh[4];
        imma16816_z(ml, ma0, ma1, bc.x);
        imma16816_z(mh, ma0, ma1, bc.y);
#pragma unroll
        for (int i = 0; i < 4; i++) M[lv][i] = ml[i] + mh[i] * 128;
    }
    const uint2 dw = fb[27 * 32];
    const float dc[2] = {__uint_as_float(dw.x), __uint_as_float(dw.y)};
    const float d0 = h2f((uint16_t)(h0.x & 0xffffu)), dm0 = h2f((uint16_t)(h0.x >> 16));
    const float d1 = h2f((uint16_t)(h1.x & 0xffffu)), dm1 = h2f((uint16_t)(h1.x >> 16));
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float sv = fmaf((float)S[2][i], kL8Inv2, fmaf((float)S[1][i], kL8Inv1, (float)S[0][i]));
        const float mv = fmaf((float)M[2][i], kL8Inv2, fmaf((float)M[1][i], kL8Inv1, (float)M[0][i]));
        const float dd = dc[i & 1];
        tot[i] += (dd * (i < 2 ? d0 : d1)) * sv - (dd * (i < 2 ? dm0 : dm1)) * mv;
    }
}

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
template <int MTB, int MPW, int CW>
IFR_DEV void issue_stage(const GemvArgs &a, const Order &o, int q, uint8_t *ring, uint64_t *full) {
    constexpr int STAGE = CW * MPW * MTB;
    const int UW = a.UW, MTG = CW * MPW / UW;
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

// MPW: M-tiles per warp per stage (a stage is 8 * MPW M-tiles = MTG row
// blocks x UW units); 1 halves each warp's serial work for small matrices
// ACT: K-quant activations, 0 exact f32 (fp16 tensor cores), 1 Q8_K (integer
// tensor cores, the reference's kernels); Q8_0 is always exact
// AM: the greedy decision of GemvArgs::am in the epilogue (its own
// instantiations, so the plain GEMVs carry none of its state)
template <int FMT, int NT, int XF, int MPW, int ACT, bool AM>
__global__ void __launch_bounds__(32 * consumers<ACT>(), 1) qgemv_kernel(GemvArgs a, AmArg<AM> aa) {
    constexpr int CW = consumers<ACT>(), NTH = 32 * CW;
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int MTB = mtile_bytes(FMT);
    constexpr int STAGE = CW * MPW * MTB;  // MTG * UW M-tiles
    constexpr int NRED = MPW * NT * 4;    // floats per lane per warp in the reduction
    const int UW = a.UW, MTG = CW * MPW / UW;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint8_t *ring = smem + 128;
    float *red = reinterpret_cast<float *>(ring + (size_t)a.S * STAGE);
    // red: two buffers of per-warp partials, so consecutive stages alternate and
    // one barrier per stage suffices
    float *acc = red + 2 * CW * NRED * 32;  // [sweep_rg * MTG * 16 rows][8 cols]
    float *ssq = acc + a.sweep_rg * MTG * 16 * 8;  // XF 3: [nu][8] sums of x^2 per unit and column
    // exact activations: the B fragments of the pass's UW units
    uint32_t *bsm = reinterpret_cast<uint32_t *>(ssq + (XF == 3 ? a.nu * 8 : 0));
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
        for (int q = 0; q < min(a.S, total); q++) issue_stage<MTB, MPW, CW>(a, o, q, ring, full);
    }
    pdl_wait();
    // RMSNorm of the input columns: 1 / sqrt(sum x^2 / K + eps) per column
    // (rmsnorm_cpu!, ModelCPU.jl:111-123), applied while building B
    __shared__ float inv_s[8];
    __shared__ float part_s[CW][8];
    __shared__ unsigned long long best_s[AM ? 8 : 1];
    __shared__ bool last_s;
    if constexpr (AM) {
        if (tid < 8) best_s[tid] = 0ull;
    }
    if (XF == 1) {
        float ss[8];
#pragma unroll
        for (int c = 0; c < 8; c++) ss[c] = 0.f;
        for (int64_t k = 4 * tid; k < a.K; k += 4 * NTH) {
#pragma unroll
            for (int c = 0; c < 8; c++) {
                if (c < a.ncols) {
                    const float4 q = __ldg(reinterpret_cast<const float4 *>(a.X + c * a.ldx + k));
                    ss[c] += q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w;
                }
            }
        }
#pragma unroll
        for (int c = 0; c < 8; c++) {
            float v = ss[c];
#pragma unroll
            for (int o2 = 16; o2; o2 >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o2);
            if (lane == 0) part_s[warp][c] = v;
        }
        __syncthreads();
        if (tid < 8) {
            float v = 0.f;
            for (int w = 0; w < CW; w++) v += part_s[w][tid];
            inv_s[tid] = 1.0f / sqrtf(v / (float)a.K + a.eps);
        }
    }
    __syncthreads();

    const int ui = warp % UW, mp = warp / UW;
    constexpr bool kI8 = FMT != 8 && ACT == 1;
    std::conditional_t<kI8, BFragI8, BView<NT>> F;
    int it = 0;
    bool dead = false;
    for (int sw = o.rg_lo; sw < o.rg_hi; sw += o.sweep_rg) {
        const int sw_hi = min(o.rg_hi, sw + o.sweep_rg);
        const int sw_rows = (sw_hi - sw) * MTG * 16;
        for (int i = tid; i < sw_rows * 8; i += NTH) acc[i] = 0.f;
        for (int p = 0; p < o.passes; p++) {
            const int64_t u = (int64_t)p * UW + ui;
            const bool active = u < a.nu;
            if constexpr (kI8) {
                if (active) build_b_i8<FMT, XF>(a, inv_s, u, lane, F);
            } else {
                // the unit's warps split its n-tiles (UW divides the warps); the
                // previous pass's fragments were last read before the barrier
                // that closed its final stage
                if (active && mp < NT)
                    build_b<FMT, NT, XF>(a, inv_s, u, lane, mp, bsm + ui * bunit_words(NT), sw == o.rg_lo ? ssq : nullptr);
                consumer_bar();
                F.at(bsm + ui * bunit_words(NT), lane);
            }
            for (int rg = sw; rg < sw_hi; rg++, it++) {
                const int s = it % a.S;
                float *redb = red + (it & 1) * (CW * NRED * 32);
                if (!dead && !mbar_wait(full + s, (uint32_t)(it / a.S) & 1)) dead = true;
                float tot[MPW][NT][4];
#pragma unroll
                for (int mm = 0; mm < MPW; mm++)
#pragma unroll
                    for (int nt = 0; nt < NT; nt++)
#pragma unroll
                        for (int i = 0; i < 4; i++) tot[mm][nt][i] = 0.f;
                if (active && !dead) {
                    const uint8_t *st = ring + (size_t)s * STAGE;
#pragma unroll
                    for (int mm = 0; mm < MPW; mm++) {
                        const int m = MPW * mp + mm;
                        if (rg * MTG + m < a.nrb) {
                            const uint8_t *tile = st + (size_t)(m * UW + ui) * MTB;
                            if constexpr (FMT == 8) mtile_q80<NT>(tile, lane, F, tot[mm]);
                            else if constexpr (kI8 && FMT == 14) mtile_q6_i8(tile, lane, F, tot[mm][0]);
                            else if constexpr (kI8) mtile_qk_i8<FMT == 13>(tile, lane, F, tot[mm][0]);
                            else if constexpr (FMT == 14) mtile_q6_h<NT>(tile, lane, F, tot[mm]);
                            else mtile_qk_h<FMT == 13, NT>(tile, lane, F, tot[mm]);
                        }
                    }
                }
#pragma unroll
                for (int mm = 0; mm < MPW; mm++)
#pragma unroll
                    for (int nt = 0; nt < NT; nt++)
#pragma unroll
                        for (int i = 0; i < 4; i++)
                            redb[((warp * MPW + mm) * NT * 4 + nt * 4 + i) * 32 + lane] = tot[mm][nt][i];
                consumer_bar();  // slot s fully read; partials visible; the other buffer's reads done
                if (tid == 0 && !dead && it + a.S < total) issue_stage<MTB, MPW, CW>(a, o, it + a.S, ring, full);
                // each thread owns outputs (m, row, col) = o, o + 256, ... in every pass
                const int base = (rg - sw) * MTG * 16;
                for (int oi = tid; oi < MTG * 128; oi += NTH) {
                    const int col = oi & 7, r16 = (oi >> 3) & 15, m = oi >> 7;
                    const int mmp = m / MPW, mm = m % MPW, half = r16 >> 3;
                    float v = 0.f;
                    if constexpr (!kI8) {
                        // C columns 2t, 2t+1 of n-tile nt are the hi and lo parts of column 4 nt + t
                        const int nt = col >> 2;
                        if (nt >= NT) continue;
                        const int ln = 4 * (r16 & 7) + (col & 3);
                        for (int q = 0; q < UW; q++) {
                            const float *pp = redb + (((mmp * UW + q) * MPW + mm) * NT * 4 + nt * 4 + 2 * half) * 32 + ln;
                            v += pp[0] + pp[32];
                        }
                    } else {
                        // C columns 2t, 2t+1 are activation columns 2t, 2t+1
                        const int ln = 4 * (r16 & 7) + (col >> 1);
                        for (int q = 0; q < UW; q++)
                            v += redb[(((mmp * UW + q) * MPW + mm) * NT * 4 + 2 * half + (col & 1)) * 32 + ln];
                    }
                    acc[(base + m * 16 + r16) * 8 + col] += v;
                }
            }
        }
        consumer_bar();  // every stage's sums are in acc
        // the sweep's rows are final: write Y (coalesced over rows)
        const int64_t row0 = (int64_t)sw * MTG * 16;
        // XF 3: W (x w) / rms(x) per column; the sums of squares in unit order
        if (XF == 3) {
            if (tid < 8) {
                float v = 0.f;
                if (tid < a.ncols)
                    for (int uu = 0; uu < a.nu; uu++) v += ssq[uu * 8 + tid];
                inv_s[tid] = tid < a.ncols ? 1.0f / sqrtf(v / (float)a.K + a.eps) : 0.f;
            }
            consumer_bar();
        }
        auto accv = [&](int r, int col) {
            const float v = acc[r * 8 + col];
            return XF == 3 ? v * inv_s[col] : v;
        };
        if (a.ep) {
            // mlp_forward (ModelCPU.jl:482-508): h = silu(gate) * up; a sweep holds whole
            // gate/up block pairs (MTG is even), local rows 32p.. gate, 32p+16.. up
            const int half_rows = sw_rows / 2;
            const int64_t j0 = row0 / 2;
            for (int i = tid; i < half_rows * a.ncols; i += NTH) {
                const int col = i / half_rows, rr = i % half_rows;
                const int gr = (rr >> 4) * 32 + (rr & 15);
                if (j0 + rr < a.M / 2 && !dead) {
                    const float gv = accv(gr, col), uv = accv(gr + 16, col);
                    a.Y[(int64_t)col * a.ldy + j0 + rr] = glu_act(a.ep, gv, uv);
                }
            }
        } else {
            if constexpr (AM) {
                int bcol = -1;
                unsigned long long bkey = 0ull;
                for (int i = tid; i < sw_rows * a.ncols; i += NTH) {
                    const int col = i / sw_rows, r = i % sw_rows;
                    if (row0 + r < a.M && !dead) {
                        const float v = accv(r, col);
                        a.Y[(int64_t)col * a.ldy + row0 + r] = v;
                        if (col != bcol) {
                            if (bcol >= 0) atomicMax(&best_s[bcol], bkey);
                            bcol = col;
                            bkey = 0ull;
                        }
                        const unsigned long long k = argmax_key(v, row0 + r);
                        bkey = k > bkey ? k : bkey;
                    }
                }
                if (bcol >= 0) atomicMax(&best_s[bcol], bkey);
            } else {
                for (int i = tid; i < sw_rows * a.ncols; i += NTH) {
                    const int col = i / sw_rows, r = i % sw_rows;
                    if (row0 + r < a.M && !dead) {
                        float *y = a.Y + (int64_t)col * a.ldy + row0 + r;
                        *y = a.accumulate ? *y + accv(r, col) : accv(r, col);
                    }
                }
            }
        }
        consumer_bar();
    }
    // stages issued but not consumed (only after a timeout) must land before exit
    if (tid == 0 && dead)
        for (int q = it; q < min(it + a.S, total); q++) mbar_wait(full + (q % a.S), (uint32_t)(q / a.S) & 1);
    if constexpr (AM) {
        // every CTA leaves its per-column best, then counts itself done; the
        // CTA that finishes last (fenced counter, nothing waits) decides
        __syncthreads();
        if (tid < a.ncols) aa.am.cand[tid * gridDim.x + blockIdx.x] = best_s[tid];
        __threadfence();
        __syncthreads();
        if (tid == 0) last_s = atomicAdd(aa.am.counter, 1u) == gridDim.x - 1;
        __syncthreads();
        if (last_s) {
            __threadfence();
            if (tid < a.ncols) {
                unsigned long long b = 0ull;
                for (unsigned c = 0; c < gridDim.x; c++) {
                    const unsigned long long k = __ldcg(aa.am.cand + tid * gridDim.x + c);
                    b = k > b ? k : b;
                }
                best_s[tid] = b;
            }
            __syncthreads();
            const int G1 = aa.am.G + 1;
            if (tid < a.ncols / G1) {
                const int b = tid;
                int32_t *ot = aa.am.out + (int64_t)b * aa.am.out_ld;
                for (int i = 0; i < G1; i++) ot[i] = -1;
                int accn = 0;
                for (int i = 0; i < G1; i++) {
                    const int tok = (int)(0xFFFFFFFFu - (uint32_t)(best_s[b * G1 + i] & 0xFFFFFFFFull));
                    ot[i] = tok;
                    if (i == aa.am.G || tok != aa.am.drafts[(int64_t)b * aa.am.draft_ld + i]) break;
                    accn++;
                }
                if (aa.am.acc) aa.am.acc[b] = accn;
            }
            if (tid == 0) *aa.am.counter = 0u;
        }
    }
}

// ---- tall matrices, exact activations: one row block per warp --------------
// For matrices of many row blocks (lm_heads, 151936 rows), in both activation
// modes, a consumer warp owns
// a whole row block over all of K, so its sums stay in registers and go
// straight to Y: no per-stage block barrier and no shared-memory reduction.
// The B fragments of every unit are built once per CTA.  Each CTA owns an
// even share of the row blocks, in groups of 15 from its first.  Warp 15
// produces: stage q = (group g, unit u) is the (up to) 15 M-tiles of the
// group's row blocks at unit u, copied with cp.async.bulk into a ring of S
// slots; full barriers count the bytes, empty barriers count the 15 consumer
// warps.  Every wait is bounded; after a timeout the kernel drains its copies
// and returns (IFR_ERR_TIMEOUT on the host).
constexpr int kRowsCW = 15;  // consumer warps (and row blocks per group)

template <int FMT, int NT, int XF, int ACT, bool AM>
__global__ void __launch_bounds__(512, 1) qgemv_rows_kernel(GemvArgs a, AmArg<AM> aa) {
    // kI8: Q8_K activations (one n-tile: columns 2t, 2t+1 of lane t), fragments
    // stored as BFragI8 [unit][lane] (80 bytes a lane: conflict-free 16-byte loads);
    // kL8: exact activations as int8 limbs (Q4_K / Q5_K; same C layout as kI8)
    constexpr bool kI8 = FMT != 8 && ACT == 1;
    constexpr bool kL8 = ACT == 0 && (FMT == 12 || FMT == 13);
    constexpr bool kIC = kI8 || kL8;  // C columns 2t, 2t+1 (else the exact fp16 layout)
    constexpr int UNITW = kI8 ? (int)(sizeof(BFragI8) / 4) * 32 : kL8 ? kL8Words : bunit_words(NT);
    constexpr int MTB = mtile_bytes(FMT);
    constexpr int STAGE = kRowsCW * MTB;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + 8;
    uint8_t *ring = smem + 128;
    uint32_t *bsm = reinterpret_cast<uint32_t *>(ring + (size_t)a.S * STAGE);
    float *ssq = reinterpret_cast<float *>(bsm + (size_t)a.nu * UNITW);  // XF 3: [nu][8]
    __shared__ float inv_s[8];
    __shared__ float part_s[16][8];
    __shared__ unsigned long long best_s[AM ? 8 : 1];
    __shared__ bool last_s;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // K halves (khalves 2): CTAs 2b and 2b + 1 take the same row groups, units
    // [0, nu/2) and [nu/2, nu); the second writes its partials to kpart
    const int kh = a.khalves == 2 ? (int)(blockIdx.x & 1) : 0;
    const int cb = a.khalves == 2 ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int ncb = a.khalves == 2 ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    const int ku0 = kh ? a.nu / 2 : 0, nku = a.khalves == 2 ? (kh ? a.nu - a.nu / 2 : a.nu / 2) : a.nu;
    // this CTA's row blocks [rb_lo, rb_hi), an even share (not whole groups:
    // the SM is issue-bound, so a last group of a few row blocks costs in
    // proportion), in groups of kRowsCW from rb_lo
    const int rb_lo = (int)((int64_t)cb * a.nrb / ncb);
    const int rb_hi = (int)((int64_t)(cb + 1) * a.nrb / ncb);
    const int ng = (rb_hi - rb_lo + kRowsCW - 1) / kRowsCW;
    const int total = ng * nku;
    if constexpr (AM) {
        if (tid < 8) best_s[tid] = 0ull;
    }
    auto issue = [&](int q) {  // one thread: stage q into its slot
        const int slot = q % a.S;
        const int gi = a.rev ? ng - 1 - q / nku : q / nku, u = ku0 + q % nku;
        const int rb0 = rb_lo + gi * kRowsCW;
        const int nrow = min(kRowsCW, rb_hi - rb0);
        fence_proxy_async();
        mbar_expect_tx(full + slot, (uint32_t)(nrow * MTB));
        for (int w = 0; w < nrow; w++) {
            const uint8_t *src = a.W + ((int64_t)(rb0 + w) * a.nu + u) * MTB;
            bulk_g2s(ring + (size_t)slot * STAGE + (size_t)w * MTB, src, (uint32_t)MTB, full + slot);
        }
    };
    pdl_trigger();
    // the weights are constant: the first stages stream in before the
    // previous kernel (producer of X) has finished
    if (tid == 0) {
        for (int s = 0; s < a.S; s++) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, kRowsCW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int q = 0; q < min(a.S, total); q++) issue(q);
    }
    pdl_wait();
    if (XF == 1) {  // RMSNorm of the input columns (rmsnorm_cpu!, ModelCPU.jl:111-123)
        float ss[8];
#pragma unroll
        for (int c = 0; c < 8; c++) ss[c] = 0.f;
        for (int64_t k = 4 * tid; k < a.K; k += 4 * 512) {
#pragma unroll
            for (int c = 0; c < 8; c++) {
                if (c < a.ncols) {
                    const float4 q = __ldg(reinterpret_cast<const float4 *>(a.X + c * a.ldx + k));
                    ss[c] += q.x * q.x + q.y * q.y + q.z * q.z + q.w * q.w;
                }
            }
        }
#pragma unroll
        for (int c = 0; c < 8; c++) {
            float v = ss[c];
#pragma unroll
            for (int o2 = 16; o2; o2 >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o2);
            if (lane == 0) part_s[warp][c] = v;
        }
        __syncthreads();
        if (tid < 8) {
            float v = 0.f;
            for (int w = 0; w < 16; w++) v += part_s[w][tid];
            inv_s[tid] = 1.0f / sqrtf(v / (float)a.K + a.eps);
        }
        __syncthreads();
    }
    // every unit's fragments, once per CTA
    if constexpr (kI8) {
        for (int u = warp; u < a.nu; u += 16) {
            BFragI8 Fr;
            build_b_i8<FMT, XF>(a, inv_s, u, lane, Fr);
            reinterpret_cast<BFragI8 *>(bsm)[u * 32 + lane] = Fr;
        }
    } else if constexpr (kL8) {
        for (int uu = warp; uu < nku; uu += 16)
            build_b_l8<FMT, XF>(a, inv_s, ku0 + uu, lane, bsm + (size_t)uu * UNITW, ssq);
    } else {
        for (int task = warp; task < nku * NT; task += 16)
            build_b<FMT, NT, XF>(a, inv_s, ku0 + task % nku, lane, task / nku, bsm + (size_t)(task % nku) * UNITW,
                                 ssq);
    }
    __syncthreads();
    if (XF == 3) {  // W (x w) / rms(x) per column; the sums of squares in unit order
        if (tid < 8) {
            float v = 0.f;
            if (tid < a.ncols)
                for (int uu = 0; uu < a.nu; uu++) v += ssq[uu * 8 + tid];
            inv_s[tid] = tid < a.ncols ? 1.0f / sqrtf(v / (float)a.K + a.eps) : 0.f;
        }
        __syncthreads();
    }
    bool dead = false;
    if (warp == kRowsCW) {
        // producer: refill each slot once its 15 consumers have released it
        if (lane == 0) {
            int q = min(a.S, total);  // stages issued so far
            while (q < total) {
                if (!mbar_wait(empty + (q % a.S), (uint32_t)((q / a.S) - 1) & 1)) break;
                issue(q++);
            }
            // the last copy into each slot has landed before the CTA exits
            // (consumed ones return at once)
            for (int r = max(0, q - a.S); r < q; r++) mbar_wait(full + (r % a.S), (uint32_t)(r / a.S) & 1);
        }
    } else {
        const int g = lane >> 2, t = lane & 3;
        // greedy keys: exact, column 4 nt + t of n-tile nt; Q8_K, column 2 t + j
        unsigned long long best[2] = {0ull, 0ull};
        int q = 0;
        for (int gi = 0; gi < ng; gi++) {
            const int gr = a.rev ? ng - 1 - gi : gi;
            const int rb = rb_lo + gr * kRowsCW + warp;
            float tot[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int i = 0; i < 4; i++) tot[nt][i] = 0.f;
            for (int u = 0; u < nku; u++, q++) {
                const int slot = q % a.S;
                if (!dead && !mbar_wait(full + slot, (uint32_t)(q / a.S) & 1)) dead = true;
                if (!dead && rb < rb_hi) {
                    const uint8_t *tile = ring + (size_t)slot * STAGE + (size_t)warp * MTB;
                    if constexpr (kI8) {
                        const BFragI8 F = reinterpret_cast<const BFragI8 *>(bsm)[u * 32 + lane];
                        if constexpr (FMT == 14) mtile_q6_i8(tile, lane, F, tot[0]);
                        else mtile_qk_i8<FMT == 13>(tile, lane, F, tot[0]);
                    } else if constexpr (kL8) {
                        mtile_qk_l8<FMT == 13>(tile, lane, reinterpret_cast<const uint2 *>(bsm + (size_t)u * UNITW) + lane,
                                               tot[0]);
                    } else {
                        BView<NT> F;
                        F.at(bsm + (size_t)u * UNITW, lane);
                        if constexpr (FMT == 8) mtile_q80<NT>(tile, lane, F, tot);
                        else if constexpr (FMT == 14) mtile_q6_h<NT>(tile, lane, F, tot);
                        else mtile_qk_h<FMT == 13, NT>(tile, lane, F, tot);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty + slot);
            }
            if (kIC && rb < rb_hi && !dead) {
                // C columns 2t, 2t+1: activation columns 2t, 2t+1
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const int col = 2 * t + j;
                    if (col >= a.ncols) continue;
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const int64_t row = (int64_t)rb * 16 + g + 8 * h;
                        if (row >= a.M) continue;
                        float v = tot[0][2 * h + j];
                        if (XF == 3) v *= inv_s[col];
                        if (kh) {  // the second K half: its partial, added by rows_khalf_add_kernel
                            a.kpart[(int64_t)col * a.M + row] = v;
                            continue;
                        }
                        float *y = a.Y + (int64_t)col * a.ldy + row;
                        if (a.accumulate) v += *y;
                        *y = v;
                        if constexpr (AM) {
                            const unsigned long long k = argmax_key(v, row);
                            best[j] = k > best[j] ? k : best[j];
                        }
                    }
                }
            }
            if (!kIC && rb < rb_hi && !dead) {
                // C columns 2t, 2t+1 of n-tile nt: hi and lo parts of column 4 nt + t
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    const int col = 4 * nt + t;
                    if (col >= a.ncols) continue;
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const int64_t row = (int64_t)rb * 16 + g + 8 * h;
                        if (row >= a.M) continue;
                        float v = tot[nt][2 * h] + tot[nt][2 * h + 1];
                        if (XF == 3) v *= inv_s[col];
                        if (kh) {  // the second K half: its partial, added by rows_khalf_add_kernel
                            a.kpart[(int64_t)col * a.M + row] = v;
                            continue;
                        }
                        float *y = a.Y + (int64_t)col * a.ldy + row;
                        if (a.accumulate) v += *y;
                        *y = v;
                        if constexpr (AM) {
                            const unsigned long long k = argmax_key(v, row);
                            best[nt] = k > best[nt] ? k : best[nt];
                        }
                    }
                }
            }
        }
        if constexpr (AM) {
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int col = kIC ? 2 * t + j : 4 * j + t;
                if ((kIC || j < NT) && col < a.ncols) atomicMax(&best_s[col], best[j]);
            }
        }
    }
    if constexpr (AM) {
        // every CTA leaves its per-column best, then counts itself done; the
        // CTA that finishes last (fenced counter, nothing waits) decides
        __syncthreads();
        if (tid < a.ncols) aa.am.cand[tid * gridDim.x + blockIdx.x] = best_s[tid];
        __threadfence();
        __syncthreads();
        if (tid == 0) last_s = atomicAdd(aa.am.counter, 1u) == gridDim.x - 1;
        __syncthreads();
        if (last_s) {
            __threadfence();
            if (tid < a.ncols) {
                unsigned long long b = 0ull;
                for (unsigned c = 0; c < gridDim.x; c++) {
                    const unsigned long long k = __ldcg(aa.am.cand + tid * gridDim.x + c);
                    b = k > b ? k : b;
                }
                best_s[tid] = b;
            }
            __syncthreads();
            const int G1 = aa.am.G + 1;
            if (tid < a.ncols / G1) {
                const int b = tid;
                int32_t *ot = aa.am.out + (int64_t)b * aa.am.out_ld;
                for (int i = 0; i < G1; i++) ot[i] = -1;
                int accn = 0;
                for (int i = 0; i < G1; i++) {
                    const int tok = (int)(0xFFFFFFFFu - (uint32_t)(best_s[b * G1 + i] & 0xFFFFFFFFull));
                    ot[i] = tok;
                    if (i == aa.am.G || tok != aa.am.drafts[(int64_t)b * aa.am.draft_ld + i]) break;
                    accn++;
                }
                if (aa.am.acc) aa.am.acc[b] = accn;
            }
            if (tid == 0) *aa.am.counter = 0u;
        }
    }
}

static int num_sms() { return device_sm_count(); }

// qgemv_rows_kernel with K halves: Y += the second half's partials, one add
// per output ((y + first half) + second half: a fixed order)
static __global__ void __launch_bounds__(256) rows_khalf_add_kernel(float *Y, int64_t ldy, const float *kpart, int64_t M,
                                                             int ncols) {
    pdl_trigger();
    pdl_wait();
    const int64_t n = M * ncols;
    for (int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x; i < n; i += (int64_t)gridDim.x * 256) {
        const int64_t col = i / M, row = i - col * M;
        Y[col * ldy + row] += kpart[i];
    }
}

template <int FMT, int NT, int XF, int MPW, int ACT, bool AM>
static cudaError_t launch_mpw(const QTensor &T, const float *X, int ncols, float *Y, bool accumulate, int64_t ldy,
                              cudaStream_t s, const XForm &xf, int UW) {
    constexpr int MTB = mtile_bytes(FMT);
    constexpr int CW = consumers<ACT>();
    constexpr int STAGE = CW * MPW * MTB;
    constexpr int kSmemMax = 226 * 1024;  // dynamic; 1 KB of the 227 KB per block stays for static shared memory
    const int MTG = CW * MPW / UW;
    const int red = 2 * CW * (MPW * NT * 4) * 32 * 4;
    const int64_t nrg = (T.nrb + MTG - 1) / MTG;
    const int grid = (int)(nrg < num_sms() ? nrg : num_sms());
    // ring stages first (2..5), then the shared accumulator gets the rest
    const int64_t per_cta = (nrg + grid - 1) / grid;
    const int64_t stages_per_cta = per_cta * ((T.nu + UW - 1) / UW);
    constexpr bool kExact = FMT == 8 || ACT == 0;
    const int bsm_bytes = kExact ? UW * bunit_words(NT) * 4 : 0;
    int S = (kSmemMax - 128 - red - bsm_bytes - 16 * 1024) / STAGE;
    S = S < 2 ? 2 : (S > 5 ? 5 : S);
    if (S > stages_per_cta) S = (int)stages_per_cta;  // small matrices: request only what is used
    const int ssq_bytes = XF == 3 ? (int)T.nu * 8 * 4 : 0;
    const int acc_bytes_avail = kSmemMax - 128 - S * STAGE - red - ssq_bytes - bsm_bytes;
    const int rg_bytes = MTG * 16 * 8 * 4;
    int sweep_rg = acc_bytes_avail / rg_bytes;
    if (sweep_rg < 1) return cudaErrorInvalidConfiguration;
    if (sweep_rg > per_cta) sweep_rg = (int)per_cta;
    const int smem = 128 + S * STAGE + red + sweep_rg * rg_bytes + ssq_bytes + bsm_bytes;
    if (smem > kSmemMax) return cudaErrorInvalidConfiguration;
    static DeviceFlags attr_set;
    if (!attr_set.test()) {
        cudaError_t e = cudaFuncSetAttribute(qgemv_kernel<FMT, NT, XF, MPW, ACT, AM>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(qgemv_kernel<FMT, NT, XF, MPW, ACT, AM>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 (int)cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) return e;
        attr_set.set();
    }
    GemvArgs a{T.data, T.rows, T.cols, (int)T.nrb, (int)T.nu, X, xf.ldx > 0 ? xf.ldx : T.cols, ncols, Y, UW, S,
               sweep_rg, accumulate ? 1 : 0, ldy, xf.kind, xf.w, xf.eps, xf.ep};
    AmArg<AM> aa{};
    if constexpr (AM) aa.am = *xf.am;
    return launch_k(qgemv_kernel<FMT, NT, XF, MPW, ACT, AM>, dim3(grid), dim3(32 * CW), (size_t)smem, s, a, aa);
}

// Tall matrices (>= 2 row groups of 15 row blocks per SM) without a SwiGLU
// input or epilogue take the row-block-per-warp kernel (either activation
// mode) when every unit's fragments and three ring slots fit in shared
// memory; returns
// cudaErrorNotSupported (nothing launched) otherwise.
template <int FMT, int NT, int XF, int ACT, bool AM>
static cudaError_t launch_rows(const QTensor &T, const float *X, int ncols, float *Y, bool accumulate, int64_t ldy,
                               cudaStream_t s, const XForm &xf) {
    constexpr int MTB = mtile_bytes(FMT);
    constexpr int STAGE = kRowsCW * MTB;
    constexpr int kSmemMax = 226 * 1024;
    constexpr bool kI8 = FMT != 8 && ACT == 1;
    const int64_t ngr = (T.nrb + kRowsCW - 1) / kRowsCW;
    if (xf.ep || ngr < 2 * num_sms()) return cudaErrorNotSupported;
    // Q4_K with Q8_K activations: the unit-split kernel (two M-tiles per warp)
    // streams faster (151936 x 4096, N = 5: 78.7 vs 90.9 us, measured)
    if (kI8 && FMT == 12) return cudaErrorNotSupported;
    constexpr bool kL8 = ACT == 0 && (FMT == 12 || FMT == 13);
    const int unit_bytes = kI8 ? (int)sizeof(BFragI8) * 32 : kL8 ? kL8Words * 4 : bunit_words(NT) * 4;
    int fixed = 128 + (int)T.nu * unit_bytes + (XF == 3 ? (int)T.nu * 8 * 4 : 0);
    int S = (kSmemMax - fixed) / STAGE;
    int khalves = 1;
    // exact activations over a long K (4096 with two n-tiles: 139 KB of
    // fragments): CTA pairs split K, each holding half the units' fragments,
    // when the caller gave scratch for the second half's partials (not with
    // the folded RMSNorm, whose scale needs every unit's sum of squares)
    if (S < 3 && !kI8 && XF != 3 && !AM && xf.kpart && xf.kpart_floats >= T.rows * ncols && T.nu >= 2) {
        fixed = 128 + (int)((T.nu + 1) / 2) * unit_bytes;
        S = (kSmemMax - fixed) / STAGE;
        khalves = 2;
    }
    if (S < 3) return cudaErrorNotSupported;  // two one-unit stages hide too little DRAM latency (measured)
    if (S > 8) S = 8;
    const int smem = fixed + S * STAGE;
    static DeviceFlags attr_set;
    if (!attr_set.test()) {
        cudaError_t e = cudaFuncSetAttribute(qgemv_rows_kernel<FMT, NT, XF, ACT, AM>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
        if (e != cudaSuccess) return e;
        attr_set.set();
    }
    const int grid = khalves == 2 ? num_sms() & ~1 : num_sms();
    GemvArgs a{T.data, T.rows, T.cols, (int)T.nrb, (int)T.nu, X, xf.ldx > 0 ? xf.ldx : T.cols, ncols, Y, 0, S,
               0, accumulate ? 1 : 0, ldy, xf.kind, xf.w, xf.eps, xf.ep, xf.rev, khalves, xf.kpart};
    AmArg<AM> aa{};
    if constexpr (AM) aa.am = *xf.am;
    cudaError_t e = launch_k(qgemv_rows_kernel<FMT, NT, XF, ACT, AM>, dim3(grid), dim3(512), (size_t)smem, s, a, aa);
    if (e != cudaSuccess || khalves == 1) return e;
    return launch_k(rows_khalf_add_kernel, dim3(2 * num_sms()), dim3(256), 0, s, Y, ldy, (const float *)xf.kpart,
                    (int64_t)T.rows, ncols);
}

// Work split: UW warps share each row block's units.  A stage: 16 warps x 1
// M-tile (exact activations: the fragments of UW units take shared memory),
// 16 warps x 2 (Q8_K activations; x 1 for Q6_K, whose larger tiles would leave
// one ring stage).  UW is the largest power of two <= 8 (and <= the units)
// whose two ring stages, fragments and partials fit in shared memory: exact
// Q8_0 (4352-byte M-tiles) with two n-tiles takes 4.
template <int FMT, int NT, int XF, int ACT>
static cudaError_t launch(const QTensor &T, const float *X, int ncols, float *Y, bool accumulate, int64_t ldy,
                          cudaStream_t s, const XForm &xf) {
    constexpr bool kExact = FMT == 8 || ACT == 0;
    constexpr int MPW = kExact ? 1 : (mtile_bytes(FMT) > 2816 ? 1 : 2);
    constexpr int CW = consumers<ACT>();
    if constexpr (XF != 2) {
        // exact Q4_K / Q5_K: the limb kernel (one n-tile of 8 columns whatever NT)
        constexpr int RNT = ACT == 0 && (FMT == 12 || FMT == 13) ? 1 : NT;
        const cudaError_t e = xf.am ? launch_rows<FMT, RNT, XF, ACT, true>(T, X, ncols, Y, accumulate, ldy, s, xf)
                                    : launch_rows<FMT, RNT, XF, ACT, false>(T, X, ncols, Y, accumulate, ldy, s, xf);
        if (e != cudaErrorNotSupported) return e;
    }
    constexpr int kSmemMax = 226 * 1024;
    int UW = 1;
    while (UW < 8 && UW * 2 <= T.nu) UW *= 2;
    for (; UW > 1; UW /= 2) {
        const int MTG = CW * MPW / UW;
        const int need = 128 + 2 * CW * MPW * mtile_bytes(FMT) + 2 * CW * (MPW * NT * 4) * 32 * 4 +
                         (kExact ? UW * bunit_words(NT) * 4 : 0) + MTG * 16 * 8 * 4 +
                         (XF == 3 ? (int)T.nu * 8 * 4 : 0);
        if (need <= kSmemMax) break;
    }
    if (xf.am) return launch_mpw<FMT, NT, XF, MPW, ACT, true>(T, X, ncols, Y, accumulate, ldy, s, xf, UW);
    return launch_mpw<FMT, NT, XF, MPW, ACT, false>(T, X, ncols, Y, accumulate, ldy, s, xf, UW);
}

template <int FMT, int NT, int XF>
static cudaError_t launch_act(const QTensor &T, const float *X, int ncols, float *Y, bool accumulate, int64_t ldy,
                              cudaStream_t s, const XForm &xf) {
    if constexpr (FMT == 8) return launch<FMT, NT, XF, 0>(T, X, ncols, Y, accumulate, ldy, s, xf);
    else if (xf.act == 1) return launch<FMT, 1, XF, 1>(T, X, ncols, Y, accumulate, ldy, s, xf);
    else return launch<FMT, NT, XF, 0>(T, X, ncols, Y, accumulate, ldy, s, xf);
}

template <int FMT>
static cudaError_t launch_fmt(const QTensor &T, const float *X, int ncols, float *Y, bool accumulate, int64_t ldy,
                              cudaStream_t s, const XForm &xf) {
    const bool two = ncols > 4 && (FMT == 8 || xf.act == 0);  // Q8_K: all 8 columns in one n-tile
    // RMSNorm input with exact activations: folded into the epilogue (W (x w)
    // / rms(x), the sums of squares formed from the loads that build B), so
    // no CTA reduces the whole input before its first MMA
    const bool fold = xf.kind == 1 && (FMT == 8 || xf.act == 0) && T.nu <= kMaxFoldUnits;
    switch (fold ? 3 : xf.kind) {
    case 0: return two ? launch_act<FMT, 2, 0>(T, X, ncols, Y, accumulate, ldy, s, xf) : launch_act<FMT, 1, 0>(T, X, ncols, Y, accumulate, ldy, s, xf);
    case 1: return two ? launch_act<FMT, 2, 1>(T, X, ncols, Y, accumulate, ldy, s, xf) : launch_act<FMT, 1, 1>(T, X, ncols, Y, accumulate, ldy, s, xf);
    case 3: return two ? launch<FMT, 2, 3, 0>(T, X, ncols, Y, accumulate, ldy, s, xf) : launch<FMT, 1, 3, 0>(T, X, ncols, Y, accumulate, ldy, s, xf);
    case 2: return two ? launch_act<FMT, 2, 2>(T, X, ncols, Y, accumulate, ldy, s, xf) : launch_act<FMT, 1, 2>(T, X, ncols, Y, accumulate, ldy, s, xf);
    }
    return cudaErrorInvalidValue;
}

#ifdef IFR_QGEMV_FMT
// this translation unit's weight format (qgemv_q4k.cu .. qgemv_q80.cu)
template <>
cudaError_t qgemm_small_fmt<IFR_QGEMV_FMT>(const QTensor &T, const float *X, int ncols, float *Y, bool accumulate,
                                           int64_t ldy, cudaStream_t s, const XForm &xf) {
    return launch_fmt<IFR_QGEMV_FMT>(T, X, ncols, Y, accumulate, ldy, s, xf);
}
template <>
cudaError_t read_dev_error_fmt<IFR_QGEMV_FMT>(int *flag, cudaStream_t s) {
    int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(flag, g_dev_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(g_dev_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    return e;
}
#endif  // IFR_QGEMV_FMT

}  // namespace ifr
