// Dense quantized GEMM on the 5th-generation tensor cores (tcgen05, TMEM):
// Y[n][r] = sum_k W[r][k] X[n][k] for many columns at once - the verify
// columns of a batch of requests, or prompt chunks - with W in Q4_K / Q5_K /
// Q6_K / Q8_0 (M-tile layout, tiles.cuh).  The N <= 8 verify GEMV (qgemv.cu)
// is HBM-bound; here the contraction is dense enough for the tensor cores.
//
// Precision (stated; this is not the exact path): weights are formed in fp16
// from their exact integer quants - Q4_K/Q5_K fma(q, fp16(d sc), -fp16(dmin m)),
// Q6_K (q - 32) fp16(d sc), Q8_0 q d, each rounded once - and every activation
// column is scaled by a power of two (max |x| -> [2^13, 2^14)) and rounded to
// fp16; products are summed in f32 in tensor memory.
//
// One CTA computes 128 output rows x a tile of up to 512 columns (MMA chunks
// of <= 256) over a range of K units (split-K over blockIdx.y when the rows
// alone give too few CTAs):
//   warp 0     weight producer: cp.async.bulk of the raw M-tiles of each
//              256-column unit into a ring of 2-3 slots (no dependency on the
//              previous kernel, so it runs ahead from the first cycle);
//   warp 1     allocates the accumulators in tensor memory; one thread issues
//              tcgen05.mma (M = 128, N = chunk, K = 16) per chunk, four K steps
//              per stage, and tcgen05.commit, which frees the stage;
//   warp 2     activation producer: cp.async.bulk of the packed fp16
//              activations of each 64-wide K stage (ring of ST);
//   warps 3-18 dequantize each stage's 128 x 64 weights into the canonical
//              K-major (no swizzle) shared-memory layout of the MMA, then read
//              the f32 accumulators back (tcgen05.ld) and write Y or the split
//              partials.
// Shared-memory operand layout (both operands K-major, 16-byte core-matrix
// rows): element (row, k) of a 64-wide stage lives at
//   (k / 8) * (rows * 16) + row * 16 + (k % 8) * 2,
// i.e. the descriptor's stride between 8-row groups is 128 bytes and between
// the two 8-element K halves of one MMA it is rows * 16 bytes.
// Every mbarrier wait is bounded (~2 s); on expiry the CTA records an error
// flag, the roles stop, in-flight copies and MMAs are drained and the host
// reports IFR_ERR_TIMEOUT.  No cluster multicast is used.
#include "common.cuh"
#include "tiles.cuh"

#include <type_traits>

namespace ifr {

__device__ int g_mma_error = 0;

namespace {

constexpr int kDqWarps = 16;
constexpr int kDqThreads = 32 * kDqWarps;
constexpr int kMmaThreads = 96 + kDqThreads;  // producer, MMA, activation producer, dequant warps
constexpr int kMaxRaw = 3;                    // raw weight ring slots (units)
constexpr int kMaxStages = 4;                 // operand stages (64-wide K)
constexpr int kBM = 128;                 // rows per CTA (8 row blocks)
// A tile: 8 K-chunks of 128 rows x 16 bytes; chunks 2112 bytes apart (2048 + 64)
// so that the two halves of a warp's 64-bit stores hit disjoint banks
constexpr int kALbo = 2112;
// A tile of a stage of KS x 64 K: 8 KS chunks
IFR_HD int a_stage_bytes(int ks) { return (8 * ks - 1) * kALbo + kBM * 16 + 64; }
constexpr int kMaxSmem = 232448;         // 227 KB per block
constexpr long long kMmaWait = 4000000000LL;  // ~2 s at 1.9 GHz

IFR_DEV uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

IFR_DEV void mb_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count) : "memory");
}
IFR_DEV void mb_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
IFR_DEV void mb_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
IFR_DEV bool mb_try(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(su32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait that also gives up once another role of the CTA has (dead)
IFR_DEV bool mb_wait(uint64_t *b, uint32_t parity, volatile int *dead) {
    if (mb_try(b, parity)) return true;
    const long long t0 = clock64();
    while (!mb_try(b, parity)) {
        if (*dead) return false;
        if (clock64() - t0 > kMmaWait) {
            *dead = 1;
            atomicExch(&g_mma_error, 1);
            return false;
        }
    }
    return true;
}
// bounded wait used only to drain (ignores the dead flag)
IFR_DEV void mb_drain(uint64_t *b, uint32_t parity) {
    const long long t0 = clock64();
    while (!mb_try(b, parity))
        if (clock64() - t0 > kMmaWait) {
            atomicExch(&g_mma_error, 1);
            return;
        }
}
IFR_DEV void bulk_copy(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(su32(dst)),
        "l"(src), "r"(bytes), "r"(su32(bar))
        : "memory");
}
IFR_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---- tcgen05 ------------------------------------------------------------------
IFR_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
IFR_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
IFR_DEV void tmem_alloc(uint32_t *holder, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(holder)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
IFR_DEV void tmem_free(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// shared-memory matrix descriptor, no swizzle: start, K-half stride (lbo),
// 8-row-group stride (sbo), all in bytes; bit 46 = descriptor version 1 (sm_100)
IFR_DEV uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// instruction descriptor of kind::f16: D f32, A and B fp16, both K-major, M = 128
IFR_HD uint32_t mma_idesc(int n) { return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24); }
IFR_DEV void mma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
IFR_DEV void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
                 : "memory");
}
// 16 consecutive f32 columns of this thread's TMEM lane
IFR_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

IFR_DEV uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
IFR_DEV uint2 lds64(const uint8_t *p) { return *reinterpret_cast<const uint2 *>(p); }
IFR_DEV uint32_t wsel(const uint4 &v, int w) { return w == 0 ? v.x : w == 1 ? v.y : w == 2 ? v.z : v.w; }
IFR_DEV uint32_t pack_h2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// ---- dequantization of one piece ------------------------------------------------
// A piece is (M-tile row r, lane quad t) of one 64-element K stage p of a unit:
// the 16 elements 64 p + 16 w + 4 t + b (run w = 0..3, b = 0..3), exactly the
// bytes the M-tile keeps together for t (tiles.cuh).  out[2 w], out[2 w + 1]
// hold run w as fp16 pairs (b = 0, 2) and (b = 1, 3): the MMA's K slots of
// every group of four hold the elements (0, 2, 1, 3), and the activations are
// packed in the same order.  Arithmetic in fp16 from exact integers
// (magic-number unpack): Q4_K/Q5_K fma(q, fp16(d sc), -fp16(dmin m)), Q6_K
// (q - 32) fp16(d sc), Q8_0 q d, each rounded once.
constexpr uint32_t kMagic = 0x64006400u;  // (1024, 1024)

IFR_DEV uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
IFR_DEV uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
IFR_DEV uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}
IFR_DEV uint32_t and_or(uint32_t a, uint32_t mask, uint32_t orv) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));
    return r;
}

// fp16 pair (lo, hi) of bytes a and b of w (0 <= byte <= 255 exactly)
IFR_DEV uint32_t byte_pair_h2(uint32_t w, uint32_t sel) { return hsub2(__byte_perm(w, 0u, sel) | kMagic, kMagic); }
constexpr uint32_t kSelB01 = 0x4140u, kSelB23 = 0x4342u;   // bytes (0, 1), (2, 3) into the two halves
IFR_DEV uint32_t dup_lo(uint32_t h2) { return __byte_perm(h2, 0u, 0x1010u); }
IFR_DEV uint32_t dup_hi(uint32_t h2) { return __byte_perm(h2, 0u, 0x3232u); }

// Per-thread dequantizer of one piece (M-tile row r, lane quad t) across the
// four stages p = 0..3 of a unit: unit() decodes the block header once,
// stage(p) produces the 16 fp16 weights of stage p.
template <bool Q5>
struct DeqK {
    const uint8_t *tile;
    int r, t;
    uint32_t dsc[4], nmn[4];  // (sub-blocks 2p, 2p+1): fp16(d sc), -fp16(dmin m)
    uint2 qh;
    uint4 qs;                 // qs piece of stages 2q, 2q+1
    IFR_DEV void unit(const uint8_t *tl, int r_, int t_) {
        tile = tl;
        r = r_;
        t = t_;
        const uint4 h = lds128(tile + qk_hdr(r));
        const uint32_t dd = (h.x & 0xffffu) * 0x10001u, dm = (h.x >> 16) * 0x10001u;
        // 6-bit scales and mins (src/Dequant.jl:345-362), byte j of word j / 4
        const uint32_t sc0 = h.y & 0x3f3f3f3fu, mn0 = h.z & 0x3f3f3f3fu;
        const uint32_t sc1 = (h.w & 0x0f0f0f0fu) | (((h.y >> 6) & 0x03030303u) << 4);
        const uint32_t mn1 = ((h.w >> 4) & 0x0f0f0f0fu) | (((h.z >> 6) & 0x03030303u) << 4);
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const uint32_t sel = (p & 1) ? kSelB23 : kSelB01;
            dsc[p] = hmul2(byte_pair_h2(p < 2 ? sc0 : sc1, sel), dd);
            nmn[p] = hmul2(byte_pair_h2(p < 2 ? mn0 : mn1, sel), dm) ^ 0x80008000u;
        }
        if (Q5) qh = lds64(tile + q5_qh(r & 7, t) + 8 * (r >> 3));
    }
    // raw qs bytes 32 p + 16 hh + 4 t + b: low nibble element 64 p + 16 hh + 4 t + b,
    // high nibble element 64 p + 32 + 16 hh + 4 t + b
    IFR_DEV void stage(int p, uint32_t (&o)[8]) {
        if ((p & 1) == 0) qs = lds128(tile + qk_qs(Q5, p >> 1, r, t));
        const uint32_t dl = dup_lo(dsc[p]), dh = dup_hi(dsc[p]), ml = dup_lo(nmn[p]), mh = dup_hi(nmn[p]);
        const int cl = 2 * p, ch = 2 * p + 1;
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
            const uint32_t W = (p & 1) ? (hh ? qs.w : qs.z) : (hh ? qs.y : qs.x);
            uint32_t l02 = and_or(W, 0x000F000Fu, kMagic), l13 = and_or(W >> 8, 0x000F000Fu, kMagic);
            uint32_t h02 = and_or(W >> 4, 0x000F000Fu, kMagic), h13 = and_or(W >> 12, 0x000F000Fu, kMagic);
            if (Q5) {
                // fifth bit: bit (sub-block) of qh byte b -> +16
                const uint32_t H = hh ? qh.y : qh.x;
                l02 |= ((H >> cl) & 0x00010001u) << 4;
                l13 |= ((H >> (8 + cl)) & 0x00010001u) << 4;
                h02 |= ((H >> ch) & 0x00010001u) << 4;
                h13 |= ((H >> (8 + ch)) & 0x00010001u) << 4;
            }
            o[2 * hh] = hfma2(hsub2(l02, kMagic), dl, ml);
            o[2 * hh + 1] = hfma2(hsub2(l13, kMagic), dl, ml);
            o[4 + 2 * hh] = hfma2(hsub2(h02, kMagic), dh, mh);
            o[4 + 2 * hh + 1] = hfma2(hsub2(h13, kMagic), dh, mh);
        }
    }
};

// Q6_K (src/Dequant.jl:558-601): element 64 p + 32 j + 16 hh + 4 t + b is raw ql
// byte 64 (p / 2) + 32 j + 16 hh + 4 t + b >> 4 (p % 2), raw qh byte
// 32 (p / 2) + 16 hh + 4 t + b >> (4 (p % 2) + 2 j), scale group 4 p + 2 j + hh
struct DeqQ6 {
    const uint8_t *tile;
    int r, t;
    uint32_t ds[8];  // (groups 2i, 2i+1): fp16(d sc)
    uint4 qh, ql;
    IFR_DEV void unit(const uint8_t *tl, int r_, int t_) {
        tile = tl;
        r = r_;
        t = t_;
        const uint32_t dd = (uint32_t)(*reinterpret_cast<const uint16_t *>(tile + q6_d(r))) * 0x10001u;
        const uint4 sc = lds128(tile + q6_sc(r));
        constexpr uint32_t k1152 = 0x64806480u;  // (1024 + 128) x 2: int8 + 128 -> int8
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint32_t b = (__byte_perm(wsel(sc, i >> 1), 0u, (i & 1) ? kSelB23 : kSelB01) ^ 0x00800080u) | kMagic;
            ds[i] = hmul2(hsub2(b, k1152), dd);
        }
        qh = lds128(tile + q6_qh(r, t));
    }
    IFR_DEV void stage(int p, uint32_t (&o)[8]) {
        constexpr uint32_t k1056 = 0x64206420u;  // (1024 + 32) x 2
        if ((p & 1) == 0) ql = lds128(tile + q6_ql(p >> 1, r, t));
        const int sl = 4 * (p & 1), n = p >> 1;
#pragma unroll
        for (int j = 0; j < 2; j++) {
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                const uint32_t L = wsel(ql, 2 * j + hh) >> sl, H = wsel(qh, 2 * n + hh) >> (sl + 2 * j);
                const uint32_t d2 = hh ? dup_hi(ds[2 * p + j]) : dup_lo(ds[2 * p + j]);
                const uint32_t q02 = and_or(L, 0x000F000Fu, kMagic) | ((H << 4) & 0x00300030u);
                const uint32_t q13 = and_or(L >> 8, 0x000F000Fu, kMagic) | ((H >> 4) & 0x00300030u);
                o[2 * (2 * j + hh)] = hmul2(hsub2(q02, k1056), d2);
                o[2 * (2 * j + hh) + 1] = hmul2(hsub2(q13, k1056), d2);
            }
        }
    }
};

// Q8_0 (src/Dequant.jl:304-321): element 64 p + 16 w + 4 t + b of the unit is
// byte b of word w of piece (p, r, t), block 2 p + w / 2
struct DeqQ8 {
    const uint8_t *tile;
    int r, t;
    uint4 dd;  // block scales, blocks (2p, 2p+1) in word p
    IFR_DEV void unit(const uint8_t *tl, int r_, int t_) {
        tile = tl;
        r = r_;
        t = t_;
        dd = lds128(tile + q8_d(r));
    }
    IFR_DEV void stage(int p, uint32_t (&o)[8]) {
        constexpr uint32_t k1152 = 0x64806480u;  // (1024 + 128) x 2
        const uint4 q = lds128(tile + q8_qs(p, r, t));
        const uint32_t d0 = dup_lo(wsel(dd, p)), d1 = dup_hi(wsel(dd, p));
#pragma unroll
        for (int w = 0; w < 4; w++) {
            const uint32_t W = wsel(q, w) ^ 0x80808080u;  // int8 + 128
            o[2 * w] = hmul2(hsub2(and_or(W, 0x00FF00FFu, kMagic), k1152), w < 2 ? d0 : d1);
            o[2 * w + 1] = hmul2(hsub2(and_or(W >> 8, 0x00FF00FFu, kMagic), k1152), w < 2 ? d0 : d1);
        }
    }
};

template <int FMT>
using Deq = std::conditional_t<FMT == 12, DeqK<false>,
                               std::conditional_t<FMT == 13, DeqK<true>, std::conditional_t<FMT == 14, DeqQ6, DeqQ8>>>;

}  // namespace

// position in a ring of n slots: slot, and how often the ring has wrapped
struct Ring {
    int n, slot = 0, round = 0;
    IFR_DEV void next() {
        if (++slot == n) {
            slot = 0;
            ++round;
        }
    }
    IFR_DEV uint32_t full_par() const { return (uint32_t)round & 1; }         // data of this round landed
    IFR_DEV uint32_t empty_par() const { return (uint32_t)(round - 1) & 1; }  // previous round consumed
};

struct MmaArgs {
    const uint8_t *W;      // M-tiles
    int nrb, nu;           // row blocks of 16, units of 256
    const uint16_t *Xp;    // packed fp16 activations [ntiles][nu * 4][8][npad][8]
    const float *xinv;     // [ntiles * npad] 2^-e of each column
    int ncols, npad, ntiles, nch, splits, RS, ST;
    float *Y;
    int64_t ldy, M;
    int accumulate, ep;
    float *ws;             // split partials [splits][ncols][nrb * 16] (splits > 1)
    const uint8_t *wf16;   // fp16 operand stages of W (QTensor::f16), or null: dequantize
};

// KS: 64-wide K sub-stages per pipeline stage (2 when the column tile is <= 256,
// so that one tcgen05.commit covers at least eight MMAs)
template <int FMT, int KS>
__global__ void __launch_bounds__(kMmaThreads, 1) qmma_kernel(MmaArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr int MTB = mtile_bytes(FMT);
    constexpr int RAW = 8 * MTB;
    const int RS = a.RS, ST = a.ST, npad = a.npad;
    uint64_t *raw_full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *raw_empty = raw_full + kMaxRaw;
    uint64_t *a_full = raw_empty + kMaxRaw;
    uint64_t *b_full = a_full + kMaxStages;
    uint64_t *ab_empty = b_full + kMaxStages;
    uint64_t *acc_full = ab_empty + kMaxStages;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(acc_full + 1);
    volatile int *dead = reinterpret_cast<volatile int *>(tmem_holder + 1);
    uint8_t *raw = smem + 1024;
    const int raw_bytes = a.wf16 ? 0 : (RS * RAW + 1023) & ~1023;  // fp16 stages: no raw ring (make_plan)
    constexpr int kAStage = a_stage_bytes(KS);
    const int bstage = npad * 128 * KS;
    const int stage_bytes = (kAStage + bstage + 1023) & ~1023;
    uint8_t *stages = raw + raw_bytes;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rt = blockIdx.x / a.ntiles, nt = blockIdx.x % a.ntiles, z = blockIdx.y;
    const int rb0 = rt * 8;
    const int nmt = min(8, a.nrb - rb0);
    const int u0 = (int)((int64_t)z * a.nu / a.splits), u1 = (int)((int64_t)(z + 1) * a.nu / a.splits);
    const int nunits = u1 - u0, nst = 4 / KS * nunits;
    const uint32_t tcols = npad <= 32 ? 32 : npad <= 64 ? 64 : npad <= 128 ? 128 : npad <= 256 ? 256 : 512;

    pdl_trigger();
    if (tid == 0) {
        for (int i = 0; i < RS; i++) {
            mb_init(raw_full + i, 1);
            mb_init(raw_empty + i, kDqThreads);
        }
        for (int i = 0; i < ST; i++) {
            mb_init(a_full + i, kDqThreads);
            mb_init(b_full + i, 1);
            mb_init(ab_empty + i, 1);
        }
        mb_init(acc_full, 1);
        *dead = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) tmem_alloc(tmem_holder, tcols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    const bool f16w = a.wf16 != nullptr;
    if (warp == 0) {
        // ---------------- weight producer (constant data: no dependency wait) ----------------
        if (lane == 0 && !f16w) {
            Ring rr{RS};
            const uint8_t *src = a.W + ((int64_t)rb0 * a.nu + u0) * MTB;
            const int64_t rb_stride = (int64_t)a.nu * MTB;
            int issued = 0;
            for (int i = 0; i < nunits && !*dead; i++, rr.next(), src += MTB) {
                if (rr.round > 0 && !mb_wait(raw_empty + rr.slot, rr.empty_par(), dead)) break;
                fence_async_smem();
                mb_expect_tx(raw_full + rr.slot, (uint32_t)(nmt * MTB));
                uint8_t *dst = raw + rr.slot * RAW;
                for (int m = 0; m < nmt; m++) bulk_copy(dst + m * MTB, src + m * rb_stride, MTB, raw_full + rr.slot);
                issued = i + 1;
            }
            // no copy may land after the CTA exits: a slot is reissued only after its
            // previous contents were consumed, so only the last RS issues can be in flight
            for (int k = 0; k < RS && k < issued; k++) {
                const int i = issued - 1 - k;
                mb_drain(raw_full + i % RS, (uint32_t)(i / RS) & 1);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const int cw = npad / a.nch;
            const uint32_t idesc = mma_idesc(cw);
            const uint32_t s0 = su32(stages);
            const uint64_t da = smem_desc(s0, kALbo, 128), db = smem_desc(s0 + kAStage, npad * 16, 128);
            Ring ab{ST};
            for (int q = 0; q < nst; q++, ab.next()) {
                if ((!f16w && !mb_wait(a_full + ab.slot, ab.full_par(), dead)) ||
                    !mb_wait(b_full + ab.slot, ab.full_par(), dead))
                    break;
                tc_fence_after();
                const uint32_t so = (uint32_t)(ab.slot * stage_bytes) >> 4;  // descriptor start fields advance in 16 B
#pragma unroll
                for (int s = 0; s < 4 * KS; s++)
                    for (int c = 0; c < a.nch; c++)
                        mma_f16(tmem + (uint32_t)(c * cw), da + so + (s * 2 * kALbo >> 4),
                                db + so + (uint32_t)((s * 2 * npad + c * cw) * 16 >> 4), idesc, (q | s) != 0);
                mma_commit(ab_empty + ab.slot);
            }
            mma_commit(acc_full);
            mb_drain(acc_full, 0);  // every MMA has completed before TMEM is released
        }
        __syncwarp();
    } else if (warp == 2) {
        // ---------------- activation producer ----------------
        if (lane == 0) {
            pdl_wait();  // the activations come from the previous kernel
            Ring ab{ST};
            const uint16_t *src = a.Xp + ((int64_t)nt * a.nu * 4 + 4 * u0) * (int64_t)npad * 64;
            // fp16 weights: the row tile's operand stages from unit u0 on, KS per stage
            const uint8_t *wsrc = f16w ? a.wf16 + ((int64_t)rt * a.nu + u0) * 4 * kF16StageBytes : nullptr;
            int issued = 0;
            for (int q = 0; q < nst && !*dead; q++, ab.next(), src += npad * 64 * KS) {
                if (ab.round > 0 && !mb_wait(ab_empty + ab.slot, ab.empty_par(), dead)) break;
                mb_expect_tx(b_full + ab.slot, (uint32_t)(bstage + (f16w ? kAStage : 0)));
                if (f16w)
                    bulk_copy(stages + ab.slot * stage_bytes, wsrc + (int64_t)q * kAStage, (uint32_t)kAStage,
                              b_full + ab.slot);
                bulk_copy(stages + ab.slot * stage_bytes + kAStage, src, (uint32_t)bstage, b_full + ab.slot);
                issued = q + 1;
            }
            for (int k = 0; k < ST && k < issued; k++) {
                const int q = issued - 1 - k;
                mb_drain(b_full + q % ST, (uint32_t)(q / ST) & 1);
            }
        }
    } else {
        // ---------------- dequant, then epilogue ----------------
        pdl_wait();
        // one piece per thread: M-tile m, row r, lane quad t, the same in every stage
        const int P = tid - 96;
        const int m = P >> 6, r = (P >> 2) & 15, t = P & 3;
        const int off = (t >> 1) * kALbo + (16 * m + r) * 16 + (t & 1) * 8;  // run w adds 2 w kALbo
        const bool has_rows = m < nmt;
        Deq<FMT> dq;
        Ring rr{RS}, ab{ST};
        for (int i = 0; i < nunits && !*dead && !f16w; i++, rr.next()) {
            if (!mb_wait(raw_full + rr.slot, rr.full_par(), dead)) break;
            if (has_rows) dq.unit(raw + rr.slot * RAW + m * MTB, r, t);
            bool ok = true;
#pragma unroll
            for (int j = 0; j < 4 / KS; j++, ab.next()) {
                if (ab.round > 0 && !mb_wait(ab_empty + ab.slot, ab.empty_par(), dead)) {
                    ok = false;
                    break;
                }
                uint8_t *A = stages + ab.slot * stage_bytes + off;
#pragma unroll
                for (int ss = 0; ss < KS; ss++) {
                    uint32_t o[8];
                    if (has_rows) {
                        dq.stage(KS * j + ss, o);
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; e++) o[e] = 0u;
                    }
#pragma unroll
                    for (int w = 0; w < 4; w++)
                        *reinterpret_cast<uint2 *>(A + (8 * ss + 2 * w) * kALbo) = make_uint2(o[2 * w], o[2 * w + 1]);
                }
                fence_async_smem();
                mb_arrive(a_full + ab.slot);
            }
            if (!ok) break;
            mb_arrive(raw_empty + rr.slot);
        }
        // epilogue: TMEM lane quarter (warp % 4) = rows 32 (warp % 4) ..; the four warps
        // of a quarter take every fourth 16-column chunk
        const bool have = __all_sync(0xffffffffu, mb_wait(acc_full, 0, dead));
        tc_fence_after();
        const int quarter = warp & 3, cgrp = (warp - 3) >> 2;
        const int64_t row = (int64_t)rb0 * 16 + 32 * quarter + lane;
        for (int c0 = 16 * cgrp; c0 < npad; c0 += 64) {
            uint32_t rv[16];
            tmem_ld16(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)c0, rv);
            if (!have) continue;
#pragma unroll
            for (int c = 0; c < 16; c++) {
                const int col = nt * npad + c0 + c;
                const float val = col < a.ncols ? __uint_as_float(rv[c]) * a.xinv[col] : 0.f;
                if (a.splits > 1) {
                    if (col < a.ncols && row < (int64_t)a.nrb * 16)
                        a.ws[((int64_t)z * a.ncols + col) * ((int64_t)a.nrb * 16) + row] = val;
                } else if (a.ep) {
                    // rows 32 P + (0..15) gate, 32 P + 16 + (0..15) up -> output 16 P + (0..15)
                    const float up = __shfl_down_sync(0xffffffffu, val, 16);
                    const int64_t j = (row >> 5) * 16 + lane;
                    if (lane < 16 && col < a.ncols && j < a.M / 2)
                        a.Y[(int64_t)col * a.ldy + j] = glu_act(a.ep, val, up);
                } else if (col < a.ncols && row < a.M) {
                    float *y = a.Y + (int64_t)col * a.ldy + row;
                    *y = a.accumulate ? *y + val : val;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_free(tmem, tcols);
    }
}

// The fp16 operand stages of W (QTensor::f16): block (row tile rt, unit u),
// 512 threads, each the piece (M-tile m, row r, lane quad t) the dequant
// warps of qmma_kernel form, written for the unit's four 64-K stages at the
// same offsets - so a stage copied from here equals the stage the kernel
// would have built (rows past the matrix are zero).
template <int FMT>
__global__ void __launch_bounds__(kDqThreads) qmma_f16_stages_kernel(const uint8_t *__restrict__ W, int nrb, int nu,
                                                                     uint8_t *__restrict__ out) {
    constexpr int MTB = mtile_bytes(FMT);
    const int rt = blockIdx.x, u = blockIdx.y, P = threadIdx.x;
    const int m = P >> 6, r = (P >> 2) & 15, t = P & 3;
    const int off = (t >> 1) * kALbo + (16 * m + r) * 16 + (t & 1) * 8;
    const bool has_rows = rt * 8 + m < nrb;
    Deq<FMT> dq;
    if (has_rows) dq.unit(W + ((int64_t)(rt * 8 + m) * nu + u) * MTB, r, t);
    uint8_t *base = out + ((int64_t)rt * nu + u) * 4 * kF16StageBytes + off;
#pragma unroll
    for (int p = 0; p < 4; p++) {
        uint32_t o[8];
        if (has_rows) {
            dq.stage(p, o);
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) o[e] = 0u;
        }
#pragma unroll
        for (int w = 0; w < 4; w++)
            *reinterpret_cast<uint2 *>(base + p * kF16StageBytes + 2 * w * kALbo) = make_uint2(o[2 * w], o[2 * w + 1]);
    }
}

// pack_x_kernel for columns too long to hold in shared memory: every pass
// (sum of squares, max, pack) reads the column again
template <int XF>
__global__ void __launch_bounds__(256) pack_x_stream_kernel(const float *__restrict__ X, int64_t ldx, int64_t K, int ncols,
                                                     int npad, int nu, const float *__restrict__ xw, float eps,
                                                     uint16_t *__restrict__ Xp, float *__restrict__ xinv) {
    __shared__ float red[8];
    __shared__ float bc;
    pdl_trigger();
    pdl_wait();
    const int col = blockIdx.x, tile = col / npad, n = col % npad;  // tiles hold consecutive columns
    const int tid = threadIdx.x;
    const int64_t nchunks = (int64_t)nu * 32;  // 8-element chunks of the padded K
    const bool has = col < ncols;
    const float *xc = X + (int64_t)col * ldx;
    auto block_reduce = [&](float v, bool is_max) {
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float w = __shfl_xor_sync(0xffffffffu, v, o);
            v = is_max ? fmaxf(v, w) : v + w;
        }
        __syncthreads();
        if ((tid & 31) == 0) red[tid >> 5] = v;
        __syncthreads();
        if (tid == 0) {
            float r = red[0];
            for (int w = 1; w < 8; w++) r = is_max ? fmaxf(r, red[w]) : r + red[w];
            bc = r;
        }
        __syncthreads();
        return bc;
    };
    float inv = 1.f;
    if (XF == 1 && has) {
        float ss = 0.f;
        for (int64_t k = tid; k < K; k += 256) ss += xc[k] * xc[k];
        ss = block_reduce(ss, false);
        inv = 1.0f / sqrtf(ss / (float)K + eps);
    }
    auto value = [&](int64_t k) -> float {
        if (!has || k >= K) return 0.f;
        float x = xc[k];
        if (XF == 1) x = x * inv * xw[k];
        if (XF == 2) x = x / (1.0f + expf(-x)) * xc[K + k];
        return x;
    };
    float mx = 0.f;
    for (int64_t k = tid; k < K; k += 256) mx = fmaxf(mx, fabsf(value(k)));
    mx = block_reduce(mx, true);
    int e = 0;
    if (mx > 0.f && !isinf(mx)) {
        int ex;
        frexpf(mx, &ex);
        e = 14 - ex;
        e = e < -100 ? -100 : (e > 100 ? 100 : e);
    }
    const float scl = __int_as_float((e + 127) << 23);
    if (tid == 0) xinv[col] = has ? __int_as_float((127 - e) << 23) : 0.f;
    for (int64_t c = tid; c < nchunks; c += 256) {
        const int64_t kst = c >> 3, ch = c & 7, k0 = 8 * c;
        const uint4 w = make_uint4(pack_h2(value(k0) * scl, value(k0 + 2) * scl),
                                   pack_h2(value(k0 + 1) * scl, value(k0 + 3) * scl),
                                   pack_h2(value(k0 + 4) * scl, value(k0 + 6) * scl),
                                   pack_h2(value(k0 + 5) * scl, value(k0 + 7) * scl));
        *reinterpret_cast<uint4 *>(Xp + ((((int64_t)tile * nu * 4 + kst) * 8 + ch) * npad + n) * 8) = w;
    }
}

// pack the columns of one n-tile to fp16 in the per-stage operand layout,
// scaled by 2^e per column (max |x| 2^e in [2^13, 2^14)), the K slots of each
// group of four holding the elements (0, 2, 1, 3) like the weights; the
// activation transform of the GEMV (RMSNorm, SwiGLU) is applied on the way.
// One CTA per column; the column is read from global memory once, in batches
// of eight loads per thread issued before their use, into shared memory
// (nu * 256 floats), and the max and pack passes read it there.  Every value
// and sum is formed in the same order as by pack_x_stream_kernel (thread tid
// sums elements tid, tid + 256, ... in turn), so the results are the same bits.
constexpr int kPackSmemMax = 192 * 1024;
template <int XF>
__global__ void __launch_bounds__(256) pack_x_kernel(const float *__restrict__ X, int64_t ldx, int64_t K, int ncols,
                                                     int npad, int nu, const float *__restrict__ xw, float eps,
                                                     uint16_t *__restrict__ Xp, float *__restrict__ xinv) {
    extern __shared__ __align__(16) float xs[];  // [nu * 256] the column's values (0 past K)
    __shared__ float red[8];
    __shared__ float bc;
    pdl_trigger();
    pdl_wait();
    const int col = blockIdx.x, tile = col / npad, n = col % npad;  // tiles hold consecutive columns
    const int tid = threadIdx.x;
    const int64_t KP = (int64_t)nu * 256, nchunks = (int64_t)nu * 32;
    const bool has = col < ncols;
    const float *xc = X + (int64_t)col * ldx;
    auto block_reduce = [&](float v, bool is_max) {
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float w = __shfl_xor_sync(0xffffffffu, v, o);
            v = is_max ? fmaxf(v, w) : v + w;
        }
        __syncthreads();
        if ((tid & 31) == 0) red[tid >> 5] = v;
        __syncthreads();
        if (tid == 0) {
            float r = red[0];
            for (int w = 1; w < 8; w++) r = is_max ? fmaxf(r, red[w]) : r + red[w];
            bc = r;
        }
        __syncthreads();
        return bc;
    };
    constexpr int LB = 8;  // loads in flight per thread
    // 1. the column (SwiGLU: silu(gate) * up) into shared memory; RMSNorm: raw
    //    values and their sum of squares
    float ss = 0.f, mx = 0.f;
    for (int64_t k0 = tid; k0 < KP; k0 += 256 * LB) {
        float g[LB], u[LB];
#pragma unroll
        for (int i = 0; i < LB; i++) {
            const int64_t k = k0 + 256 * i;
            const bool in = has && k < K;
            g[i] = in ? xc[k] : 0.f;
            u[i] = (XF == 2 && in) ? xc[K + k] : 0.f;
        }
#pragma unroll
        for (int i = 0; i < LB; i++) {
            const int64_t k = k0 + 256 * i;
            if (k < KP) {
                float v = g[i];
                if (XF == 1) ss += v * v;
                if (XF == 2) v = (has && k < K) ? v / (1.0f + expf(-v)) * u[i] : 0.f;
                if (XF != 1) mx = fmaxf(mx, fabsf(v));
                xs[k] = v;
            }
        }
    }
    if (XF == 1) {
        // 2. RMSNorm: x * inv * w in place
        const float inv = has ? 1.0f / sqrtf(block_reduce(ss, false) / (float)K + eps) : 1.f;
        for (int64_t k0 = tid; k0 < KP; k0 += 256 * LB) {
            float w[LB];
#pragma unroll
            for (int i = 0; i < LB; i++) {
                const int64_t k = k0 + 256 * i;
                w[i] = has && k < K ? xw[k] : 0.f;
            }
#pragma unroll
            for (int i = 0; i < LB; i++) {
                const int64_t k = k0 + 256 * i;
                if (k < KP) {
                    const float v = has && k < K ? xs[k] * inv * w[i] : 0.f;
                    mx = fmaxf(mx, fabsf(v));
                    xs[k] = v;
                }
            }
        }
    }
    mx = block_reduce(mx, true);  // its barriers also order the shared stores before the reads below
    int e = 0;
    if (mx > 0.f && !isinf(mx)) {
        int ex;
        frexpf(mx, &ex);
        e = 14 - ex;
        e = e < -100 ? -100 : (e > 100 ? 100 : e);
    }
    const float scl = __int_as_float((e + 127) << 23);
    if (tid == 0) xinv[col] = has ? __int_as_float((127 - e) << 23) : 0.f;
    for (int64_t c = tid; c < nchunks; c += 256) {
        const int64_t kst = c >> 3, ch = c & 7, k0 = 8 * c;
        const float4 a = *reinterpret_cast<const float4 *>(xs + k0), b = *reinterpret_cast<const float4 *>(xs + k0 + 4);
        const uint4 w = make_uint4(pack_h2(a.x * scl, a.z * scl), pack_h2(a.y * scl, a.w * scl),
                                   pack_h2(b.x * scl, b.z * scl), pack_h2(b.y * scl, b.w * scl));
        *reinterpret_cast<uint4 *>(Xp + ((((int64_t)tile * nu * 4 + kst) * 8 + ch) * npad + n) * 8) = w;
    }
}

// split-K: Y (+)= sum of the partials in split order (and the SwiGLU epilogue)
__global__ void qmma_reduce_kernel(const float *__restrict__ ws, int splits, int ncols, int64_t mpad, float *Y,
                                   int64_t ldy, int64_t M, int accumulate, int ep) {
    pdl_trigger();
    pdl_wait();
    const int64_t mo = ep ? M / 2 : M;
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= mo * ncols) return;
    const int col = (int)(i / mo);
    const int64_t r = i % mo;
    auto sum = [&](int64_t row) {
        float v = 0.f;
        for (int zz = 0; zz < splits; zz++) v += ws[((int64_t)zz * ncols + col) * mpad + row];
        return v;
    };
    if (ep) {
        const int64_t g = (r >> 4) * 32 + (r & 15);
        const float gv = sum(g), uv = sum(g + 16);
        Y[(int64_t)col * ldy + r] = glu_act(ep, gv, uv);
    } else {
        const float v = sum(r);
        float *y = Y + (int64_t)col * ldy + r;
        *y = accumulate ? *y + v : v;
    }
}

// the same sums four rows per thread: 16-byte loads of every split issued
// before the adds (each element summed in split order, as above)
__global__ void qmma_reduce4_kernel(const float *__restrict__ ws, int splits, int ncols, int64_t mpad, float *Y,
                                    int64_t ldy, int64_t M, int accumulate, int ep) {
    pdl_trigger();
    pdl_wait();
    const int64_t mo = ep ? M / 2 : M, mq = mo / 4;
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= mq * ncols) return;
    const int col = (int)(i / mq);
    const int64_t r = 4 * (i % mq);
    auto sum = [&](int64_t row) {
        constexpr int kMaxSplit = 8;
        float4 t[kMaxSplit];
#pragma unroll
        for (int zz = 0; zz < kMaxSplit; zz++)
            if (zz < splits) t[zz] = *reinterpret_cast<const float4 *>(ws + ((int64_t)zz * ncols + col) * mpad + row);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int zz = 0; zz < kMaxSplit; zz++)
            if (zz < splits) {
                v.x += t[zz].x;
                v.y += t[zz].y;
                v.z += t[zz].z;
                v.w += t[zz].w;
            }
        for (int zz = kMaxSplit; zz < splits; zz++) {
            const float4 u = *reinterpret_cast<const float4 *>(ws + ((int64_t)zz * ncols + col) * mpad + row);
            v.x += u.x;
            v.y += u.y;
            v.z += u.z;
            v.w += u.w;
        }
        return v;
    };
    float4 *y = reinterpret_cast<float4 *>(Y + (int64_t)col * ldy + r);
    if (ep) {
        const int64_t g = (r >> 4) * 32 + (r & 15);  // four rows of one 16-row gate block
        const float4 gv = sum(g), uv = sum(g + 16);
        *y = make_float4(glu_act(ep, gv.x, uv.x), glu_act(ep, gv.y, uv.y), glu_act(ep, gv.z, uv.z),
                         glu_act(ep, gv.w, uv.w));
    } else {
        const float4 v = sum(r);
        if (accumulate) {
            const float4 o = *y;
            *y = make_float4(o.x + v.x, o.y + v.y, o.z + v.z, o.w + v.w);
        } else {
            *y = v;
        }
    }
}

namespace {

int sm_count() { return device_sm_count(); }

struct Plan {
    int ntiles, npad, nch, ks, splits, RS, ST, rtiles, smem;
    int64_t xp_bytes, xinv_bytes, ws_bytes;
};

// columns per CTA up to 512 (one weight dequant serves all of them), in MMA
// chunks of <= 256; 128-wide K stages for tiles of <= 256 columns; split-K
// minimises waves x (units + start-up) per CTA
bool make_plan(const QTensor &T, int ncols, Plan &p) {
    if (ncols < 1) return false;
    const int raw1 = T.f16 ? 0 : 8 * mtile_bytes(T.type);  // fp16 stages: no raw weight ring
    bool ok = false;
    for (int cap = 512; cap >= 256 && !ok; cap -= 256) {
        p.ntiles = (ncols + cap - 1) / cap;
        const int per = (ncols + p.ntiles - 1) / p.ntiles;
        p.nch = (per + 255) / 256;
        const int cw = ((per + p.nch - 1) / p.nch + 15) / 16 * 16;
        p.npad = cw * p.nch;
        for (p.ks = p.npad <= 256 ? 2 : 1; p.ks >= 1 && !ok; p.ks--) {
            const int stage = (a_stage_bytes(p.ks) + p.npad * 128 * p.ks + 1023) & ~1023;
            for (p.RS = kMaxRaw; p.RS >= 2 && !ok; p.RS--) {
                const int raw = (p.RS * raw1 + 1023) & ~1023;
                int st = (kMaxSmem - 2048 - raw) / stage;  // 1 KB barriers, 1 KB slack
                if (st > kMaxStages) st = kMaxStages;
                if (st >= 2 && (st >= 3 || p.RS == 2)) {
                    p.ST = st;
                    p.smem = 1024 + raw + st * stage;
                    ok = true;
                }
            }
            if (ok) p.RS++;  // undo the loops' final decrements
        }
        if (ok) p.ks++;
    }
    if (!ok) return false;
    p.rtiles = (int)((T.nrb + 7) / 8);
    const int base = p.rtiles * p.ntiles, nsm = sm_count();
    p.splits = 1;
    int64_t best = -1;
    for (int s = 1; s <= T.nu && s <= 64; s++) {
        // a CTA costs its units plus ~2 units of start-up (first weights, TMEM, epilogue)
        const int64_t waves = ((int64_t)base * s + nsm - 1) / nsm;
        const int64_t cost = waves * ((T.nu + s - 1) / s + 2);
        if (best < 0 || cost < best) {
            best = cost;
            p.splits = s;
        }
    }
    p.xp_bytes = (int64_t)p.ntiles * p.npad * T.nu * 256 * 2;
    p.xinv_bytes = ((int64_t)p.ntiles * p.npad * 4 + 255) / 256 * 256;
    p.ws_bytes = p.splits > 1 ? (int64_t)p.splits * ncols * T.nrb * 16 * 4 : 0;
    return true;
}

template <int FMT, int KS>
cudaError_t launch_qmma_ks(const MmaArgs &a, const Plan &p, cudaStream_t s) {
    static DeviceFlags attr;
    if (!attr.test()) {
        cudaError_t e = cudaFuncSetAttribute(qmma_kernel<FMT, KS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kMaxSmem - 1024);
        if (e != cudaSuccess) return e;
        attr.set();
    }
    return launch_k(qmma_kernel<FMT, KS>, dim3(p.rtiles * p.ntiles, p.splits), dim3(kMmaThreads), (size_t)p.smem, s,
                    a);
}
template <int FMT>
cudaError_t launch_qmma(const MmaArgs &a, const Plan &p, cudaStream_t s) {
    return p.ks == 2 ? launch_qmma_ks<FMT, 2>(a, p, s) : launch_qmma_ks<FMT, 1>(a, p, s);
}

}  // namespace

int64_t qgemm_dense_f16_bytes(const QTensor &T) { return (T.nrb + 7) / 8 * T.nu * 4 * kF16StageBytes; }

cudaError_t qgemm_dense_prepare_f16(QTensor &T, uint8_t *dst, cudaStream_t s) {
    if (!dst || ((uintptr_t)dst & 15)) return cudaErrorInvalidValue;
    static_assert(a_stage_bytes(1) == kF16StageBytes && a_stage_bytes(2) == 2 * kF16StageBytes,
                  "a KS-stage is KS consecutive 64-K stages");
    const dim3 grid((unsigned)((T.nrb + 7) / 8), (unsigned)T.nu);
    cudaError_t e = cudaMemsetAsync(dst, 0, qgemm_dense_f16_bytes(T), s);
    if (e != cudaSuccess) return e;
    switch (T.type) {
    case 12: qmma_f16_stages_kernel<12><<<grid, kDqThreads, 0, s>>>(T.data, (int)T.nrb, (int)T.nu, dst); break;
    case 13: qmma_f16_stages_kernel<13><<<grid, kDqThreads, 0, s>>>(T.data, (int)T.nrb, (int)T.nu, dst); break;
    case 14: qmma_f16_stages_kernel<14><<<grid, kDqThreads, 0, s>>>(T.data, (int)T.nrb, (int)T.nu, dst); break;
    case 8: qmma_f16_stages_kernel<8><<<grid, kDqThreads, 0, s>>>(T.data, (int)T.nrb, (int)T.nu, dst); break;
    default: return cudaErrorInvalidValue;
    }
    e = cudaGetLastError();
    if (e == cudaSuccess) T.f16 = dst;
    return e;
}

int64_t qgemm_dense_scratch_bytes(const QTensor &T, int ncols) {
    Plan p;
    if (!make_plan(T, ncols, p)) return -1;
    return p.xp_bytes + p.xinv_bytes + p.ws_bytes;
}

// the activation packing of one GEMM: the column held in shared memory
// (pack_x_kernel) up to kPackSmemMax bytes, else re-read per pass
template <int XF>
static cudaError_t launch_pack_xf(dim3 pg, cudaStream_t s, const float *X, int64_t ldx, int64_t K, int ncols, int npad,
                                  int nu, const float *xw, float eps, uint16_t *Xp, float *xinv) {
    const int64_t smem = (int64_t)nu * 256 * 4;
    if (smem > kPackSmemMax)
        return launch_k(pack_x_stream_kernel<XF>, pg, dim3(256), 0, s, X, ldx, K, ncols, npad, nu, xw, eps, Xp, xinv);
    static DeviceFlags attr;
    if (!attr.test()) {
        const cudaError_t e =
            cudaFuncSetAttribute(pack_x_kernel<XF>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPackSmemMax);
        if (e != cudaSuccess) return e;
        attr.set();
    }
    return launch_k(pack_x_kernel<XF>, pg, dim3(256), (size_t)smem, s, X, ldx, K, ncols, npad, nu, xw, eps, Xp, xinv);
}
static cudaError_t launch_pack(int kind, dim3 pg, cudaStream_t s, const float *X, int64_t ldx, int64_t K, int ncols,
                               int npad, int nu, const float *xw, float eps, uint16_t *Xp, float *xinv) {
    switch (kind) {
    case 0: return launch_pack_xf<0>(pg, s, X, ldx, K, ncols, npad, nu, xw, eps, Xp, xinv);
    case 1: return launch_pack_xf<1>(pg, s, X, ldx, K, ncols, npad, nu, xw, eps, Xp, xinv);
    default: return launch_pack_xf<2>(pg, s, X, ldx, K, ncols, npad, nu, xw, eps, Xp, xinv);
    }
}

cudaError_t qgemm_dense(const QTensor &T, const float *X, int ncols, float *Y, bool accumulate, int64_t ldy,
                        cudaStream_t s, const XForm &xf, void *scratch, int64_t scratch_bytes) {
    Plan p;
    if (!make_plan(T, ncols, p)) return cudaErrorInvalidValue;
    if (scratch_bytes < p.xp_bytes + p.xinv_bytes + p.ws_bytes || !scratch) return cudaErrorInvalidValue;
    if (xf.kind < 0 || xf.kind > 2 || (xf.kind == 1 && !xf.w)) return cudaErrorInvalidValue;
    if (xf.ep && (accumulate || T.rows % 32)) return cudaErrorInvalidValue;
    uint8_t *sc = static_cast<uint8_t *>(scratch);
    uint16_t *Xp = reinterpret_cast<uint16_t *>(sc);
    float *xinv = reinterpret_cast<float *>(sc + p.xp_bytes);
    float *ws = p.ws_bytes ? reinterpret_cast<float *>(sc + p.xp_bytes + p.xinv_bytes) : nullptr;
    const int64_t ldx = xf.ldx > 0 ? xf.ldx : T.cols;
    const dim3 pg((unsigned)(p.ntiles * p.npad));
    cudaError_t e = launch_pack(xf.kind, pg, s, X, ldx, (int64_t)T.cols, ncols, p.npad, (int)T.nu, xf.w, xf.eps, Xp,
                                xinv);
    if (e != cudaSuccess) return e;
    MmaArgs a{T.data, (int)T.nrb, (int)T.nu, Xp, xinv, ncols, p.npad, p.ntiles, p.nch, p.splits, p.RS, p.ST,
              Y, ldy, T.rows, accumulate ? 1 : 0, xf.ep, ws, T.f16};
    switch (T.type) {
    case 12: e = launch_qmma<12>(a, p, s); break;
    case 13: e = launch_qmma<13>(a, p, s); break;
    case 14: e = launch_qmma<14>(a, p, s); break;
    case 8: e = launch_qmma<8>(a, p, s); break;
    default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess || p.splits == 1) return e;
    const int64_t mo = xf.ep ? T.rows / 2 : T.rows, n = mo * ncols, mpad = (int64_t)T.nrb * 16;
    if (mo % 4 == 0 && ldy % 4 == 0 && ((uintptr_t)Y & 15) == 0 && ((uintptr_t)ws & 15) == 0)
        return launch_k(qmma_reduce4_kernel, dim3((unsigned)((n / 4 + 255) / 256)), dim3(256), 0, s,
                        (const float *)ws, p.splits, ncols, mpad, Y, ldy, (int64_t)T.rows, accumulate ? 1 : 0, xf.ep);
    return launch_k(qmma_reduce_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, (const float *)ws,
                    p.splits, ncols, mpad, Y, ldy, (int64_t)T.rows, accumulate ? 1 : 0, xf.ep);
}

cudaError_t read_mma_error(int *flag, cudaStream_t s) {
    int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(flag, g_mma_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(g_mma_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e;
}

}  // namespace ifr
