// Dense quantized GEMM on the 5th-generation tensor cores (tcgen05, TMEM):
// Y[n][r] = sum_k W[r][k] X[n][k] for many columns at once - the verify
// columns of a batch of requests, or prompt chunks - with W in Q4_K / Q5_K /
// Q6_K / Q8_0 (M-tile layout, tiles.cuh).  The N <= 8 verify GEMV (qgemv.cu)
// is HBM-bound; here the contraction is dense enough for the tensor cores.
//
// Precision (stated; this is not the exact path): every weight is its exact
// dequantized value (src/Dequant.jl:304-601) rounded once to fp16; every
// activation column is scaled by a power of two (max |x| -> [2^13, 2^14)) and
// rounded to fp16; products are summed in f32 in tensor memory.
//
// One CTA computes 128 output rows x one tile of up to 256 columns over a
// range of K units (split-K over blockIdx.y when rows alone give too few CTAs):
//   warp 0     producer: cp.async.bulk of the raw M-tiles of each 256-column
//              unit (ring of 2) and of the packed fp16 activations of each
//              64-column K stage (ring of ST), completion on mbarriers;
//   warp 1     allocates the accumulator in tensor memory; one thread issues
//              tcgen05.mma (M = 128, N = npad, K = 16) four times per stage and
//              tcgen05.commit, which frees the stage when the MMAs are done;
//   warps 2-9  dequantize each stage's 128 x 64 weights into the canonical
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

namespace ifr {

__device__ int g_mma_error = 0;

namespace {

constexpr int kDqWarps = 8;
constexpr int kDqThreads = 32 * kDqWarps;
constexpr int kMmaThreads = 64 + kDqThreads;
constexpr int kBM = 128;                 // rows per CTA (8 row blocks)
constexpr int kBK = 64;                  // K per stage (4 MMAs of K = 16)
constexpr int kRawSlots = 2;
constexpr int kAStage = kBM * kBK * 2;   // fp16 A tile, 16 KB
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
IFR_DEV int byte_at(uint32_t w, int k) { return (int)((w >> (8 * k)) & 0xffu); }
IFR_DEV uint32_t pack_h2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// ---- dequantization of one piece ------------------------------------------------
// A piece is (M-tile row r, lane quad t) of one 64-element K stage p of a unit:
// the 16 elements 64 p + 16 w + 4 t + b (run w = 0..3, b = 0..3), exactly the
// bytes the M-tile keeps together for t (tiles.cuh).  v[4 w + b] gets the
// exact f32 value of src/Dequant.jl (separately rounded products).
template <bool Q5>
IFR_DEV void piece_qk(const uint8_t *tile, int r, int t, int p, float (&v)[16]) {
    const uint4 h = lds128(tile + qk_hdr(r));
    const float d = h2f((uint16_t)(h.x & 0xffffu)), dmin = h2f((uint16_t)(h.x >> 16));
    // 6-bit scales and mins (src/Dequant.jl:345-362), byte j of word j / 4
    const uint32_t sc0 = h.y & 0x3f3f3f3fu, mn0 = h.z & 0x3f3f3f3fu;
    const uint32_t sc1 = (h.w & 0x0f0f0f0fu) | (((h.y >> 6) & 0x03030303u) << 4);
    const uint32_t mn1 = ((h.w >> 4) & 0x0f0f0f0fu) | (((h.z >> 6) & 0x03030303u) << 4);
    const int cl = 2 * p, ch = 2 * p + 1;  // sub-blocks of the low and high nibbles
    const float dl = __fmul_rn(d, (float)byte_at(cl < 4 ? sc0 : sc1, cl & 3));
    const float ml = __fmul_rn(dmin, (float)byte_at(cl < 4 ? mn0 : mn1, cl & 3));
    const float dh = __fmul_rn(d, (float)byte_at(ch < 4 ? sc0 : sc1, ch & 3));
    const float mh = __fmul_rn(dmin, (float)byte_at(ch < 4 ? mn0 : mn1, ch & 3));
    // raw qs bytes 32 p + 16 hh + 4 t + b (hh = 0, 1): low nibble element 64 p + 16 hh + 4 t + b,
    // high nibble element 64 p + 32 + 16 hh + 4 t + b
    const uint2 q = lds64(tile + qk_qs(Q5, p >> 1, r, t) + 8 * (p & 1));
    uint2 qh = make_uint2(0u, 0u);
    if (Q5) qh = lds64(tile + q5_qh(r & 7, t) + 8 * (r >> 3));
#pragma unroll
    for (int hh = 0; hh < 2; hh++) {
        const uint32_t W = hh ? q.y : q.x, H = hh ? qh.y : qh.x;
#pragma unroll
        for (int b = 0; b < 4; b++) {
            int lo = (int)((W >> (8 * b)) & 15u), hi = (int)((W >> (8 * b + 4)) & 15u);
            if (Q5) {
                lo += (int)((H >> (8 * b + cl)) & 1u) << 4;
                hi += (int)((H >> (8 * b + ch)) & 1u) << 4;
            }
            v[4 * hh + b] = __fsub_rn(__fmul_rn(dl, (float)lo), ml);
            v[8 + 4 * hh + b] = __fsub_rn(__fmul_rn(dh, (float)hi), mh);
        }
    }
}

// Q6_K (src/Dequant.jl:558-601): element e = 64 p + 32 j + 16 hh + 4 t + b is raw
// ql byte 64 (p / 2) + 32 j + 16 hh + 4 t + b >> 4 (p % 2), raw qh byte
// 32 (p / 2) + 16 hh + 4 t + b >> (4 (p % 2) + 2 j), scale group 4 p + 2 j + hh
IFR_DEV void piece_q6(const uint8_t *tile, int r, int t, int p, float (&v)[16]) {
    const float d = h2f(*reinterpret_cast<const uint16_t *>(tile + q6_d(r)));
    const uint4 sc = lds128(tile + q6_sc(r));
    const uint4 ql = lds128(tile + q6_ql(p >> 1, r, t));
    const uint2 qh = lds64(tile + q6_qh(r, t) + 8 * (p >> 1));
    const int sl = 4 * (p & 1);
#pragma unroll
    for (int j = 0; j < 2; j++) {
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
            const uint32_t L = wsel(ql, 2 * j + hh), H = hh ? qh.y : qh.x;
            const int g = 4 * p + 2 * j + hh;
            const float ds = __fmul_rn(d, (float)(int8_t)byte_at(wsel(sc, g >> 2), g & 3));
#pragma unroll
            for (int b = 0; b < 4; b++) {
                const int q = (int)((L >> (8 * b + sl)) & 15u) | ((int)((H >> (8 * b + sl + 2 * j)) & 3u) << 4);
                v[4 * (2 * j + hh) + b] = __fmul_rn(ds, (float)(q - 32));
            }
        }
    }
}

// Q8_0 (src/Dequant.jl:304-321): element 64 p + 16 w + 4 t + b of the unit is
// byte b of word w of piece (p, r, t), block 2 p + w / 2
IFR_DEV void piece_q8(const uint8_t *tile, int r, int t, int p, float (&v)[16]) {
    const uint4 q = lds128(tile + q8_qs(p, r, t));
    const uint32_t dd = *reinterpret_cast<const uint32_t *>(tile + q8_d(r) + 4 * p);  // blocks 2p, 2p+1
    const float d0 = h2f((uint16_t)(dd & 0xffffu)), d1 = h2f((uint16_t)(dd >> 16));
#pragma unroll
    for (int w = 0; w < 4; w++) {
        const uint32_t W = wsel(q, w);
#pragma unroll
        for (int b = 0; b < 4; b++) v[4 * w + b] = __fmul_rn(w < 2 ? d0 : d1, (float)(int8_t)byte_at(W, b));
    }
}

template <int FMT>
IFR_DEV void dequant_piece(const uint8_t *tile, int r, int t, int p, float (&v)[16]) {
    if constexpr (FMT == 12) piece_qk<false>(tile, r, t, p, v);
    else if constexpr (FMT == 13) piece_qk<true>(tile, r, t, p, v);
    else if constexpr (FMT == 14) piece_q6(tile, r, t, p, v);
    else piece_q8(tile, r, t, p, v);
}

}  // namespace

struct MmaArgs {
    const uint8_t *W;      // M-tiles
    int nrb, nu;           // row blocks of 16, units of 256
    const uint16_t *Xp;    // packed fp16 activations [ntiles][nu * 4][8][npad][8]
    const float *xinv;     // [ntiles * npad] 2^-e of each column
    int ncols, npad, ntiles, splits, ST;
    float *Y;
    int64_t ldy, M;
    int accumulate, ep;
    float *ws;             // split partials [splits][ncols][nrb * 16] (splits > 1)
};

template <int FMT>
__global__ void __launch_bounds__(kMmaThreads, 1) qmma_kernel(MmaArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    constexpr int MTB = mtile_bytes(FMT);
    constexpr int RAW = 8 * MTB;
    const int ST = a.ST, npad = a.npad;
    uint64_t *raw_full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *raw_empty = raw_full + kRawSlots;
    uint64_t *a_full = raw_empty + kRawSlots;
    uint64_t *b_full = a_full + 4;
    uint64_t *ab_empty = b_full + 4;
    uint64_t *acc_full = ab_empty + 4;
    uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(acc_full + 1);
    volatile int *dead = reinterpret_cast<volatile int *>(tmem_holder + 1);
    uint8_t *raw = smem + 1024;
    const int raw_bytes = (kRawSlots * RAW + 1023) & ~1023;
    const int bstage = npad * 128;
    const int stage_bytes = (kAStage + bstage + 1023) & ~1023;
    uint8_t *stages = raw + raw_bytes;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rt = blockIdx.x / a.ntiles, nt = blockIdx.x % a.ntiles, z = blockIdx.y;
    const int rb0 = rt * 8;
    const int nmt = min(8, a.nrb - rb0);
    const int u0 = (int)((int64_t)z * a.nu / a.splits), u1 = (int)((int64_t)(z + 1) * a.nu / a.splits);
    const int nunits = u1 - u0, nst = 4 * nunits;
    const uint32_t tcols = npad <= 32 ? 32 : npad <= 64 ? 64 : npad <= 128 ? 128 : 256;

    pdl_trigger();
    if (tid == 0) {
        for (int i = 0; i < kRawSlots; i++) {
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

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            int raw_uses[kRawSlots] = {0, 0}, b_uses[4] = {0, 0, 0, 0};
            for (int i = 0; i < nunits && !*dead; i++) {
                const int rs = i % kRawSlots;
                if (i >= kRawSlots && !mb_wait(raw_empty + rs, (uint32_t)((i / kRawSlots) - 1) & 1, dead)) break;
                fence_async_smem();
                mb_expect_tx(raw_full + rs, (uint32_t)(nmt * MTB));
                for (int m = 0; m < nmt; m++)
                    bulk_copy(raw + rs * RAW + m * MTB, a.W + ((int64_t)(rb0 + m) * a.nu + u0 + i) * MTB, MTB,
                              raw_full + rs);
                raw_uses[rs]++;
                // the weights are constant; the activations come from the previous kernel
                if (i == 0) pdl_wait();
                for (int j = 0; j < 4; j++) {
                    const int q = 4 * i + j, st = q % ST;
                    if (q >= ST && !mb_wait(ab_empty + st, (uint32_t)((q / ST) - 1) & 1, dead)) break;
                    uint8_t *B = stages + st * stage_bytes + kAStage;
                    mb_expect_tx(b_full + st, (uint32_t)bstage);
                    const uint16_t *src = a.Xp + ((int64_t)nt * a.nu * 4 + 4 * (u0 + i) + j) * (int64_t)npad * 64;
                    bulk_copy(B, src, (uint32_t)bstage, b_full + st);
                    b_uses[st]++;
                }
            }
            if (nunits == 0) pdl_wait();
            // no copy may land after the CTA exits: a slot is reissued only after its
            // previous contents were consumed, so only its last use can be in flight
            for (int rs = 0; rs < kRawSlots; rs++)
                if (raw_uses[rs] > 0) mb_drain(raw_full + rs, (uint32_t)(raw_uses[rs] - 1) & 1);
            for (int st = 0; st < ST; st++)
                if (b_uses[st] > 0) mb_drain(b_full + st, (uint32_t)(b_uses[st] - 1) & 1);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = mma_idesc(npad);
            for (int q = 0; q < nst; q++) {
                const int st = q % ST;
                const uint32_t par = (uint32_t)(q / ST) & 1;
                if (!mb_wait(a_full + st, par, dead) || !mb_wait(b_full + st, par, dead)) break;
                tc_fence_after();
                const uint32_t A = su32(stages + st * stage_bytes), B = A + kAStage;
#pragma unroll
                for (int s = 0; s < 4; s++)
                    mma_f16(tmem, smem_desc(A + s * 2 * (kBM * 16), kBM * 16, 128),
                            smem_desc(B + s * 2 * (npad * 16), npad * 16, 128), idesc, (q | s) != 0);
                mma_commit(ab_empty + st);
            }
            mma_commit(acc_full);
            mb_drain(acc_full, 0);  // every MMA has completed before TMEM is released
        }
        __syncwarp();
    } else {
        // ---------------- dequant, then epilogue ----------------
        pdl_wait();
        const int dt = tid - 64;
        for (int i = 0; i < nunits && !*dead; i++) {
            const int rs = i % kRawSlots;
            if (!mb_wait(raw_full + rs, (uint32_t)(i / kRawSlots) & 1, dead)) break;
            const uint8_t *slot = raw + rs * RAW;
            bool ok = true;
            for (int j = 0; j < 4; j++) {
                const int q = 4 * i + j, st = q % ST;
                if (q >= ST && !mb_wait(ab_empty + st, (uint32_t)((q / ST) - 1) & 1, dead)) {
                    ok = false;
                    break;
                }
                uint8_t *A = stages + st * stage_bytes;
#pragma unroll
                for (int pc = 0; pc < 512 / kDqThreads; pc++) {
                    const int P = pc * kDqThreads + dt;
                    const int m = P >> 6, r = (P >> 2) & 15, t = P & 3;
                    float v[16];
                    if (m < nmt) {
                        dequant_piece<FMT>(slot + m * MTB, r, t, j, v);
                    } else {
#pragma unroll
                        for (int e = 0; e < 16; e++) v[e] = 0.f;
                    }
                    const int rr = 16 * m + r;
#pragma unroll
                    for (int w = 0; w < 4; w++) {
                        uint8_t *dst = A + (2 * w + (t >> 1)) * (kBM * 16) + rr * 16 + (t & 1) * 8;
                        *reinterpret_cast<uint2 *>(dst) =
                            make_uint2(pack_h2(v[4 * w], v[4 * w + 1]), pack_h2(v[4 * w + 2], v[4 * w + 3]));
                    }
                }
                fence_async_smem();
                mb_arrive(a_full + st);
            }
            if (!ok) break;
            mb_arrive(raw_empty + rs);
        }
        // epilogue: TMEM lane quarter (warp % 4) = rows 32 (warp % 4) ..; the two warps
        // of a quarter take alternate 16-column chunks
        const bool have = __all_sync(0xffffffffu, mb_wait(acc_full, 0, dead));
        tc_fence_after();
        const int quarter = warp & 3, chalf = (warp - 2) >> 2;
        const int64_t row = (int64_t)rb0 * 16 + 32 * quarter + lane;
        for (int c0 = 16 * chalf; c0 < npad; c0 += 32) {
            uint32_t rv[16];
            tmem_ld16(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)c0, rv);
            if (!have) continue;
#pragma unroll
            for (int c = 0; c < 16; c++) {
                const int col = nt * npad + c0 + c;
                const float val = col < a.ncols ? __uint_as_float(rv[c]) * a.xinv[col] : 0.f;
                if (a.splits > 1) {
                    if (col < a.ncols && row < (int64_t)a.nrb * 16) a.ws[((int64_t)z * a.ncols + col) * ((int64_t)a.nrb * 16) + row] = val;
                } else if (a.ep) {
                    // rows 32 P + (0..15) gate, 32 P + 16 + (0..15) up -> output 16 P + (0..15)
                    const float up = __shfl_down_sync(0xffffffffu, val, 16);
                    const int64_t j = (row >> 5) * 16 + lane;
                    if (lane < 16 && col < a.ncols && j < a.M / 2)
                        a.Y[(int64_t)col * a.ldy + j] = val / (1.0f + expf(-val)) * up;
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

// pack the columns of one n-tile to fp16 in the per-stage operand layout,
// scaled by 2^e per column (max |x| 2^e in [2^13, 2^14)); the activation
// transform of the GEMV (RMSNorm, SwiGLU) is applied on the way
template <int XF>
__global__ void __launch_bounds__(256) pack_x_kernel(const float *__restrict__ X, int64_t ldx, int64_t K, int ncols,
                                                     int npad, int nu, const float *__restrict__ xw, float eps,
                                                     uint16_t *__restrict__ Xp, float *__restrict__ xinv) {
    __shared__ float red[8];
    __shared__ float bc;
    pdl_trigger();
    pdl_wait();
    const int slot = blockIdx.x, tile = slot / npad, n = slot % npad;
    const int col = slot;  // tiles hold consecutive columns
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
    if (tid == 0) xinv[slot] = has ? __int_as_float((127 - e) << 23) : 0.f;
    for (int64_t c = tid; c < nchunks; c += 256) {
        const int64_t kst = c >> 3, ch = c & 7;
        uint32_t w[4];
#pragma unroll
        for (int i = 0; i < 4; i++) w[i] = pack_h2(value(8 * c + 2 * i) * scl, value(8 * c + 2 * i + 1) * scl);
        uint16_t *dst = Xp + ((((int64_t)tile * nu * 4 + kst) * 8 + ch) * npad + n) * 8;
        *reinterpret_cast<uint4 *>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
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
        Y[(int64_t)col * ldy + r] = gv / (1.0f + expf(-gv)) * uv;
    } else {
        const float v = sum(r);
        float *y = Y + (int64_t)col * ldy + r;
        *y = accumulate ? *y + v : v;
    }
}

namespace {

int sm_count() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

struct Plan {
    int ntiles, npad, splits, ST, rtiles, smem;
    int64_t xp_bytes, xinv_bytes, ws_bytes;
};

bool make_plan(const QTensor &T, int ncols, Plan &p) {
    if (ncols < 1) return false;
    p.ntiles = (ncols + 255) / 256;
    const int per = (ncols + p.ntiles - 1) / p.ntiles;
    p.npad = (per + 15) / 16 * 16;
    p.rtiles = (int)((T.nrb + 7) / 8);
    const int base = p.rtiles * p.ntiles;
    p.splits = 1;
    if (base < sm_count()) {
        const int want = (sm_count() + base - 1) / base;
        p.splits = (int)(want < T.nu ? want : T.nu);
        if (p.splits < 1) p.splits = 1;
    }
    const int raw = (kRawSlots * 8 * mtile_bytes(T.type) + 1023) & ~1023;
    const int stage = (kAStage + p.npad * 128 + 1023) & ~1023;
    int st = (kMaxSmem - 1024 - 1024 - raw) / stage;  // 1 KB barriers, 1 KB static/alignment slack
    if (st > 4) st = 4;
    if (st < 2) return false;
    p.ST = st;
    p.smem = 1024 + raw + st * stage;
    p.xp_bytes = (int64_t)p.ntiles * p.npad * T.nu * 256 * 2;
    p.xinv_bytes = ((int64_t)p.ntiles * p.npad * 4 + 255) / 256 * 256;
    p.ws_bytes = p.splits > 1 ? (int64_t)p.splits * ncols * T.nrb * 16 * 4 : 0;
    return true;
}

template <int FMT>
cudaError_t launch_qmma(const MmaArgs &a, const Plan &p, cudaStream_t s) {
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(qmma_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kMaxSmem - 1024);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    return launch_k(qmma_kernel<FMT>, dim3(p.rtiles * p.ntiles, p.splits), dim3(kMmaThreads), (size_t)p.smem, s, a);
}

}  // namespace

int64_t qgemm_dense_scratch_bytes(const QTensor &T, int ncols) {
    Plan p;
    if (!make_plan(T, ncols, p)) return -1;
    return p.xp_bytes + p.xinv_bytes + p.ws_bytes;
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
    cudaError_t e;
    switch (xf.kind) {
    case 0: e = launch_k(pack_x_kernel<0>, pg, dim3(256), 0, s, X, ldx, (int64_t)T.cols, ncols, p.npad, (int)T.nu, xf.w, xf.eps, Xp, xinv); break;
    case 1: e = launch_k(pack_x_kernel<1>, pg, dim3(256), 0, s, X, ldx, (int64_t)T.cols, ncols, p.npad, (int)T.nu, xf.w, xf.eps, Xp, xinv); break;
    default: e = launch_k(pack_x_kernel<2>, pg, dim3(256), 0, s, X, ldx, (int64_t)T.cols, ncols, p.npad, (int)T.nu, xf.w, xf.eps, Xp, xinv); break;
    }
    if (e != cudaSuccess) return e;
    MmaArgs a{T.data, (int)T.nrb, (int)T.nu, Xp, xinv, ncols, p.npad, p.ntiles, p.splits, p.ST,
              Y, ldy, T.rows, accumulate ? 1 : 0, xf.ep, ws};
    switch (T.type) {
    case 12: e = launch_qmma<12>(a, p, s); break;
    case 13: e = launch_qmma<13>(a, p, s); break;
    case 14: e = launch_qmma<14>(a, p, s); break;
    case 8: e = launch_qmma<8>(a, p, s); break;
    default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess || p.splits == 1) return e;
    const int64_t n = (xf.ep ? T.rows / 2 : T.rows) * ncols;
    return launch_k(qmma_reduce_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, (const float *)ws,
                    p.splits, ncols, (int64_t)T.nrb * 16, Y, ldy, (int64_t)T.rows, accumulate ? 1 : 0, xf.ep);
}

cudaError_t read_mma_error(int *flag, cudaStream_t s) {
    int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(flag, g_mma_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(g_mma_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e;
}

}  // namespace ifr
