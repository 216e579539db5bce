// Fused verify forward of one request: every decoder layer of the target (or
// the MTP layer of a draft step) as one persistent cooperative launch - one
// CTA of 512 threads per SM, the layer sequence as a list of phases in device
// memory, a grid barrier between dependent phases.  The separate-kernel path
// (engine.cu layer_forward) runs ~5 launches per layer whose latency, not
// their bytes, sets the step time at batch 1; here a phase boundary costs one
// grid barrier, and each projection's weights are prefetched to L2 one phase
// ahead so that the next phase reads them at L2 latency.
//
// Phases (reference semantics as in model.cu / qgemv_kernels.cuh):
//   GEMV   Y (+)= W f(X) for N <= 8 columns, exact f32 activations (the fp16
//          hi/lo split of the small-N kernel), K-quant M-tiles read straight
//          from global memory; every CTA takes a contiguous range of row
//          blocks with all their units (the unit fragments built once per CTA
//          in shared memory), the (row block, unit) M-tiles spread over the
//          16 warps and summed over the units in unit order; transforms: none,
//          RMSNorm folded into the epilogue; epilogues: store, accumulate into
//          the residual, silu(gate) * up / gelu_tanh(gate) * up
//   SSM    GatedDeltaNet step of one head (ssm_batch_body, 512 threads)
//   ATTN   split-KV attention slices (attn_part_body, one 256-thread virtual
//          block per CTA on named barrier 1: a slice's shared memory fills
//          the CTA's) and their combine (attn_combine_body, two 256-thread
//          virtual blocks per CTA on named barriers 1 and 2)
// Activations written by earlier phases are read with coherent loads (never
// the read-only path); a grid barrier orders them (release add, acquire poll).
// Every barrier wait is bounded (~2 s); a CTA whose wait runs out sets the
// error flag, which every other wait also checks, so the launch ends promptly
// and the host reports IFR_ERR_TIMEOUT.
// Included at the end of model.cu (it uses that file's attention and SSM
// bodies); model.cu includes qgemv_kernels.cuh for the M-tile code.
#pragma once
#include "fused.cuh"

namespace ifr {

namespace {

constexpr int kFThreads = 512, kFWarps = 16;
__device__ int g_fused_error = 0;
constexpr long long kBarrierCycles = 4000000000LL;  // ~2 s at 1.9 GHz

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void fence_acquire_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void red_release_add(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// all CTAs of the launch: the counter reaches `target` once every CTA has
// arrived at this barrier; false after a timeout or another CTA's error
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ unsigned atom_release_add(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.release.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// all CTAs of the launch: the counter reaches `target` once every CTA has
// arrived at this barrier; false after a timeout or another CTA's error.
// bt (tracing, nullable): [0] CTA 0's arrival done, [1] target seen, [2]
// acquire done; [3] the last arrival (whichever CTA made it)
__device__ bool grid_barrier(unsigned *ctr, unsigned target, int *err, unsigned long long *bt) {
    // bar.sync orders the CTA's writes before thread 0's release add (release
    // is cumulative), and its acquire poll before every thread's later reads
    __syncthreads();
    __shared__ int ok_s;
    if (threadIdx.x == 0) {
        int ok = 1;
        if (bt) {
            const unsigned old = atom_release_add(ctr, 1u);
            const unsigned long long ta = global_ns();
            if (old + 1 == target) bt[3] = ta;
            if (blockIdx.x == 0) bt[0] = ta;
        } else {
            red_release_add(ctr, 1u);
        }
        const long long t0 = clock64();
        while (ld_relaxed_u32(ctr) < target) {
            if (*(volatile int *)err) { ok = 0; break; }
            if (clock64() - t0 > kBarrierCycles) {
                atomicExch(err, 1);
                ok = 0;
                break;
            }
        }
        if (bt && blockIdx.x == 0) bt[1] = global_ns();
        fence_acquire_gpu();  // the other CTAs' phase outputs before this CTA's next reads
        if (bt && blockIdx.x == 0) bt[2] = global_ns();
        ok_s = ok;
    }
    __syncthreads();
    return ok_s != 0;
}

__device__ __forceinline__ void bulk_prefetch_l2(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// this CTA's row blocks of a GEMV phase: contiguous, in units of `gran` blocks
__device__ __forceinline__ void rb_range(const FGemv &g, int cta, int ncta, int &rb0, int &rb1) {
    const int grp = (g.nrb + g.gran - 1) / g.gran;
    rb0 = (int)((int64_t)cta * grp / ncta) * g.gran;
    rb1 = min(g.nrb, (int)((int64_t)(cta + 1) * grp / ncta) * g.gran);
}

// the L2 prefetch of this CTA's share of a GEMV phase's weights (thread 0)
__device__ void prefetch_gemv(const FPrefetch &g, int cta, int ncta) {
    if (!g.W) return;
    const int grp = (g.nrb + g.gran - 1) / g.gran;
    const int rb0 = (int)((int64_t)cta * grp / ncta) * g.gran;
    const int rb1 = min(g.nrb, (int)((int64_t)(cta + 1) * grp / ncta) * g.gran);
    if (rb1 <= rb0) return;
    const int64_t mtb = mtile_bytes(g.fmt);
    const char *p = reinterpret_cast<const char *>(g.W) + (int64_t)rb0 * g.nu * mtb;
    int64_t left = (int64_t)(rb1 - rb0) * g.nu * mtb;
    while (left > 0) {  // bulk prefetches of at most 1 MB, 16-byte multiples
        const uint32_t n = (uint32_t)(left < (1 << 20) ? left : (1 << 20));
        bulk_prefetch_l2(p, n & ~15u);
        p += n;
        left -= n;
    }
}

// the bulk copy of this CTA's M-tiles of a GEMV phase into the tile buffer
// (thread 0); false when this CTA has no rows there (nothing to wait for)
__device__ bool issue_tiles(const FPrefetch &t, int cta, int ncta, unsigned char *buf, uint64_t *bar) {
    if (!t.W) return false;
    const int grp = (t.nrb + t.gran - 1) / t.gran;
    const int rb0 = (int)((int64_t)cta * grp / ncta) * t.gran;
    const int rb1 = min(t.nrb, (int)((int64_t)(cta + 1) * grp / ncta) * t.gran);
    if (rb1 <= rb0) return false;
    const int64_t mtb = mtile_bytes(t.fmt);
    const uint32_t bytes = (uint32_t)((int64_t)(rb1 - rb0) * t.nu * mtb);
    mbar_expect_tx(bar, bytes);
    bulk_g2s(buf, t.W + (int64_t)rb0 * t.nu * mtb, bytes, bar);
    return true;
}

// bounded wait for the tile copy (~2 s; the fused error flag on timeout)
__device__ bool tiles_wait(uint64_t *bar, uint32_t parity, int *err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kBarrierCycles || *(volatile int *)err) {
            atomicExch(err, 1);
            return false;
        }
    }
    return true;
}

// the tile-buffer state of a CTA (uniform over its threads)
struct TileState {
    unsigned char *buf;
    uint64_t *bar;
    uint32_t parity;
};

template <int FMT, int NT, int XF>
__device__ void gemv_phase(const FGemv &g, bool tiles_smem, const FPrefetch &next_tiles, TileState &ts, int cta,
                           int ncta, unsigned char *smem, unsigned long long *tp, int *err) {
    constexpr int MTB = mtile_bytes(FMT);
    constexpr int BW = bunit_words(NT);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    int rb0, rb1;
    rb_range(g, cta, ncta, rb0, rb1);
    const int nrb = rb1 - rb0;
    if (nrb <= 0) {  // no rows here (uniform over the CTA): the buffer is free now
        if (tid == 0) issue_tiles(next_tiles, cta, ncta, ts.buf, ts.bar);
        return;
    }
    GemvArgs a{};
    a.W = g.W;
    a.M = g.M;
    a.K = g.K;
    a.nrb = g.nrb;
    a.nu = g.nu;
    a.X = g.X;
    a.ldx = g.ldx;
    a.ncols = g.ncols;
    a.xw = g.xw;
    a.eps = g.eps;
    // shared: fragments [nu][BW] | ssq [nu][8] | partials [nrb][nu][16][8] | inv [8]
    uint32_t *frag = reinterpret_cast<uint32_t *>(smem);
    float *ssq = reinterpret_cast<float *>(frag + g.nu * BW);
    float *part = ssq + g.nu * 8;
    float *inv = part + nrb * g.nu * 128;
    // 1. the unit fragments, (unit, n-tile) tasks over the warps
    for (int task = warp; task < g.nu * NT; task += kFWarps)
        build_b<FMT, NT, XF, true>(a, nullptr, task / NT, lane, task % NT, frag + (task / NT) * BW,
                                   XF == 3 ? ssq : nullptr);
    __syncthreads();
    if (tp) tp[1] = global_ns();
    // 2. the (row block, unit) M-tiles (from the tile buffer once its copy has
    //    landed, else from global memory); C columns 2t, 2t+1 of n-tile nt
    //    are the hi and lo parts of activation column 4 nt + t
    bool ok = true;
    if (tiles_smem) {
        ok = tiles_wait(ts.bar, ts.parity, err);
        ts.parity ^= 1u;
    }
    const uint8_t *tbase = tiles_smem ? ts.buf : g.W + (int64_t)rb0 * g.nu * MTB;
    const int gq = lane >> 2, tq = lane & 3;
    for (int task = warp; ok && task < nrb * g.nu; task += kFWarps) {
        const int rl = task / g.nu, u = task % g.nu;
        const uint8_t *tile = tbase + ((int64_t)rl * g.nu + u) * MTB;
        BView<NT> F;
        F.at(frag + u * BW, lane);
        float tot[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) tot[nt][i] = 0.f;
        if constexpr (FMT == 8) mtile_q80<NT>(tile, lane, F, tot);
        else if constexpr (FMT == 14) mtile_q6_h<NT>(tile, lane, F, tot);
        else mtile_qk_h<FMT == 13, NT>(tile, lane, F, tot);
        float *pp = part + (rl * g.nu + u) * 128;
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const int col = 4 * nt + tq;
            pp[gq * 8 + col] = tot[nt][0] + tot[nt][1];
            pp[(gq + 8) * 8 + col] = tot[nt][2] + tot[nt][3];
        }
    }
    if (XF == 3 && tid < 8) {
        // RMSNorm folded: W (x w) / rms(x) per column, the sums of squares in unit order
        float v = 0.f;
        if (tid < g.ncols)
            for (int uu = 0; uu < g.nu; uu++) v += ssq[uu * 8 + tid];
        inv[tid] = tid < g.ncols ? 1.0f / sqrtf(v / (float)g.K + g.eps) : 0.f;
    }
    __syncthreads();
    if (tp) tp[2] = global_ns();
    // the tile buffer is free: the next GEMV phase's tiles start coming
    if (tid == 0 && issue_tiles(next_tiles, cta, ncta, ts.buf, ts.bar)) {}
    // 3. epilogue: the units' partials in unit order
    auto val = [&](int rl, int r16, int col) {
        float v = 0.f;
        const float *pp = part + (rl * g.nu) * 128 + r16 * 8 + col;
        for (int uu = 0; uu < g.nu; uu++) v += pp[uu * 128];
        return XF == 3 ? v * inv[col] : v;
    };
    const int64_t row0 = (int64_t)rb0 * 16;
    if (g.ep) {
        // interleaved 16-row gate / up blocks: local rows 32 p .. gate, 32 p + 16 .. up
        const int half = nrb * 8;
        for (int i = tid; i < half * g.ncols; i += kFThreads) {
            const int col = i / half, rr = i % half;
            const int pr = rr >> 4, r16 = rr & 15;
            const int64_t j = row0 / 2 + rr;
            if (j < g.M / 2) {
                const float gv = val(2 * pr, r16, col), uv = val(2 * pr + 1, r16, col);
                g.Y[(int64_t)col * g.ldy + j] = glu_act(g.ep, gv, uv);
            }
        }
    } else {
        const int rows = nrb * 16;
        for (int i = tid; i < rows * g.ncols; i += kFThreads) {
            const int col = i / rows, r = i % rows;
            if (row0 + r < g.M) {
                float *y = g.Y + (int64_t)col * g.ldy + row0 + r;
                const float v = val(r >> 4, r & 15, col);
                *y = g.accumulate ? *y + v : v;
            }
        }
    }
}


// Row-split GatedDeltaNet step of one request (ssm_batch_body's arithmetic,
// GatedDeltaNetCPU, ModelCPU.jl:566-731): virtual block (head h, split j)
// owns the state rows r0 = j RPC .. r0 + RPC, one warp per row, each lane 4
// columns (one 16-byte vector).  Every split computes the head's q and k conv
// outputs and the alpha / beta projections itself (a few thousand MACs), so
// no split waits for another; the conv history, the replay inputs and the
// replay record are not written here (other splits of the head still read
// them) but staged and committed by the final phase.  y leaves unnormalised
// in a.y with the split's sums of squares in ssq_part.
template <int HD>
struct SplitSmem {
    static constexpr int RPC = HD / kFusedSsmSplit;
    float xq[kMaxN][HD], xk[kMaxN][HD], rk[kMaxN][HD];
    float cv[kMaxN][RPC], rv[kMaxN][RPC], ys[kMaxN][RPC];
    float rdec[kMaxN], rbeta[kMaxN], ndec[kMaxN], nbeta[kMaxN];
    float ab[3][kMaxN];
    float red[kFWarps][3 * kMaxN];
};

template <int HD>
__device__ void ssm_split_body(const SsmArgs &a, int h, int j, float *ssq_part, float *rec_stage, SplitSmem<HD> &m) {
    constexpr int RPC = HD / kFusedSsmSplit, REC = 2 * HD + 2;
    static_assert(RPC == kFWarps && HD == 128, "one warp per state row, 4 columns per lane");
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int N = a.N, K = a.K, C = a.C, qk = a.H * HD, r0 = j * RPC;
    const int r = min(max(*a.a_prev + 1, 0), kMaxN);  // tokens to replay
    // the state row (warp), loaded first
    float4 *Sp = reinterpret_cast<float4 *>(a.S + ((int64_t)h * HD + r0 + warp) * HD) + lane;
    float4 sv = *Sp;
    // 1. conv outputs of the new tokens: q and k (every dim), v (own rows)
    auto win = [&](int i, int ch) -> const float * {
        if (i < K - 1) return a.hist + (int64_t)i * C + ch;
        if (i < K - 1 + r) return a.rq + (int64_t)(i - K + 1) * C + ch;
        return a.proj + (int64_t)(i - K + 1 - r) * a.ldp + ch;
    };
    if (tid < 2 * HD + RPC) {
        const int part = tid < HD ? 0 : (tid < 2 * HD ? 1 : 2);
        const int i = part < 2 ? tid - part * HD : r0 + tid - 2 * HD;
        const int ch = part * qk + h * HD + i;
        float w[4], tap[kMaxN][4];
#pragma unroll
        for (int k = 0; k < 4; k++) w[k] = k < K ? a.conv_w[(int64_t)ch * K + k] : 0.f;
#pragma unroll
        for (int t = 0; t < kMaxN; t++)
#pragma unroll
            for (int k = 0; k < 4; k++) tap[t][k] = (t < N && k < K) ? *win(r + t + k, ch) : 0.f;
#pragma unroll
        for (int t = 0; t < kMaxN; t++) {
            if (t < N) {
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < 4; k++)
                    if (k < K) acc += tap[t][k] * w[k];
                const float o = acc / (1.0f + expf(-acc));
                if (part == 0) m.xq[t][i] = o;
                else if (part == 1) m.xk[t][i] = o;
                else m.cv[t][i - r0] = o;
            }
        }
    }
    // 2. alpha / beta projections of the new tokens over the whole d
    {
        float pa[kMaxN], pb[kMaxN], ps[kMaxN];
#pragma unroll
        for (int t = 0; t < kMaxN; t++) pa[t] = pb[t] = ps[t] = 0.f;
        const float *wa = a.ab_w + (int64_t)h * a.d, *wb = a.ab_w + (int64_t)(a.H + h) * a.d;
        for (int i = tid; i < a.d; i += kFThreads) {
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
                m.red[warp][t] = va;
                m.red[warp][kMaxN + t] = vb;
                m.red[warp][2 * kMaxN + t] = vs;
            }
        }
    }
    // 3. the previous call's replay record: k (every dim), own v rows, decay, beta
    const float *rec = a.rkv + (int64_t)h * kMaxN * REC;
    {
        constexpr int LPT = kMaxN * HD / kFThreads;
        float kr[LPT];
#pragma unroll
        for (int k = 0; k < LPT; k++) {
            const int i = tid + kFThreads * k;
            kr[k] = i < r * HD ? rec[(i / HD) * REC + i % HD] : 0.f;
        }
#pragma unroll
        for (int k = 0; k < LPT; k++) {
            const int i = tid + kFThreads * k;
            if (i < r * HD) m.rk[i / HD][i % HD] = kr[k];
        }
    }
    if (tid < r * RPC) m.rv[tid / RPC][tid % RPC] = rec[(tid / RPC) * REC + HD + r0 + tid % RPC];
    if (tid < r) {
        m.rdec[tid] = rec[tid * REC + 2 * HD];
        m.rbeta[tid] = rec[tid * REC + 2 * HD + 1];
    }
    __syncthreads();
    if (tid < 3 * N) {
        const int which = tid / N, t = tid % N;
        float v = 0.f;
        for (int w = 0; w < kFWarps; w++) v += m.red[w][which * kMaxN + t];
        if (which < 2 || !a.in_norm) m.ab[which][t] = v;
        else m.ab[2][t] = 1.0f / sqrtf(v / (float)a.d + a.eps);  // rms(x)^-1 of the folded RMSNorm
    }
    __syncthreads();
    // 4. L2 norms of q, k (warp t), gates in f64
    if (warp < N) {
        const int t = warp;
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
            const float iv = a.in_norm ? m.ab[2][t] : 1.f;
            double av = (double)(m.ab[0][t] * iv) + (double)a.dt_bias[h];
            av = av < -20.0 ? -20.0 : (av > 20.0 ? 20.0 : av);
            const double sp = log(1.0 + exp(av));
            const float dec = (float)((double)a.ssm_a[h] * sp);
            m.ndec[t] = expf(dec);
            double bv = (double)(m.ab[1][t] * iv);
            bv = bv < -20.0 ? -20.0 : (bv > 20.0 ? 20.0 : bv);
            m.nbeta[t] = (float)(1.0 / (1.0 + exp(-bv)));
        }
    }
    __syncthreads();
    // 5. this call's replay record, staged (split 0: k, decay, beta; every split its v rows)
    float *stg = rec_stage + (int64_t)h * kMaxN * REC;
    if (j == 0) {
        for (int i = tid; i < N * HD; i += kFThreads) stg[(i / HD) * REC + i % HD] = m.xk[i / HD][i % HD];
        if (tid < N) {
            stg[tid * REC + 2 * HD] = m.ndec[tid];
            stg[tid * REC + 2 * HD + 1] = m.nbeta[tid];
        }
    }
    if (tid < N * RPC) stg[(tid / RPC) * REC + HD + r0 + tid % RPC] = m.cv[tid / RPC][tid % RPC];
    // 6. the state row through the replayed tokens (committed) and the new ones
    auto update = [&](const float *kv, float dec, float beta, float vrow) {
        const float4 k4 = reinterpret_cast<const float4 *>(kv)[lane];
        sv.x *= dec;
        sv.y *= dec;
        sv.z *= dec;
        sv.w *= dec;
        float sk = sv.x * k4.x;
        sk += sv.y * k4.y;
        sk += sv.z * k4.z;
        sk += sv.w * k4.w;
        sk = warp_sum(sk);
        const float dd = beta * (vrow - sk);
        sv.x += dd * k4.x;
        sv.y += dd * k4.y;
        sv.z += dd * k4.z;
        sv.w += dd * k4.w;
    };
    for (int jj = 0; jj < r; jj++) update(m.rk[jj], m.rdec[jj], m.rbeta[jj], m.rv[jj][warp]);
    *Sp = sv;
    for (int t = 0; t < N; t++) {
        update(m.xk[t], m.ndec[t], m.nbeta[t], m.cv[t][warp]);
        const float4 q4 = reinterpret_cast<const float4 *>(m.xq[t])[lane];
        float yv = sv.x * q4.x;
        yv += sv.y * q4.y;
        yv += sv.z * q4.z;
        yv += sv.w * q4.w;
        yv = warp_sum(yv);
        if (lane == 0) {
            m.ys[t][warp] = yv;
            a.y[(int64_t)t * a.ldy + h * HD + r0 + warp] = yv;
        }
    }
    __syncthreads();
    // 7. the split's sums of y^2 per token (rows in order)
    if (tid < N) {
        float v = 0.f;
        for (int w = 0; w < RPC; w++) v += m.ys[tid][w] * m.ys[tid][w];
        ssq_part[((int64_t)h * kFusedSsmSplit + j) * kMaxN + tid] = v;
    }
}

// The final phase of the split GatedDeltaNet step, grid-wide: y = RMSNorm(y)
// per head (the splits' sums in split order) times silu(z); the conv history
// (last K-1 of history + replayed inputs), the new tokens' conv inputs and
// the staged replay record committed for the next call
template <int HD>
__device__ void ssm_final_phase(const SsmArgs &a, const float *ssq_part, const float *rec_stage, int cta, int ncta) {
    constexpr int REC = 2 * HD + 2;
    const int N = a.N, K = a.K, C = a.C, H = a.H;
    const int r = min(max(*a.a_prev + 1, 0), kMaxN);
    const int64_t n_y = (int64_t)N * H * HD, n_c = C, n_r = (int64_t)H * N * REC;
    for (int64_t i = (int64_t)cta * kFThreads + threadIdx.x; i < n_y + n_c + n_r; i += (int64_t)ncta * kFThreads) {
        if (i < n_y) {
            const int t = (int)(i / (H * HD)), h = (int)((i / HD) % H), c = (int)(i % HD);
            float ss = 0.f;
            for (int jj = 0; jj < kFusedSsmSplit; jj++) ss += ssq_part[((int64_t)h * kFusedSsmSplit + jj) * kMaxN + t];
            const float scale = 1.0f / sqrtf(ss / (float)HD + a.eps);
            const float z = a.proj[(int64_t)t * a.ldp + C + h * HD + c];
            float *y = a.y + (int64_t)t * a.ldy + h * HD + c;
            const float yn = *y * scale * a.norm_w[c];
            *y = yn * z * (1.0f / (1.0f + expf(-z)));
        } else if (i < n_y + n_c) {
            const int ch = (int)(i - n_y);
            float nh[3];
#pragma unroll
            for (int jj = 0; jj < 3; jj++) {
                const int w = r + jj;  // window element of the new committed history
                nh[jj] = jj >= K - 1 ? 0.f : (w < K - 1 ? a.hist[(int64_t)w * C + ch] : a.rq[(int64_t)(w - K + 1) * C + ch]);
            }
#pragma unroll
            for (int jj = 0; jj < 3; jj++)
                if (jj < K - 1) a.hist[(int64_t)jj * C + ch] = nh[jj];
            for (int t = 0; t < N; t++) a.rq[(int64_t)t * C + ch] = a.proj[(int64_t)t * a.ldp + ch];
        } else {
            const int64_t q = i - n_y - n_c;
            const int h = (int)(q / (N * REC)), t = (int)((q / REC) % N), e = (int)(q % REC);
            a.rkv[((int64_t)h * kMaxN + t) * REC + e] = rec_stage[((int64_t)h * kMaxN + t) * REC + e];
        }
    }
}

// GEMV format / column-tile / transform dispatch (the formats the fused step takes)
__device__ void gemv_dispatch(const FPhase &P, TileState &ts, int cta, int ncta, unsigned char *smem,
                              unsigned long long *tp, int *err) {
    const FGemv &g = P.g;
    const bool fold = g.xf == 3, tsm = P.tiles_smem != 0;
#define IFR_FGEMV(F, T, X) gemv_phase<F, T, X>(g, tsm, P.tl, ts, cta, ncta, smem, tp, err)
    if (g.fmt == 12) {
        if (g.nt == 2) fold ? IFR_FGEMV(12, 2, 3) : IFR_FGEMV(12, 2, 0);
        else fold ? IFR_FGEMV(12, 1, 3) : IFR_FGEMV(12, 1, 0);
    } else if (g.fmt == 14) {
        if (g.nt == 2) fold ? IFR_FGEMV(14, 2, 3) : IFR_FGEMV(14, 2, 0);
        else fold ? IFR_FGEMV(14, 1, 3) : IFR_FGEMV(14, 1, 0);
    }
#undef IFR_FGEMV
}

__global__ void __launch_bounds__(kFThreads, 1) fused_layers_kernel(const FPhase *__restrict__ ph, int n,
                                                                     unsigned *ctr, unsigned long long *trace) {
    int *err = &g_fused_error;
    extern __shared__ __align__(128) unsigned char fsm[];
    // the current and the next phase: each thread holds one word of the next
    // phase from the start of the current one (its load latency hidden)
    constexpr int kPW = (int)(sizeof(FPhase) / 4);
    static_assert(sizeof(FPhase) % 4 == 0 && kPW <= kFThreads, "one phase word per thread");
    __shared__ __align__(16) int pbuf[2][kPW];
    __shared__ CombineSmem<256> comb[2];
    __shared__ uint64_t tile_bar;
    const int cta = blockIdx.x, ncta = gridDim.x, tid = threadIdx.x;
    unsigned char *work = fsm + kFusedTileBytes;
    TileState ts{fsm, &tile_bar, 0u};
    int nbar = 0;
    if (tid < kPW) pbuf[0][tid] = __ldg(reinterpret_cast<const int *>(ph) + tid);
    if (tid == 0) mbar_init(&tile_bar, 1);
    __syncthreads();
    if (tid == 0 && reinterpret_cast<const FPhase *>(pbuf[0])->kind == FPhase::kGemv) {
        const FPhase &p0 = *reinterpret_cast<const FPhase *>(pbuf[0]);
        FPrefetch own;
        own.W = p0.g.W;
        own.nrb = p0.g.nrb;
        own.nu = p0.g.nu;
        own.fmt = p0.g.fmt;
        own.gran = p0.g.gran;
        if (p0.tiles_smem) issue_tiles(own, cta, ncta, ts.buf, ts.bar);
        else prefetch_gemv(own, cta, ncta);
    }
    for (int i = 0; i < n; i++) {
        const FPhase &P = *reinterpret_cast<const FPhase *>(pbuf[i & 1]);
        int next_word = 0;
        if (i + 1 < n && tid < kPW) next_word = __ldg(reinterpret_cast<const int *>(ph + i + 1) + tid);
        // trace: [phase][cta][4] start, fragments built, tiles done, phase done
        // (before the barrier), then [phase][4] the barrier detail, then the end
        unsigned long long *tp = (trace && tid == 0) ? trace + ((int64_t)i * ncta + cta) * 4 : nullptr;
        if (tp) tp[0] = tp[1] = tp[2] = global_ns();
        // later GEMV phases' weights toward L2 (planned by the host)
        if (tid == 0) {
            prefetch_gemv(P.pf[0], cta, ncta);
            prefetch_gemv(P.pf[1], cta, ncta);
            // the tile buffer is not used by this phase: the next GEMV's tiles start coming
            if (P.kind != FPhase::kGemv) issue_tiles(P.tl, cta, ncta, ts.buf, ts.bar);
        }
        switch (P.kind) {
        case FPhase::kGemv:
            gemv_dispatch(P, ts, cta, ncta, work, tp, err);
            break;
        case FPhase::kSsm: {
            SplitSmem<128> &m = *reinterpret_cast<SplitSmem<128> *>(work);
            for (int v = cta; v < P.vblocks; v += ncta) {
                ssm_split_body<128>(P.s, v / kFusedSsmSplit, v % kFusedSsmSplit, P.ssq_part, P.rec_stage, m);
                __syncthreads();
            }
            break;
        }
        case FPhase::kSsmFinal:
            ssm_final_phase<128>(P.s, P.ssq_part, P.rec_stage, cta, ncta);
            break;
        case FPhase::kAttnPart: {
            // virtual blocks (slice, row group) of one request, one per CTA on
            // its first 256 threads (the slices' shared memory fills the CTA's)
            const int vt = tid & 255;
            float *gs = reinterpret_cast<float *>(work);
            const int per_y = P.a.splits;
            for (int v = cta; v < P.vblocks; v += ncta) {
                if (tid < 256) attn_part_body<256, 1>(P.a, P.hg, P.a.splits, v % per_y, v / per_y, 0, 1, vt, gs);
                __syncthreads();
            }
            break;
        }
        case FPhase::kAttnCombine: {
            const int half = tid >> 8, vt = tid & 255;
            for (int v0 = 2 * cta; v0 < P.vblocks; v0 += 2 * ncta) {
                const int v = v0 + half;
                if (v < P.vblocks) {
                    if (half == 0) attn_combine_body<256, 1>(P.a, 1, P.a.splits, v, vt, comb[0]);
                    else attn_combine_body<256, 2>(P.a, 1, P.a.splits, v, vt, comb[1]);
                }
                __syncthreads();
            }
            break;
        }
        case FPhase::kTestAbsent:
            if (cta == 0) return;  // uniform over CTA 0: it never arrives at the barrier below
            break;
        default:
            break;
        }
        if (trace) {  // the whole CTA's end of the phase
            __syncthreads();
            if (tp) tp[3] = global_ns();
        }
        if (i + 1 < n) {
            if (tid < kPW) pbuf[(i + 1) & 1][tid] = next_word;  // visible after the barrier below
            if (P.nobar) {
                __syncthreads();
            } else if (!grid_barrier(ctr, (unsigned)(++nbar) * ncta, err, trace ? trace + (int64_t)4 * n * ncta + 4 * i : nullptr)) {
                return;
            }
        }
    }
    if (trace && cta == 0 && tid == 0) trace[(int64_t)4 * n * ncta + 4 * n] = global_ns();
    // every tile copy issued was waited for: a GEMV phase's tiles are issued
    // only by the phase before it, which exists in the list
}

}  // namespace

int fused_ctas() { return device_sm_count(); }

cudaError_t read_fused_error(int *flag, cudaStream_t s) {
    int zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(flag, g_fused_error, sizeof(int), 0, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(g_fused_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e;
}

cudaError_t fused_layers(const FPhase *phases, int n, unsigned *ctr, unsigned long long *trace, cudaStream_t s) {
    static DeviceFlags attr;
    if (!attr.test()) {
        cudaError_t e = cudaFuncSetAttribute(fused_layers_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kFusedSmem);
        if (e != cudaSuccess) return e;
        attr.set();
    }
    cudaError_t e = cudaMemsetAsync(ctr, 0, sizeof(unsigned), s);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(fused_ctas());
    cfg.blockDim = dim3(kFThreads);
    cfg.dynamicSmemBytes = kFusedSmem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once (the grid barriers)
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, fused_layers_kernel, phases, n, ctr, trace);
}

cudaError_t fused_absent_cta_test(cudaStream_t s) {
    FPhase h[2] = {};
    h[0].kind = FPhase::kTestAbsent;
    h[1].kind = FPhase::kNone;
    void *buf = nullptr;
    cudaError_t e = cudaMalloc(&buf, sizeof(h) + 256);
    if (e != cudaSuccess) return e;
    FPhase *dph = static_cast<FPhase *>(buf);
    unsigned *ctr = reinterpret_cast<unsigned *>(static_cast<char *>(buf) + sizeof(h) + 128);
    e = cudaMemcpyAsync(dph, h, sizeof(h), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = fused_layers(dph, 2, ctr, nullptr, s);
    const cudaError_t e2 = cudaStreamSynchronize(s);
    cudaFree(buf);
    return e != cudaSuccess ? e : e2;
}

bool fused_gemv_phase(const FGemv &g, FPhase &ph) {
    if (g.fmt != 12 && g.fmt != 14) return false;
    if (g.ncols < 1 || g.ncols > 4 * g.nt || g.nt < 1 || g.nt > 2 || (g.xf != 0 && g.xf != 3)) return false;
    if (g.xf == 3 && !g.xw) return false;
    if (g.ep && (g.accumulate || g.M % 32 || g.gran != 2)) return false;
    if (!g.ep && g.gran != 1) return false;
    // shared memory: fragments, sums of squares, the partials of this CTA's row blocks, inv
    const int ncta = fused_ctas();
    const int grp = (g.nrb + g.gran - 1) / g.gran;
    const int per_cta = (grp + ncta - 1) / ncta * g.gran;
    const int64_t smem = (int64_t)g.nu * bunit_words(g.nt) * 4 + g.nu * 8 * 4 + (int64_t)per_cta * g.nu * 128 * 4 + 32;
    if (smem > kFusedWorkBytes) return false;
    ph = FPhase{};
    ph.kind = FPhase::kGemv;
    ph.g = g;
    // this CTA's tiles through the tile buffer when the largest share fits
    ph.tiles_smem = (int64_t)per_cta * g.nu * mtile_bytes(g.fmt) <= kFusedTileBytes ? 1 : 0;
    return true;
}

bool fused_ssm_phases(const SsmArgs &a, int head_dim, float *ssq_part, float *rec_stage, FPhase &upd,
                      FPhase &fin) {
    if (head_dim != 128 || a.N < 1 || a.N > kMaxN || a.K < 1 || a.K > 4 || !ssq_part || !rec_stage) return false;
    if ((int)sizeof(SplitSmem<128>) > kFusedWorkBytes) return false;
    upd = FPhase{};
    upd.kind = FPhase::kSsm;
    upd.vblocks = a.H * kFusedSsmSplit;
    upd.s_hd = head_dim;
    upd.ssq_part = ssq_part;
    upd.rec_stage = rec_stage;
    upd.s = a;
    fin = upd;
    fin.kind = FPhase::kSsmFinal;
    fin.vblocks = 0;
    return true;
}

bool fused_attn_phases(const AttnArgs &a, FPhase &part, FPhase &comb) {
    if (a.hd != 256 || !a.part || a.splits < 1 || a.splits > kMaxSplits || a.N < 1 || a.N > kMaxN ||
        a.nh % a.nkv)
        return false;
    const int ratio = a.nh / a.nkv, hg = split_heads(ratio, a.N), nrg = (ratio + hg - 1) / hg;
    const int R = std::min(hg, ratio) * a.N;
    if (GrpSmem<256>::bytes(R, a.N) > kFusedWorkBytes) return false;
    part = FPhase{};
    part.kind = FPhase::kAttnPart;
    part.vblocks = a.splits * a.nkv * nrg;
    part.hg = hg;
    part.part_smem = GrpSmem<256>::bytes(R, a.N);
    part.a = a;
    comb = FPhase{};
    comb.kind = FPhase::kAttnCombine;
    comb.vblocks = a.nh * a.N;
    comb.a = a;
    return true;
}

}  // namespace ifr
