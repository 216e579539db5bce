// Shared device helpers and the internal (C++) interface between the kernel
// files and the C ABI in api.cu.  sm_100a only.
#pragma once
#include <atomic>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <utility>

#define IFR_DEV __device__ __forceinline__

namespace ifr {

// ---- device layout of the quantized tensors (see tiles.cuh) ------------------
// [row block of 16][unit of 256 columns][M-tile], same bytes as the GGUF
// blocks, re-arranged per M-tile for the tensor-core GEMV.
struct QTensor {
    int type;
    int64_t rows, cols;
    int64_t nb;         // GGUF blocks per row (256 elements, 32 for Q8_0)
    int64_t nrb;        // row blocks of 16 (rows padded up)
    int64_t nu;         // units of 256 columns (cols padded up for Q8_0)
    uint8_t *data;      // device base
    int64_t bytes;      // device bytes
    // optional (qgemm_dense_prepare_f16): the dequantized weights rounded to fp16
    // as the dense GEMM's shared-memory operand stages, [row tile][unit][stage]
    // of kF16StageBytes each; the dense GEMM then copies them instead of dequantizing
    uint8_t *f16 = nullptr;
};
constexpr int64_t kF16StageBytes = 16896;  // one 128-row x 64-K operand stage (padded chunks)

int64_t raw_row_bytes(int type, int64_t cols);
int64_t device_bytes(int type, int64_t rows, int64_t cols);

// raw GGUF bytes on the device -> device layout (dst distinct from src)
cudaError_t repack(const QTensor &t, const uint8_t *raw, cudaStream_t s);
// bit-exact dequantization (all rows, or the rows listed in idx)
cudaError_t dequant(const QTensor &t, float *out, cudaStream_t s);
cudaError_t dequant_rows(const QTensor &t, const int32_t *idx, int64_t nrows, float *out, cudaStream_t s);

// activation transform applied by the GEMV while it reads X
// Greedy decision folded into a GEMV's epilogue (qgemm_small, one launch):
// the argmax of every output column (ties to the lower row), then per
// sequence b of G + 1 consecutive columns the longest prefix whose argmax
// equals its draft, as accept_greedy_fused does: out[b * out_ld + i] = argmax
// of column b (G + 1) + i up to the first mismatch (-1 after it), acc[b] =
// accepted drafts.  cand: 8 x (grid) 64-bit scratch; counter: one unsigned at
// zero, returned to zero (launches sharing it must not overlap).
struct GemvArgmax {
    unsigned long long *cand = nullptr;
    unsigned *counter = nullptr;
    const int32_t *drafts = nullptr;  // draft b's tokens at drafts + b * draft_ld (G > 0)
    int draft_ld = 0;
    int G = 0;
    int32_t *acc = nullptr;           // may be null (G = 0)
    int32_t *out = nullptr;
    int out_ld = 0;
};
struct XForm {
    int kind = 0;              // 0: none; 1: RMSNorm x * (1/sqrt(mean x^2 + eps)) * w; 2: SwiGLU
                               // silu(X[c][k]) * X[c][K + k] (X holds [gate | up] per column)
    const float *w = nullptr;  // RMSNorm weights [cols]
    float eps = 0.f;
    int64_t ldx = 0;           // column stride of X in floats (0: the matrix's cols)
    int act = 0;               // K-quant activations: 0 = exact f32 (fp16 hi + lo),
                               // 1 = Q8_K (the reference's kernels, integer tensor cores)
    int ep = 0;                // 1: the rows are 16-row blocks of gate and up interleaved
                               // (gate 0-15, up 0-15, gate 16-31, ...); Y gets silu(gate) * up,
                               // rows/2 rows (not with accumulate); 2: gelu_tanh(gate) * up
    const GemvArgmax *am = nullptr;  // greedy decision on Y (not with ep or accumulate)
    float *kpart = nullptr;    // tall matrices, exact activations, no transform or epilogue:
    int64_t kpart_floats = 0;  // scratch for the second K half's partial sums (>= rows * ncols),
                               // which lets the row-block-per-warp kernel split K over CTA pairs
    int rev = 0;               // tall matrices: each CTA streams its row groups last to first
                               // (consecutive passes over a matrix a little larger than L2 then
                               // start on the rows the previous pass left in L2)
};
// Y[ncols][rows] (+)= W * f(X), ncols <= 8 per call; X 16-byte aligned, ldx a multiple of 4
cudaError_t qgemm_small(const QTensor &t, const float *X, int ncols, float *Y, bool accumulate, int64_t ldy,
                        cudaStream_t s, const XForm &xf = XForm());
// Dense path for many columns (qmma.cu): tcgen05 tensor cores, fp16 operands
// (weights = exact dequantized values rounded to fp16; activations scaled by a
// power of two per column), f32 accumulation.  scratch >= qgemm_dense_scratch_bytes.
cudaError_t qgemm_dense(const QTensor &t, const float *X, int ncols, float *Y, bool accumulate, int64_t ldy,
                        cudaStream_t s, const XForm &xf, void *scratch, int64_t scratch_bytes);
// bytes of t's fp16 operand stages, and their construction (into t.f16, device
// memory the caller allocated, on stream s); the dense GEMM's results are the
// same with and without them
int64_t qgemm_dense_f16_bytes(const QTensor &t);
cudaError_t qgemm_dense_prepare_f16(QTensor &t, uint8_t *dst, cudaStream_t s);
int64_t qgemm_dense_scratch_bytes(const QTensor &t, int ncols);  // -1: unsupported
cudaError_t read_mma_error(int *flag, cudaStream_t s);
// host encoder (encode.cpp): 0 on success
int quantize_host(int type, const float *x, int64_t rows, int64_t cols, uint8_t *out);
// sampled acceptance: its per-row statistics kernel has one grid row per
// logits row (gridDim.y), so batch * (2 gamma + 1) is bounded by 65535
constexpr int kAcceptMaxRows = 65535;
// device-side error flag set by bounded waits that ran out (read and cleared)
cudaError_t read_device_error(int *flag, cudaStream_t s);
// the small-N kernels of one weight format (one translation unit per format,
// qgemv_q4k.cu .. qgemv_q80.cu) and that unit's error flag
template <int FMT>
cudaError_t qgemm_small_fmt(const QTensor &t, const float *X, int ncols, float *Y, bool accumulate, int64_t ldy,
                            cudaStream_t s, const XForm &xf);
template <int FMT>
cudaError_t read_dev_error_fmt(int *flag, cudaStream_t s);

cudaError_t accept_sampled(const float *target, const float *draft, const int32_t *draft_tokens,
                           const float *uniforms, int batch, int gamma, int vocab, float T,
                           int32_t *accept_count, int32_t *out_tokens, int32_t *draft_out,
                           void *scratch, cudaStream_t s);
int64_t accept_scratch_bytes(int batch, int gamma, int vocab);
// the sampled verification on top-k / top-p / min-p filtered distributions
// (drafts drawn from the filtered draft rows); scratch >= accept_filtered_scratch_bytes
cudaError_t accept_filtered(const float *target, const float *draft, const float *uniforms, int batch, int gamma,
                            int vocab, float T, int top_k, float top_p, float min_p, int32_t *accept_count,
                            int32_t *out_tokens, int32_t *draft_out, void *scratch, cudaStream_t s);
int64_t accept_filtered_scratch_bytes(int batch, int gamma, int vocab);
cudaError_t accept_greedy(const float *target, const int32_t *draft_tokens, int batch, int gamma,
                          int vocab, int32_t *accept_count, int32_t *out_tokens, void *scratch,
                          cudaStream_t s);
int64_t accept_greedy_scratch_bytes(int batch, int gamma, int vocab);
// tensor-parallel greedy acceptance: per-row (max, off + argmax) of a vocabulary
// shard into cand[rows][2]; then, over all ranks' candidates cand[W][rows][2],
// the argmax per row and the longest matching draft prefix per sequence
cudaError_t row_argmax(const float *x, int rows, int64_t V, int off, float *cand, cudaStream_t s);
cudaError_t tp_accept(const float *cand, int W, int rows, const int32_t *drafts, int draft_ld, int B, int G,
                      int32_t *acc, int32_t *out, int out_ld, cudaStream_t s);
// the same in one launch; counter: one zero-initialised unsigned per sequence,
// left at zero (not shared by launches that can overlap); draft b's tokens at
// draft_tokens + b * draft_ld, its outputs at out_tokens + b * out_ld
// (0: gamma and gamma + 1)
cudaError_t accept_greedy_fused(const float *target, const int32_t *draft_tokens, int batch, int gamma, int vocab,
                                int32_t *accept_count, int32_t *out_tokens, void *scratch, unsigned *counter,
                                cudaStream_t s, int draft_ld = 0, int out_ld = 0);
// filtered sampling, one token per row (vocab <= 524288), and the in-place
// presence / repetition penalties (vocab <= 1048576)
cudaError_t sample_filtered(const float *logits, int rows, int vocab, float T, int top_k, float top_p, float min_p,
                            const float *uniforms, int32_t *out_tokens, cudaStream_t s);
cudaError_t apply_penalties(float *logits, int rows, int vocab, const int32_t *seen, int n_seen, float presence,
                            float repetition, cudaStream_t s);

}  // namespace ifr

// ---- small device utilities ---------------------------------------------------
namespace ifr {

IFR_DEV uint32_t lop_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
    uint32_t r;
    // (a & mask) | orv, one LOP3
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));
    return r;
}

IFR_DEV uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

IFR_DEV uint32_t hsub2_u(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

IFR_DEV uint32_t hmul2_u(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

// D = A(16x16 f16) * B(16x8 f16) + C, f32 accumulate
IFR_DEV void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                      uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A(16x16 f16) * B(16x8 f16), f32 (C = 0)
IFR_DEV void mma16816_z(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                        uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// D = A(16x32 s8) * B(32x8 s8), s32 (C = 0)
IFR_DEV void imma16832_z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                         uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// D = A(16x16 s8) * B(16x8 s8), s32 (C = 0)
IFR_DEV void imma16816_z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0));
}

// D = A(16x8 f16) * B(8x8 f16) + C, f32 accumulate
IFR_DEV void mma1688(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm(
        "mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(b0));
}

IFR_DEV float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// gelu_tanh (reference src/Gemma4.jl:253-257): 0.5 x (1 + tanh(c (x + 0.044715 x^3))),
// c = sqrt(2 / pi) in f32, evaluated left to right without contraction
IFR_DEV float gelu_tanh(float x) {
    const float c = 0.797884523868560791f;  // sqrtf(2.0f / (float)pi), correctly rounded
    const float x3 = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
    const float t = tanhf(__fmul_rn(c, __fadd_rn(x, x3)));
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
}
// the gated MLP's activation of an interleaved gate/up epilogue (XForm::ep):
// 1 silu(gate) * up (Qwen3.5, ModelCPU.jl:482-508), 2 gelu_tanh(gate) * up
// (Gemma4, Gemma4.jl:556-581)
IFR_DEV float glu_act(int ep, float g, float u) {
    if (ep == 2) return __fmul_rn(gelu_tanh(g), u);
    return g / (1.0f + expf(-g)) * u;
}

IFR_DEV uint4 ldg_nc4(const void *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }
IFR_DEV uint2 ldg_nc2(const void *p) { return __ldg(reinterpret_cast<const uint2 *>(p)); }

// ---- programmatic dependent launch ------------------------------------------
// Every kernel of the decode step is launched with programmatic stream
// serialization: the next kernel may start (prologue, weight prefetch) while
// this one runs.  Rules each kernel follows: nothing written to global memory
// and nothing read that an earlier kernel produces before pdl_wait(), which
// returns once all prerequisite grids have completed and their writes are
// visible (and is a no-op for a normal launch).  Because every kernel waits,
// completion is transitive along the stream.
IFR_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
IFR_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

bool pdl_enabled();  // IFR_PDL=0 in the environment turns it off (api.cu)

// one bit per device: per-device one-time set-up (cudaFuncSetAttribute applies
// to the current device only, and one process may drive several GPUs)
struct DeviceFlags {
    std::atomic<unsigned long long> bits{0};
    static unsigned long long bit() {
        int d = 0;
        cudaGetDevice(&d);
        return 1ull << (d & 63);
    }
    bool test() const { return (bits.load() & bit()) != 0; }
    void set() { bits.fetch_or(bit()); }
};

// multiprocessor count of the current device, cached per device (one
// process may drive several GPUs from several host threads)
inline int device_sm_count() {
    static std::atomic<int> cache[64];
    int d = 0;
    cudaGetDevice(&d);
    d &= 63;
    int n = cache[d].load(std::memory_order_relaxed);
    if (n <= 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || n <= 0) n = 148;
        cache[d].store(n, std::memory_order_relaxed);
    }
    return n;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace ifr
