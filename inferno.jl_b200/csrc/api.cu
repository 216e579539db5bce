// C ABI of libinferno_b200 (declared in include/inferno_b200.h).
#include "../../include/inferno_b200.h"
#include "common.cuh"
#include "fused.cuh"

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>

static thread_local std::string g_err;

// shared with engine.cu (hidden symbols of the library)
int ifr_fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

int ifr_cuda_fail(cudaError_t e, const char *what) {
    return ifr_fail(e == cudaErrorMemoryAllocation ? IFR_ERR_NOMEM : IFR_ERR_CUDA, "%s: %s (%s)", what,
                    cudaGetErrorString(e), cudaGetErrorName(e));
}

namespace {

#define fail ifr_fail
#define cuda_fail ifr_cuda_fail

#define IFR_CHECK_CUDA(expr, what)                  \
    do {                                            \
        cudaError_t _e = (expr);                    \
        if (_e != cudaSuccess) return cuda_fail(_e, what); \
    } while (0)

bool valid_type(int t) { return t == IFR_TYPE_Q4_K || t == IFR_TYPE_Q5_K || t == IFR_TYPE_Q6_K || t == IFR_TYPE_Q8_0; }

}  // namespace

struct ifr_ctx {
    int device = 0;
    cudaStream_t own = nullptr;
    cudaStream_t stream = nullptr;
    void *scratch = nullptr;
    size_t scratch_cap = 0;
    int act = IFR_ACT_EXACT;       // K-quant activation mode of the GEMVs
    int dense_min = IFR_DENSE_MIN_COLS_DEFAULT;  // engine GEMMs of this many columns use the dense path
    int prefill_dense = 0;                         // one-request prefill chunks may use the dense path
    int fused_layers = 0;                          // one-request verify: the layer stack as one launch
    int dense_f16 = 1;                             // batched states keep fp16 operand stages of the weights
    int kv_bf16 = 0;                               // split-KV states keep their attention caches in bf16
    std::atomic<int> refs{0};      // live models built on this context
    std::atomic<bool> closing{false};
};

struct ifr_tensor {
    ifr::QTensor q;
    int device;
};

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

int ensure_scratch(ifr_ctx *c, size_t bytes) {
    if (bytes <= c->scratch_cap) return IFR_OK;
    if (c->scratch) {
        cudaStreamSynchronize(c->stream);
        cudaFree(c->scratch);
        c->scratch = nullptr;
        c->scratch_cap = 0;
    }
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    IFR_CHECK_CUDA(cudaMalloc(&c->scratch, want), "cudaMalloc(scratch)");
    c->scratch_cap = want;
    return IFR_OK;
}

int make_tensor(int type, int64_t rows, int64_t cols, int device, ifr_tensor **out) {
    if (!valid_type(type)) return fail(IFR_ERR_ARG, "unsupported weight type %d (Q4_K=12, Q5_K=13, Q6_K=14, Q8_0=8)", type);
    if (rows < 1 || cols < 1) return fail(IFR_ERR_ARG, "rows and cols must be positive (got %lld x %lld)", (long long)rows, (long long)cols);
    int64_t rb = ifr::raw_row_bytes(type, cols);
    if (rb == 0) return fail(IFR_ERR_ARG, "cols=%lld is not a multiple of the %s block (%d)", (long long)cols,
                             type == IFR_TYPE_Q8_0 ? "Q8_0" : "K-quant", type == IFR_TYPE_Q8_0 ? 32 : 256);
    if (rows > (int64_t)1 << 31) return fail(IFR_ERR_ARG, "rows too large");
    ifr_tensor *t = new ifr_tensor();
    t->device = device;
    ifr::QTensor &q = t->q;
    q.type = type;
    q.rows = rows;
    q.cols = cols;
    q.nb = type == IFR_TYPE_Q8_0 ? cols / 32 : cols / 256;
    q.nrb = (rows + 15) / 16;
    q.nu = (cols + 255) / 256;
    q.bytes = ifr::device_bytes(type, rows, cols);
    cudaError_t e = cudaMalloc(&q.data, q.bytes);
    if (e != cudaSuccess) {
        delete t;
        return cuda_fail(e, "cudaMalloc(weights)");
    }
    *out = t;
    return IFR_OK;
}

}  // namespace

namespace ifr {
bool pdl_enabled() {
    static const bool on = [] {
        const char *e = getenv("IFR_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}
}  // namespace ifr

int ifr_ctx_device(const ifr_ctx *c) { return c->device; }
int ifr_ctx_activation(const ifr_ctx *c) { return c->act; }
int ifr_ctx_dense_min(const ifr_ctx *c) { return c->dense_min; }
int ifr_ctx_prefill_dense(const ifr_ctx *c) { return c->prefill_dense; }
int ifr_ctx_fused_layers(const ifr_ctx *c) { return c->fused_layers; }
int ifr_ctx_dense_f16(const ifr_ctx *c) { return c->dense_f16; }
int ifr_ctx_kv_bf16(const ifr_ctx *c) { return c->kv_bf16; }
static void ctx_destroy_now(ifr_ctx *c) {
    DeviceGuard g(c->device);
    cudaStreamSynchronize(c->stream);
    if (c->scratch) cudaFree(c->scratch);
    if (c->own) cudaStreamDestroy(c->own);
    delete c;
}

void ifr_ctx_retain(ifr_ctx *c) { c->refs++; }
void ifr_ctx_release(ifr_ctx *c) {
    if (--c->refs == 0 && c->closing) ctx_destroy_now(c);
}
cudaStream_t ifr_ctx_stream_of(const ifr_ctx *c) { return c->stream; }

// GGUF bytes on the host -> device M-tile tensor (caller owns q->data)
int ifr_upload_raw(ifr_ctx *c, int type, const void *host, int64_t rows, int64_t cols, ifr::QTensor *out) {
    ifr_tensor *t = nullptr;
    int rc = ifr_weights_upload(c, type, host, rows, cols, &t);
    if (rc) return rc;
    *out = t->q;
    delete t;  // the device buffer now belongs to the caller
    return IFR_OK;
}

extern "C" {

const char *ifr_last_error(void) { return g_err.c_str(); }

int ifr_version(void) { return 100; }

int ifr_ctx_create(int device, ifr_ctx **out) {
    if (!out) return fail(IFR_ERR_ARG, "out is NULL");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= n) return fail(IFR_ERR_ARG, "device %d out of range (%d devices)", device, n);
    cudaDeviceProp p;
    IFR_CHECK_CUDA(cudaGetDeviceProperties(&p, device), "cudaGetDeviceProperties");
    if (p.major != 10 || p.minor != 0)
        return fail(IFR_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a only", device, p.major, p.minor);
    DeviceGuard g(device);
    ifr_ctx *c = new ifr_ctx();
    c->device = device;
    e = cudaStreamCreateWithFlags(&c->own, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete c;
        return cuda_fail(e, "cudaStreamCreate");
    }
    c->stream = c->own;
    *out = c;
    return IFR_OK;
}

// a context outlives the models built on it: destroying it while models are
// alive only marks it, and the last ifr_model_free completes the destruction
int ifr_ctx_destroy(ifr_ctx *c) {
    if (!c) return IFR_OK;
    c->closing = true;
    if (c->refs.load() == 0) ctx_destroy_now(c);
    return IFR_OK;
}

int ifr_ctx_set_activation(ifr_ctx *c, int mode) {
    if (!c) return fail(IFR_ERR_ARG, "ctx is NULL");
    if (mode != IFR_ACT_EXACT && mode != IFR_ACT_Q8K)
        return fail(IFR_ERR_ARG, "activation mode must be IFR_ACT_EXACT (0) or IFR_ACT_Q8K (1), got %d", mode);
    c->act = mode;
    return IFR_OK;
}

int ifr_ctx_set_dense_min_cols(ifr_ctx *c, int ncols) {
    if (!c) return fail(IFR_ERR_ARG, "ctx is NULL");
    if (ncols < 1) return fail(IFR_ERR_ARG, "ncols must be >= 1 (got %d)", ncols);
    c->dense_min = ncols;
    return IFR_OK;
}

int ifr_ctx_set_prefill_dense(ifr_ctx *c, int enable) {
    if (!c) return fail(IFR_ERR_ARG, "ctx is NULL");
    c->prefill_dense = enable ? 1 : 0;
    return IFR_OK;
}

int ifr_ctx_set_dense_f16_weights(ifr_ctx *c, int enable) {
    if (!c) return fail(IFR_ERR_ARG, "ctx is NULL");
    c->dense_f16 = enable ? 1 : 0;
    return IFR_OK;
}

int ifr_ctx_set_kv_bf16(ifr_ctx *c, int enable) {
    if (!c) return fail(IFR_ERR_ARG, "ctx is NULL");
    c->kv_bf16 = enable ? 1 : 0;
    return IFR_OK;
}

int ifr_tensor_prepare_dense(ifr_ctx *c, ifr_tensor *t) {
    if (!c || !t) return fail(IFR_ERR_ARG, "NULL argument");
    if (t->device != c->device) return fail(IFR_ERR_ARG, "tensor lives on device %d, context on %d", t->device, c->device);
    if (t->q.f16) return IFR_OK;
    DeviceGuard g(c->device);
    void *p = nullptr;
    IFR_CHECK_CUDA(cudaMalloc(&p, ifr::qgemm_dense_f16_bytes(t->q)), "cudaMalloc(fp16 stages)");
    cudaError_t e = ifr::qgemm_dense_prepare_f16(t->q, static_cast<uint8_t *>(p), c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) {
        t->q.f16 = nullptr;
        cudaFree(p);
        return cuda_fail(e, "fp16 stages");
    }
    return IFR_OK;
}

int ifr_test_fused_timeout(ifr_ctx *c) {
    if (!c) return fail(IFR_ERR_ARG, "ctx is NULL");
    DeviceGuard g(c->device);
    IFR_CHECK_CUDA(ifr::fused_absent_cta_test(c->stream), "fused failure test launch");
    return ifr_sync(c);
}

int ifr_ctx_set_fused_layers(ifr_ctx *c, int enable) {
    if (!c) return fail(IFR_ERR_ARG, "ctx is NULL");
    c->fused_layers = enable ? 1 : 0;
    return IFR_OK;
}

int ifr_ctx_set_stream(ifr_ctx *c, void *s) {
    if (!c) return fail(IFR_ERR_ARG, "ctx is NULL");
    c->stream = (cudaStream_t)s;  // CUDA's convention: NULL is the default stream
    return IFR_OK;
}

int ifr_ctx_get_stream(ifr_ctx *c, void **s) {
    if (!c || !s) return fail(IFR_ERR_ARG, "NULL argument");
    *s = (void *)c->stream;
    return IFR_OK;
}

int ifr_ctx_reserve_accept(ifr_ctx *c, int batch, int gamma, int vocab) {
    if (!c || batch < 1 || gamma < 0 || gamma > 64 || vocab < 1)
        return fail(IFR_ERR_ARG, "invalid reserve arguments");
    DeviceGuard g(c->device);
    int64_t need = ifr::accept_filtered_scratch_bytes(batch, gamma < 1 ? 1 : gamma, vocab);
    int64_t g2 = ifr::accept_greedy_scratch_bytes(batch, gamma, vocab);
    return ensure_scratch(c, (size_t)(need > g2 ? need : g2));
}

int ifr_sync(ifr_ctx *c) {
    if (!c) return fail(IFR_ERR_ARG, "ctx is NULL");
    DeviceGuard g(c->device);
    IFR_CHECK_CUDA(cudaStreamSynchronize(c->stream), "cudaStreamSynchronize");
    int flag = 0;
    IFR_CHECK_CUDA(ifr::read_device_error(&flag, c->stream), "read device error flag");
    if (flag) return fail(IFR_ERR_TIMEOUT, "a bounded device-side wait ran out (pipeline stalled); results of the pending work are invalid");
    return IFR_OK;
}

int ifr_weights_from_device(ifr_ctx *c, int type, const void *dev_bytes, int64_t rows, int64_t cols,
                            ifr_tensor **out) {
    if (!c || !dev_bytes || !out) return fail(IFR_ERR_ARG, "NULL argument");
    DeviceGuard g(c->device);
    ifr_tensor *t = nullptr;
    int rc = make_tensor(type, rows, cols, c->device, &t);
    if (rc) return rc;
    cudaError_t e = ifr::repack(t->q, (const uint8_t *)dev_bytes, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) {
        cudaFree(t->q.data);
        delete t;
        return cuda_fail(e, "repack");
    }
    *out = t;
    return IFR_OK;
}

int ifr_weights_upload(ifr_ctx *c, int type, const void *host, int64_t rows, int64_t cols,
                       ifr_tensor **out) {
    if (!c || !host || !out) return fail(IFR_ERR_ARG, "NULL argument");
    DeviceGuard g(c->device);
    int64_t rb = ifr::raw_row_bytes(type, cols);
    if (!valid_type(type) || rb == 0 || rows < 1)
        return make_tensor(type, rows, cols, c->device, out);  // reports the argument error
    const int64_t raw = rb * rows;
    ifr_tensor *t = nullptr;
    int rc = make_tensor(type, rows, cols, c->device, &t);
    if (rc) return rc;
    void *tmp = nullptr;
    cudaError_t e = cudaMalloc(&tmp, raw);
    if (e == cudaSuccess) e = cudaMemcpyAsync(tmp, host, raw, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = ifr::repack(t->q, (const uint8_t *)tmp, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (tmp) cudaFree(tmp);
    if (e != cudaSuccess) {
        cudaFree(t->q.data);
        delete t;
        return cuda_fail(e, "weights upload");
    }
    *out = t;
    return IFR_OK;
}

int ifr_tensor_free(ifr_tensor *t) {
    if (!t) return IFR_OK;
    DeviceGuard g(t->device);
    cudaFree(t->q.data);
    if (t->q.f16) cudaFree(t->q.f16);
    delete t;
    return IFR_OK;
}

int ifr_tensor_info(const ifr_tensor *t, int *type, int64_t *rows, int64_t *cols, int64_t *bytes) {
    if (!t) return fail(IFR_ERR_ARG, "tensor is NULL");
    if (type) *type = t->q.type;
    if (rows) *rows = t->q.rows;
    if (cols) *cols = t->q.cols;
    if (bytes) *bytes = t->q.bytes;
    return IFR_OK;
}

int ifr_dequant(ifr_ctx *c, const ifr_tensor *t, float *out) {
    if (!c || !t || !out) return fail(IFR_ERR_ARG, "NULL argument");
    if (t->device != c->device) return fail(IFR_ERR_ARG, "tensor lives on device %d, context on %d", t->device, c->device);
    DeviceGuard g(c->device);
    IFR_CHECK_CUDA(ifr::dequant(t->q, out, c->stream), "dequant launch");
    return IFR_OK;
}

int ifr_qgemm(ifr_ctx *c, const ifr_tensor *W, const float *X, int ncols, float *Y) {
    if (!c || !W || !X || !Y) return fail(IFR_ERR_ARG, "NULL argument");
    if (ncols < 1) return fail(IFR_ERR_ARG, "ncols must be >= 1 (got %d)", ncols);
    if (W->device != c->device) return fail(IFR_ERR_ARG, "tensor lives on device %d, context on %d", W->device, c->device);
    if (((uintptr_t)X & 15) || ((uintptr_t)Y & 3)) return fail(IFR_ERR_ARG, "X must be 16-byte and Y 4-byte aligned");
    DeviceGuard g(c->device);
    // scratch for the K halves of tall matrices (second half's partials);
    // not grown while the stream is being captured
    const int64_t kp = W->q.rows * (ncols < IFR_MAX_VERIFY_COLS ? ncols : IFR_MAX_VERIFY_COLS);
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    IFR_CHECK_CUDA(cudaStreamIsCapturing(c->stream, &cap), "cudaStreamIsCapturing");
    if (cap == cudaStreamCaptureStatusNone) {
        const int rc = ensure_scratch(c, (size_t)kp * 4);
        if (rc != IFR_OK) return rc;
    }
    for (int n0 = 0; n0 < ncols; n0 += IFR_MAX_VERIFY_COLS) {
        int n = ncols - n0 < IFR_MAX_VERIFY_COLS ? ncols - n0 : IFR_MAX_VERIFY_COLS;
        ifr::XForm xf;
        xf.act = c->act;
        xf.kpart = (float *)c->scratch;
        xf.kpart_floats = (int64_t)(c->scratch_cap / 4);
        IFR_CHECK_CUDA(ifr::qgemm_small(W->q, X + (int64_t)n0 * W->q.cols, n, Y + (int64_t)n0 * W->q.rows, false,
                                        W->q.rows, c->stream, xf),
                       "qgemm launch");
    }
    return IFR_OK;
}

int ifr_qgemm_rmsnorm(ifr_ctx *c, const ifr_tensor *W, const float *X, int ncols, const float *norm_w, float eps,
                      float *Y) {
    if (!c || !W || !X || !Y || !norm_w) return fail(IFR_ERR_ARG, "NULL argument");
    if (ncols < 1) return fail(IFR_ERR_ARG, "ncols must be >= 1 (got %d)", ncols);
    if (W->device != c->device) return fail(IFR_ERR_ARG, "tensor lives on device %d, context on %d", W->device, c->device);
    if (((uintptr_t)X & 15) || ((uintptr_t)norm_w & 15) || ((uintptr_t)Y & 3))
        return fail(IFR_ERR_ARG, "X and norm_w must be 16-byte and Y 4-byte aligned");
    if (!(eps >= 0.f)) return fail(IFR_ERR_ARG, "eps must be >= 0");
    DeviceGuard g(c->device);
    for (int n0 = 0; n0 < ncols; n0 += IFR_MAX_VERIFY_COLS) {
        int n = ncols - n0 < IFR_MAX_VERIFY_COLS ? ncols - n0 : IFR_MAX_VERIFY_COLS;
        ifr::XForm xf;
        xf.act = c->act;
        xf.kind = 1;
        xf.w = norm_w;
        xf.eps = eps;
        IFR_CHECK_CUDA(ifr::qgemm_small(W->q, X + (int64_t)n0 * W->q.cols, n, Y + (int64_t)n0 * W->q.rows, false,
                                        W->q.rows, c->stream, xf),
                       "qgemm launch");
    }
    return IFR_OK;
}

int ifr_ctx_reserve_dense(ifr_ctx *c, const ifr_tensor *W, int ncols) {
    if (!c || !W) return fail(IFR_ERR_ARG, "NULL argument");
    if (ncols < 1) return fail(IFR_ERR_ARG, "ncols must be >= 1 (got %d)", ncols);
    const int64_t need = ifr::qgemm_dense_scratch_bytes(W->q, ncols);
    if (need < 0) return fail(IFR_ERR_ARG, "no dense plan for this tensor and ncols=%d", ncols);
    DeviceGuard g(c->device);
    return ensure_scratch(c, (size_t)need);
}

int ifr_qgemm_dense(ifr_ctx *c, const ifr_tensor *W, const float *X, int ncols, float *Y) {
    if (!c || !W || !X || !Y) return fail(IFR_ERR_ARG, "NULL argument");
    if (ncols < 1) return fail(IFR_ERR_ARG, "ncols must be >= 1 (got %d)", ncols);
    if (W->device != c->device) return fail(IFR_ERR_ARG, "tensor lives on device %d, context on %d", W->device, c->device);
    if (((uintptr_t)X & 15) || ((uintptr_t)Y & 3)) return fail(IFR_ERR_ARG, "X must be 16-byte and Y 4-byte aligned");
    int rc = ifr_ctx_reserve_dense(c, W, ncols);
    if (rc) return rc;
    DeviceGuard g(c->device);
    IFR_CHECK_CUDA(ifr::qgemm_dense(W->q, X, ncols, Y, false, W->q.rows, c->stream, ifr::XForm(), c->scratch,
                                    (int64_t)c->scratch_cap),
                   "qgemm_dense launch");
    return IFR_OK;
}

int ifr_quantize(int type, const float *x, int64_t rows, int64_t cols, uint8_t *out) {
    if (!x || !out) return fail(IFR_ERR_ARG, "NULL argument");
    if (!valid_type(type)) return fail(IFR_ERR_ARG, "unsupported weight type %d", type);
    if (rows < 0 || cols < 1 || ifr::raw_row_bytes(type, cols) == 0)
        return fail(IFR_ERR_ARG, "cols=%lld is not a multiple of the block size", (long long)cols);
    return ifr::quantize_host(type, x, rows, cols, out) == 0 ? IFR_OK : fail(IFR_ERR_ARG, "quantize failed");
}

int ifr_accept(ifr_ctx *c, const float *target, const float *draft, const int32_t *draft_tokens,
               const float *uniforms, int batch, int gamma, int vocab, float temperature,
               int32_t *accept_count, int32_t *out_tokens, int32_t *draft_out) {
    if (!c || !target || !draft || !uniforms || !accept_count || !out_tokens)
        return fail(IFR_ERR_ARG, "NULL argument");
    if (batch < 1 || gamma < 1 || gamma > 64 || vocab < 1)
        return fail(IFR_ERR_ARG, "invalid sizes batch=%d gamma=%d vocab=%d", batch, gamma, vocab);
    if ((int64_t)batch * (2 * gamma + 1) > ifr::kAcceptMaxRows)
        return fail(IFR_ERR_ARG, "batch=%d gamma=%d: batch * (2 gamma + 1) logits rows exceed %d", batch, gamma,
                    ifr::kAcceptMaxRows);
    if (!(temperature > 0.f) || !(temperature < 1e30f))
        return fail(IFR_ERR_ARG, "temperature must be finite and > 0 (got %g); use ifr_accept_greedy for T=0", (double)temperature);
    DeviceGuard g(c->device);
    int rc = ensure_scratch(c, (size_t)ifr::accept_scratch_bytes(batch, gamma, vocab));
    if (rc) return rc;
    IFR_CHECK_CUDA(ifr::accept_sampled(target, draft, draft_tokens, uniforms, batch, gamma, vocab,
                                       temperature, accept_count, out_tokens, draft_out, c->scratch,
                                       c->stream),
                   "accept launch");
    return IFR_OK;
}

int ifr_accept_filtered(ifr_ctx *c, const float *target, const float *draft, const float *uniforms, int batch,
                        int gamma, int vocab, float temperature, int top_k, float top_p, float min_p,
                        int32_t *accept_count, int32_t *out_tokens, int32_t *draft_out) {
    if (!c || !target || !draft || !uniforms || !accept_count || !out_tokens)
        return fail(IFR_ERR_ARG, "NULL argument");
    if (batch < 1 || gamma < 1 || gamma > 64 || vocab < 1 || vocab > 524288)
        return fail(IFR_ERR_ARG, "invalid sizes batch=%d gamma=%d vocab=%d (vocab must be in 1..524288)", batch,
                    gamma, vocab);
    if ((int64_t)batch * (2 * gamma + 1) > ifr::kAcceptMaxRows)
        return fail(IFR_ERR_ARG, "batch=%d gamma=%d: batch * (2 gamma + 1) logits rows exceed %d", batch, gamma,
                    ifr::kAcceptMaxRows);
    if (!(temperature > 0.f) || !(temperature < 1e30f))
        return fail(IFR_ERR_ARG, "temperature must be finite and > 0 (got %g)", (double)temperature);
    // _validate_sampling_parameters (src/CommonOps.jl:126-139)
    if (!std::isfinite(top_p) || top_p < 0.f || top_p > 1.f) return fail(IFR_ERR_ARG, "top_p must be in [0, 1]");
    if (top_k < 0) return fail(IFR_ERR_ARG, "top_k must be non-negative");
    if (!std::isfinite(min_p) || min_p < 0.f || min_p > 1.f) return fail(IFR_ERR_ARG, "min_p must be in [0, 1]");
    DeviceGuard g(c->device);
    int rc = ensure_scratch(c, (size_t)ifr::accept_filtered_scratch_bytes(batch, gamma, vocab));
    if (rc) return rc;
    IFR_CHECK_CUDA(ifr::accept_filtered(target, draft, uniforms, batch, gamma, vocab, temperature, top_k, top_p,
                                        min_p, accept_count, out_tokens, draft_out, c->scratch, c->stream),
                   "accept_filtered launch");
    return IFR_OK;
}

int ifr_accept_greedy(ifr_ctx *c, const float *target, const int32_t *draft_tokens, int batch,
                      int gamma, int vocab, int32_t *accept_count, int32_t *out_tokens) {
    if (!c || !target || (!draft_tokens && gamma > 0) || !accept_count || !out_tokens)
        return fail(IFR_ERR_ARG, "NULL argument");
    if (batch < 1 || gamma < 0 || vocab < 1)
        return fail(IFR_ERR_ARG, "invalid sizes batch=%d gamma=%d vocab=%d", batch, gamma, vocab);
    DeviceGuard g(c->device);
    int rc = ensure_scratch(c, (size_t)ifr::accept_greedy_scratch_bytes(batch, gamma, vocab));
    if (rc) return rc;
    IFR_CHECK_CUDA(ifr::accept_greedy(target, draft_tokens, batch, gamma, vocab, accept_count, out_tokens,
                                      c->scratch, c->stream),
                   "accept_greedy launch");
    return IFR_OK;
}

int ifr_sample(ifr_ctx *c, const float *logits, int rows, int vocab, float temperature, int top_k, float top_p,
               float min_p, const float *uniforms, int32_t *out_tokens) {
    if (!c || !logits || !uniforms || !out_tokens) return fail(IFR_ERR_ARG, "NULL argument");
    if (rows < 0 || vocab < 1 || vocab > 524288)
        return fail(IFR_ERR_ARG, "invalid sizes rows=%d vocab=%d (vocab must be in 1..524288)", rows, vocab);
    // _validate_sampling_parameters (src/CommonOps.jl:126-139)
    if (!std::isfinite(temperature) || temperature < 0.f)
        return fail(IFR_ERR_ARG, "temperature must be finite and non-negative");
    if (!std::isfinite(top_p) || top_p < 0.f || top_p > 1.f) return fail(IFR_ERR_ARG, "top_p must be in [0, 1]");
    if (top_k < 0) return fail(IFR_ERR_ARG, "top_k must be non-negative");
    if (!std::isfinite(min_p) || min_p < 0.f || min_p > 1.f) return fail(IFR_ERR_ARG, "min_p must be in [0, 1]");
    if (rows == 0) return IFR_OK;
    DeviceGuard g(c->device);
    IFR_CHECK_CUDA(ifr::sample_filtered(logits, rows, vocab, temperature, top_k, top_p, min_p, uniforms, out_tokens,
                                        c->stream),
                   "sample launch");
    return IFR_OK;
}

int ifr_apply_penalties(ifr_ctx *c, float *logits, int rows, int vocab, const int32_t *seen, int n_seen,
                        float presence, float repetition) {
    if (!c || !logits || (!seen && n_seen > 0)) return fail(IFR_ERR_ARG, "NULL argument");
    if (rows < 0 || vocab < 1 || vocab > (1 << 20) || n_seen < 0)
        return fail(IFR_ERR_ARG, "invalid sizes rows=%d vocab=%d n_seen=%d", rows, vocab, n_seen);
    if (!std::isfinite(presence)) return fail(IFR_ERR_ARG, "presence penalty must be finite");
    if (!std::isfinite(repetition) || !(repetition > 0.f))
        return fail(IFR_ERR_ARG, "repetition penalty must be finite and > 0");
    if (rows == 0 || n_seen == 0 || (presence == 0.f && repetition == 1.f)) return IFR_OK;
    DeviceGuard g(c->device);
    IFR_CHECK_CUDA(ifr::apply_penalties(logits, rows, vocab, seen, n_seen, presence, repetition, c->stream),
                   "penalty launch");
    return IFR_OK;
}

}  // extern "C"

// ------------------------------------------------------------ legacy shims ----
// The reference's symbols (src/kernels/quant_kernels.c:602-697) with host
// pointers: one default context on device 0, device buffers kept between calls.
namespace {

std::mutex g_legacy_mu;
ifr_ctx *g_legacy_ctx = nullptr;
void *g_dbuf = nullptr;
size_t g_dbuf_cap = 0;

int legacy_gemv(int type, const uint8_t *weight, const float *x, float *out, int inner, int outer) {
    if (!weight || !x || !out) return fail(IFR_ERR_ARG, "NULL argument");
    if (inner < 1 || outer < 1) return fail(IFR_ERR_ARG, "invalid dims inner=%d outer=%d", inner, outer);
    int64_t rb = ifr::raw_row_bytes(type, inner);
    if (rb == 0) return fail(IFR_ERR_ARG, "inner_dim=%d is not a multiple of the block size", inner);
    std::lock_guard<std::mutex> lk(g_legacy_mu);
    if (!g_legacy_ctx) {
        int rc = ifr_ctx_create(0, &g_legacy_ctx);
        if (rc) return rc;
        g_legacy_ctx->act = IFR_ACT_Q8K;  // the reference kernels' own activation rounding
    }
    ifr_ctx *c = g_legacy_ctx;
    DeviceGuard g(c->device);
    const size_t raw = (size_t)rb * outer, xb = (size_t)inner * 4, yb = (size_t)outer * 4;
    const size_t need = raw + xb + yb + 1024;
    if (need > g_dbuf_cap) {
        if (g_dbuf) cudaFree(g_dbuf);
        g_dbuf = nullptr;
        g_dbuf_cap = 0;
        IFR_CHECK_CUDA(cudaMalloc(&g_dbuf, need), "cudaMalloc(legacy buffers)");
        g_dbuf_cap = need;
    }
    char *draw = (char *)g_dbuf;
    float *dx = (float *)(draw + (raw + 255) / 256 * 256);
    float *dy = (float *)((char *)dx + (xb + 255) / 256 * 256);
    IFR_CHECK_CUDA(cudaMemcpyAsync(draw, weight, raw, cudaMemcpyHostToDevice, c->stream), "H2D weight");
    IFR_CHECK_CUDA(cudaMemcpyAsync(dx, x, xb, cudaMemcpyHostToDevice, c->stream), "H2D x");
    ifr_tensor *t = nullptr;
    int rc = ifr_weights_from_device(c, type, draw, outer, inner, &t);
    if (rc) return rc;
    rc = ifr_qgemm(c, t, dx, 1, dy);
    if (rc == IFR_OK) {
        cudaError_t e = cudaMemcpyAsync(out, dy, yb, cudaMemcpyDeviceToHost, c->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
        if (e != cudaSuccess) rc = cuda_fail(e, "D2H out");
    }
    ifr_tensor_free(t);
    return rc;
}

void legacy_entry(int type, const char *name, const uint8_t *w, const float *x, float *out, int inner,
                  int outer) {
    int rc = legacy_gemv(type, w, x, out, inner, outer);
    if (rc != IFR_OK) {
        fprintf(stderr, "inferno_b200 %s failed: %s\n", name, g_err.c_str());
        if (out && outer > 0)
            for (int i = 0; i < outer; i++) out[i] = nanf("");
    }
}

}  // namespace

extern "C" {
void q4_k_gemv(const uint8_t *w, const float *x, float *out, void *, int inner, int outer) {
    legacy_entry(IFR_TYPE_Q4_K, "q4_k_gemv", w, x, out, inner, outer);
}
void q5_k_gemv(const uint8_t *w, const float *x, float *out, void *, int inner, int outer) {
    legacy_entry(IFR_TYPE_Q5_K, "q5_k_gemv", w, x, out, inner, outer);
}
void q6_k_gemv(const uint8_t *w, const float *x, float *out, void *, int inner, int outer) {
    legacy_entry(IFR_TYPE_Q6_K, "q6_k_gemv", w, x, out, inner, outer);
}
void q8_0_gemv(const uint8_t *w, const float *x, float *out, int inner, int outer) {
    legacy_entry(IFR_TYPE_Q8_0, "q8_0_gemv", w, x, out, inner, outer);
}
}
