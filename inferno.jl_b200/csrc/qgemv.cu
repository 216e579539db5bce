// Small-N quantized GEMM ("verify GEMV") entry points: argument checks and
// dispatch to the kernels of each weight format (qgemv_kernels.cuh, compiled
// once per format in qgemv_q4k.cu, qgemv_q5k.cu, qgemv_q6k.cu, qgemv_q80.cu).
//
// Replaces q4_k_gemv .. q8_0_gemv (reference src/kernels/quant_kernels.c:602-697).
#include "common.cuh"
#include "fused.cuh"

namespace ifr {

cudaError_t qgemm_small(const QTensor &T, const float *X, int ncols, float *Y, bool accumulate, int64_t ldy,
                        cudaStream_t s, const XForm &xf) {
    if (ncols < 1 || ncols > 8) return cudaErrorInvalidValue;
    if (xf.kind < 0 || xf.kind > 2 || (xf.kind == 1 && !xf.w)) return cudaErrorInvalidValue;
    if (xf.ep && (accumulate || T.rows % 32)) return cudaErrorInvalidValue;
    if (xf.am && (xf.ep || accumulate || !xf.am->cand || !xf.am->counter || !xf.am->out || xf.am->G < 0 ||
                  ncols % (xf.am->G + 1) || (xf.am->G > 0 && !xf.am->drafts)))
        return cudaErrorInvalidValue;
    if (xf.act != 0 && xf.act != 1) return cudaErrorInvalidValue;
    switch (T.type) {
    case 12: return qgemm_small_fmt<12>(T, X, ncols, Y, accumulate, ldy, s, xf);
    case 13: return qgemm_small_fmt<13>(T, X, ncols, Y, accumulate, ldy, s, xf);
    case 14: return qgemm_small_fmt<14>(T, X, ncols, Y, accumulate, ldy, s, xf);
    case 8: return qgemm_small_fmt<8>(T, X, ncols, Y, accumulate, ldy, s, xf);
    }
    return cudaErrorInvalidValue;
}

// the flags of every format's kernels and of the dense kernel, read and cleared
cudaError_t read_device_error(int *flag, cudaStream_t s) {
    int f[6] = {0, 0, 0, 0, 0, 0};
    cudaError_t e = read_dev_error_fmt<12>(&f[0], s);
    if (e == cudaSuccess) e = read_dev_error_fmt<13>(&f[1], s);
    if (e == cudaSuccess) e = read_dev_error_fmt<14>(&f[2], s);
    if (e == cudaSuccess) e = read_dev_error_fmt<8>(&f[3], s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess) e = read_fused_error(&f[5], s);
    if (e == cudaSuccess) e = read_mma_error(&f[4], s);
    *flag = (f[0] | f[1] | f[2] | f[3] | f[4] | f[5]) ? 1 : 0;
    return e;
}

}  // namespace ifr
