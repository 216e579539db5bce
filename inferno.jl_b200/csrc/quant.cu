// Device layout (M-tiles, tiles.cuh): re-layout of GGUF blocks at upload, and
// the bit-exact dequantization kernels.
//
// Dequantized values follow the reference's src/Dequant.jl exactly: f32
// products rounded separately (no fused multiply-add, which Julia does not
// form there), hence the explicit __fmul_rn/__fsub_rn.
#include "common.cuh"
#include "tiles.cuh"
#include "dequant.cuh"

namespace ifr {

int64_t raw_row_bytes(int type, int64_t cols) {
    switch (type) {
    case 8: return (cols % 32) ? 0 : cols / 32 * 34;
    case 12: return (cols % 256) ? 0 : cols / 256 * 144;
    case 13: return (cols % 256) ? 0 : cols / 256 * 176;
    case 14: return (cols % 256) ? 0 : cols / 256 * 210;
    }
    return 0;
}

int64_t device_bytes(int type, int64_t rows, int64_t cols) {
    if (raw_row_bytes(type, cols) == 0) return 0;
    return (rows + 15) / 16 * ((cols + 255) / 256) * mtile_bytes(type);
}

// ---------------------------------------------------------------- repack ----
// one thread per (row, unit): that row's bits of the unit go to their M-tile
// places (tiles.cuh); padding rows and missing Q8_0 blocks become zeros.
template <int T>
__global__ void repack_kernel(const uint8_t *__restrict__ raw, uint8_t *__restrict__ dst, int64_t rows,
                              int64_t nrb, int64_t nu, int64_t nb_raw) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= nrb * 16 * nu) return;
    const int64_t u = i % nu, row = i / nu;
    const int r = (int)(row & 15);
    uint8_t *tile = dst + ((row >> 4) * nu + u) * mtile_bytes(T);
    const bool pad = row >= rows;
    const int BB = raw_block_bytes(T);
    if (T == 12 || T == 13) {
        constexpr bool q5 = T == 13;
        const uint8_t *b = raw + (row * nb_raw + u) * BB;
        const int qs0 = q5 ? 48 : 16;
        for (int k = 0; k < 16; k++) tile[qk_hdr(r) + k] = pad ? 0 : b[k];
        for (int q = 0; q < 128; q++) tile[qk_qs_byte(q5, r, q)] = pad ? 0 : b[qs0 + q];
        if (q5)
            for (int l = 0; l < 32; l++) tile[q5_qh_byte(r, l)] = pad ? 0 : b[16 + l];
    } else if (T == 14) {
        const uint8_t *b = raw + (row * nb_raw + u) * BB;
        tile[q6_d(r)] = pad ? 0 : b[208];
        tile[q6_d(r) + 1] = pad ? 0 : b[209];
        for (int k = 0; k < 16; k++) tile[q6_sc(r) + k] = pad ? 0 : b[192 + k];
        for (int q = 0; q < 128; q++) tile[q6_ql_byte(r, q)] = pad ? 0 : b[q];
        for (int h = 0; h < 64; h++) tile[q6_qh_byte(r, h)] = pad ? 0 : b[128 + h];
    } else {  // Q8_0: unit u = raw blocks 8u .. 8u+7
        for (int bl = 0; bl < 8; bl++) {
            const int64_t rb = 8 * u + bl;
            const bool miss = pad || rb >= nb_raw;
            const uint8_t *b = raw + (row * nb_raw + rb) * BB;
            tile[q8_d(r) + 2 * bl] = miss ? 0 : b[0];
            tile[q8_d(r) + 2 * bl + 1] = miss ? 0 : b[1];
            for (int p = 0; p < 32; p++) tile[q8_qs_byte(r, 32 * bl + p)] = miss ? 0 : b[2 + p];
        }
    }
}

cudaError_t repack(const QTensor &t, const uint8_t *raw, cudaStream_t s) {
    const int64_t n = t.nrb * 16 * t.nu;
    if (n == 0) return cudaSuccess;
    const int threads = 128;
    const unsigned grid = (unsigned)((n + threads - 1) / threads);
    switch (t.type) {
    case 12: repack_kernel<12><<<grid, threads, 0, s>>>(raw, t.data, t.rows, t.nrb, t.nu, t.nb); break;
    case 13: repack_kernel<13><<<grid, threads, 0, s>>>(raw, t.data, t.rows, t.nrb, t.nu, t.nb); break;
    case 14: repack_kernel<14><<<grid, threads, 0, s>>>(raw, t.data, t.rows, t.nrb, t.nu, t.nb); break;
    case 8: repack_kernel<8><<<grid, threads, 0, s>>>(raw, t.data, t.rows, t.nrb, t.nu, t.nb); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// --------------------------------------------------------------- dequant ----

// one thread per (row, unit, 32-element sub-group); writes out[row][u*256 + ...]
// (idx: optional row indices, e.g. token ids of an embedding gather; clamped
// to the tensor's rows; output row i holds source row idx[i])
template <int T>
__global__ void dequant_kernel(const uint8_t *__restrict__ w, float *__restrict__ out, int64_t rows,
                               int64_t cols, int64_t nu, int64_t nb_raw, const int32_t *__restrict__ idx,
                               int64_t src_rows) {
    pdl_trigger();
    pdl_wait();
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= rows * nu * 8) return;
    const int sub = (int)(i & 7);
    const int64_t u = (i >> 3) % nu, orow = (i >> 3) / nu;
    int64_t row = orow;
    if (idx) {
        row = idx[orow];
        row = row < 0 ? 0 : (row >= src_rows ? src_rows - 1 : row);
    }
    dequant_group<T>(w, nu, nb_raw, row, u, sub, out + orow * cols + u * 256 + 32 * sub);
}

cudaError_t dequant_rows(const QTensor &t, const int32_t *idx, int64_t nrows, float *out, cudaStream_t s) {
    const int64_t n = nrows * t.nu * 8;
    if (n == 0) return cudaSuccess;
    const int threads = 128;
    const unsigned grid = (unsigned)((n + threads - 1) / threads);
    switch (t.type) {
    case 12: return launch_k(dequant_kernel<12>, dim3(grid), dim3(threads), 0, s, (const uint8_t *)t.data, out, nrows, t.cols, t.nu, t.nb, idx, t.rows);
    case 13: return launch_k(dequant_kernel<13>, dim3(grid), dim3(threads), 0, s, (const uint8_t *)t.data, out, nrows, t.cols, t.nu, t.nb, idx, t.rows);
    case 14: return launch_k(dequant_kernel<14>, dim3(grid), dim3(threads), 0, s, (const uint8_t *)t.data, out, nrows, t.cols, t.nu, t.nb, idx, t.rows);
    case 8: return launch_k(dequant_kernel<8>, dim3(grid), dim3(threads), 0, s, (const uint8_t *)t.data, out, nrows, t.cols, t.nu, t.nb, idx, t.rows);
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t dequant(const QTensor &t, float *out, cudaStream_t s) { return dequant_rows(t, nullptr, t.rows, out, s); }

}  // namespace ifr
