// The small-N verify GEMV kernels for one weight format (GGML type 14).
#define IFR_QGEMV_FMT 14
#include "qgemv_kernels.cuh"
