// The small-N verify GEMV kernels for one weight format (GGML type 8).
#define IFR_QGEMV_FMT 8
#include "qgemv_kernels.cuh"
