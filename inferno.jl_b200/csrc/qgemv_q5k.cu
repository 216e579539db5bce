// The small-N verify GEMV kernels for one weight format (GGML type 13).
#define IFR_QGEMV_FMT 13
#include "qgemv_kernels.cuh"
