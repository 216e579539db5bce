// The small-N verify GEMV kernels for one weight format (GGML type 12).
#define IFR_QGEMV_FMT 12
#include "qgemv_kernels.cuh"
