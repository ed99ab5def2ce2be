// Instantiates the 4-bit GEMV kernels for 4 activation rows (see gemv_impl.cuh).
#include "gemv_impl.cuh"

AGXC_GEMV_INSTANTIATE(4, 4)
