// Instantiates the 4-bit GEMV kernels for 2 activation rows (see gemv_impl.cuh).
#include "gemv_impl.cuh"

AGXC_GEMV_INSTANTIATE(4, 2)
