// Instantiates the 8-bit GEMV kernels for 2 activation rows (see gemv_impl.cuh).
#include "gemv_impl.cuh"

AGXC_GEMV_INSTANTIATE(8, 2)
