// Instantiates the 8-bit GEMV kernels for 1 activation row (see gemv_impl.cuh).
#include "gemv_impl.cuh"

AGXC_GEMV_INSTANTIATE(8, 1)
