// Explicit instantiation of the block-size-16 kernels and launchers.
#include "admm_kernel.cuh"
#include "schur_pcg_kernels.cuh"

#define TMPC_NB 16
#include "inst_body.cuh"
