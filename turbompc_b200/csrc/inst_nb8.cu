// Explicit instantiation of the block-size-8 kernels and launchers.
#include "admm_kernel.cuh"
#include "schur_pcg_kernels.cuh"

#define TMPC_NB 8
#include "inst_body.cuh"
