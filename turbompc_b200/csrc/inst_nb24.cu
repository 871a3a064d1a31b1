// Explicit instantiation of the block-size-24 kernels and launchers.
#include "admm_kernel.cuh"
#include "schur_pcg_kernels.cuh"

#define TMPC_NB 24
#include "inst_body.cuh"
