// Body shared by inst_nb*.cu: instantiates every launcher for TMPC_NB.
namespace tmpc {
#define TMPC_INST(R)                                                                                          \
  template int launch_admm_nb<TMPC_NB, R>(const AdmmParams<R>&, size_t, cudaStream_t);                       \
  template int launch_admm_direct_nb<TMPC_NB, R>(const AdmmParams<R>&, size_t, cudaStream_t);                \
  template size_t admm_smem_bytes<TMPC_NB, R>(int, int, int, int, bool);                                      \
  template int launch_assemble_ref<TMPC_NB, R>(const TmpcDims*, const TmpcQP*, const R*, R, R, R*, R*,      \
                                               int32_t*, cudaStream_t);                                      \
  template int launch_assemble_packed<TMPC_NB, R>(const TmpcDims*, const TmpcQP*, const R*, R, R, R*,        \
                                                  int32_t*, cudaStream_t);                                   \
  template int launch_pcg_packed<TMPC_NB, R>(const TmpcDims*, const R*, const R*, const R*, R*, uint32_t*, R, \
                                             int, cudaStream_t);
TMPC_INST(float)
TMPC_INST(double)
#undef TMPC_INST
}  // namespace tmpc
