// Instantiation of the SpMV / SpMM launchers for T = float, Acc = float.
#include "spmv_launch.cuh"

namespace spmvb {
template spmvb_status launch_spmv<float, float>(spmvb_matrix, spmvb_kernel, int, int,
                                          const float*, float*, cudaStream_t);
template spmvb_status launch_spmm<float, float>(spmvb_matrix, int, int, int,
                                          const float*, float*, cudaStream_t);
}  // namespace spmvb
