// Instantiation of the SpMV / SpMM launchers for T = float, Acc = double.
#include "spmv_launch.cuh"

namespace spmvb {
template spmvb_status launch_spmv<float, double>(spmvb_matrix, spmvb_kernel, int, int,
                                          const float*, double*, cudaStream_t);
template spmvb_status launch_spmm<float, double>(spmvb_matrix, int, int, int,
                                          const float*, double*, cudaStream_t);
}  // namespace spmvb
