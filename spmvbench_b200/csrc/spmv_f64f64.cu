// Instantiation of the SpMV / SpMM launchers for T = double, Acc = double.
#include "spmv_launch.cuh"

namespace spmvb {
template spmvb_status launch_spmv<double, double>(spmvb_matrix, spmvb_kernel, int, int,
                                          const double*, double*, cudaStream_t);
template spmvb_status launch_spmm<double, double>(spmvb_matrix, int, int, int,
                                          const double*, double*, cudaStream_t);
}  // namespace spmvb
