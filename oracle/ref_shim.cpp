// ref_shim.cpp - extern "C" entry points over the REFERENCE's own CPU code,
// compiled together with the reference sources (oracle/Makefile) into
// oracle/_ref/libspmvref.so. Test infrastructure only: it lets the tests pin
// the C restatement in oracle.c against the reference itself, and lets
// bench.py time the reference's csr_omp as the CPU baseline.
//
// The reference namespace is renamed to spmvbench_ref at compile time
// (-Dspmvbench=spmvbench_ref) so these symbols can never collide with the
// drop-in C++ API of this repository.
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "spmvbench/bcsr.hpp"
#include "spmvbench/csr.hpp"
#include "spmvbench/ell.hpp"
#include "spmvbench/mtx_io.hpp"
#include "spmvbench/select.hpp"
#include "spmvbench/spmv_cpu.hpp"
#include "spmvbench/stats.hpp"

namespace R = spmvbench;

namespace {
template <typename T>
R::CsrMatrix<T>* make(int32_t m, int32_t n, int64_t nnz, const int32_t* rp, const int32_t* ci, const T* v) {
  auto* A = new R::CsrMatrix<T>();
  A->m = m;
  A->n = n;
  A->nnz = nnz;
  A->rowptr.assign(rp, rp + m + 1);
  A->colind.assign(ci, ci + nnz);
  A->values.assign(v, v + nnz);
  return A;
}
}  // namespace

extern "C" {

void* ref_csr_create_d(int32_t m, int32_t n, int64_t nnz, const int32_t* rp, const int32_t* ci, const double* v) {
  return make<double>(m, n, nnz, rp, ci, v);
}
void* ref_csr_create_f(int32_t m, int32_t n, int64_t nnz, const int32_t* rp, const int32_t* ci, const float* v) {
  return make<float>(m, n, nnz, rp, ci, v);
}
void ref_csr_destroy_d(void* h) { delete static_cast<R::CsrMatrix<double>*>(h); }
void ref_csr_destroy_f(void* h) { delete static_cast<R::CsrMatrix<float>*>(h); }

// read_matrix_market<double> (src/mtx_io.cpp:40-172); returns nullptr and
// copies the message on error.
void* ref_read_mtx_d(const char* path, char* err, int errcap) {
  try {
    return new R::CsrMatrix<double>(R::read_matrix_market<double>(path));
  } catch (const std::exception& e) {
    if (err && errcap > 0) std::snprintf(err, errcap, "%s", e.what());
    return nullptr;
  }
}
void ref_csr_shape_d(void* h, int32_t* m, int32_t* n, int64_t* nnz) {
  auto* A = static_cast<R::CsrMatrix<double>*>(h);
  *m = A->m;
  *n = A->n;
  *nnz = A->nnz;
}
void ref_csr_arrays_d(void* h, int32_t* rp, int32_t* ci, double* v) {
  auto* A = static_cast<R::CsrMatrix<double>*>(h);
  std::memcpy(rp, A->rowptr.data(), A->rowptr.size() * 4);
  if (A->nnz) {
    std::memcpy(ci, A->colind.data(), A->colind.size() * 4);
    std::memcpy(v, A->values.data(), A->values.size() * 8);
  }
}

void ref_spmv_csr_dd(void* h, const double* x, double* y, int nt) {
  R::spmv_csr_cpu<double, double>(*static_cast<R::CsrMatrix<double>*>(h), x, y, nt);
}
void ref_spmv_csr_ff(void* h, const float* x, float* y, int nt) {
  R::spmv_csr_cpu<float, float>(*static_cast<R::CsrMatrix<float>*>(h), x, y, nt);
}
void ref_spmv_csr_fd(void* h, const float* x, double* y, int nt) {
  R::spmv_csr_cpu<float, double>(*static_cast<R::CsrMatrix<float>*>(h), x, y, nt);
}
void ref_spmv_merge_dd(void* h, const double* x, double* y, int nt) {
  R::spmv_csr_merge_cpu<double, double>(*static_cast<R::CsrMatrix<double>*>(h), x, y, nt);
}
void ref_spmm_csr_dd(void* h, const double* B, double* Y, int k, int nt) {
  R::spmm_csr_cpu<double, double>(*static_cast<R::CsrMatrix<double>*>(h), B, Y, k, nt);
}
void ref_spmm_csr_ff(void* h, const float* B, float* Y, int k, int nt) {
  R::spmm_csr_cpu<float, float>(*static_cast<R::CsrMatrix<float>*>(h), B, Y, k, nt);
}
void ref_spmm_csr_fd(void* h, const float* B, double* Y, int k, int nt) {
  R::spmm_csr_cpu<float, double>(*static_cast<R::CsrMatrix<float>*>(h), B, Y, k, nt);
}

// csr_to_ell (src/formats.cpp:14-43): width first, then the arrays.
int32_t ref_ell_width_d(void* h) { return R::csr_to_ell(*static_cast<R::CsrMatrix<double>*>(h)).max_row_nnz; }
void ref_csr_to_ell_d(void* h, int32_t* ecol, double* ev, int32_t* rl) {
  const auto E = R::csr_to_ell(*static_cast<R::CsrMatrix<double>*>(h));
  std::memcpy(ecol, E.colind.data(), E.colind.size() * 4);
  std::memcpy(ev, E.values.data(), E.values.size() * 8);
  std::memcpy(rl, E.row_lengths.data(), E.row_lengths.size() * 4);
}
void ref_spmv_ell_dd(void* h, const double* x, double* y, int nt) {
  const auto E = R::csr_to_ell(*static_cast<R::CsrMatrix<double>*>(h));
  R::spmv_ell_cpu<double, double>(E, x, y, nt);
}

// csr_to_bcsr<double,B,B> (src/formats.cpp:45-105).
static R::BcsrMatrix<double> to_bcsr(void* h, int block) {
  const auto& A = *static_cast<R::CsrMatrix<double>*>(h);
  return block == 2 ? R::csr_to_bcsr<double, 2, 2>(A) : R::csr_to_bcsr<double, 4, 4>(A);
}
void ref_bcsr_shape_d(void* h, int block, int32_t* mb, int64_t* block_nnz) {
  const auto B = to_bcsr(h, block);
  *mb = B.mb;
  *block_nnz = B.block_nnz;
}
void ref_csr_to_bcsr_d(void* h, int block, int32_t* rp, int32_t* ci, double* v) {
  const auto B = to_bcsr(h, block);
  std::memcpy(rp, B.rowptr.data(), B.rowptr.size() * 4);
  if (B.block_nnz) {
    std::memcpy(ci, B.colind.data(), B.colind.size() * 4);
    std::memcpy(v, B.values.data(), B.values.size() * 8);
  }
}
void ref_spmv_bcsr_dd(void* h, int block, const double* x, double* y, int nt) {
  const auto B = to_bcsr(h, block);
  R::spmv_bcsr_cpu<double, double>(B, x, y, nt);
}

// compute_row_stats (src/stats.cpp:13-123), packed like orc_row_stats.
void ref_row_stats(const int32_t* rp, const int32_t* ci, int32_t m, int32_t n, int64_t nnz, double* out,
                   int64_t* hist, int64_t hist_cap) {
  const R::RowStats s = R::compute_row_stats(rp, ci, m, n, nnz);
  const double v[13] = {static_cast<double>(s.nnz), double(s.rows), double(s.cols), s.mean_row_nnz,
                        s.median_row_nnz, double(s.min_row_nnz), double(s.max_row_nnz), s.stddev_row_nnz,
                        s.cv_row_nnz, s.max_over_mean, s.ell_padding_overhead, s.frac_dense_blocks_4x4,
                        s.density};
  std::memcpy(out, v, sizeof(v));
  if (hist)
    for (size_t i = 0; i < s.row_nnz_histogram.size() && int64_t(i) < hist_cap; ++i) hist[i] = s.row_nnz_histogram[i];
}

// choose_spmv (src/select.cpp:93-165) on stats packed like orc_row_stats.
void ref_choose_spmv(const double* st, int32_t* out, char* reason, int cap) {
  R::RowStats s;
  s.nnz = static_cast<int64_t>(st[0]);
  s.rows = static_cast<int>(st[1]);
  s.cols = static_cast<int>(st[2]);
  s.mean_row_nnz = st[3];
  s.median_row_nnz = st[4];
  s.min_row_nnz = static_cast<int>(st[5]);
  s.max_row_nnz = static_cast<int>(st[6]);
  s.stddev_row_nnz = st[7];
  s.cv_row_nnz = st[8];
  s.max_over_mean = st[9];
  s.ell_padding_overhead = st[10];
  s.frac_dense_blocks_4x4 = st[11];
  s.density = st[12];
  const R::KernelChoice c = R::choose_spmv(s);
  out[0] = static_cast<int32_t>(c.kernel);
  out[1] = c.lanes;
  out[2] = c.block_r;
  out[3] = c.block_c;
  if (reason && cap > 0) std::snprintf(reason, cap, "%s", c.reason.c_str());
}

}  // extern "C"
