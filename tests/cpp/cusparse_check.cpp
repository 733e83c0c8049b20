// The reference bench's cuSPARSE baselines as the drop-in provides them
// (cusparse_spmv_csr_f32/f64, cusparse_spmm_f32/f64): built and linked like
// the reference's bench target (-lcusparse); run on a GPU, each result must
// agree with the library's SpmvRunner / spmm_csr_tiled within the gamma_n
// bound of the reference's GPU test (cuSPARSE sums in its own order).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <random>
#include <vector>

#include "spmvbench/spmm_cuda.cuh"
#include "spmvbench/spmv_cuda.cuh"

using namespace spmvbench;

static int g_fail = 0, g_pass = 0;
#define EXPECT(cond)                                                                 \
  do {                                                                               \
    if (cond) ++g_pass;                                                              \
    else { ++g_fail; std::printf("FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond); } \
  } while (0)

template <typename T>
static CsrMatrix<T> random_csr(int m, int n, int per_row, unsigned seed) {
  std::mt19937_64 rng(seed);
  std::uniform_int_distribution<int> col(0, n - 1);
  std::uniform_real_distribution<double> val(-1.0, 1.0);
  CsrMatrix<T> A(m, n);
  std::vector<char> seen(n, 0);
  for (int i = 0; i < m; ++i) {
    const int len = (i % 7 == 0) ? 0 : per_row + i % 5;  // some empty rows; distinct sorted columns
    std::vector<int> cols;
    while (static_cast<int>(cols.size()) < len) {
      const int c = col(rng);
      if (!seen[c]) { seen[c] = 1; cols.push_back(c); }
    }
    std::sort(cols.begin(), cols.end());
    for (int c : cols) {
      seen[c] = 0;
      A.colind.push_back(c);
      A.values.push_back(static_cast<T>(val(rng)));
    }
    A.rowptr[i + 1] = static_cast<Index>(A.colind.size());
  }
  A.nnz = A.rowptr[m];
  return A;
}

// |got - ref| <= 2 * gamma_len(u) * sum_j |a_ij x_j| per output, u the unit
// roundoff of T (the reference's tests/test_cuda_correctness.cpp:1-11, 88).
template <typename T>
static bool within_gamma(const CsrMatrix<T>& A, const std::vector<T>& x, int k, const std::vector<T>& ref,
                         const std::vector<T>& got) {
  const double u = std::is_same_v<T, double> ? std::ldexp(1.0, -53) : std::ldexp(1.0, -24);
  if (ref.size() != got.size()) return false;
  for (int i = 0; i < A.m; ++i) {
    const int len = A.rowptr[i + 1] - A.rowptr[i];
    const double g = len * u / (1.0 - len * u);
    for (int c = 0; c < k; ++c) {
      double s = 0.0;
      for (Index p = A.rowptr[i]; p < A.rowptr[i + 1]; ++p)
        s += std::fabs(double(A.values[p]) * double(x[static_cast<size_t>(A.colind[p]) * k + c]));
      const size_t o = static_cast<size_t>(i) * k + c;
      if (std::fabs(double(got[o]) - double(ref[o])) > 2.0 * g * s) return false;
    }
  }
  return true;
}

template <typename T>
static void check_spmv() {
  const CsrMatrix<T> A = random_csr<T>(3000, 2000, 9, 5);
  std::vector<T> x(A.n);
  std::mt19937_64 rng(6);
  std::uniform_real_distribution<double> val(-1.0, 1.0);
  for (auto& v : x) v = static_cast<T>(val(rng));
  std::vector<T> y;
  SpmvResult r;
  if constexpr (std::is_same_v<T, double>) r = cusparse_spmv_csr_f64(A, x, y, 5, 2);
  else r = cusparse_spmv_csr_f32(A, x, y, 5, 2);
  EXPECT(r.kernel == "cusparse_spmv" && r.iters == 5 && r.median_ms > 0 && r.transfer_ms > 0);
  SpmvRunner<T, T> runner(A);
  runner.set_x(x);
  runner.run(KernelId::CsrScalar, 1, 4, 4, 0);
  EXPECT(within_gamma(A, x, 1, runner.result(), y));
}

template <typename T>
static void check_spmm() {
  const CsrMatrix<T> A = random_csr<T>(2000, 1500, 7, 9);
  const int k = 24;
  std::vector<T> B(static_cast<size_t>(A.n) * k);
  std::mt19937_64 rng(10);
  std::uniform_real_distribution<double> val(-1.0, 1.0);
  for (auto& v : B) v = static_cast<T>(val(rng));
  std::vector<T> Yc, Y;
  SpmmResult r;
  if constexpr (std::is_same_v<T, double>) {
    r = cusparse_spmm_f64(A, B, k, 5, 2, Yc);
    spmm_csr_tiled_f64(A, B, k, 32, false, 1, 0, Y);
  } else {
    r = cusparse_spmm_f32(A, B, k, 5, 2, Yc);
    spmm_csr_tiled_f32(A, B, k, 32, false, 1, 0, Y);
  }
  EXPECT(r.kernel == "cusparse_spmm" && r.iters == 5 && r.median_ms > 0 && r.transfer_ms > 0);
  EXPECT(within_gamma(A, B, k, Y, Yc));
}

int main() {
  check_spmv<double>();
  check_spmv<float>();
  check_spmm<double>();
  check_spmm<float>();
  std::printf("%d passed, %d failed\n", g_pass, g_fail);
  return g_fail == 0 ? 0 : 1;
}
