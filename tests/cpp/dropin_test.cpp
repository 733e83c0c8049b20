// Drop-in API test: the reference's own test cases, written against the
// SpMVBench C++ interface (include/spmvbench), linked to libspmvb.
//   dropin_test cpu   formats, stats, selection (no GPU needed)
//   dropin_test gpu   SpmvRunner / spmm_csr_tiled_* on the device, checked
//                     like tests/test_cuda_correctness.cpp (gamma_n bound;
//                     csr_scalar and ELL bit for bit)
//   dropin_test fuzz LIB  csr_to_ell / csr_to_bcsr<2x2, 4x4> on random
//                     matrices against the reference's own conversions in
//                     LIB (oracle/_ref/libspmvref.so), bit for bit
#include <dlfcn.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <utility>
#include <vector>

#include "spmvbench/bcsr.hpp"
#include "spmvbench/ell.hpp"
#include "spmvbench/select.hpp"
#include "spmvbench/spmm_cuda.cuh"
#include "spmvbench/spmv_cuda.cuh"
#include "spmvbench/stats.hpp"

using namespace spmvbench;

static int g_fail = 0, g_pass = 0;
#define EXPECT(cond)                                                     \
  do {                                                                   \
    if (cond) ++g_pass;                                                  \
    else { ++g_fail; std::printf("FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond); } \
  } while (0)

// tests/test_util.hpp:28-51 of the reference (make_csr): rows as (col, val) lists.
static CsrMatrix<double> make_csr(int m, int n, const std::vector<std::vector<std::pair<int, double>>>& rows) {
  CsrMatrix<double> A(m, n);
  for (int i = 0; i < m; ++i) A.rowptr[i + 1] = A.rowptr[i] + static_cast<Index>(rows[i].size());
  A.nnz = A.rowptr[m];
  for (const auto& r : rows)
    for (const auto& [c, v] : r) {
      A.colind.push_back(c);
      A.values.push_back(v);
    }
  return A;
}

static std::vector<double> naive(const CsrMatrix<double>& A, const std::vector<double>& x) {
  std::vector<double> y(A.m, 0.0);
  for (int i = 0; i < A.m; ++i) {
    double s = 0.0;
    for (Index p = A.rowptr[i]; p < A.rowptr[i + 1]; ++p) s += A.values[p] * x[A.colind[p]];
    y[i] = s;
  }
  return y;
}

static CsrMatrix<double> sample() {  // tests/test_formats.cpp:13-19
  return make_csr(3, 4, {{{0, 1.0}, {3, 2.0}}, {{1, 3.0}}, {{0, 4.0}, {1, 5.0}, {2, 6.0}, {3, 7.0}}});
}

static void cpu_tests() {
  // Formats (tests/test_formats.cpp:23-107)
  const auto A = sample();
  {  // a B shorter than n*k is refused before any device work
    std::vector<double> B(A.n * 3 - 1), Y;
    bool threw = false;
    try {
      spmm_csr_tiled_f64(A, B, 3, 32, false, 1, 0, Y);
    } catch (const std::runtime_error&) {
      threw = true;
    }
    EXPECT(threw);
  }
  const auto ell = csr_to_ell(A);
  EXPECT(ell.max_row_nnz == 4 && ell.padded_nnz == 12 && ell.nnz == 7);
  EXPECT(ell.row_lengths == std::vector<int>({2, 1, 4}));
  for (int j = 1; j < 4; ++j) EXPECT(ell.colind[j * 3 + 1] == 0 && ell.values[j * 3 + 1] == 0.0);
  EXPECT(std::fabs(ell.padding_overhead() - 12.0 / 7.0) < 1e-15);
  const auto b2 = csr_to_bcsr<double, 2, 2>(A);
  EXPECT(b2.mb == 2 && b2.nb == 2 && b2.block_nnz == 4 && b2.values.size() == 16u);
  const auto b4 = csr_to_bcsr<double, 4, 4>(A);
  EXPECT(b4.mb == 1 && b4.block_nnz == 1 && b4.density() == 7.0 / 16.0);
  // Stats (tests/test_stats.cpp:10-75)
  std::vector<std::vector<std::pair<int, double>>> rows(4);
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j <= i; ++j) rows[i].push_back({j, 1.0});
  const auto s = compute_row_stats(make_csr(4, 4, rows));
  EXPECT(s.nnz == 10 && s.mean_row_nnz == 2.5 && s.median_row_nnz == 2.5);
  EXPECT(s.min_row_nnz == 1 && s.max_row_nnz == 4);
  EXPECT(std::fabs(s.stddev_row_nnz - std::sqrt(1.25)) < 1e-12);
  EXPECT(s.density == 10.0 / 16.0 && s.ell_padding_overhead == 1.6);
  EXPECT(s.row_nnz_histogram == std::vector<std::int64_t>({0, 1, 1, 1, 1}));
  // Selection: reference rules (tests/test_select.cpp:11-83) and B200 rules
  RowStats t;
  t.nnz = 1000;
  t.mean_row_nnz = 10;
  EXPECT(choose_spmv_reference(t).kernel == KernelId::CsrScalar);
  t.nnz = 1000000;
  t.mean_row_nnz = 10.0;
  t.cv_row_nnz = 0.2;
  t.max_over_mean = 2.0;
  t.ell_padding_overhead = 2.5;
  const auto c = choose_spmv_reference(t);
  EXPECT(c.kernel == KernelId::CsrVector && c.lanes == 16 && !c.reason.empty());
  t.cv_row_nnz = 5.0;
  t.max_over_mean = 200.0;
  EXPECT(choose_spmv(t).kernel == KernelId::Hyb);
  EXPECT(std::string(kernel_name(KernelId::Hyb)) == "hyb");
}

static double gamma_n(int n, double u) { return n * u / (1.0 - n * u); }

static void gpu_tests() {
  if (!gpu_available()) {
    std::printf("FAIL: gpu tests requested without a CUDA device\n");
    ++g_fail;
    return;
  }
  const GpuInfo g = query_gpu();
  EXPECT(g.major >= 10);
  // A seeded uniform matrix with mixed-magnitude x (tests/test_cuda_correctness.cpp:58-70).
  const int m = 20000, n = 20000, per = 16;
  std::mt19937 rng(1234);
  std::uniform_int_distribution<int> col(0, n - 1);
  std::uniform_real_distribution<double> val(-1.0, 1.0), e(-6.0, 6.0), bit(0.0, 1.0);
  std::vector<std::vector<std::pair<int, double>>> rows(m);
  // distinct columns per row (base + j*4729 mod n, gcd(4729, n) = 1): BCSR
  // keeps only the last of repeated (row, column) entries, CSR sums them
  for (int i = 0; i < m; ++i) {
    const int base = col(rng);
    for (int j = 0; j < per + (i % 7); ++j) rows[i].push_back({(base + j * 4729) % n, val(rng)});
  }
  const auto A = make_csr(m, n, rows);
  std::vector<double> x(n);
  for (auto& v : x) v = (bit(rng) < 0.5 ? -1.0 : 1.0) * std::pow(10.0, e(rng));
  const auto ref = naive(A, x);
  SpmvRunner<double, double> runner(A);
  runner.set_x(x);
  auto check = [&](KernelId id, int lanes, int block, bool exact, const char* label) {
    const SpmvResult r = runner.run(id, 3, lanes, block, 1);
    const auto got = runner.result();
    double worst = 0.0;
    for (int i = 0; i < m; ++i) {
      double abs_sum = 0.0;
      for (Index p = A.rowptr[i]; p < A.rowptr[i + 1]; ++p) abs_sum += std::fabs(A.values[p] * x[A.colind[p]]);
      const double bound = 2.0 * gamma_n(A.rowptr[i + 1] - A.rowptr[i], std::ldexp(1.0, -53)) * abs_sum + 1e-30;
      worst = std::max(worst, std::fabs(got[i] - ref[i]) / bound);
      if (exact && got[i] != ref[i]) worst = 1e300;
    }
    if (!(worst <= 1.0)) std::printf("kernel %s ratio %g\n", label, worst);
    EXPECT(worst <= 1.0 && r.iters == 3 && r.median_ms > 0.0);
  };
  check(KernelId::CsrScalar, 1, 1, true, "csr_scalar");
  for (int lanes : {2, 4, 8, 16, 32}) check(KernelId::CsrVector, lanes, 1, false, "csr_vector");
  check(KernelId::CsrWarp, 1, 1, false, "csr_warp");
  check(KernelId::CsrMerge, 1, 1, false, "csr_merge");
  check(KernelId::Ell, 1, 1, true, "ell");
  check(KernelId::Hyb, 1, 1, false, "hyb");
  check(KernelId::Bcsr, 1, 2, false, "bcsr2");
  check(KernelId::Bcsr, 1, 4, false, "bcsr4");
  EXPECT(runner.ell_touched_nnz() == A.nnz && runner.ell_padded_nnz() == static_cast<std::int64_t>(m) * (per + 6));
  EXPECT(runner.bcsr_block_nnz(4) > 0);
  // SpMM: tiled keeps spmm_csr_cpu's order -> bit for bit with the naive loop
  const int k = 32;
  std::vector<double> B(static_cast<size_t>(n) * k);
  for (auto& v : B) v = val(rng);
  std::vector<double> Yref(static_cast<size_t>(m) * k, 0.0);
  for (int i = 0; i < m; ++i)
    for (Index p = A.rowptr[i]; p < A.rowptr[i + 1]; ++p)
      for (int j = 0; j < k; ++j) Yref[static_cast<size_t>(i) * k + j] += A.values[p] * B[static_cast<size_t>(A.colind[p]) * k + j];
  for (int tile : {16, 32, 64})
    for (bool balanced : {false, true}) {
      std::vector<double> Y;
      const SpmmResult r = spmm_csr_tiled_f64(A, B, k, tile, balanced, 2, 1, Y);
      EXPECT(Y == Yref && r.iters == 2);
    }
}

// Random CSR: empty rows, unsorted and repeated columns, long rows, tails
// that leave partial 2x2 / 4x4 blocks.
static CsrMatrix<double> random_matrix(std::mt19937_64& rng) {
  const int m = static_cast<int>(rng() % 37), n = 1 + static_cast<int>(rng() % 45);
  CsrMatrix<double> A(m, n);
  for (int i = 0; i < m; ++i) {
    const int kind = static_cast<int>(rng() % 5);
    const int len = kind == 0 ? 0 : kind == 1 ? static_cast<int>(rng() % (2 * n + 1)) : static_cast<int>(rng() % 6);
    for (int j = 0; j < len; ++j) {
      A.colind.push_back(static_cast<Index>(rng() % n));
      A.values.push_back(static_cast<double>(static_cast<int64_t>(rng() % 2001) - 1000) / 7.0);
    }
    A.rowptr[i + 1] = static_cast<Index>(A.colind.size());
  }
  A.nnz = A.rowptr[m];
  return A;
}

template <int B>
static void fuzz_bcsr(void* lib, void* h, const CsrMatrix<double>& A) {
  auto shape = reinterpret_cast<void (*)(void*, int, int32_t*, int64_t*)>(dlsym(lib, "ref_bcsr_shape_d"));
  auto conv = reinterpret_cast<void (*)(void*, int, int32_t*, int32_t*, double*)>(dlsym(lib, "ref_csr_to_bcsr_d"));
  int32_t mb = 0;
  int64_t bn = 0;
  shape(h, B, &mb, &bn);
  std::vector<int32_t> rp(mb + 1), ci(bn > 0 ? bn : 1);
  std::vector<double> v((bn > 0 ? bn : 1) * B * B);
  conv(h, B, rp.data(), ci.data(), v.data());
  const auto mine = csr_to_bcsr<double, B, B>(A);
  EXPECT(mine.mb == mb && mine.block_nnz == bn);
  EXPECT(std::vector<int32_t>(mine.rowptr.begin(), mine.rowptr.end()) == rp);
  EXPECT(std::vector<int32_t>(mine.colind.begin(), mine.colind.end()) == std::vector<int32_t>(ci.begin(), ci.begin() + bn));
  EXPECT(mine.values == std::vector<double>(v.begin(), v.begin() + bn * B * B));
}

static void fuzz_tests(const char* libpath) {
  void* lib = dlopen(libpath, RTLD_NOW | RTLD_LOCAL);
  if (!lib) {
    std::printf("FAIL cannot load %s: %s\n", libpath, dlerror());
    ++g_fail;
    return;
  }
  auto create = reinterpret_cast<void* (*)(int32_t, int32_t, int64_t, const int32_t*, const int32_t*, const double*)>(
      dlsym(lib, "ref_csr_create_d"));
  auto destroy = reinterpret_cast<void (*)(void*)>(dlsym(lib, "ref_csr_destroy_d"));
  auto width = reinterpret_cast<int32_t (*)(void*)>(dlsym(lib, "ref_ell_width_d"));
  auto to_ell = reinterpret_cast<void (*)(void*, int32_t*, double*, int32_t*)>(dlsym(lib, "ref_csr_to_ell_d"));
  std::mt19937_64 rng(20241202);
  for (int t = 0; t < 400; ++t) {
    const CsrMatrix<double> A = random_matrix(rng);
    void* h = create(A.m, A.n, A.nnz, A.rowptr.data(), A.colind.data(), A.values.data());
    const int32_t w = width(h);
    std::vector<int32_t> ec(static_cast<size_t>(A.m) * w + 1), rl(A.m + 1);
    std::vector<double> ev(static_cast<size_t>(A.m) * w + 1);
    to_ell(h, ec.data(), ev.data(), rl.data());
    const auto mine = csr_to_ell(A);
    const size_t slots = static_cast<size_t>(A.m) * w;
    EXPECT(mine.max_row_nnz == w);
    EXPECT(std::vector<int32_t>(mine.colind.begin(), mine.colind.end()) ==
           std::vector<int32_t>(ec.begin(), ec.begin() + slots));
    EXPECT(mine.values == std::vector<double>(ev.begin(), ev.begin() + slots));
    EXPECT(mine.row_lengths == std::vector<int>(rl.begin(), rl.begin() + A.m));
    fuzz_bcsr<2>(lib, h, A);
    fuzz_bcsr<4>(lib, h, A);
    destroy(h);
  }
  dlclose(lib);
}

int main(int argc, char** argv) {
  const std::string mode = argc > 1 ? argv[1] : "cpu";
  if (mode == "cpu") cpu_tests();
  else if (mode == "fuzz") fuzz_tests(argc > 2 ? argv[2] : "");
  else gpu_tests();
  std::printf("%d passed, %d failed\n", g_pass, g_fail);
  return g_fail == 0 ? 0 : 1;
}
