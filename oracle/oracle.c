/*
 * oracle.c - CPU restatement of SpMVBench's CPU path, used ONLY as the
 * checker of the CUDA kernels (tests, the smoke check) and as the timed CPU
 * baseline of bench.py. It is test infrastructure, not part of the product:
 * nothing in spmvbench_b200/ calls it, and the product fails loudly when its
 * CUDA library is missing instead of falling back to this code.
 *
 * Parity pinning: tests/test_oracle.py checks every function here against
 * (a) the known answers of the reference's own test suite and (b) golden
 * fixtures produced by the reference itself, compiled from its sources into
 * oracle/_ref by oracle/Makefile (tests/golden/make_golden.py).
 *
 * Build: gcc -O3 -fopenmp -ffp-contract=off (no -march: baseline x86-64 SSE2
 * arithmetic, no FMA contraction - the reference's own flags, -O3 without
 * -march, CMakeLists.txt:130-132, produce the same IEEE operations).
 *
 * Citations are paths inside the SpMVBench source tree.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#define SET_THREADS(n) do { if ((n) > 0) omp_set_num_threads(n); } while (0)
#else
#define SET_THREADS(n) do { (void)(n); } while (0)
#endif

/* ---- SpMV / SpMM kernels -------------------------------------------------- */

/* spmv_csr_cpu = csr_omp (src/cpu/spmv_cpu.cpp:15-26): static schedule, each
 * row summed left to right from zero as Acc(a) * Acc(x). */
#define DEF_SPMV_CSR(NAME, T, ACC)                                            \
  void NAME(int32_t m, const int32_t* rowptr, const int32_t* colind,          \
            const T* vals, const T* x, ACC* y, int nthreads) {                \
    SET_THREADS(nthreads);                                                    \
    _Pragma("omp parallel for schedule(static)")                              \
    for (int32_t i = 0; i < m; ++i) {                                         \
      ACC sum = (ACC)0;                                                       \
      for (int32_t p = rowptr[i]; p < rowptr[i + 1]; ++p)                     \
        sum += (ACC)vals[p] * (ACC)x[colind[p]];                              \
      y[i] = sum;                                                             \
    }                                                                         \
  }
DEF_SPMV_CSR(orc_spmv_csr_dd, double, double)
DEF_SPMV_CSR(orc_spmv_csr_ff, float, float)
DEF_SPMV_CSR(orc_spmv_csr_fd, float, double)

/* spmv_ell_cpu (src/cpu/spmv_cpu.cpp:55-72): walks row_lengths[i] entries of
 * the column-major layout, p = j*m + i. */
#define DEF_SPMV_ELL(NAME, T, ACC)                                            \
  void NAME(int32_t m, const int32_t* colind, const T* vals,                  \
            const int32_t* row_lengths, const T* x, ACC* y, int nthreads) {   \
    SET_THREADS(nthreads);                                                    \
    _Pragma("omp parallel for schedule(static)")                              \
    for (int32_t i = 0; i < m; ++i) {                                         \
      ACC sum = (ACC)0;                                                       \
      for (int32_t j = 0; j < row_lengths[i]; ++j) {                          \
        const int64_t p = (int64_t)j * m + i;                                 \
        sum += (ACC)vals[p] * (ACC)x[colind[p]];                              \
      }                                                                       \
      y[i] = sum;                                                             \
    }                                                                         \
  }
DEF_SPMV_ELL(orc_spmv_ell_dd, double, double)
DEF_SPMV_ELL(orc_spmv_ell_ff, float, float)
DEF_SPMV_ELL(orc_spmv_ell_fd, float, double)

/* spmv_bcsr_cpu (src/cpu/spmv_cpu.cpp:74-105): per block row, per block,
 * per row r a partial s over columns c (stopping at the last column n-1),
 * then acc[r] += s. */
#define DEF_SPMV_BCSR(NAME, T, ACC)                                           \
  void NAME(int32_t m, int32_t n, int32_t R, int32_t C, int32_t mb,           \
            const int32_t* rowptr, const int32_t* colind, const T* vals,      \
            const T* x, ACC* y, int nthreads) {                               \
    SET_THREADS(nthreads);                                                    \
    _Pragma("omp parallel for schedule(static)")                              \
    for (int32_t bi = 0; bi < mb; ++bi) {                                     \
      ACC acc[16];                                                            \
      for (int r = 0; r < R; ++r) acc[r] = (ACC)0;                            \
      for (int32_t bp = rowptr[bi]; bp < rowptr[bi + 1]; ++bp) {              \
        const int32_t bj = colind[bp];                                        \
        const T* blk = vals + (int64_t)bp * R * C;                            \
        for (int r = 0; r < R; ++r) {                                         \
          ACC s = (ACC)0;                                                     \
          for (int c = 0; c < C; ++c) {                                       \
            const int32_t gc = bj * C + c;                                    \
            if (gc >= n) break;                                               \
            s += (ACC)blk[r * C + c] * (ACC)x[gc];                            \
          }                                                                   \
          acc[r] += s;                                                        \
        }                                                                     \
      }                                                                       \
      for (int r = 0; r < R; ++r) {                                           \
        const int32_t gi = bi * R + r;                                        \
        if (gi < m) y[gi] = acc[r];                                           \
      }                                                                       \
    }                                                                         \
  }
DEF_SPMV_BCSR(orc_spmv_bcsr_dd, double, double)
DEF_SPMV_BCSR(orc_spmv_bcsr_ff, float, float)
DEF_SPMV_BCSR(orc_spmv_bcsr_fd, float, double)

/* spmm_csr_cpu (src/cpu/spmm_cpu.cpp:10-29): Y row zeroed, then for each
 * entry in CSR order yrow[j] += Acc(a) * Acc(B[col*k + j]). */
#define DEF_SPMM(NAME, T, ACC)                                                \
  void NAME(int32_t m, int32_t k, const int32_t* rowptr,                      \
            const int32_t* colind, const T* vals, const T* B, ACC* Y,         \
            int nthreads) {                                                   \
    SET_THREADS(nthreads);                                                    \
    _Pragma("omp parallel for schedule(static)")                              \
    for (int32_t i = 0; i < m; ++i) {                                         \
      ACC* yrow = Y + (int64_t)i * k;                                         \
      for (int j = 0; j < k; ++j) yrow[j] = (ACC)0;                           \
      for (int32_t p = rowptr[i]; p < rowptr[i + 1]; ++p) {                   \
        const ACC a = (ACC)vals[p];                                           \
        const T* brow = B + (int64_t)colind[p] * k;                           \
        for (int j = 0; j < k; ++j) yrow[j] += a * (ACC)brow[j];              \
      }                                                                       \
    }                                                                         \
  }
DEF_SPMM(orc_spmm_csr_dd, double, double)
DEF_SPMM(orc_spmm_csr_ff, float, float)
DEF_SPMM(orc_spmm_csr_fd, float, double)

/* ---- format conversions ---------------------------------------------------- */

/* csr_to_ell (src/formats.cpp:14-43): width = longest row, column-major,
 * padding column 0 / value 0 (the caller passes zero-filled outputs of
 * m*width entries), row_lengths. Values are copied as elem_size bytes. */
int32_t orc_ell_width(int32_t m, const int32_t* rowptr) {
  int32_t w = 0;
  for (int32_t i = 0; i < m; ++i)
    if (rowptr[i + 1] - rowptr[i] > w) w = rowptr[i + 1] - rowptr[i];
  return w;
}

void orc_csr_to_ell(int32_t m, const int32_t* rowptr, const int32_t* colind,
                    const void* vals, int elem_size, int32_t* ecol, void* evals,
                    int32_t* row_lengths) {
  for (int32_t i = 0; i < m; ++i) {
    int32_t j = 0;
    row_lengths[i] = rowptr[i + 1] - rowptr[i];
    for (int32_t p = rowptr[i]; p < rowptr[i + 1]; ++p, ++j) {
      const int64_t s = (int64_t)j * m + i;
      ecol[s] = colind[p];
      memcpy((char*)evals + s * elem_size, (const char*)vals + (int64_t)p * elem_size, elem_size);
    }
  }
}

/* csr_to_bcsr<T,R,C> (src/formats.cpp:45-105). Per block row the blocks are
 * created in order of first touch, values are assigned (a repeated
 * (row, column) entry overwrites, so the last one in CSR order wins), and
 * blocks are emitted in ascending block-column order. Two calls: with
 * out_colind == NULL only *mb and *block_nnz are returned; then the caller
 * passes zero-filled arrays of mb+1, block_nnz and block_nnz*R*C entries. */
static int cmp_i32(const void* a, const void* b) {
  const int32_t x = *(const int32_t*)a, y = *(const int32_t*)b;
  return (x > y) - (x < y);
}

int orc_csr_to_bcsr(int32_t m, int32_t n, int32_t R, int32_t C,
                    const int32_t* rowptr, const int32_t* colind,
                    const void* vals, int elem_size, int32_t* mb_out,
                    int64_t* block_nnz_out, int32_t* out_rowptr,
                    int32_t* out_colind, void* out_vals) {
  const int32_t mb = (m + R - 1) / R;
  int64_t total = 0;
  int32_t cap = 0;
  int32_t* bcols = NULL;
  (void)n;
  for (int32_t bi = 0; bi < mb; ++bi) {
    int32_t len = 0;
    for (int r = 0; r < R && bi * R + r < m; ++r) len += rowptr[bi * R + r + 1] - rowptr[bi * R + r];
    if (len > cap) {
      cap = len;
      bcols = (int32_t*)realloc(bcols, sizeof(int32_t) * (size_t)(cap > 0 ? cap : 1));
      if (!bcols) return -1;
    }
    int32_t cnt = 0;
    for (int r = 0; r < R && bi * R + r < m; ++r)
      for (int32_t p = rowptr[bi * R + r]; p < rowptr[bi * R + r + 1]; ++p) bcols[cnt++] = colind[p] / C;
    qsort(bcols, (size_t)cnt, sizeof(int32_t), cmp_i32);
    int32_t uniq = 0;
    for (int32_t a = 0; a < cnt; ++a)
      if (a == 0 || bcols[a] != bcols[a - 1]) bcols[uniq++] = bcols[a];
    if (out_colind) {
      out_rowptr[bi] = (int32_t)total;
      for (int32_t u = 0; u < uniq; ++u) out_colind[total + u] = bcols[u];
      /* assignment in CSR order: the last write to a slot wins */
      for (int r = 0; r < R && bi * R + r < m; ++r) {
        for (int32_t p = rowptr[bi * R + r]; p < rowptr[bi * R + r + 1]; ++p) {
          const int32_t bj = colind[p] / C, cc = colind[p] % C;
          const int32_t* hit = (const int32_t*)bsearch(&bj, bcols, (size_t)uniq, sizeof(int32_t), cmp_i32);
          const int64_t blk = total + (hit - bcols);
          memcpy((char*)out_vals + (blk * R * C + r * C + cc) * elem_size,
                 (const char*)vals + (int64_t)p * elem_size, elem_size);
        }
      }
    }
    total += uniq;
  }
  if (out_colind) out_rowptr[mb] = (int32_t)total;
  free(bcols);
  *mb_out = mb;
  *block_nnz_out = total;
  return 0;
}

/* ---- statistics and selection -------------------------------------------------- */

/* compute_row_stats (src/stats.cpp:13-123). out[] holds, in order: nnz, rows,
 * cols, mean, median, min, max, stddev, cv, max/mean, ell_padding_overhead,
 * frac_dense_blocks_4x4, density. hist gets max+1 counts when non-NULL. */
static int cmp_int(const void* a, const void* b) {
  const int x = *(const int*)a, y = *(const int*)b;
  return (x > y) - (x < y);
}

int orc_row_stats(const int32_t* rowptr, const int32_t* colind, int32_t m,
                  int32_t n, int64_t nnz, double* out, int64_t* hist) {
  memset(out, 0, sizeof(double) * 13);
  out[0] = (double)nnz;
  out[1] = m;
  out[2] = n;
  out[12] = ((double)m * n > 0) ? (double)nnz / ((double)m * n) : 0.0;
  out[10] = 1.0;
  if (m <= 0) {
    if (hist) hist[0] = 0;
    return 0;
  }
  int* len = (int*)malloc(sizeof(int) * (size_t)m);
  int* sorted = (int*)malloc(sizeof(int) * (size_t)m);
  if (!len || !sorted) return -1;
  long long sum = 0;
  int mn = 0, mx = 0;
  for (int32_t i = 0; i < m; ++i) {
    const int r = rowptr[i + 1] - rowptr[i];
    len[i] = r;
    sum += r;
    if (i == 0 || r < mn) mn = r;
    if (i == 0 || r > mx) mx = r;
  }
  const double mean = (double)sum / m;
  memcpy(sorted, len, sizeof(int) * (size_t)m);
  qsort(sorted, (size_t)m, sizeof(int), cmp_int);
  const double median = (m % 2 == 1) ? sorted[m / 2] : 0.5 * ((double)((int64_t)sorted[m / 2 - 1] + sorted[m / 2]));
  double var = 0.0;
  for (int32_t i = 0; i < m; ++i) {
    const double d = len[i] - mean;
    var += d * d;
  }
  var /= m;
  const double sd = sqrt(var);
  out[3] = mean;
  out[4] = median;
  out[5] = mn;
  out[6] = mx;
  out[7] = sd;
  out[8] = mean > 0 ? sd / mean : 0.0;
  out[9] = mean > 0 ? mx / mean : 0.0;
  if (hist) {
    memset(hist, 0, sizeof(int64_t) * (size_t)(mx + 1));
    for (int32_t i = 0; i < m; ++i) hist[len[i]]++;
  }
  out[10] = nnz > 0 ? (double)m * mx / (double)nnz : 1.0;
  const int32_t mb = (m + 3) / 4, nb = (n + 3) / 4;
  int64_t dense = 0;
  if (colind && nnz > 0) {
    int32_t cap = 1;
    int32_t* bc = (int32_t*)malloc(sizeof(int32_t));
    for (int32_t bi = 0; bi < mb; ++bi) {
      int32_t cnt = 0;
      for (int r = 0; r < 4 && bi * 4 + r < m; ++r) cnt += rowptr[bi * 4 + r + 1] - rowptr[bi * 4 + r];
      if (cnt > cap) {
        cap = cnt;
        bc = (int32_t*)realloc(bc, sizeof(int32_t) * (size_t)cap);
      }
      cnt = 0;
      for (int r = 0; r < 4 && bi * 4 + r < m; ++r)
        for (int32_t p = rowptr[bi * 4 + r]; p < rowptr[bi * 4 + r + 1]; ++p) bc[cnt++] = colind[p] / 4;
      qsort(bc, (size_t)cnt, sizeof(int32_t), cmp_i32);
      for (int32_t a = 0; a < cnt;) {
        int32_t b = a;
        while (b < cnt && bc[b] == bc[a]) ++b;
        if (b - a > 8) dense++;
        a = b;
      }
    }
    free(bc);
  }
  const int64_t possible = (int64_t)mb * nb;
  out[11] = possible > 0 ? (double)dense / (double)possible : 0.0;
  free(len);
  free(sorted);
  return 0;
}

/* choose_spmv's ordered rules 0-6 (src/select.cpp:93-165). stats[] as in
 * orc_row_stats. out[]: kernel id (KernelId numbering), lanes, block_r,
 * block_c, rule index. */
void orc_choose_spmv(const double* s, int32_t* out) {
  const double nnz = s[0], mean = s[3], cv = s[8], mom = s[9], pad = s[10], dense4 = s[11];
  if (nnz < 50000) { out[0] = 0; out[1] = 1; out[2] = 1; out[3] = 1; out[4] = 0; return; }
  if (mean < 4.0) { out[0] = 0; out[1] = 1; out[2] = 1; out[3] = 1; out[4] = 1; return; }
  if (dense4 > 0.6) { out[0] = 5; out[1] = 4; out[2] = 4; out[3] = 4; out[4] = 2; return; }
  if (cv > 1.5 || mom > 50.0) { out[0] = 3; out[1] = 1; out[2] = 1; out[3] = 1; out[4] = 3; return; }
  if (mean >= 4.0 && mean < 32.0 && cv < 0.5) {
    int v = (int)ceil(mean), p = 1;
    if (v > 1) while (p < v) p <<= 1;
    out[0] = 1; out[1] = p; out[2] = 1; out[3] = 1; out[4] = 4;
    return;
  }
  if (pad < 1.2) { out[0] = 4; out[1] = 1; out[2] = 1; out[3] = 1; out[4] = 5; return; }
  out[0] = 1; out[1] = 4; out[2] = 1; out[3] = 1; out[4] = 6;
}

/* ---- gamma_n bound (tests/test_cuda_correctness.cpp:53-56,73-104) --------------- */
/* For each row: bound_i = 2*gamma_n(u)*sum_j |a_ij x_j| + 1e-30 with
 * n = row length, gamma_n = n*u / (1 - n*u); ratio_i = |got_i - ref_i| / bound_i.
 * Returns the largest ratio (<= 1 passes) and its row in *worst_row. */
double orc_gamma_check_d(int32_t m, const int32_t* rowptr, const int32_t* colind,
                         const double* vals, const double* x, const double* ref,
                         const double* got, double u, int32_t* worst_row) {
  double worst = 0.0;
  *worst_row = -1;
  for (int32_t i = 0; i < m; ++i) {
    double abs_sum = 0.0;
    for (int32_t p = rowptr[i]; p < rowptr[i + 1]; ++p) abs_sum += fabs(vals[p] * x[colind[p]]);
    const double nu = (double)(rowptr[i + 1] - rowptr[i]) * u;
    const double bound = 2.0 * (nu / (1.0 - nu)) * abs_sum + 1e-30;
    const double r = fabs(got[i] - ref[i]) / bound;
    if (r > worst) {
      worst = r;
      *worst_row = i;
    }
  }
  return worst;
}

/* ---- seeded workloads -------------------------------------------------------- */
/* A second, independent statement of the library's seeded workload generator
 * (xoshiro256** seeded through splitmix64; one stream per purpose), so that a
 * CPU timing of the reference (bench.py --impl reference) can build its
 * matrix without loading the CUDA library. tests/test_oracle.py checks that
 * both generators give identical rowptr, colind, values and vectors.
 * Workloads: 1 banded (|i-j| <= 4, diagonal + 10), 2 and 5 uniform (16
 * distinct sorted columns per row), 4 dense 4x4 blocks (8 distinct block
 * columns per block row). The power-law workload (3) is not restated. */
typedef struct { uint64_t s[4]; } OrcRng;

static uint64_t orc_splitmix(uint64_t* x) {
  uint64_t z = (*x += 0x9e3779b97f4a7c15ull);
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
static void orc_rng_init(OrcRng* r, uint64_t seed, uint64_t stream) {
  uint64_t x = seed ^ (0x632be59bd9b4e019ull * (stream + 1));
  for (int i = 0; i < 4; ++i) r->s[i] = orc_splitmix(&x);
}
static uint64_t orc_rotl(uint64_t v, int k) { return (v << k) | (v >> (64 - k)); }
static uint64_t orc_next(OrcRng* r) {
  uint64_t* s = r->s;
  const uint64_t out = orc_rotl(s[1] * 5, 7) * 9;
  const uint64_t t = s[1] << 17;
  s[2] ^= s[0];
  s[3] ^= s[1];
  s[1] ^= s[2];
  s[0] ^= s[3];
  s[2] ^= t;
  s[3] = orc_rotl(s[3], 45);
  return out;
}
/* U(-1,1): a 53-bit uniform in [0,1) times 2, minus 1. */
static double orc_sym(OrcRng* r) { return (double)(orc_next(r) >> 11) * 0x1.0p-53 * 2.0 - 1.0; }
/* [0, bound) by the high half of a 64x64-bit product. */
static uint32_t orc_below(OrcRng* r, uint32_t bound) {
  return (uint32_t)(((unsigned __int128)orc_next(r) * bound) >> 64);
}
/* k <= 64 distinct draws in [0, bound) (bound >= 4k), rejection of repeats,
 * then sorted ascending. */
static void orc_distinct_sorted(OrcRng* r, int k, uint32_t bound, int32_t* out) {
  int have = 0;
  while (have < k) {
    const int32_t c = (int32_t)orc_below(r, bound);
    int dup = 0;
    for (int i = 0; i < have; ++i) dup |= (out[i] == c);
    if (!dup) out[have++] = c;
  }
  qsort(out, (size_t)k, sizeof(int32_t), cmp_i32);
}

enum { ORC_COLUMNS = 2, ORC_VALUES = 3, ORC_VECTOR = 5 };

/* Sizes of workload `which` (scale_rows > 0 replaces the default row count);
 * with non-null arrays, also its entries. Returns 0, or -1 for a workload or
 * size it does not cover. */
int orc_generate(int which, uint64_t seed, int32_t scale_rows, int32_t* m_out, int32_t* n_out,
                 int64_t* nnz_out, int32_t* rowptr, int32_t* colind, double* vals) {
  int32_t m;
  int64_t nnz;
  if (which == 1) {
    m = scale_rows > 0 ? scale_rows : 100000;
    nnz = 0;
    for (int32_t i = 0; i < m; ++i) {
      const int32_t lo = i - 4 < 0 ? 0 : i - 4, hi = i + 4 > m - 1 ? m - 1 : i + 4;
      nnz += hi - lo + 1;
    }
  } else if (which == 2 || which == 5) {
    m = scale_rows > 0 ? scale_rows : 1000000;
    if (m < 64) return -1;
    nnz = (int64_t)m * 16;
  } else if (which == 4) {
    m = scale_rows > 0 ? (scale_rows / 4) * 4 : 500000;
    if (m < 128) return -1;
    nnz = (int64_t)m * 32;
  } else {
    return -1;
  }
  *m_out = m;
  *n_out = m;
  *nnz_out = nnz;
  if (!colind) return 0;
  OrcRng rc, rv;
  orc_rng_init(&rc, seed, ORC_COLUMNS);
  orc_rng_init(&rv, seed, ORC_VALUES);
  int64_t p = 0;
  rowptr[0] = 0;
  if (which == 1) {
    for (int32_t i = 0; i < m; ++i) {
      const int32_t lo = i - 4 < 0 ? 0 : i - 4, hi = i + 4 > m - 1 ? m - 1 : i + 4;
      for (int32_t j = lo; j <= hi; ++j, ++p) {
        colind[p] = j;
        vals[p] = orc_sym(&rv) + (j == i ? 10.0 : 0.0);
      }
      rowptr[i + 1] = (int32_t)p;
    }
  } else if (which == 2 || which == 5) {
    int32_t cols[16];
    for (int32_t i = 0; i < m; ++i) {
      orc_distinct_sorted(&rc, 16, (uint32_t)m, cols);
      for (int t = 0; t < 16; ++t, ++p) {
        colind[p] = cols[t];
        vals[p] = orc_sym(&rv);
      }
      rowptr[i + 1] = (int32_t)p;
    }
  } else {
    /* Block row b: 8 block columns, then 128 values drawn as block t, row r,
     * column c at t*16 + r*4 + c; rows are written block by block. */
    int32_t cols[8];
    double blk[128];
    for (int32_t b = 0; b < m / 4; ++b) {
      orc_distinct_sorted(&rc, 8, (uint32_t)(m / 4), cols);
      for (int q = 0; q < 128; ++q) blk[q] = orc_sym(&rv);
      for (int r = 0; r < 4; ++r) {
        for (int t = 0; t < 8; ++t)
          for (int c = 0; c < 4; ++c, ++p) {
            colind[p] = cols[t] * 4 + c;
            vals[p] = blk[t * 16 + r * 4 + c];
          }
        rowptr[b * 4 + r + 1] = (int32_t)p;
      }
    }
  }
  return 0;
}

/* `len` values U(-1,1) from the vector stream of `seed`. */
void orc_generate_vector(uint64_t seed, int64_t len, double* out) {
  OrcRng r;
  orc_rng_init(&r, seed, ORC_VECTOR);
  for (int64_t i = 0; i < len; ++i) out[i] = orc_sym(&r);
}
