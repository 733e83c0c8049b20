// Seeded synthetic matrices for the five benchmark workloads.
//
// The random source is xoshiro256** (Blackman & Vigna, "Scrambled linear
// pseudorandom number generators", 2018) seeded through splitmix64, so the
// streams are identical on every platform and compiler (std::uniform_*
// distributions are implementation defined). Each purpose (row lengths,
// columns, values, row shuffle) draws from its own stream derived from the
// seed, so sizes can be computed without generating the entries.
//
// Workloads (m x n, nnz):
//   1 banded:   100,000^2, |i-j| <= 4, off-diagonals U(-1,1), diagonal
//               U(-1,1)+10 -> nnz 899,980
//   2 uniform:  1,000,000^2, exactly 16 distinct sorted uniform columns per
//               row, U(-1,1) -> nnz 16,000,000
//   3 powerlaw: 1,000,000^2, row lengths Zipf(2.1) clipped to [1, 50,000],
//               distinct sorted uniform columns, U(-1,1), row order shuffled
//   4 blocks:   500,000^2 from dense 4x4 blocks, 8 distinct uniform block
//               columns per block row, U(-1,1) -> nnz 16,000,000
//   5 = 2 (the sparse operand of the SpMM workload)
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <string>
#include <unordered_set>
#include <vector>

#include "../internal.hpp"

namespace spmvb {
namespace {

uint64_t splitmix64(uint64_t& s) {
  uint64_t z = (s += 0x9e3779b97f4a7c15ull);
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

struct Rng {
  uint64_t s[4];
  explicit Rng(uint64_t seed, uint64_t stream) {
    uint64_t x = seed ^ (0x632be59bd9b4e019ull * (stream + 1));
    for (auto& w : s) w = splitmix64(x);
  }
  static uint64_t rotl(uint64_t v, int k) { return (v << k) | (v >> (64 - k)); }
  uint64_t next() {
    const uint64_t r = rotl(s[1] * 5, 7) * 9;
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl(s[3], 45);
    return r;
  }
  // U[0,1) with 53 random bits.
  double uniform() { return static_cast<double>(next() >> 11) * 0x1.0p-53; }
  // U(-1,1) as a*2-1 of a 53-bit uniform (never exactly 1).
  double sym() { return uniform() * 2.0 - 1.0; }
  // Integer in [0, bound) by 64x64->128 multiply-shift.
  uint32_t below(uint32_t bound) {
    return static_cast<uint32_t>((static_cast<unsigned __int128>(next()) * bound) >> 64);
  }
};

enum Stream : uint64_t { kLengths = 1, kColumns = 2, kValues = 3, kShuffle = 4, kVector = 5 };

// k distinct sorted integers in [0, bound).
void distinct_sorted(Rng& rng, int k, uint32_t bound, std::vector<int32_t>& out,
                     std::unordered_set<uint32_t>& seen) {
  out.clear();
  if (static_cast<uint64_t>(k) * 4 > bound) {
    // Dense case: partial Fisher-Yates over an explicit range.
    std::vector<int32_t> all(bound);
    for (uint32_t i = 0; i < bound; ++i) all[i] = static_cast<int32_t>(i);
    for (int i = 0; i < k; ++i) {
      const uint32_t j = i + rng.below(bound - i);
      std::swap(all[i], all[j]);
      out.push_back(all[i]);
    }
  } else if (k <= 64) {
    while (static_cast<int>(out.size()) < k) {
      const int32_t c = static_cast<int32_t>(rng.below(bound));
      bool dup = false;
      for (int32_t v : out) dup |= (v == c);
      if (!dup) out.push_back(c);
    }
  } else {
    seen.clear();
    while (static_cast<int>(out.size()) < k) {
      const uint32_t c = rng.below(bound);
      if (seen.insert(c).second) out.push_back(static_cast<int32_t>(c));
    }
  }
  std::sort(out.begin(), out.end());
}

// Zipf(alpha) on {1, 2, ...} clipped to [1, kmax]: inverse CDF over the exact
// probabilities k^-alpha / zeta(alpha) for k < kmax, with the whole tail mass
// at kmax (what clipping an unbounded draw does).
class ZipfClipped {
 public:
  ZipfClipped(double alpha, int kmax) : cdf_(kmax) {
    // zeta(alpha) = sum_{k<N} k^-a + Euler-Maclaurin tail from N.
    const int N = kmax;
    double head = 0.0;
    for (int k = N - 1; k >= 1; --k) head += std::pow(static_cast<double>(k), -alpha);
    const double Nd = N;
    const double tail = std::pow(Nd, 1.0 - alpha) / (alpha - 1.0) + 0.5 * std::pow(Nd, -alpha) +
                        alpha / 12.0 * std::pow(Nd, -alpha - 1.0);
    const double zeta = head + tail;
    double acc = 0.0;
    for (int k = 1; k < kmax; ++k) {
      acc += std::pow(static_cast<double>(k), -alpha) / zeta;
      cdf_[k - 1] = acc;
    }
    cdf_[kmax - 1] = 1.0;
  }
  int draw(Rng& rng) const {
    const double u = rng.uniform();
    const auto it = std::upper_bound(cdf_.begin(), cdf_.end(), u);
    return static_cast<int>(it - cdf_.begin()) + 1;
  }

 private:
  std::vector<double> cdf_;
};

struct Shape {
  int32_t m = 0, n = 0;
  int64_t nnz = 0;
  std::vector<int32_t> lens;  // only for the power-law workload
};

constexpr int kPowerlawMax = 50000;
constexpr double kPowerlawAlpha = 2.1;

spmvb_status shape_of(int which, uint64_t seed, int32_t scale_rows, Shape& sh) {
  switch (which) {
    case 1: {
      const int32_t m = scale_rows > 0 ? scale_rows : 100000;
      sh.m = sh.n = m;
      int64_t nnz = 0;
      for (int32_t i = 0; i < m; ++i)
        nnz += std::min<int32_t>(m - 1, i + 4) - std::max<int32_t>(0, i - 4) + 1;
      sh.nnz = nnz;
      return SPMVB_OK;
    }
    case 2:
    case 5: {
      const int32_t m = scale_rows > 0 ? scale_rows : 1000000;
      if (m < 16) return fail(SPMVB_ERR_INVALID_ARGUMENT, "uniform workload needs at least 16 rows");
      sh.m = sh.n = m;
      sh.nnz = static_cast<int64_t>(m) * 16;
      return SPMVB_OK;
    }
    case 3: {
      const int32_t m = scale_rows > 0 ? scale_rows : 1000000;
      sh.m = sh.n = m;
      const int kmax = std::min<int>(kPowerlawMax, m);
      ZipfClipped z(kPowerlawAlpha, kPowerlawMax);
      Rng rl(seed, kLengths);
      sh.lens.resize(m);
      int64_t nnz = 0;
      for (int32_t i = 0; i < m; ++i) {
        sh.lens[i] = std::min(z.draw(rl), kmax);
        nnz += sh.lens[i];
      }
      Rng rs(seed, kShuffle);
      for (int32_t i = m - 1; i > 0; --i) std::swap(sh.lens[i], sh.lens[rs.below(i + 1)]);
      sh.nnz = nnz;
      return SPMVB_OK;
    }
    case 4: {
      const int32_t m = scale_rows > 0 ? (scale_rows / 4) * 4 : 500000;
      if (m < 32) return fail(SPMVB_ERR_INVALID_ARGUMENT, "block workload needs at least 32 rows");
      sh.m = sh.n = m;
      sh.nnz = static_cast<int64_t>(m) * 32;
      return SPMVB_OK;
    }
    default:
      return fail(SPMVB_ERR_INVALID_ARGUMENT, "unknown workload " + std::to_string(which));
  }
}

}  // namespace
}  // namespace spmvb

using namespace spmvb;

extern "C" spmvb_status spmvb_generate(int which, uint64_t seed, int32_t scale_rows,
                                       int32_t* m, int32_t* n, int64_t* nnz,
                                       int32_t* h_rowptr, int32_t* h_colind,
                                       double* h_values) {
  clear_error();
  if (!m || !n || !nnz) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null size pointer");
  if (scale_rows < 0) return fail(SPMVB_ERR_INVALID_ARGUMENT, "negative scale_rows");
  Shape sh;
  SPMVB_TRY(shape_of(which, seed, scale_rows, sh));
  *m = sh.m;
  *n = sh.n;
  *nnz = sh.nnz;
  if (h_colind == nullptr) return SPMVB_OK;
  if (!h_rowptr || !h_values) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null output array");
  if (sh.nnz > INT32_MAX) return fail(SPMVB_ERR_UNSUPPORTED, "nnz exceeds int32 index range");

  Rng rc(seed, kColumns);
  Rng rv(seed, kValues);
  std::vector<int32_t> cols;
  std::unordered_set<uint32_t> seen;
  int64_t p = 0;
  h_rowptr[0] = 0;
  switch (which) {
    case 1:
      for (int32_t i = 0; i < sh.m; ++i) {
        const int32_t lo = std::max<int32_t>(0, i - 4), hi = std::min<int32_t>(sh.m - 1, i + 4);
        for (int32_t j = lo; j <= hi; ++j) {
          h_colind[p] = j;
          h_values[p] = rv.sym() + (j == i ? 10.0 : 0.0);
          ++p;
        }
        h_rowptr[i + 1] = static_cast<int32_t>(p);
      }
      break;
    case 2:
    case 5:
      for (int32_t i = 0; i < sh.m; ++i) {
        distinct_sorted(rc, 16, static_cast<uint32_t>(sh.n), cols, seen);
        for (int32_t c : cols) {
          h_colind[p] = c;
          h_values[p] = rv.sym();
          ++p;
        }
        h_rowptr[i + 1] = static_cast<int32_t>(p);
      }
      break;
    case 3:
      for (int32_t i = 0; i < sh.m; ++i) {
        distinct_sorted(rc, sh.lens[i], static_cast<uint32_t>(sh.n), cols, seen);
        for (int32_t c : cols) {
          h_colind[p] = c;
          h_values[p] = rv.sym();
          ++p;
        }
        h_rowptr[i + 1] = static_cast<int32_t>(p);
      }
      break;
    case 4: {
      const int32_t mb = sh.m / 4;
      const uint32_t nb = static_cast<uint32_t>(sh.n / 4);
      std::vector<double> blk(8 * 16);
      for (int32_t b = 0; b < mb; ++b) {
        distinct_sorted(rc, 8, nb, cols, seen);
        for (double& v : blk) v = rv.sym();  // block t, row r, col c at t*16 + r*4 + c
        for (int r = 0; r < 4; ++r) {
          for (int t = 0; t < 8; ++t) {
            for (int c = 0; c < 4; ++c) {
              h_colind[p] = cols[t] * 4 + c;
              h_values[p] = blk[t * 16 + r * 4 + c];
              ++p;
            }
          }
          h_rowptr[b * 4 + r + 1] = static_cast<int32_t>(p);
        }
      }
      break;
    }
  }
  return SPMVB_OK;
}

extern "C" spmvb_status spmvb_generate_vector(uint64_t seed, int64_t len, double* h_out) {
  clear_error();
  if (len < 0 || (len > 0 && !h_out)) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bad vector arguments");
  Rng r(seed, kVector);
  for (int64_t i = 0; i < len; ++i) h_out[i] = r.sym();
  return SPMVB_OK;
}
