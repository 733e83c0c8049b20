#pragma once
// Blocked CSR and csr_to_bcsr<T,R,C> with the layout of SpMVBench's
// csr_to_bcsr (src/formats.cpp:45-105): blocks of a block row in ascending
// block-column order, R*C row-major values, zero fill, and a repeated
// (row, column) keeps its last value in CSR order. Built by sorting each
// block row's entries (O(L log L)) instead of a linear block search.
#include <algorithm>
#include <cstdint>
#include <vector>

#include "spmvbench/csr.hpp"

namespace spmvbench {

template <typename T>
struct BcsrMatrix {
  using value_type = T;
  int m = 0;
  int n = 0;
  int R = 0;
  int C = 0;
  int mb = 0;
  int nb = 0;
  std::int64_t nnz = 0;
  std::int64_t block_nnz = 0;
  std::vector<Index> rowptr;
  std::vector<Index> colind;
  std::vector<T> values;

  double density() const {
    const std::int64_t slots = block_nnz * static_cast<std::int64_t>(R) * C;
    return slots == 0 ? 0.0 : static_cast<double>(nnz) / static_cast<double>(slots);
  }
};

template <typename T, int R, int C>
BcsrMatrix<T> csr_to_bcsr(const CsrMatrix<T>& A) {
  static_assert(R >= 1 && C >= 1, "block dimensions must be positive");
  BcsrMatrix<T> B;
  B.m = A.m;
  B.n = A.n;
  B.R = R;
  B.C = C;
  B.mb = (A.m + R - 1) / R;
  B.nb = (A.n + C - 1) / C;
  B.nnz = A.nnz;
  B.rowptr.assign(static_cast<std::size_t>(B.mb) + 1, 0);
  struct Ent {
    Index bj;
    int slot;
  };
  std::vector<Ent> ents;
  for (int bi = 0; bi < B.mb; ++bi) {
    ents.clear();
    for (int r = 0; r < R && bi * R + r < A.m; ++r)
      for (Index p = A.rowptr[bi * R + r]; p < A.rowptr[bi * R + r + 1]; ++p)
        ents.push_back({A.colind[p] / C, static_cast<int>(p)});
    std::stable_sort(ents.begin(), ents.end(), [](const Ent& a, const Ent& b) { return a.bj < b.bj; });
    for (std::size_t a = 0; a < ents.size();) {
      const std::size_t base = B.values.size();
      B.values.resize(base + static_cast<std::size_t>(R) * C, T(0));
      B.colind.push_back(ents[a].bj);
      std::size_t b = a;
      for (; b < ents.size() && ents[b].bj == ents[a].bj; ++b) {
        const Index p = ents[b].slot;
        // row of entry p inside the block row: the stable sort kept CSR order
        int r = 0;
        while (bi * R + r + 1 <= A.m && A.rowptr[bi * R + r + 1] <= p) ++r;
        B.values[base + static_cast<std::size_t>(r) * C + A.colind[p] % C] = A.values[p];
      }
      a = b;
    }
    B.rowptr[bi + 1] = static_cast<Index>(B.colind.size());
  }
  B.block_nnz = static_cast<std::int64_t>(B.colind.size());
  return B;
}

}  // namespace spmvbench
