#pragma once
// Kernel selection (same names as SpMVBench's select.hpp:11-33). KernelId
// keeps the reference's values 0..5 and adds Hyb before Count.
// choose_spmv applies the B200 rules; choose_spmv_reference the reference's
// own ordered rules 0-6 (src/select.cpp:93-165).
#include <stdexcept>
#include <string>

#include "spmvb.h"
#include "spmvbench/stats.hpp"

namespace spmvbench {

enum class KernelId : int { CsrScalar = 0, CsrVector, CsrWarp, CsrMerge, Ell, Bcsr, Hyb, Count };

inline const char* kernel_name(KernelId id) { return spmvb_kernel_name(static_cast<int>(id)); }

struct KernelChoice {
  KernelId kernel = KernelId::CsrVector;
  int lanes = 4;
  int block_r = 1;
  int block_c = 1;
  std::string reason;
};

namespace detail {
inline KernelChoice choice_from(spmvb_status st, const spmvb_choice& c) {
  if (st != SPMVB_OK) throw std::runtime_error(std::string("choose_spmv: ") + spmvb_last_error());
  KernelChoice k;
  k.kernel = static_cast<KernelId>(c.kernel);
  k.lanes = c.lanes;
  k.block_r = c.block_r;
  k.block_c = c.block_c;
  k.reason = c.reason;
  return k;
}
}  // namespace detail

inline KernelChoice choose_spmv(const RowStats& s) {
  const spmvb_row_stats c = to_c(s);
  spmvb_choice out{};
  const spmvb_status st = spmvb_choose_spmv(&c, &out);
  return detail::choice_from(st, out);
}

inline KernelChoice choose_spmv_reference(const RowStats& s) {
  const spmvb_row_stats c = to_c(s);
  spmvb_choice out{};
  const spmvb_status st = spmvb_choose_spmv_reference(&c, &out);
  return detail::choice_from(st, out);
}

}  // namespace spmvbench
