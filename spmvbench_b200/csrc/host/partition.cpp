// nnz-balanced contiguous row partition for row-sharded multi-GPU SpMV.
// The reference has no multi-GPU path; this rule is new:
//   bounds[0] = 0, bounds[parts] = m,
//   bounds[g] = lower_bound(rowptr[0..m], ceil(g * nnz / parts)) for 0 < g < parts
// i.e. part g starts at the first row whose starting offset reaches its equal
// share of nonzeros. The rule is deterministic and bounds are non-decreasing.
#include <algorithm>
#include <cstdint>

#include "../internal.hpp"

using namespace spmvb;

extern "C" spmvb_status spmvb_partition_rows(const int32_t* h_rowptr, int32_t m,
                                             int32_t parts, int32_t* h_bounds) {
  clear_error();
  if (!h_rowptr || !h_bounds) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  if (m < 0 || parts <= 0) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bad m or parts");
  const int64_t nnz = h_rowptr[m];
  h_bounds[0] = 0;
  for (int32_t g = 1; g < parts; ++g) {
    const int64_t target = (static_cast<int64_t>(g) * nnz + parts - 1) / parts;
    const int32_t* it = std::lower_bound(h_rowptr, h_rowptr + m + 1, static_cast<int32_t>(target));
    h_bounds[g] = static_cast<int32_t>(std::min<int64_t>(it - h_rowptr, m));
  }
  h_bounds[parts] = m;
  for (int32_t g = 1; g <= parts; ++g) h_bounds[g] = std::max(h_bounds[g], h_bounds[g - 1]);
  return SPMVB_OK;
}
