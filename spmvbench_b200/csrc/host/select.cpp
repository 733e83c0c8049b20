// Kernel selection.
//
// spmvb_choose_spmv_reference restates the reference's ordered rules 0-6
// (src/select.cpp:93-165) unchanged, for callers that want its exact picks.
//
// spmvb_choose_spmv is the B200 rule set, ordered by what decides the cost
// of each kernel: skewed rows need an equal share of entries per warp (the
// hybrid format's chunks),
// mostly-dense 4x4 blocks let BCSR drop 15 of 16 column indices, nearly
// uniform rows go to ELL (coalesced, all gathers in flight), long rows fill a
// warp's vector loads, and the rest take the merge path.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>

#include "../internal.hpp"

using namespace spmvb;

namespace {

int next_pow2(int v) {
  if (v <= 1) return 1;
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

// std::to_string with trailing zeros trimmed (the reference's fmt,
// src/select.cpp:59-69).
std::string fmt(double v) {
  std::string s = std::to_string(v);
  if (s.find('.') != std::string::npos) {
    while (!s.empty() && s.back() == '0') s.pop_back();
    if (!s.empty() && s.back() == '.') s.pop_back();
  }
  return s;
}

void set(spmvb_choice* c, int kernel, int lanes, int br, int bc, int rule, const std::string& why) {
  c->kernel = kernel;
  c->lanes = lanes;
  c->block_r = br;
  c->block_c = bc;
  c->rule = rule;
  std::snprintf(c->reason, sizeof(c->reason), "%s", why.c_str());
}

}  // namespace

extern "C" const char* spmvb_kernel_name(int kernel) {
  switch (kernel) {
    case SPMVB_CSR_SCALAR: return "csr_scalar";
    case SPMVB_CSR_VECTOR: return "csr_vector";
    case SPMVB_CSR_WARP: return "csr_warp";
    case SPMVB_CSR_MERGE: return "csr_merge";
    case SPMVB_ELL: return "ell";
    case SPMVB_BCSR: return "bcsr";
    case SPMVB_HYB: return "hyb";
    default: return "unknown";
  }
}

extern "C" spmvb_status spmvb_choose_spmv_reference(const spmvb_row_stats* sp, spmvb_choice* c) {
  clear_error();
  if (!sp || !c) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  const spmvb_row_stats& s = *sp;
  // Defaults of KernelChoice (include/spmvbench/select.hpp:21-27).
  set(c, SPMVB_CSR_VECTOR, 4, 1, 1, -1, "");
  if (s.nnz < 50000) {
    set(c, SPMVB_CSR_SCALAR, 1, 1, 1, 0,
        "nnz=" + std::to_string(s.nnz) +
            " < 50000: problem too small for parallel/format overhead to pay off, use scalar");
    return SPMVB_OK;
  }
  if (s.mean_row_nnz < 4.0) {
    set(c, SPMVB_CSR_SCALAR, 1, 1, 1, 1,
        "mean_row_nnz=" + fmt(s.mean_row_nnz) + " < 4: short rows, scalar (one thread/row) is cheapest");
    return SPMVB_OK;
  }
  if (s.frac_dense_blocks_4x4 > 0.6) {
    set(c, SPMVB_BCSR, 4, 4, 4, 2,
        "frac_dense_blocks_4x4=" + fmt(s.frac_dense_blocks_4x4) + " > 0.6: locally dense, use 4x4 block storage");
    return SPMVB_OK;
  }
  if (s.cv_row_nnz > 1.5 || s.max_over_mean > 50.0) {
    set(c, SPMVB_CSR_MERGE, 1, 1, 1, 3,
        "cv=" + fmt(s.cv_row_nnz) + " or max/mean=" + fmt(s.max_over_mean) +
            " indicates skew: use nnz-load-balanced csr_merge");
    return SPMVB_OK;
  }
  if (s.mean_row_nnz >= 4.0 && s.mean_row_nnz < 32.0 && s.cv_row_nnz < 0.5) {
    const int lanes = next_pow2(static_cast<int>(std::ceil(s.mean_row_nnz)));
    set(c, SPMVB_CSR_VECTOR, lanes, 1, 1, 4,
        "4 <= mean_row_nnz=" + fmt(s.mean_row_nnz) + " < 32 and cv=" + fmt(s.cv_row_nnz) +
            " < 0.5: sub-warp vector group with lanes=" + std::to_string(lanes));
    return SPMVB_OK;
  }
  if (s.ell_padding_overhead < 1.2) {
    set(c, SPMVB_ELL, 1, 1, 1, 5,
        "ell_padding_overhead=" + fmt(s.ell_padding_overhead) +
            " < 1.2: long but nearly uniform rows, coalesced ELL wins");
    return SPMVB_OK;
  }
  set(c, SPMVB_CSR_VECTOR, 4, 1, 1, 6,
      "no special signal (mean_row_nnz=" + fmt(s.mean_row_nnz) + ", cv=" + fmt(s.cv_row_nnz) +
          "): default sub-warp vector group with lanes=4");
  return SPMVB_OK;
}

extern "C" spmvb_status spmvb_choose_spmv(const spmvb_row_stats* sp, spmvb_choice* c) {
  clear_error();
  if (!sp || !c) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  const spmvb_row_stats& s = *sp;
  set(c, SPMVB_CSR_SCALAR, 1, 1, 1, -1, "");
  // (0) Skewed row lengths: the hybrid format streams every row in equal
  // chunks of entries (rows packed whole, long rows cut into segments), so
  // every warp gets the same work; on the power-law 1M matrix it runs 1.47x
  // faster than the merge path.
  if (s.cv_row_nnz > 1.5 || s.max_over_mean > 50.0) {
    set(c, SPMVB_HYB, 1, 1, 1, 0,
        "cv=" + fmt(s.cv_row_nnz) + " or max/mean=" + fmt(s.max_over_mean) +
            " indicates skew: hybrid format, rows streamed in equal chunks of entries");
    return SPMVB_OK;
  }
  // (1) Mostly dense 4x4 blocks among the occupied ones: BCSR stores one
  // column index per 16 values.
  if (s.dense_share_of_stored_4x4 > 0.6) {
    set(c, SPMVB_BCSR, 4, 4, 4, 1,
        "dense_share_of_stored_4x4=" + fmt(s.dense_share_of_stored_4x4) +
            " > 0.6: block storage cuts index traffic");
    return SPMVB_OK;
  }
  // (2) Nearly uniform rows (padded ELL at most 1.5x the entries): ELL reads
  // each row with coalesced column-major loads and keeps every row's gathers
  // in flight; on the uniform 1M x 16 matrix it runs at 94% of the device's
  // random-gather ceiling, and it sums in csr_omp order.
  if (s.ell_padding_overhead <= 1.5) {
    set(c, SPMVB_ELL, 1, 1, 1, 2,
        "ell_padding_overhead=" + fmt(s.ell_padding_overhead) +
            " <= 1.5: column-major ELL, coalesced and gather-bound");
    return SPMVB_OK;
  }
  // (3) Long rows: a full warp per row streams them with vector loads.
  if (s.mean_row_nnz >= 96.0) {
    set(c, SPMVB_CSR_VECTOR, 32, 1, 1, 3,
        "mean_row_nnz=" + fmt(s.mean_row_nnz) + " >= 96: warp-wide vector rows");
    return SPMVB_OK;
  }
  // (4) Everything else (moderately uneven rows): the merge path is balanced
  // whatever the row lengths.
  set(c, SPMVB_CSR_MERGE, 1, 1, 1, 4,
      "mean_row_nnz=" + fmt(s.mean_row_nnz) + ", cv=" + fmt(s.cv_row_nnz) +
          ", ell_padding_overhead=" + fmt(s.ell_padding_overhead) + ": balanced merge path");
  return SPMVB_OK;
}
