// On-device format conversion and block statistics (no reference
// counterpart on the device: the reference converts on the host with a
// linear search per entry, src/formats.cpp:45-105 and src/stats.cpp:96-102,
// O(L^2) per block row).
//
// BCSR R x C from the uploaded CSR, in csr_to_bcsr's layout: every entry gets
// the key ((block_row * nb + block_col) * R*C + r*C + c); one stable radix
// sort of (key, entry index) pairs orders the entries by block row, then
// ascending block column, then position inside the block, and keeps repeated
// (row, column) entries in CSR order. The first entry of each block writes
// its block column and counts the block for its block row; the last entry of
// each run of equal keys writes the value, so the last duplicate in CSR order
// wins, as in the reference; untouched slots stay zero.
//
// The 4 x 4 block census of compute_row_stats (blocks holding more than 8
// stored entries, duplicates counted, and blocks holding at least one) sorts
// the block keys alone and measures the runs.
#include <cub/cub.cuh>

#include <cstdint>
#include <string>
#include <vector>

#include "internal.hpp"

namespace spmvb {
namespace {

// Keys of every entry: one warp per row, lanes over the row's entries.
template <int R, int C>
__global__ void block_keys(const int* __restrict__ rowptr, const int* __restrict__ colind, int m, int64_t nb,
                           bool with_slot, uint64_t* __restrict__ keys, int* __restrict__ idx) {
  const int lane = threadIdx.x & 31;
  const int64_t w0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t row = w0; row < m; row += nw) {
    const uint64_t bi = static_cast<uint64_t>(row / R);
    const int r = static_cast<int>(row % R);
    const int e = rowptr[row + 1];
    for (int p = rowptr[row] + lane; p < e; p += 32) {
      const int c = colind[p];
      const uint64_t block = bi * static_cast<uint64_t>(nb) + static_cast<uint64_t>(c / C);
      keys[p] = with_slot ? block * (R * C) + static_cast<uint64_t>(r * C + c % C) : block;
      if (idx) idx[p] = p;
    }
  }
}

// 1 where a sorted entry starts a new block.
template <int RC>
__global__ void block_starts(const uint64_t* __restrict__ skeys, int64_t nnz, int* __restrict__ flag) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= nnz) return;
  flag[i] = (i == 0 || skeys[i] / RC != skeys[i - 1] / RC) ? 1 : 0;
}

template <int R, int C, typename V>
__global__ void bcsr_scatter(const uint64_t* __restrict__ skeys, const int* __restrict__ sidx,
                             const int* __restrict__ block_of, int64_t nnz, int64_t nb, const V* __restrict__ vals,
                             int* __restrict__ bcol, V* __restrict__ bval, int* __restrict__ per_row) {
  constexpr int RC = R * C;
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= nnz) return;
  const uint64_t key = skeys[i];
  const uint64_t block = key / RC;
  const int64_t b = block_of[i] - 1;  // inclusive count of block starts
  if (i == 0 || skeys[i - 1] / RC != block) {
    bcol[b] = static_cast<int>(block % static_cast<uint64_t>(nb));
    atomicAdd(per_row + block / static_cast<uint64_t>(nb), 1);
  }
  if (i == nnz - 1 || skeys[i + 1] != key) bval[b * RC + static_cast<int64_t>(key % RC)] = vals[sidx[i]];
}

// Per run of equal block keys: counts the run as stored, and as dense when
// it holds more than `dense_over` entries.
__global__ void block_census(const uint64_t* __restrict__ skeys, int64_t nnz, int dense_over,
                             unsigned long long* __restrict__ counts) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= nnz) return;
  if (i > 0 && skeys[i - 1] == skeys[i]) return;
  int64_t j = i + 1;
  while (j < nnz && skeys[j] == skeys[i] && j - i <= dense_over) ++j;
  atomicAdd(counts + 1, 1ull);
  if (j - i > dense_over) atomicAdd(counts, 1ull);
}

int key_bits(uint64_t max_key) {
  int b = 1;
  while (b < 64 && (max_key >> b) != 0) ++b;
  return b;
}

int grid_for(int64_t items, int threads = 256) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((items + threads - 1) / threads, INT32_MAX)));
}

// Sorted block keys (and, with `idx`, the entry order they came from) of A.
// `skeys`/`sidx` receive nnz entries.
template <int R, int C>
spmvb_status sorted_keys(spmvb_matrix A, bool with_slot, DevBuf& skeys, DevBuf* sidx, cudaStream_t s) {
  const int64_t nnz = A->nnz;
  const int64_t nb = (static_cast<int64_t>(A->n) + C - 1) / C;
  const int64_t mb = (static_cast<int64_t>(A->m) + R - 1) / R;
  DevBuf keys, idx;
  SPMVB_TRY(keys.alloc(nnz * 8));
  SPMVB_TRY(skeys.alloc(nnz * 8));
  if (sidx) {
    SPMVB_TRY(idx.alloc(nnz * 4));
    SPMVB_TRY(sidx->alloc(nnz * 4));
  }
  const int warps_grid = static_cast<int>(std::min<int64_t>((static_cast<int64_t>(A->m) * 32 + 255) / 256,
                                                            static_cast<int64_t>(A->ctx->sm_count) * 32));
  block_keys<R, C><<<std::max(1, warps_grid), 256, 0, s>>>(A->rowptr.as<int>(), A->colind.as<int>(), A->m, nb,
                                                            with_slot, keys.as<uint64_t>(),
                                                            sidx ? idx.as<int>() : nullptr);
  count_launch();
  SPMVB_TRY_CUDA(cudaGetLastError());
  const uint64_t max_key = static_cast<uint64_t>(std::max<int64_t>(mb * nb, 1)) * (with_slot ? R * C : 1);
  const int end_bit = key_bits(max_key - 1);
  size_t temp = 0;
  const int n = static_cast<int>(nnz);
  if (sidx) {
    SPMVB_TRY_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, temp, keys.as<uint64_t>(), skeys.as<uint64_t>(),
                                                   idx.as<int>(), sidx->as<int>(), n, 0, end_bit, s));
  } else {
    SPMVB_TRY_CUDA(cub::DeviceRadixSort::SortKeys(nullptr, temp, keys.as<uint64_t>(), skeys.as<uint64_t>(), n, 0,
                                                  end_bit, s));
  }
  DevBuf tmp;
  SPMVB_TRY(tmp.alloc(std::max<size_t>(temp, 16)));
  if (sidx) {
    SPMVB_TRY_CUDA(cub::DeviceRadixSort::SortPairs(tmp.get(), temp, keys.as<uint64_t>(), skeys.as<uint64_t>(),
                                                   idx.as<int>(), sidx->as<int>(), n, 0, end_bit, s));
  } else {
    SPMVB_TRY_CUDA(cub::DeviceRadixSort::SortKeys(tmp.get(), temp, keys.as<uint64_t>(), skeys.as<uint64_t>(), n, 0,
                                                  end_bit, s));
  }
  count_launch();
  SPMVB_TRY_CUDA(cudaStreamSynchronize(s));
  return SPMVB_OK;
}

template <int R, int C, typename V>
spmvb_status bcsr_device(spmvb_matrix A, spmvb_matrix_st::Bcsr& B, cudaStream_t s) {
  constexpr int RC = R * C;
  const int64_t nnz = A->nnz;
  const int mb = static_cast<int>((static_cast<int64_t>(A->m) + R - 1) / R);
  const int64_t nb = (static_cast<int64_t>(A->n) + C - 1) / C;
  DevBuf per_row;
  SPMVB_TRY(per_row.alloc(static_cast<size_t>(mb + 1) * 4));
  int64_t blocks = 0;
  DevBuf bcol, bval;
  if (nnz > 0) {
    DevBuf skeys, sidx, flag, block_of;
    SPMVB_TRY((sorted_keys<R, C>(A, true, skeys, &sidx, s)));
    SPMVB_TRY(flag.alloc(nnz * 4));
    SPMVB_TRY(block_of.alloc(nnz * 4));
    block_starts<RC><<<grid_for(nnz), 256, 0, s>>>(skeys.as<uint64_t>(), nnz, flag.as<int>());
    count_launch();
    size_t temp = 0;
    SPMVB_TRY_CUDA(cub::DeviceScan::InclusiveSum(nullptr, temp, flag.as<int>(), block_of.as<int>(),
                                                 static_cast<int>(nnz), s));
    DevBuf tmp;
    SPMVB_TRY(tmp.alloc(std::max<size_t>(temp, 16)));
    SPMVB_TRY_CUDA(cub::DeviceScan::InclusiveSum(tmp.get(), temp, flag.as<int>(), block_of.as<int>(),
                                                 static_cast<int>(nnz), s));
    count_launch();
    int last = 0;
    SPMVB_TRY_CUDA(cudaMemcpyAsync(&last, block_of.as<int>() + (nnz - 1), 4, cudaMemcpyDeviceToHost, s));
    SPMVB_TRY_CUDA(cudaStreamSynchronize(s));
    blocks = last;
    SPMVB_TRY(bcol.alloc((blocks + kPad) * 4));
    SPMVB_TRY(bval.alloc((blocks * RC + kPad) * sizeof(V)));
    bcsr_scatter<R, C, V><<<grid_for(nnz), 256, 0, s>>>(skeys.as<uint64_t>(), sidx.as<int>(), block_of.as<int>(),
                                                        nnz, nb, A->values.as<V>(), bcol.as<int>(), bval.as<V>(),
                                                        per_row.as<int>() + 1);
    count_launch();
    SPMVB_TRY_CUDA(cudaGetLastError());
    // Block row pointers: inclusive sum of the per-block-row counts after a
    // leading zero.
    size_t t2 = 0;
    SPMVB_TRY_CUDA(cub::DeviceScan::InclusiveSum(nullptr, t2, per_row.as<int>() + 1, per_row.as<int>() + 1, mb, s));
    DevBuf tmp2;
    SPMVB_TRY(tmp2.alloc(std::max<size_t>(t2, 16)));
    SPMVB_TRY_CUDA(cub::DeviceScan::InclusiveSum(tmp2.get(), t2, per_row.as<int>() + 1, per_row.as<int>() + 1, mb, s));
    count_launch();
    SPMVB_TRY_CUDA(cudaStreamSynchronize(s));
  } else {
    SPMVB_TRY(bcol.alloc(kPad * 4));
    SPMVB_TRY(bval.alloc(kPad * sizeof(V)));
  }
  B.rowptr = std::move(per_row);
  B.colind = std::move(bcol);
  B.values = std::move(bval);
  B.mb = mb;
  B.block_nnz = blocks;
  return SPMVB_OK;
}

}  // namespace

spmvb_status convert_bcsr_device(spmvb_matrix A, int block) {
  auto& B = block == 2 ? A->bcsr2 : A->bcsr4;
  const cudaStream_t s = nullptr;
  if (A->nnz > INT32_MAX) return fail(SPMVB_ERR_UNSUPPORTED, "nnz beyond the int32 index range");
  if (A->dtype == SPMVB_F64)
    return block == 2 ? bcsr_device<2, 2, double>(A, B, s) : bcsr_device<4, 4, double>(A, B, s);
  return block == 2 ? bcsr_device<2, 2, float>(A, B, s) : bcsr_device<4, 4, float>(A, B, s);
}

spmvb_status block_census_device(spmvb_matrix A, int64_t* dense, int64_t* stored) {
  *dense = *stored = 0;
  if (A->nnz == 0) return SPMVB_OK;
  if (A->nnz > INT32_MAX) return fail(SPMVB_ERR_UNSUPPORTED, "nnz beyond the int32 index range");
  const cudaStream_t s = nullptr;
  DevBuf skeys, counts;
  SPMVB_TRY((sorted_keys<4, 4>(A, false, skeys, nullptr, s)));
  SPMVB_TRY(counts.alloc(16));
  block_census<<<grid_for(A->nnz), 256, 0, s>>>(skeys.as<uint64_t>(), A->nnz, 8, counts.as<unsigned long long>());
  count_launch();
  SPMVB_TRY_CUDA(cudaGetLastError());
  unsigned long long h[2] = {0, 0};
  SPMVB_TRY_CUDA(cudaMemcpyAsync(h, counts.get(), 16, cudaMemcpyDeviceToHost, s));
  SPMVB_TRY_CUDA(cudaStreamSynchronize(s));
  *dense = static_cast<int64_t>(h[0]);
  *stored = static_cast<int64_t>(h[1]);
  return SPMVB_OK;
}

}  // namespace spmvb
