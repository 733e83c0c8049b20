// Merge-path SpMV that allocates nothing: spmvb_spmv_merge_noalloc.
//
// Who needs it: callers that cannot call cudaMalloc. Typical cases are a host
// application whose device memory belongs to another allocator (a framework's
// caching allocator or a pool sized at start-up, which an outside cudaMalloc
// would fragment or push over budget), and services with latency rules that
// forbid allocating after start-up, because cudaMalloc / cudaFree can
// synchronize the device and take unbounded time. Such a caller owns the CSR
// arrays, x and y on the device and passes them in; the kernels' scratch (the
// merge-path tile starts and the per-tile carries) lives in the file-scope
// array below, so no call allocates.
//
// The scratch array is a static __device__ object: every GPU that loads this
// library holds it (kNoallocScratchBytes) until the process exits. In host
// code its name only stands in for the device object, so its device address
// is fetched once per device with cudaGetSymbolAddress, with that device
// current, and passed to the kernels. Every call on a device shares the
// array: calls whose kernels overlap on the GPU (different streams, no
// ordering between them) race on it. Each call writes every scratch word it
// later reads (tile starts by the partition kernel, one carry per tile by
// the merge kernel), so nothing has to be cleared between calls.
//
// The merge kernel here is a copy of csr_merge (spmv_kernels.cuh) that stages
// products with bounds-checked scalar loads: caller-owned arrays carry no
// padding past nnz, so it never reads past the last entry.
#include <climits>
#include <cstdint>
#include <mutex>

#include "internal.hpp"
#include "spmv_kernels.cuh"

namespace spmvb {

// Merge-path tile of this entry point: 256 threads x 7 items.
constexpr int kNoallocThreads = 256;
constexpr int kNoallocIpt = 7;
constexpr int kNoallocTile = kNoallocThreads * kNoallocIpt;

// Tiles of kNoallocTile merge items; the scratch holds, per tile, its start row
// (plus one), its carry row and its carry value (8 bytes, the widest Acc),
// each region starting on a 256-byte boundary.
constexpr int kNoallocMaxTiles = 65536;
constexpr size_t kAlign256(size_t b) { return (b + 255) / 256 * 256; }
constexpr size_t kNoallocCarryRowOffset = kAlign256(static_cast<size_t>(kNoallocMaxTiles + 1) * 4);
constexpr size_t kNoallocCarryValOffset = kNoallocCarryRowOffset + kAlign256(static_cast<size_t>(kNoallocMaxTiles) * 4);
constexpr size_t kNoallocScratchBytes = kNoallocCarryValOffset + static_cast<size_t>(kNoallocMaxTiles) * 8;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

template <typename T, typename Acc, int NT, int IPT>
__global__ void __launch_bounds__(NT)
    csr_merge_scratch(CsrView A, MergeView M, const T* __restrict__ x, Acc* __restrict__ y) {
  constexpr int TILE = NT * IPT;
  __shared__ int s_rowend[TILE + 1];
  __shared__ Acc s_prod[TILE];
  __shared__ int s_crow[NT];
  __shared__ Acc s_cval[NT];
  const T* __restrict__ vals = static_cast<const T*>(A.values);
  const int t = threadIdx.x;
  const int tile = blockIdx.x;
  const int64_t d0 = static_cast<int64_t>(tile) * TILE;
  const int64_t d1 = min(d0 + TILE, M.num_items);
  const int row0 = M.tile_row[tile];
  const int row1 = M.tile_row[tile + 1];
  const int64_t j0 = d0 - row0;
  const int64_t j1 = d1 - row1;
  const int nrows_local = row1 - row0;
  const int nnz_local = static_cast<int>(j1 - j0);

  for (int i = t; i <= nrows_local; i += NT) {
    const int r = row0 + i;
    s_rowend[i] = (r < A.m) ? A.rowptr[r + 1] : INT_MAX;
  }
  // Products of this tile's entries [j0, j1), one coalesced scalar load per
  // thread and entry; j1 <= nnz, so nothing past the arrays is read.
  for (int q = t; q < nnz_local; q += NT) {
    const int64_t p = j0 + q;
    s_prod[q] = prod<Acc>(vals[p], x[A.colind[p]]);
  }
  __syncthreads();

  const int items = static_cast<int>(d1 - d0);
  const int k = min(t * IPT, items);
  int lo = max(0, k - nnz_local);
  int hi = min(k, nrows_local);
  while (lo < hi) {
    const int pivot = (lo + hi) >> 1;
    if (s_rowend[pivot] <= j0 + k - pivot - 1)
      lo = pivot + 1;
    else
      hi = pivot;
  }
  int row = row0 + lo;
  int64_t nz = j0 + k - lo;
  const int start_row = row;
  const int my_items = min(IPT, items - k);

  Acc sum = Acc(0);
  bool have = false;
  int held_row = -1;
  Acc held_val = Acc(0);
  for (int i = 0; i < my_items; ++i) {
    if (nz < s_rowend[row - row0]) {
      sum = add_rn(sum, s_prod[nz - j0]);
      have = true;
      ++nz;
    } else {
      if (row == start_row && held_row < 0) {
        held_row = row;
        held_val = sum;
      } else {
        y[row] = sum;
      }
      sum = Acc(0);
      have = false;
      ++row;
    }
  }
  s_crow[t] = have ? row : -1;
  s_cval[t] = sum;
  __syncthreads();

  if (held_row >= 0) {
    int t0 = t;
    while (t0 > 0 && s_crow[t0 - 1] == held_row) --t0;
    if (t0 < t) {
      Acc c = s_cval[t0];
      for (int u = t0 + 1; u < t; ++u) c = add_rn(c, s_cval[u]);
      y[held_row] = add_rn(c, held_val);
    } else {
      y[held_row] = held_val;
    }
  }
  if (t == NT - 1) {
    const int r = s_crow[NT - 1];
    if (r >= 0) {
      int t0 = NT - 1;
      while (t0 > 0 && s_crow[t0 - 1] == r) --t0;
      Acc c = s_cval[t0];
      for (int u = t0 + 1; u < NT; ++u) c = add_rn(c, s_cval[u]);
      M.carry_row[tile] = r;
      static_cast<Acc*>(M.carry_val)[tile] = c;
    } else {
      M.carry_row[tile] = -1;
    }
  }
}

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
unsigned char* g_noalloc_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on `device` (current), fetched on the
// first call for that device.
spmvb_status noalloc_scratch(int device, unsigned char** out) {
  if (device < 0 || device >= kMaxDevices) return fail(SPMVB_ERR_NO_DEVICE, "device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_noalloc_addr[device] = static_cast<unsigned char*>(p);
  }
  *out = g_noalloc_addr[device];
  return SPMVB_OK;
}

template <typename T, typename Acc>
void launch_noalloc(const CsrView& v, unsigned char* scratch, int tiles, const T* x, Acc* y, cudaStream_t s) {
  MergeView mv;
  int* tile_row = reinterpret_cast<int*>(scratch);
  mv.tile_row = tile_row;
  mv.carry_row = reinterpret_cast<int*>(scratch + kNoallocCarryRowOffset);
  mv.carry_val = scratch + kNoallocCarryValOffset;
  mv.num_items = static_cast<int64_t>(v.m) + v.nnz;
  mv.num_tiles = tiles;
  mv.tile_items = kNoallocTile;
  merge_partition<<<(tiles + 1 + 255) / 256, 256, 0, s>>>(v, mv.num_items, kNoallocTile, tiles, tile_row);
  csr_merge_scratch<T, Acc, kNoallocThreads, kNoallocIpt><<<tiles, kNoallocThreads, 0, s>>>(v, mv, x, y);
  merge_fixup<Acc><<<(tiles + 255) / 256, 256, 0, s>>>(mv, y);
  count_launch(3);
}

}  // namespace
}  // namespace spmvb

using namespace spmvb;

extern "C" spmvb_status spmvb_spmv_merge_noalloc(spmvb_dtype dtype, int32_t m, int32_t n, int64_t nnz,
                                                 const int32_t* d_rowptr, const int32_t* d_colind,
                                                 const void* d_values, const void* d_x, void* d_y,
                                                 spmvb_dtype acc, void* stream) {
  clear_error();
  if (dtype != SPMVB_F32 && dtype != SPMVB_F64) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bad dtype");
  if (acc != SPMVB_F32 && acc != SPMVB_F64) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bad accumulator dtype");
  if (dtype == SPMVB_F64 && acc == SPMVB_F32)
    return fail(SPMVB_ERR_UNSUPPORTED, "fp64 storage with fp32 accumulation is not instantiated");
  if (m < 0 || n < 0 || nnz < 0 || nnz > INT32_MAX) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bad m, n or nnz");
  // Every stored entry names a column of x, so entries with no columns
  // would make the kernel read an empty x.
  if (nnz > 0 && n == 0) return fail(SPMVB_ERR_INVALID_ARGUMENT, "nnz > 0 with n == 0: no column to index");
  if (m == 0) return SPMVB_OK;
  const int64_t items = static_cast<int64_t>(m) + nnz;
  const int64_t tiles = (items + kNoallocTile - 1) / kNoallocTile;
  if (tiles > kNoallocMaxTiles) {
    return fail(SPMVB_ERR_UNSUPPORTED,
                "m + nnz = " + std::to_string(items) + " exceeds the no-allocation limit of " +
                    std::to_string(static_cast<int64_t>(kNoallocMaxTiles) * kNoallocTile) +
                    " (its scratch is a fixed " + std::to_string(kNoallocScratchBytes) + "-byte device array)");
  }
  if (!d_rowptr || (nnz > 0 && (!d_colind || !d_values)) || (n > 0 && !d_x) || !d_y)
    return fail(SPMVB_ERR_INVALID_ARGUMENT, "null device pointer");
  int device = 0;
  SPMVB_TRY_CUDA(cudaGetDevice(&device));
  unsigned char* scratch = nullptr;
  SPMVB_TRY(noalloc_scratch(device, &scratch));
  CsrView v;
  v.rowptr = d_rowptr;
  v.colind = d_colind;
  v.values = d_values;
  v.m = m;
  v.n = n;
  v.nnz = nnz;
  auto s = static_cast<cudaStream_t>(stream);
  if (dtype == SPMVB_F64)
    launch_noalloc<double, double>(v, scratch, static_cast<int>(tiles), static_cast<const double*>(d_x),
                                   static_cast<double*>(d_y), s);
  else if (acc == SPMVB_F32)
    launch_noalloc<float, float>(v, scratch, static_cast<int>(tiles), static_cast<const float*>(d_x),
                                 static_cast<float*>(d_y), s);
  else
    launch_noalloc<float, double>(v, scratch, static_cast<int>(tiles), static_cast<const float*>(d_x),
                                  static_cast<double*>(d_y), s);
  SPMVB_TRY_CUDA(cudaGetLastError());
  return SPMVB_OK;
}
