// Host-side internals of libspmvb: status plumbing, device buffers, and the
// context / matrix handles behind the C ABI (include/spmvb.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/spmvb.h"
#include "views.hpp"

namespace spmvb {

// ---- status / errors -------------------------------------------------------
// Records `msg` as this thread's last error and returns `s`.
spmvb_status fail(spmvb_status s, const std::string& msg);
spmvb_status cuda_fail(cudaError_t e, const char* what);
void clear_error();

extern std::atomic<uint64_t> g_launches;
inline void count_launch(uint64_t n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }
inline void uncount_launch(uint64_t n) { g_launches.fetch_sub(n, std::memory_order_relaxed); }

#define SPMVB_TRY_CUDA(expr)                                  \
  do {                                                        \
    cudaError_t _e = (expr);                                  \
    if (_e != cudaSuccess) return ::spmvb::cuda_fail(_e, #expr); \
  } while (0)

#define SPMVB_TRY(expr)                          \
  do {                                           \
    spmvb_status _s = (expr);                    \
    if (_s != SPMVB_OK) return _s;               \
  } while (0)

// Switches to `dev` for the lifetime of the guard.
class DeviceGuard {
 public:
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev_);
    if (prev_ != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != prev_) cudaSetDevice(prev_);
  }
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;

 private:
  int prev_ = 0;
};

// Owning device allocation.
class DevBuf {
 public:
  DevBuf() = default;
  ~DevBuf() { reset(); }
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  DevBuf(DevBuf&& o) noexcept : p_(o.p_), bytes_(o.bytes_) { o.p_ = nullptr; o.bytes_ = 0; }
  DevBuf& operator=(DevBuf&& o) noexcept {
    if (this != &o) { reset(); p_ = o.p_; bytes_ = o.bytes_; o.p_ = nullptr; o.bytes_ = 0; }
    return *this;
  }
  spmvb_status alloc(size_t bytes);  // zero-filled
  void reset();
  void* get() const { return p_; }
  template <typename U> U* as() const { return static_cast<U*>(p_); }
  size_t bytes() const { return bytes_; }
  // Gives up ownership without freeing (the allocation outlives the handle).
  void* release() {
    void* p = p_;
    p_ = nullptr;
    bytes_ = 0;
    return p;
  }

 private:
  void* p_ = nullptr;
  size_t bytes_ = 0;
};

// Upload host bytes into a fresh zero-filled buffer of at least `cap` bytes.
spmvb_status upload(DevBuf& dst, const void* src, size_t bytes, size_t cap);

inline size_t dtype_size(spmvb_dtype d) { return d == SPMVB_F64 ? 8 : 4; }

}  // namespace spmvb

struct spmvb_context_st {
  int device = 0;
  int sm_count = 0;
  int l2_bytes = 0;
  int max_smem_optin = 0;
  // Device error word: kernels whose bounded waits give up write a non-zero
  // code here (see spmvb_context_check).
  spmvb::DevBuf err;
};

struct spmvb_matrix_st {
  spmvb_context ctx = nullptr;
  int device = 0;
  spmvb_dtype dtype = SPMVB_F64;
  int m = 0;
  int n = 0;
  int64_t nnz = 0;
  int max_row = 0;

  // Host copy of the CSR arrays (the reference's SpmvRunner also keeps one,
  // src/cuda/spmv_cuda.cu:147). Lazily built formats are derived from it.
  std::vector<int32_t> h_rowptr;
  std::vector<int32_t> h_colind;
  std::vector<unsigned char> h_values;

  spmvb::DevBuf rowptr, colind, values;

  // ELL (reference layout, ld = m)
  bool ell_built = false;
  int ell_width = 0;
  spmvb::DevBuf ell_colind, ell_values, ell_rowlen;
  // TMA descriptors of the ELL arrays for ell_tma: state 0 = not built yet,
  // 1 = ready, -1 = this matrix cannot use them (ell_rows runs).
  int ell_tma_state = 0;
  alignas(64) CUtensorMap ell_tm_col;
  alignas(64) CUtensorMap ell_tm_val;

  // Hybrid ELL(K) + CSR tail
  bool hyb_built = false;
  int hyb_K = 0;
  int64_t hyb_ell_nnz = 0, hyb_tail_nnz = 0;
  int hyb_n_long = 0;
  int hyb_n_chunks = 0;
  int hyb_n_split = 0;
  int hyb_n_empty = 0;
  spmvb::DevBuf hyb_colind, hyb_values, hyb_rowlen, hyb_long_rows, hyb_tail_ptr,
      hyb_tail_colind, hyb_tail_values, hyb_chunk_start, hyb_chunk_row, hyb_chunk_split, hyb_split_rows,
      hyb_split_first, hyb_split_count, hyb_empty_rows, hyb_partial;

  // BCSR 2x2 and 4x4
  struct Bcsr {
    bool built = false;
    int mb = 0;
    int64_t block_nnz = 0;
    spmvb::DevBuf rowptr, colind, values;
  } bcsr2, bcsr4;

  // Merge-path partition + carry scratch (sized for the widest accumulator)
  bool merge_built = false;
  int merge_tiles = 0;
  spmvb::DevBuf merge_tile_row, merge_carry_row, merge_carry_val;

  // SpMM column bands: rows' entries split at band_count - 1 column
  // boundaries ((band_count - 1) x m ints); band_count 0 = not built.
  // sorted_rows: every row's columns ascend (the band sweep needs it).
  int band_count = 0;
  bool sorted_rows = false;
  int spmm_bands = 0;  // requested band count (0 = automatic)
  spmvb::DevBuf band_split;

  // SpMM row buckets
  bool buckets_built = false;
  int b_short = 0, b_med = 0, b_long = 0;
  spmvb::DevBuf bucket_rows;

  // Staging buffers for the host-buffer entry points
  spmvb::DevBuf stage_in, stage_out;

  std::mutex build_mu;

  spmvb::CsrView csr_view() const {
    spmvb::CsrView v;
    v.rowptr = rowptr.as<int>();
    v.colind = colind.as<int>();
    v.values = values.get();
    v.m = m;
    v.n = n;
    v.nnz = nnz;
    return v;
  }
  int64_t device_bytes() const;
};

namespace spmvb {

// Lazy builders (formats.cpp). Each is idempotent and thread safe.
spmvb_status build_ell(spmvb_matrix A);
spmvb_status build_hyb(spmvb_matrix A, int forced_k);
spmvb_status build_bcsr(spmvb_matrix A, int block);
spmvb_status build_merge(spmvb_matrix A);
spmvb_status build_buckets(spmvb_matrix A);
// Row split points of the SpMM column-band sweep for `bands` bands.
spmvb_status build_band_splits(spmvb_matrix A, int bands);
// TMA descriptors for ell_tma (formats.cu); sets A->ell_tma_state. Needs the
// ELL built; a matrix that does not qualify (width > max_width, m not a
// multiple of 4) or a process without SPMVB_ELL_STREAM=tma gets state -1.
spmvb_status build_ell_tma(spmvb_matrix A, int max_width);

// On-device conversions (convert.cu): BCSR block x block (2 or 4) from the
// uploaded CSR into A->bcsr2 / A->bcsr4, and the 4x4 block census of
// compute_row_stats (blocks with more than 8 stored entries, blocks with any).
spmvb_status convert_bcsr_device(spmvb_matrix A, int block);
spmvb_status block_census_device(spmvb_matrix A, int64_t* dense, int64_t* stored);

// Merge-path tile shape shared by the partition builder and the kernel.
constexpr int kMergeThreads = 128;
constexpr int kMergeIpt = 11;
constexpr int kMergeTile = kMergeThreads * kMergeIpt;

// Device launchers, one instantiation per (T, Acc) in spmv_<t><acc>.cu.
template <typename T, typename Acc>
spmvb_status launch_spmv(spmvb_matrix A, spmvb_kernel kernel, int lanes,
                         int block, const T* x, Acc* y, cudaStream_t stream);
template <typename T, typename Acc>
spmvb_status launch_spmm(spmvb_matrix A, int tile, int bucketed, int k,
                         const T* X, Acc* Y, cudaStream_t stream);
spmvb_status launch_merge_partition(spmvb_matrix A, cudaStream_t stream);

// Reads (stream-ordered, then synchronizes) and clears the context's device
// error word; SPMVB_ERR_TIMEOUT if a kernel's bounded wait gave up.
spmvb_status check_err_word(spmvb_context ctx, cudaStream_t s);

// Host-buffer outputs. A kernel that stores every y element exactly once
// with a plain store (all but the merge path, whose fix-up pass adds into y)
// can write y straight into the caller's host buffer when that buffer is
// pinned and mapped into the current device's address space: the PCIe
// writes then leave from the SMs as the rows finish, and no device-to-host
// copy follows the kernel. mapped_host_ptr returns the device address of
// such a buffer on the current device, or nullptr (pageable memory, device
// memory, or pinned memory this device cannot address).
inline bool stores_y_once(spmvb_kernel k) { return k != SPMVB_CSR_MERGE; }
void* mapped_host_ptr(const void* h);

// Power-iteration vector step (vecops.cu): *norm = the 2-norm of the m-entry
// global vector held in x's padded layout (slot = owner * max_rows + local,
// bounds on the device), in a fixed reduction order (partials:
// norm_blocks(m) doubles); then every slot of x is multiplied by 1 / *norm.
int norm_blocks(int64_t m);
spmvb_status launch_norm_and_scale(spmvb_dtype dtype, void* x, int64_t m, const int* bounds, int nranks,
                                   int max_rows, double* partials, double* norm, int sm_count, cudaStream_t s);

// Peer-memory exchange launchers (peer.cu).
spmvb_status peer_launch_ell(spmvb_matrix A, const PeerView& P, const void* x, cudaStream_t s);
spmvb_status peer_launch_push(spmvb_dtype dtype, const void* y, const PeerView& P, int sm_count, cudaStream_t s);
spmvb_status peer_launch_barrier(const PeerView& P, cudaStream_t s);

}  // namespace spmvb
