// Trivially copyable device views of every storage format the kernels read.
// They are the kernel arguments; the owning buffers live in the matrix handle
// (matrix.hpp). Mirrors the role of DeviceCsr/DeviceEll/DeviceBcsr
// (include/spmvbench/spmv_cuda.cuh:53-84), plus the hybrid, merge-path and
// bucket views that have no reference counterpart.
#pragma once

#include <cstdint>

namespace spmvb {

// CSR. colind/values are padded with kPad zero entries past nnz so that
// 16-byte vector loads that round a range up to a multiple of 4 entries stay
// in bounds (padding column 0 is a valid index into x).
constexpr int kPad = 64;

struct CsrView {
  const int* rowptr = nullptr;  // m + 1
  const int* colind = nullptr;  // nnz + kPad
  const void* values = nullptr; // nnz + kPad
  int m = 0;
  int n = 0;
  int64_t nnz = 0;
};

// Column-major ELL: entry j of row i at j * ld + i. ld == m reproduces the
// reference layout (src/formats.cpp:37-39).
struct EllView {
  const int* colind = nullptr;
  const void* values = nullptr;
  const int* row_lengths = nullptr;  // m
  int m = 0;
  int n = 0;
  int width = 0;
  int64_t ld = 0;
};

// Hybrid ELL(K) + CSR. Rows with len <= K keep their entries in the
// column-major ELL part (row_lengths = len); rows longer than K ("long rows",
// row_lengths = -1) are stored whole, back to back, in a CSR part indexed by
// long-row slot. The CSR part is cut into chunks of at most kHybChunk
// entries: a "packed" chunk holds whole rows (consecutive slots
// chunk_row[c] .. chunk_row[c+1]-1); a row longer than kHybChunk is cut into
// "segment" chunks of kHybChunk entries (its last one shorter), one per
// chunk. chunk_start[c] is the chunk's first entry (chunk_start[n_chunks] =
// tail_nnz). Segments leave a partial each (partial[c]); chunk_split[c] names
// the cut row's index s among split_rows (-1 for packed chunks), split_first
// [s] its first chunk, split_count[s] counts the partials written (0 between
// launches). With K = 0 the empty rows are listed in empty_rows. One launch:
// ell_blocks blocks of ELL rows, chunk_blocks blocks of chunks, then the
// empty rows.
constexpr int kHybChunk = 256;

struct HybView {
  EllView ell;                      // width K
  const int* long_rows = nullptr;   // n_long row ids, ascending
  const int64_t* tail_ptr = nullptr;  // n_long + 1 offsets into the CSR part
  const int* tail_colind = nullptr;   // + kPad
  const void* tail_values = nullptr;
  const int64_t* chunk_start = nullptr;  // n_chunks + 1
  const int* chunk_row = nullptr;        // n_chunks + 1
  const int* chunk_split = nullptr;      // n_chunks
  const int* split_rows = nullptr;       // n_split
  const int* split_first = nullptr;      // n_split
  int* split_count = nullptr;            // n_split
  const int* empty_rows = nullptr;       // n_empty (K = 0 only)
  void* partial = nullptr;               // n_chunks, of the accumulator type
  int64_t tail_nnz = 0;
  int n_long = 0;
  int n_chunks = 0;
  int n_split = 0;
  int n_empty = 0;
  int ell_blocks = 0;
  int chunk_blocks = 0;
};

// Blocked CSR with R x C row-major blocks (src/formats.cpp:45-105 layout).
struct BcsrView {
  const int* rowptr = nullptr;  // mb + 1
  const int* colind = nullptr;  // block_nnz
  const void* values = nullptr; // block_nnz * R * C
  int m = 0;
  int n = 0;
  int R = 4;
  int C = 4;
  int mb = 0;
  int64_t block_nnz = 0;
};

// Merge-path decomposition of the (m row ends) x (nnz entries) merge grid into
// tiles of `tile_items` consecutive diagonals. tile_row[t] is the row
// coordinate where tile t starts (tile_nz[t] = t*tile_items - tile_row[t]).
// carry_row / carry_val are per-launch scratch: the partial sum a tile leaves
// for a row that continues into the next tile (carry_row = -1: none).
struct MergeView {
  const int* tile_row = nullptr;  // num_tiles + 1
  int* carry_row = nullptr;       // num_tiles
  void* carry_val = nullptr;      // num_tiles, of the accumulator type
  int64_t num_items = 0;          // m + nnz
  int num_tiles = 0;
  int tile_items = 0;
};

// Row-length buckets for SpMM (reference thresholds, src/cuda/spmm_cuda.cu:249-256):
// rows[0, n_short) have <= 8 entries, the next n_med <= 64, the rest more.
struct BucketView {
  const int* rows = nullptr;
  int n_short = 0;
  int n_med = 0;
  int n_long = 0;
};

// Peer-memory exchange of one step of row-sharded iterated SpMV (at most
// kMaxRanks ranks, one GPU each). Rank `rank` writes its `rows` results into
// every rank's next x buffer (dst[p] already points at this rank's slice of
// rank p's buffer; dst[rank] is its own). Phase counters: flags_in[q] is the
// number of operations rank q has finished, written by rank q through
// flag_out[...] of its own view; *phase is this rank's own count, kept on the
// device so that a captured graph of steps can be replayed. The operation's
// last CTA increments *phase, writes it to every other rank's counter for
// this rank once all of the operation's stores are visible, then waits until
// all of this rank's counters reach it.
constexpr int kMaxRanks = 8;

struct PeerView {
  void* dst[kMaxRanks] = {};
  unsigned long long* flag_out[kMaxRanks] = {};  // &rank p's flags_in[this rank]
  const unsigned long long* flags_in = nullptr;  // nranks counters
  unsigned int* counter = nullptr;               // finished CTAs; 0 between launches
  int* err = nullptr;                            // context error word
  unsigned long long* phase = nullptr;
  unsigned long long timeout_ns = 0;
  int nranks = 1;
  int rank = 0;
  int rows = 0;
  int cta_fence = 0;  // every CTA fences its own stores before arriving
};

}  // namespace spmvb
