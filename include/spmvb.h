/*
 * spmvb.h - C ABI of the B200 (sm_100a) sparse kernel library.
 *
 * This is the drop-in boundary for SpMVBench's `src/cuda` path. Every entry
 * point takes plain pointers and sizes and returns a status code instead of
 * aborting. The comment above each declaration names the reference interface
 * it replaces (paths relative to the SpMVBench source tree).
 *
 * Conventions
 *  - Index type is int32 (reference `Index`, include/spmvbench/dtypes.hpp:19).
 *  - Value type `dtype` is the storage type T of the matrix and of x / X;
 *    `acc` is the accumulator / output type Acc of y / Y. Supported (T, Acc):
 *    (F32, F32), (F32, F64), (F64, F64) - the instantiations of
 *    src/cuda/spmv_cuda.cu:503-505.
 *  - Pointers named d_* are device pointers, h_* host pointers.
 *  - `stream` is a cudaStream_t passed as void*; NULL is the legacy default
 *    stream, as in the reference.
 *  - A matrix handle may be used by one stream at a time (its lazily built
 *    formats and its merge-path carry buffer are per handle).
 *  - spmvb_last_error() returns a thread-local message for the last failing
 *    call made on this host thread.
 */
#ifndef SPMVB_H
#define SPMVB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SPMVB_ABI_VERSION 1

typedef enum spmvb_status {
  SPMVB_OK = 0,
  SPMVB_ERR_INVALID_ARGUMENT = 1, /* bad pointer, size, kernel id, dtype  */
  SPMVB_ERR_INVALID_MATRIX = 2,   /* rowptr/colind fail validation         */
  SPMVB_ERR_UNSUPPORTED = 3,      /* valid request this build cannot serve */
  SPMVB_ERR_OUT_OF_MEMORY = 4,    /* device or host allocation failed      */
  SPMVB_ERR_CUDA = 5,             /* CUDA runtime error (message attached) */
  SPMVB_ERR_NCCL = 6,             /* NCCL error (message attached)         */
  SPMVB_ERR_TIMEOUT = 7,          /* a bounded wait gave up                */
  SPMVB_ERR_NO_DEVICE = 8,        /* no CUDA device / bad device ordinal   */
  SPMVB_ERR_IO = 9                /* a file cannot be opened, read, written */
} spmvb_status;

typedef enum spmvb_dtype { SPMVB_F32 = 0, SPMVB_F64 = 1 } spmvb_dtype;

/* SpMV kernels. 0..5 keep the numeric values of the reference's KernelId
 * (include/spmvbench/select.hpp:11-19); SPMVB_HYB is new (hybrid ELL+CSR). */
typedef enum spmvb_kernel {
  SPMVB_CSR_SCALAR = 0, /* one row per thread, csr_omp summation order      */
  SPMVB_CSR_VECTOR = 1, /* `lanes` lanes per row (2,4,8,16,32)               */
  SPMVB_CSR_WARP = 2,   /* one warp per row                                  */
  SPMVB_CSR_MERGE = 3,  /* merge-path: equal (rows + nnz) share per thread   */
  SPMVB_ELL = 4,        /* column-major ELL, walks row_lengths               */
  SPMVB_BCSR = 5,       /* blocked CSR, `block` = 2 (2x2) or 4 (4x4)         */
  SPMVB_HYB = 6,        /* rows of <= K entries in ELL(K), longer rows whole
                           in CSR streamed in chunks of <= 256 entries        */
  SPMVB_KERNEL_COUNT = 7
} spmvb_kernel;

typedef struct spmvb_context_st* spmvb_context;
typedef struct spmvb_matrix_st* spmvb_matrix;
typedef struct spmvb_dist_st* spmvb_dist;

/* Device description. Replaces GpuInfo / query_gpu()
 * (include/spmvbench/spmv_cuda.cuh:101-111, src/cuda/spmv_cuda.cu:197-228);
 * peak_gbs is the theoretical HBM figure (2 x memory clock x bus width). */
typedef struct spmvb_gpu_info {
  char name[256];
  int major;
  int minor;
  int sm_count;
  int l2_bytes;
  int max_smem_per_block;
  int64_t global_mem_bytes;
  double peak_gbs;
  int peak_known;
} spmvb_gpu_info;

/* Storage sizes of the formats a matrix handle holds. Replaces
 * SpmvRunner::ell_padded_nnz / ell_touched_nnz / bcsr_block_nnz
 * (include/spmvbench/spmv_cuda.cuh:137-140). -1 = not built yet. */
typedef struct spmvb_matrix_info {
  int32_t m;
  int32_t n;
  int64_t nnz;
  spmvb_dtype dtype;
  int32_t max_row_nnz;
  int64_t ell_padded_nnz;  /* m * max_row_nnz                               */
  int64_t ell_touched_nnz; /* entries the ELL kernel reads (= nnz)           */
  int64_t bcsr2_block_nnz;
  int64_t bcsr4_block_nnz;
  int32_t hyb_width;       /* K of the hybrid format                        */
  int64_t hyb_ell_nnz;     /* entries held in the ELL(K) part               */
  int64_t hyb_tail_nnz;    /* entries held in the CSR tail                  */
  int32_t hyb_long_rows;   /* rows whose length exceeds K                   */
  int64_t device_bytes;    /* device memory owned by the handle             */
} spmvb_matrix_info;

/* Row statistics. Same fields and definitions as RowStats
 * (include/spmvbench/stats.hpp:14-40, src/stats.cpp:13-123). */
typedef struct spmvb_row_stats {
  int64_t nnz;
  int32_t rows;
  int32_t cols;
  double mean_row_nnz;
  double median_row_nnz;
  int32_t min_row_nnz;
  int32_t max_row_nnz;
  double stddev_row_nnz;
  double cv_row_nnz;
  double max_over_mean;
  double ell_padding_overhead;
  double frac_dense_blocks_4x4;
  double density;
  /* Not in the reference: dense 4x4 blocks (> 8 entries) over the 4x4
   * blocks that hold at least one entry. frac_dense_blocks_4x4 divides by
   * every possible block (mb*nb), so it stays near 0 for any large sparse
   * matrix, however blocky. */
  double dense_share_of_stored_4x4;
} spmvb_row_stats;

/* Kernel choice. Same fields as KernelChoice (include/spmvbench/select.hpp:21-27). */
typedef struct spmvb_choice {
  int32_t kernel; /* spmvb_kernel */
  int32_t lanes;
  int32_t block_r;
  int32_t block_c;
  int32_t rule;   /* index of the rule that fired                           */
  char reason[256];
} spmvb_choice;

/* ---- library / device -------------------------------------------------- */
const char* spmvb_version(void);
const char* spmvb_last_error(void);
const char* spmvb_status_string(spmvb_status s);
/* Kernel launches issued by this library since load (all devices). No
 * reference counterpart (the bench reports it as its launch count). */
uint64_t spmvb_launch_count(void);

/* Replaces gpu_available() (include/spmvbench/spmv_cuda.cuh:110): never aborts. */
int spmvb_gpu_available(void);
/* Replaces query_gpu() (include/spmvbench/spmv_cuda.cuh:111). */
spmvb_status spmvb_query_gpu(int device, spmvb_gpu_info* out);

/* A context binds one device. Replaces the implicit current-device state the
 * reference's SpmvRunner relies on (src/cuda/spmv_cuda.cu:233-290). */
spmvb_status spmvb_context_create(int device, spmvb_context* out);
spmvb_status spmvb_context_destroy(spmvb_context ctx);
/* Synchronizes the device and reports whether any kernel launched through
 * this context gave up a bounded wait since the last check
 * (SPMVB_ERR_TIMEOUT; the word is then cleared). The host-buffer entry
 * points perform this check on their own stream before returning. */
spmvb_status spmvb_context_check(spmvb_context ctx);
/* Launches a kernel whose bounded wait can never be satisfied (an mbarrier
 * expecting bytes no copy delivers), with a short limit, to exercise the
 * failure path; expect SPMVB_ERR_TIMEOUT. Nothing is left in flight. */
spmvb_status spmvb_selftest_wait_timeout(spmvb_context ctx);

/* ---- matrices ------------------------------------------------------------ */
/* Validate a host CSR (rowptr[0]==0, non-decreasing, rowptr[m]==nnz, every
 * column in [0,n)) and upload it. Replaces SpmvRunner(const CsrMatrix<T>&)
 * and its upload_matrix (src/cuda/spmv_cuda.cu:233-290); other formats are
 * built lazily by spmvb_matrix_prepare or on first use. Columns inside a row
 * may be unsorted, as csr.hpp:13-15 allows. */
spmvb_status spmvb_matrix_create_csr(spmvb_context ctx, spmvb_dtype dtype,
                                     int32_t m, int32_t n, int64_t nnz,
                                     const int32_t* h_rowptr,
                                     const int32_t* h_colind,
                                     const void* h_values, spmvb_matrix* out);
spmvb_status spmvb_matrix_destroy(spmvb_matrix A);
/* The host-side validation spmvb_matrix_create_csr applies, on its own (no
 * device needed). *max_row_nnz (optional) receives the longest row. */
spmvb_status spmvb_csr_validate(int32_t m, int32_t n, int64_t nnz,
                                const int32_t* h_rowptr,
                                const int32_t* h_colind,
                                int32_t* max_row_nnz);
/* Build what `kernel` needs (ELL, HYB, BCSR `block`, merge-path partition)
 * ahead of the first call; kernel = -1 builds the SpMM row-length buckets.
 * Replaces the eager conversions and uploads of SpmvRunner's constructor
 * (src/cuda/spmv_cuda.cu:234-291), done here per format and on demand.
 * param: block size for SPMVB_BCSR, forced width K for SPMVB_HYB
 * (0 = automatic). Lazy builds synchronize the device, so call this before
 * capturing a stream into a CUDA graph. */
spmvb_status spmvb_matrix_prepare(spmvb_matrix A, spmvb_kernel kernel,
                                  int param);
/* Sizes of the formats built so far. Replaces SpmvRunner::ell_padded_nnz /
 * ell_touched_nnz / bcsr_block_nnz (include/spmvbench/spmv_cuda.cuh:137-140). */
spmvb_status spmvb_matrix_get_info(spmvb_matrix A, spmvb_matrix_info* out);

/* Download a device-built format in the reference host layout, for
 * bit-exact comparison with csr_to_ell (src/formats.cpp:14-43): colind and
 * values column-major, size m*max_row_nnz, padding column 0 / value 0. */
spmvb_status spmvb_matrix_export_ell(spmvb_matrix A, int32_t* h_colind,
                                     void* h_values, int32_t* h_row_lengths);
/* Same for csr_to_bcsr<T,R,C> (src/formats.cpp:45-105), R=C=block:
 * rowptr (mb+1), block colind (block_nnz), values (block_nnz*block*block). */
spmvb_status spmvb_matrix_export_bcsr(spmvb_matrix A, int block,
                                      int32_t* h_rowptr, int32_t* h_colind,
                                      void* h_values);

/* ---- SpMV ------------------------------------------------------------------ */
/* y = A x on device buffers. x has n entries of the matrix dtype, y has m
 * entries of `acc`. `lanes` applies to SPMVB_CSR_VECTOR, `block` to
 * SPMVB_BCSR, with the reference's defaults and clamping
 * (src/cuda/spmv_cuda.cu:392-458). Replaces the launch inside
 * SpmvRunner::run (src/cuda/spmv_cuda.cu:376-464). */
spmvb_status spmvb_spmv(spmvb_matrix A, spmvb_kernel kernel, int lanes,
                        int block, const void* d_x, void* d_y,
                        spmvb_dtype acc, void* stream);
/* Same on host buffers: H2D of x, the kernel and D2H of y in stream order,
 * synchronous on return. When h_y is pinned host memory mapped into the
 * device's address space (cudaHostAlloc / cudaMallocHost, or registered
 * memory, under unified addressing), every kernel but the merge path stores
 * y into it directly instead of through a device buffer and a copy.
 * Replaces set_x + run + result (include/spmvbench/spmv_cuda.cuh:127-135). */
spmvb_status spmvb_spmv_host(spmvb_matrix A, spmvb_kernel kernel, int lanes,
                             int block, const void* h_x, void* h_y,
                             spmvb_dtype acc, void* stream);

/* The measurement of SpmvRunner::run (src/cuda/spmv_cuda.cu:466-486):
 * `warmup` launches, a synchronize, then `iters` launches each between its
 * own pair of events on `stream`, each waited for. out_ms4 receives the
 * median, mean, min and max milliseconds (the reference's summarize,
 * include/spmvbench/timer.hpp). The launches and the timing run in C++, so
 * a caller from any language gets the reference's protocol. */
spmvb_status spmvb_spmv_time(spmvb_matrix A, spmvb_kernel kernel, int lanes,
                             int block, const void* d_x, void* d_y,
                             spmvb_dtype acc, int iters, int warmup,
                             void* stream, double* out_ms4);

/* Merge-path y = A x that allocates nothing. No counterpart in the reference.
 * For callers that cannot call cudaMalloc: device memory owned by another
 * allocator (a caching allocator or a pool sized at start-up), or latency
 * rules that forbid allocation after start-up (cudaMalloc/cudaFree may
 * synchronize the device). The caller owns every array on the device: a
 * valid CSR (rowptr m+1, colind/values nnz, as spmvb_csr_validate checks), x
 * (n entries of dtype) and y (m entries of acc); the current device is used.
 * Unlike spmvb_spmv it does not inspect the pointers (host memory, another
 * device's memory or a short array are not caught): only null pointers,
 * negative sizes and nnz > 0 with n == 0 are refused, so check an untrusted
 * CSR with spmvb_csr_validate first.
 * Scratch lives in a fixed 1,048,832-byte __device__ array held by every GPU
 * that loads the library until exit, which bounds m + nnz to 117,440,512
 * (65,536 merge tiles of 1,792 items); larger requests fail with
 * SPMVB_ERR_UNSUPPORTED. The first call on a device looks the array up
 * (cudaGetSymbolAddress), so make it before any stream capture. Calls share
 * the array: calls that overlap on the GPU race; calls ordered on one stream
 * do not. Each call writes all the scratch it reads, so nothing is cleared. */
spmvb_status spmvb_spmv_merge_noalloc(spmvb_dtype dtype, int32_t m, int32_t n,
                                      int64_t nnz, const int32_t* d_rowptr,
                                      const int32_t* d_colind,
                                      const void* d_values, const void* d_x,
                                      void* d_y, spmvb_dtype acc,
                                      void* stream);

/* ---- SpMM ------------------------------------------------------------------ */
/* Y (m x k, row-major, acc) = A X (n x k, row-major, matrix dtype).
 * tile in {16,32,64}: columns of Y a row group covers per pass; bucketed != 0
 * selects the row-length-bucketed variant (buckets built once per handle).
 * Replaces the kernels behind spmm_csr_tiled_f32/f64
 * (include/spmvbench/spmm_cuda.cuh:34-41, src/cuda/spmm_cuda.cu:151-212). */
spmvb_status spmvb_spmm(spmvb_matrix A, int tile, int bucketed, int k,
                        const void* d_X, void* d_Y, spmvb_dtype acc,
                        void* stream);
/* Column bands of the plain SpMM (tile 64, X 16-byte aligned, k a multiple
 * of 16 bytes / element size, every row's columns ascending): with bands > 1
 * the product is swept in `bands` passes, pass b adding each row's entries
 * whose column lies in the b-th band of n / bands columns, so the X rows a
 * pass gathers fit the L2. Each output element still receives its terms in
 * CSR order (bit-identical to the one-pass kernel); Y is read and written
 * once per pass. 0 = automatic (the default), 1 = one pass. No reference
 * counterpart (its tiled kernel re-reads X per row, src/cuda/spmm_cuda.cu:31-60). */
spmvb_status spmvb_matrix_set_spmm_bands(spmvb_matrix A, int bands);
/* Host-buffer form (H2D X, kernel, D2H Y). Replaces run_tiled's data path
 * (src/cuda/spmm_cuda.cu:214-325) without its per-call malloc/free. */
spmvb_status spmvb_spmm_host(spmvb_matrix A, int tile, int bucketed, int k,
                             const void* h_X, void* h_Y, spmvb_dtype acc,
                             void* stream);

/* Measures this device's random-gather ceiling: 8-byte loads at random
 * positions of an L2-resident vector of n doubles (`gathers` of them, in
 * one launch, best of 6 after 2 warm-up launches). SpMV on matrices whose
 * column indices have no locality is bounded by this rate, not by HBM
 * bandwidth. No reference counterpart (its roofline is HBM only). */
spmvb_status spmvb_probe_gather_rate(spmvb_context ctx, int64_t n,
                                     int64_t gathers, double* gathers_per_s);

/* ---- statistics and kernel selection ---------------------------------------- */
/* Replaces compute_row_stats (include/spmvbench/stats.hpp:44-52). histogram
 * (optional) receives max_row_nnz+1 counts when hist_cap is large enough;
 * the dense-block scan is hashed, O(nnz) instead of O(L^2) per block row. */
spmvb_status spmvb_compute_row_stats(const int32_t* h_rowptr, const int32_t* h_colind,
                             int32_t m, int32_t n, int64_t nnz,
                             spmvb_row_stats* out, int64_t* h_histogram,
                             int64_t hist_cap);
/* The same statistics, bit for bit, of a matrix already on the device: the
 * 4x4 block census (the O(nnz) part, src/stats.cpp:85-118 in the reference,
 * O(L^2) per block row there) runs on the GPU as one radix sort of block
 * keys; lengths, median and variance come from the handle's host rowptr in
 * the reference's order. Replaces compute_row_stats for uploaded matrices. */
spmvb_status spmvb_matrix_row_stats(spmvb_matrix A, spmvb_row_stats* out,
                                    int64_t* h_histogram, int64_t hist_cap);
/* Replaces choose_spmv (include/spmvbench/select.hpp:33) with rules
 * calibrated on B200 measurements. */
spmvb_status spmvb_choose_spmv(const spmvb_row_stats* stats,
                               spmvb_choice* out);
/* The reference's own rule set, unchanged (src/select.cpp:93-165). */
spmvb_status spmvb_choose_spmv_reference(const spmvb_row_stats* stats,
                                         spmvb_choice* out);
/* Replaces kernel_name (src/select.cpp:73-91); adds "hyb". */
const char* spmvb_kernel_name(int kernel);

/* ---- synthetic inputs ------------------------------------------------------ */
/* Seeded generators for the five benchmark matrices (no reference
 * counterpart; the reference reads .mtx files). `which`: 1 banded 100k hb=4,
 * 2 uniform 1M x 16, 3 power-law Zipf(2.1) <= 50,000, 4 dense-4x4-block 500k,
 * 5 = 2 (the SpMM operand). `scale_rows` (0 = full size) shrinks m for tests.
 * Two calls: with h_colind == NULL the sizes are returned in *m,*n,*nnz;
 * then the caller allocates and calls again. Values are f64. */
spmvb_status spmvb_generate(int which, uint64_t seed, int32_t scale_rows,
                            int32_t* m, int32_t* n, int64_t* nnz,
                            int32_t* h_rowptr, int32_t* h_colind,
                            double* h_values);
/* x_i ~ U(-1,1) from a seeded 64-bit generator, shared by oracle and GPU. */
spmvb_status spmvb_generate_vector(uint64_t seed, int64_t len, double* h_out);

/* ---- streamed SpMV over host buffers ------------------------------------------- */
/* No reference counterpart (SpmvRunner copies x in, runs and copies y out
 * synchronously, src/cuda/spmv_cuda.cu:292-330,476-498). A pipeline keeps
 * up to `depth` (1..16) host-buffer SpMVs in flight, each on its own stream
 * and device staging, so with pinned host buffers one call's copy of x in,
 * another's kernel and a third's output overlap. y is written by the kernel
 * straight into a pinned, mapped h_y (all kernels but the merge path), else
 * staged on the device and copied out. */
typedef struct spmvb_pipeline_st* spmvb_pipeline;
spmvb_status spmvb_pipeline_create(spmvb_matrix A, int depth,
                                   spmvb_pipeline* out);
/* Later submissions start after the work already enqueued on `stream`. */
spmvb_status spmvb_pipeline_fork(spmvb_pipeline P, void* stream);
/* Enqueues y = A x (host x: n entries, host y: m entries of `acc`) on the
 * next slot and returns. h_x must stay unchanged and h_y must not be read
 * until the call is waited for (spmvb_pipeline_wait, or work joined onto a
 * stream); a slot's staging is reused only after its previous call ends. */
spmvb_status spmvb_pipeline_submit(spmvb_pipeline P, spmvb_kernel kernel,
                                   int lanes, int block, const void* h_x,
                                   void* h_y, spmvb_dtype acc);
/* `stream` waits for every call submitted so far. */
spmvb_status spmvb_pipeline_join(spmvb_pipeline P, void* stream);
/* Waits for every call submitted so far; reports a kernel's bounded-wait
 * failure like the other host entry points. */
spmvb_status spmvb_pipeline_wait(spmvb_pipeline P);
spmvb_status spmvb_pipeline_destroy(spmvb_pipeline P);

/* ---- input formats ------------------------------------------------------------- */
/* Host CSR read from a file (f64 values; a caller wanting f32 converts with
 * round-to-nearest, as the reference's static_cast<float> does). */
typedef struct spmvb_host_csr_st* spmvb_host_csr;
/* Replaces read_matrix_market<T> (src/mtx_io.cpp:40-172, declared in
 * include/spmvbench/mtx_io.hpp): coordinate real / integer / pattern,
 * general / symmetric; the same CSR (rows sorted by column with the
 * reference's sort, so repeated entries keep its order) and the same error
 * texts ("Matrix Market: <path>: ..."; SPMVB_ERR_IO when the file cannot be
 * opened, SPMVB_ERR_INVALID_MATRIX for a malformed file). The entry lines are
 * parsed by `threads` threads (0 = all hardware threads). */
spmvb_status spmvb_read_matrix_market(const char* path, int threads,
                                      spmvb_host_csr* out);
/* Binary CSR cache (no reference counterpart): a 40-byte header ("SPMVBCSR",
 * version 1, value bytes 8, m, n, nnz) then rowptr, colind, f64 values. The
 * CSR is validated on write and on read. */
spmvb_status spmvb_csr_cache_write(const char* path, int32_t m, int32_t n,
                                   int64_t nnz, const int32_t* h_rowptr,
                                   const int32_t* h_colind,
                                   const double* h_values);
spmvb_status spmvb_csr_cache_read(const char* path, spmvb_host_csr* out);
/* Sizes and pointers into the handle's arrays (valid until it is freed). */
spmvb_status spmvb_host_csr_get(spmvb_host_csr A, int32_t* m, int32_t* n,
                                int64_t* nnz, const int32_t** rowptr,
                                const int32_t** colind, const double** values);
void spmvb_host_csr_free(spmvb_host_csr A);

/* ---- multi-GPU row sharding ---------------------------------------------------- */
/* No reference counterpart: SpMVBench runs on one GPU. These entry points add
 * the row-sharded multi-GPU SpMV (one process per GPU) and its x exchange. */
/* nnz-balanced contiguous row blocks: bounds[g] = lower_bound(rowptr,
 * ceil(g*nnz/parts)) for g in 1..parts-1, bounds[0]=0, bounds[parts]=m. */
spmvb_status spmvb_partition_rows(const int32_t* h_rowptr, int32_t m,
                                  int32_t parts, int32_t* h_bounds);
/* Host-only shard planning used by spmvb_dist_create: rank `rank`'s rows
 * [bounds[rank], bounds[rank+1]) of a square m x m CSR with every column c
 * renumbered to its padded gather slot owner(c)*max_rows + (c -
 * bounds[owner(c)]), max_rows = the largest part. With h_out_colind == NULL
 * only *max_rows and *local_nnz are returned. h_out_rowptr has
 * local_rows+1 entries. */
spmvb_status spmvb_shard_csr(int32_t m, const int32_t* h_rowptr,
                             const int32_t* h_colind, int nranks, int rank,
                             const int32_t* h_bounds, int32_t* max_rows,
                             int64_t* local_nnz, int32_t* h_out_rowptr,
                             int32_t* h_out_colind);
/* NCCL unique id (NCCL_UNIQUE_ID_BYTES = 128) created on one rank and
 * broadcast by the caller. */
spmvb_status spmvb_nccl_unique_id(void* h_out, size_t cap);
/* One rank's shard of a square row-partitioned matrix for iterated y = A x
 * with x <- y. The caller passes the global rowptr/colind/values (host) and
 * the bounds from spmvb_partition_rows; the shard's columns are renumbered
 * into the padded gather layout once (slot = owner*max_rows + local). */
spmvb_status spmvb_dist_create(spmvb_context ctx, int nranks, int rank,
                               const void* h_unique_id, spmvb_dtype dtype,
                               int32_t m, int64_t nnz,
                               const int32_t* h_rowptr,
                               const int32_t* h_colind, const void* h_values,
                               const int32_t* h_bounds, spmvb_dist* out);
spmvb_status spmvb_dist_destroy(spmvb_dist D);
/* Load the global x (host, m entries) into this rank's padded x buffer. */
spmvb_status spmvb_dist_set_x(spmvb_dist D, const void* h_x, void* stream);
/* `iters` steps of: y_local = A_local x (kernel), then the exchange of the
 * padded y slices into x (ncclAllGather, or the peer exchange below). The
 * final x (global, m entries) can be read back with spmvb_dist_get_x. */
spmvb_status spmvb_dist_iterate(spmvb_dist D, spmvb_kernel kernel, int lanes,
                                int iters, void* stream);
/* Same, with the steps enqueued back to back and timed on device events:
 * *step_ms = milliseconds from the first step's start to the last step's
 * end; *kernel_ms = the SpMV part of each step (for the fused peer ELL step,
 * the whole step), summed over the steps. */
spmvb_status spmvb_dist_iterate_timed(spmvb_dist D, spmvb_kernel kernel,
                                      int lanes, int iters, void* stream,
                                      double* kernel_ms, double* step_ms);
spmvb_status spmvb_dist_get_x(spmvb_dist D, void* h_x, void* stream);
/* Power iteration on the row-sharded matrix: `iters` steps of
 *   x <- A x (kernel, then the exchange of the slices), lambda = ||x||_2,
 *   x <- x / lambda,
 * with the norm taken by every rank over the whole vector it now holds, in a
 * fixed order that does not depend on the number of ranks (so every rank,
 * and a one-rank run, gets the same bits when the kernel keeps csr_omp's
 * order). *h_lambda receives the last step's norm (an estimate of the
 * dominant eigenvalue's magnitude); synchronizes. Collective, like
 * spmvb_dist_iterate; works on either exchange. No reference counterpart
 * (the reference has no solver loop). */
spmvb_status spmvb_dist_power_iterate(spmvb_dist D, spmvb_kernel kernel,
                                      int lanes, int iters, double* h_lambda,
                                      void* stream);

/* Exchange of x slices between the steps of spmvb_dist_iterate. */
typedef enum {
  SPMVB_EXCHANGE_NCCL = 0, /* SpMV, then ncclAllGather (default) */
  SPMVB_EXCHANGE_PEER = 1  /* SpMV stores each slice into every rank's x */
} spmvb_exchange;
/* Collective (every rank calls it): switch to the peer exchange. Each rank
 * maps the other ranks' double-buffered x and phase counters through CUDA
 * IPC; a step then runs the SpMV, stores its slice straight into every
 * rank's next x over NVLink and ends in a barrier (its last CTA publishes
 * this rank's phase and waits for every other rank's): one kernel for
 * SPMVB_ELL, the SpMV plus a copy kernel for the others. With one rank the
 * SpMV writes the next x itself. No NCCL call is on the data path.
 * Needs one GPU per rank and at most 8 ranks; otherwise every rank gets
 * SPMVB_ERR_UNSUPPORTED and stays on ncclAllGather. Waits give up after
 * SPMVB_PEER_TIMEOUT_MS (environment, default 10000) with
 * SPMVB_ERR_TIMEOUT, after which the handle only accepts destroy. Until
 * destroy, every rank must make the same sequence of set_x / iterate /
 * get_x calls. No reference counterpart. */
spmvb_status spmvb_dist_enable_peer(spmvb_dist D, void* stream);
/* SPMVB_EXCHANGE_NCCL or SPMVB_EXCHANGE_PEER. */
int spmvb_dist_exchange(spmvb_dist D);
spmvb_status spmvb_dist_get_info(spmvb_dist D, int32_t* row_begin,
                                 int32_t* row_end, int32_t* max_rows,
                                 int64_t* local_nnz);

/* Single product y = A x over host buffers, row-sharded: each rank passes its
 * own rows' slice of x (rows bounds[rank]..bounds[rank+1]-1, host) and gets
 * its rows of y (host). The slices are all-gathered on the devices over
 * NVLink (ncclAllGather), so each entry of x crosses PCIe once per job, not
 * once per GPU. Up to `depth` calls in flight, as in spmvb_pipeline; keep x
 * unchanged and y unread until the call is waited for. Collective: every
 * rank submits the same sequence of calls. Pinned, mapped y is written by
 * the kernel directly (every kernel but the merge path). Runs on the NCCL
 * exchange (not after spmvb_dist_enable_peer). Destroying the dist handle
 * first waits for the pipeline's calls; the pipeline's later calls then fail
 * and only its destroy remains valid. No reference counterpart (the reference's
 * SpmvRunner copies the whole x to its one GPU,
 * src/cuda/spmv_cuda.cu:292-330). */
typedef struct spmvb_dist_pipeline_st* spmvb_dist_pipeline;
spmvb_status spmvb_dist_pipeline_create(spmvb_dist D, int depth,
                                        spmvb_dist_pipeline* out);
spmvb_status spmvb_dist_pipeline_fork(spmvb_dist_pipeline P, void* stream);
spmvb_status spmvb_dist_pipeline_submit(spmvb_dist_pipeline P,
                                        spmvb_kernel kernel, int lanes,
                                        const void* h_x_local, void* h_y_local);
spmvb_status spmvb_dist_pipeline_join(spmvb_dist_pipeline P, void* stream);
spmvb_status spmvb_dist_pipeline_wait(spmvb_dist_pipeline P);
spmvb_status spmvb_dist_pipeline_destroy(spmvb_dist_pipeline P);

#ifdef __cplusplus
}
#endif

#endif /* SPMVB_H */
