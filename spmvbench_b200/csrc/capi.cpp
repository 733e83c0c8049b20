// C ABI implementation: contexts, matrix handles, dispatch to the per-(T, Acc)
// launchers, host-buffer entry points and format export.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "internal.hpp"

namespace spmvb {

std::atomic<uint64_t> g_launches{0};

static thread_local std::string t_last_error;

spmvb_status fail(spmvb_status s, const std::string& msg) {
  t_last_error = msg;
  return s;
}

spmvb_status cuda_fail(cudaError_t e, const char* what) {
  const spmvb_status s = (e == cudaErrorMemoryAllocation) ? SPMVB_ERR_OUT_OF_MEMORY
                         : (e == cudaErrorNoDevice || e == cudaErrorInvalidDevice || e == cudaErrorInsufficientDriver)
                             ? SPMVB_ERR_NO_DEVICE
                             : SPMVB_ERR_CUDA;
  return fail(s, std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

void clear_error() { t_last_error.clear(); }

spmvb_status DevBuf::alloc(size_t bytes) {
  reset();
  if (bytes == 0) bytes = 16;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_fail(e, "cudaMalloc");
  }
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "cudaMemset");
  }
  p_ = p;
  bytes_ = bytes;
  return SPMVB_OK;
}

void DevBuf::reset() {
  if (p_) cudaFree(p_);
  p_ = nullptr;
  bytes_ = 0;
}

spmvb_status upload(DevBuf& dst, const void* src, size_t bytes, size_t cap) {
  SPMVB_TRY(dst.alloc(std::max(bytes, cap)));
  if (bytes) SPMVB_TRY_CUDA(cudaMemcpy(dst.get(), src, bytes, cudaMemcpyHostToDevice));
  return SPMVB_OK;
}

// Device-pointer check through the driver's address-range query (fetched by
// the runtime, so the library has no link-time dependency on libcuda): the
// pointer must be device-accessible from `device` and its allocation must
// hold `bytes` from the pointer on. A host pointer or an undersized buffer is
// rejected before any kernel can touch it.
using AddrRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
static AddrRangeFn addr_range_fn() {
  static AddrRangeFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<AddrRangeFn>(f);
  }();
  return fn;
}

static spmvb_status check_device_ptr(const void* p, size_t bytes, int device, const char* name) {
  if (bytes == 0) return SPMVB_OK;
  if (!p) return fail(SPMVB_ERR_INVALID_ARGUMENT, std::string(name) + " is null");
  cudaPointerAttributes at{};
  cudaError_t e = cudaPointerGetAttributes(&at, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(SPMVB_ERR_INVALID_ARGUMENT, std::string(name) + " is not a CUDA pointer");
  }
  if (at.type == cudaMemoryTypeUnregistered || (at.type == cudaMemoryTypeHost && at.devicePointer == nullptr))
    return fail(SPMVB_ERR_INVALID_ARGUMENT, std::string(name) + " is host memory; pass a device pointer");
  if (at.type == cudaMemoryTypeDevice && at.device != device)
    return fail(SPMVB_ERR_INVALID_ARGUMENT, std::string(name) + " lives on another device");
  if (at.type == cudaMemoryTypeDevice) {
    if (AddrRangeFn fn = addr_range_fn()) {
      CUdeviceptr base = 0;
      size_t size = 0;
      if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(p)) == CUDA_SUCCESS) {
        const size_t avail = static_cast<size_t>(base + size - reinterpret_cast<CUdeviceptr>(p));
        if (avail < bytes) {
          char msg[200];
          std::snprintf(msg, sizeof(msg), "%s holds %zu bytes past the pointer, %zu needed", name, avail, bytes);
          return fail(SPMVB_ERR_INVALID_ARGUMENT, msg);
        }
      }
    }
  }
  return SPMVB_OK;
}

}  // namespace spmvb

using namespace spmvb;

int64_t spmvb_matrix_st::device_bytes() const {
  int64_t b = rowptr.bytes() + colind.bytes() + values.bytes();
  b += ell_colind.bytes() + ell_values.bytes() + ell_rowlen.bytes();
  b += hyb_colind.bytes() + hyb_values.bytes() + hyb_rowlen.bytes() + hyb_long_rows.bytes() +
       hyb_tail_ptr.bytes() + hyb_tail_colind.bytes() + hyb_tail_values.bytes() + hyb_chunk_start.bytes() +
       hyb_chunk_row.bytes() + hyb_chunk_split.bytes() + hyb_split_rows.bytes() + hyb_split_first.bytes() +
       hyb_split_count.bytes() + hyb_empty_rows.bytes() + hyb_partial.bytes();
  for (const auto* B : {&bcsr2, &bcsr4}) b += B->rowptr.bytes() + B->colind.bytes() + B->values.bytes();
  b += merge_tile_row.bytes() + merge_carry_row.bytes() + merge_carry_val.bytes();
  b += bucket_rows.bytes() + stage_in.bytes() + stage_out.bytes();
  return b;
}

extern "C" {

const char* spmvb_version(void) { return "spmvb 0.1.0 (sm_100a)"; }
const char* spmvb_last_error(void) { return t_last_error.c_str(); }
uint64_t spmvb_launch_count(void) { return g_launches.load(); }

const char* spmvb_status_string(spmvb_status s) {
  switch (s) {
    case SPMVB_OK: return "ok";
    case SPMVB_ERR_INVALID_ARGUMENT: return "invalid argument";
    case SPMVB_ERR_INVALID_MATRIX: return "invalid matrix";
    case SPMVB_ERR_UNSUPPORTED: return "unsupported";
    case SPMVB_ERR_OUT_OF_MEMORY: return "out of memory";
    case SPMVB_ERR_CUDA: return "CUDA error";
    case SPMVB_ERR_NCCL: return "NCCL error";
    case SPMVB_ERR_TIMEOUT: return "timeout";
    case SPMVB_ERR_NO_DEVICE: return "no device";
    case SPMVB_ERR_IO: return "i/o error";
  }
  return "unknown status";
}

int spmvb_gpu_available(void) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return count > 0;
}

spmvb_status spmvb_query_gpu(int device, spmvb_gpu_info* out) {
  clear_error();
  if (!out) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null output");
  if (!spmvb_gpu_available()) return fail(SPMVB_ERR_NO_DEVICE, "no CUDA device");
  cudaDeviceProp prop{};
  SPMVB_TRY_CUDA(cudaGetDeviceProperties(&prop, device));
  std::memset(out, 0, sizeof(*out));
  std::snprintf(out->name, sizeof(out->name), "%s", prop.name);
  out->major = prop.major;
  out->minor = prop.minor;
  out->sm_count = prop.multiProcessorCount;
  out->l2_bytes = prop.l2CacheSize;
  out->max_smem_per_block = static_cast<int>(prop.sharedMemPerBlockOptin);
  out->global_mem_bytes = static_cast<int64_t>(prop.totalGlobalMem);
  int mem_khz = 0, bus_bits = 0;
  if (cudaDeviceGetAttribute(&mem_khz, cudaDevAttrMemoryClockRate, device) == cudaSuccess &&
      cudaDeviceGetAttribute(&bus_bits, cudaDevAttrGlobalMemoryBusWidth, device) == cudaSuccess &&
      mem_khz > 0 && bus_bits > 0) {
    out->peak_gbs = 2.0 * mem_khz * 1e3 * (bus_bits / 8.0) / 1e9;
    out->peak_known = 1;
  }
  cudaGetLastError();
  return SPMVB_OK;
}

spmvb_status spmvb_context_create(int device, spmvb_context* out) {
  clear_error();
  if (!out) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null output");
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    cudaGetLastError();
    return fail(SPMVB_ERR_NO_DEVICE, "no CUDA device");
  }
  if (device < 0 || device >= count) return fail(SPMVB_ERR_NO_DEVICE, "device ordinal out of range");
  auto c = std::make_unique<spmvb_context_st>();
  c->device = device;
  DeviceGuard g(device);
  SPMVB_TRY_CUDA(cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, device));
  SPMVB_TRY_CUDA(cudaDeviceGetAttribute(&c->l2_bytes, cudaDevAttrL2CacheSize, device));
  SPMVB_TRY_CUDA(cudaDeviceGetAttribute(&c->max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
  SPMVB_TRY(c->err.alloc(16));
  *out = c.release();
  return SPMVB_OK;
}

spmvb_status spmvb_context_destroy(spmvb_context ctx) {
  clear_error();
  if (ctx) {
    DeviceGuard g(ctx->device);
    delete ctx;
  }
  return SPMVB_OK;
}

spmvb_status spmvb_context_check(spmvb_context ctx) {
  clear_error();
  if (!ctx) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null context");
  DeviceGuard g(ctx->device);
  SPMVB_TRY_CUDA(cudaDeviceSynchronize());
  int code = 0;
  SPMVB_TRY_CUDA(cudaMemcpy(&code, ctx->err.get(), sizeof(int), cudaMemcpyDeviceToHost));
  if (code != 0) {
    SPMVB_TRY_CUDA(cudaMemset(ctx->err.get(), 0, sizeof(int)));
    return fail(SPMVB_ERR_TIMEOUT, "a kernel's bounded wait gave up (device error code " + std::to_string(code) + ")");
  }
  return SPMVB_OK;
}

spmvb_status spmvb_matrix_create_csr(spmvb_context ctx, spmvb_dtype dtype, int32_t m, int32_t n,
                                     int64_t nnz, const int32_t* h_rowptr, const int32_t* h_colind,
                                     const void* h_values, spmvb_matrix* out) {
  clear_error();
  if (!ctx || !out) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null context or output");
  if (dtype != SPMVB_F32 && dtype != SPMVB_F64) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bad dtype");
  int max_row = 0;
  SPMVB_TRY(spmvb_csr_validate(m, n, nnz, h_rowptr, h_colind, &max_row));
  if (nnz > 0 && !h_values) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null values");
  DeviceGuard g(ctx->device);
  auto* A = new spmvb_matrix_st;
  A->ctx = ctx;
  A->device = ctx->device;
  A->dtype = dtype;
  A->m = m;
  A->n = n;
  A->nnz = nnz;
  A->max_row = max_row;
  const size_t es = dtype_size(dtype);
  A->h_rowptr.assign(h_rowptr, h_rowptr + m + 1);
  A->sorted_rows = true;
  for (int32_t i = 0; i < m && A->sorted_rows; ++i)
    for (int32_t p = h_rowptr[i] + 1; p < h_rowptr[i + 1]; ++p)
      if (h_colind[p] < h_colind[p - 1]) {
        A->sorted_rows = false;
        break;
      }
  if (nnz > 0) {
    A->h_colind.assign(h_colind, h_colind + nnz);
    const auto* vb = static_cast<const unsigned char*>(h_values);
    A->h_values.assign(vb, vb + nnz * es);
  }
  spmvb_status s = upload(A->rowptr, A->h_rowptr.data(), (m + 1) * 4, (m + 1) * 4);
  if (s == SPMVB_OK) s = upload(A->colind, A->h_colind.data(), nnz * 4, (nnz + kPad) * 4);
  if (s == SPMVB_OK) s = upload(A->values, A->h_values.data(), nnz * es, (nnz + kPad) * es);
  if (s != SPMVB_OK) {
    delete A;
    return s;
  }
  *out = A;
  return SPMVB_OK;
}

spmvb_status spmvb_matrix_set_spmm_bands(spmvb_matrix A, int bands) {
  clear_error();
  if (!A) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null matrix");
  if (bands < 0 || bands > 64) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bands must be in [0, 64]");
  A->spmm_bands = bands;
  return SPMVB_OK;
}

spmvb_status spmvb_csr_validate(int32_t m, int32_t n, int64_t nnz, const int32_t* h_rowptr,
                                const int32_t* h_colind, int32_t* max_row_nnz) {
  clear_error();
  if (m < 0 || n < 0 || nnz < 0) return fail(SPMVB_ERR_INVALID_MATRIX, "negative dimension or nnz");
  if (nnz > INT32_MAX - kPad) return fail(SPMVB_ERR_UNSUPPORTED, "nnz exceeds the int32 index range");
  if (!h_rowptr) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null rowptr");
  if (nnz > 0 && !h_colind) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null colind");
  if (h_rowptr[0] != 0) return fail(SPMVB_ERR_INVALID_MATRIX, "rowptr[0] != 0");
  int32_t max_row = 0;
  for (int32_t i = 0; i < m; ++i) {
    if (h_rowptr[i + 1] < h_rowptr[i]) return fail(SPMVB_ERR_INVALID_MATRIX, "rowptr decreases at row " + std::to_string(i));
    max_row = std::max(max_row, h_rowptr[i + 1] - h_rowptr[i]);
  }
  if (h_rowptr[m] != nnz) return fail(SPMVB_ERR_INVALID_MATRIX, "rowptr[m] != nnz");
  for (int64_t p = 0; p < nnz; ++p) {
    if (h_colind[p] < 0 || h_colind[p] >= n)
      return fail(SPMVB_ERR_INVALID_MATRIX, "column index out of range at entry " + std::to_string(p));
  }
  if (max_row_nnz) *max_row_nnz = max_row;
  return SPMVB_OK;
}

spmvb_status spmvb_matrix_destroy(spmvb_matrix A) {
  clear_error();
  if (!A) return SPMVB_OK;
  DeviceGuard g(A->device);
  delete A;
  return SPMVB_OK;
}

spmvb_status spmvb_matrix_prepare(spmvb_matrix A, spmvb_kernel kernel, int param) {
  clear_error();
  if (!A) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null matrix");
  switch (kernel) {
    case SPMVB_CSR_SCALAR:
    case SPMVB_CSR_VECTOR:
    case SPMVB_CSR_WARP: return SPMVB_OK;
    case SPMVB_CSR_MERGE: return build_merge(A);
    case SPMVB_ELL: return build_ell(A);
    case SPMVB_HYB: return build_hyb(A, param);
    case SPMVB_BCSR: return build_bcsr(A, param <= 2 ? 2 : 4);
    default: break;
  }
  if (static_cast<int>(kernel) == -1) return build_buckets(A);  // SpMM buckets
  return fail(SPMVB_ERR_INVALID_ARGUMENT, "unknown kernel id");
}

spmvb_status spmvb_matrix_get_info(spmvb_matrix A, spmvb_matrix_info* out) {
  clear_error();
  if (!A || !out) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  std::lock_guard<std::mutex> lk(A->build_mu);
  spmvb_matrix_info i{};
  i.m = A->m;
  i.n = A->n;
  i.nnz = A->nnz;
  i.dtype = A->dtype;
  i.max_row_nnz = A->max_row;
  i.ell_padded_nnz = static_cast<int64_t>(A->m) * A->max_row;
  i.ell_touched_nnz = A->nnz;
  i.bcsr2_block_nnz = A->bcsr2.built ? A->bcsr2.block_nnz : -1;
  i.bcsr4_block_nnz = A->bcsr4.built ? A->bcsr4.block_nnz : -1;
  i.hyb_width = A->hyb_built ? A->hyb_K : -1;
  i.hyb_ell_nnz = A->hyb_built ? A->hyb_ell_nnz : -1;
  i.hyb_tail_nnz = A->hyb_built ? A->hyb_tail_nnz : -1;
  i.hyb_long_rows = A->hyb_built ? A->hyb_n_long : -1;
  i.device_bytes = A->device_bytes();
  *out = i;
  return SPMVB_OK;
}

spmvb_status spmvb_matrix_export_ell(spmvb_matrix A, int32_t* h_colind, void* h_values, int32_t* h_row_lengths) {
  clear_error();
  if (!A) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null matrix");
  SPMVB_TRY(build_ell(A));
  DeviceGuard g(A->device);
  const int64_t slots = static_cast<int64_t>(A->m) * A->ell_width;
  if (h_colind && slots) SPMVB_TRY_CUDA(cudaMemcpy(h_colind, A->ell_colind.get(), slots * 4, cudaMemcpyDeviceToHost));
  if (h_values && slots) SPMVB_TRY_CUDA(cudaMemcpy(h_values, A->ell_values.get(), slots * dtype_size(A->dtype), cudaMemcpyDeviceToHost));
  if (h_row_lengths && A->m) SPMVB_TRY_CUDA(cudaMemcpy(h_row_lengths, A->ell_rowlen.get(), int64_t(A->m) * 4, cudaMemcpyDeviceToHost));
  return SPMVB_OK;
}

spmvb_status spmvb_matrix_export_bcsr(spmvb_matrix A, int block, int32_t* h_rowptr, int32_t* h_colind, void* h_values) {
  clear_error();
  if (!A) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null matrix");
  if (block != 2 && block != 4) return fail(SPMVB_ERR_INVALID_ARGUMENT, "block must be 2 or 4");
  SPMVB_TRY(build_bcsr(A, block));
  DeviceGuard g(A->device);
  const auto& B = block == 2 ? A->bcsr2 : A->bcsr4;
  if (h_rowptr) SPMVB_TRY_CUDA(cudaMemcpy(h_rowptr, B.rowptr.get(), (int64_t(B.mb) + 1) * 4, cudaMemcpyDeviceToHost));
  if (h_colind && B.block_nnz) SPMVB_TRY_CUDA(cudaMemcpy(h_colind, B.colind.get(), B.block_nnz * 4, cudaMemcpyDeviceToHost));
  if (h_values && B.block_nnz)
    SPMVB_TRY_CUDA(cudaMemcpy(h_values, B.values.get(), B.block_nnz * block * block * dtype_size(A->dtype), cudaMemcpyDeviceToHost));
  return SPMVB_OK;
}

// Reads the context's device error word after `s` has been synchronized.
}  // extern "C"

spmvb_status spmvb::check_err_word(spmvb_context ctx, cudaStream_t s) {
  int code = 0;
  SPMVB_TRY_CUDA(cudaMemcpyAsync(&code, ctx->err.get(), sizeof(int), cudaMemcpyDeviceToHost, s));
  SPMVB_TRY_CUDA(cudaStreamSynchronize(s));
  if (code != 0) {
    SPMVB_TRY_CUDA(cudaMemsetAsync(ctx->err.get(), 0, sizeof(int), s));
    return fail(SPMVB_ERR_TIMEOUT, "a kernel's bounded wait gave up (device error code " + std::to_string(code) + ")");
  }
  return SPMVB_OK;
}

void* spmvb::mapped_host_ptr(const void* h) {
  if (!h) return nullptr;
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, h) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return at.type == cudaMemoryTypeHost ? at.devicePointer : nullptr;
}

extern "C" {

static spmvb_status check_pair(spmvb_matrix A, spmvb_dtype acc) {
  if (!A) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null matrix");
  if (acc != SPMVB_F32 && acc != SPMVB_F64) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bad accumulator dtype");
  if (A->dtype == SPMVB_F64 && acc == SPMVB_F32)
    return fail(SPMVB_ERR_UNSUPPORTED, "fp64 storage with fp32 accumulation is not instantiated");
  return SPMVB_OK;
}

static spmvb_status dispatch_spmv(spmvb_matrix A, spmvb_kernel kernel, int lanes, int block, const void* x, void* y,
                                  spmvb_dtype acc, cudaStream_t s) {
  if (A->dtype == SPMVB_F64)
    return launch_spmv<double, double>(A, kernel, lanes, block, static_cast<const double*>(x), static_cast<double*>(y), s);
  if (acc == SPMVB_F32)
    return launch_spmv<float, float>(A, kernel, lanes, block, static_cast<const float*>(x), static_cast<float*>(y), s);
  return launch_spmv<float, double>(A, kernel, lanes, block, static_cast<const float*>(x), static_cast<double*>(y), s);
}

static spmvb_status dispatch_spmm(spmvb_matrix A, int tile, int bucketed, int k, const void* X, void* Y,
                                  spmvb_dtype acc, cudaStream_t s) {
  if (A->dtype == SPMVB_F64)
    return launch_spmm<double, double>(A, tile, bucketed, k, static_cast<const double*>(X), static_cast<double*>(Y), s);
  if (acc == SPMVB_F32)
    return launch_spmm<float, float>(A, tile, bucketed, k, static_cast<const float*>(X), static_cast<float*>(Y), s);
  return launch_spmm<float, double>(A, tile, bucketed, k, static_cast<const float*>(X), static_cast<double*>(Y), s);
}

spmvb_status spmvb_spmv(spmvb_matrix A, spmvb_kernel kernel, int lanes, int block, const void* d_x, void* d_y,
                        spmvb_dtype acc, void* stream) {
  clear_error();
  SPMVB_TRY(check_pair(A, acc));
  if (kernel < 0 || kernel >= SPMVB_KERNEL_COUNT) return fail(SPMVB_ERR_INVALID_ARGUMENT, "unknown kernel id");
  DeviceGuard g(A->device);
  SPMVB_TRY(check_device_ptr(d_x, size_t(A->n) * dtype_size(A->dtype), A->device, "x"));
  SPMVB_TRY(check_device_ptr(d_y, size_t(A->m) * dtype_size(acc), A->device, "y"));
  return dispatch_spmv(A, kernel, lanes, block, d_x, d_y, acc, static_cast<cudaStream_t>(stream));
}

spmvb_status spmvb_spmv_time(spmvb_matrix A, spmvb_kernel kernel, int lanes, int block, const void* d_x, void* d_y,
                             spmvb_dtype acc, int iters, int warmup, void* stream, double* out_ms4) {
  clear_error();
  if (!out_ms4 || iters < 1 || warmup < 0) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bad timing arguments");
  SPMVB_TRY(check_pair(A, acc));
  if (kernel < 0 || kernel >= SPMVB_KERNEL_COUNT) return fail(SPMVB_ERR_INVALID_ARGUMENT, "unknown kernel id");
  DeviceGuard g(A->device);
  SPMVB_TRY(check_device_ptr(d_x, size_t(A->n) * dtype_size(A->dtype), A->device, "x"));
  SPMVB_TRY(check_device_ptr(d_y, size_t(A->m) * dtype_size(acc), A->device, "y"));
  SPMVB_TRY(spmvb_matrix_prepare(A, kernel, kernel == SPMVB_BCSR ? (block <= 2 ? 2 : 4) : 0));
  auto s = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < warmup; ++i) SPMVB_TRY(dispatch_spmv(A, kernel, lanes, block, d_x, d_y, acc, s));
  SPMVB_TRY_CUDA(cudaStreamSynchronize(s));
  struct Ev {
    cudaEvent_t a = nullptr, b = nullptr;
    ~Ev() {
      if (a) cudaEventDestroy(a);
      if (b) cudaEventDestroy(b);
    }
  } ev;
  SPMVB_TRY_CUDA(cudaEventCreate(&ev.a));
  SPMVB_TRY_CUDA(cudaEventCreate(&ev.b));
  std::vector<double> t(static_cast<size_t>(iters));
  for (int i = 0; i < iters; ++i) {
    SPMVB_TRY_CUDA(cudaEventRecord(ev.a, s));
    SPMVB_TRY(dispatch_spmv(A, kernel, lanes, block, d_x, d_y, acc, s));
    SPMVB_TRY_CUDA(cudaEventRecord(ev.b, s));
    SPMVB_TRY_CUDA(cudaEventSynchronize(ev.b));
    float ms = 0.f;
    SPMVB_TRY_CUDA(cudaEventElapsedTime(&ms, ev.a, ev.b));
    t[static_cast<size_t>(i)] = ms;
  }
  SPMVB_TRY(check_err_word(A->ctx, s));
  std::vector<double> sorted = t;
  std::sort(sorted.begin(), sorted.end());
  const size_t n = sorted.size();
  out_ms4[0] = n % 2 ? sorted[n / 2] : 0.5 * (sorted[n / 2 - 1] + sorted[n / 2]);
  double sum = 0.0;
  for (double v : t) sum += v;
  out_ms4[1] = sum / static_cast<double>(n);
  out_ms4[2] = sorted.front();
  out_ms4[3] = sorted.back();
  return SPMVB_OK;
}

spmvb_status spmvb_spmv_host(spmvb_matrix A, spmvb_kernel kernel, int lanes, int block, const void* h_x, void* h_y,
                             spmvb_dtype acc, void* stream) {
  clear_error();
  SPMVB_TRY(check_pair(A, acc));
  if (kernel < 0 || kernel >= SPMVB_KERNEL_COUNT) return fail(SPMVB_ERR_INVALID_ARGUMENT, "unknown kernel id");
  if ((A->n && !h_x) || (A->m && !h_y)) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null host buffer");
  DeviceGuard g(A->device);
  const size_t xb = size_t(A->n) * dtype_size(A->dtype), yb = size_t(A->m) * dtype_size(acc);
  // Pinned, mapped y: the kernel stores into it directly (no copy out).
  void* y_direct = (yb && stores_y_once(kernel)) ? mapped_host_ptr(h_y) : nullptr;
  if (A->stage_in.bytes() < xb + 16) SPMVB_TRY(A->stage_in.alloc(xb + 16));
  if (!y_direct && A->stage_out.bytes() < yb + 16) SPMVB_TRY(A->stage_out.alloc(yb + 16));
  auto s = static_cast<cudaStream_t>(stream);
  if (xb) SPMVB_TRY_CUDA(cudaMemcpyAsync(A->stage_in.get(), h_x, xb, cudaMemcpyHostToDevice, s));
  if (y_direct) {
    SPMVB_TRY(dispatch_spmv(A, kernel, lanes, block, A->stage_in.get(), y_direct, acc, s));
  } else {
    SPMVB_TRY(dispatch_spmv(A, kernel, lanes, block, A->stage_in.get(), A->stage_out.get(), acc, s));
    if (yb) SPMVB_TRY_CUDA(cudaMemcpyAsync(h_y, A->stage_out.get(), yb, cudaMemcpyDeviceToHost, s));
  }
  SPMVB_TRY_CUDA(cudaStreamSynchronize(s));
  return check_err_word(A->ctx, s);
}

spmvb_status spmvb_spmm(spmvb_matrix A, int tile, int bucketed, int k, const void* d_X, void* d_Y, spmvb_dtype acc,
                        void* stream) {
  clear_error();
  SPMVB_TRY(check_pair(A, acc));
  if (k < 0) return fail(SPMVB_ERR_INVALID_ARGUMENT, "negative k");
  DeviceGuard g(A->device);
  SPMVB_TRY(check_device_ptr(d_X, size_t(A->n) * k * dtype_size(A->dtype), A->device, "X"));
  SPMVB_TRY(check_device_ptr(d_Y, size_t(A->m) * k * dtype_size(acc), A->device, "Y"));
  return dispatch_spmm(A, tile, bucketed, k, d_X, d_Y, acc, static_cast<cudaStream_t>(stream));
}

spmvb_status spmvb_spmm_host(spmvb_matrix A, int tile, int bucketed, int k, const void* h_X, void* h_Y,
                             spmvb_dtype acc, void* stream) {
  clear_error();
  SPMVB_TRY(check_pair(A, acc));
  if (k < 0) return fail(SPMVB_ERR_INVALID_ARGUMENT, "negative k");
  const size_t xb = size_t(A->n) * k * dtype_size(A->dtype), yb = size_t(A->m) * k * dtype_size(acc);
  if ((xb && !h_X) || (yb && !h_Y)) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null host buffer");
  DeviceGuard g(A->device);
  if (A->stage_in.bytes() < xb + 16) SPMVB_TRY(A->stage_in.alloc(xb + 16));
  if (A->stage_out.bytes() < yb + 16) SPMVB_TRY(A->stage_out.alloc(yb + 16));
  auto s = static_cast<cudaStream_t>(stream);
  if (xb) SPMVB_TRY_CUDA(cudaMemcpyAsync(A->stage_in.get(), h_X, xb, cudaMemcpyHostToDevice, s));
  SPMVB_TRY(dispatch_spmm(A, tile, bucketed, k, A->stage_in.get(), A->stage_out.get(), acc, s));
  if (yb) SPMVB_TRY_CUDA(cudaMemcpyAsync(h_Y, A->stage_out.get(), yb, cudaMemcpyDeviceToHost, s));
  SPMVB_TRY_CUDA(cudaStreamSynchronize(s));
  return SPMVB_OK;
}

}  // extern "C"
