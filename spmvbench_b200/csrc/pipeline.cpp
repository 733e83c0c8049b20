// Streamed SpMV over host buffers (no reference counterpart; the reference's
// SpmvRunner copies x in, runs and copies y out synchronously,
// src/cuda/spmv_cuda.cu:292-330, 476-498).
//
// A pipeline owns `depth` slots, each a non-blocking stream with its own
// device staging for x and y. spmvb_pipeline_submit enqueues, on the next
// slot, the copy of the caller's host x in, the SpMV, and the copy of y out,
// and returns without waiting. Work on one slot is ordered by its stream
// (its staging is reused only after its previous call has finished), and
// the slots run side by side: with pinned host buffers one call's copy in
// overlaps another's kernel and a third's output. When the caller's y is
// pinned and mapped, kernels that store each y element once write it there
// directly; otherwise y is staged on the device and copied out.
#include <cuda_runtime.h>

#include <memory>
#include <vector>

#include "internal.hpp"

using namespace spmvb;

struct spmvb_pipeline_st {
  spmvb_matrix A = nullptr;
  struct Slot {
    cudaStream_t stream = nullptr;
    cudaEvent_t done = nullptr;
    DevBuf x, y;
    bool used = false;
  };
  std::vector<Slot> slots;
  cudaEvent_t fork = nullptr;
  int next = 0;

  ~spmvb_pipeline_st() {
    for (auto& s : slots) {
      if (s.stream) cudaStreamSynchronize(s.stream);
      if (s.done) cudaEventDestroy(s.done);
      if (s.stream) cudaStreamDestroy(s.stream);
    }
    if (fork) cudaEventDestroy(fork);
  }
};

extern "C" {

spmvb_status spmvb_pipeline_create(spmvb_matrix A, int depth, spmvb_pipeline* out) {
  clear_error();
  if (!A || !out) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  if (depth < 1 || depth > 16) return fail(SPMVB_ERR_INVALID_ARGUMENT, "depth must be in [1, 16]");
  *out = nullptr;
  DeviceGuard g(A->device);
  auto P = std::make_unique<spmvb_pipeline_st>();
  P->A = A;
  P->slots.resize(depth);
  SPMVB_TRY_CUDA(cudaEventCreateWithFlags(&P->fork, cudaEventDisableTiming));
  for (auto& s : P->slots) {
    SPMVB_TRY_CUDA(cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking));
    SPMVB_TRY_CUDA(cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming));
    // Room for either accumulator type.
    SPMVB_TRY(s.x.alloc(size_t(A->n) * dtype_size(A->dtype) + 16));
    SPMVB_TRY(s.y.alloc(size_t(A->m) * 8 + 16));
  }
  *out = P.release();
  return SPMVB_OK;
}

spmvb_status spmvb_pipeline_fork(spmvb_pipeline P, void* stream) {
  clear_error();
  if (!P) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null pipeline");
  DeviceGuard g(P->A->device);
  SPMVB_TRY_CUDA(cudaEventRecord(P->fork, static_cast<cudaStream_t>(stream)));
  for (auto& s : P->slots) SPMVB_TRY_CUDA(cudaStreamWaitEvent(s.stream, P->fork, 0));
  return SPMVB_OK;
}

spmvb_status spmvb_pipeline_submit(spmvb_pipeline P, spmvb_kernel kernel, int lanes, int block, const void* h_x,
                                   void* h_y, spmvb_dtype acc) {
  clear_error();
  if (!P) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null pipeline");
  spmvb_matrix A = P->A;
  if ((A->n && !h_x) || (A->m && !h_y)) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null host buffer");
  if (acc != SPMVB_F32 && acc != SPMVB_F64) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bad accumulator dtype");
  if (A->dtype == SPMVB_F64 && acc == SPMVB_F32)
    return fail(SPMVB_ERR_UNSUPPORTED, "fp64 storage with fp32 accumulation is not instantiated");
  if (kernel < 0 || kernel >= SPMVB_KERNEL_COUNT) return fail(SPMVB_ERR_INVALID_ARGUMENT, "unknown kernel id");
  DeviceGuard g(A->device);
  // Formats are built (synchronously) before anything is enqueued.
  SPMVB_TRY(spmvb_matrix_prepare(A, kernel, kernel == SPMVB_BCSR ? block : 0));
  auto& s = P->slots[P->next];
  P->next = (P->next + 1) % static_cast<int>(P->slots.size());
  const size_t xb = size_t(A->n) * dtype_size(A->dtype), yb = size_t(A->m) * dtype_size(acc);
  // Pinned, mapped y: the kernel stores into it directly, so only the copy
  // engine's host-to-device direction is busy and the SpMV's PCIe writes
  // replace the device-to-host copy (that copy slowed down while a
  // neighbouring slot's L2-bound SpMV ran).
  void* y_direct = (yb && stores_y_once(kernel)) ? mapped_host_ptr(h_y) : nullptr;
  if (xb) SPMVB_TRY_CUDA(cudaMemcpyAsync(s.x.get(), h_x, xb, cudaMemcpyHostToDevice, s.stream));
  if (y_direct) {
    SPMVB_TRY(spmvb_spmv(A, kernel, lanes, block, s.x.get(), y_direct, acc, s.stream));
  } else {
    SPMVB_TRY(spmvb_spmv(A, kernel, lanes, block, s.x.get(), s.y.get(), acc, s.stream));
    if (yb) SPMVB_TRY_CUDA(cudaMemcpyAsync(h_y, s.y.get(), yb, cudaMemcpyDeviceToHost, s.stream));
  }
  SPMVB_TRY_CUDA(cudaEventRecord(s.done, s.stream));
  s.used = true;
  return SPMVB_OK;
}

spmvb_status spmvb_pipeline_join(spmvb_pipeline P, void* stream) {
  clear_error();
  if (!P) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null pipeline");
  DeviceGuard g(P->A->device);
  for (auto& s : P->slots)
    if (s.used) SPMVB_TRY_CUDA(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), s.done, 0));
  return SPMVB_OK;
}

spmvb_status spmvb_pipeline_wait(spmvb_pipeline P) {
  clear_error();
  if (!P) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null pipeline");
  DeviceGuard g(P->A->device);
  for (auto& s : P->slots) SPMVB_TRY_CUDA(cudaStreamSynchronize(s.stream));
  return check_err_word(P->A->ctx, P->slots[0].stream);
}

spmvb_status spmvb_pipeline_destroy(spmvb_pipeline P) {
  clear_error();
  if (!P) return SPMVB_OK;
  DeviceGuard g(P->A->device);
  delete P;
  return SPMVB_OK;
}

}  // extern "C"
