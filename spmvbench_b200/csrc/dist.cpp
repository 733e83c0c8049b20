// Row-sharded multi-GPU SpMV with NCCL all-gather of x (no reference
// counterpart; the reference is single-GPU).
//
// One process per GPU. Rank g owns rows [bounds[g], bounds[g+1]) of a square
// matrix (bounds from spmvb_partition_rows, nnz-balanced). NCCL has no
// all-gather-v, so every rank's slice of x is padded to max_rows entries and
// x lives in a padded layout of nranks*max_rows slots: global column c owned
// by rank r sits in slot r*max_rows + (c - bounds[r]). Columns are renumbered
// into that layout once, when the shard is built, so each step is
//   y_local = A_local * x_pad        (this library's SpMV kernel)
//   x_pad   = all_gather(y_local)    (ncclAllGather over NVLink)
// with no other copies. Communicator set-up is non-blocking with a bounded
// wait: a rank that never joins makes spmvb_dist_create return
// SPMVB_ERR_TIMEOUT after the communicator is aborted.
//
// Peer exchange (spmvb_dist_enable_peer, collective): every rank maps the
// other ranks' x buffers through CUDA IPC and the step becomes
//   y_local = A_local * x[cur]; store y_local into x[cur^1] of every rank;
//   barrier (publish this rank's phase, wait for every peer's)
// in one kernel for ELL (peer.cu) and SpMV + push for the other kernels,
// with no NCCL call on the data path. x is double-buffered: step k reads
// x[k%2] and writes x[(k+1)%2]; a rank's step k+1 writes a peer's x[k%2]
// only after its own step k barrier, which needs the peer to have finished
// step k, and with it every read of x[k%2].
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "internal.hpp"

using namespace spmvb;

struct spmvb_dist_st {
  spmvb_context ctx = nullptr;
  int nranks = 1;
  int rank = 0;
  spmvb_dtype dtype = SPMVB_F64;
  ncclComm_t comm = nullptr;
  std::vector<int32_t> bounds;
  int32_t m = 0;
  int32_t max_rows = 0;
  spmvb_matrix local = nullptr;
  DevBuf x_pad, y_loc;
  DevBuf bounds_dev;   // bounds on the device (power iteration's norm)
  DevBuf norm_work;    // norm partials, then the norm itself

  // Peer exchange state.
  bool peer = false;
  bool broken = false;       // a peer wait gave up; the phases no longer agree
  DevBuf pmem;               // [x0 | x1 | nranks phase counters], IPC-exported
  size_t xbytes = 0;         // bytes of one padded x buffer (256-aligned)
  void* peer_base[kMaxRanks] = {};  // other ranks' pmem, mapped here
  DevBuf counter;            // finished-CTA counter (offset 0) and phase (offset 64)
  int cur = 0;
  unsigned long long timeout_ns = 0;
  // Captured pairs of peer steps (x parity returns to where it started),
  // keyed by kernel, lanes and starting parity; and captured single NCCL
  // steps (parity -1).
  struct Graph {
    int kernel, lanes, parity;
    cudaGraphExec_t exec;
    uint64_t kernels;  // kernel launches per replay
  };
  std::vector<Graph> graphs;
  cudaStream_t capture = nullptr;
  // Host-buffer pipelines made on this handle: their work drains before the
  // communicator and the matrix go.
  std::vector<spmvb_dist_pipeline_st*> pipelines;

  void close_peers() {
    for (int q = 0; q < kMaxRanks; ++q)
      if (peer_base[q]) {
        cudaIpcCloseMemHandle(peer_base[q]);
        peer_base[q] = nullptr;
      }
  }
  ~spmvb_dist_st() {
    for (auto& g : graphs) cudaGraphExecDestroy(g.exec);
    if (capture) cudaStreamDestroy(capture);
    close_peers();
    spmvb_matrix_destroy(local);
  }
};

namespace {

spmvb_status nccl_fail(ncclResult_t r, const char* what) {
  return fail(SPMVB_ERR_NCCL, std::string(what) + ": " + ncclGetErrorString(r));
}

// Bounded wait for a non-blocking communicator operation to settle. A
// collective's enqueue settles in microseconds, so the first 20 ms poll with
// a yield between tries; only a slow operation (communicator set-up) falls
// back to 1 ms sleeps.
spmvb_status nccl_wait(ncclComm_t comm, double timeout_s, const char* what) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t r = ncclCommGetAsyncError(comm, &st);
    if (r != ncclSuccess) return nccl_fail(r, what);
    if (st == ncclSuccess) return SPMVB_OK;
    if (st != ncclInProgress) return nccl_fail(st, what);
    const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > timeout_s) return fail(SPMVB_ERR_TIMEOUT, std::string(what) + ": timed out after " + std::to_string(timeout_s) + " s");
    if (el < 0.02)
      std::this_thread::yield();
    else
      std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
}

// A non-blocking communicator may return ncclInProgress from a collective
// while it is still being enqueued (the first call sets up connections); the
// next NCCL call on that communicator must wait until it reports success.
spmvb_status nccl_enqueued(ncclComm_t comm, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return SPMVB_OK;
  if (r != ncclInProgress) return nccl_fail(r, what);
  return nccl_wait(comm, 120.0, what);
}

double peer_timeout_ms() {
  const char* e = std::getenv("SPMVB_PEER_TIMEOUT_MS");
  const double v = (e && *e) ? std::atof(e) : 10000.0;
  return v > 0 ? v : 10000.0;
}

unsigned char* x_buf(spmvb_dist D, int which) { return D->pmem.as<unsigned char>() + size_t(which) * D->xbytes; }

// Kernel view of the next peer operation: write this rank's slice of
// x[cur^1] of every rank, then publish the next phase and wait for every
// peer to reach it.
PeerView peer_view(spmvb_dist D) {
  PeerView P;
  const size_t es = dtype_size(D->dtype);
  const size_t slice = size_t(D->rank) * D->max_rows * es;
  const size_t next = size_t(D->cur ^ 1) * D->xbytes + slice;
  const size_t flags = 2 * D->xbytes;
  for (int q = 0; q < D->nranks; ++q) {
    unsigned char* base = q == D->rank ? D->pmem.as<unsigned char>() : static_cast<unsigned char*>(D->peer_base[q]);
    P.dst[q] = base + next;
    P.flag_out[q] = reinterpret_cast<unsigned long long*>(base + flags) + D->rank;
  }
  P.flags_in = reinterpret_cast<const unsigned long long*>(D->pmem.as<unsigned char>() + flags);
  P.counter = D->counter.as<unsigned int>();
  P.err = D->ctx->err.as<int>();
  P.phase = reinterpret_cast<unsigned long long*>(D->counter.as<unsigned char>() + 64);
  P.timeout_ns = D->timeout_ns;
  P.nranks = D->nranks;
  P.rank = D->rank;
  P.rows = D->bounds[D->rank + 1] - D->bounds[D->rank];
  return P;
}

// Reads the device error word after a peer operation; a peer wait that gave
// up leaves the ranks' phases out of step, so the handle refuses further
// steps.
spmvb_status peer_check(spmvb_dist D, cudaStream_t s) {
  const spmvb_status st = check_err_word(D->ctx, s);
  if (st == SPMVB_ERR_TIMEOUT) D->broken = true;
  return st;
}

double init_timeout_s() {
  const char* e = std::getenv("SPMVB_NCCL_INIT_TIMEOUT_S");
  return (e && *e) ? std::atof(e) : 120.0;
}

}  // namespace

extern "C" {

spmvb_status spmvb_shard_csr(int32_t m, const int32_t* h_rowptr, const int32_t* h_colind, int nranks, int rank,
                             const int32_t* h_bounds, int32_t* max_rows, int64_t* local_nnz,
                             int32_t* h_out_rowptr, int32_t* h_out_colind) {
  clear_error();
  if (!h_rowptr || !h_bounds || !max_rows || !local_nnz) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  if (nranks < 1 || rank < 0 || rank >= nranks || m < 0) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bad rank / nranks / m");
  if (h_bounds[0] != 0 || h_bounds[nranks] != m) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bounds must span [0, m]");
  int32_t mr = 0;
  for (int g = 0; g < nranks; ++g) {
    if (h_bounds[g + 1] < h_bounds[g]) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bounds must be non-decreasing");
    mr = std::max(mr, h_bounds[g + 1] - h_bounds[g]);
  }
  const int32_t r0 = h_bounds[rank], r1 = h_bounds[rank + 1];
  const int64_t p0 = h_rowptr[r0], p1 = h_rowptr[r1];
  *max_rows = mr;
  *local_nnz = p1 - p0;
  if (!h_out_colind) return SPMVB_OK;
  if (!h_out_rowptr) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null output rowptr");
  for (int32_t i = 0; i <= r1 - r0; ++i) h_out_rowptr[i] = static_cast<int32_t>(h_rowptr[r0 + i] - p0);
  for (int64_t p = p0; p < p1; ++p) {
    const int32_t c = h_colind[p];
    if (c < 0 || c >= m) return fail(SPMVB_ERR_INVALID_MATRIX, "column index out of range");
    const int owner = static_cast<int>(std::upper_bound(h_bounds, h_bounds + nranks + 1, c) - h_bounds) - 1;
    h_out_colind[p - p0] = owner * mr + (c - h_bounds[owner]);
  }
  return SPMVB_OK;
}

spmvb_status spmvb_nccl_unique_id(void* h_out, size_t cap) {
  clear_error();
  if (!h_out || cap < sizeof(ncclUniqueId)) return fail(SPMVB_ERR_INVALID_ARGUMENT, "buffer smaller than ncclUniqueId");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  std::memcpy(h_out, &id, sizeof(id));
  return SPMVB_OK;
}

spmvb_status spmvb_dist_create(spmvb_context ctx, int nranks, int rank, const void* h_unique_id, spmvb_dtype dtype,
                               int32_t m, int64_t nnz, const int32_t* h_rowptr, const int32_t* h_colind,
                               const void* h_values, const int32_t* h_bounds, spmvb_dist* out) {
  clear_error();
  if (!ctx || !out || !h_rowptr || !h_bounds) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  if (nranks < 1 || rank < 0 || rank >= nranks) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bad rank / nranks");
  if (nranks > 1 && !h_unique_id) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null NCCL unique id");
  if (dtype != SPMVB_F32 && dtype != SPMVB_F64) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bad dtype");
  if (m < 0 || nnz < 0 || h_rowptr[m] != nnz) return fail(SPMVB_ERR_INVALID_MATRIX, "rowptr[m] != nnz");
  if (h_bounds[0] != 0 || h_bounds[nranks] != m) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bounds must span [0, m]");
  for (int g = 0; g < nranks; ++g)
    if (h_bounds[g + 1] < h_bounds[g]) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bounds must be non-decreasing");
  DeviceGuard guard(ctx->device);
  auto D = std::make_unique<spmvb_dist_st>();
  D->ctx = ctx;
  D->nranks = nranks;
  D->rank = rank;
  D->dtype = dtype;
  D->m = m;
  D->bounds.assign(h_bounds, h_bounds + nranks + 1);

  // Local shard with renumbered columns.
  const int32_t r0 = h_bounds[rank], r1 = h_bounds[rank + 1];
  const int32_t ml = r1 - r0;
  const size_t es = dtype_size(dtype);
  int64_t lnnz = 0;
  SPMVB_TRY(spmvb_shard_csr(m, h_rowptr, h_colind, nranks, rank, h_bounds, &D->max_rows, &lnnz, nullptr, nullptr));
  std::vector<int32_t> rp(ml + 1), ci(std::max<int64_t>(lnnz, 1));
  SPMVB_TRY(spmvb_shard_csr(m, h_rowptr, h_colind, nranks, rank, h_bounds, &D->max_rows, &lnnz, rp.data(), ci.data()));
  const int64_t p0 = h_rowptr[r0];
  const unsigned char* vv = static_cast<const unsigned char*>(h_values) + p0 * es;
  const int32_t npad = nranks * D->max_rows;
  SPMVB_TRY(spmvb_matrix_create_csr(ctx, dtype, ml, npad, lnnz, rp.data(), ci.data(), vv, &D->local));
  SPMVB_TRY(D->x_pad.alloc(size_t(std::max(npad, 1)) * es));
  SPMVB_TRY(D->y_loc.alloc(size_t(std::max(D->max_rows, 1)) * es));

  if (nranks > 1) {
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclUniqueId id;
    std::memcpy(&id, h_unique_id, sizeof(id));
    ncclResult_t r = ncclCommInitRankConfig(&D->comm, nranks, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) return nccl_fail(r, "ncclCommInitRankConfig");
    spmvb_status s = nccl_wait(D->comm, init_timeout_s(), "ncclCommInitRankConfig");
    if (s != SPMVB_OK) {
      const std::string msg = spmvb_last_error();
      ncclCommAbort(D->comm);
      D->comm = nullptr;
      return fail(s, msg);
    }
  }
  *out = D.release();
  return SPMVB_OK;
}

static void detach_pipeline(spmvb_dist_pipeline_st* P);

spmvb_status spmvb_dist_destroy(spmvb_dist D) {
  clear_error();
  if (!D) return SPMVB_OK;
  DeviceGuard g(D->ctx->device);
  if (D->peer && D->nranks > 1) {
    // A last barrier: once every rank has reached it, no rank stores into
    // another's buffers again. If it fails, the buffers are left allocated
    // rather than freed under a possible writer.
    bool quiet = cudaDeviceSynchronize() == cudaSuccess && !D->broken;
    if (quiet) {
      quiet = peer_launch_barrier(peer_view(D), nullptr) == SPMVB_OK && check_err_word(D->ctx, nullptr) == SPMVB_OK;
    }
    D->close_peers();
    if (!quiet) (void)D->pmem.release();
  }
  // Graphs that hold NCCL calls go before the communicator does.
  for (auto& gr : D->graphs) cudaGraphExecDestroy(gr.exec);
  D->graphs.clear();
  for (auto* P : D->pipelines) detach_pipeline(P);
  D->pipelines.clear();
  if (D->comm) {
    ncclCommFinalize(D->comm);
    nccl_wait(D->comm, 30.0, "ncclCommFinalize");
    ncclCommDestroy(D->comm);
  }
  delete D;
  return SPMVB_OK;
}

spmvb_status spmvb_dist_enable_peer(spmvb_dist D, void* stream) {
  clear_error();
  if (!D) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  if (D->peer) return SPMVB_OK;
  if (D->nranks > kMaxRanks)
    return fail(SPMVB_ERR_UNSUPPORTED, "the peer exchange supports at most " + std::to_string(kMaxRanks) + " ranks");
  DeviceGuard g(D->ctx->device);
  auto s = static_cast<cudaStream_t>(stream);
  const size_t es = dtype_size(D->dtype);
  const size_t npad_bytes = size_t(D->nranks) * D->max_rows * es;
  D->xbytes = std::max<size_t>(256, (npad_bytes + 255) / 256 * 256);
  SPMVB_TRY(D->pmem.alloc(2 * D->xbytes + 256));
  SPMVB_TRY(D->counter.alloc(256));
  D->timeout_ns = static_cast<unsigned long long>(peer_timeout_ms() * 1e6);
  // The zero-filled counters must be in place before any rank can map them.
  SPMVB_TRY_CUDA(cudaDeviceSynchronize());

  if (D->nranks > 1) {
    struct Record {
      cudaIpcMemHandle_t handle;
      unsigned char uuid[16];
      int32_t ok;
      int32_t pad[3];
    };
    Record mine;
    std::memset(&mine, 0, sizeof(mine));
    mine.ok = cudaIpcGetMemHandle(&mine.handle, D->pmem.get()) == cudaSuccess;
    cudaGetLastError();
    cudaDeviceProp prop;
    SPMVB_TRY_CUDA(cudaGetDeviceProperties(&prop, D->ctx->device));
    std::memcpy(mine.uuid, &prop.uuid, sizeof(mine.uuid));
    std::vector<Record> all(D->nranks);
    DevBuf dsend, drecv, dok;
    SPMVB_TRY(dsend.alloc(sizeof(Record)));
    SPMVB_TRY(drecv.alloc(sizeof(Record) * D->nranks));
    SPMVB_TRY(dok.alloc(sizeof(int32_t)));
    SPMVB_TRY_CUDA(cudaMemcpyAsync(dsend.get(), &mine, sizeof(Record), cudaMemcpyHostToDevice, s));
    SPMVB_TRY(nccl_enqueued(D->comm, ncclAllGather(dsend.get(), drecv.get(), sizeof(Record), ncclChar, D->comm, s),
                            "ncclAllGather(peer records)"));
    SPMVB_TRY_CUDA(cudaMemcpyAsync(all.data(), drecv.get(), sizeof(Record) * D->nranks, cudaMemcpyDeviceToHost, s));
    SPMVB_TRY_CUDA(cudaStreamSynchronize(s));

    // Every rank sees the same records, so these checks agree everywhere.
    std::string why;
    for (int q = 0; q < D->nranks && why.empty(); ++q)
      if (!all[q].ok) why = "rank " + std::to_string(q) + " could not export its buffers";
    for (int q = 0; q < D->nranks && why.empty(); ++q)
      for (int r = q + 1; r < D->nranks && why.empty(); ++r)
        if (std::memcmp(all[q].uuid, all[r].uuid, sizeof(all[q].uuid)) == 0)
          why = "ranks " + std::to_string(q) + " and " + std::to_string(r) +
                " share one GPU; the peer kernels wait on one another and need one GPU per rank";
    int32_t ok = why.empty();
    for (int q = 0; q < D->nranks && ok; ++q) {
      if (q == D->rank) continue;
      const cudaError_t e = cudaIpcOpenMemHandle(&D->peer_base[q], all[q].handle, cudaIpcMemLazyEnablePeerAccess);
      if (e != cudaSuccess) {
        cudaGetLastError();
        D->peer_base[q] = nullptr;
        ok = 0;
        why = "cudaIpcOpenMemHandle(rank " + std::to_string(q) + "): " + cudaGetErrorString(e);
      }
    }
    // All ranks must agree before any of them stores into another's memory.
    SPMVB_TRY_CUDA(cudaMemcpyAsync(dok.get(), &ok, sizeof(ok), cudaMemcpyHostToDevice, s));
    SPMVB_TRY(nccl_enqueued(D->comm, ncclAllReduce(dok.get(), dok.get(), 1, ncclInt32, ncclMin, D->comm, s),
                            "ncclAllReduce(peer agreement)"));
    int32_t all_ok = 0;
    SPMVB_TRY_CUDA(cudaMemcpyAsync(&all_ok, dok.get(), sizeof(all_ok), cudaMemcpyDeviceToHost, s));
    SPMVB_TRY_CUDA(cudaStreamSynchronize(s));
    if (!all_ok) {
      // Every rank unmaps the others' buffers; only after all have done so
      // (the second collective) does a rank free its own.
      D->close_peers();
      SPMVB_TRY(nccl_enqueued(D->comm, ncclAllReduce(dok.get(), dok.get(), 1, ncclInt32, ncclMin, D->comm, s),
                              "ncclAllReduce(peer release)"));
      SPMVB_TRY_CUDA(cudaStreamSynchronize(s));
      D->pmem.reset();
      D->counter.reset();
      return fail(SPMVB_ERR_UNSUPPORTED,
                  "peer exchange unavailable: " + (why.empty() ? std::string("another rank could not map peer memory") : why));
    }
  }
  if (npad_bytes)
    SPMVB_TRY_CUDA(cudaMemcpyAsync(x_buf(D, 0), D->x_pad.get(), npad_bytes, cudaMemcpyDeviceToDevice, s));
  SPMVB_TRY_CUDA(cudaStreamSynchronize(s));
  D->cur = 0;
  D->peer = true;
  return SPMVB_OK;
}

int spmvb_dist_exchange(spmvb_dist D) { return D && D->peer ? SPMVB_EXCHANGE_PEER : SPMVB_EXCHANGE_NCCL; }

spmvb_status spmvb_dist_set_x(spmvb_dist D, const void* h_x, void* stream) {
  clear_error();
  if (!D || (D->m && !h_x)) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  if (D->broken) return fail(SPMVB_ERR_TIMEOUT, "an earlier peer wait gave up; recreate the handle");
  DeviceGuard g(D->ctx->device);
  const size_t es = dtype_size(D->dtype);
  std::vector<unsigned char> pad(size_t(D->nranks) * D->max_rows * es, 0);
  for (int r = 0; r < D->nranks; ++r) {
    const int32_t b = D->bounds[r], cnt = D->bounds[r + 1] - b;
    std::memcpy(pad.data() + size_t(r) * D->max_rows * es, static_cast<const unsigned char*>(h_x) + size_t(b) * es, size_t(cnt) * es);
  }
  auto s = static_cast<cudaStream_t>(stream);
  if (!D->peer) {
    if (!pad.empty()) SPMVB_TRY_CUDA(cudaMemcpyAsync(D->x_pad.get(), pad.data(), pad.size(), cudaMemcpyHostToDevice, s));
    SPMVB_TRY_CUDA(cudaStreamSynchronize(s));
    return SPMVB_OK;
  }
  // Peer exchange: the previous operation's barrier saw every peer's stores
  // into x[cur] land, and no peer writes x[cur] before this rank's next step
  // has read it.
  if (!pad.empty()) SPMVB_TRY_CUDA(cudaMemcpyAsync(x_buf(D, D->cur), pad.data(), pad.size(), cudaMemcpyHostToDevice, s));
  return peer_check(D, s);
}

// One peer-exchange step. One rank: the SpMV writes the other x buffer.
// Several: the fused ELL kernel, or the SpMV into y_loc and the push kernel.
static spmvb_status peer_step(spmvb_dist D, spmvb_kernel kernel, int lanes, cudaStream_t s, cudaEvent_t mark) {
  void* x = x_buf(D, D->cur);
  if (D->nranks == 1) {
    SPMVB_TRY(spmvb_spmv(D->local, kernel, lanes, 4, x, x_buf(D, D->cur ^ 1), D->dtype, s));
    if (mark) SPMVB_TRY_CUDA(cudaEventRecord(mark, s));
  } else if (kernel == SPMVB_ELL) {
    SPMVB_TRY(peer_launch_ell(D->local, peer_view(D), x, s));
    if (mark) SPMVB_TRY_CUDA(cudaEventRecord(mark, s));
  } else {
    SPMVB_TRY(spmvb_spmv(D->local, kernel, lanes, 4, x, D->y_loc.get(), D->dtype, s));
    if (mark) SPMVB_TRY_CUDA(cudaEventRecord(mark, s));
    SPMVB_TRY(peer_launch_push(D->dtype, D->y_loc.get(), peer_view(D), D->ctx->sm_count, s));
  }
  D->cur ^= 1;
  return SPMVB_OK;
}

static bool graphs_enabled() {
  const char* e = std::getenv("SPMVB_DIST_GRAPHS");
  return !(e && *e == '0');
}

// The graph of two peer steps from the current parity, captured on a
// private stream on first use (the formats are built by then: the caller ran
// one eager step).
static spmvb_status peer_graph(spmvb_dist D, spmvb_kernel kernel, int lanes, cudaGraphExec_t* exec, uint64_t* kernels) {
  for (const auto& g : D->graphs)
    if (g.kernel == kernel && g.lanes == lanes && g.parity == D->cur) {
      *exec = g.exec;
      *kernels = g.kernels;
      return SPMVB_OK;
    }
  if (!D->capture) SPMVB_TRY_CUDA(cudaStreamCreateWithFlags(&D->capture, cudaStreamNonBlocking));
  const int parity = D->cur;
  const uint64_t before = spmvb_launch_count();
  SPMVB_TRY_CUDA(cudaStreamBeginCapture(D->capture, cudaStreamCaptureModeRelaxed));
  spmvb_status st = peer_step(D, kernel, lanes, D->capture, nullptr);
  if (st == SPMVB_OK) st = peer_step(D, kernel, lanes, D->capture, nullptr);
  cudaGraph_t graph = nullptr;
  const cudaError_t e = cudaStreamEndCapture(D->capture, &graph);
  const uint64_t captured = spmvb_launch_count() - before;
  uncount_launch(captured);  // counted when captured, not run
  D->cur = parity;
  if (st != SPMVB_OK || e != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    return st != SPMVB_OK ? st : cuda_fail(e, "cudaStreamEndCapture");
  }
  cudaGraphExec_t ex = nullptr;
  const cudaError_t ei = cudaGraphInstantiate(&ex, graph, 0);
  cudaGraphDestroy(graph);
  if (ei != cudaSuccess) return cuda_fail(ei, "cudaGraphInstantiate");
  D->graphs.push_back({static_cast<int>(kernel), lanes, parity, ex, captured});
  *exec = ex;
  *kernels = captured;
  return SPMVB_OK;
}

static spmvb_status dist_step(spmvb_dist D, spmvb_kernel kernel, int lanes, cudaStream_t s);

// The graph of one NCCL-exchange step (SpMV, then the all-gather into x),
// captured on a private stream on first use (the caller ran one eager step,
// so formats and NCCL connections exist). Keyed with parity -1.
static spmvb_status nccl_graph(spmvb_dist D, spmvb_kernel kernel, int lanes, cudaGraphExec_t* exec, uint64_t* kernels) {
  for (const auto& g : D->graphs)
    if (g.kernel == kernel && g.lanes == lanes && g.parity == -1) {
      *exec = g.exec;
      *kernels = g.kernels;
      return SPMVB_OK;
    }
  if (!D->capture) SPMVB_TRY_CUDA(cudaStreamCreateWithFlags(&D->capture, cudaStreamNonBlocking));
  const uint64_t before = spmvb_launch_count();
  SPMVB_TRY_CUDA(cudaStreamBeginCapture(D->capture, cudaStreamCaptureModeRelaxed));
  const spmvb_status st = dist_step(D, kernel, lanes, D->capture);
  cudaGraph_t graph = nullptr;
  const cudaError_t e = cudaStreamEndCapture(D->capture, &graph);
  const uint64_t captured = spmvb_launch_count() - before;
  uncount_launch(captured);
  if (st != SPMVB_OK || e != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    return st != SPMVB_OK ? st : cuda_fail(e, "cudaStreamEndCapture");
  }
  cudaGraphExec_t ex = nullptr;
  const cudaError_t ei = cudaGraphInstantiate(&ex, graph, 0);
  cudaGraphDestroy(graph);
  if (ei != cudaSuccess) return cuda_fail(ei, "cudaGraphInstantiate");
  D->graphs.push_back({static_cast<int>(kernel), lanes, -1, ex, captured});
  *exec = ex;
  *kernels = captured;
  return SPMVB_OK;
}

static spmvb_status dist_step(spmvb_dist D, spmvb_kernel kernel, int lanes, cudaStream_t s) {
  SPMVB_TRY(spmvb_spmv(D->local, kernel, lanes, 4, D->x_pad.get(), D->y_loc.get(), D->dtype, s));
  if (D->nranks > 1) {
    const ncclDataType_t t = D->dtype == SPMVB_F64 ? ncclFloat64 : ncclFloat32;
    SPMVB_TRY(nccl_enqueued(D->comm, ncclAllGather(D->y_loc.get(), D->x_pad.get(), size_t(D->max_rows), t, D->comm, s),
                            "ncclAllGather"));
  } else {
    SPMVB_TRY_CUDA(cudaMemcpyAsync(D->x_pad.get(), D->y_loc.get(), size_t(D->max_rows) * dtype_size(D->dtype),
                                   cudaMemcpyDeviceToDevice, s));
  }
  return SPMVB_OK;
}

spmvb_status spmvb_dist_iterate(spmvb_dist D, spmvb_kernel kernel, int lanes, int iters, void* stream) {
  clear_error();
  if (!D || iters < 0) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bad argument");
  if (D->broken) return fail(SPMVB_ERR_TIMEOUT, "an earlier peer wait gave up; recreate the handle");
  DeviceGuard g(D->ctx->device);
  auto s = static_cast<cudaStream_t>(stream);
  if (D->peer) {
    // Asynchronous: a bounded wait that gives up is reported by the next
    // set_x, get_x or iterate_timed. From three steps on, pairs of steps
    // replay a captured graph.
    int left = iters;
    if (left >= 3 && graphs_enabled()) {
      SPMVB_TRY(peer_step(D, kernel, lanes, s, nullptr));
      --left;
      cudaGraphExec_t ex = nullptr;
      uint64_t nk = 0;
      SPMVB_TRY(peer_graph(D, kernel, lanes, &ex, &nk));
      for (; left >= 2; left -= 2) {
        SPMVB_TRY_CUDA(cudaGraphLaunch(ex, s));
        count_launch(nk);
      }
    }
    for (; left > 0; --left) SPMVB_TRY(peer_step(D, kernel, lanes, s, nullptr));
    return SPMVB_OK;
  }
  // NCCL exchange: from two steps on, one eager step, then replays of the
  // captured step (no host enqueue work between steps).
  int left = iters;
  if (left >= 2 && graphs_enabled()) {
    SPMVB_TRY(dist_step(D, kernel, lanes, s));
    --left;
    cudaGraphExec_t ex = nullptr;
    uint64_t nk = 0;
    SPMVB_TRY(nccl_graph(D, kernel, lanes, &ex, &nk));
    for (; left > 0; --left) {
      SPMVB_TRY_CUDA(cudaGraphLaunch(ex, s));
      count_launch(nk);
    }
  }
  for (; left > 0; --left) SPMVB_TRY(dist_step(D, kernel, lanes, s));
  return SPMVB_OK;
}

spmvb_status spmvb_dist_iterate_timed(spmvb_dist D, spmvb_kernel kernel, int lanes, int iters, void* stream,
                                      double* kernel_ms, double* step_ms) {
  clear_error();
  if (!D || iters < 0 || !kernel_ms || !step_ms) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bad argument");
  if (D->broken) return fail(SPMVB_ERR_TIMEOUT, "an earlier peer wait gave up; recreate the handle");
  DeviceGuard g(D->ctx->device);
  auto s = static_cast<cudaStream_t>(stream);
  *kernel_ms = 0.0;
  *step_ms = 0.0;
  if (iters == 0) return SPMVB_OK;
  // Steps are enqueued back to back (no host synchronization between them);
  // event i*2 opens step i, i*2+1 follows its SpMV, the last closes the run.
  struct Events {
    std::vector<cudaEvent_t> e;
    ~Events() {
      for (auto v : e)
        if (v) cudaEventDestroy(v);
    }
  } ev;
  ev.e.resize(size_t(2) * iters + 1, nullptr);
  for (auto& v : ev.e) SPMVB_TRY_CUDA(cudaEventCreate(&v));
  for (int it = 0; it < iters; ++it) {
    SPMVB_TRY_CUDA(cudaEventRecord(ev.e[2 * it], s));
    if (D->peer) {
      SPMVB_TRY(peer_step(D, kernel, lanes, s, ev.e[2 * it + 1]));
    } else {
      SPMVB_TRY(spmvb_spmv(D->local, kernel, lanes, 4, D->x_pad.get(), D->y_loc.get(), D->dtype, s));
      SPMVB_TRY_CUDA(cudaEventRecord(ev.e[2 * it + 1], s));
      if (D->nranks > 1) {
        const ncclDataType_t t = D->dtype == SPMVB_F64 ? ncclFloat64 : ncclFloat32;
        SPMVB_TRY(nccl_enqueued(D->comm, ncclAllGather(D->y_loc.get(), D->x_pad.get(), size_t(D->max_rows), t, D->comm, s),
                                "ncclAllGather"));
      } else {
        SPMVB_TRY_CUDA(cudaMemcpyAsync(D->x_pad.get(), D->y_loc.get(), size_t(D->max_rows) * dtype_size(D->dtype),
                                       cudaMemcpyDeviceToDevice, s));
      }
    }
  }
  SPMVB_TRY_CUDA(cudaEventRecord(ev.e[2 * iters], s));
  SPMVB_TRY_CUDA(cudaEventSynchronize(ev.e[2 * iters]));
  if (D->peer) SPMVB_TRY(peer_check(D, s));
  double k_ms = 0.0;
  for (int it = 0; it < iters; ++it) {
    float a = 0.f;
    SPMVB_TRY_CUDA(cudaEventElapsedTime(&a, ev.e[2 * it], ev.e[2 * it + 1]));
    k_ms += a;
  }
  float b = 0.f;
  SPMVB_TRY_CUDA(cudaEventElapsedTime(&b, ev.e[0], ev.e[2 * iters]));
  *kernel_ms = k_ms;
  *step_ms = b;
  return SPMVB_OK;
}

spmvb_status spmvb_dist_get_x(spmvb_dist D, void* h_x, void* stream) {
  clear_error();
  if (!D || (D->m && !h_x)) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  if (D->broken) return fail(SPMVB_ERR_TIMEOUT, "an earlier peer wait gave up; recreate the handle");
  DeviceGuard g(D->ctx->device);
  const size_t es = dtype_size(D->dtype);
  std::vector<unsigned char> pad(size_t(D->nranks) * D->max_rows * es);
  auto s = static_cast<cudaStream_t>(stream);
  // Peer exchange: the last step's barrier saw every peer's stores land.
  const void* src = D->peer ? x_buf(D, D->cur) : D->x_pad.get();
  if (!pad.empty()) SPMVB_TRY_CUDA(cudaMemcpyAsync(pad.data(), src, pad.size(), cudaMemcpyDeviceToHost, s));
  SPMVB_TRY_CUDA(cudaStreamSynchronize(s));
  if (D->peer) SPMVB_TRY(peer_check(D, s));
  for (int r = 0; r < D->nranks; ++r) {
    const int32_t b = D->bounds[r], cnt = D->bounds[r + 1] - b;
    std::memcpy(static_cast<unsigned char*>(h_x) + size_t(b) * es, pad.data() + size_t(r) * D->max_rows * es, size_t(cnt) * es);
  }
  return SPMVB_OK;
}

spmvb_status spmvb_dist_power_iterate(spmvb_dist D, spmvb_kernel kernel, int lanes, int iters, double* h_lambda,
                                      void* stream) {
  clear_error();
  if (!D || iters < 1 || !h_lambda) return fail(SPMVB_ERR_INVALID_ARGUMENT, "bad argument");
  if (D->broken) return fail(SPMVB_ERR_TIMEOUT, "an earlier peer wait gave up; recreate the handle");
  DeviceGuard g(D->ctx->device);
  auto s = static_cast<cudaStream_t>(stream);
  const int parts = norm_blocks(D->m);
  if (!D->bounds_dev.get()) {
    SPMVB_TRY(upload(D->bounds_dev, D->bounds.data(), D->bounds.size() * 4, D->bounds.size() * 4));
    SPMVB_TRY(D->norm_work.alloc(size_t(parts + 1) * 8));
  }
  double* partials = D->norm_work.as<double>();
  double* norm = partials + parts;
  for (int it = 0; it < iters; ++it) {
    void* x;
    if (D->peer) {
      SPMVB_TRY(peer_step(D, kernel, lanes, s, nullptr));
      x = x_buf(D, D->cur);
    } else {
      SPMVB_TRY(dist_step(D, kernel, lanes, s));
      x = D->x_pad.get();
    }
    // Every rank now holds the whole product: each takes its norm (same
    // bits everywhere) and scales its own copy, so no other collective runs.
    // Peers store only into the other x buffer, never into this one.
    SPMVB_TRY(launch_norm_and_scale(D->dtype, x, D->m, D->bounds_dev.as<int>(), D->nranks, D->max_rows, partials,
                                    norm, D->ctx->sm_count, s));
  }
  SPMVB_TRY_CUDA(cudaMemcpyAsync(h_lambda, norm, 8, cudaMemcpyDeviceToHost, s));
  SPMVB_TRY_CUDA(cudaStreamSynchronize(s));
  if (D->peer) SPMVB_TRY(peer_check(D, s));
  return SPMVB_OK;
}

spmvb_status spmvb_dist_get_info(spmvb_dist D, int32_t* row_begin, int32_t* row_end, int32_t* max_rows,
                                 int64_t* local_nnz) {
  clear_error();
  if (!D) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  if (row_begin) *row_begin = D->bounds[D->rank];
  if (row_end) *row_end = D->bounds[D->rank + 1];
  if (max_rows) *max_rows = D->max_rows;
  if (local_nnz) *local_nnz = D->local->nnz;
  return SPMVB_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Host-buffer product over the row shards: every rank passes its own rows'
// slice of x (host) and receives its rows of y (host). On the device the
// slices are all-gathered over NVLink (ncclAllGather, in place into the
// padded x of the call's slot), so each entry of x crosses PCIe once per job
// instead of once per GPU. Slots as in spmvb_pipeline (pipeline.cpp): each
// has its own stream, padded x and staging y; every all-gather runs on one
// communication stream, in submit order, which is the same on every rank.
// ---------------------------------------------------------------------------
struct spmvb_dist_pipeline_st {
  spmvb_dist D = nullptr;  // null once the dist handle was destroyed first
  int device = 0;
  struct Slot {
    cudaStream_t stream = nullptr;
    cudaEvent_t copied = nullptr, gathered = nullptr, done = nullptr;
    DevBuf x, y;
    bool used = false;
  };
  std::vector<Slot> slots;
  cudaStream_t comm = nullptr;
  cudaEvent_t fork = nullptr;
  int next = 0;

  ~spmvb_dist_pipeline_st() {
    if (comm) cudaStreamSynchronize(comm);
    for (auto& s : slots) {
      if (s.stream) cudaStreamSynchronize(s.stream);
      for (cudaEvent_t e : {s.copied, s.gathered, s.done})
        if (e) cudaEventDestroy(e);
      if (s.stream) cudaStreamDestroy(s.stream);
    }
    if (comm) cudaStreamDestroy(comm);
    if (fork) cudaEventDestroy(fork);
  }
};

// The dist handle goes first: let the pipeline's work finish (its kernels
// read the handle's matrix and its all-gathers use the handle's
// communicator), then make its later calls fail.
static void detach_pipeline(spmvb_dist_pipeline_st* P) {
  if (P->comm) cudaStreamSynchronize(P->comm);
  for (auto& s : P->slots)
    if (s.stream) cudaStreamSynchronize(s.stream);
  P->D = nullptr;
}


extern "C" {

spmvb_status spmvb_dist_pipeline_create(spmvb_dist D, int depth, spmvb_dist_pipeline* out) {
  clear_error();
  if (!D || !out) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null argument");
  if (depth < 1 || depth > 16) return fail(SPMVB_ERR_INVALID_ARGUMENT, "depth must be in [1, 16]");
  if (D->peer) return fail(SPMVB_ERR_UNSUPPORTED, "the host-buffer product runs on the NCCL exchange, not after enable_peer");
  *out = nullptr;
  DeviceGuard g(D->ctx->device);
  auto P = std::make_unique<spmvb_dist_pipeline_st>();
  P->D = D;
  P->device = D->ctx->device;
  P->slots.resize(depth);
  const size_t es = dtype_size(D->dtype);
  SPMVB_TRY_CUDA(cudaStreamCreateWithFlags(&P->comm, cudaStreamNonBlocking));
  SPMVB_TRY_CUDA(cudaEventCreateWithFlags(&P->fork, cudaEventDisableTiming));
  for (auto& s : P->slots) {
    SPMVB_TRY_CUDA(cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking));
    for (cudaEvent_t* e : {&s.copied, &s.gathered, &s.done})
      SPMVB_TRY_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
    SPMVB_TRY(s.x.alloc(size_t(std::max(D->nranks * D->max_rows, 1)) * es));
    SPMVB_TRY(s.y.alloc(size_t(std::max(D->max_rows, 1)) * es));
  }
  D->pipelines.push_back(P.get());
  *out = P.release();
  return SPMVB_OK;
}

static const char* kDetached = "the pipeline's dist handle was destroyed";

spmvb_status spmvb_dist_pipeline_fork(spmvb_dist_pipeline P, void* stream) {
  clear_error();
  if (!P) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null pipeline");
  if (!P->D) return fail(SPMVB_ERR_INVALID_ARGUMENT, kDetached);
  DeviceGuard g(P->device);
  SPMVB_TRY_CUDA(cudaEventRecord(P->fork, static_cast<cudaStream_t>(stream)));
  SPMVB_TRY_CUDA(cudaStreamWaitEvent(P->comm, P->fork, 0));
  for (auto& s : P->slots) SPMVB_TRY_CUDA(cudaStreamWaitEvent(s.stream, P->fork, 0));
  return SPMVB_OK;
}

spmvb_status spmvb_dist_pipeline_submit(spmvb_dist_pipeline P, spmvb_kernel kernel, int lanes,
                                        const void* h_x_local, void* h_y_local) {
  clear_error();
  if (!P) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null pipeline");
  if (!P->D) return fail(SPMVB_ERR_INVALID_ARGUMENT, kDetached);
  spmvb_dist D = P->D;
  const int32_t rows = D->bounds[D->rank + 1] - D->bounds[D->rank];
  if (rows && (!h_x_local || !h_y_local)) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null host buffer");
  if (kernel < 0 || kernel >= SPMVB_KERNEL_COUNT) return fail(SPMVB_ERR_INVALID_ARGUMENT, "unknown kernel id");
  DeviceGuard g(D->ctx->device);
  SPMVB_TRY(spmvb_matrix_prepare(D->local, kernel, 0));
  auto& s = P->slots[P->next];
  P->next = (P->next + 1) % static_cast<int>(P->slots.size());
  const size_t es = dtype_size(D->dtype);
  unsigned char* mine = s.x.as<unsigned char>() + size_t(D->rank) * D->max_rows * es;
  if (rows) SPMVB_TRY_CUDA(cudaMemcpyAsync(mine, h_x_local, size_t(rows) * es, cudaMemcpyHostToDevice, s.stream));
  if (D->nranks > 1) {
    SPMVB_TRY_CUDA(cudaEventRecord(s.copied, s.stream));
    SPMVB_TRY_CUDA(cudaStreamWaitEvent(P->comm, s.copied, 0));
    const ncclDataType_t t = D->dtype == SPMVB_F64 ? ncclFloat64 : ncclFloat32;
    SPMVB_TRY(nccl_enqueued(D->comm, ncclAllGather(mine, s.x.get(), size_t(D->max_rows), t, D->comm, P->comm),
                            "ncclAllGather(x slices)"));
    SPMVB_TRY_CUDA(cudaEventRecord(s.gathered, P->comm));
    SPMVB_TRY_CUDA(cudaStreamWaitEvent(s.stream, s.gathered, 0));
  }
  void* y_direct = (rows && stores_y_once(kernel)) ? mapped_host_ptr(h_y_local) : nullptr;
  if (y_direct) {
    SPMVB_TRY(spmvb_spmv(D->local, kernel, lanes, 4, s.x.get(), y_direct, D->dtype, s.stream));
  } else {
    SPMVB_TRY(spmvb_spmv(D->local, kernel, lanes, 4, s.x.get(), s.y.get(), D->dtype, s.stream));
    if (rows) SPMVB_TRY_CUDA(cudaMemcpyAsync(h_y_local, s.y.get(), size_t(rows) * es, cudaMemcpyDeviceToHost, s.stream));
  }
  SPMVB_TRY_CUDA(cudaEventRecord(s.done, s.stream));
  s.used = true;
  return SPMVB_OK;
}

spmvb_status spmvb_dist_pipeline_join(spmvb_dist_pipeline P, void* stream) {
  clear_error();
  if (!P) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null pipeline");
  if (!P->D) return fail(SPMVB_ERR_INVALID_ARGUMENT, kDetached);
  DeviceGuard g(P->device);
  for (auto& s : P->slots)
    if (s.used) SPMVB_TRY_CUDA(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), s.done, 0));
  return SPMVB_OK;
}

spmvb_status spmvb_dist_pipeline_wait(spmvb_dist_pipeline P) {
  clear_error();
  if (!P) return fail(SPMVB_ERR_INVALID_ARGUMENT, "null pipeline");
  if (!P->D) return fail(SPMVB_ERR_INVALID_ARGUMENT, kDetached);
  DeviceGuard g(P->device);
  SPMVB_TRY_CUDA(cudaStreamSynchronize(P->comm));
  for (auto& s : P->slots) SPMVB_TRY_CUDA(cudaStreamSynchronize(s.stream));
  return check_err_word(P->D->ctx, P->slots[0].stream);
}

spmvb_status spmvb_dist_pipeline_destroy(spmvb_dist_pipeline P) {
  clear_error();
  if (!P) return SPMVB_OK;
  DeviceGuard g(P->device);
  if (P->D) {
    auto& v = P->D->pipelines;
    v.erase(std::remove(v.begin(), v.end(), P), v.end());
  }
  delete P;
  return SPMVB_OK;
}

}  // extern "C"
