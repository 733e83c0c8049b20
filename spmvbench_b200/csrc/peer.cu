// Kernels of the peer-memory exchange for row-sharded iterated SpMV (no
// reference counterpart; the reference is single-GPU).
//
// Each rank maps every other rank's x buffers and phase counters (CUDA IPC,
// set up by spmvb_dist_enable_peer) and, instead of a separate all-gather,
// stores its slice of the next x straight into every rank's buffer over
// NVLink while it computes it.
//
// Every peer operation ends in a barrier run by the last CTA of its final
// kernel: CTAs count themselves finished with a gpu-scope release (their
// stores, local and remote, ordered before it); the last one fences at
// system scope, writes the new phase number into every other rank's counter
// for this rank (its own count, kept on the device, so a captured graph of
// steps replays unchanged), then waits until every other rank's counter for
// it reaches the same phase. The next kernel on the stream starts after
// that, so it reads x with no wait of its own, and a rank stores into a
// peer's x buffer only after that peer has finished the step that read it.
//
//   ell_rows_peer  one launch per step: ELL rows (same order as ell_rows, so
//                  bit-identical to csr_omp), each row's sum stored to every
//                  rank, barrier. Each thread takes 4 rows in turn on a shard
//                  of at most 160k rows, else 1 (SPMVB_PEER_ROWS_PER_THREAD
//                  overrides); SPMVB_PEER_CTA_FENCE=1 makes every CTA fence
//                  its own stores at system scope before arriving (slower at
//                  8 ranks, off by default).
//   peer_push      after a non-fused SpMV: copy the local slice to every
//                  rank, barrier.
//   peer_barrier   barrier only.
//
// The wait is bounded by a wall-clock limit (%globaltimer) and an iteration
// cap; a wait that gives up writes kErrPeerWait to the context error word.
// Once the word is set no barrier publishes or waits, so every later step
// and every other rank gives up too instead of reading stale x.
#include <algorithm>
#include <cstdint>
#include <cstdlib>

#include "internal.hpp"
#include "spmv_kernels.cuh"

namespace spmvb {

namespace {

constexpr int kErrPeerWait = 3;
constexpr int kPeerRowThreads = 256;
constexpr uint32_t kPeerSpinCap = 1u << 28;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ int ld_volatile(const int* p) { return *static_cast<const volatile int*>(p); }

// One thread: true once every other rank's counter for this rank has
// reached `phase`, false if the error word is (or becomes) set or the wait
// runs past P.timeout_ns.
__device__ bool peer_wait_all(const PeerView& P, unsigned long long phase) {
  const unsigned long long t0 = globaltimer_ns();
  for (int q = 0; q < P.nranks; ++q) {
    if (q == P.rank) continue;
    uint32_t spins = 0;
    while (ld_acquire_sys(P.flags_in + q) < phase) {
      ++spins;
      if ((spins & 63) == 0) {
        if (ld_volatile(P.err) != 0) return false;
        if (globaltimer_ns() - t0 > P.timeout_ns || spins >= kPeerSpinCap) {
          atomicExch(P.err, kErrPeerWait);
          return false;
        }
      }
      __nanosleep(64);
    }
  }
  return true;
}

// All threads of every CTA, after the CTA's last store: the barrier above.
// With P.cta_fence, each CTA first makes its own stores visible at system
// scope (the barrier orders the CTA's threads before thread 0's fence, which
// covers what thread 0 has observed), so the remote stores drain while other
// CTAs still compute and the last CTA's fence only waits for its own.
__device__ void peer_arrive(const PeerView& P) {
  __syncthreads();
  if (threadIdx.x == 0) {
    if (P.cta_fence) __threadfence_system();
    unsigned prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(P.counter) : "memory");
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      atomicExch(P.counter, 0u);
      const unsigned long long phase = *P.phase + 1;
      *P.phase = phase;
      if (ld_volatile(P.err) == 0) {
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q)
          if (q < P.nranks && q != P.rank) st_release_sys(P.flag_out[q], phase);
        peer_wait_all(P, phase);
      }
    }
  }
}

template <typename T>
__device__ __forceinline__ void store_all(const PeerView& P, int i, T v) {
#pragma unroll
  for (int q = 0; q < kMaxRanks; ++q)
    if (q < P.nranks) static_cast<T*>(P.dst[q])[i] = v;
}

// Sum of ELL row `row` with up to 16 of its gathers in flight at once, left
// to right from zero (the order of ell_row_sum, so the same bits).
template <typename T>
__device__ __forceinline__ T ell_row_sum16(const EllView& E, int row, int L, const T* __restrict__ x, uint64_t ps,
                                           uint64_t pk) {
  const T* __restrict__ vals = static_cast<const T*>(E.values);
  T sum = T(0);
  for (int j0 = 0; j0 < L; j0 += 16) {
    T a[16], xv[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      if (j0 + u < L) {
        const int64_t p = row + static_cast<int64_t>(j0 + u) * E.ld;
        a[u] = ld_stream(vals + p, ps);
        xv[u] = ld_keep(x + ld_stream(E.colind + p, ps), pk);
      }
    }
#pragma unroll
    for (int u = 0; u < 16; ++u)
      if (j0 + u < L) sum = add_rn(sum, mul_rn(a[u], xv[u]));
  }
  return sum;
}

// Rows are dealt round-robin over the grid; with a grid smaller than the
// rows, each thread finishes its rows one after another, so the stores to
// the peers leave while the rest of the step is still computing instead of
// in one burst at the end.
template <typename T>
__global__ void __launch_bounds__(kPeerRowThreads) ell_rows_peer(EllView E, const T* __restrict__ x, PeerView P) {
  const uint64_t ps = policy_evict_first();
  const uint64_t pk = policy_evict_last();
  for (int row = blockIdx.x * blockDim.x + threadIdx.x; row < E.m; row += gridDim.x * blockDim.x)
    store_all<T>(P, row, ell_row_sum16<T>(E, row, E.row_lengths[row], x, ps, pk));
  peer_arrive(P);
}

template <typename T>
__global__ void __launch_bounds__(256) peer_push(const T* __restrict__ y, PeerView P) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < P.rows; i += gridDim.x * blockDim.x)
    store_all<T>(P, i, y[i]);
  peer_arrive(P);
}

__global__ void peer_barrier(PeerView P) { peer_arrive(P); }

}  // namespace

// Grid of the grid-stride peer kernels: at most 8 CTAs of 256 threads per
// SM, so few CTAs pay for the barrier's per-CTA release, and at least
// `rows_per_thread` rows per thread.
static int peer_grid(int rows, int sm_count, int rows_per_thread = 1) {
  const int per = std::max(1, rows_per_thread);
  return std::max(1, std::min((rows + 256 * per - 1) / (256 * per), sm_count * 8));
}

static bool peer_cta_fence() {
  static const bool v = [] {
    const char* e = std::getenv("SPMVB_PEER_CTA_FENCE");
    return e && *e == '1';
  }();
  return v;
}

// Rows each thread of the fused SpMV + push takes in turn. A shard of at most
// 160k rows (one row per thread would fill under 40 % of the GPU's threads,
// so every row finishes and pushes at about the same time) gets 4, which
// spreads the remote stores over the kernel: 37.6 against 42.1 us per step at
// 8 ranks x 125k rows. Larger shards keep 1. SPMVB_PEER_ROWS_PER_THREAD
// overrides both.
static int peer_rows_per_thread(int rows) {
  static const int forced = [] {
    const char* e = std::getenv("SPMVB_PEER_ROWS_PER_THREAD");
    const int r = (e && *e) ? std::atoi(e) : 0;
    return r > 0 ? r : 0;
  }();
  if (forced) return forced;
  return rows <= 160000 ? 4 : 1;
}

spmvb_status peer_launch_ell(spmvb_matrix A, const PeerView& P, const void* x, cudaStream_t s) {
  SPMVB_TRY(build_ell(A));
  EllView e;
  e.colind = A->ell_colind.as<int>();
  e.values = A->ell_values.get();
  e.row_lengths = A->ell_rowlen.as<int>();
  e.m = A->m;
  e.n = A->n;
  e.width = A->ell_width;
  e.ld = A->m;
  const int grid = peer_grid(A->m, A->ctx->sm_count, peer_rows_per_thread(A->m));
  PeerView V = P;
  V.cta_fence = peer_cta_fence() ? 1 : 0;
  if (A->dtype == SPMVB_F64)
    ell_rows_peer<double><<<grid, kPeerRowThreads, 0, s>>>(e, static_cast<const double*>(x), V);
  else
    ell_rows_peer<float><<<grid, kPeerRowThreads, 0, s>>>(e, static_cast<const float*>(x), V);
  count_launch();
  SPMVB_TRY_CUDA(cudaGetLastError());
  return SPMVB_OK;
}

spmvb_status peer_launch_push(spmvb_dtype dtype, const void* y, const PeerView& P, int sm_count, cudaStream_t s) {
  const int grid = peer_grid(P.rows, sm_count);
  PeerView V = P;
  V.cta_fence = peer_cta_fence() ? 1 : 0;
  if (dtype == SPMVB_F64)
    peer_push<double><<<grid, 256, 0, s>>>(static_cast<const double*>(y), V);
  else
    peer_push<float><<<grid, 256, 0, s>>>(static_cast<const float*>(y), V);
  count_launch();
  SPMVB_TRY_CUDA(cudaGetLastError());
  return SPMVB_OK;
}

spmvb_status peer_launch_barrier(const PeerView& P, cudaStream_t s) {
  peer_barrier<<<1, 32, 0, s>>>(P);
  count_launch();
  SPMVB_TRY_CUDA(cudaGetLastError());
  return SPMVB_OK;
}

}  // namespace spmvb
