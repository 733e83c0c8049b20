// Device-side building blocks shared by every kernel of the library.
//
// Loads: the matrix arrays are streamed once per SpMV, so they are read
// through the non-coherent path with L1 no-allocate and an L2 evict-first
// policy; x (or the dense X of SpMM) is gathered with an L2 evict-last policy
// so it stays resident in the 126 MB L2 while the stream passes through.
//
// Arithmetic: products and sums use explicit round-to-nearest intrinsics
// (__dmul_rn/__dadd_rn, __fmul_rn/__fadd_rn). That forbids FMA contraction,
// so a kernel that adds in the same order as the reference's csr_omp
// (src/cpu/spmv_cpu.cpp:19-25: sum += Acc(a) * Acc(x), left to right, from 0)
// produces bit-identical results.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace spmvb {

constexpr int kWarp = 32;

// ---- cache policies --------------------------------------------------------
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- streamed (read-once) loads --------------------------------------------
__device__ __forceinline__ int ld_stream(const int* p, uint64_t pol) {
  int r;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.s32 %0, [%1], %2;"
      : "=r"(r) : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ int2 ld_stream2(const int* p, uint64_t pol) {
  int2 r;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.s32 {%0,%1}, [%2], %3;"
      : "=r"(r.x), "=r"(r.y) : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ int4 ld_stream4(const int* p, uint64_t pol) {
  int4 r;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.s32 {%0,%1,%2,%3}, [%4], %5;"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ double ld_stream(const double* p, uint64_t pol) {
  double r;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.f64 %0, [%1], %2;"
      : "=d"(r) : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ float ld_stream(const float* p, uint64_t pol) {
  float r;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.f32 %0, [%1], %2;"
      : "=f"(r) : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ double2 ld_stream2(const double* p, uint64_t pol) {
  double2 r;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.f64 {%0,%1}, [%2], %3;"
      : "=d"(r.x), "=d"(r.y) : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ float2 ld_stream2(const float* p, uint64_t pol) {
  float2 r;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.f32 {%0,%1}, [%2], %3;"
      : "=f"(r.x), "=f"(r.y) : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ float4 ld_stream4(const float* p, uint64_t pol) {
  float4 r;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.f32 {%0,%1,%2,%3}, [%4], %5;"
      : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(p), "l"(pol));
  return r;
}

// ---- gathered (reused) loads -------------------------------------------------
// Scalar gathers keep x in L2 (evict-last) but skip L1 allocation: random
// 8-byte gathers from a multi-MB x hit L1 a few percent of the time.
__device__ __forceinline__ double ld_keep(const double* p, uint64_t pol) {
  double r;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.f64 %0, [%1], %2;"
      : "=d"(r) : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ float ld_keep(const float* p, uint64_t pol) {
  float r;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.f32 %0, [%1], %2;"
      : "=f"(r) : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ double2 ld_keep2(const double* p, uint64_t pol) {
  double2 r;
  asm("ld.global.nc.L2::cache_hint.v2.f64 {%0,%1}, [%2], %3;"
      : "=d"(r.x), "=d"(r.y) : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ float4 ld_keep4(const float* p, uint64_t pol) {
  float4 r;
  asm("ld.global.nc.L2::cache_hint.v4.f32 {%0,%1,%2,%3}, [%4], %5;"
      : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ float2 ld_keep2(const float* p, uint64_t pol) {
  float2 r;
  asm("ld.global.nc.L2::cache_hint.v2.f32 {%0,%1}, [%2], %3;"
      : "=f"(r.x), "=f"(r.y) : "l"(p), "l"(pol));
  return r;
}

// ---- streamed stores ---------------------------------------------------------
template <typename T>
__device__ __forceinline__ void st_stream(T* p, T v) {
  __stcs(p, v);
}

// ---- exact-order arithmetic ----------------------------------------------------
__device__ __forceinline__ double mul_rn(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double add_rn(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }

// One term of the reference inner product: Acc(a) * Acc(x), rounded.
template <typename Acc, typename T>
__device__ __forceinline__ Acc prod(T a, T x) {
  return mul_rn(static_cast<Acc>(a), static_cast<Acc>(x));
}

// Butterfly sum over a group of G lanes (G a power of two <= 32, groups
// aligned within the warp). Every lane of the group ends with the total.
template <int G, typename Acc>
__device__ __forceinline__ Acc group_sum(Acc v) {
#pragma unroll
  for (int off = G / 2; off > 0; off >>= 1)
    v = add_rn(v, __shfl_xor_sync(0xffffffffu, v, off, G));
  return v;
}

// ---- TMA bulk copies and mbarriers (sm_90+ PTX, used on sm_100a) --------------
// Spin limit of every mbarrier wait. try_wait suspends the thread for a
// hardware-chosen interval per attempt, so 2^20 attempts is well over a
// second; a wait that gives up makes the kernel record an error and return.
constexpr uint32_t kWaitLimit = 1u << 20;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// True once the barrier's phase `parity` has completed; false after
// kWaitLimit attempts.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity,
                                          uint32_t limit = kWaitLimit) {
  for (uint32_t i = 0; i < limit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}
}  // namespace spmvb
