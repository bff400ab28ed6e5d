// sm100_primitives.cuh -- thin inline-PTX wrappers for the sm_100a features
// the kernels use: mbarriers, 1D bulk copies (TMA) global->shared, L2 bulk
// prefetch, streaming loads and packed f32x2 arithmetic.
//
// No multicast form is used anywhere (every bulk copy reads this GPU's own
// global memory into this CTA's own shared memory).
#pragma once

#include <cstdint>

namespace to_b200 {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Arrive once and announce `bytes` of transaction to be completed by bulk copies.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait on one phase of an mbarrier.  Returns false if `max_polls`
// try_wait probes (each one a hardware-bounded suspend) all failed.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint32_t max_polls) {
  for (uint32_t n = 0; n < max_polls; ++n)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// 1D bulk copy global -> this CTA's shared memory, completing on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 bulk prefetch of `bytes` (rounded down to 16) at 16-byte aligned `p`.
__device__ __forceinline__ void l2_prefetch_bulk(const void* p, uint32_t bytes) {
  bytes &= ~15u;
  if (bytes == 0) return;
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

template <typename T>
__device__ __forceinline__ T ld_stream(const T* p) {
  return __ldg(p);
}

// ---- two-lane values: packed f32x2 on sm_100a, plain pairs otherwise ----
template <typename T>
struct V2;
template <>
struct V2<float> {
  float2 v;
};
template <>
struct V2<double> {
  double2 v;
};

__device__ __forceinline__ V2<float> mk2(float a, float b) { return {make_float2(a, b)}; }
__device__ __forceinline__ V2<double> mk2(double a, double b) { return {make_double2(a, b)}; }
__device__ __forceinline__ V2<float> fma2(V2<float> a, V2<float> b, V2<float> c) {
  return {__ffma2_rn(a.v, b.v, c.v)};
}
__device__ __forceinline__ V2<float> mul2(V2<float> a, V2<float> b) {
  return {__fmul2_rn(a.v, b.v)};
}
__device__ __forceinline__ V2<float> add2(V2<float> a, V2<float> b) {
  return {__fadd2_rn(a.v, b.v)};
}
__device__ __forceinline__ V2<double> fma2(V2<double> a, V2<double> b, V2<double> c) {
  return {make_double2(fma(a.v.x, b.v.x, c.v.x), fma(a.v.y, b.v.y, c.v.y))};
}
__device__ __forceinline__ V2<double> mul2(V2<double> a, V2<double> b) {
  return {make_double2(a.v.x * b.v.x, a.v.y * b.v.y)};
}
__device__ __forceinline__ V2<double> add2(V2<double> a, V2<double> b) {
  return {make_double2(a.v.x + b.v.x, a.v.y + b.v.y)};
}
// scalar overloads so one template body serves single points too
__device__ __forceinline__ float fma2(float a, float b, float c) { return fmaf(a, b, c); }
__device__ __forceinline__ float mul2(float a, float b) { return a * b; }
__device__ __forceinline__ float add2(float a, float b) { return a + b; }
__device__ __forceinline__ double fma2(double a, double b, double c) { return fma(a, b, c); }
__device__ __forceinline__ double mul2(double a, double b) { return a * b; }
__device__ __forceinline__ double add2(double a, double b) { return a + b; }

}  // namespace to_b200

namespace to_b200 {

// L2 cache policy that evicts first: for data streamed exactly once.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void l2_prefetch_bulk_hint(const void* p, uint32_t bytes,
                                                      uint64_t policy) {
  bytes &= ~15u;
  if (bytes == 0) return;
  asm volatile("cp.async.bulk.prefetch.L2.global.L2::cache_hint [%0], %1, %2;" ::"l"(p),
               "r"(bytes), "l"(policy)
               : "memory");
}

}  // namespace to_b200
