// Shared device helpers for the select-step kernels: bulk copies with
// mbarriers and bounded waits, exact division, block reductions and sorts.
#pragma once
#include <stdint.h>
#include <cuda_runtime.h>

namespace yapd {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegInf = -__builtin_inff();

// --------------------------------------------------------------------- math

// 2^x on the SFU (PTX ex2.approx, relative error about 2^-22).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Correctly rounded a / b from the correctly rounded reciprocal rb = RN(1/b):
// q = RN(a*rb); r = a - b*q (exact with one FMA); RN(q + r*rb) (Markstein,
// IBM J. Res. Dev. 34(1), 1990).  Outside the normal range it defers to the
// IEEE divide.
__device__ __forceinline__ float div_rn(float a, float b, float rb) {
  const float q = __fmul_rn(a, rb);
  const float r = __fmaf_rn(-q, b, a);
  const float q2 = __fmaf_rn(r, rb, q);
  const float aq = fabsf(q2);
  if (!(aq > 1e-30f && aq < 1e30f)) return (a == 0.0f) ? q2 : __fdiv_rn(a, b);
  return q2;
}

// Order-preserving map float -> uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t ord_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord_key_inv(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Two fp32 values in one 64-bit register pair, for the sm_100 packed
// arithmetic (add/fma .f32x2: both halves rounded exactly as the scalar ops).
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// The two bf16 halves of w as a packed fp32 pair (exact).
__device__ __forceinline__ unsigned long long f2_bf16(uint32_t w) { return f2_pack(bf16lo(w), bf16hi(w)); }

// ------------------------------------------------------------ bulk / mbarrier

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Global -> shared bulk copy completing on `bar` (no multicast, CTA-local).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// As mbar_try_wait, suspending the thread for up to `hint_ns` nanoseconds
// while the phase is incomplete.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Hint: bring [src, src + bytes) into L2 (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait for phase `parity` of `bar`, giving up after `limit_ns` nanoseconds;
// a negative limit gives up without waiting (the failure path, for tests).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int64_t limit_ns) {
  if (limit_ns < 0) return false;
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    // the thread sleeps in the wait until the phase completes (or 20 us pass)
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (globaltimer_ns() - t0 > (uint64_t)limit_ns) return false;
  }
}

// ---------------------------------------------------------------- reductions

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Bitonic sort of one value per lane across a warp, DESCENDING.
__device__ __forceinline__ unsigned long long warp_bitonic_desc(unsigned long long x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const unsigned long long y = __shfl_xor_sync(0xffffffffu, x, j);
      const bool up = ((lane & k) == 0);        // this pair sorts descending
      const bool lower = ((lane & j) == 0);     // this lane holds the first slot
      const bool take_max = (up == lower);
      x = take_max ? (x > y ? x : y) : (x < y ? x : y);
    }
  }
  return x;
}

// Ascending bitonic sort of one float per lane across a warp (values only).
__device__ __forceinline__ float warp_bitonic_asc_f(float x) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 2; k <= 32; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      const float y = __shfl_xor_sync(0xffffffffu, x, j);
      const bool up = ((lane & k) == 0);
      const bool lower = ((lane & j) == 0);
      const bool take_min = (up == lower);
      x = take_min ? fminf(x, y) : fmaxf(x, y);
    }
  }
  return x;
}

}  // namespace yapd

namespace yapd {

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Named barrier `id` over `count` threads (a multiple of the warp size).
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

}  // namespace yapd
