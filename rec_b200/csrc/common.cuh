// Shared device helpers for the rec_b200 decode kernels (sm_100a).
//
// Every floating-point step on the decode path is written with an explicit
// rounding (the library is compiled with -fmad=false), so a CPU restatement
// that performs the same operations in the same order reproduces the results
// bit for bit.  The canonical orders are described next to each kernel.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <mutex>
#include <set>
#include <utility>

namespace rec {

// Raises a kernel's dynamic shared-memory limit once per (device, kernel):
// the attribute is per device, so a process that drives several GPUs sets it
// on each of them.  Host only; thread safe.
inline cudaError_t set_smem_limit(const void* kern, size_t smem) {
  static std::mutex mu;
  static std::set<std::pair<int, const void*>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> g(mu);
  if (done.count({dev, kern})) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e == cudaSuccess) done.insert({dev, kern});
  return e;
}

// ----------------------------------------------------------------------------
// Status words.  Kernels never trap: a bounded wait that runs out records a
// code in the session status word and the kernel returns.
// ----------------------------------------------------------------------------
enum : int {
  kStatusOk = 0,
  kStatusBulkTimeout = 1,    // an mbarrier wait on a bulk copy ran out
  kStatusCounterTimeout = 2, // a cross-CTA handoff wait ran out
  kStatusBadToken = 3,       // token id outside the vocabulary
  kStatusBadPosition = 4,    // position outside the KV capacity
};

constexpr uint32_t kSpinLimit = 1u << 22;  // polling bound (seconds at most), then give up

__device__ __forceinline__ void report(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// ----------------------------------------------------------------------------
// bf16 / fp16 conversions (round to nearest even, as torch and MLX do).
// ----------------------------------------------------------------------------
__device__ __forceinline__ float bf(uint16_t v) { return __uint_as_float(uint32_t(v) << 16); }
__device__ __forceinline__ uint16_t to_bf(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float rbf(float f) { return bf(to_bf(f)); }  // round through bf16
__device__ __forceinline__ float hf(uint16_t v) { return __half2float(__ushort_as_half(v)); }

// Scale/bias element type of a quantized tensor: 0 = fp16, 1 = bf16.
template <int SD>
__device__ __forceinline__ float sb(uint16_t v) {
  if constexpr (SD == 0) return hf(v); else return bf(v);
}
// SD == 2: the type is a runtime flag (1 = bf16).
template <int SD>
__device__ __forceinline__ float sb(uint16_t v, int sd_rt) {
  if constexpr (SD == 2) return sd_rt ? bf(v) : hf(v); else return sb<SD>(v);
}

// ----------------------------------------------------------------------------
// Deterministic exp.  Cody-Waite reduction x = n*ln2 + r with ln2 split in a
// 16-bit head and a tail, e^r by its degree-7 Taylor polynomial in Horner form
// (all steps fused multiply-adds), result scaled by 2^n through the exponent
// field.  |r| <= ln2/2 keeps the truncation error below 2^-27.  The same
// sequence of IEEE operations is restated by the CPU oracle.
// exp(-inf) = 0, exp(+inf) = inf, exp(nan) = nan.
// ----------------------------------------------------------------------------
__device__ __forceinline__ float rexp(float x) {
  if (!(x > -104.0f)) return (x != x) ? x : 0.0f;   // also catches -inf
  if (x > 88.8f) return __int_as_float(0x7f800000);
  const float log2e = 1.44269504088896341f;
  const float ln2_hi = 0.693145751953125f;          // 16 significant bits
  const float ln2_lo = 1.42860682030941723e-6f;     // ln2 - ln2_hi
  float n = rintf(__fmul_rn(x, log2e));
  float r = __fmaf_rn(-n, ln2_hi, x);
  r = __fmaf_rn(-n, ln2_lo, r);
  float p = 1.98412698412698413e-4f;                // 1/7!
  p = __fmaf_rn(p, r, 1.38888888888888889e-3f);     // 1/6!
  p = __fmaf_rn(p, r, 8.33333333333333333e-3f);     // 1/5!
  p = __fmaf_rn(p, r, 4.16666666666666667e-2f);     // 1/4!
  p = __fmaf_rn(p, r, 1.66666666666666667e-1f);     // 1/3!
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int e = int(n);
  // split the scale so that results in the subnormal range are formed by
  // two exact-or-single-rounding multiplications
  int e1 = e / 2, e2 = e - e1;
  p = __fmul_rn(p, __int_as_float((e1 + 127) << 23));
  return __fmul_rn(p, __int_as_float((e2 + 127) << 23));
}

// Natural logarithm shared by the kernels and the oracle (the sampler's
// log-sum-exp and Gumbel noise).  Argument reduction x = m * 2^e with m in
// [sqrt(1/2), sqrt(2)), then the atanh series ln m = 2f + 2f(f^2/3 + f^4/5 +
// ... + f^12/13), f = (m-1)/(m+1), by Horner in f^2 with fused
// multiply-adds; ln x = e*ln2_hi + (e*ln2_lo + ln m).  ln(+-0) = -inf,
// ln(x<0) = NaN, ln(inf) = inf.
__device__ __forceinline__ float rlog(float x) {
  if (x != x) return x;
  if (x == 0.0f) return __int_as_float(0xff800000);
  if (x < 0.0f) return __int_as_float(0x7fc00000);
  if (x == __int_as_float(0x7f800000)) return x;
  uint32_t u = __float_as_uint(x);
  int e = 0;
  if (u < 0x00800000u) {  // subnormal: scale by 2^24 (exact)
    u = __float_as_uint(__fmul_rn(x, 16777216.0f));
    e = -24;
  }
  e += int(u >> 23) - 127;
  float m = __uint_as_float((u & 0x007fffffu) | 0x3f800000u);
  if (m > 1.41421353816986084f) {
    m = __fmul_rn(m, 0.5f);
    e += 1;
  }
  const float f = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
  const float f2 = __fmul_rn(f, f);
  float p = 7.69230769230769231e-2f;            // 1/13
  p = __fmaf_rn(p, f2, 9.09090909090909091e-2f);  // 1/11
  p = __fmaf_rn(p, f2, 1.11111111111111111e-1f);  // 1/9
  p = __fmaf_rn(p, f2, 1.42857142857142857e-1f);  // 1/7
  p = __fmaf_rn(p, f2, 2.00000000000000000e-1f);  // 1/5
  p = __fmaf_rn(p, f2, 3.33333333333333333e-1f);  // 1/3
  p = __fmul_rn(p, f2);
  const float f2x = __fmul_rn(2.0f, f);
  const float lnm = __fmaf_rn(f2x, p, f2x);
  const float ef = float(e);
  return __fmaf_rn(ef, 0.693145751953125f, __fmaf_rn(ef, 1.42860682030941723e-6f, lnm));
}

// SiLU factor used by the reference's routed experts:
// tail = 1/(1+exp(|g|)), sigmoid = g<0 ? tail : 1-tail.
__device__ __forceinline__ float rsigmoid(float g) {
  float tail = __fdiv_rn(1.0f, __fadd_rn(1.0f, rexp(fabsf(g))));
  return g < 0.0f ? tail : __fsub_rn(1.0f, tail);
}

// ----------------------------------------------------------------------------
// Warp reductions with a fixed xor-butterfly tree: after the loop every lane
// holds the same value, v(l) + v(l^16) first, then ^8, ^4, ^2, ^1.
// ----------------------------------------------------------------------------
template <int WIDTH = 32>
__device__ __forceinline__ float bfly_sum(float v) {
#pragma unroll
  for (int off = WIDTH / 2; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}
template <int WIDTH = 32>
__device__ __forceinline__ float bfly_max(float v) {
#pragma unroll
  for (int off = WIDTH / 2; off >= 1; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// ----------------------------------------------------------------------------
// mbarrier + bulk async copy (global -> shared) wrappers.
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// Bounded wait.  Returns false when the limit runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
// 16-byte asynchronous copy global -> shared through L2 only (data written
// by other CTAs of the same launch), and the wait for a thread's copies.
__device__ __forceinline__ void cp_async_cg16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// 1-D bulk copy; dst, src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// ----------------------------------------------------------------------------
// Programmatic dependent launch.  Kernels prefetch weights (which no earlier
// kernel writes) before grid_wait(); everything that reads activations comes
// after it.  grid_launch_dependents() lets the next kernel start its prologue.
// ----------------------------------------------------------------------------
__device__ __forceinline__ void grid_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_addr(p)));
  return v;
}
__device__ __forceinline__ uint4 ldg128_nc(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// Coherent 128-bit load of data written by an earlier kernel of this step.
__device__ __forceinline__ uint4 ldg128(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}

}  // namespace rec
