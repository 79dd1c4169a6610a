// Exchange buffer of one decode session split over several GPUs: each
// rank's buffer is peer-mapped on every rank (torch symmetric memory), and
// ranks write their contributions into the others' buffers with plain peer
// stores over NVLink, then raise a counter with a system-scope atomic.
// Used by the persistent kernel (mega.cuh) and by the standalone kernels of
// the sharded graph schedule (attn_shard.cuh, moe.cuh k_down).
#pragma once
#include "attn_core.cuh"
#include "qdot.cuh"

namespace rec {

// Exchange buffer of one rank (identical layout on every rank); two copies
// of everything, selected by the parity of the global layer-step counter.
constexpr int kMaxWorld = 8;
// Waits on other GPUs: ranks launch independently, so allow more host jitter
// than for waits inside one GPU (still bounded: a few seconds).
constexpr uint32_t kPeerSpinLimit = kSpinLimit * 8;
constexpr int kMaxGrid = 1024;
constexpr int kXchMaxTopK = 8;  // expert slots per token in the exchange (= kMaxTopK)
struct XchLayout {
  size_t head_cnt;  // unsigned [2][Hq]: super-chunk partials received per head
  size_t xcnt;      // unsigned [2][kMaxGrid]: expert-output contributions received per CTA
  size_t supers;    // float [2][Hq][n_super][132]
  size_t xd;        // bf16 [2][kXchMaxTopK][H]: per-slot expert outputs
  size_t total;
  int hq, n_super, H;
};
inline __host__ __device__ size_t xch_align(size_t x) { return (x + 255) / 256 * 256; }
inline __host__ __device__ XchLayout xch_layout(int hq, int n_super, int H) {
  XchLayout x;
  x.hq = hq;
  x.n_super = n_super;
  x.H = H;
  x.head_cnt = 0;
  x.xcnt = xch_align(x.head_cnt + size_t(2) * hq * 4);
  x.supers = xch_align(x.xcnt + size_t(2) * kMaxGrid * 4);
  x.xd = xch_align(x.supers + size_t(2) * hq * n_super * kPartialFloats * 4);
  x.total = xch_align(x.xd + size_t(2) * kXchMaxTopK * H * 2);
  return x;
}
__device__ __forceinline__ unsigned* xch_head_cnt(uint8_t* b, const XchLayout& x, int par, int h) {
  return reinterpret_cast<unsigned*>(b + x.head_cnt) + par * x.hq + h;
}
__device__ __forceinline__ unsigned* xch_xcnt(uint8_t* b, const XchLayout& x, int par, int cta) {
  return reinterpret_cast<unsigned*>(b + x.xcnt) + par * kMaxGrid + cta;
}
__device__ __forceinline__ float* xch_super(uint8_t* b, const XchLayout& x, int par, int h, int s) {
  return reinterpret_cast<float*>(b + x.supers) + ((size_t(par) * x.hq + h) * x.n_super + s) * kPartialFloats;
}
__device__ __forceinline__ uint16_t* xch_xd(uint8_t* b, const XchLayout& x, int par, int slot) {
  return reinterpret_cast<uint16_t*>(b + x.xd) + (size_t(par) * kXchMaxTopK + slot) * x.H;
}


__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

}  // namespace rec
