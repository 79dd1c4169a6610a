// Attention exchange of a decode session split over several GPUs on the
// graph schedule (standalone kernels; the persistent kernel has its own copy
// of this exchange in mega.cuh).
//
// Rank r holds the cache of super-chunks [super_lo, super_hi) (64 blocks of
// 256 tokens each) and computes their item partials with k_attn_partial.
//   k_attn_combine_xch: one warp per (q head, local super-chunk) folds the
//     super-chunk's items in order, stores the partial into every rank's
//     exchange buffer with plain peer stores (NVLink); after a warp barrier
//     lane 0 fences at system scope and raises each rank's per-head counter
//     with a system-scope atomic.  The warp of (head h, first local slot)
//     then waits (bounded) until its own counter holds every super-chunk of
//     the context, folds [sink] and the super-chunks in order -- the
//     single-GPU combine, so every rank's output equals the one-GPU output
//     bit for bit -- writes the output and resets the counter.  Every CTA of
//     the grid is resident while it waits (32 x local-slot one-warp CTAs),
//     and the next kernel launches only after each of them has started.
// The exchange slots alternate between two copies by the parity of the
// global layer step (steps completed, a device counter, times n_layers plus
// the layer), so a rank one layer ahead never overwrites data a peer is
// still reading.  A wait that runs out records kStatusCounterTimeout.
// Reference: split-KV partials and the LSE merge (megakernel.py:276-318,
// 619-693); BASELINE configs 2 and 4 (split-KV across GPUs).
#pragma once
#include "attn.cuh"
#include "xch.cuh"

namespace rec {

struct AttnXchArgs {
  const float* partials;  // this rank's item partials [Hq, items_cap(capacity), 132], local item index
  int capacity;           // local cache capacity
  int token_base, super_lo, super_hi;
  const int* position;    // global position p of the step (T = p + 1)
  const int* seq;         // steps completed (device counter): exchange parity
  int layer, n_layers;
  int world, rank, hq;
  uint8_t* xch[kMaxWorld];
  XchLayout xl;
  const uint16_t* sinks;  // bf16 [Hq] or null
  uint16_t* out;          // bf16 [Hq * 128]
  int* status;
  int pdl;                // launched as a programmatic dependent of the previous kernel
};

__device__ __forceinline__ int xch_layer_parity(const AttnXchArgs& a) {
  return int((unsigned(*a.seq) * unsigned(a.n_layers) + unsigned(a.layer)) & 1u);
}

// Items and super-chunks of a context of T tokens (the standalone kernels' plan).
struct AttnCounts {
  int nblk, nbi, n_items, per_super, n_super;
};
__device__ __forceinline__ AttnCounts attn_counts(int T) {
  AttnCounts c;
  c.nblk = (T + kAttBlock - 1) / kAttBlock;
  c.nbi = item_blocks(c.nblk);
  c.n_items = (c.nblk + c.nbi - 1) / c.nbi;
  c.per_super = super_items(c.nblk);
  c.n_super = (c.n_items + c.per_super - 1) / c.per_super;
  return c;
}

__global__ void __launch_bounds__(32) k_attn_combine_xch(const AttnXchArgs a) {
  const int lane = threadIdx.x;
  if (a.pdl) grid_wait();  // the item partials of k_attn_partial
  grid_launch_dependents();
  const AttnCounts C = attn_counts(*a.position + 1);
  const int h = blockIdx.x, s = a.super_lo + blockIdx.y;
  const int par = xch_layer_parity(a);
  if (s < min(a.super_hi, C.n_super)) {
    const int item0 = a.token_base / (kAttBlock * C.nbi);
    const int icap = items_cap(a.capacity);
    Partial4 P = empty_partial();
    fold_partials(P, a.partials + size_t(h) * icap * kPartialFloats, s * C.per_super - item0,
                  min((s + 1) * C.per_super, C.n_items) - item0);
    for (int q = 0; q < a.world; ++q) store_partial(xch_super(a.xch[q], a.xl, par, h, s), P);
    __syncwarp();
    if (lane == 0) {
      __threadfence_system();  // cumulative over the warp's stores (ordered by the warp barrier)
      for (int q = 0; q < a.world; ++q) atomicAdd_system(xch_head_cnt(a.xch[q], a.xl, par, h), 1u);
    }
  }
  if (blockIdx.y != 0) return;
  // CTA (h, 0) of every rank (present even when the rank holds no
  // super-chunk of this context yet): wait for every super-chunk of head h,
  // then the single-GPU combine
  uint8_t* own = a.xch[a.rank];
  unsigned* cnt = xch_head_cnt(own, a.xl, par, h);
  int ok = 1;
  if (lane == 0) {
    uint32_t spins = 0;
    while (ld_acquire_sys_u32(cnt) < unsigned(C.n_super)) {
      if (++spins > kPeerSpinLimit) {
        report(a.status, kStatusCounterTimeout);
        ok = 0;
        break;
      }
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (!ok) return;
  __syncwarp();
  Partial4 F = empty_partial();
  if (a.sinks) {
    F.m = bf(a.sinks[h]);
    F.l = 1.0f;
  }
  fold_partials(F, xch_super(own, a.xl, par, h, 0), 0, C.n_super);
  uint2 o;
  o.x = uint32_t(to_bf(__fdiv_rn(F.a[0], F.l))) | (uint32_t(to_bf(__fdiv_rn(F.a[1], F.l))) << 16);
  o.y = uint32_t(to_bf(__fdiv_rn(F.a[2], F.l))) | (uint32_t(to_bf(__fdiv_rn(F.a[3], F.l))) << 16);
  *reinterpret_cast<uint2*>(a.out + h * 128 + 4 * lane) = o;
  __syncwarp();
  if (lane == 0) *reinterpret_cast<volatile unsigned*>(cnt) = 0u;
}

}  // namespace rec
