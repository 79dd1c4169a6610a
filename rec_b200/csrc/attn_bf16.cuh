// Decode attention over a bf16 (16-bit) KV cache: the reference's production
// megakernel keeps K and V unquantized in bf16 (megakernel.py:619-693,
// `attention_partial_path_w53`; kv_format "bf16").  Same work items,
// super-chunks and combine as the quantized path (attn.cuh); only the tile
// math differs.
//
// Cache layout: K, V bf16 [Hkv, C, 128] (the RecKVLayer codes pointers; no
// scales or biases).
//
// Canonical order (restated by oracle/rec_oracle.c att_tile_bf16):
//   * qs = fp32(q) * (1/sqrt(128)) in fp32 (q: the bf16 q after its head
//     norm and RoPE; no bf16 rounding of qs, as the reference's bf16 path);
//   * score of the token at tile row r (0..31) = fp32 fused multiply-adds
//     over its 32 four-dim chunks in the order c' = (c + r) mod 32, c = 0..31,
//     dims 4c'..4c'+3 within a chunk (no bf16 rounding of the score);
//   * per tile and head: m' = max(m, tile max); alpha = aexp(m - m');
//     p_r = aexp(s_r - m') (0 for rows outside [first, nvalid));
//     l' = fma(l, alpha, butterfly sum of p over the 32 rows);
//     acc_d' = fma(acc_d, alpha, PV_d), PV_d = fma chain over the valid rows
//     in order, from 0: PV = fma(p_r, v_rd, PV);
//   * warp states, items, super-chunks, sinks and the output as attn.cuh.
// The products and sums are fp32 on the CUDA cores: the tensor cores'
// accumulation order is not restatable.
#pragma once
#include "attn.cuh"

namespace rec {

// A block's 256 rows in four 64-row quarters, one per warp pair: pair q
// (warps 2q, 2q+1) folds tiles 2q, 2q+1 of every block from its own quarter
// slot, and the pairs stream their quarters independently (one pair's copy
// overlaps another pair's math).
constexpr int kBfQuarter = 64;
struct AttnBfSmem {
  alignas(128) uint16_t k[4][kBfQuarter * 128];  // per pair: K rows of its quarter
  alignas(128) uint16_t v[4][kBfQuarter * 128];  // and V rows
  alignas(16) float q[kHeadsPerKv][128];         // scaled queries of the kv head's 8 heads
  alignas(16) float p[kAttWarps][kAttTile][kHeadsPerKv];  // per warp: softmax weights [row][head]
  alignas(16) uint16_t knew[128], vnew[128];     // the new token's K (normed, RoPE'd) and V
  AttnScratch sc;                                // query preparation scratch and the warp-state tree fold
  uint64_t bar[4];                               // per pair: its quarter's K and V copies
  int issued[4];                                 // per pair: a copy of the current block is in flight
  int failed;                                    // a bounded wait ran out
};

// Rows [r0, r0 + 64) of a kv head that some attended position needs (below
// T, and the quarter reaches the window start lo): the count copied (0: none).
__device__ __forceinline__ int bf16_quarter_rows(int r0, int T, int lo) {
  const int n = min(kBfQuarter, T - r0);
  return (n > 0 && r0 + kBfQuarter > lo) ? n : 0;
}
__device__ __forceinline__ void issue_bf16_quarter(AttnBfSmem& sm, int pair, const AttnArgs& a, int g, int r0,
                                                   int n) {
  const size_t row = size_t(g) * a.capacity + size_t(r0) - size_t(a.token_base);
  const uint32_t bytes = uint32_t(n) * 256u;
  mbar_expect_tx(&sm.bar[pair], 2 * bytes);
  bulk_g2s(sm.k[pair], reinterpret_cast<const uint8_t*>(a.k_codes) + row * 256u, bytes, &sm.bar[pair]);
  bulk_g2s(sm.v[pair], reinterpret_cast<const uint8_t*>(a.v_codes) + row * 256u, bytes, &sm.bar[pair]);
}

// Warp w: query of head 8g + w (norm, RoPE, scale) into sm.q[w].
__device__ __forceinline__ void prep_q_bf16(const AttnArgs& a, AttnBfSmem& sm, int g, const float* cs, int warp) {
  const int lane = threadIdx.x & 31;
  const uint16_t* qr = a.qkv + (g * kHeadsPerKv + warp) * 128;
  float x[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) x[j] = bf(__ldcg(reinterpret_cast<const unsigned short*>(qr + 4 * lane + j)));
  if (a.q_norm) head_norm4(x, a.q_norm, a.eps);
  rope4(x, cs, reinterpret_cast<float*>(sm.sc.u.wbuf[warp]));
#pragma unroll
  for (int j = 0; j < 4; ++j) sm.q[warp][4 * lane + j] = __fmul_rn(x[j], kQScale);
}

// Warps 0 (K: head norm, RoPE) and 1 (V): the new token's row of kv head g
// into the cache (row `slot`) and into sm.knew / sm.vnew.
__device__ __forceinline__ void prep_new_bf16(const AttnArgs& a, AttnBfSmem& sm, int g, const float* cs, int warp,
                                              size_t slot) {
  if (warp >= 2) return;
  const int lane = threadIdx.x & 31;
  const bool is_k = warp == 0;
  const uint16_t* src = a.qkv + (a.hq + (is_k ? 0 : a.hkv) + g) * 128;
  float x[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) x[j] = bf(__ldcg(reinterpret_cast<const unsigned short*>(src + 4 * lane + j)));
  if (is_k) {
    if (a.k_norm) head_norm4(x, a.k_norm, a.eps);
    rope4(x, cs, reinterpret_cast<float*>(sm.sc.u.wbuf[warp]));
  }
  uint16_t* dst = is_k ? sm.knew : sm.vnew;
  uint16_t* gdst = reinterpret_cast<uint16_t*>(is_k ? a.k_codes : a.v_codes) + slot * 128;
  const uint2 w = make_uint2(uint32_t(to_bf(x[0])) | (uint32_t(to_bf(x[1])) << 16),
                             uint32_t(to_bf(x[2])) | (uint32_t(to_bf(x[3])) << 16));
  *reinterpret_cast<uint2*>(dst + 4 * lane) = w;
  *reinterpret_cast<uint2*>(gdst + 4 * lane) = w;
}

// Per-warp running state of the bf16 tile: m, l of all 8 heads in every lane;
// acc[4h + j] = head h, dim 4 lane + j (each V element is converted once and
// used for the 8 heads).
struct BfState {
  float m[kHeadsPerKv], l[kHeadsPerKv];
  float acc[32];
};

// The tile whose 32 K / V rows start at kt / vt (rows [first, nvalid) of it
// valid) folded into st.
__device__ __forceinline__ void tile_fold_bf16(const uint16_t* kt, const uint16_t* vt, const float (&q)[8][128],
                                               float (&p_sm)[kAttTile][kHeadsPerKv], int first, int nvalid,
                                               BfState& st) {
  const int lane = threadIdx.x & 31;
  // ---- scores: lane = row
  const uint16_t* krow = kt + lane * 128;
  float s[kHeadsPerKv];
#pragma unroll
  for (int h = 0; h < kHeadsPerKv; ++h) s[h] = 0.0f;
#pragma unroll 4
  for (int c = 0; c < 32; ++c) {
    const int cc = (c + lane) & 31;
    const uint2 kk = *reinterpret_cast<const uint2*>(krow + 4 * cc);
    const float k0 = __uint_as_float(kk.x << 16), k1 = __uint_as_float(kk.x & 0xFFFF0000u);
    const float k2 = __uint_as_float(kk.y << 16), k3 = __uint_as_float(kk.y & 0xFFFF0000u);
#pragma unroll
    for (int h = 0; h < kHeadsPerKv; ++h) {
      const float4 qq = *reinterpret_cast<const float4*>(&q[h][4 * cc]);
      s[h] = __fmaf_rn(qq.x, k0, s[h]);
      s[h] = __fmaf_rn(qq.y, k1, s[h]);
      s[h] = __fmaf_rn(qq.z, k2, s[h]);
      s[h] = __fmaf_rn(qq.w, k3, s[h]);
    }
  }
  // ---- softmax per head (all lanes keep every head's m, l)
  const bool valid = lane >= first && lane < nvalid;
  float alpha[kHeadsPerKv], pr[kHeadsPerKv];
#pragma unroll
  for (int h = 0; h < kHeadsPerKv; ++h) {
    const float sh = valid ? s[h] : -INFINITY;
    const float mn = fmaxf(st.m[h], bfly_max(sh));
    alpha[h] = aexp(__fsub_rn(st.m[h], mn));
    pr[h] = valid ? aexp(__fsub_rn(sh, mn)) : 0.0f;
    st.l[h] = __fmaf_rn(st.l[h], alpha[h], bfly_sum(pr[h]));
    st.m[h] = mn;
  }
  *reinterpret_cast<float4*>(&p_sm[lane][0]) = make_float4(pr[0], pr[1], pr[2], pr[3]);
  *reinterpret_cast<float4*>(&p_sm[lane][4]) = make_float4(pr[4], pr[5], pr[6], pr[7]);
  __syncwarp();
  // ---- P.V: lane l, dims 4l..4l+3 of every head (rows in order)
  float pv[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) pv[i] = 0.0f;
#pragma unroll 4
  for (int r = first; r < nvalid; ++r) {
    const float4 pa = *reinterpret_cast<const float4*>(&p_sm[r][0]);
    const float4 pb = *reinterpret_cast<const float4*>(&p_sm[r][4]);
    const uint2 vv = *reinterpret_cast<const uint2*>(vt + r * 128 + 4 * lane);
    const float v[4] = {__uint_as_float(vv.x << 16), __uint_as_float(vv.x & 0xFFFF0000u),
                        __uint_as_float(vv.y << 16), __uint_as_float(vv.y & 0xFFFF0000u)};
    const float ph[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
#pragma unroll
    for (int h = 0; h < kHeadsPerKv; ++h)
#pragma unroll
      for (int j = 0; j < 4; ++j) pv[4 * h + j] = __fmaf_rn(ph[h], v[j], pv[4 * h + j]);
  }
#pragma unroll
  for (int h = 0; h < kHeadsPerKv; ++h)
#pragma unroll
    for (int j = 0; j < 4; ++j) st.acc[4 * h + j] = __fmaf_rn(st.acc[4 * h + j], alpha[h], pv[4 * h + j]);
  __syncwarp();  // p_sm is rewritten by the next tile
}

// Item partials over a bf16 cache.  Persistent grid, one CTA per SM (the
// four quarter slots take 128 KB); item it = (kv head it % Hkv, item
// i_first + it / Hkv).  Each warp pair waits for its quarter of a block,
// patches the new row into it, folds its two tiles and issues its quarter of
// the next block; the pairs meet only at the item's start and end.
static __global__ void __launch_bounds__(kAttWarps * 32, 1) k_attn_partial_bf16(const AttnArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AttnBfSmem& sm = *reinterpret_cast<AttnBfSmem*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = warp >> 1, half = warp & 1;
  const bool leader = half == 0 && lane == 0;
  volatile int* failed = &sm.failed;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(&sm.bar[i], 1);
    fence_barrier_init();
    sm.sc.qg = -1;
    sm.failed = 0;
  }
  __syncthreads();
  if (a.pdl) grid_wait();
  grid_launch_dependents();
  const int p = *a.position;
  const int T = p + 1;
  if (p < 0 || p >= a.capacity) {
    if (blockIdx.x == 0 && threadIdx.x == 0) report(a.status, kStatusBadPosition);
    return;
  }
  const int nblk = (T + kAttBlock - 1) / kAttBlock;
  const int nbi = item_blocks(nblk);
  const int n_items = (nblk + nbi - 1) / nbi;
  const int lo = window_start(p, a.window);
  const int i_first = lo / (kAttBlock * nbi);
  const int items = max(0, n_items - i_first) * a.hkv;
  const float* cs = a.rope ? a.rope + size_t(p) * 128 : nullptr;
  const int icap = items_cap(a.capacity);
  uint32_t phase = 0;  // parity of this pair's barrier
  bool ok = true;      // this thread's waits all completed
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const int g = it % a.hkv, item = i_first + it / a.hkv;
    const int b0 = item * nbi, b1 = min(b0 + nbi, nblk);
    if (leader) {
      const int r0 = b0 * kAttBlock + kBfQuarter * pair, n = bf16_quarter_rows(r0, T, lo);
      if (n && !*failed) issue_bf16_quarter(sm, pair, a, g, r0, n);
      sm.issued[pair] = n && !*failed;
    }
    if (sm.sc.qg != g) prep_q_bf16(a, sm, g, cs, warp);
    const bool has_new = p >= b0 * kAttBlock && p < b1 * kAttBlock;
    if (has_new) prep_new_bf16(a, sm, g, cs, warp, size_t(g) * a.capacity + size_t(p));
    __syncthreads();
    if (threadIdx.x == 0) sm.sc.qg = g;
    BfState st;
#pragma unroll
    for (int h = 0; h < kHeadsPerKv; ++h) {
      st.m[h] = -INFINITY;
      st.l[h] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) st.acc[i] = 0.0f;
    for (int b = b0; b < b1; ++b) {
      const int r0 = b * kAttBlock + kBfQuarter * pair;
      const int n = bf16_quarter_rows(r0, T, lo);
      // every copy this pair issued is waited for (bounded), whatever the
      // other pairs do; after a failure no further copy is issued
      const bool issued = sm.issued[pair] != 0;
      if (issued) {
        if (mbar_wait(&sm.bar[pair], phase)) {
          phase ^= 1u;
        } else {
          ok = false;
          *failed = 1;
        }
      }
      const int t0 = kAttTile * half;  // this warp's tile inside the quarter
      const int nvalid = min(kAttTile, n - t0), first = max(0, lo - r0 - t0);
      uint16_t* kt = sm.k[pair] + t0 * 128;
      uint16_t* vt = sm.v[pair] + t0 * 128;
      const int new_row = p - r0 - t0;  // the new token's row in this tile, if it is there
      const bool go = __all_sync(0xffffffffu, issued && ok && !*failed);  // uniform over the warp
      if (go && nvalid > first) {
        if (has_new && new_row >= 0 && new_row < kAttTile) {
          *reinterpret_cast<uint2*>(kt + new_row * 128 + 4 * lane) = *reinterpret_cast<const uint2*>(sm.knew + 4 * lane);
          *reinterpret_cast<uint2*>(vt + new_row * 128 + 4 * lane) = *reinterpret_cast<const uint2*>(sm.vnew + 4 * lane);
          __syncwarp();
        }
        tile_fold_bf16(kt, vt, sm.q, sm.p[warp], first, nvalid, st);
      }
      // both warps of the pair are done with the slot (the generic-proxy
      // patch and the reads come before the next bulk copy into it)
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("bar.sync %0, %1;" ::"r"(1 + pair), "r"(64));
      if (leader && b + 1 < b1) {
        const int n1 = bf16_quarter_rows(r0 + kAttBlock, T, lo);
        const bool go1 = n1 && !*failed;
        if (go1) issue_bf16_quarter(sm, pair, a, g, r0 + kAttBlock, n1);
        sm.issued[pair] = go1;
      }
      asm volatile("bar.sync %0, %1;" ::"r"(1 + pair), "r"(64));  // issued[pair] seen by the pair
    }
    if (__syncthreads_or(!ok)) {
      if (!ok) mbar_wait(&sm.bar[pair], phase);  // the copy that did not land (bounded)
      if (threadIdx.x == 0) report(a.status, kStatusBulkTimeout);
      return;
    }
    // to the WarpState layout (lane 4gq + tq: head gq, dims state_dim(i, tq))
    // through this warp's 4 KB of the K slots (every copy has been consumed)
    WarpState ws;
    const int gq = lane >> 2, tq = lane & 3;
    ws.m = st.m[0];
    ws.l = st.l[0];
#pragma unroll
    for (int h = 1; h < kHeadsPerKv; ++h) {
      ws.m = gq == h ? st.m[h] : ws.m;
      ws.l = gq == h ? st.l[h] : ws.l;
    }
    float(*tr)[128] = reinterpret_cast<float(*)[128]>(&sm.k[0][0]) + warp * kHeadsPerKv;
#pragma unroll
    for (int h = 0; h < kHeadsPerKv; ++h)
      *reinterpret_cast<float4*>(&tr[h][4 * lane]) =
          make_float4(st.acc[4 * h], st.acc[4 * h + 1], st.acc[4 * h + 2], st.acc[4 * h + 3]);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 32; ++i) ws.acc[i] = tr[gq][state_dim(i, tq)];
    // the next item's copies into the K slots come after these generic-proxy accesses
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    // (the barrier above ends every warp's tiles: the fold scratch overlays
    // the query-preparation buffers)
    warps_fold_store(ws, warp, sm.sc, CtaSync{}, a.partials + (size_t(g * kHeadsPerKv) * icap + item) * kPartialFloats,
                     size_t(icap) * kPartialFloats);
    __syncthreads();
  }
}

}  // namespace rec
