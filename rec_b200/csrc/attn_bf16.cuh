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

struct AttnBfSmem {
  alignas(128) uint16_t k[kAttBlock * 128];  // one block of K rows
  alignas(128) uint16_t v[kAttBlock * 128];  // and of V rows
  alignas(16) float q[kHeadsPerKv][128];     // scaled queries of the kv head's 8 heads
  float p[kAttWarps][kHeadsPerKv][33];       // per warp: softmax weights [head][row] (padded)
  alignas(16) uint16_t knew[128], vnew[128]; // the new token's K (normed, RoPE'd) and V
  AttnScratch sc;                            // query preparation scratch and the warp-state tree fold
  uint64_t bar[2];                           // K, V copies
};

// Bulk copies of the K (which = 0) or V (1) rows of block b of kv head g.
__device__ __forceinline__ void issue_bf16_rows(AttnBfSmem& sm, int which, const AttnArgs& a, int g, int b, int T) {
  const int n = min(kAttBlock, T - b * kAttBlock);
  const size_t row = size_t(g) * a.capacity + size_t(b) * kAttBlock - size_t(a.token_base);
  const uint32_t bytes = uint32_t(n) * 256u;
  mbar_expect_tx(&sm.bar[which], bytes);
  const uint32_t* src = which ? a.v_codes : a.k_codes;
  bulk_g2s(which ? sm.v : sm.k, reinterpret_cast<const uint8_t*>(src) + row * 256u, bytes, &sm.bar[which]);
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
// acc in the WarpState layout (lane 4gq + tq: head gq, dims state_dim(i, tq)).
struct BfState {
  float m[kHeadsPerKv], l[kHeadsPerKv];
  float acc[32];
};

// The tile (rows [32 warp, 32 warp + 32) of the block; rows [first, nvalid)
// of it valid) folded into st.
__device__ __forceinline__ void tile_fold_bf16(const AttnBfSmem& sm, float (&p_sm)[kHeadsPerKv][33], int warp,
                                               int first, int nvalid, BfState& st) {
  const int lane = threadIdx.x & 31, gq = lane >> 2, tq = lane & 3;
  // ---- scores: lane = row
  const uint16_t* krow = sm.k + (warp * kAttTile + lane) * 128;
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
      const float4 qq = *reinterpret_cast<const float4*>(&sm.q[h][4 * cc]);
      s[h] = __fmaf_rn(qq.x, k0, s[h]);
      s[h] = __fmaf_rn(qq.y, k1, s[h]);
      s[h] = __fmaf_rn(qq.z, k2, s[h]);
      s[h] = __fmaf_rn(qq.w, k3, s[h]);
    }
  }
  // ---- softmax per head (all lanes keep every head's m, l)
  const bool valid = lane >= first && lane < nvalid;
  float alpha[kHeadsPerKv];
#pragma unroll
  for (int h = 0; h < kHeadsPerKv; ++h) {
    const float sh = valid ? s[h] : -INFINITY;
    const float mn = fmaxf(st.m[h], bfly_max(sh));
    alpha[h] = aexp(__fsub_rn(st.m[h], mn));
    const float p = valid ? aexp(__fsub_rn(sh, mn)) : 0.0f;
    st.l[h] = __fmaf_rn(st.l[h], alpha[h], bfly_sum(p));
    st.m[h] = mn;
    p_sm[h][lane] = p;
  }
  __syncwarp();
  // ---- P.V: lane (gq, tq), head gq, dims state_dim(i, tq)
  float a_h = alpha[0], pv[32];
#pragma unroll
  for (int h = 1; h < kHeadsPerKv; ++h) a_h = gq == h ? alpha[h] : a_h;
#pragma unroll
  for (int i = 0; i < 32; ++i) pv[i] = 0.0f;
  for (int r = first; r < nvalid; ++r) {
    const float pr = p_sm[gq][r];
    const uint16_t* vrow = sm.v + (warp * kAttTile + r) * 128 + 16 * tq;
    uint32_t w[16];
    {
      const uint4 a0 = *reinterpret_cast<const uint4*>(vrow);
      const uint4 a1 = *reinterpret_cast<const uint4*>(vrow + 8);
      const uint4 b0 = *reinterpret_cast<const uint4*>(vrow + 64);
      const uint4 b1 = *reinterpret_cast<const uint4*>(vrow + 72);
      w[0] = a0.x; w[1] = a0.y; w[2] = a0.z; w[3] = a0.w; w[4] = a1.x; w[5] = a1.y; w[6] = a1.z; w[7] = a1.w;
      w[8] = b0.x; w[9] = b0.y; w[10] = b0.z; w[11] = b0.w; w[12] = b1.x; w[13] = b1.y; w[14] = b1.z; w[15] = b1.w;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      pv[2 * j] = __fmaf_rn(pr, __uint_as_float(w[j] << 16), pv[2 * j]);
      pv[2 * j + 1] = __fmaf_rn(pr, __uint_as_float(w[j] & 0xFFFF0000u), pv[2 * j + 1]);
    }
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) st.acc[i] = __fmaf_rn(st.acc[i], a_h, pv[i]);
  __syncwarp();  // p_sm is rewritten by the next tile
}

// Item partials over a bf16 cache.  Persistent grid, one CTA per SM (a block
// of K and V rows takes 128 KB); item it = (kv head it % Hkv, item
// i_first + it / Hkv).  Each block is copied, patched with the new row and
// folded; the CTAs of the grid keep HBM busy between them.
static __global__ void __launch_bounds__(kAttWarps * 32, 1) k_attn_partial_bf16(const AttnArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AttnBfSmem& sm = *reinterpret_cast<AttnBfSmem*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&sm.bar[0], 1);
    mbar_init(&sm.bar[1], 1);
    fence_barrier_init();
    sm.sc.qg = -1;
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
  uint32_t phase = 0;  // bit 0: K barrier parity, bit 1: V
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const int g = it % a.hkv, item = i_first + it / a.hkv;
    const int b0 = item * nbi, b1 = min(b0 + nbi, nblk);
    if (threadIdx.x == 0) {
      issue_bf16_rows(sm, 0, a, g, b0, T);
      issue_bf16_rows(sm, 1, a, g, b0, T);
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
    bool ok = true;
    for (int b = b0; b < b1; ++b) {
      const int n = min(kAttBlock, T - b * kAttBlock);
      const int t0 = warp * kAttTile;
      const int nvalid = min(kAttTile, n - t0), first = max(0, lo - b * kAttBlock - t0);
      const bool tile = nvalid > first;
      const int new_row = (has_new && p / kAttBlock == b) ? p - b * kAttBlock : -1;
      const bool mine = new_row >= t0 && new_row < t0 + kAttTile;
      ok = mbar_wait(&sm.bar[0], phase & 1u) && ok;
      phase ^= 1u;
      if (!__syncthreads_and(ok)) break;
      if (mine) *reinterpret_cast<uint2*>(sm.k + new_row * 128 + 4 * lane) =
          *reinterpret_cast<const uint2*>(sm.knew + 4 * lane);
      ok = mbar_wait(&sm.bar[1], (phase >> 1) & 1u) && ok;
      phase ^= 2u;
      if (!__syncthreads_and(ok)) break;
      if (mine) *reinterpret_cast<uint2*>(sm.v + new_row * 128 + 4 * lane) =
          *reinterpret_cast<const uint2*>(sm.vnew + 4 * lane);
      __syncwarp();
      if (tile) tile_fold_bf16(sm, sm.p[warp], warp, first, nvalid, st);
      // both buffers are read; the next block's copies may overwrite them
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncthreads();
      if (threadIdx.x == 0 && b + 1 < b1) {
        issue_bf16_rows(sm, 0, a, g, b + 1, T);
        issue_bf16_rows(sm, 1, a, g, b + 1, T);
      }
    }
    if (!ok) {
      if (threadIdx.x == 0) {
        report(a.status, kStatusBulkTimeout);
        for (int s = 0; s < 2; ++s) mbar_wait(&sm.bar[s], (phase >> s) & 1u);
      }
      return;
    }
    WarpState ws;
    const int gq = lane >> 2;
    ws.m = st.m[0];
    ws.l = st.l[0];
#pragma unroll
    for (int h = 1; h < kHeadsPerKv; ++h) {
      ws.m = gq == h ? st.m[h] : ws.m;
      ws.l = gq == h ? st.l[h] : ws.l;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) ws.acc[i] = st.acc[i];
    __syncthreads();  // the fold scratch overlays the query-preparation buffers
    warps_fold_store(ws, warp, sm.sc, CtaSync{}, a.partials + (size_t(g * kHeadsPerKv) * icap + item) * kPartialFloats,
                     size_t(icap) * kPartialFloats);
    __syncthreads();
  }
}

}  // namespace rec
