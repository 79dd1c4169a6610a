// GQA decode attention over the quantized KV cache: split-KV item partials
// with fused RoPE / quantize-on-append, and the log-sum-exp combine.  The
// tile math and its canonical order are in attn_core.cuh.
//
// Work item = (kv head g, item_blocks(nblk) consecutive blocks of 256
// tokens: 1 up to one super-chunk of context, 4 beyond) for all 8 q heads of g.  Warp w folds tile w (32 tokens) of each of the item's blocks
// into a running state; the 8 warp states are folded as a tree
// ((w0 w1)(w2 w3))((w4 w5)(w6 w7)); super-chunks (64 blocks) fold
// their items in order; the output folds [sink] and the super-chunks in order.
//
// Reference: engine/src/rec_mlx/model.py:45-82 (quantize-on-append),
// model.py:108-139 (scores, sink, softmax), megakernel.py:619-693 (split-KV
// partials (max, sum, acc)), megakernel.py:276-318 (LSE merge).
#pragma once
#include "attn_core.cuh"

namespace rec {

constexpr int kHeadsPerKv = 8;                          // q heads per kv head
constexpr int kShortItems = 6;  // item partials per head folded by the last item's CTA (one super-chunk)

// Blocks per work item: 1 while the context fits one super-chunk (short
// contexts want many small items), 4 beyond (fewer per-item overheads).
__host__ __device__ inline int item_blocks(int nblk) { return nblk <= kAttSuper ? 1 : 4; }
__host__ __device__ inline int super_items(int nblk) { return kAttSuper / item_blocks(nblk); }

struct AttnArgs {
  const uint16_t* qkv;     // bf16 [Hq*128 | Hkv*128 | Hkv*128] pre-RoPE projections
  uint32_t* k_codes;       // [Hkv, C, 128*bits/32]
  uint16_t* k_scales;      // [Hkv, C, 2]
  uint16_t* k_biases;
  uint32_t* v_codes;
  uint16_t* v_scales;
  uint16_t* v_biases;
  int capacity;            // C, multiple of 256
  int hq, hkv;
  const float* rope;       // [positions, 128] cos | sin, row = absolute position; null: no RoPE (NoPE layer)
  const uint16_t* q_norm;  // bf16 [128] or null
  const uint16_t* k_norm;
  float eps;
  const int* position;     // device position p; T = p + 1
  float* partials;         // [Hq, n_items_cap, 132]
  float* supers;           // [Hq, n_super_max, 132]
  unsigned* head_counters; // [Hq]
  uint16_t* out;           // bf16 [Hq*128]
  const uint16_t* sinks;   // bf16 [Hq] or null
  int n_super_max;
  int* status;
  int pdl;
  // a session split over ranks: this rank's cache holds positions from
  // token_base on, and it computes the items of super-chunks [super_lo,
  // super_hi) (one GPU: token_base 0, super_lo 0, super_hi kAttAllSupers)
  int token_base;
  int super_lo, super_hi;
  // > 0: a sliding-window layer attends positions [max(0, p - window + 1), p]
  int window;
};
constexpr int kAttAllSupers = 1 << 30;

// First attended position of a step at position p (sliding window or 0).
__host__ __device__ inline int window_start(int p, int window) { return window > 0 && p + 1 > window ? p + 1 - window : 0; }

// Item partial slots per head: one per block covers every item size.
__host__ __device__ inline int items_cap(int capacity) { return capacity / kAttBlock; }

// Shared-memory scratch of the attention items of one CTA.
struct AttnScratch {
  QFrags qf;                               // queries of the 8 heads
  union alignas(16) {
    uint8_t wbuf[kAttWarps][1024];         // per-warp scratch of the query / new-row preparation
    float tree[kAttWarps / 2][36][32];     // warp states during the tree fold
    float stage[kAttWarps][4][kPartialFloats];  // per-warp partials being merged
    float items[kHeadsPerKv][kShortItems][kPartialFloats];  // a head group's item partials (short contexts)
  } u;
  uint32_t kpatch[32], vpatch[32];         // quantized K / V row of the new token
  uint16_t kps[2], kpb[2], vps[2], vpb[2];
  int qg;                                  // kv head whose queries are in qh (-1: none)
};

// Queries of the 8 heads of kv head g: warp w prepares head 8g + w.
template <int BITS>
__device__ __forceinline__ void prep_q_heads(const uint16_t* qkv, int g, const float* cs, const uint16_t* q_norm,
                                             float eps, AttnScratch& sc, int warp) {
  const int lane = threadIdx.x & 31;
  const uint16_t* qr = qkv + (g * kHeadsPerKv + warp) * 128;
  float x[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) x[j] = bf(__ldcg(reinterpret_cast<const unsigned short*>(qr + 4 * lane + j)));
  if (q_norm) head_norm4(x, q_norm, eps);
  float* scratch = reinterpret_cast<float*>(sc.u.wbuf[warp]);
  rope4(x, cs, scratch);
  prep_qhead<BITS>(x, sc.qf, warp, reinterpret_cast<int*>(scratch));
}

// The new token's K and V of kv head g, RoPE'd (K) and quantized into the
// patch rows; warps 0,1 = K groups, 2,3 = V groups (K codes BITS wide, V
// codes VBITS wide).  With g_* non-null the rows are also stored into the cache.
template <int BITS, int VBITS = BITS>
__device__ __forceinline__ void prep_new_kv(const uint16_t* qkv, int hq_total, int hkv, int g, const float* cs,
                                            const uint16_t* k_norm, float eps, AttnScratch& sc, int warp,
                                            uint32_t* g_kc, uint32_t* g_vc, uint16_t* g_ks, uint16_t* g_kb,
                                            uint16_t* g_vs, uint16_t* g_vb) {
  if (warp >= 4) return;
  const int lane = threadIdx.x & 31;
  const bool is_k = warp < 2;
  const int grp = warp & 1;
  const uint16_t* src = qkv + (hq_total + (is_k ? 0 : hkv) + g) * 128;
  float kv4[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) kv4[j] = bf(__ldcg(reinterpret_cast<const unsigned short*>(src + 4 * lane + j)));
  float* tmp = reinterpret_cast<float*>(sc.u.wbuf[warp]);
  if (is_k) {
    if (k_norm) head_norm4(kv4, k_norm, eps);
    rope4(kv4, cs, tmp);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) tmp[4 * lane + j] = kv4[j];
  __syncwarp();
  const float v0 = tmp[64 * grp + 2 * lane], v1 = tmp[64 * grp + 2 * lane + 1];
  const int bits = is_k ? BITS : VBITS;
  const QGroupParams qp = warp_group_params(v0, v1, bits);
  const uint32_t word = warp_pack(quant_code(v0, qp, bits), quant_code(v1, qp, bits), bits);
  const int GW = 64 * bits / 32;
  uint32_t* prow = (is_k ? sc.kpatch : sc.vpatch) + grp * GW;
  if (lane < GW) prow[lane] = word;
  const uint16_t scb = to_bf(qp.scale), bib = to_bf(qp.bias);
  if (lane == 0) {
    (is_k ? sc.kps : sc.vps)[grp] = scb;
    (is_k ? sc.kpb : sc.vpb)[grp] = bib;
  }
  if (g_kc) {
    uint32_t* gc = (is_k ? g_kc : g_vc) + grp * GW;
    if (lane < GW) gc[lane] = word;
    if (lane == 0) {
      (is_k ? g_ks : g_vs)[grp] = scb;
      (is_k ? g_kb : g_vb)[grp] = bib;
    }
  }
  __syncwarp();
}

// One warp copies the patch rows into row `row` of a K / V tile pair.
template <int BITS, int VBITS = BITS>
__device__ __forceinline__ void patch_row(uint32_t* kc, uint16_t* ks, uint16_t* kb, uint32_t* vc, uint16_t* vs,
                                          uint16_t* vb, int row, const AttnScratch& sc) {
  constexpr int RW = 128 * BITS / 32;
  constexpr int RWV = 128 * VBITS / 32;
  const int lane = threadIdx.x & 31;
  if (lane < RW) kc[row * RW + lane] = sc.kpatch[lane];
  if (lane < RWV) vc[row * RWV + lane] = sc.vpatch[lane];
  if (lane < 2) {
    ks[row * 2 + lane] = sc.kps[lane];
    kb[row * 2 + lane] = sc.kpb[lane];
    vs[row * 2 + lane] = sc.vps[lane];
    vb[row * 2 + lane] = sc.vpb[lane];
  }
  __syncwarp();
}

// Tree fold of the 8 warp states ((w0 w1)(w2 w3))((w4 w5)(w6 w7)) and the
// store of the item partial of heads 0..7 to dst + head * head_stride (m, l,
// pad, pad, acc[128]).  All warps call it (sync: a barrier over the 8 warps)
// after a barrier that ends every warp's tiles: the scratch overlays the
// per-warp buffers.  Level 1 goes through the scratch in the thread layout
// (senders 1,3,5,7 write slot w/2); receivers 0,2,4,6 rewrite their slot as
// [head][m, l, pad, pad, dim]; then warp w folds head w's four level-1
// states in registers (lane l: dims 4l..4l+3) and stores it.
template <typename Sync>
__device__ __forceinline__ void warps_fold_store(WarpState& st, int warp, AttnScratch& sc, Sync sync, float* dst,
                                                 size_t head_stride) {
  const int lane = threadIdx.x & 31, gq = lane >> 2, tq = lane & 3;
  float(*d)[32] = sc.u.tree[warp >> 1];
  if (warp & 1) {
    d[0][lane] = st.m;
    d[1][lane] = st.l;
#pragma unroll
    for (int i = 0; i < 32; ++i) d[2 + i][lane] = st.acc[i];
  }
  sync();
  if (!(warp & 1)) {
    WarpState y;
    y.m = d[0][lane];
    y.l = d[1][lane];
#pragma unroll
    for (int i = 0; i < 32; ++i) y.acc[i] = d[2 + i][lane];
    state_merge(st, y);
    __syncwarp();  // the slot is rewritten below: every lane has read it
    float* hs = &d[0][0] + gq * kPartialFloats;
    if (tq == 0) {
      hs[0] = st.m;
      hs[1] = st.l;
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {  // dims 64(r>>1) + 16tq + 8(r&1) + 0..7
      float4* o = reinterpret_cast<float4*>(hs + 4 + 64 * (r >> 1) + 16 * tq + 8 * (r & 1));
      o[0] = make_float4(st.acc[8 * r], st.acc[8 * r + 1], st.acc[8 * r + 2], st.acc[8 * r + 3]);
      o[1] = make_float4(st.acc[8 * r + 4], st.acc[8 * r + 5], st.acc[8 * r + 6], st.acc[8 * r + 7]);
    }
  }
  sync();
  Partial4 q[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const float* hs = &sc.u.tree[r][0][0] + warp * kPartialFloats;
    q[r].m = hs[0];
    q[r].l = hs[1];
    const float4 v = *reinterpret_cast<const float4*>(hs + 4 + 4 * lane);
    q[r].a[0] = v.x; q[r].a[1] = v.y; q[r].a[2] = v.z; q[r].a[3] = v.w;
  }
  merge_into(q[0], q[1]);
  merge_into(q[2], q[3]);
  merge_into(q[0], q[2]);
  store_partial(dst + size_t(warp) * head_stride, q[0]);
}

// This warp's tile (tile `warp`) of one block held in the given K / V tiles
// (rows [first, n) of the block valid: first > 0 only in the block where a
// sliding window starts; new_row >= 0: that row is the new token).  A tile
// with no valid row leaves the state unchanged.
// SPLIT: full tiles take the unmasked instance of tile_fold (same results);
// the persistent kernel keeps one instance for its instruction footprint.
template <int BITS, bool SPLIT = false, int VBITS = BITS>
__device__ __forceinline__ void block_tiles(uint32_t* kc, uint16_t* ks, uint16_t* kb, uint32_t* vc, uint16_t* vs,
                                            uint16_t* vb, int n, int new_row, const AttnScratch& sc, int warp,
                                            WarpState& st, int first = 0) {
  constexpr int RW = 128 * BITS / 32;
  constexpr int RWV = 128 * VBITS / 32;
  const int t0 = warp * kAttTile;
  const int nvalid = min(kAttTile, n - t0);
  const int tfirst = max(0, first - t0);
  if (nvalid <= tfirst) return;
  if (new_row >= t0 && new_row < t0 + kAttTile) patch_row<BITS, VBITS>(kc, ks, kb, vc, vs, vb, new_row, sc);
  if (SPLIT && nvalid == kAttTile && tfirst == 0)
    tile_fold<BITS, true, VBITS>(kc + t0 * RW, ks + 2 * t0, kb + 2 * t0, vc + t0 * RWV, vs + 2 * t0, vb + 2 * t0,
                                 nvalid, sc.qf, st);
  else
    tile_fold<BITS, false, VBITS>(kc + t0 * RW, ks + 2 * t0, kb + 2 * t0, vc + t0 * RWV, vs + 2 * t0, vb + 2 * t0,
                                  nvalid, sc.qf, st, tfirst);
}

// ---------------------------------------------------------------------------
// Standalone kernels (the graph schedule)
// ---------------------------------------------------------------------------
template <int BITS, int VBITS = BITS>
struct AttnStage {
  static constexpr int ROW_WORDS = 128 * BITS / 32;    // K
  static constexpr int VROW_WORDS = 128 * VBITS / 32;  // V
  alignas(128) uint32_t kc[kAttBlock * ROW_WORDS];
  alignas(128) uint32_t vc[kAttBlock * VROW_WORDS];
  alignas(16) uint16_t ks[kAttBlock * 2];
  alignas(16) uint16_t kb[kAttBlock * 2];
  alignas(16) uint16_t vs[kAttBlock * 2];
  alignas(16) uint16_t vb[kAttBlock * 2];
};
template <int BITS, int VBITS = BITS>
struct AttnSmem {
  AttnStage<BITS, VBITS> st[2];
  AttnScratch sc;
  uint64_t bar[2];
};

// Bulk copies of block b (global index) of kv head g into stage s.
template <int BITS, int VBITS = BITS>
__device__ __forceinline__ void issue_block(AttnSmem<BITS, VBITS>& sm, int s, const AttnArgs& a, int g, int b,
                                            int T) {
  constexpr int RW = AttnStage<BITS, VBITS>::ROW_WORDS;
  constexpr int RWV = AttnStage<BITS, VBITS>::VROW_WORDS;
  const int n = min(kAttBlock, T - b * kAttBlock);
  const int n4 = (n + 3) & ~3;
  const size_t slot = size_t(g) * a.capacity + size_t(b) * kAttBlock - size_t(a.token_base);
  const uint32_t cb = uint32_t(n4) * RW * 4, cbv = uint32_t(n4) * RWV * 4, sbytes = uint32_t(n4) * 4;
  mbar_expect_tx(&sm.bar[s], cb + cbv + 4 * sbytes);
  bulk_g2s(sm.st[s].kc, a.k_codes + slot * RW, cb, &sm.bar[s]);
  bulk_g2s(sm.st[s].vc, a.v_codes + slot * RWV, cbv, &sm.bar[s]);
  bulk_g2s(sm.st[s].ks, a.k_scales + slot * 2, sbytes, &sm.bar[s]);
  bulk_g2s(sm.st[s].kb, a.k_biases + slot * 2, sbytes, &sm.bar[s]);
  bulk_g2s(sm.st[s].vs, a.v_scales + slot * 2, sbytes, &sm.bar[s]);
  bulk_g2s(sm.st[s].vb, a.v_biases + slot * 2, sbytes, &sm.bar[s]);
}

struct CtaSync {
  __device__ void operator()() const { __syncthreads(); }
};

// Item partials.  Persistent grid; item it = (kv head it % Hkv, item it / Hkv).
template <int BITS, int VBITS = BITS>
__global__ void __launch_bounds__(kAttWarps * 32, 2) k_attn_partial(const AttnArgs a) {
  constexpr int RW = AttnStage<BITS, VBITS>::ROW_WORDS;
  constexpr int RWV = AttnStage<BITS, VBITS>::VROW_WORDS;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AttnSmem<BITS, VBITS>& sm = *reinterpret_cast<AttnSmem<BITS, VBITS>*>(smem_raw);
  const int warp = threadIdx.x >> 5;
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
  if (p < 0 || (a.super_hi >= kAttAllSupers && p >= a.capacity)) {
    if (blockIdx.x == 0 && threadIdx.x == 0) report(a.status, kStatusBadPosition);
    return;
  }
  const int nblk = (T + kAttBlock - 1) / kAttBlock;
  const int nbi = item_blocks(nblk);
  const int n_items = (nblk + nbi - 1) / nbi;
  const int per_super = super_items(nblk);
  // this rank's items: those of super-chunks [super_lo, super_hi)
  // a sliding window skips the items below its first position (their
  // partials are never read)
  const int lo = window_start(p, a.window);
  const int i_first = lo / (kAttBlock * nbi);
  const int i_lo = max(i_first, min(a.super_lo, (n_items + per_super - 1) / per_super) * per_super);
  const int i_hi = a.super_hi >= (n_items + per_super - 1) / per_super ? n_items : a.super_hi * per_super;
  const int items = max(0, i_hi - i_lo) * a.hkv;
  const int item0 = a.token_base / (kAttBlock * nbi);  // local index of the first item held here
  const float* cs = a.rope ? a.rope + size_t(p) * 128 : nullptr;
  const int icap = items_cap(a.capacity);
  uint32_t phase = 0;  // bit s: parity of stage s
  for (int it = blockIdx.x; it < items; it += gridDim.x) {
    const int g = it % a.hkv, item = i_lo + it / a.hkv;
    const int b0 = item * nbi, b1 = min(b0 + nbi, nblk);
    if (threadIdx.x == 0) issue_block<BITS, VBITS>(sm, 0, a, g, b0, T);
    if (sm.sc.qg != g) prep_q_heads<BITS>(a.qkv, g, cs, a.q_norm, a.eps, sm.sc, warp);
    const bool has_new = p >= b0 * kAttBlock && p < b1 * kAttBlock;
    if (has_new) {
      const size_t slot = size_t(g) * a.capacity + size_t(p - a.token_base);
      prep_new_kv<BITS, VBITS>(a.qkv, a.hq, a.hkv, g, cs, a.k_norm, a.eps, sm.sc, warp, a.k_codes + slot * RW,
                               a.v_codes + slot * RWV, a.k_scales + slot * 2, a.k_biases + slot * 2,
                               a.v_scales + slot * 2, a.v_biases + slot * 2);
    }
    __syncthreads();
    if (threadIdx.x == 0) sm.sc.qg = g;
    WarpState st;
    state_empty(st);
    bool ok = true;
    for (int b = b0; b < b1; ++b) {
      const int s = (b - b0) & 1;
      if (threadIdx.x == 0 && b + 1 < b1) issue_block<BITS, VBITS>(sm, s ^ 1, a, g, b + 1, T);
      ok = mbar_wait(&sm.bar[s], (phase >> s) & 1u) && ok;
      phase ^= 1u << s;
      if (!__syncthreads_and(ok)) break;
      const int n = min(kAttBlock, T - b * kAttBlock);
      const int new_row = (has_new && p / kAttBlock == b) ? p - b * kAttBlock : -1;
      AttnStage<BITS, VBITS>& S = sm.st[s];
      block_tiles<BITS, true, VBITS>(S.kc, S.ks, S.kb, S.vc, S.vs, S.vb, n, new_row, sm.sc, warp, st,
                                     lo - b * kAttBlock);
      // the tile may have been patched through the generic proxy, and the
      // next bulk copy into this stage must not overtake this block's reads
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncthreads();
    }
    if (!ok) {
      if (threadIdx.x == 0) {
        report(a.status, kStatusBulkTimeout);
        for (int s = 0; s < 2; ++s) mbar_wait(&sm.bar[s], (phase >> s) & 1u);
      }
      return;
    }
    warps_fold_store(st, warp, sm.sc, CtaSync{},
                     a.partials + (size_t(g * kHeadsPerKv) * icap + (item - item0)) * kPartialFloats,
                     size_t(icap) * kPartialFloats);
    __syncthreads();
  }
}

// Combine: one warp per (q head, super-chunk) folds its items in order; the
// last warp of a head folds [sink] and the super-chunks into out.
static __global__ void __launch_bounds__(32) k_attn_combine(const AttnArgs a) {
  if (a.pdl) grid_wait();
  grid_launch_dependents();
  const int lane = threadIdx.x;
  const int p = *a.position;
  const int T = p + 1;
  const int nblk = (T + kAttBlock - 1) / kAttBlock;
  const int nbi = item_blocks(nblk), per_super = super_items(nblk);
  const int n_items = (nblk + nbi - 1) / nbi;
  const int n_super = (n_items + per_super - 1) / per_super;
  const int i_first = window_start(p, a.window) / (kAttBlock * nbi);  // items below a sliding window are empty
  const int h = blockIdx.x;
  const int icap = items_cap(a.capacity);
  for (int s = blockIdx.y; s < n_super; s += gridDim.y) {
    Partial4 P = empty_partial();
    fold_partials(P, a.partials + size_t(h) * icap * kPartialFloats, max(s * per_super, i_first),
                  min((s + 1) * per_super, n_items));
    float* dst = a.supers + (size_t(h) * a.n_super_max + s) * kPartialFloats;
    if (lane == 0) {
      dst[0] = P.m;
      dst[1] = P.l;
    }
    *reinterpret_cast<float4*>(dst + 4 + 4 * lane) = make_float4(P.a[0], P.a[1], P.a[2], P.a[3]);
  }
  // the last arriving warp of head h merges the super-chunks in order
  __threadfence();
  unsigned prev = 0;
  if (lane == 0) prev = atomicAdd(a.head_counters + h, 1u);
  prev = __shfl_sync(0xffffffffu, prev, 0);
  if (prev != gridDim.y - 1) return;
  __threadfence();
  Partial4 F = empty_partial();
  if (a.sinks) {
    F.m = bf(a.sinks[h]);
    F.l = 1.0f;
  }
  fold_partials(F, a.supers + size_t(h) * a.n_super_max * kPartialFloats, 0, n_super);
  uint2 o;
  o.x = uint32_t(to_bf(__fdiv_rn(F.a[0], F.l))) | (uint32_t(to_bf(__fdiv_rn(F.a[1], F.l))) << 16);
  o.y = uint32_t(to_bf(__fdiv_rn(F.a[2], F.l))) | (uint32_t(to_bf(__fdiv_rn(F.a[3], F.l))) << 16);
  *reinterpret_cast<uint2*>(a.out + h * 128 + 4 * lane) = o;
  if (lane == 0) a.head_counters[h] = 0;
}

}  // namespace rec
