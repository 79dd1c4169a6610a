// GQA decode attention over the quantized KV cache: split-KV block partials
// with fused RoPE / quantize-on-append, and the log-sum-exp combine.  The
// math and its canonical order are in attn_core.cuh.
//
// Reference: engine/src/rec_mlx/model.py:45-82 (quantize-on-append),
// model.py:108-139 (scores, sink, softmax), megakernel.py:619-693 (split-KV
// partials (max, sum, acc)), megakernel.py:276-318 (LSE merge).
#pragma once
#include "attn_core.cuh"

namespace rec {

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
  const float* rope;       // [C, 128] cos | sin
  const uint16_t* q_norm;  // bf16 [128] or null
  const uint16_t* k_norm;
  float eps;
  const int* position;     // device position p; T = p + 1
  int token_base;          // first global position stored in this cache (split-KV ranks)
  int block_begin, block_end;  // global block range this rank computes (split-KV)
  float* partials;         // [Hq, capacity/256, 132]
  float* supers;           // [Hq, n_super_max, 132]
  unsigned* head_counters; // [Hq]
  uint16_t* out;           // bf16 [Hq*128]
  const uint16_t* sinks;   // bf16 [Hq] or null
  int n_super_max;
  int final_merge;         // 1: combine also merges super-chunks into out
  int* status;
  int pdl;
};

// Shared-memory scratch of one attention item (hq <= kMaxHq heads).
struct AttnScratch {
  QHead qh[kMaxHq];
  alignas(16) float p[kAttWarps][kMaxHq][kAttTile];
  alignas(16) float wacc[kAttWarps][kMaxHq][128];
  float wm[kAttWarps][kMaxHq], wl[kAttWarps][kMaxHq];
};

// Tile of one (block, kv head): codes then scales then biases for K and V,
// rows padded to a multiple of 4 tokens.
struct TileView {
  uint32_t *kc, *vc;
  uint16_t *ks, *kb, *vs, *vb;
};

// One work item: one block (n tokens) of kv head g for q heads [h0, h0+hq).
// Called by all kAttWarps warps of a group (ids warp 0..7, synchronised by
// `sync`); warp h < hq returns the block partial of head h0 + h.
struct AttnBlock {
  const uint16_t* qkv;
  int hq_total, hkv;
  int g, h0, hq, n;
  const float* cs;              // cos/sin row of pos
  const uint16_t *q_norm, *k_norm;
  float eps;
  bool has_new;                 // the block holds position pos
  int tnew;                     // its row in the tile
  uint32_t* g_kcodes;           // non-null: publish the new token here (row slot)
  uint32_t* g_vcodes;
  uint16_t *g_ks, *g_kb, *g_vs, *g_vb;
};

struct NoMark {
  __device__ void operator()(int) const {}
};

// mark(i) is called by every warp after the query/append step (i = 0) and
// after the tiles (i = 1): a hook for timeline stamps.
template <int BITS, typename Sync, typename Mark = NoMark>
__device__ __forceinline__ void attn_block(const AttnBlock& it, TileView tv, AttnScratch& sc, int warp, Sync sync,
                                           Partial4& P, Mark mark = Mark()) {
  constexpr int RW = 128 * BITS / 32;
  const int lane = threadIdx.x & 31;
  // --- queries (warps 4..7) and the new token's K/V (warps 0..3) --------------
  if (warp >= 4) {
    const int hh = warp - 4;
    if (hh < it.hq) {
      const uint16_t* qr = it.qkv + (it.h0 + hh) * 128;
      float x[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = bf(__ldcg(reinterpret_cast<const unsigned short*>(qr + 4 * lane + j)));
      if (it.q_norm) head_norm4(x, it.q_norm, it.eps);
      float* scratch = sc.wacc[warp][0];
      rope4(x, it.cs, scratch);
      prep_qhead<BITS>(x, sc.qh[hh], scratch);
    }
  } else if (it.has_new) {
    const bool is_k = warp < 2;
    const int grp = warp & 1;
    const uint16_t* src = it.qkv + (it.hq_total + (is_k ? 0 : it.hkv) + it.g) * 128;
    float kv4[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) kv4[j] = bf(__ldcg(reinterpret_cast<const unsigned short*>(src + 4 * lane + j)));
    float* tmp = sc.wacc[warp][0];
    if (is_k) {
      if (it.k_norm) head_norm4(kv4, it.k_norm, it.eps);
      rope4(kv4, it.cs, tmp);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) tmp[4 * lane + j] = kv4[j];
    __syncwarp();
    const float v0 = tmp[64 * grp + 2 * lane], v1 = tmp[64 * grp + 2 * lane + 1];
    const QGroupParams qp = warp_group_params(v0, v1, BITS);
    const uint32_t word = warp_pack(quant_code(v0, qp, BITS), quant_code(v1, qp, BITS), BITS);
    constexpr int GW = 64 * BITS / 32;
    uint32_t* crow = (is_k ? tv.kc : tv.vc) + it.tnew * RW + grp * GW;
    if (lane < GW) crow[lane] = word;
    const uint16_t scb = to_bf(qp.scale), bib = to_bf(qp.bias);
    if (lane == 0) {
      (is_k ? tv.ks : tv.vs)[it.tnew * 2 + grp] = scb;
      (is_k ? tv.kb : tv.vb)[it.tnew * 2 + grp] = bib;
    }
    if (it.g_kcodes) {
      uint32_t* gc = (is_k ? it.g_kcodes : it.g_vcodes) + grp * GW;
      if (lane < GW) gc[lane] = word;
      if (lane == 0) {
        (is_k ? it.g_ks : it.g_vs)[grp] = scb;
        (is_k ? it.g_kb : it.g_vb)[grp] = bib;
      }
    }
  }
  sync();
  mark(0);
  // --- warp w: tile w ------------------------------------------------------------
  const int hq = it.hq;
  float m[kMaxHq], l[kMaxHq], acc[kMaxHq][4];
#pragma unroll
  for (int h = 0; h < kMaxHq; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[h][j] = 0.0f;
  }
  const int base = warp * kAttTile;
  if (base < it.n) {
    const int tl = base + lane;
    const bool valid = tl < it.n;
    const int row = valid ? tl : base;
    const float s0 = bf(tv.ks[row * 2]), s1 = bf(tv.ks[row * 2 + 1]);
    const float b0 = bf(tv.kb[row * 2]), b1 = bf(tv.kb[row * 2 + 1]);
    tile_scores<BITS>(tv.kc + row * RW, valid, s0, b0, s1, b1, sc.qh, hq, m, l, sc.p[warp]);
    __syncwarp();
    const int nt = min(kAttTile, it.n - base);
    const int grp = lane >> 4;
    // two tokens per iteration: every shared-memory load of the pair is
    // issued before its multiply-adds; acc still adds tokens in order
    auto vvals = [&](int tok, float (&v)[4]) {
      uint32_t c4;
      if constexpr (BITS == 4) c4 = reinterpret_cast<const uint16_t*>(tv.vc + tok * RW)[lane];
      else c4 = tv.vc[tok * RW + lane];
      const float vsc = bf(tv.vs[tok * 2 + grp]), vbi = bf(tv.vb[tok * 2 + grp]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t c = BITS == 4 ? (c4 >> (4 * j)) & 15u : (c4 >> (8 * j)) & 255u;
        v[j] = __fmaf_rn(vsc, code_f(c), vbi);
      }
    };
    int t = 0;
    for (; t + 2 <= nt; t += 2) {
      float v[2][4];
#pragma unroll
      for (int q = 0; q < 2; ++q) vvals(base + t + q, v[q]);
#pragma unroll
      for (int h = 0; h < kMaxHq; ++h) {
        if (h >= hq) break;
        const float2 p2 = *reinterpret_cast<const float2*>(&sc.p[warp][h][t]);
        const float pq[2] = {p2.x, p2.y};
#pragma unroll
        for (int q = 0; q < 2; ++q)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[h][j] = __fmaf_rn(pq[q], v[q][j], acc[h][j]);
      }
    }
    for (; t < nt; ++t) {
      float v[4];
      vvals(base + t, v);
#pragma unroll
      for (int h = 0; h < kMaxHq; ++h) {
        if (h >= hq) break;
        const float pp = sc.p[warp][h][t];
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[h][j] = __fmaf_rn(pp, v[j], acc[h][j]);
      }
    }
  }
#pragma unroll
  for (int h = 0; h < kMaxHq; ++h) {
    if (h >= hq) break;
    if (lane == 0) {
      sc.wm[warp][h] = m[h];
      sc.wl[warp][h] = l[h];
    }
    *reinterpret_cast<float4*>(&sc.wacc[warp][h][4 * lane]) = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
  }
  sync();
  mark(1);
  // --- block partial: warps merged in order ----------------------------------
  P = empty_partial();
  if (warp < hq) {
    const int h = warp;
    for (int w = 0; w < kAttWarps; ++w) {
      Partial4 Q;
      Q.m = sc.wm[w][h];
      Q.l = sc.wl[w][h];
      const float4 a4 = *reinterpret_cast<const float4*>(&sc.wacc[w][h][4 * lane]);
      Q.a[0] = a4.x; Q.a[1] = a4.y; Q.a[2] = a4.z; Q.a[3] = a4.w;
      if (w * kAttTile >= it.n) Q = empty_partial();
      merge_into(P, Q);
    }
  }
}

__device__ __forceinline__ void store_partial(float* dst, const Partial4& P) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) {
    dst[0] = P.m;
    dst[1] = P.l;
  }
  *reinterpret_cast<float4*>(dst + 4 + 4 * lane) = make_float4(P.a[0], P.a[1], P.a[2], P.a[3]);
}

__device__ __forceinline__ int att_hq(int hkv, int nblk, int slots) {
  // q heads per work item: as few as possible while the items fit `slots`
  int hq = 1;
  while (hq < kMaxHq && hkv * (8 / hq) * nblk > slots) hq *= 2;
  return hq;
}

template <int BITS>
struct AttnSmem {
  static constexpr int ROW_WORDS = 128 * BITS / 32;
  alignas(128) uint32_t kc[kAttBlock * ROW_WORDS];
  alignas(128) uint32_t vc[kAttBlock * ROW_WORDS];
  alignas(16) uint16_t ks[kAttBlock * 2];
  alignas(16) uint16_t kb[kAttBlock * 2];
  alignas(16) uint16_t vs[kAttBlock * 2];
  alignas(16) uint16_t vb[kAttBlock * 2];
  AttnScratch sc;
  uint64_t bar;
};

// Issue the bulk copies of block b (local index) of kv head g, n tokens
// (rounded up to 4).
template <int BITS>
__device__ __forceinline__ void issue_kv_tile(AttnSmem<BITS>& sm, const AttnArgs& a, int g, int b_local, int n) {
  constexpr int RW = AttnSmem<BITS>::ROW_WORDS;
  const int n4 = (n + 3) & ~3;
  const size_t slot = size_t(g) * a.capacity + size_t(b_local) * kAttBlock;
  const uint32_t cb = uint32_t(n4) * RW * 4, sbytes = uint32_t(n4) * 4;
  mbar_expect_tx(&sm.bar, 2 * cb + 4 * sbytes);
  bulk_g2s(sm.kc, a.k_codes + slot * RW, cb, &sm.bar);
  bulk_g2s(sm.vc, a.v_codes + slot * RW, cb, &sm.bar);
  bulk_g2s(sm.ks, a.k_scales + slot * 2, sbytes, &sm.bar);
  bulk_g2s(sm.kb, a.k_biases + slot * 2, sbytes, &sm.bar);
  bulk_g2s(sm.vs, a.v_scales + slot * 2, sbytes, &sm.bar);
  bulk_g2s(sm.vb, a.v_biases + slot * 2, sbytes, &sm.bar);
}

struct CtaSync {
  __device__ void operator()() const { __syncthreads(); }
};

// Block partials.  Persistent grid; work item = (block, kv head, q-head slice).
template <int BITS>
__global__ void __launch_bounds__(kAttWarps * 32, 2) k_attn_partial(const AttnArgs a) {
  constexpr int RW = AttnSmem<BITS>::ROW_WORDS;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AttnSmem<BITS>& sm = *reinterpret_cast<AttnSmem<BITS>*>(smem_raw);
  const int warp = threadIdx.x >> 5;

  if (threadIdx.x == 0) {
    mbar_init(&sm.bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  const int p = *a.position;
  const int T = p + 1;
  const int nblk_total = (T + kAttBlock - 1) / kAttBlock;
  const int b0 = a.block_begin, b1 = min(a.block_end, nblk_total);
  const int nblk = max(b1 - b0, 0);
  const int hq = att_hq(a.hkv, max(nblk, 1), gridDim.x);
  const int nq = (a.hq / a.hkv) / hq;
  const int items = nblk * a.hkv * nq;
  const bool pos_ok = p >= a.token_base && p < a.capacity + a.token_base;
  const int blk0 = a.token_base / kAttBlock;

  auto coords = [&](int it, int& b, int& g, int& qsub) {
    qsub = it % nq;
    g = (it / nq) % a.hkv;
    b = b0 + it / (nq * a.hkv);
  };
  auto block_tokens = [&](int b) { return min(kAttBlock, T - b * kAttBlock); };

  uint32_t phase = 0;
  int it = blockIdx.x;
  bool pending = false;
  if (threadIdx.x == 0 && it < items && pos_ok) {
    int b, g, q_;
    coords(it, b, g, q_);
    issue_kv_tile<BITS>(sm, a, g, b - blk0, block_tokens(b));
  }
  pending = it < items && pos_ok;
  if (a.pdl) grid_wait();
  grid_launch_dependents();
  if (!pos_ok) {
    if (blockIdx.x == 0 && threadIdx.x == 0) report(a.status, kStatusBadPosition);
    return;
  }
  const float* cs = a.rope + size_t(p) * 128;  // rows are absolute positions
  for (; it < items; it += gridDim.x) {
    int b, g, qsub;
    coords(it, b, g, qsub);
    const int n = block_tokens(b);
    if (!pending && threadIdx.x == 0) issue_kv_tile<BITS>(sm, a, g, b - blk0, n);
    pending = false;
    const bool ok = mbar_wait(&sm.bar, phase);
    phase ^= 1;
    if (!__syncthreads_and(ok)) {
      if (threadIdx.x == 0) {
        report(a.status, kStatusBulkTimeout);
        mbar_wait(&sm.bar, phase ^ 1);
      }
      return;
    }
    AttnBlock ai = {};
    ai.qkv = a.qkv;
    ai.hq_total = a.hq;
    ai.hkv = a.hkv;
    ai.g = g;
    ai.h0 = g * (a.hq / a.hkv) + qsub * hq;
    ai.hq = hq;
    ai.n = n;
    ai.cs = cs;
    ai.q_norm = a.q_norm;
    ai.k_norm = a.k_norm;
    ai.eps = a.eps;
    ai.has_new = p >= b * kAttBlock && p < b * kAttBlock + n;
    ai.tnew = p - b * kAttBlock;
    if (ai.has_new && qsub == 0) {
      const size_t slot = size_t(g) * a.capacity + size_t(p - a.token_base);
      ai.g_kcodes = a.k_codes + slot * RW;
      ai.g_vcodes = a.v_codes + slot * RW;
      ai.g_ks = a.k_scales + slot * 2;
      ai.g_kb = a.k_biases + slot * 2;
      ai.g_vs = a.v_scales + slot * 2;
      ai.g_vb = a.v_biases + slot * 2;
    }
    TileView tv = {sm.kc, sm.vc, sm.ks, sm.kb, sm.vs, sm.vb};
    Partial4 P;
    attn_block<BITS>(ai, tv, sm.sc, warp, CtaSync{}, P);
    if (warp < hq) {
      const int nblk_cap = a.capacity / kAttBlock;
      store_partial(a.partials + (size_t(ai.h0 + warp) * nblk_cap + (b - blk0)) * kPartialFloats, P);
    }
    // the tile was patched by the generic proxy; order that before the next
    // bulk copy overwrites it
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
  }
}

// Combine: one warp per (q head, super-chunk) merges its blocks in order; the
// last warp of a head merges the super-chunks (and the sink) into out.
__global__ void __launch_bounds__(32) k_attn_combine(const AttnArgs a) {
  if (a.pdl) grid_wait();
  grid_launch_dependents();
  const int lane = threadIdx.x;
  const int p = *a.position;
  const int T = p + 1;
  const int nblk_total = (T + kAttBlock - 1) / kAttBlock;
  const int b0 = a.block_begin, b1 = min(a.block_end, nblk_total);
  const int s_first = b0 / kAttSuper;
  const int s_last = b1 > b0 ? (b1 - 1) / kAttSuper : s_first - 1;
  const int n_local = s_last - s_first + 1;
  const int h = blockIdx.x;
  const int nblk_cap = a.capacity / kAttBlock;
  for (int si = blockIdx.y; si < max(n_local, 0); si += gridDim.y) {
    const int s = s_first + si;
    Partial4 P = empty_partial();
    const int bb0 = max(s * kAttSuper, b0), bb1 = min((s + 1) * kAttSuper, b1);
    for (int b = bb0; b < bb1; ++b) {
      const float* src = a.partials + (size_t(h) * nblk_cap + (b - a.token_base / kAttBlock)) * kPartialFloats;
      Partial4 Q;
      Q.m = __ldcg(src);
      Q.l = __ldcg(src + 1);
      const float4 v = __ldcg(reinterpret_cast<const float4*>(src + 4) + lane);
      Q.a[0] = v.x; Q.a[1] = v.y; Q.a[2] = v.z; Q.a[3] = v.w;
      merge_into(P, Q);
    }
    float* dst = a.supers + (size_t(h) * a.n_super_max + s) * kPartialFloats;
    if (lane == 0) {
      dst[0] = P.m;
      dst[1] = P.l;
    }
    *reinterpret_cast<float4*>(dst + 4 + 4 * lane) = make_float4(P.a[0], P.a[1], P.a[2], P.a[3]);
  }
  if (!a.final_merge) return;
  // last arriving warp of head h merges the super-chunks in order
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
  const int n_super_total = (nblk_total + kAttSuper - 1) / kAttSuper;
  for (int s = 0; s < n_super_total; ++s) {
    const float* src = a.supers + (size_t(h) * a.n_super_max + s) * kPartialFloats;
    Partial4 Q;
    Q.m = __ldcg(src);
    Q.l = __ldcg(src + 1);
    const float4 v = __ldcg(reinterpret_cast<const float4*>(src + 4) + lane);
    Q.a[0] = v.x; Q.a[1] = v.y; Q.a[2] = v.z; Q.a[3] = v.w;
    merge_into(F, Q);
  }
  uint2 o;
  o.x = uint32_t(to_bf(__fdiv_rn(F.a[0], F.l))) | (uint32_t(to_bf(__fdiv_rn(F.a[1], F.l))) << 16);
  o.y = uint32_t(to_bf(__fdiv_rn(F.a[2], F.l))) | (uint32_t(to_bf(__fdiv_rn(F.a[3], F.l))) << 16);
  *reinterpret_cast<uint2*>(a.out + h * 128 + 4 * lane) = o;
  if (lane == 0) a.head_counters[h] = 0;
}

}  // namespace rec
