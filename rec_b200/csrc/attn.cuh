// GQA decode attention over the quantized KV cache: split-KV partials with
// fused RoPE / quantize-on-append, and the log-sum-exp combine.
//
// Reference: engine/src/rec_mlx/model.py:45-82 (quantize-on-append),
// model.py:108-139 (scores, sink, softmax), megakernel.py:619-693 (split-KV
// partials (max, sum, acc)), megakernel.py:276-318 (LSE merge).
//
// Canonical order (restated by oracle/rec_oracle.c):
//   * q is RoPE'd (pairs (i, i+64), fp32 table of cos/sin), scaled and
//     rounded: qs = bf16(q * 1/sqrt(128)); QS_g = sum of qs over group g
//     (4 accumulators by d mod 4, then (a0+a1)+(a2+a3)).
//   * score(t) = bf16(fma(b1, QS1, fma(s1, A1, fma(b0, QS0, s0*A0)))) with
//     A_g = sum_d qs_d * code_d in the same 4-accumulator order.
//   * tokens are cut into blocks of 256 and tiles of 32; warp w of 4 owns
//     tiles w and w+4 of a block and runs an online softmax over them:
//     m' = max(m, tile max); alpha = exp(m - m'); p_t = exp(s_t - m');
//     l = fma(l, alpha, butterfly-sum(p)); acc = acc*alpha, then
//     acc = fma(p_t, v_t, acc) in token order, v = fma(scale, code, bias).
//   * warp partials merge in order into a block partial; blocks merge in
//     order into super-chunks of 64 blocks; super-chunks merge in order
//     (after the sink partial (sink, 1, 0) when sinks are on);
//     merge: m = max; a_i = exp(m_i - m); l = fma(l1, a1, l2*a2);
//     acc = fma(acc1, a1, acc2*a2); an empty side is the identity.
//   * out = bf16(acc / l).
#pragma once
#include "common.cuh"
#include "quant.cuh"

namespace rec {

constexpr int kAttBlock = 256;
constexpr int kAttTile = 32;
constexpr int kAttWarps = 4;
constexpr int kAttSuper = 64;          // blocks per super-chunk
constexpr int kPartialFloats = 132;    // m, l, pad, pad, acc[128]
constexpr float kQScale = 0.0883883476483184405f;  // 1/sqrt(128)

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

struct Partial4 {  // lane-distributed partial: dims 4*lane .. 4*lane+3
  float m, l;
  float a[4];
};

__device__ __forceinline__ void merge_into(Partial4& x, const Partial4& y) {
  if (y.m == -INFINITY) return;
  if (x.m == -INFINITY) { x = y; return; }
  const float m = fmaxf(x.m, y.m);
  const float a1 = rexp(__fsub_rn(x.m, m)), a2 = rexp(__fsub_rn(y.m, m));
  x.l = __fmaf_rn(x.l, a1, __fmul_rn(y.l, a2));
#pragma unroll
  for (int j = 0; j < 4; ++j) x.a[j] = __fmaf_rn(x.a[j], a1, __fmul_rn(y.a[j], a2));
  x.m = m;
}

// Per-head RMSNorm over 128 dims (q_norm / k_norm): lane l holds 4l..4l+3.
__device__ __forceinline__ void head_norm4(float (&x)[4], const uint16_t* w, float eps) {
  const int lane = threadIdx.x & 31;
  float a = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) a = __fmaf_rn(x[j], x[j], a);
  a = bfly_sum(a);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(a, 128.0f), eps)));
#pragma unroll
  for (int j = 0; j < 4; ++j) x[j] = rbf(__fmul_rn(bf(w[4 * lane + j]), rbf(__fmul_rn(x[j], inv))));
}

template <int BITS>
struct AttnTile {
  static constexpr int ROW_WORDS = 128 * BITS / 32;  // 16 or 32
  static constexpr int ROW_BYTES = ROW_WORDS * 4;
  alignas(128) uint32_t kc[kAttBlock * ROW_WORDS];
  alignas(128) uint32_t vc[kAttBlock * ROW_WORDS];
  alignas(16) uint16_t ks[kAttBlock * 2];
  alignas(16) uint16_t kb[kAttBlock * 2];
  alignas(16) uint16_t vs[kAttBlock * 2];
  alignas(16) uint16_t vb[kAttBlock * 2];
};

template <int BITS>
struct AttnSmem {
  AttnTile<BITS> tile;
  alignas(16) float qs[8][128];
  float QS[8][2];
  alignas(16) float p[kAttWarps][8][kAttTile];
  Partial4 wp_dummy;
  alignas(16) float wacc[kAttWarps][8][128];
  float wm[kAttWarps][8], wl[kAttWarps][8];
  uint64_t bar;
};

__device__ __forceinline__ uint32_t code_of(const uint32_t* row, int bits, int d) {
  return bits == 4 ? (row[d >> 3] >> (4 * (d & 7))) & 15u : (row[d >> 2] >> (8 * (d & 3))) & 255u;
}

// Issue the bulk copies of block b of kv head g (n tokens, rounded up to 4).
template <int BITS>
__device__ __forceinline__ void issue_kv_tile(AttnSmem<BITS>& sm, const AttnArgs& a, int g, int b_local, int n) {
  using Tl = AttnTile<BITS>;
  const int n4 = (n + 3) & ~3;
  const size_t slot = size_t(g) * a.capacity + size_t(b_local) * kAttBlock;
  const uint32_t cb = uint32_t(n4) * Tl::ROW_BYTES, sbytes = uint32_t(n4) * 4;
  mbar_expect_tx(&sm.bar, 2 * cb + 4 * sbytes);
  bulk_g2s(sm.tile.kc, a.k_codes + slot * Tl::ROW_WORDS, cb, &sm.bar);
  bulk_g2s(sm.tile.vc, a.v_codes + slot * Tl::ROW_WORDS, cb, &sm.bar);
  bulk_g2s(sm.tile.ks, a.k_scales + slot * 2, sbytes, &sm.bar);
  bulk_g2s(sm.tile.kb, a.k_biases + slot * 2, sbytes, &sm.bar);
  bulk_g2s(sm.tile.vs, a.v_scales + slot * 2, sbytes, &sm.bar);
  bulk_g2s(sm.tile.vb, a.v_biases + slot * 2, sbytes, &sm.bar);
}

__device__ __forceinline__ int att_hq(int hkv, int nblk, int grid) {
  // q heads per work item: as few as possible while keeping ~2 items per CTA
  int hq = 1;
  while (hq < 8 && hkv * (8 / hq) * nblk > 2 * grid) hq *= 2;
  return hq;
}

// Score of the lane's token for one head; krow holds the token's code words.
template <int BITS>
__device__ __forceinline__ float att_score(const uint32_t (&krow)[AttnTile<BITS>::ROW_WORDS], const float* qs,
                                           const float* QS, float s0, float b0, float s1, float b1) {
  float A[2];
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    float acc4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int d0 = 64 * g; d0 < 64 * g + 64; d0 += 4) {
      const float4 q4 = *reinterpret_cast<const float4*>(qs + d0);
      const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int d = d0 + j;
        const uint32_t c = BITS == 4 ? (krow[d >> 3] >> (4 * (d & 7))) & 15u : (krow[d >> 2] >> (8 * (d & 3))) & 255u;
        acc4[j] = __fmaf_rn(qv[j], float(c), acc4[j]);
      }
    }
    A[g] = __fadd_rn(__fadd_rn(acc4[0], acc4[1]), __fadd_rn(acc4[2], acc4[3]));
  }
  float t = __fmaf_rn(b0, QS[0], __fmul_rn(s0, A[0]));
  t = __fmaf_rn(s1, A[1], t);
  t = __fmaf_rn(b1, QS[1], t);
  return rbf(t);
}

// Block partials.  Persistent grid; work item = (block, kv head, q-head slice).
template <int BITS>
__global__ void __launch_bounds__(128, 2) k_attn_partial(const AttnArgs a) {
  using Tl = AttnTile<BITS>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AttnSmem<BITS>& sm = *reinterpret_cast<AttnSmem<BITS>*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

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
  const int nq = (a.hq / a.hkv) / hq;  // q-head slices per kv head
  const int items = nblk * a.hkv * nq;
  const bool pos_ok = p >= 0 && p < a.capacity + a.token_base && p >= a.token_base - 0;

  auto item_coords = [&](int it, int& b, int& g, int& qsub) {
    qsub = it % nq;
    g = (it / nq) % a.hkv;
    b = b0 + it / (nq * a.hkv);
  };
  auto block_tokens = [&](int b) { return min(kAttBlock, T - b * kAttBlock); };

  uint32_t phase = 0;
  bool pending = false;
  int it = blockIdx.x;
  if (threadIdx.x == 0 && it < items && pos_ok) {
    int b, g, qs_;
    item_coords(it, b, g, qs_);
    issue_kv_tile<BITS>(sm, a, g, b - a.token_base / kAttBlock, block_tokens(b));
  }
  pending = it < items && pos_ok;
  if (a.pdl) grid_wait();
  grid_launch_dependents();
  if (!pos_ok) {
    if (blockIdx.x == 0 && threadIdx.x == 0) report(a.status, kStatusBadPosition);
    return;
  }

  for (; it < items; it += gridDim.x) {
    int b, g, qsub;
    item_coords(it, b, g, qsub);
    const int n = block_tokens(b);
    const int h0 = g * (a.hq / a.hkv) + qsub * hq;
    if (!pending && threadIdx.x == 0) issue_kv_tile<BITS>(sm, a, g, b - a.token_base / kAttBlock, n);
    pending = false;

    // --- queries: (norm,) RoPE, scale, group sums ---------------------------
    const float* cs = a.rope + size_t(p - a.token_base) * 128;
    for (int hh = warp; hh < hq; hh += kAttWarps) {
      const uint16_t* qr = a.qkv + (h0 + hh) * 128;
      float x[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) x[j] = bf(qr[4 * lane + j]);
      if (a.q_norm) head_norm4(x, a.q_norm, a.eps);
      // RoPE on pairs (i, i+64): exchange halves through shared memory
#pragma unroll
      for (int j = 0; j < 4; ++j) sm.qs[hh][4 * lane + j] = x[j];
      __syncwarp();
      float y[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int d = 4 * lane + j, i = d & 63;
        const float c = cs[i], s = cs[64 + i];
        const float lo = sm.qs[hh][i], hi = sm.qs[hh][i + 64];
        y[j] = d < 64 ? rbf(__fmaf_rn(lo, c, -__fmul_rn(hi, s))) : rbf(__fmaf_rn(lo, s, __fmul_rn(hi, c)));
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 4; ++j) sm.qs[hh][4 * lane + j] = rbf(__fmul_rn(y[j], kQScale));
      __syncwarp();
      if (lane < 2) {
        float a4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int d = 64 * lane; d < 64 * lane + 64; ++d) a4[d & 3] = __fadd_rn(a4[d & 3], sm.qs[hh][d]);
        sm.QS[hh][lane] = __fadd_rn(__fadd_rn(a4[0], a4[1]), __fadd_rn(a4[2], a4[3]));
      }
    }

    // --- tile arrival -------------------------------------------------------
    bool ok = mbar_wait(&sm.bar, phase);
    phase ^= 1;
    if (!__syncthreads_and(ok)) {
      if (threadIdx.x == 0) report(a.status, kStatusBulkTimeout);
      if (threadIdx.x == 0) mbar_wait(&sm.bar, phase ^ 1);
      return;
    }

    // --- the new token: RoPE'd k and v, quantized, patched into the tile ----
    if (p >= b * kAttBlock && p < b * kAttBlock + n) {
      const int tloc = p - b * kAttBlock;
      // warps 0,1: k groups 0,1; warps 2,3: v groups 0,1
      const bool is_k = warp < 2;
      const int grp = warp & 1;
      const uint16_t* src = a.qkv + (a.hq + (is_k ? 0 : a.hkv) + g) * 128;
      float kv4[4];
      // each warp needs the full head for norm/RoPE of k; compute all 128 dims
#pragma unroll
      for (int j = 0; j < 4; ++j) kv4[j] = bf(src[4 * lane + j]);
      if (is_k) {
        if (a.k_norm) head_norm4(kv4, a.k_norm, a.eps);
        float* tmp = sm.wacc[warp][0];
#pragma unroll
        for (int j = 0; j < 4; ++j) tmp[4 * lane + j] = kv4[j];
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int d = 4 * lane + j, i = d & 63;
          const float c = cs[i], s = cs[64 + i];
          const float lo = tmp[i], hi = tmp[i + 64];
          kv4[j] = d < 64 ? rbf(__fmaf_rn(lo, c, -__fmul_rn(hi, s))) : rbf(__fmaf_rn(lo, s, __fmul_rn(hi, c)));
        }
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 4; ++j) tmp[4 * lane + j] = kv4[j];
      } else {
        float* tmp = sm.wacc[warp][0];
#pragma unroll
        for (int j = 0; j < 4; ++j) tmp[4 * lane + j] = kv4[j];
      }
      __syncwarp();
      const float* tmp = sm.wacc[warp][0];
      const float v0 = tmp[64 * grp + 2 * lane], v1 = tmp[64 * grp + 2 * lane + 1];
      QGroupParams qp = warp_group_params(v0, v1, BITS);
      const uint32_t word = warp_pack(quant_code(v0, qp, BITS), quant_code(v1, qp, BITS), BITS);
      constexpr int GW = 64 * BITS / 32;  // words per group
      uint32_t* crow = (is_k ? sm.tile.kc : sm.tile.vc) + tloc * Tl::ROW_WORDS + grp * GW;
      if (lane < GW) crow[lane] = word;
      const uint16_t sc = to_bf(qp.scale), bi = to_bf(qp.bias);
      if (lane == 0) {
        (is_k ? sm.tile.ks : sm.tile.vs)[tloc * 2 + grp] = sc;
        (is_k ? sm.tile.kb : sm.tile.vb)[tloc * 2 + grp] = bi;
      }
      if (qsub == 0) {  // one writer per kv head publishes the new slot
        const size_t slot = size_t(g) * a.capacity + size_t(p - a.token_base);
        uint32_t* gc = (is_k ? a.k_codes : a.v_codes) + slot * Tl::ROW_WORDS + grp * GW;
        if (lane < GW) gc[lane] = word;
        if (lane == 0) {
          (is_k ? a.k_scales : a.v_scales)[slot * 2 + grp] = sc;
          (is_k ? a.k_biases : a.v_biases)[slot * 2 + grp] = bi;
        }
      }
    }
    __syncthreads();

    // --- per-warp online softmax over tiles w, w+4 --------------------------
    float m[8], l[8], acc[8][4];
#pragma unroll
    for (int hh = 0; hh < 8; ++hh) {
      m[hh] = -INFINITY;
      l[hh] = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[hh][j] = 0.0f;
    }
    for (int tile = warp; tile < kAttBlock / kAttTile; tile += kAttWarps) {
      const int base = tile * kAttTile;
      if (base >= n) break;
      const int tl = base + lane;
      const bool valid = tl < n;
      // scores (lane = token)
      uint32_t krow[Tl::ROW_WORDS];
#pragma unroll
      for (int w = 0; w < Tl::ROW_WORDS; w += 4) {
        const uint4 q4 = *reinterpret_cast<const uint4*>(&sm.tile.kc[(valid ? tl : 0) * Tl::ROW_WORDS + w]);
        krow[w] = q4.x;
        krow[w + 1] = q4.y;
        krow[w + 2] = q4.z;
        krow[w + 3] = q4.w;
      }
      const float s0 = bf(sm.tile.ks[(valid ? tl : 0) * 2]), s1 = bf(sm.tile.ks[(valid ? tl : 0) * 2 + 1]);
      const float bb0 = bf(sm.tile.kb[(valid ? tl : 0) * 2]), bb1 = bf(sm.tile.kb[(valid ? tl : 0) * 2 + 1]);
      for (int hh = 0; hh < hq; ++hh) {
        const float sc = valid ? att_score<BITS>(krow, sm.qs[hh], sm.QS[hh], s0, bb0, s1, bb1) : -INFINITY;
        const float tmax = bfly_max(sc);
        const float mnew = fmaxf(m[hh], tmax);
        const float alpha = rexp(__fsub_rn(m[hh], mnew));
        const float pt = valid ? rexp(__fsub_rn(sc, mnew)) : 0.0f;
        const float ts = bfly_sum(pt);
        l[hh] = __fmaf_rn(l[hh], alpha, ts);
        m[hh] = mnew;
        sm.p[warp][hh][lane] = pt;
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[hh][j] = __fmul_rn(acc[hh][j], alpha);
      }
      __syncwarp();
      // P*V (lane = 4 dims)
      const int nt = min(kAttTile, n - base);
      const int grp = lane >> 4;
      for (int t = 0; t < nt; ++t) {
        const int tok = base + t;
        uint32_t c4;
        if constexpr (BITS == 4) {
          const uint16_t* row16 = reinterpret_cast<const uint16_t*>(sm.tile.vc + tok * Tl::ROW_WORDS);
          c4 = row16[lane];
        } else {
          c4 = sm.tile.vc[tok * Tl::ROW_WORDS + lane];
        }
        const float vs = bf(sm.tile.vs[tok * 2 + grp]), vb = bf(sm.tile.vb[tok * 2 + grp]);
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t c = BITS == 4 ? (c4 >> (4 * j)) & 15u : (c4 >> (8 * j)) & 255u;
          v[j] = __fmaf_rn(vs, float(c), vb);
        }
        for (int hh = 0; hh < hq; ++hh) {
          const float pp = sm.p[warp][hh][t];
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[hh][j] = __fmaf_rn(pp, v[j], acc[hh][j]);
        }
      }
      __syncwarp();
    }
    // --- warp partials -> block partial (warps merged in order) --------------
    for (int hh = 0; hh < hq; ++hh) {
      if (lane == 0) {
        sm.wm[warp][hh] = m[hh];
        sm.wl[warp][hh] = l[hh];
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) sm.wacc[warp][hh][4 * lane + j] = acc[hh][j];
    }
    __syncthreads();
    for (int hh = warp; hh < hq; hh += kAttWarps) {
      Partial4 P;
      P.m = -INFINITY;
      P.l = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) P.a[j] = 0.0f;
      for (int w = 0; w < kAttWarps; ++w) {
        Partial4 Q;
        Q.m = sm.wm[w][hh];
        Q.l = sm.wl[w][hh];
#pragma unroll
        for (int j = 0; j < 4; ++j) Q.a[j] = sm.wacc[w][hh][4 * lane + j];
        merge_into(P, Q);
      }
      float* dst = a.partials + (size_t(h0 + hh) * (a.capacity / kAttBlock) + (b - a.token_base / kAttBlock)) * kPartialFloats;
      if (lane == 0) {
        dst[0] = P.m;
        dst[1] = P.l;
      }
      *reinterpret_cast<float4*>(dst + 4 + 4 * lane) = make_float4(P.a[0], P.a[1], P.a[2], P.a[3]);
    }
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
    Partial4 P;
    P.m = -INFINITY;
    P.l = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) P.a[j] = 0.0f;
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
  Partial4 F;
  F.m = -INFINITY;
  F.l = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) F.a[j] = 0.0f;
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
