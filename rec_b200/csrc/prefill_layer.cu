// The per-token kernels of a chunked prompt prefill (rec_prefill_chunk in
// decode.cu strings them together with the tensor-core GEMMs of prefill.cu):
// embedding rows, row RMSNorm, q / k head norms and RoPE, causal attention of
// the chunk's queries over the quantized cache, the residual add, and the
// router of every token.
//
// Reference: the chunked prefill of QATSession.prefill
// (engine/src/rec_mlx/quantized.py:102-148) running the native MLX model
// (model.py:108-139 attention with sinks over the quantized cache,
// model.py:216-271 norms, router and residuals) and the reference's prefill
// kernels (engine/src/rec_mlx/m4_max_prefill.py:6-104,
// kernels/m4_max_prefill.py:49-144).
//
// Numerics: the projections run on the tensor cores with fp32 accumulation
// (prefill.cu), so a prefilled chunk matches the token-by-token decode path
// within a tolerance, not bit for bit.  The attention follows the reference's
// rounding points: q is scaled by 1/sqrt(128) and rounded to bf16, scores are
// rounded to bf16, the softmax runs in fp32 with the sink logit in the
// normaliser.  K enters the score MMAs as two fp16 parts (k_hi = fp16(k),
// k_lo = fp16(k - k_hi): ~22 significant bits, so a score is exact to fp32
// before its bf16 rounding), V is dequantized to fp16 (2^-11 relative), and
// q_s and the probabilities enter the MMAs as fp16, with fp32 accumulation.  The router and the expert selection are the decode path's
// (canonical logit order, softmax or sigmoid + bias, top-k with the lowest id
// on ties, weights p / (sum + 1e-20)).
#include "attn_core.cuh"
#include "capi_common.h"
#include "moe.cuh"
#include "prefill_layer.h"

namespace rec {
namespace {

// ---------------------------------------------------------------------------
// embedding rows: h[t] = bf16(fma(scale, q, bias)) of token tokens[t]
// ---------------------------------------------------------------------------
__global__ void k_pf_embed(QMatDev emb, int sd, const int* __restrict__ tokens, int T, int H, int V,
                           uint16_t* __restrict__ h, int* status) {
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    int tok = tokens[t];
    if (tok < 0 || tok >= V) {
      if (threadIdx.x == 0) report(status, kStatusBadToken);
      tok = 0;
    }
    const uint32_t* w = emb.w + size_t(tok) * (H / 8);
    for (int i = threadIdx.x; i < H; i += blockDim.x) {
      const float q = float((w[i >> 3] >> (4 * (i & 7))) & 15u);
      const float s = sb<2>(emb.s[size_t(tok) * (H / 64) + (i >> 6)], sd);
      const float b = sb<2>(emb.b[size_t(tok) * (H / 64) + (i >> 6)], sd);
      h[size_t(t) * H + i] = to_bf(__fmaf_rn(s, q, b));
    }
  }
}

// ---------------------------------------------------------------------------
// row RMSNorm (H = 2048, 256 threads, thread i owns elements 8i..8i+7):
// out = bf16(w * bf16(x * inv)), inv = 1 / sqrt(mean(x^2) + eps)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_pf_rmsnorm(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                                    int T, float eps, uint16_t* __restrict__ out) {
  __shared__ float red[8];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const uint4 wv = *reinterpret_cast<const uint4*>(w + t * 8);
  for (int row = blockIdx.x; row < T; row += gridDim.x) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + size_t(row) * 2048 + t * 8);
    const uint32_t us[4] = {u.x, u.y, u.z, u.w};
    float v[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      v[2 * q] = __uint_as_float(us[q] << 16);
      v[2 * q + 1] = __uint_as_float(us[q] & 0xFFFF0000u);
    }
    float acc = 0.0f;
#pragma unroll
    for (int q = 0; q < 8; ++q) acc = __fmaf_rn(v[q], v[q], acc);
    acc = bfly_sum(acc);
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    float total = 0.0f;
    for (int g = 0; g < 8; ++g) total = __fadd_rn(total, red[g]);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, 2048.0f), eps)));
    const uint32_t ws_[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t lo = to_bf(__fmul_rn(__uint_as_float(ws_[q] << 16), rbf(__fmul_rn(v[2 * q], inv))));
      const uint32_t hi = to_bf(__fmul_rn(__uint_as_float(ws_[q] & 0xFFFF0000u), rbf(__fmul_rn(v[2 * q + 1], inv))));
      o[q] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4*>(out + size_t(row) * 2048 + t * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    __syncthreads();  // red is rewritten by the next row
  }
}

// ---------------------------------------------------------------------------
// q and k heads of every token: optional head RMSNorm, then RoPE at position
// p0 + t (pairs (i, i + 64), the session's fp32 cos | sin table), in place.
// One warp per (token, head); heads 0..hq-1 of q, then 0..hkv-1 of k.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_pf_qk(uint16_t* __restrict__ q, int hq, uint16_t* __restrict__ k, int hkv,
                                               int T, int p0, const float* __restrict__ rope,
                                               const uint16_t* __restrict__ qn, const uint16_t* __restrict__ kn,
                                               float eps) {
  __shared__ float scratch[8][128];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per = hq + hkv;
  for (int item = blockIdx.x * 8 + warp; item < T * per; item += gridDim.x * 8) {
    const int t = item / per, hh = item % per;
    const bool is_q = hh < hq;
    uint16_t* row = is_q ? q + (size_t(t) * hq + hh) * 128 : k + (size_t(t) * hkv + (hh - hq)) * 128;
    float x[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = bf(row[4 * lane + j]);
    const uint16_t* nw = is_q ? qn : kn;
    if (nw) head_norm4(x, nw, eps);
    rope4(x, rope + size_t(p0 + t) * 128, scratch[warp]);
#pragma unroll
    for (int j = 0; j < 4; ++j) row[4 * lane + j] = to_bf(x[j]);
  }
}

// h = bf16(h + o)
__global__ void k_pf_add(uint16_t* __restrict__ h, const uint16_t* __restrict__ o, size_t n) {
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    h[i] = to_bf(__fadd_rn(bf(h[i]), bf(o[i])));
}

// ---------------------------------------------------------------------------
// router of every token: one CTA (8 warps) per token; warp w computes the
// logits of experts w, w + 8, ... in the decode path's canonical order (lane l
// owns 8-element chunks l, l + 32, ...; fmas in order; butterfly; bf16), then
// warp 0 selects the top-k exactly as the decode path's router does.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_pf_router(const uint16_t* __restrict__ xn, const uint16_t* __restrict__ wr,
                                                   const float* __restrict__ bias, int T, int E, int k, int mode,
                                                   int* __restrict__ ids, float* __restrict__ wts) {
  __shared__ float p[kMaxExperts];
  __shared__ unsigned keys[kMaxExperts];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    const uint16_t* x = xn + size_t(t) * 2048;
    for (int e = warp; e < E; e += 8) {
      const uint16_t* w = wr + size_t(e) * 2048;
      float acc = 0.0f;
#pragma unroll 2
      for (int m = 0; m < 8; ++m) {
        const int c = lane + 32 * m;
        const uint4 wv = *reinterpret_cast<const uint4*>(w + c * 8);
        const uint4 xv = *reinterpret_cast<const uint4*>(x + c * 8);
        const uint32_t ws_[4] = {wv.x, wv.y, wv.z, wv.w};
        const uint32_t xs_[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          acc = __fmaf_rn(__uint_as_float(ws_[q] << 16), __uint_as_float(xs_[q] << 16), acc);
          acc = __fmaf_rn(__uint_as_float(ws_[q] & 0xFFFF0000u), __uint_as_float(xs_[q] & 0xFFFF0000u), acc);
        }
      }
      acc = bfly_sum(acc);
      if (lane == 0) p[e] = rbf(acc);
    }
    __syncthreads();
    if (warp == 0) {
      if (mode == 0) {
        float mx = -INFINITY;
        for (int i = lane; i < E; i += 32) mx = fmaxf(mx, p[i]);
        mx = bfly_max(mx);
        float s = 0.0f;
        for (int i = lane; i < E; i += 32) {
          const float c = rexp(__fsub_rn(p[i], mx));
          p[i] = c;
          s = __fadd_rn(s, c);
        }
        s = bfly_sum(s);
        for (int i = lane; i < E; i += 32) {
          const float pi = __fdiv_rn(p[i], s);
          p[i] = pi;
          keys[i] = route_key(pi);
        }
      } else {
        for (int i = lane; i < E; i += 32) {
          const float pi = rsigmoid(p[i]);
          p[i] = pi;
          keys[i] = route_key(__fadd_rn(pi, bias[i]));
        }
      }
      __syncwarp();
      unsigned bk = 0u;
      int bi = 0;
      for (int i = lane; i < E; i += 32)
        if (keys[i] > bk) { bk = keys[i]; bi = i; }
      float s2 = 0.0f, my_p = 0.0f;
      int my_id = 0;
      for (int r = 0; r < k; ++r) {
        const unsigned wbest = __reduce_max_sync(0xffffffffu, bk);
        int widx = int(__reduce_min_sync(0xffffffffu, (bk == wbest && bk) ? unsigned(bi) : ~0u));
        if (unsigned(widx) >= unsigned(E)) widx = 0;
        const float pw = p[widx];
        if (lane == (widx & 31)) {
          keys[widx] = 0u;
          bk = 0u;
          bi = 0;
          for (int i = lane; i < E; i += 32)
            if (keys[i] > bk) { bk = keys[i]; bi = i; }
        }
        if (lane == r) {
          my_id = widx;
          my_p = pw;
        }
        s2 = __fadd_rn(s2, pw);
      }
      s2 = __fadd_rn(s2, 1e-20f);
      if (lane < k) {
        ids[size_t(t) * k + lane] = my_id;
        wts[size_t(t) * k + lane] = __fdiv_rn(my_p, s2);
      }
    }
    __syncthreads();  // p and keys are rewritten by the next token
  }
}

// ---------------------------------------------------------------------------
// Causal attention of a chunk's queries over the quantized cache.  CTA =
// (16 query tokens, kv head g); warp w = q head 8g + w, its 16 rows = the 16
// tokens.  KV blocks of 64 tokens are dequantized by the CTA into shared
// memory (K as an fp16 pair k_hi + k_lo, V as fp16, rows padded to 136
// elements so the fragment loads are conflict-free); per block each warp
// computes S = Q K_hi^T + Q K_lo^T with mma.sync m16n8k16 (fp16, fp32
// accumulate), rounds S to bf16, masks the
// future, folds an online softmax (fp32) and accumulates P V (fp16 P, fp32
// accumulate).  Row t attends to positions 0 .. p0 + t.
// ---------------------------------------------------------------------------
constexpr int kPaQ = 16, kPaKV = 64, kPaLd = 136;

struct PaArgs {
  const uint16_t* q;  // bf16 [T, hq, 128], RoPE'd
  const uint32_t* k_codes;
  const uint16_t* k_scales;
  const uint16_t* k_biases;
  const uint32_t* v_codes;
  const uint16_t* v_scales;
  const uint16_t* v_biases;
  int capacity, hq, p0, T;
  const uint16_t* sinks;  // bf16 [hq] or null
  uint16_t* out;          // bf16 [T, hq * 128]
};

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
               : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// exp for the prefill softmax (x <= 0 or -inf): the library's own exp, 0 at -inf
__device__ __forceinline__ float pexp(float x) { return x == -INFINITY ? 0.0f : rexp(x); }

struct PaSmem {
  alignas(16) uint16_t ks[kPaKV * kPaLd];   // K as fp16: k_hi
  alignas(16) uint16_t ks2[kPaKV * kPaLd];  // fp16(k - k_hi)
  alignas(16) uint16_t vs[kPaKV * kPaLd];
};

template <int BITS>
__global__ void __launch_bounds__(256, 1) k_pf_attn(const PaArgs a) {
  extern __shared__ __align__(16) uint8_t pa_smem_raw[];
  PaSmem& sm = *reinterpret_cast<PaSmem*>(pa_smem_raw);
  uint16_t* ks = sm.ks;
  uint16_t* ks2 = sm.ks2;
  uint16_t* vs = sm.vs;
  constexpr int RW = 128 * BITS / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, tq = lane & 3;
  const int t0 = blockIdx.x * kPaQ, g = blockIdx.y;
  const int h = g * 8 + warp;
  // query fragments: rows gq / gq + 8 = tokens t0 + gq / t0 + gq + 8;
  // k-step ks covers dims 16 ks .. 16 ks + 15 (a0, a2: row gq; a1, a3: row gq + 8)
  uint32_t qa[8][4];
  {
    const int r0 = t0 + gq, r1 = t0 + gq + 8;
    const uint16_t* q0 = a.q + (size_t(r0) * a.hq + h) * 128;
    const uint16_t* q1 = a.q + (size_t(r1) * a.hq + h) * 128;
    // q_s = bf16(q / sqrt(128)) (the reference's rounding), carried as fp16
    // (exact for |q_s| in [2^-14, 65504]) so that K can enter as fp16 too
    auto ld = [&](const uint16_t* row, bool ok, int d) -> uint32_t {
      if (!ok) return 0u;
      const uint32_t w = *reinterpret_cast<const uint32_t*>(row + d);
      const float lo = rbf(__fmul_rn(__uint_as_float(w << 16), kQScale));
      const float hi = rbf(__fmul_rn(__uint_as_float(w & 0xFFFF0000u), kQScale));
      return pack_h2(lo, hi);
    };
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      qa[s][0] = ld(q0, r0 < a.T, 16 * s + 2 * tq);
      qa[s][1] = ld(q1, r1 < a.T, 16 * s + 2 * tq);
      qa[s][2] = ld(q0, r0 < a.T, 16 * s + 8 + 2 * tq);
      qa[s][3] = ld(q1, r1 < a.T, 16 * s + 8 + 2 * tq);
    }
  }
  float m[2], l[2];
  const float sink = a.sinks ? bf(a.sinks[h]) : -INFINITY;
  m[0] = m[1] = sink;
  l[0] = l[1] = a.sinks ? 1.0f : 0.0f;
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  const int qpos0 = a.p0 + t0 + gq, qpos1 = qpos0 + 8;  // positions of this lane's two rows
  const int last = a.p0 + min(t0 + kPaQ, a.T) - 1;
  const int nblk = last / kPaKV + 1;
  const uint32_t vbase = uint32_t(__cvta_generic_to_shared(vs));
  for (int b = 0; b < nblk; ++b) {
    __syncthreads();  // the previous block's fragments have been read
    {
      // dequantize: thread = (token, quarter of 32 dims)
      const int tok = threadIdx.x >> 2, qd = threadIdx.x & 3;
      const int pos = b * kPaKV + tok;
      uint4* kd = reinterpret_cast<uint4*>(ks + tok * kPaLd + qd * 32);
      uint4* kd2 = reinterpret_cast<uint4*>(ks2 + tok * kPaLd + qd * 32);
      uint4* vd = reinterpret_cast<uint4*>(vs + tok * kPaLd + qd * 32);
      if (pos <= last) {
        const size_t row = size_t(g) * a.capacity + pos;
        const int grp = qd >> 1;
        const float s_k = bf(a.k_scales[row * 2 + grp]), b_k = bf(a.k_biases[row * 2 + grp]);
        const float s_v = bf(a.v_scales[row * 2 + grp]), b_v = bf(a.v_biases[row * 2 + grp]);
        constexpr int WPQ = 32 * BITS / 32;  // code words per 32 dims
        uint32_t kw[WPQ], vw[WPQ];
#pragma unroll
        for (int i = 0; i < WPQ; i += 4) {
          const uint4 x = *reinterpret_cast<const uint4*>(a.k_codes + row * RW + qd * WPQ + i);
          const uint4 y = *reinterpret_cast<const uint4*>(a.v_codes + row * RW + qd * WPQ + i);
          kw[i] = x.x; kw[i + 1] = x.y; kw[i + 2] = x.z; kw[i + 3] = x.w;
          vw[i] = y.x; vw[i + 1] = y.y; vw[i + 2] = y.z; vw[i + 3] = y.w;
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {  // 8 dims per 16-byte store
          uint32_t kp[4], kp2[4], vp[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float k2[2], v2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int d = 8 * c + 2 * j + e;  // dim within the quarter
              uint32_t kc, vc;
              if constexpr (BITS == 4) {
                kc = (kw[d >> 3] >> (4 * (d & 7))) & 15u;
                vc = (vw[d >> 3] >> (4 * (d & 7))) & 15u;
              } else {
                kc = (kw[d >> 2] >> (8 * (d & 3))) & 255u;
                vc = (vw[d >> 2] >> (8 * (d & 3))) & 255u;
              }
              k2[e] = __fmaf_rn(s_k, code_f(kc), b_k);
              v2[e] = __fmaf_rn(s_v, code_f(vc), b_v);
            }
            const __half2 hk = __floats2half2_rn(k2[0], k2[1]);
            kp[j] = *reinterpret_cast<const uint32_t*>(&hk);
            kp2[j] = pack_h2(__fsub_rn(k2[0], __low2float(hk)), __fsub_rn(k2[1], __high2float(hk)));
            vp[j] = pack_h2(v2[0], v2[1]);
          }
          kd[c] = make_uint4(kp[0], kp[1], kp[2], kp[3]);
          kd2[c] = make_uint4(kp2[0], kp2[1], kp2[2], kp2[3]);
          vd[c] = make_uint4(vp[0], vp[1], vp[2], vp[3]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) kd[c] = kd2[c] = vd[c] = make_uint4(0, 0, 0, 0);
      }
    }
    __syncthreads();
    // S = Q K^T: n-tile nt = tokens b*64 + 8 nt .. + 7
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
      const uint16_t* krow = ks + (8 * nt + gq) * kPaLd + 2 * tq;
      const uint16_t* krow2 = ks2 + (8 * nt + gq) * kPaLd + 2 * tq;
#pragma unroll
      for (int st = 0; st < 8; ++st) {
        mma_f16_16816(s[nt], qa[st], *reinterpret_cast<const uint32_t*>(krow + 16 * st),
                      *reinterpret_cast<const uint32_t*>(krow + 16 * st + 8));
        mma_f16_16816(s[nt], qa[st], *reinterpret_cast<const uint32_t*>(krow2 + 16 * st),
                      *reinterpret_cast<const uint32_t*>(krow2 + 16 * st + 8));
      }
    }
    // bf16 scores, causal mask, online softmax of the lane's two rows
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int pos = b * kPaKV + 8 * nt + 2 * tq + (e & 1);
        const int qp = e < 2 ? qpos0 : qpos1;
        const bool ok = pos <= qp && (e < 2 ? t0 + gq : t0 + gq + 8) < a.T;
        s[nt][e] = ok ? rbf(s[nt][e]) : -INFINITY;
        mx[e >> 1] = fmaxf(mx[e >> 1], s[nt][e]);
      }
    float alpha[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
      const float mn = fmaxf(m[i], mx[i]);
      alpha[i] = mn == -INFINITY ? 1.0f : pexp(__fsub_rn(m[i], mn));
      m[i] = mn;
    }
    float rs[2] = {0.0f, 0.0f};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = e >> 1;
        const float pv = m[i] == -INFINITY ? 0.0f : pexp(__fsub_rn(s[nt][e], m[i]));
        s[nt][e] = pv;
        rs[i] = __fadd_rn(rs[i], pv);
      }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      rs[i] = __fadd_rn(rs[i], __shfl_xor_sync(0xffffffffu, rs[i], 1));
      rs[i] = __fadd_rn(rs[i], __shfl_xor_sync(0xffffffffu, rs[i], 2));
      l[i] = __fmaf_rn(l[i], alpha[i], rs[i]);
    }
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] = __fmul_rn(o[n][0], alpha[0]);
      o[n][1] = __fmul_rn(o[n][1], alpha[0]);
      o[n][2] = __fmul_rn(o[n][2], alpha[1]);
      o[n][3] = __fmul_rn(o[n][3], alpha[1]);
    }
    // O += P V: k-step kk = tokens 16 kk .. 16 kk + 15 (n-tiles 2kk, 2kk + 1)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_h2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_h2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_h2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_h2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
      // ldmatrix.trans: thread j*8 + i addresses row 16 kk + 8 (j & 1) + i,
      // dims 8 (nd + (j >> 1)) .. of V
      const int j = lane >> 3, i = lane & 7;
#pragma unroll
      for (int nd = 0; nd < 16; nd += 2) {
        const uint32_t addr =
            vbase + uint32_t(((16 * kk + 8 * (j & 1) + i) * kPaLd + 8 * (nd + (j >> 1))) * 2);
        uint32_t r0, r1, r2, r3;
        ldsm_x4_trans(addr, r0, r1, r2, r3);
        mma_f16_16816(o[nd], pa, r0, r1);
        mma_f16_16816(o[nd + 1], pa, r2, r3);
      }
    }
  }
  // out = bf16(o / l): row gq -> c0, c1; row gq + 8 -> c2, c3 (dims 8 n + 2 tq, + 1)
  const int r0 = t0 + gq, r1 = t0 + gq + 8;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    const int d = 8 * n + 2 * tq;
    if (r0 < a.T) {
      const uint32_t v = uint32_t(to_bf(__fdiv_rn(o[n][0], l[0]))) | (uint32_t(to_bf(__fdiv_rn(o[n][1], l[0]))) << 16);
      *reinterpret_cast<uint32_t*>(a.out + (size_t(r0) * a.hq + h) * 128 + d) = v;
    }
    if (r1 < a.T) {
      const uint32_t v = uint32_t(to_bf(__fdiv_rn(o[n][2], l[1]))) | (uint32_t(to_bf(__fdiv_rn(o[n][3], l[1]))) << 16);
      *reinterpret_cast<uint32_t*>(a.out + (size_t(r1) * a.hq + h) * 128 + d) = v;
    }
  }
}

}  // namespace

cudaError_t pf_embed(const QMatDev& emb, int sd, const int* tokens, int T, int H, int V, uint16_t* h, int* status,
                     cudaStream_t st) {
  k_pf_embed<<<min(T, 4 * sm_count()), 256, 0, st>>>(emb, sd, tokens, T, H, V, h, status);
  return cudaGetLastError();
}

cudaError_t pf_rmsnorm(const uint16_t* x, const uint16_t* w, int T, float eps, uint16_t* out, cudaStream_t st) {
  k_pf_rmsnorm<<<min(T, 4 * sm_count()), 256, 0, st>>>(x, w, T, eps, out);
  return cudaGetLastError();
}

cudaError_t pf_qk(uint16_t* q, int hq, uint16_t* k, int hkv, int T, int p0, const float* rope, const uint16_t* qn,
                  const uint16_t* kn, float eps, cudaStream_t st) {
  const int items = T * (hq + hkv);
  k_pf_qk<<<min((items + 7) / 8, 8 * sm_count()), 256, 0, st>>>(q, hq, k, hkv, T, p0, rope, qn, kn, eps);
  return cudaGetLastError();
}

cudaError_t pf_add(uint16_t* h, const uint16_t* o, size_t n, cudaStream_t st) {
  k_pf_add<<<4 * sm_count(), 256, 0, st>>>(h, o, n);
  return cudaGetLastError();
}

cudaError_t pf_router(const uint16_t* xn, const uint16_t* router, const float* bias, int T, int E, int k, int mode,
                      int* ids, float* wts, cudaStream_t st) {
  k_pf_router<<<min(T, 8 * sm_count()), 256, 0, st>>>(xn, router, bias, T, E, k, mode, ids, wts);
  return cudaGetLastError();
}

cudaError_t pf_attention(const uint16_t* q, int hq, int hkv, const RecKVLayer& kv, int capacity, int bits, int p0,
                         int T, const uint16_t* sinks, uint16_t* out, cudaStream_t st) {
  PaArgs a;
  a.q = q;
  a.k_codes = static_cast<const uint32_t*>(kv.k_codes);
  a.k_scales = static_cast<const uint16_t*>(kv.k_scales);
  a.k_biases = static_cast<const uint16_t*>(kv.k_biases);
  a.v_codes = static_cast<const uint32_t*>(kv.v_codes);
  a.v_scales = static_cast<const uint16_t*>(kv.v_scales);
  a.v_biases = static_cast<const uint16_t*>(kv.v_biases);
  a.capacity = capacity;
  a.hq = hq;
  a.p0 = p0;
  a.T = T;
  a.sinks = sinks;
  a.out = out;
  dim3 grid((T + kPaQ - 1) / kPaQ, hkv);
  const size_t smem = sizeof(PaSmem);
  const void* kern = bits == 4 ? reinterpret_cast<const void*>(k_pf_attn<4>) : reinterpret_cast<const void*>(k_pf_attn<8>);
  cudaError_t e = set_smem_limit(kern, smem);
  if (e != cudaSuccess) return e;
  if (bits == 4) k_pf_attn<4><<<grid, 256, smem, st>>>(a);
  else k_pf_attn<8><<<grid, 256, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace rec
