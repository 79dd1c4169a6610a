// Attention math shared by the standalone split-KV kernel and the persistent
// decode kernel: query preparation, exact-integer scores, the per-warp online
// softmax over one 32-token tile, and partial merges.
//
// Canonical order (restated by oracle/rec_oracle.c):
//   * q is RoPE'd (pairs (i, i+64), fp32 cos/sin table), scaled and rounded:
//     qs = bf16(q * 1/sqrt(128)).  Each head gets a 16-bit fixed point:
//     F = min(14 - exponent(max|qs|), 100), qi = rint(qs * 2^F);
//     QS_g = sum of qi over group g (64 dims), exact.
//   * score(t) = bf16(fma(b1, QS1, fma(s1, D1, fma(b0, QS0, s0*D0))) * 2^-F)
//     with D_g = sum_d qi_d * code_d exact (int32) and s, b the token's K
//     scale/bias of group g.
//   * a block of 256 tokens is 8 tiles of 32; warp w of 8 owns tile w:
//     m = tile max; p_t = exp(s_t - m); l = butterfly-sum(p);
//     acc = sum_t fma(p_t, v_t, acc) in token order, v = fma(scale, code, bias).
//   * block partial = warps merged in order; super-chunk = 64 blocks merged in
//     order; final = [sink (sink, 1, 0)] then super-chunks in order;
//     merge: m = max; a_i = exp(m_i - m); l = fma(l1, a1, l2*a2);
//     acc = fma(acc1, a1, acc2*a2); an empty side is the identity.
//   * out = bf16(acc / l).
// Reference: model.py:108-139 (scores, sink, softmax), megakernel.py:619-693
// (split-KV partials), megakernel.py:276-318 (merge).
#pragma once
#include "common.cuh"
#include "quant.cuh"

namespace rec {

constexpr int kAttBlock = 256;
constexpr int kAttTile = 32;
constexpr int kAttWarps = 8;
constexpr int kAttSuper = 64;          // blocks per super-chunk
constexpr int kPartialFloats = 132;    // m, l, pad, pad, acc[128]
constexpr float kQScale = 0.0883883476483184405f;  // 1/sqrt(128)
constexpr int kMaxHq = 4;              // query heads per work item

// Byte dot product: unsigned bytes of a times signed bytes of b, plus c.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

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

__device__ __forceinline__ Partial4 empty_partial() {
  Partial4 p;
  p.m = -INFINITY;
  p.l = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) p.a[j] = 0.0f;
  return p;
}

// Exact small-integer to float: 2^23 + c has c in the low mantissa bits.
__device__ __forceinline__ float code_f(uint32_t c) {
  return __fsub_rn(__uint_as_float(0x4B000000u | c), 8388608.0f);
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

// RoPE of a 128-dim head held by a warp (lane l: dims 4l..4l+3), through a
// 128-float shared scratch.  Pairs (i, i+64): lo' = bf16(fma(lo, c, -hi*s)),
// hi' = bf16(fma(lo, s, hi*c)).
__device__ __forceinline__ void rope4(float (&x)[4], const float* cs, float* scratch) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int j = 0; j < 4; ++j) scratch[4 * lane + j] = x[j];
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int d = 4 * lane + j, i = d & 63;
    const float c = cs[i], s = cs[64 + i];
    const float lo = scratch[i], hi = scratch[i + 64];
    x[j] = d < 64 ? rbf(__fmaf_rn(lo, c, -__fmul_rn(hi, s))) : rbf(__fmaf_rn(lo, s, __fmul_rn(hi, c)));
  }
  __syncwarp();
}

// Prepared query of one head in shared memory: byte limbs in the layout of
// the K code words (8-bit: word w = dims 4w..4w+3; 4-bit: word w = dims
// 8w..8w+7 split in even / odd nibble lanes).
struct QHead {
  uint32_t hi[32], lo[32];  // 8-bit: [w]; 4-bit: [2w] even, [2w+1] odd
  float QS[2];              // float(sum qi) per group, exact
  float down;               // 2^-F
  float pad;
};

// One warp prepares head h: x = its (normed, RoPE'd) dims 4l..4l+3.
template <int BITS>
__device__ __forceinline__ void prep_qhead(const float (&x)[4], QHead& q, float* scratch) {
  const int lane = threadIdx.x & 31;
  float qs[4];
  float mx = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    qs[j] = rbf(__fmul_rn(x[j], kQScale));
    mx = fmaxf(mx, fabsf(qs[j]));
  }
  mx = bfly_max(mx);
  const int E = int((__float_as_uint(mx) >> 23) & 0xFF) - 127;
  int F = 14 - E;
  F = F > 100 ? 100 : F;
  const float up = __uint_as_float(uint32_t(F + 127) << 23);
  int qi[4];
  int part = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    qi[j] = __float2int_rn(__fmul_rn(qs[j], up));
    part += qi[j];
  }
  // group sums: lanes 0..15 hold group 0, 16..31 group 1 (exact integers)
#pragma unroll
  for (int off = 8; off >= 1; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
  if (lane == 0) q.QS[0] = float(part);
  if (lane == 16) q.QS[1] = float(part);
  if (lane == 0) q.down = __uint_as_float(uint32_t(127 - F) << 23);
  if constexpr (BITS == 8) {
    // lane l owns dims 4l..4l+3 = word l
    uint32_t h = 0, lo = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      h |= (uint32_t(qi[j] >> 8) & 0xFFu) << (8 * j);
      lo |= (uint32_t(qi[j]) & 0xFFu) << (8 * j);
    }
    q.hi[lane] = h;
    q.lo[lane] = lo;
  } else {
    // word w = dims 8w..8w+7: even dims from lanes 2w (dims 0,2) and 2w+1
    // (dims 4,6); odd dims likewise.  Exchange through the scratch.
    int* si = reinterpret_cast<int*>(scratch);
#pragma unroll
    for (int j = 0; j < 4; ++j) si[4 * lane + j] = qi[j];
    __syncwarp();
    if (lane < 16) {
      const int w = lane;
      uint32_t he = 0, ho = 0, le = 0, lo = 0;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const int ve = si[8 * w + 2 * q4], vo = si[8 * w + 2 * q4 + 1];
        he |= (uint32_t(ve >> 8) & 0xFFu) << (8 * q4);
        ho |= (uint32_t(vo >> 8) & 0xFFu) << (8 * q4);
        le |= (uint32_t(ve) & 0xFFu) << (8 * q4);
        lo |= (uint32_t(vo) & 0xFFu) << (8 * q4);
      }
      q.hi[2 * w] = he;
      q.hi[2 * w + 1] = ho;
      q.lo[2 * w] = le;
      q.lo[2 * w + 1] = lo;
    }
    __syncwarp();
  }
}

// Scores of the lane's token for heads [0, hq) and the tile's online
// softmax; writes p into pbuf[h][lane] and returns (m, l) per head.
// krow: the token's code words in shared memory (row of RW words).
template <int BITS>
__device__ __forceinline__ void tile_scores(const uint32_t* krow, bool valid, float s0, float b0, float s1,
                                            float b1, const QHead* qh, int hq, float (&m)[kMaxHq],
                                            float (&l)[kMaxHq], float (*pbuf)[kAttTile]) {
  const int lane = threadIdx.x & 31;
  int dhi0[kMaxHq], dlo0[kMaxHq], dhi1[kMaxHq], dlo1[kMaxHq];
#pragma unroll
  for (int h = 0; h < kMaxHq; ++h) dhi0[h] = dlo0[h] = dhi1[h] = dlo1[h] = 0;
  // 16-byte chunks of the row, visited in a per-lane rotated order (sums are
  // exact, so the order is free) so that the lanes of a quarter warp hit
  // different banks.
  constexpr int CHUNKS = BITS == 8 ? 8 : 4;
  const int rot = BITS == 8 ? lane : (lane >> 1);
  // not unrolled: this runs once per layer from a cold instruction cache
#pragma unroll 1
  for (int j = 0; j < CHUNKS; ++j) {
    const int c = (j + rot) & (CHUNKS - 1);
    const uint4 kw = *reinterpret_cast<const uint4*>(krow + 4 * c);
    const uint32_t ks[4] = {kw.x, kw.y, kw.z, kw.w};
    const bool g1 = c >= CHUNKS / 2;
#pragma unroll
    for (int h = 0; h < kMaxHq; ++h) {
      if (h >= hq) break;
      int hi = 0;
      unsigned lo = 0;
      if constexpr (BITS == 8) {
        const uint4 qh4 = *reinterpret_cast<const uint4*>(&qh[h].hi[4 * c]);
        const uint4 ql4 = *reinterpret_cast<const uint4*>(&qh[h].lo[4 * c]);
        const uint32_t qhs[4] = {qh4.x, qh4.y, qh4.z, qh4.w};
        const uint32_t qls[4] = {ql4.x, ql4.y, ql4.z, ql4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          hi = dp4a_us(ks[i], qhs[i], hi);  // unsigned codes x signed high limbs
          lo = __dp4a(ks[i], qls[i], lo);
        }
      } else {
        const uint4 qh0 = *reinterpret_cast<const uint4*>(&qh[h].hi[8 * c]);
        const uint4 qh1 = *reinterpret_cast<const uint4*>(&qh[h].hi[8 * c + 4]);
        const uint4 ql0 = *reinterpret_cast<const uint4*>(&qh[h].lo[8 * c]);
        const uint4 ql1 = *reinterpret_cast<const uint4*>(&qh[h].lo[8 * c + 4]);
        const uint32_t qhs[8] = {qh0.x, qh0.y, qh0.z, qh0.w, qh1.x, qh1.y, qh1.z, qh1.w};
        const uint32_t qls[8] = {ql0.x, ql0.y, ql0.z, ql0.w, ql1.x, ql1.y, ql1.z, ql1.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t e = ks[i] & 0x0F0F0F0Fu, o = (ks[i] >> 4) & 0x0F0F0F0Fu;
          hi = dp4a_us(e, qhs[2 * i], hi);
          hi = dp4a_us(o, qhs[2 * i + 1], hi);
          lo = __dp4a(e, qls[2 * i], lo);
          lo = __dp4a(o, qls[2 * i + 1], lo);
        }
      }
      if (g1) {
        dhi1[h] += hi;
        dlo1[h] += int(lo);
      } else {
        dhi0[h] += hi;
        dlo0[h] += int(lo);
      }
    }
  }
#pragma unroll
  for (int h = 0; h < kMaxHq; ++h) {
    if (h >= hq) break;
    const int D0 = dhi0[h] * 256 + dlo0[h], D1 = dhi1[h] * 256 + dlo1[h];
    float t = __fmaf_rn(b0, qh[h].QS[0], __fmul_rn(s0, float(D0)));
    t = __fmaf_rn(s1, float(D1), t);
    t = __fmaf_rn(b1, qh[h].QS[1], t);
    const float sc = valid ? rbf(__fmul_rn(t, qh[h].down)) : -INFINITY;
    const float mx = bfly_max(sc);
    const float pt = valid ? rexp(__fsub_rn(sc, mx)) : 0.0f;
    m[h] = mx;
    l[h] = bfly_sum(pt);
    pbuf[h][lane] = pt;
  }
}

}  // namespace rec
