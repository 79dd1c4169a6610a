// Attention math shared by the standalone split-KV kernel and the persistent
// decode kernel: query preparation, exact-integer scores, the per-warp online
// softmax over one 32-token tile, and partial merges.
//
// Canonical order (restated by oracle/rec_oracle.c):
//   * q is RoPE'd (pairs (i, i+64), fp32 cos/sin table), scaled and rounded:
//     qs = bf16(q * 1/sqrt(128)).  Each head gets a 16-bit fixed point:
//     F = min(14 - exponent(max|qs| * (1 + 2^-7)), 100), qi = rint(qs * 2^F);
//     QS_g = sum of qi over group g (64 dims), exact.
//   * score(t) = bf16(fma(b1, QS1, fma(s1, D1, fma(b0, QS0, s0*D0))) * 2^-F)
//     with D_g = sum_d qi_d * code_d exact (int32) and s, b the token's K
//     scale/bias of group g.
//   * a block of 256 tokens is 8 tiles of 32; warp w folds tile w of each
//     block of a work item into a running (m, l, acc) state (tile_fold):
//     m' = max(m, tile max); alpha = aexp(m - m'); p = aexp(s - m');
//     l' = fma(l, alpha, sum p); acc' = fma(acc, alpha, PV) with PV from
//     fixed-point weights (exact integer dot, one rounding per dim).
//   * item partial = the 8 warp states folded as a tree; super-chunk = its
//     items merged in order; final = [sink (sink, 1, 0)] then super-chunks in
//     order; merge: m = max; a_i = exp(m_i - m); l = fma(l1, a1, l2*a2);
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
  // the factor of the side holding the max is exp(0) = 1: only the other
  // one is computed
  const bool xm = x.m >= y.m;
  const float m = xm ? x.m : y.m;
  const float e = rexp(__fsub_rn(xm ? y.m : x.m, m));
  const float a1 = xm ? 1.0f : e, a2 = xm ? e : 1.0f;
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

__device__ __forceinline__ void store_partial(float* dst, const Partial4& P) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) {
    dst[0] = P.m;
    dst[1] = P.l;
  }
  *reinterpret_cast<float4*>(dst + 4 + 4 * lane) = make_float4(P.a[0], P.a[1], P.a[2], P.a[3]);
}

// Folds partials [i0, i1) of a [*, kPartialFloats] array (L2 reads) into P in
// order, with kBatch loads in flight.
__device__ __forceinline__ void fold_partials(Partial4& P, const float* base, int i0, int i1) {
  constexpr int kBatch = 16;  // loads in flight before the in-order merges
  const int lane = threadIdx.x & 31;
  for (int i = i0; i < i1; i += kBatch) {
    Partial4 Q[kBatch];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      if (i + j < i1) {
        const float* src = base + size_t(i + j) * kPartialFloats;
        Q[j].m = __ldcg(src);
        Q[j].l = __ldcg(src + 1);
        const float4 v = __ldcg(reinterpret_cast<const float4*>(src + 4) + lane);
        Q[j].a[0] = v.x; Q[j].a[1] = v.y; Q[j].a[2] = v.z; Q[j].a[3] = v.w;
      }
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j)
      if (i + j < i1) merge_into(P, Q[j]);
  }
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
// hi' = bf16(fma(lo, s, hi*c)).  cs == nullptr: a layer without rotary
// embedding (x unchanged).
__device__ __forceinline__ void rope4(float (&x)[4], const float* cs, float* scratch) {
  if (!cs) return;
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

// ---------------------------------------------------------------------------
// Exp of the attention softmax, for x <= 0 (a score minus a running max, or
// the difference of two running maxima).  Cody-Waite reduction with a 16-bit
// head of ln2; the integer n = rint(x*log2e) comes from the fused
// multiply-add fma(x, log2e, 1.5*2^23) (one rounding), whose bits also give
// the scale 2^n; e^r by the degree-7 Taylor polynomial in Horner form.
// Results below 2^-125 (x <= -87) are flushed to 0; exp(-inf) = 0.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float aexp(float x) {
  if (!(x > -87.0f)) return 0.0f;
  const float t = __fmaf_rn(x, 1.44269504088896341f, 12582912.0f);
  const float n = __fsub_rn(t, 12582912.0f);
  float r = __fmaf_rn(-n, 0.693145751953125f, x);
  r = __fmaf_rn(-n, 1.42860682030941723e-6f, r);
  float p = 1.98412698412698413e-4f;
  p = __fmaf_rn(p, r, 1.38888888888888889e-3f);
  p = __fmaf_rn(p, r, 8.33333333333333333e-3f);
  p = __fmaf_rn(p, r, 4.16666666666666667e-2f);
  p = __fmaf_rn(p, r, 1.66666666666666667e-1f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  // bits(t) = 0x4B400000 + n  ->  exponent field n + 127
  const uint32_t sc = (__float_as_uint(t) + uint32_t(127 - 0x4B400000)) << 23;
  return __fmul_rn(p, __uint_as_float(sc));
}

// ---------------------------------------------------------------------------
// Tile computation on the tensor cores (integer mma.sync m16n8k32, signed
// A, unsigned B).  Fragment layout (lane = 4*gq + tq):
//   A 16x32 (row): a0 = A[gq][4tq..+3], a1 = A[gq+8][4tq..+3],
//                  a2 = A[gq][16+4tq..+3], a3 = A[gq+8][16+4tq..+3]
//   B 32x8  (col): b0 = B[4tq..+3][gq], b1 = B[16+4tq..+3][gq]
//   C 16x8:        c0 = C[gq][2tq], c1 = C[gq][2tq+1], c2 = C[gq+8][2tq],
//                  c3 = C[gq+8][2tq+1]
// (byte i of a register = k index 4tq+i, resp. 16+4tq+i).
//
// A rows gq and gq+8 carry the high and low signed byte limbs of head gq
// (v = 256*hi + lo, hi = (v+128)>>8), so a thread owns one head: gq.
//   scores:  A = query limbs, B = K codes of n-tile nt (tokens 8nt..8nt+7);
//            the thread gets head gq, tokens 8nt+2tq, 8nt+2tq+1.
//   PV:      A = fixed-point weights of the thread's own 8 tokens (k index
//            4tq+i <-> token 8(i>>1)+2tq+(i&1), 16+4tq+i <-> that + 16),
//            B = V codes (n-tile nt: column n = dim 8n+nt of group 0, nt < 8,
//            or 64+8n+(nt-8)); the thread gets dims 16tq+{0..15} and
//            64+16tq+{0..15} of head gq.
// The K dims are permuted within a k-step (qk_dim) so that a thread's B
// registers come straight from its code words; the query uses the same
// permutation.  All integer sums are exact, so the permutations and the MMA
// summation order do not change any result.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_s8u8(int (&c)[4], const uint4& a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1));
}

// Dim of K/query k index (k-step ks, thread tq, side r: 0 = k 4tq+i, 1 = k
// 16+4tq+i, byte i).  4-bit: word w = 8(ks>>1) + 2tq + (ks&1), low nibbles
// (even dims) on side 0, high nibbles on side 1.  8-bit: words w0 = 16(ks>>1)
// + 4tq + 2(ks&1) (side 0) and w0+1 (side 1).  k-steps 0,1 cover group 0.
template <int BITS>
__host__ __device__ __forceinline__ int qk_dim(int ks, int tq, int r, int i) {
  if constexpr (BITS == 4) {
    const int w = 8 * (ks >> 1) + 2 * tq + (ks & 1);
    return 8 * w + 2 * i + r;
  } else {
    const int w = 16 * (ks >> 1) + 4 * tq + 2 * (ks & 1) + r;
    return 4 * w + i;
  }
}

// Prepared queries of the 8 heads of a kv head: A fragments per k-step and
// lane (head lane>>2), and per head (QS0, QS1, 2^-F, 0).
struct QFrags {
  uint4 frag[4][32];
  float4 meta[8];
};

// 4x4 byte transpose with the pairs (w0, w1), (w2, w3) given in either
// order: selectors (0x5140, 0x7362) for the natural order, (0x1504, 0x3726)
// for swapped pairs.
__device__ __forceinline__ void transpose4s(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, uint32_t sa,
                                            uint32_t sb, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  const uint32_t x0 = __byte_perm(w0, w1, sa), x1 = __byte_perm(w0, w1, sb);
  const uint32_t x2 = __byte_perm(w2, w3, sa), x3 = __byte_perm(w2, w3, sb);
  r0 = __byte_perm(x0, x2, 0x5410);
  r1 = __byte_perm(x0, x2, 0x7632);
  r2 = __byte_perm(x1, x3, 0x5410);
  r3 = __byte_perm(x1, x3, 0x7632);
}

// 4x4 byte transpose: r_k = byte k of w0..w3 (w0 in the low byte).
__device__ __forceinline__ void transpose4(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, uint32_t& r0,
                                           uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  const uint32_t x0 = __byte_perm(w0, w1, 0x5140), x1 = __byte_perm(w0, w1, 0x7362);
  const uint32_t x2 = __byte_perm(w2, w3, 0x5140), x3 = __byte_perm(w2, w3, 0x7362);
  r0 = __byte_perm(x0, x2, 0x5410);
  r1 = __byte_perm(x0, x2, 0x7632);
  r2 = __byte_perm(x1, x3, 0x5410);
  r3 = __byte_perm(x1, x3, 0x7632);
}

// Signed byte limbs of v (|v| <= 32639): hi = (v + 128) >> 8, lo = v - 256 hi.
__device__ __forceinline__ uint32_t limb_hi(int v) { return uint32_t((v + 128) >> 8) & 0xFFu; }
__device__ __forceinline__ uint32_t limb_lo(int v) { return uint32_t(v) & 0xFFu; }

// One warp prepares head `head` (0..7) of the kv head: x = its (normed,
// RoPE'd) dims 4l..4l+3.  scratch: 512 bytes of the warp's shared memory.
//   qs = bf16(x / sqrt(128)); F = min(14 - exponent(max|qs| * (1 + 2^-7)), 100)
//   (keeps |qi| <= 32512, so both limbs are signed bytes); qi = rint(qs 2^F);
//   QS_g = exact sum of qi over group g.
template <int BITS>
__device__ __forceinline__ void prep_qhead(const float (&x)[4], QFrags& q, int head, int* scratch) {
  const int lane = threadIdx.x & 31;
  float qs[4];
  float mx = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    qs[j] = rbf(__fmul_rn(x[j], kQScale));
    mx = fmaxf(mx, fabsf(qs[j]));
  }
  mx = bfly_max(mx);
  const int E = int((__float_as_uint(__fmul_rn(mx, 1.0078125f)) >> 23) & 0xFF) - 127;
  int F = 14 - E;
  F = F > 100 ? 100 : F;
  const float up = __uint_as_float(uint32_t(F + 127) << 23);
  int part = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int qi = __float2int_rn(__fmul_rn(qs[j], up));
    scratch[4 * lane + j] = qi;
    part += qi;
  }
  // group sums: lanes 0..15 hold group 0, 16..31 group 1 (exact integers)
#pragma unroll
  for (int off = 8; off >= 1; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
  const int qs1 = __shfl_sync(0xffffffffu, part, 16);
  if (lane == 0) q.meta[head] = make_float4(float(part), float(qs1), __uint_as_float(uint32_t(127 - F) << 23), 0.0f);
  __syncwarp();
  if (lane < 16) {
    const int ks = lane >> 2, tq = lane & 3;
    uint32_t r[4] = {0, 0, 0, 0};  // a0 (hi, side 0), a1 (lo, side 0), a2, a3
#pragma unroll
    for (int side = 0; side < 2; ++side)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int v = scratch[qk_dim<BITS>(ks, tq, side, i)];
        r[2 * side] |= limb_hi(v) << (8 * i);
        r[2 * side + 1] |= limb_lo(v) << (8 * i);
      }
    q.frag[ks][4 * head + tq] = make_uint4(r[0], r[1], r[2], r[3]);
  }
  __syncwarp();
}

// Running state of one warp: head gq of the kv head, dims 16tq + (0..15) and
// 64 + 16tq + (0..15): acc[16 grp + 8 c + k] = dim 64 grp + 16 tq + 8 c + k.
struct WarpState {
  float m, l;
  float acc[32];
};
__device__ __forceinline__ void state_empty(WarpState& s) {
  s.m = -INFINITY;
  s.l = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) s.acc[i] = 0.0f;
}
// x <- x (+) y (the merge rule of merge_into).
__device__ __forceinline__ void state_merge(WarpState& x, const WarpState& y) {
  if (y.m == -INFINITY) return;
  if (x.m == -INFINITY) {
    x = y;
    return;
  }
  const bool xm = x.m >= y.m;
  const float m = xm ? x.m : y.m;
  const float e = rexp(__fsub_rn(xm ? y.m : x.m, m));
  const float a1 = xm ? 1.0f : e, a2 = xm ? e : 1.0f;
  x.l = __fmaf_rn(x.l, a1, __fmul_rn(y.l, a2));
#pragma unroll
  for (int i = 0; i < 32; ++i) x.acc[i] = __fmaf_rn(x.acc[i], a1, __fmul_rn(y.acc[i], a2));
  x.m = m;
}
__device__ __forceinline__ int state_dim(int i, int tq) { return 64 * (i >> 4) + 16 * tq + (i & 15); }

// Sum over the 32 tokens of a tile of the values v[2nt + j] (token 8nt + 2tq
// + j) of the 4 threads of a head: ((v0+v1)+(v2+v3)) + ((v4+v5)+(v6+v7)) per
// thread, then (S0+S1)+(S2+S3) by a butterfly over tq.
__device__ __forceinline__ float tile_sum(const float (&v)[8]) {
  float s = __fadd_rn(__fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3])),
                      __fadd_rn(__fadd_rn(v[4], v[5]), __fadd_rn(v[6], v[7])));
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 1));
  return __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 2));
}
__device__ __forceinline__ float tile_max(const float (&v)[8]) {
  float m = fmaxf(fmaxf(fmaxf(v[0], v[1]), fmaxf(v[2], v[3])), fmaxf(fmaxf(v[4], v[5]), fmaxf(v[6], v[7])));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  return fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
}

// One tile of 32 tokens (FULL: all 32 valid, the masks compile away; rows of
// the K and V tiles in shared memory, row
// stride RW words; scales/biases [token][2], 8-byte aligned) for the 8 q
// heads, folded into the warp state (canonical order):
//   s_t = score of token t (first..nvalid-1), -inf outside (first > 0: the
//   start of a sliding window inside the tile);
//   m' = max(m, max_t s_t); alpha = aexp(m - m'); p_t = aexp(s_t - m');
//   l' = fma(l, alpha, tile_sum(p));
//   per V group: w_t = p_t scale_t, x_t = p_t bias_t (0 beyond nvalid);
//     F = min(14 - exponent(max|w| (1 + 2^-7)), 100); wq_t = rint(w_t 2^F)
//     (|wq| <= 32514: signed byte limbs);
//     acc_d' = fma(acc_d, alpha, fma(float(sum_t wq_t code_td), 2^-F, tile_sum(x))).
// BITS: the K codes' width; VBITS: the V codes' (the reference's mixed cache
// keeps K at 8 and V at 4 bits, model.py:35-37,40-82).
template <int BITS, bool FULL = false, int VBITS = BITS>
__device__ __forceinline__ void tile_fold(const uint32_t* kc, const uint16_t* ks, const uint16_t* kb,
                                          const uint32_t* vc, const uint16_t* vs, const uint16_t* vb, int nvalid,
                                          const QFrags& qf, WarpState& st, int first = 0) {
  constexpr int RW = 128 * BITS / 32;
  constexpr int RWV = 128 * VBITS / 32;
  constexpr uint32_t M4 = 0x0F0F0F0Fu;
  const int lane = threadIdx.x & 31, gq = lane >> 2, tq = lane & 3;
  // ---- scores: C[group][nt]
  int C[2][4][4];
#pragma unroll
  for (int g = 0; g < 2; ++g)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) C[g][nt][e] = 0;
  {
    uint4 A[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) A[k] = qf.frag[k][lane];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const uint32_t* row = kc + (8 * nt + gq) * RW;
      if constexpr (BITS == 4) {
        const uint2 x = *reinterpret_cast<const uint2*>(row + 2 * tq);
        const uint2 y = *reinterpret_cast<const uint2*>(row + 8 + 2 * tq);
        mma_s8u8(C[0][nt], A[0], x.x & M4, (x.x >> 4) & M4);
        mma_s8u8(C[0][nt], A[1], x.y & M4, (x.y >> 4) & M4);
        mma_s8u8(C[1][nt], A[2], y.x & M4, (y.x >> 4) & M4);
        mma_s8u8(C[1][nt], A[3], y.y & M4, (y.y >> 4) & M4);
      } else {
        const uint4 x = *reinterpret_cast<const uint4*>(row + 4 * tq);
        const uint4 y = *reinterpret_cast<const uint4*>(row + 16 + 4 * tq);
        mma_s8u8(C[0][nt], A[0], x.x, x.y);
        mma_s8u8(C[0][nt], A[1], x.z, x.w);
        mma_s8u8(C[1][nt], A[2], y.x, y.y);
        mma_s8u8(C[1][nt], A[3], y.z, y.w);
      }
    }
  }
  // ---- scores of head gq, tokens 8nt + 2tq + j  (v = 2nt + j)
  float p[8];
  float alpha;
  {
    const float4 meta = qf.meta[gq];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      const int t = 8 * nt + 2 * tq;
      const uint2 sp = *reinterpret_cast<const uint2*>(ks + 2 * t);
      const uint2 bp = *reinterpret_cast<const uint2*>(kb + 2 * t);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const uint32_t sw = j ? sp.y : sp.x, bw = j ? bp.y : bp.x;
        const float s0 = __uint_as_float(sw << 16), s1 = __uint_as_float(sw & 0xFFFF0000u);
        const float b0 = __uint_as_float(bw << 16), b1 = __uint_as_float(bw & 0xFFFF0000u);
        const int D0 = C[0][nt][j] * 256 + C[0][nt][2 + j];
        const int D1 = C[1][nt][j] * 256 + C[1][nt][2 + j];
        float u = __fmaf_rn(b0, meta.x, __fmul_rn(s0, float(D0)));
        u = __fmaf_rn(s1, float(D1), u);
        u = __fmaf_rn(b1, meta.y, u);
        p[2 * nt + j] = (FULL || (t + j >= first && t + j < nvalid)) ? rbf(__fmul_rn(u, meta.z)) : -INFINITY;
      }
    }
    const float mt = tile_max(p);
    const float mn = fmaxf(st.m, mt);
    alpha = aexp(__fsub_rn(st.m, mn));
    st.m = mn;
#pragma unroll
    for (int v = 0; v < 8; ++v) p[v] = aexp(__fsub_rn(p[v], mn));
    st.l = __fmaf_rn(st.l, alpha, tile_sum(p));
  }
  // ---- PV per V group
  uint2 vsp[4], vbp[4];
#pragma unroll
  for (int nt = 0; nt < 4; ++nt) {
    const int t = 8 * nt + 2 * tq;
    vsp[nt] = *reinterpret_cast<const uint2*>(vs + 2 * t);
    vbp[nt] = *reinterpret_cast<const uint2*>(vb + 2 * t);
  }
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    float w[8], x[8];
    float mx = 0.0f;
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int v = 2 * nt + j;
        const uint32_t sw = j ? vsp[nt].y : vsp[nt].x, bw = j ? vbp[nt].y : vbp[nt].x;
        const float sc = __uint_as_float(g ? (sw & 0xFFFF0000u) : (sw << 16));
        const float bi = __uint_as_float(g ? (bw & 0xFFFF0000u) : (bw << 16));
        const int tt = 8 * nt + 2 * tq + j;
        const bool ok = FULL || (tt >= first && tt < nvalid);
        w[v] = ok ? __fmul_rn(p[v], sc) : 0.0f;
        x[v] = ok ? __fmul_rn(p[v], bi) : 0.0f;
        mx = fmaxf(mx, fabsf(w[v]));
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const int E = int((__float_as_uint(__fmul_rn(mx, 1.0078125f)) >> 23) & 0xFF) - 127;
    int F = 14 - E;
    F = F > 100 ? 100 : F;
    const float up = __uint_as_float(uint32_t(F + 127) << 23);
    const float dn = __uint_as_float(uint32_t(127 - F) << 23);
    const float B = tile_sum(x);
    // wq = rint(w 2^F) as bits 0x4B400000 + wq of fma(w, 2^F, 1.5*2^23);
    // byte 0 of those bits is the low limb, byte 1 of (bits + 128) the high.
    uint32_t lo[8], hp[8];
#pragma unroll
    for (int v = 0; v < 8; ++v) {
      lo[v] = __float_as_uint(__fmaf_rn(w[v], up, 12582912.0f));
      hp[v] = lo[v] + 128u;
    }
    uint4 Aw;
    Aw.x = __byte_perm(__byte_perm(hp[0], hp[1], 0x0051), __byte_perm(hp[2], hp[3], 0x0051), 0x5410);
    Aw.y = __byte_perm(__byte_perm(lo[0], lo[1], 0x0040), __byte_perm(lo[2], lo[3], 0x0040), 0x5410);
    Aw.z = __byte_perm(__byte_perm(hp[4], hp[5], 0x0051), __byte_perm(hp[6], hp[7], 0x0051), 0x5410);
    Aw.w = __byte_perm(__byte_perm(lo[4], lo[5], 0x0040), __byte_perm(lo[6], lo[7], 0x0040), 0x5410);
    // V codes of the thread's tokens: side 0 = tokens 2tq, 2tq+1, 8+2tq,
    // 9+2tq; side 1 = those + 16.  Transposed to (dim, 4 tokens) bytes.
    uint32_t bt[2][8];  // [side][nt & 7]
#pragma unroll
    for (int side = 0; side < 2; ++side) {
      const int tb = 16 * side + 2 * tq;
      const int rows[4] = {tb, tb + 1, tb + 8, tb + 9};
      if constexpr (VBITS == 4) {
        // odd tq reads each row pair in swapped order: the four threads of a
        // column then hit two rows of each parity (two bank halves)
        const int odd = tq & 1;
        uint32_t wv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) wv[i] = vc[(tb + 8 * (i >> 1) + ((i & 1) ^ odd)) * RWV + 8 * g + gq];
        uint32_t r[4];
        transpose4s(wv[0], wv[1], wv[2], wv[3], odd ? 0x1504u : 0x5140u, odd ? 0x3726u : 0x7362u, r[0], r[1], r[2],
                    r[3]);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          bt[side][2 * k] = r[k] & M4;
          bt[side][2 * k + 1] = (r[k] >> 4) & M4;
        }
      } else {
        uint2 wv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) wv[i] = *reinterpret_cast<const uint2*>(vc + rows[i] * RWV + 16 * g + 2 * gq);
        transpose4(wv[0].x, wv[1].x, wv[2].x, wv[3].x, bt[side][0], bt[side][1], bt[side][2], bt[side][3]);
        transpose4(wv[0].y, wv[1].y, wv[2].y, wv[3].y, bt[side][4], bt[side][5], bt[side][6], bt[side][7]);
      }
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      int P[4] = {0, 0, 0, 0};
      mma_s8u8(P, Aw, bt[0][k], bt[1][k]);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int ai = P[c] * 256 + P[2 + c];
        const float v = __fmaf_rn(float(ai), dn, B);
        float& a = st.acc[16 * g + 8 * c + k];
        a = __fmaf_rn(a, alpha, v);
      }
    }
  }
}

}  // namespace rec
