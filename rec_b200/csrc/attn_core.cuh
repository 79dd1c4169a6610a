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
  constexpr int kBatch = 4;
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

// ---------------------------------------------------------------------------
// Tile computation on the tensor cores (integer mma.sync m16n8k32).  Scores
// D_g = sum qi*code and the PV dot sum wq*code are exact int32 sums, so the
// MMA gives the same bits as any other summation order.
//
// Fragment layout (lane = 4*gq + tq):
//   A 16x32 (row): a0 = A[gq][4tq..], a1 = A[gq+8][4tq..], a2 = A[gq][16+4tq..],
//                  a3 = A[gq+8][16+4tq..]  (four 8-bit values per register)
//   B 32x8  (col): b0 = B[4tq..][gq], b1 = B[16+4tq..][gq]
//   C 16x8:        c0 = C[gq][2tq], c1 = C[gq][2tq+1], c2 = C[gq+8][2tq],
//                  c3 = C[gq+8][2tq+1]
// A thread owns the tile's tokens gq, gq+8, 16+gq, 24+gq and the heads 2tq,
// 2tq+1; for PV it owns 16 dims: dim_of(li) below.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_u8u8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
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

// PV dims of a thread: local index li (0..15) -> dim.
template <int BITS>
__device__ __forceinline__ int dim_of(int li, int gq) {
  if constexpr (BITS == 8) return 32 * (li >> 2) + 4 * gq + (li & 3);
  else return 64 * (li >> 3) + 8 * gq + (li & 7);
}

// Running (m, l, acc) of one warp for heads 2tq, 2tq+1 and the thread's dims.
struct WarpState {
  float m[2], l[2];
  float acc[2][16];
};
__device__ __forceinline__ void state_empty(WarpState& s) {
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    s.m[hh] = -INFINITY;
    s.l[hh] = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) s.acc[hh][i] = 0.0f;
  }
}
// x <- x (+) y for one head (the merge rule of merge_into).
__device__ __forceinline__ void state_merge(WarpState& x, const WarpState& y) {
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    if (y.m[hh] == -INFINITY) continue;
    if (x.m[hh] == -INFINITY) {
      x.m[hh] = y.m[hh];
      x.l[hh] = y.l[hh];
#pragma unroll
      for (int i = 0; i < 16; ++i) x.acc[hh][i] = y.acc[hh][i];
      continue;
    }
    const float m = fmaxf(x.m[hh], y.m[hh]);
    const float a1 = rexp(__fsub_rn(x.m[hh], m)), a2 = rexp(__fsub_rn(y.m[hh], m));
    x.l[hh] = __fmaf_rn(x.l[hh], a1, __fmul_rn(y.l[hh], a2));
#pragma unroll
    for (int i = 0; i < 16; ++i) x.acc[hh][i] = __fmaf_rn(x.acc[hh][i], a1, __fmul_rn(y.acc[hh][i], a2));
    x.m[hh] = m;
  }
}

__device__ __forceinline__ float sum_tokens(float v00, float v01, float v10, float v11) {
  // (t[gq] + t[gq+8]) + (t[16+gq] + t[24+gq]), then a butterfly over gq
  float s = __fadd_rn(__fadd_rn(v00, v01), __fadd_rn(v10, v11));
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 16));
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 8));
  s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 4));
  return s;
}
__device__ __forceinline__ float max_tokens(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
  return v;
}

// One tile of 32 tokens (rows of the K and V tiles in shared memory, row
// stride RW words; scales/biases [token][2]) for the 8 q heads in qh, folded
// into the warp state.  nvalid: tokens of the tile below T (1..32).
// wbuf: 1 KB of the warp's shared memory.
template <int BITS>
__device__ __forceinline__ void tile_fold(const uint32_t* kc, const uint16_t* ks, const uint16_t* kb,
                                          const uint32_t* vc, const uint16_t* vs, const uint16_t* vb, int nvalid,
                                          const QHead* qh, uint8_t* wbuf, WarpState& st) {
  constexpr int RW = 128 * BITS / 32;
  const int lane = threadIdx.x & 31, gq = lane >> 2, tq = lane & 3;
  // ---- scores: C[group][half][limb]
  int C[2][2][2][4];
#pragma unroll
  for (int g = 0; g < 2; ++g)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf)
#pragma unroll
      for (int lb = 0; lb < 2; ++lb)
#pragma unroll
        for (int e = 0; e < 4; ++e) C[g][hf][lb][e] = 0;
#pragma unroll
  for (int kq = 0; kq < 4; ++kq) {
    const uint32_t bh0 = qh[gq].hi[8 * kq + tq], bh1 = qh[gq].hi[8 * kq + 4 + tq];
    const uint32_t bl0 = qh[gq].lo[8 * kq + tq], bl1 = qh[gq].lo[8 * kq + 4 + tq];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const uint32_t* r0 = kc + (16 * hf + gq) * RW;
      const uint32_t* r1 = r0 + 8 * RW;
      uint32_t a0, a1, a2, a3;
      if constexpr (BITS == 8) {
        a0 = r0[8 * kq + tq];
        a1 = r1[8 * kq + tq];
        a2 = r0[8 * kq + 4 + tq];
        a3 = r1[8 * kq + 4 + tq];
      } else {
        const int w0 = 4 * kq + (tq >> 1), w2 = w0 + 2, sh = (tq & 1) * 4;
        a0 = (r0[w0] >> sh) & 0x0F0F0F0Fu;
        a1 = (r1[w0] >> sh) & 0x0F0F0F0Fu;
        a2 = (r0[w2] >> sh) & 0x0F0F0F0Fu;
        a3 = (r1[w2] >> sh) & 0x0F0F0F0Fu;
      }
      mma_u8s8(C[kq >> 1][hf][0], a0, a1, a2, a3, bh0, bh1);
      mma_u8u8(C[kq >> 1][hf][1], a0, a1, a2, a3, bl0, bl1);
    }
  }
  // ---- scores, tile max, p, l   (element e = 2r + hh: token 16hf + 8r + gq, head 2tq + hh)
  float p[2][2][2];  // [hf][r][hh]
  float mt[2];
  {
    float sc[2][2][2];
    float QS0[2], QS1[2], dn[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      QS0[hh] = qh[2 * tq + hh].QS[0];
      QS1[hh] = qh[2 * tq + hh].QS[1];
      dn[hh] = qh[2 * tq + hh].down;
    }
#pragma unroll
    for (int hf = 0; hf < 2; ++hf)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int j = 16 * hf + 8 * r + gq;
        const uint32_t sp = *reinterpret_cast<const uint32_t*>(ks + 2 * j);
        const uint32_t bp = *reinterpret_cast<const uint32_t*>(kb + 2 * j);
        const float s0 = __uint_as_float(sp << 16), s1 = __uint_as_float(sp & 0xFFFF0000u);
        const float b0 = __uint_as_float(bp << 16), b1 = __uint_as_float(bp & 0xFFFF0000u);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int e = 2 * r + hh;
          const int D0 = C[0][hf][0][e] * 256 + C[0][hf][1][e];
          const int D1 = C[1][hf][0][e] * 256 + C[1][hf][1][e];
          float t = __fmaf_rn(b0, QS0[hh], __fmul_rn(s0, float(D0)));
          t = __fmaf_rn(s1, float(D1), t);
          t = __fmaf_rn(b1, QS1[hh], t);
          sc[hf][r][hh] = j < nvalid ? rbf(__fmul_rn(t, dn[hh])) : -INFINITY;
        }
      }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float m = fmaxf(fmaxf(sc[0][0][hh], sc[0][1][hh]), fmaxf(sc[1][0][hh], sc[1][1][hh]));
      m = max_tokens(m);
      mt[hh] = m;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int j = 16 * hf + 8 * r + gq;
          p[hf][r][hh] = j < nvalid ? rexp(__fsub_rn(sc[hf][r][hh], m)) : 0.0f;
        }
    }
  }
  float lt[2];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) lt[hh] = sum_tokens(p[0][0][hh], p[0][1][hh], p[1][0][hh], p[1][1][hh]);
  // merge factors of the state and the tile
  float as[2], at[2];
  bool first[2];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    first[hh] = st.m[hh] == -INFINITY;
    const float m = first[hh] ? mt[hh] : fmaxf(st.m[hh], mt[hh]);
    as[hh] = first[hh] ? 0.0f : rexp(__fsub_rn(st.m[hh], m));
    at[hh] = first[hh] ? 1.0f : rexp(__fsub_rn(mt[hh], m));
    st.l[hh] = first[hh] ? lt[hh] : __fmaf_rn(st.l[hh], as[hh], __fmul_rn(lt[hh], at[hh]));
    st.m[hh] = m;
  }
  // ---- PV per V group: fixed-point weights, exact integer dot, fold
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    float dnw[2], B[2];
    float vsc[2][2], vbi[2][2];  // V scale / bias of the thread's tokens, group g
#pragma unroll
    for (int hf = 0; hf < 2; ++hf)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int j = 16 * hf + 8 * r + gq;
        vsc[hf][r] = bf(vs[2 * j + g]);
        vbi[hf][r] = bf(vb[2 * j + g]);
      }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float w[2][2], x[2][2];
      float mx = 0.0f;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int j = 16 * hf + 8 * r + gq;
          const bool v = j < nvalid;
          w[hf][r] = v ? __fmul_rn(p[hf][r][hh], vsc[hf][r]) : 0.0f;
          x[hf][r] = v ? __fmul_rn(p[hf][r][hh], vbi[hf][r]) : 0.0f;
          mx = fmaxf(mx, fabsf(w[hf][r]));
        }
      mx = max_tokens(mx);
      const int E = int((__float_as_uint(mx) >> 23) & 0xFF) - 127;
      int F = 13 - E;
      F = F > 100 ? 100 : F;
      const float up = __uint_as_float(uint32_t(F + 127) << 23);
      dnw[hh] = __uint_as_float(uint32_t(127 - F) << 23);
      B[hh] = sum_tokens(x[0][0], x[0][1], x[1][0], x[1][1]);
      // limbs -> wbuf[limb][head][token] bytes
#pragma unroll
      for (int hf = 0; hf < 2; ++hf)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int j = 16 * hf + 8 * r + gq, head = 2 * tq + hh;
          const int q = __float2int_rn(__fmul_rn(w[hf][r], up));
          wbuf[head * 32 + j] = uint8_t((q >> 8) & 0xFF);
          wbuf[256 + head * 32 + j] = uint8_t(q & 0xFF);
        }
    }
    __syncwarp();
    const uint32_t* wb32 = reinterpret_cast<const uint32_t*>(wbuf);
    const uint32_t bh0 = wb32[gq * 8 + tq], bh1 = wb32[gq * 8 + 4 + tq];
    const uint32_t bl0 = wb32[64 + gq * 8 + tq], bl1 = wb32[64 + gq * 8 + 4 + tq];
    int P[4][2][4];  // [block][limb][e]
#pragma unroll
    for (int bk = 0; bk < 4; ++bk)
#pragma unroll
      for (int lb = 0; lb < 2; ++lb)
#pragma unroll
        for (int e = 0; e < 4; ++e) P[bk][lb][e] = 0;
    if constexpr (BITS == 8) {
      // 32-dim groups p = 2g, 2g+1: words (8p + gq) of tokens 4tq+i and 16+4tq+i
#pragma unroll
      for (int pp = 0; pp < 2; ++pp) {
        const int wi = 8 * (2 * g + pp) + gq;
        uint32_t r0, r1, r2, r3, s0, s1, s2, s3;
        transpose4(vc[(4 * tq + 0) * RW + wi], vc[(4 * tq + 1) * RW + wi], vc[(4 * tq + 2) * RW + wi],
                   vc[(4 * tq + 3) * RW + wi], r0, r1, r2, r3);
        transpose4(vc[(16 + 4 * tq + 0) * RW + wi], vc[(16 + 4 * tq + 1) * RW + wi],
                   vc[(16 + 4 * tq + 2) * RW + wi], vc[(16 + 4 * tq + 3) * RW + wi], s0, s1, s2, s3);
        mma_u8s8(P[2 * pp][0], r0, r1, s0, s1, bh0, bh1);
        mma_u8u8(P[2 * pp][1], r0, r1, s0, s1, bl0, bl1);
        mma_u8s8(P[2 * pp + 1][0], r2, r3, s2, s3, bh0, bh1);
        mma_u8u8(P[2 * pp + 1][1], r2, r3, s2, s3, bl0, bl1);
      }
    } else {
      const int wi = 8 * g + gq;
      uint32_t w4[4], z4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        w4[i] = vc[(4 * tq + i) * RW + wi];
        z4[i] = vc[(16 + 4 * tq + i) * RW + wi];
      }
      uint32_t e0, e1, e2, e3, o0, o1, o2, o3, f0, f1, f2, f3, q0, q1, q2, q3;
      transpose4(w4[0] & 0x0F0F0F0Fu, w4[1] & 0x0F0F0F0Fu, w4[2] & 0x0F0F0F0Fu, w4[3] & 0x0F0F0F0Fu, e0, e1, e2, e3);
      transpose4((w4[0] >> 4) & 0x0F0F0F0Fu, (w4[1] >> 4) & 0x0F0F0F0Fu, (w4[2] >> 4) & 0x0F0F0F0Fu,
                 (w4[3] >> 4) & 0x0F0F0F0Fu, o0, o1, o2, o3);
      transpose4(z4[0] & 0x0F0F0F0Fu, z4[1] & 0x0F0F0F0Fu, z4[2] & 0x0F0F0F0Fu, z4[3] & 0x0F0F0F0Fu, f0, f1, f2, f3);
      transpose4((z4[0] >> 4) & 0x0F0F0F0Fu, (z4[1] >> 4) & 0x0F0F0F0Fu, (z4[2] >> 4) & 0x0F0F0F0Fu,
                 (z4[3] >> 4) & 0x0F0F0F0Fu, q0, q1, q2, q3);
      // blocks: dims (+0,+2), (+4,+6), (+1,+3), (+5,+7) of the thread's 8
      mma_u8s8(P[0][0], e0, e1, f0, f1, bh0, bh1);
      mma_u8u8(P[0][1], e0, e1, f0, f1, bl0, bl1);
      mma_u8s8(P[1][0], e2, e3, f2, f3, bh0, bh1);
      mma_u8u8(P[1][1], e2, e3, f2, f3, bl0, bl1);
      mma_u8s8(P[2][0], o0, o1, q0, q1, bh0, bh1);
      mma_u8u8(P[2][1], o0, o1, q0, q1, bl0, bl1);
      mma_u8s8(P[3][0], o2, o3, q2, q3, bh0, bh1);
      mma_u8u8(P[3][1], o2, o3, q2, q3, bl0, bl1);
    }
    __syncwarp();
    // element (block bk, row r, head hh) -> local dim li
#pragma unroll
    for (int bk = 0; bk < 4; ++bk)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        int li;
        if constexpr (BITS == 8) li = 8 * g + 4 * (bk >> 1) + 2 * (bk & 1) + r;
        else li = 8 * g + (bk == 0 ? 2 * r : bk == 1 ? 4 + 2 * r : bk == 2 ? 1 + 2 * r : 5 + 2 * r);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int e = 2 * r + hh;
          const int acc_int = P[bk][0][e] * 256 + P[bk][1][e];
          const float v = __fmaf_rn(float(acc_int), dnw[hh], B[hh]);
          st.acc[hh][li] = first[hh] ? v : __fmaf_rn(st.acc[hh][li], as[hh], __fmul_rn(v, at[hh]));
        }
      }
  }
}

}  // namespace rec
