// int4 g64 row dot products in the MLX affine layout, and the shared-memory
// weight pipeline that feeds them.
//
// Layout (reference: engine/src/rec_mlx/kernels/megakernel.py:161-170,189-232;
// MLX nn.quantize bits=4 group_size=64 mode="affine"):
//   weights  uint32[N, K/8]: element j of a row is (word[j/8] >> 4*(j%8)) & 15
//   scales   [N, K/64] fp16 or bf16, biases [N, K/64]
//   w[n, j] = scale[n, j/64] * q[n, j] + bias[n, j/64]
//
// Canonical order of one row (what the CPU oracle restates):
//   * the row is cut into 32-element chunks c (16 bytes of codes, half a group);
//   * every sum starts from +0.0 and adds its terms one at a time;
//   * in a chunk, two accumulators run over the words k = 0..3 and nibbles
//     i = 0..3: lo += x[8k+i] q[8k+i], hi += x[8k+4+i] q[8k+4+i] (fused
//     multiply-adds of exact products); D_c = lo + hi.  X_c (sum of x over the
//     chunk) is formed the same way;
//   * a lane owns a fixed set of chunks and folds them in order:
//     acc = fma(scale_g, D_c, acc); acc = fma(bias_g, X_c, acc)  (g = c/2);
//   * lanes are combined with an xor butterfly over T lanes;
//   * K % 2048 == 0: T = 32, the row is split in 2048-element segments, lane l
//     of segment s owns chunks 64s+l and 64s+l+32, and segment sums are added
//     in order.  Otherwise (K = 256*n, n <= 4): T = 8, lane l owns chunks
//     l, l+8, ... and there is one segment.
//   * the result is rounded once to bf16.
//
// The multiply uses x prescaled by a power of two so that each nibble can be
// turned into a float with a single AND/OR (exponent-magic) and a subtraction
// of 2^23, without shifting it down first.  Prescaling by 2^-p is exact for
// every bf16 input, so products are unchanged.
#pragma once
#include "common.cuh"

namespace rec {

// --- x preparation -----------------------------------------------------------
// xp[k][i] = (x'lo, x'hi) pair for word k, nibble pair i of one chunk.
struct ChunkX {
  float2 p[4][4];
  float X;  // sum of x over the chunk, canonical order
};

__device__ __forceinline__ void prep_chunk(const float* x32, ChunkX& cx) {
  // x32: the 32 chunk values as floats (already rounded to bf16 values).
  // lo nibble i is masked in place from the word (value q*2^(4i)); hi nibble
  // 4+i from the word shifted right by 12 (value q*2^(4i+4)).
  const float lo_scale[4] = {1.0f, 0.0625f, 0.00390625f, 0.000244140625f};          // 2^-4i
  const float hi_scale[4] = {0.0625f, 0.00390625f, 0.000244140625f, 1.52587890625e-05f};  // 2^-(4i+4)
  float xl = 0.0f, xh = 0.0f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a = x32[8 * k + i], b = x32[8 * k + 4 + i];
      cx.p[k][i] = make_float2(__fmul_rn(a, lo_scale[i]), __fmul_rn(b, hi_scale[i]));
      xl = __fadd_rn(xl, a);
      xh = __fadd_rn(xh, b);
    }
  }
  cx.X = __fadd_rn(xl, xh);
}

// --- one 16-byte chunk against prepared x -------------------------------------
__device__ __forceinline__ float2 u64_as_float2(unsigned long long v) {
  float2 f;
  f.x = __uint_as_float(uint32_t(v));
  f.y = __uint_as_float(uint32_t(v >> 32));
  return f;
}

__device__ __forceinline__ float chunk_dot(uint4 w, const ChunkX& cx) {
  // (word, word >> 12) form one 64-bit register pair; each 64-bit AND/OR
  // yields a (lo, hi) float pair ready for the packed f32x2 add and FMA.
  const unsigned long long M = 0x4B0000004B000000ull;
  const float2 off = make_float2(-8388608.0f, -8388608.0f);
  float2 acc = make_float2(0.0f, 0.0f);
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const unsigned long long p = (static_cast<unsigned long long>(ws[k] >> 12) << 32) | ws[k];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const unsigned long long mask = (static_cast<unsigned long long>(0xF0u << (4 * i)) << 32) | (0xFu << (4 * i));
      const float2 f = __fadd2_rn(u64_as_float2((p & mask) | M), off);
      acc = __ffma2_rn(cx.p[k][i], f, acc);
    }
  }
  return __fadd_rn(acc.x, acc.y);
}

// Fold one chunk into a lane accumulator.
__device__ __forceinline__ float fold_chunk(float acc, float d, float X, float s, float b) {
  acc = __fmaf_rn(s, d, acc);
  return __fmaf_rn(b, X, acc);
}

// --- K configurations ----------------------------------------------------------
// T lanes per row, CH chunks per lane (per segment), SEG segments.
template <int K>
struct KCfg {
  static_assert(K % 256 == 0, "K must be a multiple of 256");
  static constexpr bool wide = (K % 2048 == 0);
  static constexpr int T = wide ? 32 : 8;
  static constexpr int SEG = wide ? K / 2048 : 1;
  static constexpr int CH = wide ? 2 : K / 256;
  static_assert(wide || K / 256 <= 4, "K = 256*n needs n <= 4");
  static constexpr int CHUNKS = K / 32;
  static constexpr int ROW_BYTES = K / 2;
  static constexpr int GROUPS = K / 64;
  // chunk index owned by (segment, lane-in-row, m)
  __device__ static __forceinline__ int chunk(int seg, int l, int m) {
    return wide ? seg * 64 + l + 32 * m : l + 8 * m;
  }
};

// Prepare a lane's chunks of x (bf16 in global or shared memory, given as a
// generic pointer to uint16) for segment `seg`.
template <int K>
__device__ __forceinline__ void prep_lane_x(const uint16_t* x, int seg, int l, ChunkX (&cx)[KCfg<K>::CH]) {
#pragma unroll
  for (int m = 0; m < KCfg<K>::CH; ++m) {
    int c = KCfg<K>::chunk(seg, l, m);
    float v[32];
    const uint4* src = reinterpret_cast<const uint4*>(x + c * 32);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 u = src[q];
      const uint32_t us[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        v[8 * q + 2 * t] = __uint_as_float(us[t] << 16);
        v[8 * q + 2 * t + 1] = __uint_as_float(us[t] & 0xFFFF0000u);
      }
    }
    prep_chunk(v, cx[m]);
  }
}

// Lane partial of one row whose codes/scales/biases sit in shared memory.
template <int K, int SD>
__device__ __forceinline__ float lane_row_partial(const uint8_t* wrow, const uint16_t* srow,
                                                  const uint16_t* brow, int seg, int l,
                                                  const ChunkX (&cx)[KCfg<K>::CH]) {
  float acc = 0.0f;
#pragma unroll
  for (int m = 0; m < KCfg<K>::CH; ++m) {
    int c = KCfg<K>::chunk(seg, l, m);
    uint4 w = lds128(wrow + c * 16);
    float d = chunk_dot(w, cx[m]);
    float s = sb<SD>(srow[c >> 1]), b = sb<SD>(brow[c >> 1]);
    acc = fold_chunk(acc, d, cx[m].X, s, b);
  }
  return acc;
}

// Lane partials of ILP rows at once (independent chains for the scheduler);
// row i lives at wrow0 + i*row_stride etc.  valid[i] false rows give 0.
template <int K, int SD, int ILP>
__device__ __forceinline__ void lane_rows_partial(const uint8_t* wbase, const uint16_t* sbase,
                                                  const uint16_t* bbase, const int (&rows)[ILP],
                                                  int seg, int l, const ChunkX (&cx)[KCfg<K>::CH],
                                                  float (&out)[ILP]) {
  float acc[ILP];
#pragma unroll
  for (int i = 0; i < ILP; ++i) acc[i] = 0.0f;
#pragma unroll
  for (int m = 0; m < KCfg<K>::CH; ++m) {
    const int c = KCfg<K>::chunk(seg, l, m);
    uint4 w[ILP];
#pragma unroll
    for (int i = 0; i < ILP; ++i) w[i] = lds128(wbase + rows[i] * KCfg<K>::ROW_BYTES + c * 16);
    float d[ILP];
#pragma unroll
    for (int i = 0; i < ILP; ++i) d[i] = chunk_dot(w[i], cx[m]);
#pragma unroll
    for (int i = 0; i < ILP; ++i) {
      const float s = sb<SD>(sbase[rows[i] * KCfg<K>::GROUPS + (c >> 1)]);
      const float b = sb<SD>(bbase[rows[i] * KCfg<K>::GROUPS + (c >> 1)]);
      acc[i] = fold_chunk(acc[i], d[i], cx[m].X, s, b);
    }
  }
#pragma unroll
  for (int i = 0; i < ILP; ++i) out[i] = acc[i];
}

// --- shared-memory stage pipeline ---------------------------------------------
// A stage holds up to RS consecutive rows of one matrix: codes, then scales,
// then biases, each copied with one bulk copy.
template <int K, int RS>
struct StageLayout {
  static constexpr int W_BYTES = RS * KCfg<K>::ROW_BYTES;
  static constexpr int S_BYTES = ((RS * KCfg<K>::GROUPS * 2) + 15) / 16 * 16;
  static constexpr int BYTES = W_BYTES + 2 * S_BYTES;
};

struct QMatDev {
  const uint32_t* w;
  const uint16_t* s;
  const uint16_t* b;
};

// Issue the copies of rows [row0, row0+nrows) of matrix m into a stage.
// Sizes: nrows*K/2 and nrows*K/32 bytes must be multiples of 16 (nrows even
// for K = 768).
template <int K, int RS>
__device__ __forceinline__ void issue_stage(uint8_t* stage, uint64_t* bar, const QMatDev& m, int row0,
                                            int nrows) {
  using L = StageLayout<K, RS>;
  const uint32_t wb = uint32_t(nrows) * KCfg<K>::ROW_BYTES;
  const uint32_t sbytes = uint32_t(nrows) * KCfg<K>::GROUPS * 2;
  mbar_expect_tx(bar, wb + 2 * sbytes);
  bulk_g2s(stage, reinterpret_cast<const uint8_t*>(m.w) + size_t(row0) * KCfg<K>::ROW_BYTES, wb, bar);
  bulk_g2s(stage + L::W_BYTES, m.s + size_t(row0) * KCfg<K>::GROUPS, sbytes, bar);
  bulk_g2s(stage + L::W_BYTES + L::S_BYTES, m.b + size_t(row0) * KCfg<K>::GROUPS, sbytes, bar);
}

template <int K, int RS>
__device__ __forceinline__ const uint8_t* stage_wrow(const uint8_t* stage, int r) {
  return stage + r * KCfg<K>::ROW_BYTES;
}
template <int K, int RS>
__device__ __forceinline__ const uint16_t* stage_srow(const uint8_t* stage, int r) {
  return reinterpret_cast<const uint16_t*>(stage + StageLayout<K, RS>::W_BYTES) + r * KCfg<K>::GROUPS;
}
template <int K, int RS>
__device__ __forceinline__ const uint16_t* stage_brow(const uint8_t* stage, int r) {
  return reinterpret_cast<const uint16_t*>(stage + StageLayout<K, RS>::W_BYTES + StageLayout<K, RS>::S_BYTES) +
         r * KCfg<K>::GROUPS;
}

// Balanced split of `units` work units over `parts`: [begin, end) of part p.
__device__ __forceinline__ void split_range(int units, int parts, int p, int& begin, int& end) {
  begin = int((long long)units * p / parts);
  end = int((long long)units * (p + 1) / parts);
}

}  // namespace rec
