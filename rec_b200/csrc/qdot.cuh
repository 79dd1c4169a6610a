// int4 g64 row dot products in the MLX affine layout, and the shared-memory
// weight pipeline that feeds them.
//
// Layout (reference: engine/src/rec_mlx/kernels/megakernel.py:161-170,189-232;
// MLX nn.quantize bits=4 group_size=64 mode="affine"):
//   weights  uint32[N, K/8]: element j of a row is (word[j/8] >> 4*(j%8)) & 15
//   scales   [N, K/64] fp16 or bf16, biases [N, K/64]
//   w[n, j] = scale[n, j/64] * q[n, j] + bias[n, j/64]
//   y[n] = sum_g scale_g * sum_{j in g} x_j q_j + bias_g * sum_{j in g} x_j
//
// Canonical arithmetic (restated by oracle/rec_oracle.c):
//   * the input vector x (bf16[K]) is put in 16-bit fixed point with one
//     power-of-two scale for the whole vector: E = exponent of max|x|,
//     F = min(14 - E, 100), xi_j = rint(x_j * 2^F) (|xi| <= 32640);
//   * per group g of 64: D_g = sum_j q_j * xi_j and X_g = sum_j xi_j are
//     exact integers (int32), computed with byte dot products on the
//     limbs xi = 256*hi + lo (hi signed, lo unsigned), so their order is
//     irrelevant;
//   * a lane owns groups and folds them in order, starting from +0:
//     acc = fma(scale_g, float(D_g), acc); acc = fma(bias_g, float(X_g), acc);
//   * K % 2048 == 0: 32 lanes per row, lane l of 2048-element segment s owns
//     group 32s + l; segments are reduced by an xor butterfly and added in
//     order.  K = 256*n (n <= 4): 4 lanes per row, lane l owns groups
//     l, l+4, l+8, ...; butterfly over the 4 lanes;
//   * y = bf16(row_sum * 2^-F).
// Every fixed-point element within 2^7 of max|x| is exact; smaller ones are
// rounded to a multiple of 2^-F, which moves y by ~1e-4 of its size — an
// order of magnitude below the bf16 rounding of y.
#pragma once
#include "common.cuh"

namespace rec {

template <int K>
struct KCfg {
  static_assert(K % 256 == 0, "K must be a multiple of 256");
  static constexpr bool wide = (K % 2048 == 0);
  static constexpr int T = wide ? 32 : 4;           // lanes per row
  static constexpr int SEG = wide ? K / 2048 : 1;   // segments per row
  static constexpr int GROUPS = K / 64;
  static constexpr int GPL = wide ? 1 : GROUPS / 4;  // groups per lane (per segment)
  static_assert(wide || K / 256 <= 4, "K = 256*n needs n <= 4");
  static constexpr int ROW_BYTES = K / 2;
  __device__ static __forceinline__ int group(int seg, int l, int m) { return wide ? 32 * seg + l : l + 4 * m; }
};

// Fixed-point scale of a vector: returns F; 2^F and 2^-F as floats.
struct FixScale {
  int F;
  float up, down;
};
__device__ __forceinline__ FixScale fix_scale_from_max(float maxabs) {
  const int E = int((__float_as_uint(maxabs) >> 23) & 0xFF) - 127;
  int F = 14 - E;
  F = F > 100 ? 100 : F;
  return {F, __uint_as_float(uint32_t(F + 127) << 23), __uint_as_float(uint32_t(127 - F) << 23)};
}

// Max |x| over a bf16 vector in shared/global memory, reduced over the
// threads [t0, t0 + nthreads) that call it; red: shared scratch of
// nthreads/32 floats.  Returns the same value to all callers.
__device__ __forceinline__ float block_maxabs(const uint16_t* x, int n, int tid, int nthreads, float* red,
                                              int bar_id) {
  float m = 0.0f;
  for (int i = tid * 8; i < n; i += nthreads * 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + i);
    const uint32_t us[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) m = fmaxf(m, fmaxf(fabsf(__uint_as_float(us[q] << 16)),
                                                   fabsf(__uint_as_float(us[q] & 0xFFFF0000u))));
  }
  m = bfly_max(m);
  if ((tid & 31) == 0) red[tid >> 5] = m;
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthreads));
  float r = 0.0f;
  for (int w = 0; w < nthreads / 32; ++w) r = fmaxf(r, red[w]);
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthreads));
  return r;
}

// Max |x| over a bf16 vector, reduced within one warp (all lanes call it).
__device__ __forceinline__ float warp_maxabs(const uint16_t* x, int n) {
  const int lane = threadIdx.x & 31;
  float m = 0.0f;
  for (int i = lane * 8; i < n; i += 256) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + i);
    const uint32_t us[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) m = fmaxf(m, fmaxf(fabsf(__uint_as_float(us[q] << 16)),
                                                   fabsf(__uint_as_float(us[q] & 0xFFFF0000u))));
  }
  return bfly_max(m);
}

// A lane's prepared group of x: per word w of the group, byte-packed limbs
// matching the even nibbles (0,2,4,6) and odd nibbles (1,3,5,7) of the
// weight word.  Lanes with bit 2 set (wide rows, see lane_half) hold the
// group's two 16-byte halves in swapped order (words 4..7, then 0..3), like
// the weight words they read; the dot product is an exact integer sum, so
// the order does not change it.
struct GroupX {
  uint32_t hi_e[8], hi_o[8], lo_e[8], lo_o[8];
  float X;  // float(sum of xi over the group), exact
};

// Which half of its 32-byte group a lane of a wide row (32 lanes per row,
// lane l owning group l) reads first: lanes 0-3 of each quarter-warp the
// low half, lanes 4-7 the high half, so that the quarter-warp's 128-bit
// shared loads cover all 32 banks (the plain order puts lanes l and l + 4
// on the same banks).
__device__ __forceinline__ int lane_half(int l) { return (l >> 2) & 1; }

__device__ __forceinline__ void prep_group(const uint16_t* xg, FixScale fs, GroupX& gx, int sw = 0) {
  int sum = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const uint4 u = *reinterpret_cast<const uint4*>(xg + 8 * (w ^ (4 * sw)));
    const uint32_t us[4] = {u.x, u.y, u.z, u.w};
    int xi[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      xi[2 * q] = __float2int_rn(__fmul_rn(__uint_as_float(us[q] << 16), fs.up));
      xi[2 * q + 1] = __float2int_rn(__fmul_rn(__uint_as_float(us[q] & 0xFFFF0000u), fs.up));
    }
    uint32_t he = 0, ho = 0, le = 0, lo = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int a = xi[2 * q], b = xi[2 * q + 1];
      he |= (uint32_t(a >> 8) & 0xFFu) << (8 * q);
      ho |= (uint32_t(b >> 8) & 0xFFu) << (8 * q);
      le |= (uint32_t(a) & 0xFFu) << (8 * q);
      lo |= (uint32_t(b) & 0xFFu) << (8 * q);
      sum += a + b;
    }
    gx.hi_e[w] = he;
    gx.hi_o[w] = ho;
    gx.lo_e[w] = le;
    gx.lo_o[w] = lo;
  }
  gx.X = float(sum);
}

// Exact integer dot of one group (32 bytes of codes) with prepared x.
__device__ __forceinline__ int group_dot(const uint4 (&w)[2], const GroupX& gx) {
  int hi = 0;
  unsigned lo = 0;
  const uint32_t ws[8] = {w[0].x, w[0].y, w[0].z, w[0].w, w[1].x, w[1].y, w[1].z, w[1].w};
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t e = ws[k] & 0x0F0F0F0Fu, o = (ws[k] >> 4) & 0x0F0F0F0Fu;
    hi = __dp4a(int(e), int(gx.hi_e[k]), hi);
    hi = __dp4a(int(o), int(gx.hi_o[k]), hi);
    lo = __dp4a(e, gx.lo_e[k], lo);
    lo = __dp4a(o, gx.lo_o[k], lo);
  }
  return hi * 256 + int(lo);
}

__device__ __forceinline__ float fold_group(float acc, int D, float X, float s, float b) {
  acc = __fmaf_rn(s, float(D), acc);
  return __fmaf_rn(b, X, acc);
}

// Prepare a lane's groups of x (bf16 vector in shared memory) for segment seg.
template <int K>
__device__ __forceinline__ void prep_lane_x(const uint16_t* x, FixScale fs, int seg, int l,
                                            GroupX (&gx)[KCfg<K>::GPL]) {
#pragma unroll
  for (int m = 0; m < KCfg<K>::GPL; ++m)
    prep_group(x + KCfg<K>::group(seg, l, m) * 64, fs, gx[m], KCfg<K>::wide ? lane_half(l) : 0);
}

// Fixed-point limbs of n_groups groups of 64 bf16 values at x (shared
// memory), prepared once for all lanes and written in place in the layout
// [chunk 0..7][group] of uint4 (chunks 0,1 = hi_e, 2,3 = hi_o, 4,5 = lo_e,
// 6,7 = lo_o), with X[g] = float(exact sum of the group's xi).  Group g uses
// the up-scale upf(g).  Threads [0, NT) of the calling group call it (sync:
// a barrier over them); n_groups * 8 <= MAXI * NT.  The values are those of
// prep_group.
template <int MAXI, int NT, class UpF, class Sync>
__device__ __forceinline__ void prep_limbs_inplace(uint16_t* x, float* X, int n_groups, int t, UpF upf, Sync sync) {
  uint32_t he[MAXI], ho[MAXI], le[MAXI], lo[MAXI];
  const int n_items = n_groups * 8;
#pragma unroll
  for (int q = 0; q < MAXI; ++q) {
    const int idx = t + q * NT;
    int part = 0;
    he[q] = ho[q] = le[q] = lo[q] = 0;
    if (idx < n_items) {
      const uint4 u = *reinterpret_cast<const uint4*>(x + idx * 8);
      const float up = upf(idx >> 3);
      const uint32_t us[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int a = __float2int_rn(__fmul_rn(__uint_as_float(us[k] << 16), up));
        const int b = __float2int_rn(__fmul_rn(__uint_as_float(us[k] & 0xFFFF0000u), up));
        he[q] |= (uint32_t(a >> 8) & 0xFFu) << (8 * k);
        ho[q] |= (uint32_t(b >> 8) & 0xFFu) << (8 * k);
        le[q] |= (uint32_t(a) & 0xFFu) << (8 * k);
        lo[q] |= (uint32_t(b) & 0xFFu) << (8 * k);
        part += a + b;
      }
    }
    // the 8 items of a group are 8 consecutive lanes of one warp
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    part += __shfl_xor_sync(0xffffffffu, part, 4);
    if (idx < n_items && (idx & 7) == 0) X[idx >> 3] = float(part);
  }
  sync();
  uint32_t* L = reinterpret_cast<uint32_t*>(x);
#pragma unroll
  for (int q = 0; q < MAXI; ++q) {
    const int idx = t + q * NT;
    if (idx < n_items) {
      const int g = idx >> 3, w = idx & 7, c = w >> 2, j = w & 3;
      L[((0 + c) * n_groups + g) * 4 + j] = he[q];
      L[((2 + c) * n_groups + g) * 4 + j] = ho[q];
      L[((4 + c) * n_groups + g) * 4 + j] = le[q];
      L[((6 + c) * n_groups + g) * 4 + j] = lo[q];
    }
  }
  sync();
}

// The same limbs written to a separate buffer `out` (one pass; callers
// synchronize before reading them).
template <int NT, class UpF>
__device__ __forceinline__ void prep_limbs_to(const uint16_t* x, uint16_t* out, float* X, int n_groups, int t,
                                              UpF upf) {
  const int n_items = n_groups * 8;
  uint32_t* L = reinterpret_cast<uint32_t*>(out);
  for (int base = 0; base < n_items; base += NT) {
    const int idx = base + t;
    int part = 0;
    uint32_t he = 0, ho = 0, le = 0, lo = 0;
    if (idx < n_items) {
      const uint4 u = *reinterpret_cast<const uint4*>(x + idx * 8);
      const float up = upf(idx >> 3);
      const uint32_t us[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int a = __float2int_rn(__fmul_rn(__uint_as_float(us[k] << 16), up));
        const int b = __float2int_rn(__fmul_rn(__uint_as_float(us[k] & 0xFFFF0000u), up));
        he |= (uint32_t(a >> 8) & 0xFFu) << (8 * k);
        ho |= (uint32_t(b >> 8) & 0xFFu) << (8 * k);
        le |= (uint32_t(a) & 0xFFu) << (8 * k);
        lo |= (uint32_t(b) & 0xFFu) << (8 * k);
        part += a + b;
      }
      const int g = idx >> 3, w = idx & 7, c = w >> 2, j = w & 3;
      L[((0 + c) * n_groups + g) * 4 + j] = he;
      L[((2 + c) * n_groups + g) * 4 + j] = ho;
      L[((4 + c) * n_groups + g) * 4 + j] = le;
      L[((6 + c) * n_groups + g) * 4 + j] = lo;
    }
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    part += __shfl_xor_sync(0xffffffffu, part, 4);
    if (idx < n_items && (idx & 7) == 0) X[idx >> 3] = float(part);
  }
}

// A lane's prepared group g from the shared limbs of prep_limbs_inplace.
__device__ __forceinline__ void load_limbs(const uint16_t* x, const float* X, int n_groups, int g, GroupX& gx,
                                           int sw = 0) {
  const uint4* L = reinterpret_cast<const uint4*>(x);
  uint4 c[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) c[k] = L[(k ^ sw) * n_groups + g];  // sw: halves swapped (lane_half)
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    gx.hi_e[4 * k] = c[k].x; gx.hi_e[4 * k + 1] = c[k].y; gx.hi_e[4 * k + 2] = c[k].z; gx.hi_e[4 * k + 3] = c[k].w;
    gx.hi_o[4 * k] = c[2 + k].x; gx.hi_o[4 * k + 1] = c[2 + k].y; gx.hi_o[4 * k + 2] = c[2 + k].z;
    gx.hi_o[4 * k + 3] = c[2 + k].w;
    gx.lo_e[4 * k] = c[4 + k].x; gx.lo_e[4 * k + 1] = c[4 + k].y; gx.lo_e[4 * k + 2] = c[4 + k].z;
    gx.lo_e[4 * k + 3] = c[4 + k].w;
    gx.lo_o[4 * k] = c[6 + k].x; gx.lo_o[4 * k + 1] = c[6 + k].y; gx.lo_o[4 * k + 2] = c[6 + k].z;
    gx.lo_o[4 * k + 3] = c[6 + k].w;
  }
  gx.X = X[g];
}

// Lane partials of ILP rows at once (independent chains for the scheduler).
template <int K, int SD, int ILP>
__device__ __forceinline__ void lane_rows_partial(const uint8_t* wbase, const uint16_t* sbase,
                                                  const uint16_t* bbase, const int (&rows)[ILP], int seg, int l,
                                                  const GroupX (&gx)[KCfg<K>::GPL], float (&out)[ILP],
                                                  int sd_rt = 0) {
  float acc[ILP];
#pragma unroll
  for (int i = 0; i < ILP; ++i) acc[i] = 0.0f;
  // wide rows: the halves in the lane's order (lane_half); gx matches it
  const int h0 = KCfg<K>::wide ? 16 * lane_half(l) : 0;
#pragma unroll
  for (int m = 0; m < KCfg<K>::GPL; ++m) {
    const int g = KCfg<K>::group(seg, l, m);
    uint4 w[ILP][2];
#pragma unroll
    for (int i = 0; i < ILP; ++i) {
      const uint8_t* p = wbase + rows[i] * KCfg<K>::ROW_BYTES + g * 32;
      w[i][0] = lds128(p + h0);
      w[i][1] = lds128(p + (16 - h0));
    }
    int D[ILP];
#pragma unroll
    for (int i = 0; i < ILP; ++i) D[i] = group_dot(w[i], gx[m]);
#pragma unroll
    for (int i = 0; i < ILP; ++i) {
      const float s = sb<SD>(sbase[rows[i] * KCfg<K>::GROUPS + g], sd_rt);
      const float b = sb<SD>(bbase[rows[i] * KCfg<K>::GROUPS + g], sd_rt);
      acc[i] = fold_group(acc[i], D[i], gx[m].X, s, b);
    }
  }
#pragma unroll
  for (int i = 0; i < ILP; ++i) out[i] = acc[i];
}

// lane_rows_partial with the lane's groups read from the shared limbs of
// prep_limbs_inplace one at a time (group index g0 + KCfg<K>::group(0, l, m)).
template <int K, int SD, int ILP>
__device__ __forceinline__ void lane_rows_partial_shared(const uint8_t* wbase, const uint16_t* sbase,
                                                         const uint16_t* bbase, const int (&rows)[ILP], int l,
                                                         const uint16_t* limbs, const float* X, int n_groups,
                                                         int g0, float (&out)[ILP], int sd_rt = 0) {
  float acc[ILP];
#pragma unroll
  for (int i = 0; i < ILP; ++i) acc[i] = 0.0f;
#pragma unroll
  for (int m = 0; m < KCfg<K>::GPL; ++m) {
    const int g = KCfg<K>::group(0, l, m);
    GroupX gx;
    load_limbs(limbs, X, n_groups, g0 + g, gx);
    uint4 w[ILP][2];
#pragma unroll
    for (int i = 0; i < ILP; ++i) {
      const uint8_t* p = wbase + rows[i] * KCfg<K>::ROW_BYTES + g * 32;
      w[i][0] = lds128(p);
      w[i][1] = lds128(p + 16);
    }
#pragma unroll
    for (int i = 0; i < ILP; ++i) {
      const int D = group_dot(w[i], gx);
      const float s = sb<SD>(sbase[rows[i] * KCfg<K>::GROUPS + g], sd_rt);
      const float b = sb<SD>(bbase[rows[i] * KCfg<K>::GROUPS + g], sd_rt);
      acc[i] = fold_group(acc[i], D, gx.X, s, b);
    }
  }
#pragma unroll
  for (int i = 0; i < ILP; ++i) out[i] = acc[i];
}

// Butterfly over the lanes of one row.
template <int K>
__device__ __forceinline__ float row_reduce(float v) {
  return bfly_sum<KCfg<K>::T>(v);
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
