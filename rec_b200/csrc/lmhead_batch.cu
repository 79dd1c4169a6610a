// int4 g64 GEMV for up to 8 input vectors at once (the batch-8 sampling
// head's final norm + lm_head), on the tensor cores: one pass over the
// weights instead of one per vector.
//
// The result is bit-identical to k_gemv (gemv.cuh) run once per vector: the
// same RMSNorm, the same per-vector fixed-point scale and limbs, the same
// exact integer group dots, and the same fold order:
//   f_g = fma(bias_g, X_g, fma(scale_g, float(D_g), 0))   (one group per lane)
//   y   = bf16(butterfly_32(f) * 2^-F)                   (xor 16, 8, 4, 2, 1)
// Only the integer dots move: D_g for 8 weight rows x 8 vectors comes from
// mma.sync m16n8k32 (A = the vectors' limbs, B = the weight codes), with the
// hi limb (signed) and the lo limb (unsigned) in separate MMAs.  The butterfly
// is evaluated as the same binary tree over the 32 groups, taken in
// bit-reversed order so that a small stack of partial sums suffices.
//
// Layout: CTA of 8 warps; a stage holds 64 weight rows (8 tiles of 8 rows),
// one tile per warp.  Code rows are copied one bulk copy per row into rows
// of 1,056 bytes (1,024 + 32), so that the B fragments (8 rows, same column)
// fall in distinct banks.  Warp 0 issues the copies.
#include "capi_common.h"
#include "gemv.cuh"

namespace rec {

constexpr int kLbRows = 64;          // rows per stage (8 tiles of 8)
constexpr int kLbStride = 1056;      // shared row stride of the codes
constexpr int kLbStages = 2;
constexpr int kLbMaxB = 8;
constexpr int kLbLimbStride = 4112;  // bytes per vector's limbs (4,096 + 16: conflict-free A loads)

struct LbSmem {
  alignas(128) uint8_t codes[kLbStages][kLbRows * kLbStride];
  alignas(16) uint16_t sc[kLbStages][kLbRows * 32];
  alignas(16) uint16_t bi[kLbStages][kLbRows * 32];
  alignas(16) uint8_t limbs[kLbMaxB * kLbLimbStride];
  float X[kLbMaxB][32];
  float down[kLbMaxB];
  alignas(16) uint16_t xn[2048];
  float red[40];
  uint64_t full[kLbStages];
};

struct LbArgs {
  QMatDev w;             // [V, 2048] int4 g64
  int V, B;
  const uint16_t* h;     // bf16 [B, 2048]
  const uint16_t* norm;  // final RMSNorm weight
  float eps;
  uint16_t* out;         // bf16 [B, V]
  int* status;
};

// A = {a0, 0, a2, 0}: rows 0..7 of the tile hold the 8 vectors' limbs, rows
// 8..15 are zero.
__device__ __forceinline__ void mma_s8u8_lb(int (&c)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_u8u8_lb(int (&c)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

// Stage s <- rows [row0, row0 + n) (warp 0, all lanes).
__device__ __forceinline__ void lb_issue(LbSmem& sm, int s, const LbArgs& a, int row0, int n, int lane) {
  if (lane == 0) mbar_expect_tx(&sm.full[s], uint32_t(n) * (1024 + 2 * 64));
  __syncwarp();
  for (int r = lane; r < n; r += 32)
    bulk_g2s(sm.codes[s] + r * kLbStride, reinterpret_cast<const uint8_t*>(a.w.w) + size_t(row0 + r) * 1024, 1024,
             &sm.full[s]);
  if (lane == 0) {
    bulk_g2s(sm.sc[s], a.w.s + size_t(row0) * 32, uint32_t(n) * 64, &sm.full[s]);
    bulk_g2s(sm.bi[s], a.w.b + size_t(row0) * 32, uint32_t(n) * 64, &sm.full[s]);
  }
}

template <int SD>
__global__ void __launch_bounds__(kThreads, 1) k_gemv_batch(const LbArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  LbSmem& sm = *reinterpret_cast<LbSmem*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gq = lane >> 2, tq = lane & 3;
  // this CTA's 8-row tiles
  int t0, t1;
  split_range(a.V / 8, gridDim.x, blockIdx.x, t0, t1);
  const int row_begin = 8 * t0, row_end = 8 * t1;
  const int n_stages = (row_end - row_begin + kLbRows - 1) / kLbRows;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kLbStages; ++s) mbar_init(&sm.full[s], 1);
    fence_barrier_init();
  }
  __syncthreads();
  int issued = 0;  // stages issued (warp 0)
  if (warp == 0)
    for (int s = 0; s < kLbStages && s < n_stages; ++s, ++issued)
      lb_issue(sm, s, a, row_begin + s * kLbRows, min(kLbRows, row_end - row_begin - s * kLbRows), lane);

  // per vector: RMSNorm, fixed-point scale, limbs [b][group][tq][word parity]
  // = uint4 {hi even, hi odd, lo even, lo odd}, exact group sums X
  for (int b = 0; b < kLbMaxB; ++b) {
    uint32_t he = 0, ho = 0, le = 0, lo = 0;
    int part = 0;
    float down = 0.0f;
    if (b < a.B) {
      cta_rmsnorm(a.h + size_t(b) * 2048, a.norm, 2048, a.eps, sm.xn, sm.red);
      const FixScale fs = fix_scale_from_max(block_maxabs(sm.xn, 2048, threadIdx.x, kThreads, sm.red, 0));
      down = fs.down;
      const uint4 u = *reinterpret_cast<const uint4*>(sm.xn + threadIdx.x * 8);  // word threadIdx.x
      const uint32_t us[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int x0 = __float2int_rn(__fmul_rn(__uint_as_float(us[q] << 16), fs.up));
        const int x1 = __float2int_rn(__fmul_rn(__uint_as_float(us[q] & 0xFFFF0000u), fs.up));
        he |= (uint32_t(x0 >> 8) & 0xFFu) << (8 * q);
        ho |= (uint32_t(x1 >> 8) & 0xFFu) << (8 * q);
        le |= (uint32_t(x0) & 0xFFu) << (8 * q);
        lo |= (uint32_t(x1) & 0xFFu) << (8 * q);
        part += x0 + x1;
      }
    }
    // the 8 words of a group are 8 consecutive threads
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    part += __shfl_xor_sync(0xffffffffu, part, 4);
    const int w = threadIdx.x, g = w >> 3, wg = w & 7;
    *reinterpret_cast<uint4*>(sm.limbs + b * kLbLimbStride + ((g * 4 + (wg >> 1)) * 2 + (wg & 1)) * 16) =
        make_uint4(he, ho, le, lo);
    if ((w & 7) == 0) sm.X[b][g] = float(part);
    if (threadIdx.x == 0) sm.down[b] = down;
    __syncthreads();
  }

  const uint8_t* my_limbs = sm.limbs + gq * kLbLimbStride + tq * 32;
  const float down = sm.down[gq];
  bool failed = false;
  int j = 0;
  for (; j < n_stages; ++j) {
    const int s = j % kLbStages;
    const int row0 = row_begin + j * kLbRows;
    const int n = min(kLbRows, row_end - row0);
    if (!mbar_wait(&sm.full[s], (j / kLbStages) & 1)) failed = true;
    if (!failed && 8 * warp < n) {
      const uint8_t* crow = sm.codes[s] + (8 * warp + gq) * kLbStride + tq * 8;  // B: weight row gq of the tile
      const uint16_t* srow = sm.sc[s] + (8 * warp + 2 * tq) * 32;               // rows 2tq, 2tq+1 of the tile
      const uint16_t* brow = sm.bi[s] + (8 * warp + 2 * tq) * 32;
      float st0[5], st1[5];  // partial sums of the butterfly tree, per level
      float r0 = 0.0f, r1 = 0.0f;
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const int g = ((k & 1) << 4) | ((k & 2) << 2) | (k & 4) | ((k & 8) >> 2) | ((k & 16) >> 4);  // bitrev5
        const uint2 wv = *reinterpret_cast<const uint2*>(crow + g * 32);
        const uint4 L0 = *reinterpret_cast<const uint4*>(my_limbs + g * 128);
        const uint4 L1 = *reinterpret_cast<const uint4*>(my_limbs + g * 128 + 16);
        const uint32_t e0 = wv.x & 0x0F0F0F0Fu, o0 = (wv.x >> 4) & 0x0F0F0F0Fu;
        const uint32_t e1 = wv.y & 0x0F0F0F0Fu, o1 = (wv.y >> 4) & 0x0F0F0F0Fu;
        int Hd[4] = {0, 0, 0, 0}, Ld[4] = {0, 0, 0, 0};
        mma_s8u8_lb(Hd, L0.x, L0.y, e0, o0);
        mma_s8u8_lb(Hd, L1.x, L1.y, e1, o1);
        mma_u8u8_lb(Ld, L0.z, L0.w, e0, o0);
        mma_u8u8_lb(Ld, L1.z, L1.w, e1, o1);
        const int D0 = Hd[0] * 256 + Ld[0], D1 = Hd[1] * 256 + Ld[1];  // vector gq, rows 2tq, 2tq+1
        const float X = sm.X[gq][g];
        float f0 = __fmaf_rn(sb<SD>(srow[g]), float(D0), 0.0f);
        f0 = __fmaf_rn(sb<SD>(brow[g]), X, f0);
        float f1 = __fmaf_rn(sb<SD>(srow[32 + g]), float(D1), 0.0f);
        f1 = __fmaf_rn(sb<SD>(brow[32 + g]), X, f1);
        // leaf k: climb while this node is a right child
#pragma unroll
        for (int lvl = 0; lvl < 5; ++lvl) {
          if ((k >> lvl) & 1) {
            f0 = __fadd_rn(st0[lvl], f0);
            f1 = __fadd_rn(st1[lvl], f1);
          } else {
            st0[lvl] = f0;
            st1[lvl] = f1;
            break;
          }
        }
        if (k == 31) {
          r0 = f0;
          r1 = f1;
        }
      }
      const int row = row0 + 8 * warp + 2 * tq;
      if (gq < a.B) {
        const uint32_t o = uint32_t(to_bf(__fmul_rn(r0, down))) | (uint32_t(to_bf(__fmul_rn(r1, down))) << 16);
        *reinterpret_cast<uint32_t*>(a.out + size_t(gq) * a.V + row) = o;
      }
    }
    if (__syncthreads_or(failed)) {
      failed = true;
      break;
    }
    // slot s is free: its next stage
    if (warp == 0 && j + kLbStages < n_stages) {
      const int nr = row_begin + (j + kLbStages) * kLbRows;
      lb_issue(sm, s, a, nr, min(kLbRows, row_end - nr), lane);
      ++issued;
    }
  }
  if (failed && warp == 0 && lane == 0) {
    report(a.status, kStatusBulkTimeout);
    // let the copies still in flight into this CTA's shared memory land
    for (int q = j; q < issued; ++q) mbar_wait(&sm.full[q % kLbStages], (q / kLbStages) & 1);
  }
}

// Final RMSNorm + lm_head for B <= 8 hidden rows (K = 2048, V % 8 == 0).
int lmhead_batch(const RecQMat* w, int sd, int V, const void* h, int B, const void* norm, float eps, void* out,
                 int* status, cudaStream_t st) {
  LbArgs a = {};
  a.w = {static_cast<const uint32_t*>(w->w), static_cast<const uint16_t*>(w->scales),
         static_cast<const uint16_t*>(w->biases)};
  a.V = V;
  a.B = B;
  a.h = static_cast<const uint16_t*>(h);
  a.norm = static_cast<const uint16_t*>(norm);
  a.eps = eps;
  a.out = static_cast<uint16_t*>(out);
  a.status = status;
  const size_t smem = sizeof(LbSmem);
  auto kern = sd == REC_SCALE_FP16 ? k_gemv_batch<0> : k_gemv_batch<1>;
  REC_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
  kern<<<sm_count(), kThreads, smem, st>>>(a);
  REC_CHECK_CUDA(cudaGetLastError());
  return REC_OK;
}

}  // namespace rec
