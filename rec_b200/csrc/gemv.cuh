// Streaming int4 GEMV kernel used for the dense projections (QKV, O) and the
// lm_head, plus the CTA-level RMSNorm prologue they share.
#pragma once
#include "qdot.cuh"

namespace rec {

constexpr int kThreads = 256;  // 8 warps per CTA for all GEMV-type kernels
constexpr int kWarps = kThreads / 32;

// --- RMSNorm of a bf16 vector into shared memory -----------------------------
// Canonical order: H/8 chunks of 8 elements summed sequentially (fused
// multiply-adds of squares), groups of 32 chunks combined by butterfly, group
// sums added in order; inv = 1/sqrt(ss/H + eps); out = bf16(w * bf16(h*inv)).
// Reference: megakernel.py:726-744 (rms_256_w4).  Needs H % 256 == 0 and
// H/256 <= 32.  All threads of the CTA must call it.
__device__ __forceinline__ void cta_rmsnorm(const uint16_t* h, const uint16_t* w, int H, float eps,
                                            uint16_t* out_smem, float* red_smem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = H >> 8;
  for (int g = warp; g < groups; g += kWarps) {
    uint4 u = ldg128(h + (g * 32 + lane) * 8);
    const uint32_t us[4] = {u.x, u.y, u.z, u.w};
    float a = 0.0f;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      float x0 = __uint_as_float(us[t] << 16), x1 = __uint_as_float(us[t] & 0xFFFF0000u);
      a = __fmaf_rn(x0, x0, a);
      a = __fmaf_rn(x1, x1, a);
    }
    a = bfly_sum(a);
    if (lane == 0) red_smem[g] = a;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float total = 0.0f;
    for (int g = 0; g < groups; ++g) total = __fadd_rn(total, red_smem[g]);
    float mean = __fdiv_rn(total, float(H));
    red_smem[32] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  }
  __syncthreads();
  const float inv = red_smem[32];
  for (int i = threadIdx.x; i < H; i += kThreads)
    out_smem[i] = to_bf(__fmul_rn(bf(w[i]), rbf(__fmul_rn(bf(h[i]), inv))));
  __syncthreads();
}

// --- generic streaming GEMV ---------------------------------------------------
enum EpiKind { kEpiStore = 0, kEpiResidual = 1, kEpiArgmax = 2 };

struct GemvArgs {
  QMatDev mat[3];
  int rows[3];       // rows of each matrix (concatenated in order)
  int total_rows;
  const uint16_t* x;       // bf16[K] input (raw h when norm_w != null)
  const uint16_t* norm_w;  // bf16[K] RMSNorm weight or null
  float eps;
  uint16_t* out;           // bf16 rows (kEpiStore, kEpiArgmax)
  uint16_t* resid;         // bf16 residual updated in place (kEpiResidual)
  uint16_t* trace_out;     // kEpiResidual: also a copy of the updated rows (a layer's trace row), or null
  float* cand_val;         // kEpiArgmax: per-CTA best value
  int* cand_idx;           //             per-CTA best index
  unsigned* counter;       //             CTA arrival counter (reset by the last CTA)
  int* token_out;          //             argmax result
  int* status;
  int pdl;                 // griddepcontrol.wait before reading x
};

template <int K, int RS, int NS>
struct GemvSmem {
  using L = StageLayout<K, RS>;
  alignas(128) uint8_t stage[NS][L::BYTES];
  alignas(16) uint16_t xn[K];
  uint64_t full[NS];
  float red[40];
  float seg_part[kWarps][RS];  // team partials (SEG > 1)
  float best_val[kWarps];
  int best_idx[kWarps];
  int is_last;
};

// Cursor over the stages of a CTA's row range (stages never cross matrices).
struct StageCursor {
  int cur, end;
  __device__ bool next(const GemvArgs& a, int rs, int& mat, int& row0, int& nrows, int& grow0) {
    if (cur >= end) return false;
    int base = 0, mi = 0;
    while (mi < 2 && cur >= base + a.rows[mi]) base += a.rows[mi++];
    int stop = min(min(cur + rs, end), base + a.rows[mi]);
    mat = mi;
    row0 = cur - base;
    nrows = stop - cur;
    grow0 = cur;
    cur = stop;
    return true;
  }
};

// Rows computed together by one warp (independent dependency chains).
template <int K>
constexpr int gemv_ilp() { return KCfg<K>::wide ? 4 : 1; }
// Stage rows: one full pass of the CTA over its row slots (K = 6144: two
// teams of three warps; the other two warps only wait on the stages).
template <int K>
constexpr int gemv_rs() {
  return (kWarps / (KCfg<K>::wide ? KCfg<K>::SEG : 1)) * (32 / KCfg<K>::T) * gemv_ilp<K>();
}

template <int K, int SD, int RS, int NS, int EPI>
__global__ void __launch_bounds__(kThreads, 1) k_gemv(const GemvArgs a) {
  constexpr int ILP = gemv_ilp<K>();
  static_assert(RS >= ILP, "stage must hold one row per ILP slot");
  using C = KCfg<K>;
  using S = GemvSmem<K, RS, NS>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  S& sm = *reinterpret_cast<S*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  int r_begin, r_end;
  split_range(a.total_rows / 2, gridDim.x, blockIdx.x, r_begin, r_end);
  r_begin *= 2;
  r_end = (blockIdx.x == gridDim.x - 1) ? a.total_rows : r_end * 2;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(&sm.full[s], 1);
    fence_barrier_init();
  }
  __syncthreads();

  StageCursor prod{r_begin, r_end}, cons{r_begin, r_end};
  int issued = 0;  // meaningful in thread 0 only
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      int mat, row0, nrows, g0;
      if (!prod.next(a, RS, mat, row0, nrows, g0)) break;
      issue_stage<K, RS>(sm.stage[s], &sm.full[s], a.mat[mat], row0, nrows);
      ++issued;
    }
  }
  if (a.pdl) grid_wait();
  grid_launch_dependents();

  // x (optionally normalised) into shared memory, then the lane's chunks.
  if (a.norm_w) {
    cta_rmsnorm(a.x, a.norm_w, K, a.eps, sm.xn, sm.red);
  } else {
    for (int i = threadIdx.x * 8; i < K; i += kThreads * 8)
      *reinterpret_cast<uint4*>(sm.xn + i) = ldg128(a.x + i);
    __syncthreads();
  }
  const FixScale fs = fix_scale_from_max(block_maxabs(sm.xn, K, threadIdx.x, kThreads, sm.red, 0));
  // Team layout: TEAM warps per row for SEG > 1 (one segment each); for
  // narrow K, 8 rows per warp with 4 lanes each.
  constexpr int SEG = C::SEG;
  constexpr int TEAM = C::wide ? SEG : 1;
  constexpr int TEAMS = kWarps / TEAM;
  static_assert(TEAMS >= 1, "a row needs at most 8 warps");
  constexpr int ROWS_PER_WARP = 32 / C::T;
  const int seg = C::wide ? warp % TEAM : 0;
  const int team = warp / TEAM;
  const int sub = lane / C::T;  // row slot inside the warp
  const int l = lane % C::T;    // lane inside the row
  GroupX gx[C::GPL];
  prep_lane_x<K>(sm.xn, fs, seg, l, gx);

  float best = -INFINITY;
  int best_i = 0x7fffffff;
  bool failed = false;
  int j = 0;
  int mat, row0, nrows, g0;
  while (cons.next(a, RS, mat, row0, nrows, g0)) {
    const int slot = j % NS;
    const uint32_t parity = (j / NS) & 1;
    if (!mbar_wait(&sm.full[slot], parity)) failed = true;
    if (!failed) {
      const uint8_t* st = sm.stage[slot];
      const uint8_t* wbase = stage_wrow<K, RS>(st, 0);
      const uint16_t* sbase = stage_srow<K, RS>(st, 0);
      const uint16_t* bbase = stage_brow<K, RS>(st, 0);
      // Row slots are walked uniformly by whole warps so that shuffles see
      // every lane; slots past the stage's rows compute nothing.
      constexpr int SLOTS = TEAMS * ROWS_PER_WARP;  // rows per sub-pass
      // warps outside the teams (kWarps % TEAM of them) compute nothing
      for (int rb = 0; team < TEAMS && rb < nrows; rb += SLOTS * ILP) {
        int rows[ILP];
        bool valid[ILP];
#pragma unroll
        for (int i = 0; i < ILP; ++i) {
          const int r = rb + i * SLOTS + team * ROWS_PER_WARP + sub;
          valid[i] = r < nrows;
          rows[i] = valid[i] ? r : 0;
        }
        float v[ILP];
        lane_rows_partial<K, SD, ILP>(wbase, sbase, bbase, rows, seg, l, gx, v);
#pragma unroll
        for (int i = 0; i < ILP; ++i) {
          if (!valid[i]) v[i] = 0.0f;
          v[i] = row_reduce<K>(v[i]);
        }
        if constexpr (SEG > 1) {
          // segment partials added in order by the team's first warp
          if (lane == 0) {
#pragma unroll
            for (int i = 0; i < ILP; ++i) sm.seg_part[warp][i] = v[i];
          }
          asm volatile("bar.sync %0, %1;" ::"r"(1 + team), "r"(TEAM * 32));
          if (seg == 0) {
#pragma unroll
            for (int i = 0; i < ILP; ++i) {
              float t = v[i];
              for (int s2 = 1; s2 < SEG; ++s2) t = __fadd_rn(t, sm.seg_part[warp + s2][i]);
              v[i] = t;
            }
          }
          asm volatile("bar.sync %0, %1;" ::"r"(1 + team), "r"(TEAM * 32));
        }
        // residual rows read before any store, so the loads are in flight together
        float res[ILP];
#pragma unroll
        for (int i = 0; i < ILP; ++i) {
          res[i] = 0.0f;
          if constexpr (EPI == kEpiResidual)
            if (valid[i] && (C::wide ? (lane == 0 && seg == 0) : (l == 0))) res[i] = bf(a.resid[g0 + rows[i]]);
        }
#pragma unroll
        for (int i = 0; i < ILP; ++i) {
          const bool writer = valid[i] && (C::wide ? (lane == 0 && seg == 0) : (l == 0));
          v[i] = __fmul_rn(v[i], fs.down);
          if (writer) {
            const int grow = g0 + rows[i];
            if constexpr (EPI == kEpiStore) {
              a.out[grow] = to_bf(v[i]);
            } else if constexpr (EPI == kEpiResidual) {
              const uint16_t hn = to_bf(__fadd_rn(res[i], rbf(v[i])));
              a.resid[grow] = hn;
              if (a.trace_out) a.trace_out[grow] = hn;
            } else {
              uint16_t o = to_bf(v[i]);
              a.out[grow] = o;
              float fv = bf(o);
              if (fv > best || (fv == best && grow < best_i)) { best = fv; best_i = grow; }
            }
          }
        }
      }
    }
    if (__syncthreads_or(failed)) {
      failed = true;
      break;
    }
    if (threadIdx.x == 0) {
      int m2, r2, n2, gg;
      if (prod.next(a, RS, m2, r2, n2, gg)) {
        issue_stage<K, RS>(sm.stage[slot], &sm.full[slot], a.mat[m2], r2, n2);
        ++issued;
      }
    }
    ++j;
  }
  if (failed) {
    if (threadIdx.x == 0) {
      report(a.status, kStatusBulkTimeout);
      // drain copies still in flight into this CTA's shared memory
      for (int s = j; s < issued; ++s) mbar_wait(&sm.full[s % NS], (s / NS) & 1);
    }
    return;
  }

  if constexpr (EPI == kEpiArgmax) {
    // CTA best (lowest index among equal maxima), then the last CTA reduces.
    for (int off = 16; off >= 1; off >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, best, off);
      int oi = __shfl_xor_sync(0xffffffffu, best_i, off);
      if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
    }
    if (lane == 0) { sm.best_val[warp] = best; sm.best_idx[warp] = best_i; }
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int w = 1; w < kWarps; ++w)
        if (sm.best_val[w] > best || (sm.best_val[w] == best && sm.best_idx[w] < best_i)) {
          best = sm.best_val[w]; best_i = sm.best_idx[w];
        }
      a.cand_val[blockIdx.x] = best;
      a.cand_idx[blockIdx.x] = best_i;
      __threadfence();
      unsigned prev = atomicAdd(a.counter, 1u);
      sm.is_last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (sm.is_last) {
      __threadfence();
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int c = threadIdx.x; c < gridDim.x; c += kThreads) {
        float v = __ldcg(a.cand_val + c);
        int i = __ldcg(a.cand_idx + c);
        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
      }
      for (int off = 16; off >= 1; off >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
      if (lane == 0) { sm.best_val[warp] = bv; sm.best_idx[warp] = bi; }
      __syncthreads();
      if (threadIdx.x == 0) {
        for (int w = 0; w < kWarps; ++w)
          if (sm.best_val[w] > bv || (sm.best_val[w] == bv && sm.best_idx[w] < bi)) {
            bv = sm.best_val[w]; bi = sm.best_idx[w];
          }
        *a.token_out = bi;
        *a.counter = 0;
      }
    }
  }
}

template <int K, int SD, int RS, int NS, int EPI>
inline cudaError_t launch_gemv(const GemvArgs& a, int grid, cudaStream_t st, bool pdl) {
  auto kern = k_gemv<K, SD, RS, NS, EPI>;
  const size_t smem = sizeof(GemvSmem<K, RS, NS>);
  if (smem > 48 * 1024) {
    cudaError_t e = set_smem_limit(reinterpret_cast<const void*>(kern), smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  GemvArgs b = a;
  b.pdl = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, b);
}

}  // namespace rec
