// Prefill projection GEMM on the 5th-generation tensor cores (tcgen05):
//   Y[T, N] = X[T, K] . W[N, K]^T
// X bf16 row-major (the prompt's activations), W int4 g64 in the MLX affine
// layout (uint32 nibbles, fp16 or bf16 scale and bias per 64 weights), Y bf16.
// Reference: the prefill of QATSession.prefill / m4_max_prefill
// (engine/src/rec_mlx/quantized.py:102-148, kernels/m4_max_prefill.py:49-144),
// whose projections are mx.quantized_matmul over the prompt's tokens.
//
// One CTA computes a 128 x 256 tile of Y with K walked in steps of 64 (one
// quantization group), through a 2-stage shared-memory ring:
//   * the X tile (128 tokens x 64) arrives by TMA (cp.async.bulk.tensor, 128B
//     swizzle) on the stage's mbarrier;
//   * the W tile (256 rows x 64) is dequantized by the 256 threads (one row
//     each, its codes fetched one K step ahead), w = fma(scale, q, bias) in
//     fp32, and written as two bf16 tiles in the same 128B-swizzled K-major
//     layout: w_hi = bf16(w) and w_lo = bf16(w - w_hi);
//   * thread 0 issues eight tcgen05.mma kind::f16 (M 128, N 256, K 16, bf16
//     in, fp32 accumulate in tensor memory: X w_hi^T and X w_lo^T into the
//     same accumulator) and commits them to the stage's "empty" mbarrier,
//     which frees the stage for the next K step;
//   * after the last step the accumulator (128 lanes x 256 columns of TMEM) is
//     read with tcgen05.ld, rounded to bf16 and stored.
// Every wait is bounded: a wait that runs out records kStatusBulkTimeout, the
// CTA drains what it issued, frees its tensor memory and returns.
//
// Numerics: the products are exact (bf16 x bf16 in fp32) and the tensor core
// accumulates in fp32 in its own order, so results are compared with a
// tolerance.  Splitting each dequantized weight into w_hi + w_lo keeps ~16
// significant bits of it (one bf16 operand alone would round it at 2^-9),
// which puts the prefill's hidden states within the decode path's tolerance.
#include <cuda.h>

#include "capi_common.h"
#include "common.cuh"
#include "gemv.cuh"

namespace rec {
namespace {

constexpr int kPBM = 128, kPBN = 256, kPBK = 64, kPStages = 2, kPThreads = 256;
constexpr uint32_t kATileBytes = kPBM * kPBK * 2;  // 16 KB
constexpr uint32_t kBTileBytes = kPBN * kPBK * 2;  // 32 KB
constexpr uint32_t kTmemCols = kPBN;               // fp32 accumulator columns

// b: the dequantized weights rounded to bf16 (w_hi); b2: the remainder
// bf16(w - w_hi).  Both multiply the same X tile into one fp32 accumulator,
// so the weights enter with ~16 significant bits instead of 8.
struct PrefillSmem {
  alignas(1024) uint8_t a[kPStages][kATileBytes];
  alignas(1024) uint8_t b[kPStages][kBTileBytes];
  alignas(1024) uint8_t b2[kPStages][kBTileBytes];
  uint64_t full[kPStages], empty[kPStages], done;
  uint32_t tmem_base;
};

// Shared-memory matrix descriptor of a K-major, 128B-swizzled operand whose
// rows are 128 bytes (64 bf16) and whose 8-row groups are 1,024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = uint64_t((saddr >> 4) & 0x3FFFu);  // start address
  d |= uint64_t(1) << 16;                          // leading byte offset (unused for this layout)
  d |= uint64_t(1024 >> 4) << 32;                  // stride byte offset: 8 rows x 128 B
  d |= uint64_t(1) << 46;                          // descriptor version
  d |= uint64_t(2) << 61;                          // 128-byte swizzle
  return d;
}
// Instruction descriptor: bf16 A and B, fp32 D, both K-major, M = 128, N = 256.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(kPBN >> 3) << 17) |
                            (uint32_t(kPBM >> 4) << 24);

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(kIdesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cta(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y)
      : "memory");
}
// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// tiles (grouped mode, one matrix per expert): tile blockIdx.y is rows
// [row0, row0 + rows) of X and Y multiplied by expert e's W (rows e N ..);
// {e, row0, rows, 0}, rows 0 = no tile.  tiles null: dense, tile blockIdx.y =
// rows 128 blockIdx.y .. of X.
template <int SD>
__global__ void __launch_bounds__(kPThreads, 1)
    k_prefill_gemm(const __grid_constant__ CUtensorMap xmap, const QMatDev w, int K, int N, int T,
                   uint16_t* __restrict__ y, int* status, const int4* __restrict__ tiles) {
  extern __shared__ uint8_t smem_raw[];
  PrefillSmem& sm = *reinterpret_cast<PrefillSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                    ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * kPBN;
  int m0 = blockIdx.y * kPBM, mrows = kPBM;
  size_t wrow0 = 0;
  if (tiles) {
    const int4 tl = tiles[blockIdx.y];
    if (tl.z <= 0) return;  // the whole CTA, before any barrier or tensor memory
    m0 = tl.y;
    mrows = tl.z;
    wrow0 = size_t(tl.x) * N;
  }
  const int KT = K / kPBK;
  if (tid == 0) {
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(&sm.full[s], kPThreads + 1);  // every thread's W rows + the X bytes
      mbar_init(&sm.empty[s], 1);             // the MMAs that read the stage
    }
    mbar_init(&sm.done, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&sm.tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  bool ok = true;
  int issued = 0;  // K steps whose MMAs thread 0 issued
  // this thread's W row (tid): codes, scale and bias of the next K step are
  // loaded one step ahead
  constexpr int RPT = kPBN / kPThreads;  // rows per thread
  uint4 nc[RPT][2];
  uint16_t ns[RPT], nb[RPT];
  auto fetch = [&](int kt) {
#pragma unroll
    for (int rr = 0; rr < RPT; ++rr) {
      const size_t row = wrow0 + size_t(n0 + tid + rr * kPThreads);
      const uint4* src = reinterpret_cast<const uint4*>(w.w + row * (K / 8) + size_t(kt) * 8);
      nc[rr][0] = ldg128_nc(src);
      nc[rr][1] = ldg128_nc(src + 1);
      ns[rr] = w.s[row * (K / 64) + kt];
      nb[rr] = w.b[row * (K / 64) + kt];
    }
  };
  fetch(0);
  for (int kt = 0; kt < KT && ok; ++kt) {
    const int s = kt % kPStages;
    const uint32_t use = uint32_t(kt / kPStages);
    uint4 cc[RPT][2];
    uint16_t cs[RPT], cb[RPT];
#pragma unroll
    for (int rr = 0; rr < RPT; ++rr) {
      cc[rr][0] = nc[rr][0];
      cc[rr][1] = nc[rr][1];
      cs[rr] = ns[rr];
      cb[rr] = nb[rr];
    }
    if (kt + 1 < KT) fetch(kt + 1);
    if (kt >= kPStages && !mbar_wait(&sm.empty[s], (use - 1) & 1u)) {
      ok = false;
      break;
    }
    if (tid == 0) {
      mbar_expect_tx(&sm.full[s], kATileBytes);
      tma_load_2d(sm.a[s], &xmap, kt * kPBK, m0, &sm.full[s]);
    }
    // dequantize: float(q) from the bits 0x4B000000 | q minus 2^23 (exact),
    // w = fma(scale, q, bias); w_hi = bf16(w), w_lo = bf16(w - w_hi)
#pragma unroll
    for (int rr = 0; rr < RPT; ++rr) {
      const int r = tid + rr * kPThreads;
      const float sc = sb<SD>(cs[rr]), bi = sb<SD>(cb[rr]);
      const uint32_t words[8] = {cc[rr][0].x, cc[rr][0].y, cc[rr][0].z, cc[rr][0].w,
                                 cc[rr][1].x, cc[rr][1].y, cc[rr][1].z, cc[rr][1].w};
      uint8_t* brow = sm.b[s] + r * 128;
      uint8_t* brow2 = sm.b2[s] + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {  // word c = elements 8c .. 8c+7 = one 16-byte chunk
        uint32_t p[4], p2[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float q0 = __fsub_rn(__uint_as_float(((words[c] >> (8 * j)) & 15u) | 0x4B000000u), 8388608.0f);
          const float q1 = __fsub_rn(__uint_as_float(((words[c] >> (8 * j + 4)) & 15u) | 0x4B000000u), 8388608.0f);
          const float w0 = __fmaf_rn(sc, q0, bi), w1 = __fmaf_rn(sc, q1, bi);
          const __nv_bfloat162 v = __floats2bfloat162_rn(w0, w1);
          p[j] = *reinterpret_cast<const uint32_t*>(&v);
          const __nv_bfloat162 v2 = __floats2bfloat162_rn(__fsub_rn(w0, __uint_as_float(p[j] << 16)),
                                                          __fsub_rn(w1, __uint_as_float(p[j] & 0xFFFF0000u)));
          p2[j] = *reinterpret_cast<const uint32_t*>(&v2);
        }
        *reinterpret_cast<uint4*>(brow + ((c ^ (r & 7)) << 4)) = make_uint4(p[0], p[1], p[2], p[3]);
        *reinterpret_cast<uint4*>(brow2 + ((c ^ (r & 7)) << 4)) = make_uint4(p2[0], p2[1], p2[2], p2[3]);
      }
    }
    fence_proxy_async_smem();  // the tensor core reads these writes through the async proxy
    mbar_arrive_cta(&sm.full[s]);
    if (tid == 0) {
      if (!mbar_wait(&sm.full[s], use & 1u)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t a0 = smem_addr(sm.a[s]), b0 = smem_addr(sm.b[s]), b1 = smem_addr(sm.b2[s]);
#pragma unroll
      for (int ks = 0; ks < kPBK / 16; ++ks) {
        umma_bf16(tmem, sw128_desc(a0 + ks * 32), sw128_desc(b0 + ks * 32), (kt | ks) != 0);
        umma_bf16(tmem, sw128_desc(a0 + ks * 32), sw128_desc(b1 + ks * 32), 1u);
      }
      umma_commit(&sm.empty[s]);
      ++issued;
    }
  }
  // the accumulator is complete once every issued MMA has finished
  if (tid == 0) umma_commit(&sm.done);
  const bool done = mbar_wait(&sm.done, 0);
  tc_fence_after();
  ok = __syncthreads_and(ok && done && (tid != 0 || issued == KT));
  if (ok) {
    // warp w reads TMEM lanes 32 (w % 4) .. +31 (its lane quarter) and the
    // column half w / 4
    const int quarter = warp & 3, half = warp >> 2;
    const int row = m0 + quarter * 32 + lane;
#pragma unroll 1
    for (int c = half * (kPBN / 64); c < (half + 1) * (kPBN / 64); ++c) {
      uint32_t r[32];
      tmem_ld32(tmem + (uint32_t(quarter * 32) << 16) + uint32_t(c * 32), r);
      if (row < T && quarter * 32 + lane < mrows) {
        uint4* dst = reinterpret_cast<uint4*>(y + size_t(row) * N + n0 + c * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j)
            o[j] = uint32_t(to_bf(__uint_as_float(r[8 * q + 2 * j]))) |
                   (uint32_t(to_bf(__uint_as_float(r[8 * q + 2 * j + 1]))) << 16);
          dst[q] = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
  } else if (tid == 0) {
    report(status, kStatusBulkTimeout);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

bool valid_qmat3(const RecQMat& m) {
  return m.w && m.scales && m.biases && aligned16(m.w) && aligned16(m.scales) && aligned16(m.biases);
}

EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  }
  return fn;
}

template <int SD>
cudaError_t launch_prefill(const CUtensorMap& map, const QMatDev& w, int K, int N, int T, uint16_t* y, int* status,
                           cudaStream_t st, const int4* tiles = nullptr, int n_tiles = 0) {
  const size_t smem = sizeof(PrefillSmem) + 1024;
  cudaError_t e = cudaFuncSetAttribute(k_prefill_gemm<SD>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  dim3 grid(N / kPBN, tiles ? n_tiles : (T + kPBM - 1) / kPBM);
  k_prefill_gemm<SD><<<grid, kPThreads, smem, st>>>(map, w, K, N, T, y, status, tiles);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// MoE block of a prefill chunk: the (token, rank) pairs of the routing are
// grouped by expert, each expert's rows multiply its gate / up / down
// matrices in one grouped GEMM launch each, and the expert outputs are mixed
// per token in rank order (the decode path's bf16 rounding points).
// ---------------------------------------------------------------------------
constexpr int kMoeThreads = 256;

__global__ void k_moe_count(const int* __restrict__ ids, int n_pairs, int E, int* counts, int* status) {
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < n_pairs; p += gridDim.x * blockDim.x) {
    const int e = ids[p];
    if (e < 0 || e >= E) {
      report(status, kStatusBadToken);
      continue;
    }
    atomicAdd(&counts[e], 1);
  }
}

// Offsets of the experts' row groups, the grouped GEMMs' tile table (rows
// 128 at a time inside each group; unused entries have 0 rows) and zeroed
// cursors.  One thread: E and the tile count are small.
__global__ void k_moe_plan(const int* __restrict__ counts, int E, int* off, int* cursor, int4* tiles,
                           int n_tiles_max) {
  if (threadIdx.x != 0) return;
  int o = 0, ti = 0;
  for (int e = 0; e < E; ++e) {
    const int n = counts[e];
    off[e] = o;
    cursor[e] = 0;
    for (int m = 0; m < n && ti < n_tiles_max; m += kPBM) tiles[ti++] = make_int4(e, o + m, min(kPBM, n - m), 0);
    o += n;
  }
  for (; ti < n_tiles_max; ++ti) tiles[ti] = make_int4(0, 0, 0, 0);
}

// One warp per pair (t, r): its slot in expert e's group (the order inside a
// group does not change any result) and the copy of x row t there.
__global__ void k_moe_gather(const int* __restrict__ ids, int n_pairs, int k, int E, const uint16_t* __restrict__ x,
                             int H, const int* __restrict__ off, int* cursor, int* pos, uint16_t* __restrict__ xg) {
  const int lane = threadIdx.x & 31;
  const int nw = gridDim.x * (blockDim.x >> 5);
  for (int p = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; p < n_pairs; p += nw) {
    const int e = ids[p];
    int slot = -1;
    if (lane == 0 && e >= 0 && e < E) slot = off[e] + atomicAdd(&cursor[e], 1);
    slot = __shfl_sync(0xffffffffu, slot, 0);
    if (lane == 0) pos[p] = slot;
    if (slot < 0) continue;
    const uint4* src = reinterpret_cast<const uint4*>(x + size_t(p / k) * H);
    uint4* dst = reinterpret_cast<uint4*>(xg + size_t(slot) * H);
    for (int i = lane; i < H / 8; i += 32) dst[i] = ldg128(src + i);
  }
}

// act = bf16(bf16(g * bf16(sigmoid(g))) * u), in place over g (as the decode
// path's gate/up epilogue).
__global__ void k_moe_swiglu(uint16_t* __restrict__ g, const uint16_t* __restrict__ u, size_t n) {
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    const float gg = bf(g[i]), uu = bf(u[i]);
    g[i] = to_bf(__fmul_rn(rbf(__fmul_rn(gg, rbf(rsigmoid(gg)))), uu));
  }
}

// y[t] = (resid[t] +) the pairs' outputs d * bf16(w) summed in rank order
// with a bf16 rounding after each add (the decode path's mix).
__global__ void k_moe_mix(const uint16_t* __restrict__ d, const int* __restrict__ pos, const float* __restrict__ wts,
                          int T, int k, int H, const uint16_t* __restrict__ resid, uint16_t* __restrict__ y) {
  const size_t n = size_t(T) * H;
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
    const int t = int(i / H), h = int(i % H);
    float mix = 0.0f;
    bool first = true;
    for (int r = 0; r < k; ++r) {
      const int slot = pos[size_t(t) * k + r];
      if (slot < 0) continue;
      const float term = __fadd_rn(rbf(__fmul_rn(bf(d[size_t(slot) * H + h]), rbf(wts[size_t(t) * k + r]))), 0.0f);
      mix = first ? term : rbf(__fadd_rn(term, mix));
      first = false;
    }
    y[i] = resid ? to_bf(__fadd_rn(bf(resid[i]), mix)) : to_bf(mix);
  }
}

struct MoeLayout {
  size_t counts, cursor, off, tiles, pos, xg, g, u, d, total;
  int n_tiles_max;
};
MoeLayout moe_layout(int64_t T, int k, int H, int I, int E) {
  MoeLayout L;
  const int64_t P = T * k;
  L.n_tiles_max = int((P + kPBM - 1) / kPBM) + E;
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = (o + bytes + 255) / 256 * 256;
    return at;
  };
  L.counts = take(size_t(E) * 4);
  L.cursor = take(size_t(E) * 4);
  L.off = take(size_t(E) * 4);
  L.tiles = take(size_t(L.n_tiles_max) * 16);
  L.pos = take(size_t(P) * 4);
  L.xg = take(size_t(P) * H * 2);
  L.g = take(size_t(P) * I * 2);
  L.u = take(size_t(P) * I * 2);
  L.d = take(size_t(P) * H * 2);
  L.total = o;
  return L;
}

int encode_rows(CUtensorMap* map, const void* base, int64_t rows, int cols) {
  EncodeTiled enc = encode_fn();
  if (!enc) return -1;
  const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(cols) * 2};
  const cuuint32_t box[2] = {kPBK, kPBM};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? 0
             : -1;
}

}  // namespace
}  // namespace rec

using namespace rec;

REC_API size_t rec_prefill_moe_workspace_bytes(int64_t t, int32_t k, int32_t hidden, int32_t inter,
                                               int32_t n_experts) {
  if (t <= 0 || k <= 0 || hidden <= 0 || inter <= 0 || n_experts <= 0) return 0;
  return moe_layout(t, k, hidden, inter, n_experts).total;
}

REC_API int rec_prefill_moe(const RecQMat* gate, const RecQMat* up, const RecQMat* down, int32_t scale_dtype,
                            int32_t n_experts, int32_t inter, int32_t hidden, const void* x_dev, int64_t t,
                            int32_t k, const int32_t* ids_dev, const float* weights_dev, const void* resid_dev,
                            void* y_dev, void* workspace, size_t workspace_bytes, int32_t* status_dev, void* stream) {
  REC_CHECK_ARG(gate && up && down && x_dev && ids_dev && weights_dev && y_dev && workspace && status_dev,
                "rec_prefill_moe: null pointer");
  REC_CHECK_ARG(valid_qmat3(*gate) && valid_qmat3(*up) && valid_qmat3(*down),
                "rec_prefill_moe: expert matrices must be non-null and 16-byte aligned");
  REC_CHECK_ARG(scale_dtype == REC_SCALE_FP16 || scale_dtype == REC_SCALE_BF16, "bad scale dtype");
  REC_CHECK_ARG(n_experts > 0 && n_experts <= 4096, "rec_prefill_moe: n_experts %d outside 1..4096", n_experts);
  REC_CHECK_ARG(k >= 1 && k <= 16 && k <= n_experts, "rec_prefill_moe: k %d outside 1..min(16, n_experts)", k);
  REC_CHECK_ARG(hidden % kPBN == 0 && inter % kPBN == 0,
                "rec_prefill_moe: hidden %d and inter %d must be multiples of %d", hidden, inter, kPBN);
  REC_CHECK_ARG(t > 0 && t * k < (1ll << 31), "rec_prefill_moe: bad token count");
  REC_CHECK_ARG(aligned16(x_dev) && aligned16(y_dev) && (!resid_dev || aligned16(resid_dev)) &&
                    (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
                "rec_prefill_moe: x, y, resid 16-byte and workspace 256-byte aligned");
  const MoeLayout L = moe_layout(t, k, hidden, inter, n_experts);
  REC_CHECK_ARG(workspace_bytes >= L.total, "rec_prefill_moe: workspace %zu < %zu bytes", workspace_bytes, L.total);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int* counts = reinterpret_cast<int*>(ws + L.counts);
  int* cursor = reinterpret_cast<int*>(ws + L.cursor);
  int* off = reinterpret_cast<int*>(ws + L.off);
  int4* tiles = reinterpret_cast<int4*>(ws + L.tiles);
  int* pos = reinterpret_cast<int*>(ws + L.pos);
  uint16_t* xg = reinterpret_cast<uint16_t*>(ws + L.xg);
  uint16_t* g = reinterpret_cast<uint16_t*>(ws + L.g);
  uint16_t* u = reinterpret_cast<uint16_t*>(ws + L.u);
  uint16_t* d = reinterpret_cast<uint16_t*>(ws + L.d);
  const int P = int(t * k);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap xmap, amap;
  REC_CHECK_ARG(encode_rows(&xmap, xg, P, hidden) == 0 && encode_rows(&amap, g, P, inter) == 0,
                "rec_prefill_moe: tensor map encoding failed");
  const int blocks = 4 * sm_count();
  REC_CHECK_CUDA(cudaMemsetAsync(counts, 0, size_t(n_experts) * 4, st));
  k_moe_count<<<blocks, kMoeThreads, 0, st>>>(ids_dev, P, n_experts, counts, status_dev);
  k_moe_plan<<<1, 32, 0, st>>>(counts, n_experts, off, cursor, tiles, L.n_tiles_max);
  k_moe_gather<<<blocks, kMoeThreads, 0, st>>>(ids_dev, P, k, n_experts, static_cast<const uint16_t*>(x_dev), hidden,
                                               off, cursor, pos, xg);
  REC_CHECK_CUDA(cudaGetLastError());
  const QMatDev wg = {static_cast<const uint32_t*>(gate->w), static_cast<const uint16_t*>(gate->scales),
                      static_cast<const uint16_t*>(gate->biases)};
  const QMatDev wu = {static_cast<const uint32_t*>(up->w), static_cast<const uint16_t*>(up->scales),
                      static_cast<const uint16_t*>(up->biases)};
  const QMatDev wd = {static_cast<const uint32_t*>(down->w), static_cast<const uint16_t*>(down->scales),
                      static_cast<const uint16_t*>(down->biases)};
  auto gemm = [&](const CUtensorMap& m, const QMatDev& w, int K, int N, uint16_t* out) {
    return scale_dtype == REC_SCALE_FP16 ? launch_prefill<0>(m, w, K, N, P, out, status_dev, st, tiles, L.n_tiles_max)
                                         : launch_prefill<1>(m, w, K, N, P, out, status_dev, st, tiles, L.n_tiles_max);
  };
  REC_CHECK_CUDA(gemm(xmap, wg, hidden, inter, g));
  REC_CHECK_CUDA(gemm(xmap, wu, hidden, inter, u));
  k_moe_swiglu<<<blocks, kMoeThreads, 0, st>>>(g, u, size_t(P) * inter);
  REC_CHECK_CUDA(cudaGetLastError());
  REC_CHECK_CUDA(gemm(amap, wd, inter, hidden, d));
  k_moe_mix<<<blocks, kMoeThreads, 0, st>>>(d, pos, weights_dev, int(t), k, hidden,
                                            static_cast<const uint16_t*>(resid_dev), static_cast<uint16_t*>(y_dev));
  REC_CHECK_CUDA(cudaGetLastError());
  return REC_OK;
}

REC_API int rec_prefill_gemm(const RecQMat* w, int32_t scale_dtype, int64_t n, int32_t k, const void* x_dev,
                             int64_t t, void* y_dev, int32_t* status_dev, void* stream) {
  REC_CHECK_ARG(w && w->w && w->scales && w->biases && x_dev && y_dev && status_dev, "rec_prefill_gemm: null pointer");
  REC_CHECK_ARG(n > 0 && n % kPBN == 0 && n < (1ll << 30), "rec_prefill_gemm: N=%lld must be a multiple of %d",
                (long long)n, kPBN);
  REC_CHECK_ARG(k >= kPBK && k % kPBK == 0, "rec_prefill_gemm: K=%d must be a positive multiple of %d", k, kPBK);
  REC_CHECK_ARG(t > 0 && t < (1ll << 31), "rec_prefill_gemm: bad token count");
  REC_CHECK_ARG(aligned16(x_dev) && aligned16(y_dev) && aligned16(w->w), "rec_prefill_gemm: buffers must be 16-byte aligned");
  REC_CHECK_ARG(scale_dtype == REC_SCALE_FP16 || scale_dtype == REC_SCALE_BF16, "bad scale dtype");
  EncodeTiled enc = encode_fn();
  REC_CHECK_ARG(enc, "rec_prefill_gemm: cuTensorMapEncodeTiled is unavailable");
  CUtensorMap map;
  const cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(t)};
  const cuuint64_t strides[1] = {cuuint64_t(k) * 2};
  const cuuint32_t box[2] = {kPBK, kPBM};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x_dev), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  REC_CHECK_ARG(r == CUDA_SUCCESS, "rec_prefill_gemm: tensor map encoding failed (%d)", int(r));
  const QMatDev wd = {static_cast<const uint32_t*>(w->w), static_cast<const uint16_t*>(w->scales),
                      static_cast<const uint16_t*>(w->biases)};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = scale_dtype == REC_SCALE_FP16
                      ? launch_prefill<0>(map, wd, k, int(n), int(t), static_cast<uint16_t*>(y_dev), status_dev, st)
                      : launch_prefill<1>(map, wd, k, int(n), int(t), static_cast<uint16_t*>(y_dev), status_dev, st);
  REC_CHECK_CUDA(e);
  return REC_OK;
}
