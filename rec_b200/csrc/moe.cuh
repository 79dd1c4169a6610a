// MoE block kernels: router (RMSNorm + bf16 logits + selection), expert
// gate/up GEMV with fused SwiGLU, expert down GEMV with the fused bf16 mix
// and residual.
//
// Reference: engine/src/rec_mlx/model.py:227-254 (Router, SparseMoeBlock),
// megakernel.py:406-435,696-725 (router dot, top-k), rank_routing.py:12-32
// (lowest index wins ties), megakernel.py:747-798 (expert gate/up/down),
// megakernel.py:944-969 + mixed_bits.py:32-54 (bf16 logits, bf16 mix).
#pragma once
#include "gemv.cuh"
#include "xch.cuh"

namespace rec {

constexpr int kMaxExperts = 1024;
constexpr int kMaxTopK = 8;

// --- router ---------------------------------------------------------------
struct RouterArgs {
  const uint16_t* h;       // bf16 [H] residual
  const uint16_t* norm_w;  // post-attention RMSNorm weight
  float eps;
  const uint16_t* w;       // bf16 [E, H]
  const float* expert_bias;
  int E, k, mode;
  float* logits;           // [E]
  uint16_t* xn_out;        // [H]
  int* ids;                // [k]
  float* wts;              // [k]
  unsigned* counter;
  int* status;
  int pdl;
  int norm_only;           // a dense-MLP layer: only the RMSNorm into xn_out (one CTA), no routing
};

template <int H>
struct RouterSmem {
  alignas(16) uint16_t xn[H];
  float red[40];
  float p[kMaxExperts];
  float choice[kMaxExperts];
  int is_last;
};

// Order-preserving key of a float (+0 and -0 canonicalised first); NaN gets
// key 1, below every number, so it is chosen last (lowest index among NaNs).
__device__ __forceinline__ unsigned route_key(float x) {
  const unsigned u = __float_as_uint(__fadd_rn(x, 0.0f));
  if ((u & 0x7fffffffu) > 0x7f800000u) return 1u;  // NaN ranks below every number (and -inf)
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Canonical router logit: lane l owns 8-element chunks l, l+32, ...; fused
// multiply-adds in order; butterfly; rounded to bf16 (mixed_bits.py:32-38).
template <int H>
__global__ void __launch_bounds__(kThreads) k_router(const RouterArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  RouterSmem<H>& sm = *reinterpret_cast<RouterSmem<H>*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int CH = H / 256;
  const int e = blockIdx.x * kWarps + warp;
  uint4 wv[CH];
  if (e < a.E) {
#pragma unroll
    for (int m = 0; m < CH; ++m) wv[m] = ldg128_nc(a.w + size_t(e) * H + (lane + 32 * m) * 8);
  }
  if (a.pdl) grid_wait();
  grid_launch_dependents();
  cta_rmsnorm(a.h, a.norm_w, H, a.eps, sm.xn, sm.red);
  if (blockIdx.x == 0)
    for (int i = threadIdx.x * 8; i < H; i += kThreads * 8)
      *reinterpret_cast<uint4*>(a.xn_out + i) = *reinterpret_cast<const uint4*>(sm.xn + i);
  if (a.norm_only) return;
  if (e < a.E) {
    float acc = 0.0f;
#pragma unroll
    for (int m = 0; m < CH; ++m) {
      const uint4 xv = *reinterpret_cast<const uint4*>(sm.xn + (lane + 32 * m) * 8);
      const uint32_t ws_[4] = {wv[m].x, wv[m].y, wv[m].z, wv[m].w};
      const uint32_t xs_[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        acc = __fmaf_rn(__uint_as_float(ws_[t] << 16), __uint_as_float(xs_[t] << 16), acc);
        acc = __fmaf_rn(__uint_as_float(ws_[t] & 0xFFFF0000u), __uint_as_float(xs_[t] & 0xFFFF0000u), acc);
      }
    }
    acc = bfly_sum(acc);
    if (lane == 0) a.logits[e] = rbf(acc);
  }
  // the last CTA selects the experts
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    sm.is_last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!sm.is_last || warp != 0) return;
  __threadfence();
  const int E = a.E;
  // the logits once into shared memory (all loads in flight together)
  for (int i = lane; i < E; i += 32) sm.p[i] = __ldcg(a.logits + i);
  __syncwarp();
  // selection keys (route_key order; 0 = taken) over the choice storage
  unsigned* keys = reinterpret_cast<unsigned*>(sm.choice);
  if (a.mode == 0) {
    float mx = -INFINITY;
    for (int i = lane; i < E; i += 32) mx = fmaxf(mx, sm.p[i]);
    mx = bfly_max(mx);
    float s = 0.0f;
    for (int i = lane; i < E; i += 32) {
      const float c = rexp(__fsub_rn(sm.p[i], mx));
      sm.choice[i] = c;
      s = __fadd_rn(s, c);
    }
    s = bfly_sum(s);
    for (int i = lane; i < E; i += 32) {
      const float pi = __fdiv_rn(sm.choice[i], s);
      sm.p[i] = pi;
      keys[i] = route_key(pi);
    }
  } else {
    for (int i = lane; i < E; i += 32) {
      const float pi = rsigmoid(sm.p[i]);
      sm.p[i] = pi;
      keys[i] = route_key(__fadd_rn(pi, a.expert_bias[i]));
    }
  }
  __syncwarp();
  // k rounds of (largest choice, lowest id among equals): each lane keeps the
  // best of its own experts lane + 32 j; the warp reduces those, and only the
  // lane that owned the winner rescans its experts
  unsigned bk = 0u;
  int bi = 0;
  for (int i = lane; i < E; i += 32)
    if (keys[i] > bk) { bk = keys[i]; bi = i; }
  float s2 = 0.0f, my_p = 0.0f;
  int my_id = 0;
  for (int r = 0; r < a.k; ++r) {
    const unsigned wbest = __reduce_max_sync(0xffffffffu, bk);
    int widx = int(__reduce_min_sync(0xffffffffu, (bk == wbest && bk) ? unsigned(bi) : ~0u));
    if (unsigned(widx) >= unsigned(E)) widx = 0;  // only for NaN choices
    const float pw = sm.p[widx];
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
  if (lane < a.k) {
    a.ids[lane] = my_id;
    a.wts[lane] = __fdiv_rn(my_p, s2);
  }
  if (lane == 0) *a.counter = 0;
}

// --- expert gate/up + SwiGLU ---------------------------------------------------
struct GateUpArgs {
  QMatDev gate, up;        // stacked [E*I, H]
  const uint16_t* xn;      // bf16 [H]
  const int* ids;          // [k]
  int k, I;
  int expert_lo, expert_hi;  // experts computed here (expert parallelism)
  uint16_t* act;           // bf16 [k, I] (then the shared expert's [Is])
  // an always-on shared expert (Is > 0): its Is gate/up pairs follow the
  // routed ones as "rank k", from these matrices
  QMatDev sgate, sup;
  int Is;
  int* status;
  int pdl;
};

template <int RSP, int NS>
struct GateUpSmem {
  using L = StageLayout<2048, 2 * RSP>;
  alignas(128) uint8_t stage[NS][L::BYTES];
  alignas(16) uint16_t xn[2048];
  float red[kWarps];
  uint64_t full[NS];
};

// Row pairs (gate row i, up row i) of expert rank r form work units
// u = r*I + i; a stage holds up to RSP consecutive pairs of one rank.  A
// shared expert's pairs follow as rank k: u = k*I + i, i < Is.
struct PairCursor {
  int cur, end, I, rsp, kI, Is;
  __device__ bool next(int& r, int& i0, int& n) {
    if (cur >= end) return false;
    if (cur < kI) {
      r = cur / I;
      i0 = cur % I;
      n = min(min(rsp, end - cur), I - i0);
    } else {
      r = kI / I;
      i0 = cur - kI;
      n = min(min(rsp, end - cur), Is - i0);
    }
    cur += n;
    return true;
  }
};

// expert < 0: the shared expert (rows i0.. of its own matrices).
template <int RSP>
__device__ __forceinline__ void issue_pairs(uint8_t* stage, uint64_t* bar, const GateUpArgs& a, int expert, int i0,
                                            int n) {
  using L = StageLayout<2048, 2 * RSP>;
  constexpr int RB = KCfg<2048>::ROW_BYTES, G = KCfg<2048>::GROUPS;
  const bool sh = expert < 0;
  const QMatDev& gm = sh ? a.sgate : a.gate;
  const QMatDev& um = sh ? a.sup : a.up;
  const size_t row = sh ? size_t(i0) : size_t(expert) * a.I + i0;
  const uint32_t wb = uint32_t(n) * RB, sbytes = uint32_t(n) * G * 2;
  mbar_expect_tx(bar, 2 * wb + 4 * sbytes);
  bulk_g2s(stage, reinterpret_cast<const uint8_t*>(gm.w) + row * RB, wb, bar);
  bulk_g2s(stage + RSP * RB, reinterpret_cast<const uint8_t*>(um.w) + row * RB, wb, bar);
  uint8_t* s = stage + L::W_BYTES;
  uint8_t* b = stage + L::W_BYTES + L::S_BYTES;
  bulk_g2s(s, gm.s + row * G, sbytes, bar);
  bulk_g2s(s + RSP * G * 2, um.s + row * G, sbytes, bar);
  bulk_g2s(b, gm.b + row * G, sbytes, bar);
  bulk_g2s(b + RSP * G * 2, um.b + row * G, sbytes, bar);
}

template <int SD, int RSP, int NS>
__global__ void __launch_bounds__(kThreads, 1) k_gateup(const GateUpArgs a) {
  using S = GateUpSmem<RSP, NS>;
  using L = typename S::L;
  constexpr int K = 2048;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  S& sm = *reinterpret_cast<S*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(&sm.full[s], 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (a.pdl) grid_wait();
  grid_launch_dependents();

  int u0, u1;
  const int kI = a.k * a.I;
  split_range((kI + a.Is) / 2, gridDim.x, blockIdx.x, u0, u1);
  u0 *= 2;
  u1 *= 2;
  PairCursor prod{u0, u1, a.I, RSP, kI, a.Is}, cons{u0, u1, a.I, RSP, kI, a.Is};
  // Slot s completes one barrier phase per issued (local) stage; both sides
  // track the parity per slot, and `outstanding` (thread 0) the slots with a
  // copy in flight.
  uint32_t phase_bits = 0, outstanding = 0;
  // rank k is the shared expert (expert_of -1 - expert_lo: issue_pairs takes it by its sign)
  auto expert_of = [&](int r) { return r < a.k ? a.ids[r] : -1 + a.expert_lo; };
  auto local = [&](int r) {
    if (r >= a.k) return true;
    const int e = expert_of(r);
    return e >= a.expert_lo && e < a.expert_hi;
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      int r, i0, n;
      if (!prod.next(r, i0, n)) break;
      if (local(r)) {
        issue_pairs<RSP>(sm.stage[s], &sm.full[s], a, expert_of(r) - a.expert_lo, i0, n);
        outstanding |= 1u << s;
      }
    }
  }
  for (int i = threadIdx.x * 8; i < K; i += kThreads * 8)
    *reinterpret_cast<uint4*>(sm.xn + i) = ldg128(a.xn + i);
  __syncthreads();
  const FixScale fs = fix_scale_from_max(block_maxabs(sm.xn, K, threadIdx.x, kThreads, sm.red, 0));
  GroupX gx[1];
  prep_lane_x<K>(sm.xn, fs, 0, lane, gx);

  bool failed = false;
  int j = 0, r, i0, n;
  while (cons.next(r, i0, n)) {
    const int slot = j % NS;
    const bool here = local(r);
    if (here) {
      if (mbar_wait(&sm.full[slot], (phase_bits >> slot) & 1u)) {
        phase_bits ^= 1u << slot;
        outstanding &= ~(1u << slot);
      } else {
        failed = true;
      }
    }
    if (here && !failed) {
      const uint8_t* st = sm.stage[slot];
      const uint8_t* wbase = stage_wrow<K, 2 * RSP>(st, 0);
      const uint16_t* sbase = stage_srow<K, 2 * RSP>(st, 0);
      const uint16_t* bbase = stage_brow<K, 2 * RSP>(st, 0);
      // each warp: 2 pairs per pass (ILP 4 rows: g0, u0, g1, u1)
      for (int pb = 0; pb < n; pb += 2 * kWarps) {
        const int pa = pb + warp, pc = pb + kWarps + warp;
        const bool va = pa < n, vc = pc < n;
        int rows[4] = {va ? pa : 0, va ? RSP + pa : 0, vc ? pc : 0, vc ? RSP + pc : 0};
        float v[4];
        lane_rows_partial<K, SD, 4>(wbase, sbase, bbase, rows, 0, lane, gx, v);
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = __fmul_rn(bfly_sum(v[q]), fs.down);
        // lanes 0 and 1 finish pairs pa and pc side by side (the sums are
        // on every lane after the butterflies)
        if (lane < 2 && (lane == 0 ? va : vc)) {
          const float g = rbf(lane == 0 ? v[0] : v[2]), u = rbf(lane == 0 ? v[1] : v[3]);
          const float sig = rbf(rsigmoid(g));
          a.act[r * a.I + i0 + (lane == 0 ? pa : pc)] = to_bf(__fmul_rn(rbf(__fmul_rn(g, sig)), u));
        }
      }
    }
    if (__syncthreads_or(failed)) {
      failed = true;
      break;
    }
    if (threadIdx.x == 0) {
      int r2, i2, n2;
      if (prod.next(r2, i2, n2) && local(r2)) {
        issue_pairs<RSP>(sm.stage[slot], &sm.full[slot], a, expert_of(r2) - a.expert_lo, i2, n2);
        outstanding |= 1u << slot;
      }
    }
    ++j;
  }
  if (failed && threadIdx.x == 0) {
    report(a.status, kStatusBulkTimeout);
    // wait (bounded) for the copies still in flight into this CTA
    for (int s = 0; s < NS; ++s)
      if (outstanding & (1u << s)) mbar_wait(&sm.full[s], (phase_bits >> s) & 1u);
  }
}

// --- expert down + bf16 mix + residual -----------------------------------------
struct DownArgs {
  QMatDev down;            // stacked [E*H, I]
  const uint16_t* act;     // bf16 [k, I]
  const int* ids;
  const float* wts;
  int k, H;
  int expert_lo, expert_hi;
  uint16_t* h;             // residual (mix mode)
  uint16_t* trace_row;     // bf16 [H] copy of the new residual, or null
  uint16_t* dout;          // expert-parallel mode: bf16 [k, H] expert outputs (local ranks only)
  // the shared expert's output bf16 [H] (Flint MoE layers), or null: added to
  // the routed mix as mlp = bf16(mix + shared) before the residual
  // (megakernel.py:955-958)
  const uint16_t* shared_out;
  // or computed here (k_down<I, SD, IS> with IS > 0): the shared expert's down
  // matrix [H, IS]; its activations follow the routed ones in act (k * I on)
  QMatDev sdown;
  int* status;
  int pdl;
  // a session split over ranks (world > 1): the local experts' outputs go
  // into every rank's exchange buffer, then each CTA mixes its rows of all k
  // slots in rank order once every rank has delivered them
  int world, rank, layer, n_layers;
  const int* seq;          // steps completed (device counter): exchange parity
  uint8_t* xch[kMaxWorld];
  XchLayout xl;
};

template <int I>
struct DownSmem {
  static constexpr int RMAX = 16;  // output rows per CTA (H / grid rounded up to even)
  using L = StageLayout<I, RMAX>;
  alignas(128) uint8_t stage[kMaxTopK][L::BYTES];
  alignas(16) uint16_t act[kMaxTopK][I];
  float d[kMaxTopK][RMAX];
  uint64_t bar;
};
// The shared expert's part (k_down<I, SD, IS>), after DownSmem<I> in shared memory.
template <int IS>
struct DownSharedSmem {
  using L = StageLayout<IS, DownSmem<256>::RMAX>;
  alignas(128) uint8_t stage[L::BYTES];
  alignas(16) uint16_t act[IS];
  float d[DownSmem<256>::RMAX];
};
template <int I, int IS>
constexpr size_t down_smem_bytes() {
  return IS ? (sizeof(DownSmem<I>) + 127) / 128 * 128 + sizeof(DownSharedSmem<IS ? IS : 256>) : sizeof(DownSmem<I>);
}

// One warp: rows [0, n) of a stage of K-wide down rows (8 rows per pass, 4
// lanes per row) against activations x, into d[row] = bf16(row dot).
template <int K, int SD, int RMAX>
__device__ __forceinline__ void down_rows(const uint8_t* st, const uint16_t* x, int n, float* d) {
  using C = KCfg<K>;
  const int lane = threadIdx.x & 31;
  const FixScale fs = fix_scale_from_max(warp_maxabs(x, K));
  GroupX gx[C::GPL];
  const int sub = lane >> 2, l = lane & 3;
  prep_lane_x<K>(x, fs, 0, l, gx);
  for (int rb = 0; rb < n; rb += 16) {
    int rows[2];
    bool valid[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int rr = rb + 8 * q + sub;
      valid[q] = rr < n;
      rows[q] = valid[q] ? rr : 0;
    }
    float v[2];
    lane_rows_partial<K, SD, 2>(stage_wrow<K, RMAX>(st, 0), stage_srow<K, RMAX>(st, 0), stage_brow<K, RMAX>(st, 0),
                                rows, 0, l, gx, v);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      v[q] = bfly_sum<4>(valid[q] ? v[q] : 0.0f);
      if (valid[q] && l == 0) d[rows[q]] = rbf(__fmul_rn(v[q], fs.down));
    }
  }
}

// Mix mode (single device): every CTA owns output rows [i0, i1) and computes
// them for all k experts (warp r = rank r), then mixes in rank order:
// m = bf16(d_0*bf16(w_0)) + 0; m = bf16(bf16(d_r*bf16(w_r)) + 0 + m);
// with a shared expert m = bf16(m + shared); h = bf16(h + m).  IS > 0: the
// shared expert's down rows (K = IS) are computed here by warp k (k < 8),
// from a.sdown and the activations at act + k * I.
template <int I, int SD, int IS = 0>
__global__ void __launch_bounds__(kThreads, 1) k_down(const DownArgs a) {
  using S = DownSmem<I>;
  using L = typename S::L;
  using C = KCfg<I>;
  static_assert(!C::wide, "down projection expects a narrow K");
  extern __shared__ __align__(128) uint8_t smem_raw[];
  S& sm = *reinterpret_cast<S*>(smem_raw);
  using SS = DownSharedSmem<IS ? IS : 256>;
  using CS = KCfg<IS ? IS : 256>;
  SS& ss = *reinterpret_cast<SS*>(smem_raw + (sizeof(S) + 127) / 128 * 128);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int i0, i1;
  split_range(a.H / 2, gridDim.x, blockIdx.x, i0, i1);
  i0 *= 2;
  i1 *= 2;
  const int n = i1 - i0;
  if (threadIdx.x == 0) {
    mbar_init(&sm.bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  // ids were written two kernels earlier (the router); the weights of the
  // selected experts can stream in before this kernel's inputs are ready.
  auto local = [&](int r) { const int e = a.ids[r]; return e >= a.expert_lo && e < a.expert_hi; };
  if (threadIdx.x == 0 && n > 0) {
    uint32_t total = 0;
    for (int r = 0; r < a.k; ++r)
      if (local(r)) total += uint32_t(n) * (C::ROW_BYTES + 2 * C::GROUPS * 2);
    if constexpr (IS > 0) total += uint32_t(n) * (CS::ROW_BYTES + 2 * CS::GROUPS * 2);
    mbar_expect_tx(&sm.bar, total);
    if constexpr (IS > 0) {
      using LS = typename SS::L;
      const size_t row = size_t(i0);
      bulk_g2s(ss.stage, reinterpret_cast<const uint8_t*>(a.sdown.w) + row * CS::ROW_BYTES, n * CS::ROW_BYTES,
               &sm.bar);
      bulk_g2s(ss.stage + LS::W_BYTES, a.sdown.s + row * CS::GROUPS, n * CS::GROUPS * 2, &sm.bar);
      bulk_g2s(ss.stage + LS::W_BYTES + LS::S_BYTES, a.sdown.b + row * CS::GROUPS, n * CS::GROUPS * 2, &sm.bar);
    }
    for (int r = 0; r < a.k; ++r) {
      if (!local(r)) continue;
      const size_t row = size_t(a.ids[r] - a.expert_lo) * a.H + i0;
      bulk_g2s(sm.stage[r], reinterpret_cast<const uint8_t*>(a.down.w) + row * C::ROW_BYTES, n * C::ROW_BYTES, &sm.bar);
      bulk_g2s(sm.stage[r] + L::W_BYTES, a.down.s + row * C::GROUPS, n * C::GROUPS * 2, &sm.bar);
      bulk_g2s(sm.stage[r] + L::W_BYTES + L::S_BYTES, a.down.b + row * C::GROUPS, n * C::GROUPS * 2, &sm.bar);
    }
  }
  if (a.pdl) grid_wait();
  grid_launch_dependents();
  for (int i = threadIdx.x * 8; i < a.k * I; i += kThreads * 8)
    *reinterpret_cast<uint4*>(&sm.act[0][0] + i) = ldg128(a.act + i);
  if constexpr (IS > 0)
    for (int i = threadIdx.x * 8; i < IS; i += kThreads * 8)
      *reinterpret_cast<uint4*>(ss.act + i) = ldg128(a.act + a.k * I + i);
  __syncthreads();
  bool ok = n == 0 || mbar_wait(&sm.bar, 0);
  if (!__syncthreads_and(ok)) {
    if (threadIdx.x == 0) {
      report(a.status, kStatusBulkTimeout);
      mbar_wait(&sm.bar, 0);
    }
    return;
  }
  const int r = warp;
  if (r < a.k && local(r)) down_rows<I, SD, S::RMAX>(sm.stage[r], sm.act[r], n, sm.d[r]);
  if constexpr (IS > 0)
    if (r == a.k) down_rows<IS, SD, S::RMAX>(ss.stage, ss.act, n, ss.d);
  __syncthreads();
  if (a.dout) {
    for (int t = threadIdx.x; t < a.k * n; t += kThreads) {
      const int rr = t / n, i = t % n;
      if (local(rr)) a.dout[rr * a.H + i0 + i] = to_bf(sm.d[rr][i]);
    }
    return;
  }
  if (a.world > 1) {
    // rows [i0, i1) of the local slots to every rank (this one included) as
    // bf16 pairs (n and i0 are even); after the CTA barrier one thread fences
    // at system scope (cumulative over the CTA's stores) and raises each
    // rank's counter for this CTA's rows; then wait (bounded) for all ranks'
    // rows and mix them from this rank's buffer, the single-GPU mix order
    const int par = int((unsigned(*a.seq) * unsigned(a.n_layers) + unsigned(a.layer)) & 1u);
    const int n2 = n / 2;
    for (int q = 0; q < a.world; ++q)
      for (int t = threadIdx.x; t < a.k * n2; t += kThreads) {
        const int rr = t / n2, i = 2 * (t % n2);
        if (local(rr))
          *reinterpret_cast<uint32_t*>(xch_xd(a.xch[q], a.xl, par, rr) + i0 + i) =
              uint32_t(to_bf(sm.d[rr][i])) | (uint32_t(to_bf(sm.d[rr][i + 1])) << 16);
      }
    __syncthreads();
    __shared__ int xok;
    unsigned* cnt = xch_xcnt(a.xch[a.rank], a.xl, par, blockIdx.x);
    if (threadIdx.x == 0) {
      __threadfence_system();
      for (int q = 0; q < a.world; ++q) atomicAdd_system(xch_xcnt(a.xch[q], a.xl, par, blockIdx.x), 1u);
      int ok = 1;
      uint32_t spins = 0;
      while (ld_acquire_sys_u32(cnt) < unsigned(a.world)) {
        if (++spins > kPeerSpinLimit) {
          report(a.status, kStatusCounterTimeout);
          ok = 0;
          break;
        }
      }
      xok = ok;
    }
    __syncthreads();
    if (!xok) return;
    const uint8_t* own = a.xch[a.rank];
    for (int i = threadIdx.x; i < n; i += kThreads) {
      float m = 0.0f;
      for (int rr = 0; rr < a.k; ++rr) {
        const float d = bf(__ldcg(reinterpret_cast<const unsigned short*>(
            xch_xd(const_cast<uint8_t*>(own), a.xl, par, rr) + i0 + i)));
        const float t = __fadd_rn(rbf(__fmul_rn(d, rbf(a.wts[rr]))), 0.0f);
        m = rr == 0 ? t : rbf(__fadd_rn(t, m));
      }
      const uint16_t hn = to_bf(__fadd_rn(bf(a.h[i0 + i]), m));
      a.h[i0 + i] = hn;
      if (a.trace_row) a.trace_row[i0 + i] = hn;
    }
    __syncthreads();
    if (threadIdx.x == 0) *reinterpret_cast<volatile unsigned*>(cnt) = 0u;
    return;
  }
  for (int i = threadIdx.x; i < n; i += kThreads) {
    float m = 0.0f;
    for (int rr = 0; rr < a.k; ++rr) {
      const float t = __fadd_rn(rbf(__fmul_rn(sm.d[rr][i], rbf(a.wts[rr]))), 0.0f);
      m = rr == 0 ? t : rbf(__fadd_rn(t, m));
    }
    if (a.shared_out) m = rbf(__fadd_rn(m, bf(a.shared_out[i0 + i])));
    if constexpr (IS > 0) m = rbf(__fadd_rn(m, ss.d[i]));
    const uint16_t hn = to_bf(__fadd_rn(bf(a.h[i0 + i]), m));
    a.h[i0 + i] = hn;
    if (a.trace_row) a.trace_row[i0 + i] = hn;
  }
}

// Expert-parallel mix: gathered expert outputs dg [ranks, k, H] (each rank
// row valid only for the experts it owns) are mixed in rank order.
struct MixArgs {
  const uint16_t* dg;
  const int* ids;
  const float* wts;
  int k, H, world;
  int experts_per_rank;
  uint16_t* h;
  uint16_t* trace_row;
  int pdl;
};

static __global__ void __launch_bounds__(kThreads) k_mix(const MixArgs a) {
  if (a.pdl) grid_wait();
  grid_launch_dependents();
  for (int i = blockIdx.x * kThreads + threadIdx.x; i < a.H; i += gridDim.x * kThreads) {
    float m = 0.0f;
    for (int r = 0; r < a.k; ++r) {
      const int owner = a.ids[r] / a.experts_per_rank;
      const float d = bf(a.dg[(size_t(owner) * a.k + r) * a.H + i]);
      const float t = __fadd_rn(rbf(__fmul_rn(d, rbf(a.wts[r]))), 0.0f);
      m = r == 0 ? t : rbf(__fadd_rn(t, m));
    }
    const uint16_t hn = to_bf(__fadd_rn(bf(a.h[i]), m));
    a.h[i] = hn;
    if (a.trace_row) a.trace_row[i] = hn;
  }
}

}  // namespace rec
