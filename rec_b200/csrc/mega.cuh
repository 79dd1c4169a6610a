// Persistent decode kernel: the whole decode step (or a packet of steps) in
// one cooperative launch with one CTA per SM.
//
// Warp 0 of every CTA is a producer: it walks the step's fixed schedule of
// weight (and KV) chunks for this CTA and streams them with cp.async.bulk into
// a ring of shared-memory slots (full/empty mbarriers).  Weights do not depend
// on activations, so the producer runs ahead across phase and layer
// boundaries; only the expert chunks wait for this layer's routing, which
// the producer warp computes itself from the router logits as they land
// (flag+value words, no grid barrier before G).  Warps
// 1..8 are consumers: they take the chunks in the same order and run the same
// math as the standalone kernels (gemv.cuh, attn.cuh, moe.cuh), in the same
// canonical order, so results are bit-identical to them and to the oracle.
//
// Phases of a layer, separated by bounded software grid barriers (except
// R -> G):
//   Q  RMSNorm + QKV rows                       -> qkv
//   A  split-KV attention items (+RoPE, quantize-on-append); the last CTA to
//      finish a super-chunk / head merges it (log-sum-exp)   -> attn
//   O  O rows + residual (rows owned like D)   -> h
//   R  RMSNorm + router logits                 -> router_ll (flag + value)
//   G  expert gate/up pairs + SwiGLU (selection by each CTA's producer) -> act
//   D  expert down rows for all k experts + bf16 mix + residual -> h, trace
// then H (final RMSNorm + lm_head + CTA argmax) and E (global argmax, done
// redundantly by every CTA, so the next token needs no extra barrier).
//
// Reference counterpart: the persistent Metal megakernel
// (engine/src/rec_mlx/kernels/megakernel.py:823-975) with its spin-capped
// grid barrier (megakernel.py:137-159) and 8-token resident loop
// (resident_block.py:62-88).
#pragma once
#include "attn.cuh"
#include "moe.cuh"
#include "xch.cuh"

namespace rec {

static_assert(kXchMaxTopK == kMaxTopK, "exchange slots must cover the top-k");
constexpr int kMegaCons = 8;                        // consumer warps
constexpr int kMegaThreads = 32 * (kMegaCons + 1);  // + producer warp
constexpr int kSlotBytes = 36864;
constexpr int kSlots = 4;
constexpr int kMergeChunk = 8;  // partials per head in one merge slot (8 heads x 8 x 528 B)
constexpr int kBarCons = 1;   // named barrier: all consumer warps
constexpr int kBarTeam0 = 2;  // named barriers 2..5: warp pairs (K = 4096 rows)
constexpr int kQRows = 32;    // rows per Q / H chunk (K = 2048)
constexpr int kORows = 16;    // rows per O chunk (K = 4096)
constexpr int kGPairs = 16;   // gate/up pairs per G chunk
constexpr int kDExperts = 4;  // experts per D chunk
constexpr int kDRowsMax = 16; // output rows per CTA in O / D
constexpr int kMaxLayers = 64;  // layer descriptors kept in shared memory
constexpr int kMegaMaxExperts = 256;  // the producer warp's routing holds 8 experts per lane

struct MegaLayer {
  QMatDev q, k, v, o, gate, up, down;
  const uint16_t* input_norm;
  const uint16_t* post_norm;
  const uint16_t* router;
  const float* expert_bias;
  const uint16_t* sinks;
  const uint16_t* q_norm;
  const uint16_t* k_norm;
  uint32_t* k_codes;
  uint16_t* k_scales;
  uint16_t* k_biases;
  uint32_t* v_codes;
  uint16_t* v_scales;
  uint16_t* v_biases;
};

struct MegaArgs {
  const MegaLayer* layers;
  int n_layers, H, hq, hkv, E, k, I, V, kv_bits, router_mode, capacity, n_super_max;
  int sd;  // scale/bias type of the int4 weights: 0 fp16, 1 bf16
  float eps;
  QMatDev embed, lm_head;
  const uint16_t* final_norm;
  const float* rope;
  int* ctl;            // control block (token, position, EOS, recorded ids)
  unsigned* gbar;      // [0] grid barrier arrivals (zeroed before launch), [1] abort flag
  unsigned* cnt;       // [Hq] head counters, then [Hq * n_super_max] super counters
  uint16_t *h, *qkv, *attn, *act, *logits, *trace;
  float *partials, *supers, *router_logits, *cand_val;
  // router logits as (flag << 32 | value bits) words, [2][E] by flag parity:
  // the flag is the layer's running sequence number (route_flag), so the
  // producer warps see each logit land without a grid barrier
  unsigned long long* router_ll;
  int* cand_idx;
  int steps;
  // one session over several GPUs (world > 1): experts [e_lo, e_hi) and
  // super-chunks [super_lo, super_hi) are local; xch[q] is rank q's exchange
  // buffer (peer-mapped), laid out by XchLayout
  int world, rank, e_lo, e_hi, super_lo, super_hi, token_base;
  unsigned layer_seq0;  // layer steps run before this launch (exchange parity)
  XchLayout xl;
  uint8_t* xch[kMaxWorld];
  // kSegAll: the whole step(s).  Otherwise one segment of a step whose
  // attention runs as separate kernels (steps == 1): seg == -1 is the
  // embedding + Q of layer 0; seg == l >= 0 is O, R, G, D of layer l, then
  // Q of layer l + 1 (or H and E after the last layer)
  int seg;
  // poll bound of the grid barrier, and a CTA that skips its arrivals (-1:
  // none): the failure path's tests make the bounded wait run out with them
  unsigned bar_spin_limit;
  int skip_arrive_cta;
  unsigned long long* prof;  // optional: [barrier][cta] x (arrive, release) globaltimer stamps
  unsigned long long* prof2; // optional: [cta][64] stamps inside layer prof_layer of step 0
  int prof_layer;
};

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

struct MegaSmem {
  alignas(128) uint8_t ring[kSlots][kSlotBytes];
  MegaLayer layers[kMaxLayers];  // descriptors, copied once per launch
  alignas(16) uint16_t h0[2048];
  alignas(16) uint16_t xn[4096];
  alignas(16) uint16_t act[kMaxTopK * 1024];
  AttnScratch att;
  float red[40];
  float seg_part[kMegaCons][4];
  float best_val[kMegaCons];
  int best_idx[kMegaCons];
  float gX[kMaxTopK * 16];   // exact group sums of the shared fixed-point limbs
  float dmax[kMaxTopK];      // D: max |activation| per selected expert
  float route_p[kMegaMaxExperts];     // the producer's routing: logits, then p
  unsigned route_k[kMegaMaxExperts];  // selection keys (0 = taken)
  int ids[kMaxTopK];
  float wts[kMaxTopK];
  int loc[kMaxTopK];   // selection slots whose expert is local, in slot order
  int lids[kMaxTopK];  // their local expert indices
  int n_loc;
  int xok;             // world > 1: the expert-output exchange completed
  float dsm[kMaxTopK][kDRowsMax];
  uint64_t full[kSlots], empty[kSlots];
  uint64_t mfull;      // a short-context head group's item partials have landed
  unsigned mpar;       // its phase parity
  uint16_t hown[kDRowsMax];  // this CTA's rows of h (it owns them in embed, O and D)
  volatile int route_seq;
  volatile int merge_seq;  // 2 (step n_layers + layer) + k: consumers passed merge barrier k
  int token;
  int token0, pos0;  // starting token / position, read once at kernel entry
};

// D stages the experts' fixed-point limbs (k * I * 2 bytes) in the attention scratch.
static_assert(sizeof(decltype(AttnScratch::u)) >= kMaxTopK * 1024 * 2, "attention scratch too small for D limbs");

__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync %0, %1;" ::"r"(kBarCons), "r"(kMegaCons * 32)); }
struct ConsSync {
  __device__ void operator()() const { cons_sync(); }
};
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Data written by other CTAs during this launch is read through L2 only
// (L1 is not coherent across SMs inside one kernel).
__device__ __forceinline__ uint4 ldcg128(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ float ldcg_bf(const uint16_t* p) {
  return bf(__ldcg(reinterpret_cast<const unsigned short*>(p)));
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// 64-bit flag+value words (single-copy atomic: aligned scalar 64-bit accesses)
__device__ __forceinline__ unsigned long long ld_relaxed64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// ---------------------------------------------------------------------------
// Static partition of the step's work over CTAs (shared by both roles)
// ---------------------------------------------------------------------------
struct Part {
  int q0, q1;   // QKV rows
  int o0, o1;   // output rows of O and D (same owner)
  int g0, g1;   // gate/up pair units
};
__device__ __forceinline__ Part partition(const MegaArgs& a) {
  Part p;
  const int G = gridDim.x, c = blockIdx.x;
  const int qrows = (a.hq + 2 * a.hkv) * 128;
  split_range(qrows / 2, G, c, p.q0, p.q1);
  p.q0 *= 2;
  p.q1 *= 2;
  split_range(a.H / 2, G, c, p.o0, p.o1);
  p.o0 *= 2;
  p.o1 *= 2;
  split_range(a.k * a.I / 2, G, c, p.g0, p.g1);
  p.g0 *= 2;
  p.g1 *= 2;
  return p;
}

struct AttnPlan {
  int T, nblk, n_items, n_super;  // global: tokens, blocks, items, super-chunks
  int nbi, per_super;             // blocks per item, items per super-chunk
  int i_lo, i_hi;                 // this rank's items (global indices)
  int items;                      // work items of this rank: local items x kv heads
};
__device__ __forceinline__ AttnPlan attn_plan(const MegaArgs& a, int pos) {
  AttnPlan p;
  p.T = pos + 1;
  p.nblk = (p.T + kAttBlock - 1) / kAttBlock;
  p.nbi = item_blocks(p.nblk);
  p.per_super = super_items(p.nblk);
  p.n_items = (p.nblk + p.nbi - 1) / p.nbi;
  p.n_super = (p.n_items + p.per_super - 1) / p.per_super;
  p.i_lo = min(a.super_lo * p.per_super, p.n_items);
  p.i_hi = min(a.super_hi * p.per_super, p.n_items);
  p.items = (p.i_hi - p.i_lo) * a.hkv;
  return p;
}
// One rank, one super-chunk of at most kShortItems items per head: the CTA
// that stores a head group's last item partial folds the group itself
// (Consumers::short_tail); otherwise the folds run after a grid barrier from
// partials the producer stages (merge_phase, final_phase).
__device__ __forceinline__ bool short_merge(const MegaArgs& a, const AttnPlan& P) {
  return a.world == 1 && P.n_super == 1 && P.n_items <= kShortItems;
}
// Work item it of this rank: kv head g and global item index.
__device__ __forceinline__ void attn_coords(const AttnPlan& P, int hkv, int it, int& g, int& item) {
  g = it % hkv;
  item = P.i_lo + it / hkv;
}
// Parity of the global layer step: selects one of the two exchange copies.
__device__ __forceinline__ int xch_parity(const MegaArgs& a, int step, int layer) {
  return int((a.layer_seq0 + unsigned(step) * unsigned(a.n_layers) + unsigned(layer)) & 1u);
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// In-layer stamps are compiled in only with -DREC_LAYER_STAMPS (diagnostic
// builds): each site costs instructions in code that runs once per layer.
__device__ __forceinline__ void stamp(const MegaArgs& a, int step, int layer, int slot) {
#ifdef REC_LAYER_STAMPS
  if (a.prof2 && step == 0 && layer == a.prof_layer) {
    unsigned long long t;
    // the memory clobber keeps the site between the loads and stores around it
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t) :: "memory");
    a.prof2[blockIdx.x * 64 + slot] = t;
  }
#endif
}
// Adds v to a per-CTA diagnostic slot of the same layer profile.
__device__ __forceinline__ void prof_add(const MegaArgs& a, int step, int layer, int slot, unsigned long long v) {
#ifdef REC_LAYER_STAMPS
  if (a.prof2 && step == 0 && layer == a.prof_layer) a.prof2[blockIdx.x * 64 + slot] += v;
#endif
}

constexpr int kSegAll = -2;
__device__ __forceinline__ int seg_l0(const MegaArgs& a) { return a.seg == kSegAll ? 0 : max(0, a.seg); }
__device__ __forceinline__ int seg_l1(const MegaArgs& a) {
  return a.seg == kSegAll ? a.n_layers : min(a.n_layers, a.seg + 2);
}
__device__ __forceinline__ bool seg_q(const MegaArgs& a, int l) { return a.seg == kSegAll || l == a.seg + 1; }
__device__ __forceinline__ bool seg_orgd(const MegaArgs& a, int l) { return a.seg == kSegAll || l == a.seg; }
__device__ __forceinline__ bool seg_h(const MegaArgs& a) { return a.seg == kSegAll || a.seg == a.n_layers - 1; }

// Grid barrier index of a phase: each step has 6 per layer + 1 (after H).
// Phase 3 (router logits -> selection) is not a grid barrier: its timeline
// slot records when the CTA's selection became ready.
__device__ __forceinline__ unsigned bar_index(const MegaArgs& a, int step, int layer, int ph) {
  return unsigned(step * (6 * a.n_layers + 1) + 6 * layer + ph);
}
// Flag of a layer's router-logit words: unique over the context's launches
// (never 0, the value of a cleared word).
__device__ __forceinline__ unsigned route_flag(const MegaArgs& a, int step, int layer) {
  return a.layer_seq0 + unsigned(step) * unsigned(a.n_layers) + unsigned(layer) + 1u;
}

__device__ __forceinline__ bool aborted(const MegaArgs& a) {
  return *reinterpret_cast<volatile unsigned*>(a.gbar + 1) != 0;
}
// Waits that poll shared memory look at the abort word (a global load, one
// L2 round trip) every 8th time round only, so that the load seldom delays
// the moment the wait sees its own condition.
__device__ __forceinline__ bool aborted_every8(const MegaArgs& a, uint32_t spins) {
  return (spins & 7u) == 7u && aborted(a);
}
__device__ __forceinline__ void set_abort(const MegaArgs& a, int code) {
  report(a.ctl + 0, code);
  atomicExch(a.gbar + 1, 1u);
}

// Bounded grid barrier among consumers of all CTAs.  Returns false on abort.
// seq: the launch's running barrier count (every CTA passes the same
// sequence); idx: the timeline slot, or kNoStamp for barriers the timeline
// does not record (the long-context merge phase).
constexpr unsigned kNoStamp = 0xffffffffu;
__device__ __forceinline__ bool grid_barrier(const MegaArgs& a, unsigned seq, unsigned idx) {
  cons_sync();
  __shared__ int ok_flag;
  if (threadIdx.x == 32) {
    if (a.prof && idx != kNoStamp) a.prof[(size_t(idx) * gridDim.x + blockIdx.x) * 2] = globaltimer();
    // release: the CTA's writes (ordered before this thread by the barrier
    // above) become visible to every CTA that acquires the count
    if (int(blockIdx.x) != a.skip_arrive_cta)
      asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(a.gbar), "r"(1u) : "memory");
    const unsigned target = gridDim.x * (seq + 1);
    int ok = 1;
    uint32_t spins = 0;
    while (true) {
      // the abort word's load is issued first and overlaps the count's
      // acquire load: one L2 round trip per poll.  A CTA that leaves while
      // another raises the abort stops at its next wait (every wait reads it).
      const bool ab = aborted(a);
      if (ld_acquire(a.gbar) >= target) break;
      if (ab) { ok = 0; break; }
      if (++spins > a.bar_spin_limit) {
        set_abort(a, kStatusCounterTimeout);
        ok = 0;
        break;
      }
    }
    if (a.prof && idx != kNoStamp) a.prof[(size_t(idx) * gridDim.x + blockIdx.x) * 2 + 1] = globaltimer();
    ok_flag = ok;
  }
  cons_sync();
  return ok_flag != 0;
}

// ---------------------------------------------------------------------------
// Producer
// ---------------------------------------------------------------------------
struct Producer {
  const MegaArgs& a;
  MegaSmem& sm;
  uint32_t chunk = 0;
  bool ok = true;
  uint32_t issued_mask = 0, last_par = 0;  // per slot: ever issued, parity of its last phase

  __device__ Producer(const MegaArgs& a_, MegaSmem& sm_) : a(a_), sm(sm_) {}

  __device__ void issued(int slot) {
    issued_mask |= 1u << slot;
    last_par = (last_par & ~(1u << slot)) | (((chunk / kSlots) & 1u) << slot);
    ++chunk;
  }
  // lane 0 only
  __device__ uint8_t* acquire(int& slot) {
    slot = chunk % kSlots;
    if (chunk >= kSlots) {
      const uint32_t par = ((chunk / kSlots) - 1) & 1;
      uint32_t spins = 0;
      while (!mbar_try_wait(&sm.empty[slot], par)) {
        if (aborted_every8(a, spins)) { ok = false; return nullptr; }
        if (++spins > kSpinLimit) {
          set_abort(a, kStatusBulkTimeout);
          ok = false;
          return nullptr;
        }
      }
    }
#ifdef REC_LAYER_STAMPS
    if (acq_stamp >= 0) {
      stamp_cur(acq_stamp);
      acq_stamp = -1;
    }
#endif
    return sm.ring[slot];
  }
  __device__ void gemv_chunk(const QMatDev& m, int K, int row0, int n) {
    int slot;
    uint8_t* dst = acquire(slot);
    if (!dst) return;
    const uint32_t wb = uint32_t(n) * (K / 2), sbytes = uint32_t(n) * (K / 32);
    const uint32_t soff = wb, boff = wb + ((sbytes + 15) & ~15u);
    mbar_expect_tx(&sm.full[slot], wb + 2 * sbytes);
    bulk_g2s(dst, reinterpret_cast<const uint8_t*>(m.w) + size_t(row0) * (K / 2), wb, &sm.full[slot]);
    bulk_g2s(dst + soff, m.s + size_t(row0) * (K / 64), sbytes, &sm.full[slot]);
    bulk_g2s(dst + boff, m.b + size_t(row0) * (K / 64), sbytes, &sm.full[slot]);
    issued(slot);
  }
  // G chunk: n gate/up pairs, rows [i0, i0 + nA) of expert eA then rows
  // [0, n - nA) of expert eB (a chunk may span two experts, so every CTA's
  // share of pairs takes the same number of chunks).  Slot layout: gate rows,
  // up rows, gate scales, up scales, gate biases, up biases (pair q = row q).
  __device__ void pair_chunk(const MegaLayer& L, int eA, int i0, int nA, int eB, int n) {
    int slot;
    uint8_t* dst = acquire(slot);
    if (!dst) return;
    const uint32_t wb = uint32_t(n) * 1024, sbytes = uint32_t(n) * 64;
    mbar_expect_tx(&sm.full[slot], 2 * wb + 4 * sbytes);
    for (int part = 0; part < 2; ++part) {
      const int np = part ? n - nA : nA;
      if (np == 0) continue;
      const size_t row = part ? size_t(eB) * a.I : size_t(eA) * a.I + i0;
      const uint32_t q0 = part ? uint32_t(nA) : 0u;  // first pair of this part
      const uint32_t pw = uint32_t(np) * 1024, ps = uint32_t(np) * 64;
      bulk_g2s(dst + q0 * 1024, reinterpret_cast<const uint8_t*>(L.gate.w) + row * 1024, pw, &sm.full[slot]);
      bulk_g2s(dst + wb + q0 * 1024, reinterpret_cast<const uint8_t*>(L.up.w) + row * 1024, pw, &sm.full[slot]);
      bulk_g2s(dst + 2 * wb + q0 * 64, L.gate.s + row * 32, ps, &sm.full[slot]);
      bulk_g2s(dst + 2 * wb + sbytes + q0 * 64, L.up.s + row * 32, ps, &sm.full[slot]);
      bulk_g2s(dst + 2 * wb + 2 * sbytes + q0 * 64, L.gate.b + row * 32, ps, &sm.full[slot]);
      bulk_g2s(dst + 2 * wb + 3 * sbytes + q0 * 64, L.up.b + row * 32, ps, &sm.full[slot]);
    }
    issued(slot);
  }
  // D chunk: experts ids[r0..r1) rows [o0, o0+n) of the down matrices (K = I)
  __device__ void down_chunk(const MegaLayer& L, const int* ids, int r0, int r1, int o0, int n) {
    int slot;
    uint8_t* dst = acquire(slot);
    if (!dst) return;
    const uint32_t wb = uint32_t(n) * (a.I / 2), sbytes = uint32_t(n) * (a.I / 32);
    const uint32_t per = wb + 2 * ((sbytes + 15) & ~15u);
    mbar_expect_tx(&sm.full[slot], uint32_t(r1 - r0) * (wb + 2 * sbytes));
    for (int r = r0; r < r1; ++r) {
      const size_t row = size_t(ids[r]) * a.H + o0;
      uint8_t* d = dst + (r - r0) * per;
      bulk_g2s(d, reinterpret_cast<const uint8_t*>(L.down.w) + row * (a.I / 2), wb, &sm.full[slot]);
      bulk_g2s(d + wb, L.down.s + row * (a.I / 64), sbytes, &sm.full[slot]);
      bulk_g2s(d + wb + ((sbytes + 15) & ~15u), L.down.b + row * (a.I / 64), sbytes, &sm.full[slot]);
    }
    issued(slot);
  }
  // One router row (bf16 [H]) of expert e.
  __device__ void router_chunk(const MegaLayer& L, int e) {
    int slot;
    uint8_t* dst = acquire(slot);
    if (!dst) return;
    const uint32_t bytes = uint32_t(a.H) * 2;
    mbar_expect_tx(&sm.full[slot], bytes);
    bulk_g2s(dst, L.router + size_t(e) * a.H, bytes, &sm.full[slot]);
    issued(slot);
  }
  __device__ void kv_chunk(const uint32_t* codes, const uint16_t* sc, const uint16_t* bi, int g, int b, int n) {
    int slot;
    uint8_t* dst = acquire(slot);
    if (!dst) return;
    const int rw = 128 * a.kv_bits / 32;
    const int n4 = (n + 3) & ~3;
    const size_t s0 = size_t(g) * a.capacity + size_t(b - a.token_base / kAttBlock) * kAttBlock;
    const uint32_t cb = uint32_t(n4) * rw * 4, sbytes = uint32_t(n4) * 4;
    mbar_expect_tx(&sm.full[slot], cb + 2 * sbytes);
    bulk_g2s(dst, codes + s0 * rw, cb, &sm.full[slot]);
    bulk_g2s(dst + cb, sc + s0 * 2, sbytes, &sm.full[slot]);
    bulk_g2s(dst + cb + sbytes, bi + s0 * 2, sbytes, &sm.full[slot]);
    issued(slot);
  }

  // 4-bit caches: K and V of one block fill exactly one slot (2 x 18,432 B).
  __device__ void kv_pair_chunk(const MegaLayer& L, int g, int b, int n) {
    int slot;
    uint8_t* dst = acquire(slot);
    if (!dst) return;
    constexpr int rw = 16;
    const int n4 = (n + 3) & ~3;
    const size_t s0 = size_t(g) * a.capacity + size_t(b - a.token_base / kAttBlock) * kAttBlock;
    const uint32_t cb = uint32_t(n4) * rw * 4, sbytes = uint32_t(n4) * 4, half = cb + 2 * sbytes;
    mbar_expect_tx(&sm.full[slot], 2 * half);
    bulk_g2s(dst, L.k_codes + s0 * rw, cb, &sm.full[slot]);
    bulk_g2s(dst + cb, L.k_scales + s0 * 2, sbytes, &sm.full[slot]);
    bulk_g2s(dst + cb + sbytes, L.k_biases + s0 * 2, sbytes, &sm.full[slot]);
    bulk_g2s(dst + half, L.v_codes + s0 * rw, cb, &sm.full[slot]);
    bulk_g2s(dst + half + cb, L.v_scales + s0 * 2, sbytes, &sm.full[slot]);
    bulk_g2s(dst + half + cb + sbytes, L.v_biases + s0 * 2, sbytes, &sm.full[slot]);
    issued(slot);
  }

  // 8 heads x n partials (kPartialFloats floats each): head h's run starts at
  // src0 + h * head_stride; slot layout [head][n][kPartialFloats].
  __device__ void partials_chunk(const float* src0, size_t head_stride, int n) {
    int slot;
    uint8_t* dst = acquire(slot);
    if (!dst) return;
    const uint32_t bytes = uint32_t(n) * kPartialFloats * 4;
    mbar_expect_tx(&sm.full[slot], kHeadsPerKv * bytes);
    for (int h = 0; h < kHeadsPerKv; ++h) bulk_g2s(dst + h * bytes, src0 + h * head_stride, bytes, &sm.full[slot]);
    issued(slot);
  }
  // Waits (bounded) until the consumers have passed merge barrier `target`.
  // The partials were written by other CTAs before it: order the async-proxy
  // reads after the consumers' acquire.
  __device__ void wait_merge(int target) {
    uint32_t spins = 0;
    while (sm.merge_seq < target) {
      __nanosleep(32);
      if (aborted_every8(a, spins)) { ok = false; return; }
      if (++spins > kSpinLimit * 64) {
        set_abort(a, kStatusCounterTimeout);
        ok = false;
        return;
      }
    }
    stamp_cur(30);
    __threadfence();
    asm volatile("fence.proxy.async.global;" ::: "memory");
    stamp_cur(25);
  }
  // The merge phases of one layer's attention (the consumers' merge_phase
  // and final_phase take the same chunks in the same order).
  int cur_step = 0, cur_layer = 0;  // for the diagnostics stamps
  int acq_stamp = -1;                // diagnostics: stamp slot of the next slot acquisition
  __device__ void stamp_cur(int slot) { stamp(a, cur_step, cur_layer, slot); }
  __device__ void merge_chunks(const AttnPlan& AP, int step, int l) {
    if (short_merge(a, AP)) return;
    cur_step = step;
    cur_layer = l;
    const int seq = 2 * (step * a.n_layers + l);
    wait_merge(seq + 1);
    const int icap = items_cap(a.capacity);
    const int item0 = a.token_base / (kAttBlock * AP.nbi);
    const int n_local = max(0, min(a.super_hi, AP.n_super) - a.super_lo);
    for (int t = blockIdx.x; t < n_local * a.hkv && ok; t += gridDim.x) {
      const int g = t % a.hkv, s = a.super_lo + t / a.hkv;
      const int lo = s * AP.per_super - item0, hi = min((s + 1) * AP.per_super, AP.n_items) - item0;
      for (int i0 = lo; i0 < hi && ok; i0 += kMergeChunk)
        partials_chunk(a.partials + (size_t(g * kHeadsPerKv) * icap + i0) * kPartialFloats,
                       size_t(icap) * kPartialFloats, min(kMergeChunk, hi - i0));
    }
    if (AP.n_super > 1 && a.world == 1 && ok) {
      wait_merge(seq + 2);
      for (int c = blockIdx.x; c < a.hkv && ok; c += gridDim.x)
        for (int s0 = 0; s0 < AP.n_super && ok; s0 += kMergeChunk)
          partials_chunk(a.supers + (size_t(c * kHeadsPerKv) * a.n_super_max + s0) * kPartialFloats,
                         size_t(a.n_super_max) * kPartialFloats, min(kMergeChunk, AP.n_super - s0));
    }
  }

  // Routing in the producer warp (all lanes): the router logits arrive as
  // flag+value words, so the selection needs no grid barrier, and the
  // expert copies are issued right after it.  Lane l handles experts l,
  // l+32, ...  Softmax (router_mode 0: max, exp(l - max), the sum lane by
  // lane in that order then a butterfly, p = exp / sum) or sigmoid + bias
  // (1: p = sigmoid(l), c = p + bias); the top-k by c, lowest index on ties,
  // in k rounds of a warp arg-max; weights p / (sum of the selected p in
  // rank order + 1e-20).  Publishes ids, wts and the local-expert lists in
  // shared memory, then route_seq = seq.  Compact loops: this code runs
  // once per layer, so its size (instruction fetch) matters more than ILP.
  __device__ bool route_ll(const MegaLayer& L, int step, int l, int lane) {
    constexpr int J = kMegaMaxExperts / 32;
    const unsigned flag = route_flag(a, step, l);
    const int E = a.E;
    const unsigned long long* buf = a.router_ll + size_t(flag & 1u) * E;
    unsigned pending = 0;
#pragma unroll 1
    for (int j = 0; j < J; ++j)
      if (lane + 32 * j < E) pending |= 1u << j;
    const unsigned valid = pending;
    uint32_t spins = 0;
    while (true) {
      const bool ab = aborted(a);  // in flight with the logit loads
      unsigned long long v[J];
#pragma unroll
      for (int j = 0; j < J; ++j) v[j] = ((pending >> j) & 1u) ? ld_relaxed64(buf + lane + 32 * j) : 0ull;
#pragma unroll
      for (int j = 0; j < J; ++j)
        if (((pending >> j) & 1u) && unsigned(v[j] >> 32) == flag) {
          sm.route_p[lane + 32 * j] = __uint_as_float(unsigned(v[j]));
          pending &= ~(1u << j);
        }
      if (__all_sync(0xffffffffu, pending == 0)) break;
      if (__any_sync(0xffffffffu, ab)) return false;
      if (++spins > kSpinLimit * 4) {
        if (lane == 0) set_abort(a, kStatusCounterTimeout);
        return false;
      }
    }
    if (lane == 0) stamp(a, step, l, 14);
    if (a.router_mode == 0) {
      float mx = -INFINITY;
#pragma unroll 1
      for (int i = lane; i < E; i += 32) mx = fmaxf(mx, sm.route_p[i]);
      mx = bfly_max(mx);
      float sum = 0.0f;
#pragma unroll 1
      for (int i = lane; i < E; i += 32) {
        const float c = rexp(__fsub_rn(sm.route_p[i], mx));
        sm.route_p[i] = c;
        sum = __fadd_rn(sum, c);
      }
      sum = bfly_sum(sum);
#pragma unroll 1
      for (int i = lane; i < E; i += 32) {
        const float pi = __fdiv_rn(sm.route_p[i], sum);
        sm.route_p[i] = pi;
        sm.route_k[i] = route_key(pi);
      }
    } else {
#pragma unroll 1
      for (int i = lane; i < E; i += 32) {
        const float pi = rsigmoid(sm.route_p[i]);
        sm.route_p[i] = pi;
        sm.route_k[i] = route_key(__fadd_rn(pi, L.expert_bias[i]));
      }
    }
    __syncwarp();
    if (lane == 0) stamp(a, step, l, 49);
    unsigned key[J];  // this lane's keys in registers for the k rounds (0 = absent or taken)
#pragma unroll
    for (int j = 0; j < J; ++j) key[j] = ((valid >> j) & 1u) ? sm.route_k[lane + 32 * j] : 0u;
    float s2 = 0.0f, my_p = 0.0f;
    int my_id = 0;
#pragma unroll 1
    for (int r = 0; r < a.k; ++r) {
      unsigned best = 0;
      int bj = 0;
#pragma unroll
      for (int j = 0; j < J; ++j)
        if (key[j] > best) {
          best = key[j];
          bj = j;
        }
      const unsigned wbest = __reduce_max_sync(0xffffffffu, best);
      int widx = int(__reduce_min_sync(0xffffffffu, (best == wbest && best) ? unsigned(lane + 32 * bj) : ~0u));
      if (unsigned(widx) >= unsigned(E)) widx = 0;  // no key left (top_k > E); never read outside route_p
      const float pw = sm.route_p[widx];
      if (lane == (widx & 31)) {
#pragma unroll
        for (int j = 0; j < J; ++j)
          if (j == (widx >> 5)) key[j] = 0u;  // taken
      }
      if (lane == r) {
        my_id = widx;
        my_p = pw;
      }
      s2 = __fadd_rn(s2, pw);
    }
    s2 = __fadd_rn(s2, 1e-20f);
    const bool sel = lane < a.k;
    const bool local = sel && my_id >= a.e_lo && my_id < a.e_hi;
    const unsigned lm = __ballot_sync(0xffffffffu, local);
    if (sel) {
      sm.ids[lane] = my_id;
      sm.wts[lane] = __fdiv_rn(my_p, s2);
    }
    if (local) {
      const int at = __popc(lm & ((1u << lane) - 1u));
      sm.loc[at] = lane;
      sm.lids[at] = my_id - a.e_lo;
    }
    if (lane == 0) sm.n_loc = __popc(lm);
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      sm.route_seq = step * a.n_layers + l + 1;
      stamp(a, step, l, 15);
    }
    __syncwarp();
    return true;
  }

  __device__ void run() {
    const int lane = threadIdx.x & 31;
    const Part P = partition(a);
    const int pos0 = sm.pos0;
    const int qrows[3] = {a.hq * 128, a.hkv * 128, a.hkv * 128};
    const bool attn_in = a.seg == kSegAll;
    for (int step = 0; step < a.steps && ok; ++step) {
      const int pos = pos0 + step;
      const AttnPlan AP = attn_plan(a, pos);
      for (int l = seg_l0(a); l < seg_l1(a) && ok; ++l) {
        const MegaLayer& L = sm.layers[l];
        const bool orgd = seg_orgd(a, l);
        if (lane == 0) {
          // Q rows (q | k | v), chunks never cross matrices
          for (int r = P.q0; r < P.q1 && ok && seg_q(a, l);) {
            int m = 0, base = 0;
            while (m < 2 && r >= base + qrows[m]) base += qrows[m++];
            const int n = min(min(kQRows, P.q1 - r), base + qrows[m] - r);
            gemv_chunk(m == 0 ? L.q : (m == 1 ? L.k : L.v), a.H, r - base, n);
            r += n;
          }
          // A: K and V tiles of this CTA's items
          for (int it = blockIdx.x; it < AP.items && ok && attn_in; it += gridDim.x) {
            int g, item;
            attn_coords(AP, a.hkv, it, g, item);
            const int b1 = min(item * AP.nbi + AP.nbi, AP.nblk);
            for (int b = item * AP.nbi; b < b1 && ok; ++b) {
              const int n = min(kAttBlock, AP.T - b * kAttBlock);
              if (a.kv_bits == 4) {
                kv_pair_chunk(L, g, b, n);
              } else {
                kv_chunk(L.k_codes, L.k_scales, L.k_biases, g, b, n);
                kv_chunk(L.v_codes, L.v_scales, L.v_biases, g, b, n);
              }
            }
            stamp(a, step, l, 24);
          }
          if (ok && attn_in) merge_chunks(AP, step, l);
          // O rows
          for (int r = P.o0; r < P.o1 && ok && orgd; r += kORows)
            gemv_chunk(L.o, a.hq * 128, r, min(kORows, P.o1 - r));
          // R: this CTA's router rows
          for (int e = blockIdx.x; e < a.E && ok && orgd; e += gridDim.x) router_chunk(L, e);
        }
        __syncwarp();
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!orgd) continue;
        // G / D need this layer's routing: the warp selects the experts as
        // soon as every router logit has landed
        if (ok) ok = route_ll(L, step, l, lane);
        if (lane == 0) stamp(a, step, l, 20);
        if (lane == 0 && ok) {
          // this rank's selected experts only (all of them when world == 1)
          int lids[kMaxTopK];
          const int nl = sm.n_loc;
          for (int j = 0; j < nl; ++j) lids[j] = sm.lids[j];
          int g0, g1;
          split_range(nl * a.I / 2, gridDim.x, blockIdx.x, g0, g1);
          g0 *= 2;
          g1 *= 2;
#ifdef REC_LAYER_STAMPS
          cur_step = step;
          cur_layer = l;
          acq_stamp = 50;
#endif
          for (int u = g0; u < g1 && ok;) {
            const int j = u / a.I, i0 = u % a.I;
            const int n = min(kGPairs, g1 - u), nA = min(n, a.I - i0);
            pair_chunk(L, lids[j], i0, nA, nA < n ? lids[j + 1] : 0, n);
            stamp(a, step, l, 21 + min((u - g0) / kGPairs, 3));
            u += n;
          }
          if (P.o1 > P.o0)
            for (int j0 = 0; j0 < nl && ok; j0 += kDExperts)
              down_chunk(L, lids, j0, min(nl, j0 + kDExperts), P.o0, P.o1 - P.o0);
        }
        __syncwarp();
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
      if (lane == 0 && seg_h(a)) {
        int v0, v1;
        split_range(a.V / 2, gridDim.x, blockIdx.x, v0, v1);
        v0 *= 2;
        v1 *= 2;
        for (int r = v0; r < v1 && ok; r += kQRows) gemv_chunk(a.lm_head, a.H, r, min(kQRows, v1 - r));
      }
      __syncwarp();
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    // on abort: let the copies already issued land before the CTA exits
    if (lane == 0 && !ok) {
      for (int s = 0; s < kSlots; ++s)
        if (issued_mask & (1u << s)) mbar_wait(&sm.full[s], (last_par >> s) & 1u);
    }
  }
};

// ---------------------------------------------------------------------------
// Consumers
// ---------------------------------------------------------------------------
struct Consumers {
  const MegaArgs& a;
  MegaSmem& sm;
  const int warp, lane;  // warp in 0..7
  uint32_t chunk = 0;
  unsigned nbar = 0;  // grid barriers passed in this launch

  __device__ bool gbar(unsigned idx) { return grid_barrier(a, nbar++, idx); }
  int slot = 0;
  bool ok = true;

  __device__ Consumers(const MegaArgs& a_, MegaSmem& sm_)
      : a(a_), sm(sm_), warp((threadIdx.x >> 5) - 1), lane(threadIdx.x & 31) {}

  __device__ const uint8_t* take() {
    slot = chunk % kSlots;
    const uint32_t par = (chunk / kSlots) & 1;
    uint32_t spins = 0;
    while (!mbar_try_wait(&sm.full[slot], par)) {
      if (aborted_every8(a, spins)) { ok = false; break; }
      if (++spins > kSpinLimit) {
        set_abort(a, kStatusBulkTimeout);  // every CTA leaves at its next grid barrier
        ok = false;
        break;
      }
    }
    return sm.ring[slot];
  }
  __device__ void release(bool wrote_smem = false) {
    if (wrote_smem) fence_proxy_async();
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[slot]);
    ++chunk;
  }

  // The fixed-point limbs of x (n_groups groups of 64, one scale) shared by
  // every lane of the CTA: prepared once, in place.
  __device__ void share_limbs(uint16_t* x, int n_groups, const FixScale& fs) {
    const float up = fs.up;
    prep_limbs_inplace<2, kMegaCons * 32>(x, sm.gX, n_groups, threadIdx.x - 32, [up](int) { return up; },
                                          ConsSync{});
  }

  // RMSNorm of src (bf16[2048], global or shared) into sm.xn, canonical
  // order: consumer thread t owns chunk t (8 elements) = group t/32 = its warp.
  __device__ FixScale norm(const uint16_t* src, const uint16_t* w, bool from_smem = false) {
    const int t = threadIdx.x - 32;
    const uint4 u = from_smem ? *reinterpret_cast<const uint4*>(src + t * 8) : ldcg128(src + t * 8);
    const uint4 wv = ldg128_nc(w + t * 8);
    const uint32_t us[4] = {u.x, u.y, u.z, u.w};
    float x[8];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      x[2 * q] = __uint_as_float(us[q] << 16);
      x[2 * q + 1] = __uint_as_float(us[q] & 0xFFFF0000u);
    }
    float acc = 0.0f;
#pragma unroll
    for (int q = 0; q < 8; ++q) acc = __fmaf_rn(x[q], x[q], acc);
    acc = bfly_sum(acc);
    if (lane == 0) sm.red[warp] = acc;
    cons_sync();
    if (warp == 0 && lane == 0) {
      float total = 0.0f;
      for (int g = 0; g < kMegaCons; ++g) total = __fadd_rn(total, sm.red[g]);
      sm.red[32] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, 2048.0f), a.eps)));
    }
    cons_sync();
    const float inv = sm.red[32];
    const uint32_t ws_[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
    float mx = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t lo = to_bf(__fmul_rn(__uint_as_float(ws_[q] << 16), rbf(__fmul_rn(x[2 * q], inv))));
      const uint32_t hi = to_bf(__fmul_rn(__uint_as_float(ws_[q] & 0xFFFF0000u), rbf(__fmul_rn(x[2 * q + 1], inv))));
      o[q] = lo | (hi << 16);
      mx = fmaxf(mx, fmaxf(fabsf(bf(uint16_t(lo))), fabsf(bf(uint16_t(hi)))));
    }
    *reinterpret_cast<uint4*>(sm.xn + t * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    mx = bfly_max(mx);
    if (lane == 0) sm.red[8 + warp] = mx;
    cons_sync();
    float r = 0.0f;
    for (int g = 0; g < kMegaCons; ++g) r = fmaxf(r, sm.red[8 + g]);
    return fix_scale_from_max(r);
  }
  // Copies n bf16 (n <= 4096 * ... multiple of 2048) into dst with every load issued
  // before the first store.
  __device__ void load_vec(uint16_t* dst, const uint16_t* src, int n) {
    constexpr int kMax = 4;
    const int t = threadIdx.x - 32, stride = kMegaCons * 32 * 8;
    uint4 v[kMax];
#pragma unroll
    for (int q = 0; q < kMax; ++q)
      if (t * 8 + q * stride < n) v[q] = ldcg128(src + t * 8 + q * stride);
#pragma unroll
    for (int q = 0; q < kMax; ++q)
      if (t * 8 + q * stride < n) *reinterpret_cast<uint4*>(dst + t * 8 + q * stride) = v[q];
    cons_sync();
  }
  // Loads x into sm.xn and returns its fixed-point scale.
  __device__ FixScale load_x(const uint16_t* src, int n, int step_ = -1, int layer_ = -1) {
    load_vec(sm.xn, src, n);
    if (warp == 0 && lane == 0) stamp(a, step_, layer_, 48);
    return fix_scale_from_max(block_maxabs(sm.xn, n, threadIdx.x - 32, kMegaCons * 32, sm.red, kBarCons));
  }

  // --- Q and H: K = 2048 rows, 8 warps x ILP 4 ---------------------------------
  template <bool HEAD>
  __device__ void rows2048(const uint8_t* st, int n, int grow0, const GroupX (&gx)[1], FixScale fs, uint16_t* out,
                           float& best, int& best_i) {
    const uint32_t wb = uint32_t(n) * 1024, sbytes = uint32_t(n) * 64;
    const uint8_t* wbase = st;
    const uint16_t* sbase = reinterpret_cast<const uint16_t*>(st + wb);
    const uint16_t* bbase = reinterpret_cast<const uint16_t*>(st + wb + ((sbytes + 15) & ~15u));
    int rows[4];
    bool valid[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = warp + i * kMegaCons;
      valid[i] = r < n;
      rows[i] = valid[i] ? r : 0;
    }
    float v[4];
    lane_rows_partial<2048, 2, 4>(wbase, sbase, bbase, rows, 0, lane, gx, v, a.sd);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[i] = __fmul_rn(bfly_sum(valid[i] ? v[i] : 0.0f), fs.down);
      if (valid[i] && lane == 0) {
        const int g = grow0 + rows[i];
        const uint16_t o = to_bf(v[i]);
        out[g] = o;
        if (HEAD) {
          const float fv = bf(o);
          if (fv > best || (fv == best && g < best_i)) { best = fv; best_i = g; }
        }
      }
    }
  }

  // --- O with K = 2048 (n_q_heads = 16): 8 warps x ILP 4, residual into own rows
  __device__ void rows2048_resid(const uint8_t* st, int n, int grow0, int own0, const GroupX (&gx)[1], FixScale fs) {
    const uint32_t wb = uint32_t(n) * 1024, sbytes = uint32_t(n) * 64;
    const uint8_t* wbase = st;
    const uint16_t* sbase = reinterpret_cast<const uint16_t*>(st + wb);
    const uint16_t* bbase = reinterpret_cast<const uint16_t*>(st + wb + ((sbytes + 15) & ~15u));
    int rows[4];
    bool valid[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = warp + i * kMegaCons;
      valid[i] = r < n;
      rows[i] = valid[i] ? r : 0;
    }
    float v[4];
    lane_rows_partial<2048, 2, 4>(wbase, sbase, bbase, rows, 0, lane, gx, v, a.sd);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[i] = __fmul_rn(bfly_sum(valid[i] ? v[i] : 0.0f), fs.down);
      if (valid[i] && lane == 0) {
        const int g = grow0 + rows[i];
        const int own = g - own0;
        const uint16_t hn = to_bf(__fadd_rn(bf(sm.hown[own]), rbf(v[i])));
        sm.hown[own] = hn;
        a.h[g] = hn;
      }
    }
  }

  // --- O: K = 4096 rows, warp pairs (one 2048 segment each) x ILP 4 ---------
  __device__ void rows4096(const uint8_t* st, int n, int grow0, int own0, const GroupX (&gx)[1], FixScale fs) {
    // always called by every consumer warp: the team barriers below must match
    const int seg = warp & 1, team = warp >> 1;
    const uint32_t wb = uint32_t(n) * 2048, sbytes = uint32_t(n) * 128;
    const uint8_t* wbase = st;
    const uint16_t* sbase = reinterpret_cast<const uint16_t*>(st + wb);
    const uint16_t* bbase = reinterpret_cast<const uint16_t*>(st + wb + sbytes);
    int rows[4];
    bool valid[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = team + 4 * i;
      valid[i] = r < n;
      rows[i] = valid[i] ? r : 0;
    }
    float v[4];
    lane_rows_partial<4096, 2, 4>(wbase, sbase, bbase, rows, seg, lane, gx, v, a.sd);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = bfly_sum(valid[i] ? v[i] : 0.0f);
    if (lane == 0)
      for (int i = 0; i < 4; ++i) sm.seg_part[warp][i] = v[i];
    asm volatile("bar.sync %0, %1;" ::"r"(kBarTeam0 + team), "r"(64));
    if (seg == 0 && lane == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (!valid[i]) continue;
        const float t = __fmul_rn(__fadd_rn(v[i], sm.seg_part[warp + 1][i]), fs.down);
        const int g = grow0 + rows[i];
        const int own = g - own0;
        const uint16_t hn = to_bf(__fadd_rn(bf(sm.hown[own]), rbf(t)));
        sm.hown[own] = hn;
        a.h[g] = hn;
      }
    }
    asm volatile("bar.sync %0, %1;" ::"r"(kBarTeam0 + team), "r"(64));
  }

  // --- attention ----------------------------------------------------------------
  // All consumer warps: item `item` (nbi blocks) of kv head g for its 8 q
  // heads, blocks streamed through the ring (4-bit: K and V in one slot;
  // 8-bit: a K slot and a V slot); the item partial is stored for
  // merge_phase.
  template <int BITS>
  __device__ void attn_item(const MegaLayer& L, const AttnPlan& P, int pos, int g, int item, int step_,
                            int layer_) {
    constexpr int RW = 128 * BITS / 32;
    const int b0 = item * P.nbi, b1 = min(b0 + P.nbi, P.nblk);
    const float* cs = a.rope + size_t(pos) * 128;
    cons_sync();  // a previous item's merges may still use the scratch
    if (sm.att.qg != g) prep_q_heads<BITS>(a.qkv, g, cs, L.q_norm, a.eps, sm.att, warp);
    const bool has_new = pos >= b0 * kAttBlock && pos < b1 * kAttBlock;
    if (has_new) {
      const size_t sl = size_t(g) * a.capacity + size_t(pos - a.token_base);
      prep_new_kv<BITS>(a.qkv, a.hq, a.hkv, g, cs, L.k_norm, a.eps, sm.att, warp, L.k_codes + sl * RW,
                        L.v_codes + sl * RW, L.k_scales + sl * 2, L.k_biases + sl * 2, L.v_scales + sl * 2,
                        L.v_biases + sl * 2);
    }
    cons_sync();
    if (warp == 0 && lane == 0) {
      sm.att.qg = g;
      stamp(a, step_, layer_, 19);
    }
    WarpState st;
    state_empty(st);
    for (int b = b0; b < b1; ++b) {
      const int n = min(kAttBlock, P.T - b * kAttBlock), n4 = (n + 3) & ~3;
      uint8_t* kt = const_cast<uint8_t*>(take());
      if (warp == 0 && lane == 0 && b == b0) stamp(a, step_, layer_, 29);
      const int kslot = slot;
      uint8_t* vt;
      int vslot = -1;
      if constexpr (BITS == 4) {
        vt = kt + n4 * RW * 4 + n4 * 8;  // V half of the same slot
      } else {
        ++chunk;
        vt = const_cast<uint8_t*>(take());
        vslot = slot;
        --chunk;
      }
      uint32_t* kc = reinterpret_cast<uint32_t*>(kt);
      uint16_t* ks = reinterpret_cast<uint16_t*>(kt + n4 * RW * 4);
      uint32_t* vc = reinterpret_cast<uint32_t*>(vt);
      uint16_t* vs = reinterpret_cast<uint16_t*>(vt + n4 * RW * 4);
      const int new_row = (has_new && pos / kAttBlock == b) ? pos - b * kAttBlock : -1;
      block_tiles<BITS>(kc, ks, ks + n4 * 2, vc, vs, vs + n4 * 2, n, new_row, sm.att, warp, st);
      if (warp == 0 && lane == 0 && b == b0) stamp(a, step_, layer_, 16);
      slot = kslot;
      release(true);
      if (vslot >= 0) {
        slot = vslot;
        release(true);
      }
    }
    if (warp == 0 && lane == 0) stamp(a, step_, layer_, 17);
    cons_sync();  // the fold scratch overlays the query-preparation buffers
    // item partial of the 8 heads (local item index)
    const int icap = items_cap(a.capacity);
    const int item0 = a.token_base / (kAttBlock * P.nbi);
    warps_fold_store(st, warp, sm.att, ConsSync{},
                     a.partials + (size_t(g * kHeadsPerKv) * icap + (item - item0)) * kPartialFloats,
                     size_t(icap) * kPartialFloats);
    if (warp == 0 && lane == 0) stamp(a, step_, layer_, 18);
    if (short_merge(a, P)) short_tail(L, P, g, step_, layer_);
  }

  // Short contexts: an acq_rel counter per kv head finds the CTA that stored
  // the group's last item partial; it bulk-copies the group's partials into
  // its scratch and warp w folds head 8g + w: [sink], then the items in order.
  __device__ void short_tail(const MegaLayer& L, const AttnPlan& P, int g, int step_, int layer_) {
    cons_sync();  // every warp's partial stores precede the counter update
    if (warp == 0 && lane == 0) {
      unsigned* cnt = a.cnt + a.hq + g * a.n_super_max;
      unsigned prev;
      asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(cnt) : "memory");
      const bool last = prev == unsigned(P.n_items - 1);
      sm.xok = last ? 1 : 0;
      if (last) {
        *cnt = 0u;  // the next layer's items come after grid barriers
        asm volatile("fence.proxy.async.global;" ::: "memory");
        const int icap = items_cap(a.capacity);
        const uint32_t bytes = uint32_t(P.n_items) * kPartialFloats * 4;
        mbar_expect_tx(&sm.mfull, kHeadsPerKv * bytes);
        for (int h = 0; h < kHeadsPerKv; ++h)
          bulk_g2s(&sm.att.u.items[h][0][0], a.partials + size_t(g * kHeadsPerKv + h) * icap * kPartialFloats,
                   bytes, &sm.mfull);
      }
    }
    cons_sync();
    if (!sm.xok) return;
    const bool ok = mbar_wait(&sm.mfull, sm.mpar & 1u);
    if (ok) {
      const int h = g * kHeadsPerKv + warp;
      Partial4 F = sink_partial(L, h);
      for (int j = 0; j < P.n_items; ++j) merge_into(F, smem_partial(&sm.att.u.items[warp][j][0]));
      write_attn(h, F);
      if (warp == 0 && lane == 0) stamp(a, step_, layer_, 31);
    } else if (warp == 0 && lane == 0) {
      set_abort(a, kStatusBulkTimeout);
    }
    cons_sync();
    if (warp == 0 && lane == 0) sm.mpar += 1;
  }

  // Folds super-chunk s of the 8 heads of kv head g from the merge slots
  // (items in order; warp w = head 8g + w), then finishes it: several ranks
  // publish it, one rank with one super-chunk writes the output, otherwise
  // it is stored for final_phase.
  template <int BITS>
  __device__ void merge_phase(const MegaLayer& L, const AttnPlan& P, int step_, int layer_) {
    const int n_local = max(0, min(a.super_hi, P.n_super) - a.super_lo);
    const int item0 = a.token_base / (kAttBlock * P.nbi);
    for (int t = blockIdx.x; t < n_local * a.hkv; t += gridDim.x) {
      const int g = t % a.hkv, s = a.super_lo + t / a.hkv;
      const int lo = s * P.per_super - item0, hi = min((s + 1) * P.per_super, P.n_items) - item0;
      Partial4 S = empty_partial();
      for (int i0 = lo; i0 < hi; i0 += kMergeChunk) {
        const int n = min(kMergeChunk, hi - i0);
        const float* st = reinterpret_cast<const float*>(take()) + warp * n * kPartialFloats;
        if (warp == 0 && lane == 0 && i0 == lo) stamp(a, step_, layer_, 37);
        for (int j = 0; j < n; ++j) merge_into(S, smem_partial(st + j * kPartialFloats));
        release();
      }
      if (warp == 0 && lane == 0) stamp(a, step_, layer_, 38);
      const int h = g * kHeadsPerKv + warp;
      if (a.world > 1) {
        // publish the super-chunk to every rank; each merges them itself
        const int par = xch_parity(a, step_, layer_);
        for (int q = 0; q < a.world; ++q) store_partial(xch_super(a.xch[q], a.xl, par, h, s), S);
        __syncwarp();
        if (lane == 0) {
          __threadfence_system();  // cumulative over the warp's stores (ordered by the warp barrier)
          for (int q = 0; q < a.world; ++q) atomicAdd_system(xch_head_cnt(a.xch[q], a.xl, par, h), 1u);
        }
      } else if (P.n_super == 1) {
        Partial4 F = sink_partial(L, h);
        merge_into(F, S);
        write_attn(h, F);
        if (warp == 0 && lane == 0) stamp(a, step_, layer_, 31);
      } else {
        store_partial(a.supers + (size_t(h) * a.n_super_max + s) * kPartialFloats, S);
      }
    }
  }

  // One rank, several super-chunks: heads 8c + w fold [sink] and the
  // super-chunks in order from the merge slots.
  __device__ void final_phase(const MegaLayer& L, const AttnPlan& P, int step_, int layer_) {
    for (int c = blockIdx.x; c < a.hkv; c += gridDim.x) {
      const int h = c * kHeadsPerKv + warp;
      Partial4 F = sink_partial(L, h);
      for (int s0 = 0; s0 < P.n_super; s0 += kMergeChunk) {
        const int n = min(kMergeChunk, P.n_super - s0);
        const float* st = reinterpret_cast<const float*>(take()) + warp * n * kPartialFloats;
        for (int j = 0; j < n; ++j) merge_into(F, smem_partial(st + j * kPartialFloats));
        release();
      }
      write_attn(h, F);
      if (warp == 0 && lane == 0) stamp(a, step_, layer_, 31);
    }
  }

  __device__ Partial4 smem_partial(const float* p) const {
    Partial4 Q;
    Q.m = p[0];
    Q.l = p[1];
    const float4 v = *reinterpret_cast<const float4*>(p + 4 + 4 * lane);
    Q.a[0] = v.x; Q.a[1] = v.y; Q.a[2] = v.z; Q.a[3] = v.w;
    return Q;
  }
  __device__ Partial4 sink_partial(const MegaLayer& L, int h) const {
    Partial4 F = empty_partial();
    if (L.sinks) {
      F.m = bf(L.sinks[h]);
      F.l = 1.0f;
    }
    return F;
  }

  // world > 1: send this rank's expert slots of rows [o0, o1) to every other
  // rank, then take the other ranks' slots from this rank's exchange buffer.
  // All consumer warps call it; false when a bounded wait ran out.
  __device__ bool exchange_down(const Part& P, int n, int par) {
    const int t = threadIdx.x - 32, nt = kMegaCons * 32;
    const int nl = sm.n_loc;
    uint8_t* own = a.xch[a.rank];
    const int n2 = n / 2;  // rows as bf16 pairs (n and P.o0 are even)
    for (int q = 0; q < a.world; ++q) {
      if (q == a.rank) continue;
      for (int idx = t; idx < nl * n2; idx += nt) {
        const int j = idx / n2, i = 2 * (idx - j * n2);
        const int rr = sm.loc[j];
        *reinterpret_cast<uint32_t*>(xch_xd(a.xch[q], a.xl, par, rr) + P.o0 + i) =
            uint32_t(to_bf(sm.dsm[rr][i])) | (uint32_t(to_bf(sm.dsm[rr][i + 1])) << 16);
      }
    }
    cons_sync();
    if (t == 0) {
      __threadfence_system();  // cumulative over the consumers' stores (ordered by the barrier)
      for (int q = 0; q < a.world; ++q)
        if (q != a.rank) atomicAdd_system(xch_xcnt(a.xch[q], a.xl, par, blockIdx.x), 1u);
      unsigned* c = xch_xcnt(own, a.xl, par, blockIdx.x);
      bool ok = true;
      uint32_t spins = 0;
      while (true) {
        const bool ab = aborted(a);
        if (ld_acquire_sys(c) >= unsigned(a.world - 1)) break;
        if (ab) { ok = false; break; }
        if (++spins > kPeerSpinLimit) {
          set_abort(a, kStatusCounterTimeout);
          ok = false;
          break;
        }
      }
      if (ok) *reinterpret_cast<volatile unsigned*>(c) = 0u;
      sm.xok = ok ? 1 : 0;
    }
    cons_sync();
    if (!sm.xok) return false;
    for (int idx = t; idx < a.k * n; idx += nt) {
      const int rr = idx / n, i = idx - rr * n;
      bool mine = false;
      for (int j = 0; j < nl; ++j) mine = mine || sm.loc[j] == rr;
      if (!mine)
        sm.dsm[rr][i] = bf(__ldcg(reinterpret_cast<const unsigned short*>(xch_xd(own, a.xl, par, rr) + P.o0 + i)));
    }
    cons_sync();
    return true;
  }

  __device__ __noinline__ void write_attn(int h, const Partial4& F) {
    uint2 o;
    o.x = uint32_t(to_bf(__fdiv_rn(F.a[0], F.l))) | (uint32_t(to_bf(__fdiv_rn(F.a[1], F.l))) << 16);
    o.y = uint32_t(to_bf(__fdiv_rn(F.a[2], F.l))) | (uint32_t(to_bf(__fdiv_rn(F.a[3], F.l))) << 16);
    *reinterpret_cast<uint2*>(a.attn + h * 128 + 4 * lane) = o;
  }

  // world > 1: heads h = blockIdx.x (mod grid) wait for every rank's
  // super-chunk partials of this layer, then merge them in order.  Warp 0.
  __device__ bool attn_final_sharded(const MegaLayer& L, const AttnPlan& P, int par) {
    for (int h = blockIdx.x; h < a.hq; h += gridDim.x) {
      unsigned* cnt = xch_head_cnt(a.xch[a.rank], a.xl, par, h);
      uint32_t spins = 0;
      bool ok = true;
      if (lane == 0) {
        while (true) {
          const bool ab = aborted(a);
          if (ld_acquire_sys(cnt) >= unsigned(P.n_super)) break;
          if (ab) { ok = false; break; }
          if (++spins > kPeerSpinLimit) {
            set_abort(a, kStatusCounterTimeout);
            ok = false;
            break;
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) return false;
      __syncwarp();
      Partial4 F = empty_partial();
      if (L.sinks) {
        F.m = bf(L.sinks[h]);
        F.l = 1.0f;
      }
      const Partial4 none = empty_partial();
      merge_range(F, xch_super(a.xch[a.rank], a.xl, par, h, 0), 0, P.n_super, -1, none);
      write_attn(h, F);
      __syncwarp();
      if (lane == 0) *reinterpret_cast<volatile unsigned*>(cnt) = 0u;
    }
    return true;
  }

  // Merges partials [i0, i1) of a [*, kPartialFloats] array into P in order;
  // entry `own` is taken from registers.  Chunks of 4 partials are copied
  // into this warp's shared staging with cp.async (all in flight together),
  // then merged from shared memory.  Callers keep the other warps away from
  // the staging (it overlays the attention scratch).
  __device__ void merge_range(Partial4& P, const float* base, int i0, int i1, int own, const Partial4& own_p) {
    constexpr int kChunk = 4;
    float(*stage)[kPartialFloats] = sm.att.u.stage[warp];
    for (int i = i0; i < i1; i += kChunk) {
      const int n = min(kChunk, i1 - i);
      for (int j = 0; j < n; ++j) {
        if (i + j == own) continue;
        const float* src = base + size_t(i + j) * kPartialFloats;
        cp_async_cg16(&stage[j][4 + 4 * lane], src + 4 + 4 * lane);
        if (lane == 0) cp_async_cg16(&stage[j][0], src);  // m, l, pad, pad
      }
      cp_async_wait_all();
      __syncwarp();
      for (int j = 0; j < n; ++j) {
        if (i + j == own) {
          merge_into(P, own_p);
          continue;
        }
        Partial4 Q;
        Q.m = stage[j][0];
        Q.l = stage[j][1];
        const float4 v = *reinterpret_cast<const float4*>(&stage[j][4 + 4 * lane]);
        Q.a[0] = v.x; Q.a[1] = v.y; Q.a[2] = v.z; Q.a[3] = v.w;
        merge_into(P, Q);
      }
      __syncwarp();
    }
  }

  // Waits (thread 32, bounded) until the producer warp has published this
  // layer's selection (route_ll); the timeline slot of phase 3 records the
  // wait.  Returns false on abort.
  __device__ bool wait_route(int seq, unsigned idx) {
    __shared__ int ok_route;
    if (threadIdx.x == 32) {
      if (a.prof) a.prof[(size_t(idx) * gridDim.x + blockIdx.x) * 2] = globaltimer();
      int ok = 1;
      uint32_t spins = 0;
      while (sm.route_seq < seq) {
        if (aborted_every8(a, spins)) { ok = 0; break; }
        if (++spins > kSpinLimit * 4) {
          set_abort(a, kStatusCounterTimeout);
          ok = 0;
          break;
        }
      }
      __threadfence_block();
      if (a.prof) a.prof[(size_t(idx) * gridDim.x + blockIdx.x) * 2 + 1] = globaltimer();
      ok_route = ok;
    }
    cons_sync();
    return ok_route != 0;
  }

  template <int I, int BITS>
  __device__ void run() {
    const Part P = partition(a);
    int token = sm.token0;
    const int pos0 = sm.pos0;
    const int H = a.H;
    float best = -INFINITY;
    int best_i = 0x7fffffff;
    for (int step = 0; step < a.steps; ++step) {
      const int pos = pos0 + step;
      const AttnPlan AP = attn_plan(a, pos);
      // embedding (every CTA, for its own layer-0 norm); owners publish rows
      if (a.seg != kSegAll && a.seg >= 0) {
        // a later segment of the step: this CTA's rows of h from the
        // previous segment (same partition)
        for (int i = threadIdx.x - 32; i < P.o1 - P.o0; i += kMegaCons * 32) sm.hown[i] = __ldcg(a.h + P.o0 + i);
        cons_sync();
      } else {
        const int tok = (token >= 0 && token < a.V) ? token : 0;
        if (tok != token && blockIdx.x == 0 && warp == 0 && lane == 0) report(a.ctl + 0, kStatusBadToken);
        const uint32_t* w = a.embed.w + size_t(tok) * (H / 8);
        for (int i = threadIdx.x - 32; i < H; i += kMegaCons * 32) {
          const float q = float((w[i >> 3] >> (4 * (i & 7))) & 15u);
          const float s = sb<2>(a.embed.s[size_t(tok) * (H / 64) + (i >> 6)], a.sd);
          const float bb = sb<2>(a.embed.b[size_t(tok) * (H / 64) + (i >> 6)], a.sd);
          const uint16_t v = to_bf(__fmaf_rn(s, q, bb));
          sm.h0[i] = v;
          if (i >= P.o0 && i < P.o1) {
            a.h[i] = v;
            sm.hown[i - P.o0] = v;
          }
          if (blockIdx.x == 0) a.trace[i] = v;
        }
        cons_sync();
      }
      const bool attn_in = a.seg == kSegAll;
      for (int l = seg_l0(a); l < seg_l1(a); ++l) {
        const MegaLayer& L = sm.layers[l];
        // ---- Q
        if (seg_q(a, l)) {
          const FixScale fq = norm(l == 0 ? sm.h0 : a.h, L.input_norm, l == 0);
          GroupX gx[1];
          share_limbs(sm.xn, 32, fq);
          load_limbs(sm.xn, sm.gX, 32, lane, gx[0], lane_half(lane));
          const int qrows[3] = {a.hq * 128, a.hkv * 128, a.hkv * 128};
          for (int r = P.q0; r < P.q1;) {
            int m = 0, base = 0;
            while (m < 2 && r >= base + qrows[m]) base += qrows[m++];
            const int n = min(min(kQRows, P.q1 - r), base + qrows[m] - r);
            const uint8_t* st = take();
            rows2048<false>(st, n, r, gx, fq, a.qkv, best, best_i);
            release();
            r += n;
          }
          if (!attn_in) continue;  // a segment ends with Q: attention runs as separate kernels
          if (!gbar(bar_index(a, step, l, 0))) return;
        }
        // ---- A
        if (attn_in) {
        if (warp == 0 && lane == 0) stamp(a, step, l, 11);
        if (warp == 0 && lane == 0) sm.att.qg = -1;  // queries change every layer
        cons_sync();
        for (int it = blockIdx.x; it < AP.items; it += gridDim.x) {
          int g, item;
          attn_coords(AP, a.hkv, it, g, item);
          if (warp == 0 && lane == 0) stamp(a, step, l, 12);
          attn_item<BITS>(L, AP, pos, g, item, step, l);
          if (warp == 0 && lane == 0) stamp(a, step, l, 13);
        }
        if (!short_merge(a, AP)) {
          // item partials -> super-chunks (-> output); the producer stages
          // the partials into the ring once every CTA has stored its items
          const int seq = 2 * (step * a.n_layers + l);
          if (!gbar(kNoStamp)) return;
          if (warp == 0 && lane == 0) {
            sm.merge_seq = seq + 1;
            stamp(a, step, l, 26);
          }
          merge_phase<BITS>(L, AP, step, l);
          if (warp == 0 && lane == 0) stamp(a, step, l, 27);
          if (AP.n_super > 1 && a.world == 1) {
            if (!gbar(kNoStamp)) return;
            if (warp == 0 && lane == 0) {
              sm.merge_seq = seq + 2;
              stamp(a, step, l, 28);
            }
            final_phase(L, AP, step, l);
          }
        }
        if (a.world > 1 && warp == 0) attn_final_sharded(L, AP, xch_parity(a, step, l));
        if (!gbar(bar_index(a, step, l, 1))) return;
        }
        if (!seg_orgd(a, l)) continue;
        // ---- O
        {
          if (warp == 0 && lane == 0) stamp(a, step, l, 40);
          const FixScale fo = load_x(a.attn, a.hq * 128, step, l);
          if (warp == 0 && lane == 0) stamp(a, step, l, 41);
          GroupX gx[1];
          if (a.hq * 128 == 4096) {
            share_limbs(sm.xn, 64, fo);
            load_limbs(sm.xn, sm.gX, 64, KCfg<4096>::group(warp & 1, lane, 0), gx[0], lane_half(lane));
            for (int r = P.o0; r < P.o1; r += kORows) {
              const int n = min(kORows, P.o1 - r);
              const uint8_t* st = take();
              rows4096(st, n, r, P.o0, gx, fo);
              release();
            }
          } else {
            share_limbs(sm.xn, 32, fo);
            load_limbs(sm.xn, sm.gX, 32, lane, gx[0], lane_half(lane));
            for (int r = P.o0; r < P.o1; r += kORows) {
              const int n = min(kORows, P.o1 - r);
              const uint8_t* st = take();
              rows2048_resid(st, n, r, P.o0, gx, fo);
              release();
            }
          }
          if (warp == 0 && lane == 0) stamp(a, step, l, 42);
        }
        if (!gbar(bar_index(a, step, l, 2))) return;
        // ---- R
        if (warp == 0 && lane == 0) stamp(a, step, l, 43);
        const FixScale fr = norm(a.h, L.post_norm);
        if (warp == 0 && lane == 0) stamp(a, step, l, 44);
        {
          int j = 0;
          for (int e = blockIdx.x; e < a.E; e += gridDim.x, ++j) {
            // the row was staged by the producer; warp j % 8 computes it
            const uint16_t* wrow = reinterpret_cast<const uint16_t*>(take());
            if ((j % kMegaCons) != warp) {
              release();
              continue;
            }
            float acc = 0.0f;
            for (int mm = 0; mm < H / 256; ++mm) {
              const int c = lane + 32 * mm;
              const uint4 wv = *reinterpret_cast<const uint4*>(wrow + c * 8);
              const uint4 xv = *reinterpret_cast<const uint4*>(sm.xn + c * 8);
              const uint32_t ws_[4] = {wv.x, wv.y, wv.z, wv.w};
              const uint32_t xs_[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
              for (int t = 0; t < 4; ++t) {
                acc = __fmaf_rn(__uint_as_float(ws_[t] << 16), __uint_as_float(xs_[t] << 16), acc);
                acc = __fmaf_rn(__uint_as_float(ws_[t] & 0xFFFF0000u), __uint_as_float(xs_[t] & 0xFFFF0000u), acc);
              }
            }
            acc = bfly_sum(acc);
            if (lane == 0) {
              const unsigned flag = route_flag(a, step, l);
              st_relaxed64(a.router_ll + size_t(flag & 1u) * a.E + e,
                           (static_cast<unsigned long long>(flag) << 32) | __float_as_uint(rbf(acc)));
            }
            release();
          }
          if (warp == 0 && lane == 0) stamp(a, step, l, 45);
        }
        // ---- G: the selection (the producer's route_ll), then gate/up pairs
        if (warp == 0 && lane == 0) stamp(a, step, l, 0);
        if (!wait_route(step * a.n_layers + l + 1, bar_index(a, step, l, 3))) return;
        if (warp == 0 && lane == 0) stamp(a, step, l, 1);
        {
          GroupX gx[1];
          share_limbs(sm.xn, 32, fr);
          load_limbs(sm.xn, sm.gX, 32, lane, gx[0], lane_half(lane));
          int g0, g1;
          split_range(sm.n_loc * a.I / 2, gridDim.x, blockIdx.x, g0, g1);
          g0 *= 2;
          g1 *= 2;
          for (int u = g0; u < g1;) {
            const int n = min(kGPairs, g1 - u);  // pairs u .. u + n - 1 (at most two experts)
            const uint8_t* st = take();
            if (warp == 0 && lane == 0) stamp(a, step, l, 2 + 2 * min((u - g0) / kGPairs, 3));
            {
              const uint32_t wb = uint32_t(n) * 1024, sbytes = uint32_t(n) * 64;
              const uint16_t* sbase = reinterpret_cast<const uint16_t*>(st + 2 * wb);
              const uint16_t* bbase = reinterpret_cast<const uint16_t*>(st + 2 * wb + 2 * sbytes);
              // rows: gate i at row i, up i at row n + i (scales likewise)
              const int pa = warp, pc = warp + kMegaCons;
              const bool va = pa < n, vc = pc < n;
              int rows[4] = {va ? pa : 0, va ? n + pa : 0, vc ? pc : 0, vc ? n + pc : 0};
              float v[4];
              lane_rows_partial<2048, 2, 4>(st, sbase, bbase, rows, 0, lane, gx, v, a.sd);
#pragma unroll
              for (int q = 0; q < 4; ++q) v[q] = __fmul_rn(bfly_sum(v[q]), fr.down);
              // pair u + q: selection slot loc[(u + q) / I], row (u + q) % I;
              // lanes 0 and 1 finish pairs pa and pc side by side
              if (lane < 2 && (lane == 0 ? va : vc)) {
                const float gg = rbf(lane == 0 ? v[0] : v[2]), uu = rbf(lane == 0 ? v[1] : v[3]);
                const int gu = u + (lane == 0 ? pa : pc);
                a.act[sm.loc[gu / a.I] * a.I + gu % a.I] =
                    to_bf(__fmul_rn(rbf(__fmul_rn(gg, rbf(rsigmoid(gg)))), uu));
              }
            }
            release();
            if (warp == 0 && lane == 0) stamp(a, step, l, 3 + 2 * min((u - g0) / kGPairs, 3));
            u += n;
          }
        }
        if (warp == 0 && lane == 0) stamp(a, step, l, 10);
        if (!gbar(bar_index(a, step, l, 4))) return;
        // ---- D: down rows of all k experts, mix, residual
        {
          if (warp == 0 && lane == 0) stamp(a, step, l, 39);
          load_vec(sm.act, a.act, a.k * I);
          // per selected expert: fixed-point scale, then the shared limbs
          for (int r = warp; r < a.k; r += kMegaCons) {
            const float m = warp_maxabs(sm.act + r * I, I);
            if (lane == 0) sm.dmax[r] = m;
          }
          cons_sync();
          // limbs into the attention scratch (free during D)
          uint16_t* dl = reinterpret_cast<uint16_t*>(&sm.att.u);
          prep_limbs_to<kMegaCons * 32>(sm.act, dl, sm.gX, a.k * (I / 64), threadIdx.x - 32,
                                        [&](int g) { return fix_scale_from_max(sm.dmax[g / (I / 64)]).up; });
          cons_sync();
          if (warp == 0 && lane == 0) stamp(a, step, l, 33);
          const int n = P.o1 - P.o0;
          const int nl = sm.n_loc;
          if (n > 0) {
            for (int j0 = 0; j0 < nl; j0 += kDExperts) {
              const int j1 = min(nl, j0 + kDExperts);
              const uint8_t* st = take();
              if (warp == 0 && lane == 0 && j0 == 0) stamp(a, step, l, 34);
              // warp w: local expert j0 + (w % 4), rows of half (w / 4)
              const int jj = j0 + (warp % kDExperts), half = warp / kDExperts;
              if (jj < j1) {
                using C = KCfg<I>;
                const int rr = sm.loc[jj];
                const uint32_t wb = uint32_t(n) * (I / 2), sbytes = uint32_t(n) * (I / 32);
                const uint32_t per = wb + 2 * ((sbytes + 15) & ~15u);
                const uint8_t* e0 = st + (jj - j0) * per;
                const uint16_t* sbase = reinterpret_cast<const uint16_t*>(e0 + wb);
                const uint16_t* bbase = reinterpret_cast<const uint16_t*>(e0 + wb + ((sbytes + 15) & ~15u));
                const FixScale fd = fix_scale_from_max(sm.dmax[rr]);
                const int sub = lane >> 2, l4 = lane & 3;  // 8 rows per pass, 4 lanes per row
                const int rbeg = half * ((n + 1) / 2), rend = half == 0 ? (n + 1) / 2 : n;
                for (int rb = rbeg; rb < rend; rb += 8) {
                  int rows[1];
                  const int x = rb + sub;
                  const bool valid = x < rend;
                  rows[0] = valid ? x : rbeg;
                  float v[1];
                  lane_rows_partial_shared<I, 2, 1>(e0, sbase, bbase, rows, l4, dl, sm.gX, a.k * (I / 64),
                                                    rr * (I / 64), v, a.sd);
                  v[0] = bfly_sum<4>(valid ? v[0] : 0.0f);
                  if (valid && l4 == 0) sm.dsm[rr][rows[0]] = rbf(__fmul_rn(v[0], fd.down));
                }
              }
              if (warp == 0 && lane == 0) stamp(a, step, l, j0 == 0 ? 46 : 47);
              release();
            }
            cons_sync();
          }
          if (warp == 0 && lane == 0) stamp(a, step, l, 35);
          if (a.world > 1 && !exchange_down(P, n, xch_parity(a, step, l))) return;
          if (n > 0) {
            for (int i = threadIdx.x - 32; i < n; i += kMegaCons * 32) {
              float mix = 0.0f;
              for (int r = 0; r < a.k; ++r) {
                const float t = __fadd_rn(rbf(__fmul_rn(sm.dsm[r][i], rbf(sm.wts[r]))), 0.0f);
                mix = r == 0 ? t : rbf(__fadd_rn(t, mix));
              }
              const uint16_t hn = to_bf(__fadd_rn(bf(sm.hown[i]), mix));
              sm.hown[i] = hn;
              a.h[P.o0 + i] = hn;
              a.trace[size_t(l + 1) * H + P.o0 + i] = hn;
            }
          }
          if (warp == 0 && lane == 0) stamp(a, step, l, 36);
        }
        if (!gbar(bar_index(a, step, l, 5))) return;
      }
      if (!seg_h(a)) continue;  // a segment that ends before the last layer's D
      // ---- H: final norm + lm_head + CTA argmax
      const FixScale fh = norm(a.h, a.final_norm);
      {
        GroupX gx[1];
        share_limbs(sm.xn, 32, fh);
        load_limbs(sm.xn, sm.gX, 32, lane, gx[0], lane_half(lane));
        best = -INFINITY;
        best_i = 0x7fffffff;
        int v0, v1;
        split_range(a.V / 2, gridDim.x, blockIdx.x, v0, v1);
        v0 *= 2;
        v1 *= 2;
        for (int r = v0; r < v1; r += kQRows) {
          const int n = min(kQRows, v1 - r);
          const uint8_t* st = take();
          rows2048<true>(st, n, r, gx, fh, a.logits, best, best_i);
          release();
        }
        for (int off = 16; off >= 1; off >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, best, off);
          const int oi = __shfl_xor_sync(0xffffffffu, best_i, off);
          if (ov > best || (ov == best && oi < best_i)) { best = ov; best_i = oi; }
        }
        if (lane == 0) {
          sm.best_val[warp] = best;
          sm.best_idx[warp] = best_i;
        }
        cons_sync();
        if (warp == 0 && lane == 0) {
          float bv = sm.best_val[0];
          int bi = sm.best_idx[0];
          for (int w = 1; w < kMegaCons; ++w)
            if (sm.best_val[w] > bv || (sm.best_val[w] == bv && sm.best_idx[w] < bi)) {
              bv = sm.best_val[w];
              bi = sm.best_idx[w];
            }
          a.cand_val[blockIdx.x] = bv;
          a.cand_idx[blockIdx.x] = bi;
        }
      }
      if (!gbar(bar_index(a, step, a.n_layers, 0))) return;
      // ---- E: global argmax (every CTA), bookkeeping (CTA 0)
      if (warp == 0) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int c = lane; c < gridDim.x; c += 32) {
          const float v = __ldcg(a.cand_val + c);
          const int i = __ldcg(a.cand_idx + c);
          if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
        }
        for (int off = 16; off >= 1; off >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
          if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) {
          sm.token = bi;
          if (blockIdx.x == 0 && a.ctl[80]) {
            // sampled packet: the sampler records the id and feeds it back
            a.ctl[7] = bi;
            a.ctl[2] = pos + 1;
            a.ctl[5] += 1;
          } else if (blockIdx.x == 0) {
            int* ctl = a.ctl;
            if (ctl[3]) {  // active
              if (ctl[5] < 64) ctl[16 + ctl[5]] = bi;
              ctl[4] += 1;
              for (int i = 0; i < ctl[6]; ++i)
                if (ctl[8 + i] == bi) ctl[3] = 0;
            }
            ctl[7] = bi;
            ctl[1] = bi;
            ctl[2] = pos + 1;
            ctl[5] += 1;
          }
        }
      }
      cons_sync();
      token = sm.token;
    }
  }
};

template <int I, int BITS>
// 168 registers per thread at most: the register file is split over the
// SM's four schedulers, and nine warps put three on one of them
// (3 x 32 x 170 <= 16,384).  The code is written to that budget.
__global__ void __launch_bounds__(kMegaThreads, 1) k_decode_mega(const MegaArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  MegaSmem& sm = *reinterpret_cast<MegaSmem*>(smem_raw);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kMegaCons);
    }
    sm.route_seq = 0;
    sm.merge_seq = 0;
    mbar_init(&sm.mfull, 1);
    sm.mpar = 0;
    sm.token0 = a.ctl[1];
    sm.pos0 = a.ctl[2];
    fence_barrier_init();
  }
  {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(a.layers);
    uint32_t* dst = reinterpret_cast<uint32_t*>(sm.layers);
    // the layers this launch runs (all of them, or a segment's one or two)
    constexpr int per = int(sizeof(MegaLayer) / 4);
    for (int i = seg_l0(a) * per + threadIdx.x; i < seg_l1(a) * per; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    Producer p(a, sm);
    p.run();
  } else {
    Consumers c(a, sm);
    c.template run<I, BITS>();
  }
}

}  // namespace rec
