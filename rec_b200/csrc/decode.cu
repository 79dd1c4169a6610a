// Decode session: workspace layout, the per-token launch sequence (captured
// once into a CUDA graph) and the session entry points of the C ABI.
//
// Replaces FullModel.forward / ResidentSampler.block of the reference
// (engine/src/rec_mlx/kernels/megakernel.py:1224-1301, sampling.py:62-169):
// one persistent Metal dispatch with ~390 software grid barriers per token
// becomes a graph of ~7 kernels per layer chained with programmatic
// dependent launch, so each kernel streams its weights while the previous one
// finishes.
#include <cmath>
#include <cstring>
#include <mutex>
#include <set>
#include <vector>

#include <cstdlib>

#include "attn.cuh"
#include "attn_bf16.cuh"
#include "attn_shard.cuh"
#include "capi_common.h"
#include "mega.cuh"
#include "moe.cuh"
#include "prefill_layer.h"
#include "sample.cuh"

namespace rec {

// --- control block (device ints) ---------------------------------------------
enum Ctrl : int {
  kCtlStatus = 0,
  kCtlToken = 1,
  kCtlPosition = 2,
  kCtlActive = 3,
  kCtlProduced = 4,
  kCtlStep = 5,
  kCtlNEos = 6,
  kCtlArgmax = 7,
  kCtlEos = 8,       // 8 slots
  kCtlRecorded = 16, // 64 slots: ids produced by the current packet
  kCtlSampled = 80,  // 1: a sampled packet; the sampler feeds the next token back
  kCtlSeq = 81,      // steps completed since the workspace was set (exchange parity of sharded graph steps)
  kCtlInts = 96,
};
constexpr int kMaxPacket = 64;
constexpr int kMaxEos = 8;

// token < 0: continue from the token and position held on the device.
__global__ void k_set_step(int* ctl, int token, int position, int n_eos, const int4 eos_lo, const int4 eos_hi,
                           int sampled) {
  if (threadIdx.x == 0) {
    ctl[kCtlSampled] = sampled;
    if (token >= 0) {
      ctl[kCtlToken] = token;
      ctl[kCtlPosition] = position;
    }
    ctl[kCtlActive] = 1;
    ctl[kCtlProduced] = 0;
    ctl[kCtlStep] = 0;
    ctl[kCtlNEos] = n_eos;
    const int e[8] = {eos_lo.x, eos_lo.y, eos_lo.z, eos_lo.w, eos_hi.x, eos_hi.y, eos_hi.z, eos_hi.w};
    for (int i = 0; i < kMaxEos; ++i) ctl[kCtlEos + i] = e[i];
  }
}

// Embedding row (int4 or int8 g64): h = bf16(fma(scale, q, bias)).  Also the
// first trace row.  Reference megakernel.py:850-860 (int4), mixed_bits.py:25-30
// (the production checkpoint's int8 codes).
template <int SD>
__global__ void __launch_bounds__(256) k_embed(int* ctl, QMatDev emb, int H, int V, int capacity, int token_base,
                                               uint16_t* h, uint16_t* trace, int bits) {
  int tok = ctl[kCtlToken];
  const int pos = ctl[kCtlPosition];
  if (tok < 0 || tok >= V) {
    if (threadIdx.x == 0) report(ctl + kCtlStatus, kStatusBadToken);
    tok = 0;
  }
  if ((pos < 0 || pos - token_base >= capacity) && threadIdx.x == 0) report(ctl + kCtlStatus, kStatusBadPosition);
  grid_launch_dependents();
  const uint32_t* w = emb.w + size_t(tok) * (H * bits / 32);
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float q = bits == 8 ? float((w[i >> 2] >> (8 * (i & 3))) & 255u) : float((w[i >> 3] >> (4 * (i & 7))) & 15u);
    const float s = sb<SD>(emb.s[size_t(tok) * (H / 64) + (i >> 6)]);
    const float b = sb<SD>(emb.b[size_t(tok) * (H / 64) + (i >> 6)]);
    const uint16_t v = to_bf(__fmaf_rn(s, q, b));
    h[i] = v;
    trace[i] = v;
  }
}

// End of a step: record the argmax, stop after EOS, advance the position.
__global__ void k_step_end(int* ctl) {
  grid_wait();
  if (threadIdx.x == 0) ctl[kCtlSeq] += 1;
  if (threadIdx.x == 0) {
    const int t = ctl[kCtlArgmax];
    const int step = ctl[kCtlStep];
    if (ctl[kCtlSampled]) {  // the sampler records the id and feeds it back
      ctl[kCtlPosition] += 1;
      ctl[kCtlStep] = step + 1;
      return;
    }
    if (ctl[kCtlActive]) {
      if (step < kMaxPacket) ctl[kCtlRecorded + step] = t;
      ctl[kCtlProduced] += 1;
      for (int i = 0; i < ctl[kCtlNEos]; ++i)
        if (ctl[kCtlEos + i] == t) ctl[kCtlActive] = 0;
    }
    ctl[kCtlToken] = t;
    ctl[kCtlPosition] += 1;
    ctl[kCtlStep] = step + 1;
  }
}

// --- launch helper ----------------------------------------------------------------
template <typename Kern, typename... Args>
cudaError_t launch(Kern kern, dim3 grid, int block, size_t smem, cudaStream_t st, bool pdl, Args... args) {
  if (smem > 48 * 1024) {
    cudaError_t e = set_smem_limit(reinterpret_cast<const void*>(kern), smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

}  // namespace rec

// ------------------------------------------------------------------------------
// Session
// ------------------------------------------------------------------------------
using namespace rec;

struct RecCtx {
  RecModelDesc d;
  std::vector<RecLayerWeights> layers;
  RecGlobalWeights g = {};
  bool has_weights = false;
  std::vector<RecKVLayer> kv;
  int capacity = 0;
  int token_base = 0;       // split-KV: first position held by this rank
  int block_begin = 0, block_end = 1 << 30;
  // one session over several GPUs (rec_set_shard)
  int world = 1, rank = 0, e_lo = 0, e_hi = 0, super_lo = 0, super_hi = 0, cap_total = 0;
  bool shard_graph = false;  // a split session on the graph schedule (RecShard.schedule), fixed for its lifetime
  uint8_t* xch[kMaxWorld] = {};
  unsigned layer_seq = 0;  // layer steps run so far (exchange parity)
  uint8_t* ws = nullptr;
  size_t ws_bytes = 0;
  bool usable = true;
  // workspace views
  int* ctl = nullptr;
  unsigned* counters = nullptr;
  uint16_t *h = nullptr, *qkv = nullptr, *attn = nullptr, *xn = nullptr, *act = nullptr, *logits = nullptr,
           *trace = nullptr;
  // Flint layer options (a shared expert, dense-MLP / NoPE / sliding layers):
  // the model runs on the graph schedule
  bool flint = false;
  uint16_t *act_shared = nullptr, *d_shared = nullptr;  // shared expert activations and output
  int* one_id = nullptr;     // device constant {0}: the single "expert" of a dense MLP or shared expert
  float* one_wt = nullptr;   // device constant {1.0f}
  float *router_logits = nullptr, *wts = nullptr, *cand_val = nullptr, *partials = nullptr, *supers = nullptr,
        *rope = nullptr;
  int *ids = nullptr, *cand_idx = nullptr;
  int n_super_max = 0;
  int grid = 148;
  cudaStream_t cap_stream = nullptr;
  cudaGraphExec_t step_exec = nullptr;
  // persistent schedule
  int sched = 0;  // kSchedMega / kSchedGraph / kSchedSplit of the current call
  MegaLayer* mega_layers = nullptr;  // device table, in the workspace
  unsigned long long* router_ll = nullptr;  // [2][E] flag+value router logits of the persistent kernel
  unsigned* mega_cnt = nullptr;      // [2] grid barrier + abort, [Hq] heads, [Hq*n_super] supers
  unsigned long long* prof = nullptr;  // optional phase timeline
  size_t prof_entries = 0;
  unsigned long long* prof2 = nullptr;  // optional stamps inside one layer
  int prof_layer = -1;
  int kv_rows = 0;     // cache rows backed by memory (rec_set_kv_rows; <= capacity, the head stride)
  int rope_done = 0;   // RoPE table rows filled (the table grows with kv_rows)
  int layers_run = 0;  // > 0: the current call runs only the first layers_run layers (rec_decode_layers)
  // failure-path tests (rec_set_fault_injection): the grid barrier's poll
  // bound, and one CTA that never arrives at a grid barrier (-1: none)
  uint32_t bar_spin_limit = kSpinLimit * 4;
  int skip_arrive_cta = -1;
};

namespace {

constexpr int kSuperTokens = kAttBlock * kAttSuper;  // tokens per super-chunk

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

enum { kSchedMega = 0, kSchedGraph = 1, kSchedSplit = 2 };

struct Layout {
  size_t off[24];
  size_t total;
};

enum Region {
  rCtl, rCounters, rMegaCnt, rRouterLL, rH, rQkv, rAttn, rXn, rAct, rLogits, rTrace, rRouter, rIds, rWts, rCandV, rCandI,
  rPartials, rSupers, rMegaLayers, rRope, rFlint, rCount
};

// Positions the RoPE table covers: the local cache, or the whole context when
// the session is split over ranks (every rank rotates every query).
int rope_rows(const RecCtx* c) { return c->world > 1 ? c->cap_total : c->capacity; }

Layout layout_of(const RecCtx* c) {
  const RecModelDesc& d = c->d;
  const int grid = c->grid;
  const int nblk = c->capacity / kAttBlock;
  const int nsup = (nblk + kAttSuper - 1) / kAttSuper;
  size_t sz[rCount];
  sz[rCtl] = kCtlInts * 4;
  sz[rCounters] = (64 + d.n_q_heads) * 4;
  sz[rMegaCnt] = size_t(2 + d.n_q_heads + d.n_q_heads * nsup) * 4;
  sz[rRouterLL] = size_t(2) * d.n_experts * 8;  // zeroed with the control block
  sz[rMegaLayers] = size_t(d.n_layers) * sizeof(MegaLayer);
  sz[rH] = size_t(d.hidden) * 2;
  sz[rQkv] = size_t(d.n_q_heads + 2 * d.n_kv_heads) * 128 * 2;
  sz[rAttn] = size_t(d.n_q_heads) * 128 * 2;
  sz[rXn] = size_t(d.hidden) * 2;
  // routed activations, then the shared expert's; a dense MLP's in the same space
  sz[rAct] = std::max(size_t(d.top_k) * d.moe_inter + size_t(d.shared_inter), size_t(d.dense_inter)) * 2;
  sz[rLogits] = size_t(d.vocab) * 2;
  sz[rTrace] = size_t(d.n_layers + 1) * d.hidden * 2;
  sz[rRouter] = size_t(d.n_experts) * 4;
  sz[rIds] = kMaxTopK * 4;
  sz[rWts] = kMaxTopK * 4;
  sz[rCandV] = size_t(grid) * 4;
  sz[rCandI] = size_t(grid) * 4;
  sz[rPartials] = size_t(d.n_q_heads) * nblk * kPartialFloats * 4;
  sz[rSupers] = size_t(d.n_q_heads) * nsup * kPartialFloats * 4;
  sz[rRope] = size_t(rope_rows(c)) * 128 * 4;
  sz[rFlint] = size_t(d.hidden) * 2 + 16;  // shared expert output bf16 [H], then {0} and {1.0f}
  Layout L;
  size_t o = 0;
  for (int i = 0; i < rCount; ++i) {
    L.off[i] = o;
    o = align_up(o + sz[i], 256);
  }
  L.total = o;
  return L;
}

// Kernels of one decode step, in launch order (per layer: kKQkv..kKDown; a
// layer with a shared expert runs kKSharedDown between kKGateUp, which also
// takes the shared expert's gate/up pairs, and kKDown; kKSharedGateUp runs
// those pairs alone, for timing).
enum KernelKind { kKEmbed = 0, kKQkv, kKAttn, kKCombine, kKOproj, kKRouter, kKGateUp, kKDown, kKHead, kKStepEnd,
                  kKCount, kKSharedGateUp = kKCount, kKSharedDown, kKAll };

bool layer_dense(const RecCtx* c, int li) { return (c->layers[li].kind & REC_LAYER_DENSE) != 0; }
bool layer_shared(const RecCtx* c, int li) { return c->d.shared_inter > 0 && !layer_dense(c, li); }
// The routed k_down computes the shared expert's down rows itself (one warp
// beside the k routed ones): k < 8 and a shared intermediate it is built for.
bool shared_down_fused(const RecCtx* c, int li) {
  return layer_shared(c, li) && c->d.top_k < kMaxTopK && (c->d.shared_inter == 512 || c->d.shared_inter == 1024);
}

// The routed down + mix kernel for intermediate I, with the shared expert's
// down rows fused when is > 0.
template <int SD, int I>
cudaError_t launch_down(const DownArgs& a, int dgrid, int is, cudaStream_t st, bool pdl) {
  switch (is) {
    case 0: return launch(k_down<I, SD>, dgrid, kThreads, sizeof(DownSmem<I>), st, pdl, a);
    case 512: return launch(k_down<I, SD, 512>, dgrid, kThreads, down_smem_bytes<I, 512>(), st, pdl, a);
    case 1024: return launch(k_down<I, SD, 1024>, dgrid, kThreads, down_smem_bytes<I, 1024>(), st, pdl, a);
    default: return cudaErrorInvalidValue;
  }
}

template <int SD>
cudaError_t enqueue_kernel_sd(RecCtx* c, int kind, int li, cudaStream_t st, bool pdl) {
  const RecModelDesc& d = c->d;
  const int H = d.hidden;
  const int grid = c->grid;
  // the gate/up kernel fits two CTAs per SM (85 registers, 115 KB of shared
  // memory): twice the warps to hide its latency (7.5 vs 8.0 us at config 3).
  // The GEMV kernels do not (a second wave: slower)
  const int grid2 = 2 * grid;
  cudaError_t e = cudaSuccess;
  int* status = c->ctl + kCtlStatus;
  if (kind == kKEmbed)  // a split session checks the position against the whole context
    return launch(k_embed<SD>, 1, 256, 0, st, false, c->ctl, QMatDev{(const uint32_t*)c->g.embed.w,
                  (const uint16_t*)c->g.embed.scales, (const uint16_t*)c->g.embed.biases}, H, d.vocab,
                  c->world > 1 ? c->cap_total : c->capacity, c->world > 1 ? 0 : c->token_base, c->h, c->trace,
                  d.embed_bits == 8 ? 8 : 4);
  if (kind == kKStepEnd) return launch(k_step_end, 1, 32, 0, st, pdl, c->ctl);
  if (kind != kKHead) {
    const RecLayerWeights& L = c->layers[li];
    const RecKVLayer& kv = c->kv[li];
    switch (kind) {
    case kKQkv: {  // RMSNorm + QKV projection
      GemvArgs a = {};
      a.mat[0] = {(const uint32_t*)L.q.w, (const uint16_t*)L.q.scales, (const uint16_t*)L.q.biases};
      a.mat[1] = {(const uint32_t*)L.k.w, (const uint16_t*)L.k.scales, (const uint16_t*)L.k.biases};
      a.mat[2] = {(const uint32_t*)L.v.w, (const uint16_t*)L.v.scales, (const uint16_t*)L.v.biases};
      a.rows[0] = d.n_q_heads * 128;
      a.rows[1] = d.n_kv_heads * 128;
      a.rows[2] = d.n_kv_heads * 128;
      a.total_rows = a.rows[0] + a.rows[1] + a.rows[2];
      a.x = c->h;
      a.norm_w = (const uint16_t*)L.input_norm;
      a.eps = d.rms_eps;
      a.out = c->qkv;
      a.status = status;
      a.pdl = pdl;
      using Kq = GemvSmem<2048, gemv_rs<2048>(), 3>;
      e = launch(k_gemv<2048, SD, gemv_rs<2048>(), 3, kEpiStore>, grid, kThreads, sizeof(Kq), st, pdl, a);
      return e;
    }
    case kKAttn:
    case kKCombine: {  // attention partials (+ RoPE, quantize-on-append) / combine
      AttnArgs a = {};
      a.qkv = c->qkv;
      a.k_codes = (uint32_t*)kv.k_codes;
      a.k_scales = (uint16_t*)kv.k_scales;
      a.k_biases = (uint16_t*)kv.k_biases;
      a.v_codes = (uint32_t*)kv.v_codes;
      a.v_scales = (uint16_t*)kv.v_scales;
      a.v_biases = (uint16_t*)kv.v_biases;
      a.capacity = c->capacity;
      a.token_base = c->world > 1 ? c->token_base : 0;
      a.super_lo = c->world > 1 ? c->super_lo : 0;
      a.super_hi = c->world > 1 ? c->super_hi : kAttAllSupers;
      a.hq = d.n_q_heads;
      a.hkv = d.n_kv_heads;
      a.rope = (L.kind & REC_LAYER_NO_ROPE) ? nullptr : c->rope;
      a.window = (L.kind & REC_LAYER_SLIDING) ? d.sliding_window : 0;
      a.q_norm = (d.flags & REC_FLAG_QK_NORM) ? (const uint16_t*)L.q_norm : nullptr;
      a.k_norm = (d.flags & REC_FLAG_QK_NORM) ? (const uint16_t*)L.k_norm : nullptr;
      a.eps = d.rms_eps;
      a.position = c->ctl + kCtlPosition;
      a.partials = c->partials;
      a.supers = c->supers;
      a.head_counters = c->counters + 2;
      a.out = c->attn;
      a.sinks = (d.flags & REC_FLAG_SINKS) ? (const uint16_t*)L.sinks : nullptr;
      a.n_super_max = c->n_super_max;
      a.status = status;
      a.pdl = pdl;
      const int agrid = sm_count() * (d.kv_bits == 4 ? 2 : 1);  // 4-bit stages fit two CTAs per SM
      if (kind == kKAttn && d.kv_bits == 16)  // a bf16 cache: one block of K and V rows per CTA
        return launch(k_attn_partial_bf16, sm_count(), kAttWarps * 32, sizeof(AttnBfSmem), st, pdl, a);
      const int vbits = d.kv_value_bits ? d.kv_value_bits : d.kv_bits;
      if (kind == kKAttn && vbits != d.kv_bits)  // a mixed cache (K and V codes of different widths)
        return d.kv_bits == 8
                   ? launch(k_attn_partial<8, 4>, sm_count(), kAttWarps * 32, sizeof(AttnSmem<8, 4>), st, pdl, a)
                   : launch(k_attn_partial<4, 8>, sm_count(), kAttWarps * 32, sizeof(AttnSmem<4, 8>), st, pdl, a);
      if (kind == kKAttn)
        return d.kv_bits == 4 ? launch(k_attn_partial<4>, agrid, kAttWarps * 32, sizeof(AttnSmem<4>), st, pdl, a)
                              : launch(k_attn_partial<8>, agrid, kAttWarps * 32, sizeof(AttnSmem<8>), st, pdl, a);
      if (c->world > 1) {
        // this rank's super-chunks to every rank, then the in-order merge
        AttnXchArgs x = {};
        x.partials = c->partials;
        x.capacity = c->capacity;
        x.token_base = c->token_base;
        x.super_lo = c->super_lo;
        x.super_hi = c->super_hi;
        x.position = c->ctl + kCtlPosition;
        x.seq = c->ctl + kCtlSeq;
        x.layer = li;
        x.n_layers = d.n_layers;
        x.world = c->world;
        x.rank = c->rank;
        x.hq = d.n_q_heads;
        for (int q = 0; q < kMaxWorld; ++q) x.xch[q] = c->xch[q];
        x.xl = xch_layout(d.n_q_heads, (c->cap_total + kSuperTokens - 1) / kSuperTokens, H);
        x.sinks = a.sinks;
        x.out = c->attn;
        x.status = status;
        x.pdl = pdl;
        const int local = std::max(1, c->super_hi - c->super_lo);
        return launch(k_attn_combine_xch, dim3(d.n_q_heads, local), 32, 0, st, pdl, x);
      }
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(d.n_q_heads, std::max(1, c->n_super_max));
      cfg.blockDim = dim3(32);
      cfg.stream = st;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      return cudaLaunchKernelEx(&cfg, k_attn_combine, a);
    }
    case kKOproj: {  // O projection + residual
      GemvArgs a = {};
      a.mat[0] = {(const uint32_t*)L.o.w, (const uint16_t*)L.o.scales, (const uint16_t*)L.o.biases};
      a.rows[0] = H;
      a.total_rows = H;
      a.x = c->attn;
      a.resid = c->h;
      a.status = status;
      a.pdl = pdl;
      if (d.n_q_heads * 128 == 4096) {
        using Ko = GemvSmem<4096, gemv_rs<4096>(), 3>;
        e = launch(k_gemv<4096, SD, gemv_rs<4096>(), 3, kEpiResidual>, grid, kThreads, sizeof(Ko), st, pdl, a);
      } else {
        using Ko = GemvSmem<2048, gemv_rs<2048>(), 3>;
        e = launch(k_gemv<2048, SD, gemv_rs<2048>(), 3, kEpiResidual>, grid, kThreads, sizeof(Ko), st, pdl, a);
      }
      return e;
    }
    case kKRouter: {
      RouterArgs a = {};
      a.h = c->h;
      a.norm_w = (const uint16_t*)L.post_norm;
      a.eps = d.rms_eps;
      a.w = (const uint16_t*)L.router;
      a.expert_bias = (const float*)L.expert_bias;
      a.E = d.n_experts;
      a.k = d.top_k;
      a.mode = d.router_mode;
      a.logits = c->router_logits;
      a.xn_out = c->xn;
      a.ids = c->ids;
      a.wts = c->wts;
      a.counter = c->counters + 1;
      a.status = status;
      a.pdl = pdl;
      if (layer_dense(c, li)) {  // a dense MLP: the post-attention norm only (no router rows to read)
        a.norm_only = 1;
        a.w = nullptr;
        a.E = 0;
        return launch(k_router<2048>, 1, kThreads, sizeof(RouterSmem<2048>), st, pdl, a);
      }
      e = launch(k_router<2048>, (d.n_experts + kWarps - 1) / kWarps, kThreads, sizeof(RouterSmem<2048>), st, pdl, a);
      return e;
    }
    case kKGateUp:         // experts gate/up + SwiGLU (a dense layer: its MLP as one "expert"; a
                           // shared expert's pairs follow the routed ones in the same launch)
    case kKSharedGateUp: {  // the shared expert's gate/up alone (diagnostics: rec_launch_kernel)
      const bool one = kind == kKSharedGateUp || layer_dense(c, li);
      const RecQMat& G = kind == kKSharedGateUp ? L.shared_gate : L.gate;
      const RecQMat& U = kind == kKSharedGateUp ? L.shared_up : L.up;
      GateUpArgs a = {};
      a.gate = {(const uint32_t*)G.w, (const uint16_t*)G.scales, (const uint16_t*)G.biases};
      a.up = {(const uint32_t*)U.w, (const uint16_t*)U.scales, (const uint16_t*)U.biases};
      a.xn = c->xn;
      a.ids = one ? c->one_id : c->ids;
      a.k = one ? 1 : d.top_k;
      a.I = kind == kKSharedGateUp ? d.shared_inter : (layer_dense(c, li) ? d.dense_inter : d.moe_inter);
      a.expert_lo = c->world > 1 && !one ? c->e_lo : 0;
      a.expert_hi = one ? 1 : (c->world > 1 ? c->e_hi : d.n_experts);
      a.act = kind == kKSharedGateUp ? c->act_shared : c->act;
      if (kind == kKGateUp && layer_shared(c, li)) {  // act_shared = act + k * I: rank k of the same units
        a.sgate = {(const uint32_t*)L.shared_gate.w, (const uint16_t*)L.shared_gate.scales,
                   (const uint16_t*)L.shared_gate.biases};
        a.sup = {(const uint32_t*)L.shared_up.w, (const uint16_t*)L.shared_up.scales,
                 (const uint16_t*)L.shared_up.biases};
        a.Is = d.shared_inter;
      }
      a.status = status;
      a.pdl = pdl;
      constexpr int RSP = 16;
      e = launch(k_gateup<SD, RSP, 3>, grid2, kThreads, sizeof(GateUpSmem<RSP, 3>), st, pdl, a);
      return e;
    }
    case kKSharedDown: {  // the shared expert's down projection into d_shared
      DownArgs a = {};
      a.down = {(const uint32_t*)L.shared_down.w, (const uint16_t*)L.shared_down.scales,
                (const uint16_t*)L.shared_down.biases};
      a.act = c->act_shared;
      a.ids = c->one_id;
      a.wts = c->one_wt;
      a.k = 1;
      a.H = H;
      a.expert_lo = 0;
      a.expert_hi = 1;
      a.h = c->h;
      a.dout = c->d_shared;
      a.world = 1;
      a.status = status;
      a.pdl = pdl;
      const int dgrid = std::max(grid, H / (2 * DownSmem<768>::RMAX / 2));
      switch (d.shared_inter) {
        case 256: return launch(k_down<256, SD>, dgrid, kThreads, sizeof(DownSmem<256>), st, pdl, a);
        case 512: return launch(k_down<512, SD>, dgrid, kThreads, sizeof(DownSmem<512>), st, pdl, a);
        case 768: return launch(k_down<768, SD>, dgrid, kThreads, sizeof(DownSmem<768>), st, pdl, a);
        case 1024: return launch(k_down<1024, SD>, dgrid, kThreads, sizeof(DownSmem<1024>), st, pdl, a);
        default: return cudaErrorInvalidValue;
      }
    }
    case kKDown: {  // experts down + bf16 mix + residual
      if (layer_dense(c, li)) {  // a dense MLP's down projection + residual (the trace row too)
        GemvArgs g = {};
        g.mat[0] = {(const uint32_t*)L.down.w, (const uint16_t*)L.down.scales, (const uint16_t*)L.down.biases};
        g.rows[0] = H;
        g.total_rows = H;
        g.x = c->act;
        g.resid = c->h;
        g.trace_out = c->trace + size_t(li + 1) * H;
        g.status = status;
        g.pdl = pdl;
        switch (d.dense_inter) {
          case 2048: {
            using Kd = GemvSmem<2048, gemv_rs<2048>(), 3>;
            return launch(k_gemv<2048, SD, gemv_rs<2048>(), 3, kEpiResidual>, grid, kThreads, sizeof(Kd), st, pdl, g);
          }
          case 4096: {
            using Kd = GemvSmem<4096, gemv_rs<4096>(), 3>;
            return launch(k_gemv<4096, SD, gemv_rs<4096>(), 3, kEpiResidual>, grid, kThreads, sizeof(Kd), st, pdl, g);
          }
          case 6144: {
            using Kd = GemvSmem<6144, gemv_rs<6144>(), 3>;
            return launch(k_gemv<6144, SD, gemv_rs<6144>(), 3, kEpiResidual>, grid, kThreads, sizeof(Kd), st, pdl, g);
          }
          default: return cudaErrorInvalidValue;
        }
      }
      DownArgs a = {};
      const bool fused = shared_down_fused(c, li);
      a.shared_out = layer_shared(c, li) && !fused ? c->d_shared : nullptr;
      if (fused)
        a.sdown = {(const uint32_t*)L.shared_down.w, (const uint16_t*)L.shared_down.scales,
                   (const uint16_t*)L.shared_down.biases};
      const int is = fused ? d.shared_inter : 0;
      a.down = {(const uint32_t*)L.down.w, (const uint16_t*)L.down.scales, (const uint16_t*)L.down.biases};
      a.act = c->act;
      a.ids = c->ids;
      a.wts = c->wts;
      a.k = d.top_k;
      a.H = H;
      a.expert_lo = c->world > 1 ? c->e_lo : 0;
      a.expert_hi = c->world > 1 ? c->e_hi : d.n_experts;
      a.h = c->h;
      a.trace_row = c->trace + size_t(li + 1) * H;
      a.world = c->world;
      a.rank = c->rank;
      a.layer = li;
      a.n_layers = d.n_layers;
      a.seq = c->ctl + kCtlSeq;
      for (int q = 0; q < kMaxWorld; ++q) a.xch[q] = c->xch[q];
      if (c->world > 1) a.xl = xch_layout(d.n_q_heads, (c->cap_total + kSuperTokens - 1) / kSuperTokens, H);
      a.status = status;
      a.pdl = pdl;
      const int dgrid = std::max(grid, H / (2 * DownSmem<768>::RMAX / 2));
      switch (d.moe_inter) {
        case 256: return launch_down<SD, 256>(a, dgrid, is, st, pdl);
        case 512: return launch_down<SD, 512>(a, dgrid, is, st, pdl);
        case 768: return launch_down<SD, 768>(a, dgrid, is, st, pdl);
        case 1024: return launch_down<SD, 1024>(a, dgrid, is, st, pdl);
        default: return cudaErrorInvalidValue;
      }
    }
    default:
      return cudaErrorInvalidValue;
    }
  }
  {  // final norm + lm_head + argmax
    GemvArgs a = {};
    a.mat[0] = {(const uint32_t*)c->g.lm_head.w, (const uint16_t*)c->g.lm_head.scales,
                (const uint16_t*)c->g.lm_head.biases};
    a.rows[0] = d.vocab;
    a.total_rows = d.vocab;
    a.x = c->h;
    a.norm_w = (const uint16_t*)c->g.final_norm;
    a.eps = d.rms_eps;
    a.out = c->logits;
    a.cand_val = c->cand_val;
    a.cand_idx = c->cand_idx;
    a.counter = c->counters + 0;
    a.token_out = c->ctl + kCtlArgmax;
    a.status = status;
    a.pdl = pdl;
    using Kh = GemvSmem<2048, gemv_rs<2048>(), 3>;
    return launch(k_gemv<2048, SD, gemv_rs<2048>(), 3, kEpiArgmax>, grid, kThreads, sizeof(Kh), st, pdl, a);
  }
}

// The FFN kernels of layer li from the router on (a shared expert's gate/up
// pairs ride in the routed gate/up launch; its down projection runs between
// that and the routed down + mix).
template <int SD>
cudaError_t enqueue_ffn_sd(RecCtx* c, int li, cudaStream_t st, bool pdl) {
  cudaError_t e = enqueue_kernel_sd<SD>(c, kKRouter, li, st, pdl);
  if (e == cudaSuccess) e = enqueue_kernel_sd<SD>(c, kKGateUp, li, st, pdl);
  if (e == cudaSuccess && layer_shared(c, li) && !shared_down_fused(c, li))
    e = enqueue_kernel_sd<SD>(c, kKSharedDown, li, st, pdl);
  if (e == cudaSuccess) e = enqueue_kernel_sd<SD>(c, kKDown, li, st, pdl);
  return e;
}

// One step through the first n_layers layers (all of them in the captured
// graph; fewer for a partial-depth call), the lm_head and the step end.
template <int SD>
cudaError_t enqueue_step_sd(RecCtx* c, cudaStream_t st, int n_layers) {
  cudaError_t e = enqueue_kernel_sd<SD>(c, kKEmbed, 0, st, false);
  for (int li = 0; li < n_layers && e == cudaSuccess; ++li) {
    for (int k = kKQkv; k <= kKOproj && e == cudaSuccess; ++k) e = enqueue_kernel_sd<SD>(c, k, li, st, true);
    if (e == cudaSuccess) e = enqueue_ffn_sd<SD>(c, li, st, true);
  }
  if (e == cudaSuccess) e = enqueue_kernel_sd<SD>(c, kKHead, 0, st, true);
  if (e == cudaSuccess) e = enqueue_kernel_sd<SD>(c, kKStepEnd, 0, st, true);
  return e;
}

cudaError_t enqueue_step(RecCtx* c, cudaStream_t st, int n_layers) {
  return c->d.scale_dtype == REC_SCALE_FP16 ? enqueue_step_sd<0>(c, st, n_layers)
                                            : enqueue_step_sd<1>(c, st, n_layers);
}

int ensure_graph(RecCtx* c) {
  if (c->step_exec) return REC_OK;
  if (!c->cap_stream) REC_CHECK_CUDA(cudaStreamCreateWithFlags(&c->cap_stream, cudaStreamNonBlocking));
  cudaGraph_t graph = nullptr;
  REC_CHECK_CUDA(cudaStreamBeginCapture(c->cap_stream, cudaStreamCaptureModeThreadLocal));
  cudaError_t e = enqueue_step(c, c->cap_stream, c->d.n_layers);
  cudaError_t e2 = cudaStreamEndCapture(c->cap_stream, &graph);
  if (e != cudaSuccess || e2 != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    set_error("step capture failed: %s", cudaGetErrorString(e != cudaSuccess ? e : e2));
    return REC_ECUDA;
  }
  e = cudaGraphInstantiate(&c->step_exec, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) {
    c->step_exec = nullptr;
    set_error("graph instantiate failed: %s", cudaGetErrorString(e));
    return REC_ECUDA;
  }
  return REC_OK;
}

void drop_graph(RecCtx* c) {
  if (c->step_exec) cudaGraphExecDestroy(c->step_exec);
  c->step_exec = nullptr;
}

// Options of the model description that put it on the graph schedule: a
// shared expert, a bf16 or mixed cache, an int8 embedding (layer kinds add to
// them at rec_set_weights).
bool desc_options(const RecModelDesc& d) {
  return d.shared_inter > 0 || d.kv_bits == 16 || d.embed_bits == 8 ||
         (d.kv_value_bits != 0 && d.kv_value_bits != d.kv_bits);
}

bool valid_qmat(const RecQMat& m) {
  return m.w && m.scales && m.biases && aligned16(m.w) && aligned16(m.scales) && aligned16(m.biases);
}

}  // namespace

// ------------------------------------------------------------------------------
// C ABI
// ------------------------------------------------------------------------------
REC_API int rec_create(const RecModelDesc* desc, RecCtx** out) {
  REC_CHECK_ARG(desc && out, "rec_create: null argument");
  const RecModelDesc& d = *desc;
  REC_CHECK_ARG(d.hidden == 2048, "hidden must be 2048 (got %d)", d.hidden);
  REC_CHECK_ARG(d.head_dim == 128, "head_dim must be 128");
  REC_CHECK_ARG(d.n_kv_heads > 0 && d.n_q_heads == 8 * d.n_kv_heads, "need 8 query heads per KV head");
  REC_CHECK_ARG(d.n_q_heads * 128 == 2048 || d.n_q_heads * 128 == 4096, "n_q_heads must be 16 or 32");
  REC_CHECK_ARG(d.n_experts > 0 && d.n_experts <= kMaxExperts, "n_experts must be in 1..%d", kMaxExperts);
  REC_CHECK_ARG(d.top_k >= 1 && d.top_k <= kMaxTopK && d.top_k <= d.n_experts, "top_k must be in 1..8");
  REC_CHECK_ARG(d.moe_inter == 256 || d.moe_inter == 512 || d.moe_inter == 768 || d.moe_inter == 1024,
                "moe_inter must be 256, 512, 768 or 1024");
  REC_CHECK_ARG(d.vocab > 0 && d.vocab % 2 == 0, "vocab must be even");
  REC_CHECK_ARG(d.group_size == 64, "group_size must be 64");
  REC_CHECK_ARG(d.scale_dtype == REC_SCALE_FP16 || d.scale_dtype == REC_SCALE_BF16, "bad scale dtype");
  REC_CHECK_ARG(d.kv_bits == 4 || d.kv_bits == 8 || d.kv_bits == 16, "kv_bits must be 4, 8 or 16");
  REC_CHECK_ARG(d.router_mode == REC_ROUTER_SOFTMAX || d.router_mode == REC_ROUTER_SIGMOID, "bad router mode");
  REC_CHECK_ARG(d.n_layers >= 1 && d.n_layers <= kMaxLayers, "n_layers must be in 1..%d", kMaxLayers);
  REC_CHECK_ARG(d.shared_inter == 0 || d.shared_inter == 256 || d.shared_inter == 512 || d.shared_inter == 768 ||
                    d.shared_inter == 1024,
                "shared_inter must be 0, 256, 512, 768 or 1024");
  REC_CHECK_ARG(d.dense_inter == 0 || d.dense_inter == 2048 || d.dense_inter == 4096 || d.dense_inter == 6144,
                "dense_inter must be 0, 2048, 4096 or 6144");
  REC_CHECK_ARG(d.sliding_window >= 0, "sliding_window must be >= 0");
  REC_CHECK_ARG(d.embed_bits == 0 || d.embed_bits == 4 || d.embed_bits == 8, "embed_bits must be 4 or 8");
  REC_CHECK_ARG(d.kv_value_bits == 0 || d.kv_value_bits == d.kv_bits ||
                    (d.kv_bits != 16 && (d.kv_value_bits == 4 || d.kv_value_bits == 8)),
                "kv_value_bits must be 0 or, with 4- or 8-bit K codes, 4 or 8");
  RecCtx* c = new RecCtx();
  c->d = d;
  c->flint = desc_options(d);
  c->grid = sm_count();
  *out = c;
  return REC_OK;
}

REC_API int rec_set_shard(RecCtx* c, const RecShard* sh) {
  REC_CHECK_ARG(c && sh, "rec_set_shard: null argument");
  const RecShard& s = *sh;
  REC_CHECK_ARG(s.world >= 1 && s.world <= kMaxWorld, "world size must be 1..%d", kMaxWorld);
  REC_CHECK_ARG(s.world == 1 || !c->flint, "a model with layer options (shared expert, dense / NoPE / sliding "
                "layers) runs on one GPU");
  REC_CHECK_ARG(s.rank >= 0 && s.rank < s.world, "rank outside the world");
  REC_CHECK_ARG(c->grid <= kMaxGrid, "too many SMs for the exchange layout");
  REC_CHECK_ARG(s.capacity_total > 0 && s.capacity_total % kAttBlock == 0,
                "capacity_total must be a positive multiple of %d", kAttBlock);
  const int n_super = (s.capacity_total + kSuperTokens - 1) / kSuperTokens;
  REC_CHECK_ARG(s.super_lo >= 0 && s.super_lo <= s.super_hi && s.super_hi <= n_super, "bad super-chunk range");
  REC_CHECK_ARG(s.expert_lo >= 0 && s.expert_lo < s.expert_hi && s.expert_hi <= c->d.n_experts, "bad expert range");
  c->world = s.world;
  c->rank = s.rank;
  c->e_lo = s.expert_lo;
  c->e_hi = s.expert_hi;
  c->super_lo = s.super_lo;
  c->super_hi = s.super_hi;
  c->cap_total = s.capacity_total;
  REC_CHECK_ARG(s.schedule == 0 || s.schedule == 1, "RecShard.schedule must be 0 or 1");
  if (c->shard_graph != (s.schedule == 1)) drop_graph(c);
  c->shard_graph = s.world > 1 && s.schedule == 1;
  c->token_base = s.super_lo * kSuperTokens;
  bool all = true;
  for (int q = 0; q < kMaxWorld; ++q) {
    c->xch[q] = q < s.world ? static_cast<uint8_t*>(s.exchange[q]) : nullptr;
    if (q < s.world) all = all && c->xch[q] != nullptr;
  }
  for (int q = 0; q < s.world && all; ++q)
    REC_CHECK_ARG((reinterpret_cast<uintptr_t>(c->xch[q]) & 255u) == 0, "exchange buffers must be 256-byte aligned");
  c->layer_seq = 0;
  c->ws = nullptr;  // the workspace layout depends on the split
  c->ws_bytes = 0;
  drop_graph(c);
  return REC_OK;
}

REC_API size_t rec_exchange_bytes(const RecCtx* c) {
  if (!c || c->world < 1 || c->cap_total <= 0) return 0;
  return xch_layout(c->d.n_q_heads, (c->cap_total + kSuperTokens - 1) / kSuperTokens, c->d.hidden).total;
}

REC_API void rec_destroy(RecCtx* ctx) {
  if (!ctx) return;
  drop_graph(ctx);
  if (ctx->cap_stream) cudaStreamDestroy(ctx->cap_stream);
  delete ctx;
}

REC_API int rec_set_weights(RecCtx* c, const RecLayerWeights* layers, int32_t n_layers, const RecGlobalWeights* g) {
  REC_CHECK_ARG(c && layers && g, "rec_set_weights: null argument");
  REC_CHECK_ARG(n_layers == c->d.n_layers, "expected %d layers, got %d", c->d.n_layers, n_layers);
  bool flint = desc_options(c->d);  // and any layer kind below
  for (int i = 0; i < n_layers; ++i) {
    const RecLayerWeights& L = layers[i];
    const bool dense = (L.kind & REC_LAYER_DENSE) != 0;
    REC_CHECK_ARG((L.kind & ~(REC_LAYER_DENSE | REC_LAYER_NO_ROPE | REC_LAYER_SLIDING)) == 0,
                  "layer %d: unknown kind bits 0x%x", i, L.kind);
    REC_CHECK_ARG(!dense || c->d.dense_inter > 0, "layer %d: a dense-MLP layer needs dense_inter", i);
    REC_CHECK_ARG(!(L.kind & REC_LAYER_SLIDING) || c->d.sliding_window > 0,
                  "layer %d: a sliding-window layer needs sliding_window", i);
    REC_CHECK_ARG(c->world == 1 || L.kind == 0, "layer %d: layer options need an unsharded session", i);
    flint = flint || L.kind != 0;
    REC_CHECK_ARG(L.input_norm && L.post_norm && (dense || L.router), "layer %d: missing norm/router weights", i);
    REC_CHECK_ARG(valid_qmat(L.q) && valid_qmat(L.k) && valid_qmat(L.v) && valid_qmat(L.o) && valid_qmat(L.gate) &&
                      valid_qmat(L.up) && valid_qmat(L.down),
                  "layer %d: quantized matrices must be non-null and 16-byte aligned", i);
    REC_CHECK_ARG(dense || c->d.shared_inter == 0 ||
                      (valid_qmat(L.shared_gate) && valid_qmat(L.shared_up) && valid_qmat(L.shared_down)),
                  "layer %d: shared-expert matrices must be non-null and 16-byte aligned", i);
    if (dense) continue;
    REC_CHECK_ARG(aligned16(L.router), "layer %d: router must be 16-byte aligned", i);
    REC_CHECK_ARG(c->d.router_mode != REC_ROUTER_SIGMOID || L.expert_bias, "layer %d: sigmoid router needs a bias", i);
    REC_CHECK_ARG(!(c->d.flags & REC_FLAG_SINKS) || L.sinks, "layer %d: sinks enabled but missing", i);
    REC_CHECK_ARG(!(c->d.flags & REC_FLAG_QK_NORM) || (L.q_norm && L.k_norm), "layer %d: qk norm missing", i);
  }
  REC_CHECK_ARG(valid_qmat(g->embed) && valid_qmat(g->lm_head) && g->final_norm, "global weights incomplete");
  c->layers.assign(layers, layers + n_layers);
  c->g = *g;
  c->has_weights = true;
  c->flint = flint;
  drop_graph(c);
  return REC_OK;
}

REC_API int rec_set_kv(RecCtx* c, const RecKVLayer* layers, int32_t n_layers, int32_t capacity) {
  REC_CHECK_ARG(c && layers, "rec_set_kv: null argument");
  REC_CHECK_ARG(n_layers == c->d.n_layers, "expected %d KV layers", c->d.n_layers);
  REC_CHECK_ARG(capacity > 0 && capacity % kAttBlock == 0, "capacity must be a positive multiple of %d", kAttBlock);
  for (int i = 0; i < n_layers; ++i) {
    const RecKVLayer& k = layers[i];
    if (c->d.kv_bits == 16) {  // bf16 rows; no scales or biases
      REC_CHECK_ARG(k.k_codes && k.v_codes && aligned16(k.k_codes) && aligned16(k.v_codes),
                    "KV layer %d: bf16 K / V buffers must be non-null and 16-byte aligned", i);
      continue;
    }
    REC_CHECK_ARG(k.k_codes && k.k_scales && k.k_biases && k.v_codes && k.v_scales && k.v_biases &&
                      aligned16(k.k_codes) && aligned16(k.v_codes) && aligned16(k.k_scales) &&
                      aligned16(k.k_biases) && aligned16(k.v_scales) && aligned16(k.v_biases),
                  "KV layer %d: buffers must be non-null and 16-byte aligned", i);
  }
  const bool grow = capacity != c->capacity;
  c->kv.assign(layers, layers + n_layers);
  c->capacity = capacity;
  c->kv_rows = capacity;
  const int nblk = capacity / kAttBlock;
  c->n_super_max = (nblk + kAttSuper - 1) / kAttSuper;
  if (grow) {
    c->ws = nullptr;  // workspace must be re-sized
    c->ws_bytes = 0;
  }
  drop_graph(c);
  return REC_OK;
}

static int fill_rope(RecCtx* c, int rows);

REC_API int rec_set_kv_rows(RecCtx* c, int32_t rows) {
  REC_CHECK_ARG(c && c->capacity > 0, "rec_set_kv_rows: set the KV cache first");
  REC_CHECK_ARG(c->world == 1, "rec_set_kv_rows: an unsharded session only");
  REC_CHECK_ARG(rows > 0 && rows <= c->capacity && rows % kAttBlock == 0,
                "rec_set_kv_rows: rows %d must be a multiple of %d in (0, %d]", rows, kAttBlock, c->capacity);
  c->kv_rows = rows;
  return fill_rope(c, rows);
}

REC_API size_t rec_workspace_bytes(const RecCtx* c) {
  if (!c || c->capacity <= 0) return 0;
  return layout_of(c).total;
}

// RoPE table rows [rope_done, rows): cos/sin of pos * theta^(-i/64) in
// double, rounded to float (row p = absolute position p).
static int fill_rope(RecCtx* c, int rows) {
  rows = rows < rope_rows(c) ? rows : rope_rows(c);
  if (!c->rope || rows <= c->rope_done) return REC_OK;
  const int p0 = c->rope_done;
  std::vector<float> cs(size_t(rows - p0) * 128);
  for (int p = p0; p < rows; ++p)
    for (int i = 0; i < 64; ++i) {
      const double inv = std::pow(double(c->d.rope_theta), -double(i) / 64.0);
      const double ang = double(p) * inv;
      cs[size_t(p - p0) * 128 + i] = float(std::cos(ang));
      cs[size_t(p - p0) * 128 + 64 + i] = float(std::sin(ang));
    }
  REC_CHECK_CUDA(cudaMemcpy(c->rope + size_t(p0) * 128, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
  c->rope_done = rows;
  return REC_OK;
}

REC_API int rec_set_workspace(RecCtx* c, void* ws, size_t bytes) {
  int rc_rope = 0;
  REC_CHECK_ARG(c && ws, "rec_set_workspace: null argument");
  REC_CHECK_ARG(c->capacity > 0, "call rec_set_kv before rec_set_workspace");
  const Layout L = layout_of(c);
  REC_CHECK_ARG(bytes >= L.total, "workspace too small: %zu < %zu", bytes, L.total);
  REC_CHECK_ARG((reinterpret_cast<uintptr_t>(ws) & 255u) == 0, "workspace must be 256-byte aligned");
  uint8_t* b = static_cast<uint8_t*>(ws);
  c->ws = b;
  c->ws_bytes = bytes;
  c->ctl = reinterpret_cast<int*>(b + L.off[rCtl]);
  c->counters = reinterpret_cast<unsigned*>(b + L.off[rCounters]);
  c->h = reinterpret_cast<uint16_t*>(b + L.off[rH]);
  c->qkv = reinterpret_cast<uint16_t*>(b + L.off[rQkv]);
  c->attn = reinterpret_cast<uint16_t*>(b + L.off[rAttn]);
  c->xn = reinterpret_cast<uint16_t*>(b + L.off[rXn]);
  c->act = reinterpret_cast<uint16_t*>(b + L.off[rAct]);
  c->logits = reinterpret_cast<uint16_t*>(b + L.off[rLogits]);
  c->trace = reinterpret_cast<uint16_t*>(b + L.off[rTrace]);
  c->router_logits = reinterpret_cast<float*>(b + L.off[rRouter]);
  c->router_ll = reinterpret_cast<unsigned long long*>(b + L.off[rRouterLL]);
  c->ids = reinterpret_cast<int*>(b + L.off[rIds]);
  c->wts = reinterpret_cast<float*>(b + L.off[rWts]);
  c->cand_val = reinterpret_cast<float*>(b + L.off[rCandV]);
  c->cand_idx = reinterpret_cast<int*>(b + L.off[rCandI]);
  c->partials = reinterpret_cast<float*>(b + L.off[rPartials]);
  c->supers = reinterpret_cast<float*>(b + L.off[rSupers]);
  c->rope = reinterpret_cast<float*>(b + L.off[rRope]);
  c->mega_cnt = reinterpret_cast<unsigned*>(b + L.off[rMegaCnt]);
  c->mega_layers = reinterpret_cast<MegaLayer*>(b + L.off[rMegaLayers]);
  c->act_shared = c->act + size_t(c->d.top_k) * c->d.moe_inter;
  c->d_shared = reinterpret_cast<uint16_t*>(b + L.off[rFlint]);
  c->one_id = reinterpret_cast<int*>(b + L.off[rFlint] + size_t(c->d.hidden) * 2);
  c->one_wt = reinterpret_cast<float*>(c->one_id + 1);
  {
    const int one[2] = {0, 0x3f800000};  // {0, 1.0f}
    REC_CHECK_CUDA(cudaMemcpy(c->one_id, one, sizeof(one), cudaMemcpyHostToDevice));
  }
  // control block and counters start at zero
  REC_CHECK_CUDA(cudaMemset(b, 0, L.off[rH]));
  // layer table of the persistent kernel
  {
    const bool qk = (c->d.flags & REC_FLAG_QK_NORM) != 0, sinks = (c->d.flags & REC_FLAG_SINKS) != 0;
    auto q = [](const RecQMat& m) {
      return QMatDev{(const uint32_t*)m.w, (const uint16_t*)m.scales, (const uint16_t*)m.biases};
    };
    std::vector<MegaLayer> t(c->d.n_layers);
    for (int i = 0; i < c->d.n_layers; ++i) {
      const RecLayerWeights& W = c->layers[i];
      const RecKVLayer& K = c->kv[i];
      t[i] = MegaLayer{q(W.q), q(W.k), q(W.v), q(W.o), q(W.gate), q(W.up), q(W.down),
                       (const uint16_t*)W.input_norm, (const uint16_t*)W.post_norm, (const uint16_t*)W.router,
                       (const float*)W.expert_bias, sinks ? (const uint16_t*)W.sinks : nullptr,
                       qk ? (const uint16_t*)W.q_norm : nullptr, qk ? (const uint16_t*)W.k_norm : nullptr,
                       (uint32_t*)K.k_codes, (uint16_t*)K.k_scales, (uint16_t*)K.k_biases, (uint32_t*)K.v_codes,
                       (uint16_t*)K.v_scales, (uint16_t*)K.v_biases};
    }
    if (c->has_weights)
      REC_CHECK_CUDA(cudaMemcpy(c->mega_layers, t.data(), t.size() * sizeof(MegaLayer), cudaMemcpyHostToDevice));
  }
  // RoPE table rows for the positions the cache backs (more as it grows)
  c->rope_done = 0;
  rc_rope = fill_rope(c, c->world > 1 ? rope_rows(c) : c->kv_rows);
  if (rc_rope) return rc_rope;
  c->usable = true;
  drop_graph(c);
  return REC_OK;
}

// Schedule of a step at `position`: the persistent kernel (kSchedMega), the
// CUDA graph of separate kernels (kSchedGraph), or the split schedule
// (kSchedSplit: persistent-kernel segments around the standalone attention
// kernels of each layer).  REC_SCHEDULE=mega / graph / split forces one;
// otherwise the persistent kernel runs while one layer's attended KV is
// below kMegaAttnBytes and the graph above it.  At long contexts attention
// dominates, and its standalone kernel (two 8-warp CTAs per SM) outruns the
// persistent kernel's 8 consumer warps per SM, while the graph overlaps
// consecutive kernels (programmatic dependent launch).  Measured tok/s
// (mega / split / graph): 8-bit 16K 347 / 344 / 330; 8-bit 32K 311 / 313 /
// 326; 4-bit 64K 268 / 292 / 307; 4-bit 128K 188 / 206 / 242.  The split
// schedule (each segment starts cold, without the weight prefetch across
// the attention launches) is never the fastest and runs only when forced.
// More than kMegaMaxExperts experts take the graph; a session split over
// ranks always runs on the persistent kernel.
constexpr double kMegaAttnBytes = 24.0 * 1024 * 1024;
static int schedule_for(const RecCtx* c, int position) {
  if (c->flint) return kSchedGraph;  // layer options exist on the graph schedule only
  const char* sched = std::getenv("REC_SCHEDULE");
  if (sched && std::strcmp(sched, "graph") == 0) return kSchedGraph;
  if (c->d.n_experts > kMegaMaxExperts) return kSchedGraph;
  if (c->world > 1) return c->shard_graph ? kSchedGraph : kSchedMega;
  if (sched && std::strcmp(sched, "mega") == 0) return kSchedMega;
  if (sched && std::strcmp(sched, "split") == 0) return kSchedSplit;
  const double bytes = double(position + 1) * double(c->d.n_kv_heads) * (c->d.kv_bits == 4 ? 144.0 : 272.0);
  return bytes < kMegaAttnBytes ? kSchedMega : kSchedGraph;
}
static bool mega_for(const RecCtx* c, int position) { return schedule_for(c, position) == kSchedMega; }

static int check_ready(RecCtx* c) {
  REC_CHECK_ARG(c, "null context");
  if (!c->usable) {
    set_error("Session was invalidated by a GPU synchronization failure");
    return REC_ESTATE;
  }
  if (!c->has_weights || !c->ws || c->kv.empty()) {
    set_error("session not configured (weights, KV and workspace are required)");
    return REC_ESTATE;
  }
  if (c->world > 1) {
    REC_CHECK_ARG(c->shard_graph || c->d.n_experts <= kMegaMaxExperts,
                  "a split session on the persistent kernel needs n_experts <= %d", kMegaMaxExperts);
    for (int q = 0; q < c->world; ++q)
      if (!c->xch[q]) {
        set_error("rec_set_shard: exchange buffer of rank %d not set", q);
        return REC_ESTATE;
      }
  }
  return REC_OK;
}

// Picks the schedule of a call whose last step runs at `last_position` and
// builds the CUDA graph on first use.
static int select_schedule(RecCtx* c, int last_position) {
  c->sched = schedule_for(c, last_position);
  // the split schedule launches the graph's attention kernels, whose set-up
  // the capture does
  return c->sched == kSchedMega ? REC_OK : ensure_graph(c);
}

// Position limit of the session (global when split over ranks).
static int position_limit(const RecCtx* c) {
  return c->world > 1 ? c->cap_total : c->token_base + (c->kv_rows < c->capacity ? c->kv_rows : c->capacity);
}

// One cooperative launch of the persistent kernel for `steps` tokens.
template <int I, int BITS>
static cudaError_t launch_mega_t(RecCtx* c, int steps, cudaStream_t st, int seg) {
  const RecModelDesc& d = c->d;
  MegaArgs A = {};
  A.seg = seg;
  A.layers = c->mega_layers;
  A.n_layers = c->layers_run > 0 ? c->layers_run : d.n_layers;
  A.bar_spin_limit = c->bar_spin_limit;
  A.skip_arrive_cta = c->skip_arrive_cta;
  A.H = d.hidden;
  A.hq = d.n_q_heads;
  A.hkv = d.n_kv_heads;
  A.E = d.n_experts;
  A.k = d.top_k;
  A.I = d.moe_inter;
  A.V = d.vocab;
  A.kv_bits = d.kv_bits;
  A.router_mode = d.router_mode;
  A.sd = d.scale_dtype == REC_SCALE_BF16 ? 1 : 0;
  A.capacity = c->capacity;
  A.n_super_max = c->n_super_max;
  A.eps = d.rms_eps;
  A.embed = {(const uint32_t*)c->g.embed.w, (const uint16_t*)c->g.embed.scales, (const uint16_t*)c->g.embed.biases};
  A.lm_head = {(const uint32_t*)c->g.lm_head.w, (const uint16_t*)c->g.lm_head.scales,
               (const uint16_t*)c->g.lm_head.biases};
  A.final_norm = (const uint16_t*)c->g.final_norm;
  A.rope = c->rope;
  A.ctl = c->ctl;
  A.gbar = c->mega_cnt;
  A.cnt = c->mega_cnt + 2;
  A.h = c->h;
  A.qkv = c->qkv;
  A.attn = c->attn;
  A.act = c->act;
  A.logits = c->logits;
  A.trace = c->trace;
  A.partials = c->partials;
  A.supers = c->supers;
  A.router_logits = c->router_logits;
  A.router_ll = c->router_ll;
  A.cand_val = c->cand_val;
  A.cand_idx = c->cand_idx;
  A.steps = steps;
  A.world = c->world;
  A.rank = c->rank;
  A.e_lo = c->world > 1 ? c->e_lo : 0;
  A.e_hi = c->world > 1 ? c->e_hi : d.n_experts;
  A.super_lo = c->world > 1 ? c->super_lo : 0;
  A.super_hi = c->world > 1 ? c->super_hi : c->n_super_max;
  A.token_base = c->token_base;
  A.layer_seq0 = c->layer_seq;
  A.xl = xch_layout(d.n_q_heads, c->world > 1 ? (c->cap_total + kSuperTokens - 1) / kSuperTokens : 1, d.hidden);
  for (int q = 0; q < kMaxWorld; ++q) A.xch[q] = c->xch[q];
  const size_t need = size_t(steps) * (6 * d.n_layers + 1) * c->grid * 2;
  A.prof = (c->prof && c->prof_entries >= need && seg == kSegAll) ? c->prof : nullptr;
  A.prof2 = c->prof2;
  A.prof_layer = c->prof_layer;
  auto kern = k_decode_mega<I, BITS>;
  const size_t smem = sizeof(MegaSmem);
  cudaError_t e = set_smem_limit(reinterpret_cast<const void*>(kern), smem);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(c->mega_cnt, 0, 2 * sizeof(unsigned), st);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(c->grid);
  cfg.blockDim = dim3(kMegaThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, A);
  // a segmented step advances the layer sequence once, after its last segment
  if (e == cudaSuccess && seg == kSegAll) c->layer_seq += unsigned(steps) * unsigned(A.n_layers);
  return e;
}

static cudaError_t launch_mega(RecCtx* c, int steps, cudaStream_t st, int seg = kSegAll) {
  const bool kv4 = c->d.kv_bits == 4;
  switch (c->d.moe_inter) {
    case 256: return kv4 ? launch_mega_t<256, 4>(c, steps, st, seg) : launch_mega_t<256, 8>(c, steps, st, seg);
    case 512: return kv4 ? launch_mega_t<512, 4>(c, steps, st, seg) : launch_mega_t<512, 8>(c, steps, st, seg);
    case 768: return kv4 ? launch_mega_t<768, 4>(c, steps, st, seg) : launch_mega_t<768, 8>(c, steps, st, seg);
    case 1024: return kv4 ? launch_mega_t<1024, 4>(c, steps, st, seg) : launch_mega_t<1024, 8>(c, steps, st, seg);
    default: return cudaErrorInvalidValue;
  }
}

// One step on the split schedule: persistent-kernel segments for everything
// but attention (embedding + Q of layer 0, then per layer O, R, G, D and the
// next layer's Q, the last one ending with H and E), and the standalone
// attention kernels of each layer between them.
static cudaError_t launch_split_step(RecCtx* c, cudaStream_t st) {
  const int L = c->d.n_layers;
  cudaError_t e = launch_mega(c, 1, st, -1);
  for (int l = 0; l < L && e == cudaSuccess; ++l) {
    e = c->d.scale_dtype == REC_SCALE_FP16 ? enqueue_kernel_sd<0>(c, kKAttn, l, st, true)
                                           : enqueue_kernel_sd<1>(c, kKAttn, l, st, true);
    if (e == cudaSuccess)
      e = c->d.scale_dtype == REC_SCALE_FP16 ? enqueue_kernel_sd<0>(c, kKCombine, l, st, true)
                                             : enqueue_kernel_sd<1>(c, kKCombine, l, st, true);
    if (e == cudaSuccess) e = launch_mega(c, 1, st, l);
  }
  if (e == cudaSuccess) c->layer_seq += unsigned(L);
  return e;
}

// One step (graph schedule or split schedule) or a packet of steps
// (persistent kernel) on the schedule chosen for the call.
static cudaError_t launch_steps(RecCtx* c, int steps, cudaStream_t st) {
  cudaError_t e = cudaSuccess;
  if (c->sched == kSchedMega) return launch_mega(c, steps, st);
  for (int i = 0; i < steps && e == cudaSuccess; ++i)
    e = c->sched == kSchedGraph ? cudaGraphLaunch(c->step_exec, st) : launch_split_step(c, st);
  return e;
}

REC_API int rec_decode_step(RecCtx* c, int32_t token, int32_t position, void* logits_dev, void* trace_dev,
                            void* stream) {
  int rc = check_ready(c);
  if (rc) return rc;
  if (position < 0 || position >= position_limit(c)) {
    set_error("position %d outside the KV capacity", position);
    return REC_ELIMIT;
  }
  REC_CHECK_ARG(token >= 0 && token < c->d.vocab, "token %d outside the vocabulary", token);
  rc = select_schedule(c, position);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  k_set_step<<<1, 32, 0, st>>>(c->ctl, token, position, 0, make_int4(0, 0, 0, 0), make_int4(0, 0, 0, 0), 0);
  REC_CHECK_CUDA(cudaGetLastError());
  REC_CHECK_CUDA(launch_steps(c, 1, st));
  if (logits_dev)
    REC_CHECK_CUDA(cudaMemcpyAsync(logits_dev, c->logits, size_t(c->d.vocab) * 2, cudaMemcpyDeviceToDevice, st));
  if (trace_dev)
    REC_CHECK_CUDA(cudaMemcpyAsync(trace_dev, c->trace, size_t(c->d.n_layers + 1) * c->d.hidden * 2,
                                   cudaMemcpyDeviceToDevice, st));
  return REC_OK;
}

REC_API int rec_decode_layers(RecCtx* c, int32_t token, int32_t position, int32_t layer_count, void* logits_dev,
                              void* trace_dev, void* stream) {
  int rc = check_ready(c);
  if (rc) return rc;
  REC_CHECK_ARG(layer_count >= 1 && layer_count <= c->d.n_layers, "layer_count %d outside 1..%d", layer_count,
                c->d.n_layers);
  if (layer_count == c->d.n_layers) return rec_decode_step(c, token, position, logits_dev, trace_dev, stream);
  REC_CHECK_ARG(c->flint || c->d.n_experts <= kMegaMaxExperts, "a partial-depth step needs at most %d experts",
                kMegaMaxExperts);
  if (position < 0 || position >= position_limit(c)) {
    set_error("position %d outside the KV capacity", position);
    return REC_ELIMIT;
  }
  REC_CHECK_ARG(token >= 0 && token < c->d.vocab, "token %d outside the vocabulary", token);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  k_set_step<<<1, 32, 0, st>>>(c->ctl, token, position, 0, make_int4(0, 0, 0, 0), make_int4(0, 0, 0, 0), 0);
  REC_CHECK_CUDA(cudaGetLastError());
  if (c->flint) {
    // layer options: the graph schedule's kernels for the first layers,
    // launched directly (the captured graph runs every layer)
    c->sched = kSchedGraph;
    REC_CHECK_CUDA(enqueue_step(c, st, layer_count));
  } else {
    // the persistent kernel with a shorter layer loop (its H phase follows
    // the last layer run)
    c->sched = kSchedMega;
    c->layers_run = layer_count;
    const cudaError_t e = launch_mega(c, 1, st);
    c->layers_run = 0;
    REC_CHECK_CUDA(e);
  }
  if (logits_dev)
    REC_CHECK_CUDA(cudaMemcpyAsync(logits_dev, c->logits, size_t(c->d.vocab) * 2, cudaMemcpyDeviceToDevice, st));
  if (trace_dev)
    REC_CHECK_CUDA(cudaMemcpyAsync(trace_dev, c->trace, size_t(layer_count + 1) * c->d.hidden * 2,
                                   cudaMemcpyDeviceToDevice, st));
  return REC_OK;
}

// ---------------------------------------------------------------------------
// Chunked prompt prefill (quantized.py:102-148): t tokens at positions
// [position, position + t) through every layer, dense work on the tensor cores
// (rec_prefill_gemm, rec_prefill_moe), causal attention over the quantized
// cache (prefill_layer.cu), the chunk's K / V quantized into the cache
// (rec_kv_append_bulk); optionally the last token's logits.
// ---------------------------------------------------------------------------
namespace {
struct PrefillLayout {
  size_t h, xn, q, k, v, att, o, ids, wts, moe, total;
  size_t moe_bytes;
};
PrefillLayout prefill_layout(const RecModelDesc& d, int64_t t) {
  PrefillLayout L;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes, 256);
    return at;
  };
  const size_t H = size_t(d.hidden), Q = size_t(d.n_q_heads) * 128, KV = size_t(d.n_kv_heads) * 128;
  L.h = take(size_t(t) * H * 2);
  L.xn = take(size_t(t) * H * 2);
  L.q = take(size_t(t) * Q * 2);
  L.k = take(size_t(t) * KV * 2);
  L.v = take(size_t(t) * KV * 2);
  L.att = take(size_t(t) * Q * 2);
  L.o = take(size_t(t) * H * 2);
  L.ids = take(size_t(t) * d.top_k * 4);
  L.wts = take(size_t(t) * d.top_k * 4);
  L.moe_bytes = rec_prefill_moe_workspace_bytes(t, d.top_k, d.hidden, d.moe_inter, d.n_experts);
  L.moe = take(L.moe_bytes);
  L.total = off;
  return L;
}
}  // namespace

REC_API size_t rec_prefill_workspace_bytes(const RecCtx* c, int32_t t) {
  if (!c || t <= 0) return 0;
  return prefill_layout(c->d, t).total;
}

REC_API int rec_prefill_chunk_layers(RecCtx* c, const int32_t* tokens_dev, int32_t position, int32_t t,
                                     int32_t layer_begin, int32_t layer_end, void* logits_dev, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  int rc = check_ready(c);
  if (rc) return rc;
  const RecModelDesc& d = c->d;
  REC_CHECK_ARG(workspace && (tokens_dev || layer_begin > 0), "rec_prefill_chunk: null pointer");
  REC_CHECK_ARG(layer_begin >= 0 && layer_begin < layer_end && layer_end <= d.n_layers,
                "rec_prefill_chunk: layers [%d, %d) outside [0, %d)", layer_begin, layer_end, d.n_layers);
  REC_CHECK_ARG(c->world == 1, "rec_prefill_chunk: an unsharded session only");
  REC_CHECK_ARG(!c->flint, "rec_prefill_chunk: layer options (shared expert, dense / NoPE / sliding layers) are "
                "prefilled by decode steps");
  REC_CHECK_ARG(d.hidden == 2048 && d.moe_inter % 256 == 0, "rec_prefill_chunk: hidden 2048 and I a multiple of 256");
  REC_CHECK_ARG(t >= 1 && t <= 16384, "rec_prefill_chunk: %d tokens outside 1..16384", t);
  if (position < 0 || int64_t(position) + t > position_limit(c)) {
    set_error("Decode context limit exhausted");
    return REC_ELIMIT;
  }
  const PrefillLayout L = prefill_layout(d, t);
  REC_CHECK_ARG(workspace_bytes >= L.total && (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
                "rec_prefill_chunk: workspace must be 256-byte aligned and hold %zu bytes", L.total);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  uint16_t* h = reinterpret_cast<uint16_t*>(w + L.h);
  uint16_t* xn = reinterpret_cast<uint16_t*>(w + L.xn);
  uint16_t* q = reinterpret_cast<uint16_t*>(w + L.q);
  uint16_t* k = reinterpret_cast<uint16_t*>(w + L.k);
  uint16_t* v = reinterpret_cast<uint16_t*>(w + L.v);
  uint16_t* att = reinterpret_cast<uint16_t*>(w + L.att);
  uint16_t* o = reinterpret_cast<uint16_t*>(w + L.o);
  int* ids = reinterpret_cast<int*>(w + L.ids);
  float* wts = reinterpret_cast<float*>(w + L.wts);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* status = c->ctl + kCtlStatus;
  const int sd = d.scale_dtype;
  const int H = d.hidden, Q = d.n_q_heads * 128, KV = d.n_kv_heads * 128;
  const QMatDev emb = {(const uint32_t*)c->g.embed.w, (const uint16_t*)c->g.embed.scales,
                       (const uint16_t*)c->g.embed.biases};
  // the chunk's hidden states stay in the workspace between layer ranges
  if (layer_begin == 0)
    REC_CHECK_CUDA(pf_embed(emb, sd == REC_SCALE_BF16 ? 1 : 0, tokens_dev, t, H, d.vocab, h, status, st));
  const bool qk = (d.flags & REC_FLAG_QK_NORM) != 0, sinks = (d.flags & REC_FLAG_SINKS) != 0;
  for (int l = layer_begin; l < layer_end; ++l) {
    const RecLayerWeights& W = c->layers[l];
    REC_CHECK_CUDA(pf_rmsnorm(h, (const uint16_t*)W.input_norm, t, d.rms_eps, xn, st));
    if ((rc = rec_prefill_gemm(&W.q, sd, Q, H, xn, t, q, status, st))) return rc;
    if ((rc = rec_prefill_gemm(&W.k, sd, KV, H, xn, t, k, status, st))) return rc;
    if ((rc = rec_prefill_gemm(&W.v, sd, KV, H, xn, t, v, status, st))) return rc;
    REC_CHECK_CUDA(pf_qk(q, d.n_q_heads, k, d.n_kv_heads, t, position, c->rope,
                         qk ? (const uint16_t*)W.q_norm : nullptr, qk ? (const uint16_t*)W.k_norm : nullptr,
                         d.rms_eps, st));
    if ((rc = rec_kv_append_bulk(&c->kv[l], d.n_kv_heads, c->capacity, d.kv_bits, k, v, position, t, st)))
      return rc;
    REC_CHECK_CUDA(pf_attention(q, d.n_q_heads, d.n_kv_heads, c->kv[l], c->capacity, d.kv_bits, position, t,
                                sinks ? (const uint16_t*)W.sinks : nullptr, att, st));
    if ((rc = rec_prefill_gemm(&W.o, sd, H, Q, att, t, o, status, st))) return rc;
    REC_CHECK_CUDA(pf_add(h, o, size_t(t) * H, st));
    REC_CHECK_CUDA(pf_rmsnorm(h, (const uint16_t*)W.post_norm, t, d.rms_eps, xn, st));
    REC_CHECK_CUDA(pf_router(xn, (const uint16_t*)W.router, (const float*)W.expert_bias, t, d.n_experts, d.top_k,
                             d.router_mode, ids, wts, st));
    if ((rc = rec_prefill_moe(&W.gate, &W.up, &W.down, sd, d.n_experts, d.moe_inter, H, xn, t, d.top_k, ids, wts, h,
                              h, w + L.moe, L.moe_bytes, status, st)))
      return rc;
  }
  if (logits_dev && layer_end == d.n_layers)
    return rec_gemv_int4(&c->g.lm_head, sd, d.vocab, H, h + size_t(t - 1) * H, c->g.final_norm, d.rms_eps, logits_dev,
                         st);
  return REC_OK;
}

REC_API int rec_prefill_chunk(RecCtx* c, const int32_t* tokens_dev, int32_t position, int32_t t, void* logits_dev,
                              void* workspace, size_t workspace_bytes, void* stream) {
  if (!c) return check_ready(c);
  return rec_prefill_chunk_layers(c, tokens_dev, position, t, 0, c->d.n_layers, logits_dev, workspace,
                                  workspace_bytes, stream);
}

REC_API int rec_prefill_attention(const void* q_dev, int32_t n_q_heads, int32_t n_kv_heads, const RecKVLayer* kv,
                                  int32_t capacity, int32_t kv_bits, int32_t position, int32_t t, const void* sinks_dev,
                                  void* out_dev, void* stream) {
  REC_CHECK_ARG(q_dev && kv && out_dev, "rec_prefill_attention: null pointer");
  REC_CHECK_ARG(n_kv_heads >= 1 && n_q_heads == 8 * n_kv_heads, "rec_prefill_attention: 8 q heads per kv head");
  REC_CHECK_ARG(kv_bits == 4 || kv_bits == 8, "rec_prefill_attention: kv_bits 4 or 8");
  REC_CHECK_ARG(t >= 1 && position >= 0 && int64_t(position) + t <= capacity,
                "rec_prefill_attention: positions [%d, %d) outside the capacity %d", position, position + t, capacity);
  REC_CHECK_ARG(aligned16(kv->k_codes) && aligned16(kv->v_codes), "rec_prefill_attention: codes 16-byte aligned");
  REC_CHECK_CUDA(pf_attention(static_cast<const uint16_t*>(q_dev), n_q_heads, n_kv_heads, *kv, capacity, kv_bits,
                              position, t, static_cast<const uint16_t*>(sinks_dev), static_cast<uint16_t*>(out_dev),
                              static_cast<cudaStream_t>(stream)));
  return REC_OK;
}

REC_API int rec_set_fault_injection(RecCtx* c, uint32_t barrier_spin_limit, int32_t skip_arrive_cta) {
  REC_CHECK_ARG(c, "null context");
  c->bar_spin_limit = barrier_spin_limit ? barrier_spin_limit : kSpinLimit * 4;
  c->skip_arrive_cta = skip_arrive_cta;
  return REC_OK;
}

REC_API int rec_decode_greedy(RecCtx* c, int32_t token, int32_t position, int32_t count, const int32_t* eos,
                              int32_t n_eos, int32_t* ids_dev, int32_t* produced_dev, void* stream) {
  int rc = check_ready(c);
  if (rc) return rc;
  REC_CHECK_ARG(count >= 1 && count <= kMaxPacket, "packet must contain between 1 and %d tokens", kMaxPacket);
  REC_CHECK_ARG(n_eos >= 0 && n_eos <= kMaxEos && (n_eos == 0 || eos), "between 0 and %d EOS ids", kMaxEos);
  REC_CHECK_ARG(token >= -1 && token < c->d.vocab, "token %d outside the vocabulary", token);
  if (position < 0 || position + count > position_limit(c)) {
    set_error("Decode context limit exhausted");
    return REC_ELIMIT;
  }
  rc = select_schedule(c, position + count - 1);
  if (rc) return rc;
  int e8[8] = {-1, -1, -1, -1, -1, -1, -1, -1};
  for (int i = 0; i < n_eos; ++i) e8[i] = eos[i];
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  k_set_step<<<1, 32, 0, st>>>(c->ctl, token, position, n_eos, make_int4(e8[0], e8[1], e8[2], e8[3]),
                               make_int4(e8[4], e8[5], e8[6], e8[7]), 0);
  REC_CHECK_CUDA(cudaGetLastError());
  REC_CHECK_CUDA(launch_steps(c, count, st));
  if (ids_dev)
    REC_CHECK_CUDA(cudaMemcpyAsync(ids_dev, c->ctl + kCtlRecorded, size_t(count) * 4, cudaMemcpyDeviceToDevice, st));
  if (produced_dev)
    REC_CHECK_CUDA(cudaMemcpyAsync(produced_dev, c->ctl + kCtlProduced, 4, cudaMemcpyDeviceToDevice, st));
  return REC_OK;
}

REC_API int rec_decode_sampled(RecCtx* c, int32_t token, int32_t position, int32_t count,
                               const RecSampling* params, const float* uniforms_dev, int32_t* history_dev,
                               int32_t* history_len_dev, int32_t history_cap, const int32_t* eos, int32_t n_eos,
                               int32_t* ids_dev, int32_t* produced_dev, void* stream) {
  int rc = check_ready(c);
  if (rc) return rc;
  const int V = c->d.vocab;
  REC_CHECK_ARG(params && uniforms_dev, "rec_decode_sampled: null parameters or uniforms");
  REC_CHECK_ARG(count >= 1 && count <= kMaxPacket, "packet must contain between 1 and %d tokens", kMaxPacket);
  REC_CHECK_ARG(n_eos >= 0 && n_eos <= kMaxEos && (n_eos == 0 || eos), "between 0 and %d EOS ids", kMaxEos);
  REC_CHECK_ARG(token >= 0 && token < V, "token %d outside the vocabulary", token);
  REC_CHECK_ARG(V <= kSampleMaxVocab, "vocabulary above %d", kSampleMaxVocab);
  const RecSampling& p = *params;
  REC_CHECK_ARG(p.temperature > 0.0f && p.temperature < 1e30f, "rec_decode_sampled: temperature must be positive");
  REC_CHECK_ARG(p.repetition_penalty > 0.0f, "repetition penalty must be positive");
  REC_CHECK_ARG(p.top_k >= 0 && p.top_k < V && p.top_k <= kSampleMaxTopK, "top_k must be between 0 and %d",
                V - 1 < kSampleMaxTopK ? V - 1 : kSampleMaxTopK);
  REC_CHECK_ARG(p.top_p > 0.0f, "top_p must be positive");
  REC_CHECK_ARG(p.top_k > 0 || p.top_p >= 1.0f, "top_p < 1 needs top_k > 0");
  REC_CHECK_ARG(history_cap >= 0 && (history_cap == 0 || (history_dev && history_len_dev)),
                "rec_decode_sampled: a history needs its buffer and length");
  if (position < 0 || position + count > position_limit(c)) {
    set_error("Decode context limit exhausted");
    return REC_ELIMIT;
  }
  rc = select_schedule(c, position + count - 1);
  if (rc) return rc;
  int e8[8] = {-1, -1, -1, -1, -1, -1, -1, -1};
  for (int i = 0; i < n_eos; ++i) e8[i] = eos[i];
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  k_set_step<<<1, 32, 0, st>>>(c->ctl, token, position, n_eos, make_int4(e8[0], e8[1], e8[2], e8[3]),
                               make_int4(e8[4], e8[5], e8[6], e8[7]), 1);
  REC_CHECK_CUDA(cudaGetLastError());
  SampleArgs sa = {};
  sa.logits = c->logits;
  sa.stride = V;
  sa.V = V;
  sa.history = history_cap ? history_dev : nullptr;
  sa.n_hist = 0;
  sa.temperature = p.temperature;
  sa.top_k = p.top_k;
  sa.top_p = p.top_p;
  sa.rep = p.repetition_penalty;
  sa.presence = p.presence_penalty;
  sa.ids = c->ctl + kCtlArgmax;  // the id also lands in the packet's record and next-token slots
  sa.ctl = c->ctl;
  sa.hist_len = history_cap ? history_len_dev : nullptr;
  sa.hist_out = history_cap ? history_dev : nullptr;
  sa.hist_cap = history_cap;
  for (int i = 0; i < count; ++i) {
    REC_CHECK_CUDA(launch_steps(c, 1, st));
    sa.uniforms = uniforms_dev + size_t(i) * V;
    REC_CHECK_CUDA(launch_sample(sa, 1, st));
  }
  if (ids_dev)
    REC_CHECK_CUDA(cudaMemcpyAsync(ids_dev, c->ctl + kCtlRecorded, size_t(count) * 4, cudaMemcpyDeviceToDevice, st));
  if (produced_dev)
    REC_CHECK_CUDA(cudaMemcpyAsync(produced_dev, c->ctl + kCtlProduced, 4, cudaMemcpyDeviceToDevice, st));
  return REC_OK;
}

REC_API int32_t rec_schedule_for(const RecCtx* c, int32_t position) {
  if (!c) return -1;
  return schedule_for(c, position);
}

REC_API int rec_launch_kernel(RecCtx* c, int32_t kind, int32_t layer, void* stream) {
  int rc = check_ready(c);
  if (rc) return rc;
  REC_CHECK_ARG(kind >= 0 && kind < kKAll, "unknown kernel kind %d", kind);
  rc = ensure_graph(c);
  if (rc) return rc;
  REC_CHECK_ARG(layer >= 0 && layer < c->d.n_layers, "layer %d out of range", layer);
  REC_CHECK_ARG(kind < kKCount || layer_shared(c, layer), "layer %d has no shared expert", layer);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = c->d.scale_dtype == REC_SCALE_FP16 ? enqueue_kernel_sd<0>(c, kind, layer, st, false)
                                                     : enqueue_kernel_sd<1>(c, kind, layer, st, false);
  REC_CHECK_CUDA(e);
  return REC_OK;
}

REC_API int rec_router_moe(RecCtx* c, int32_t layer, void* h_dev, int32_t* ids_dev, float* weights_dev,
                           void* stream) {
  int rc = check_ready(c);
  if (rc) return rc;
  REC_CHECK_ARG(h_dev, "rec_router_moe: null residual");
  REC_CHECK_ARG(layer >= 0 && layer < c->d.n_layers, "layer %d out of range", layer);
  REC_CHECK_ARG(c->world == 1, "rec_router_moe runs on an unsharded session");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t hb = size_t(c->d.hidden) * 2;
  REC_CHECK_CUDA(cudaMemcpyAsync(c->h, h_dev, hb, cudaMemcpyDeviceToDevice, st));
  REC_CHECK_CUDA(c->d.scale_dtype == REC_SCALE_FP16 ? enqueue_ffn_sd<0>(c, layer, st, false)
                                                    : enqueue_ffn_sd<1>(c, layer, st, false));
  REC_CHECK_CUDA(cudaMemcpyAsync(h_dev, c->h, hb, cudaMemcpyDeviceToDevice, st));
  if (ids_dev)
    REC_CHECK_CUDA(cudaMemcpyAsync(ids_dev, c->ids, size_t(c->d.top_k) * 4, cudaMemcpyDeviceToDevice, st));
  if (weights_dev)
    REC_CHECK_CUDA(cudaMemcpyAsync(weights_dev, c->wts, size_t(c->d.top_k) * 4, cudaMemcpyDeviceToDevice, st));
  return REC_OK;
}

REC_API int rec_set_profile(RecCtx* c, void* buf_dev, size_t entries) {
  REC_CHECK_ARG(c, "null context");
  c->prof = static_cast<unsigned long long*>(buf_dev);
  c->prof_entries = buf_dev ? entries : 0;
  return REC_OK;
}

REC_API int rec_set_layer_profile(RecCtx* c, void* buf_dev, int32_t layer) {
  REC_CHECK_ARG(c, "null context");
  REC_CHECK_ARG(!buf_dev || (layer >= 0 && layer < c->d.n_layers), "layer out of range");
  c->prof2 = static_cast<unsigned long long*>(buf_dev);
  c->prof_layer = buf_dev ? layer : -1;
  return REC_OK;
}

REC_API int rec_check_status(RecCtx* c, void* stream) {
  REC_CHECK_ARG(c && c->ctl, "rec_check_status: session not configured");
  int s = 0;
  REC_CHECK_CUDA(cudaMemcpyAsync(&s, c->ctl + kCtlStatus, 4, cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream)));
  REC_CHECK_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  if (s != 0) {
    c->usable = false;
    set_error("GPU synchronization failed: device status %d", s);
  }
  return s;
}
