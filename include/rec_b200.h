/*
 * rec_b200 — C ABI of the B200 decode hot path of rec (single-session,
 * batch-1 decode of the Flint-style MoE transformer).
 *
 * Conventions
 *   - Every pointer named *_dev is device memory owned by the caller (torch);
 *     the library keeps non-owning views and allocates no device memory.
 *   - Every call is stream-ordered and non-blocking unless stated otherwise;
 *     `stream` is a cudaStream_t passed as void*.
 *   - Return codes: 0 ok; < 0 argument error (the Python shim raises
 *     ValueError); > 0 device status (a bounded device wait ran out or the
 *     device rejected an input; the shim raises RuntimeError and marks the
 *     session unusable).  Details: rec_last_error().
 *   - bf16 / fp16 tensors are passed as uint16_t storage.
 *
 * Reference interfaces replaced (paths inside recursive-oss/rec):
 *   engine/src/rec_mlx/kernels/megakernel.py:983-1337  FullModel (forward,
 *       prefill_state, ensure_capacity), the `flint_decode` Metal kernel
 *   engine/src/rec_mlx/kernels/sampling.py:17-169       ResidentSampler.block
 *   engine/src/rec_mlx/kernels/masked_sampling.py:7-212 filtered sampling
 *   engine/src/rec_mlx/kernels/resident_block.py:12-88   grid argmax packet
 *   engine/src/rec_mlx/cache.py:6-46                     KV write kernels
 *   engine/src/rec_mlx/model.py:40-139,216-254           native MLX ops
 */
#ifndef REC_B200_H
#define REC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
#define REC_EXTERN extern "C"
#else
#define REC_EXTERN
#endif
#define REC_API REC_EXTERN __attribute__((visibility("default")))

enum {
  REC_OK = 0,
  REC_EINVAL = -1,      /* bad argument / unsupported shape */
  REC_ECUDA = -2,       /* CUDA runtime error at launch */
  REC_ESTATE = -3,      /* session unusable or not configured */
  REC_ELIMIT = -4,      /* context limit exhausted */
  REC_DEV_BULK_TIMEOUT = 1,
  REC_DEV_COUNTER_TIMEOUT = 2,
  REC_DEV_BAD_TOKEN = 3,
  REC_DEV_BAD_POSITION = 4,
};

/* Scale/bias storage type of quantized weights. */
enum { REC_SCALE_FP16 = 0, REC_SCALE_BF16 = 1 };
/* Router modes: softmax -> top-k -> renormalise; sigmoid + bias selection
 * (reference model.py:245-254). */
enum { REC_ROUTER_SOFTMAX = 0, REC_ROUTER_SIGMOID = 1 };
/* Model flags. */
enum { REC_FLAG_SINKS = 1, REC_FLAG_QK_NORM = 2 };
/* Layer kinds (RecLayerWeights.kind bits), the reference Flint model's layer
 * options (engine/src/rec_mlx/model.py:14-37,155-163,216-271):
 *   REC_LAYER_DENSE    the FFN is a dense SwiGLU MLP of dense_inter rows
 *                      (`mlp_only_layers`, model.py:216-224,262-266) instead of
 *                      the routed experts; gate/up/down hold its matrices;
 *   REC_LAYER_NO_ROPE  no rotary embedding of q and k (`no_rope_layer_indices`,
 *                      the "global" layers, model.py:158-163,196-198);
 *   REC_LAYER_SLIDING  attention over the last sliding_window positions only
 *                      (`layer_types` "sliding_attention", model.py:281-313).
 * A model that uses any of them, or a shared expert, runs on the graph
 * schedule of separate kernels. */
enum { REC_LAYER_DENSE = 1, REC_LAYER_NO_ROPE = 2, REC_LAYER_SLIDING = 4 };

/* Model shape (reference ModelArgs, engine/src/rec_mlx/model.py:14-37). */
typedef struct RecModelDesc {
  int32_t hidden;      /* H = 2048 */
  int32_t n_layers;    /* 1..64 */
  int32_t n_q_heads;   /* 8 * n_kv_heads, with n_q_heads * 128 = 2048 or 4096 */
  int32_t n_kv_heads;
  int32_t head_dim;    /* 128 */
  int32_t n_experts;   /* E <= 1024 */
  int32_t top_k;       /* k <= 8 */
  int32_t moe_inter;   /* I: 256, 512, 768 or 1024 */
  int32_t vocab;       /* V */
  int32_t group_size;  /* 64 */
  int32_t scale_dtype; /* REC_SCALE_* of the int4 weights */
  int32_t kv_bits;     /* 4 or 8 (KV scales/biases are bf16); 16: bf16 K / V rows,
                        * the reference megakernel's kv_format "bf16" (graph
                        * schedule; RecKVLayer codes = bf16 [Hkv, C, 128], no
                        * scales or biases) */
  int32_t router_mode; /* REC_ROUTER_* */
  int32_t flags;       /* REC_FLAG_* */
  float rms_eps;
  float rope_theta;
  /* Flint layer options (0 = off).  shared_inter: rows of the always-on
   * shared SwiGLU expert of every MoE layer (256, 512, 768 or 1024), added to
   * the routed mix as mlp = bf16(mix + shared) before the residual
   * (model.py:243,254; megakernel.py:955-958).  dense_inter: rows of the
   * dense MLP of REC_LAYER_DENSE layers (2048, 4096 or 6144).  sliding_window:
   * positions a REC_LAYER_SLIDING layer attends, the current one included
   * (the reference's window is 513). */
  int32_t shared_inter;
  int32_t dense_inter;
  int32_t sliding_window;
  /* bits of the embedding's affine g64 codes: 4 (0 means 4) or 8 (the
   * production checkpoint's embedding, mixed_bits.py:25-30;
   * graph schedule) */
  int32_t embed_bits;
  /* bits of the V codes when they differ from the K codes' (kv_bits): 0
   * (same), 4 or 8 -- the reference's MixedQuantizedKVCache keeps K at 8 and
   * V at 4 bits (model.py:35-37,40-82); a mixed cache runs on the graph
   * schedule, V codes uint32[Hkv, C, 128*kv_value_bits/32] */
  int32_t kv_value_bits;
} RecModelDesc;

/* int4 g64 affine matrix in MLX layout: codes uint32[N, K/8], scales and
 * biases [N, K/64] (reference megakernel.py:161-170). */
typedef struct RecQMat {
  const void* w;
  const void* scales;
  const void* biases;
} RecQMat;

typedef struct RecLayerWeights {
  const void* input_norm; /* bf16 [H] */
  const void* post_norm;  /* bf16 [H] */
  RecQMat q, k, v, o;     /* [Hq*D, H], [Hkv*D, H] x2, [H, Hq*D] */
  const void* router;     /* bf16 [E, H] */
  const void* expert_bias;/* fp32 [E] (sigmoid router) or NULL */
  RecQMat gate, up, down; /* [E*I, H], [E*I, H], [E*H, I] */
  const void* sinks;      /* bf16 [Hq] or NULL */
  const void* q_norm;     /* bf16 [D] or NULL */
  const void* k_norm;     /* bf16 [D] or NULL */
  int32_t kind;           /* REC_LAYER_* bits (0: routed experts, RoPE, full attention) */
  /* the shared expert of an MoE layer when shared_inter > 0: [Is, H], [Is, H],
   * [H, Is]; otherwise unused.  A REC_LAYER_DENSE layer has no router: its
   * gate/up/down are [Id, H], [Id, H], [H, Id] and router may be NULL. */
  RecQMat shared_gate, shared_up, shared_down;
} RecLayerWeights;

typedef struct RecGlobalWeights {
  RecQMat embed;          /* int4 [V, H] (int8 with embed_bits = 8: codes uint32[V, H/4]) */
  const void* final_norm; /* bf16 [H] */
  RecQMat lm_head;        /* int4 [V, H] */
} RecGlobalWeights;

/* One layer of quantized KV cache (reference MixedQuantizedKVCache,
 * model.py:40-82): codes uint32[Hkv, C, D*bits/32], scales/biases bf16
 * [Hkv, C, D/64]. */
typedef struct RecKVLayer {
  void* k_codes;
  void* k_scales;
  void* k_biases;
  void* v_codes;
  void* v_scales;
  void* v_biases;
} RecKVLayer;

/* Sampling parameters of the sampling head (reference engine.py:206-212,
 * masked_sampling.py:98-125, filtered_sampling.py:7-22). */
typedef struct RecSampling {
  float temperature;        /* 0 = greedy */
  int32_t top_k;            /* 0 = off; <= 256 */
  float top_p;              /* >= 1 = off; < 1 needs top_k > 0 */
  float repetition_penalty; /* 1 = off: x<0 ? x*p : x/p for ids in the history */
  float presence_penalty;   /* 0 = off: x - p for ids in the history */
} RecSampling;

typedef struct RecCtx RecCtx;

/* ---- session ----------------------------------------------------------- */
REC_API int rec_create(const RecModelDesc* desc, RecCtx** out);
REC_API void rec_destroy(RecCtx* ctx);
REC_API int rec_set_weights(RecCtx* ctx, const RecLayerWeights* layers, int32_t n_layers,
                            const RecGlobalWeights* global);
/* capacity: KV slots per layer (multiple of 256). */
REC_API int rec_set_kv(RecCtx* ctx, const RecKVLayer* layers, int32_t n_layers, int32_t capacity);
/* Rows [0, rows) of every head of the cache are backed by memory; positions
 * at or above rows are refused (REC_ELIMIT) while `capacity` stays the head
 * stride.  For a cache reserved at its final capacity in virtual memory and
 * backed block by block as the context grows (no copy of the rows already
 * written; rec_b200/vmm.py).  rows: a multiple of 256, at most the capacity;
 * rec_set_kv resets it to the capacity.  Replaces the reference's KV growth by
 * appended bank blocks (engine/src/rec_mlx/cache.py:47-84). */
REC_API int rec_set_kv_rows(RecCtx* ctx, int32_t rows);
REC_API size_t rec_workspace_bytes(const RecCtx* ctx);
REC_API int rec_set_workspace(RecCtx* ctx, void* workspace_dev, size_t bytes);
/* One decode step: embeds `token` at `position`, runs every layer, writes
 * bf16 logits[V] and (optional) the residual trace bf16[L+1, H].  Replaces
 * FullModel.forward (megakernel.py:1224-1301). */
REC_API int rec_decode_step(RecCtx* ctx, int32_t token, int32_t position, void* logits_dev,
                            void* trace_dev, void* stream);
/* rec_decode_step through the first layer_count layers only (1 <= layer_count
 * <= n_layers): the final norm and lm_head follow the last layer run, the
 * trace holds rows 0..layer_count, and the deeper layers' cache rows at this
 * position are not written.  Runs on the persistent kernel (n_experts <=
 * 256).  Replaces FullModel.forward(state, token, layer_count)
 * (engine/src/rec_mlx/kernels/megakernel.py:824,861,1224-1233,1272). */
REC_API int rec_decode_layers(RecCtx* ctx, int32_t token, int32_t position, int32_t layer_count, void* logits_dev,
                              void* trace_dev, void* stream);
/* Tests of the failure path only (no reference counterpart; the reference's
 * spin-capped grid barrier is megakernel.py:137-159): the persistent
 * kernel's grid-barrier poll bound (0 restores the default) and one CTA
 * (index, or -1 for none) that never arrives at a grid barrier.  With a CTA
 * skipping, every CTA's bounded wait runs out, the kernel sets device status
 * REC_DEV_COUNTER_TIMEOUT and returns; the next rec_check_status reports it
 * and marks the session unusable. */
REC_API int rec_set_fault_injection(RecCtx* ctx, uint32_t barrier_spin_limit, int32_t skip_arrive_cta);
/* Up to `count` greedy steps with the argmax fed back on the device; stops
 * after an EOS id.  ids_dev int32[count] receives the produced ids, produced_dev
 * int32[1] their number.  token = -1 continues from the token and position
 * the device holds after the previous call (no host round trip).  Replaces
 * ResidentSampler.block for temperature 0 (sampling.py:62-169,
 * resident_block.py:12-88). */
REC_API int rec_decode_greedy(RecCtx* ctx, int32_t token, int32_t position, int32_t count,
                              const int32_t* eos, int32_t n_eos, int32_t* ids_dev,
                              int32_t* produced_dev, void* stream);
/* A packet of up to 64 tokens sampled on the device (temperature > 0):
 * each step decodes one token and samples the next id from the logits with
 * that step's uniforms (fp32 [count, vocab]; the rules of rec_sample_logits),
 * and the id is fed back without a host round trip.  history_dev (int32
 * [history_cap]) holds *history_len_dev ids that the penalties apply to; each
 * sampled id is appended (up to history_cap).  Ids are recorded until an EOS
 * id (included); ids_dev / produced_dev as for rec_decode_greedy.  Replaces
 * ResidentSampler.block at temperature > 0 with its device-side Gumbel
 * feedback (engine/src/rec_mlx/kernels/sampling.py:17-60,62-169,
 * resident_block.py:62-88). */
REC_API int rec_decode_sampled(RecCtx* ctx, int32_t token, int32_t position, int32_t count,
                               const RecSampling* params, const float* uniforms_dev, int32_t* history_dev,
                               int32_t* history_len_dev, int32_t history_cap, const int32_t* eos, int32_t n_eos,
                               int32_t* ids_dev, int32_t* produced_dev, void* stream);
/* ---- one session over several GPUs (one process per GPU) ----------------
 * Expert parallelism + split-KV along the sequence: rank r holds experts
 * [expert_lo, expert_hi) (its layer weights' gate/up/down hold only those,
 * stacked in order) and the KV of super-chunks [super_lo, super_hi) (64
 * blocks of 256 tokens each; its cache starts at token_base = super_lo *
 * 16384 and rec_set_kv gets its local capacity).  Dense weights, embedding
 * and lm_head are replicated.  The persistent kernel exchanges super-chunk
 * attention partials and per-expert outputs between the ranks through peer
 * stores into each rank's exchange buffer (NVLink), with bounded waits; the
 * merges keep the single-GPU order, so every rank's logits equal the
 * single-GPU ones bit for bit.  Replaces the reference's planned split-KV /
 * expert-parallel partitioning (BASELINE configs 2 and 4); no reference
 * counterpart in code.  Call order: rec_create, rec_set_shard,
 * rec_set_weights, rec_set_kv, rec_exchange_bytes (allocate the exchange
 * buffer as peer-mapped memory, zeroed, on every rank), rec_set_shard again
 * with the peer pointers, rec_set_workspace. */
typedef struct RecShard {
  int32_t world, rank;
  int32_t expert_lo, expert_hi;
  int32_t super_lo, super_hi;
  int32_t capacity_total;  /* global context capacity (positions), multiple of 256 */
  void* exchange[8];       /* rank q's exchange buffer as mapped in this process */
  int32_t schedule;        /* 0: the persistent kernel; 1: the graph of standalone kernels
                              (attention on each rank's KV with the standalone kernel, the
                              super-chunk and expert-output exchanges as separate kernels);
                              fixed for the session's lifetime */
} RecShard;
REC_API int rec_set_shard(RecCtx* ctx, const RecShard* shard);
REC_API size_t rec_exchange_bytes(const RecCtx* ctx);

/* Schedule of a decode step at `position`: 0 = one persistent cooperative
 * kernel per call; 1 = a CUDA graph of separate kernels per step (7 per layer
 * + 3); 2 = split: per step, persistent-kernel segments (embedding + Q of
 * layer 0; then per layer O, router, experts and the next layer's Q, the
 * last with the lm_head) around each layer's standalone attention kernels
 * (3 per layer + 1 launches).  REC_SCHEDULE=mega / graph / split forces one;
 * otherwise 0 while one layer's attended KV is below 24 MiB (about 43K
 * tokens with a 4-bit cache, 23K with an 8-bit one) and 1 above it, where
 * the standalone attention kernel is faster; 2 runs only when forced.  More
 * than 256 experts always take 1; sessions split over ranks run on 0.  -1
 * for a null context.  (The
 * reference's step is always its single Metal dispatch,
 * megakernel.py:1224-1301.) */
REC_API int32_t rec_schedule_for(const RecCtx* ctx, int32_t position);
/* Kernels of one step, in launch order; layer kernels repeat per layer. */
enum {
  REC_K_EMBED = 0, REC_K_QKV = 1, REC_K_ATTN = 2, REC_K_COMBINE = 3, REC_K_OPROJ = 4, REC_K_ROUTER = 5,
  REC_K_GATEUP = 6, REC_K_DOWN = 7, REC_K_HEAD = 8, REC_K_STEP_END = 9
};
/* Launches one kernel of the step on `stream` against the session's current
 * state (profiling and per-kernel timing; no reference counterpart: the
 * reference's step is a single Metal dispatch). */
REC_API int rec_launch_kernel(RecCtx* ctx, int32_t kind, int32_t layer, void* stream);
/* The MoE block of one layer on a residual vector, with the session's
 * weights: x = RMSNorm(h, post_norm); logits = bf16(Wr x); softmax or
 * sigmoid + bias selection of top_k experts, weights renormalised;
 * h <- bf16(h + mix), mix = the selected experts' bf16 SwiGLU FFN outputs
 * times bf16(weight), summed in bf16 in selection order.  h_dev (bf16
 * [hidden]) is read and overwritten; ids_dev (int32 [top_k]) and weights_dev
 * (float [top_k]) receive the selection when non-NULL.  Replaces Router /
 * SparseMoeBlock.__call__ (engine/src/rec_mlx/model.py:227-254), mlx-lm's
 * SwitchGLU and the reference's route/expert kernels (megakernel.py:406-435,
 * 696-798; mixed_bits.py:32-54).  Unsharded sessions only. */
REC_API int rec_router_moe(RecCtx* ctx, int32_t layer, void* h_dev, int32_t* ids_dev, float* weights_dev,
                           void* stream);
/* Optional phase timeline of the persistent decode kernel: when set, every
 * CTA stamps %globaltimer (ns) at each grid-barrier arrival and release into
 * buf_dev as uint64 [barrier][cta][2]; a step has 6*n_layers + 1 barriers.
 * Counterpart of the reference's PROFILE schedule flag
 * (megakernel.py:151,1269-1299).  NULL disables. */
REC_API int rec_set_profile(RecCtx* ctx, void* buf_dev, size_t entries);
/* Optional stamps inside one layer (step 0 of a launch) of the persistent
 * kernel: uint64 [cta][64] %globaltimer values at fixed points of the
 * attention and expert phases (diagnostics; no reference counterpart).  The
 * stamps exist only in a library built with REC_LAYER_STAMPS=1 (see
 * rec_b200/build.py); otherwise the buffer is left untouched. */
REC_API int rec_set_layer_profile(RecCtx* ctx, void* buf_dev, int32_t layer);
/* Reads the device status word (synchronises `stream`).  Non-zero marks the
 * session unusable. */
REC_API int rec_check_status(RecCtx* ctx, void* stream);
REC_API int rec_last_error(char* buf, size_t len);

/* Quantize-on-append of one token's K and V rows (bf16 [n_kv_heads * 128]
 * each, K already RoPE'd) into row *position_dev of every head of a cache
 * layer: MLX affine quantization, group 64 along head_dim, bf16 scale and
 * bias.  Replaces the append of MixedQuantizedKVCache.update_and_fetch
 * (engine/src/rec_mlx/model.py:45-82) and the KV write kernels
 * (cache.py:6-46); the persistent decode kernel fuses the same step into its
 * attention phase.  A position outside [0, capacity) sets *status_dev to 4
 * and writes nothing. */
REC_API int rec_kv_append(const RecKVLayer* kv, int32_t n_kv_heads, int32_t capacity, int32_t kv_bits,
                          const void* k_dev, const void* v_dev, const int32_t* position_dev, int32_t* status_dev,
                          void* stream);
/* rec_kv_append for a prefill chunk: the t tokens' K and V rows (bf16
 * [t, n_kv_heads * 128] each, K already RoPE'd) into rows [position,
 * position + t) of every head, with the same arithmetic per row (the bulk
 * quantize-on-append of the reference's prefill: update_and_fetch over a
 * chunk, model.py:45-82).  Rows outside [0, capacity) are an argument
 * error. */
REC_API int rec_kv_append_bulk(const RecKVLayer* kv, int32_t n_kv_heads, int32_t capacity, int32_t kv_bits,
                               const void* k_dev, const void* v_dev, int32_t position, int32_t t, void* stream);

/* ---- kernel entry points used by the unit tests -------------------------- */
/* y = W x (int4 g64) with an optional fused RMSNorm prologue on x. */
REC_API int rec_gemv_int4(const RecQMat* w, int32_t scale_dtype, int64_t n, int32_t k,
                          const void* x_dev, const void* norm_weight_dev, float eps, void* y_dev,
                          void* stream);
/* y = W x (int4 g64, optional fused RMSNorm on x) and the greedy token
 * argmax(y) (lowest index among equal maxima, as the decode step's lm_head)
 * without any caller-provided scratch.  No counterpart in the reference: its
 * argmax kernel always runs inside a session that owns its buffers.
 *
 * For callers that cannot allocate device memory: a plain C or ctypes host
 * that has no device allocator of its own (the library allocates nothing, and
 * every other entry point that needs scratch takes it from a session
 * workspace), or a sampler that runs in a process whose HBM is already handed
 * out in full to weight banks and the KV pool, where an extra cudaMalloc
 * fails or fragments the pool.
 *
 * The cross-CTA scratch (arrival counter, per-CTA candidates and, when y_dev
 * is NULL, the bf16 logits) is one static device array of 532,736 bytes per
 * device.  Limits: N <= 262,144 rows when y_dev is NULL (larger N is rejected
 * with REC_EINVAL; pass y_dev for a larger vocabulary); N even, K as in
 * rec_gemv_int4.  token_dev receives -1 if a bounded device wait ran out;
 * the logits in y_dev (when given) are then undefined, possibly partly
 * written.
 * The first call on each device looks up the array's device address (with
 * that device current) and sets the kernels' shared-memory limit; make that
 * first call before any stream capture.  Every call shares the array and it
 * keeps the last call's contents (each call clears what must start at zero):
 * calls that overlap on the GPU (different streams or threads) race on it.
 * The call allocates nothing: no cudaMalloc, no cudaFree, no library
 * allocator. */
REC_API int rec_gemv_int4_argmax_noalloc(const RecQMat* w, int32_t scale_dtype, int64_t n, int32_t k,
                                         const void* x_dev, const void* norm_weight_dev, float eps,
                                         void* y_dev, int32_t* token_dev, void* stream);
/* Samples one id per row of bf16 logits [batch, stride] (vocab <= 262,144):
 * penalties over the row's history (int32 [batch, history_len]), then greedy
 * argmax (temperature 0), or temperature / top-k / top-p with the injected
 * uniforms (fp32 [batch, vocab], u in [0, 1)) as Gumbel noise -log(-log u).
 * Replaces the reference's sampler step (engine.py:279-301,
 * masked_sampling.py:98-125, filtered_sampling.py:7-22, sampling.py:48-52).
 * ids_dev[b] = -1 when more than 1,024 logits tie at the top-k threshold. */
REC_API int rec_sample_logits(const void* logits_dev, int32_t batch, int32_t vocab, int64_t stride,
                              const int32_t* history_dev, int32_t history_len, const RecSampling* params,
                              const float* uniforms_dev, int32_t* ids_dev, void* stream);
/* rec_sample_logits with a grammar allow-mask: allow_dev (uint32 [batch,
 * allow_stride], allow_stride >= ceil(vocab / 32)) has bit (i & 31) of word
 * i >> 5 set for each allowed id i of the row.  Disallowed ids get -inf after
 * the penalties (the reference's grammar handoff, masked_sampling.py:101-110);
 * top-k counts allowed ids only; a row with no allowed id gives -1.  NULL
 * allow_dev is rec_sample_logits. */
REC_API int rec_sample_logits_masked(const void* logits_dev, int32_t batch, int32_t vocab, int64_t stride,
                                     const int32_t* history_dev, int32_t history_len, const RecSampling* params,
                                     const float* uniforms_dev, const uint32_t* allow_dev, int64_t allow_stride,
                                     int32_t* ids_dev, void* stream);
/* Log-probability of each row's chosen id (ids_dev int32 [batch]) as the
 * reference reports it: report = x / T (temperature > 0) or x, x the logits
 * after the penalties over the history and the optional grammar mask (the
 * rules of rec_sample_logits_masked); logprob_dev[b] = report[id] -
 * logsumexp(report) over the whole vocabulary (fp32, the library's own exp
 * and log).  NaN for an id outside [0, vocab); -inf when no logit is finite.
 * top_k / top_p do not enter.  Replaces the logprob report of the reference
 * (engine/src/rec_mlx/engine.py:294-296; kernels/masked_sampling.py:126-128,
 * 145-146, 205-206). */
REC_API int rec_token_logprob(const void* logits_dev, int32_t batch, int32_t vocab, int64_t stride,
                              const int32_t* history_dev, int32_t history_len, const RecSampling* params,
                              const uint32_t* allow_dev, int64_t allow_stride, const int32_t* ids_dev,
                              float* logprob_dev, void* stream);
/* The sampling head for `batch` hidden rows (bf16 [batch, hidden]):
 * logits[b] = lm_head . RMSNorm(h[b], final_norm) (int4 g64 GEMV into
 * logits_dev, bf16 [batch, vocab]), then rec_sample_logits on those rows with
 * the history, parameters and uniforms as documented there.  Replaces the
 * final norm + lm_head of Model.__call__ (engine/src/rec_mlx/model.py:324-327)
 * followed by the reference's sampler step (engine.py:279-301). */
REC_API int rec_lmhead_sample(const RecQMat* lm_head, int32_t scale_dtype, int32_t vocab, int32_t hidden,
                              const void* h_dev, int32_t batch, const void* final_norm_dev, float eps,
                              const int32_t* history_dev, int32_t history_len, const RecSampling* params,
                              const float* uniforms_dev, void* logits_dev, int32_t* ids_dev, void* stream);
/* Workspace (bytes) of rec_prefill_chunk for a chunk of t tokens. */
REC_API size_t rec_prefill_workspace_bytes(const RecCtx* ctx, int32_t t);
/* Chunked prompt prefill: the t tokens of tokens_dev (int32) at positions
 * [position, position + t) through every layer of the session -- embedding,
 * RMSNorm, q / k / v / o projections and the MoE block on the tensor cores
 * (rec_prefill_gemm, rec_prefill_moe), q / k head norms and RoPE, the chunk's
 * K / V quantized into the cache (rec_kv_append_bulk), causal attention of
 * every token over the quantized cache at positions 0 .. its own, the
 * router of every token -- and, when logits_dev is non-NULL, the bf16 logits
 * of the last token (final norm + lm_head).  The cache rows then hold what
 * the chunk wrote, and decoding continues at position + t.  Dense work
 * accumulates in fp32 on the tensor cores, so results match the
 * token-by-token decode within a tolerance, not bit for bit.  workspace:
 * 256-byte aligned, rec_prefill_workspace_bytes(ctx, t) bytes.  Unsharded
 * sessions, hidden 2048.  Replaces QATSession.prefill's chunk step
 * (engine/src/rec_mlx/quantized.py:102-148; m4_max_prefill.py:6-104;
 * kernels/m4_max_prefill.py:49-144). */
REC_API int rec_prefill_chunk(RecCtx* ctx, const int32_t* tokens_dev, int32_t position, int32_t t, void* logits_dev,
                              void* workspace, size_t workspace_bytes, void* stream);
/* rec_prefill_chunk over layers [layer_begin, layer_end) only, so that a
 * caller can stop between layers: the range starting at 0 embeds tokens_dev
 * (which later ranges may pass as NULL), the chunk's hidden states stay in
 * the workspace between ranges (the same workspace, the same t and
 * position), and the range ending at the last layer writes the logits.
 * Layer ranges that cover 0 .. n_layers in order give the same bits as one
 * rec_prefill_chunk.  Replaces the per-layer stop poll of the reference's
 * prefill (quantized.py:129-133 with interrupt_between_layers;
 * model.py:309-314). */
REC_API int rec_prefill_chunk_layers(RecCtx* ctx, const int32_t* tokens_dev, int32_t position, int32_t t,
                                     int32_t layer_begin, int32_t layer_end, void* logits_dev, void* workspace,
                                     size_t workspace_bytes, void* stream);
/* The causal attention step of rec_prefill_chunk alone: q_dev bf16 [t,
 * n_q_heads, 128] (RoPE'd, not scaled) at positions [position, position + t)
 * attends over cache rows 0 .. its own position (the chunk's rows already
 * appended): scores bf16(bf16(q / sqrt(128)) . k), fp32 softmax with the
 * optional sink logit, P . V with fp16 P and V, fp32 accumulation; out bf16
 * [t, n_q_heads * 128].  Replaces the prefill path of
 * quantized_attention_with_sinks (engine/src/rec_mlx/model.py:108-139). */
REC_API int rec_prefill_attention(const void* q_dev, int32_t n_q_heads, int32_t n_kv_heads, const RecKVLayer* kv,
                                  int32_t capacity, int32_t kv_bits, int32_t position, int32_t t, const void* sinks_dev,
                                  void* out_dev, void* stream);
/* Prefill projection on the tensor cores: Y[t, n] = X[t, k] . W[n, k]^T with
 * X bf16 [t, k] row-major (16-byte aligned), W int4 g64 (MLX affine layout,
 * scale_dtype scales and biases), Y bf16 [t, n].  n a multiple of 256, k a
 * multiple of 64.  tcgen05 MMAs accumulate in fp32 in tensor memory from bf16
 * operands (the weights are dequantized to bf16), so results match an fp32
 * GEMM of the dequantized weights within bf16 rounding, not bit for bit.
 * *status_dev is set to 1 if a bounded device wait ran out.  Replaces the
 * quantized projections of the reference's chunked prefill
 * (engine/src/rec_mlx/quantized.py:102-148, kernels/m4_max_prefill.py:49-144). */
REC_API int rec_prefill_gemm(const RecQMat* w, int32_t scale_dtype, int64_t n, int32_t k, const void* x_dev,
                             int64_t t, void* y_dev, int32_t* status_dev, void* stream);
/* Workspace (bytes) of rec_prefill_moe for t tokens, k experts per token, the
 * hidden and expert-intermediate sizes and the expert count; 0 for bad sizes. */
REC_API size_t rec_prefill_moe_workspace_bytes(int64_t t, int32_t k, int32_t hidden, int32_t inter,
                                               int32_t n_experts);
/* MoE block of a prefill chunk on the tensor cores.  x bf16 [t, hidden]: the
 * post-attention RMSNorm of the tokens; ids int32 [t, k] and weights fp32
 * [t, k]: each token's experts in rank order and their renormalised weights
 * (the router's output); gate, up int4 g64 [n_experts * inter, hidden] and
 * down [n_experts * hidden, inter] (the layer's stacked expert matrices).
 * The (token, rank) pairs are grouped by expert and each expert's rows go
 * through one grouped tcgen05 GEMM per matrix (rec_prefill_gemm's kernel,
 * one 128-row tile table for all experts); act = bf16(bf16(g * bf16(
 * sigmoid(g))) * u); y[t] = resid[t] + the pairs' d * bf16(w) summed in rank
 * order with a bf16 rounding after each add (resid may be null: y = the
 * mix).  hidden and inter multiples of 256.  workspace: 256-byte aligned,
 * rec_prefill_moe_workspace_bytes of it; *status_dev is set when a bounded
 * wait runs out or an expert id is outside [0, n_experts) (that pair is
 * skipped).  Replaces the grouped expert GEMMs of the reference's prefill
 * (engine/src/rec_mlx/m4_max_prefill.py:27-46 PrefillSwitchGLU,
 * kernels/m4_max_prefill.py:111-144 gate_up) and the SwitchGLU of
 * model.py:242-254 over the prompt's tokens. */
REC_API int rec_prefill_moe(const RecQMat* gate, const RecQMat* up, const RecQMat* down, int32_t scale_dtype,
                            int32_t n_experts, int32_t inter, int32_t hidden, const void* x_dev, int64_t t,
                            int32_t k, const int32_t* ids_dev, const float* weights_dev, const void* resid_dev,
                            void* y_dev, void* workspace, size_t workspace_bytes, int32_t* status_dev, void* stream);
/* Decode attention of one layer alone (unit tests, the attention sweep):
 * quantizes the new K / V of `*position_dev` from qkv_dev (bf16 [Hq*128 |
 * Hkv*128 | Hkv*128], RoPE from rope_dev [positions][cos 64 | sin 64]) into
 * the cache, then attends q over positions [0, position] with optional sinks;
 * out bf16 [Hq*128].  scratch_dev: rec_attn_scratch_bytes(Hq, capacity) bytes,
 * 256-byte aligned.  Replaces quantized_attention_with_sinks + the KV write
 * (model.py:45-82,108-139; megakernel.py:276-318,619-693). */
REC_API size_t rec_attn_scratch_bytes(int32_t n_q_heads, int32_t capacity);
REC_API int rec_attn_decode(const void* qkv_dev, int32_t n_q_heads, int32_t n_kv_heads, const RecKVLayer* kv,
                            int32_t capacity, int32_t kv_bits, const float* rope_dev, const void* sinks_dev,
                            const int32_t* position_dev, void* scratch_dev, size_t scratch_bytes, void* out_dev,
                            int32_t* status_dev, void* stream);
/* MLX affine quantization of fp32 groups into codes + (bf16|fp16) scale/bias. */
REC_API int rec_quantize_affine(const float* w_dev, int64_t n_groups, int32_t bits,
                                int32_t scale_dtype, void* codes_dev, void* scales_dev,
                                void* biases_dev, void* stream);
/* The SiLU table: out_dev bf16[65536], entry i = bf16(bf16(g * bf16(sigmoid(g)))
 * * 1) for the gate g whose bf16 bits are i — the decode path's gate/up
 * epilogue with u = 1.  Replaces the engine's `silu` table
 * (megakernel.py:1110-1112: swiglu over every bf16 gate, up = 1). */
REC_API int rec_silu_table(void* out_dev, void* stream);

#endif /* REC_B200_H */
