// Log-probability of the chosen token, as the reference engine reports it
// (engine/src/rec_mlx/engine.py:294-296 for the first token,
// kernels/masked_sampling.py:126-128 inside resident packets):
//   report = x / T (T > 0) or x (T = 0), x = the logits after the penalties
//   and the grammar mask (the sampler's x, sample.cuh);
//   logprob = report[id] - logsumexp(report).
// It is computed over the full vocabulary, not over the top-k / top-p
// survivors, exactly as the reference does.
//
// Canonical order (restated by oracle/rec_oracle.c:orc_token_logprob): one
// CTA of 1024 threads per row; M = max report (exact); thread t sums
// exp(report_i - M) for i = t, t + 1024, ... in order, then a butterfly over
// the warp (xor 16, 8, 4, 2, 1), then the 32 warp sums in order: S;
// lse = M + log(S) with the library's own exp and log (common.cuh).  An id
// outside [0, V) gives NaN; a row with no finite logit gives -inf.
#include "capi_common.h"
#include "common.cuh"

using namespace rec;

namespace {

constexpr int kLpThreads = 1024;
constexpr int kLpMaxVocab = 262144;

struct LogprobArgs {
  const uint16_t* logits;
  int64_t stride;
  int V;
  const int* history;
  int n_hist;
  float temperature, rep, presence;
  const uint32_t* allow;
  int64_t allow_stride;
  const int* ids;
  float* out;
};

__global__ void __launch_bounds__(kLpThreads) k_token_logprob(const LogprobArgs a) {
  __shared__ unsigned seen[kLpMaxVocab / 32];
  __shared__ float red[32];
  __shared__ float Mshared;
  const int b = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const uint16_t* lg = a.logits + size_t(b) * a.stride;
  const uint32_t* allow = a.allow ? a.allow + size_t(b) * a.allow_stride : nullptr;
  const bool pen = a.rep != 1.0f || a.presence != 0.0f;
  if (pen) {
    for (int i = t; i < (a.V + 31) / 32; i += kLpThreads) seen[i] = 0u;
    __syncthreads();
    for (int i = t; i < a.n_hist; i += kLpThreads) {
      const int id = a.history[size_t(b) * a.n_hist + i];
      if (id >= 0 && id < a.V) atomicOr(&seen[id >> 5], 1u << (id & 31));
    }
    __syncthreads();
  }
  auto Y = [&](int i) -> float {
    if (allow && !((allow[i >> 5] >> (i & 31)) & 1u)) return -INFINITY;
    float x = bf(lg[i]);
    if (pen && ((seen[i >> 5] >> (i & 31)) & 1u)) {
      if (a.rep != 1.0f) x = x < 0.0f ? __fmul_rn(x, a.rep) : __fdiv_rn(x, a.rep);
      if (a.presence != 0.0f) x = __fsub_rn(x, a.presence);
    }
    x = __fadd_rn(x, 0.0f);
    return a.temperature > 0.0f ? __fdiv_rn(x, a.temperature) : x;
  };
  float m = -INFINITY;
  for (int i = t; i < a.V; i += kLpThreads) m = fmaxf(m, Y(i));
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (t == 0) {
    float r = red[0];
    for (int w = 1; w < 32; ++w) r = fmaxf(r, red[w]);
    Mshared = r;
  }
  __syncthreads();
  const float M = Mshared;
  __syncthreads();  // red is reused below
  float s = 0.0f;
  if (M != -INFINITY)
    for (int i = t; i < a.V; i += kLpThreads) s = __fadd_rn(s, rexp(__fsub_rn(Y(i), M)));
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (t == 0) {
    float S = 0.0f;
    for (int w = 0; w < 32; ++w) S = __fadd_rn(S, red[w]);
    const int id = a.ids[b];
    float lp;
    if (id < 0 || id >= a.V) lp = __int_as_float(0x7fc00000);
    else if (M == -INFINITY) lp = -INFINITY;
    else lp = __fsub_rn(Y(id), __fadd_rn(M, rlog(S)));
    a.out[b] = lp;
  }
}

}  // namespace

REC_API int rec_token_logprob(const void* logits_dev, int32_t batch, int32_t vocab, int64_t stride,
                              const int32_t* history_dev, int32_t history_len, const RecSampling* params,
                              const uint32_t* allow_dev, int64_t allow_stride, const int32_t* ids_dev,
                              float* logprob_dev, void* stream) {
  REC_CHECK_ARG(logits_dev && params && ids_dev && logprob_dev, "rec_token_logprob: null pointer");
  REC_CHECK_ARG(batch >= 1 && batch <= 64, "rec_token_logprob: batch %d outside 1..64", batch);
  REC_CHECK_ARG(vocab >= 1 && vocab <= kLpMaxVocab, "rec_token_logprob: vocab %d outside 1..%d", vocab,
                kLpMaxVocab);
  REC_CHECK_ARG(stride >= vocab, "rec_token_logprob: row stride %lld < vocab", (long long)stride);
  REC_CHECK_ARG(history_len >= 0 && (history_len == 0 || history_dev), "rec_token_logprob: bad history");
  REC_CHECK_ARG(!allow_dev || allow_stride >= (vocab + 31) / 32, "rec_token_logprob: allow rows too short");
  const RecSampling& p = *params;
  REC_CHECK_ARG(p.temperature >= 0.0f && p.temperature < 1e30f, "rec_token_logprob: bad temperature");
  REC_CHECK_ARG(p.repetition_penalty > 0.0f, "rec_token_logprob: repetition penalty must be positive");
  LogprobArgs a = {};
  a.logits = static_cast<const uint16_t*>(logits_dev);
  a.stride = stride;
  a.V = vocab;
  a.history = history_dev;
  a.n_hist = history_len;
  a.temperature = p.temperature;
  a.rep = p.repetition_penalty;
  a.presence = p.presence_penalty;
  a.allow = allow_dev;
  a.allow_stride = allow_stride;
  a.ids = ids_dev;
  a.out = logprob_dev;
  k_token_logprob<<<batch, kLpThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
  REC_CHECK_CUDA(cudaGetLastError());
  return REC_OK;
}
