// C-ABI entry point of the sampling head over bf16 logits.
#include "capi_common.h"
#include "sample.cuh"

using namespace rec;

namespace rec {
int lmhead_batch(const RecQMat* w, int sd, int V, const void* h, int B, const void* norm, float eps, void* out,
                 int* status, cudaStream_t st);  // lmhead_batch.cu
}

REC_API int rec_sample_logits_masked(const void* logits_dev, int32_t batch, int32_t vocab, int64_t stride,
                                     const int32_t* history_dev, int32_t history_len, const RecSampling* params,
                                     const float* uniforms_dev, const uint32_t* allow_dev, int64_t allow_stride,
                                     int32_t* ids_dev, void* stream) {
  REC_CHECK_ARG(!allow_dev || allow_stride >= (vocab + 31) / 32, "rec_sample_logits_masked: allow rows too short");
  REC_CHECK_ARG(logits_dev && ids_dev && params, "rec_sample_logits: null pointer");
  REC_CHECK_ARG(batch >= 1 && batch <= 64, "rec_sample_logits: batch %d outside 1..64", batch);
  REC_CHECK_ARG(vocab >= 2 && vocab <= kSampleMaxVocab, "rec_sample_logits: vocab %d outside 2..%d", vocab,
                kSampleMaxVocab);
  REC_CHECK_ARG(stride >= vocab, "rec_sample_logits: row stride %lld < vocab", (long long)stride);
  REC_CHECK_ARG(history_len >= 0 && (history_len == 0 || history_dev), "rec_sample_logits: bad history");
  const RecSampling& p = *params;
  REC_CHECK_ARG(p.temperature >= 0.0f && p.temperature < 1e30f, "rec_sample_logits: bad temperature");
  REC_CHECK_ARG(p.repetition_penalty > 0.0f, "rec_sample_logits: repetition penalty must be positive");
  if (p.temperature > 0.0f) {
    REC_CHECK_ARG(uniforms_dev, "rec_sample_logits: temperature > 0 needs uniforms");
    REC_CHECK_ARG(p.top_k >= 0 && p.top_k < vocab && p.top_k <= kSampleMaxTopK,
                  "top_k must be between 0 and %d", vocab - 1 < kSampleMaxTopK ? vocab - 1 : kSampleMaxTopK);
    REC_CHECK_ARG(p.top_p > 0.0f, "top_p must be positive");
    REC_CHECK_ARG(p.top_k > 0 || p.top_p >= 1.0f, "top_p < 1 needs top_k > 0");
  }
  SampleArgs a = {};
  a.logits = static_cast<const uint16_t*>(logits_dev);
  a.stride = stride;
  a.V = vocab;
  a.history = history_dev;
  a.n_hist = history_len;
  a.temperature = p.temperature;
  a.top_k = p.top_k;
  a.top_p = p.top_p;
  a.rep = p.repetition_penalty;
  a.presence = p.presence_penalty;
  a.uniforms = uniforms_dev;
  a.allow = allow_dev;
  a.allow_stride = allow_stride;
  a.ids = ids_dev;
  REC_CHECK_CUDA(launch_sample(a, batch, static_cast<cudaStream_t>(stream)));
  return REC_OK;
}

REC_API int rec_sample_logits(const void* logits_dev, int32_t batch, int32_t vocab, int64_t stride,
                              const int32_t* history_dev, int32_t history_len, const RecSampling* params,
                              const float* uniforms_dev, int32_t* ids_dev, void* stream) {
  return rec_sample_logits_masked(logits_dev, batch, vocab, stride, history_dev, history_len, params, uniforms_dev,
                                  nullptr, 0, ids_dev, stream);
}

REC_API int rec_lmhead_sample(const RecQMat* lm_head, int32_t scale_dtype, int32_t vocab, int32_t hidden,
                              const void* h_dev, int32_t batch, const void* final_norm_dev, float eps,
                              const int32_t* history_dev, int32_t history_len, const RecSampling* params,
                              const float* uniforms_dev, void* logits_dev, int32_t* ids_dev, void* stream) {
  REC_CHECK_ARG(lm_head && h_dev && final_norm_dev && params && logits_dev && ids_dev,
                "rec_lmhead_sample: null pointer");
  REC_CHECK_ARG(batch >= 1 && batch <= 64, "rec_lmhead_sample: batch %d outside 1..64", batch);
  REC_CHECK_ARG(hidden > 0 && vocab > 0, "rec_lmhead_sample: bad shape");
  const uint16_t* h = static_cast<const uint16_t*>(h_dev);
  uint16_t* lg = static_cast<uint16_t*>(logits_dev);
  const bool batched = batch > 1 && hidden == 2048 && vocab % 8 == 0 && lm_head->w && lm_head->scales &&
                       lm_head->biases && aligned16(lm_head->w) && aligned16(lm_head->scales) &&
                       aligned16(lm_head->biases) && aligned16(h_dev) && (reinterpret_cast<uintptr_t>(lg) & 3u) == 0;
  if (batched) {
    // up to 8 rows per pass over the weights, on the tensor cores
    // (bit-identical to the per-row GEMV)
    REC_CHECK_ARG(scale_dtype == REC_SCALE_FP16 || scale_dtype == REC_SCALE_BF16, "bad scale dtype");
    for (int b0 = 0; b0 < batch; b0 += 8) {
      const int rc = lmhead_batch(lm_head, scale_dtype, vocab, h + size_t(b0) * hidden,
                                  batch - b0 < 8 ? batch - b0 : 8, final_norm_dev, eps, lg + size_t(b0) * vocab,
                                  nullptr, static_cast<cudaStream_t>(stream));
      if (rc) return rc;
    }
  } else {
    for (int b = 0; b < batch; ++b) {
      const int rc = rec_gemv_int4(lm_head, scale_dtype, vocab, hidden, h + size_t(b) * hidden, final_norm_dev, eps,
                                   lg + size_t(b) * vocab, stream);
      if (rc) return rc;
    }
  }
  return rec_sample_logits(logits_dev, batch, vocab, vocab, history_dev, history_len, params, uniforms_dev, ids_dev,
                           stream);
}

