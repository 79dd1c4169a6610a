// Launchers of the per-token prefill kernels (prefill_layer.cu), used by the
// chunk driver rec_prefill_chunk (decode.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/rec_b200.h"
#include "gemv.cuh"

namespace rec {

cudaError_t pf_embed(const QMatDev& emb, int sd, const int* tokens, int T, int H, int V, uint16_t* h, int* status,
                     cudaStream_t st);
cudaError_t pf_rmsnorm(const uint16_t* x, const uint16_t* w, int T, float eps, uint16_t* out, cudaStream_t st);
cudaError_t pf_qk(uint16_t* q, int hq, uint16_t* k, int hkv, int T, int p0, const float* rope, const uint16_t* qn,
                  const uint16_t* kn, float eps, cudaStream_t st);
cudaError_t pf_add(uint16_t* h, const uint16_t* o, size_t n, cudaStream_t st);
cudaError_t pf_router(const uint16_t* xn, const uint16_t* router, const float* bias, int T, int E, int k, int mode,
                      int* ids, float* wts, cudaStream_t st);
cudaError_t pf_attention(const uint16_t* q, int hq, int hkv, const RecKVLayer& kv, int capacity, int bits, int p0,
                         int T, const uint16_t* sinks, uint16_t* out, cudaStream_t st);

}  // namespace rec
