// C-ABI entry point of the decode attention kernels alone (unit tests and
// the attention sweep): quantize-on-append of the new K/V at `position`, item
// partials over [0, position], combine into bf16 [Hq, 128].
#include "attn.cuh"
#include "capi_common.h"

using namespace rec;

namespace {

struct AttnScratchLayout {
  size_t partials, supers, counters, total;
  int icap, n_super;
};
AttnScratchLayout attn_scratch_layout(int hq, int capacity) {
  AttnScratchLayout L;
  L.icap = items_cap(capacity);
  L.n_super = (capacity / kAttBlock + kAttSuper - 1) / kAttSuper;
  L.partials = 0;
  L.supers = (size_t(hq) * L.icap * kPartialFloats * 4 + 255) / 256 * 256;
  L.counters = L.supers + (size_t(hq) * L.n_super * kPartialFloats * 4 + 255) / 256 * 256;
  L.total = L.counters + (size_t(hq) * 4 + 255) / 256 * 256;
  return L;
}

// Persistent grid: as many CTAs as fit on every SM.
template <class K>
cudaError_t launch_smem(K kern, int threads, size_t smem, cudaStream_t st, const AttnArgs& a) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return e;
  int per_sm = 1;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
  if (e != cudaSuccess) return e;
  kern<<<sm_count() * (per_sm > 0 ? per_sm : 1), threads, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace

REC_API size_t rec_attn_scratch_bytes(int32_t n_q_heads, int32_t capacity) {
  if (n_q_heads <= 0 || capacity <= 0) return 0;
  return attn_scratch_layout(n_q_heads, capacity).total;
}

REC_API int rec_attn_decode(const void* qkv_dev, int32_t n_q_heads, int32_t n_kv_heads, const RecKVLayer* kv,
                            int32_t capacity, int32_t kv_bits, const float* rope_dev, const void* sinks_dev,
                            const int32_t* position_dev, void* scratch_dev, size_t scratch_bytes, void* out_dev,
                            int32_t* status_dev, void* stream) {
  REC_CHECK_ARG(qkv_dev && kv && rope_dev && position_dev && scratch_dev && out_dev && status_dev,
                "rec_attn_decode: null pointer");
  REC_CHECK_ARG(n_kv_heads > 0 && n_q_heads == kHeadsPerKv * n_kv_heads, "need 8 query heads per KV head");
  REC_CHECK_ARG(capacity > 0 && capacity % kAttBlock == 0, "capacity must be a positive multiple of %d", kAttBlock);
  REC_CHECK_ARG(kv_bits == 4 || kv_bits == 8, "kv_bits must be 4 or 8");
  REC_CHECK_ARG(kv->k_codes && kv->k_scales && kv->k_biases && kv->v_codes && kv->v_scales && kv->v_biases &&
                    aligned16(kv->k_codes) && aligned16(kv->v_codes) && aligned16(kv->k_scales) &&
                    aligned16(kv->k_biases) && aligned16(kv->v_scales) && aligned16(kv->v_biases),
                "rec_attn_decode: KV buffers must be non-null and 16-byte aligned");
  const AttnScratchLayout L = attn_scratch_layout(n_q_heads, capacity);
  REC_CHECK_ARG(scratch_bytes >= L.total && (reinterpret_cast<uintptr_t>(scratch_dev) & 255u) == 0,
                "rec_attn_decode: scratch must be 256-byte aligned and hold %zu bytes", L.total);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* s = static_cast<uint8_t*>(scratch_dev);
  REC_CHECK_CUDA(cudaMemsetAsync(s + L.counters, 0, size_t(n_q_heads) * 4, st));
  AttnArgs a = {};
  a.qkv = static_cast<const uint16_t*>(qkv_dev);
  a.k_codes = static_cast<uint32_t*>(kv->k_codes);
  a.k_scales = static_cast<uint16_t*>(kv->k_scales);
  a.k_biases = static_cast<uint16_t*>(kv->k_biases);
  a.v_codes = static_cast<uint32_t*>(kv->v_codes);
  a.v_scales = static_cast<uint16_t*>(kv->v_scales);
  a.v_biases = static_cast<uint16_t*>(kv->v_biases);
  a.capacity = capacity;
  a.hq = n_q_heads;
  a.hkv = n_kv_heads;
  a.rope = rope_dev;
  a.eps = 1e-6f;
  a.position = position_dev;
  a.partials = reinterpret_cast<float*>(s + L.partials);
  a.supers = reinterpret_cast<float*>(s + L.supers);
  a.head_counters = reinterpret_cast<unsigned*>(s + L.counters);
  a.out = static_cast<uint16_t*>(out_dev);
  a.sinks = static_cast<const uint16_t*>(sinks_dev);
  a.n_super_max = L.n_super;
  a.status = status_dev;
  a.pdl = 0;
  cudaError_t e = kv_bits == 4 ? launch_smem(k_attn_partial<4>, kAttWarps * 32, sizeof(AttnSmem<4>), st, a)
                               : launch_smem(k_attn_partial<8>, kAttWarps * 32, sizeof(AttnSmem<8>), st, a);
  REC_CHECK_CUDA(e);
  k_attn_combine<<<dim3(n_q_heads, L.n_super), 32, 0, st>>>(a);
  REC_CHECK_CUDA(cudaGetLastError());
  return REC_OK;
}
