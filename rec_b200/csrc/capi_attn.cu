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

// Quantize-on-append: one warp per (kv head, K or V, group of 64 dims) of
// the new token's rows, stored at row *position of each head.
__global__ void k_kv_append(const uint16_t* __restrict__ k, const uint16_t* __restrict__ v, RecKVLayer kv, int hkv,
                            int capacity, int bits, const int* __restrict__ position, int* status) {
  const int lane = threadIdx.x & 31;
  const int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (task >= hkv * 4) return;
  const int p = *position;
  if (p < 0 || p >= capacity) {
    if (task == 0 && lane == 0) report(status, kStatusBadPosition);
    return;
  }
  const int g = task >> 2, is_v = (task >> 1) & 1, grp = task & 1;
  const uint32_t pair = reinterpret_cast<const uint32_t*>((is_v ? v : k) + g * 128 + 64 * grp)[lane];
  const float v0 = bf(uint16_t(pair & 0xFFFFu)), v1 = bf(uint16_t(pair >> 16));
  const QGroupParams qp = warp_group_params(v0, v1, bits);
  const uint32_t word = warp_pack(quant_code(v0, qp, bits), quant_code(v1, qp, bits), bits);
  const int gw = 64 * bits / 32, rw = 2 * gw;
  const size_t slot = size_t(g) * capacity + size_t(p);
  uint32_t* codes = static_cast<uint32_t*>(is_v ? kv.v_codes : kv.k_codes);
  uint16_t* sc = static_cast<uint16_t*>(is_v ? kv.v_scales : kv.k_scales);
  uint16_t* bi = static_cast<uint16_t*>(is_v ? kv.v_biases : kv.k_biases);
  if (lane < gw) codes[slot * rw + grp * gw + lane] = word;
  if (lane == 0) {
    sc[slot * 2 + grp] = to_bf(qp.scale);
    bi[slot * 2 + grp] = to_bf(qp.bias);
  }
}

// Bulk form for a prefill chunk: token j of k, v (bf16 [t, hkv * 128]) goes
// to row p0 + j; one warp per (token, head, K or V, group), the same
// arithmetic as k_kv_append.
__global__ void k_kv_append_bulk(const uint16_t* __restrict__ k, const uint16_t* __restrict__ v, RecKVLayer kv,
                                 int hkv, int capacity, int bits, int p0, int t) {
  const int lane = threadIdx.x & 31;
  const long long task = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (task >= (long long)t * hkv * 4) return;
  const int j = int(task / (hkv * 4)), r = int(task % (hkv * 4));
  const int g = r >> 2, is_v = (r >> 1) & 1, grp = r & 1;
  const uint32_t pair =
      reinterpret_cast<const uint32_t*>((is_v ? v : k) + (size_t(j) * hkv + g) * 128 + 64 * grp)[lane];
  const float v0 = bf(uint16_t(pair & 0xFFFFu)), v1 = bf(uint16_t(pair >> 16));
  const QGroupParams qp = warp_group_params(v0, v1, bits);
  const uint32_t word = warp_pack(quant_code(v0, qp, bits), quant_code(v1, qp, bits), bits);
  const int gw = 64 * bits / 32, rw = 2 * gw;
  const size_t slot = size_t(g) * capacity + size_t(p0 + j);
  uint32_t* codes = static_cast<uint32_t*>(is_v ? kv.v_codes : kv.k_codes);
  uint16_t* sc = static_cast<uint16_t*>(is_v ? kv.v_scales : kv.k_scales);
  uint16_t* bi = static_cast<uint16_t*>(is_v ? kv.v_biases : kv.k_biases);
  if (lane < gw) codes[slot * rw + grp * gw + lane] = word;
  if (lane == 0) {
    sc[slot * 2 + grp] = to_bf(qp.scale);
    bi[slot * 2 + grp] = to_bf(qp.bias);
  }
}

}  // namespace

REC_API int rec_kv_append_bulk(const RecKVLayer* kv, int32_t n_kv_heads, int32_t capacity, int32_t kv_bits,
                               const void* k_dev, const void* v_dev, int32_t position, int32_t t, void* stream) {
  REC_CHECK_ARG(kv && k_dev && v_dev, "rec_kv_append_bulk: null pointer");
  REC_CHECK_ARG(n_kv_heads > 0 && capacity > 0, "rec_kv_append_bulk: n_kv_heads and capacity must be positive");
  REC_CHECK_ARG(kv_bits == 4 || kv_bits == 8, "kv_bits must be 4 or 8");
  REC_CHECK_ARG(t >= 1 && position >= 0 && int64_t(position) + t <= capacity,
                "rec_kv_append_bulk: rows [%d, %lld) outside the capacity %d", position,
                (long long)position + t, capacity);
  REC_CHECK_ARG(kv->k_codes && kv->k_scales && kv->k_biases && kv->v_codes && kv->v_scales && kv->v_biases &&
                    aligned16(kv->k_codes) && aligned16(kv->v_codes) && aligned16(k_dev) && aligned16(v_dev),
                "rec_kv_append_bulk: KV buffers and k/v rows must be non-null and 16-byte aligned");
  const long long warps = (long long)t * n_kv_heads * 4;
  k_kv_append_bulk<<<unsigned((warps + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(k_dev), static_cast<const uint16_t*>(v_dev), *kv, n_kv_heads, capacity, kv_bits,
      position, t);
  REC_CHECK_CUDA(cudaGetLastError());
  return REC_OK;
}

REC_API int rec_kv_append(const RecKVLayer* kv, int32_t n_kv_heads, int32_t capacity, int32_t kv_bits,
                          const void* k_dev, const void* v_dev, const int32_t* position_dev, int32_t* status_dev,
                          void* stream) {
  REC_CHECK_ARG(kv && k_dev && v_dev && position_dev && status_dev, "rec_kv_append: null pointer");
  REC_CHECK_ARG(n_kv_heads > 0 && capacity > 0, "rec_kv_append: n_kv_heads and capacity must be positive");
  REC_CHECK_ARG(kv_bits == 4 || kv_bits == 8, "kv_bits must be 4 or 8");
  REC_CHECK_ARG(kv->k_codes && kv->k_scales && kv->k_biases && kv->v_codes && kv->v_scales && kv->v_biases &&
                    aligned16(kv->k_codes) && aligned16(kv->v_codes) && aligned16(k_dev) && aligned16(v_dev),
                "rec_kv_append: KV buffers and k/v rows must be non-null and 16-byte aligned");
  const int warps = n_kv_heads * 4;
  k_kv_append<<<(warps + 7) / 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(k_dev), static_cast<const uint16_t*>(v_dev), *kv, n_kv_heads, capacity, kv_bits,
      position_dev, status_dev);
  REC_CHECK_CUDA(cudaGetLastError());
  return REC_OK;
}

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
  a.super_hi = kAttAllSupers;
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
