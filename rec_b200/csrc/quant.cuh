// MLX affine quantization of one group of 64 values, as used by nn.quantize
// for the weights and by the quantized KV cache on append
// (reference: engine/src/rec_mlx/quantized.py:26-36, model.py:45-82; the
// algorithm is mlx 0.32.0's affine_quantize):
//   scale = max((max - min) / (2^bits - 1), 1e-7), negated unless |min| > |max|
//   edge  = |min| > |max| ? min : max;  q0 = rint(edge / scale)
//   if q0 != 0: scale = edge / q0, bias = edge  else bias = 0
//   code  = clamp(rint((w - bias) / scale), 0, 2^bits - 1)
// Scale and bias are stored rounded to the storage type; the codes are formed
// with the unrounded fp32 values.
#pragma once
#include "common.cuh"

namespace rec {

struct QGroupParams {
  float scale, bias;
};

// All 32 lanes of a warp call this with the group's values v0 = w[2*lane],
// v1 = w[2*lane+1].  Every lane returns the same parameters.
__device__ __forceinline__ QGroupParams warp_group_params(float v0, float v1, int bits) {
  float mx = fmaxf(v0, v1), mn = fminf(v0, v1);
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
  }
  const float n_bins = float((1 << bits) - 1);
  float scale = __fdiv_rn(__fsub_rn(mx, mn), n_bins);
  scale = scale > 1e-7f ? scale : 1e-7f;
  const bool side = fabsf(mn) > fabsf(mx);
  scale = side ? scale : -scale;
  const float edge = side ? mn : mx;
  const float q0 = rintf(__fdiv_rn(edge, scale));
  float bias = 0.0f;
  if (q0 != 0.0f) {
    scale = __fdiv_rn(edge, q0);
    bias = edge;
  }
  return {scale, bias};
}

__device__ __forceinline__ uint32_t quant_code(float w, QGroupParams p, int bits) {
  const float n_bins = float((1 << bits) - 1);
  float q = rintf(__fdiv_rn(__fsub_rn(w, p.bias), p.scale));
  q = q < 0.0f ? 0.0f : (q > n_bins ? n_bins : q);
  return uint32_t(q);
}

// Pack the warp's 64 codes (two per lane) into words; lane w (< 64*bits/32)
// returns word w.
__device__ __forceinline__ uint32_t warp_pack(uint32_t c0, uint32_t c1, int bits) {
  const int lane = threadIdx.x & 31;
  uint32_t pair = c0 | (c1 << bits);  // elements 2l, 2l+1
  const int pairs_per_word = 16 / bits;  // 4 (4-bit) or 2 (8-bit)
  uint32_t word = 0;
  for (int t = 0; t < pairs_per_word; ++t) {
    uint32_t p = __shfl_sync(0xffffffffu, pair, (lane * pairs_per_word + t) & 31);
    word |= p << (2 * bits * t);
  }
  return word;
}

}  // namespace rec
