// C-ABI entry points for single kernels (used by the unit tests and by the
// weight generator): int4 GEMV and MLX affine quantization.
#include "capi_common.h"
#include "gemv.cuh"
#include "quant.cuh"

namespace rec {

static thread_local std::string g_error;

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_error = buf;
}

int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// --- quantization ----------------------------------------------------------
// One warp per group of 64 values.
__global__ void k_quantize(const float* __restrict__ w, int64_t n_groups, int bits, int sd,
                           uint32_t* __restrict__ codes, uint16_t* __restrict__ scales,
                           uint16_t* __restrict__ biases) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t g = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); g < n_groups; g += warps) {
    const float2 v = reinterpret_cast<const float2*>(w + g * 64)[lane];
    QGroupParams p = warp_group_params(v.x, v.y, bits);
    uint32_t word = warp_pack(quant_code(v.x, p, bits), quant_code(v.y, p, bits), bits);
    const int words = 64 * bits / 32;
    if (lane < words) codes[g * words + lane] = word;
    if (lane == 0) {
      if (sd == REC_SCALE_FP16) {
        scales[g] = __half_as_ushort(__float2half_rn(p.scale));
        biases[g] = __half_as_ushort(__float2half_rn(p.bias));
      } else {
        scales[g] = to_bf(p.scale);
        biases[g] = to_bf(p.bias);
      }
    }
  }
}

template <int K, int SD>
static cudaError_t gemv_store(const GemvArgs& a, cudaStream_t st) {
  return launch_gemv<K, SD, gemv_rs<K>(), 3, kEpiStore>(a, sm_count(), st, false);
}

template <int SD>
static cudaError_t gemv_dispatch(int k, const GemvArgs& a, cudaStream_t st) {
  switch (k) {
    case 256: return gemv_store<256, SD>(a, st);
    case 512: return gemv_store<512, SD>(a, st);
    case 768: return gemv_store<768, SD>(a, st);
    case 1024: return gemv_store<1024, SD>(a, st);
    case 2048: return gemv_store<2048, SD>(a, st);
    case 4096: return gemv_store<4096, SD>(a, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace rec

using namespace rec;

REC_API int rec_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return REC_EINVAL;
  snprintf(buf, len, "%s", g_error.c_str());
  return REC_OK;
}

REC_API int rec_gemv_int4(const RecQMat* w, int32_t scale_dtype, int64_t n, int32_t k, const void* x_dev,
                          const void* norm_weight_dev, float eps, void* y_dev, void* stream) {
  REC_CHECK_ARG(w && w->w && w->scales && w->biases && x_dev && y_dev, "rec_gemv_int4: null pointer");
  REC_CHECK_ARG(k == 256 || k == 512 || k == 768 || k == 1024 || k == 2048 || k == 4096,
                "rec_gemv_int4: unsupported K=%d", k);
  REC_CHECK_ARG(n > 0 && n % 2 == 0 && n < (1ll << 30), "rec_gemv_int4: N=%lld must be even", (long long)n);
  REC_CHECK_ARG(scale_dtype == REC_SCALE_FP16 || scale_dtype == REC_SCALE_BF16, "bad scale dtype");
  REC_CHECK_ARG(!norm_weight_dev || k % 256 == 0, "norm needs K % 256 == 0");
  REC_CHECK_ARG(aligned16(w->w) && aligned16(w->scales) && aligned16(w->biases) && aligned16(x_dev),
                "rec_gemv_int4: operands must be 16-byte aligned");
  GemvArgs a = {};
  a.mat[0] = {static_cast<const uint32_t*>(w->w), static_cast<const uint16_t*>(w->scales),
              static_cast<const uint16_t*>(w->biases)};
  a.rows[0] = int(n);
  a.total_rows = int(n);
  a.x = static_cast<const uint16_t*>(x_dev);
  a.norm_w = static_cast<const uint16_t*>(norm_weight_dev);
  a.eps = eps;
  a.out = static_cast<uint16_t*>(y_dev);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = scale_dtype == REC_SCALE_FP16 ? gemv_dispatch<0>(k, a, st) : gemv_dispatch<1>(k, a, st);
  REC_CHECK_CUDA(e);
  return REC_OK;
}

REC_API int rec_quantize_affine(const float* w_dev, int64_t n_groups, int32_t bits, int32_t scale_dtype,
                                void* codes_dev, void* scales_dev, void* biases_dev, void* stream) {
  REC_CHECK_ARG(w_dev && codes_dev && scales_dev && biases_dev, "rec_quantize_affine: null pointer");
  REC_CHECK_ARG(bits == 4 || bits == 8, "rec_quantize_affine: bits must be 4 or 8");
  REC_CHECK_ARG(n_groups > 0, "rec_quantize_affine: no groups");
  REC_CHECK_ARG(scale_dtype == REC_SCALE_FP16 || scale_dtype == REC_SCALE_BF16, "bad scale dtype");
  REC_CHECK_ARG((reinterpret_cast<uintptr_t>(w_dev) & 7u) == 0, "rec_quantize_affine: input must be 8-byte aligned");
  const int threads = 256;
  int64_t blocks = (n_groups + 7) / 8;
  if (blocks > int64_t(sm_count()) * 16) blocks = int64_t(sm_count()) * 16;
  k_quantize<<<int(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      w_dev, n_groups, bits, scale_dtype, static_cast<uint32_t*>(codes_dev), static_cast<uint16_t*>(scales_dev),
      static_cast<uint16_t*>(biases_dev));
  REC_CHECK_CUDA(cudaGetLastError());
  return REC_OK;
}

// The SiLU table: entry i = bf16(bf16(g * bf16(sigmoid(g))) * 1) for the gate
// g whose bf16 bits are i, the decode path's gate/up epilogue with u = 1.
__global__ void k_silu_table(uint16_t* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;  // grid covers exactly 65,536
  const float gg = bf(uint16_t(i));
  out[i] = to_bf(__fmul_rn(rbf(__fmul_rn(gg, rbf(rsigmoid(gg)))), 1.0f));
}

REC_API int rec_silu_table(void* out_dev, void* stream) {
  REC_CHECK_ARG(out_dev, "rec_silu_table: null pointer");
  REC_CHECK_ARG((reinterpret_cast<uintptr_t>(out_dev) & 1u) == 0, "rec_silu_table: output must be 2-byte aligned");
  k_silu_table<<<65536 / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint16_t*>(out_dev));
  REC_CHECK_CUDA(cudaGetLastError());
  return REC_OK;
}
