// int4 GEMV + greedy argmax for callers that cannot allocate device memory.
//
// The same kernel as the lm_head step (k_gemv with the argmax epilogue); its
// cross-CTA scratch (arrival counter, status word, per-CTA candidates and,
// when the caller passes no logits buffer, the logits themselves) lives in
// one file-scope device array instead of a caller workspace.
//
// Scratch layout (kNaScratchBytes = 532,736 bytes):
//   [0, 256)           unsigned counter, int status      (zeroed by every call)
//   [256, 4352)        float cand_val[kNaMaxCtas]        (written before read)
//   [4352, 8448)       int   cand_idx[kNaMaxCtas]        (written before read)
//   [8448, 532736)     bf16  logits[kNaMaxRows]          (only when y_dev is NULL)
//
// Every call shares the array and it keeps the previous call's contents, so
// calls whose kernels overlap on the GPU (other streams, other threads) race
// on it; calls on one stream are ordered.
#include <mutex>

#include "capi_common.h"
#include "gemv.cuh"

namespace rec {
namespace {

constexpr int kNaMaxCtas = 1024;
constexpr int64_t kNaMaxRows = 262144;
constexpr size_t kNaHeader = 256;
constexpr size_t kNaCandVal = kNaHeader;
constexpr size_t kNaCandIdx = kNaCandVal + sizeof(float) * kNaMaxCtas;
constexpr size_t kNaLogits = kNaCandIdx + sizeof(int) * kNaMaxCtas;
constexpr size_t kNaScratchBytes = kNaLogits + sizeof(uint16_t) * kNaMaxRows;
constexpr int kNaMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNaScratchBytes];

struct DeviceSetup {
  uint8_t* scratch = nullptr;  // device address of g_noalloc_scratch
};
std::mutex g_setup_mu;
DeviceSetup g_setup[kNaMaxDevices];

template <int K, int SD>
cudaError_t configure_one() {
  using S = GemvSmem<K, gemv_rs<K>(), 3>;
  return cudaFuncSetAttribute(k_gemv<K, SD, gemv_rs<K>(), 3, kEpiArgmax>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, int(sizeof(S)));
}

template <int SD>
cudaError_t configure_sd() {
  cudaError_t e;
  if ((e = configure_one<256, SD>()) != cudaSuccess) return e;
  if ((e = configure_one<512, SD>()) != cudaSuccess) return e;
  if ((e = configure_one<768, SD>()) != cudaSuccess) return e;
  if ((e = configure_one<1024, SD>()) != cudaSuccess) return e;
  if ((e = configure_one<2048, SD>()) != cudaSuccess) return e;
  return configure_one<4096, SD>();
}

// Once per device, with that device current: the scratch's device address
// and the kernels' shared-memory limit.
int setup_current_device(uint8_t** scratch) {
  int dev = 0;
  REC_CHECK_CUDA(cudaGetDevice(&dev));
  REC_CHECK_ARG(dev >= 0 && dev < kNaMaxDevices, "rec_gemv_int4_argmax_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_setup_mu);
  DeviceSetup& s = g_setup[dev];
  if (!s.scratch) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      set_error("rec_gemv_int4_argmax_noalloc: cudaGetSymbolAddress of the scratch failed on device %d: %s", dev,
                cudaGetErrorString(e));
      return REC_ECUDA;
    }
    REC_CHECK_CUDA(configure_sd<0>());
    REC_CHECK_CUDA(configure_sd<1>());
    s.scratch = static_cast<uint8_t*>(p);
  }
  *scratch = s.scratch;
  return REC_OK;
}

template <int K, int SD>
cudaError_t launch_one(const GemvArgs& a, int grid, cudaStream_t st) {
  using S = GemvSmem<K, gemv_rs<K>(), 3>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = sizeof(S);
  cfg.stream = st;
  return cudaLaunchKernelEx(&cfg, k_gemv<K, SD, gemv_rs<K>(), 3, kEpiArgmax>, a);
}

template <int SD>
cudaError_t launch_sd(int k, const GemvArgs& a, int grid, cudaStream_t st) {
  switch (k) {
    case 256: return launch_one<256, SD>(a, grid, st);
    case 512: return launch_one<512, SD>(a, grid, st);
    case 768: return launch_one<768, SD>(a, grid, st);
    case 1024: return launch_one<1024, SD>(a, grid, st);
    case 2048: return launch_one<2048, SD>(a, grid, st);
    case 4096: return launch_one<4096, SD>(a, grid, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace
}  // namespace rec

using namespace rec;

REC_API int rec_gemv_int4_argmax_noalloc(const RecQMat* w, int32_t scale_dtype, int64_t n, int32_t k,
                                         const void* x_dev, const void* norm_weight_dev, float eps, void* y_dev,
                                         int32_t* token_dev, void* stream) {
  REC_CHECK_ARG(w && w->w && w->scales && w->biases && x_dev && token_dev,
                "rec_gemv_int4_argmax_noalloc: null pointer");
  REC_CHECK_ARG(k == 256 || k == 512 || k == 768 || k == 1024 || k == 2048 || k == 4096,
                "rec_gemv_int4_argmax_noalloc: unsupported K=%d", k);
  REC_CHECK_ARG(n > 0 && n % 2 == 0 && n < (1ll << 30), "rec_gemv_int4_argmax_noalloc: N=%lld must be even",
                (long long)n);
  REC_CHECK_ARG(y_dev || n <= kNaMaxRows,
                "rec_gemv_int4_argmax_noalloc: N=%lld rows exceed the %lld-row logits scratch; pass y_dev",
                (long long)n, (long long)kNaMaxRows);
  REC_CHECK_ARG(scale_dtype == REC_SCALE_FP16 || scale_dtype == REC_SCALE_BF16, "bad scale dtype");
  REC_CHECK_ARG(!norm_weight_dev || k % 256 == 0, "norm needs K % 256 == 0");
  REC_CHECK_ARG(aligned16(w->w) && aligned16(w->scales) && aligned16(w->biases) && aligned16(x_dev),
                "rec_gemv_int4_argmax_noalloc: operands must be 16-byte aligned");
  const int grid = sm_count() < kNaMaxCtas ? sm_count() : kNaMaxCtas;
  REC_CHECK_ARG(grid > 0 && grid <= kNaMaxCtas, "rec_gemv_int4_argmax_noalloc: %d CTAs exceed the %d candidate slots",
                grid, kNaMaxCtas);
  uint8_t* scratch = nullptr;
  const int rc = setup_current_device(&scratch);
  if (rc != REC_OK) return rc;

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // counter and status must start at zero (a call whose wait ran out leaves
  // them set); the token reads -1 until the last CTA writes it
  REC_CHECK_CUDA(cudaMemsetAsync(scratch, 0, kNaHeader, st));
  REC_CHECK_CUDA(cudaMemsetAsync(token_dev, 0xFF, sizeof(int32_t), st));

  GemvArgs a = {};
  a.mat[0] = {static_cast<const uint32_t*>(w->w), static_cast<const uint16_t*>(w->scales),
              static_cast<const uint16_t*>(w->biases)};
  a.rows[0] = int(n);
  a.total_rows = int(n);
  a.x = static_cast<const uint16_t*>(x_dev);
  a.norm_w = static_cast<const uint16_t*>(norm_weight_dev);
  a.eps = eps;
  a.out = y_dev ? static_cast<uint16_t*>(y_dev) : reinterpret_cast<uint16_t*>(scratch + kNaLogits);
  a.cand_val = reinterpret_cast<float*>(scratch + kNaCandVal);
  a.cand_idx = reinterpret_cast<int*>(scratch + kNaCandIdx);
  a.counter = reinterpret_cast<unsigned*>(scratch);
  a.status = reinterpret_cast<int*>(scratch + sizeof(unsigned));
  a.token_out = token_dev;
  a.pdl = 0;
  const cudaError_t e = scale_dtype == REC_SCALE_FP16 ? launch_sd<0>(k, a, grid, st) : launch_sd<1>(k, a, grid, st);
  REC_CHECK_CUDA(e);
  return REC_OK;
}
