// Host-side helpers shared by the C-ABI translation units.
#pragma once
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string>

#include "../../include/rec_b200.h"

namespace rec {

void set_error(const char* fmt, ...);

#define REC_CHECK_ARG(cond, ...)      \
  do {                                \
    if (!(cond)) {                    \
      ::rec::set_error(__VA_ARGS__);  \
      return REC_EINVAL;              \
    }                                 \
  } while (0)

#define REC_CHECK_CUDA(expr)                                                           \
  do {                                                                                 \
    cudaError_t e_ = (expr);                                                           \
    if (e_ != cudaSuccess) {                                                           \
      ::rec::set_error("%s failed: %s", #expr, cudaGetErrorString(e_));                \
      return REC_ECUDA;                                                                \
    }                                                                                  \
  } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int sm_count();

}  // namespace rec
