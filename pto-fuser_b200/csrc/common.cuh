// Shared host/device definitions for the GDN chunk-forward kernels.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/pto_fuser_gdn.h"

namespace ptof {

constexpr int kChunk = 64;  // chunk length C of every kernel in this library

// Strides (in elements) of a [B,H,T,D]-shaped logical tensor, whatever its
// physical layout: heads-outer [B,H,T,D] or token-major [B,T,H,D].
struct Strides4 {
  int64_t b, h, t;  // innermost (d) stride is 1
};
// Strides of a per-token scalar [B,H,T] (heads-outer) or [B,T,H] (token-major).
struct Strides3 {
  int64_t b, h, t;
};

__host__ __device__ inline Strides4 make_strides4(int layout, int H, int T, int D) {
  Strides4 s;
  if (layout == PTOF_LAYOUT_BHTD) {
    s.t = D;
    s.h = static_cast<int64_t>(T) * D;
    s.b = static_cast<int64_t>(H) * T * D;
  } else {
    s.h = D;
    s.t = static_cast<int64_t>(H) * D;
    s.b = static_cast<int64_t>(T) * H * D;
  }
  return s;
}
__host__ __device__ inline Strides3 make_strides3(int layout, int H, int T) {
  Strides3 s;
  if (layout == PTOF_LAYOUT_BHTD) {
    s.t = 1;
    s.h = T;
    s.b = static_cast<int64_t>(H) * T;
  } else {
    s.h = 1;
    s.t = H;
    s.b = static_cast<int64_t>(T) * H;
  }
  return s;
}

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Element i of a beta array of element type dt (PTOF_F32 / F16 / BF16) as fp32.
__device__ __forceinline__ float ld_beta_any(const void* p, int dt, int64_t i) {
  if (dt == PTOF_F32) return static_cast<const float*>(p)[i];
  if (dt == PTOF_F16) return __half2float(static_cast<const __half*>(p)[i]);
  return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

// Decay coefficients, written exactly as the reference forward writes them
// (examples/attention/_gdn_full.py:53-54 `_safe_exp`, :90-91 `exp(min(.,0))`).
__device__ __forceinline__ float kkt_coef(float gi, float gj) {  // where(x<=0, exp(x), 0)
  const float x = gi - gj;
  return x <= 0.f ? __expf(x) : 0.f;
}
__device__ __forceinline__ float qk_coef(float gi, float gj) {  // exp(min(x, 0))
  return __expf(fminf(gi - gj, 0.f));
}

}  // namespace ptof
