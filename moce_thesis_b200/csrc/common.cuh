// Shared helpers for the MoCE sm_100a kernels: dtype conversion, warp
// reductions, status reporting and launch bookkeeping.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "../../include/moce_b200.h"

namespace moce {

constexpr unsigned kFull = 0xffffffffu;

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

// Max that propagates NaN the way torch's softmax does (NaN wins).
__device__ __forceinline__ float nan_max(float a, float b) {
  return (a != a || a > b) ? a : b;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = nan_max(v, __shfl_xor_sync(kFull, v, o));
  return v;
}

__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

// Effective temperature, MoCE.py:218 (eval form): clamp(min + range*sigmoid(g), 1e-3).
// A NaN gate logit stays NaN (torch.clamp keeps NaN).
__device__ __forceinline__ float temperature(float g, float tmin_tau, float trange_tau, float* sig_out) {
  const float sig = 1.0f / (1.0f + expf(-g));
  if (sig_out) *sig_out = sig;
  const float t = tmin_tau + trange_tau * sig;
  return (t < 1e-3f) ? 1e-3f : t;
}

// Output epilogue: the caller's eval-mode BatchNorm folded to a per-channel
// affine (scale, shift) and an optional ReLU, applied to a finished output
// value before it is rounded and stored (models_unified.py:158-165 runs
// MoCE -> bn1 -> relu1).  A NaN stays NaN through the ReLU, as in torch.
struct OutEpilogue {
  const float* scale;   // [E] or null (no epilogue)
  const float* shift;   // [E]
  int relu;
};

__device__ __forceinline__ float apply_epilogue(float v, float sc, float sh, int relu) {
  const float r = fmaf(v, sc, sh);
  return (relu && r < 0.0f) ? 0.0f : r;
}

// ---------------------------------------------------------------- host side

// Records the message for moce_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);
int num_sms();  // SM count of the current device (cached per device)

template <typename T> struct DTypeOf;
template <> struct DTypeOf<float> { static constexpr int value = MOCE_F32; };
template <> struct DTypeOf<__nv_bfloat16> { static constexpr int value = MOCE_BF16; };
template <> struct DTypeOf<__half> { static constexpr int value = MOCE_F16; };

inline size_t dtype_size(int dtype) { return dtype == MOCE_F32 ? 4 : 2; }
inline bool dtype_ok(int dtype) { return dtype == MOCE_F32 || dtype == MOCE_BF16 || dtype == MOCE_F16; }

inline size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

// Dispatch a functor templated on the element type.
template <typename F>
int dispatch_dtype(int dtype, F&& f) {
  switch (dtype) {
    case MOCE_F32: return f(float{});
    case MOCE_BF16: return f(__nv_bfloat16{});
    case MOCE_F16: return f(__half{});
    default: return set_error(MOCE_ERR_INVALID, "unknown dtype %d", dtype);
  }
}

}  // namespace moce

#define MOCE_REQUIRE(cond, code, ...)                      \
  do {                                                     \
    if (!(cond)) return ::moce::set_error((code), __VA_ARGS__); \
  } while (0)
