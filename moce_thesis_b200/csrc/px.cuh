// Helpers of the lanes-over-pixels CUDA-core kernels (simt.cu, backward.cu):
// four-element shared-memory loads and global stores, and the staging of one
// sample's rows into shared memory.
#pragma once

#include "common.cuh"

namespace moce {

// four consecutive elements from shared memory (16 B fp32, 8 B for 16-bit)
template <typename T>
__device__ __forceinline__ void ld4(const T* p, float* f);
template <>
__device__ __forceinline__ void ld4<float>(const float* p, float* f) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  f[0] = v.x;
  f[1] = v.y;
  f[2] = v.z;
  f[3] = v.w;
}
template <>
__device__ __forceinline__ void ld4<__nv_bfloat16>(const __nv_bfloat16* p, float* f) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  f[0] = __uint_as_float(v.x << 16);
  f[1] = __uint_as_float(v.x & 0xffff0000u);
  f[2] = __uint_as_float(v.y << 16);
  f[3] = __uint_as_float(v.y & 0xffff0000u);
}
template <>
__device__ __forceinline__ void ld4<__half>(const __half* p, float* f) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
  f[0] = a.x;
  f[1] = a.y;
  f[2] = b.x;
  f[3] = b.y;
}

template <typename T>
__device__ __forceinline__ void st4(T* p, const float* f);
template <>
__device__ __forceinline__ void st4<float>(float* p, const float* f) {
  *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
}
template <>
__device__ __forceinline__ void st4<__nv_bfloat16>(__nv_bfloat16* p, const float* f) {
  const __nv_bfloat162 a = __floats2bfloat162_rn(f[0], f[1]);
  const __nv_bfloat162 b = __floats2bfloat162_rn(f[2], f[3]);
  uint2 v;
  v.x = *reinterpret_cast<const uint32_t*>(&a);
  v.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = v;
}
template <>
__device__ __forceinline__ void st4<__half>(__half* p, const float* f) {
  const __half2 a = __floats2half2_rn(f[0], f[1]);
  const __half2 b = __floats2half2_rn(f[2], f[3]);
  uint2 v;
  v.x = *reinterpret_cast<const uint32_t*>(&a);
  v.y = *reinterpret_cast<const uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = v;
}

// X_b [C, HW] into shared rows of HWp elements (HWp % 4 == 0); padding
// columns are zeroed.  A flat 16-byte copy when the rows are unpadded; padded
// rows of an aligned sample take the same 16-byte loads, each element then
// stored to its row and column.
template <typename T>
__device__ __forceinline__ void px_stage_rows(T* s_x, const T* xb, int C, int HW, int HWp) {
  const size_t n = (size_t)C * HW;
  if (HWp != HW && ((((uintptr_t)xb) | (n * sizeof(T))) & 15) == 0) {
    constexpr int V = 16 / sizeof(T);
    const int4* s4 = reinterpret_cast<const int4*>(xb);
    const int n16 = (int)(n * sizeof(T) / 16);
    for (int q0 = threadIdx.x; q0 < n16; q0 += 8 * blockDim.x) {
      int4 r[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int q = q0 + u * blockDim.x;
        if (q < n16) r[u] = __ldg(s4 + q);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int q = q0 + u * blockDim.x;
        if (q < n16) {
          union {
            int4 v;
            T e[V];
          } w;
          w.v = r[u];
          int c = (q * V) / HW, p = q * V - c * HW;
#pragma unroll
          for (int t = 0; t < V; ++t) {
            s_x[(size_t)c * HWp + p] = w.e[t];
            if (++p == HW) {
              p = 0;
              ++c;
            }
          }
        }
      }
    }
    const int padw = HWp - HW;
    for (int i = threadIdx.x; i < C * padw; i += blockDim.x) {
      const int c = i / padw;
      s_x[(size_t)c * HWp + HW + (i - c * padw)] = from_f<T>(0.0f);
    }
    return;
  }
  if (HWp == HW && ((((uintptr_t)xb) | (n * sizeof(T))) & 15) == 0) {
    const int4* s4 = reinterpret_cast<const int4*>(xb);
    int4* d4 = reinterpret_cast<int4*>(s_x);
    const int n16 = (int)(n * sizeof(T) / 16);
    for (int q0 = threadIdx.x; q0 < n16; q0 += 8 * blockDim.x) {
      int4 r[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int q = q0 + u * blockDim.x;
        if (q < n16) r[u] = __ldg(s4 + q);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int q = q0 + u * blockDim.x;
        if (q < n16) d4[q] = r[u];
      }
    }
  } else {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int c = warp; c < C; c += nw) {
      const T* row = xb + (size_t)c * HW;
      T* dst = s_x + (size_t)c * HWp;
      for (int p = lane; p < HWp; p += 32) dst[p] = (p < HW) ? row[p] : from_f<T>(0.0f);
    }
  }
}

}  // namespace moce
