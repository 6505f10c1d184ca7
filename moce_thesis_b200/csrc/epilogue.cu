// Eval-mode BatchNorm of a bottleneck's other convolutions, fused with what
// follows it (models_unified.py:155-169):
//   relu2(bn2(conv2(.)))                        -> y = relu(x * s + t)
//   relu3(bn3(conv3(.)) + shortcut)             -> y = relu(x * s + t + r)
//   relu3(bn3(conv3(.)) + bn_sc(conv_sc(.)))    -> y = relu(x * s + t + r * rs + rt)
// with each BatchNorm folded to a per-channel affine (s, t) in fp32 by the
// caller.  One pass over NCHW tensors: torch runs the BatchNorm, the add and
// the ReLU as two to four passes.  Every value is computed in fp32 and
// rounded once to the output type.
#include "common.cuh"

namespace moce {
namespace {

constexpr int kEpThreads = 256;

struct BnActArgs {
  const void* x;
  const float* scale;
  const float* shift;
  const void* r;         // residual or null
  const float* r_scale;  // residual's own affine or null
  const float* r_shift;
  void* y;
  uint32_t n_vec;        // vectors of V elements
  uint32_t C, HW;
  int relu;
};

template <typename T, int V>
struct Vec {
  T e[V];
};

// V elements per vector over the flat tensor (N*C*HW < 2^31).  kCross: H*W
// is not a multiple of V (7x7 maps), so a vector may cross into the next
// channel row once (H*W >= V); both rows' affines are loaded and each element
// selects its own, without branches.
template <typename T, int V, bool kCross>
__global__ void __launch_bounds__(kEpThreads) bn_act_kernel(BnActArgs a) {
  using VT = Vec<T, V>;
  const VT* x = static_cast<const VT*>(a.x);
  const VT* r = static_cast<const VT*>(a.r);
  VT* y = static_cast<VT*>(a.y);
  const bool raff = r && a.r_scale;
  const uint32_t stride = gridDim.x * kEpThreads;
  for (uint32_t i0 = blockIdx.x * kEpThreads + threadIdx.x; i0 < a.n_vec; i0 += 4 * stride) {
    VT xv[4], rv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t i = i0 + u * stride;
      if (i < a.n_vec) {
        xv[u] = x[i];
        if (r) rv[u] = r[i];
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t i = i0 + u * stride;
      if (i < a.n_vec) {
        const uint32_t e = i * V, row = e / a.HW;
        const uint32_t c0 = row % a.C;
        // elements of this vector in row c0 (the rest are in the next row)
        const uint32_t rem = kCross ? a.HW - (e - row * a.HW) : V;
        const uint32_t c1 = c0 + 1 == a.C ? 0 : c0 + 1;
        const float s0 = a.scale[c0], t0 = a.shift[c0];
        const float s1 = kCross ? a.scale[c1] : s0, t1 = kCross ? a.shift[c1] : t0;
        float rs0 = 1.0f, rt0 = 0.0f, rs1 = 1.0f, rt1 = 0.0f;
        if (raff) {
          rs0 = a.r_scale[c0];
          rt0 = a.r_shift[c0];
          rs1 = kCross ? a.r_scale[c1] : rs0;
          rt1 = kCross ? a.r_shift[c1] : rt0;
        }
        VT o;
#pragma unroll
        for (int j = 0; j < V; ++j) {
          const bool first = !kCross || (uint32_t)j < rem;
          float v = fmaf(to_f(xv[u].e[j]), first ? s0 : s1, first ? t0 : t1);
          if (r) v += fmaf(to_f(rv[u].e[j]), first ? rs0 : rs1, first ? rt0 : rt1);
          // a NaN stays NaN through the ReLU, as in torch
          if (a.relu && v < 0.0f) v = 0.0f;
          o.e[j] = from_f<T>(v);
        }
        y[i] = o;
      }
    }
  }
}

template <typename T, int V, bool kCross>
int bn_act_launch(const BnActArgs& a, void* stream) {
  const long long want = ((long long)a.n_vec + kEpThreads * 4 - 1) / (kEpThreads * 4);
  const long long cap = 8LL * num_sms();
  const unsigned grid = (unsigned)(want < 1 ? 1 : want > cap ? cap : want);
  bn_act_kernel<T, V, kCross><<<grid, kEpThreads, 0, (cudaStream_t)stream>>>(a);
  return check_launch("bn_act_kernel");
}

template <typename T, int V>
int bn_act_pick(const BnActArgs& a, void* stream) {
  return a.HW % V == 0 ? bn_act_launch<T, V, false>(a, stream) : bn_act_launch<T, V, true>(a, stream);
}

}  // namespace
}  // namespace moce

using namespace moce;

extern "C" int moce_bn_act(const void* x, int dtype, int64_t N, int64_t C, int64_t HW, const float* scale,
                           const float* shift, const void* residual, const float* r_scale, const float* r_shift,
                           int relu, void* y, void* stream) {
  if (N == 0) return MOCE_OK;  // an empty batch is a no-op
  MOCE_REQUIRE(x && scale && shift && y, MOCE_ERR_INVALID, "moce_bn_act: null pointer argument");
  MOCE_REQUIRE(!r_scale == !r_shift, MOCE_ERR_INVALID, "moce_bn_act: r_scale and r_shift go together");
  MOCE_REQUIRE(!r_scale || residual, MOCE_ERR_INVALID, "moce_bn_act: r_scale without a residual");
  MOCE_REQUIRE(dtype_ok(dtype), MOCE_ERR_INVALID, "moce_bn_act: unknown dtype %d", dtype);
  MOCE_REQUIRE(N > 0 && C >= 1 && HW >= 1, MOCE_ERR_INVALID, "moce_bn_act: invalid shape");
  MOCE_REQUIRE(N * C * HW < ((int64_t)1 << 31), MOCE_ERR_UNSUPPORTED, "moce_bn_act: shape too large");
  const size_t es = dtype_size(dtype);
  const uintptr_t al = (uintptr_t)x | (uintptr_t)y | (uintptr_t)residual;
  const int64_t n = N * C * HW;
  // the widest vector that divides the tensor, that every pointer admits and
  // that crosses at most one channel row boundary (V <= H*W)
  int V = 1;
  for (int v : {16 / (int)es, 8 / (int)es, 4 / (int)es})
    if (v > 1 && n % v == 0 && al % (v * es) == 0 && v <= HW) {
      V = v;
      break;
    }
  BnActArgs a{x, scale, shift, residual, r_scale, r_shift, y, (uint32_t)(n / V), (uint32_t)C, (uint32_t)HW,
              relu ? 1 : 0};
  return dispatch_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    if constexpr (sizeof(T) == 2) {
      switch (V) {
        case 8: return bn_act_pick<T, 8>(a, stream);
        case 4: return bn_act_pick<T, 4>(a, stream);
        case 2: return bn_act_pick<T, 2>(a, stream);
        default: return bn_act_launch<T, 1, false>(a, stream);
      }
    } else {
      switch (V) {
        case 4: return bn_act_pick<T, 4>(a, stream);
        case 2: return bn_act_pick<T, 2>(a, stream);
        default: return bn_act_launch<T, 1, false>(a, stream);
      }
    }
  });
}
