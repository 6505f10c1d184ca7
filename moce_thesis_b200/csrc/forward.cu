// Forward kernels of the MoCE layer on sm_100a.
//
// Pass 1 (gate_kernel): global average pool of X fused with the shared
// Linear(k,1) temperature gate -> z [B,C] and T [B,E_r].
//   Reference: MoCE.py:174-178 (train), MoCE.py:212-218 (eval).
// Pass 2 (mix_kernel): per-expert softmax of ln/T, the convex gather-mix of
// the k selected channels, and the residual expert, from a shared-memory tile
// of all C channels of one sample, so X is read from HBM once and Y written
// once.
//   Reference: MoCE.py:188-199 (train), MoCE.py:219-229 -> moce_kernel.cu:57-231.
#include "common.cuh"

namespace moce {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// ------------------------------------------------------------------ pass 1
// grid (n_chunks, B).  Every CTA pools its sample (CTAs of one sample share
// the X read through L2), then each warp evaluates the gate for experts of its
// chunk: lanes stride the k supports, a warp sum gives the logit.
template <typename T>
__global__ void __launch_bounds__(kThreads) gate_kernel(
    const T* __restrict__ x, const float* __restrict__ pooled_in, int C, int HW,
    const int32_t* __restrict__ idx, int E_r, int k, const float* __restrict__ gate_w,
    const float* __restrict__ gate_b, float tmin_tau, float trange_tau, float* __restrict__ z,
    float* __restrict__ Tout) {
  extern __shared__ float s_mem[];
  float* s_z = s_mem;          // C
  float* s_w = s_mem + C;      // k
  const int b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (pooled_in) {
    for (int c = threadIdx.x; c < C; c += kThreads) s_z[c] = pooled_in[(size_t)b * C + c];
  } else {
    const T* xb = x + (size_t)b * C * HW;
    const float inv_hw = 1.0f / (float)HW;
    for (int c = warp; c < C; c += kWarps) {
      const T* row = xb + (size_t)c * HW;
      float s = 0.0f;
      for (int p = lane; p < HW; p += 32) s += to_f(row[p]);
      s = warp_sum(s);
      if (lane == 0) {
        const float m = s * inv_hw;
        s_z[c] = m;
        if (z && blockIdx.x == 0) z[(size_t)b * C + c] = m;
      }
    }
  }
  for (int i = threadIdx.x; i < k; i += kThreads) s_w[i] = gate_w[i];
  __syncthreads();
  const float bias = (E_r > 0) ? gate_b[0] : 0.0f;
  const int per = (E_r + gridDim.x - 1) / gridDim.x;
  const int e0 = blockIdx.x * per, e1 = min(E_r, e0 + per);
  for (int e = e0 + warp; e < e1; e += kWarps) {
    const int32_t* ie = idx + (size_t)e * k;
    float g = 0.0f;
    for (int i = lane; i < k; i += 32) g += s_w[i] * s_z[ie[i]];
    g = warp_sum(g) + bias;
    if (lane == 0) Tout[(size_t)b * E_r + e] = temperature(g, tmin_tau, trange_tau, nullptr);
  }
}

// ------------------------------------------------------------------ pass 2
// grid (n_ptiles * n_chunks, B), 256 threads.  The CTA stages X[b, :, tile]
// (all C channels, TP pixels, pitch TP) in shared memory, then each warp owns
// experts of its chunk: lane i of the warp computes the softmax weight and
// channel offset of support i, and the warp walks the supports with shuffles,
// every lane accumulating VP pixels (p = lane + 32 v) in fp32.  Expert E_r is
// the residual: the mean over channels with mask[c] == 1.
struct MixArgs {
  const void* x;
  void* y;
  const void* idx;        // int32 or int64 [E_r, k]
  const float* ln;        // [E_r, k] (computed weights)
  const float* T;         // [B, E_r] (computed weights)
  const float* weights;   // [B, E_r, k] (given weights)
  const int32_t* mask;    // [C]
  int C, HW, E_r, k;
  int TP, n_ptiles, n_chunks;
};

template <typename T, typename IdxT, bool kGiven, int VP>
__global__ void __launch_bounds__(kThreads) mix_kernel(MixArgs a) {
  extern __shared__ __align__(16) unsigned char s_raw[];
  T* s_x = reinterpret_cast<T*>(s_raw);
  const int b = blockIdx.y;
  const int pt = blockIdx.x % a.n_ptiles, ch = blockIdx.x / a.n_ptiles;
  const int C = a.C, HW = a.HW, TP = a.TP, k = a.k, E_r = a.E_r;
  const int p0 = pt * TP;
  const int tp = min(TP, HW - p0);
  const T* xb = static_cast<const T*>(a.x) + (size_t)b * C * HW;

  // ---- stage the tile: rows of tp pixels, pitch TP
  if (tp == HW && TP == HW) {
    const size_t n = (size_t)C * HW;
    const size_t bytes = n * sizeof(T);
    if ((bytes & 15) == 0 && ((uintptr_t)xb & 15) == 0) {
      const int4* src = reinterpret_cast<const int4*>(xb);
      int4* dst = reinterpret_cast<int4*>(s_x);
      for (size_t q = threadIdx.x; q < bytes / 16; q += kThreads) dst[q] = __ldg(src + q);
    } else {
      for (size_t q = threadIdx.x; q < n; q += kThreads) s_x[q] = xb[q];
    }
  } else {
    for (int c = threadIdx.x >> 5; c < C; c += kWarps) {
      const T* row = xb + (size_t)c * HW + p0;
      for (int p = threadIdx.x & 31; p < tp; p += 32) s_x[c * TP + p] = row[p];
    }
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = E_r + 1;
  const int per = (E + a.n_chunks - 1) / a.n_chunks;
  const int e0 = ch * per, e1 = min(E, e0 + per);
  const IdxT* idx = static_cast<const IdxT*>(a.idx);
  T* yb = static_cast<T*>(a.y) + (size_t)b * E * HW + p0;

  for (int e = e0 + warp; e < e1; e += kWarps) {
    float acc[VP];
#pragma unroll
    for (int v = 0; v < VP; ++v) acc[v] = 0.0f;
    if (e < E_r) {
      float t = 1.0f, m = 0.0f, ssum = 1.0f;
      if (!kGiven) {
        t = a.T[(size_t)b * E_r + e];
        const float* lne = a.ln + (size_t)e * k;
        m = -INFINITY;
        for (int i = lane; i < k; i += 32) m = nan_max(m, lne[i] / t);
        m = warp_max(m);
        ssum = 0.0f;
        for (int i = lane; i < k; i += 32) ssum += expf(lne[i] / t - m);
        ssum = warp_sum(ssum);
      }
      for (int i0 = 0; i0 < k; i0 += 32) {
        const int i = i0 + lane;
        float w_l = 0.0f;
        int off_l = 0;
        if (i < k) {
          off_l = (int)idx[(size_t)e * k + i] * TP;
          if (kGiven) w_l = a.weights[((size_t)b * E_r + e) * k + i];
          else w_l = expf(a.ln[(size_t)e * k + i] / t - m) / ssum;
        }
        const int n = min(32, k - i0);
        for (int j = 0; j < n; ++j) {
          const float w = __shfl_sync(kFull, w_l, j);
          const int off = __shfl_sync(kFull, off_l, j);
#pragma unroll
          for (int v = 0; v < VP; ++v) {
            const int p = lane + 32 * v;
            if (p < tp) acc[v] += w * to_f(s_x[off + p]);
          }
        }
      }
    } else {
      // residual expert: mean over uncovered channels (0 if none)
      int cnt = 0;
      for (int c = 0; c < C; ++c) {
        if (a.mask[c] == 1) {
          ++cnt;
#pragma unroll
          for (int v = 0; v < VP; ++v) {
            const int p = lane + 32 * v;
            if (p < tp) acc[v] += to_f(s_x[c * TP + p]);
          }
        }
      }
#pragma unroll
      for (int v = 0; v < VP; ++v) acc[v] = (cnt > 0) ? acc[v] / (float)cnt : 0.0f;
    }
    T* ye = yb + (size_t)e * HW;
#pragma unroll
    for (int v = 0; v < VP; ++v) {
      const int p = lane + 32 * v;
      if (p < tp) ye[p] = from_f<T>(acc[v]);
    }
  }
}

constexpr size_t kSmemBudget = 200 * 1024;   // per CTA, of the 227 KB opt-in

struct MixPlan {
  int TP, VP, n_ptiles, n_chunks;
  size_t smem;
};

int plan_mix(int64_t B, int64_t C, int64_t HW, int64_t E_r, size_t esize, MixPlan* pl) {
  int64_t max_tp = (int64_t)(kSmemBudget / ((size_t)C * esize));
  if (max_tp < 1)
    return set_error(MOCE_ERR_UNSUPPORTED, "mix: C=%lld channels do not fit one pixel column in shared memory", (long long)C);
  int64_t tp = HW < 256 ? HW : 256;
  if (tp > max_tp) tp = max_tp;
  int vp = (int)((tp + 31) / 32);
  int VP = vp <= 1 ? 1 : vp <= 2 ? 2 : vp <= 4 ? 4 : 8;
  pl->TP = (int)tp;
  pl->VP = VP;
  pl->n_ptiles = (int)((HW + tp - 1) / tp);
  const int64_t E = E_r + 1;
  const int64_t units = B * pl->n_ptiles;
  const int64_t target = 4LL * num_sms();
  int64_t nch = units >= target ? 1 : (target + units - 1) / units;
  const int64_t max_ch = (E + kWarps - 1) / kWarps;
  if (nch > max_ch) nch = max_ch;
  if (nch < 1) nch = 1;
  pl->n_chunks = (int)nch;
  pl->smem = (size_t)C * tp * esize;
  return MOCE_OK;
}

template <typename T, typename IdxT, bool kGiven>
int launch_mix(const MixArgs& a0, int64_t B, const MixPlan& pl, cudaStream_t st) {
  MixArgs a = a0;
  a.TP = pl.TP;
  a.n_ptiles = pl.n_ptiles;
  a.n_chunks = pl.n_chunks;
  void (*kern)(MixArgs) = nullptr;
  switch (pl.VP) {
    case 1: kern = mix_kernel<T, IdxT, kGiven, 1>; break;
    case 2: kern = mix_kernel<T, IdxT, kGiven, 2>; break;
    case 4: kern = mix_kernel<T, IdxT, kGiven, 4>; break;
    default: kern = mix_kernel<T, IdxT, kGiven, 8>; break;
  }
  if (pl.smem > 48 * 1024) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem) != cudaSuccess)
      return set_error(MOCE_ERR_CUDA, "mix: cannot reserve %zu B shared memory", pl.smem);
  }
  dim3 grid((unsigned)(pl.n_ptiles * pl.n_chunks), (unsigned)B);
  kern<<<grid, kThreads, pl.smem, st>>>(a);
  return check_launch("mix_kernel");
}

template <typename T>
int launch_gate(const void* x, const float* pooled_in, int64_t B, int64_t C, int64_t HW,
                const int32_t* idx, int64_t E_r, int64_t k, const float* gw, const float* gb,
                float tmin_tau, float trange_tau, float* z, float* Tout, cudaStream_t st) {
  const size_t smem = (size_t)(C + k) * 4;
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(gate_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return set_error(MOCE_ERR_UNSUPPORTED, "gate: C=%lld too large", (long long)C);
  }
  const int64_t target = 2LL * num_sms();
  int64_t nch = B >= target ? 1 : (target + B - 1) / B;
  const int64_t max_ch = (E_r + kWarps - 1) / kWarps;
  if (nch > max_ch) nch = max_ch;
  if (nch < 1) nch = 1;
  dim3 grid((unsigned)nch, (unsigned)B);
  gate_kernel<T><<<grid, kThreads, smem, st>>>(static_cast<const T*>(x), pooled_in, (int)C, (int)HW, idx,
                                               (int)E_r, (int)k, gw, gb, tmin_tau, trange_tau, z, Tout);
  return check_launch("gate_kernel");
}

// int64 -> int32 index conversion for the reference-compatible entry points.
__global__ void idx64_to_32(const int64_t* __restrict__ in, int32_t* __restrict__ out, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = (int32_t)in[i];
}

}  // namespace

int check_shapes(const char* fn, int64_t B, int64_t C, int64_t HW, int64_t E_r, int64_t k) {
  MOCE_REQUIRE(B >= 0 && C >= 1 && HW >= 1 && E_r >= 1 && k >= 1 && k <= C, MOCE_ERR_INVALID,
               "%s: invalid shape B=%lld C=%lld HW=%lld E_r=%lld k=%lld", fn, (long long)B,
               (long long)C, (long long)HW, (long long)E_r, (long long)k);
  MOCE_REQUIRE(B < 65536 && C * HW < (int64_t)1 << 31 && (E_r + 1) * HW < (int64_t)1 << 31 &&
                   E_r * k < (int64_t)1 << 31 && (E_r + 1) * k < (int64_t)1 << 31,
               MOCE_ERR_UNSUPPORTED, "%s: shape too large (B=%lld C=%lld HW=%lld E_r=%lld k=%lld)", fn,
               (long long)B, (long long)C, (long long)HW, (long long)E_r, (long long)k);
  return MOCE_OK;
}

}  // namespace moce

using namespace moce;

extern "C" int moce_pool(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, float* pooled,
                         void* stream) {
  if (B == 0) return MOCE_OK;  // an empty batch is a no-op
  MOCE_REQUIRE(x && pooled, MOCE_ERR_INVALID, "moce_pool: null pointer argument");
  MOCE_REQUIRE(dtype_ok(dtype), MOCE_ERR_INVALID, "moce_pool: unknown dtype %d", dtype);
  int rc = check_shapes("moce_pool", B, C, HW, 1, 1);
  if (rc) return rc;
  if (B == 0) return MOCE_OK;
  // the gate kernel with E_r = 0 experts is a pure pool
  return dispatch_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    const size_t smem = (size_t)C * 4;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(gate_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return set_error(MOCE_ERR_UNSUPPORTED, "moce_pool: C too large");
    dim3 grid(1, (unsigned)B);
    gate_kernel<T><<<grid, kThreads, smem, (cudaStream_t)stream>>>(
        static_cast<const T*>(x), nullptr, (int)C, (int)HW, nullptr, 0, 0, nullptr, nullptr, 0.f, 0.f,
        pooled, nullptr);
    return check_launch("moce_pool");
  });
}

extern "C" int moce_gate_temperature(const void* x, int dtype, const float* pooled_in, int64_t B,
                                     int64_t C, int64_t HW, const int32_t* idx, int64_t E_r,
                                     int64_t k, const float* gate_w, const float* gate_b,
                                     float tmin_tau, float trange_tau, float* z, float* T,
                                     void* stream) {
  if (B == 0) return MOCE_OK;  // an empty batch is a no-op
  MOCE_REQUIRE((x || pooled_in) && idx && gate_w && gate_b && T, MOCE_ERR_INVALID,
               "moce_gate_temperature: null pointer argument");
  MOCE_REQUIRE(dtype_ok(dtype), MOCE_ERR_INVALID, "moce_gate_temperature: unknown dtype %d", dtype);
  int rc = check_shapes("moce_gate_temperature", B, C, HW, E_r, k);
  if (rc) return rc;
  if (B == 0) return MOCE_OK;
  return dispatch_dtype(dtype, [&](auto tag) {
    using Tt = decltype(tag);
    return launch_gate<Tt>(x, pooled_in, B, C, HW, idx, E_r, k, gate_w, gate_b, tmin_tau, trange_tau, z, T,
                           (cudaStream_t)stream);
  });
}

extern "C" int moce_mix(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const int32_t* idx,
                        const float* ln, const float* T, int64_t E_r, int64_t k, const int32_t* mask, void* y,
                        void* stream) {
  if (B == 0) return MOCE_OK;  // an empty batch is a no-op
  MOCE_REQUIRE(x && idx && ln && T && mask && y, MOCE_ERR_INVALID, "moce_mix: null pointer argument");
  MOCE_REQUIRE(dtype_ok(dtype), MOCE_ERR_INVALID, "moce_mix: unknown dtype %d", dtype);
  int rc = check_shapes("moce_mix", B, C, HW, E_r, k);
  if (rc) return rc;
  if (B == 0) return MOCE_OK;
  MixPlan pl;
  rc = plan_mix(B, C, HW, E_r, dtype_size(dtype), &pl);
  if (rc) return rc;
  MixArgs a{x, y, idx, ln, T, nullptr, mask, (int)C, (int)HW, (int)E_r, (int)k, 0, 0, 0};
  return dispatch_dtype(dtype, [&](auto tag) {
    using Tt = decltype(tag);
    return launch_mix<Tt, int32_t, false>(a, B, pl, (cudaStream_t)stream);
  });
}

extern "C" int moce_forward_dynamic_temp(const void* x, int dtype, const void* indices, int index_bits,
                                         const float* weights, const int32_t* mask, void* y, int64_t B,
                                         int64_t C, int64_t HW, int64_t E_r, int64_t K, void* stream) {
  if (B == 0) return MOCE_OK;  // an empty batch is a no-op
  MOCE_REQUIRE(x && indices && weights && mask && y, MOCE_ERR_INVALID,
               "moce_forward_dynamic_temp: null pointer argument");
  MOCE_REQUIRE(dtype_ok(dtype), MOCE_ERR_INVALID, "moce_forward_dynamic_temp: unknown dtype %d", dtype);
  MOCE_REQUIRE(index_bits == 32 || index_bits == 64, MOCE_ERR_INVALID,
               "moce_forward_dynamic_temp: index_bits must be 32 or 64");
  int rc = check_shapes("moce_forward_dynamic_temp", B, C, HW, E_r, K);
  if (rc) return rc;
  if (B == 0) return MOCE_OK;
  MixPlan pl;
  rc = plan_mix(B, C, HW, E_r, dtype_size(dtype), &pl);
  if (rc) return rc;
  MixArgs a{x, y, indices, nullptr, nullptr, weights, mask, (int)C, (int)HW, (int)E_r, (int)K, 0, 0, 0};
  return dispatch_dtype(dtype, [&](auto tag) {
    using Tt = decltype(tag);
    if (index_bits == 64) return launch_mix<Tt, int64_t, true>(a, B, pl, (cudaStream_t)stream);
    return launch_mix<Tt, int32_t, true>(a, B, pl, (cudaStream_t)stream);
  });
}

extern "C" size_t moce_gate_route_workspace_bytes(int64_t B, int64_t C, int64_t E_r) {
  (void)C;
  // T [B, E_r] fp32, then int32 indices [E_r, K] are converted in place of a
  // second buffer sized for K <= C
  return align256((size_t)B * E_r * 4) + align256((size_t)B * C * 4) + align256((size_t)E_r * C * 4);
}

extern "C" int moce_gate_route(const void* x, int dtype, const float* pooled, const void* indices, int index_bits,
                               const float* logits_norm, const float* gate_w, const float* gate_b,
                               const int32_t* mask, float temp_min, float temp_max, float tau, void* y, int64_t B,
                               int64_t C, int64_t HW, int64_t E_r, int64_t K, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (B == 0) return MOCE_OK;  // an empty batch is a no-op
  MOCE_REQUIRE(x && indices && logits_norm && gate_w && gate_b && mask && y, MOCE_ERR_INVALID,
               "moce_gate_route: null pointer argument");
  MOCE_REQUIRE(dtype_ok(dtype), MOCE_ERR_INVALID, "moce_gate_route: unknown dtype %d", dtype);
  MOCE_REQUIRE(index_bits == 32 || index_bits == 64, MOCE_ERR_INVALID,
               "moce_gate_route: index_bits must be 32 or 64");
  int rc = check_shapes("moce_gate_route", B, C, HW, E_r, K);
  if (rc) return rc;
  const size_t need = moce_gate_route_workspace_bytes(B, C, E_r);
  MOCE_REQUIRE(workspace && workspace_bytes >= need && ((uintptr_t)workspace & 255) == 0, MOCE_ERR_WORKSPACE,
               "moce_gate_route: workspace of %zu bytes (256-aligned) required", need);
  if (B == 0) return MOCE_OK;
  cudaStream_t st = (cudaStream_t)stream;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  float* Tb = reinterpret_cast<float*>(ws);
  float* zb = reinterpret_cast<float*>(ws + align256((size_t)B * E_r * 4));
  int32_t* idx32 = reinterpret_cast<int32_t*>(ws + align256((size_t)B * E_r * 4) + align256((size_t)B * C * 4));
  if (index_bits == 64) {
    const int n = (int)(E_r * K);
    idx64_to_32<<<(n + 255) / 256, 256, 0, st>>>(static_cast<const int64_t*>(indices), idx32, n);
    rc = check_launch("moce_gate_route/idx");
    if (rc) return rc;
  } else {
    idx32 = const_cast<int32_t*>(static_cast<const int32_t*>(indices));
  }
  // reference form: clamp((tmin + (tmax - tmin) * sigmoid(g)) * tau, 1e-3)
  rc = moce_gate_temperature(x, dtype, pooled, B, C, HW, idx32, E_r, K, gate_w, gate_b, temp_min * tau,
                             (temp_max - temp_min) * tau, pooled ? nullptr : zb, Tb, stream);
  if (rc) return rc;
  return moce_mix(x, dtype, B, C, HW, idx32, logits_norm, Tb, E_r, K, mask, y, stream);
}
