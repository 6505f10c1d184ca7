// Backward kernels of the MoCE layer on sm_100a.
//
// The reference has no backward kernel: it trains through autograd over
// MoCE.forward_train (MoCE.py:153-201).  The gradients below are that graph's,
// derived by hand (u = ln/T, a = softmax(u)):
//   da[b,e,i] = sum_p dY[b,e,p] X[b,S_ei,p]
//   du = a (da - sum_j a_j da_j);  dln_b = du / T;  dT = -sum_i du_i u_i / T
//   dT passes the 1e-3 clamp only where the unclamped value >= 1e-3
//   dg = dT * (tmax - tmin) * tau * sigmoid(g) (1 - sigmoid(g))
//   dgate_w[i] = sum_{b,e} dg z[b,S_ei];  dgate_b = sum dg;  dz[b,S_ei] += dg w_i
//   dX[b,c,p] = sum_{(e,i): S_ei = c} a dY[b,e,p] + mask[c]/n_u dY[b,E_r,p] + dz[b,c]/HW
//   dL[e,S_e] = backward of ln = (sel - mean) / max(std, 1) applied to sum_b dln_b
// Batch reductions run in a fixed order (no atomics), so results are
// deterministic.
//
// Given-temperature mode (gate_w == nullptr; moce_backward_t): T came from a
// gate the caller differentiates itself (the two-layer gate), so the kernels
// stop at dT -- stored where dg goes, without the clamp mask or the sigmoid
// factor, which belong to the caller's gate -- and add no dz term to dX.
#include "px.cuh"

namespace moce {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

int bwd_chunks(int64_t B, int64_t E_r) {
  // depends on shapes only, so the workspace size is device independent
  const int64_t target = 1184;  // 8 CTAs x 148 SMs
  int64_t nch = B >= target ? 1 : (target + B - 1) / B;
  const int64_t max_ch = (E_r + kWarps - 1) / kWarps;
  if (nch > max_ch) nch = max_ch;
  return nch < 1 ? 1 : (int)nch;
}

struct BwdWs {
  float* a;       // [B, E_r, k] softmax weights
  float* dlnb;    // [B, E_r, k] per-sample d ln
  float* dg;      // [B, E_r]
  float* part_w;  // [B * nch, k]
  float* part_b;  // [B * nch]
  float* dln;     // [E_r, k]
};

size_t ws_layout(int64_t B, int64_t E_r, int64_t k, unsigned char* base, BwdWs* w) {
  const int nch = bwd_chunks(B, E_r);
  const size_t sz[6] = {(size_t)B * E_r * k * 4, (size_t)B * E_r * k * 4, (size_t)B * E_r * 4,
                        (size_t)B * nch * k * 4, (size_t)B * nch * 4, (size_t)E_r * k * 4};
  size_t off = 0;
  float* ptr[6];
  for (int i = 0; i < 6; ++i) {
    ptr[i] = base ? reinterpret_cast<float*>(base + off) : nullptr;
    off += align256(sz[i] ? sz[i] : 1);
  }
  if (w) *w = BwdWs{ptr[0], ptr[1], ptr[2], ptr[3], ptr[4], ptr[5]};
  return off;
}

// grid (nch, B): warp per expert.  da by warp-reduced dot products over the
// pixels, then the softmax / temperature / gate chain per (b, e).
template <typename T>
__global__ void __launch_bounds__(kThreads) bwd_route_kernel(
    const T* __restrict__ x, const T* __restrict__ dy, int C, int HW, const int32_t* __restrict__ idx,
    const float* __restrict__ ln, int E_r, int k, const float* __restrict__ gate_w,
    const float* __restrict__ gate_b, float tmin_tau, float trange_tau, const float* __restrict__ z,
    const float* __restrict__ Tb, BwdWs ws) {
  extern __shared__ float s_mem[];
  float* s_z = s_mem;                     // C
  float* s_w = s_z + C;                   // k
  float* s_pw = s_w + k;                  // kWarps * k
  float* s_pb = s_pw + kWarps * k;        // kWarps
  const int b = blockIdx.y, ch = blockIdx.x, nch = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool tg = gate_w == nullptr;       // given-temperature mode
  if (!tg) {
    for (int c = threadIdx.x; c < C; c += kThreads) s_z[c] = z[(size_t)b * C + c];
    for (int i = threadIdx.x; i < k; i += kThreads) s_w[i] = gate_w[i];
  }
  for (int i = threadIdx.x; i < kWarps * k; i += kThreads) s_pw[i] = 0.0f;
  if (threadIdx.x < kWarps) s_pb[threadIdx.x] = 0.0f;
  __syncthreads();
  const float bias = tg ? 0.0f : gate_b[0];
  const int per = (E_r + nch - 1) / nch;
  const int e0 = ch * per, e1 = min(E_r, e0 + per);
  const int E = E_r + 1;
  const T* xb = x + (size_t)b * C * HW;
  for (int e = e0 + warp; e < e1; e += kWarps) {
    const int32_t* ie = idx + (size_t)e * k;
    const float* lne = ln + (size_t)e * k;
    const size_t be = (size_t)b * E_r + e;
    const float t = Tb[be];
    float g = 0.0f;
    if (!tg)
      for (int i = lane; i < k; i += 32) g += s_w[i] * s_z[ie[i]];
    g = warp_sum(g) + bias;
    float m = -INFINITY;
    for (int i = lane; i < k; i += 32) m = nan_max(m, lne[i] / t);
    m = warp_max(m);
    float ssum = 0.0f;
    for (int i = lane; i < k; i += 32) ssum += expf(lne[i] / t - m);
    ssum = warp_sum(ssum);
    const T* dye = dy + ((size_t)b * E + e) * HW;
    float S = 0.0f;
    for (int i0 = 0; i0 < k; i0 += 32) {
      const int i = i0 + lane;
      const int c_l = (i < k) ? ie[i] : 0;
      const float a_l = (i < k) ? expf(lne[i] / t - m) / ssum : 0.0f;
      float da_l = 0.0f;
      const int n = min(32, k - i0);
      for (int j = 0; j < n; ++j) {
        const int c = __shfl_sync(kFull, c_l, j);
        const T* xr = xb + (size_t)c * HW;
        float part = 0.0f;
        for (int p = lane; p < HW; p += 32) part += to_f(dye[p]) * to_f(xr[p]);
        part = warp_sum(part);
        if (lane == j) da_l = part;
      }
      if (i < k) {
        ws.a[be * k + i] = a_l;
        ws.dlnb[be * k + i] = da_l;   // holds da until the second sweep
      }
      S += a_l * da_l;
    }
    S = warp_sum(S);
    float dTp = 0.0f;
    for (int i0 = 0; i0 < k; i0 += 32) {
      const int i = i0 + lane;
      if (i < k) {
        const float a_l = ws.a[be * k + i];
        const float du = a_l * (ws.dlnb[be * k + i] - S);
        ws.dlnb[be * k + i] = du / t;
        dTp += du * (lne[i] / t);
      }
    }
    float dT = -warp_sum(dTp) / t;
    float dg = dT;                          // given-temperature mode: dT itself
    if (!tg) {
      const float sig = 1.0f / (1.0f + expf(-g));
      const float t_raw = tmin_tau + trange_tau * sig;
      if (!(t_raw >= 1e-3f)) dT = 0.0f;
      dg = dT * trange_tau * sig * (1.0f - sig);
    }
    if (lane == 0) {
      ws.dg[be] = dg;
      s_pb[warp] += dg;
    }
    if (!tg)
      for (int i = lane; i < k; i += 32) s_pw[warp * k + i] += dg * s_z[ie[i]];
  }
  __syncthreads();
  const size_t q = (size_t)b * nch + ch;
  for (int i = threadIdx.x; i < k; i += kThreads) {
    float s = 0.0f;
    for (int w = 0; w < kWarps; ++w) s += s_pw[w * k + i];
    ws.part_w[q * k + i] = s;
  }
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int w = 0; w < kWarps; ++w) s += s_pb[w];
    ws.part_b[q] = s;
  }
}

// grid (ceil(C / 8), B): warp per input channel c.  Gathers the transposed
// list of c (every (e, i) with S_ei = c) against dY rows.
template <typename T>
__global__ void __launch_bounds__(kThreads) bwd_dx_kernel(
    const T* __restrict__ dy, int C, int HW, int E_r, int k, const int32_t* __restrict__ mask,
    const int32_t* __restrict__ meta, const int32_t* __restrict__ toff, const int32_t* __restrict__ tslot,
    const float* __restrict__ gate_w, BwdWs ws, T* __restrict__ dx) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * kWarps + warp;
  const int b = blockIdx.y;
  if (c >= C) return;
  const int s0 = toff[c], s1 = toff[c + 1];
  const size_t bek = (size_t)b * E_r * k;
  float dz = 0.0f;
  if (gate_w)
    for (int s = s0 + lane; s < s1; s += 32) {
      const int slot = tslot[s];
      dz += ws.dg[(size_t)b * E_r + slot / k] * gate_w[slot % k];
    }
  dz = warp_sum(dz);
  const int n_u = meta[0];
  const float rw = (mask[c] == 1 && n_u > 0) ? 1.0f / (float)n_u : 0.0f;
  const float dz_hw = dz / (float)HW;
  const int E = E_r + 1;
  const T* dyb = dy + (size_t)b * E * HW;
  T* dxr = dx + ((size_t)b * C + c) * HW;
  for (int p0 = 0; p0 < HW; p0 += 32) {
    const int p = p0 + lane;
    float acc = 0.0f;
    for (int sc = s0; sc < s1; sc += 32) {
      const int s = sc + lane;
      int e_l = 0;
      float a_l = 0.0f;
      if (s < s1) {
        const int slot = tslot[s];
        e_l = slot / k;
        a_l = ws.a[bek + slot];
      }
      const int n = min(32, s1 - sc);
      for (int j = 0; j < n; ++j) {
        const int e = __shfl_sync(kFull, e_l, j);
        const float a = __shfl_sync(kFull, a_l, j);
        if (p < HW) acc += a * to_f(dyb[(size_t)e * HW + p]);
      }
    }
    if (p < HW) {
      if (rw != 0.0f) acc += rw * to_f(dyb[(size_t)E_r * HW + p]);
      dxr[p] = from_f<T>(acc + dz_hw);
    }
  }
}

// ---------------------------------------------------------------------
// Lanes over pixels (H*W <= 512, k <= 32): the same gradients with X_b
// staged in shared memory once per CTA and every support row read as
// consecutive words by the whole warp (no bank conflicts), four pixels per
// lane per 128-pixel slab.

constexpr int kPxThreadsB = 512;
constexpr int kPxWarpsB = kPxThreadsB / 32;

// lane L of the result holds sum over the 32 lanes of v[L] (31 shuffles)
__device__ __forceinline__ float reduce_scatter32(float (&v)[32], int lane) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool up = (lane & off) != 0;
#pragma unroll
    for (int j = 0; j < off; ++j) {
      const float send = up ? v[j] : v[j + off];
      const float keep = up ? v[j + off] : v[j];
      v[j] = keep + __shfl_xor_sync(kFull, send, off);
    }
  }
  return v[0];
}

size_t px_route_smem(int64_t C, int64_t HW, int64_t k, size_t esize) {
  const int64_t HWp = (HW + 3) / 4 * 4;
  return (((size_t)C * HWp * esize + 15) & ~size_t(15)) + (size_t)(C + k + kPxWarpsB * k + kPxWarpsB) * 4;
}

// grid (nch, B): warp per expert; the dY row in registers, the k dot
// products against the support rows, one reduce-scatter, then the softmax /
// temperature / gate chain of bwd_route_kernel.
template <typename T, int NSLAB>
__global__ void __launch_bounds__(kPxThreadsB, 1) bwd_px_route_kernel(
    const T* __restrict__ x, const T* __restrict__ dy, int C, int HW, int HWp, const int32_t* __restrict__ idx,
    const float* __restrict__ ln, int E_r, int k, const float* __restrict__ gate_w,
    const float* __restrict__ gate_b, float tmin_tau, float trange_tau, const float* __restrict__ z,
    const float* __restrict__ Tb, BwdWs ws, int vec_dy) {
  extern __shared__ __align__(16) unsigned char s_raw[];
  T* s_x = reinterpret_cast<T*>(s_raw);                                                 // C x HWp
  float* s_z = reinterpret_cast<float*>(s_raw + (((size_t)C * HWp * sizeof(T) + 15) & ~size_t(15)));  // C
  float* s_w = s_z + C;                                                                 // k
  float* s_pw = s_w + k;                                                                // warps x k
  float* s_pb = s_pw + kPxWarpsB * k;                                                   // warps
  const int b = blockIdx.y, ch = blockIdx.x, nch = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  px_stage_rows<T>(s_x, x + (size_t)b * C * HW, C, HW, HWp);
  const bool tg = gate_w == nullptr;       // given-temperature mode
  if (!tg) {
    for (int c = threadIdx.x; c < C; c += kPxThreadsB) s_z[c] = z[(size_t)b * C + c];
    for (int i = threadIdx.x; i < k; i += kPxThreadsB) s_w[i] = gate_w[i];
  }
  for (int i = threadIdx.x; i < kPxWarpsB * k; i += kPxThreadsB) s_pw[i] = 0.0f;
  if (threadIdx.x < kPxWarpsB) s_pb[threadIdx.x] = 0.0f;
  __syncthreads();
  const float bias = tg ? 0.0f : gate_b[0];
  const int per = (E_r + nch - 1) / nch;
  const int e0 = ch * per, e1 = min(E_r, e0 + per);
  const int E = E_r + 1;
  const bool valid = lane < k;
  // the expert's dY row (four pixels per lane per slab), supports, logits and
  // temperature are loaded one expert ahead, overlapping the current one
  auto load_dy = [&](int e, float (&d)[NSLAB][4]) {
    const T* dyr = dy + ((size_t)b * E + e) * HW;
#pragma unroll
    for (int sl = 0; sl < NSLAB; ++sl) {
      const int p = 128 * sl + 4 * lane;
      if (p + 3 < HW && vec_dy) {
        ld4<T>(dyr + p, d[sl]);
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) d[sl][j] = (p + j < HW) ? to_f(dyr[p + j]) : 0.0f;
      }
    }
  };
  float d_n[NSLAB][4];
  int c_n = 0;
  float ln_n = 0.0f, t_n = 1.0f;
  if (e0 + warp < e1) {
    load_dy(e0 + warp, d_n);
    c_n = valid ? idx[(size_t)(e0 + warp) * k + lane] : 0;
    ln_n = valid ? ln[(size_t)(e0 + warp) * k + lane] : 0.0f;
    t_n = Tb[(size_t)b * E_r + e0 + warp];
  }
  for (int e = e0 + warp; e < e1; e += kPxWarpsB) {
    const size_t be = (size_t)b * E_r + e;
    const float t = t_n;
    const int c_l = c_n;
    const float ln_l = ln_n;
    float d[NSLAB][4];
#pragma unroll
    for (int sl = 0; sl < NSLAB; ++sl)
#pragma unroll
      for (int j = 0; j < 4; ++j) d[sl][j] = d_n[sl][j];
    if (e + kPxWarpsB < e1) {
      load_dy(e + kPxWarpsB, d_n);
      c_n = valid ? idx[(size_t)(e + kPxWarpsB) * k + lane] : 0;
      ln_n = valid ? ln[(size_t)(e + kPxWarpsB) * k + lane] : 0.0f;
      t_n = Tb[be + kPxWarpsB];
    }
    const float g = warp_sum((valid && !tg) ? s_w[lane] * s_z[c_l] : 0.0f) + bias;
    const float u = valid ? ln_l / t : -INFINITY;
    const float m = warp_max(u);
    const float ex = valid ? expf(u - m) : 0.0f;
    const float a_l = ex / warp_sum(ex);
    float part[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      float sum = 0.0f;
      if (i < k) {
        const int c = __shfl_sync(kFull, c_l, i);
        const T* row = s_x + (size_t)c * HWp + 4 * lane;
#pragma unroll
        for (int sl = 0; sl < NSLAB; ++sl) {
          if (128 * sl + 4 * lane < HW) {
            float f[4];
            ld4<T>(row + 128 * sl, f);
#pragma unroll
            for (int j = 0; j < 4; ++j) sum = fmaf(d[sl][j], f[j], sum);
          }
        }
      }
      part[i] = sum;
    }
    const float da = reduce_scatter32(part, lane);
    const float S = warp_sum(valid ? a_l * da : 0.0f);
    const float du = valid ? a_l * (da - S) : 0.0f;
    float dT = -warp_sum(du * (valid ? u : 0.0f)) / t;
    float dg = dT;                          // given-temperature mode: dT itself
    if (!tg) {
      const float sig = 1.0f / (1.0f + expf(-g));
      const float t_raw = tmin_tau + trange_tau * sig;
      if (!(t_raw >= 1e-3f)) dT = 0.0f;
      dg = dT * trange_tau * sig * (1.0f - sig);
    }
    if (valid) {
      ws.a[be * k + lane] = a_l;
      ws.dlnb[be * k + lane] = du / t;
      if (!tg) s_pw[warp * k + lane] += dg * s_z[c_l];
    }
    if (lane == 0) {
      ws.dg[be] = dg;
      s_pb[warp] += dg;
    }
  }
  __syncthreads();
  const size_t q = (size_t)b * nch + ch;
  for (int i = threadIdx.x; i < k; i += kPxThreadsB) {
    float s = 0.0f;
    for (int w = 0; w < kPxWarpsB; ++w) s += s_pw[w * k + i];
    ws.part_w[q * k + i] = s;
  }
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int w = 0; w < kPxWarpsB; ++w) s += s_pb[w];
    ws.part_b[q] = s;
  }
}

// grid (ceil(HW / 32), B): a 32-pixel tile of dY for all E experts, as fp32,
// in shared memory (dY read from HBM once); warp per input channel, lane per
// pixel, the channel's transposed list gathered in list order as in
// bwd_dx_kernel.  Each chunk of 32 list entries is staged as (row offset,
// weight) pairs in a buffer of the warp after dY, and read two entries per
// 16-byte broadcast load (one shared load per entry for the dY value, where
// two shuffles per entry were needed before).
constexpr int kDxThreads = 1024;          // 32 warps (56 registers a thread): more channel rows in flight
constexpr int kDxCwStride = 17;           // float4 per warp: 32 entries and a 16-byte skew
template <typename T>
__global__ void __launch_bounds__(kDxThreads, 1) bwd_px_dx_kernel(
    const T* __restrict__ dy, int C, int HW, int E_r, int k, const int32_t* __restrict__ mask,
    const int32_t* __restrict__ meta, const int32_t* __restrict__ toff, const int32_t* __restrict__ tslot,
    const float* __restrict__ gate_w, BwdWs ws, T* __restrict__ dx) {
  extern __shared__ __align__(16) unsigned char s_raw[];
  float* s_dy = reinterpret_cast<float*>(s_raw);            // E x 32
  const int b = blockIdx.y, p0 = blockIdx.x * 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = E_r + 1;
  float4* cw = reinterpret_cast<float4*>(s_raw + (size_t)E * 32 * 4) + (size_t)warp * kDxCwStride;
  const T* dyb = dy + (size_t)b * E * HW;
  for (int q = threadIdx.x; q < E * 32; q += kDxThreads) {
    const int p = p0 + (q & 31);
    s_dy[q] = (p < HW) ? to_f(dyb[(size_t)(q >> 5) * HW + p]) : 0.0f;
  }
  __syncthreads();
  const int n_u = meta[0];
  const int p = p0 + lane;
  const size_t bek = (size_t)b * E_r * k;
  // metadata of 32 list entries per lane-load: (expert, weight, gate term);
  // the next chunk (of this channel or the warp's next one) is fetched
  // before the current chunk's 32 entries are summed
  auto fetch = [&](int c, int sc, int& e_l, float& a_l, float& g_l) {
    const int s1 = toff[c + 1];
    const int s = sc + lane;
    e_l = 0;
    a_l = 0.0f;
    g_l = 0.0f;
    if (s < s1) {
      const int slot = tslot[s];
      e_l = slot / k;
      a_l = ws.a[bek + slot];
      g_l = gate_w ? ws.dg[(size_t)b * E_r + e_l] * gate_w[slot - e_l * k] : 0.0f;
    }
  };
  int c = warp, sc = (c < C) ? toff[c] : 0;
  int e_n = 0;
  float a_n = 0.0f, g_n = 0.0f;
  if (c < C) fetch(c, sc, e_n, a_n, g_n);
  float acc = 0.0f, dzp = 0.0f;
  while (c < C) {
    const int s1 = toff[c + 1];
    const int e_l = e_n;
    const float a_l = a_n;
    dzp += g_n;
    const int n = min(32, s1 - sc);
    // advance to the next chunk and prefetch it
    int c2 = c, sc2 = sc + 32;
    if (sc2 >= s1) {
      c2 = c + (kDxThreads / 32);
      sc2 = (c2 < C) ? toff[c2] : 0;
    }
    if (c2 < C) fetch(c2, sc2, e_n, a_n, g_n);
    reinterpret_cast<float2*>(cw)[lane] = make_float2(__int_as_float(e_l * 32), a_l);
    __syncwarp();
    for (int j2 = 0; 2 * j2 < n; ++j2) {
      const float4 v = cw[j2];                                // entries 2 j2 and 2 j2 + 1
      acc = fmaf(v.y, s_dy[__float_as_int(v.x) + lane], acc);
      if (2 * j2 + 1 < n) acc = fmaf(v.w, s_dy[__float_as_int(v.z) + lane], acc);
    }
    __syncwarp();                                             // read before the next chunk's writes
    if (c2 == c) {
      sc = sc2;
      continue;
    }
    // channel c complete
    const float dz = warp_sum(dzp);
    const float rw = (mask[c] == 1 && n_u > 0) ? 1.0f / (float)n_u : 0.0f;
    if (p < HW) {
      if (rw != 0.0f) acc += rw * s_dy[E_r * 32 + lane];
      dx[((size_t)b * C + c) * HW + p] = from_f<T>(acc + dz / (float)HW);
    }
    acc = 0.0f;
    dzp = 0.0f;
    c = c2;
    sc = sc2;
  }
}

int smem_optin() {
  int dev = 0, smem_max = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  return smem_max;
}

// grid ceil(E_r / 8): warp per expert.  Sums d ln over the batch in order,
// then back-propagates the centring / std normalisation into dL[e, S_e].
__global__ void __launch_bounds__(kThreads) bwd_logits_kernel(
    const float* __restrict__ L, int C, int B, const int32_t* __restrict__ idx, int E_r, int k, BwdWs ws,
    float* __restrict__ dL) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * kWarps + warp;
  if (e >= E_r) return;
  const float* Le = L + (size_t)e * C;
  const int32_t* ie = idx + (size_t)e * k;
  float* dLe = dL + (size_t)e * C;
  for (int c = lane; c < C; c += 32) dLe[c] = 0.0f;
  double ssel = 0.0;
  for (int i = lane; i < k; i += 32) {
    // eight independent partial sums over the batch (loads in flight),
    // combined in a fixed order
    float p8[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    const size_t stride = (size_t)E_r * k;
    const float* src = ws.dlnb + (size_t)e * k + i;
    int b = 0;
    for (; b + 8 <= B; b += 8) {
#pragma unroll
      for (int u = 0; u < 8; ++u) p8[u] += src[(size_t)(b + u) * stride];
    }
    for (; b < B; ++b) p8[b & 7] += src[(size_t)b * stride];
    const float s = ((p8[0] + p8[1]) + (p8[2] + p8[3])) + ((p8[4] + p8[5]) + (p8[6] + p8[7]));
    ws.dln[(size_t)e * k + i] = s;
    ssel += (double)Le[ie[i]];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ssel += __shfl_xor_sync(kFull, ssel, o);
  const double mean = ssel / (double)k;
  double ss = 0.0, sdc = 0.0;
  for (int i = lane; i < k; i += 32) {
    const double cen = (double)Le[ie[i]] - mean;
    ss += cen * cen;
    sdc += (double)ws.dln[(size_t)e * k + i] * cen;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ss += __shfl_xor_sync(kFull, ss, o);
    sdc += __shfl_xor_sync(kFull, sdc, o);
  }
  const double sd = (k > 1) ? sqrt(ss / (double)(k - 1)) : (double)NAN;
  const double scale = (sd != sd) ? sd : (sd < 1.0 ? 1.0 : sd);
  // d scale = -sum(dln * cen) / scale^2 ; flows into sel only where sd >= 1
  const double g_sd = (sd >= 1.0) ? (-sdc / (scale * scale)) / ((double)(k - 1) * sd) : 0.0;
  double sdcen = 0.0;
  for (int i = lane; i < k; i += 32) {
    const double cen = (double)Le[ie[i]] - mean;
    sdcen += (double)ws.dln[(size_t)e * k + i] / scale + g_sd * cen;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sdcen += __shfl_xor_sync(kFull, sdcen, o);
  const double mdc = sdcen / (double)k;
  __syncwarp();
  for (int i = lane; i < k; i += 32) {
    const double cen = (double)Le[ie[i]] - mean;
    const double dcen = (double)ws.dln[(size_t)e * k + i] / scale + g_sd * cen;
    dLe[ie[i]] = (float)(dcen - mdc);
  }
}

// Fixed-order sum of the per-CTA gate partials: warp w handles gate weight
// w (w == k: the bias); lane l sums the contiguous range l of the nq
// partials, then the lanes combine in a fixed butterfly (deterministic).
__global__ void bwd_gate_reduce_kernel(BwdWs ws, int nq, int k, float* __restrict__ dgw, float* __restrict__ dgb) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (w > k) return;
  const int per = (nq + 31) / 32;
  const int q0 = lane * per, q1 = min(nq, q0 + per);
  float s = 0.0f;
  if (w < k) {
    for (int q = q0; q < q1; ++q) s += ws.part_w[(size_t)q * k + w];
  } else {
    for (int q = q0; q < q1; ++q) s += ws.part_b[q];
  }
  s = warp_sum(s);
  if (lane == 0) {
    if (w < k) dgw[w] = s;
    else dgb[0] = s;
  }
}

int check_bwd_shapes(int64_t B, int64_t C, int64_t HW, int64_t E_r, int64_t k) {
  MOCE_REQUIRE(B >= 0 && C >= 1 && HW >= 1 && E_r >= 1 && k >= 1 && k <= C, MOCE_ERR_INVALID,
               "moce_backward: invalid shape");
  MOCE_REQUIRE(B < 65536 && C * HW < (int64_t)1 << 31 && (E_r + 1) * HW < (int64_t)1 << 31 &&
                   B * E_r * k < (int64_t)1 << 40 && E_r * k < (int64_t)1 << 31 && k <= 4096 && C <= 32768,
               MOCE_ERR_UNSUPPORTED, "moce_backward: shape too large");
  return MOCE_OK;
}

}  // namespace
}  // namespace moce

using namespace moce;

extern "C" size_t moce_backward_workspace_bytes(int64_t B, int64_t C, int64_t HW, int64_t E_r, int64_t k) {
  (void)C;
  (void)HW;
  return ws_layout(B, E_r, k, nullptr, nullptr);
}

// The linear-gate backward (gate_w given: dgate_w, dgate_b out) or the
// given-temperature backward (gate_w null: dT out).
static int backward_run(const void* x, const void* dy, int dtype, int64_t B, int64_t C, int64_t HW,
                        const float* logits, const int32_t* idx, const float* ln, const int32_t* mask,
                        const int32_t* meta, const int32_t* toff, const int32_t* tslot, int64_t E_r, int64_t k,
                        const float* gate_w, const float* gate_b, float tmin_tau, float trange_tau, const float* z,
                        const float* T, void* dx, float* dL, float* dgate_w, float* dgate_b, float* dT,
                        void* workspace, size_t workspace_bytes, void* stream) {
  const bool tg = gate_w == nullptr;
  MOCE_REQUIRE(logits && idx && ln && mask && meta && toff && tslot && dL &&
                   (tg ? dT != nullptr : (gate_b && dgate_w && dgate_b)),
               MOCE_ERR_INVALID, "moce_backward: null pointer argument");
  MOCE_REQUIRE(B == 0 || (x && dy && (tg || z) && T && dx), MOCE_ERR_INVALID, "moce_backward: null pointer argument");
  MOCE_REQUIRE(dtype_ok(dtype), MOCE_ERR_INVALID, "moce_backward: unknown dtype %d", dtype);
  int rc = check_bwd_shapes(B, C, HW, E_r, k);
  if (rc) return rc;
  const size_t need = moce_backward_workspace_bytes(B, C, HW, E_r, k);
  MOCE_REQUIRE(workspace && workspace_bytes >= need && ((uintptr_t)workspace & 255) == 0, MOCE_ERR_WORKSPACE,
               "moce_backward: workspace of %zu bytes (256-aligned) required", need);
  cudaStream_t st = (cudaStream_t)stream;
  BwdWs ws;
  ws_layout(B, E_r, k, static_cast<unsigned char*>(workspace), &ws);
  const int nch = bwd_chunks(B, E_r);
  if (B == 0) {
    if (cudaMemsetAsync(dL, 0, (size_t)E_r * C * 4, st) != cudaSuccess ||
        (!tg && (cudaMemsetAsync(dgate_w, 0, (size_t)k * 4, st) != cudaSuccess ||
                 cudaMemsetAsync(dgate_b, 0, 4, st) != cudaSuccess)))
      return set_error(MOCE_ERR_CUDA, "moce_backward: memset failed");
    return MOCE_OK;
  }
  rc = dispatch_dtype(dtype, [&](auto tag) {
    using Tt = decltype(tag);
    const int smem_max = smem_optin();
    const size_t es = sizeof(Tt);
    const size_t smem_pr = px_route_smem(C, HW, k, es);
    if (HW <= 512 && k <= 32 && smem_pr <= (size_t)smem_max) {
      const int HWp = (int)((HW + 3) / 4 * 4);
      const int nslab = (int)((HW + 127) / 128);
      const int vec = (HW % 4 == 0) && (((uintptr_t)dy) % 16 == 0);
      void (*kern)(const Tt*, const Tt*, int, int, int, const int32_t*, const float*, int, int, const float*,
                   const float*, float, float, const float*, const float*, BwdWs, int) =
          nslab == 1 ? bwd_px_route_kernel<Tt, 1> : nslab == 2 ? bwd_px_route_kernel<Tt, 2>
          : nslab == 3 ? bwd_px_route_kernel<Tt, 3> : bwd_px_route_kernel<Tt, 4>;
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_pr) != cudaSuccess)
        return set_error(MOCE_ERR_CUDA, "moce_backward: route smem %zu", smem_pr);
      kern<<<dim3(nch, (unsigned)B), kPxThreadsB, smem_pr, st>>>(
          static_cast<const Tt*>(x), static_cast<const Tt*>(dy), (int)C, (int)HW, HWp, idx, ln, (int)E_r, (int)k,
          gate_w, gate_b, tmin_tau, trange_tau, z, T, ws, vec);
    } else {
      const size_t smem = (size_t)(C + k + kWarps * k + kWarps) * 4;
      if (smem > 48 * 1024 &&
          cudaFuncSetAttribute(bwd_route_kernel<Tt>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
              cudaSuccess)
        return set_error(MOCE_ERR_UNSUPPORTED, "moce_backward: route smem %zu", smem);
      bwd_route_kernel<Tt><<<dim3(nch, (unsigned)B), kThreads, smem, st>>>(
          static_cast<const Tt*>(x), static_cast<const Tt*>(dy), (int)C, (int)HW, idx, ln, (int)E_r, (int)k,
          gate_w, gate_b, tmin_tau, trange_tau, z, T, ws);
    }
    int r = check_launch("moce_backward/route");
    if (r) return r;
    const size_t smem_dx = (size_t)(E_r + 1) * 32 * 4 + (size_t)(kDxThreads / 32) * kDxCwStride * 16;
    if (smem_dx <= (size_t)smem_max) {
      if (cudaFuncSetAttribute(bwd_px_dx_kernel<Tt>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_dx) !=
          cudaSuccess)
        return set_error(MOCE_ERR_CUDA, "moce_backward: dx smem %zu", smem_dx);
      bwd_px_dx_kernel<Tt><<<dim3((unsigned)((HW + 31) / 32), (unsigned)B), kDxThreads, smem_dx, st>>>(
          static_cast<const Tt*>(dy), (int)C, (int)HW, (int)E_r, (int)k, mask, meta, toff, tslot, gate_w, ws,
          static_cast<Tt*>(dx));
    } else {
      bwd_dx_kernel<Tt><<<dim3((unsigned)((C + kWarps - 1) / kWarps), (unsigned)B), kThreads, 0, st>>>(
          static_cast<const Tt*>(dy), (int)C, (int)HW, (int)E_r, (int)k, mask, meta, toff, tslot, gate_w, ws,
          static_cast<Tt*>(dx));
    }
    return check_launch("moce_backward/dx");
  });
  if (rc) return rc;
  bwd_logits_kernel<<<(unsigned)((E_r + kWarps - 1) / kWarps), kThreads, 0, st>>>(logits, (int)C, (int)B, idx,
                                                                                  (int)E_r, (int)k, ws, dL);
  rc = check_launch("moce_backward/logits");
  if (rc) return rc;
  if (tg) {
    // dT [B, E_r] lies in the workspace where dg goes
    if (cudaMemcpyAsync(dT, ws.dg, (size_t)B * E_r * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
      return set_error(MOCE_ERR_CUDA, "moce_backward_t: copy of dT failed");
    return MOCE_OK;
  }
  bwd_gate_reduce_kernel<<<(unsigned)((k + 1 + 7) / 8), 256, 0, st>>>(ws, (int)(B * nch), (int)k, dgate_w, dgate_b);
  return check_launch("moce_backward/gate");
}

extern "C" int moce_backward(const void* x, const void* dy, int dtype, int64_t B, int64_t C, int64_t HW,
                             const float* logits, const int32_t* idx, const float* ln, const int32_t* mask,
                             const int32_t* meta, const int32_t* toff, const int32_t* tslot, int64_t E_r,
                             int64_t k, const float* gate_w, const float* gate_b, float tmin_tau,
                             float trange_tau, const float* z, const float* T, void* dx, float* dL,
                             float* dgate_w, float* dgate_b, void* workspace, size_t workspace_bytes,
                             void* stream) {
  MOCE_REQUIRE(gate_w, MOCE_ERR_INVALID, "moce_backward: null gate_w (moce_backward_t takes given temperatures)");
  return backward_run(x, dy, dtype, B, C, HW, logits, idx, ln, mask, meta, toff, tslot, E_r, k, gate_w, gate_b,
                      tmin_tau, trange_tau, z, T, dx, dL, dgate_w, dgate_b, nullptr, workspace, workspace_bytes,
                      stream);
}

extern "C" int moce_backward_t(const void* x, const void* dy, int dtype, int64_t B, int64_t C, int64_t HW,
                               const float* logits, const int32_t* idx, const float* ln, const int32_t* mask,
                               const int32_t* meta, const int32_t* toff, const int32_t* tslot, int64_t E_r,
                               int64_t k, const float* T, void* dx, float* dL, float* dT, void* workspace,
                               size_t workspace_bytes, void* stream) {
  return backward_run(x, dy, dtype, B, C, HW, logits, idx, ln, mask, meta, toff, tslot, E_r, k, nullptr, nullptr, 0.f,
                      0.f, nullptr, T, dx, dL, nullptr, nullptr, dT, workspace, workspace_bytes, stream);
}
