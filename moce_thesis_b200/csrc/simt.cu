// Pass 2 on CUDA cores with lanes over pixels (any dtype, H*W <= 512).
//
// The scheduled mix (mix.cu) puts experts on lanes, so every lane gathers a
// different channel row and a bank-conflict-free order of the supports has to
// be planned per route.  Here a warp owns one expert at a time and its lanes
// own the pixels: every support is one warp-uniform channel row, read as
// consecutive 16-byte (fp32) or 8-byte (16-bit) words, conflict-free by
// construction, four pixels per lane per 128-pixel slab.  This suits maps of
// a few hundred pixels (the 14x14 and 28x28 stages); X_b sits whole in shared
// memory, so the sample is read from HBM once per CTA.
//
// Per expert (MoCE.py:216-221 / 175-188): lane i holds support i (i and
// i + 32 for k <= 64); the gate Linear(k,1) on z[S_e], the temperature, and
// the softmax of ln / T are warp reductions; then the k weighted rows are
// summed pixel by pixel in support order and the row of Y is stored directly.
#include <cooperative_groups.h>

#include "px.cuh"

namespace moce {
namespace {

// threads per CTA: 1024 (32 warps, more loads in flight per SM) for maps of
// at most two 128-pixel slabs, where the accumulators leave room at 64
// registers a thread; 512 for larger maps.  At batch 1024 the 1024-thread
// CTAs cut the C=1024 14x14 mix from 1.97 to 1.19 ms and the C=2048 7x7
// (k=128) mix from 3.51 to 2.26 ms.
__host__ __device__ constexpr int px_threads(int nslab) { return nslab <= 2 ? 1024 : 512; }

struct PxArgs {
  const void* x;
  void* y;
  const float* z;
  const int32_t* idx;
  const float* ln;
  const float* gate_w;
  const float* gate_b;
  float* T_out;
  float tmin_tau, trange_tau;
  const float* T_in;              // given temperatures [B, E_r] (z and the gate unused), or null
  int B, C, HW, HWp, E_r, k;
  int vec_out;                    // Y rows allow 4-element vector stores
  int vec_in;                     // X rows allow 4-element vector loads (global-memory kernel)
  int csplit;                     // channels staged per CTA (C, or ceil(C/2) in a CTA pair)
};

// grid (n_echunks, B); kPxThreads threads; warp per expert.  CL == 2: the
// two CTAs of a cluster (consecutive expert chunks of one sample) each stage
// half of X_b's channels, and a support row of the other half is read from
// the peer's shared memory (distributed shared memory), so samples of up to
// twice the shared memory of one CTA (C = 1024 at 14x14) stay on chip.
// kCw: the expert's supports are staged as (channel, weight) pairs in a
// buffer of the warp in shared memory and read two per 16-byte broadcast
// load, in place of two shuffles per support (when the buffers fit).
template <typename T, int NSLAB, int KL, int CL, bool kCw>
__global__ void __launch_bounds__(px_threads(NSLAB), 1) mix_px_kernel(PxArgs a) {
  constexpr int kPxThreads = px_threads(NSLAB), kPxWarps = kPxThreads / 32;
  constexpr int kCwStride = KL * 16 + 1;                                               // float4 per warp
  extern __shared__ __align__(16) unsigned char s_raw[];
  const int C = a.C, HW = a.HW, HWp = a.HWp, k = a.k, E_r = a.E_r;
  const int Ch = (CL == 1) ? C : a.csplit;                                             // channels per CTA
  int rank = 0;
  if constexpr (CL > 1) rank = (int)cooperative_groups::this_cluster().block_rank();
  const int cs0 = rank * Ch, chn = min(C, cs0 + Ch) - cs0;                             // staged here
  T* s_x = reinterpret_cast<T*>(s_raw);                                                // Ch x HWp
  float* s_z = reinterpret_cast<float*>(s_raw + (((size_t)Ch * HWp * sizeof(T) + 15) & ~size_t(15)));  // C
  float* s_gw = s_z + C;                                                               // k
  // kCw: [warp][kCwStride] float4, after z and the gate weights
  float4* s_cw = reinterpret_cast<float4*>(
      s_raw + ((reinterpret_cast<unsigned char*>(s_gw + k) - s_raw + 15) & ~(ptrdiff_t)15));
  const int b = blockIdx.y, ch = blockIdx.x, nch = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const T* xg = static_cast<const T*>(a.x);
  px_stage_rows<T>(s_x, xg + ((size_t)b * C + cs0) * HW, chn, HW, HWp);
  if (!a.T_in) {
    for (int c = threadIdx.x; c < C; c += kPxThreads) s_z[c] = a.z[(size_t)b * C + c];
    for (int i = threadIdx.x; i < k; i += kPxThreads) s_gw[i] = a.gate_w[i];
  }
  __syncthreads();
  const T* s_peer = nullptr;
  if constexpr (CL > 1) {
    auto cluster = cooperative_groups::this_cluster();
    cluster.sync();                                     // both halves staged
    s_peer = cluster.map_shared_rank(s_x, rank ^ 1);
  }
  const float bias = a.T_in ? 0.0f : a.gate_b[0];
  const int per = (E_r + nch - 1) / nch;
  const int e0 = ch * per, e1 = min(E_r, e0 + per);
  const int E = E_r + 1;
  T* yg = static_cast<T*>(a.y);
  // the next expert's supports and logits are loaded one iteration ahead,
  // so that their global-memory latency overlaps the current expert's mix
  int c_n[KL];
  float ln_n[KL];
#pragma unroll
  for (int q = 0; q < KL; ++q) {
    const int i = lane + 32 * q;
    const bool v = i < k && e0 + warp < e1;
    c_n[q] = v ? a.idx[(size_t)(e0 + warp) * k + i] : 0;
    ln_n[q] = v ? a.ln[(size_t)(e0 + warp) * k + i] : -INFINITY;
  }
  for (int e = e0 + warp; e < e1; e += kPxWarps) {
    int c_l[KL];
    float u_l[KL];
#pragma unroll
    for (int q = 0; q < KL; ++q) {
      c_l[q] = c_n[q];
      u_l[q] = ln_n[q];
      const int i = lane + 32 * q;
      const bool v = i < k && e + kPxWarps < e1;
      c_n[q] = v ? a.idx[(size_t)(e + kPxWarps) * k + i] : 0;
      ln_n[q] = v ? a.ln[(size_t)(e + kPxWarps) * k + i] : -INFINITY;
    }
    float gp = 0.0f;
#pragma unroll
    for (int q = 0; q < KL; ++q) {
      const int i = lane + 32 * q;
      if (i >= k) u_l[q] = -INFINITY;
      else if (!a.T_in) gp += s_gw[i] * s_z[c_l[q]];
    }
    const float g = warp_sum(gp) + bias;
    const float t = a.T_in ? a.T_in[(size_t)b * E_r + e] : temperature(g, a.tmin_tau, a.trange_tau, nullptr);
    if (a.T_out && lane == 0) a.T_out[(size_t)b * E_r + e] = t;
    float m = -INFINITY;
#pragma unroll
    for (int q = 0; q < KL; ++q) {
      if (lane + 32 * q < k) u_l[q] = u_l[q] / t;
      m = nan_max(m, u_l[q]);
    }
    m = warp_max(m);
    float a_l[KL], s = 0.0f;
#pragma unroll
    for (int q = 0; q < KL; ++q) {
      a_l[q] = (lane + 32 * q < k) ? expf(u_l[q] - m) : 0.0f;
      s += a_l[q];
    }
    s = warp_sum(s);
#pragma unroll
    for (int q = 0; q < KL; ++q) a_l[q] /= s;

    float acc[NSLAB][4];
#pragma unroll
    for (int sl = 0; sl < NSLAB; ++sl)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[sl][j] = 0.0f;
    // one support's row into the accumulators (the row's owner is uniform
    // across the warp: one support at a time)
    auto mix_support = [&](int c, float w) {
      auto mix_row = [&](const T* row) {
#pragma unroll
        for (int sl = 0; sl < NSLAB; ++sl) {
          if (128 * sl + 4 * lane < HW) {
            float f[4];
            ld4<T>(row + 128 * sl, f);
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) acc[sl][jj] = fmaf(w, f[jj], acc[sl][jj]);
          }
        }
      };
      if constexpr (CL == 1) {
        mix_row(s_x + (size_t)c * HWp + 4 * lane);
      } else {
        if (c >= cs0 && c < cs0 + chn) mix_row(s_x + (size_t)(c - cs0) * HWp + 4 * lane);
        else mix_row(s_peer + (size_t)(c - (rank ^ 1) * Ch) * HWp + 4 * lane);
      }
    };
    if constexpr (kCw) {
      float4* cw = s_cw + (size_t)warp * kCwStride;
      float2* cw2 = reinterpret_cast<float2*>(cw);
#pragma unroll
      for (int q = 0; q < KL; ++q) cw2[lane + 32 * q] = make_float2(__int_as_float(c_l[q]), a_l[q]);
      __syncwarp();
#pragma unroll 2
      for (int j2 = 0; 2 * j2 < k; ++j2) {
        const float4 v = cw[j2];                              // supports 2 j2 and 2 j2 + 1
        mix_support(__float_as_int(v.x), v.y);
        if (2 * j2 + 1 < k) mix_support(__float_as_int(v.z), v.w);
      }
      __syncwarp();                                           // read before the next expert's writes
    } else {
#pragma unroll
      for (int q = 0; q < KL; ++q) {
        const int nq = min(32, k - 32 * q);
#pragma unroll 4
        for (int j = 0; j < nq; ++j) mix_support(__shfl_sync(kFull, c_l[q], j), __shfl_sync(kFull, a_l[q], j));
      }
    }
    T* yr = yg + ((size_t)b * E + e) * HW;
#pragma unroll
    for (int sl = 0; sl < NSLAB; ++sl) {
      const int p = 128 * sl + 4 * lane;
      if (p + 3 < HW && a.vec_out) {
        st4<T>(yr + p, acc[sl]);
      } else {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
          if (p + jj < HW) yr[p + jj] = from_f<T>(acc[sl][jj]);
      }
    }
  }
  // the peer reads this CTA's rows until it is done
  if constexpr (CL > 1) cooperative_groups::this_cluster().sync();
}

// Maps of at most 64 pixels (7x7): a warp mixes two experts at once, one per
// half-warp (16 lanes x 4 pixels), so 26 of 32 lanes carry pixels at 7x7
// instead of 13.  Lane i of a half holds supports i, i + 16, ... (KL16 of
// them, k <= 16 KL16); the gate, temperature and softmax reduce over the 16
// lanes of the half, and each support's channel and weight reach the half by
// a width-16 shuffle.  X_b in one CTA's shared memory, as mix_px_kernel.
//
// kCw: each half writes its expert's supports as (row offset, weight) pairs
// into a buffer of the warp in shared memory, and the pixel loop reads two
// supports per 16-byte load (a broadcast within each half; the halves'
// buffers 16 bytes out of bank step) instead of two width-16 shuffles per
// support.  Taken when the buffers fit beside X_b.
template <typename T, int KL16, bool kCw>
__global__ void __launch_bounds__(px_threads(1), 1) mix_px_half_kernel(PxArgs a) {
  constexpr int kPxThreads = px_threads(1), kPxWarps = kPxThreads / 32;
  constexpr int kCwStride = KL16 * 8 + 1;                                              // float4 per half
  extern __shared__ __align__(16) unsigned char s_raw[];
  const int C = a.C, HW = a.HW, HWp = a.HWp, k = a.k, E_r = a.E_r;
  T* s_x = reinterpret_cast<T*>(s_raw);                                                // C x HWp
  float* s_z = reinterpret_cast<float*>(s_raw + (((size_t)C * HWp * sizeof(T) + 15) & ~size_t(15)));  // C
  float* s_gw = s_z + C;                                                               // k
  // kCw: [warp][half][kCwStride] float4, after z and the gate weights
  float4* s_cw = reinterpret_cast<float4*>(
      s_raw + ((reinterpret_cast<unsigned char*>(s_gw + k) - s_raw + 15) & ~(ptrdiff_t)15));
  const int b = blockIdx.y, ch = blockIdx.x, nch = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hl = lane & 15, hsel = lane >> 4;
  const T* xg = static_cast<const T*>(a.x);
  px_stage_rows<T>(s_x, xg + (size_t)b * C * HW, C, HW, HWp);
  if (!a.T_in) {
    for (int c = threadIdx.x; c < C; c += kPxThreads) s_z[c] = a.z[(size_t)b * C + c];
    for (int i = threadIdx.x; i < k; i += kPxThreads) s_gw[i] = a.gate_w[i];
  }
  __syncthreads();
  const float bias = a.T_in ? 0.0f : a.gate_b[0];
  const int per = (E_r + nch - 1) / nch;
  const int e0 = ch * per, e1 = min(E_r, e0 + per);
  const int E = E_r + 1;
  T* yg = static_cast<T*>(a.y);
  for (int eb = e0 + 2 * warp; eb < e1; eb += 2 * kPxWarps) {       // uniform across the warp
    const int e = eb + hsel;
    const bool ve = e < e1;                                         // uniform across the half
    int c_l[KL16];
    float u_l[KL16];
#pragma unroll
    for (int q = 0; q < KL16; ++q) {
      const int i = hl + 16 * q;
      const bool v = ve && i < k;
      c_l[q] = v ? a.idx[(size_t)e * k + i] : 0;
      u_l[q] = v ? a.ln[(size_t)e * k + i] : -INFINITY;
    }
    float gp = 0.0f;
#pragma unroll
    for (int q = 0; q < KL16; ++q)
      if (hl + 16 * q < k && !a.T_in) gp += s_gw[hl + 16 * q] * s_z[c_l[q]];
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) gp += __shfl_xor_sync(kFull, gp, o);
    const float g = gp + bias;
    const float t = a.T_in ? (ve ? a.T_in[(size_t)b * E_r + e] : 1.0f)
                           : temperature(g, a.tmin_tau, a.trange_tau, nullptr);
    if (a.T_out && ve && hl == 0) a.T_out[(size_t)b * E_r + e] = t;
    float m = -INFINITY;
#pragma unroll
    for (int q = 0; q < KL16; ++q) {
      if (hl + 16 * q < k) u_l[q] = u_l[q] / t;
      m = nan_max(m, u_l[q]);
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) m = nan_max(m, __shfl_xor_sync(kFull, m, o));
    float a_l[KL16], sum = 0.0f;
#pragma unroll
    for (int q = 0; q < KL16; ++q) {
      a_l[q] = (hl + 16 * q < k) ? expf(u_l[q] - m) : 0.0f;
      sum += a_l[q];
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
#pragma unroll
    for (int q = 0; q < KL16; ++q) a_l[q] /= sum;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const int p = 4 * hl;
    if constexpr (kCw) {
      float4* cw = s_cw + (size_t)(2 * warp + hsel) * kCwStride;
      float2* cw2 = reinterpret_cast<float2*>(cw);
#pragma unroll
      for (int q = 0; q < KL16; ++q)
        cw2[hl + 16 * q] = make_float2(__int_as_float(c_l[q] * HWp), a_l[q]);
      __syncwarp();
#pragma unroll 4
      for (int j2 = 0; 2 * j2 < k; ++j2) {
        const float4 v = cw[j2];                              // supports 2 j2 and 2 j2 + 1
        if (p < HW) {
          float f[4];
          ld4<T>(s_x + __float_as_int(v.x) + p, f);
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) acc[jj] = fmaf(v.y, f[jj], acc[jj]);
          if (2 * j2 + 1 < k) {
            ld4<T>(s_x + __float_as_int(v.z) + p, f);
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) acc[jj] = fmaf(v.w, f[jj], acc[jj]);
          }
        }
      }
      __syncwarp();                                           // read before the next pair's writes
    } else {
#pragma unroll
      for (int q = 0; q < KL16; ++q) {
        const int nq = min(16, k - 16 * q);
#pragma unroll 4
        for (int j = 0; j < nq; ++j) {
          const int c = __shfl_sync(kFull, c_l[q], j, 16);
          const float w = __shfl_sync(kFull, a_l[q], j, 16);
          if (p < HW) {
            float f[4];
            ld4<T>(s_x + (size_t)c * HWp + p, f);
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) acc[jj] = fmaf(w, f[jj], acc[jj]);
          }
        }
      }
    }
    if (ve) {
      T* yr = yg + ((size_t)b * E + e) * HW;
      if (p + 3 < HW && a.vec_out) {
        st4<T>(yr + p, acc);
      } else {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
          if (p + jj < HW) yr[p + jj] = from_f<T>(acc[jj]);
      }
    }
  }
}

// k <= 32: the weights of 32 experts are computed at once with lanes over
// experts (each lane runs its expert's gate, temperature and softmax alone,
// no warp reductions), then the warp walks those experts with lanes over
// pixels, taking each support's channel and weight by shuffle from the
// expert's lane.  KMAX = 16 or 32 supports per lane in registers.
template <typename T, int NSLAB, int KMAX>
__global__ void __launch_bounds__(px_threads(NSLAB), 1) mix_px_grouped_kernel(PxArgs a) {
  constexpr int kPxThreads = px_threads(NSLAB), kPxWarps = kPxThreads / 32;
  extern __shared__ __align__(16) unsigned char s_raw[];
  const int C = a.C, HW = a.HW, HWp = a.HWp, k = a.k, E_r = a.E_r;
  T* s_x = reinterpret_cast<T*>(s_raw);                                                // C x HWp
  float* s_z = reinterpret_cast<float*>(s_raw + (((size_t)C * HWp * sizeof(T) + 15) & ~size_t(15)));  // C
  float* s_gw = s_z + C;                                                               // k
  const int b = blockIdx.y, ch = blockIdx.x, nch = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const T* xg = static_cast<const T*>(a.x);
  px_stage_rows<T>(s_x, xg + (size_t)b * C * HW, C, HW, HWp);
  if (!a.T_in) {
    for (int c = threadIdx.x; c < C; c += kPxThreads) s_z[c] = a.z[(size_t)b * C + c];
    for (int i = threadIdx.x; i < k; i += kPxThreads) s_gw[i] = a.gate_w[i];
  }
  __syncthreads();
  const float bias = a.T_in ? 0.0f : a.gate_b[0];
  const int per = (E_r + nch - 1) / nch;
  const int e0 = ch * per, e1 = min(E_r, e0 + per);
  const int E = E_r + 1;
  T* yg = static_cast<T*>(a.y);
  // warp w owns the G consecutive experts [e0 + w G, e0 + (w + 1) G) of the chunk
  const int G = min(32, (e1 - e0 + kPxWarps - 1) / kPxWarps);
  const int gb = e0 + warp * G;
  const int ge = min(e1, gb + G);
  if (gb < ge) {
    // ---- weights, lane = expert gb + lane
    const int em = gb + lane;
    const bool has = em < ge;
    int cr[KMAX];
    float ar[KMAX];
#pragma unroll
    for (int i = 0; i < KMAX; ++i) {
      const bool v = has && i < k;
      cr[i] = v ? a.idx[(size_t)em * k + i] : 0;
      ar[i] = v ? a.ln[(size_t)em * k + i] : -INFINITY;
    }
    float g = 0.0f;
#pragma unroll
    for (int i = 0; i < KMAX; ++i)
      if (i < k && !a.T_in) g += s_gw[i] * s_z[cr[i]];
    const float t = a.T_in ? (has ? a.T_in[(size_t)b * E_r + em] : 1.0f)
                           : temperature(g + bias, a.tmin_tau, a.trange_tau, nullptr);
    if (a.T_out && has) a.T_out[(size_t)b * E_r + em] = t;
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < KMAX; ++i) {
      if (i < k) ar[i] = ar[i] / t;
      m = nan_max(m, ar[i]);
    }
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < KMAX; ++i) {
      ar[i] = (i < k) ? expf(ar[i] - m) : 0.0f;
      sum += ar[i];
    }
    const float is = 1.0f / sum;
#pragma unroll
    for (int i = 0; i < KMAX; ++i) ar[i] *= is;
    // ---- mix, lanes = pixels, one expert of the group at a time
    for (int j = 0; j < ge - gb; ++j) {
      float acc[NSLAB][4];
#pragma unroll
      for (int sl = 0; sl < NSLAB; ++sl)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) acc[sl][jj] = 0.0f;
#pragma unroll
      for (int i = 0; i < KMAX; ++i) {
        if (i < k) {
          const int c = __shfl_sync(kFull, cr[i], j);
          const float w = __shfl_sync(kFull, ar[i], j);
          const T* row = s_x + (size_t)c * HWp + 4 * lane;
#pragma unroll
          for (int sl = 0; sl < NSLAB; ++sl) {
            if (128 * sl + 4 * lane < HW) {
              float f[4];
              ld4<T>(row + 128 * sl, f);
#pragma unroll
              for (int jj = 0; jj < 4; ++jj) acc[sl][jj] = fmaf(w, f[jj], acc[sl][jj]);
            }
          }
        }
      }
      T* yr = yg + ((size_t)b * E + gb + j) * HW;
#pragma unroll
      for (int sl = 0; sl < NSLAB; ++sl) {
        const int p = 128 * sl + 4 * lane;
        if (p + 3 < HW && a.vec_out) {
          st4<T>(yr + p, acc[sl]);
        } else {
#pragma unroll
          for (int jj = 0; jj < 4; ++jj)
            if (p + jj < HW) yr[p + jj] = from_f<T>(acc[sl][jj]);
        }
      }
    }
  }
}


// Pass 2 on CUDA cores for samples that do not fit shared memory (C of 1024
// and more at 14x14, 2048 at 7x7, 512 at 28x28): the same warp per expert
// and lanes over pixels as mix_px_kernel, but each support row is read from
// global memory, where the CTAs of one sample (consecutive blocks) keep X_b
// resident in L2 and L1 while they walk its experts.  Up to KL x 32 = 128
// supports per expert (lane i holds supports i, i + 32, ...) and NSLAB x 128
// pixels per row; rows with H*W % 4 == 0 are read as 4-element vectors.
template <typename T, int NSLAB, int KL>
__global__ void __launch_bounds__(px_threads(NSLAB), 1) mix_gx_kernel(PxArgs a) {
  constexpr int kPxThreads = px_threads(NSLAB), kPxWarps = kPxThreads / 32;
  extern __shared__ __align__(16) unsigned char s_raw[];
  const int C = a.C, HW = a.HW, k = a.k, E_r = a.E_r;
  float* s_z = reinterpret_cast<float*>(s_raw);                                        // C
  float* s_gw = s_z + C;                                                               // k
  const int b = blockIdx.y, ch = blockIdx.x, nch = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const T* xb = static_cast<const T*>(a.x) + (size_t)b * C * HW;
  if (!a.T_in) {
    for (int c = threadIdx.x; c < C; c += kPxThreads) s_z[c] = a.z[(size_t)b * C + c];
    for (int i = threadIdx.x; i < k; i += kPxThreads) s_gw[i] = a.gate_w[i];
  }
  __syncthreads();
  const float bias = a.T_in ? 0.0f : a.gate_b[0];
  const int per = (E_r + nch - 1) / nch;
  const int e0 = ch * per, e1 = min(E_r, e0 + per);
  const int E = E_r + 1;
  const bool vin = a.vec_in != 0;
  T* yg = static_cast<T*>(a.y);
  for (int e = e0 + warp; e < e1; e += kPxWarps) {
    int c_l[KL];
    float u_l[KL];
#pragma unroll
    for (int q = 0; q < KL; ++q) {
      const int i = lane + 32 * q;
      c_l[q] = i < k ? a.idx[(size_t)e * k + i] : 0;
      u_l[q] = i < k ? a.ln[(size_t)e * k + i] : -INFINITY;
    }
    float gp = 0.0f;
#pragma unroll
    for (int q = 0; q < KL; ++q)
      if (lane + 32 * q < k && !a.T_in) gp += s_gw[lane + 32 * q] * s_z[c_l[q]];
    const float g = warp_sum(gp) + bias;
    const float t = a.T_in ? a.T_in[(size_t)b * E_r + e] : temperature(g, a.tmin_tau, a.trange_tau, nullptr);
    if (a.T_out && lane == 0) a.T_out[(size_t)b * E_r + e] = t;
    float m = -INFINITY;
#pragma unroll
    for (int q = 0; q < KL; ++q) {
      if (lane + 32 * q < k) u_l[q] = u_l[q] / t;
      m = nan_max(m, u_l[q]);
    }
    m = warp_max(m);
    float a_l[KL], sum = 0.0f;
#pragma unroll
    for (int q = 0; q < KL; ++q) {
      a_l[q] = (lane + 32 * q < k) ? expf(u_l[q] - m) : 0.0f;
      sum += a_l[q];
    }
    sum = warp_sum(sum);
#pragma unroll
    for (int q = 0; q < KL; ++q) a_l[q] /= sum;

    float acc[NSLAB][4];
#pragma unroll
    for (int sl = 0; sl < NSLAB; ++sl)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[sl][j] = 0.0f;
#pragma unroll
    for (int q = 0; q < KL; ++q) {
      const int nq = min(32, k - 32 * q);
#pragma unroll 4
      for (int j = 0; j < nq; ++j) {
        const int c = __shfl_sync(kFull, c_l[q], j);
        const float w = __shfl_sync(kFull, a_l[q], j);
        const T* row = xb + (size_t)c * HW;
#pragma unroll
        for (int sl = 0; sl < NSLAB; ++sl) {
          const int p = 128 * sl + 4 * lane;
          float f[4];
          if (vin && p + 3 < HW) {
            ld4<T>(row + p, f);
          } else {
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) f[jj] = (p + jj < HW) ? to_f(row[p + jj]) : 0.0f;
          }
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) acc[sl][jj] = fmaf(w, f[jj], acc[sl][jj]);
        }
      }
    }
    T* yr = yg + ((size_t)b * E + e) * HW;
#pragma unroll
    for (int sl = 0; sl < NSLAB; ++sl) {
      const int p = 128 * sl + 4 * lane;
      if (p + 3 < HW && a.vec_out) {
        st4<T>(yr + p, acc[sl]);
      } else {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
          if (p + jj < HW) yr[p + jj] = from_f<T>(acc[sl][jj]);
      }
    }
  }
}

}  // namespace

size_t px_smem_bytes(int64_t C, int64_t HW, int64_t k, size_t esize) {
  const int64_t HWp = (HW + 3) / 4 * 4;
  return (((size_t)C * HWp * esize + 15) & ~size_t(15)) + (size_t)C * 4 + (size_t)k * 4;
}

// shared memory of one CTA staging Ch of the sample's C channels
static size_t px_smem_split(int64_t C, int64_t Ch, int64_t HW, int64_t k, size_t esize) {
  const int64_t HWp = (HW + 3) / 4 * 4;
  return (((size_t)Ch * HWp * esize + 15) & ~size_t(15)) + (size_t)C * 4 + (size_t)k * 4;
}

static int px_smem_max() {
  int dev = 0, smem_max = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  return smem_max;
}

// CTAs per cluster that hold one sample: 1 if X_b fits one CTA's shared
// memory, 2 if half of it does, 0 otherwise
static int px_cluster(int dtype, int64_t C, int64_t HW, int64_t k) {
  const size_t es = dtype_size(dtype), mx = (size_t)px_smem_max();
  if (px_smem_split(C, C, HW, k, es) <= mx) return 1;
  if (px_smem_split(C, (C + 1) / 2, HW, k, es) <= mx) return 2;
  return 0;
}

int px_supported(int dtype, int64_t C, int64_t HW, int64_t k) {
  if (!dtype_ok(dtype) || HW < 1 || HW > 512 || k < 1 || k > 128) return 0;
  return px_cluster(dtype, C, HW, k) > 0 ? 1 : 0;
}

int gx_supported(int dtype, int64_t C, int64_t HW, int64_t k) {
  return (dtype_ok(dtype) && HW >= 1 && HW <= 1024 && k >= 1 && k <= 128 && C >= 1 && C <= 16384) ? 1 : 0;
}

}  // namespace moce

using namespace moce;

extern "C" int moce_px_supported(int dtype, int64_t C, int64_t HW, int64_t k) { return px_supported(dtype, C, HW, k); }

// the gate from z and gate_w / gate_b, or (T_in given) the temperatures as given
static int mix_px_run(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const float* z,
                        const int32_t* idx, const float* ln, int64_t E_r, int64_t k, const float* gate_w,
                        const float* gate_b, float tmin_tau, float trange_tau, void* y, float* T_out,
                        const float* T_in, void* stream) {
  if (B == 0) return MOCE_OK;  // an empty batch is a no-op
  MOCE_REQUIRE(x && idx && ln && y && (T_in || (z && gate_w && gate_b)), MOCE_ERR_INVALID,
               "moce_mix_px: null pointer argument");
  MOCE_REQUIRE(dtype_ok(dtype), MOCE_ERR_INVALID, "moce_mix_px: unknown dtype %d", dtype);
  MOCE_REQUIRE(B > 0 && C >= 1 && HW >= 1 && E_r >= 1 && k >= 1 && k <= C, MOCE_ERR_INVALID,
               "moce_mix_px: invalid shape");
  MOCE_REQUIRE(B < 65536 && (E_r + 1) * HW < (int64_t)1 << 31 && C * HW < (int64_t)1 << 31, MOCE_ERR_UNSUPPORTED,
               "moce_mix_px: shape too large");
  MOCE_REQUIRE(px_supported(dtype, C, HW, k), MOCE_ERR_UNSUPPORTED,
               "moce_mix_px: needs H*W <= 512, k <= 128 and X_b within the shared memory of two CTAs");
  const size_t esize = dtype_size(dtype);
  const int HWp = (int)((HW + 3) / 4 * 4);
  const int CL = px_cluster(dtype, C, HW, k);
  const int64_t Ch = CL == 1 ? C : (C + 1) / 2;
  size_t smem = px_smem_split(C, Ch, HW, k, esize);
  const int nslab = (int)((HW + 127) / 128);
  const int nthr = px_threads(nslab), kPxWarps = nthr / 32;
  // CTAs per sample: the count whose rounds over the SMs waste least.  A
  // CTA costs its share of the sample's experts plus a fixed part (staging
  // X_b, the prologue), taken as 1/16 of a whole sample; the busiest SM runs
  // ceil(B * nch / SMs) CTAs.  (Small batches used to take enough CTAs per
  // sample to cover the SMs four times, each restaging X_b.)
  const int64_t max_ch = (E_r + kPxWarps - 1) / kPxWarps;
  const int64_t n_sm = num_sms();
  int64_t nch = CL;
  double best = 1e30;
  for (int64_t c = CL; c <= max_ch && c <= 64; c += CL) {
    const double cost = (double)((B * c + n_sm - 1) / n_sm) * (1.0 / (double)c + 1.0 / 16.0);
    if (cost < best - 1e-9) {
      best = cost;
      nch = c;
    }
  }
  // grouped weights (k <= 16) pay off with at least 8 experts per warp; a
  // group holds at most 32
  const int64_t per = (E_r + nch - 1) / nch;
  const bool grouped = CL == 1 && k <= 16 && per >= 8 * kPxWarps;
  if (grouped && per > 32 * kPxWarps) nch = (E_r + 32 * kPxWarps - 1) / (32 * kPxWarps);
  const int vec = (HW % 4 == 0) && (((uintptr_t)y) % 16 == 0);
  PxArgs a{x, y, z, idx, ln, gate_w, gate_b, T_in ? nullptr : T_out, tmin_tau, trange_tau, T_in,
           (int)B, (int)C, (int)HW, HWp, (int)E_r, (int)k, vec, 0, (int)Ch};
  // warp buffers of (channel, weight) pairs for the warp-per-expert kernel
  const int kl32 = k <= 32 ? 1 : k <= 64 ? 2 : 4;
  const size_t cw_end = ((smem + 15) & ~size_t(15)) + (size_t)kPxWarps * (kl32 * 16 + 1) * 16;
  const bool cw_fits = cw_end <= (size_t)px_smem_max();
  return dispatch_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    void (*kern)(PxArgs) = nullptr;
#define MOCE_PX_KL(NS, CLN) (k <= 32 ? mix_px_kernel<T, NS, 1, CLN, false> : k <= 64 ? mix_px_kernel<T, NS, 2, CLN, false> \
                                                                          : mix_px_kernel<T, NS, 4, CLN, false>)
#define MOCE_PX_KLC(NS, CLN) (k <= 32 ? mix_px_kernel<T, NS, 1, CLN, true> : k <= 64 ? mix_px_kernel<T, NS, 2, CLN, true> \
                                                                           : mix_px_kernel<T, NS, 4, CLN, true>)
#define MOCE_PX_PICK(NS)                                                                          \
  case NS:                                                                                        \
    kern = grouped ? mix_px_grouped_kernel<T, NS, 16>                                             \
           : cw_fits ? (CL == 2 ? MOCE_PX_KLC(NS, 2) : MOCE_PX_KLC(NS, 1))                        \
                     : (CL == 2 ? MOCE_PX_KL(NS, 2) : MOCE_PX_KL(NS, 1));                          \
    if (!grouped && cw_fits) smem = cw_end;                                                       \
    break;
    // maps of at most 64 pixels: two experts per warp (half-warps), with the
    // supports staged per warp in shared memory when that fits
    const bool half = CL == 1 && HW <= 64 && !grouped;
    if (half) {
      const int kl16 = k <= 16 ? 1 : k <= 32 ? 2 : k <= 64 ? 4 : 8;
      const size_t cw_end = ((smem + 15) & ~size_t(15)) + (size_t)kPxWarps * 2 * (kl16 * 8 + 1) * 16;
      const bool cw = cw_end <= (size_t)px_smem_max();
      if (cw) smem = cw_end;
      kern = k <= 16 ? (cw ? mix_px_half_kernel<T, 1, true> : mix_px_half_kernel<T, 1, false>)
             : k <= 32 ? (cw ? mix_px_half_kernel<T, 2, true> : mix_px_half_kernel<T, 2, false>)
             : k <= 64 ? (cw ? mix_px_half_kernel<T, 4, true> : mix_px_half_kernel<T, 4, false>)
                       : (cw ? mix_px_half_kernel<T, 8, true> : mix_px_half_kernel<T, 8, false>);
    } else switch (nslab) {
      MOCE_PX_PICK(1)
      MOCE_PX_PICK(2)
      MOCE_PX_PICK(3)
      MOCE_PX_PICK(4)
      default: return set_error(MOCE_ERR_UNSUPPORTED, "moce_mix_px: H*W=%lld", (long long)HW);
    }
#undef MOCE_PX_PICK
#undef MOCE_PX_KL
#undef MOCE_PX_KLC
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return set_error(MOCE_ERR_CUDA, "moce_mix_px: cannot reserve %zu B shared memory", smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)nch, (unsigned)B);
    cfg.blockDim = dim3(nthr);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = CL > 1 ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, kern, a) != cudaSuccess) return check_launch("mix_px_kernel");
    return check_launch("mix_px_kernel");
  });
}


extern "C" int moce_gx_supported(int dtype, int64_t C, int64_t HW, int64_t k) { return gx_supported(dtype, C, HW, k); }

// the gate from z and gate_w / gate_b, or (T_in given) the temperatures as given
static int mix_gx_run(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const float* z,
                        const int32_t* idx, const float* ln, int64_t E_r, int64_t k, const float* gate_w,
                        const float* gate_b, float tmin_tau, float trange_tau, void* y, float* T_out,
                        const float* T_in, void* stream) {
  if (B == 0) return MOCE_OK;  // an empty batch is a no-op
  MOCE_REQUIRE(x && idx && ln && y && (T_in || (z && gate_w && gate_b)), MOCE_ERR_INVALID,
               "moce_mix_gx: null pointer argument");
  MOCE_REQUIRE(dtype_ok(dtype), MOCE_ERR_INVALID, "moce_mix_gx: unknown dtype %d", dtype);
  MOCE_REQUIRE(B > 0 && C >= 1 && HW >= 1 && E_r >= 1 && k >= 1 && k <= C, MOCE_ERR_INVALID,
               "moce_mix_gx: invalid shape");
  MOCE_REQUIRE(B < 65536 && (E_r + 1) * HW < (int64_t)1 << 31 && C * HW < (int64_t)1 << 31, MOCE_ERR_UNSUPPORTED,
               "moce_mix_gx: shape too large");
  MOCE_REQUIRE(gx_supported(dtype, C, HW, k), MOCE_ERR_UNSUPPORTED,
               "moce_mix_gx: needs H*W <= 1024, k <= 128 and C <= 16384");
  const size_t esize = dtype_size(dtype);
  const size_t smem = (size_t)C * 4 + (size_t)k * 4;
  const int nslab = (int)((HW + 127) / 128);
  const int ns_t = nslab <= 1 ? 1 : nslab <= 2 ? 2 : nslab <= 4 ? 4 : 8;   // slabs of the instantiation
  const int nthr = px_threads(ns_t), kPxWarps = nthr / 32;
  // expert chunks per sample: enough CTAs to cover the SMs four times over
  int64_t nch = (4LL * num_sms() + B - 1) / B;
  const int64_t max_ch = (E_r + kPxWarps - 1) / kPxWarps;
  if (nch > max_ch) nch = max_ch;
  if (nch < 1) nch = 1;
  const int vout = (HW % 4 == 0) && (((uintptr_t)y) % 16 == 0);
  const int vin = (HW % 4 == 0) && (((uintptr_t)x) % (4 * esize) == 0);
  PxArgs a{x, y, z, idx, ln, gate_w, gate_b, T_in ? nullptr : T_out, tmin_tau, trange_tau, T_in,
           (int)B, (int)C, (int)HW, (int)HW, (int)E_r, (int)k, vout, vin, (int)C};
  return dispatch_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    void (*kern)(PxArgs) = nullptr;
    const int ns = ns_t;
#define MOCE_GX_PICK(NS)                                                                          \
  case NS:                                                                                        \
    kern = k <= 32 ? mix_gx_kernel<T, NS, 1> : k <= 64 ? mix_gx_kernel<T, NS, 2> : mix_gx_kernel<T, NS, 4>; \
    break;
    switch (ns) {
      MOCE_GX_PICK(1)
      MOCE_GX_PICK(2)
      MOCE_GX_PICK(4)
      MOCE_GX_PICK(8)
      default: return set_error(MOCE_ERR_UNSUPPORTED, "moce_mix_gx: H*W=%lld", (long long)HW);
    }
#undef MOCE_GX_PICK
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return set_error(MOCE_ERR_CUDA, "moce_mix_gx: cannot reserve %zu B shared memory", smem);
    kern<<<dim3((unsigned)nch, (unsigned)B), nthr, smem, (cudaStream_t)stream>>>(a);
    return check_launch("mix_gx_kernel");
  });
}

extern "C" int moce_mix_px(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const float* z,
                           const int32_t* idx, const float* ln, int64_t E_r, int64_t k, const float* gate_w,
                           const float* gate_b, float tmin_tau, float trange_tau, void* y, float* T_out,
                           void* stream) {
  return mix_px_run(x, dtype, B, C, HW, z, idx, ln, E_r, k, gate_w, gate_b, tmin_tau, trange_tau, y, T_out, nullptr,
                    stream);
}

extern "C" int moce_mix_px_t(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const float* T,
                             const int32_t* idx, const float* ln, int64_t E_r, int64_t k, void* y, void* stream) {
  MOCE_REQUIRE(T || B == 0, MOCE_ERR_INVALID, "moce_mix_px_t: null T");
  return mix_px_run(x, dtype, B, C, HW, nullptr, idx, ln, E_r, k, nullptr, nullptr, 0.f, 0.f, y, nullptr, T, stream);
}

extern "C" int moce_mix_gx(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const float* z,
                           const int32_t* idx, const float* ln, int64_t E_r, int64_t k, const float* gate_w,
                           const float* gate_b, float tmin_tau, float trange_tau, void* y, float* T_out,
                           void* stream) {
  return mix_gx_run(x, dtype, B, C, HW, z, idx, ln, E_r, k, gate_w, gate_b, tmin_tau, trange_tau, y, T_out, nullptr,
                    stream);
}

extern "C" int moce_mix_gx_t(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const float* T,
                             const int32_t* idx, const float* ln, int64_t E_r, int64_t k, void* y, void* stream) {
  MOCE_REQUIRE(T || B == 0, MOCE_ERR_INVALID, "moce_mix_gx_t: null T");
  return mix_gx_run(x, dtype, B, C, HW, nullptr, idx, ln, E_r, k, nullptr, nullptr, 0.f, 0.f, y, nullptr, T, stream);
}
