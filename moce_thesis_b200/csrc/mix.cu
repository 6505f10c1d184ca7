// Fast forward path of the MoCE layer on sm_100a.
//
// Pass 1 (pool_residual_kernel): one coalesced read of X per sample, staged
// through shared memory in channel chunks, gives
//   z[b,c]      = mean_p X[b,c,p]                      (MoCE.py:174 / 212)
//   Y[b,E_r,p]  = mean over uncovered channels of X    (MoCE.py:191-196,
//                 0 when every channel is covered       moce_kernel.cu:148-231)
// Pass 2 (mix_sched_kernel): routed experts.  Lanes own experts (one warp =
// one schedule group of 32 experts); the per-sample prologue evaluates the
// Linear(k,1) gate on z, the temperature and the softmax of ln/T in
// registers (MoCE.py:216-221 / 175-188), then every lane sweeps the pixels of
// a shared-memory X tile, reading one 32-bit word (1 fp32 or 2 bf16/fp16
// pixels) per support per step from a bank that no other lane uses in that
// step (see schedule.cu).  Results are staged per warp in shared memory and
// written as contiguous expert rows.
#include <cooperative_groups.h>

#include "common.cuh"

extern "C" int moce_schedule_steps(int64_t k);

namespace moce {
namespace {

constexpr unsigned kIdle = 0xFFFFu;

// ------------------------------------------------------------------ loaders
// Flat copy of n elements (16-byte aligned source, destination and size):
// eight 16-byte loads in flight per thread before their stores.
template <typename T>
__device__ __forceinline__ void load_flat(T* dst, const T* src, size_t n) {
  const int4* s = reinterpret_cast<const int4*>(src);
  int4* d = reinterpret_cast<int4*>(dst);
  const int n16 = (int)(n * sizeof(T) / 16);
  constexpr int U = 8;
  for (int q0 = threadIdx.x; q0 < n16; q0 += U * blockDim.x) {
    int4 r[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int q = q0 + u * blockDim.x;
      if (q < n16) r[u] = __ldg(s + q);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int q = q0 + u * blockDim.x;
      if (q < n16) d[q] = r[u];
    }
  }
}

// Whole sample [C, HW] from a 16-byte aligned source into rows of `pe`
// elements: 16-byte loads (four in flight per thread) scattered by element.
// Row/column of each chunk advance incrementally (no division in the loop).
template <typename T>
__device__ __forceinline__ void load_pitched(T* dst, const T* src, int C, int HW, int pe) {
  constexpr int V = 16 / sizeof(T);
  constexpr int U = 4;
  const int n16 = (int)((size_t)C * HW * sizeof(T) / 16);
  const int4* s = reinterpret_cast<const int4*>(src);
  const int stride = U * blockDim.x * V;                 // elements per outer step
  const int dc = stride / HW, dp = stride - dc * HW;
  int c0 = (threadIdx.x * V) / HW;
  int p0 = threadIdx.x * V - c0 * HW;
  const int ustride = blockDim.x * V;
  const int uc = ustride / HW, up = ustride - uc * HW;
  for (int q0 = threadIdx.x; q0 < n16; q0 += U * blockDim.x) {
    int4 r[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int q = q0 + u * blockDim.x;
      if (q < n16) r[u] = __ldg(s + q);
    }
    int c = c0, p = p0;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int q = q0 + u * blockDim.x;
      if (q < n16) {
        const T* v = reinterpret_cast<const T*>(&r[u]);
        int cc = c, pp = p;
#pragma unroll
        for (int j = 0; j < V; ++j) {
          dst[cc * pe + pp] = v[j];
          if (++pp == HW) {
            pp = 0;
            ++cc;
          }
        }
      }
      c += uc;
      p += up;
      if (p >= HW) {
        p -= HW;
        ++c;
      }
    }
    c0 += dc;
    p0 += dp;
    if (p0 >= HW) {
      p0 -= HW;
      ++c0;
    }
  }
}

// ------------------------------------------------------------------ pass 1
// grid (ncl, B), 256 threads, clusters of ncl CTAs along x: CTA r of a
// sample's cluster takes channels [r per, (r + 1) per), in chunks [c0, c0 +
// cc) that are contiguous in X and are copied flat; z per channel (one
// thread per channel row when rows are short, one warp per row otherwise),
// the residual per pixel by a thread loop over the chunk's uncovered
// channels, the CTAs' partial sums added up by rank 0 through distributed
// shared memory.  (Several CTAs per sample keep the SMs busy at small
// batches.)
template <typename T>
__global__ void __launch_bounds__(256) pool_residual_kernel(const T* __restrict__ x, int C, int HW, int cc, int per,
                                                            const int32_t* __restrict__ mask,
                                                            const int32_t* __restrict__ meta, float* __restrict__ z,
                                                            T* __restrict__ y, int E) {
  extern __shared__ __align__(16) unsigned char s_raw[];
  T* s_x = reinterpret_cast<T*>(s_raw);                                  // cc * HW
  float* s_res = reinterpret_cast<float*>(s_raw + (((size_t)cc * HW * sizeof(T) + 15) & ~size_t(15)));  // HW
  int* s_ulist = reinterpret_cast<int*>(s_res + HW);                    // cc
  __shared__ int s_nu;
  cooperative_groups::cluster_group cluster = cooperative_groups::this_cluster();
  const int b = blockIdx.y, rank = (int)cluster.block_rank(), ncl = (int)cluster.num_blocks();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int n_u = (mask && meta) ? meta[0] : 0;
  const T* xb = x + (size_t)b * C * HW;
  if (n_u > 0)
    for (int p = threadIdx.x; p < HW; p += blockDim.x) s_res[p] = 0.0f;
  const float inv_hw = 1.0f / (float)HW;
  const int c_end = min(C, (rank + 1) * per);
  for (int c0 = rank * per; c0 < c_end; c0 += cc) {
    const int cn = min(cc, c_end - c0);
    const T* src = xb + (size_t)c0 * HW;
    const size_t n = (size_t)cn * HW;
    __syncthreads();
    if ((((uintptr_t)src) | (n * sizeof(T))) % 16 == 0) {
      load_flat(s_x, src, n);
    } else {
#pragma unroll 4
      for (size_t q = threadIdx.x; q < n; q += blockDim.x) s_x[q] = src[q];
    }
    if (threadIdx.x == 0) s_nu = 0;
    __syncthreads();
    if (HW <= 64) {
      for (int c = threadIdx.x; c < cn; c += blockDim.x) {
        const T* row = s_x + (size_t)c * HW;
        float s = 0.0f;
        for (int p = 0; p < HW; ++p) s += to_f(row[p]);
        z[(size_t)b * C + c0 + c] = s * inv_hw;
      }
    } else {
      for (int c = warp; c < cn; c += nw) {
        float s = 0.0f;
        for (int p = lane; p < HW; p += 32) s += to_f(s_x[(size_t)c * HW + p]);
        s = warp_sum(s);
        if (lane == 0) z[(size_t)b * C + c0 + c] = s * inv_hw;
      }
    }
    if (n_u > 0) {
      if (warp == 0) {
        // ordered compaction of the chunk's uncovered channels
        int base = 0;
        for (int c = lane; c - lane < cn; c += 32) {
          const bool u = c < cn && mask[c0 + c] == 1;
          const unsigned bal = __ballot_sync(kFull, u);
          if (u) s_ulist[base + __popc(bal & ((1u << lane) - 1u))] = c;
          base += __popc(bal);
        }
        if (lane == 0) s_nu = base;
      }
      __syncthreads();
      const int nl = s_nu;
      for (int p = threadIdx.x; p < HW; p += blockDim.x) {
        float r = s_res[p];
        for (int j = 0; j < nl; ++j) r += to_f(s_x[(size_t)s_ulist[j] * HW + p]);
        s_res[p] = r;
      }
    }
  }
  __syncthreads();
  if (ncl > 1 && n_u > 0) cluster.sync();                 // every CTA's partial sums are complete
  if (y && rank == 0) {
    T* yr = y + ((size_t)b * E + (E - 1)) * HW;
    for (int p = threadIdx.x; p < HW; p += blockDim.x) {
      float r = 0.0f;
      if (n_u > 0)
        for (int q = 0; q < ncl; ++q) r += q == 0 ? s_res[p] : cluster.map_shared_rank(s_res, q)[p];
      yr[p] = from_f<T>(n_u > 0 ? r / (float)n_u : 0.0f);
    }
  }
  if (ncl > 1 && n_u > 0) cluster.sync();                 // peers' shared memory stays until rank 0 has read it
}

// ------------------------------------------------------------------ pass 2
struct SchedMixArgs {
  const void* x;
  void* y;
  const float* z;
  const float* ln;
  const float* gate_w;
  const float* gate_b;
  const int32_t* group_expert;
  const int32_t* sched;
  float* T_out;
  float tmin_tau, trange_tau;
  int B, C, HW, E_r, k, S, G;
  int TP, pitch_w, n_ptiles, n_gchunks, n_bsplit;
};

constexpr int kYW = 33;                     // staging row pitch in words (odd)

template <typename T>
__device__ __forceinline__ void unpack(uint32_t w, float* v);
template <>
__device__ __forceinline__ void unpack<float>(uint32_t w, float* v) { v[0] = __uint_as_float(w); }
template <>
__device__ __forceinline__ void unpack<__nv_bfloat16>(uint32_t w, float* v) {
  v[0] = __uint_as_float(w << 16);
  v[1] = __uint_as_float(w & 0xffff0000u);
}
template <>
__device__ __forceinline__ void unpack<__half>(uint32_t w, float* v) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
  v[0] = f.x;
  v[1] = f.y;
}

template <typename T>
__device__ __forceinline__ uint32_t pack(const float* v);
template <>
__device__ __forceinline__ uint32_t pack<float>(const float* v) { return __float_as_uint(v[0]); }
template <>
__device__ __forceinline__ uint32_t pack<__nv_bfloat16>(const float* v) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(v[0], v[1]);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack<__half>(const float* v) {
  const __half2 h = __floats2half2_rn(v[0], v[1]);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Two fp32 FMAs with one packed instruction (fma.rn.f32x2, sm_100):
// (a0, a1) += w * (v0, v1), each lane rounded like fmaf.
__device__ __forceinline__ void fma2(float& a0, float& a1, float w, float v0, float v1) {
  asm("{\n\t.reg .b64 ra, rw, rv;\n\t"
      "mov.b64 ra, {%0, %1};\n\t"
      "mov.b64 rw, {%2, %2};\n\t"
      "mov.b64 rv, {%3, %4};\n\t"
      "fma.rn.f32x2 ra, rw, rv, ra;\n\t"
      "mov.b64 {%0, %1}, ra;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(w), "f"(v0), "f"(v1));
}

// grid (n_gchunks * n_bsplit); WPB warps, warp w of chunk q owns schedule
// group q*WPB + w.  S (schedule steps) and PUW (words per lane per inner
// iteration) are compile-time so the step loop unrolls without bounds checks.
template <typename T, int S, int PUW, int WPB>
__global__ void __launch_bounds__(WPB * 32, (S <= 40 ? 2 : 1)) mix_sched_kernel(SchedMixArgs a) {
  constexpr int EPW = 4 / sizeof(T);       // elements per 32-bit word
  constexpr int CHW = PUW * (32 / PUW);    // words per staged chunk
  constexpr int SP = (S + 1) / 2;
  extern __shared__ __align__(16) unsigned char s_raw[];
  const int C = a.C, HW = a.HW, k = a.k, E_r = a.E_r, pitch_w = a.pitch_w;
  uint32_t* s_x = reinterpret_cast<uint32_t*>(s_raw);                  // C * pitch_w (+ PUW slack)
  float* s_z = reinterpret_cast<float*>(s_x + (size_t)C * pitch_w + PUW);
  float* s_gw = s_z + C;
  uint32_t* s_y = reinterpret_cast<uint32_t*>(s_gw + ((k + 3) & ~3));  // WPB * 32 * kYW
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gchunk = blockIdx.x % a.n_gchunks, bsplit = blockIdx.x / a.n_gchunks;
  const int g = gchunk * WPB + warp;
  const bool active = g < a.G;
  const int e = active ? a.group_expert[g * 32 + lane] : -1;
  const int32_t* sch = a.sched + (size_t)(active ? g : 0) * S * 32 + lane;
  uint32_t* ys = s_y + (size_t)(warp * 32) * kYW;

  // word offsets of the channel rows, two 16-bit offsets per register
  uint32_t offp[SP];
  float w[S];
#pragma unroll
  for (int j = 0; j < SP; ++j) offp[j] = 0;
#pragma unroll
  for (int s = 0; s < S; ++s) {
    w[s] = 0.0f;
    const uint32_t o = active ? (((unsigned)sch[s * 32]) & 0xFFFFu) * (uint32_t)pitch_w : 0u;
    offp[s >> 1] |= (s & 1) ? (o << 16) : o;
  }
  for (int i = threadIdx.x; i < k; i += blockDim.x) s_gw[i] = a.gate_w[i];
  const float bias = a.gate_b[0];
  const int E = E_r + 1;
  const int b0 = (int)((long long)bsplit * a.B / a.n_bsplit);
  const int b1 = (int)((long long)(bsplit + 1) * a.B / a.n_bsplit);
  const T* xg = static_cast<const T*>(a.x);
  T* yg = static_cast<T*>(a.y);

  for (int b = b0; b < b1; ++b) {
    const T* xb = xg + (size_t)b * C * HW;
    for (int pt = 0; pt < a.n_ptiles; ++pt) {
      const int p0 = pt * a.TP;
      const int tp = min(a.TP, HW - p0);
      const int nwords = (tp + EPW - 1) / EPW;
      __syncthreads();
      // ---- stage the X tile: row c holds pixels p0 .. p0+tp-1, pitch_w words
      const bool aligned16 = ((((uintptr_t)xb) | ((size_t)C * HW * sizeof(T))) & 15) == 0;
      if (tp == HW && pitch_w * EPW == HW && aligned16) {
        load_flat(reinterpret_cast<T*>(s_x), xb, (size_t)C * HW);
      } else if (tp == HW && aligned16) {
        load_pitched(reinterpret_cast<T*>(s_x), xb, C, HW, pitch_w * EPW);
      } else {
        T* sx = reinterpret_cast<T*>(s_x);
        const int pe = pitch_w * EPW;
        for (int c = warp; c < C; c += WPB) {
          const T* row = xb + (size_t)c * HW + p0;
#pragma unroll 4
          for (int p = lane; p < tp; p += 32) sx[(size_t)c * pe + p] = row[p];
        }
      }
      if (pt == 0)
        for (int c = threadIdx.x; c < C; c += blockDim.x) s_z[c] = a.z[(size_t)b * C + c];
      __syncthreads();
      if (pt == 0 && e >= 0) {
        // ---- gate -> temperature -> softmax weights, per lane (= expert)
        float gs = bias;
        {
          unsigned ent[S];
#pragma unroll
          for (int s = 0; s < S; ++s) ent[s] = (unsigned)__ldg(sch + s * 32);
#pragma unroll
          for (int s = 0; s < S; ++s) {
            const unsigned i = ent[s] >> 16;
            if (i != kIdle) gs += s_gw[i] * s_z[ent[s] & 0xFFFFu];
          }
        }
        const float t = temperature(gs, a.tmin_tau, a.trange_tau, nullptr);
        if (a.T_out) a.T_out[(size_t)b * E_r + e] = t;
        const float it = 1.0f / t;
        const float* lne = a.ln + (size_t)e * k;
        float m = -INFINITY;
#pragma unroll
        for (int s = 0; s < S; ++s) {
          const unsigned i = ((unsigned)__ldg(sch + s * 32)) >> 16;
          w[s] = (i != kIdle) ? __ldg(lne + i) * it : -INFINITY;
        }
#pragma unroll
        for (int s = 0; s < S; ++s) m = nan_max(m, w[s]);
        float zs = 0.0f;
#pragma unroll
        for (int s = 0; s < S; ++s) {
          w[s] = expf(w[s] - m);
          zs += w[s];
        }
        const float iz = 1.0f / zs;
#pragma unroll
        for (int s = 0; s < S; ++s) w[s] *= iz;
      }
      // ---- the mix: chunks of CHW words staged in ys, then rows out
      for (int c0 = 0; c0 < nwords; c0 += CHW) {
        const int cw = min(CHW, nwords - c0);
        for (int q0 = 0; q0 < cw; q0 += PUW) {
          const uint32_t* base = s_x + c0 + q0;
          float acc[PUW * EPW];
#pragma unroll
          for (int u = 0; u < PUW * EPW; ++u) acc[u] = 0.0f;
#pragma unroll
          for (int s = 0; s < S; ++s) {
            const uint32_t o = (s & 1) ? (offp[s >> 1] >> 16) : (offp[s >> 1] & 0xFFFFu);
            const uint32_t* src = base + o;
            uint32_t v[PUW];
#pragma unroll
            for (int u = 0; u < PUW; ++u) v[u] = src[u];
            float f[PUW * EPW];
#pragma unroll
            for (int u = 0; u < PUW; ++u) unpack<T>(v[u], &f[u * EPW]);
#pragma unroll
            for (int h = 0; h + 1 < PUW * EPW; h += 2) fma2(acc[h], acc[h + 1], w[s], f[h], f[h + 1]);
            if ((PUW * EPW) & 1) acc[PUW * EPW - 1] = fmaf(w[s], f[PUW * EPW - 1], acc[PUW * EPW - 1]);
          }
#pragma unroll
          for (int u = 0; u < PUW; ++u)
            if (q0 + u < cw) ys[lane * kYW + q0 + u] = pack<T>(&acc[u * EPW]);
        }
        __syncwarp();
        const int pc0 = c0 * EPW;                          // first pixel of the chunk
        const int pcn = min(cw * EPW, tp - pc0);
        const T* yst = reinterpret_cast<const T*>(ys);
#pragma unroll 4
        for (int r = 0; r < 32; ++r) {
          const int er = __shfl_sync(kFull, e, r);
          if (er >= 0) {
            T* yr = yg + ((size_t)b * E + er) * HW + p0 + pc0;
            for (int q = lane; q < pcn; q += 32) yr[q] = yst[r * kYW * EPW + q];
          }
        }
        __syncwarp();
      }
    }
  }
}

struct SchedPlan {
  int TP, pitch_w, n_ptiles, n_gchunks, n_bsplit, S, PUW;
  size_t smem;
};

template <int WPB>
int plan_sched(int64_t B, int64_t C, int64_t HW, int64_t E_r, int64_t k, size_t esize, SchedPlan* pl) {
  const int EPW = (int)(4 / esize);
  const size_t fixed = (size_t)C * 4 + (size_t)((k + 3) & ~3) * 4 + (size_t)WPB * 32 * kYW * 4 + 8 * 4;
  const size_t budget = 110 * 1024;       // two CTAs per SM
  const size_t hard = 220 * 1024;
  int64_t words = (HW + EPW - 1) / EPW;
  int64_t pw = words | 1;                 // odd pitch: bank = bijection of channel
  size_t need = fixed + (size_t)C * pw * 4;
  int64_t tp = HW;
  if (need > budget) {
    // largest tile (in words, odd pitch) within the budget
    int64_t maxw = (int64_t)((budget > fixed ? budget - fixed : 0) / ((size_t)C * 4));
    if (maxw < 1) maxw = (int64_t)((hard > fixed ? hard - fixed : 0) / ((size_t)C * 4));
    if (maxw < 1) return set_error(MOCE_ERR_UNSUPPORTED, "mix: C=%lld too large for the scheduled kernel", (long long)C);
    pw = (maxw % 2 == 1) ? maxw : maxw - 1;
    if (pw < 1) pw = 1;
    tp = pw * EPW;
    if (tp > HW) tp = HW;
    need = fixed + (size_t)C * pw * 4;
    if (need > hard) return set_error(MOCE_ERR_UNSUPPORTED, "mix: tile does not fit shared memory");
  }
  if ((int64_t)C * pw >= 65536) return set_error(MOCE_ERR_UNSUPPORTED, "mix: tile offsets exceed 16 bits");
  pl->TP = (int)tp;
  pl->pitch_w = (int)pw;
  pl->n_ptiles = (int)((HW + tp - 1) / tp);
  // words per inner iteration: the candidate that wastes the fewest word slots
  const int64_t tw = (tp + EPW - 1) / EPW;
  const int cand[3] = {7, 5, 4};
  int best = 4;
  int64_t best_waste = 1 << 30;
  for (int c : cand) {
    const int64_t chw = c * (32 / c);
    int64_t waste = 0, rem = tw;
    while (rem > 0) {
      const int64_t cw = rem < chw ? rem : chw;
      waste += ((cw + c - 1) / c) * c - cw;
      rem -= cw;
    }
    if (waste < best_waste) {
      best_waste = waste;
      best = c;
    }
  }
  pl->PUW = best;
  const int64_t G = (E_r + 31) / 32;
  pl->n_gchunks = (int)((G + WPB - 1) / WPB);
  pl->S = moce_schedule_steps(k);
  const int per_sm = (need <= budget && pl->S <= 40) ? 2 : 1;
  const int64_t target = (int64_t)per_sm * num_sms();
  int64_t bs = (target + pl->n_gchunks - 1) / pl->n_gchunks;
  if (bs > B) bs = B;
  if (bs < 1) bs = 1;
  pl->n_bsplit = (int)bs;
  pl->smem = need;
  return MOCE_OK;
}

template <typename T, int S, int WPB>
void (*pick_puw(int puw))(SchedMixArgs) {
  switch (puw) {
    case 7: return mix_sched_kernel<T, S, 7, WPB>;
    case 5: return mix_sched_kernel<T, S, 5, WPB>;
    default: return mix_sched_kernel<T, S, 4, WPB>;
  }
}

template <typename T, int WPB>
int launch_sched(const SchedMixArgs& a0, const SchedPlan& pl, cudaStream_t st) {
  SchedMixArgs a = a0;
  a.TP = pl.TP;
  a.pitch_w = pl.pitch_w;
  a.n_ptiles = pl.n_ptiles;
  a.n_gchunks = pl.n_gchunks;
  a.n_bsplit = pl.n_bsplit;
  a.S = pl.S;
  void (*kern)(SchedMixArgs) = nullptr;
  switch (pl.S) {
    case 12: kern = pick_puw<T, 12, WPB>(pl.PUW); break;
    case 20: kern = pick_puw<T, 20, WPB>(pl.PUW); break;
    case 28: kern = pick_puw<T, 28, WPB>(pl.PUW); break;
    case 40: kern = pick_puw<T, 40, WPB>(pl.PUW); break;
    case 52: kern = pick_puw<T, 52, WPB>(pl.PUW); break;
    default: return set_error(MOCE_ERR_UNSUPPORTED, "mix: schedule of %d steps exceeds the register budget", pl.S);
  }
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem) != cudaSuccess)
    return set_error(MOCE_ERR_CUDA, "mix: cannot reserve %zu B shared memory", pl.smem);
  kern<<<(unsigned)(pl.n_gchunks * pl.n_bsplit), WPB * 32, pl.smem, st>>>(a);
  return check_launch("mix_sched_kernel");
}

constexpr int kWPB = 8;

}  // namespace

int sched_supported(int64_t k) { return moce_schedule_steps(k) <= 52; }

}  // namespace moce

using namespace moce;

extern "C" int moce_pool_residual(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const int32_t* mask,
                                  const int32_t* meta, float* z, void* y, int64_t E_r, void* stream) {
  if (B == 0) return MOCE_OK;  // an empty batch is a no-op
  MOCE_REQUIRE(x && z, MOCE_ERR_INVALID, "moce_pool_residual: null pointer argument");
  MOCE_REQUIRE(!y || (mask && meta), MOCE_ERR_INVALID, "moce_pool_residual: the residual needs mask and meta");
  MOCE_REQUIRE(dtype_ok(dtype), MOCE_ERR_INVALID, "moce_pool_residual: unknown dtype %d", dtype);
  MOCE_REQUIRE(B >= 0 && C >= 1 && HW >= 1 && E_r >= 0, MOCE_ERR_INVALID, "moce_pool_residual: invalid shape");
  MOCE_REQUIRE(B < 65536 && C * HW < (int64_t)1 << 31 && HW <= 16384, MOCE_ERR_UNSUPPORTED,
               "moce_pool_residual: shape too large");
  if (B == 0) return MOCE_OK;
  const size_t es = dtype_size(dtype);
  // channel chunk: a multiple of m channels so chunk starts stay 16-byte aligned
  int64_t m = 1;
  while ((m * HW * (int64_t)es) % 16 != 0 && m < 16) m *= 2;
  // CTAs per sample (a cluster): enough for about four CTAs per SM, at most 8
  int64_t ncl = (4LL * num_sms() + B - 1) / B;
  if (ncl > 8) ncl = 8;
  if (ncl < 1) ncl = 1;
  const int64_t per = ((C + ncl - 1) / ncl + m - 1) / m * m;    // channels per CTA
  ncl = (C + per - 1) / per;
  int64_t cc = (int64_t)(96 * 1024 / ((size_t)HW * es));
  cc = (cc / m) * m;
  if (cc < 1) cc = 1;
  if (cc > per) cc = per;
  const size_t smem = (((size_t)cc * HW * es + 15) & ~size_t(15)) + (size_t)HW * 4 + (size_t)cc * 4;
  return dispatch_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(pool_residual_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
      return set_error(MOCE_ERR_CUDA, "moce_pool_residual: smem %zu", smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ncl, (unsigned)B);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)ncl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, pool_residual_kernel<T>, static_cast<const T*>(x), (int)C, (int)HW, (int)cc,
                           (int)per, mask, meta, z, static_cast<T*>(y), (int)(E_r + 1)) != cudaSuccess)
      return check_launch("pool_residual_kernel");
    return check_launch("pool_residual_kernel");
  });
}

extern "C" int moce_mix_scheduled(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const float* z,
                                  const float* ln, int64_t E_r, int64_t k, const int32_t* group_expert,
                                  const int32_t* sched, const float* gate_w, const float* gate_b, float tmin_tau,
                                  float trange_tau, void* y, float* T_out, void* stream) {
  if (B == 0) return MOCE_OK;  // an empty batch is a no-op
  MOCE_REQUIRE(x && z && ln && group_expert && sched && gate_w && gate_b && y, MOCE_ERR_INVALID,
               "moce_mix_scheduled: null pointer argument");
  MOCE_REQUIRE(dtype_ok(dtype), MOCE_ERR_INVALID, "moce_mix_scheduled: unknown dtype %d", dtype);
  MOCE_REQUIRE(B >= 0 && C >= 1 && HW >= 1 && E_r >= 1 && k >= 1 && k <= C, MOCE_ERR_INVALID,
               "moce_mix_scheduled: invalid shape");
  MOCE_REQUIRE(B < 65536 && C * HW < (int64_t)1 << 31 && (E_r + 1) * HW < (int64_t)1 << 31 && C <= 65535,
               MOCE_ERR_UNSUPPORTED, "moce_mix_scheduled: shape too large");
  MOCE_REQUIRE(sched_supported(k), MOCE_ERR_UNSUPPORTED, "moce_mix_scheduled: k=%lld exceeds the scheduled kernel",
               (long long)k);
  if (B == 0) return MOCE_OK;
  SchedPlan pl;
  int rc = plan_sched<kWPB>(B, C, HW, E_r, k, dtype_size(dtype), &pl);
  if (rc) return rc;
  SchedMixArgs a{x, y, z, ln, gate_w, gate_b, group_expert, sched, T_out, tmin_tau, trange_tau,
                 (int)B, (int)C, (int)HW, (int)E_r, (int)k, 0, (int)((E_r + 31) / 32), 0, 0, 0, 0, 0};
  return dispatch_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    return launch_sched<T, kWPB>(a, pl, (cudaStream_t)stream);
  });
}
