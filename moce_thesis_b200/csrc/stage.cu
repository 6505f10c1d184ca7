// Pass 1 of the tensor-core path (16-bit inputs): one read of X
// gives
//   z[b,c]       = mean_p X[b,c,p]                     (MoCE.py:174 / 212)
//   Y[b,E_r,p]   = mean over uncovered channels of X   (MoCE.py:191-196,
//                  0 when every channel is covered      moce_kernel.cu:148-231)
//   xstage[b]    = X_b in the tensor-core operand layout of the mix
// Maps of at most 64 pixels (7x7): each sample is one cluster of kStageCtas
// CTAs, one channel quarter per CTA, so that a sample's loads spread over
// several SMs and many loads are in flight per SM; the per-pixel residual
// sums of the quarters are added up by cluster rank 0 through distributed
// shared memory.  Larger maps (14x14 and up): pool_stage_rows_kernel, a warp
// per channel row and no shared memory (below).
//
// Operand layout (matches the B operand of mix_tc.cu): per sample NT pixel
// tiles of NP pixels (a multiple of 16, at most 256; the last tile shorter),
// each padded to NA = NP / 64 rounded up atoms of 64 pixels, and four
// K-quarters of Kq = Kp / 4 channels, stored
// [tile][quarter][atom][Kq rows][128 bytes]; in row c of atom a of tile t the
// 16-byte unit j holds pixels t NP + 64 a + 8 (j ^ (c & 7)) .. +7 (zero
// beyond the tile or H*W); rows C .. Kp-1 are zero.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace moce {
namespace {

constexpr int kStageCtas = 4;
constexpr int kStageThreads = 256;

template <typename T, bool kTiled>
__global__ void __cluster_dims__(kStageCtas, 1, 1) __launch_bounds__(kStageThreads)
    pool_stage_kernel(const T* __restrict__ x, int C, int HW, int cc, const int32_t* __restrict__ mask,
                      const int32_t* __restrict__ meta, float* __restrict__ z, T* __restrict__ y, int E,
                      int4* __restrict__ xstage, int Kp, int NP, int NT, int NA, OutEpilogue ep) {
  extern __shared__ __align__(16) unsigned char s_raw[];
  T* s_x = reinterpret_cast<T*>(s_raw);                                            // cc x HW
  float* s_res = reinterpret_cast<float*>(s_raw + (((size_t)cc * HW * sizeof(T) + 15) & ~size_t(15)));  // HW
  int* s_ulist = reinterpret_cast<int*>(s_res + ((HW + 3) & ~3));                 // cc
  __shared__ int s_nu;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = blockIdx.x, b = blockIdx.y;
  // a programmatic dependent (the tensor-core mix) may start its prologue
  // once every CTA of this grid is running; it waits for this grid's results
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c0 = rank * cc;
  const int c1 = min(C, c0 + cc);
  const int cn = max(0, c1 - c0);
  const int n_u = (mask && meta) ? meta[0] : 0;
  const T* src = x + ((size_t)b * C + c0) * HW;
  const size_t n = (size_t)cn * HW;

  for (int p = tid; p < HW; p += kStageThreads) s_res[p] = 0.0f;
  if (cn > 0) {
    // contiguous rows c0 .. c1-1: 16-byte loads, eight in flight per thread
    if ((((uintptr_t)src) | (n * sizeof(T))) % 16 == 0) {
      const int4* s4 = reinterpret_cast<const int4*>(src);
      int4* d4 = reinterpret_cast<int4*>(s_x);
      const int n16 = (int)(n * sizeof(T) / 16);
      for (int q0 = tid; q0 < n16; q0 += 8 * kStageThreads) {
        int4 r[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int q = q0 + u * kStageThreads;
          if (q < n16) r[u] = __ldg(s4 + q);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int q = q0 + u * kStageThreads;
          if (q < n16) d4[q] = r[u];
        }
      }
    } else {
#pragma unroll 4
      for (size_t q = tid; q < n; q += kStageThreads) s_x[q] = src[q];
    }
  }
  if (tid == 0) s_nu = 0;
  __syncthreads();
  // z: two threads per channel, one half of the pixels each
  const float inv_hw = 1.0f / (float)HW;
  for (int c = tid >> 1; c - (tid >> 1) < cn; c += kStageThreads / 2) {
    float s = 0.0f;
    if (c < cn)
      for (int p = tid & 1; p < HW; p += 2) s += to_f(s_x[(size_t)c * HW + p]);
    s += __shfl_xor_sync(kFull, s, 1);
    if (c < cn && (tid & 1) == 0) z[(size_t)b * C + c0 + c] = s * inv_hw;
  }
  // residual: partial sums over this quarter's uncovered channels
  if (n_u > 0 && cn > 0) {
    if (warp == 0) {
      int base = 0;
      for (int c = lane; c - lane < cn; c += 32) {
        const bool un = c < cn && mask[c0 + c] == 1;
        const unsigned bal = __ballot_sync(kFull, un);
        if (un) s_ulist[base + __popc(bal & ((1u << lane) - 1u))] = c;
        base += __popc(bal);
      }
      if (lane == 0) s_nu = base;
    }
    __syncthreads();
    const int nl = s_nu;
    for (int p = tid; p < HW; p += kStageThreads) {
      float r = 0.0f;
      for (int j = 0; j < nl; ++j) r += to_f(s_x[(size_t)s_ulist[j] * HW + p]);
      s_res[p] = r;
    }
  }
  // the partial sums are published before the (much larger) operand stores,
  // so that the cluster barrier's release does not wait for those stores
  if (n_u > 0) asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  // operand layout; the CTA holding channel C-1 also writes the zero rows
  {
    int4* xs = xstage + (size_t)b * NT * Kp * NA * 8;
    const int Kq = Kp / 4;
    const int row_end = (cn > 0 && c1 == C) ? Kp : c1;
    const int units = (row_end - c0) * NT * NA * 8;          // 16-byte units: channel, tile, atom, chunk
    for (int q = tid; q < units; q += kStageThreads) {
      const int j = q & 7;
      int at = 0, tl = 0, c = c0 + (q >> 3);
      if constexpr (kTiled) {                                 // (one tile of one atom: no division)
        int rest = q >> 3;
        at = rest % NA;
        rest /= NA;
        tl = rest % NT;
        c = c0 + rest / NT;
      }
      const int pend = min(HW, (tl + 1) * NP);                // end of this tile's pixels
      const int pb = tl * NP + at * 64 + (j ^ (c & 7)) * 8;
      union {
        int4 v;
        T e[8];
      } u;
#pragma unroll
      for (int t = 0; t < 8; ++t)
        u.e[t] = (c < C && pb + t < pend) ? s_x[(size_t)(c - c0) * HW + pb + t] : from_f<T>(0.0f);
      if constexpr (!kTiled)
        xs[(size_t)c * 8 + j] = u.v;                          // [quarter][rows] == [channel rows]
      else
        xs[((((size_t)tl * 4 + c / Kq) * NA + at) * Kq + (c % Kq)) * 8 + j] = u.v;
    }
  }
  // residual row, with the output epilogue of channel E-1 when one is given
  const float esc = ep.scale ? ep.scale[E - 1] : 1.0f, esh = ep.scale ? ep.shift[E - 1] : 0.0f;
  if (n_u > 0) {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (rank == 0 && y) {
      T* yr = y + ((size_t)b * E + (E - 1)) * HW;
      for (int p = tid; p < HW; p += kStageThreads) {
        float r = 0.0f;
        for (int q = 0; q < kStageCtas; ++q) r += cluster.map_shared_rank(s_res, q)[p];
        r = r / (float)n_u;
        yr[p] = from_f<T>(ep.scale ? apply_epilogue(r, esc, esh, ep.relu) : r);
      }
    }
    cluster.sync();                                 // peers' shared memory stays until rank 0 has read it
  } else if (rank == 0 && y) {
    T* yr = y + ((size_t)b * E + (E - 1)) * HW;
    const T zv = from_f<T>(ep.scale ? apply_epilogue(0.0f, esc, esh, ep.relu) : 0.0f);
    for (int p = tid; p < HW; p += kStageThreads) yr[p] = zv;
  }
}

// eight 16-bit values of one 16-byte unit, summed in order
template <typename T>
__device__ __forceinline__ float sum8(const int4& v) {
  union {
    int4 v;
    T e[8];
  } u;
  u.v = v;
  float s = 0.0f;
#pragma unroll
  for (int t = 0; t < 8; ++t) s += to_f(u.e[t]);
  return s;
}

constexpr int kRowsWarps = 8;                 // channels per block of pool_stage_rows_kernel

// Pixels 8u .. 8u+7 of one channel row (zero past H*W) as one 16-byte unit:
// one 16-byte load (VEC 8: H*W % 8 == 0, X 16-byte aligned), two 8-byte
// loads (VEC 4: H*W % 4 == 0, X 8-byte aligned) or element loads.
template <typename T, int VEC>
__device__ __forceinline__ int4 load_chunk(const T* __restrict__ row, int u, int HW) {
  if constexpr (VEC == 8) {
    return __ldg(reinterpret_cast<const int4*>(row) + u);
  } else if constexpr (VEC == 4) {
    const uint2* r2 = reinterpret_cast<const uint2*>(row) + 2 * u;
    const uint2 lo = __ldg(r2);
    const uint2 hi = (8 * u + 4 < HW) ? __ldg(r2 + 1) : make_uint2(0u, 0u);
    return make_int4((int)lo.x, (int)lo.y, (int)hi.x, (int)hi.y);
  } else {
    union {
      int4 v;
      T e[8];
    } w;
#pragma unroll
    for (int t = 0; t < 8; ++t) w.e[t] = (8 * u + t < HW) ? row[8 * u + t] : from_f<T>(0.0f);
    return w.v;
  }
}

// Pass 1 for maps of more than 64 pixels.  Every 8-pixel chunk of a channel
// row is one 16-byte unit of the operand layout, where it only moves to
// position (chunk ^ (c & 7)) of its 128-byte row.  A warp streams one channel
// row of one sample: chunk loads, the same units stored at their
// operand-layout positions (a warp's 32 units fill whole 128-byte rows, so
// stores stay coalesced), and the channel sum accumulated on the way (z,
// MoCE.py:174 / 212).  Rows C..Kp-1 and the pixels past H*W in the last tile
// are written as zeros.  One extra block per sample writes the residual
// expert's row: the mean over the uncovered channels, in ascending channel
// order (MoCE.py:191-196), or zeros.
template <typename T, int VEC>
__global__ void __launch_bounds__(kRowsWarps * 32)
    pool_stage_rows_kernel(const T* __restrict__ x, int C, int HW, const int32_t* __restrict__ mask,
                           const int32_t* __restrict__ meta, float* __restrict__ z, T* __restrict__ y, int E,
                           int4* __restrict__ xstage, int Kp, int NP, int NT, int NA, int nblk_ch,
                           OutEpilogue ep) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nv = (HW + 7) >> 3;                           // chunks of a channel row
  if ((int)blockIdx.x == nblk_ch) {
    if (!y) return;
    const int n_u = (mask && meta) ? meta[0] : 0;
    T* yr = y + ((size_t)b * E + (E - 1)) * HW;
    const T* xb = x + (size_t)b * C * HW;
    for (int q = threadIdx.x; q < nv; q += blockDim.x) {
      float acc[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) acc[t] = 0.0f;
      if (n_u > 0) {
        for (int c = 0; c < C; ++c) {
          if (mask[c] != 1) continue;                     // uniform across the block
          union {
            int4 v;
            T e[8];
          } w;
          w.v = load_chunk<T, VEC>(xb + (size_t)c * HW, q, HW);
#pragma unroll
          for (int t = 0; t < 8; ++t) acc[t] += to_f(w.e[t]);
        }
      }
      union {
        int4 v;
        T e[8];
      } o;
      const float esc = ep.scale ? ep.scale[E - 1] : 1.0f, esh = ep.scale ? ep.shift[E - 1] : 0.0f;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const float r = n_u > 0 ? acc[t] / (float)n_u : 0.0f;
        o.e[t] = from_f<T>(ep.scale ? apply_epilogue(r, esc, esh, ep.relu) : r);
      }
      if constexpr (VEC == 8) {
        reinterpret_cast<int4*>(yr)[q] = o.v;             // Y rows 16-byte aligned (checked by the host)
      } else {
#pragma unroll
        for (int t = 0; t < 8; ++t)
          if (8 * q + t < HW) yr[8 * q + t] = o.e[t];
      }
    }
    return;
  }
  const int c = blockIdx.x * kRowsWarps + warp;
  if (c >= Kp) return;
  const int Kq = Kp >> 2;
  const int npc = NP >> 3;                                // units per pixel tile
  const int nck = NT * npc;                               // units including the last tile's padding
  int4* xs = xstage + (size_t)b * NT * Kp * NA * 8 + ((size_t)(c / Kq) * NA * Kq + (c % Kq)) * 8;
  const size_t tile_units = (size_t)Kp * NA * 8;
  const T* src = x + ((size_t)b * C + (c < C ? c : 0)) * HW;
  const int sw = c & 7;
  const bool real = c < C;
  float s = 0.0f;
  constexpr int U = 4;
  for (int u0 = lane; u0 < nck; u0 += 32 * U) {
    int4 v[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int u = u0 + 32 * j;
      v[j] = make_int4(0, 0, 0, 0);
      if (real && u < nv) v[j] = load_chunk<T, VEC>(src, u, HW);
    }
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int u = u0 + 32 * j;
      if (u < nck) {
        const int t = u / npc, pin = u - t * npc;
        xs[(size_t)t * tile_units + (size_t)(pin >> 3) * Kq * 8 + ((pin & 7) ^ sw)] = v[j];
        s += sum8<T>(v[j]);
      }
    }
  }
  s = warp_sum(s);
  if (real && lane == 0) z[(size_t)b * C + c] = s * (1.0f / (float)HW);
}

}  // namespace

// channels per CTA: a multiple of 8, so that every chunk starts on a 16-byte
// boundary of the sample
int pool_stage_cc(int64_t C) { return (int)(((C + kStageCtas - 1) / kStageCtas + 7) / 8 * 8); }

// shared memory of the per-sample cluster kernel (maps of at most 64 pixels;
// larger maps stream channel rows without shared memory)
size_t pool_stage_smem(int64_t C, int64_t HW) {
  if (HW > 64) return 0;
  const int64_t cc = pool_stage_cc(C);
  return (((size_t)cc * HW * 2 + 15) & ~size_t(15)) + (size_t)((HW + 3) & ~3) * 4 + (size_t)cc * 4;
}

}  // namespace moce

using namespace moce;

namespace moce {
void tc_stage_tiling(int64_t C, int64_t HW, int* NP, int* NT, int* NA);   // mix_tc.cu
int pool_stage_run(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const int32_t* mask,
                   const int32_t* meta, float* z, void* y, int64_t E_r, void* xstage, OutEpilogue ep, void* stream);
}

extern "C" int moce_pool_stage(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const int32_t* mask,
                               const int32_t* meta, float* z, void* y, int64_t E_r, void* xstage, void* stream) {
  return pool_stage_run(x, dtype, B, C, HW, mask, meta, z, y, E_r, xstage, OutEpilogue{nullptr, nullptr, 0},
                        stream);
}

// pass 1 with an optional output epilogue on the residual row
int moce::pool_stage_run(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const int32_t* mask,
                         const int32_t* meta, float* z, void* y, int64_t E_r, void* xstage, OutEpilogue ep,
                         void* stream) {
  if (B == 0) return MOCE_OK;  // an empty batch is a no-op
  MOCE_REQUIRE(x && z && xstage, MOCE_ERR_INVALID, "moce_pool_stage: null pointer argument");
  MOCE_REQUIRE(((uintptr_t)xstage & 15) == 0, MOCE_ERR_INVALID,
               "moce_pool_stage: xstage must be a 16-byte aligned buffer");
  MOCE_REQUIRE(!y || (mask && meta), MOCE_ERR_INVALID, "moce_pool_stage: the residual needs mask and meta");
  MOCE_REQUIRE(dtype == MOCE_BF16 || dtype == MOCE_F16, MOCE_ERR_UNSUPPORTED, "moce_pool_stage: 16-bit inputs only");
  MOCE_REQUIRE(B > 0 && C >= 1 && HW >= 1 && E_r >= 0, MOCE_ERR_INVALID, "moce_pool_stage: invalid shape");
  MOCE_REQUIRE(HW <= 65536, MOCE_ERR_UNSUPPORTED, "moce_pool_stage: H*W too large");
  MOCE_REQUIRE(B < 65536 && C <= 4096, MOCE_ERR_UNSUPPORTED, "moce_pool_stage: shape too large");
  if (HW <= 64) {
    int dev = 0, smem_max = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    MOCE_REQUIRE(pool_stage_smem(C, HW) <= (size_t)smem_max, MOCE_ERR_UNSUPPORTED,
                 "moce_pool_stage: a quarter of the sample exceeds shared memory");
  }
  const int cc = pool_stage_cc(C);
  const size_t smem = pool_stage_smem(C, HW);
  const int Kp = (int)((C + 63) / 64 * 64);
  // pixel tiling of the tensor-core mix
  int NP, NT, NA;
  tc_stage_tiling(C, HW, &NP, &NT, &NA);
  // maps of more than 64 pixels stream channel rows, smaller maps go
  // through the per-sample cluster
  const bool rows = HW > 64;
  const int vec = (HW % 8 == 0 && ((uintptr_t)x & 15) == 0 && (!y || ((uintptr_t)y & 15) == 0)) ? 8
                  : (HW % 4 == 0 && ((uintptr_t)x & 7) == 0) ? 4 : 1;
  return dispatch_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    if constexpr (sizeof(T) != 2) {
      return set_error(MOCE_ERR_UNSUPPORTED, "moce_pool_stage: 16-bit inputs only");
    } else if (rows) {
      const int nblk_ch = (Kp + kRowsWarps - 1) / kRowsWarps;
      const dim3 grid((unsigned)(nblk_ch + 1), (unsigned)B);
      auto kern = vec == 8 ? pool_stage_rows_kernel<T, 8> : vec == 4 ? pool_stage_rows_kernel<T, 4>
                                                                     : pool_stage_rows_kernel<T, 1>;
      kern<<<grid, kRowsWarps * 32, 0, (cudaStream_t)stream>>>(
          static_cast<const T*>(x), (int)C, (int)HW, mask, meta, z, static_cast<T*>(y), (int)(E_r + 1),
          reinterpret_cast<int4*>(xstage), Kp, NP, NT, NA, nblk_ch, ep);
      return check_launch("pool_stage_rows_kernel");
    } else {
      auto kern = (NT * NA > 1) ? pool_stage_kernel<T, true> : pool_stage_kernel<T, false>;
      if (smem > 48 * 1024 &&
          cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return set_error(MOCE_ERR_CUDA, "moce_pool_stage: cannot reserve %zu B shared memory", smem);
      const dim3 grid(kStageCtas, (unsigned)B);
      kern<<<grid, kStageThreads, smem, (cudaStream_t)stream>>>(
          static_cast<const T*>(x), (int)C, (int)HW, cc, mask, meta, z, static_cast<T*>(y), (int)(E_r + 1),
          reinterpret_cast<int4*>(xstage), Kp, NP, NT, NA, ep);
      return check_launch("pool_stage_kernel");
    }
  });
}
