// Temperature kernels: the per-(sample, expert) temperature T[b, e] from the
// pooled means z [B, C], computed between pass 1 (pool) and pass 2 (mix) so
// that the mix reads one float per expert row and sample instead of
// gathering its gate inputs.
//
// Linear gate (the reference's, MoCE.py:66-68, eval MoCE.py:216-218, train
// MoCE.py:175-178): one Linear(k, 1) shared by all experts, applied to the
// pooled values of the expert's own supports:
//     g[b, e] = gate_w . z[b, S_e] + gate_b;
//     T[b, e] = max(tmin_tau + trange_tau * sigmoid(g), 1e-3)
// temp_linear_kernel: lanes over samples (see the kernel), so the gathers of
// z are conflict-free shared-memory reads.
//
// Two-layer gate (opt-in, no reference counterpart: the two-layer gate of the
// benchmark configurations, C -> C/16 -> E_r with ReLU):
//     h[b, :] = relu(W1 z[b, :] + b1);   g[b, e] = W2[e, :] . h[b, :] + b2[e]
// mlp_hidden_kernel computes h (a warp per sample, W1 through L1), then
// mlp_temp_kernel the logits and temperatures (expert-major, W2 rows in
// registers).  Neither uses the tensor cores: the gate is 3 orders of
// magnitude smaller than the mix.
#include "common.cuh"

namespace moce {
namespace {

constexpr int kGateThreads = 256;
constexpr int kGateRows = 128;                 // experts per CTA (two threads each)

// expert tiles x groups of `spb` samples: each CTA loads its samples' input
// rows in one coalesced pass (no load latency per sample); the group size
// keeps that staging within `smem_cap` bytes and the grid at several CTAs
// per SM
void gate_grid(int64_t B, int64_t E_r, int64_t row_floats, int* n_tiles, int* spb, int* n_groups) {
  *n_tiles = (int)((E_r + kGateRows - 1) / kGateRows);
  int64_t g = 8;
  while (g > 1 && g * row_floats * 4 > 48 * 1024) g /= 2;
  while (g > 1 && *n_tiles * ((B + g - 1) / g) < 4LL * num_sms()) g /= 2;
  *spb = (int)g;
  *n_groups = (int)((B + g - 1) / g);
}

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Linear gate with lanes over samples.  A CTA owns a tile of 32 samples and
// a range of experts.  z of the 32 samples is staged transposed, zt[c][b]
// (row pitch 33 words), so that for one support channel the warp's 32 lanes
// (32 samples) read 32 consecutive banks: one conflict-free wavefront per
// support step.  The expert's supports and gate weights are warp-uniform
// (one load per lane, broadcast by shuffle).  Temperatures of 32 experts x
// 32 samples collect in a shared tile and leave as rows of T [B, E_r].
constexpr int kTs = 32;                        // samples per CTA
constexpr int kTeWarp = 4;                     // experts per warp per round (32 per CTA round of 8 warps)

__global__ void __launch_bounds__(kGateThreads) temp_linear_kernel(
    const float* __restrict__ z, int B, int C, const int32_t* __restrict__ idx, int E_r, int k,
    const float* __restrict__ gate_w, const float* __restrict__ gate_b, float tmin_tau, float trange_tau,
    float* __restrict__ T, int n_stiles, int e_per_cta) {
  extern __shared__ float s_zt[];                          // C x 33: z transposed
  __shared__ float s_t[kTs][33];                           // 32 experts x 32 samples of T
  grid_dep_launch();                                       // the mix may start its prologue
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int st = blockIdx.x % n_stiles, eg = blockIdx.x / n_stiles;
  const int b0 = st * kTs, nb = min(kTs, B - b0);
  const int ea = eg * e_per_cta, eb = min(E_r, ea + e_per_cta);
  const float bias = gate_b[0];
  grid_dep_wait();                                         // z comes from pass 1
  // z[b0 .. b0+nb, :] -> zt[c][b]: consecutive threads take consecutive
  // channels of one sample (coalesced reads, conflict-free writes)
  for (int q = threadIdx.x; q < nb * C; q += kGateThreads) {
    const int bb = q / C, c = q - bb * C;
    s_zt[c * 33 + bb] = z[(size_t)(b0 + bb) * C + c];
  }
  __syncthreads();
  for (int e00 = ea; e00 < eb; e00 += 8 * kTeWarp) {       // rounds of 32 experts
#pragma unroll
    for (int r = 0; r < kTeWarp; ++r) {
      const int el = warp * kTeWarp + r;                   // expert within the round, 0..31
      const int e = e00 + el;
      float g = 0.0f;
      if (e < eb) {                                        // uniform across the warp
        for (int i0 = 0; i0 < k; i0 += 32) {
          const int i = i0 + lane;
          const int c_l = i < k ? idx[(size_t)e * k + i] : 0;
          const float w_l = i < k ? gate_w[i] : 0.0f;
          const int n = min(32, k - i0);
          for (int j = 0; j < n; ++j) {
            const int c = __shfl_sync(kFull, c_l, j);
            const float w = __shfl_sync(kFull, w_l, j);
            g += w * s_zt[c * 33 + lane];
          }
        }
      }
      s_t[el][lane] = temperature(g + bias, tmin_tau, trange_tau, nullptr);
    }
    __syncthreads();
    // rows of T: sample b0 + bb, experts e00 .. e00+31
    for (int q = threadIdx.x; q < kTs * 32; q += kGateThreads) {
      const int bb = q >> 5, el = q & 31;
      if (bb < nb && e00 + el < eb) T[(size_t)(b0 + bb) * E_r + e00 + el] = s_t[el][bb];
    }
    __syncthreads();
  }
}

// h[b, j] = relu(W1[j, :] . z[b, :] + b1[j]); a warp per sample, lanes over C
__global__ void __launch_bounds__(kGateThreads) mlp_hidden_kernel(const float* __restrict__ z, int B, int C, int Hd,
                                                                  const float* __restrict__ w1,
                                                                  const float* __restrict__ b1,
                                                                  float* __restrict__ h) {
  grid_dep_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x * (kGateThreads / 32) + warp;
  grid_dep_wait();
  if (b >= B) return;
  const float* zb = z + (size_t)b * C;
  for (int j = 0; j < Hd; ++j) {
    const float* wr = w1 + (size_t)j * C;
    float s = 0.0f;
    for (int c = lane; c < C; c += 32) s += wr[c] * zb[c];
    s = warp_sum(s) + b1[j];
    if (lane == 0) h[(size_t)b * Hd + j] = s > 0.0f ? s : 0.0f;
  }
}

// g[b, e] = W2[e, :] . h[b, :] + b2[e] -> T; threads 2r, 2r+1 hold half of
// row r of W2 each (HH values), h of a sample is broadcast from shared memory
template <int HH>
__global__ void __launch_bounds__(kGateThreads) mlp_temp_kernel(
    const float* __restrict__ h, int B, int Hd, const float* __restrict__ w2, const float* __restrict__ b2,
    int E_r, float tmin_tau, float trange_tau, float* __restrict__ T, int n_tiles, int spb) {
  extern __shared__ float s_h[];                           // spb x Hd
  grid_dep_launch();
  const int tid = threadIdx.x, row = tid >> 1, part = tid & 1;
  const int tile = blockIdx.x % n_tiles, grp = blockIdx.x / n_tiles;
  const int e = tile * kGateRows + row;
  const bool has = e < E_r;
  const int b0 = grp * spb, nb = min(spb, B - b0);
  float w[HH];
#pragma unroll
  for (int j = 0; j < HH; ++j) {
    const int i = part * HH + j;
    w[j] = (has && i < Hd) ? w2[(size_t)e * Hd + i] : 0.0f;
  }
  const float bias = has ? b2[e] : 0.0f;
  grid_dep_wait();                                         // h comes from mlp_hidden_kernel
  const int n = nb * Hd;
  const float* hs = h + (size_t)b0 * Hd;
#pragma unroll 4
  for (int q = tid; q < n; q += kGateThreads) s_h[q] = hs[q];
  __syncthreads();
  for (int s = 0; s < nb; ++s) {
    const float* hc = s_h + s * Hd;
    float g = 0.0f;
#pragma unroll
    for (int j = 0; j < HH; ++j)
      if (part * HH + j < Hd) g += w[j] * hc[part * HH + j];
    g += __shfl_xor_sync(kFull, g, 1);
    if (has && part == 0) T[(size_t)(b0 + s) * E_r + e] = temperature(g + bias, tmin_tau, trange_tau, nullptr);
  }
}

// Launch with programmatic stream serialization when `dependent` (the
// kernel's griddepcontrol.wait then orders its reads after the previous
// kernel on the stream).
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool dependent,
               const char* what, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = dependent ? 1 : 0;
  if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return set_error(MOCE_ERR_UNSUPPORTED, "%s: %zu B of shared memory not available", what, smem);
  cudaLaunchKernelEx(&cfg, kern, args...);
  return check_launch(what);
}

}  // namespace

// Linear-gate temperatures from pooled means (also used inside the fused
// forward passes, as a programmatic dependent of pass 1 when `dependent`).
int temperature_run(const float* z, int64_t B, int64_t C, const int32_t* idx, int64_t E_r, int64_t k,
                    const float* gate_w, const float* gate_b, float tmin_tau, float trange_tau, float* T,
                    void* stream, bool dependent) {
  if (B == 0) return MOCE_OK;
  MOCE_REQUIRE(z && idx && gate_w && gate_b && T, MOCE_ERR_INVALID, "moce_temperature: null pointer argument");
  MOCE_REQUIRE(B > 0 && C >= 1 && E_r >= 1 && k >= 1 && k <= C, MOCE_ERR_INVALID, "moce_temperature: invalid shape");
  MOCE_REQUIRE(B * E_r < ((int64_t)1 << 40) && E_r * k < ((int64_t)1 << 31), MOCE_ERR_UNSUPPORTED,
               "moce_temperature: shape too large");
  // channels beyond the transposed staging's shared memory: the general gate
  // kernel from the pooled means (a warp per expert row)
  if (C * 33 * 4 > 200 * 1024)
    return moce_gate_temperature(nullptr, MOCE_F32, z, B, C, 1, idx, E_r, k, gate_w, gate_b, tmin_tau, trange_tau,
                                 nullptr, T, stream);
  // 32-sample tiles x expert ranges (multiples of 32): about two CTAs per SM
  const int n_stiles = (int)((B + kTs - 1) / kTs);
  const int64_t rounds = (E_r + 31) / 32;
  int64_t n_eg = (2LL * num_sms() + n_stiles - 1) / n_stiles;
  if (n_eg > rounds) n_eg = rounds;
  if (n_eg < 1) n_eg = 1;
  const int e_per_cta = (int)(((rounds + n_eg - 1) / n_eg) * 32);
  n_eg = (E_r + e_per_cta - 1) / e_per_cta;
  const dim3 grid((unsigned)(n_stiles * n_eg)), block(kGateThreads);
  const size_t smem = (size_t)C * 33 * 4;
  return launch_pdl(temp_linear_kernel, grid, block, smem, (cudaStream_t)stream, dependent, "temp_linear_kernel", z,
                    (int)B, (int)C, idx, (int)E_r, (int)k, gate_w, gate_b, tmin_tau, trange_tau, T, n_stiles,
                    e_per_cta);
}

int temperature_mlp_run(const float* z, int64_t B, int64_t C, int64_t Hd, int64_t E_r, const float* w1,
                        const float* b1, const float* w2, const float* b2, float tmin_tau, float trange_tau,
                        float* h, float* T, void* stream, bool dependent) {
  if (B == 0) return MOCE_OK;
  MOCE_REQUIRE(z && w1 && b1 && w2 && b2 && h && T, MOCE_ERR_INVALID, "moce_temperature_mlp: null pointer argument");
  MOCE_REQUIRE(B > 0 && C >= 1 && Hd >= 1 && E_r >= 1, MOCE_ERR_INVALID, "moce_temperature_mlp: invalid shape");
  MOCE_REQUIRE(Hd <= 256 && B * E_r < ((int64_t)1 << 40) && B * C < ((int64_t)1 << 40), MOCE_ERR_UNSUPPORTED,
               "moce_temperature_mlp: hidden width <= 256");
  cudaStream_t st = (cudaStream_t)stream;
  const int Bi = (int)B, Ci = (int)C, Hi = (int)Hd, Ei = (int)E_r;
  int rc = launch_pdl(mlp_hidden_kernel, dim3((unsigned)((B + 7) / 8)), dim3(kGateThreads), 0, st, dependent,
                      "mlp_hidden_kernel", z, Bi, Ci, Hi, w1, b1, h);
  if (rc) return rc;
  int n_tiles, spb, n_groups;
  gate_grid(B, E_r, Hd, &n_tiles, &spb, &n_groups);
  const dim3 grid((unsigned)(n_tiles * n_groups)), block(kGateThreads);
  const size_t smem = (size_t)spb * Hd * 4;
  if (Hd <= 32)
    return launch_pdl(mlp_temp_kernel<16>, grid, block, smem, st, true, "mlp_temp_kernel", (const float*)h, Bi, Hi,
                      w2, b2, Ei, tmin_tau, trange_tau, T, n_tiles, spb);
  if (Hd <= 64)
    return launch_pdl(mlp_temp_kernel<32>, grid, block, smem, st, true, "mlp_temp_kernel", (const float*)h, Bi, Hi,
                      w2, b2, Ei, tmin_tau, trange_tau, T, n_tiles, spb);
  if (Hd <= 128)
    return launch_pdl(mlp_temp_kernel<64>, grid, block, smem, st, true, "mlp_temp_kernel", (const float*)h, Bi, Hi,
                      w2, b2, Ei, tmin_tau, trange_tau, T, n_tiles, spb);
  return launch_pdl(mlp_temp_kernel<128>, grid, block, smem, st, true, "mlp_temp_kernel", (const float*)h, Bi, Hi,
                    w2, b2, Ei, tmin_tau, trange_tau, T, n_tiles, spb);
}

}  // namespace moce

using namespace moce;

extern "C" int moce_temperature(const float* z, int64_t B, int64_t C, const int32_t* idx, int64_t E_r, int64_t k,
                                const float* gate_w, const float* gate_b, float tmin_tau, float trange_tau, float* T,
                                void* stream) {
  return temperature_run(z, B, C, idx, E_r, k, gate_w, gate_b, tmin_tau, trange_tau, T, stream, false);
}

extern "C" int moce_temperature_mlp(const float* z, int64_t B, int64_t C, int64_t Hd, int64_t E_r, const float* w1,
                                    const float* b1, const float* w2, const float* b2, float tmin_tau,
                                    float trange_tau, float* h, float* T, void* stream) {
  return temperature_mlp_run(z, B, C, Hd, E_r, w1, b1, w2, b2, tmin_tau, trange_tau, h, T, stream, false);
}
