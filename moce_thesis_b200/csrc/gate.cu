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
// temp_linear_kernel: a CTA owns a tile of 128 experts and a group of up to
// 8 samples; threads 2r and 2r+1 hold half of row r's supports and gate
// weights in registers, the group's z rows (contiguous) are staged in shared
// memory in one coalesced pass, then each thread pair gathers its row's
// inputs for every sample of the group.
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

template <int KH>
__global__ void __launch_bounds__(kGateThreads) temp_linear_kernel(
    const float* __restrict__ z, int B, int C, const int32_t* __restrict__ idx, int E_r, int k,
    const float* __restrict__ gate_w, const float* __restrict__ gate_b, float tmin_tau, float trange_tau,
    float* __restrict__ T, int n_tiles, int spb) {
  extern __shared__ float s_zb[];                          // spb x C: z of this CTA's samples
  grid_dep_launch();                                       // the mix may start its prologue
  const int tid = threadIdx.x, row = tid >> 1, part = tid & 1;
  const int tile = blockIdx.x % n_tiles, grp = blockIdx.x / n_tiles;
  const int e = tile * kGateRows + row;
  const bool has = e < E_r;
  const int b0 = grp * spb, nb = min(spb, B - b0);
  int ch[KH];
  float w[KH];
#pragma unroll
  for (int j = 0; j < KH; ++j) {
    const int i = part * KH + j;
    ch[j] = 0;
    w[j] = 0.0f;
    if (has && i < k) {
      ch[j] = idx[(size_t)e * k + i];
      w[j] = gate_w[i];
    }
  }
  const float bias = gate_b[0];
  grid_dep_wait();                                         // z comes from pass 1
  // the samples' z rows are contiguous: one coalesced copy, many loads in flight
  const int n = nb * C;
  const float* zs = z + (size_t)b0 * C;
#pragma unroll 4
  for (int q = tid; q < n; q += kGateThreads) s_zb[q] = zs[q];
  __syncthreads();
  for (int s = 0; s < nb; ++s) {
    const float* zc = s_zb + s * C;
    float g = 0.0f;
#pragma unroll
    for (int j = 0; j < KH; ++j) g += w[j] * zc[ch[j]];
    g += __shfl_xor_sync(kFull, g, 1);
    if (has && part == 0) T[(size_t)(b0 + s) * E_r + e] = temperature(g + bias, tmin_tau, trange_tau, nullptr);
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
  MOCE_REQUIRE(k <= 128, MOCE_ERR_UNSUPPORTED, "moce_temperature: k <= 128");
  MOCE_REQUIRE(B * E_r < ((int64_t)1 << 40) && C * 4 <= 200 * 1024, MOCE_ERR_UNSUPPORTED,
               "moce_temperature: shape too large");
  int n_tiles, spb, n_groups;
  gate_grid(B, E_r, C, &n_tiles, &spb, &n_groups);
  const dim3 grid((unsigned)(n_tiles * n_groups)), block(kGateThreads);
  const size_t smem = (size_t)spb * C * 4;
  cudaStream_t st = (cudaStream_t)stream;
  const int ki = (int)k, Ci = (int)C, Ei = (int)E_r, Bi = (int)B;
  if (k <= 16)
    return launch_pdl(temp_linear_kernel<8>, grid, block, smem, st, dependent, "temp_linear_kernel", z, Bi, Ci, idx,
                      Ei, ki, gate_w, gate_b, tmin_tau, trange_tau, T, n_tiles, spb);
  if (k <= 32)
    return launch_pdl(temp_linear_kernel<16>, grid, block, smem, st, dependent, "temp_linear_kernel", z, Bi, Ci,
                      idx, Ei, ki, gate_w, gate_b, tmin_tau, trange_tau, T, n_tiles, spb);
  if (k <= 64)
    return launch_pdl(temp_linear_kernel<32>, grid, block, smem, st, dependent, "temp_linear_kernel", z, Bi, Ci,
                      idx, Ei, ki, gate_w, gate_b, tmin_tau, trange_tau, T, n_tiles, spb);
  return launch_pdl(temp_linear_kernel<64>, grid, block, smem, st, dependent, "temp_linear_kernel", z, Bi, Ci, idx,
                    Ei, ki, gate_w, gate_b, tmin_tau, trange_tau, T, n_tiles, spb);
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
