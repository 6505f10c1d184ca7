// Route cache build: support selection (top-k), selected-logit normalisation,
// channel coverage and the transposed (channel -> slots) lists.
//
// Reference semantics: MoCE.build_eval_cache (MoCE.py:85-109) and the per-step
// topk/normalisation of MoCE.forward_train (MoCE.py:160, 182-187).
#include "common.cuh"

namespace moce {
namespace {

// Total order on fp32 keys matching torch.topk: NaN above everything,
// -0.0 == +0.0.
__device__ __forceinline__ uint32_t order_key(float f) {
  if (f != f) return 0xffffffffu;
  if (f == 0.0f) f = 0.0f;
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One CTA per expert row.  Rank of element j = #{i : key_i > key_j} +
// #{i < j : key_i == key_j}; elements of rank < k are the support, written at
// their rank (descending logit, ties by ascending channel).  Then one warp
// normalises the k selected logits in double precision.
__global__ void select_kernel(const float* __restrict__ L, int C, int k,
                              int32_t* __restrict__ idx, float* __restrict__ ln) {
  extern __shared__ uint32_t s_key[];          // C keys, then k selected channels
  int32_t* s_sel = reinterpret_cast<int32_t*>(s_key + C);
  const int row = blockIdx.x;
  const float* Lr = L + (size_t)row * C;
  for (int j = threadIdx.x; j < C; j += blockDim.x) s_key[j] = order_key(Lr[j]);
  __syncthreads();
  for (int j = threadIdx.x; j < C; j += blockDim.x) {
    const uint32_t kj = s_key[j];
    int r = 0;
    for (int i = 0; i < C && r < k; ++i) {
      const uint32_t ki = s_key[i];
      r += (ki > kj) | ((ki == kj) & (i < j));
    }
    if (r < k) s_sel[r] = j;
  }
  __syncthreads();
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  double sum = 0.0;
  for (int i = lane; i < k; i += 32) sum += (double)Lr[s_sel[i]];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
  const double mean = sum / (double)k;
  double ss = 0.0;
  for (int i = lane; i < k; i += 32) {
    const double c = (double)Lr[s_sel[i]] - mean;
    ss += c * c;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(kFull, ss, o);
  // unbiased std; k == 1 gives 0/0 = NaN and torch.clamp keeps the NaN
  const double sd = (k > 1) ? sqrt(ss / (double)(k - 1)) : (double)NAN;
  const double scale = (sd != sd) ? sd : (sd < 1.0 ? 1.0 : sd);
  for (int i = lane; i < k; i += 32) {
    const int c = s_sel[i];
    idx[(size_t)row * k + i] = c;
    ln[(size_t)row * k + i] = (float)(((double)Lr[c] - mean) / scale);
  }
}

// Single CTA: per-channel selection counts -> mask, number of uncovered
// channels and (optionally) the CSR offsets of the transposed lists.
__global__ void cover_kernel(const int32_t* __restrict__ idx, int total, int C,
                             int32_t* __restrict__ mask, int32_t* __restrict__ meta,
                             int32_t* __restrict__ toff) {
  extern __shared__ int32_t s_cnt[];           // C counts
  __shared__ int32_t s_part[1024];
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int c = tid; c < C; c += nt) s_cnt[c] = 0;
  __syncthreads();
  for (int s = tid; s < total; s += nt) atomicAdd(&s_cnt[idx[s]], 1);
  __syncthreads();
  // contiguous chunk per thread for the scan
  const int per = (C + nt - 1) / nt;
  const int c0 = min(C, tid * per), c1 = min(C, c0 + per);
  int local = 0, unc = 0;
  for (int c = c0; c < c1; ++c) {
    local += s_cnt[c];
    unc += (s_cnt[c] == 0);
  }
  s_part[tid] = local;
  __syncthreads();
  // Hillis-Steele inclusive scan over the per-thread partials
  for (int off = 1; off < nt; off <<= 1) {
    const int v = (tid >= off) ? s_part[tid - off] : 0;
    __syncthreads();
    s_part[tid] += v;
    __syncthreads();
  }
  int run = s_part[tid] - local;               // exclusive prefix
  for (int c = c0; c < c1; ++c) {
    mask[c] = (s_cnt[c] == 0) ? 1 : 0;
    if (toff) toff[c] = run;
    run += s_cnt[c];
  }
  if (toff && tid == nt - 1) toff[C] = s_part[nt - 1];
  // number of uncovered channels
  unc = warp_sum_i(unc);
  __syncthreads();
  if ((tid & 31) == 0) s_part[tid >> 5] = unc;
  __syncthreads();
  if (tid == 0) {
    int n = 0;
    for (int w = 0; w < nt / 32; ++w) n += s_part[w];
    meta[0] = n;
    meta[1] = 0;
  }
}

// Warp per channel: append, in ascending slot order, every slot s with
// idx[s] == c (ballot compaction keeps the order deterministic).
__global__ void transpose_kernel(const int32_t* __restrict__ idx, int total, int C,
                                 const int32_t* __restrict__ toff, int32_t* __restrict__ tslot) {
  const int lane = threadIdx.x & 31;
  const int c = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (c >= C) return;
  int n = toff[c];
  for (int s0 = 0; s0 < total; s0 += 32) {
    const int s = s0 + lane;
    const bool hit = (s < total) && (idx[s] == c);
    const unsigned bal = __ballot_sync(kFull, hit);
    if (hit) tslot[n + __popc(bal & ((1u << lane) - 1u))] = s;
    n += __popc(bal);
  }
}

}  // namespace
}  // namespace moce

using namespace moce;

extern "C" int moce_route_build(const float* logits, int64_t E_r, int64_t C, int64_t k,
                                int32_t* idx, float* ln, int32_t* mask, int32_t* meta,
                                int32_t* toff, int32_t* tslot, void* stream) {
  MOCE_REQUIRE(logits && idx && ln && mask && meta, MOCE_ERR_INVALID,
               "moce_route_build: null pointer argument");
  MOCE_REQUIRE(E_r >= 1 && C >= 1 && k >= 1 && k <= C, MOCE_ERR_INVALID,
               "moce_route_build: need E_r >= 1, C >= 1, 1 <= k <= C (got E_r=%lld C=%lld k=%lld)",
               (long long)E_r, (long long)C, (long long)k);
  MOCE_REQUIRE((toff == nullptr) == (tslot == nullptr), MOCE_ERR_INVALID,
               "moce_route_build: toff and tslot must both be given or both be NULL");
  MOCE_REQUIRE(C <= 49152 && E_r * k < (int64_t)1 << 31, MOCE_ERR_UNSUPPORTED,
               "moce_route_build: C=%lld or E_r*k too large", (long long)C);
  cudaStream_t st = (cudaStream_t)stream;
  const size_t sel_smem = (size_t)(C + k) * 4;
  if (sel_smem > 48 * 1024) {
    if (cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sel_smem) != cudaSuccess)
      return set_error(MOCE_ERR_UNSUPPORTED, "moce_route_build: C=%lld needs %zu B shared memory", (long long)C, sel_smem);
  }
  select_kernel<<<(unsigned)E_r, 256, sel_smem, st>>>(logits, (int)C, (int)k, idx, ln);
  int rc = check_launch("moce_route_build/select");
  if (rc) return rc;
  const size_t cov_smem = (size_t)C * 4;
  if (cov_smem > 48 * 1024) {
    if (cudaFuncSetAttribute(cover_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cov_smem) != cudaSuccess)
      return set_error(MOCE_ERR_UNSUPPORTED, "moce_route_build: cover smem %zu", cov_smem);
  }
  const int total = (int)(E_r * k);
  cover_kernel<<<1, 1024, cov_smem, st>>>(idx, total, (int)C, mask, meta, toff);
  rc = check_launch("moce_route_build/cover");
  if (rc) return rc;
  if (toff) {
    const int wpb = 8;
    transpose_kernel<<<(unsigned)((C + wpb - 1) / wpb), wpb * 32, 0, st>>>(idx, total, (int)C, toff, tslot);
    rc = check_launch("moce_route_build/transpose");
  }
  return rc;
}
