// Support schedule for the lanes-by-experts mix kernel.
//
// In the mix kernel each lane of a warp owns one routed expert and walks its
// k supports; at step s every lane reads X[c_s][p] from a shared-memory tile
// whose row pitch (in 32-bit words) is odd, so the bank of that read is a
// bijection of (c_s mod 32).  The schedule orders each lane's supports so
// that, step by step, the 32 lanes of a warp hit 32 different banks -- one
// shared-memory wavefront per step instead of ~3.5 for random supports.
//
// 1. group_kernel (optional "balance"): assigns experts to warps (groups of
//    32) greedily, each expert to the group whose per-bank support count
//    stays flattest, so every group can be scheduled in ~k steps.
// 2. sched_kernel: per group, S steps; at each step lanes (most remaining
//    supports first) take a support whose bank is still free.  A lane that
//    must place an entry in every remaining step takes one even on a used
//    bank (a conflict costs time, never correctness).  Idle lanes are given
//    a free bank's channel so they do not collide either.
// Entry encoding: (slot i << 16) | channel c; slot 0xFFFF marks an idle step.
#include "common.cuh"

namespace moce {
namespace {

constexpr int kIdleSlot = 0xFFFF;

__global__ void identity_group_kernel(int E_r, int G, int32_t* __restrict__ group_expert) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t < G * 32) group_expert[t] = t < E_r ? t : -1;
}

// Single CTA of 1024 threads; thread t evaluates group t (G <= 1024).
__global__ void __launch_bounds__(1024) group_kernel(const int32_t* __restrict__ idx, int E_r, int k, int G,
                                                     int32_t* __restrict__ group_expert) {
  extern __shared__ uint16_t s_gh[];             // [32][G] bank counts per group
  __shared__ int s_hist[32];
  __shared__ unsigned long long s_best[32];
  __shared__ int s_cnt[1024];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  for (int q = t; q < 32 * G; q += blockDim.x) s_gh[q] = 0;
  for (int q = t; q < G; q += blockDim.x) s_cnt[q] = 0;
  for (int q = t; q < G * 32; q += blockDim.x) group_expert[q] = -1;
  __syncthreads();
  for (int e = 0; e < E_r; ++e) {
    if (warp == 0) {
      int h = 0;
      for (int j = 0; j < k; ++j) h += ((idx[(size_t)e * k + j] & 31) == lane);
      s_hist[lane] = h;
    }
    __syncthreads();
    unsigned long long key = ~0ull;
    if (t < G && s_cnt[t] < 32) {
      unsigned mx = 0;
      unsigned long long ss = 0;
      for (int b = 0; b < 32; ++b) {
        const unsigned v = (unsigned)s_gh[b * G + t] + (unsigned)s_hist[b];
        mx = v > mx ? v : mx;
        ss += (unsigned long long)v * v;
      }
      key = ((unsigned long long)mx << 40) | (ss << 10) | (unsigned long long)t;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(kFull, key, o);
      key = other < key ? other : key;
    }
    if (lane == 0) s_best[warp] = key;
    __syncthreads();
    if (warp == 0) {
      unsigned long long v = s_best[lane];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(kFull, v, o);
        v = other < v ? other : v;
      }
      if (lane == 0) s_best[0] = v;
    }
    __syncthreads();
    const int win = (int)(s_best[0] & 1023ull);
    if (t == win) {
      for (int b = 0; b < 32; ++b) s_gh[b * G + t] = (uint16_t)(s_gh[b * G + t] + s_hist[b]);
      group_expert[t * 32 + s_cnt[t]] = e;
      s_cnt[t] += 1;
    }
    __syncthreads();
  }
}

// Warp per group.  s_rem holds each lane's unplaced supports as entries.
template <int WPB>
__global__ void __launch_bounds__(WPB * 32) sched_kernel(const int32_t* __restrict__ idx, int k, int C, int G, int S,
                                                         const int32_t* __restrict__ group_expert,
                                                         int32_t* __restrict__ sched) {
  extern __shared__ int32_t s_rem_all[];          // WPB * k * 32
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = blockIdx.x * WPB + warp;
  if (g >= G) return;
  int32_t* rem = s_rem_all + (size_t)warp * k * 32;
  const int e = group_expert[g * 32 + lane];
  int cnt = 0;
  if (e >= 0) {
    for (int j = 0; j < k; ++j) rem[j * 32 + lane] = (j << 16) | idx[(size_t)e * k + j];
    cnt = k;
  }
  __syncwarp();
  for (int s = 0; s < S; ++s) {
    // priority rank: more remaining first, then rotating lane order
    int rank = 0;
    const int my_key = cnt * 64 + ((lane - s) & 31);
    for (int o = 0; o < 32; ++o) {
      const int ok = __shfl_sync(kFull, my_key, o);
      rank += (ok > my_key);
    }
    unsigned taken = 0;
    int pick = -1;
    for (int r = 0; r < 32; ++r) {
      const unsigned who = __ballot_sync(kFull, rank == r);
      const int src = __ffs(who) - 1;
      unsigned bit = 0;
      if (lane == src && cnt > 0) {
        const bool forced = cnt >= S - s;
        int j_sel = -1;
        for (int j = 0; j < cnt; ++j) {
          const int c = rem[j * 32 + lane] & 0xFFFF;
          if (!((taken >> (c & 31)) & 1u)) {
            j_sel = j;
            break;
          }
        }
        if (j_sel < 0 && forced) j_sel = 0;
        if (j_sel >= 0) {
          pick = rem[j_sel * 32 + lane];
          rem[j_sel * 32 + lane] = rem[(cnt - 1) * 32 + lane];
          --cnt;
          bit = 1u << ((pick & 0xFFFF) & 31);
        }
      }
      taken |= __shfl_sync(kFull, bit, src < 0 ? 0 : src);
    }
    // idle lanes take distinct free banks
    const unsigned idle = __ballot_sync(kFull, pick < 0);
    if (pick < 0) {
      const int my_idle_rank = __popc(idle & ((1u << lane) - 1u));
      unsigned free_banks = ~taken;
      int bank = 0;
      for (int q = 0; q <= my_idle_rank && free_banks; ++q) {
        bank = __ffs(free_banks) - 1;
        free_banks &= free_banks - 1;
      }
      const int c = C > 0 ? bank % C : 0;
      pick = (int)(((unsigned)kIdleSlot << 16) | (unsigned)c);
    }
    sched[((size_t)g * S + s) * 32 + lane] = pick;
    __syncwarp();
  }
}

}  // namespace
}  // namespace moce

using namespace moce;

// Steps per schedule: k plus slack for bank balancing, rounded up to the
// step counts the mix kernel is compiled for (so its step loop has no
// runtime bound).
extern "C" int moce_schedule_steps(int64_t k) {
  if (k <= 0) return 0;
  const int64_t need = k + (k + 7) / 8 + 2;
  const int64_t buckets[] = {12, 20, 28, 40, 52};
  for (int64_t b : buckets)
    if (need <= b) return (int)b;
  return (int)need;
}

extern "C" int moce_schedule_build(const int32_t* idx, int64_t E_r, int64_t C, int64_t k, int balance,
                                   int32_t* group_expert, int32_t* sched, void* stream) {
  MOCE_REQUIRE(idx && group_expert && sched, MOCE_ERR_INVALID, "moce_schedule_build: null pointer argument");
  MOCE_REQUIRE(E_r >= 1 && C >= 1 && k >= 1 && k <= C, MOCE_ERR_INVALID,
               "moce_schedule_build: invalid shape E_r=%lld C=%lld k=%lld", (long long)E_r, (long long)C,
               (long long)k);
  const int64_t G = (E_r + 31) / 32;
  MOCE_REQUIRE(C <= 65535 && k <= 256 && G <= 1024, MOCE_ERR_UNSUPPORTED,
               "moce_schedule_build: needs C <= 65535, k <= 256, E_r <= 32768");
  // the balancing score packs counts into 64-bit keys; beyond k = 128 use the identity grouping
  if (k > 128) balance = 0;
  const int S = moce_schedule_steps(k);
  cudaStream_t st = (cudaStream_t)stream;
  if (balance) {
    const size_t smem = (size_t)32 * G * 2;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return set_error(MOCE_ERR_CUDA, "moce_schedule_build: group smem");
    group_kernel<<<1, 1024, smem, st>>>(idx, (int)E_r, (int)k, (int)G, group_expert);
  } else {
    identity_group_kernel<<<(unsigned)((G * 32 + 255) / 256), 256, 0, st>>>((int)E_r, (int)G, group_expert);
  }
  int rc = check_launch("moce_schedule_build/group");
  if (rc) return rc;
  constexpr int WPB = 4;
  const size_t smem = (size_t)WPB * k * 32 * 4;
  MOCE_REQUIRE(smem <= 200 * 1024, MOCE_ERR_UNSUPPORTED, "moce_schedule_build: k=%lld too large", (long long)k);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(sched_kernel<WPB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return set_error(MOCE_ERR_CUDA, "moce_schedule_build: sched smem");
  sched_kernel<WPB><<<(unsigned)((G + WPB - 1) / WPB), WPB * 32, smem, st>>>(idx, (int)k, (int)C, (int)G, S,
                                                                               group_expert, sched);
  return check_launch("moce_schedule_build/sched");
}
