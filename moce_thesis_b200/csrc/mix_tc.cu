// Tensor-core mix for 16-bit inputs (bf16 / fp16) on sm_100a: tcgen05.mma
// with the accumulator in tensor memory.
//
// Per sample b and tile of 128 consecutive routed experts the routed output
// is a dense product
//     Y_b[e, p] = sum_c A_b[e, c] X_b[c, p],   A_b[e, S_ei] = a_bei, 0 elsewhere,
// i.e. the convex gather-mix of MoCE.py:188-189 / moce_kernel.cu:57-141
// written as D[M=128, N=64] = A[128, K=C] B[K=C, N=64] with the pixels padded
// to N = 64 (HW <= 64, e.g. the 7x7 stage-4 maps).  A is 1/16 dense for the
// stage-4 layer; the tensor cores absorb that redundancy far faster than the
// CUDA cores can run the sparse form.
//
// Shared memory operands (canonical UMMA layouts, 128-byte swizzle):
//   A  K-major : K-blocks of 64 channels, 16 KB each = 16 groups of 8 rows x 128 B
//   B  MN-major: 8-channel groups of 1024 B, each channel row = 64 pixels x 2 B
// The CTA owns one expert tile for a range of samples.  The sparsity pattern
// of A is fixed, so A is zeroed once and each sample rewrites only its k
// nonzeros per row.  X_b arrives already in the B layout (pass 1 stages it),
// so the operand moves are plain bulk copies into a ring of K-quarter slots.
//
// An M=128, N=64, K=16 MMA reads 6 KB of operands from shared memory, so the
// loop is bound by shared-memory bandwidth (about 48 cycles per MMA at
// 128 B/clk), and a single issuing thread reaches only about one MMA per 70
// cycles.  Hence two issuers (one per K-half, each into its own partial
// accumulator), A rewritten per K-half as soon as the previous sample's MMAs
// release it, and the staged-X copies running several quarters ahead.
//
// Every wait is bounded in time (%globaltimer): a wait on another role that
// runs out (TcArgs::wait_ns, about one second unless the caller sets it with
// moce_tc_wait_limit_ns) sets g_tc_fault, the roles leave their loops
// together, the copies and MMAs already in flight complete (waits bounded by
// kOwnWaitNs), and the kernel returns after releasing its tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace moce {

__device__ int g_tc_fault = 0;

// Where the first wait that ran out gave up (diagnostics; moce_tc_fault_info):
// [0] set, [1] wait site (TcWaitSite), [2] parity, [3] unit or sample index,
// [4] block, [5] thread, [6] C, [7] H*W, [8] E_r, [9] k, [10] B, [11] pixel
// tiles per sample, [12] MMA N, [13] nanoseconds waited
constexpr int kFaultInfoLen = 14;
__device__ long long g_tc_fault_info[kFaultInfoLen];

namespace {

constexpr int kTcMaxN = 256;              // pixels per MMA (N), padded to 16
// bound of a wait for this thread's own copies or MMAs already in flight,
// which the hardware completes by itself
constexpr uint64_t kOwnWaitNs = 2000000000ull;
constexpr long long kDefaultWaitNs = 1ll << 30;   // about 1.07 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  // start address, leading / stride byte offsets (16-byte units), version 1,
  // base offset 0, 128-byte swizzle (layout type 2 in bits 61..63)
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// kind::f16 instruction descriptor: D fp32, A and B of the same 16-bit type
// (fmt 0 = f16, 1 = bf16), A K-major, B MN-major, N >> 3, M >> 4.
__host__ __device__ constexpr uint32_t umma_idesc(int fmt, int M, int N) {
  return (1u << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | (0u << 15) | (1u << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool mbar_try(uint32_t a, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(a), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait for this thread's own copies or MMAs in flight (bounded by
// kOwnWaitNs); returns false if the bound ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try(a, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try(a, parity)) return true;
    if (global_ns() - t0 > kOwnWaitNs) return false;
  }
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void proxy_fence_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(da), "l"(db), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// byte offset of A[row, c] in the K-major 128B-swizzled layout
__device__ __forceinline__ uint32_t a_off(int row, int c) {
  return (uint32_t)((c >> 6) * 16384 + (row >> 3) * 1024 + (row & 7) * 128 + ((((c & 63) >> 3) ^ (row & 7)) << 4) +
                    ((c & 7) << 1));
}

struct TcArgs {
  const void* xstage;             // [B, Kp, 128 B] operand-layout copy of X (pass 1)
  void* y;
  const float* z;                 // [B, C] pooled means (pass 1), for the Linear(k,1) gate in the weight rows
  const int32_t* idx;
  const float* ln;
  const float* gate_w;
  const float* gate_b;
  float* T_out;                   // [B, E_r] temperatures out, or null
  float tmin_tau, trange_tau;
  const float* T;                 // [B, E_r] temperatures given (kTin: a gate computed before the pass)
  int B, C, HW, E_r, k, Kp;       // Kp: C rounded up to 64
  int n_tiles, n_bsplit;
  int ns;                         // X quarter slots in the ring
  int NP, NA, P;                  // MMA N (pixel tile, a multiple of 16), 64-pixel atoms, partial accumulators
  int NT;                         // pixel tiles per sample (NP pixels each, the last one shorter)
  uint32_t tmem_cols;             // tensor-memory columns allocated (power of 2)
  unsigned long long wait_ns;     // bound of a wait on another role
  int drain;                      // output path, one of the TcDrain values
  int stg_pitch;                  // staging row pitch: elements (kDrainOneTile, kDrainRowsLegacy), bytes (kDrainRows)
  int nsb;                        // staging buffers (kDrainRows)
  uint32_t stage_bytes;           // shared memory of the output staging area
  OutEpilogue ep;                 // caller's folded BatchNorm + ReLU on the outputs (scale null: none)
};

// How the drain moves a finished accumulator to Y.
enum TcDrain {
  kDrainOneTile = 0,              // one pixel tile: the tile's rows are one contiguous range of Y, staged in
                                  // shared memory and written by one bulk copy
  kDrainRows = 1,                 // pixel tiles of 16-byte aligned rows: 16-byte stores into rows padded by
                                  // 16 bytes (conflict-free), one bulk copy per row, `nsb` buffers
  kDrainDirect = 2,               // 16-byte stores from registers straight to Y (when staging does not fit)
  kDrainRowsLegacy = 3,           // other pixel tiles: 16-bit stores into rows of NP elements
  kDrainTma = 4,                  // pixel tiles of a multiple of 64 pixels, 16-byte aligned rows: 64-pixel
                                  // column blocks staged in the 128-byte swizzled layout, each written by
                                  // one TMA tensor store of up to 128 rows (Y as [B][E_r][H*W], so the
                                  // residual row is outside the map)
};

constexpr int kMaxSlots = 8;

// A is written and released in two halves along K, each with a full and a
// free barrier.  With two MMA issuers, kSplitK: issuer h takes K-quarters h
// and h + 2 (one of each half), so that both finish half 0 before half 1 and
// the next sample's half 0 is written while half 1's MMAs run; otherwise
// issuer h takes both quarters of half h.
#ifndef MOCE_TC_SPLITK
#define MOCE_TC_SPLITK 1
#endif
constexpr bool kSplitK = MOCE_TC_SPLITK != 0;
constexpr int kAPieces = 2;

struct TcBars {
  uint64_t full_b[kMaxSlots];     // X quarter landed in the slot (bulk copy, tx bytes)
  uint64_t slot_free[kMaxSlots];  // MMAs reading the slot done
  uint64_t a_full[kAPieces];      // weight rows wrote the A piece (one arrival per weight warp)
  uint64_t a_free[kAPieces];      // MMAs reading the A piece done
  uint64_t d_full[2];             // accumulator buffer complete (one commit per issuer)
  uint64_t d_empty[2];            // accumulator buffer drained (128 arrivals)
  uint64_t fin[2];                // per issuer: every MMA it issued has completed
  uint32_t tmem;
  int abort;
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// One arrival for the whole warp: every lane's preceding writes (ordered for
// the async proxy, or its tensor-memory loads, by the fence the caller ran)
// are covered by the warp barrier, then lane 0 arrives.
__device__ __forceinline__ void mbar_arrive_warp(uint64_t* bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// The waits on another role, by barrier (recorded when one runs out).
enum TcWaitSite {
  kSiteSlotFree = 1,      // producer: a ring slot's MMAs done
  kSiteDEmptySample = 2,  // issuer: accumulator buffer drained (one tile per sample)
  kSiteAFull = 3,         // issuer: weights of a K-quarter written
  kSiteDEmptyTile = 4,    // issuer: accumulator buffer drained (pixel tiles)
  kSiteFullB = 5,         // issuer: staged X quarter landed
  kSiteAFree = 6,         // weight rows: a K-quarter's MMAs of the previous sample done
  kSiteDFull = 7,         // drain: accumulator complete
};

// Wait on another role, bounded by limit_ns; also gives up when another role
// has aborted.  Returns 1 when the phase completed, 0 when another role
// aborted, -1 when this wait ran out (the CTA's abort flag and g_tc_fault
// are then raised).
__device__ __forceinline__ int mbar_wait_peer(uint64_t* bar, uint32_t parity, volatile int* abort, uint64_t limit_ns,
                                              uint64_t* waited) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try(a, parity)) return 1;
  const uint64_t t0 = global_ns();
  uint64_t dt = 0;
  for (;;) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try(a, parity)) return 1;
    if (*abort) return 0;
    dt = global_ns() - t0;
    if (dt > limit_ns) break;
  }
  *abort = 1;
  atomicExch(&g_tc_fault, 1);
  *waited = dt;
  return -1;
}

// Records the first wait that ran out on the device (later ones are dropped).
__device__ __noinline__ void record_tc_fault(int site, int parity, int unit, int C, int HW, int E_r, int k, int B,
                                             int NT, int NP, uint64_t waited) {
  if (atomicCAS(reinterpret_cast<unsigned long long*>(&g_tc_fault_info[0]), 0ull, 1ull) != 0ull) return;
  const long long v[kFaultInfoLen] = {1, site, parity, unit, (long long)blockIdx.x, (long long)threadIdx.x, C, HW,
                                      E_r, k, B, NT, NP, (long long)waited};
  for (int i = 1; i < kFaultInfoLen; ++i) g_tc_fault_info[i] = v[i];
  __threadfence();
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void bulk_s2g(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// every bulk group of this thread but the most recent one has read its source
__device__ __forceinline__ void bulk_wait_read_all_but1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// TMA store of one box of the tensor map from shared memory (box start at
// pixel x, expert y, sample z); the caller commits the bulk group
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Named barrier over the 128 threads of one role that also ANDs a flag, so
// that every thread of the role takes the same branch after a bounded wait.
__device__ __forceinline__ bool role_sync_and(int id, int nthreads, bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)ok), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// 2^x on the MUFU unit (ex2.approx, relative error about 2^-22; results that
// would be subnormal flush to zero).  The weights it feeds are rounded to
// 16 bits right after.
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void st_shared_u16(uint32_t addr, unsigned short v) {
  asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}

template <typename T>
__device__ __forceinline__ unsigned short bits16(T v) {
  static_assert(sizeof(T) == 2, "16-bit element");
  return *reinterpret_cast<const unsigned short*>(&v);
}

// two outputs as one 32-bit word, the first in the low half (lower address)
template <typename T>
__device__ __forceinline__ uint32_t pack2_16(float lo, float hi) {
  return (uint32_t)bits16(from_f<T>(lo)) | ((uint32_t)bits16(from_f<T>(hi)) << 16);
}

// Programmatic dependent launch: wait until the prerequisite grid has
// completed and its memory is visible (returns at once without one).
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void role_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// 32 lanes x 32 bit x 32 columns, no wait (the caller waits once for several).
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

constexpr int kTcThreads = 480;           // 15 warps, roles below
constexpr int kWeightThreads = 256, kDrainThreads = 128;
constexpr int kBarWeights = 1, kBarDrain = 2;
constexpr int kWarpIssuer0 = 12, kWarpProducer = 14;

// Roles (warp-specialized, one CTA per SM):
//   warps 0-7   weight rows: threads 2r and 2r+1 share expert row e0 + r,
//               each with half of its supports (a pair of adjacent lanes
//               combines sums by shuffle); per sample the gate and
//               temperature (MoCE.py:216-218 / 175-178; kTin: T[b, e] read
//               from a gate computed before the pass) and the softmax
//               (MoCE.py:219-221 / 188), written as bf16/fp16 into A one
//               K-half at a time, as soon as the MMAs of the previous sample
//               have released that half
//   warps 8-11  drain: sum of the two partial accumulators (tcgen05.ld),
//               output rows through a shared staging block, one bulk store
//   warp 12, 13 lane 0: MMA issuers, K-half 0 / 1, each into its own partial
//               accumulator (one thread issues a tcgen05.mma only about
//               every 70 cycles, two keep the tensor pipe fed)
//   warp 14     lane 0: producer, bulk copies of the staged X quarters into
//               a ring of `ns` slots, running ahead of the MMAs
// Tensor memory: 2 accumulator buffers x 2 partials x 64 columns.
// kGen: N, atoms, partials and tiles from the arguments; otherwise the 7x7
// stage-4 case (N = 64, one atom, two partials, one tile) as constants.
// kEp: the output epilogue is applied (a separate instantiation: even an
// untaken epilogue branch cost the tiled drain 14 %).
// kW1 (pixel-tiled maps with padded staging rows, k <= 16): one weight
// thread per row (warps 0-3; the weights change once per sample, every NT
// tiles) and eight drain warps (4-11), two per tensor-memory lane quarter,
// each taking one half of a tile's 32-column chunks: the drain of a
// 128 x 256 tile, not the MMAs, sets the pace of these maps.
template <typename T, int KMAX, bool kGen, bool kEp, bool kW1, bool kTin>
__global__ void __launch_bounds__(kTcThreads, 1) mix_tc_kernel(TcArgs a, const __grid_constant__ CUtensorMap tmap_y,
                                                          const __grid_constant__ CUtensorMap tmap_r) {
  constexpr int WT = kW1 ? 128 : kWeightThreads;              // weight threads
  constexpr int DT = kW1 ? 256 : kDrainThreads;               // drain threads
  extern __shared__ unsigned char s_dyn[];
  // 1024-byte aligned operand base, offset from s_dyn so that every pointer
  // below stays in the shared address space (LDS/STS, not generic accesses)
  unsigned char* base = s_dyn + ((1024u - (smem_u32(s_dyn) & 1023u)) & 1023u);
  const int C = a.C, HW = a.HW, k = a.k, Kp = a.Kp, E_r = a.E_r, NS = a.ns;
  const int NP = kGen ? a.NP : 64, NA = kGen ? a.NA : 1, P = kGen ? a.P : 2, NT = kGen ? a.NT : 1;
  const uint32_t sbytes = (uint32_t)Kp * NA * 128;            // one staged (sample, pixel tile)
  const uint32_t qbytes = sbytes / 4;                         // a quarter of the channels, all atoms
  unsigned char* sA = base;                                   // 128 x Kp : Kp * 256 B
  unsigned char* sB = sA + (size_t)Kp * 256;                  // NS quarter slots
  T* stg = reinterpret_cast<T*>(sB + (size_t)NS * qbytes);    // output staging area
  float* s_z = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(stg) + a.stage_bytes);
  float* s_gw = s_z + 2 * Kp;
  TcBars* bars = reinterpret_cast<TcBars*>(s_gw + KMAX);
  volatile int* abort = &bars->abort;
  const uint64_t wlim = a.wait_ns;
  const int Bn = a.B;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // a bounded wait on another role; one that runs out records where
  auto wait_peer = [&](uint64_t* bar, uint32_t parity, int site, int unit) -> bool {
    uint64_t waited = 0;
    const int r = mbar_wait_peer(bar, parity, abort, wlim, &waited);
    if (r < 0) record_tc_fault(site, (int)parity, unit, C, HW, E_r, k, Bn, NT, NP, waited);
    return r > 0;
  };
  const int tile = blockIdx.x % a.n_tiles, bsplit = blockIdx.x / a.n_tiles;
  const int e0 = tile * 128;
  const int rows = min(128, E_r - e0);
  // this CTA's units: [u0, u1) of the B * NT (sample, pixel tile) units of
  // its expert tile, in sample-major order; it touches samples b0 .. b0+nb-1
  // (the first from tile t0 on, the last up to unit u1 - 1), and writes the
  // weights of each sample it touches
  const long long n_units = (long long)a.B * NT;
  const int u0 = (int)(bsplit * n_units / a.n_bsplit), u1 = (int)((bsplit + 1) * n_units / a.n_bsplit);
  const int b0 = u0 / NT, t0 = u0 - (u0 / NT) * NT;
  const int nb = u1 > u0 ? (u1 - 1) / NT - b0 + 1 : 0;
  const int E = E_r + 1;

  // ---- prologue.  The producer initializes the barriers and starts the
  // first X copies, and the weight rows start their register loads, before
  // all threads zero A, so that those latencies overlap the zeroing.
  const unsigned char* xs = static_cast<const unsigned char*>(a.xstage) + (size_t)u0 * sbytes;
  const int nu = u1 - u0;                                     // units (sample, pixel tile) of this CTA
  // X quarter n = 4u + q of unit u goes to a slot of the ring.  With two
  // issuers (P == 2) issuer h consumes its two quarters of every unit (q = h
  // and h + 2, or 2h and 2h + 1; see kSplitK) from a ring of its own (slots
  // [0, NS0) for issuer 0, [NS0, NS) for issuer 1), so that every slot's full
  // barrier has one consumer, which has waited for each earlier phase of it.
  // (A slot shared by the two issuers lets one of them wait for a copy while
  // the slot's previous copy, consumed by the other, is still landing; a
  // parity wait for a phase two ahead of the barrier then passes at once,
  // and the ring's accounting breaks.)
  const int NS0 = (P == 2) ? (NS + 1) / 2 : NS, NS1 = (P == 2) ? NS / 2 : 0;
  auto ring_slot = [&](int n, int& slot, int& use) {
    if (P == 2) {
      const int q = n & 3;
      const int h = kSplitK ? (q & 1) : (q >> 1);             // ring (issuer)
      const int m = 2 * (n >> 2) + (kSplitK ? (q >> 1) : (q & 1));  // copy of that ring
      const int nsh = h ? NS1 : NS0;
      slot = (h ? NS0 : 0) + m % nsh;
      use = m / nsh;
    } else {
      slot = n % NS;
      use = n / NS;
    }
  };
  // the producer warp feeds each ring from a lane of its own (lane r, ring r),
  // so a ring waiting for a slot never holds back the other ring's copies;
  // copy m of ring r is X quarter n = ring_copy(r, m)
  const int n_rings = (P == 2) ? 2 : 1;
  auto ring_copy = [&](int r, int m) -> int {
    if (P != 2) return m;
    return 4 * (m >> 1) + (kSplitK ? r + 2 * (m & 1) : 2 * r + (m & 1));
  };
  const int ring_len = (P == 2) ? 2 * nu : 4 * nu;             // copies per ring
  int m_pre = 0;                                              // copies this lane issued in the prologue
  if (warp == kWarpProducer && lane == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&bars->full_b[s], 1);
      mbar_init(&bars->slot_free[s], 1);
    }
    for (int q = 0; q < kAPieces; ++q) {
      mbar_init(&bars->a_full[q], WT / 32);                    // one arrival per weight warp
      mbar_init(&bars->a_free[q], (P == 2 && kSplitK) ? 2 : 1); // one commit per issuer reading the half
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&bars->d_full[h], P);
      mbar_init(&bars->d_empty[h], DT / 32);                   // one arrival per drain warp
      mbar_init(&bars->fin[h], 1);
    }
    bars->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kWarpProducer) {
    __syncwarp();                                             // the barriers are initialized
    if (lane < n_rings) {
      // staged X comes from pass 1, which may still run when this grid is a
      // programmatic dependent of it (moce_forward_tc); a no-op otherwise
      grid_dep_wait();
      // the leading copies that take a slot's first use need no wait
      for (; m_pre < ring_len; ++m_pre) {
        const int n = ring_copy(lane, m_pre);
        int slot, use;
        ring_slot(n, slot, use);
        if (use > 0) break;
        mbar_expect_tx(&bars->full_b[slot], qbytes);
        bulk_g2s(smem_u32(sB) + (uint32_t)slot * qbytes, xs + (size_t)(n >> 2) * sbytes + (size_t)(n & 3) * qbytes,
                 qbytes, &bars->full_b[slot]);
      }
    }
  }
  // weight rows: threads 2r and 2r+1 share expert row e0 + r, each with KH
  // of its supports (kW1: thread r alone, with all of them)
  constexpr int KH = kW1 ? KMAX : KMAX / 2;
  const int row = kW1 ? tid : tid >> 1, part = kW1 ? 0 : tid & 1;
  const bool w_row = tid < WT && row < rows;
  uint32_t chp[KH];                                           // K-quarter << 30 | channel << 17 | byte offset in A
  float ln2[KH];
  float mx2 = -INFINITY;
  float t_next = 1.0f;                                        // kTin: this row's temperature, one sample ahead
  // !kTin: gate weights of this thread's supports in registers (k <= 32),
  // else read from shared memory per sample; z of the next sample in flight
  constexpr bool kGwReg = KMAX <= 32 && !kTin;
  float gwr[kGwReg ? KH : 1];
  constexpr int ZPT = kTin ? 1 : 512 / WT;                    // z values per weight thread (C <= 512)
  float zr[ZPT];
  if (tid < WT) {
#pragma unroll
    for (int jj = 0; jj < KH; ++jj) {
      const int j = part * KH + jj;
      chp[jj] = 0;
      ln2[jj] = -INFINITY;
      if (j < k && w_row) {
        const size_t o = (size_t)(e0 + row) * k + j;
        const int c = a.idx[o];
        chp[jj] = ((uint32_t)(4 * c / Kp) << 30) | ((uint32_t)c << 17) | a_off(row, c);
        ln2[jj] = a.ln[o] * 1.4426950408889634f;            // log2(e)
        mx2 = nan_max(mx2, ln2[jj]);
      }
      if constexpr (kGwReg) gwr[jj] = (j < k) ? a.gate_w[j] : 0.0f;
    }
    grid_dep_wait();                                          // z or T come from the launch before (see above)
    if constexpr (kTin) {
      if (nb > 0 && w_row) t_next = a.T[(size_t)b0 * E_r + e0 + row];
    } else {
#pragma unroll
      for (int u = 0; u < ZPT; ++u) {
        const int c = tid + u * WT;
        zr[u] = (nb > 0 && c < C) ? a.z[(size_t)b0 * C + c] : 0.0f;
      }
    }
  }
  for (int q = tid; q < Kp * 256 / 16; q += blockDim.x) reinterpret_cast<int4*>(sA)[q] = make_int4(0, 0, 0, 0);
  if constexpr (!kTin)
    for (int i = tid; i < k; i += blockDim.x) s_gw[i] = a.gate_w[i];
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&bars->tmem)),
                 "r"(a.tmem_cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  proxy_fence_smem();                                         // zeroed A visible to the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;

  if (warp == kWarpProducer) {
    // ===================== producer: lane r feeds ring r
    if (lane < n_rings) {
      const uint32_t aB = smem_u32(sB);
      int m = m_pre;
      for (; m < ring_len; ++m) {
        const int n = ring_copy(lane, m);
        int slot, use;
        ring_slot(n, slot, use);
        if (use >= 1 && !wait_peer(&bars->slot_free[slot], (use - 1) & 1, kSiteSlotFree, n)) break;
        mbar_expect_tx(&bars->full_b[slot], qbytes);
        bulk_g2s(aB + (uint32_t)slot * qbytes, xs + (size_t)(n >> 2) * sbytes + (size_t)(n & 3) * qbytes, qbytes,
                 &bars->full_b[slot]);
      }
      // copies still in flight land before the block can exit (no-op on the
      // normal path: the issuers consumed every slot): the most recent use
      // of every slot of this ring
      const int nsh = (P == 2 && lane) ? NS1 : NS0, base = lane ? NS0 : 0;
      for (int j = max(0, m - nsh); j < m; ++j)
        if (!mbar_wait(&bars->full_b[base + j % nsh], (j / nsh) & 1)) atomicExch(&g_tc_fault, 1);
    }
  } else if (warp == kWarpIssuer0 || warp == kWarpIssuer0 + 1) {
    // ===================== MMA issuers.  P == 2: issuer h takes K-half h
    // into partial accumulator h.  P == 1 (wide N, where two buffers of two
    // partials would not fit tensor memory and one thread keeps the
    // longer MMAs fed): issuer 0 takes both halves into one accumulator.
    const int hi = warp - kWarpIssuer0;
    if (lane == 0 && hi < P) {
      const uint32_t idesc = umma_idesc(DTypeOf<T>::value == MOCE_BF16 ? 1 : 0, 128, NP);
      const uint64_t da0 = umma_desc(smem_u32(sA), 16, 1024);
      const uint32_t aB = smem_u32(sB);
      const int kq = Kp / 64;                                 // K-steps (16 channels) per quarter
      // B slot: NA atoms of Kq channel rows x 128 B; atoms Kq * 128 B apart
      // (leading byte offset), 8-row groups 1024 B apart (stride byte offset)
      const uint32_t atom_stride = (uint32_t)(Kp / 4) * 128;
      const int nq = (P == 2) ? 2 : 4;                        // K-quarters of a unit this issuer takes
      bool run = true;
      for (int i = 0; i < nb && run; ++i) {
        // one tile per sample: the accumulator buffer first, as it frees
        // earlier than the next weights
        if (NT == 1 && i >= 2 && !wait_peer(&bars->d_empty[i & 1], ((i - 2) >> 1) & 1, kSiteDEmptySample, i)) break;
        // this sample's tiles in the CTA's range (one tile per sample: the
        // tile, and unit i)
        const int t_beg = (NT == 1 || i > 0) ? 0 : t0;
        const int t_end = (NT == 1 || i < nb - 1) ? NT : u1 - (b0 + i) * NT;
        for (int t = t_beg; t < t_end && run; ++t) {
          const int u = NT == 1 ? i : (b0 + i) * NT + t - u0, s = u & 1;   // unit of this CTA
          if (NT > 1 && u >= 2) {
            if (!wait_peer(&bars->d_empty[s], ((u - 2) >> 1) & 1, kSiteDEmptyTile, u)) {
              run = false;
              break;
            }
            tc_fence_after();
          }
          {
            const uint32_t d = tmem + (uint32_t)(s * P * NP + (P == 2 ? hi : 0) * NP);
            for (int qi = 0; qi < nq; ++qi) {
              const int q = (P == 2) ? (kSplitK ? hi + 2 * qi : 2 * hi + qi) : qi, n = 4 * u + q;
              // the sample's weights of this half of K (before this issuer's
              // first quarter of it, first tile), then the quarter's X
              const int pc = q >> 1;
              const bool pfirst = (P == 2) ? (kSplitK || qi == 0) : (q & 1) == 0;
              const bool plast = (P == 2) ? (kSplitK || qi == 1) : (q & 1) == 1;
              if (t == t_beg && pfirst && !wait_peer(&bars->a_full[pc], i & 1, kSiteAFull, i)) {
                run = false;
                break;
              }
              int slot, use;
              ring_slot(n, slot, use);
              if (!wait_peer(&bars->full_b[slot], use & 1, kSiteFullB, n)) {
                run = false;
                break;
              }
              tc_fence_after();
              const uint64_t db0 = umma_desc(aB + (uint32_t)slot * qbytes, atom_stride, 1024);
              for (int jj = 0; jj < kq; ++jj) {
                const int j = q * kq + jj;                      // K-step over all channels
                // start-address fields advance in 16-byte units (no carry:
                // shared addresses are below 2^18)
                const uint64_t da = da0 + (uint64_t)(((j >> 2) * 16384 + (j & 3) * 32) >> 4);
                const uint64_t db = db0 + (uint64_t)(jj * 128);
                const bool first = qi == 0 && jj == 0;
                umma_f16(d, da, db, idesc, first ? 0u : 1u);
              }
              umma_commit(&bars->slot_free[slot]);
              // the last tile of the sample releases the half's weights
              if (t == t_end - 1 && plast) umma_commit(&bars->a_free[pc]);
            }
          }
          if (!run) break;
          // every tile releases its accumulator buffer
          umma_commit(&bars->d_full[s]);
        }
        if (!run) break;
      }
      // every MMA of this thread completes before the block exits
      umma_commit(&bars->fin[hi]);
      if (!mbar_wait(&bars->fin[hi], 0)) atomicExch(&g_tc_fault, 1);
    }
  } else if (tid < WT) {
    // ===================== weight rows (pairs of threads per row)
    const int e = e0 + row;
    const bool has_row = w_row;
    const uint32_t sAu = smem_u32(sA);
    // the unnormalized weights of the sample stay in registers between the
    // softmax sum and the four quarter writes (k <= 32); for k <= 64 they are
    // recomputed per quarter to stay within the register budget
    constexpr bool kKeepW = KMAX <= 32;
    if constexpr (!kW1) mx2 = nan_max(mx2, __shfl_xor_sync(kFull, mx2, 1));
    const float bias = kTin ? 0.0f : a.gate_b[0];
    bool ok = true;
    for (int i = 0; i < nb; ++i) {
      const int b = b0 + i;
      float t;
      if constexpr (kTin) {
        // the temperature computed before the pass, the next sample's load
        // in flight behind this sample's softmax and stores
        t = t_next;
        if (i + 1 < nb && has_row) t_next = a.T[(size_t)(b + 1) * E_r + e];
      } else {
        // the shared Linear(k,1) gate on the pooled values of this row's
        // supports and the temperature (MoCE.py:216-218 / 175-178)
        float* szb = s_z + (i & 1) * Kp;
#pragma unroll
        for (int u = 0; u < ZPT; ++u)
          if (tid + u * WT < C) szb[tid + u * WT] = zr[u];
        // the weight warps agree here, once per sample, on whether to go on
        // (a warp whose wait ran out below comes here with ok false)
        ok = role_sync_and(kBarWeights, WT, ok);
        if (!ok) break;
        if (i + 1 < nb) {
#pragma unroll
          for (int u = 0; u < ZPT; ++u) {
            const int c = tid + u * WT;
            if (c < C) zr[u] = a.z[(size_t)(b + 1) * C + c];
          }
        }
        float gp = 0.0f;
#pragma unroll
        for (int jj = 0; jj < KH; ++jj)
          if (part * KH + jj < k && has_row) gp += (kGwReg ? gwr[jj] : s_gw[part * KH + jj]) * szb[(chp[jj] >> 17) & 0x1FFu];
        const float g = bias + gp + (kW1 ? 0.0f : __shfl_xor_sync(kFull, gp, 1));
        t = temperature(g, a.tmin_tau, a.trange_tau, nullptr);
        if (a.T_out && has_row && part == 0) a.T_out[(size_t)b * E_r + e] = t;
      }
      const float it = 1.0f / t;
      const float m2 = mx2 * it;
      float wv[kKeepW ? KH : 1];
      float zp = 0.0f;
#pragma unroll
      for (int jj = 0; jj < KH; ++jj) {
        const float ev = ex2_approx(ln2[jj] * it - m2);
        if constexpr (kKeepW) wv[jj] = ev;
        zp += ev;
      }
      const float iz = 1.0f / (zp + (kW1 ? 0.0f : __shfl_xor_sync(kFull, zp, 1)));
      // the halves in order; each warp waits for the previous sample's MMAs
      // of a half by itself and writes it, while the MMAs of the other half
      // run
#pragma unroll
      for (int q = 0; q < kAPieces; ++q) {
        const bool w_ok = i < 1 || wait_peer(&bars->a_free[q], (i - 1) & 1, kSiteAFree, i);
        if (!__all_sync(kFull, w_ok)) {
          ok = false;
          break;
        }
        if (has_row) {
#pragma unroll
          for (int jj = 0; jj < KH; ++jj) {
            if (part * KH + jj < k && (int)(chp[jj] >> 31) == q) {
              float ev;
              if constexpr (kKeepW) ev = wv[jj];
              else ev = ex2_approx(ln2[jj] * it - m2);
              st_shared_u16(sAu + (chp[jj] & 0x1FFFFu), bits16(from_f<T>(ev * iz)));
            }
          }
        }
        proxy_fence_smem();
        mbar_arrive_warp(&bars->a_full[q]);
      }
      if (kTin && !ok) break;                                 // (!kTin: the warps agree above)
    }
  } else if (tid < WT + DT) {
    // ===================== drain (warps 8-11; kW1: 4-11): TMEM lane quarter = warp % 4
    const int dt = (warp & 3) * 32 + lane;                    // row within the tile
    const int dhalf = kW1 ? (warp - 4) >> 2 : 0;              // kW1: which half of the tile's chunks
    const bool dlead = tid == WT;                             // waits for the accumulator
    const bool has_row = dt < rows;
    // output epilogue of this thread's row (expert e0 + dt)
    constexpr bool hep = kEp;
    const float esc = (hep && has_row) ? a.ep.scale[e0 + dt] : 1.0f;
    const float esh = (hep && has_row) ? a.ep.shift[e0 + dt] : 0.0f;
    const int erelu = a.ep.relu;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    T* yg = static_cast<T*>(a.y);
    const int drain = kGen ? a.drain : (int)kDrainOneTile;  // kW1: one tile or padded rows (host)
    if (drain == kDrainOneTile) {
      // One pixel tile per sample: the tile's rows are one contiguous range of
      // Y, staged in shared memory at a pitch of H*W elements with 16-bit
      // stores and written by one bulk copy.  (16-byte, 8-byte or paired
      // 4-byte staging stores, by the rows' alignment, measured slower here:
      // 90.4 against 82.7 us at 7x7, 86 against 69 us at 14x14.)
      for (int u = 0; u < nu; ++u) {
        const int s = u & 1;
        bool ok = true;
        if (dlead) ok = wait_peer(&bars->d_full[s], (u >> 1) & 1, kSiteDFull, u);
        if (dlead) bulk_wait_read();                          // the previous sample's copy left the block
        if (!role_sync_and(kBarDrain, DT, ok)) break;
        tc_fence_after();
        const uint32_t tb = tmem + lane_base + (uint32_t)(s * P * NP);
        // this thread's columns: the whole row, or (kW1) one half of its
        // 32-column chunks
        int c_lo = 0, c_hi = HW;
        if constexpr (kW1) {
          const int mid = min(HW, ((HW + 31) / 32 + 1) / 2 * 32);
          c_lo = dhalf ? mid : 0;
          c_hi = dhalf ? HW : mid;
        }
#pragma unroll
        for (int cb = 0; cb < (kGen ? kTcMaxN : 64); cb += 32) {
          if (cb >= c_hi) break;                              // uniform across the warp
          if (cb < c_lo) continue;
          uint32_t r0[32], r1[32];
          tmem_ld32_nowait(tb + cb, r0);
          if (P == 2) tmem_ld32_nowait(tb + NP + cb, r1);
          tmem_wait_ld();
          if (has_row) {
            float v[32];
#pragma unroll
            for (int p = 0; p < 32; ++p)
              v[p] = (P == 2) ? __uint_as_float(r0[p]) + __uint_as_float(r1[p]) : __uint_as_float(r0[p]);
            if constexpr (hep) {
#pragma unroll
              for (int p = 0; p < 32; ++p) v[p] = apply_epilogue(v[p], esc, esh, erelu);
            }
#pragma unroll
            for (int p = 0; p < 32; ++p)
              if (cb + p < HW) stg[dt * HW + cb + p] = from_f<T>(v[p]);
          }
        }
        tc_fence_before();
        mbar_arrive_warp(&bars->d_empty[s]);
        proxy_fence_smem();
        role_sync(kBarDrain, DT);
        T* dst = yg + ((size_t)(b0 + u) * E + e0) * HW;
        const uint32_t nbytes = (uint32_t)(rows * HW * sizeof(T));
        if (((((uintptr_t)dst) | nbytes) & 15) == 0) {
          if (dlead) bulk_s2g(dst, smem_u32(stg), nbytes);
        } else {
          for (int q = tid - WT; q < rows * HW; q += DT) dst[q] = stg[q];
          role_sync(kBarDrain, DT);
        }
      }
    } else if (drain == kDrainRows || drain == kDrainTma) {
      // Pixel tiles of 16-byte aligned rows; `nsb` staging buffers alternate.
      // kDrainRows: each thread stages its row with 16-byte stores into rows
      // 2 NP + 16 bytes apart (the 16-byte skew puts the 32 rows of a warp's
      // store in distinct bank quads), then copies it out with one bulk copy.
      // (Warp-coalesced row stores in place of the bulk copies measured 249
      // against 228 us at 56x56, C=64.)
      // kDrainTma: the tile is staged as 64-pixel column blocks of 128 rows x
      // 128 bytes in the 128-byte swizzled layout (16-byte unit j of row r at
      // r * 128 + ((j ^ (r & 7)) << 4): a warp's 32 rows fill the banks once
      // per 8 rows), and one thread writes each block with one TMA tensor
      // store; 128 row copies per tile took the drain's time at 56x56.
      const bool tma = drain == kDrainTma;
      const uint32_t pitch = (uint32_t)a.stg_pitch;
      unsigned char* row0 = reinterpret_cast<unsigned char*>(stg) + (size_t)dt * pitch;
      for (int u = 0; u < nu; ++u) {
        const int s = u & 1, ug = u0 + u, i = ug / NT - b0, t = ug - (ug / NT) * NT;
        const int p0 = t * NP, tp = min(NP, HW - p0);       // a multiple of 8
        unsigned char* row = row0 + (size_t)(u % a.nsb) * 128u * pitch;
        unsigned char* blk = reinterpret_cast<unsigned char*>(stg) + (size_t)(u % a.nsb) * (size_t)NP * 256u;
        bool ok = true;
        if (dlead) ok = wait_peer(&bars->d_full[s], (u >> 1) & 1, kSiteDFull, u);
        // this thread's copy out of this buffer, nsb units ago, has read it
        if (a.nsb == 2) bulk_wait_read_all_but1();
        else bulk_wait_read();
        if (!role_sync_and(kBarDrain, DT, ok)) break;
        tc_fence_after();
        const uint32_t tb = tmem + lane_base + (uint32_t)(s * P * NP);
        // 32 columns (two partials when P == 2) into the staging row
        auto put = [&](const uint32_t* ra, const uint32_t* rb, int cb) {
          if (has_row) {
            float v[32];
#pragma unroll
            for (int p = 0; p < 32; ++p)
              v[p] = (P == 2) ? __uint_as_float(ra[p]) + __uint_as_float(rb[p]) : __uint_as_float(ra[p]);
            if constexpr (hep) {
#pragma unroll
              for (int p = 0; p < 32; ++p) v[p] = apply_epilogue(v[p], esc, esh, erelu);
            }
            uint4 q[4];
#pragma unroll
            for (int g = 0; g < 4; ++g)
              q[g] = make_uint4(pack2_16<T>(v[8 * g], v[8 * g + 1]), pack2_16<T>(v[8 * g + 2], v[8 * g + 3]),
                                pack2_16<T>(v[8 * g + 4], v[8 * g + 5]), pack2_16<T>(v[8 * g + 6], v[8 * g + 7]));
            if (tma && (cb >> 6) < (NP >> 6)) {
              // the chunk lies in one 64-pixel block (32-column chunks start
              // on 32-column boundaries)
              unsigned char* b = blk + (size_t)(cb >> 6) * 16384u + (size_t)dt * 128u;
              const int j0 = (cb & 63) >> 3;
#pragma unroll
              for (int g = 0; g < 4; ++g)
                if (cb + 8 * g < tp) *reinterpret_cast<uint4*>(b + (size_t)(((j0 + g) ^ (dt & 7)) << 4)) = q[g];
            } else if (tma) {
              // the tile's last NP % 64 pixels: rows of (NP % 64) * 2 bytes,
              // unswizzled, after the full blocks
              const int full = NP >> 6, rb = (NP & 63) * 2;
              unsigned char* b = blk + (size_t)full * 16384u + (size_t)dt * rb + (size_t)(cb - 64 * full) * 2;
#pragma unroll
              for (int g = 0; g < 4; ++g)
                if (cb + 8 * g < tp) *reinterpret_cast<uint4*>(b + 16 * g) = q[g];
            } else {
#pragma unroll
              for (int g = 0; g < 4; ++g)
                if (cb + 8 * g < tp) *reinterpret_cast<uint4*>(row + (size_t)(cb + 8 * g) * 2) = q[g];
            }
          }
        };
        // this thread's columns: the whole tile, or (kW1) one half of its
        // 32-column chunks (the halves start on 32-column boundaries)
        int c_lo = 0, c_hi = tp;
        if constexpr (kW1) {
          const int mid = min(tp, ((tp + 31) / 32 + 1) / 2 * 32);
          c_lo = dhalf ? mid : 0;
          c_hi = dhalf ? tp : mid;
        }
        if (c_lo >= c_hi) {                                   // nothing to read (uniform across the warp)
          tc_fence_before();
          mbar_arrive_warp(&bars->d_empty[s]);
        } else if (P == 1) {
          // one accumulator: two 32-column chunks in flight (r0 / r1), so
          // each load's latency overlaps the conversion and stores of the
          // chunk before it; the buffer is released after its last load
          uint32_t r0[32], r1[32];
          tmem_ld32_nowait(tb + c_lo, r0);
          tmem_wait_ld();
          for (int cb = c_lo; cb < c_hi; cb += 64) {          // uniform across the warp
            if (cb + 32 < c_hi) {
              tmem_ld32_nowait(tb + cb + 32, r1);
            } else {
              tc_fence_before();
              mbar_arrive_warp(&bars->d_empty[s]);
            }
            put(r0, r0, cb);
            if (cb + 32 >= c_hi) break;
            tmem_wait_ld();
            if (cb + 64 < c_hi) {
              tmem_ld32_nowait(tb + cb + 64, r0);
            } else {
              tc_fence_before();
              mbar_arrive_warp(&bars->d_empty[s]);
            }
            put(r1, r1, cb + 32);
            tmem_wait_ld();
          }
        } else {
          for (int cb = c_lo; cb < c_hi; cb += 32) {          // uniform across the warp
            uint32_t r0[32], r1[32];
            tmem_ld32_nowait(tb + cb, r0);
            tmem_ld32_nowait(tb + NP + cb, r1);
            tmem_wait_ld();
            if (cb + 32 >= c_hi) {                            // last read of the buffer
              tc_fence_before();
              mbar_arrive_warp(&bars->d_empty[s]);
            }
            put(r0, r1, cb);
          }
        }
        if (tma) {
          // every row's blocks written (and visible to the async proxy), then
          // one store per 64-pixel block; pixels past H*W and experts past
          // E_r are outside the map and are not written
          proxy_fence_smem();
          role_sync(kBarDrain, DT);
          if (dlead) {
            const int full = NP >> 6;
            for (int at = 0; at < full && at * 64 < tp; ++at)
              tma_store_3d(&tmap_y, smem_u32(blk) + (uint32_t)at * 16384u, p0 + 64 * at, e0, b0 + i);
            if ((NP & 63) && 64 * full < tp)
              tma_store_3d(&tmap_r, smem_u32(blk) + (uint32_t)full * 16384u, p0 + 64 * full, e0, b0 + i);
            bulk_commit();
          }
        } else if (has_row && c_hi > c_lo) {
          proxy_fence_smem();
          bulk_s2g(yg + ((size_t)(b0 + i) * E + e0 + dt) * HW + p0 + c_lo, smem_u32(row + (size_t)c_lo * 2),
                   (uint32_t)(c_hi - c_lo) * (uint32_t)sizeof(T));
        }
      }
    } else if (drain == kDrainDirect) {
      // pixel tiles of 16-byte aligned rows when no staging buffer fits:
      // 16-byte stores from registers straight to Y
      for (int u = 0; u < nu; ++u) {
        const int s = u & 1, ug = u0 + u, i = ug / NT - b0, t = ug - (ug / NT) * NT;
        const int p0 = t * NP, tp = min(NP, HW - p0);
        bool ok = true;
        if (dlead) ok = wait_peer(&bars->d_full[s], (u >> 1) & 1, kSiteDFull, u);
        if (!role_sync_and(kBarDrain, DT, ok)) break;
        tc_fence_after();
        const uint32_t tb = tmem + lane_base + (uint32_t)(s * P * NP);
        T* dst = yg + ((size_t)(b0 + i) * E + e0 + dt) * HW + p0;
        for (int cb = 0; cb < tp; cb += 32) {                 // uniform across the warp
          uint32_t r0[32], r1[32];
          tmem_ld32_nowait(tb + cb, r0);
          if (P == 2) tmem_ld32_nowait(tb + NP + cb, r1);
          tmem_wait_ld();
          if (cb + 32 >= tp) {                                // last read of the buffer
            tc_fence_before();
            mbar_arrive_warp(&bars->d_empty[s]);
          }
          if (has_row) {
            float v[32];
#pragma unroll
            for (int p = 0; p < 32; ++p)
              v[p] = (P == 2) ? __uint_as_float(r0[p]) + __uint_as_float(r1[p]) : __uint_as_float(r0[p]);
            if constexpr (hep) {
#pragma unroll
              for (int p = 0; p < 32; ++p) v[p] = apply_epilogue(v[p], esc, esh, erelu);
            }
            if (cb + 32 <= tp) {
#pragma unroll
              for (int g = 0; g < 4; ++g) {
                int4 w;
                w.x = (int)pack2_16<T>(v[8 * g + 0], v[8 * g + 1]);
                w.y = (int)pack2_16<T>(v[8 * g + 2], v[8 * g + 3]);
                w.z = (int)pack2_16<T>(v[8 * g + 4], v[8 * g + 5]);
                w.w = (int)pack2_16<T>(v[8 * g + 6], v[8 * g + 7]);
                *reinterpret_cast<int4*>(dst + cb + 8 * g) = w;
              }
            } else {
#pragma unroll
              for (int p = 0; p < 32; ++p)
                if (cb + p < tp) dst[cb + p] = from_f<T>(v[p]);
            }
          }
        }
      }
    } else {
      // other pixel tiles: 16-bit stores into rows of the tile's width, one
      // bulk copy (or element copy) per row
      for (int u = 0; u < nu; ++u) {
        const int s = u & 1, ug = u0 + u, i = ug / NT - b0, t = ug - (ug / NT) * NT;
        const int p0 = t * NP, tp = min(NP, HW - p0);         // this tile's pixels
        bool ok = true;
        if (dlead) ok = wait_peer(&bars->d_full[s], (u >> 1) & 1, kSiteDFull, u);
        bulk_wait_read();                                     // this thread's copy left the staging area
        if (!role_sync_and(kBarDrain, DT, ok)) break;
        tc_fence_after();
        const uint32_t tb = tmem + lane_base + (uint32_t)(s * P * NP);
        for (int cb = 0; cb < tp; cb += 32) {                 // uniform across the warp
          uint32_t r0[32], r1[32];
          tmem_ld32_nowait(tb + cb, r0);
          if (P == 2) tmem_ld32_nowait(tb + NP + cb, r1);
          tmem_wait_ld();
          if (has_row) {
#pragma unroll
            for (int p = 0; p < 32; ++p) {
              float v = (P == 2) ? __uint_as_float(r0[p]) + __uint_as_float(r1[p]) : __uint_as_float(r0[p]);
              if constexpr (hep) v = apply_epilogue(v, esc, esh, erelu);
              if (cb + p < tp) stg[dt * tp + cb + p] = from_f<T>(v);
            }
          }
        }
        tc_fence_before();
        mbar_arrive_warp(&bars->d_empty[s]);
        if (has_row) {
          T* dst = yg + ((size_t)(b0 + i) * E + e0 + dt) * HW + p0;
          const uint32_t nbytes = (uint32_t)(tp * sizeof(T));
          const uint32_t src = smem_u32(stg) + (uint32_t)(dt * tp) * (uint32_t)sizeof(T);
          if (((((uintptr_t)dst) | nbytes | src) & 15) == 0) {
            proxy_fence_smem();
            bulk_s2g(dst, src, nbytes);
          } else {
            for (int p = 0; p < tp; ++p) dst[p] = stg[dt * tp + p];
          }
        }
      }
    }
    bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols));
}

}  // namespace

struct TcShape {
  int Kp, NP, NT, NA, P, KMAX;
  int drain, stg_pitch, nsb;      // output path (TcDrain), staging pitch, staging buffers
  uint32_t stage_bytes;           // shared memory of the output staging area
  uint32_t tmem_cols;
  size_t fixed, qbytes;           // shared memory without the X ring, bytes per ring slot
  int ns;                         // X quarter slots in the ring
};

// pixel tiling: NT tiles of NP pixels (a multiple of 16, at most np_max), the
// last tile shorter
void tc_tiling(int64_t HW, int np_max, int* NP, int* NT, int* NA) {
  const int64_t nt0 = (HW + np_max - 1) / np_max;
  int64_t np = ((HW + nt0 - 1) / nt0 + 15) / 16 * 16;
  if (np > np_max) np = np_max;
  *NP = (int)np;
  *NT = (int)((HW + np - 1) / np);
  *NA = (int)((np + 63) / 64);
}

int smem_optin_tc();

// The driver's tensor-map encoder, looked up once through the runtime (no
// link against the driver library); null when the driver does not offer it.
PFN_cuTensorMapEncodeTiled_v12000 tma_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

// The kernel's shape for (C, H*W, k) and a Y that is (or is not) 16-byte
// aligned: tiling, accumulators, output path and shared-memory plan.
// ns == 0 when the shape does not fit shared memory.
TcShape tc_shape(int64_t C, int64_t HW, int64_t k, bool y_aligned, int np_max) {
  TcShape t;
  t.Kp = (int)((C + 63) / 64 * 64);
  tc_tiling(HW, np_max, &t.NP, &t.NT, &t.NA);
  // the drain reads 32 columns at a time, so the last read of a region whose
  // width is not a multiple of 32 reaches 16 columns past it: allocate that
  const int over = (t.NP % 32) ? 16 : 0;
  t.P = (4 * t.NP + over <= 512) ? 2 : 1;
  uint32_t cols = 32;
  while (cols < (uint32_t)(2 * t.P * t.NP + over)) cols <<= 1;
  t.tmem_cols = cols;
  t.KMAX = k <= 16 ? 16 : k <= 32 ? 32 : 64;
  t.qbytes = (size_t)t.Kp * t.NA * 32;
  const size_t base = 1024 + (size_t)t.Kp * 256 + (size_t)t.Kp * 8 + (size_t)t.KMAX * 4 + sizeof(TcBars);
  const size_t smem_max = (size_t)smem_optin_tc();
  auto slots = [&](size_t stage) -> int {
    const size_t f = base + stage;
    return f < smem_max ? (int)std::min<size_t>((size_t)kMaxSlots, (smem_max - f) / t.qbytes) : 0;
  };
  auto pick = [&](int drain, int pitch, int nsb, size_t stage) {
    t.drain = drain;
    t.stg_pitch = pitch;
    t.nsb = nsb;
    t.stage_bytes = (uint32_t)((stage + 15) & ~size_t(15));
    t.fixed = base + t.stage_bytes;
    t.ns = slots(t.stage_bytes);
  };
  if (t.NT == 1) {
    // one tile: the block is the tile's rows, H*W apart
    pick(kDrainOneTile, (int)HW, 1, (size_t)128 * HW * 2);
  } else if (HW % 8 == 0 && y_aligned) {
    // rows of 16-byte aligned segments: 64-pixel column blocks (and the
    // tile's remaining NP % 64 pixels) for TMA stores, else padded staging
    // rows; two
    // buffers if three ring slots still fit, else one with two slots, else
    // no staging
    const int pitch = 2 * t.NP + 16;
    const size_t one = (size_t)128 * pitch, blocks = (size_t)t.NP * 256;
    const bool tma = tma_encode_fn() != nullptr;
    if (tma && slots(2 * blocks) >= 3) pick(kDrainTma, pitch, 2, 2 * blocks);
    else if (tma && slots(blocks) >= 2) pick(kDrainTma, pitch, 1, blocks);
    else if (slots(2 * one) >= 3) pick(kDrainRows, pitch, 2, 2 * one);
    else if (slots(one) >= 2) pick(kDrainRows, pitch, 1, one);
    else pick(kDrainDirect, 0, 0, 0);
  } else {
    pick(kDrainRowsLegacy, t.NP, 1, (size_t)128 * t.NP * 2);
  }
  return t;
}

// The largest pixel tile (256, 128 or 64 pixels) whose kernel fits shared
// memory with at least three (else two) ring slots, for an aligned and an
// unaligned Y and any k <= 64; 0 if none does.  Wide C (a 128 KB weight tile at C = 512)
// needs the smaller tiles: at 28x28, 208-pixel tiles make 64 KB ring slots.
// The staged layout of pass 1 follows the same choice (tc_stage_tiling).
int tc_np_max(int64_t C, int64_t HW) {
  // first choice: three ring slots for an aligned Y (copies run ahead of the
  // MMAs); else two
  for (int need = 3; need >= 2; --need)
    for (int npm = kTcMaxN; npm >= 64; npm /= 2)
      if (tc_shape(C, HW, 64, true, npm).ns >= need && tc_shape(C, HW, 64, false, npm).ns >= 2) return npm;
  return 0;
}

void tc_stage_tiling(int64_t C, int64_t HW, int* NP, int* NT, int* NA) {
  int npm = tc_np_max(C, HW);
  tc_tiling(HW, npm > 0 ? npm : kTcMaxN, NP, NT, NA);
}

TcShape tc_shape_for(int64_t C, int64_t HW, int64_t k, bool y_aligned) {
  const int npm = tc_np_max(C, HW);
  return tc_shape(C, HW, k, y_aligned, npm > 0 ? npm : kTcMaxN);
}

int smem_optin_tc() {
  int dev = 0, smem_max = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  return smem_max;
}

size_t pool_stage_smem(int64_t C, int64_t HW);   // stage.cu

int tc_supported(int dtype, int64_t C, int64_t HW, int64_t k) {
  if (!(dtype == MOCE_BF16 || dtype == MOCE_F16) || HW < 1 || HW > 65536 || k < 1 || k > 64 || C < 1 || C > 512)
    return 0;
  // the shapes of an aligned and of an unaligned Y both have to fit
  const size_t smem_max = (size_t)smem_optin_tc();
  return (tc_np_max(C, HW) > 0 && tc_shape_for(C, HW, k, true).ns >= 2 && tc_shape_for(C, HW, k, false).ns >= 2 &&
          pool_stage_smem(C, HW) <= smem_max) ? 1 : 0;
}

}  // namespace moce

using namespace moce;

extern "C" int moce_tc_supported(int dtype, int64_t C, int64_t HW, int64_t k) {
  return tc_supported(dtype, C, HW, k);
}

extern "C" size_t moce_tc_stage_bytes(int64_t B, int64_t C, int64_t HW) {
  if (HW < 1) return 0;
  int NP, NT, NA;
  tc_stage_tiling(C, HW, &NP, &NT, &NA);
  return (size_t)B * (size_t)NT * (size_t)((C + 63) / 64 * 64) * (size_t)NA * 128;
}

// Pass 2 with the Linear(k,1) gate computed in the weight rows from z, or
// (T_in given) from temperatures computed before the pass.
struct TcGate {
  const float* z;
  const float* gate_w;
  const float* gate_b;
  float tmin_tau, trange_tau;
  float* T_out;
  const float* T_in;
};

static int mix_tc_launch(const void* xstage, int dtype, int64_t B, int64_t C, int64_t HW, const int32_t* idx,
                         const float* ln, int64_t E_r, int64_t k, TcGate gate, void* y, void* stream, bool dependent,
                         OutEpilogue ep);

// bound of the kernel's waits on another role, taken at each launch
static std::atomic<long long> g_wait_ns{kDefaultWaitNs};

extern "C" int64_t moce_tc_wait_limit_ns(int64_t ns) {
  return (int64_t)(ns > 0 ? g_wait_ns.exchange((long long)ns) : g_wait_ns.load());
}

extern "C" int moce_mix_tc(const void* xstage, int dtype, int64_t B, int64_t C, int64_t HW, const float* z,
                           const int32_t* idx, const float* ln, int64_t E_r, int64_t k, const float* gate_w,
                           const float* gate_b, float tmin_tau, float trange_tau, void* y, float* T_out,
                           void* stream) {
  MOCE_REQUIRE(B == 0 || (z && gate_w && gate_b), MOCE_ERR_INVALID, "moce_mix_tc: null pointer argument");
  return mix_tc_launch(xstage, dtype, B, C, HW, idx, ln, E_r, k,
                       TcGate{z, gate_w, gate_b, tmin_tau, trange_tau, T_out, nullptr}, y, stream, false,
                       OutEpilogue{nullptr, nullptr, 0});
}

extern "C" int moce_mix_tc_t(const void* xstage, int dtype, int64_t B, int64_t C, int64_t HW, const float* T,
                             const int32_t* idx, const float* ln, int64_t E_r, int64_t k, void* y, void* stream) {
  MOCE_REQUIRE(B == 0 || T, MOCE_ERR_INVALID, "moce_mix_tc_t: null T");
  return mix_tc_launch(xstage, dtype, B, C, HW, idx, ln, E_r, k, TcGate{nullptr, nullptr, nullptr, 0.f, 0.f, nullptr, T},
                       y, stream, false, OutEpilogue{nullptr, nullptr, 0});
}

namespace moce {
int pool_stage_run(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const int32_t* mask,
                   const int32_t* meta, float* z, void* y, int64_t E_r, void* xstage, OutEpilogue ep, void* stream);
int temperature_mlp_run(const float* z, int64_t B, int64_t C, int64_t Hd, int64_t E_r, const float* w1,
                        const float* b1, const float* w2, const float* b2, float tmin_tau, float trange_tau,
                        float* h, float* T, void* stream, bool dependent);                    // gate.cu
}

// Pass 1 (pool, residual, operand staging), then pass 2 as a programmatic
// dependent of it: the mix's prologue (A zeroing, tensor-memory allocation,
// route loads) overlaps pass 1's tail, and its reads of z and the staged X
// wait for pass 1's results.
static int forward_tc_run(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const int32_t* mask,
                          const int32_t* meta, const int32_t* idx, const float* ln, int64_t E_r, int64_t k,
                          const float* gate_w, const float* gate_b, float tmin_tau, float trange_tau, float* z,
                          void* xstage, void* y, float* T_out, OutEpilogue ep, void* stream) {
  if (B == 0) return MOCE_OK;
  MOCE_REQUIRE(gate_w && gate_b, MOCE_ERR_INVALID, "moce_forward_tc: null gate");
  int rc = pool_stage_run(x, dtype, B, C, HW, mask, meta, z, y, E_r, xstage, ep, stream);
  if (rc) return rc;
  return mix_tc_launch(xstage, dtype, B, C, HW, idx, ln, E_r, k,
                       TcGate{z, gate_w, gate_b, tmin_tau, trange_tau, T_out, nullptr}, y, stream, true, ep);
}

extern "C" int moce_forward_tc(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const int32_t* mask,
                               const int32_t* meta, const int32_t* idx, const float* ln, int64_t E_r, int64_t k,
                               const float* gate_w, const float* gate_b, float tmin_tau, float trange_tau, float* z,
                               void* xstage, void* y, float* T_out, void* stream) {
  return forward_tc_run(x, dtype, B, C, HW, mask, meta, idx, ln, E_r, k, gate_w, gate_b, tmin_tau, trange_tau, z,
                        xstage, y, T_out, OutEpilogue{nullptr, nullptr, 0}, stream);
}

extern "C" int moce_forward_tc_ep(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const int32_t* mask,
                                  const int32_t* meta, const int32_t* idx, const float* ln, int64_t E_r, int64_t k,
                                  const float* gate_w, const float* gate_b, float tmin_tau, float trange_tau,
                                  const float* out_scale, const float* out_shift, int out_relu, float* z,
                                  void* xstage, void* y, float* T_out, void* stream) {
  MOCE_REQUIRE(out_scale && out_shift, MOCE_ERR_INVALID, "moce_forward_tc_ep: null scale or shift");
  return forward_tc_run(x, dtype, B, C, HW, mask, meta, idx, ln, E_r, k, gate_w, gate_b, tmin_tau, trange_tau, z,
                        xstage, y, T_out, OutEpilogue{out_scale, out_shift, out_relu ? 1 : 0}, stream);
}

// pass 1 -> the two-layer gate's temperatures -> pass 2 from given T, each a
// programmatic dependent of the launch before
extern "C" int moce_forward_tc_mlp(const void* x, int dtype, int64_t B, int64_t C, int64_t HW, const int32_t* mask,
                                   const int32_t* meta, const int32_t* idx, const float* ln, int64_t E_r, int64_t k,
                                   int64_t Hd, const float* w1, const float* b1, const float* w2, const float* b2,
                                   float tmin_tau, float trange_tau, float* z, float* h, void* xstage, void* y,
                                   float* T, void* stream) {
  if (B == 0) return MOCE_OK;
  MOCE_REQUIRE(T, MOCE_ERR_INVALID, "moce_forward_tc_mlp: T (fp32 [B, E_r]) is required");
  int rc = pool_stage_run(x, dtype, B, C, HW, mask, meta, z, y, E_r, xstage, OutEpilogue{nullptr, nullptr, 0},
                          stream);
  if (rc) return rc;
  rc = temperature_mlp_run(z, B, C, Hd, E_r, w1, b1, w2, b2, tmin_tau, trange_tau, h, T, stream, true);
  if (rc) return rc;
  return mix_tc_launch(xstage, dtype, B, C, HW, idx, ln, E_r, k, TcGate{nullptr, nullptr, nullptr, 0.f, 0.f, nullptr, T},
                       y, stream, true, OutEpilogue{nullptr, nullptr, 0});
}

static int mix_tc_launch(const void* xstage, int dtype, int64_t B, int64_t C, int64_t HW, const int32_t* idx,
                         const float* ln, int64_t E_r, int64_t k, TcGate gate, void* y, void* stream, bool dependent,
                         OutEpilogue ep) {
  if (B == 0) return MOCE_OK;
  MOCE_REQUIRE(xstage && idx && ln && y, MOCE_ERR_INVALID, "moce_mix_tc: null pointer argument");
  MOCE_REQUIRE(B > 0 && C >= 1 && HW >= 1 && E_r >= 1 && k >= 1 && k <= C, MOCE_ERR_INVALID,
               "moce_mix_tc: invalid shape");
  MOCE_REQUIRE(tc_supported(dtype, C, HW, k), MOCE_ERR_UNSUPPORTED,
               "moce_mix_tc: needs bf16/fp16, C <= 512, k <= 64 within shared memory");
  MOCE_REQUIRE(((uintptr_t)xstage & 15) == 0, MOCE_ERR_INVALID, "moce_mix_tc: xstage must be 16-byte aligned");
  MOCE_REQUIRE(B < 65536 && (E_r + 1) * HW < (int64_t)1 << 31, MOCE_ERR_UNSUPPORTED, "moce_mix_tc: shape too large");
  const bool tin = gate.T_in != nullptr;
  MOCE_REQUIRE(!tin || ep.scale == nullptr, MOCE_ERR_UNSUPPORTED, "moce_mix_tc: given temperatures take no epilogue");
  const TcShape sh = tc_shape_for(C, HW, k, (((uintptr_t)y) & 15) == 0);
  const int Kp = sh.Kp, KMAX = sh.KMAX;
  const size_t qbytes = sh.qbytes, fixed = sh.fixed;
  const int ns = sh.ns;
  MOCE_REQUIRE(ns >= 2, MOCE_ERR_UNSUPPORTED, "moce_mix_tc: not enough shared memory (%d B)", smem_optin_tc());
  const size_t smem = fixed + (size_t)ns * qbytes;
  const int n_tiles = (int)((E_r + 127) / 128);
  // CTAs per expert tile: one per SM over all tiles, each with a range of
  // (sample, pixel tile) units (a range may start and end inside a sample)
  int n_bsplit = num_sms() / n_tiles;
  if (n_bsplit < 1) n_bsplit = 1;
  if (n_bsplit > B * sh.NT) n_bsplit = (int)(B * sh.NT);
  TcArgs a{xstage, y, gate.z, idx, ln, gate.gate_w, gate.gate_b, gate.T_out, gate.tmin_tau, gate.trange_tau, gate.T_in,
           (int)B, (int)C, (int)HW, (int)E_r, (int)k, Kp, n_tiles, n_bsplit, ns, sh.NP, sh.NA, sh.P, sh.NT,
           sh.tmem_cols, (unsigned long long)g_wait_ns.load(), sh.drain, sh.stg_pitch, sh.nsb, sh.stage_bytes, ep};
  // kDrainTma: Y as [B][E_r][H*W] (the residual row E_r lies outside), boxes
  // of 64 pixels x 128 experts x 1 sample in the 128-byte swizzled layout
  // (tmap_r: the same with boxes of the tile's last NP % 64 pixels, unswizzled)
  CUtensorMap tmap, tmap_r;
  memset(&tmap, 0, sizeof(tmap));
  memset(&tmap_r, 0, sizeof(tmap_r));
  if (sh.drain == kDrainTma) {
    const cuuint64_t dims[3] = {(cuuint64_t)HW, (cuuint64_t)E_r, (cuuint64_t)B};
    const cuuint64_t strides[2] = {(cuuint64_t)HW * 2, (cuuint64_t)(E_r + 1) * (cuuint64_t)HW * 2};
    const cuuint32_t rows = (cuuint32_t)std::min<int64_t>(128, E_r);
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapDataType dt = dtype == MOCE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const cuuint32_t box[3] = {64, rows, 1};
    CUresult r = tma_encode_fn()(&tmap, dt, 3, y, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                 CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r == CUDA_SUCCESS && (sh.NP & 63)) {
      const cuuint32_t box_r[3] = {(cuuint32_t)(sh.NP & 63), rows, 1};
      r = tma_encode_fn()(&tmap_r, dt, 3, y, dims, strides, box_r, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    MOCE_REQUIRE(r == CUDA_SUCCESS, MOCE_ERR_CUDA, "moce_mix_tc: cannot encode the output tensor map (%d)", (int)r);
  }
  return dispatch_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    if constexpr (sizeof(T) != 2) {
      return set_error(MOCE_ERR_UNSUPPORTED, "moce_mix_tc: 16-bit inputs only");
    } else {
      const bool gen = !(sh.NP == 64 && sh.NA == 1 && sh.P == 2 && sh.NT == 1 && sh.drain == kDrainOneTile);
      const bool epi = ep.scale != nullptr;
#define MOCE_TC_KMAX(G, EP, TI)                                                                         \
  (KMAX == 16 ? mix_tc_kernel<T, 16, G, EP, false, TI>                                                 \
              : KMAX == 32 ? mix_tc_kernel<T, 32, G, EP, false, TI> : mix_tc_kernel<T, 64, G, EP, false, TI>)
      // pixel-tiled maps with padded staging rows and k <= 16: one weight
      // thread per row and eight drain warps (with one tile per sample the
      // weights are rewritten every unit and the split measured slower:
      // 74.7 against 68.6 us at 14x14)
      const bool w1 = gen && (sh.drain == kDrainRows || sh.drain == kDrainTma) && KMAX == 16;
      void (*kern)(TcArgs, CUtensorMap, CUtensorMap) = nullptr;
      if (tin) {
        kern = w1 ? mix_tc_kernel<T, 16, true, false, true, true>
                  : gen ? MOCE_TC_KMAX(true, false, true) : MOCE_TC_KMAX(false, false, true);
      } else {
        kern = w1 ? (epi ? mix_tc_kernel<T, 16, true, true, true, false> : mix_tc_kernel<T, 16, true, false, true, false>)
                  : gen ? (epi ? MOCE_TC_KMAX(true, true, false) : MOCE_TC_KMAX(true, false, false))
                        : (epi ? MOCE_TC_KMAX(false, true, false) : MOCE_TC_KMAX(false, false, false));
      }
#undef MOCE_TC_KMAX
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return set_error(MOCE_ERR_CUDA, "moce_mix_tc: cannot reserve %zu B shared memory", smem);
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)(n_tiles * n_bsplit));
      cfg.blockDim = dim3(kTcThreads);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = (cudaStream_t)stream;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = dependent ? 1 : 0;
      if (cudaLaunchKernelEx(&cfg, kern, a, tmap, tmap_r) != cudaSuccess) return check_launch("mix_tc_kernel");
      return check_launch("mix_tc_kernel");
    }
  });
}

extern "C" int moce_tc_fault_info(int64_t* info, int n, int clear) {
  MOCE_REQUIRE(info && n >= 1, MOCE_ERR_INVALID, "moce_tc_fault_info: null pointer");
  long long v[kFaultInfoLen];
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpyFromSymbol(v, g_tc_fault_info, sizeof(v)) != cudaSuccess)
    return set_error(MOCE_ERR_CUDA, "moce_tc_fault_info: read failed");
  for (int i = 0; i < n; ++i) info[i] = i < kFaultInfoLen ? (int64_t)v[i] : 0;
  if (clear) {
    const long long zero[kFaultInfoLen] = {};
    if (cudaMemcpyToSymbol(g_tc_fault_info, zero, sizeof(zero)) != cudaSuccess)
      return set_error(MOCE_ERR_CUDA, "moce_tc_fault_info: clear failed");
  }
  return MOCE_OK;
}

extern "C" int moce_tc_fault(int* flag, int clear) {
  MOCE_REQUIRE(flag, MOCE_ERR_INVALID, "moce_tc_fault: null pointer");
  // every stream's launches (not only the legacy stream's) have finished
  if (cudaDeviceSynchronize() != cudaSuccess) return set_error(MOCE_ERR_CUDA, "moce_tc_fault: synchronize failed");
  if (cudaMemcpyFromSymbol(flag, g_tc_fault, sizeof(int)) != cudaSuccess)
    return set_error(MOCE_ERR_CUDA, "moce_tc_fault: read failed");
  if (clear) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_tc_fault, &zero, sizeof(int)) != cudaSuccess)
      return set_error(MOCE_ERR_CUDA, "moce_tc_fault: clear failed");
  }
  return MOCE_OK;
}
