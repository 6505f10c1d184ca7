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
// nonzeros per row.  One thread per expert row computes the gate, the
// temperature and the softmax weights of its expert (MoCE.py:216-221 /
// 175-188) and writes them into A; the warps stage X_b into B; one thread
// issues the MMAs and commits them to an mbarrier; all threads then drain the
// accumulator with tcgen05.ld and write the rows through a shared staging
// block as contiguous stores.
//
// Every wait is bounded: a wait that runs out sets g_tc_fault and the kernel
// returns after releasing its tensor memory.
#include "common.cuh"

namespace moce {

__device__ int g_tc_fault = 0;

namespace {

constexpr int kTcThreads = 128;           // one thread per expert row
constexpr int kTcN = 64;                  // padded pixels
constexpr long long kSpinLimit = 1ll << 28;

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

// Bounded parity wait; returns false if the limit ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  for (long long it = 0; it < kSpinLimit; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
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

// 32 lanes x 32 bit x 64 columns: thread t of warp w gets row 32w + t.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
      "%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
      "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// byte offset of A[row, c] in the K-major 128B-swizzled layout
__device__ __forceinline__ uint32_t a_off(int row, int c) {
  return (uint32_t)((c >> 6) * 16384 + (row >> 3) * 1024 + (row & 7) * 128 + ((((c & 63) >> 3) ^ (row & 7)) << 4) +
                    ((c & 7) << 1));
}

// byte offset of B[c, p] (channel c, pixel p) in the MN-major 128B-swizzled layout
__device__ __forceinline__ uint32_t b_off(int c, int p) {
  return (uint32_t)((c >> 3) * 1024 + (c & 7) * 128 + ((((p >> 3) ^ (c & 7))) << 4) + ((p & 7) << 1));
}

struct TcArgs {
  const void* xstage;             // [B, Kp, 128 B] operand-layout copy of X (pass 1)
  void* y;
  const float* z;
  const int32_t* idx;
  const float* ln;
  const float* gate_w;
  const float* gate_b;
  float* T_out;
  float tmin_tau, trange_tau;
  int B, C, HW, E_r, k, Kp;       // Kp: C rounded up to 64
  int n_tiles, n_bsplit;
};

constexpr int kQ = 4;             // K quarters: pipeline stages of the operands

struct TcBars {
  uint64_t full_b[kQ];            // B quarter landed (bulk copy, tx bytes)
  uint64_t mma_q[kQ];             // MMAs of a quarter done: A and B quarter free
  uint64_t a_full[kQ];            // rows wrote the A quarter (128 arrivals)
  uint64_t d_full[2];             // accumulator buffer complete
  uint64_t d_empty[2];            // accumulator buffer drained (128 arrivals)
  uint32_t tmem;
  int abort;
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Bounded wait that also gives up when another role has aborted.
__device__ __forceinline__ bool mbar_wait_abort(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const uint32_t a = smem_u32(bar);
  for (long long it = 0; it < kSpinLimit; ++it) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
    if ((it & 1023) == 1023 && *abort) return false;
  }
  *abort = 1;
  atomicExch(&g_tc_fault, 1);
  return false;
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
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void row_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// 160 threads: warps 0..3 own the 128 expert rows of the tile (softmax
// weights into A, accumulator drain, output), lane 0 of warp 4 moves the
// operands (bulk copies of the staged X quarters) and issues the MMAs.
template <typename T, int KMAX>
__global__ void __launch_bounds__(160, 1) mix_tc_kernel(TcArgs a) {
  extern __shared__ unsigned char s_dyn[];
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(s_dyn) + 1023) & ~uintptr_t(1023));
  const int C = a.C, HW = a.HW, k = a.k, Kp = a.Kp, E_r = a.E_r;
  const int Kq = Kp / kQ;                                     // channels per quarter (multiple of 16)
  // kQ stages pipeline the X operand (bulk copies); the weight operand is
  // rewritten per sample after the sample's last MMA (mma_q[kQ - 1])
  unsigned char* sA = base;                                   // 128 x Kp : Kp * 256 B
  unsigned char* sB = base + (size_t)Kp * 256;                // Kp x 64  : Kp * 128 B
  T* stg = reinterpret_cast<T*>(sB + (size_t)Kp * 128);       // 128 x HW output block
  float* s_z = reinterpret_cast<float*>(sB + (size_t)Kp * 128 + 128 * kTcN * sizeof(T));  // 2 x Kp
  float* s_gw = s_z + 2 * Kp;
  TcBars* bars = reinterpret_cast<TcBars*>(s_gw + KMAX);
  volatile int* abort = &bars->abort;

  const int tid = threadIdx.x, warp = tid >> 5;
  const int tile = blockIdx.x % a.n_tiles, bsplit = blockIdx.x / a.n_tiles;
  const int e0 = tile * 128;
  const int rows = min(128, E_r - e0);
  const int b0 = (int)((long long)bsplit * a.B / a.n_bsplit);
  const int b1 = (int)((long long)(bsplit + 1) * a.B / a.n_bsplit);
  const int nb = b1 - b0;
  const int E = E_r + 1;

  for (int q = tid; q < Kp * 256 / 16; q += blockDim.x) reinterpret_cast<int4*>(sA)[q] = make_int4(0, 0, 0, 0);
  for (int i = tid; i < k; i += blockDim.x) s_gw[i] = a.gate_w[i];
  if (tid == 0) {
    for (int q = 0; q < kQ; ++q) {
      mbar_init(&bars->full_b[q], 1);
      mbar_init(&bars->mma_q[q], 1);
      mbar_init(&bars->a_full[q], 128);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->d_full[s], 1);
      mbar_init(&bars->d_empty[s], 128);
    }
    bars->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&bars->tmem)),
                 "r"(2 * kTcN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;

  if (warp == 4) {
    // ===================== operand mover + MMA issuer (one thread)
    if (tid == 128) {
      const uint32_t idesc = umma_idesc(DTypeOf<T>::value == MOCE_BF16 ? 1 : 0, 128, kTcN);
      const uint32_t aA = smem_u32(sA), aB = smem_u32(sB);
      const unsigned char* xs = static_cast<const unsigned char*>(a.xstage);
      const uint32_t qbytes = (uint32_t)Kq * 128;
      const uint64_t da0 = umma_desc(aA, 16, 1024);
      const uint64_t db0 = umma_desc(aB, (uint32_t)Kp * 128, 1024);
      bool run = nb > 0;
      if (run)
        for (int q = 0; q < kQ; ++q) {
          mbar_expect_tx(&bars->full_b[q], qbytes);
          bulk_g2s(aB + q * qbytes, xs + (size_t)b0 * Kp * 128 + (size_t)q * qbytes, qbytes, &bars->full_b[q]);
        }
      for (int i = 0; i < nb && run; ++i) {
        const int s = i & 1;
        if (i >= 2 && !mbar_wait_abort(&bars->d_empty[s], ((i - 2) >> 1) & 1, abort)) break;
        const uint32_t d = tmem + (uint32_t)(s * kTcN);
        for (int q = 0; q < kQ && run; ++q) {
          if (!mbar_wait_abort(&bars->full_b[q], i & 1, abort) || !mbar_wait_abort(&bars->a_full[q], i & 1, abort)) {
            run = false;
            break;
          }
          tc_fence_after();
          for (int j = q * Kq / 16; j < (q + 1) * Kq / 16; ++j) {
            // start-address fields advance in 16-byte units (no carry: shared
            // addresses are below 2^18)
            const uint64_t da = da0 + (uint64_t)(((j >> 2) * 16384 + (j & 3) * 32) >> 4);
            const uint64_t db = db0 + (uint64_t)(j * 128);
            umma_f16(d, da, db, idesc, j > 0 ? 1u : 0u);
          }
          umma_commit(&bars->mma_q[q]);
        }
        if (!run) break;
        umma_commit(&bars->d_full[s]);
        if (i + 1 < nb) {
          for (int q = 0; q < kQ; ++q) {
            if (!mbar_wait_abort(&bars->mma_q[q], i & 1, abort)) {
              run = false;
              break;
            }
            mbar_expect_tx(&bars->full_b[q], qbytes);
            bulk_g2s(aB + q * qbytes, xs + (size_t)(b0 + i + 1) * Kp * 128 + (size_t)q * qbytes, qbytes,
                     &bars->full_b[q]);
          }
        }
      }
    }
  } else {
    // ===================== expert rows: weights -> A, accumulator -> Y
    const int e = e0 + tid;
    const bool has_row = tid < rows;
    int ch[KMAX];
    float ln2[KMAX];
    float mx2 = -INFINITY;
#pragma unroll
    for (int i = 0; i < KMAX; ++i) {
      ch[i] = 0;
      ln2[i] = -INFINITY;
      if (i < k && has_row) {
        ch[i] = a.idx[(size_t)e * k + i];
        ln2[i] = a.ln[(size_t)e * k + i] * 1.4426950408889634f;   // log2(e)
        mx2 = nan_max(mx2, ln2[i]);
      }
    }
    const float bias = a.gate_b[0];
    T* yg = static_cast<T*>(a.y);
    float w[KMAX];
    constexpr int ZPT = 4;                           // z values per thread (C <= 512)
    float zr[ZPT];
#pragma unroll
    for (int u = 0; u < ZPT; ++u) {
      const int c = tid + u * 128;
      zr[u] = (nb > 0 && c < C) ? a.z[(size_t)b0 * C + c] : 0.0f;
    }
    for (int i = 0; i <= nb; ++i) {
      if (i < nb) {
        const int b = b0 + i;
        float* szb = s_z + (i & 1) * Kp;
#pragma unroll
        for (int u = 0; u < ZPT; ++u)
          if (tid + u * 128 < C) szb[tid + u * 128] = zr[u];
        row_bar();
        if (i + 1 < nb) {
#pragma unroll
          for (int u = 0; u < ZPT; ++u) {
            const int c = tid + u * 128;
            if (c < C) zr[u] = a.z[(size_t)(b + 1) * C + c];
          }
        }
        if (has_row) {
          float g = bias;
#pragma unroll
          for (int j = 0; j < KMAX; ++j)
            if (j < k) g += s_gw[j] * szb[ch[j]];
          const float t = temperature(g, a.tmin_tau, a.trange_tau, nullptr);
          if (a.T_out) a.T_out[(size_t)b * E_r + e] = t;
          const float it = 1.0f / t;
          const float m2 = mx2 * it;
          float zs = 0.0f;
#pragma unroll
          for (int j = 0; j < KMAX; ++j) {
            w[j] = exp2f(ln2[j] * it - m2);
            zs += w[j];
          }
          const float iz = 1.0f / zs;
#pragma unroll
          for (int j = 0; j < KMAX; ++j) w[j] *= iz;
        }
        // A is rewritten once the previous sample's MMAs are all done; one
        // proxy fence makes the new weights visible to the tensor cores
        if (i >= 1 && !mbar_wait_abort(&bars->mma_q[kQ - 1], (i - 1) & 1, abort)) break;
        if (has_row) {
#pragma unroll
          for (int j = 0; j < KMAX; ++j)
            if (j < k) *reinterpret_cast<T*>(sA + a_off(tid, ch[j])) = from_f<T>(w[j]);
        }
        proxy_fence_smem();
        for (int q = 0; q < kQ; ++q) mbar_arrive(&bars->a_full[q]);
      }
      if (i >= 1) {
        // drain sample i-1
        const int j = i - 1, s = j & 1;
        if (!mbar_wait_abort(&bars->d_full[s], (j >> 1) & 1, abort)) break;
        tc_fence_after();
        float v[kTcN];
        tmem_ld64(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(s * kTcN), v);
        tc_fence_before();
        mbar_arrive(&bars->d_empty[s]);
        if (tid == 0) bulk_wait_read();               // previous block left the staging area
        row_bar();
        if (has_row) {
#pragma unroll
          for (int p = 0; p < kTcN; ++p)
            if (p < HW) stg[tid * HW + p] = from_f<T>(v[p]);
        }
        proxy_fence_smem();
        row_bar();
        T* dst = yg + ((size_t)(b0 + j) * E + e0) * HW;
        const uint32_t nbytes = (uint32_t)(rows * HW * sizeof(T));
        if (((((uintptr_t)dst) | nbytes) & 15) == 0) {
          if (tid == 0) bulk_s2g(dst, smem_u32(stg), nbytes);
        } else {
          for (int q = tid; q < rows * HW; q += 128) dst[q] = stg[q];
          row_bar();
        }
      }
    }
    if (tid == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kTcN));
}

}  // namespace

int tc_supported(int dtype, int64_t C, int64_t HW, int64_t k) {
  return (dtype == MOCE_BF16 || dtype == MOCE_F16) && HW >= 1 && HW <= kTcN && k <= 64 && C <= 512;
}

}  // namespace moce

using namespace moce;

extern "C" size_t moce_tc_stage_bytes(int64_t B, int64_t C) {
  return (size_t)B * (size_t)((C + 63) / 64 * 64) * 128;
}

extern "C" int moce_mix_tc(const void* xstage, int dtype, int64_t B, int64_t C, int64_t HW, const float* z,
                           const int32_t* idx, const float* ln, int64_t E_r, int64_t k, const float* gate_w,
                           const float* gate_b, float tmin_tau, float trange_tau, void* y, float* T_out,
                           void* stream) {
  if (B == 0) return MOCE_OK;
  MOCE_REQUIRE(xstage && z && idx && ln && gate_w && gate_b && y, MOCE_ERR_INVALID,
               "moce_mix_tc: null pointer argument");
  MOCE_REQUIRE(B > 0 && C >= 1 && HW >= 1 && E_r >= 1 && k >= 1 && k <= C, MOCE_ERR_INVALID,
               "moce_mix_tc: invalid shape");
  MOCE_REQUIRE(tc_supported(dtype, C, HW, k), MOCE_ERR_UNSUPPORTED,
               "moce_mix_tc: needs bf16/fp16, H*W <= 64, C <= 512, k <= 64");
  MOCE_REQUIRE(((uintptr_t)xstage & 15) == 0, MOCE_ERR_INVALID, "moce_mix_tc: xstage must be 16-byte aligned");
  MOCE_REQUIRE(B < 65536 && (E_r + 1) * HW < (int64_t)1 << 31, MOCE_ERR_UNSUPPORTED, "moce_mix_tc: shape too large");
  const int Kp = (int)((C + 63) / 64 * 64);
  const int KMAX = k <= 16 ? 16 : k <= 32 ? 32 : 64;
  const size_t smem = 1024 + (size_t)Kp * 256 + (size_t)Kp * 128 + (size_t)128 * 64 * 2 + (size_t)Kp * 8 +
                      (size_t)KMAX * 4 + sizeof(TcBars) + 16;
  const int n_tiles = (int)((E_r + 127) / 128);
  int n_bsplit = num_sms() / n_tiles;
  if (n_bsplit < 1) n_bsplit = 1;
  if (n_bsplit > B) n_bsplit = (int)B;
  TcArgs a{xstage, y, z, idx, ln, gate_w, gate_b, T_out, tmin_tau, trange_tau,
           (int)B, (int)C, (int)HW, (int)E_r, (int)k, Kp, n_tiles, n_bsplit};
  return dispatch_dtype(dtype, [&](auto tag) {
    using T = decltype(tag);
    if constexpr (sizeof(T) != 2) {
      return set_error(MOCE_ERR_UNSUPPORTED, "moce_mix_tc: 16-bit inputs only");
    } else {
      void (*kern)(TcArgs) = KMAX == 16 ? mix_tc_kernel<T, 16> : KMAX == 32 ? mix_tc_kernel<T, 32>
                                                                            : mix_tc_kernel<T, 64>;
      if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return set_error(MOCE_ERR_CUDA, "moce_mix_tc: cannot reserve %zu B shared memory", smem);
      kern<<<(unsigned)(n_tiles * n_bsplit), 160, smem, (cudaStream_t)stream>>>(a);
      return check_launch("mix_tc_kernel");
    }
  });
}

extern "C" int moce_tc_fault(int* flag, int clear) {
  MOCE_REQUIRE(flag, MOCE_ERR_INVALID, "moce_tc_fault: null pointer");
  if (cudaMemcpyFromSymbol(flag, g_tc_fault, sizeof(int)) != cudaSuccess)
    return set_error(MOCE_ERR_CUDA, "moce_tc_fault: read failed");
  if (clear) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_tc_fault, &zero, sizeof(int)) != cudaSuccess)
      return set_error(MOCE_ERR_CUDA, "moce_tc_fault: clear failed");
  }
  return MOCE_OK;
}
