// The auxiliary (coverage) loss of the layer and its gradient with respect to
// the routing logits, MoCE._compute_aux_losses (MoCE.py:118-151):
//   P        = softmax(L / tau) over channels                  [E_r, C]
//   usage_c  = mean_e P[e,c] = s_c / E_r,  s_c = sum_e P[e,c]
//   balance  = mean_c (usage_c - mean(usage))^2
//   q[e,c]   = P[e,c] / max(s_c, 1e-8)
//   H_c      = -sum_e q log(max(q, 1e-8))
//   spec     = mean_c relu(H_c - log(max(E_r k / C, 1)))
//   div      = mean of the off-diagonal of P P^T
//            = (sum_c s_c^2 - sum_{e,c} P^2) / (E_r (E_r - 1))   (0 when E_r == 1)
//   aux      = w_b balance + w_s spec + w_d div
// The P P^T of the reference (an E_r x C x E_r product) is never formed: its
// sum is the sum of squared column sums and its trace the sum of squares.
//
// Kernels (every reduction in a fixed order, no atomics, so the result is
// deterministic; sums over rows and columns in double):
//   aux_rows_kernel   a warp per expert row: max and 1 / sum exp of L / tau
//   aux_cols_kernel   32 channels x 8 row groups per CTA, rows split over
//                     grid.y: partial column sums of P and P^2 (mode 0), of
//                     q log q (mode 1, needs s), of the entropy gradient
//                     weighted by P (mode 2, backward)
//   aux_colsum_kernel the partials added in split order
//   aux_scalar_kernel one CTA: balance, spec, div, aux
//   aux_bwd_rows_kernel a warp per row: dP from the three terms, then the
//                     softmax backward dL = P (dP - sum_c P dP) / tau
#include <algorithm>

#include "common.cuh"

namespace moce {
namespace {

constexpr int kAuxCols = 32, kAuxGroups = 8;        // CTA of aux_cols_kernel: 32 columns x 8 row groups
constexpr int kAuxRowsPerSplit = 128;
constexpr float kEps = 1e-8f;

int aux_splits(int64_t E_r) { return (int)std::max<int64_t>(1, (E_r + kAuxRowsPerSplit - 1) / kAuxRowsPerSplit); }

struct AuxWs {
  float* rmax;    // [E_r]  max_c L / tau
  float* rinv;    // [E_r]  1 / sum_c exp(L / tau - max)
  double* part;   // [splits, C, 2]
  double* colS;   // [C]  s_c
  double* colQ;   // [C]  sum_e P^2
  double* colH;   // [C]  H_c
  double* colA;   // [C]  sum_e gq P (backward)
  double* stat;   // [8]  balance, spec, div, aux, mean usage
};

size_t aux_layout(int64_t E_r, int64_t C, unsigned char* base, AuxWs* w) {
  const size_t sz[8] = {(size_t)E_r * 4, (size_t)E_r * 4, (size_t)aux_splits(E_r) * C * 2 * 8, (size_t)C * 8,
                        (size_t)C * 8, (size_t)C * 8, (size_t)C * 8, 8 * 8};
  size_t off = 0;
  void* p[8];
  for (int i = 0; i < 8; ++i) {
    p[i] = base ? base + off : nullptr;
    off += align256(sz[i]);
  }
  if (w)
    *w = AuxWs{(float*)p[0], (float*)p[1], (double*)p[2], (double*)p[3], (double*)p[4], (double*)p[5], (double*)p[6],
               (double*)p[7]};
  return off;
}

struct AuxParams {
  int E, C;
  float tau, wb, ws, wd, log_target;
};

__device__ __forceinline__ float p_of(const float* Lrow, int c, float tau, float m, float inv) {
  return expf(Lrow[c] / tau - m) * inv;
}

// dH/dq of -q log(max(q, eps)), with torch's clamp gradient (passes at q >= eps)
__device__ __forceinline__ double dent_dq(float q) {
  return -((double)logf(fmaxf(q, kEps)) + (q >= kEps ? 1.0 : 0.0));
}

__global__ void __launch_bounds__(256) aux_rows_kernel(const float* __restrict__ L, AuxParams ap, AuxWs w) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * 8 + warp;
  if (e >= ap.E) return;
  const float* row = L + (size_t)e * ap.C;
  float m = -INFINITY;
  for (int c = lane; c < ap.C; c += 32) m = nan_max(m, row[c] / ap.tau);
  m = warp_max(m);
  double s = 0.0;
  for (int c = lane; c < ap.C; c += 32) s += (double)expf(row[c] / ap.tau - m);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
  if (lane == 0) {
    w.rmax[e] = m;
    w.rinv[e] = (float)(1.0 / s);
  }
}

// grid (ceil(C / 32), splits); thread (column cl = tid & 31, row group tid >> 5)
__global__ void __launch_bounds__(kAuxCols * kAuxGroups) aux_cols_kernel(const float* __restrict__ L, AuxParams ap,
                                                                         AuxWs w, int mode) {
  __shared__ double s_a[kAuxGroups][kAuxCols], s_b[kAuxGroups][kAuxCols];
  const int cl = threadIdx.x & 31, rg = threadIdx.x >> 5;
  const int c = blockIdx.x * kAuxCols + cl;
  const int e0 = blockIdx.y * kAuxRowsPerSplit, e1 = min(ap.E, e0 + kAuxRowsPerSplit);
  double a = 0.0, b = 0.0;
  if (c < ap.C) {
    const double s = (mode > 0) ? w.colS[c] : 1.0;
    const float sd = (float)fmax(s, (double)kEps);
    const bool active = (mode == 2) && (w.colH[c] - (double)ap.log_target > 0.0);
    for (int e = e0 + rg; e < e1; e += kAuxGroups) {
      const float p = p_of(L + (size_t)e * ap.C, c, ap.tau, w.rmax[e], w.rinv[e]);
      if (mode == 0) {
        a += (double)p;
        b += (double)p * (double)p;
      } else if (mode == 1) {
        const float q = p / sd;
        a += (double)q * (double)logf(fmaxf(q, kEps));
      } else if (active) {
        a += dent_dq(p / sd) * (double)p;
      }
    }
  }
  s_a[rg][cl] = a;
  s_b[rg][cl] = b;
  __syncthreads();
  if (rg == 0 && c < ap.C) {
    double ta = 0.0, tb = 0.0;
    for (int g = 0; g < kAuxGroups; ++g) {
      ta += s_a[g][cl];
      tb += s_b[g][cl];
    }
    double* out = w.part + ((size_t)blockIdx.y * ap.C + c) * 2;
    out[0] = ta;
    out[1] = tb;
  }
}

// column totals over the row splits, in split order: mode 0 -> (s, Q),
// mode 1 -> H = -sum, mode 2 -> A
__global__ void aux_colsum_kernel(AuxParams ap, AuxWs w, int splits, int mode) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= ap.C) return;
  double a = 0.0, b = 0.0;
  for (int sp = 0; sp < splits; ++sp) {
    a += w.part[((size_t)sp * ap.C + c) * 2];
    b += w.part[((size_t)sp * ap.C + c) * 2 + 1];
  }
  if (mode == 0) {
    w.colS[c] = a;
    w.colQ[c] = b;
  } else if (mode == 1) {
    w.colH[c] = -a;
  } else {
    w.colA[c] = a;
  }
}

// one CTA of 256 threads: the three terms and the loss
__global__ void __launch_bounds__(256) aux_scalar_kernel(AuxParams ap, AuxWs w, float* __restrict__ aux_out) {
  __shared__ double red[3][8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const double E = (double)ap.E, C = (double)ap.C;
  // mean usage first (fixed-order block sum)
  double su = 0.0;
  for (int c = threadIdx.x; c < ap.C; c += 256) su += w.colS[c] / E;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) su += __shfl_xor_sync(kFull, su, o);
  if (lane == 0) red[0][warp] = su;
  __syncthreads();
  double ubar = 0.0;
  for (int i = 0; i < 8; ++i) ubar += red[0][i];
  ubar /= C;
  __syncthreads();
  double bal = 0.0, spec = 0.0, sq = 0.0;
  for (int c = threadIdx.x; c < ap.C; c += 256) {
    const double du = w.colS[c] / E - ubar;
    bal += du * du;
    const double h = w.colH[c] - (double)ap.log_target;
    spec += h > 0.0 ? h : 0.0;
    sq += w.colS[c] * w.colS[c] - w.colQ[c];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    bal += __shfl_xor_sync(kFull, bal, o);
    spec += __shfl_xor_sync(kFull, spec, o);
    sq += __shfl_xor_sync(kFull, sq, o);
  }
  if (lane == 0) {
    red[0][warp] = bal;
    red[1][warp] = spec;
    red[2][warp] = sq;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double tb = 0.0, ts = 0.0, tq = 0.0;
    for (int i = 0; i < 8; ++i) {
      tb += red[0][i];
      ts += red[1][i];
      tq += red[2][i];
    }
    const double balance = tb / C, specialization = ts / C;
    const double diversity = ap.E > 1 ? tq / (E * (E - 1.0)) : 0.0;
    const double aux = (double)ap.wb * balance + (double)ap.ws * specialization + (double)ap.wd * diversity;
    w.stat[0] = balance;
    w.stat[1] = specialization;
    w.stat[2] = diversity;
    w.stat[3] = aux;
    w.stat[4] = ubar;
    if (aux_out) aux_out[0] = (float)aux;
  }
}

// a warp per expert row: dP, the row dot sum_c P dP, then dL
__global__ void __launch_bounds__(256) aux_bwd_rows_kernel(const float* __restrict__ L, AuxParams ap, AuxWs w,
                                                           const float* __restrict__ grad_aux, float* __restrict__ dL) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * 8 + warp;
  if (e >= ap.E) return;
  const float* row = L + (size_t)e * ap.C;
  const float m = w.rmax[e], inv = w.rinv[e];
  const double go = (double)grad_aux[0];
  const double E = (double)ap.E, C = (double)ap.C;
  const double ubar = w.stat[4];
  const double kb = (double)ap.wb * 2.0 / (C * E);
  const double ks = (double)ap.ws / C;
  const double kd = ap.E > 1 ? (double)ap.wd * 2.0 / (E * (E - 1.0)) : 0.0;
  auto dP_of = [&](int c, float p) -> double {
    const double s = w.colS[c];
    double d = kb * (s / E - ubar) + kd * (s - (double)p);
    if (w.colH[c] - (double)ap.log_target > 0.0) {
      if (s >= (double)kEps) {
        const float q = p / (float)s;
        d += ks * (dent_dq(q) / s - w.colA[c] / (s * s));
      } else {
        d += ks * dent_dq(p / kEps) / (double)kEps;
      }
    }
    return go * d;
  };
  double dot = 0.0;
  for (int c = lane; c < ap.C; c += 32) {
    const float p = p_of(row, c, ap.tau, m, inv);
    dot += (double)p * dP_of(c, p);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(kFull, dot, o);
  for (int c = lane; c < ap.C; c += 32) {
    const float p = p_of(row, c, ap.tau, m, inv);
    dL[(size_t)e * ap.C + c] = (float)((double)p * (dP_of(c, p) - dot) / (double)ap.tau);
  }
}

int aux_forward_run(const float* L, AuxParams ap, AuxWs w, float* aux_out, cudaStream_t st) {
  const int splits = aux_splits(ap.E);
  aux_rows_kernel<<<(unsigned)((ap.E + 7) / 8), 256, 0, st>>>(L, ap, w);
  const dim3 gcols((unsigned)((ap.C + kAuxCols - 1) / kAuxCols), (unsigned)splits);
  const unsigned gsum = (unsigned)((ap.C + 255) / 256);
  aux_cols_kernel<<<gcols, kAuxCols * kAuxGroups, 0, st>>>(L, ap, w, 0);
  aux_colsum_kernel<<<gsum, 256, 0, st>>>(ap, w, splits, 0);
  aux_cols_kernel<<<gcols, kAuxCols * kAuxGroups, 0, st>>>(L, ap, w, 1);
  aux_colsum_kernel<<<gsum, 256, 0, st>>>(ap, w, splits, 1);
  aux_scalar_kernel<<<1, 256, 0, st>>>(ap, w, aux_out);
  return check_launch("moce_aux_loss");
}

int aux_check(const float* L, int64_t E_r, int64_t C, float tau, void* workspace, size_t workspace_bytes,
              const char* fn) {
  MOCE_REQUIRE(L && workspace, MOCE_ERR_INVALID, "%s: null pointer argument", fn);
  MOCE_REQUIRE(E_r >= 1 && C >= 1 && E_r < (1 << 30) && C < (1 << 30) && E_r * C < ((int64_t)1 << 40),
               MOCE_ERR_INVALID, "%s: invalid shape", fn);
  MOCE_REQUIRE(tau > 0.0f, MOCE_ERR_INVALID, "%s: tau must be positive", fn);
  const size_t need = aux_layout(E_r, C, nullptr, nullptr);
  MOCE_REQUIRE(workspace_bytes >= need && ((uintptr_t)workspace & 255) == 0, MOCE_ERR_WORKSPACE,
               "%s: workspace of %zu bytes (256-aligned) required", fn, need);
  return MOCE_OK;
}

}  // namespace
}  // namespace moce

using namespace moce;

extern "C" size_t moce_aux_workspace_bytes(int64_t E_r, int64_t C) { return aux_layout(E_r, C, nullptr, nullptr); }

extern "C" int moce_aux_loss(const float* logits, int64_t E_r, int64_t C, float tau, float balance_weight,
                             float specialization_weight, float diversity_weight, float log_target, float* aux_out,
                             void* workspace, size_t workspace_bytes, void* stream) {
  int rc = aux_check(logits, E_r, C, tau, workspace, workspace_bytes, "moce_aux_loss");
  if (rc) return rc;
  MOCE_REQUIRE(aux_out, MOCE_ERR_INVALID, "moce_aux_loss: null aux_out");
  AuxWs w;
  aux_layout(E_r, C, static_cast<unsigned char*>(workspace), &w);
  const AuxParams ap{(int)E_r, (int)C, tau, balance_weight, specialization_weight, diversity_weight, log_target};
  return aux_forward_run(logits, ap, w, aux_out, (cudaStream_t)stream);
}

extern "C" int moce_aux_loss_backward(const float* logits, int64_t E_r, int64_t C, float tau, float balance_weight,
                                      float specialization_weight, float diversity_weight, float log_target,
                                      const float* grad_aux, float* dL, void* workspace, size_t workspace_bytes,
                                      void* stream) {
  int rc = aux_check(logits, E_r, C, tau, workspace, workspace_bytes, "moce_aux_loss_backward");
  if (rc) return rc;
  MOCE_REQUIRE(grad_aux && dL, MOCE_ERR_INVALID, "moce_aux_loss_backward: null pointer argument");
  AuxWs w;
  aux_layout(E_r, C, static_cast<unsigned char*>(workspace), &w);
  const AuxParams ap{(int)E_r, (int)C, tau, balance_weight, specialization_weight, diversity_weight, log_target};
  cudaStream_t st = (cudaStream_t)stream;
  // the forward statistics again (cheap next to the backward itself), then
  // the entropy gradient's column sums and the row pass
  rc = aux_forward_run(logits, ap, w, nullptr, st);
  if (rc) return rc;
  const int splits = aux_splits(E_r);
  aux_cols_kernel<<<dim3((unsigned)((C + kAuxCols - 1) / kAuxCols), (unsigned)splits), kAuxCols * kAuxGroups, 0,
                    st>>>(logits, ap, w, 2);
  aux_colsum_kernel<<<(unsigned)((C + 255) / 256), 256, 0, st>>>(ap, w, splits, 2);
  aux_bwd_rows_kernel<<<(unsigned)((E_r + 7) / 8), 256, 0, st>>>(logits, ap, w, grad_aux, dL);
  return check_launch("moce_aux_loss_backward");
}
