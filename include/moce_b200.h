/*
 * moce_b200.h -- C ABI of the B200 (sm_100a) MoCE layer kernels.
 *
 * Plain pointers and sizes only: every tensor argument is a device pointer to
 * a dense, contiguous array laid out as documented; no allocation happens
 * inside any entry point (callers pass outputs and, where noted, a workspace
 * sized by the matching *_workspace_bytes query).  Every call is asynchronous
 * on `stream` (a cudaStream_t; NULL = legacy default stream) and returns a
 * moce_status; moce_last_error() gives a message for the calling thread.
 *
 * Shapes: B batch, C input channels, HW = H*W spatial positions, E_r routed
 * experts (the layer has E = E_r + 1 output channels, the last one is the
 * residual expert), k supports per expert.  X is [B, C, HW]; Y is [B, E, HW].
 *
 * Reference interfaces replaced (Elianiluk/MoCE_thesis):
 *   moce_fixed/moce_layer_cuda.cpp  -- pybind wrappers of the 7 entry points
 *   moce_fixed/moce_kernel.cu       -- their CUDA implementations
 *   MoCE.py                         -- the ATen parts of the layer (cache
 *                                      build, pooling, gate, softmax)
 */
#ifndef MOCE_B200_H
#define MOCE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden symbol visibility: only the entry points
 * declared here are exported, so a process that loads two builds of it (or
 * another library with the same internal names) cannot bind one build's
 * internal calls to the other's. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef enum {
  MOCE_OK = 0,
  MOCE_ERR_INVALID = 1,      /* bad pointer, shape or dtype */
  MOCE_ERR_UNSUPPORTED = 2,  /* shape outside the supported range */
  MOCE_ERR_CUDA = 3,         /* a CUDA runtime call or launch failed */
  MOCE_ERR_WORKSPACE = 4     /* workspace missing or too small */
} moce_status;

typedef enum { MOCE_F32 = 0, MOCE_BF16 = 1, MOCE_F16 = 2 } moce_dtype;

/* Message for the last non-OK status returned on the calling thread. */
const char* moce_last_error(void);

/* Library version string. */
const char* moce_version(void);

/*
 * Support selection, logit normalisation and coverage (the eval cache).
 * Replaces MoCE.build_eval_cache (MoCE.py:85-109) and the per-step topk of
 * MoCE.forward_train (MoCE.py:160-187).
 *   logits  fp32 [E_r, C]      routing logits L
 *   idx     int32 [E_r, k]     out: TopK(L_e, k), descending logit, ties by
 *                              ascending channel (torch.topk order when the
 *                              row has no ties)
 *   ln      fp32 [E_r, k]      out: (sel - mean) / max(std_unbiased, 1)
 *   mask    int32 [C]          out: 1 where no expert selects the channel
 *   meta    int32 [2]          out: {number of uncovered channels, 0}
 *   toff    int32 [C+1]        out (optional, NULL to skip): CSR offsets of
 *   tslot   int32 [E_r*k]      the per-channel list of flat slots e*k+i with
 *                              idx[e,i] == c, ascending (used by backward)
 */
int moce_route_build(const float* logits, int64_t E_r, int64_t C, int64_t k,
                     int32_t* idx, float* ln, int32_t* mask, int32_t* meta,
                     int32_t* toff, int32_t* tslot, void* stream);

/*
 * Support schedule for the scheduled mix (no reference counterpart: it is a
 * layout of the supports chosen at cache-build time).  Experts are grouped
 * 32 per warp (balance != 0: greedily, so each group's supports spread over
 * the 32 shared-memory banks; balance == 0: experts 32g .. 32g+31), and each
 * group's supports are ordered into moce_schedule_steps(k) steps in which the
 * 32 lanes read 32 different banks.
 *   group_expert int32 [G*32], G = ceil(E_r/32)    out: expert of each lane, -1 if none
 *   sched        int32 [G*S*32], S = moce_schedule_steps(k)
 *                out: entry (slot << 16) | channel, slot 0xFFFF = idle step
 * Requires k <= 256, C <= 65535, E_r <= 32768.
 */
int moce_schedule_steps(int64_t k);
int moce_schedule_build(const int32_t* idx, int64_t E_r, int64_t C, int64_t k,
                        int balance, int32_t* group_expert, int32_t* sched,
                        void* stream);

/*
 * Pass 1 of the fast path: one read of X gives the pooled means z (fp32
 * [B, C], MoCE.py:174 / 212) and, if y is not NULL, the residual expert
 * channel y[:, E_r, :] (mean over channels with mask[c] == 1, 0 if none;
 * MoCE.py:191-196, moce_kernel.cu:148-231).  y is [B, E_r+1, HW] in the dtype
 * of X; meta is the route cache's {n_uncovered, 0}.
 */
int moce_pool_residual(const void* x, int dtype, int64_t B, int64_t C,
                       int64_t HW, const int32_t* mask, const int32_t* meta,
                       float* z, void* y, int64_t E_r, void* stream);

/*
 * Pass 2 of the fast path: routed experts 0 .. E_r-1 of y from X, the pooled
 * z of pass 1, the normalised logits ln [E_r, k] and the schedule.  Fuses
 * the gate and temperature (MoCE.py:216-218 / 175-178), the softmax of ln/T
 * (MoCE.py:219-221 / 188) and the gather-mix (moce_kernel.cu:57-141).  If
 * T_out is not NULL the temperatures fp32 [B, E_r] are written there (the
 * backward needs them).  Requires moce_schedule_steps(k) <= 52 (k <= 44).
 */
int moce_mix_scheduled(const void* x, int dtype, int64_t B, int64_t C,
                       int64_t HW, const float* z, const float* ln,
                       int64_t E_r, int64_t k, const int32_t* group_expert,
                       const int32_t* sched, const float* gate_w,
                       const float* gate_b, float tmin_tau, float trange_tau,
                       void* y, float* T_out, void* stream);

/*
 * Temperatures from the pooled means z fp32 [B, C] (pass 1's output), the
 * step between the two passes:
 *   T[b,e] = max(tmin_tau + trange_tau * sigmoid(g[b,e]), 1e-3)  fp32 [B, E_r]
 * moce_temperature: the shared Linear(k,1) gate of the reference
 * (MoCE.py:66-68, eval MoCE.py:216-218, train MoCE.py:175-178),
 *   g[b,e] = gate_w . z[b, idx[e,:]] + gate_b[0];  k <= 128.
 * moce_temperature_mlp: the two-layer gate C -> Hd -> E_r with ReLU of the
 * benchmark configurations (no reference counterpart; the reference has only
 * the Linear(k,1) gate),
 *   h[b,:] = relu(w1 z[b,:] + b1)  (fp32 [B, Hd] out),
 *   g[b,e] = w2[e,:] . h[b,:] + b2[e];
 * w1 fp32 [Hd, C], b1 [Hd], w2 [E_r, Hd], b2 [E_r]; Hd <= 256.
 */
int moce_temperature(const float* z, int64_t B, int64_t C, const int32_t* idx,
                     int64_t E_r, int64_t k, const float* gate_w,
                     const float* gate_b, float tmin_tau, float trange_tau,
                     float* T, void* stream);
int moce_temperature_mlp(const float* z, int64_t B, int64_t C, int64_t Hd,
                         int64_t E_r, const float* w1, const float* b1,
                         const float* w2, const float* b2, float tmin_tau,
                         float trange_tau, float* h, float* T, void* stream);

/*
 * Tensor-core fast path, for bf16 / fp16 inputs with C <= 512 and k <= 64
 * (any H*W) whose operands fit the shared memory of one CTA (the ResNet-50
 * maps from 56x56 to 7x7); moce_tc_supported returns 1 for those.
 *
 * moce_pool_stage: pass 1 as moce_pool_residual, plus a copy of X in the
 * tensor-core operand layout: per sample, NT pixel tiles of NP pixels (NP a
 * multiple of 16 of at most 256, 128 or 64, chosen from C and H*W so that
 * pass 2 fits shared memory; the last tile shorter), each with Kp = C
 * rounded up to 64 channel rows in four K-quarters and NA = ceil(NP / 64)
 * atoms of 64 pixels; stored [tile][quarter][atom][Kp/4 rows][128 bytes],
 * each row's 16-byte units swizzled by (channel mod 8).  moce_tc_stage_bytes
 * gives its size.
 *
 * moce_mix_tc: pass 2.  Same outputs as moce_mix_scheduled; the routed
 * experts are computed per sample as a dense product of the 128-expert weight
 * tile (zero off the supports) with the staged X (bulk copies into shared
 * memory, tcgen05.mma with the accumulator in tensor memory).  The gate and
 * temperature (MoCE.py:216-218) and the softmax of ln / T (MoCE.py:219-221)
 * are computed in the kernel from z.  Weights are rounded to the input's
 * 16-bit type before the product (fp32 accumulation).
 * moce_mix_tc_t: the same with the temperatures T fp32 [B, E_r] given (e.g.
 * from moce_temperature_mlp) in place of z and the Linear(k,1) gate.
 *
 * Waits inside the kernel are bounded in time.  If a wait of one role of the
 * kernel on another runs out (about one second by default), the kernel sets a
 * device flag and abandons the launch, so part of y is left unwritten.  The
 * copies and MMAs already in flight complete, the kernel returns, and the
 * CUDA context stays usable.  moce_tc_fault reads (and optionally clears)
 * that flag.  It synchronises with the device, so check it after a batch of
 * calls, not after each one.  moce_tc_wait_limit_ns(ns) sets the bound, in
 * nanoseconds, for launches made after it when ns > 0, and returns the bound
 * that was in effect; ns <= 0 only queries.  (No reference counterpart: the
 * reference kernels have no waits.)
 */
int moce_tc_supported(int dtype, int64_t C, int64_t HW, int64_t k);
size_t moce_tc_stage_bytes(int64_t B, int64_t C, int64_t HW);
int moce_pool_stage(const void* x, int dtype, int64_t B, int64_t C,
                    int64_t HW, const int32_t* mask, const int32_t* meta,
                    float* z, void* y, int64_t E_r, void* xstage,
                    void* stream);
int moce_mix_tc(const void* xstage, int dtype, int64_t B, int64_t C,
                int64_t HW, const float* z, const int32_t* idx,
                const float* ln, int64_t E_r, int64_t k, const float* gate_w,
                const float* gate_b, float tmin_tau, float trange_tau,
                void* y, float* T_out, void* stream);
int moce_mix_tc_t(const void* xstage, int dtype, int64_t B, int64_t C,
                  int64_t HW, const float* T, const int32_t* idx,
                  const float* ln, int64_t E_r, int64_t k, void* y,
                  void* stream);
int moce_tc_fault(int* flag, int clear);
int64_t moce_tc_wait_limit_ns(int64_t ns);
/* Where the first wait that ran out gave up, for diagnostics (synchronises):
 * info[0] 1 if recorded, [1] wait site (1 producer: ring slot free, 2 issuer:
 * accumulator drained (one tile per sample), 3 issuer: weights written,
 * 4 issuer: accumulator drained (pixel tiles), 5 issuer: X quarter landed,
 * 6 weight rows: previous sample's MMAs done, 7 drain: accumulator
 * complete), [2] parity, [3] unit or sample index, [4] block, [5] thread,
 * [6] C, [7] H*W, [8] E_r, [9] k, [10] B, [11] pixel tiles per sample,
 * [12] MMA N, [13] nanoseconds waited.  Fills min(n, 14) entries. */
int moce_tc_fault_info(int64_t* info, int n, int clear);

/*
 * Both tensor-core passes in one call: moce_pool_stage, then moce_mix_tc
 * launched as a programmatic dependent of it (the mix's prologue overlaps
 * pass 1; its reads of z and xstage wait for pass 1 to complete).  Same
 * buffers and conditions as the two calls.
 */
int moce_forward_tc(const void* x, int dtype, int64_t B, int64_t C, int64_t HW,
                    const int32_t* mask, const int32_t* meta,
                    const int32_t* idx, const float* ln, int64_t E_r,
                    int64_t k, const float* gate_w, const float* gate_b,
                    float tmin_tau, float trange_tau, float* z, void* xstage,
                    void* y, float* T_out, void* stream);

/*
 * The tensor-core forward with the two-layer temperature gate
 * (moce_temperature_mlp) in place of the shared Linear(k, 1): pass 1, the
 * gate, then moce_mix_tc_t, each a programmatic dependent of the launch
 * before.  z, the hidden layer h fp32 [B, Hd] and T (required) are outputs.
 * No reference counterpart (see moce_temperature_mlp).
 */
int moce_forward_tc_mlp(const void* x, int dtype, int64_t B, int64_t C,
                        int64_t HW, const int32_t* mask, const int32_t* meta,
                        const int32_t* idx, const float* ln, int64_t E_r,
                        int64_t k, int64_t Hd, const float* w1,
                        const float* b1, const float* w2, const float* b2,
                        float tmin_tau, float trange_tau, float* z, float* h,
                        void* xstage, void* y, float* T, void* stream);

/*
 * moce_forward_tc with the caller's next two ops folded into the output
 * store: every output channel e (routed experts and the residual) becomes
 *   relu?(y[b,e,p] * out_scale[e] + out_shift[e])
 * computed in fp32 before the one rounding to the 16-bit output type.
 * out_scale / out_shift are fp32 [E] (E = E_r + 1): an eval-mode
 * BatchNorm2d folded to scale = weight / sqrt(running_var + eps),
 * shift = bias - running_mean * scale.  Replaces the MoCE -> bn1 -> relu1
 * sequence of BottleneckWithMoCEProjection.forward (models_unified.py:155-165).
 * T_out (when given) and z are the layer's own values, before the epilogue.
 */
int moce_forward_tc_ep(const void* x, int dtype, int64_t B, int64_t C,
                       int64_t HW, const int32_t* mask, const int32_t* meta,
                       const int32_t* idx, const float* ln, int64_t E_r,
                       int64_t k, const float* gate_w, const float* gate_b,
                       float tmin_tau, float trange_tau,
                       const float* out_scale, const float* out_shift,
                       int out_relu, float* z, void* xstage, void* y,
                       float* T_out, void* stream);

/*
 * CUDA-core pass 2 with lanes over pixels, any dtype, H*W <= 512, k <= 64,
 * for maps of a few hundred pixels (14x14, 28x28 stages; fp32 anywhere).
 * Same inputs and outputs as moce_mix_tc with X itself in place of the
 * staged copy (pass 1 is moce_pool_residual): a warp per expert computes the
 * gate, temperature and softmax (MoCE.py:216-221 / 175-188) and sums its k
 * support rows (moce_kernel.cu:57-141) from X_b held in shared memory.
 * moce_px_supported returns 1 when the shape fits (X_b within the shared
 * memory of one CTA).
 */
int moce_px_supported(int dtype, int64_t C, int64_t HW, int64_t k);
int moce_mix_px(const void* x, int dtype, int64_t B, int64_t C, int64_t HW,
                const float* z, const int32_t* idx, const float* ln,
                int64_t E_r, int64_t k, const float* gate_w,
                const float* gate_b, float tmin_tau, float trange_tau,
                void* y, float* T_out, void* stream);
/* moce_mix_px with the temperatures given (fp32 [B, E_r], e.g. from
 * moce_temperature_mlp) in place of the gate's inputs. */
int moce_mix_px_t(const void* x, int dtype, int64_t B, int64_t C, int64_t HW,
                  const float* T, const int32_t* idx, const float* ln,
                  int64_t E_r, int64_t k, void* y, void* stream);

/*
 * Pass 2 on CUDA cores for samples too large for shared memory (C >= 1024 at
 * 14x14, 2048 at 7x7, 512 at 28x28: the deep ResNet-50 bottlenecks,
 * models_unified.py:227-258).  Same inputs, outputs and arithmetic as
 * moce_mix_px (replacing moce_kernel.cu:57-141 with the gate and softmax of
 * MoCE.py:216-221), but each expert's k support rows are read from X in
 * global memory, where a sample stays in L2 while its CTAs run.
 * moce_gx_supported: H*W <= 1024, k <= 128, C <= 16384.
 */
int moce_gx_supported(int dtype, int64_t C, int64_t HW, int64_t k);
int moce_mix_gx(const void* x, int dtype, int64_t B, int64_t C, int64_t HW,
                const float* z, const int32_t* idx, const float* ln,
                int64_t E_r, int64_t k, const float* gate_w,
                const float* gate_b, float tmin_tau, float trange_tau,
                void* y, float* T_out, void* stream);
/* moce_mix_gx with the temperatures given (fp32 [B, E_r]). */
int moce_mix_gx_t(const void* x, int dtype, int64_t B, int64_t C, int64_t HW,
                  const float* T, const int32_t* idx, const float* ln,
                  int64_t E_r, int64_t k, void* y, void* stream);

/*
 * Global average pool: pooled[b,c] = mean_p X[b,c,p] (fp32 out).
 * Replaces moce_pool (moce_layer_cuda.cpp:8-10, moce_kernel.cu:849-861).
 * pooled has the dtype of X in the reference; here it is always fp32.
 */
int moce_pool(const void* x, int dtype, int64_t B, int64_t C, int64_t HW,
              float* pooled, void* stream);

/*
 * Pass 1: global average pool fused with the shared Linear(k,1) temperature
 * gate.  Replaces the ATen code of MoCE.forward_eval (MoCE.py:212-218) and
 * MoCE.forward_train (MoCE.py:174-178):
 *   z[b,c]  = mean_p X[b,c,p]                         (fp32 [B, C], out)
 *   g       = gate_w . z[b, idx[e,:]] + gate_b[0]
 *   T[b,e]  = max(tmin_tau + trange_tau * sigmoid(g), 1e-3)  (fp32 [B, E_r], out)
 * with tmin_tau = temp_min * tau and trange_tau = (temp_max - temp_min) * tau.
 * gate_w fp32 [k], gate_b fp32 [1] are device pointers.  If `pooled_in` is
 * not NULL it is used as z (fp32 [B, C]) and X is not read (x may be NULL).
 */
int moce_gate_temperature(const void* x, int dtype, const float* pooled_in,
                          int64_t B, int64_t C, int64_t HW, const int32_t* idx,
                          int64_t E_r, int64_t k, const float* gate_w,
                          const float* gate_b, float tmin_tau, float trange_tau,
                          float* z, float* T, void* stream);

/*
 * Pass 2: per-expert softmax of ln[e,:] / T[b,e], the convex gather-mix of
 * the k selected channels, and the residual expert (mean over channels with
 * mask[c] == 1, or 0 when there are none).  Y has the dtype of X.
 * Replaces MoCE.py:219-229 and fused_moce_forward_dynamic_temp's kernels
 * (moce_kernel.cu:57-231).
 */
int moce_mix(const void* x, int dtype, int64_t B, int64_t C, int64_t HW,
             const int32_t* idx, const float* ln, const float* T,
             int64_t E_r, int64_t k, const int32_t* mask, void* y,
             void* stream);

/*
 * Drop-in for fused_moce_forward_dynamic_temp(input, indices, weights,
 * mask_int) (moce_layer_cuda.cpp:19-26, moce_kernel.cu:1079-1153): the mix
 * with caller-computed per-sample weights fp32 [B, E_r, K].  `indices` is
 * [E_r, K] int64 (index_bits = 64, as MoCE.py passes) or int32 (32).
 */
int moce_forward_dynamic_temp(const void* x, int dtype, const void* indices,
                              int index_bits, const float* weights,
                              const int32_t* mask, void* y, int64_t B,
                              int64_t C, int64_t HW, int64_t E_r, int64_t K,
                              void* stream);

/*
 * Drop-in for fused_moce_gate_route (moce_layer_cuda.cpp:36-45,
 * moce_kernel.cu:396-485; pooled given) and fused_moce_gate_route_all
 * (moce_layer_cuda.cpp:89-98, moce_kernel.cu:867-942; pooled == NULL, pool
 * computed here).  logits_norm fp32 [E_r, K] is used as given; T is
 * max((temp_min + (temp_max - temp_min) * sigmoid(g)) * tau, 1e-3).
 * workspace: moce_gate_route_workspace_bytes(B, C, E_r) bytes, 256-aligned.
 */
size_t moce_gate_route_workspace_bytes(int64_t B, int64_t C, int64_t E_r);
int moce_gate_route(const void* x, int dtype, const float* pooled,
                    const void* indices, int index_bits,
                    const float* logits_norm, const float* gate_w,
                    const float* gate_b, const int32_t* mask, float temp_min,
                    float temp_max, float tau, void* y, int64_t B, int64_t C,
                    int64_t HW, int64_t E_r, int64_t K, void* workspace,
                    size_t workspace_bytes, void* stream);

/*
 * moce_gate_route without a workspace argument.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory at the
 * call (for example a plugin inside an inference engine that gets a fixed
 * memory budget and no allocator, or a latency-critical path that cannot
 * take cudaMalloc's device-wide synchronisation).  Same arguments and results
 * as moce_gate_route minus the workspace; the scratch it needs comes from a
 * fixed array inside the library of moce_noalloc_scratch_bytes() bytes
 * (4 MiB), which every GPU that loads the library holds until exit.  Shapes
 * needing more (moce_gate_route_workspace_bytes) fail with
 * MOCE_ERR_UNSUPPORTED.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress) with that device current and keeps
 * it for the life of the process; make that first call before any stream
 * capture.  Calls across a cudaDeviceReset of that device are not supported
 * (the kept address belongs to the context the reset destroyed).  All calls
 * share the array: calls that overlap on the GPU race and must be serialised
 * by the caller.  It never calls cudaMalloc or cudaFree.
 */
size_t moce_noalloc_scratch_bytes(void);
int moce_gate_route_noalloc(const void* x, int dtype, const float* pooled,
                            const void* indices, int index_bits,
                            const float* logits_norm, const float* gate_w,
                            const float* gate_b, const int32_t* mask,
                            float temp_min, float temp_max, float tau,
                            void* y, int64_t B, int64_t C, int64_t HW,
                            int64_t E_r, int64_t K, void* stream);

/*
 * Backward of the layer (no reference kernel: the reference trains through
 * autograd over MoCE.forward_train, MoCE.py:153-201).  Given dY [B, E, HW]
 * (dtype of X), the forward's z and T, and the route cache (including the
 * transposed lists), writes
 *   dX      [B, C, HW]   dtype of X
 *   dL      fp32 [E_r, C]  gradient of the routing logits through the
 *                           selected-logit normalisation (zero off-support;
 *                           the auxiliary-loss gradient is not included)
 *   dgate_w fp32 [k], dgate_b fp32 [1]
 * Reductions over the batch are deterministic (fixed order, no atomics).
 * workspace: moce_backward_workspace_bytes(...) bytes.
 */
size_t moce_backward_workspace_bytes(int64_t B, int64_t C, int64_t HW,
                                     int64_t E_r, int64_t k);
int moce_backward(const void* x, const void* dy, int dtype, int64_t B,
                  int64_t C, int64_t HW, const float* logits,
                  const int32_t* idx, const float* ln, const int32_t* mask,
                  const int32_t* meta, const int32_t* toff,
                  const int32_t* tslot, int64_t E_r, int64_t k,
                  const float* gate_w, const float* gate_b, float tmin_tau,
                  float trange_tau, const float* z, const float* T, void* dx,
                  float* dL, float* dgate_w, float* dgate_b, void* workspace,
                  size_t workspace_bytes, void* stream);

/*
 * moce_backward for temperatures that came from a gate the caller
 * differentiates itself (the two-layer gate of moce_temperature_mlp): the
 * same dX (mix and residual terms only, no gate term) and dL, and instead of
 * the gate gradients dT fp32 [B, E_r], the gradient of the loss with respect
 * to the temperatures the mix used.  The caller adds the gate's own
 * contribution through z (dz / H*W per channel) to dX.  Same workspace.
 * (No reference counterpart, as for moce_backward.)
 */
int moce_backward_t(const void* x, const void* dy, int dtype, int64_t B,
                    int64_t C, int64_t HW, const float* logits,
                    const int32_t* idx, const float* ln, const int32_t* mask,
                    const int32_t* meta, const int32_t* toff,
                    const int32_t* tslot, int64_t E_r, int64_t k,
                    const float* T, void* dx, float* dL, float* dT,
                    void* workspace, size_t workspace_bytes, void* stream);

/*
 * The auxiliary (coverage) loss of the layer, MoCE._compute_aux_losses
 * (MoCE.py:118-151), and its gradient with respect to the routing logits:
 *   P = softmax(logits / tau) over channels, logits fp32 [E_r, C]
 *   aux = balance_weight * var_c(mean_e P)
 *       + specialization_weight * mean_c relu(H_c - log_target)
 *       + diversity_weight * mean of the off-diagonal of P P^T
 * with H_c the entropy of column c of P normalised to sum 1 (clamped at
 * 1e-8 as the reference does) and log_target = log(max(E_r k / C, 1)).  The
 * E_r x E_r product is not formed (its sum is the sum of squared column sums,
 * its trace the sum of squares).  aux_out: fp32 [1] on the device.
 * moce_aux_loss_backward writes dL fp32 [E_r, C] = grad_aux[0] * d aux /
 * d logits (grad_aux fp32 [1] on the device).  Both are deterministic.
 * workspace: moce_aux_workspace_bytes(E_r, C) bytes, 256-aligned.
 */
size_t moce_aux_workspace_bytes(int64_t E_r, int64_t C);
int moce_aux_loss(const float* logits, int64_t E_r, int64_t C, float tau,
                  float balance_weight, float specialization_weight,
                  float diversity_weight, float log_target, float* aux_out,
                  void* workspace, size_t workspace_bytes, void* stream);
int moce_aux_loss_backward(const float* logits, int64_t E_r, int64_t C,
                           float tau, float balance_weight,
                           float specialization_weight, float diversity_weight,
                           float log_target, const float* grad_aux, float* dL,
                           void* workspace, size_t workspace_bytes,
                           void* stream);

/*
 * The bottleneck's other eval-mode BatchNorms, fused with what follows them
 * (models_unified.py:155-169: relu2(bn2(conv2)), relu3(bn3(conv3) +
 * shortcut)), in one pass over NCHW tensors [N, C, HW] of x's dtype:
 *   y = act(x * scale[c] + shift[c] + (residual ? residual * rs[c] + rt[c] : 0))
 * with rs = 1, rt = 0 when r_scale / r_shift are null (an identity shortcut)
 * and act the ReLU when relu != 0 (a NaN stays NaN).  scale / shift (and
 * r_scale / r_shift, for a shortcut convolution's BatchNorm) are the
 * BatchNorms folded to fp32 per-channel affines: scale = weight /
 * sqrt(running_var + eps), shift = bias - running_mean * scale.  y may be x.
 * No reference counterpart (the reference runs the BatchNorm, add and ReLU
 * as torch ops).
 */
int moce_bn_act(const void* x, int dtype, int64_t N, int64_t C, int64_t HW,
                const float* scale, const float* shift, const void* residual,
                const float* r_scale, const float* r_shift, int relu, void* y,
                void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* MOCE_B200_H */
