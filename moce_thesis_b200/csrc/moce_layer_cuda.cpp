// PyTorch binding of the MoCE C ABI, importable as `moce_fixed.moce_cuda`.
//
// Mirrors the reference binding (moce_fixed/moce_layer_cuda.cpp:117-138):
// the same seven functions with the same arguments and return lists, so the
// reference MoCE.py (`import moce_fixed.moce_cuda`, MoCE.py:7, call at
// MoCE.py:224) runs on these kernels unchanged.  Differences, all supersets:
//   * kernels launch on the current CUDA stream (the reference uses the
//     legacy default stream, moce_kernel.cu:1116);
//   * input may be float32, bfloat16 or float16 (the reference accepts
//     float32 only); indices may be int64 (as MoCE.py passes) or int32;
//   * K is not limited to 64 (moce_kernel.cu:424 and others).
// Additional functions expose the native pipeline (route build, pass 1,
// pass 2, backward) used by moce_thesis_b200.MoCE.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <vector>

#include "../../include/moce_b200.h"

namespace {

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be CUDA")
#define CHECK_CONTIGUOUS(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
#define CHECK_INPUT(x) \
  CHECK_CUDA(x);       \
  CHECK_CONTIGUOUS(x)

void ok(int rc) { TORCH_CHECK(rc == MOCE_OK, "moce_b200: ", moce_last_error()); }

int dtype_of(const torch::Tensor& t) {
  switch (t.scalar_type()) {
    case torch::kFloat32: return MOCE_F32;
    case torch::kBFloat16: return MOCE_BF16;
    case torch::kFloat16: return MOCE_F16;
    default: TORCH_CHECK(false, "input must be float32, bfloat16 or float16");
  }
  return -1;
}

int index_bits(const torch::Tensor& t) {
  TORCH_CHECK(t.scalar_type() == torch::kInt64 || t.scalar_type() == torch::kInt32,
              "indices must be int64 or int32");
  return t.scalar_type() == torch::kInt64 ? 64 : 32;
}

void* cur_stream() { return (void*)at::cuda::getCurrentCUDAStream().stream(); }

struct Dims {
  int64_t B, C, H, W, HW, E_r, K;
};

Dims dims(const torch::Tensor& input, const torch::Tensor& indices) {
  TORCH_CHECK(input.dim() == 4, "input must be (B, C, H, W)");
  TORCH_CHECK(indices.dim() == 2, "indices must be (E_routed, K)");
  Dims d;
  d.B = input.size(0);
  d.C = input.size(1);
  d.H = input.size(2);
  d.W = input.size(3);
  d.HW = d.H * d.W;
  d.E_r = indices.size(0);
  d.K = indices.size(1);
  return d;
}

torch::Tensor f32_opts_like(const torch::Tensor& t, at::IntArrayRef shape) {
  return torch::empty(shape, t.options().dtype(torch::kFloat32));
}

// Events on the current stream around a callable; returns elapsed ms.
template <typename F>
float timed(F&& f) {
  cudaStream_t st = at::cuda::getCurrentCUDAStream().stream();
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  cudaEventRecord(a, st);
  f();
  cudaEventRecord(b, st);
  cudaEventSynchronize(b);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return ms;
}

// ------------------------------------------------------- reference surface

std::vector<torch::Tensor> py_moce_pool(torch::Tensor input) {
  CHECK_INPUT(input);
  TORCH_CHECK(input.dim() == 4, "input must be (B, C, H, W)");
  const c10::cuda::CUDAGuard guard(input.device());
  const int64_t B = input.size(0), C = input.size(1), HW = input.size(2) * input.size(3);
  auto pooled = f32_opts_like(input, {B, C});
  ok(::moce_pool(input.data_ptr(), dtype_of(input), B, C, HW, pooled.data_ptr<float>(), cur_stream()));
  // the reference returns pooled in the input dtype (moce_kernel.cu:853)
  return {input.scalar_type() == torch::kFloat32 ? pooled : pooled.to(input.scalar_type())};
}

std::vector<torch::Tensor> fused_moce_forward_dynamic_temp(torch::Tensor input, torch::Tensor indices,
                                                           torch::Tensor weights, torch::Tensor mask_int) {
  CHECK_INPUT(input);
  CHECK_INPUT(indices);
  CHECK_INPUT(weights);
  CHECK_INPUT(mask_int);
  TORCH_CHECK(weights.scalar_type() == torch::kFloat32, "weights must be float32");
  TORCH_CHECK(mask_int.scalar_type() == torch::kInt32, "mask_int must be int32");
  const c10::cuda::CUDAGuard guard(input.device());
  Dims d = dims(input, indices);
  TORCH_CHECK(weights.dim() == 3 && weights.size(0) == d.B && weights.size(1) == d.E_r && weights.size(2) == d.K,
              "weights must be (B, E_routed, K)");
  TORCH_CHECK(mask_int.numel() == d.C, "mask_int must have C entries");
  auto out = torch::empty({d.B, d.E_r + 1, d.H, d.W}, input.options());
  ok(moce_forward_dynamic_temp(input.data_ptr(), dtype_of(input), indices.data_ptr(), index_bits(indices),
                               weights.data_ptr<float>(), mask_int.data_ptr<int32_t>(), out.data_ptr(), d.B, d.C,
                               d.HW, d.E_r, d.K, cur_stream()));
  return {out};
}

void check_gate_route_args(const torch::Tensor& input, const torch::Tensor& indices, const torch::Tensor& logits_norm,
                           const torch::Tensor& gate_weight, const torch::Tensor& gate_bias,
                           const torch::Tensor& mask_int, const Dims& d) {
  CHECK_INPUT(input);
  CHECK_INPUT(indices);
  CHECK_INPUT(logits_norm);
  CHECK_INPUT(gate_weight);
  CHECK_INPUT(gate_bias);
  CHECK_INPUT(mask_int);
  TORCH_CHECK(logits_norm.scalar_type() == torch::kFloat32, "logits_norm must be float32");
  TORCH_CHECK(gate_weight.scalar_type() == torch::kFloat32, "gate_weight must be float32");
  TORCH_CHECK(gate_bias.scalar_type() == torch::kFloat32, "gate_bias must be float32");
  TORCH_CHECK(mask_int.scalar_type() == torch::kInt32, "mask_int must be int32");
  TORCH_CHECK(logits_norm.numel() == d.E_r * d.K, "logits_norm must be (E_routed, K)");
  TORCH_CHECK(gate_weight.numel() == d.K, "gate_weight must have K entries");
  TORCH_CHECK(gate_bias.numel() >= 1, "gate_bias must have one entry");
  TORCH_CHECK(mask_int.numel() == d.C, "mask_int must have C entries");
}

torch::Tensor gate_route_impl(torch::Tensor input, const torch::Tensor* pooled, torch::Tensor indices,
                              torch::Tensor logits_norm, torch::Tensor gate_weight, torch::Tensor gate_bias,
                              torch::Tensor mask_int, double temp_min, double temp_max, double tau) {
  Dims d = dims(input, indices);
  check_gate_route_args(input, indices, logits_norm, gate_weight, gate_bias, mask_int, d);
  const float* pooled_ptr = nullptr;
  torch::Tensor pooled_f32;
  if (pooled) {
    CHECK_INPUT(*pooled);
    TORCH_CHECK(pooled->numel() == d.B * d.C, "pooled must be (B, C)");
    pooled_f32 = pooled->scalar_type() == torch::kFloat32 ? *pooled : pooled->to(torch::kFloat32);
    pooled_ptr = pooled_f32.data_ptr<float>();
  }
  auto out = torch::empty({d.B, d.E_r + 1, d.H, d.W}, input.options());
  const size_t wsb = moce_gate_route_workspace_bytes(d.B, d.C, d.E_r);
  auto ws = torch::empty({(int64_t)wsb + 256}, input.options().dtype(torch::kUInt8));
  void* wsp = (void*)(((uintptr_t)ws.data_ptr() + 255) & ~(uintptr_t)255);
  ok(moce_gate_route(input.data_ptr(), dtype_of(input), pooled_ptr, indices.data_ptr(), index_bits(indices),
                     logits_norm.data_ptr<float>(), gate_weight.data_ptr<float>(), gate_bias.data_ptr<float>(),
                     mask_int.data_ptr<int32_t>(), (float)temp_min, (float)temp_max, (float)tau, out.data_ptr(),
                     d.B, d.C, d.HW, d.E_r, d.K, wsp, wsb, cur_stream()));
  return out;
}

std::vector<torch::Tensor> fused_moce_gate_route(torch::Tensor input, torch::Tensor pooled, torch::Tensor indices,
                                                 torch::Tensor logits_norm, torch::Tensor gate_weight,
                                                 torch::Tensor gate_bias, torch::Tensor mask_int, double temp_min,
                                                 double temp_max, double tau) {
  const c10::cuda::CUDAGuard guard(input.device());
  return {gate_route_impl(input, &pooled, indices, logits_norm, gate_weight, gate_bias, mask_int, temp_min,
                          temp_max, tau)};
}

std::vector<torch::Tensor> fused_moce_gate_route_all(torch::Tensor input, torch::Tensor indices,
                                                     torch::Tensor logits_norm, torch::Tensor gate_weight,
                                                     torch::Tensor gate_bias, torch::Tensor mask_int, double temp_min,
                                                     double temp_max, double tau) {
  const c10::cuda::CUDAGuard guard(input.device());
  return {gate_route_impl(input, nullptr, indices, logits_norm, gate_weight, gate_bias, mask_int, temp_min, temp_max,
                          tau)};
}

// Timed variants.  The reference reports separate routed / residual kernel
// times and clock64 sections inside its routed kernel (moce_kernel.cu:493-579,
// 759-843, 951-1063).  Here the pipeline is two fused passes, timed with CUDA
// events on the current stream:
//   kernel_times (2): [pass 1 (pool + gate + temperature) ms, pass 2 (softmax + mix + residual) ms]
//   kernel_times (3): [pass 1 ms, pass 2 ms, 0 (residual is fused into pass 2)]
//   section_us  (4): [pass 1 us, 0 (temperature fused into pass 1), 0 (softmax fused into pass 2), pass 2 us]
struct TwoPass {
  torch::Tensor out;
  float ms1, ms2;
};

TwoPass gate_route_two_pass(torch::Tensor input, const torch::Tensor* pooled, torch::Tensor indices,
                            torch::Tensor logits_norm, torch::Tensor gate_weight, torch::Tensor gate_bias,
                            torch::Tensor mask_int, double temp_min, double temp_max, double tau) {
  Dims d = dims(input, indices);
  check_gate_route_args(input, indices, logits_norm, gate_weight, gate_bias, mask_int, d);
  torch::Tensor idx32 = indices.scalar_type() == torch::kInt32 ? indices : indices.to(torch::kInt32);
  torch::Tensor pooled_f32;
  const float* pooled_ptr = nullptr;
  if (pooled) {
    CHECK_INPUT(*pooled);
    TORCH_CHECK(pooled->numel() == d.B * d.C, "pooled must be (B, C)");
    pooled_f32 = pooled->scalar_type() == torch::kFloat32 ? *pooled : pooled->to(torch::kFloat32);
    pooled_ptr = pooled_f32.data_ptr<float>();
  }
  auto out = torch::empty({d.B, d.E_r + 1, d.H, d.W}, input.options());
  auto T = f32_opts_like(input, {d.B, d.E_r});
  auto z = f32_opts_like(input, {d.B, d.C});
  TwoPass r;
  r.ms1 = timed([&] {
    ok(moce_gate_temperature(input.data_ptr(), dtype_of(input), pooled_ptr, d.B, d.C, d.HW,
                             idx32.data_ptr<int32_t>(), d.E_r, d.K, gate_weight.data_ptr<float>(),
                             gate_bias.data_ptr<float>(), (float)(temp_min * tau), (float)((temp_max - temp_min) * tau),
                             pooled ? nullptr : z.data_ptr<float>(), T.data_ptr<float>(), cur_stream()));
  });
  r.ms2 = timed([&] {
    ok(moce_mix(input.data_ptr(), dtype_of(input), d.B, d.C, d.HW, idx32.data_ptr<int32_t>(),
                logits_norm.data_ptr<float>(), T.data_ptr<float>(), d.E_r, d.K, mask_int.data_ptr<int32_t>(),
                out.data_ptr(), cur_stream()));
  });
  r.out = out;
  return r;
}

std::vector<torch::Tensor> fused_moce_gate_route_timed(torch::Tensor input, torch::Tensor pooled,
                                                       torch::Tensor indices, torch::Tensor logits_norm,
                                                       torch::Tensor gate_weight, torch::Tensor gate_bias,
                                                       torch::Tensor mask_int, double temp_min, double temp_max,
                                                       double tau) {
  const c10::cuda::CUDAGuard guard(input.device());
  auto r = gate_route_two_pass(input, &pooled, indices, logits_norm, gate_weight, gate_bias, mask_int, temp_min,
                               temp_max, tau);
  return {r.out, torch::tensor({r.ms1, r.ms2})};
}

std::vector<torch::Tensor> fused_moce_gate_route_section_timed(torch::Tensor input, torch::Tensor pooled,
                                                               torch::Tensor indices, torch::Tensor logits_norm,
                                                               torch::Tensor gate_weight, torch::Tensor gate_bias,
                                                               torch::Tensor mask_int, double temp_min,
                                                               double temp_max, double tau) {
  const c10::cuda::CUDAGuard guard(input.device());
  auto r = gate_route_two_pass(input, &pooled, indices, logits_norm, gate_weight, gate_bias, mask_int, temp_min,
                               temp_max, tau);
  return {r.out, torch::tensor({r.ms1 * 1000.f, 0.f, 0.f, r.ms2 * 1000.f})};
}

std::vector<torch::Tensor> fused_moce_gate_route_all_timed(torch::Tensor input, torch::Tensor indices,
                                                           torch::Tensor logits_norm, torch::Tensor gate_weight,
                                                           torch::Tensor gate_bias, torch::Tensor mask_int,
                                                           double temp_min, double temp_max, double tau) {
  const c10::cuda::CUDAGuard guard(input.device());
  auto r = gate_route_two_pass(input, nullptr, indices, logits_norm, gate_weight, gate_bias, mask_int, temp_min,
                               temp_max, tau);
  return {r.out, torch::tensor({r.ms1, r.ms2, 0.f}), torch::tensor({r.ms1 * 1000.f, 0.f, 0.f, r.ms2 * 1000.f})};
}

// ------------------------------------------------------- native pipeline

std::vector<torch::Tensor> route_build(torch::Tensor logits, int64_t k, bool transposed) {
  CHECK_INPUT(logits);
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.dim() == 2, "logits must be float32 (E_r, C)");
  const c10::cuda::CUDAGuard guard(logits.device());
  const int64_t E_r = logits.size(0), C = logits.size(1);
  auto i32 = logits.options().dtype(torch::kInt32);
  auto idx = torch::empty({E_r, k}, i32);
  auto ln = torch::empty({E_r, k}, logits.options());
  auto mask = torch::empty({C}, i32);
  auto meta = torch::empty({2}, i32);
  torch::Tensor toff, tslot;
  if (transposed) {
    toff = torch::empty({C + 1}, i32);
    tslot = torch::empty({E_r * k}, i32);
  } else {
    toff = torch::empty({0}, i32);
    tslot = torch::empty({0}, i32);
  }
  ok(moce_route_build(logits.data_ptr<float>(), E_r, C, k, idx.data_ptr<int32_t>(), ln.data_ptr<float>(),
                      mask.data_ptr<int32_t>(), meta.data_ptr<int32_t>(),
                      transposed ? toff.data_ptr<int32_t>() : nullptr, transposed ? tslot.data_ptr<int32_t>() : nullptr,
                      cur_stream()));
  return {idx, ln, mask, meta, toff, tslot};
}

std::vector<torch::Tensor> gate_temperature(torch::Tensor x, torch::Tensor idx, torch::Tensor gate_w,
                                            torch::Tensor gate_b, double tmin_tau, double trange_tau) {
  CHECK_INPUT(x);
  CHECK_INPUT(idx);
  CHECK_INPUT(gate_w);
  CHECK_INPUT(gate_b);
  TORCH_CHECK(idx.scalar_type() == torch::kInt32, "idx must be int32");
  TORCH_CHECK(gate_w.scalar_type() == torch::kFloat32 && gate_b.scalar_type() == torch::kFloat32,
              "gate parameters must be float32");
  const c10::cuda::CUDAGuard guard(x.device());
  Dims d = dims(x, idx);
  TORCH_CHECK(gate_w.numel() == d.K && gate_b.numel() >= 1, "gate shape mismatch");
  auto z = f32_opts_like(x, {d.B, d.C});
  auto T = f32_opts_like(x, {d.B, d.E_r});
  ok(moce_gate_temperature(x.data_ptr(), dtype_of(x), nullptr, d.B, d.C, d.HW, idx.data_ptr<int32_t>(), d.E_r, d.K,
                           gate_w.data_ptr<float>(), gate_b.data_ptr<float>(), (float)tmin_tau, (float)trange_tau,
                           z.data_ptr<float>(), T.data_ptr<float>(), cur_stream()));
  return {z, T};
}

torch::Tensor mix(torch::Tensor x, torch::Tensor idx, torch::Tensor ln, torch::Tensor T, torch::Tensor mask,
                  c10::optional<torch::Tensor> out_opt) {
  CHECK_INPUT(x);
  CHECK_INPUT(idx);
  CHECK_INPUT(ln);
  CHECK_INPUT(T);
  CHECK_INPUT(mask);
  TORCH_CHECK(idx.scalar_type() == torch::kInt32 && mask.scalar_type() == torch::kInt32, "idx/mask must be int32");
  TORCH_CHECK(ln.scalar_type() == torch::kFloat32 && T.scalar_type() == torch::kFloat32, "ln/T must be float32");
  const c10::cuda::CUDAGuard guard(x.device());
  Dims d = dims(x, idx);
  TORCH_CHECK(ln.numel() == d.E_r * d.K && T.numel() == d.B * d.E_r && mask.numel() == d.C, "shape mismatch");
  torch::Tensor out;
  if (out_opt.has_value()) {
    out = *out_opt;
    CHECK_INPUT(out);
    TORCH_CHECK(out.scalar_type() == x.scalar_type() && out.numel() == d.B * (d.E_r + 1) * d.HW, "out mismatch");
  } else {
    out = torch::empty({d.B, d.E_r + 1, d.H, d.W}, x.options());
  }
  ok(moce_mix(x.data_ptr(), dtype_of(x), d.B, d.C, d.HW, idx.data_ptr<int32_t>(), ln.data_ptr<float>(),
              T.data_ptr<float>(), d.E_r, d.K, mask.data_ptr<int32_t>(), out.data_ptr(), cur_stream()));
  return out;
}

std::vector<torch::Tensor> backward(torch::Tensor x, torch::Tensor dy, torch::Tensor logits, torch::Tensor idx,
                                    torch::Tensor ln, torch::Tensor mask, torch::Tensor meta, torch::Tensor toff,
                                    torch::Tensor tslot, torch::Tensor gate_w, torch::Tensor gate_b, double tmin_tau,
                                    double trange_tau, torch::Tensor z, torch::Tensor T) {
  for (auto* t : {&x, &dy, &logits, &idx, &ln, &mask, &meta, &toff, &tslot, &gate_w, &gate_b, &z, &T}) {
    CHECK_INPUT(*t);
  }
  TORCH_CHECK(dy.scalar_type() == x.scalar_type(), "dy must have the dtype of x");
  const c10::cuda::CUDAGuard guard(x.device());
  Dims d = dims(x, idx);
  TORCH_CHECK(dy.numel() == d.B * (d.E_r + 1) * d.HW, "dy must be (B, E, H, W)");
  TORCH_CHECK(toff.numel() == d.C + 1 && tslot.numel() == d.E_r * d.K, "transposed lists missing");
  auto dx = torch::empty_like(x);
  auto dL = f32_opts_like(x, {d.E_r, d.C});
  auto dgw = f32_opts_like(x, {1, d.K});
  auto dgb = f32_opts_like(x, {1});
  const size_t wsb = moce_backward_workspace_bytes(d.B, d.C, d.HW, d.E_r, d.K);
  auto ws = torch::empty({(int64_t)wsb + 256}, x.options().dtype(torch::kUInt8));
  void* wsp = (void*)(((uintptr_t)ws.data_ptr() + 255) & ~(uintptr_t)255);
  ok(moce_backward(x.data_ptr(), dy.data_ptr(), dtype_of(x), d.B, d.C, d.HW, logits.data_ptr<float>(),
                   idx.data_ptr<int32_t>(), ln.data_ptr<float>(), mask.data_ptr<int32_t>(), meta.data_ptr<int32_t>(),
                   toff.data_ptr<int32_t>(), tslot.data_ptr<int32_t>(), d.E_r, d.K, gate_w.data_ptr<float>(),
                   gate_b.data_ptr<float>(), (float)tmin_tau, (float)trange_tau, z.data_ptr<float>(),
                   T.data_ptr<float>(), dx.data_ptr(), dL.data_ptr<float>(), dgw.data_ptr<float>(),
                   dgb.data_ptr<float>(), wsp, wsb, cur_stream()));
  return {dx, dL, dgw, dgb};
}


// ------------------------------------------------------- fast path

std::vector<torch::Tensor> schedule_build(torch::Tensor idx, int64_t C, bool balance) {
  CHECK_INPUT(idx);
  TORCH_CHECK(idx.scalar_type() == torch::kInt32 && idx.dim() == 2, "idx must be int32 (E_r, k)");
  const c10::cuda::CUDAGuard guard(idx.device());
  const int64_t E_r = idx.size(0), k = idx.size(1);
  const int64_t G = (E_r + 31) / 32;
  const int64_t S = moce_schedule_steps(k);
  auto i32 = idx.options();
  auto group_expert = torch::empty({G * 32}, i32);
  auto sched = torch::empty({G * S * 32}, i32);
  ok(moce_schedule_build(idx.data_ptr<int32_t>(), E_r, C, k, balance ? 1 : 0, group_expert.data_ptr<int32_t>(),
                         sched.data_ptr<int32_t>(), cur_stream()));
  return {group_expert, sched};
}

bool schedule_supported(int64_t k) { return k >= 1 && moce_schedule_steps(k) <= 52; }

// pass 1 (pool + residual) and pass 2 (gate, temperature, softmax, mix)
std::vector<torch::Tensor> forward_scheduled(torch::Tensor x, torch::Tensor ln, torch::Tensor mask, torch::Tensor meta,
                                             torch::Tensor group_expert, torch::Tensor sched, torch::Tensor gate_w,
                                             torch::Tensor gate_b, double tmin_tau, double trange_tau, bool want_T,
                                             c10::optional<torch::Tensor> out_opt) {
  for (auto* t : {&x, &ln, &mask, &meta, &group_expert, &sched, &gate_w, &gate_b}) {
    CHECK_INPUT(*t);
  }
  TORCH_CHECK(x.dim() == 4 && ln.dim() == 2, "x must be (B, C, H, W), ln (E_r, k)");
  TORCH_CHECK(gate_w.scalar_type() == torch::kFloat32 && gate_b.scalar_type() == torch::kFloat32 &&
                  ln.scalar_type() == torch::kFloat32,
              "gate and ln must be float32");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t B = x.size(0), C = x.size(1), H = x.size(2), W = x.size(3), HW = H * W;
  const int64_t E_r = ln.size(0), k = ln.size(1);
  TORCH_CHECK(mask.numel() == C && gate_w.numel() == k, "shape mismatch");
  torch::Tensor y;
  if (out_opt.has_value()) {
    y = *out_opt;
    CHECK_INPUT(y);
    TORCH_CHECK(y.scalar_type() == x.scalar_type() && y.numel() == B * (E_r + 1) * HW, "out mismatch");
  } else {
    y = torch::empty({B, E_r + 1, H, W}, x.options());
  }
  auto z = f32_opts_like(x, {B, C});
  auto T = want_T ? f32_opts_like(x, {B, E_r}) : f32_opts_like(x, {0});
  ok(moce_pool_residual(x.data_ptr(), dtype_of(x), B, C, HW, mask.data_ptr<int32_t>(), meta.data_ptr<int32_t>(),
                        z.data_ptr<float>(), y.data_ptr(), E_r, cur_stream()));
  ok(moce_mix_scheduled(x.data_ptr(), dtype_of(x), B, C, HW, z.data_ptr<float>(), ln.data_ptr<float>(), E_r, k,
                        group_expert.data_ptr<int32_t>(), sched.data_ptr<int32_t>(), gate_w.data_ptr<float>(),
                        gate_b.data_ptr<float>(), (float)tmin_tau, (float)trange_tau, y.data_ptr(),
                        want_T ? T.data_ptr<float>() : nullptr, cur_stream()));
  return {y, z, T};
}


// Shape, dtype and device checks shared by the fast-path bindings below
// (forward_tc, forward_tc_ep, forward_px, forward_gx): every route tensor
// must match x and idx, and live on x's device, before any pointer reaches
// a kernel.
void check_route_args(const torch::Tensor& x, const torch::Tensor& idx, const torch::Tensor& ln,
                      const torch::Tensor& mask, const torch::Tensor& meta, const torch::Tensor& gate_w,
                      const torch::Tensor& gate_b, const Dims& d) {
  TORCH_CHECK(idx.scalar_type() == torch::kInt32 && ln.scalar_type() == torch::kFloat32, "idx int32, ln float32");
  TORCH_CHECK(mask.scalar_type() == torch::kInt32 && meta.scalar_type() == torch::kInt32, "mask and meta int32");
  TORCH_CHECK(gate_w.scalar_type() == torch::kFloat32 && gate_b.scalar_type() == torch::kFloat32,
              "gate_w and gate_b must be float32");
  TORCH_CHECK(ln.numel() == d.E_r * d.K, "ln must be (E_r, k)");
  TORCH_CHECK(mask.numel() == d.C, "mask must have C entries");
  TORCH_CHECK(meta.numel() >= 2, "meta must have 2 entries");
  TORCH_CHECK(gate_w.numel() == d.K, "gate_w must have k entries");
  TORCH_CHECK(gate_b.numel() >= 1, "gate_b must have one entry");
  for (const torch::Tensor* t : {&idx, &ln, &mask, &meta, &gate_w, &gate_b})
    TORCH_CHECK(t->device() == x.device(), "all tensors must be on the device of x");
}

bool tc_supported(torch::Tensor x, int64_t k) {
  if (!(x.scalar_type() == torch::kBFloat16 || x.scalar_type() == torch::kFloat16) || x.dim() != 4) return false;
  return moce_tc_supported(dtype_of(x), x.size(1), x.size(2) * x.size(3), k) != 0;
}

// pass 1 (pool + residual) and the tensor-core pass 2
std::vector<torch::Tensor> forward_tc(torch::Tensor x, torch::Tensor idx, torch::Tensor ln, torch::Tensor mask,
                                      torch::Tensor meta, torch::Tensor gate_w, torch::Tensor gate_b,
                                      double tmin_tau, double trange_tau, bool want_T,
                                      c10::optional<torch::Tensor> out_opt) {
  for (auto* t : {&x, &idx, &ln, &mask, &meta, &gate_w, &gate_b}) {
    CHECK_INPUT(*t);
  }
  const c10::cuda::CUDAGuard guard(x.device());
  Dims d = dims(x, idx);
  check_route_args(x, idx, ln, mask, meta, gate_w, gate_b, d);
  torch::Tensor y;
  if (out_opt.has_value()) {
    y = *out_opt;
    CHECK_INPUT(y);
    TORCH_CHECK(y.scalar_type() == x.scalar_type() && y.numel() == d.B * (d.E_r + 1) * d.HW, "out mismatch");
    TORCH_CHECK(y.device() == x.device(), "out must be on the device of x");
  } else {
    y = torch::empty({d.B, d.E_r + 1, d.H, d.W}, x.options());
  }
  auto z = f32_opts_like(x, {d.B, d.C});
  auto T = want_T ? f32_opts_like(x, {d.B, d.E_r}) : f32_opts_like(x, {0});
  auto xstage = torch::empty({(int64_t)moce_tc_stage_bytes(d.B, d.C, d.HW)}, x.options().dtype(torch::kUInt8));
  ok(moce_forward_tc(x.data_ptr(), dtype_of(x), d.B, d.C, d.HW, mask.data_ptr<int32_t>(), meta.data_ptr<int32_t>(),
                     idx.data_ptr<int32_t>(), ln.data_ptr<float>(), d.E_r, d.K, gate_w.data_ptr<float>(),
                     gate_b.data_ptr<float>(), (float)tmin_tau, (float)trange_tau, z.data_ptr<float>(),
                     xstage.data_ptr(), y.data_ptr(), want_T ? T.data_ptr<float>() : nullptr, cur_stream()));
  return {y, z, T};
}

// the tensor-core forward with the caller's eval BatchNorm (folded to a
// per-channel scale / shift over the E outputs) and ReLU applied in the store
torch::Tensor forward_tc_ep(torch::Tensor x, torch::Tensor idx, torch::Tensor ln, torch::Tensor mask,
                            torch::Tensor meta, torch::Tensor gate_w, torch::Tensor gate_b, double tmin_tau,
                            double trange_tau, torch::Tensor out_scale, torch::Tensor out_shift, bool relu,
                            c10::optional<torch::Tensor> out_opt) {
  for (auto* t : {&x, &idx, &ln, &mask, &meta, &gate_w, &gate_b, &out_scale, &out_shift}) {
    CHECK_INPUT(*t);
  }
  const c10::cuda::CUDAGuard guard(x.device());
  Dims d = dims(x, idx);
  check_route_args(x, idx, ln, mask, meta, gate_w, gate_b, d);
  TORCH_CHECK(out_scale.scalar_type() == torch::kFloat32 && out_shift.scalar_type() == torch::kFloat32 &&
                  out_scale.numel() == d.E_r + 1 && out_shift.numel() == d.E_r + 1,
              "out_scale / out_shift must be float32 [E]");
  TORCH_CHECK(out_scale.device() == x.device() && out_shift.device() == x.device(),
              "out_scale / out_shift must be on the device of x");
  torch::Tensor y;
  if (out_opt.has_value()) {
    y = *out_opt;
    CHECK_INPUT(y);
    TORCH_CHECK(y.scalar_type() == x.scalar_type() && y.numel() == d.B * (d.E_r + 1) * d.HW, "out mismatch");
    TORCH_CHECK(y.device() == x.device(), "out must be on the device of x");
  } else {
    y = torch::empty({d.B, d.E_r + 1, d.H, d.W}, x.options());
  }
  auto z = f32_opts_like(x, {d.B, d.C});
  auto xstage = torch::empty({(int64_t)moce_tc_stage_bytes(d.B, d.C, d.HW)}, x.options().dtype(torch::kUInt8));
  ok(moce_forward_tc_ep(x.data_ptr(), dtype_of(x), d.B, d.C, d.HW, mask.data_ptr<int32_t>(),
                        meta.data_ptr<int32_t>(), idx.data_ptr<int32_t>(), ln.data_ptr<float>(), d.E_r, d.K,
                        gate_w.data_ptr<float>(), gate_b.data_ptr<float>(), (float)tmin_tau, (float)trange_tau,
                        out_scale.data_ptr<float>(), out_shift.data_ptr<float>(), relu ? 1 : 0, z.data_ptr<float>(),
                        xstage.data_ptr(), y.data_ptr(), nullptr, cur_stream()));
  return y;
}

// a bottleneck's eval BatchNorm (folded to scale / shift per channel), an
// optional residual with its own optional affine, and an optional ReLU in one
// pass; in place when out is x
torch::Tensor bn_act(torch::Tensor x, torch::Tensor scale, torch::Tensor shift, c10::optional<torch::Tensor> r_opt,
                     c10::optional<torch::Tensor> rs_opt, c10::optional<torch::Tensor> rt_opt, bool relu,
                     c10::optional<torch::Tensor> out_opt) {
  CHECK_INPUT(x);
  CHECK_INPUT(scale);
  CHECK_INPUT(shift);
  const c10::cuda::CUDAGuard guard(x.device());
  TORCH_CHECK(x.dim() == 4, "x must be [N, C, H, W]");
  const int64_t N = x.size(0), C = x.size(1), HW = x.size(2) * x.size(3);
  auto f32c = [&](const torch::Tensor& t, const char* name) {
    TORCH_CHECK(t.scalar_type() == torch::kFloat32 && t.numel() == C, name, " must be float32 [C]");
    TORCH_CHECK(t.device() == x.device(), name, " must be on the device of x");
  };
  f32c(scale, "scale");
  f32c(shift, "shift");
  const void* r = nullptr;
  const float* rs = nullptr;
  const float* rt = nullptr;
  if (r_opt.has_value()) {
    CHECK_INPUT(*r_opt);
    TORCH_CHECK(r_opt->sizes() == x.sizes() && r_opt->scalar_type() == x.scalar_type() &&
                    r_opt->device() == x.device(),
                "residual must match x");
    r = r_opt->data_ptr();
  }
  TORCH_CHECK(rs_opt.has_value() == rt_opt.has_value(), "r_scale and r_shift go together");
  if (rs_opt.has_value()) {
    TORCH_CHECK(r != nullptr, "r_scale without a residual");
    CHECK_INPUT(*rs_opt);
    CHECK_INPUT(*rt_opt);
    f32c(*rs_opt, "r_scale");
    f32c(*rt_opt, "r_shift");
    rs = rs_opt->data_ptr<float>();
    rt = rt_opt->data_ptr<float>();
  }
  torch::Tensor y;
  if (out_opt.has_value()) {
    y = *out_opt;
    CHECK_INPUT(y);
    TORCH_CHECK(y.sizes() == x.sizes() && y.scalar_type() == x.scalar_type() && y.device() == x.device(),
                "out must match x");
  } else {
    y = torch::empty_like(x);
  }
  ok(moce_bn_act(x.data_ptr(), dtype_of(x), N, C, HW, scale.data_ptr<float>(), shift.data_ptr<float>(), r, rs, rt,
                 relu ? 1 : 0, y.data_ptr(), cur_stream()));
  return y;
}

bool px_supported(torch::Tensor x, int64_t k) {
  if (x.dim() != 4) return false;
  return moce_px_supported(dtype_of(x), x.size(1), x.size(2) * x.size(3), k) != 0;
}

// pass 1 (pool + residual) and the lanes-over-pixels CUDA-core pass 2
std::vector<torch::Tensor> forward_px(torch::Tensor x, torch::Tensor idx, torch::Tensor ln, torch::Tensor mask,
                                      torch::Tensor meta, torch::Tensor gate_w, torch::Tensor gate_b,
                                      double tmin_tau, double trange_tau, bool want_T,
                                      c10::optional<torch::Tensor> out_opt) {
  for (auto* t : {&x, &idx, &ln, &mask, &meta, &gate_w, &gate_b}) {
    CHECK_INPUT(*t);
  }
  const c10::cuda::CUDAGuard guard(x.device());
  Dims d = dims(x, idx);
  check_route_args(x, idx, ln, mask, meta, gate_w, gate_b, d);
  torch::Tensor y;
  if (out_opt.has_value()) {
    y = *out_opt;
    CHECK_INPUT(y);
    TORCH_CHECK(y.scalar_type() == x.scalar_type() && y.numel() == d.B * (d.E_r + 1) * d.HW, "out mismatch");
    TORCH_CHECK(y.device() == x.device(), "out must be on the device of x");
  } else {
    y = torch::empty({d.B, d.E_r + 1, d.H, d.W}, x.options());
  }
  auto z = f32_opts_like(x, {d.B, d.C});
  auto T = want_T ? f32_opts_like(x, {d.B, d.E_r}) : f32_opts_like(x, {0});
  ok(moce_pool_residual(x.data_ptr(), dtype_of(x), d.B, d.C, d.HW, mask.data_ptr<int32_t>(),
                        meta.data_ptr<int32_t>(), z.data_ptr<float>(), y.data_ptr(), d.E_r, cur_stream()));
  ok(moce_mix_px(x.data_ptr(), dtype_of(x), d.B, d.C, d.HW, z.data_ptr<float>(), idx.data_ptr<int32_t>(),
                 ln.data_ptr<float>(), d.E_r, d.K, gate_w.data_ptr<float>(), gate_b.data_ptr<float>(),
                 (float)tmin_tau, (float)trange_tau, y.data_ptr(), want_T ? T.data_ptr<float>() : nullptr,
                 cur_stream()));
  return {y, z, T};
}

bool gx_supported(torch::Tensor x, int64_t k) {
  if (x.dim() != 4) return false;
  return moce_gx_supported(dtype_of(x), x.size(1), x.size(2) * x.size(3), k) != 0;
}

// pass 1 (pool + residual) and the CUDA-core pass 2 reading X from global memory
std::vector<torch::Tensor> forward_gx(torch::Tensor x, torch::Tensor idx, torch::Tensor ln, torch::Tensor mask,
                                      torch::Tensor meta, torch::Tensor gate_w, torch::Tensor gate_b,
                                      double tmin_tau, double trange_tau, bool want_T,
                                      c10::optional<torch::Tensor> out_opt) {
  for (auto* t : {&x, &idx, &ln, &mask, &meta, &gate_w, &gate_b}) {
    CHECK_INPUT(*t);
  }
  const c10::cuda::CUDAGuard guard(x.device());
  Dims d = dims(x, idx);
  check_route_args(x, idx, ln, mask, meta, gate_w, gate_b, d);
  torch::Tensor y;
  if (out_opt.has_value()) {
    y = *out_opt;
    CHECK_INPUT(y);
    TORCH_CHECK(y.scalar_type() == x.scalar_type() && y.numel() == d.B * (d.E_r + 1) * d.HW, "out mismatch");
    TORCH_CHECK(y.device() == x.device(), "out must be on the device of x");
  } else {
    y = torch::empty({d.B, d.E_r + 1, d.H, d.W}, x.options());
  }
  auto z = f32_opts_like(x, {d.B, d.C});
  auto T = want_T ? f32_opts_like(x, {d.B, d.E_r}) : f32_opts_like(x, {0});
  ok(moce_pool_residual(x.data_ptr(), dtype_of(x), d.B, d.C, d.HW, mask.data_ptr<int32_t>(),
                        meta.data_ptr<int32_t>(), z.data_ptr<float>(), y.data_ptr(), d.E_r, cur_stream()));
  ok(moce_mix_gx(x.data_ptr(), dtype_of(x), d.B, d.C, d.HW, z.data_ptr<float>(), idx.data_ptr<int32_t>(),
                 ln.data_ptr<float>(), d.E_r, d.K, gate_w.data_ptr<float>(), gate_b.data_ptr<float>(),
                 (float)tmin_tau, (float)trange_tau, y.data_ptr(), want_T ? T.data_ptr<float>() : nullptr,
                 cur_stream()));
  return {y, z, T};
}

// ------------------------------------------------------- two-layer gate

void check_mlp(const torch::Tensor& z, const torch::Tensor& w1, const torch::Tensor& b1, const torch::Tensor& w2,
               const torch::Tensor& b2, int64_t C, int64_t E_r) {
  for (const torch::Tensor* t : {&z, &w1, &b1, &w2, &b2}) {
    CHECK_INPUT(*t);
    TORCH_CHECK(t->scalar_type() == torch::kFloat32, "two-layer gate tensors must be float32");
    TORCH_CHECK(t->device() == z.device(), "all tensors must be on one device");
  }
  TORCH_CHECK(w1.dim() == 2 && w1.size(1) == C, "w1 must be (Hd, C)");
  const int64_t Hd = w1.size(0);
  TORCH_CHECK(b1.numel() == Hd && w2.dim() == 2 && w2.size(0) == E_r && w2.size(1) == Hd && b2.numel() == E_r,
              "b1 (Hd), w2 (E_r, Hd), b2 (E_r) expected");
}

// temperatures of the two-layer gate from pooled means z [B, C]: (T, h)
std::vector<torch::Tensor> temperature_mlp(torch::Tensor z, torch::Tensor w1, torch::Tensor b1, torch::Tensor w2,
                                           torch::Tensor b2, double tmin_tau, double trange_tau) {
  TORCH_CHECK(z.dim() == 2, "z must be (B, C)");
  const c10::cuda::CUDAGuard guard(z.device());
  const int64_t B = z.size(0), C = z.size(1), E_r = w2.size(0), Hd = w1.size(0);
  check_mlp(z, w1, b1, w2, b2, C, E_r);
  auto T = f32_opts_like(z, {B, E_r});
  auto h = f32_opts_like(z, {B, Hd});
  ok(moce_temperature_mlp(z.data_ptr<float>(), B, C, Hd, E_r, w1.data_ptr<float>(), b1.data_ptr<float>(),
                          w2.data_ptr<float>(), b2.data_ptr<float>(), (float)tmin_tau, (float)trange_tau,
                          h.data_ptr<float>(), T.data_ptr<float>(), cur_stream()));
  return {T, h};
}

// temperatures of the shared Linear(k,1) gate from pooled means z [B, C]
torch::Tensor temperature(torch::Tensor z, torch::Tensor idx, torch::Tensor gate_w, torch::Tensor gate_b,
                          double tmin_tau, double trange_tau) {
  for (auto* t : {&z, &idx, &gate_w, &gate_b}) {
    CHECK_INPUT(*t);
    TORCH_CHECK(t->device() == z.device(), "all tensors must be on one device");
  }
  TORCH_CHECK(z.dim() == 2 && idx.dim() == 2 && idx.scalar_type() == torch::kInt32 &&
                  z.scalar_type() == torch::kFloat32, "z float32 (B, C), idx int32 (E_r, k)");
  TORCH_CHECK(gate_w.numel() == idx.size(1) && gate_b.numel() >= 1 && gate_w.scalar_type() == torch::kFloat32 &&
                  gate_b.scalar_type() == torch::kFloat32, "gate shape mismatch");
  const c10::cuda::CUDAGuard guard(z.device());
  auto T = f32_opts_like(z, {z.size(0), idx.size(0)});
  ok(moce_temperature(z.data_ptr<float>(), z.size(0), z.size(1), idx.data_ptr<int32_t>(), idx.size(0), idx.size(1),
                      gate_w.data_ptr<float>(), gate_b.data_ptr<float>(), (float)tmin_tau, (float)trange_tau,
                      T.data_ptr<float>(), cur_stream()));
  return T;
}

// tensor-core forward with the two-layer gate: (y, z, T, h)
std::vector<torch::Tensor> forward_tc_mlp(torch::Tensor x, torch::Tensor idx, torch::Tensor ln, torch::Tensor mask,
                                          torch::Tensor meta, torch::Tensor w1, torch::Tensor b1, torch::Tensor w2,
                                          torch::Tensor b2, double tmin_tau, double trange_tau,
                                          c10::optional<torch::Tensor> out_opt) {
  for (auto* t : {&x, &idx, &ln, &mask, &meta}) {
    CHECK_INPUT(*t);
  }
  const c10::cuda::CUDAGuard guard(x.device());
  Dims d = dims(x, idx);
  TORCH_CHECK(idx.scalar_type() == torch::kInt32 && ln.scalar_type() == torch::kFloat32 && ln.numel() == d.E_r * d.K &&
                  mask.numel() == d.C && meta.numel() >= 2, "route tensors do not match x");
  auto z = f32_opts_like(x, {d.B, d.C});
  check_mlp(z, w1, b1, w2, b2, d.C, d.E_r);
  torch::Tensor y;
  if (out_opt.has_value()) {
    y = *out_opt;
    CHECK_INPUT(y);
    TORCH_CHECK(y.scalar_type() == x.scalar_type() && y.numel() == d.B * (d.E_r + 1) * d.HW, "out mismatch");
  } else {
    y = torch::empty({d.B, d.E_r + 1, d.H, d.W}, x.options());
  }
  const int64_t Hd = w1.size(0);
  auto T = f32_opts_like(x, {d.B, d.E_r});
  auto h = f32_opts_like(x, {d.B, Hd});
  auto xstage = torch::empty({(int64_t)moce_tc_stage_bytes(d.B, d.C, d.HW)}, x.options().dtype(torch::kUInt8));
  ok(moce_forward_tc_mlp(x.data_ptr(), dtype_of(x), d.B, d.C, d.HW, mask.data_ptr<int32_t>(),
                         meta.data_ptr<int32_t>(), idx.data_ptr<int32_t>(), ln.data_ptr<float>(), d.E_r, d.K, Hd,
                         w1.data_ptr<float>(), b1.data_ptr<float>(), w2.data_ptr<float>(), b2.data_ptr<float>(),
                         (float)tmin_tau, (float)trange_tau, z.data_ptr<float>(), h.data_ptr<float>(),
                         xstage.data_ptr(), y.data_ptr(), T.data_ptr<float>(), cur_stream()));
  return {y, z, T, h};
}

// pass 1 of the CUDA-core paths: (y with the residual row written, z)
std::vector<torch::Tensor> pool_residual(torch::Tensor x, torch::Tensor mask, torch::Tensor meta, int64_t E_r,
                                         c10::optional<torch::Tensor> out_opt) {
  for (auto* t : {&x, &mask, &meta}) {
    CHECK_INPUT(*t);
    TORCH_CHECK(t->device() == x.device(), "all tensors must be on one device");
  }
  TORCH_CHECK(x.dim() == 4 && mask.numel() == x.size(1) && meta.numel() >= 2 && mask.scalar_type() == torch::kInt32 &&
                  meta.scalar_type() == torch::kInt32, "x (B, C, H, W), mask int32 [C], meta int32 [2]");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t B = x.size(0), C = x.size(1), H = x.size(2), W = x.size(3);
  torch::Tensor y;
  if (out_opt.has_value()) {
    y = *out_opt;
    CHECK_INPUT(y);
    TORCH_CHECK(y.scalar_type() == x.scalar_type() && y.numel() == B * (E_r + 1) * H * W, "out mismatch");
  } else {
    y = torch::empty({B, E_r + 1, H, W}, x.options());
  }
  auto z = f32_opts_like(x, {B, C});
  ok(moce_pool_residual(x.data_ptr(), dtype_of(x), B, C, H * W, mask.data_ptr<int32_t>(), meta.data_ptr<int32_t>(),
                        z.data_ptr<float>(), y.data_ptr(), E_r, cur_stream()));
  return {y, z};
}

// the routed experts of y from given temperatures T [B, E_r]: the
// lanes-over-pixels mix, the global-memory mix, or the general mix (which
// also rewrites the residual row), by shape
void mix_given_t(torch::Tensor x, torch::Tensor idx, torch::Tensor ln, torch::Tensor mask, torch::Tensor T,
                 torch::Tensor y) {
  for (auto* t : {&x, &idx, &ln, &mask, &T, &y}) {
    CHECK_INPUT(*t);
    TORCH_CHECK(t->device() == x.device(), "all tensors must be on one device");
  }
  const c10::cuda::CUDAGuard guard(x.device());
  Dims d = dims(x, idx);
  TORCH_CHECK(idx.scalar_type() == torch::kInt32 && ln.scalar_type() == torch::kFloat32 && ln.numel() == d.E_r * d.K &&
                  mask.numel() == d.C && T.scalar_type() == torch::kFloat32 && T.numel() == d.B * d.E_r,
              "route tensors or T do not match x");
  TORCH_CHECK(y.scalar_type() == x.scalar_type() && y.numel() == d.B * (d.E_r + 1) * d.HW, "out mismatch");
  const int dt = dtype_of(x);
  if (moce_px_supported(dt, d.C, d.HW, d.K)) {
    ok(moce_mix_px_t(x.data_ptr(), dt, d.B, d.C, d.HW, T.data_ptr<float>(), idx.data_ptr<int32_t>(),
                     ln.data_ptr<float>(), d.E_r, d.K, y.data_ptr(), cur_stream()));
  } else if (moce_gx_supported(dt, d.C, d.HW, d.K)) {
    ok(moce_mix_gx_t(x.data_ptr(), dt, d.B, d.C, d.HW, T.data_ptr<float>(), idx.data_ptr<int32_t>(),
                     ln.data_ptr<float>(), d.E_r, d.K, y.data_ptr(), cur_stream()));
  } else {
    ok(moce_mix(x.data_ptr(), dt, d.B, d.C, d.HW, idx.data_ptr<int32_t>(), ln.data_ptr<float>(),
                T.data_ptr<float>(), d.E_r, d.K, mask.data_ptr<int32_t>(), y.data_ptr(), cur_stream()));
  }
}

// pass 1 and the mix from given temperatures T [B, E_r]: the tensor-core
// path (operand staging, tcgen05 mix) where it takes the input, else the
// CUDA-core pass 1 and mix_given_t; returns y
torch::Tensor forward_given_t(torch::Tensor x, torch::Tensor idx, torch::Tensor ln, torch::Tensor mask,
                              torch::Tensor meta, torch::Tensor T, c10::optional<torch::Tensor> out_opt) {
  for (auto* t : {&x, &idx, &ln, &mask, &meta, &T}) {
    CHECK_INPUT(*t);
    TORCH_CHECK(t->device() == x.device(), "all tensors must be on one device");
  }
  const c10::cuda::CUDAGuard guard(x.device());
  Dims d = dims(x, idx);
  TORCH_CHECK(idx.scalar_type() == torch::kInt32 && ln.scalar_type() == torch::kFloat32 && ln.numel() == d.E_r * d.K &&
                  mask.numel() == d.C && meta.numel() >= 2 && T.scalar_type() == torch::kFloat32 &&
                  T.numel() == d.B * d.E_r, "route tensors or T do not match x");
  torch::Tensor y;
  if (out_opt.has_value()) {
    y = *out_opt;
    CHECK_INPUT(y);
    TORCH_CHECK(y.scalar_type() == x.scalar_type() && y.numel() == d.B * (d.E_r + 1) * d.HW, "out mismatch");
  } else {
    y = torch::empty({d.B, d.E_r + 1, d.H, d.W}, x.options());
  }
  auto z = f32_opts_like(x, {d.B, d.C});
  const int dt = dtype_of(x);
  if (tc_supported(x, d.K)) {
    auto xstage = torch::empty({(int64_t)moce_tc_stage_bytes(d.B, d.C, d.HW)}, x.options().dtype(torch::kUInt8));
    ok(moce_pool_stage(x.data_ptr(), dt, d.B, d.C, d.HW, mask.data_ptr<int32_t>(), meta.data_ptr<int32_t>(),
                       z.data_ptr<float>(), y.data_ptr(), d.E_r, xstage.data_ptr(), cur_stream()));
    ok(moce_mix_tc_t(xstage.data_ptr(), dt, d.B, d.C, d.HW, T.data_ptr<float>(), idx.data_ptr<int32_t>(),
                     ln.data_ptr<float>(), d.E_r, d.K, y.data_ptr(), cur_stream()));
  } else {
    ok(moce_pool_residual(x.data_ptr(), dt, d.B, d.C, d.HW, mask.data_ptr<int32_t>(), meta.data_ptr<int32_t>(),
                          z.data_ptr<float>(), y.data_ptr(), d.E_r, cur_stream()));
    mix_given_t(x, idx, ln, mask, T, y);
  }
  return y;
}

// backward from given temperatures: (dx, dL, dT)
std::vector<torch::Tensor> backward_t(torch::Tensor x, torch::Tensor dy, torch::Tensor logits, torch::Tensor idx,
                                      torch::Tensor ln, torch::Tensor mask, torch::Tensor meta, torch::Tensor toff,
                                      torch::Tensor tslot, torch::Tensor T) {
  for (auto* t : {&x, &dy, &logits, &idx, &ln, &mask, &meta, &toff, &tslot, &T}) {
    CHECK_INPUT(*t);
    TORCH_CHECK(t->device() == x.device(), "all tensors must be on one device");
  }
  const c10::cuda::CUDAGuard guard(x.device());
  Dims d = dims(x, idx);
  TORCH_CHECK(dy.scalar_type() == x.scalar_type() && dy.numel() == d.B * (d.E_r + 1) * d.HW, "dy must be (B, E, H, W)");
  TORCH_CHECK(toff.numel() == d.C + 1 && tslot.numel() == d.E_r * d.K, "transposed lists missing");
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.numel() == d.E_r * d.C && T.numel() == d.B * d.E_r &&
                  T.scalar_type() == torch::kFloat32 && ln.numel() == d.E_r * d.K && mask.numel() == d.C,
              "shape mismatch");
  auto dx = torch::empty_like(x);
  auto dL = f32_opts_like(x, {d.E_r, d.C});
  auto dT = f32_opts_like(x, {d.B, d.E_r});
  const size_t nb = moce_backward_workspace_bytes(d.B, d.C, d.HW, d.E_r, d.K);
  auto ws = torch::empty({(int64_t)nb + 256}, x.options().dtype(torch::kUInt8));
  void* wp = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(ws.data_ptr()) + 255) & ~uintptr_t(255));
  ok(moce_backward_t(x.data_ptr(), dy.data_ptr(), dtype_of(x), d.B, d.C, d.HW, logits.data_ptr<float>(),
                     idx.data_ptr<int32_t>(), ln.data_ptr<float>(), mask.data_ptr<int32_t>(), meta.data_ptr<int32_t>(),
                     toff.data_ptr<int32_t>(), tslot.data_ptr<int32_t>(), d.E_r, d.K, T.data_ptr<float>(),
                     dx.data_ptr(), dL.data_ptr<float>(), dT.data_ptr<float>(), wp, nb, cur_stream()));
  return {dx, dL, dT};
}

// ------------------------------------------------------- auxiliary loss

torch::Tensor aux_workspace(const torch::Tensor& logits, void** wp, size_t* nb) {
  *nb = moce_aux_workspace_bytes(logits.size(0), logits.size(1));
  auto ws = torch::empty({(int64_t)*nb + 256}, logits.options().dtype(torch::kUInt8));
  *wp = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(ws.data_ptr()) + 255) & ~uintptr_t(255));
  return ws;
}

void check_logits(const torch::Tensor& logits) {
  CHECK_INPUT(logits);
  TORCH_CHECK(logits.dim() == 2 && logits.scalar_type() == torch::kFloat32, "logits must be float32 (E_r, C)");
}

// the auxiliary loss as a 0-d float32 tensor
torch::Tensor aux_loss(torch::Tensor logits, double tau, double wb, double ws_, double wd, double log_target) {
  check_logits(logits);
  const c10::cuda::CUDAGuard guard(logits.device());
  void* wp;
  size_t nb;
  auto ws = aux_workspace(logits, &wp, &nb);
  auto out = torch::empty({}, logits.options());
  ok(moce_aux_loss(logits.data_ptr<float>(), logits.size(0), logits.size(1), (float)tau, (float)wb, (float)ws_,
                   (float)wd, (float)log_target, out.data_ptr<float>(), wp, nb, cur_stream()));
  return out;
}

// grad * d aux / d logits
torch::Tensor aux_loss_backward(torch::Tensor logits, double tau, double wb, double ws_, double wd, double log_target,
                                torch::Tensor grad) {
  check_logits(logits);
  CHECK_INPUT(grad);
  TORCH_CHECK(grad.numel() == 1 && grad.scalar_type() == torch::kFloat32 && grad.device() == logits.device(),
              "grad must be one float32 on the device of logits");
  const c10::cuda::CUDAGuard guard(logits.device());
  void* wp;
  size_t nb;
  auto ws = aux_workspace(logits, &wp, &nb);
  auto dL = torch::empty_like(logits);
  ok(moce_aux_loss_backward(logits.data_ptr<float>(), logits.size(0), logits.size(1), (float)tau, (float)wb,
                            (float)ws_, (float)wd, (float)log_target, grad.data_ptr<float>(), dL.data_ptr<float>(), wp,
                            nb, cur_stream()));
  return dL;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  // reference surface (moce_layer_cuda.cpp:117-138)
  m.def("moce_pool", &py_moce_pool, "Channel average pool (B,C,H,W) -> [(B,C)]");
  m.def("fused_moce_forward_dynamic_temp", &fused_moce_forward_dynamic_temp,
        "Weighted sum + residual with caller weights (B,E_routed,K); returns [out]");
  m.def("fused_moce_gate_route", &fused_moce_gate_route, "Pooled given: gate+temperature+softmax+mix; returns [out]");
  m.def("fused_moce_gate_route_timed", &fused_moce_gate_route_timed,
        "Timed fused_moce_gate_route; returns [out, kernel_ms[pass1, pass2]]");
  m.def("fused_moce_gate_route_section_timed", &fused_moce_gate_route_section_timed,
        "Section-timed fused_moce_gate_route; returns [out, section_us[pass1, 0, 0, pass2]]");
  m.def("fused_moce_gate_route_all", &fused_moce_gate_route_all, "Pool+gate+temperature+softmax+mix; returns [out]");
  m.def("fused_moce_gate_route_all_timed", &fused_moce_gate_route_all_timed,
        "Timed fused_moce_gate_route_all; returns [out, kernel_ms[pass1, pass2, 0], section_us]");
  // native pipeline
  m.def("route_build", &route_build, "Top-k supports, normalised logits, mask, meta, transposed lists",
        py::arg("logits"), py::arg("k"), py::arg("transposed") = true);
  m.def("gate_temperature", &gate_temperature, "Pass 1: (z, T)");
  m.def("mix", &mix, "Pass 2: softmax + gather-mix + residual", py::arg("x"), py::arg("idx"), py::arg("ln"),
        py::arg("T"), py::arg("mask"), py::arg("out") = py::none());
  m.def("backward", &backward, "Layer backward: (dx, dL, dgate_w, dgate_b)");
  m.def("schedule_build", &schedule_build, "Warp groups and bank-conflict-free support schedule",
        py::arg("idx"), py::arg("C"), py::arg("balance") = true);
  m.def("schedule_supported", &schedule_supported, "Whether k fits the scheduled mix kernel");
  m.def("forward_scheduled", &forward_scheduled, "Fast path: (y, z, T)", py::arg("x"), py::arg("ln"), py::arg("mask"),
        py::arg("meta"), py::arg("group_expert"), py::arg("sched"), py::arg("gate_w"), py::arg("gate_b"),
        py::arg("tmin_tau"), py::arg("trange_tau"), py::arg("want_T") = false, py::arg("out") = py::none());
  m.def("tc_supported", &tc_supported, "Whether the tensor-core mix takes this input");
  m.def("bn_act", &bn_act,
        "y = act(x * scale + shift + residual * r_scale + r_shift): a folded eval BatchNorm with an optional "
        "residual (its own optional affine) and ReLU, one pass over NCHW",
        py::arg("x"), py::arg("scale"), py::arg("shift"), py::arg("residual") = py::none(),
        py::arg("r_scale") = py::none(), py::arg("r_shift") = py::none(), py::arg("relu") = true,
        py::arg("out") = py::none());
  m.def("forward_tc_ep", &forward_tc_ep,
        "Tensor-core forward with a folded BatchNorm (scale, shift per output channel) and ReLU on the outputs",
        py::arg("x"), py::arg("idx"), py::arg("ln"), py::arg("mask"), py::arg("meta"), py::arg("gate_w"),
        py::arg("gate_b"), py::arg("tmin_tau"), py::arg("trange_tau"), py::arg("out_scale"), py::arg("out_shift"),
        py::arg("relu"), py::arg("out") = py::none());
  m.def("forward_tc", &forward_tc, "Pool + residual, then the tensor-core mix: (y, z, T)", py::arg("x"),
        py::arg("idx"), py::arg("ln"), py::arg("mask"), py::arg("meta"), py::arg("gate_w"), py::arg("gate_b"),
        py::arg("tmin_tau"), py::arg("trange_tau"), py::arg("want_T") = false, py::arg("out") = py::none());
  m.def("gx_supported", &gx_supported, "Whether the global-memory CUDA-core mix takes this input");
  m.def("forward_gx", &forward_gx, "Pool + residual, then the CUDA-core mix reading X from global memory: (y, z, T)",
        py::arg("x"), py::arg("idx"), py::arg("ln"), py::arg("mask"), py::arg("meta"), py::arg("gate_w"),
        py::arg("gate_b"), py::arg("tmin_tau"), py::arg("trange_tau"), py::arg("want_T") = false,
        py::arg("out") = py::none());
  m.def("px_supported", &px_supported, "Whether the lanes-over-pixels CUDA-core mix takes this input");
  m.def("forward_px", &forward_px, "Pool + residual, then the lanes-over-pixels CUDA-core mix: (y, z, T)",
        py::arg("x"), py::arg("idx"), py::arg("ln"), py::arg("mask"), py::arg("meta"), py::arg("gate_w"),
        py::arg("gate_b"), py::arg("tmin_tau"), py::arg("trange_tau"), py::arg("want_T") = false,
        py::arg("out") = py::none());
  m.def("version", []() { return std::string(moce_version()); });
  m.def("temperature", &temperature, "Linear-gate temperatures T [B, E_r] from pooled means z [B, C]");
  m.def("temperature_mlp", &temperature_mlp, "Two-layer-gate temperatures from pooled means: (T, h)");
  m.def("forward_tc_mlp", &forward_tc_mlp, "Tensor-core forward with the two-layer gate: (y, z, T, h)",
        py::arg("x"), py::arg("idx"), py::arg("ln"), py::arg("mask"), py::arg("meta"), py::arg("w1"), py::arg("b1"),
        py::arg("w2"), py::arg("b2"), py::arg("tmin_tau"), py::arg("trange_tau"), py::arg("out") = py::none());
  m.def("pool_residual", &pool_residual, "Pass 1 of the CUDA-core paths: (y with the residual row, z)",
        py::arg("x"), py::arg("mask"), py::arg("meta"), py::arg("E_r"), py::arg("out") = py::none());
  m.def("mix_given_t", &mix_given_t, "Routed experts of y from given temperatures (CUDA-core mix)");
  m.def("forward_given_t", &forward_given_t, "Pass 1 and the mix from given temperatures: y", py::arg("x"),
        py::arg("idx"), py::arg("ln"), py::arg("mask"), py::arg("meta"), py::arg("T"), py::arg("out") = py::none());
  m.def("backward_t", &backward_t, "Backward from given temperatures: (dx, dL, dT)");
  m.def("aux_loss", &aux_loss, "Auxiliary (coverage) loss of the routing logits, a 0-d tensor");
  m.def("aux_loss_backward", &aux_loss_backward, "grad * d aux / d logits");
  m.def("tc_fault", [](bool clear) {
    int flag = 0;
    ok(moce_tc_fault(&flag, clear ? 1 : 0));
    return flag;
  }, "Device flag set when a bounded wait inside a tensor-core kernel ran out (synchronises)",
        py::arg("clear") = true);
  m.def("tc_fault_info", [](bool clear) {
    std::vector<int64_t> v(14, 0);
    ok(moce_tc_fault_info(v.data(), 14, clear ? 1 : 0));
    return v;
  }, "Where the first bounded wait that ran out gave up (14 integers, see moce_tc_fault_info)",
        py::arg("clear") = true);
}
