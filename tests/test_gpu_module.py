"""GPU tests of the nn.Module surface and of the ``moce_fixed.moce_cuda``
binding (the reference module path), against the reference golden vectors.

The layer is built the way ``tests/golden/make_golden.py`` builds the
reference one (sampling_factor=1, then E, the logits and the gate forced to
the case's values).  Tolerances as in ``test_gpu_parity.py``.
"""
import os

import numpy as np
import pytest
import torch

from inputs import CASES, make_inputs
from moce_thesis_b200 import MoCE, native

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
FULL = [n for n, c in CASES.items() if not c.get("summary")]
DEV = "cuda:0"


def load(name):
    return dict(np.load(os.path.join(GOLD, f"{name}.npz")))


def close(a, b, rtol=1e-5, floor=1e-6):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return bool(np.all(np.abs(a - b) <= rtol * np.abs(b) + floor * max(np.abs(b).max(), 1e-30)))


def maxrel(a, b, floor=1e-3):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), floor))


def build_layer(case, t):
    C, E, k = case["C"], case["E"], case["k"]
    m = MoCE(in_channels=C, sampling_factor=1, k=k, tau=case["tau"], temp_min=case["tmin"], temp_max=case["tmax"])
    m.num_experts = E
    m.routing_logits = torch.nn.Parameter(t["L"].clone())
    m.target_experts_per_channel = (max(E - 1, 1) * k) / max(float(C), 1.0)
    with torch.no_grad():
        m.gate.weight.copy_(t["gate_w"])
        m.gate.bias.copy_(t["gate_b"])
    return m.to(DEV)


@pytest.mark.parametrize("name", FULL)
def test_module_train_forward_backward(name):
    g, c = load(name), CASES[name]
    t = make_inputs(c)
    m = build_layer(c, t)
    m.train()
    x = t["X"].to(DEV).requires_grad_(True)
    y = m(x)
    assert close(y.detach().cpu().numpy(), g["Y_train"])
    assert abs(float(m.aux_loss) - float(g["aux"])) <= 1e-5 * max(abs(float(g["aux"])), 1e-6)
    (y * t["dY"].to(DEV)).sum().backward()
    assert maxrel(x.grad.cpu().numpy(), g["dX"]) < 1e-5
    assert maxrel(m.gate.weight.grad.cpu().numpy(), g["dgate_w"]) < 1e-5
    assert maxrel(m.gate.bias.grad.cpu().numpy(), g["dgate_b"]) < 1e-5
    # routing-logit gradient = main path + auxiliary loss (reference autograd of both)
    m.zero_grad()
    y = m(t["X"].to(DEV))
    ((y * t["dY"].to(DEV)).sum() + m.aux_loss).backward()
    assert maxrel(m.routing_logits.grad.cpu().numpy(), g["dL"] + g["dL_aux"]) < 1e-5


@pytest.mark.parametrize("name", FULL)
def test_module_eval(name):
    g, c = load(name), CASES[name]
    t = make_inputs(c)
    m = build_layer(c, t).eval()
    with pytest.raises(RuntimeError, match="eval cache not built"):
        m(t["X"].to(DEV))
    m.build_eval_cache()
    np.testing.assert_array_equal(m.cached_indices.cpu().numpy(), g["idx"])
    assert m.cached_indices.dtype == torch.int64
    np.testing.assert_array_equal(m.cached_mask_int.cpu().numpy(), g["mask"])
    with torch.no_grad():
        y = m(t["X"].to(DEV))
        yb = m(t["X"].to(DEV, torch.bfloat16))
    assert close(y.cpu().numpy(), g["Y_eval"])
    assert yb.dtype == torch.bfloat16
    assert close(yb.float().cpu().numpy(), g["Y_eval"], rtol=2e-2, floor=1e-2)


def test_state_dict_keys_match_reference_layout():
    m = MoCE(in_channels=32, sampling_factor=2, k=4).to(DEV)
    assert set(m.state_dict()) == {"routing_logits", "gate.weight", "gate.bias"}
    m.eval()
    m.build_eval_cache()
    # after the cache build the reference state_dict also carries these
    assert {"cached_indices", "cached_selected_logits_norm", "cached_gate_bias"} <= set(m.state_dict())


@pytest.mark.parametrize("name", ["small_resid", "covered_odd", "k40"])
def test_binding_reference_functions(name):
    """The seven reference entry points, called the way MoCE.py would."""
    g, c = load(name), CASES[name]
    mc = native()
    X = torch.from_numpy(g["X"]).to(DEV)
    idx64 = torch.from_numpy(g["idx"]).to(DEV)
    w = torch.from_numpy(g["weights"]).to(DEV)
    mask = torch.from_numpy(g["mask"]).to(DEV)
    ln = torch.from_numpy(g["ln"]).to(DEV)
    gw = torch.from_numpy(g["gate_w"].reshape(-1)).to(DEV)
    gb = torch.from_numpy(g["gate_b"]).to(DEV)
    out, = mc.fused_moce_forward_dynamic_temp(X, idx64, w, mask)
    assert close(out.cpu().numpy(), g["Y_eval"])
    pooled, = mc.moce_pool(X)
    assert close(pooled.cpu().numpy(), X.mean((2, 3)).cpu().numpy())
    args = (idx64, ln, gw, gb, mask, c["tmin"], c["tmax"], c["tau"])
    for fn in (mc.fused_moce_gate_route, mc.fused_moce_gate_route_timed, mc.fused_moce_gate_route_section_timed):
        res = fn(X, pooled, *args)
        assert close(res[0].cpu().numpy(), g["Y_eval"]), fn.__name__
    for fn in (mc.fused_moce_gate_route_all, mc.fused_moce_gate_route_all_timed):
        res = fn(X, *args)
        assert close(res[0].cpu().numpy(), g["Y_eval"]), fn.__name__
    _, kt = mc.fused_moce_gate_route_timed(X, pooled, *args)
    assert kt.shape == (2,) and float(kt.min()) >= 0.0
    _, kt3, sec = mc.fused_moce_gate_route_all_timed(X, *args)
    assert kt3.shape == (3,) and sec.shape == (4,)


def test_binding_errors_match_reference_checks():
    mc = native()
    X = torch.rand(2, 8, 3, 3, device=DEV)
    idx = torch.zeros(3, 2, dtype=torch.int64, device=DEV)
    mask = torch.zeros(8, dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="must be CUDA"):
        mc.fused_moce_forward_dynamic_temp(X.cpu(), idx, torch.rand(2, 3, 2, device=DEV), mask)
    with pytest.raises(RuntimeError, match="weights must be"):
        mc.fused_moce_forward_dynamic_temp(X, idx, torch.rand(2, 3, 3, device=DEV), mask)
    with pytest.raises(RuntimeError, match="mask_int must be int32"):
        mc.fused_moce_forward_dynamic_temp(X, idx, torch.rand(2, 3, 2, device=DEV), mask.long())


@pytest.mark.parametrize("dtype,B,C,Hh,E,k,slices", [
    (torch.bfloat16, 37, 128, 7, 200, 16, 8),    # runs of 5 samples, the last one of 2; tensor-core path
    (torch.float32, 9, 64, 14, 70, 8, 4),        # fp32: lanes-over-pixels path
    (torch.bfloat16, 3, 64, 28, 40, 8, 8),       # fewer samples than runs
])
def test_forward_host_matches_forward_eval(dtype, B, C, Hh, E, k, slices):
    """MoCE.forward_host (pinned host X in, host Y out, copies and passes
    overlapped on three streams) gives the bits of forward_eval on the
    device, on two calls in a row (buffers reused) and after a call of
    another batch size (buffers replaced)."""
    gen = torch.Generator().manual_seed(B + C)
    torch.manual_seed(B)
    m = MoCE(in_channels=C, sampling_factor=1, k=k, temp_min=0.1, temp_max=10.0)
    m.num_experts = E
    m.routing_logits = torch.nn.Parameter(torch.randn(E - 1, C, generator=gen))
    m = m.to(DEV).eval()
    m.build_eval_cache()
    with torch.no_grad():
        for b in (B, B, B + 1, B):
            xh = torch.randn(b, C, Hh, Hh, generator=gen).abs().to(dtype).pin_memory()
            ref = m(xh.to(DEV)).cpu()
            yh = m.forward_host(xh, slices=slices)
            torch.cuda.current_stream().synchronize()
            assert yh.is_pinned() and yh.shape == ref.shape and yh.dtype == dtype
            assert torch.equal(yh, ref)


@pytest.mark.parametrize("dtype,C,Hh,E,k", [
    (torch.bfloat16, 128, 14, 64, 8),    # tensor-core path: epilogue in the kernels
    (torch.float32, 64, 7, 40, 8),       # fp32: forward_eval, then torch BatchNorm and ReLU
])
def test_forward_eval_bn_relu(dtype, C, Hh, E, k):
    """MoCE.forward_eval_bn_relu equals relu(bn(forward_eval(x))) for an
    eval-mode BatchNorm2d (bf16 / fp32 tolerances)."""
    gen = torch.Generator().manual_seed(C)
    torch.manual_seed(C)
    m = MoCE(in_channels=C, sampling_factor=1, k=k, temp_min=0.1, temp_max=10.0)
    m.num_experts = E
    m.routing_logits = torch.nn.Parameter(torch.randn(E - 1, C, generator=gen))
    m = m.to(DEV).eval()
    m.build_eval_cache()
    bn = torch.nn.BatchNorm2d(E).to(DEV).eval()
    with torch.no_grad():
        bn.weight.copy_(torch.rand(E, generator=gen) + 0.5)
        bn.bias.copy_(torch.randn(E, generator=gen) * 0.3)
        bn.running_mean.copy_(torch.randn(E, generator=gen) * 0.1)
        bn.running_var.copy_(torch.rand(E, generator=gen) + 0.5)
        x = torch.randn(4, C, Hh, Hh, generator=gen).abs().to(DEV, dtype)
        ref = torch.relu(bn(m(x).float())).cpu().numpy()
        got = m.forward_eval_bn_relu(x, bn).float().cpu().numpy()
    tol = (1e-2, 1e-3) if dtype != torch.float32 else (1e-5, 1e-6)
    assert close(got, ref, *tol), maxrel(got, ref)


def test_resnet_inference_paths_agree():
    """ResNet-50 + MoCE on a small batch: with MoCE -> bn1 -> relu1 fused in
    the MoCE kernels the logits equal the reference-order eval output within
    bf16 tolerance (relative to the largest logit)."""
    from moce_thesis_b200 import resnet
    torch.manual_seed(0)
    kcfg = [[4, 16, 16], [16, 32, 32, 32], [32, 64, 64, 64, 64, 64], [64, 128, 128]]
    m = resnet.resnet50_moce_projection(dataset="imagenet", num_classes=1000, k=kcfg).to(DEV, torch.bfloat16).eval()
    # BatchNorms with non-trivial statistics, so that the epilogue is exercised
    g = torch.Generator().manual_seed(1)
    with torch.no_grad():
        for mod in m.modules():
            if isinstance(mod, torch.nn.BatchNorm2d):
                n = mod.num_features
                mod.weight.copy_(torch.rand(n, generator=g) * 0.5 + 0.75)
                mod.bias.copy_(torch.randn(n, generator=g) * 0.05)
                mod.running_mean.copy_(torch.randn(n, generator=g) * 0.05)
                mod.running_var.copy_(torch.rand(n, generator=g) * 0.5 + 0.75)
    resnet.build_moce_cache(m)
    x = torch.randn(4, 3, 224, 224, generator=g).to(DEV, torch.bfloat16)
    with torch.no_grad():
        resnet.set_fused_epilogue(m, False)
        ref = m(x).float()
        resnet.set_fused_epilogue(m, True)
        fused = m(x).float()
    scale = ref.abs().max().item()
    assert (fused - ref).abs().max().item() <= 5e-2 * scale


def test_resnet_forward_replays_as_cuda_graph():
    """The eval forward of ResNet-50 + MoCE (tensor-core, lanes-over-pixels
    and CTA-pair kernels, the fused epilogue) captured once as a CUDA graph
    and replayed gives the eager output bit for bit."""
    from moce_thesis_b200 import resnet
    torch.manual_seed(0)
    kcfg = [[4, 16, 16], [16, 32, 32, 32], [32, 64, 64, 64, 64, 64], [64, 128, 128]]
    m = resnet.resnet50_moce_projection(dataset="imagenet", num_classes=1000, k=kcfg).to(DEV, torch.bfloat16).eval()
    resnet.build_moce_cache(m)
    x = torch.randn(4, 3, 224, 224, generator=torch.Generator().manual_seed(2)).to(DEV, torch.bfloat16)
    with torch.no_grad():
        want = m(x).clone()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            m(x)
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = m(x)
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize()
        got = out.clone()
        del g
    assert torch.equal(got, want)
