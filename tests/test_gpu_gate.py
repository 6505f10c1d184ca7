"""GPU parity of the temperature kernels and the opt-in two-layer gate.

* moce_temperature (the reference's shared Linear(k,1) gate, MoCE.py:216-218)
  against the oracle's temperatures, fp32 within 1e-5;
* moce_temperature_mlp (two-layer gate C -> C/16 -> E-1, no reference
  counterpart) against the oracle's restatement, T and the hidden layer;
* the layer with the two-layer gate, eval (the fused tensor-core chain and
  the CUDA-core paths) and train (forward, then dX, dL and the gate's
  gradients through autograd from the native given-temperature backward),
  against the oracle: fp32 1e-5, bf16 1e-2, gradients 1e-5 of their largest
  magnitude;
* moce_backward_t's dT against the oracle.
"""
import numpy as np
import pytest
import torch

from oracle import moce_oracle as O
import capi_helpers as H

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
TMIN, TMAX, TAU = 0.1, 10.0, 1.0


def close(a, b, rtol, floor):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return bool(np.all(np.abs(a - b) <= rtol * np.abs(b) + floor * max(np.abs(b).max(), 1e-30)))


def maxrel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def mlp_params(C, E, seed):
    g = torch.Generator().manual_seed(seed)
    Hd = max(1, C // 16)
    w1 = torch.randn(Hd, C, generator=g) * (2.0 / C) ** 0.5
    b1 = torch.randn(Hd, generator=g) * 0.1
    w2 = torch.randn(E - 1, Hd, generator=g) * (2.0 / Hd) ** 0.5
    b2 = torch.randn(E - 1, generator=g) * 0.1
    return w1, b1, w2, b2


@pytest.mark.parametrize("B,C,E,k", [(256, 512, 2048, 32), (7, 64, 300, 8), (3, 100, 130, 40), (2, 2048, 512, 128)])
def test_linear_temperature_kernel(B, C, E, k):
    g = torch.Generator().manual_seed(B + C + k)
    z = torch.rand(B, C, generator=g)
    L = torch.randn(E - 1, C, generator=g)
    gw = torch.rand(k, generator=g) - 0.5
    gb = torch.randn(1, generator=g) * 0.1
    r = H.route_build(L.to(DEV), k, transposed=False)
    T = H.temperature(z.to(DEV), r["idx"], gw.to(DEV), gb.to(DEV), TMIN * TAU, (TMAX - TMIN) * TAU)
    want, _ = O.gate_temperature(z.numpy(), r["idx"].long().cpu().numpy(), gw.numpy(), gb.numpy(), TMIN, TMAX, TAU)
    assert close(T.cpu().numpy(), want, 1e-5, 1e-6), maxrel(T.cpu().numpy(), want)


@pytest.mark.parametrize("B,C,E", [(256, 512, 2048), (5, 64, 300), (3, 2048, 512), (2, 48, 9)])
def test_mlp_temperature_kernel(B, C, E):
    g = torch.Generator().manual_seed(B + C + E)
    z = torch.rand(B, C, generator=g)
    w1, b1, w2, b2 = mlp_params(C, E, seed=C + E)
    T, h = H.temperature_mlp(z.to(DEV), *(t.to(DEV) for t in (w1, b1, w2, b2)), TMIN * TAU, (TMAX - TMIN) * TAU)
    want, _, hw = O.gate_temperature_mlp(z.numpy(), w1.numpy(), b1.numpy(), w2.numpy(), b2.numpy(), TMIN, TMAX, TAU)
    assert close(h.cpu().numpy(), hw, 1e-5, 1e-6), maxrel(h.cpu().numpy(), hw)
    assert close(T.cpu().numpy(), want, 1e-5, 1e-6), maxrel(T.cpu().numpy(), want)


@pytest.mark.parametrize("B,C,Hh,E,k", [(32, 512, 7, 2048, 32), (3, 64, 56, 140, 8), (4, 256, 14, 300, 16)])
def test_forward_tc_mlp_matches_oracle(B, C, Hh, E, k):
    """The fused tensor-core chain with the two-layer gate (bf16)."""
    g = torch.Generator().manual_seed(B * 7 + C)
    X = torch.randn(B, C, Hh, Hh, generator=g).abs()
    L = torch.randn(E - 1, C, generator=g)
    prm = mlp_params(C, E, seed=B + E)
    x = X.to(DEV, torch.bfloat16)
    r = H.route_build(L.to(DEV), k, transposed=False)
    assert H.tc_supported(x, k)
    H.tc_fault(clear=True)
    y, z, T, h = H.forward_tc_mlp(x, r, *(t.to(DEV) for t in prm), TMIN * TAU, (TMAX - TMIN) * TAU)
    torch.cuda.synchronize()
    assert H.tc_fault() == 0
    mlp = tuple(t.numpy() for t in prm)
    ref, aux = O.forward(x.float().cpu().numpy(), L.numpy(), None, None, k, TMIN, TMAX, TAU, mode="eval",
                         return_aux=True, mlp=mlp)
    assert close(T.cpu().numpy(), aux["T"], 1e-5, 1e-6), maxrel(T.cpu().numpy(), aux["T"])
    got = y.float().cpu().numpy()
    assert close(got, ref, 1e-2, 1e-3), maxrel(got, ref)


@pytest.mark.parametrize("B,C,Hh,E,k,dtype", [
    (8, 256, 14, 1024, 16, torch.float32),     # lanes-over-pixels path, fp32
    (4, 512, 7, 2048, 32, torch.bfloat16),     # fused tensor-core chain
    (2, 1024, 14, 256, 64, torch.bfloat16),    # C > 512: CUDA-core path, bf16
    (3, 64, 40, 65, 8, torch.float32),         # H*W = 1600: the general mix
])
def test_module_eval_mlp_gate(B, C, Hh, E, k, dtype):
    from moce_thesis_b200 import MoCE
    g = torch.Generator().manual_seed(B + C + k)
    X = torch.randn(B, C, Hh, Hh, generator=g).abs()
    L = torch.randn(E - 1, C, generator=g)
    torch.manual_seed(3)
    m = MoCE(in_channels=C, sampling_factor=1, k=k, temp_min=TMIN, temp_max=TMAX, gate_type="mlp")
    m.num_experts = E
    m.routing_logits = torch.nn.Parameter(L)
    m.reset_gate_mlp()
    m = m.to(DEV).eval()
    m.build_eval_cache()
    x = X.to(DEV, dtype)
    with torch.no_grad():
        y = m(x)
    torch.cuda.synchronize()
    mlp = tuple(t.detach().cpu().numpy() for t in (m.gate_mlp[0].weight, m.gate_mlp[0].bias,
                                                   m.gate_mlp[2].weight, m.gate_mlp[2].bias))
    ref = O.forward(x.float().cpu().numpy(), L.numpy(), None, None, k, TMIN, TMAX, TAU, mode="eval", mlp=mlp)
    rtol = 1e-5 if dtype == torch.float32 else 1e-2
    got = y.float().cpu().numpy()
    assert close(got, ref, rtol, 1e-3), maxrel(got, ref)


@pytest.mark.parametrize("B,C,Hh,E,k", [(4, 64, 7, 65, 8), (2, 256, 14, 1024, 16), (3, 96, 5, 4, 8)])
def test_module_train_mlp_gate(B, C, Hh, E, k):
    """Train forward and backward with the two-layer gate (fp32)."""
    from moce_thesis_b200 import MoCE
    g = torch.Generator().manual_seed(B * 13 + C)
    X = torch.randn(B, C, Hh, Hh, generator=g).abs()
    L = torch.randn(E - 1, C, generator=g)
    dY = torch.randn(B, E, Hh, Hh, generator=g)
    torch.manual_seed(4)
    m = MoCE(in_channels=C, sampling_factor=1, k=k, temp_min=TMIN, temp_max=TMAX, gate_type="mlp")
    m.num_experts = E
    m.routing_logits = torch.nn.Parameter(L.clone())
    m.reset_gate_mlp()
    m = m.to(DEV).train()
    x = X.to(DEV).requires_grad_(True)
    y = m(x)
    (y * dY.to(DEV)).sum().backward()
    torch.cuda.synchronize()
    lin1, lin2 = m.gate_mlp[0], m.gate_mlp[2]
    mlp = tuple(t.detach().cpu().numpy() for t in (lin1.weight, lin1.bias, lin2.weight, lin2.bias))
    ref = O.forward(X.numpy(), L.numpy(), None, None, k, TMIN, TMAX, TAU, mode="train", mlp=mlp)
    assert close(y.detach().cpu().numpy(), ref, 1e-5, 1e-3), maxrel(y.detach().cpu().numpy(), ref)
    d = O.backward(X.numpy(), L.numpy(), None, None, k, dY.numpy(), TMIN, TMAX, TAU, mlp=mlp)
    # the routing logits also get the aux-loss gradient; compare the main path
    m.routing_logits.grad = None
    got = {"dX": x.grad, "dw1": lin1.weight.grad, "db1": lin1.bias.grad, "dw2": lin2.weight.grad,
           "db2": lin2.bias.grad}
    for key, t in got.items():
        assert maxrel(t.cpu().numpy(), d[key]) < 1e-5, (key, maxrel(t.cpu().numpy(), d[key]))


def test_backward_t_dT_matches_oracle():
    """moce_backward_t through the binding: dT, dL and dX (no gate term)."""
    from moce_thesis_b200 import native
    g = torch.Generator().manual_seed(77)
    B, C, Hh, E, k = 3, 128, 9, 200, 16
    X = torch.randn(B, C, Hh, Hh, generator=g).abs()
    L = torch.randn(E - 1, C, generator=g)
    dY = torch.randn(B, E, Hh, Hh, generator=g)
    prm = mlp_params(C, E, seed=5)
    mlp = tuple(t.numpy() for t in prm)
    _, aux = O.forward(X.numpy(), L.numpy(), None, None, k, TMIN, TMAX, TAU, mode="train", return_aux=True, mlp=mlp)
    d = O.backward(X.numpy(), L.numpy(), None, None, k, dY.numpy(), TMIN, TMAX, TAU, mlp=mlp)
    r = H.route_build(L.to(DEV), k, transposed=True)
    T = torch.from_numpy(aux["T"]).float().to(DEV)
    dx, dL, dT = native().backward_t(X.to(DEV), dY.to(DEV), L.to(DEV), r["idx"], r["ln"], r["mask"], r["meta"],
                                     r["toff"], r["tslot"], T)
    torch.cuda.synchronize()
    assert maxrel(dT.cpu().numpy(), d["dT"]) < 1e-5
    assert maxrel(dL.cpu().numpy(), d["dL"]) < 1e-5
    # dX without the gate's term through z (the caller's autograd adds it)
    HW = Hh * Hh
    w1, b1, w2, b2 = (np.asarray(t, dtype=np.float64) for t in mlp)
    h = aux["h"]
    sig = 1.0 / (1.0 + np.exp(-aux["g"]))
    T_raw = (TMIN + (TMAX - TMIN) * sig) * TAU
    dg = np.where(T_raw >= 1e-3, d["dT"], 0.0) * TAU * (TMAX - TMIN) * sig * (1 - sig)
    dz = ((dg @ w2) * (h > 0)) @ w1
    dX_mix = d["dX"] - dz[:, :, None, None] / HW
    assert maxrel(dx.cpu().numpy(), dX_mix) < 1e-5


@pytest.mark.parametrize("B,C,Hh,E,k", [(9, 512, 7, 300, 32), (3, 128, 28, 90, 16), (2, 64, 56, 40, 8)])
def test_mix_tc_given_T_matches_in_kernel_gate(B, C, Hh, E, k):
    """moce_mix_tc_t fed the temperatures moce_mix_tc computed from z gives
    the same bits (the same weights reach the same MMAs)."""
    g = torch.Generator().manual_seed(B + C + E)
    x = torch.randn(B, C, Hh, Hh, generator=g).abs().to(DEV, torch.bfloat16)
    L = torch.randn(E - 1, C, generator=g).to(DEV)
    gw = (torch.rand(k, generator=g) - 0.5).to(DEV)
    gb = (torch.randn(1, generator=g) * 0.1).to(DEV)
    r = H.route_build(L, k, transposed=False)
    H.tc_fault(clear=True)
    y, z, T = H.forward_tc(x, r, gw, gb, TMIN * TAU, (TMAX - TMIN) * TAU, want_T=True)
    y2 = H.forward_tc_t(x, r, T)
    torch.cuda.synchronize()
    assert H.tc_fault() == 0
    assert torch.equal(y, y2)
