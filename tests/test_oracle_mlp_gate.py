"""The oracle's two-layer temperature gate against torch autograd (CPU).

The two-layer gate (C -> C/16 -> E-1, ReLU) has no counterpart in the
reference, so its oracle is a restatement: ``gate_temperature_mlp`` and the
hand-derived ``backward(..., mlp=...)``.  This pins that restatement to a
float64 torch expression of the same layer differentiated by autograd
(forward through the reference's temperature map, softmax and gather-mix).
"""
import numpy as np
import torch

from oracle import moce_oracle as O


def _torch_layer(X, L, w1, b1, w2, b2, k, tmin, tmax, tau):
    idx = torch.from_numpy(O.select_supports(L.detach().numpy(), k))
    sel = torch.gather(L, 1, idx)
    cen = sel - sel.mean(1, keepdim=True)
    ln = cen / sel.std(1, keepdim=True).clamp(min=1.0)
    z = X.mean((2, 3))
    g = torch.relu(z @ w1.T + b1) @ w2.T + b2
    T = ((tmin + (tmax - tmin) * torch.sigmoid(g)) * tau).clamp(min=1e-3)
    a = torch.softmax(ln[None] / T[:, :, None], dim=-1)
    B, C, H, W = X.shape
    Xf = X.reshape(B, C, H * W)
    y = (a[..., None] * Xf[:, idx, :]).sum(2)
    mask = torch.from_numpy(O.uncovered_mask(C, idx.numpy()).astype(bool))
    res = Xf[:, mask, :].mean(1, keepdim=True) if mask.any() else torch.zeros(B, 1, H * W, dtype=X.dtype)
    return torch.cat([y, res], 1).reshape(B, -1, H, W), T


def test_mlp_gate_oracle_matches_autograd():
    g = torch.Generator().manual_seed(5)
    B, C, H, W, E, k = 3, 32, 4, 4, 21, 6
    Hd = C // 16
    X = torch.randn(B, C, H, W, generator=g, dtype=torch.float64).abs().requires_grad_(True)
    # fp32-representable logits: the oracle reads L as fp32, as the reference stores it
    L = torch.randn(E - 1, C, generator=g).double().requires_grad_(True)
    w1 = (torch.randn(Hd, C, generator=g, dtype=torch.float64) * (2.0 / C) ** 0.5).requires_grad_(True)
    b1 = (torch.randn(Hd, generator=g, dtype=torch.float64) * 0.1).requires_grad_(True)
    w2 = (torch.randn(E - 1, Hd, generator=g, dtype=torch.float64) * (2.0 / Hd) ** 0.5).requires_grad_(True)
    b2 = (torch.randn(E - 1, generator=g, dtype=torch.float64) * 0.1).requires_grad_(True)
    dY = torch.randn(B, E, H, W, generator=g, dtype=torch.float64)
    tmin, tmax, tau = 0.1, 10.0, 1.0
    Y, T = _torch_layer(X, L, w1, b1, w2, b2, k, tmin, tmax, tau)
    mlp = tuple(t.detach().numpy() for t in (w1, b1, w2, b2))
    Yo, aux = O.forward(X.detach().numpy(), L.detach().numpy(), None, None, k, tmin, tmax, tau, mode="train",
                        return_aux=True, mlp=mlp)
    assert np.allclose(Yo, Y.detach().numpy(), rtol=1e-12, atol=1e-12)
    assert np.allclose(aux["T"], T.detach().numpy(), rtol=1e-12, atol=1e-12)
    (Y * dY).sum().backward()
    d = O.backward(X.detach().numpy(), L.detach().numpy(), None, None, k, dY.numpy(), tmin, tmax, tau, mlp=mlp)
    for name, t in (("dX", X), ("dL", L), ("dw1", w1), ("db1", b1), ("dw2", w2), ("db2", b2)):
        assert np.allclose(d[name], t.grad.numpy(), rtol=1e-9, atol=1e-12), name
