"""GPU parity of the native auxiliary (coverage) loss and its gradient.

moce_aux_loss / moce_aux_loss_backward (through the binding) against
* the float64 oracle ``aux_loss`` (a restatement of MoCE.py:118-151, pinned
  to the reference's own aux values by the golden tests), within 1e-5
  relative, and
* torch autograd of the reference expression in float64 for d aux / d L,
  within 1e-5 of the gradient's largest magnitude,
at the training shape (E=1024, C=256, k=16), the stage-4 shape, a shape whose
entropy term is partly inactive, and E_r = 1 (no diversity term).
"""
import math

import numpy as np
import pytest
import torch

from oracle import moce_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
W = (0.05, 0.1, 0.01)


def reference_aux(L, k, tau, wb, ws, wd):
    """MoCE._compute_aux_losses restated in torch (float64), for autograd."""
    E_r, C = L.shape
    P = torch.softmax(L / tau, dim=1)
    usage = P.mean(dim=0)
    balance = (usage - usage.mean()).pow(2).mean()
    per_channel = P / P.sum(dim=0, keepdim=True).clamp(min=1e-8)
    entropy = -(per_channel * per_channel.clamp(min=1e-8).log()).sum(dim=0)
    target = math.log(max(E_r * k / C, 1.0))
    spec = torch.relu(entropy - target).mean()
    if E_r > 1:
        ov = P @ P.t()
        div = ov[~torch.eye(E_r, dtype=torch.bool)].mean()
    else:
        div = P.new_zeros(())
    return wb * balance + ws * spec + wd * div


@pytest.mark.parametrize("E_r,C,k,tau,scale", [
    (1023, 256, 16, 1.0, 1.0),     # training shape
    (2047, 512, 32, 1.0, 1.0),     # stage-4 shape
    (63, 256, 4, 0.5, 3.0),        # peaked rows: low entropy, the relu partly inactive
    (1, 40, 8, 1.0, 1.0),          # one routed expert: no diversity term
    (300, 130, 40, 2.0, 0.3),      # ragged sizes, flat rows
])
def test_aux_loss_and_gradient(E_r, C, k, tau, scale):
    from moce_thesis_b200 import native
    g = torch.Generator().manual_seed(E_r + C + k)
    L = torch.randn(E_r, C, generator=g) * scale
    target = math.log(max(E_r * k / C, 1.0))
    aux = native().aux_loss(L.to(DEV), tau, *W, target)
    want = O.aux_loss(L.numpy(), k, tau, *W)
    assert abs(float(aux) - want) <= 1e-5 * abs(want) + 1e-12, (float(aux), want)
    Ld = L.double().requires_grad_(True)
    reference_aux(Ld, k, tau, *W).backward()
    gsc = 1.7
    dL = native().aux_loss_backward(L.to(DEV), tau, *W, target, torch.tensor([gsc], device=DEV))
    torch.cuda.synchronize()
    ref = gsc * Ld.grad.numpy()
    err = float(np.abs(dL.cpu().numpy() - ref).max() / max(np.abs(ref).max(), 1e-30))
    assert err < 1e-5, err


def test_aux_loss_deterministic():
    from moce_thesis_b200 import native
    L = torch.randn(1023, 256, generator=torch.Generator().manual_seed(3)).to(DEV)
    a = native().aux_loss_backward(L, 1.0, *W, 1.2, torch.ones(1, device=DEV))
    b = native().aux_loss_backward(L, 1.0, *W, 1.2, torch.ones(1, device=DEV))
    assert torch.equal(a, b)
    assert torch.equal(native().aux_loss(L, 1.0, *W, 1.2), native().aux_loss(L, 1.0, *W, 1.2))
