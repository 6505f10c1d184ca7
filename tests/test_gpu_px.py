"""GPU parity of the lanes-over-pixels CUDA-core mix (moce_mix_px) and of
the backward kernels that use the same layout, against the oracle.

fp32 within 1e-5 relative, bf16/fp16 within 1e-2 relative of the fp32
oracle on the rounded input; temperatures within 1e-5.
"""
import numpy as np
import pytest
import torch

from oracle import moce_oracle as O
import capi_helpers as H

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def close(a, b, rtol, floor):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return bool(np.all(np.abs(a - b) <= rtol * np.abs(b) + floor * max(np.abs(b).max(), 1e-30)))


def relerr(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float((np.abs(a - b) / np.maximum(np.abs(b), 1e-6 * max(np.abs(b).max(), 1e-30))).max())


@pytest.mark.parametrize("B,C,H_,W_,E,k,dtype", [
    (3, 256, 14, 14, 64, 16, torch.float32),     # the 14x14 stage: two slabs, unpadded rows (flat copy)
    (2, 512, 7, 7, 80, 32, torch.float32),       # HW = 49: padded rows, one partial slab
    (2, 64, 16, 32, 30, 8, torch.float32),       # HW = 512: four full slabs
    (2, 40, 15, 20, 33, 40, torch.float32),      # HW = 300, k > 32: two supports per lane
    (2, 48, 1, 1, 9, 48, torch.float32),         # HW = 1, k == C
    (2, 37, 9, 9, 12, 5, torch.float32),         # odd C, HW = 81, uncovered channels (residual)
    (3, 256, 14, 14, 64, 16, torch.bfloat16),
    (2, 128, 11, 13, 40, 64, torch.float16),     # HW = 143, k = 64
    (2, 2048, 7, 7, 60, 128, torch.bfloat16),    # k = 128 (four supports per lane), 221 KB sample in one CTA
    (2, 1024, 14, 14, 100, 64, torch.bfloat16),  # 401 KB sample: two CTAs of a cluster hold one half each
    (3, 600, 13, 13, 70, 100, torch.float32),    # fp32 split over a CTA pair, odd C and H*W, k = 100
])
def test_px_mix_matches_oracle(B, C, H_, W_, E, k, dtype):
    gen = torch.Generator().manual_seed(B * 100 + C + k)
    X = torch.randn(B, C, H_, W_, generator=gen).abs()
    L = torch.randn(E - 1, C, generator=gen)
    gw = torch.rand(1, k, generator=gen) - 0.5
    gb = torch.randn(1, generator=gen) * 0.1
    x = X.to(DEV, dtype)
    assert H.px_supported(x, k)
    y, st = H.forward(x, L.to(DEV), gw.to(DEV), gb.to(DEV), k, 0.1, 10.0, 1.0, path="px")
    xr = x.float().cpu().numpy()
    ref, aux = O.forward(xr, L.numpy(), gw.numpy(), gb.numpy(), k, 0.1, 10.0, 1.0, mode="eval", return_aux=True)
    rt = 1e-5 if dtype == torch.float32 else 1e-2
    got = y.float().cpu().numpy()
    assert close(got, ref, rt, rt / 10), relerr(got, ref)
    assert close(st["T"].cpu().numpy(), aux["T"], 1e-5, 1e-6)


def test_px_unsupported_shape_is_rejected():
    x = torch.empty(1, 16, 32, 32, device=DEV)          # HW = 1024
    assert not H.px_supported(x, 8)
    r = H.route_build(torch.randn(7, 16, device=DEV), 8, transposed=False)
    with pytest.raises(RuntimeError, match="moce_mix_px"):
        H.forward_px(x, r, torch.zeros(8, device=DEV), torch.zeros(1, device=DEV), 0.1, 9.9)


@pytest.mark.parametrize("B,C,H_,W_,E,k", [
    (3, 256, 14, 14, 64, 16),       # lanes-over-pixels route and dX kernels
    (2, 96, 13, 11, 50, 20),        # padded rows, partial slab
    (2, 32, 16, 32, 20, 32),        # HW = 512, k = 32
])
def test_px_backward_matches_oracle(B, C, H_, W_, E, k):
    gen = torch.Generator().manual_seed(B * 7 + C + k)
    X = torch.randn(B, C, H_, W_, generator=gen).abs()
    L = torch.randn(E - 1, C, generator=gen)
    gw = torch.rand(1, k, generator=gen) - 0.5
    gb = torch.randn(1, generator=gen) * 0.1
    dY = torch.randn(B, E, H_, W_, generator=gen)
    x = X.to(DEV)
    y, st = H.forward(x, L.to(DEV), gw.to(DEV), gb.to(DEV), k, 0.1, 10.0, 1.0, path="px")
    r = H.route_build(L.to(DEV), k)
    r.update(z=st["z"], T=st["T"])
    d = H.backward(x, dY.to(DEV), L.to(DEV), r, gw.to(DEV), gb.to(DEV), 0.1, 9.9)
    want = O.backward(X.numpy(), L.numpy(), gw.numpy(), gb.numpy(), k, dY.numpy(), 0.1, 10.0, 1.0, mode="eval")
    for key in ("dX", "dL", "dgate_w", "dgate_b"):
        got = d[key].cpu().numpy().reshape(np.shape(want[key]))
        w = np.asarray(want[key], dtype=np.float64)
        err = float(np.abs(got - w).max() / max(np.abs(w).max(), 1e-3))
        assert err < 1e-5, (key, err)
