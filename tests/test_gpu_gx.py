"""GPU parity of the CUDA-core mix that reads X from global memory
(moce_mix_gx: samples larger than shared memory, k up to 128) against the
oracle.  fp32 within 1e-5 relative, 16-bit within 1e-2 relative of the fp32
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


@pytest.mark.parametrize("B,C,H_,W_,E,k,dtype", [
    (2, 1024, 14, 14, 256, 64, torch.bfloat16),   # ResNet-50 layer3 bottleneck entrance (k = C/16)
    (2, 2048, 7, 7, 64, 128, torch.bfloat16),     # layer4: k = 128, rows of 49 pixels (element loads)
    (2, 512, 28, 28, 128, 32, torch.bfloat16),    # layer2: 784 pixels over seven 128-pixel slabs
    (3, 96, 5, 7, 40, 40, torch.float32),         # fp32, k not a multiple of 32, odd H*W
    (2, 64, 32, 32, 20, 8, torch.float16),        # 1024 pixels (eight slabs), uncovered channels
    (1, 300, 9, 9, 50, 100, torch.bfloat16),      # k = 100 (four support registers per lane)
])
def test_gx_mix_matches_oracle(B, C, H_, W_, E, k, dtype):
    gen = torch.Generator().manual_seed(B * 100 + C + k)
    X = torch.randn(B, C, H_, W_, generator=gen).abs()
    L = torch.randn(E - 1, C, generator=gen)
    gw = torch.rand(1, k, generator=gen) - 0.5
    gb = torch.randn(1, generator=gen) * 0.1
    x = X.to(DEV, dtype)
    assert H.gx_supported(x, k)
    y, st = H.forward(x, L.to(DEV), gw.to(DEV), gb.to(DEV), k, 0.1, 10.0, 1.0, path="gx")
    torch.cuda.synchronize()
    ref, aux = O.forward(x.float().cpu().numpy(), L.numpy(), gw.numpy(), gb.numpy(), k, 0.1, 10.0, 1.0,
                         mode="eval", return_aux=True)
    tol = (1e-5, 1e-6) if dtype == torch.float32 else (1e-2, 1e-3)
    assert close(y.float().cpu().numpy(), ref, *tol)
    assert close(st["T"].cpu().numpy(), aux["T"], 1e-5, 1e-6)


def test_gx_rejects_shapes_beyond_its_limits():
    x = torch.zeros(1, 8, 33, 33, device=DEV)                       # 1089 pixels
    assert not H.gx_supported(x, 4)
    assert not H.gx_supported(torch.zeros(1, 256, 4, 4, device=DEV), 129)
