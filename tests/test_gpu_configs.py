"""GPU parity at the benchmark configurations' own shapes (through the C ABI).

Each test runs the layer at one of the workload shapes the benchmarks time
and compares every output element with the float64 oracle (a restatement of
MoCE.py:153-230, itself pinned to goldens made by the unmodified reference):

* the ResNet-50 stage-4 layer (N=256, C=512, 7x7, E=2048, k=32), bf16 on the
  tensor-core path with all 256 samples, and fp32 on the lanes-over-pixels
  path with 64 samples, all 2047 routed experts each;
* the four per-stage sweep shapes at their exact C, H*W, E and k (bf16);
* the training shape (C=256, 14x14, E=1024, k=16, fp32) forward and
  backward (dX, dL, dgate) at a small batch;
* every distinct MoCE layer of ResNet-50 with k = C_in/16, on the kernel the
  layer module picks for it.

Inputs follow the benchmarks' recipe: half-normal X, N(0,1) logits, a
uniform gate weight, temp_min 0.1, temp_max 10.  Tolerances: fp32 outputs
1e-5 relative, bf16 1e-2 relative (both with a floor of 1e-3 of the largest
magnitude, for elements near zero), gradients 1e-5 of their largest
magnitude.
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


def worst(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float((np.abs(a - b) / np.maximum(np.abs(b), 1e-3 * max(np.abs(b).max(), 1e-30))).max())


def inputs(B, C, Hh, E, k, seed):
    """Benchmark recipe: X = |N(0,1)|, L ~ N(0,1), gate weight U(-a, a) with
    a = sqrt(6 / (k + 1)) (xavier_uniform of Linear(k, 1), MoCE.py:66-68)."""
    X = torch.randn(B, C, Hh, Hh, generator=torch.Generator().manual_seed(seed)).abs()
    L = torch.randn(E - 1, C, generator=torch.Generator().manual_seed(seed + 1))
    gw = (torch.rand(1, k, generator=torch.Generator().manual_seed(seed + 2)) * 2 - 1) * (6.0 / (k + 1)) ** 0.5
    gb = torch.zeros(1)
    return X, L, gw, gb


def path_for(x, k):
    """The kernel moce_thesis_b200.MoCE picks for this input (moce.py _Route.forward)."""
    if H.tc_supported(x, k):
        return "tc"
    if H.px_supported(x, k):
        return "px"
    if H.gx_supported(x, k):
        return "gx"
    return "fast" if H.schedule_supported(k) else "general"


def oracle_forward(Xf, L, gw, gb, k, chunk=32):
    """O.forward over the batch in chunks of samples (bounded host memory)."""
    outs = [O.forward(Xf[i:i + chunk], L, gw, gb, k, TMIN, TMAX, TAU, mode="eval")
            for i in range(0, Xf.shape[0], chunk)]
    return np.concatenate(outs, axis=0)


def run_and_check(B, C, Hh, E, k, dtype, seed, expect_path=None):
    X, L, gw, gb = inputs(B, C, Hh, E, k, seed)
    x = X.to(DEV, dtype)
    path = path_for(x, k)
    if expect_path is not None:
        assert path == expect_path, path
    H.tc_fault(clear=True)
    y, st = H.forward(x, L.to(DEV), gw.to(DEV), gb.to(DEV), k, TMIN, TMAX, TAU, path=path)
    torch.cuda.synchronize()
    assert H.tc_fault() == 0
    # supports bit-exact against torch.topk's order (tie-free N(0,1) rows)
    assert torch.equal(st["idx"].long().cpu(), torch.topk(L, k, dim=1).indices)
    Xf = x.float().cpu().numpy()
    ref = oracle_forward(Xf, L.numpy(), gw.numpy(), gb.numpy(), k)
    got = y.float().cpu().numpy()
    rtol = 1e-5 if dtype == torch.float32 else 1e-2
    assert close(got, ref, rtol, 1e-3), (path, worst(got, ref))
    return path


def test_stage4_bf16_all_samples():
    """The headline workload, every sample and expert against the oracle."""
    run_and_check(256, 512, 7, 2048, 32, torch.bfloat16, seed=1000, expect_path="tc")


def test_stage4_fp32_reference_precision():
    """The stage-4 layer in the reference's own precision (fp32)."""
    run_and_check(64, 512, 7, 2048, 32, torch.float32, seed=1001)


@pytest.mark.parametrize("C,Hh,E,k", [(64, 56, 256, 8), (128, 28, 512, 16), (256, 14, 1024, 16), (512, 7, 2048, 32)])
def test_sweep_shapes_exact(C, Hh, E, k):
    """The per-stage sweep at its exact C, H*W, E, k (bf16), two samples."""
    run_and_check(2, C, Hh, E, k, torch.bfloat16, seed=3000 + C, expect_path="tc")


@pytest.mark.parametrize("C,Hh,E,k", [
    (64, 56, 64, 4),        # layer1, block 0 (sampling factor 1)
    (256, 56, 64, 16),      # layer1, blocks 1-2
    (256, 56, 128, 16),     # layer2, block 0 (sampling factor 2, before the stride)
    (512, 28, 128, 32),     # layer2, blocks 1-3
    (512, 28, 256, 32),     # layer3, block 0
    (1024, 14, 256, 64),    # layer3, blocks 1-5
    (1024, 14, 512, 64),    # layer4, block 0
    (2048, 7, 512, 128),    # layer4, blocks 1-2
])
def test_resnet50_layers_k_cin_over_16(C, Hh, E, k):
    """Every distinct MoCE layer of ResNet-50 + MoCE with k = C_in / 16
    (models_unified.py:227-258), bf16, two samples, on the kernel the layer
    module dispatches to."""
    run_and_check(2, C, Hh, E, k, torch.bfloat16, seed=5000 + C + E)


def test_training_shape_gradients():
    """The training configuration's layer (C=256, 14x14, E=1024, k=16, fp32):
    forward, then dX, dL and dgate against the oracle's hand-derived
    backward (MoCE.py:153-201 under autograd), at batch 2."""
    B, C, Hh, E, k = 2, 256, 14, 1024, 16
    X, L, gw, gb = inputs(B, C, Hh, E, k, seed=2000)
    dY = torch.randn(B, E, Hh, Hh, generator=torch.Generator().manual_seed(2003))
    x, Ld, gwd, gbd = X.to(DEV), L.to(DEV), gw.to(DEV), gb.to(DEV)
    r = H.route_build(Ld, k, transposed=True)
    path = path_for(x, k)
    y, st = H.forward(x, Ld, gwd, gbd, k, TMIN, TMAX, TAU, route=r, path=path)
    d = H.backward(x, dY.to(DEV), Ld, st, gwd, gbd, TMIN * TAU, (TMAX - TMIN) * TAU)
    torch.cuda.synchronize()
    ref_y = O.forward(X.numpy(), L.numpy(), gw.numpy(), gb.numpy(), k, TMIN, TMAX, TAU, mode="train")
    assert close(y.cpu().numpy(), ref_y, 1e-5, 1e-3), worst(y.cpu().numpy(), ref_y)
    g = O.backward(X.numpy(), L.numpy(), gw.numpy(), gb.numpy(), k, dY.numpy(), TMIN, TMAX, TAU)
    for key in ("dX", "dL", "dgate_w", "dgate_b"):
        got = d[key].cpu().numpy().reshape(g[key].shape)
        want = g[key]
        err = float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))
        assert err < 1e-5, (key, err)
