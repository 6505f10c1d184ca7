"""moce_gate_route_noalloc against moce_gate_route (GPU, through the C ABI).

The no-allocation entry point serves callers that cannot allocate device
memory at the call (an engine plugin with a fixed budget and no allocator, a
latency-critical path that cannot take cudaMalloc's synchronisation).  It
must give the same output as the workspace entry point, also on a second
call in a row (its scratch array keeps the previous call's contents), and
reject shapes whose scratch exceeds the library's fixed array.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from moce_thesis_b200 import capi
from moce_thesis_b200.capi import ptr, stream_handle
import capi_helpers as H

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _inputs(seed, B, C, Hh, W, E, k, dtype):
    g = torch.Generator().manual_seed(seed)
    X = torch.randn(B, C, Hh, W, generator=g).abs().to(DEV, dtype)
    L = torch.randn(E - 1, C, generator=g).to(DEV)
    r = H.route_build(L, k, transposed=False)
    gw = (torch.rand(k, generator=g) - 0.5).to(DEV)
    gb = (torch.randn(1, generator=g) * 0.1).to(DEV)
    return X, r, gw, gb


def _noalloc(x, pooled, idx, r, gw, gb, tmin, tmax, tau):
    B, C, Hh, W = x.shape
    E_r, k = idx.shape
    bits = 64 if idx.dtype == torch.int64 else 32
    y = torch.empty(B, E_r + 1, Hh, W, dtype=x.dtype, device=x.device)
    rc = capi.lib().moce_gate_route_noalloc(ptr(x), capi.dtype_code(x), ptr(pooled), ptr(idx), bits,
                                            ptr(r["ln"]), ptr(gw), ptr(gb), ptr(r["mask"]), tmin, tmax, tau,
                                            ptr(y), B, C, Hh * W, E_r, k, stream_handle())
    capi.check(rc, "moce_gate_route_noalloc")
    return y


@pytest.mark.parametrize("index_bits", [32, 64])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("pooled_given", [False, True])
def test_noalloc_matches_workspace_entry_twice(dtype, pooled_given, index_bits):
    """Three different calls in a row: none may see an earlier call's
    scratch.  The last shape has k close to C, so its indices fill most of
    the scratch region that 64-bit indices are converted into."""
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    lib = capi.lib()
    for seed, shape in ((1, (4, 64, 7, 7, 65, 8)), (2, (3, 96, 5, 5, 33, 12)), (3, (2, 64, 3, 3, 1001, 60))):
        B, C, Hh, W, E, k = shape
        assert lib.moce_gate_route_workspace_bytes(B, C, E - 1) <= lib.moce_noalloc_scratch_bytes()
        x, r, gw, gb = _inputs(seed, B, C, Hh, W, E, k, dtype)
        idx = r["idx"].long().contiguous() if index_bits == 64 else r["idx"]
        pooled = x.float().mean((2, 3)).contiguous() if pooled_given else None
        want = H.gate_route(x, pooled, idx, r["ln"], gw, gb, r["mask"], 0.1, 10.0, 1.0)
        got = _noalloc(x, pooled, idx, r, gw, gb, 0.1, 10.0, 1.0)
        torch.cuda.synchronize()
        a, b = got.float().cpu().numpy(), want.float().cpu().numpy()
        assert np.all(np.abs(a - b) <= tol * np.abs(b) + 1e-6 * np.abs(b).max()), float(np.abs(a - b).max())


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = capi.lib()
    cap = lib.moce_noalloc_scratch_bytes()
    assert cap == 4 << 20
    B, C, E_r, k = 4096, 512, 2047, 32
    assert lib.moce_gate_route_workspace_bytes(B, C, E_r) > cap
    dummy = torch.empty(16, device=DEV)
    p = ptr(dummy)
    rc = lib.moce_gate_route_noalloc(p, 0, None, p, 32, p, p, p, p, 0.1, 10.0, 1.0, p, B, C, 49, E_r, k,
                                     stream_handle())
    assert rc == capi.MOCE_ERR_UNSUPPORTED
    assert b"scratch" in lib.moce_last_error()
