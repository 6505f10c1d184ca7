"""The tensor-core mix's bounded waits, made to run out on purpose.

Every wait of one role of mix_tc_kernel on another (weight rows, MMA issuers,
copy producer, drain) is bounded in time.  Setting the bound to one
nanosecond (moce_tc_wait_limit_ns) makes the first wait that does not succeed
at once give up: the kernel must then set its fault flag, let its copies and
MMAs in flight finish, release its tensor memory and return, leaving the
context usable.  These tests check exactly that, on the three kernel forms
(the 7x7 specialisation, the general one-tile form, the pixel-tiled form with
one weight thread per row): the launch returns without a CUDA error, the
flag reads 1 (through the C ABI and through ``check_faults``), and a launch
made afterwards with the default bound matches the oracle with the flag
clear.  No kernel traps, faults or waits without a bound here.
"""
import numpy as np
import pytest
import torch

from moce_thesis_b200 import capi, check_faults
from oracle import moce_oracle as O
import capi_helpers as H

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _case(B, C, Hh, E, k, seed):
    gen = torch.Generator().manual_seed(seed)
    X = torch.randn(B, C, Hh, Hh, generator=gen).abs()
    L = torch.randn(E - 1, C, generator=gen)
    gw = torch.rand(1, k, generator=gen) - 0.5
    gb = torch.randn(1, generator=gen) * 0.1
    return X, L, gw, gb


@pytest.mark.parametrize("B,C,Hh,E,k", [
    (24, 512, 7, 600, 32),     # 7x7: the specialised one-tile kernel, two issuers
    (8, 256, 14, 300, 16),     # 14x14: general one-tile kernel, one accumulator
    (2, 64, 56, 140, 8),       # 56x56: pixel tiles, one weight thread per row, eight drain warps
])
def test_wait_that_runs_out_aborts_cleanly(B, C, Hh, E, k):
    lib = capi.lib()
    X, L, gw, gb = _case(B, C, Hh, E, k, seed=B + C + k)
    x = X.to(DEV, torch.bfloat16)
    Ld, gwd, gbd = L.to(DEV), gw.to(DEV), gb.to(DEV)
    assert H.tc_supported(x, k)
    r = H.route_build(Ld, k, transposed=False)
    torch.cuda.synchronize()
    H.tc_fault(clear=True)
    default = lib.moce_tc_wait_limit_ns(0)
    assert default >= 10 ** 9 // 2
    prev = lib.moce_tc_wait_limit_ns(1)
    try:
        assert prev == default
        H.forward(x, Ld, gwd, gbd, k, 0.1, 10.0, 1.0, route=r, path="tc")
        torch.cuda.synchronize()                        # returns: no hang, no CUDA error
    finally:
        lib.moce_tc_wait_limit_ns(prev)
    assert lib.moce_tc_wait_limit_ns(0) == default
    with pytest.raises(RuntimeError, match="bounded wait ran out"):
        check_faults(clear=False)
    assert H.tc_fault(clear=True) == 1
    # the context is usable and tensor memory was released: a normal launch
    # gives the oracle's output with the flag clear
    y, st = H.forward(x, Ld, gwd, gbd, k, 0.1, 10.0, 1.0, route=r, path="tc")
    torch.cuda.synchronize()
    assert H.tc_fault() == 0
    check_faults()
    ref = O.forward(x.float().cpu().numpy(), L.numpy(), gw.numpy(), gb.numpy(), k, 0.1, 10.0, 1.0, mode="eval")
    got = y.float().cpu().numpy()
    err = np.abs(got - ref) - (1e-2 * np.abs(ref) + 1e-3 * np.abs(ref).max())
    assert float(err.max()) <= 0.0


def test_wait_limit_query_does_not_change_it():
    lib = capi.lib()
    a = lib.moce_tc_wait_limit_ns(0)
    b = lib.moce_tc_wait_limit_ns(-5)
    assert a == b > 0
