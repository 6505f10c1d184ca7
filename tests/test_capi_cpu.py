"""CPU-side checks of the native library: it loads, exports every symbol the
header declares, and rejects invalid arguments before touching a GPU.
"""
import os
import re

import pytest

from moce_thesis_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "moce_b200.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(moce_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_the_abi():
    names = header_functions()
    assert "moce_mix" in names and "moce_backward" in names and len(names) >= 10


def test_library_exports_every_declared_symbol():
    lib = capi.lib()
    for name in header_functions():
        assert hasattr(lib, name), name
        assert name in capi.SIGNATURES, name


def test_version_and_error_strings():
    assert b"sm_100a" in capi.lib().moce_version()
    assert capi.lib().moce_last_error() is not None


def test_workspace_queries_are_host_only():
    lib = capi.lib()
    assert lib.moce_backward_workspace_bytes(4, 16, 9, 7, 3) > 0
    assert lib.moce_backward_workspace_bytes(4, 16, 9, 7, 3) % 256 == 0
    assert lib.moce_gate_route_workspace_bytes(4, 16, 7) >= 4 * 7 * 4


@pytest.mark.parametrize("call", [
    lambda l: l.moce_mix(None, 0, 1, 4, 4, None, None, None, 3, 2, None, None, None),
    lambda l: l.moce_route_build(1, 3, 4, 5, 1, 1, 1, 1, None, None, None),          # k > C
    lambda l: l.moce_route_build(1, 3, 4, 2, 1, 1, 1, 1, 1, None, None),             # toff without tslot
    lambda l: l.moce_pool(1, 7, 1, 4, 4, 1, None),                                     # bad dtype
    lambda l: l.moce_forward_dynamic_temp(1, 0, 1, 16, 1, 1, 1, 1, 4, 4, 3, 2, None),  # bad index width
    lambda l: l.moce_gate_temperature(1, 0, None, -1, 4, 4, 1, 3, 2, 1, 1, 0.1, 1.0, None, 1, None),
    lambda l: l.moce_bn_act(1, 0, 2, 4, 9, None, 1, None, None, None, 1, 1, None),        # no scale
    lambda l: l.moce_bn_act(1, 0, 2, 4, 9, 1, 1, None, 1, 1, 1, 1, None),                 # affine without residual
    lambda l: l.moce_bn_act(1, 0, 2, 4, 9, 1, 1, 1, 1, None, 1, 1, None),                 # r_scale without r_shift
])
def test_invalid_arguments_rejected_on_host(call):
    lib = capi.lib()
    assert call(lib) == capi.MOCE_ERR_INVALID
    assert len(lib.moce_last_error()) > 0


def test_workspace_too_small_rejected():
    lib = capi.lib()
    rc = lib.moce_gate_route(1, 0, None, 1, 64, 1, 1, 1, 1, 0.1, 1.0, 1.0, 1, 2, 4, 4, 3, 2, 256, 8, None)
    assert rc == capi.MOCE_ERR_WORKSPACE
