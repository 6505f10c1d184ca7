"""Build the reference's own CUDA extension from its sources -- TEST
INFRASTRUCTURE ONLY (the second oracle and the reference GPU timing).

    python oracle/build_ref.py [<path of the reference checkout>]

Compiles ``moce_fixed/moce_kernel.cu`` and ``moce_fixed/moce_layer_cuda.cpp``
of Elianiluk/MoCE_thesis, unmodified and where they lie, with the flags of the
reference's ``moce_fixed/setup.py:37-58`` (``-O3 --use_fast_math -lineinfo``)
for sm_100a, into ``oracle/_ref/moce_cuda_ref<EXT_SUFFIX>``: a torch extension
importable as ``moce_cuda_ref`` with the reference's seven functions.  The
reference's own build system (its ``setup.py``) is not run, and nothing is
written outside ``oracle/_ref/`` (objects included).  The shipped binaries of
the reference are never used.

Only the tests, ``__graft_entry__.smoke()`` and ``bench.py --impl reference``
load the result, as a checker and as the reference GPU path to time.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
EXT_SUFFIX = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
MODULE = "moce_cuda_ref"
TARGET = os.path.join(OUT, MODULE + EXT_SUFFIX)
DEFAULT_REF = "/root/reference"
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _sources(ref_root):
    d = os.path.join(ref_root, "moce_fixed")
    return os.path.join(d, "moce_kernel.cu"), os.path.join(d, "moce_layer_cuda.cpp")


def available(ref_root=DEFAULT_REF):
    return all(os.path.isfile(p) for p in _sources(ref_root))


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout[-4000:] + r.stderr[-4000:])
        raise RuntimeError(f"reference build step failed: {cmd[0]} (exit {r.returncode})")


def build(ref_root=DEFAULT_REF, verbose=False, force=False):
    """Compile the reference extension; returns the path of the module, or
    None when the reference sources are not present (e.g. on a GPU box, which
    uses the module built beforehand)."""
    if not available(ref_root):
        return TARGET if os.path.exists(TARGET) else None
    cu, cpp = _sources(ref_root)
    if not force and os.path.exists(TARGET) and os.path.getmtime(TARGET) >= max(os.path.getmtime(cu),
                                                                                os.path.getmtime(cpp)):
        return TARGET
    import torch
    import torch.utils.cpp_extension as ce
    os.makedirs(OUT, exist_ok=True)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    inc = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"]]
    libs = ce.library_paths(device_type="cuda")
    defs = [f"-DTORCH_EXTENSION_NAME={MODULE}", "-DTORCH_API_INCLUDE_EXTENSION_H",
            f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]
    incs = [f"-I{p}" for p in inc]
    o_cu = os.path.join(OUT, "moce_kernel.o")
    o_cpp = os.path.join(OUT, "moce_layer_cuda.o")
    # the reference's nvcc flags (moce_fixed/setup.py:49-54), for sm_100a only
    _run([os.path.join(CUDA_HOME, "bin", "nvcc"), "-gencode", "arch=compute_100a,code=sm_100a", "-O3",
          "--use_fast_math", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-w"] + defs + incs +
         ["-c", cu, "-o", o_cu], verbose)
    _run(["g++", "-O3", "-fPIC", "-std=c++17", "-w"] + defs + incs + ["-c", cpp, "-o", o_cpp], verbose)
    _run(["g++", "-shared", "-o", TARGET + ".tmp", o_cpp, o_cu] + [f"-L{p}" for p in libs] +
         ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python", "-lcudart"] +
         [f"-Wl,-rpath,{p}" for p in libs], verbose)
    os.replace(TARGET + ".tmp", TARGET)
    return TARGET


def load():
    """Import the built reference extension (raises ImportError if unbuilt)."""
    import importlib.util
    if not os.path.exists(TARGET):
        raise ImportError(f"{TARGET} is not built; run `python oracle/build_ref.py <reference checkout>`")
    spec = importlib.util.spec_from_file_location(MODULE, TARGET)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else DEFAULT_REF
    path = build(root, verbose=True, force="--force" in sys.argv)
    print(path if path else f"reference sources not found under {root}")
