"""Build the native parts in-tree.

* ``moce_thesis_b200/lib/libmoce_b200.so`` -- the CUDA kernels and the C ABI
  declared in ``include/moce_b200.h``; nvcc for sm_100a only.
* ``moce_fixed/moce_cuda<EXT_SUFFIX>`` -- the PyTorch binding (reference
  module path ``moce_fixed.moce_cuda``), linked against the library above.

Run ``python -m moce_thesis_b200.build``, or ``python setup.py build_ext``
(``setup.py`` at the repository root drives the same two steps).
Objects go to ``_build/``; nothing is written outside the repository.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "moce_thesis_b200")
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libmoce_b200.so")
BUILD = os.path.join(ROOT, "_build")
BINDING_DIR = os.path.join(ROOT, "moce_fixed")
EXT_SUFFIX = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
BINDING = os.path.join(BINDING_DIR, "moce_cuda" + EXT_SUFFIX)

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                     "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]

CU_SOURCES = ["status.cu", "route.cu", "schedule.cu", "forward.cu", "mix.cu", "stage.cu", "gate.cu", "mix_tc.cu", "simt.cu",
              "backward.cu", "aux.cu", "noalloc.cu", "epilogue.cu"]


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} (exit {r.returncode})")
    if verbose and (r.stdout or r.stderr):
        sys.stdout.write(r.stdout + r.stderr)


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _headers():
    hs = [os.path.join(ROOT, "include", "moce_b200.h")]
    hs += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs


def build_native(verbose=False, force=False, extra_flags=()):
    """Compile every .cu for sm_100a and link libmoce_b200.so."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    objs = []
    hdrs = _headers()
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        if force or _stale(o, [s] + hdrs):
            _run([NVCC] + NVCC_FLAGS + list(extra_flags) + ["-c", s, "-o", o], verbose)
        objs.append(o)
    if force or _stale(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-Xlinker", "-soname=libmoce_b200.so", "-o", LIB] + objs +
             ["-lcudart"], verbose)
    return LIB


def build_binding(verbose=False, force=False):
    """Compile the torch binding against libmoce_b200.so."""
    import torch
    import torch.utils.cpp_extension as ce

    src = os.path.join(CSRC, "moce_layer_cuda.cpp")
    if not (force or _stale(BINDING, [src, LIB] + _headers())):
        return BINDING
    os.makedirs(BINDING_DIR, exist_ok=True)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    inc = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"]]
    libs = ce.library_paths(device_type="cuda")
    cmd = ["g++", "-shared", "-fPIC", "-O2", "-std=c++17", "-w",
           "-DTORCH_EXTENSION_NAME=moce_cuda", "-DTORCH_API_INCLUDE_EXTENSION_H",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]
    cmd += [f"-I{p}" for p in inc]
    cmd += [src, "-o", BINDING + ".tmp"]
    cmd += [f"-L{p}" for p in libs] + [f"-L{LIBDIR}"]
    cmd += ["-lmoce_b200", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
            "-ltorch_python", "-lcudart"]
    cmd += ["-Wl,-rpath,$ORIGIN/../moce_thesis_b200/lib"] + [f"-Wl,-rpath,{p}" for p in libs]
    _run(cmd, verbose)
    shutil.move(BINDING + ".tmp", BINDING)
    return BINDING


def build(verbose=False, force=False):
    build_native(verbose=verbose, force=force)
    build_binding(verbose=verbose, force=force)


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)
