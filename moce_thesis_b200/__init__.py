"""B200-native (sm_100a) MoCE layer hot path.

The package holds the CUDA kernels and C ABI (``csrc/``, built into
``lib/libmoce_b200.so``), the PyTorch binding that mirrors the reference
``moce_fixed.moce_cuda`` module, and ``MoCE`` -- the reference layer's
nn.Module surface (Elianiluk/MoCE_thesis ``MoCE.py``) routed through those
kernels in both eval and train mode.
"""
from .moce import MoCE, MoCEFunction, check_faults, native  # noqa: F401

__all__ = ["MoCE", "MoCEFunction", "check_faults", "native"]
