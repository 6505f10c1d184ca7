"""Drop-in replacement for the reference package ``moce_fixed``.

``moce_fixed.moce_cuda`` is the compiled PyTorch binding of the sm_100a MoCE
kernels (source: ``moce_thesis_b200/csrc/moce_layer_cuda.cpp``), exporting the
seven functions of the reference binding (``moce_fixed/moce_layer_cuda.cpp``
in Elianiluk/MoCE_thesis) with the same arguments and return values, so
the reference ``MoCE.py`` (``import moce_fixed.moce_cuda``) runs on it
unchanged.  Build it with ``python -m moce_thesis_b200.build``; importing it
unbuilt raises ImportError (there is no CPU fallback).
"""
