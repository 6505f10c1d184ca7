"""Build the MoCE sm_100a kernels and their PyTorch binding in place.

    python setup.py build_ext          # (or: python -m moce_thesis_b200.build)

Two steps, both for sm_100a (B200) only -- nvcc ``-gencode
arch=compute_100a,code=sm_100a``, no other architecture, no Triton, no CPU
fallback:

* ``moce_thesis_b200/lib/libmoce_b200.so``: every CUDA source under
  ``moce_thesis_b200/csrc`` and the C ABI of ``include/moce_b200.h``;
* ``moce_fixed/moce_cuda<EXT_SUFFIX>``: the PyTorch binding importable as
  ``moce_fixed.moce_cuda``, the module path the reference's ``MoCE.py``
  imports (the reference builds it with its own ``moce_fixed/setup.py``).

Both land inside the repository; ``build_ext --force`` rebuilds everything.
"""
from setuptools import Command, setup


class BuildExt(Command):
    description = "compile the sm_100a kernels and the moce_fixed.moce_cuda binding in place"
    user_options = [("force", "f", "rebuild everything")]
    boolean_options = ["force"]

    def initialize_options(self):
        self.force = False

    def finalize_options(self):
        self.force = bool(self.force)

    def run(self):
        from moce_thesis_b200 import build
        build.build(verbose=True, force=self.force)


setup(
    name="moce_thesis_b200",
    version="0.2.0",
    description="B200-native (sm_100a) MoCE layer kernels behind the reference's moce_fixed.moce_cuda surface",
    packages=["moce_thesis_b200", "moce_fixed"],
    cmdclass={"build_ext": BuildExt},
)
