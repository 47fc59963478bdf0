"""Wheel build of the mamba_onnx package with its CUDA library.

The reference's build backend (build_backend.py:83-89) copies only its cpp
and zig libraries into the wheel. Here `build_py` first runs the Makefile
(nvcc, sm_100a) so that mamba_onnx/libmamba_ops_cuda.so is built and packaged
with the Python modules; the wheel is platform-specific. Build from a
checkout of this repository (the Makefile reads ../include):

    python -m pip wheel --no-build-isolation --no-deps mamba-onnx_b200
"""
import os
import subprocess
from pathlib import Path

from setuptools import Distribution, setup
from setuptools.command.build_py import build_py

HERE = Path(__file__).resolve().parent


class BuildWithMake(build_py):
    def run(self):
        subprocess.check_call(["make", "-C", str(HERE), f"-j{min(8, os.cpu_count() or 4)}"])
        if not (HERE / "mamba_onnx" / "libmamba_ops_cuda.so").exists():
            raise RuntimeError("make did not produce mamba_onnx/libmamba_ops_cuda.so")
        super().run()


class BinaryDistribution(Distribution):
    """Carries a compiled library: tag the wheel for this platform."""

    def has_ext_modules(self):
        return True


setup(cmdclass={"build_py": BuildWithMake}, distclass=BinaryDistribution)
