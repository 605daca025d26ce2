# SPDX-License-Identifier: Apache-2.0
"""Packaging: `pip install .` builds libvccl.so and the native tools with the
Makefile (nvcc, sm_100a) before the Python package is copied."""

import os
import subprocess

from setuptools import setup
from setuptools.command.build_py import build_py
from setuptools.dist import Distribution


class BuildNative(build_py):
    def run(self):
        root = os.path.dirname(os.path.abspath(__file__))
        subprocess.check_call(["make", "-j", str(os.cpu_count() or 8)], cwd=root)
        super().run()


class NativeDistribution(Distribution):
    """The package ships a compiled library (libvccl.so and the tools), so
    its wheel is tagged for the platform, not as pure Python."""

    def has_ext_modules(self):
        return True


setup(cmdclass={"build_py": BuildNative}, distclass=NativeDistribution)
