# SPDX-License-Identifier: Apache-2.0
"""Packaging: `pip install .` builds libvccl.so and the native tools with the
Makefile (nvcc, sm_100a) before the Python package is copied."""

import os
import subprocess

from setuptools import setup
from setuptools.command.build_py import build_py


class BuildNative(build_py):
    def run(self):
        root = os.path.dirname(os.path.abspath(__file__))
        subprocess.check_call(["make", "-j", str(os.cpu_count() or 8)], cwd=root)
        super().run()


setup(cmdclass={"build_py": BuildNative})
