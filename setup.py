"""Builds the native library before the package's files are collected (see pyproject.toml)."""
import importlib.util
import os

from setuptools import Distribution, setup
from setuptools.command.build_py import build_py

HERE = os.path.dirname(os.path.abspath(__file__))


class BuildWithNative(build_py):
    def run(self):
        # The build script alone (importing the package would load the library it builds).
        spec = importlib.util.spec_from_file_location("_bccl_build", os.path.join(HERE, "originccl_b200", "_build.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
        super().run()


class NativeDistribution(Distribution):
    """The package carries a compiled library: platform-specific wheels."""

    def has_ext_modules(self):
        return True


setup(cmdclass={"build_py": BuildWithNative}, distclass=NativeDistribution)
