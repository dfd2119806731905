"""Builds the `ZipMoE` Python module (csrc/zipmoe_module.cpp) in place, linked
against libzmoe.so in this directory:

    python setup_zipmoe.py build_ext --inplace --build-temp _build/pyext
"""
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

setup(
    name="ZipMoE",
    ext_modules=[CUDAExtension(
        "ZipMoE",
        [os.path.join("csrc", "zipmoe_module.cpp")],
        include_dirs=[os.path.join(ROOT, "include")],
        library_dirs=[HERE],
        libraries=["zmoe"],
        extra_compile_args={"cxx": ["-O2", "-g0", "-Wall", "-Wno-unused-parameter"]},
        extra_link_args=["-Wl,-rpath,$ORIGIN"],
    )],
    cmdclass={"build_ext": BuildExtension},
)
