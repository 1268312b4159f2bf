"""Build the revpp CUDA extension in-tree for sm_100a.

    python setup.py build_ext --inplace        # -> revpp/_C.*.so

Only sm_100a code is generated (the explicit -gencode flag stops torch from
adding its own arch list).
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))

# Build with the system toolchain, which links libstdc++ dynamically: a second,
# statically linked C++ runtime inside the extension breaks C++ exceptions that
# cross into torch's runtime.
for _var, _val in (("CC", "/usr/bin/gcc"), ("CXX", "/usr/bin/g++"), ("LDSHARED", "/usr/bin/g++ -shared")):
    if os.path.exists(_val.split()[0]):
        os.environ[_var] = _val
CSRC = os.path.join(HERE, "csrc")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
sources = [os.path.relpath(s, HERE) for s in sources]

nvcc_flags = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-ccbin=/usr/bin/g++",
    "-Xptxas=-v" if os.environ.get("REVPP_PTXAS_VERBOSE") else "-Xptxas=-O3",
]
if os.environ.get("REVPP_DEBUG_BOUNDS"):
    nvcc_flags.append("-DREVPP_DEBUG_BOUNDS=1")

setup(
    name="revpp",
    ext_modules=[
        CUDAExtension(
            name="revpp._C",
            sources=sources,
            include_dirs=[CSRC],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
