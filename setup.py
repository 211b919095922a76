"""In-tree build of the sm_100a extension: `python setup.py build_ext --inplace` writes
phung5_b200/_C*.so (built for sm_100a only; no other architecture is targeted)."""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]

nvcc_flags = GENCODE + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xptxas=-v"
                        if os.environ.get("PHX_PTXAS_VERBOSE") == "1" else "-DPHX_QUIET"]

setup(
    name="phung5_b200",
    ext_modules=[
        CUDAExtension(
            name="phung5_b200._C",
            sources=sorted(glob.glob(os.path.join("csrc", "*.cu"))) + ["csrc/bindings.cpp"],
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
