"""Build the in-tree sm_100a extensions: ``python setup.py build_ext --inplace``.

Only ``-gencode arch=compute_100a,code=sm_100a`` is emitted (B200); torch's own arch list is not used.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xptxas=-v"
               if os.environ.get("BARQ_PTXAS_V") else "-DBARQ_QUIET=1"]
# BARQ_DIAG=1: compile the mainloop diagnostic switches (BARQ_GEMM_EXP / BARQ_GEMV_EXP) in
if os.environ.get("BARQ_DIAG"):
    NVCC.append("-DBARQ_DIAG=1")
if os.environ.get("BARQ_GEMM_TS"):  # 0: weight operand through shared memory for every tile size
    NVCC.append("-DBARQ_GEMM_TS=" + os.environ["BARQ_GEMM_TS"])
CXX = ["-O3", "-std=c++17"]

kernels = sorted(glob.glob(os.path.join("csrc", "kernels", "*.cu")))

ext_modules = [
    CUDAExtension(
        name="barq_inference_b200._C",
        sources=["csrc/bindings.cpp", *kernels],
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={"cxx": CXX, "nvcc": NVCC},
        libraries=["cuda"],
    ),
    CUDAExtension(
        name="barq_inference_b200._cpu_ref",
        sources=sorted(glob.glob(os.path.join("csrc", "cpu_ref", "*.cpp"))),
        extra_compile_args={"cxx": CXX, "nvcc": NVCC},
    ),
    CppExtension(
        name="barq_inference_b200._native",
        sources=sorted(glob.glob(os.path.join("csrc", "native", "*.cpp"))),
        extra_compile_args={"cxx": CXX},
    ),
]

setup(
    name="barq_inference_b200",
    version="0.1.0",
    packages=["barq_inference_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    # the reference's binary name, so scripts written for it keep working after a pip install
    entry_points={"console_scripts": ["barq-inference=barq_inference_b200.cli:main", "barq=barq_inference_b200.cli:main"]},
)
