"""Build the heiretsu_b200 native extension in-tree for B200 (sm_100a).

    python setup.py build_ext --inplace
    HB_DEBUG=1 python setup.py build_ext --inplace     # with device-side invariant checks

produces heiretsu_b200/_C*.so next to the Python sources. Kernel files
(*.cu) are torch-free and compile in parallel; *.cpp files hold the
torch-facing argument checks and bindings.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("heiretsu_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__",
]
CXX_FLAGS = ["-O2", "-std=c++17"]
if os.environ.get("HB_DEBUG", "0") == "1":
    # Kernels check invariants the host cannot see (MoE row positions within
    # the staging capacity, barrier epochs) and record failures in the status word.
    NVCC_FLAGS.append("-DHB_DEBUG")


def sources():
    files = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    return [os.path.relpath(f, HERE) for f in files]


os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 8))

setup(
    name="heiretsu_b200",
    version="0.1.0",
    packages=["heiretsu_b200"],
    ext_modules=[
        CUDAExtension(
            name="heiretsu_b200._C",
            sources=sources(),
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
