"""Build the sm_100a CUDA extension in place:

    python setup.py build_ext --inplace

produces ``nano_megatron_b200/_C*.so`` next to the Python sources, so it
travels with the repository (no JIT cache). Only sm_100a code is generated.
"""

import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("nano_megatron_b200", "csrc")

SOURCES = [
    "bindings.cpp",
    "elementwise_bindings.cpp",
    "gemm.cu",
    "kernels.cu",
    "attention.cu",
    "attention_tc.cu",
    "attention_bwd_tc.cu",
    "fused_tp.cu", "dp_reduce.cu",
    "noalloc.cu",
    "fp32.cu",
    "tc_probe.cu",
]

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas=-warn-spills",
]

setup(
    name="nano_megatron_b200",
    version="0.1.0",
    description="Megatron-style TP x SP x PP x DP GPT training with hand-written sm_100a (B200) kernels",
    python_requires=">=3.10",
    install_requires=["torch>=2.4"],
    packages=find_packages(include=["nano_megatron_b200", "nano_megatron_b200.*"]),
    ext_modules=[
        CUDAExtension(
            name="nano_megatron_b200._C",
            sources=[os.path.join(CSRC, s) for s in SOURCES],
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
