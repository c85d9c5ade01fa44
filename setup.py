"""Build script for my_muon_fsdp2_b200 and its sm_100a extension.

    python setup.py build_ext --inplace     # builds my_muon_fsdp2_b200/_C*.so in the tree
    MMF_DEVICE_CHECKS=1 python setup.py build_ext --inplace --force   # debug build with device checks

The extension is compiled for Blackwell only (``-gencode arch=compute_100a,code=sm_100a``);
passing the arch flag explicitly bypasses torch's own TORCH_CUDA_ARCH_LIST handling.
"""
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("my_muon_fsdp2_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]
CXX_FLAGS = ["-O3", "-std=c++17"]
if os.environ.get("MMF_DEVICE_CHECKS", "0") == "1":
    # debug build: device-side index / segment checks that record an error code and skip
    NVCC_FLAGS.append("-DMMF_DEVICE_CHECKS")
    CXX_FLAGS.append("-DMMF_DEVICE_CHECKS")

SOURCES = [
    "bindings.cpp",
    "tc_gemm.cu",
    "linear_gemm.cu",
    "optim_kernels.cu",
    "model_kernels.cu",
    "attention.cu",
    "symm_comm.cu",
    "noalloc.cu",
]


def ext_modules():
    srcs = [os.path.join(CSRC, s) for s in SOURCES if os.path.exists(os.path.join(HERE, CSRC, s))]
    return [
        CUDAExtension(
            name="my_muon_fsdp2_b200._C",
            sources=srcs,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        )
    ]


setup(
    name="my-muon-fsdp2-b200",
    version="0.1.0",
    description="Blackwell-native (sm_100a) FSDP2 + Muon training library",
    packages=find_packages(include=["my_muon_fsdp2_b200", "my_muon_fsdp2_b200.*"]),
    python_requires=">=3.10",
    ext_modules=ext_modules(),
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={
        "console_scripts": [
            "muon-fsdp=my_muon_fsdp2_b200.cli:muon_fsdp_main",
            "fsdp2-utils=my_muon_fsdp2_b200.cli:fsdp2_utils_main",
        ]
    },
)
