"""Build the in-tree extensions of mesh_b200.

``python setup.py build_ext --inplace`` compiles
* ``mesh_b200/_C``       : the sm_100a CUDA kernels (tcgen05 GEMM, attention, fused all-reduce, ...)
* ``mesh_b200/_runtime`` : the native host runtime (KV page allocator, decode scheduler, TCP framing)
Only sm_100a code is generated (``-gencode arch=compute_100a,code=sm_100a``).
"""
import os
from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension, CppExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xptxas=-v" if os.environ.get("MESH_PTXAS_V") else "-DMESH_QUIET"]
CXX = ["-O3", "-std=c++17"]

ext_modules = [
    CUDAExtension(
        name="mesh_b200._C",
        sources=[
            "csrc/bindings.cpp",
            "csrc/kernels/gemm_tcgen05.cu",
            "csrc/kernels/elementwise.cu",
            "csrc/kernels/attn_decode.cu",
            "csrc/kernels/attn_prefill.cu",
            "csrc/kernels/attn_prefill_tc.cu",
            "csrc/kernels/kv_pages.cu",
            "csrc/kernels/gemm_2sm.cu",
            "csrc/kernels/sampling.cu",
            "csrc/kernels/allreduce.cu",
        ],
        include_dirs=[os.path.join(ROOT, "csrc", "include")],
        extra_compile_args={"cxx": CXX, "nvcc": NVCC},
    ),
]
from pybind11.setup_helpers import Pybind11Extension  # noqa: E402

ext_modules.append(Pybind11Extension(
    "mesh_b200._runtime",
    sources=["csrc/runtime/runtime.cpp"],
    extra_compile_args=CXX,
    cxx_std=17,
))

setup(
    name="mesh_b200",
    version="0.1.0",
    packages=["mesh_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={"console_scripts": ["mesh=mesh_b200.cli.main:main",
                                      "mesh-control-plane=mesh_b200.control_plane.app:main"]},
)
