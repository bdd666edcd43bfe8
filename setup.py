"""Build the native extensions of starry_unigraph in-tree.

    python setup.py build_ext --inplace

* ``starry_unigraph._C``      CUDA kernels for sm_100a (tcgen05 GEMMs, TGN step,
                              DTDG ops, peer-memory collectives, fused Adam).
* ``starry_unigraph._native`` host C++ (OpenMP): temporal neighbour sampler with
                              the reference sampler's policies, T-CSR, TPPR,
                              adaptive time split, graph partitioner.

Only sm_100a is targeted; the CUDA architecture list is pinned so that torch
does not add other -gencode targets.
"""
from __future__ import annotations

import glob
import os

from setuptools import setup

os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))

from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
SKIP_CUDA = os.environ.get("SU_SKIP_CUDA", "0") == "1"

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-v" if os.environ.get("SU_PTXAS_VERBOSE") else "-O3",
]
CXX_FLAGS = ["-O3", "-std=c++17"]

ext_modules = []
if not SKIP_CUDA:
    # .cu files are torch-free (fast nvcc); torch wrappers are plain C++.
    cuda_sources = sorted(glob.glob(os.path.join("csrc", "cuda", "*.cu"))) + sorted(
        glob.glob(os.path.join("csrc", "ops", "*.cpp"))
    )
    ext_modules.append(
        CUDAExtension(
            name="starry_unigraph._C",
            sources=cuda_sources,
            include_dirs=[os.path.join(ROOT, "csrc", "cuda"), os.path.join(ROOT, "csrc", "ops")],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        )
    )

def _omp_flags():
    """Link libgomp explicitly: the active gcc prefix may ship omp.h without libgomp."""
    for d in sorted(glob.glob("/usr/lib/gcc/x86_64-linux-gnu/*"), reverse=True):
        if os.path.exists(os.path.join(d, "libgomp.so")):
            return [], ["-L" + d, "-lgomp", "-Wl,-rpath,/usr/lib/x86_64-linux-gnu"]
    return [], ["-fopenmp"]


OMP_INC, OMP_LINK = _omp_flags()

host_sources = sorted(glob.glob(os.path.join("csrc", "host", "*.cpp")))
if host_sources:
    ext_modules.append(
        CppExtension(
            name="starry_unigraph._native",
            sources=host_sources,
            include_dirs=[os.path.join(ROOT, "csrc", "host")],
            extra_compile_args=CXX_FLAGS + ["-fopenmp"] + OMP_INC,
            extra_link_args=OMP_LINK,
        )
    )

setup(
    name="starry_unigraph",
    version="0.2.0",
    packages=[],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
