"""Build the sm_100a kernel library in-tree:  python setup.py build_ext --inplace"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("vllm_sly_radiance_b200", "csrc")

NVCC_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
]
if os.environ.get("RADIANCE_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + [os.path.join(CSRC, "bindings.cpp")]


def build_noalloc_lib():
    """The allocation-free argmax C entry point alone, in a library that links only the CUDA
    runtime (for C / C++ hosts without torch): vllm_sly_radiance_b200/libradiance_noalloc.so."""
    import subprocess
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    src = os.path.join(HERE, CSRC, "argmax_noalloc.cu")
    out = os.path.join(HERE, "vllm_sly_radiance_b200", "libradiance_noalloc.so")
    if os.path.exists(out) and os.path.getmtime(out) >= max(
            os.path.getmtime(src), os.path.getmtime(os.path.join(HERE, CSRC, "radiance_noalloc.h"))):
        return
    subprocess.run([nvcc, *[f for f in NVCC_FLAGS if f != "-DNDEBUG"], "-shared",
                    "-Xcompiler", "-fPIC", "-I", os.path.join(HERE, CSRC), src, "-o", out],
                   check=True)


class Build(BuildExtension):
    def run(self):
        super().run()
        build_noalloc_lib()

setup(
    name="vllm_sly_radiance_b200",
    version="0.1.0",
    packages=["vllm_sly_radiance_b200"],
    ext_modules=[
        CUDAExtension(
            name="vllm_sly_radiance_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": Build.with_options(use_ninja=True)},
)
