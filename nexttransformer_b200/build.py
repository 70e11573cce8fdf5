"""Build the native extensions in place: ``python -m nexttransformer_b200.build``.

``_C`` holds the sm_100a CUDA kernels; ``_native`` the host-side C++ runtime (best-fit data
packing, BPE merge training).

The kernels live in ``nexttransformer_b200/csrc``.  They are compiled only for Blackwell
(``-gencode arch=compute_100a,code=sm_100a``) and linked into ``nexttransformer_b200/_C*.so``
next to this file, so the built library travels with the source tree.  ``nvcc`` cross-compiles
without a GPU; ninja rebuilds only the translation units that changed.
"""
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SOURCES = ["bindings.cpp", "gemm_sm100.cu", "gemm_noalloc.cu", "elementwise.cu", "optim.cu", "attention_sm100.cu",
           "comm.cu", "linear_attn.cu", "delta_scan.cu", "delta_prep.cu", "moe.cu", "moe_route.cu", "sparse_attn.cu", "sparse_teacher.cu", "nsa_compress.cu", "msar.cu", "residual.cu", "probe_sm100.cu", "plugin_ops.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__",
]


def build(verbose=False):
    """Compile every CUDA source of the package into ``nexttransformer_b200/_C``."""
    from setuptools import setup
    from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

    os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
    ext = CUDAExtension(
        name="nexttransformer_b200._C",
        sources=[str(HERE / "csrc" / s) for s in SOURCES],
        include_dirs=[str(HERE / "csrc")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
    )
    host = CppExtension(
        name="nexttransformer_b200._native",
        sources=[str(HERE / "csrc" / "native_host.cpp")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"]},
    )
    build_temp = HERE.parent / "build" / "nt_ext"
    argv = ["build_ext", "--inplace", "--build-temp", str(build_temp)]
    cwd = os.getcwd()
    os.chdir(HERE.parent)
    try:
        setup(name="nexttransformer_b200_ext", ext_modules=[ext, host],
              cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
              script_args=argv if verbose else ["-q", *argv])
    finally:
        os.chdir(cwd)


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
