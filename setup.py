"""Builds the cascadia_b200 CUDA extension in-tree for sm_100a (B200).

    python setup.py build_ext --inplace

produces ``cascadia_b200/_C*.so``.  Only Blackwell (``compute_100a``) code is
generated: the kernels use tcgen05 / TMA / TMEM instructions that exist on no
other architecture.
"""
import os

# Keep torch from adding its own multi-arch -gencode list.
os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")

import pybind11  # noqa: E402
from setuptools import Extension, setup  # noqa: E402
from torch.utils.cpp_extension import BuildExtension, CUDAExtension  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")

SOURCES = [
    "bindings.cpp",
    "gemm_w4a16.cu",
    "gemm_bf16.cu",
    "hc.cu",
    "attention.cu",
    "elementwise.cu",
    "comm.cu",
    "moe.cu",
    "gemv_w4a16.cu",
    "ep.cu",
    "mla.cu",
    "gdn.cu",
    "ffn_sparse.cu",
]

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode=arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_HALF2_OPERATORS__",
]
if os.environ.get("CASCADIA_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")


def main():
    setup(
        name="cascadia_b200",
        version="0.1.0",
        packages=[],
        ext_modules=[
            CUDAExtension(
                name="cascadia_b200._C",
                sources=[os.path.join("csrc", s) for s in SOURCES],
                include_dirs=[CSRC],
                extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
            ),
            # Native runtime (no CUDA): TCP stage transport, KV block allocator.
            Extension(
                name="cascadia_b200._runtime",
                sources=[os.path.join("csrc", "runtime", "runtime.cpp")],
                include_dirs=[pybind11.get_include()],
                extra_compile_args=["-O2", "-std=c++17", "-fvisibility=hidden"],
                language="c++",
            ),
        ],
        cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    )


if __name__ == "__main__":
    main()
