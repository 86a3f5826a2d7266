"""In-tree build of the native modules (``python setup.py build_ext --inplace``).

* ``bitresearch_b200._native_data``: C++ document source + best-fit packer (CPU).
* ``bitresearch_b200._C``: the sm_100a CUDA kernels and their bindings. Compiled only for
  ``sm_100a`` (``-gencode arch=compute_100a,code=sm_100a``); torch's own arch list is bypassed.
"""
import glob
import os

from setuptools import find_packages, setup

ROOT = os.path.dirname(os.path.abspath(__file__))


def _ext_modules():
    import pybind11
    from setuptools import Extension
    from torch.utils.cpp_extension import CUDAExtension

    data = Extension(
        "bitresearch_b200._native_data",
        ["csrc/data/packer.cpp", "csrc/data/bpe.cpp"],
        include_dirs=[pybind11.get_include()],
        extra_compile_args=["-O3", "-std=c++17"],
        language="c++",
    )
    cu = sorted(glob.glob(os.path.join(ROOT, "csrc", "kernels", "*.cu")))
    cpp = sorted(glob.glob(os.path.join(ROOT, "csrc", "kernels", "*.cpp")))
    nvcc = [
        "-O3", "-std=c++17", "-lineinfo",
        "-gencode", "arch=compute_100a,code=sm_100a",
        "--expt-relaxed-constexpr", "--use_fast_math",
        "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
        "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__",
        "-Xptxas", "-v" if os.environ.get("BR_PTXAS_VERBOSE") else "-O3",
    ]
    cuda = CUDAExtension(
        "bitresearch_b200._C",
        [os.path.relpath(p, ROOT) for p in cpp + cu],
        include_dirs=[os.path.join(ROOT, "csrc", "kernels")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc},
        libraries=["cuda"],
    )
    return [data, cuda] if cu else [data]


def _cmdclass():
    from torch.utils.cpp_extension import BuildExtension
    return {"build_ext": BuildExtension.with_options(use_ninja=True)}


os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")  # the explicit -gencode above is what is compiled
setup(
    name="bitresearch_b200",
    version="0.1.0",
    packages=find_packages(include=["bitresearch_b200", "bitresearch_b200.*"]),
    ext_modules=_ext_modules(),
    cmdclass=_cmdclass(),
)
