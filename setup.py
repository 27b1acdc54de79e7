"""Build the native parts in place:

    python setup.py build_ext --inplace

* ``rs_nanogpt_b200/_host*.so``  -- C++17 host core (tokenizer, trainer, packers).
* ``rs_nanogpt_b200/_C*.so``     -- sm_100a CUDA kernels (skipped when
  ``NANOGPT_SKIP_CUDA`` is set; nvcc cross-compiles without a GPU).
* ``rs_nanogpt_b200/_C_bounds*.so`` -- the tcgen05 GEMM and flash-attention
  kernels again, built with ``-DNANOGPT_DEBUG_BOUNDS`` (tile-index checks that
  record an error code instead of faulting); used by the debug tests.
"""
import glob
import os

from setuptools import setup

ROOT = os.path.dirname(os.path.abspath(__file__))


def host_extension():
    from pybind11.setup_helpers import Pybind11Extension

    srcs = sorted(glob.glob(os.path.join("csrc", "host", "*.cpp")))
    return Pybind11Extension(
        "rs_nanogpt_b200._host", srcs, cxx_std=17,
        extra_compile_args=["-O3", "-pthread", "-fvisibility=hidden"], extra_link_args=["-pthread", "-static-libstdc++", "-static-libgcc"])


def cuda_extension():
    from torch.utils.cpp_extension import CUDAExtension

    srcs = sorted(glob.glob(os.path.join("csrc", "kernels", "*.cu"))) + sorted(
        glob.glob(os.path.join("csrc", "kernels", "*.cpp")))
    return CUDAExtension(
        "rs_nanogpt_b200._C", srcs,
        include_dirs=[os.path.join(ROOT, "csrc", "kernels")],
        extra_compile_args={
            "cxx": ["-O3", "-std=c++17"],
            "nvcc": ["-O3", "-std=c++17", "-lineinfo", "-gencode", "arch=compute_100a,code=sm_100a",
                     "--expt-relaxed-constexpr"]
            + (["-Xptxas=-v"] if os.environ.get("NANOGPT_PTXAS_VERBOSE") else []),
        })


def bounds_extension():
    from torch.utils.cpp_extension import CUDAExtension

    srcs = sorted(glob.glob(os.path.join("csrc", "kernels", "bounds", "*.cu"))) + [
        os.path.join("csrc", "kernels", "bounds", "bindings_bounds.cpp")]
    return CUDAExtension(
        "rs_nanogpt_b200._C_bounds", srcs,
        include_dirs=[os.path.join(ROOT, "csrc", "kernels")],
        extra_compile_args={
            "cxx": ["-O3", "-std=c++17"],
            "nvcc": ["-O3", "-std=c++17", "-lineinfo", "-gencode", "arch=compute_100a,code=sm_100a",
                     "--expt-relaxed-constexpr"],
        })


def main():
    exts = [host_extension()]
    cmdclass = {}
    if not os.environ.get("NANOGPT_SKIP_CUDA"):
        from torch.utils.cpp_extension import BuildExtension

        exts.append(cuda_extension())
        if not os.environ.get("NANOGPT_SKIP_BOUNDS"):
            exts.append(bounds_extension())
        cmdclass["build_ext"] = BuildExtension.with_options(use_ninja=True)
    setup(name="rs_nanogpt_b200", version="0.1.0", packages=[], ext_modules=exts, cmdclass=cmdclass)


if __name__ == "__main__":
    main()
