"""Build the sm_100a CUDA extension in-tree: ``python setup.py build_ext --inplace``."""
import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
HERE = os.path.dirname(os.path.abspath(__file__))
NVCC_FLAGS = ["-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
              "--expt-relaxed-constexpr", "--expt-extended-lambda", "-DNDEBUG"]
if os.environ.get("MIMIR_PTXAS_VERBOSE") == "1":
    NVCC_FLAGS += ["-Xptxas", "-v"]

sources = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + ["csrc/bindings.cpp"]
# Link the system's shared libstdc++ (the one torch itself uses).  Where the compiler's own
# unversioned libstdc++.so link is missing, the linker would otherwise fall back to the static
# archive and every extension would carry a private copy of the C++ runtime (its stream/locale
# state is not set up on threads other than the main one, so formatting an error message there
# crashed).
LINK_ARGS = []
for candidate in ("/usr/lib/x86_64-linux-gnu/libstdc++.so.6", "/usr/lib64/libstdc++.so.6"):
    if os.path.exists(candidate):
        LINK_ARGS = [candidate]
        break
host_sources = sorted(glob.glob(os.path.join("csrc", "host", "*.cpp")))

setup(
    name="mimir_b200",
    version="0.1.0",
    packages=find_packages(include=["mimir_b200", "mimir_b200.*"]),
    package_data={"mimir_b200": ["conf/**/*.yaml", "evaluation/suites/*.json"]},
    ext_modules=[CUDAExtension("mimir_b200._C", sources=sources,
                               include_dirs=[os.path.join(HERE, "csrc")],
                               extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
                               extra_link_args=LINK_ARGS),
                 CppExtension("mimir_b200._host", sources=host_sources,
                              extra_compile_args={"cxx": ["-O3", "-std=c++17"]}, extra_link_args=LINK_ARGS)],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={"console_scripts": ["mimir=mimir_b200.cli:main"]},
)
