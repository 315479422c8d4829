"""In-tree build of the native parts of tutti_b200.

    python setup.py build_ext --inplace

builds
  * tutti_b200/_core*.so  - StorageRuntime, resolvers, object store, emulated
                            NVMe controllers, DataPaths and the fused GPU io kernel;
  * tutti_b200/_ops*.so   - torch-facing sm_100a kernels (paged KV copy, fp8
                            block quantisation, prefix hashing, NVLink fan-out).
Every CUDA source is compiled for sm_100a only.
"""
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("tutti_b200", "csrc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xptxas", "-v"] + ARCH
CXX = ["-O3", "-std=c++17", "-fvisibility=hidden", "-Wno-unused-parameter"]
INCLUDE = [os.path.join(ROOT, CSRC, "include"), os.path.join(ROOT, CSRC)]


def src(*parts):
    return os.path.join(CSRC, *parts)


CORE_SOURCES = [
    src("runtime", "storage_runtime.cpp"),
    src("nvme", "host_memory.cpp"),
    src("nvme", "emulated_controller.cpp"),
    src("nvme", "snvme_client.cpp"),
    src("testing", "fake_snvme.cpp"),
    src("resolvers", "file_resolvers.cpp"),
    src("datapaths", "gpu_nvme_data_path.cpp"),
    src("datapaths", "posix_data_path.cpp"),
    src("kernels", "io_kernel.cu"),
    src("kernels", "io_noalloc.cu"),
    src("objects", "object_store.cpp"),
    src("config", "yaml_lite.cpp"),
    src("config", "runtime_spec.cpp"),
    src("daemon", "lease_ledger.cpp"),
    src("daemon", "daemon_client.cpp"),
    src("runtime", "tutti_runtime.cpp"),
    src("python", "presets.cpp"),
    src("python", "core_module.cpp"),
]

OPS_SOURCES = [
    src("kernels", "ops_module.cpp"),
    src("kernels", "paged_copy.cu"),
    src("kernels", "fp8_block.cu"),
    src("kernels", "blake2b.cu"),
    src("kernels", "probe_kernels.cu"),
    src("kernels", "ready_flags.cu"),
]

ext_modules = [
    CUDAExtension(
        "tutti_b200._core",
        CORE_SOURCES,
        include_dirs=INCLUDE,
        extra_compile_args={"cxx": CXX, "nvcc": NVCC},
        libraries=["cudart"],
    ),
]
if all(os.path.exists(os.path.join(ROOT, s)) for s in OPS_SOURCES):
    ext_modules.append(
        CUDAExtension(
            "tutti_b200._ops",
            OPS_SOURCES,
            include_dirs=INCLUDE,
            extra_compile_args={"cxx": CXX, "nvcc": NVCC},
            libraries=["cudart"],
        )
    )

setup(
    name="tutti_b200",
    version="0.1.0",
    packages=["tutti_b200", "tutti", "tutti_runtime"],  # tutti / tutti_runtime: Tutti's import paths
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
