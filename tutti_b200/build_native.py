"""Builds the standalone native executables next to the package:

* ``tutti_b200/bin/tutti_daemon``        - the device-manager daemon (queue leases);
* ``tutti_b200/bin/tutti_posix_roundtrip`` - the public C++ API end to end on the POSIX data path
* ``tutti_b200/bin/tutti_native_tests``  - C++ contract tests of the runtime
  (StorageRuntime against the mock DataPath kit, object store, config spec);
* ``tutti_b200/bin/tutti_snvme_smoke``   - bring-up check of one controller behind
  the snvme driver (``--node /dev/snvmN``) or the fake driver (``--fake``).

    python -m tutti_b200.build_native
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
BIN = os.path.join(PKG, "bin")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")

CXX = ["g++", "-O2", "-std=c++17", "-pthread", "-I", os.path.join(CSRC, "include"), "-I", CSRC,
       "-I", os.path.join(CUDA, "include")]

TARGETS = {
    "tutti_daemon": (["daemon/daemon_main.cpp", "daemon/lease_ledger.cpp", "daemon/host_admin.cpp",
                      "config/yaml_lite.cpp", "nvme/snvme_client.cpp", "nvme/host_memory.cpp",
                      "nvme/emulated_controller.cpp"],
                     ["-L", os.path.join(CUDA, "lib64"), "-lcudart", "-Wl,-rpath," + os.path.join(CUDA, "lib64")]),
    "tutti_native_tests": ([
        "tests/native_tests.cpp", "tests/runtime_contract_tests.cpp", "tests/datapath_contract_tests.cpp",
        "tests/snvme_client_tests.cpp", "nvme/snvme_client.cpp", "testing/fake_snvme.cpp",
        "tests/host_admin_tests.cpp", "daemon/host_admin.cpp",
        "runtime/storage_runtime.cpp", "datapaths/posix_data_path.cpp", "objects/object_store.cpp",
        "config/yaml_lite.cpp", "config/runtime_spec.cpp", "daemon/lease_ledger.cpp",
        "resolvers/file_resolvers.cpp", "nvme/emulated_controller.cpp", "nvme/host_memory.cpp",
    ], ["-L", os.path.join(CUDA, "lib64"), "-lcudart", "-Wl,-rpath," + os.path.join(CUDA, "lib64")]),
    "tutti_snvme_smoke": ([
        "examples/snvme_smoke.cpp", "nvme/snvme_client.cpp", "testing/fake_snvme.cpp",
        "nvme/emulated_controller.cpp", "nvme/host_memory.cpp",
    ], ["-L", os.path.join(CUDA, "lib64"), "-lcudart", "-Wl,-rpath," + os.path.join(CUDA, "lib64")]),
    # the public C++ API without a GPU: runtime assembly, open, register, submit, wait
    "tutti_posix_roundtrip": ([
        "examples/posix_roundtrip.cpp", "runtime/storage_runtime.cpp", "resolvers/file_resolvers.cpp",
        "datapaths/posix_data_path.cpp",
    ], ["-L", os.path.join(CUDA, "lib64"), "-lcudart", "-Wl,-rpath," + os.path.join(CUDA, "lib64")]),
}


def build(names=None) -> None:
    os.makedirs(BIN, exist_ok=True)
    for name, (srcs, libs) in TARGETS.items():
        if names and name not in names:
            continue
        paths = [os.path.join(CSRC, s) for s in srcs]
        if not all(os.path.exists(p) for p in paths):
            continue
        out = os.path.join(BIN, name)
        newest = max(os.path.getmtime(os.path.join(d, f)) for d, _, fs in os.walk(CSRC) for f in fs
                     if f.endswith((".h", ".cpp", ".cuh", ".cu")))
        if os.path.exists(out) and newest <= os.path.getmtime(out):
            continue
        subprocess.run(CXX + paths + ["-o", out] + libs, check=True)


if __name__ == "__main__":
    build(sys.argv[1:] or None)
