"""Command line for operators: build, status, daemon, probes, tests and benchmarks.

    python -m tutti_b200 build                 # CUDA extensions (sm_100a) + native executables
    python -m tutti_b200 status [--json]       # GPUs, extensions, native binaries, a runtime's capabilities
    python -m tutti_b200 daemon --config F     # run tutti_daemon (queue leases) in the foreground
    python -m tutti_b200 selftest              # C++ contract suite (no GPU needed)
    python -m tutti_b200 fiemap FILE           # extents the FIEMAP resolver sees
    python -m tutti_b200 probe-raid0 md0 [--sysfs /sys]
    python -m tutti_b200 topology [--sysfs /sys]   # NVMe drive -> affine GPU over the PCIe tree
    python -m tutti_b200 bench {kernels,ttft,fanout,mla,trace} [args...]

Parity: reference scripts/tutti-env.sh (build, build-ext, test, daemon, status
subcommands), scripts/tutti-md (md RAID0 inspection) and
scripts/pci_topology_check.sh (drive / GPU switch affinity).
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
BENCHES = {"kernels": "kernels", "ttft": "ttft", "fanout": "fanout", "mla": "mla_indexer", "trace": "serving_trace"}


def _bin(name: str) -> str:
    return os.path.join(PKG, "bin", name)


def cmd_build(_args) -> int:
    r = subprocess.run([sys.executable, "setup.py", "build_ext", "--inplace"], cwd=ROOT)
    if r.returncode:
        return r.returncode
    from . import build_native

    build_native.build()
    return 0


def status() -> dict:
    out = {"package": PKG, "binaries": {n: os.path.exists(_bin(n)) for n in ("tutti_daemon", "tutti_native_tests")}}
    try:
        import torch

        out["torch"] = torch.__version__
        out["cuda_available"] = torch.cuda.is_available()
        out["gpus"] = [torch.cuda.get_device_name(i) for i in range(torch.cuda.device_count())]
    except Exception as e:  # noqa: BLE001
        out["torch_error"] = str(e)
    for mod in ("_core", "_ops"):
        try:
            importlib.import_module(f"tutti_b200.{mod}")
            out[mod] = "loaded"
        except ImportError as e:
            out[mod] = f"missing ({e})"
    if out.get("_core") == "loaded":
        from ._native import core

        out["native_cuda_device"] = bool(core().cuda_device_present())
    return out


def cmd_status(args) -> int:
    s = status()
    if args.json:
        print(json.dumps(s))
    else:
        for k, v in s.items():
            print(f"{k:>20}: {v}")
    return 0


def cmd_daemon(args) -> int:
    exe = _bin("tutti_daemon")
    if not os.path.exists(exe):
        print("tutti_daemon is not built: python -m tutti_b200 build", file=sys.stderr)
        return 2
    os.execv(exe, [exe, "--config", args.config] + list(args.rest))
    return 0  # not reached


def cmd_selftest(_args) -> int:
    exe = _bin("tutti_native_tests")
    if not os.path.exists(exe):
        print("tutti_native_tests is not built: python -m tutti_b200 build", file=sys.stderr)
        return 2
    return subprocess.run([exe]).returncode


def cmd_fiemap(args) -> int:
    from ._native import core

    for logical, physical, length, flags in core().fiemap(args.file):
        print(f"logical {logical:>14} physical {physical:>16} length {length:>12} flags 0x{flags:x}")
    return 0


def cmd_probe_raid0(args) -> int:
    from ._native import core

    print(json.dumps(core().probe_md_raid0(args.sysfs, args.md)))
    return 0


def cmd_topology(args) -> int:
    from .parallel.topology import affinity, discover

    devs = discover(args.sysfs)
    gpus = [d for d in devs if d.kind == "gpu"]
    drives = [d for d in devs if d.kind == "nvme"]
    aff = affinity(drives, gpus) if drives and gpus else []
    out = {"gpus": [d.bdf for d in gpus], "drives": [d.bdf for d in drives], "affine_gpus": aff}
    print(json.dumps(out))
    return 0


def cmd_bench(args) -> int:
    mod = importlib.import_module(f"tutti_b200.benchmarks.{BENCHES[args.which]}")
    rc = mod.main(list(args.rest))
    return int(rc or 0) if not isinstance(rc, dict) else 0


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="python -m tutti_b200")
    sub = p.add_subparsers(dest="cmd", required=True)
    sub.add_parser("build").set_defaults(fn=cmd_build)
    s = sub.add_parser("status")
    s.add_argument("--json", action="store_true")
    s.set_defaults(fn=cmd_status)
    d = sub.add_parser("daemon")
    d.add_argument("--config", required=True)
    d.add_argument("rest", nargs=argparse.REMAINDER)
    d.set_defaults(fn=cmd_daemon)
    sub.add_parser("selftest").set_defaults(fn=cmd_selftest)
    f = sub.add_parser("fiemap")
    f.add_argument("file")
    f.set_defaults(fn=cmd_fiemap)
    r = sub.add_parser("probe-raid0")
    r.add_argument("md")
    r.add_argument("--sysfs", default="/sys")
    r.set_defaults(fn=cmd_probe_raid0)
    t = sub.add_parser("topology")
    t.add_argument("--sysfs", default="/sys")
    t.set_defaults(fn=cmd_topology)
    b = sub.add_parser("bench")
    b.add_argument("which", choices=sorted(BENCHES))
    b.add_argument("rest", nargs=argparse.REMAINDER)
    b.set_defaults(fn=cmd_bench)
    args = p.parse_args(argv)
    return args.fn(args)


if __name__ == "__main__":
    sys.exit(main())
