"""Command line for operators: build, status, daemon, probes, tests and benchmarks.

    python -m tutti_b200 build                 # CUDA extensions (sm_100a) + native executables
    python -m tutti_b200 status [--json]       # GPUs, extensions, native binaries, a runtime's capabilities
    python -m tutti_b200 daemon --config F     # run tutti_daemon (queue leases) in the foreground
    python -m tutti_b200 daemon-grpc --socket S [--listen 127.0.0.1:50051]   # Tutti's NvmeService over it
    python -m tutti_b200 selftest              # C++ contract suite (no GPU needed)
    python -m tutti_b200 fiemap FILE           # extents the FIEMAP resolver sees
    python -m tutti_b200 probe-raid0 md0 [--sysfs /sys]
    python -m tutti_b200 topology [--sysfs /sys]   # NVMe drive -> affine GPU over the PCIe tree
    python -m tutti_b200 nvme-bind BDF [--driver nvme|snvme]    # move one controller to a driver
    python -m tutti_b200 nvme-unbind [BDF ...] [--driver snvme] # release controllers (all by default)
    python -m tutti_b200 raid0-create DEV DEV ... [--chunk-kib 64] --yes   # destroys the drives' data
    python -m tutti_b200 raid0-delete mdN --yes                 # stops the array
    python -m tutti_b200 snvme-smoke (--node /dev/snvmN | --fake) [--write] ...   # controller bring-up check
    python -m tutti_b200 bench {kernels,ttft,fanout,mla,trace,sweep,plumbing,vllm} [args...]
    python -m tutti_b200 test [--gpu] [--dry-run] [pytest args...]   # pytest suites + C++ contract suite
    python -m tutti_b200 vllm-config --root R [--mounts M ...] [--preset JSON] ...   # --kv-transfer-config JSON
    python -m tutti_b200 vllm-serve MODEL --root R [...] [--dry-run] -- [vllm serve args...]

Parity: reference scripts/tutti-env.sh (build, build-ext, test, daemon, status
subcommands), scripts/tutti-md (md RAID0 inspection),
scripts/pci_topology_check.sh (drive / GPU switch affinity),
scripts/{bind_nvme_device,unbind,raid0_create,raid0_delete}.sh (through
``device_admin``) and scripts/vllm/run/serve-8gpu-striped.sh (vLLM serve with
the connector).
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
BENCHES = {"kernels": "kernels", "ttft": "ttft", "fanout": "fanout", "mla": "mla_indexer", "trace": "serving_trace",
           "sweep": "io_sweep", "plumbing": "cpu_plumbing", "vllm": "vllm_e2e"}


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
    out = {"package": PKG, "binaries": {n: os.path.exists(_bin(n)) for n in ("tutti_daemon", "tutti_native_tests",
                                                                          "tutti_posix_roundtrip", "tutti_snvme_smoke")}}
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


def cmd_daemon_grpc(args) -> int:
    from . import daemon_grpc

    return daemon_grpc.main(list(args.rest))


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


def _admin(fn) -> int:
    from .device_admin import AdminError

    try:
        rep = fn()
    except AdminError as e:
        print(f"error: {e}", file=sys.stderr)
        return 1
    for line in getattr(rep, "steps", []):
        print(line)
    return 0


def cmd_nvme_bind(args) -> int:
    from . import device_admin as da

    return _admin(lambda: da.bind_driver(args.bdf, args.driver, da.Host(sysfs=args.sysfs)))


def cmd_nvme_unbind(args) -> int:
    from . import device_admin as da

    return _admin(lambda: da.unbind_driver(args.driver, list(args.bdfs) or None, da.Host(sysfs=args.sysfs)))


def cmd_raid0_create(args) -> int:
    from . import device_admin as da

    return _admin(lambda: da.raid0_create(list(args.devices), args.chunk_kib, args.yes)[1])


def cmd_raid0_delete(args) -> int:
    from . import device_admin as da

    return _admin(lambda: da.raid0_delete(args.md, args.yes))


def cmd_snvme_smoke(args) -> int:
    exe = _bin("tutti_snvme_smoke")
    if not os.path.exists(exe):
        print("tutti_snvme_smoke is not built (python -m tutti_b200 build)", file=sys.stderr)
        return 1
    return subprocess.run([exe] + list(args.rest)).returncode


def cmd_bench(args) -> int:
    mod = importlib.import_module(f"tutti_b200.benchmarks.{BENCHES[args.which]}")
    rc = mod.main(list(args.rest))
    return int(rc or 0) if not isinstance(rc, dict) else 0


def cmd_test(args) -> int:
    cmds = [[sys.executable, "-m", "pytest", os.path.join(ROOT, "tests"), "-q", "-m", "gpu" if args.gpu else "not gpu",
             *args.rest]]
    if not args.gpu:
        cmds.append([_bin("tutti_native_tests")])
    for c in cmds:
        if args.dry_run:
            print(" ".join(c))
            continue
        rc = subprocess.run(c, cwd=ROOT).returncode
        if rc:
            return rc
    return 0


def kv_transfer_config(args) -> dict:
    """The ``--kv-transfer-config`` of a vLLM deployment with this connector (Tutti's module path and schema)."""
    options = {"root": args.root}
    if args.mounts:
        options["mounts"] = list(args.mounts)
    if args.capacity:
        options["capacity"] = args.capacity
    if args.preset:
        options["preset"] = json.loads(args.preset)
    if args.stored_format != "native":
        options["stored_format"] = args.stored_format
    extra = {"chunk_tokens": args.chunk_tokens, "load_mode": args.load_mode,
             "store": {"type": "tutti_nvme", "options": options}}
    from .integration.vllm.factory import ConnectorConfig

    ConnectorConfig.from_extra(extra)  # fail here, not inside vLLM's workers
    return {"kv_connector": "TuttiConnectorV1", "kv_connector_module_path": "tutti.integration.vllm.connector",
            "kv_role": "kv_both", "kv_load_failure_policy": args.failure_policy, "kv_connector_extra_config": extra}


def cmd_vllm_config(args) -> int:
    print(json.dumps(kv_transfer_config(args)))
    return 0


def cmd_vllm_serve(args) -> int:
    rest = [a for a in args.rest if a != "--"]
    cmd = ["vllm", "serve", args.model, "--kv-transfer-config", json.dumps(kv_transfer_config(args)), *rest]
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    if args.dry_run:
        print(" ".join(cmd[:4]) + " '" + cmd[4] + "' " + " ".join(cmd[5:]))
        return 0
    return subprocess.run(cmd, env=env).returncode


def _vllm_args(q) -> None:
    q.add_argument("--root", required=True, help="store root ({LOCAL_RANK} / {RANK} expand per worker)")
    q.add_argument("--mounts", nargs="*", default=[], help="one drive per mount")
    q.add_argument("--capacity", default="", help='e.g. "64 GiB"')
    q.add_argument("--preset", default="", help="drives by device id, as JSON (daemon_config, device_groups)")
    q.add_argument("--chunk-tokens", type=int, default=256)
    q.add_argument("--load-mode", choices=["sync", "async", "auto"], default="sync")
    q.add_argument("--failure-policy", choices=["recompute", "fail"], default="recompute")
    q.add_argument("--stored-format", choices=["native", "fp8_block128"], default="native")


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
    dg = sub.add_parser("daemon-grpc")
    dg.set_defaults(fn=cmd_daemon_grpc, passthrough=True)  # --socket/--listen go to the gateway
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
    nb = sub.add_parser("nvme-bind")
    nb.add_argument("bdf")
    nb.add_argument("--driver", choices=["nvme", "snvme"], default="nvme")
    nb.add_argument("--sysfs", default="/sys")
    nb.set_defaults(fn=cmd_nvme_bind)
    nu = sub.add_parser("nvme-unbind")
    nu.add_argument("bdfs", nargs="*")
    nu.add_argument("--driver", choices=["nvme", "snvme"], default="snvme")
    nu.add_argument("--sysfs", default="/sys")
    nu.set_defaults(fn=cmd_nvme_unbind)
    rc = sub.add_parser("raid0-create")
    rc.add_argument("devices", nargs="+")
    rc.add_argument("--chunk-kib", type=int, default=64)
    rc.add_argument("--yes", action="store_true", help="confirm: every byte on the drives is lost")
    rc.set_defaults(fn=cmd_raid0_create)
    rd = sub.add_parser("raid0-delete")
    rd.add_argument("md")
    rd.add_argument("--yes", action="store_true", help="confirm: the array is stopped")
    rd.set_defaults(fn=cmd_raid0_delete)
    sm = sub.add_parser("snvme-smoke")
    sm.set_defaults(fn=cmd_snvme_smoke, passthrough=True)  # arguments go to tutti_snvme_smoke
    b = sub.add_parser("bench")
    b.add_argument("which", choices=sorted(BENCHES))
    b.add_argument("rest", nargs=argparse.REMAINDER)
    b.set_defaults(fn=cmd_bench)
    te = sub.add_parser("test")
    te.add_argument("--gpu", action="store_true", help="the B200 suite instead of the host suites")
    te.add_argument("--dry-run", action="store_true")
    te.set_defaults(fn=cmd_test, passthrough=True)  # other arguments go to pytest
    vc = sub.add_parser("vllm-config")
    _vllm_args(vc)
    vc.set_defaults(fn=cmd_vllm_config)
    vs = sub.add_parser("vllm-serve")
    vs.add_argument("model")
    _vllm_args(vs)
    vs.add_argument("--dry-run", action="store_true")
    vs.set_defaults(fn=cmd_vllm_serve, passthrough=True)  # other arguments go to vllm serve
    args, extra = p.parse_known_args(argv)
    if extra and not getattr(args, "passthrough", False):
        p.error(f"unrecognized arguments: {' '.join(extra)}")
    if getattr(args, "passthrough", False):
        args.rest = extra
    return args.fn(args)


if __name__ == "__main__":
    sys.exit(main())
