"""Operator command line (host only)."""
import json
import subprocess
import sys

import pytest


def test_status_json_reports_native_pieces(capsys):
    from tutti_b200.cli import main

    assert main(["status", "--json"]) == 0
    s = json.loads(capsys.readouterr().out)
    assert s["_core"] == "loaded" and s["_ops"] == "loaded"
    assert s["binaries"]["tutti_native_tests"]


def test_selftest_runs_native_contract_suite():
    r = subprocess.run([sys.executable, "-m", "tutti_b200", "selftest"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]


def test_fiemap_and_raid0_probe(tmp_path, capsys):
    from tutti_b200.cli import main

    f = tmp_path / "x.bin"
    f.write_bytes(b"\1" * 65536)
    assert main(["fiemap", str(f)]) == 0
    md = tmp_path / "block" / "md9" / "md"
    (md / "rd0").mkdir(parents=True)
    (md / "level").write_text("raid0\n")
    (md / "chunk_size").write_text("65536\n")
    (md / "raid_disks").write_text("1\n")
    (md / "rd0" / "slot").write_text("0\n")
    (md / "rd0" / "offset").write_text("8\n")
    capsys.readouterr()
    assert main(["probe-raid0", "md9", "--sysfs", str(tmp_path)]) == 0
    assert json.loads(capsys.readouterr().out)["chunk_bytes"] == 65536


def test_topology_command_on_empty_sysfs(tmp_path, capsys):
    from tutti_b200.cli import main

    assert main(["topology", "--sysfs", str(tmp_path)]) == 0
    assert json.loads(capsys.readouterr().out) == {"gpus": [], "drives": [], "affine_gpus": []}


def test_vllm_config_and_serve_command(capsys):
    import json

    from tutti_b200.cli import main
    from tutti_b200.integration.vllm.factory import ConnectorConfig

    assert main(["vllm-config", "--root", "/kv/{LOCAL_RANK}", "--capacity", "64 GiB", "--load-mode", "auto",
                 "--preset", '{"type": "nvme-device-group", "device_groups": [[0], [1]]}']) == 0
    ktc = json.loads(capsys.readouterr().out)
    assert ktc["kv_connector_module_path"] == "tutti.integration.vllm.connector"
    c = ConnectorConfig.from_extra(ktc["kv_connector_extra_config"])
    assert c.capacity_bytes == 64 << 30 and c.load_mode == "auto" and c.preset["device_groups"] == [[0], [1]]
    assert main(["vllm-serve", "/models/llama", "--root", "/kv", "--dry-run", "--", "--tensor-parallel-size", "8"]) == 0
    out = capsys.readouterr().out
    assert out.startswith("vllm serve /models/llama --kv-transfer-config '{") and "--tensor-parallel-size 8" in out
    with pytest.raises(ValueError):  # a bad config fails before vLLM starts
        main(["vllm-config", "--root", "/kv", "--preset", '["not", "a", "mapping"]'])


def test_test_command_runs_the_suites(capsys):
    from tutti_b200.cli import main

    assert main(["test", "--dry-run", "-k", "cli"]) == 0
    out = capsys.readouterr().out.splitlines()
    assert "-m not gpu" in out[0] and out[0].endswith("-k cli") and out[1].endswith("tutti_native_tests")


def test_cpp_api_example_round_trip(tmp_path):
    import os

    exe = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "tutti_b200", "bin",
                       "tutti_posix_roundtrip")
    if not os.path.exists(exe):
        pytest.skip("native examples not built")
    out = subprocess.run([exe, str(tmp_path)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == "OK 1048576"


def test_device_admin_commands_on_a_plain_sysfs_tree(tmp_path, capsys):
    from tutti_b200.cli import main

    # a plain tree (no kernel behind it): writes land in files, so a bind cannot be verified
    drv = tmp_path / "bus" / "pci" / "drivers"
    dev = tmp_path / "bus" / "pci" / "devices" / "0000:1b:00.0"
    for d in (drv / "nvme", drv / "snvme", dev):
        d.mkdir(parents=True)
    for f in ("bind", "unbind"):
        (drv / "snvme" / f).write_text("")
        (drv / "nvme" / f).write_text("")
    for name, value in (("class", "0x010802"), ("vendor", "0x144d"), ("device", "0xa80a"), ("driver_override", "")):
        (dev / name).write_text(value + "\n")
    (drv / "snvme" / "0000:1b:00.0").symlink_to(dev)
    (dev / "driver").symlink_to(drv / "snvme")
    assert main(["nvme-unbind", "--sysfs", str(tmp_path)]) == 0
    assert "0000:1b:00.0: unbound from snvme" in capsys.readouterr().out
    assert (drv / "snvme" / "unbind").read_text() == "0000:1b:00.0"
    assert main(["nvme-bind", "0000:1b:00.0", "--driver", "nvme", "--sysfs", str(tmp_path)]) == 1
    assert "instead of nvme" in capsys.readouterr().err
    assert main(["raid0-create", "/dev/nonexistent0", "/dev/nonexistent1"]) == 1
    err = capsys.readouterr().err  # mdadm is checked first; either way nothing is created
    assert "mdadm is not installed" in err or "not a block device" in err


def test_snvme_smoke_rounds_against_the_fake_driver():
    import os

    exe = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "tutti_b200", "bin",
                       "tutti_snvme_smoke")
    if not os.path.exists(exe):
        pytest.skip("native executables not built")
    for args in (["--fake"], ["--fake", "--write", "--queues", "3", "--rounds", "6", "--bytes", "1048576"],
                 ["--fake", "--write", "--bytes", "8192"]):
        r = subprocess.run([exe] + args, capture_output=True, text=True, timeout=120)
        assert r.returncode == 0, r.stdout + r.stderr
        res = json.loads(r.stdout.strip().splitlines()[-1])
        assert res["ok"] and res["fake"] and len(res["read_us"]) >= 4
    r = subprocess.run([exe, "--node", "/dev/no_such_snvme_node"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "cannot open snvme node" in r.stdout
    r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert r.returncode == 2 and "exactly one of" in r.stderr
