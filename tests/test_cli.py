"""Operator command line (host only)."""
import json
import subprocess
import sys


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
