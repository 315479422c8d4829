"""Drive presets: device ids resolved through daemon configs, device groups per TP rank."""
import pytest

from tutti_b200.integration.vllm.factory import ConnectorConfig, store_mounts
from tutti_b200.storage.preset import load_daemon_devices, prepare_preset, preset_mounts

OURS = """
service: {socket: /tmp/x.sock}
devices:
  - {id: 0, kind: emulated, mount: /mnt/nvme0, pci: "0000:1b:00.0", nsid: 1}
  - {id: 1, kind: emulated, mount: /mnt/nvme1, pci: "0000:1c:00.0"}
"""
TUTTI = """
nvmes:
  - {device_id: 2, pci_addr: "0000:3b:00.0", backing_mount_path: /mnt/nvme2, namespace_id: 1}
  - {device_id: 3, pci_addr: "0000:3c:00.0", backing_mount_path: /mnt/nvme3}
"""


@pytest.fixture
def daemons(tmp_path):
    a, b = tmp_path / "ours.yaml", tmp_path / "tutti.yaml"
    a.write_text(OURS)
    b.write_text(TUTTI)
    return f"{a},{b}"


def test_both_daemon_schemas_merge(daemons, tmp_path):
    facts = load_daemon_devices(daemons)
    assert facts[1] == {"mount_path": "/mnt/nvme1", "pci_bdf": "0000:1c:00.0", "namespace_id": 1}
    assert facts[3]["mount_path"] == "/mnt/nvme3" and sorted(facts) == [0, 1, 2, 3]
    dup = tmp_path / "dup.yaml"
    dup.write_text(OURS)
    with pytest.raises(ValueError, match="more than one"):
        load_daemon_devices([str(dup), daemons.split(",")[0]])


def test_device_groups_pick_each_ranks_drives(daemons):
    preset = {"type": "nvme-device-group", "daemon_config": daemons, "device_groups": [["0", "1"], [2, 3]]}
    assert preset_mounts(prepare_preset(preset, rank=0, tp_size=4)) == ["/mnt/nvme0", "/mnt/nvme1"]
    p3 = prepare_preset(preset, rank=3, tp_size=4)
    assert preset_mounts(p3) == ["/mnt/nvme2", "/mnt/nvme3"] and p3["devices"][0]["pci_bdf"] == "0000:3b:00.0"
    with pytest.raises(ValueError, match="multiple"):
        prepare_preset(preset, rank=0, tp_size=3)
    local = prepare_preset({"type": "local", "daemon_config": daemons, "device_id": 2})
    assert preset_mounts(local) == ["/mnt/nvme2"]
    explicit = prepare_preset({"type": "nvme-device-group", "devices": [{"mount_path": "/x", "device_id": 1}],
                               "daemon_config": daemons})
    assert preset_mounts(explicit) == ["/x"]  # explicit fields win over the daemon's


def test_invalid_presets(daemons):
    with pytest.raises(ValueError, match="unknown preset type"):
        prepare_preset({"type": "jbod"})
    with pytest.raises(ValueError, match="raid0"):  # members on different mounts
        prepare_preset({"type": "raid0", "daemon_config": daemons, "devices": [{"device_id": 0}, {"device_id": 1}]})
    ok = prepare_preset({"type": "raid0", "devices": [{"mount_path": "/md0"}, {"mount_path": "/md0"}]})
    assert preset_mounts(ok) == ["/md0"]
    with pytest.raises(ValueError, match="no daemon config entry"):
        prepare_preset({"type": "local", "daemon_config": daemons, "device_id": 9})


def test_connector_config_takes_its_mounts_from_the_preset(daemons):
    cfg = ConnectorConfig.from_extra({"store": {"type": "tutti_nvme", "options": {
        "root": "/kv/{LOCAL_RANK}", "preset": {"type": "nvme-device-group", "daemon_config": daemons,
                                               "device_groups": [[0, 1], [2, 3]]}}}})
    assert store_mounts(cfg, rank=1, local_rank=1, world=2) == ["/mnt/nvme2", "/mnt/nvme3"]
    explicit = ConnectorConfig.from_extra({"store": {"type": "tutti_nvme", "options": {
        "root": "/kv", "mounts": ["/a{LOCAL_RANK}"], "preset": {"type": "local", "device_id": 0}}}})
    assert store_mounts(explicit, rank=0, local_rank=5, world=1) == ["/a5"]  # explicit mounts win


def test_preset_from_environment_is_parsed_and_checked(monkeypatch, daemons):
    from tutti_b200.storage.preset import runtime_from_env

    monkeypatch.delenv("TUTTI_NVME_PRESET", raising=False)
    with pytest.raises(ValueError, match="not set"):
        runtime_from_env()
    monkeypatch.setenv("TUTTI_NVME_PRESET", "[1, 2]")
    with pytest.raises(ValueError, match="mapping"):
        runtime_from_env()
    monkeypatch.setenv("TUTTI_NVME_PRESET", '{"type": "local", "device_id": 7, "daemon_config": "%s"}' % daemons)
    with pytest.raises(ValueError, match="device id 7"):
        runtime_from_env()


def test_raid0_preset_over_a_tutti_style_daemon_file(tmp_path):
    d = tmp_path / "daemon_kv.yaml"
    lines = ["nvmes:"]
    for i in range(4):
        lines += [f"- device_id: {i}", f'  pci_addr: "0000:0{i}:00.0"', "  backing_mount_path: /mnt/md_kv",
                  "  namespace_id: 1", "  kernel_ioq_cap: 16", "  allowed_accel_ids: [0, 1, 2, 3]",
                  "  auto_mount: false"]
    lines += ["raid0_arrays:", "- name: kv", "  device_ids: [0, 1, 2, 3]", "  mount_path: /mnt/md_kv"]
    d.write_text("\n".join(lines) + "\n")
    p = prepare_preset({"type": "raid0", "daemon_config": [str(d)], "gpu_id": "{LOCAL_RANK}",
                        "device_groups": [[0, 1, 2, 3]]}, rank=5, tp_size=8)
    assert preset_mounts(p) == ["/mnt/md_kv"] and [x["pci_bdf"] for x in p["devices"]][-1] == "0000:03:00.0"
