"""md RAID0 probe (fake sysfs root) and offset mapping against a byte oracle."""
import numpy as np
import pytest

from tutti_b200._native import core


def _fake_md(root, name="md0", level="raid0", chunk=512 * 1024, members=((1, 2048), (0, 4096))):
    md = root / "block" / name / "md"
    md.mkdir(parents=True)
    (md / "level").write_text(level + "\n")
    (md / "chunk_size").write_text(f"{chunk}\n")
    (md / "raid_disks").write_text(f"{len(members)}\n")
    for i, (slot, off) in enumerate(members):
        rd = md / f"rd{i}"
        rd.mkdir()
        (rd / "slot").write_text(f"{slot}\n")
        (rd / "offset").write_text(f"{off}\n")  # sectors
    return md


def test_probe_orders_members_by_slot(tmp_path):
    _fake_md(tmp_path)
    g = core().probe_md_raid0(str(tmp_path), "md0")
    assert g["chunk_bytes"] == 512 * 1024
    # slot 0 is rd1 (offset 4096 sectors), slot 1 is rd0 (2048 sectors)
    assert g["members"] == [(0, 4096 * 512, "rd1"), (1, 2048 * 512, "rd0")]


def test_probe_rejects_other_levels_and_holes(tmp_path):
    _fake_md(tmp_path, name="md1", level="raid1")
    with pytest.raises(Exception, match="raid1"):
        core().probe_md_raid0(str(tmp_path), "md1")
    md = _fake_md(tmp_path, name="md2")
    (md / "rd1" / "offset").unlink()
    with pytest.raises(Exception, match="missing md member"):
        core().probe_md_raid0(str(tmp_path), "md2")
    _fake_md(tmp_path, name="md3", members=((0, 0), (0, 8)))
    with pytest.raises(Exception, match="bad md slot"):
        core().probe_md_raid0(str(tmp_path), "md3")


def test_raid0_map_matches_striping_oracle():
    chunk, offs = 64 * 1024, [1 << 20, 3 << 20, 0]
    n = len(offs)
    rng = np.random.default_rng(0)
    # byte oracle: an md image striped over member images, chunk by chunk
    md_bytes = 48 * chunk
    image = rng.integers(0, 256, md_bytes, dtype=np.uint8)
    members = [np.zeros(offs[m] + (md_bytes // n) + chunk, dtype=np.uint8) for m in range(n)]
    for c in range(md_bytes // chunk):
        m, row = c % n, c // n
        members[m][offs[m] + row * chunk: offs[m] + (row + 1) * chunk] = image[c * chunk: (c + 1) * chunk]
    for off in list(rng.integers(0, md_bytes - 1, 200)) + [0, chunk - 1, chunk, md_bytes - 1]:
        m, moff, contig = core().raid0_map(chunk, offs, int(off))
        assert contig == chunk - (off % chunk)
        assert members[m][moff] == image[off]
        k = min(contig, md_bytes - off)
        assert np.array_equal(members[m][moff: moff + k], image[off: off + k])


def test_md_array_found_from_a_mount(tmp_path):
    import os

    mnt = tmp_path / "mnt"
    mnt.mkdir()
    st = os.stat(mnt)
    sysfs = tmp_path / "sys"
    _fake_md(sysfs, name="md7")
    (sysfs / "devices" / "virtual" / "block" / "md7").mkdir(parents=True)
    (sysfs / "dev" / "block").mkdir(parents=True)
    os.symlink("../../devices/virtual/block/md7", sysfs / "dev" / "block" / f"{os.major(st.st_dev)}:{os.minor(st.st_dev)}")
    assert core().find_md_array(str(sysfs), str(mnt)) == "md7"
    other = tmp_path / "sys2"
    (other / "dev" / "block").mkdir(parents=True)
    os.symlink("../../devices/pci/nvme0n1", other / "dev" / "block" / f"{os.major(st.st_dev)}:{os.minor(st.st_dev)}")
    with pytest.raises(Exception, match="not on an md array"):
        core().find_md_array(str(other), str(mnt))


def test_tutti_style_runtime_config_validates():
    # Tutti's runtime YAML conventions: an explicit device selection, and a raid0
    # resolver that finds its md array from the mount instead of naming it
    text = """
accelerator: {profile: CUDA}
runtime: {accel_id: 0}
storage:
  resources:
    - id: nvme-local-0
      type: nvme
      provider: {type: nvme-service, endpoint: "127.0.0.1:50051"}
      allocation: {selection: explicit, device_ids: [0, 1], queues_per_controller: 4}
  resolvers:
    - {id: raid0-resolver, type: local-file, scheme: file, config: {topology: raid0}}
  datapaths:
    - {id: dp, type: nvme-device-group, config: {}}
  backends:
    - {id: storage, contract: nvme-device-group, resolver: raid0-resolver, datapath: dp, resource: nvme-local-0, config: {}}
"""
    spec = core().parse_runtime_config(text, True)
    assert spec["resources"][0]["provider"] == "nvme-service" and spec["backends"]
