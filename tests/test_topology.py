"""PCIe drive -> GPU affinity from a fake sysfs tree (host only)."""
import os

from tutti_b200.parallel.topology import affine_gpus, affinity, discover


def _dev(root, chain, cls, vendor):
    """Create /sys/devices/<chain...> and the /sys/bus/pci/devices/<bdf> link to it."""
    real = os.path.join(root, "devices", "pci0000:00", *chain)
    os.makedirs(real, exist_ok=True)
    with open(os.path.join(real, "class"), "w") as f:
        f.write(cls + "\n")
    with open(os.path.join(real, "vendor"), "w") as f:
        f.write(vendor + "\n")
    link_dir = os.path.join(root, "bus", "pci", "devices")
    os.makedirs(link_dir, exist_ok=True)
    os.symlink(real, os.path.join(link_dir, chain[-1]))


def test_drives_map_to_gpu_behind_the_same_switch(tmp_path):
    root = str(tmp_path)
    # two PCIe switches under two root ports; a GPU and two drives behind switch A, a GPU and one drive behind B
    sw_a = ["0000:00:01.0", "0000:01:00.0"]
    sw_b = ["0000:00:02.0", "0000:11:00.0"]
    _dev(root, sw_a + ["0000:02:00.0", "0000:03:00.0"], "0x030200", "0x10de")   # GPU 0
    _dev(root, sw_a + ["0000:02:01.0", "0000:04:00.0"], "0x010802", "0x144d")   # nvme, switch A
    _dev(root, sw_b + ["0000:12:00.0", "0000:13:00.0"], "0x030200", "0x10de")   # GPU 1
    _dev(root, sw_b + ["0000:12:01.0", "0000:14:00.0"], "0x010802", "0x144d")   # nvme, switch B
    _dev(root, sw_a + ["0000:02:02.0", "0000:05:00.0"], "0x010802", "0x8086")   # nvme, switch A
    _dev(root, ["0000:00:1f.0"], "0x060100", "0x8086")                          # an ISA bridge: ignored
    devs = discover(root)
    assert [d.kind for d in devs].count("gpu") == 2 and [d.kind for d in devs].count("nvme") == 3
    # drives in PCI address order: 04:00.0 (A), 05:00.0 (A), 14:00.0 (B)
    assert affine_gpus(root) == [0, 0, 1]
    gpus = [d for d in devs if d.kind == "gpu"]
    drives = [d for d in devs if d.kind == "nvme"]
    assert affinity(drives, gpus[::-1]) == [1, 1, 0]


def test_no_devices_means_no_affinity(tmp_path):
    assert affine_gpus(str(tmp_path)) == []
