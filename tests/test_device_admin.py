"""Device administration (driver binding, md RAID0 create/stop) against a fake host: a sysfs tree
in a temporary directory whose attribute writes the fake kernel acts on, fake block devices,
and recorded commands. Nothing touches the real host."""
import os

import pytest

from tutti_b200 import device_admin as da

NVME_BDF = "0000:1b:00.0"
NIC_BDF = "0000:3a:00.0"


class FakeHost(da.Host):
    def __init__(self, tmp, root=True):
        super().__init__(sysfs=str(tmp / "sys"), dev=str(tmp / "dev"), proc=str(tmp / "proc"))
        self.root = root
        self.block = set()
        self.commands = []
        # argv[0:2] -> (rc, out, err); a clean drive: no signature, no md superblock
        self.answers = {("blkid", "-p"): (2, "", ""),
                        ("mdadm", "--examine"): (1, "", "mdadm: No md superblock detected")}
        self.refuse_bind = set()
        os.makedirs(os.path.join(self.sysfs, "bus", "pci", "drivers"))
        os.makedirs(os.path.join(self.sysfs, "bus", "pci", "devices"))
        os.makedirs(self.dev)
        os.makedirs(os.path.join(self.proc, "self"))
        with open(os.path.join(self.proc, "self", "mountinfo"), "w") as f:
            f.write("22 1 259:1 / / rw,relatime shared:1 - ext4 /dev/nvme9n1p1 rw\n")

    # -- the fake tree ---------------------------------------------------------
    def add_driver(self, name):
        d = os.path.join(self.sysfs, "bus", "pci", "drivers", name)
        os.makedirs(d)
        for f in ("bind", "unbind"):
            open(os.path.join(d, f), "w").close()

    def add_device(self, bdf, cls, driver=None):
        d = os.path.join(self.sysfs, "bus", "pci", "devices", bdf)
        os.makedirs(d)
        for name, value in (("class", f"0x{cls:06x}"), ("vendor", "0x144d"), ("device", "0xa80a"),
                            ("driver_override", "(null)")):
            with open(os.path.join(d, name), "w") as f:
                f.write(value + "\n")
        if driver:
            self._link(bdf, driver)

    def _link(self, bdf, driver):
        dd = os.path.join(self.sysfs, "bus", "pci", "drivers", driver)
        dev = os.path.join(self.sysfs, "bus", "pci", "devices", bdf)
        os.symlink(dd, os.path.join(dev, "driver"))
        os.symlink(dev, os.path.join(dd, bdf))
        if driver == "nvme":
            os.makedirs(os.path.join(dev, "nvme", "nvme3"), exist_ok=True)

    def _unlink(self, bdf, driver):
        dd = os.path.join(self.sysfs, "bus", "pci", "drivers", driver)
        dev = os.path.join(self.sysfs, "bus", "pci", "devices", bdf)
        os.unlink(os.path.join(dev, "driver"))
        os.unlink(os.path.join(dd, bdf))

    # -- the fake kernel and tools ---------------------------------------------
    def write(self, path, value):
        super().write(path, value)
        parent, attr = os.path.split(path)
        drivers = os.path.join(self.sysfs, "bus", "pci", "drivers")
        if os.path.dirname(parent) == drivers:
            driver = os.path.basename(parent)
            if attr == "unbind":
                if not os.path.islink(os.path.join(parent, value)):
                    raise OSError(19, "No such device")
                self._unlink(value, driver)
            elif attr == "bind":
                dev = os.path.join(self.sysfs, "bus", "pci", "devices", value)
                override = self.read(os.path.join(dev, "driver_override"))
                if value in self.refuse_bind or override not in (driver, "(null)", ""):
                    raise OSError(19, "No such device")
                if os.path.islink(os.path.join(dev, "driver")):
                    raise OSError(16, "Device or resource busy")
                self._link(value, driver)

    def is_block_device(self, path):
        return path in self.block

    def run(self, argv):
        self.commands.append(list(argv))
        return self.answers.get(tuple(argv[:2]), (0, "", ""))

    def is_root(self):
        return self.root


@pytest.fixture
def host(tmp_path):
    h = FakeHost(tmp_path)
    h.add_driver("nvme")
    h.add_driver("snvme")
    h.add_device(NVME_BDF, da.NVME_CLASS, driver="nvme")
    h.add_device(NIC_BDF, 0x020000)
    return h


def test_bind_moves_a_controller_to_snvme_and_back(host):
    rep = da.bind_driver(NVME_BDF, "snvme", host)
    assert da.pci_device(host, NVME_BDF).driver == "snvme"
    assert any("unbound from nvme" in s for s in rep.steps) and any("bound to snvme" in s for s in rep.steps)
    assert da.bound_devices("snvme", host) == [NVME_BDF]
    # pinned to this device only (driver_override), not a vendor:device id for every drive
    assert host.read(os.path.join(host.sysfs, "bus/pci/devices", NVME_BDF, "driver_override")) == "snvme"
    rep = da.bind_driver(NVME_BDF, "nvme", host)
    assert da.pci_device(host, NVME_BDF).driver == "nvme"
    assert "block controller nvme3" in rep.steps[-1]


def test_bind_checks_before_it_touches_anything(host, tmp_path):
    with pytest.raises(da.AdminError, match="not an NVMe controller"):
        da.bind_driver(NIC_BDF, "nvme", host)
    with pytest.raises(da.AdminError, match="not a PCI address"):
        da.bind_driver("1b:00.0", "nvme", host)
    with pytest.raises(da.AdminError, match="not found"):
        da.bind_driver("0000:99:00.0", "nvme", host)
    with pytest.raises(da.AdminError, match="driver must be"):
        da.bind_driver(NVME_BDF, "vfio-pci", host)
    assert da.bind_driver(NVME_BDF, "nvme", host).steps[1].endswith("already bound to nvme")
    nonroot = FakeHost(tmp_path / "other", root=False)
    with pytest.raises(da.AdminError, match="root"):
        da.bind_driver(NVME_BDF, "nvme", nonroot)


def test_bind_reports_a_driver_that_is_not_loaded_and_a_refused_bind(tmp_path):
    h = FakeHost(tmp_path)
    h.add_driver("nvme")
    h.add_device(NVME_BDF, da.NVME_CLASS, driver="nvme")
    with pytest.raises(da.AdminError, match="modprobe snvme"):
        da.bind_driver(NVME_BDF, "snvme", h)
    assert da.pci_device(h, NVME_BDF).driver == "nvme"  # nothing was unbound
    h.add_driver("snvme")
    h.refuse_bind.add(NVME_BDF)
    with pytest.raises(da.AdminError, match="refused to bind"):
        da.bind_driver(NVME_BDF, "snvme", h)


def test_unbind_releases_every_snvme_device_or_the_named_ones(host):
    other = "0000:1c:00.0"
    host.add_device(other, da.NVME_CLASS, driver="snvme")
    da.bind_driver(NVME_BDF, "snvme", host)
    assert da.bound_devices("snvme", host) == [NVME_BDF, other]
    rep = da.unbind_driver("snvme", [other], host)
    assert da.bound_devices("snvme", host) == [NVME_BDF] and rep.steps == [f"{other}: unbound from snvme"]
    with pytest.raises(da.AdminError, match="not bound"):
        da.unbind_driver("snvme", [other], host)
    da.unbind_driver("snvme", None, host)
    assert da.bound_devices("snvme", host) == []
    # the override is cleared: the kernel's own driver may probe the device again
    assert host.read(os.path.join(host.sysfs, "bus/pci/devices", NVME_BDF, "driver_override")) == ""
    assert da.unbind_driver("snvme", None, host).steps == ["no device is bound to snvme"]


def test_raid0_create_checks_drives_and_needs_confirmation(host):
    drives = [os.path.join(host.dev, f"nvme{i}n1") for i in range(3)]
    host.block.update(drives)
    open(os.path.join(host.dev, "md0"), "w").close()  # md0 is taken
    with pytest.raises(da.AdminError, match="confirm"):
        da.raid0_create(drives, host=host)
    assert not any(c[:2] == ["mdadm", "--create"] for c in host.commands)
    md, rep = da.raid0_create(drives, chunk_kib=64, confirm=True, host=host)
    assert md == os.path.join(host.dev, "md1")
    create = [c for c in host.commands if c[:2] == ["mdadm", "--create"]][-1]
    assert create == ["mdadm", "--create", md, "--level=0", "--raid-devices=3", *drives, "--chunk=64K", "--run",
                      "--verbose"]
    assert rep.steps[-1].endswith("created")


def test_raid0_create_refuses_unsafe_drives(host):
    a, b = os.path.join(host.dev, "nvme0n1"), os.path.join(host.dev, "nvme1n1")
    host.block.update([a, b])
    with pytest.raises(da.AdminError, match="at least two"):
        da.raid0_create([a], confirm=True, host=host)
    with pytest.raises(da.AdminError, match="named twice"):
        da.raid0_create([a, a], confirm=True, host=host)
    with pytest.raises(da.AdminError, match="not a block device"):
        da.raid0_create([a, os.path.join(host.dev, "sdz")], confirm=True, host=host)
    with pytest.raises(da.AdminError, match="power of two"):
        da.raid0_create([a, b], chunk_kib=48, confirm=True, host=host)
    mounted = "/dev/nvme9n1p1"
    host.block.add(mounted)
    with pytest.raises(da.AdminError, match="mounted"):
        da.raid0_create([a, mounted], confirm=True, host=host)
    host.answers[("blkid", "-p")] = (0, "ext4\n", "")
    with pytest.raises(da.AdminError, match="ext4 file system"):
        da.raid0_create([a, b], confirm=True, host=host)
    host.answers[("blkid", "-p")] = (2, "", "")
    host.answers[("mdadm", "--examine")] = (0, "Magic : a92b4efc\n", "")
    with pytest.raises(da.AdminError, match="md superblock"):
        da.raid0_create([a, b], confirm=True, host=host)
    host.answers[("mdadm", "--examine")] = (1, "", "No md superblock detected")
    host.answers[("mdadm", "--version")] = (127, "", "not found")
    with pytest.raises(da.AdminError, match="mdadm is not installed"):
        da.raid0_create([a, b], confirm=True, host=host)
    host.answers[("mdadm", "--version")] = (0, "mdadm - v4.2", "")
    host.answers[("mdadm", "--create")] = (1, "", "mdadm: cannot open /dev/nvme0n1: Device or resource busy")
    with pytest.raises(da.AdminError, match="resource busy"):
        da.raid0_create([a, b], confirm=True, host=host)


def test_raid0_delete_stops_an_unmounted_array_once_confirmed(host):
    md = os.path.join(host.dev, "md127")
    host.block.add(md)
    with pytest.raises(da.AdminError, match="confirmation"):
        da.raid0_delete("md127", host=host)
    assert da.raid0_delete("/dev/md127", confirm=True, host=host).steps == [f"{md}: stopped"]
    assert host.commands[-1] == ["mdadm", "--stop", md]
    with pytest.raises(da.AdminError, match="not an md device"):
        da.raid0_delete("nvme0n1", confirm=True, host=host)
    with pytest.raises(da.AdminError, match="not a block device"):
        da.raid0_delete("md5", confirm=True, host=host)
    with open(os.path.join(host.proc, "self", "mountinfo"), "a") as f:
        f.write(f"40 22 9:127 / /mnt/kv rw - xfs {md} rw\n")
    with pytest.raises(da.AdminError, match="mounted"):
        da.raid0_delete("md127", confirm=True, host=host)
