"""Native runtime configuration (YAML spec, validation, assembly) and tutti_daemon leases."""
import os
import signal
import socket
import subprocess
import sys
import textwrap
import time

import numpy as np
import pytest
import torch

from tutti_b200._native import core

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DAEMON = os.path.join(ROOT, "tutti_b200", "bin", "tutti_daemon")

DEVICE_GROUP = """
# nvme-device-group over two emulated drives
accelerator:
  profile: CUDA
runtime:
  accel_id: 0
storage:
  resources:
    - id: nvme-group
      type: nvme
      provider: {type: emulated}
      allocation:
        selection: device-group
        device_ids: [0, 1]
        queues_per_controller: 16
      config:
        mounts: ["{m0}", "{m1}"]
        controller_threads: 2
  resolvers:
    - id: file-resolver
      type: local-file
      scheme: file
      config: {topology: multi-mount}
  datapaths:
    - id: dg
      type: nvme-device-group
      config: {leases: 16, slots_per_lease: 4}
  backends:
    - id: storage
      contract: nvme-device-group
      resolver: file-resolver
      datapath: dg
      resource: nvme-group
      config: {}
"""

POSIX = """
storage:
  resolvers:
    - {id: r, type: local-file, config: {topology: multi-mount}}
  resources:
    - id: mem
      type: memory
      config: {mounts: ["{m0}"]}
  datapaths:
    - {id: p, type: posix, config: {threads: 2, direct_io: false}}
  backends:
    - {id: b, contract: posix, resolver: r, datapath: p, resource: mem}
"""


def test_parse_device_group_spec(tmp_path):
    d = core().parse_runtime_config(DEVICE_GROUP.replace("{m0}", "/a").replace("{m1}", "/b"))
    assert d["resources"][0]["device_ids"] == [0, 1]
    assert d["resources"][0]["mounts"] == ["/a", "/b"]
    assert d["resolvers"][0]["topology"] == "multi-mount"
    assert d["backends"][0]["contract"] == "nvme-device-group"
    assert d["datapaths"][0]["leases"] == 16


@pytest.mark.parametrize("mutation,needle", [
    (lambda s: s.replace("topology: multi-mount", "topology: multi-mount, bogus: 1"),
     "storage.resolvers[0].config.bogus: unknown field"),
    (lambda s: s.replace("contract: nvme-device-group", "contract: nfs"), "unknown contract"),
    (lambda s: s.replace("datapath: dg", "datapath: nope"), "unknown datapath"),
    (lambda s: s.replace("id: dg", "id: file-resolver"), "duplicate id"),
    (lambda s: s.replace("type: nvme-device-group\n", "type: posix\n"), "needs an nvme datapath"),
    (lambda s: s.replace("slots_per_lease: 4", "slots_per_lease: 99"), "slots_per_lease"),
    (lambda s: s.replace("profile: CUDA", "profile: MUSA"), "CUDA"),
])
def test_spec_validation_fails_closed_with_paths(mutation, needle):
    text = mutation(DEVICE_GROUP.replace("{m0}", "/a").replace("{m1}", "/b"))
    with pytest.raises(ValueError) as e:
        core().parse_runtime_config(text)
    assert needle in str(e.value)


def test_yaml_errors_name_lines():
    with pytest.raises(ValueError) as e:
        core().parse_runtime_config("storage:\n  resolvers:\n    - id: x\n      type: [unclosed\n")
    assert "line 4" in str(e.value)
    with pytest.raises(ValueError):
        core().parse_runtime_config("storage:\n  a: 1\n  a: 2\n")


def test_posix_runtime_assembled_from_config_roundtrip(tmp_path):
    m0 = tmp_path / "m0"
    m0.mkdir()
    f = m0 / "obj.bin"
    f.write_bytes(bytes(range(256)) * 64)
    rt = core().make_runtime_from_config(POSIX.replace("{m0}", str(m0)))
    try:
        buf = torch.zeros(16384, dtype=torch.uint8)
        mh = rt.register_memory(buf.data_ptr(), buf.numel(), "host", -1)
        th = rt.open(str(f))
        assert rt.query_target(th)["size"] == 16384
        r = rt.submit_arrays("read", np.array([mh], np.uint64), np.array([0], np.uint64), np.array([th], np.uint64),
                             np.array([0], np.uint64), np.array([16384], np.uint64), 0, True)
        res = rt.wait(r["io"], 10000)
        rt.release_io(r["io"])
        assert res["ok"] and res["confirmed_bytes"] == 16384
        assert bytes(buf.numpy()) == f.read_bytes()
    finally:
        rt.shutdown(5000)


def test_daemon_protocol_in_process():
    out = core().daemon_handle_request_selftest(
        ["HELLO client=t pid=0", "ACQUIRE session=1 devices=0,1 queues=8", "LIST",
         "ACQUIRE session=1 devices=1 queues=60", "RELEASE lease=2", "ACQUIRE session=1 devices=1 queues=60",
         "NOPE"],
        [{"id": 0, "mount": "/m0", "queues": 64}, {"id": 1, "mount": "/m1", "queues": 64}])
    assert out[0].startswith("OK") and "session=1" in out[0]
    assert "lease=2" in out[1] and "mounts=/m0,/m1" in out[1] and "first_queue=0,0" in out[1]
    assert "free_queues=56,56" in out[2]
    assert out[3].startswith("ERR") and "RESOURCE_EXHAUSTED" in out[3]  # all-or-nothing budget
    assert out[4].startswith("OK")
    assert out[5].startswith("OK")
    assert out[6].startswith("ERR")


class Client:
    def __init__(self, path):
        self.s = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        self.s.connect(path)
        self.f = self.s.makefile("rwb")

    def __call__(self, line):
        self.f.write((line + "\n").encode())
        self.f.flush()
        return self.f.readline().decode().strip()

    def kv(self, line):
        rsp = self(line)
        assert rsp.startswith("OK"), rsp
        return dict(t.split("=", 1) for t in rsp.split()[1:])


@pytest.fixture
def daemon(tmp_path):
    if not os.path.exists(DAEMON):
        pytest.skip("tutti_daemon not built")
    sock = str(tmp_path / "d.sock")
    cfg = tmp_path / "daemon.yaml"
    cfg.write_text(textwrap.dedent(f"""
        service: {{socket: {sock}}}
        lease: {{heartbeat_timeout_s: 1, reap_interval_ms: 100}}
        devices:
          - {{id: 0, kind: emulated, mount: {tmp_path}/nvme0, queues: 32}}
          - {{id: 1, kind: emulated, mount: {tmp_path}/nvme1, queues: 32}}
        """))
    p = subprocess.Popen([DAEMON, "--config", str(cfg)], stderr=subprocess.PIPE)
    for _ in range(100):
        if os.path.exists(sock):
            break
        time.sleep(0.05)
    yield sock
    p.send_signal(signal.SIGTERM)
    p.wait(timeout=10)


def test_daemon_lease_heartbeat_expiry(daemon):
    c = Client(daemon)
    sess = c.kv(f"HELLO client=test pid={os.getpid()}")["session"]
    lease = c.kv(f"ACQUIRE session={sess} devices=0,1 queues=16")["lease"]
    assert c.kv("LIST")["free_queues"] == "16,16"
    for _ in range(3):
        time.sleep(0.5)
        c.kv(f"HEARTBEAT lease={lease}")
    assert c.kv("STATUS")["leases"] == "1"
    time.sleep(2.0)  # no heartbeat for > 1 s: reaped
    assert c.kv("STATUS")["leases"] == "0"
    assert c.kv("LIST")["free_queues"] == "32,32"


def test_daemon_reaps_a_crashed_client(daemon):
    code = textwrap.dedent(f"""
        import socket, os, time
        s = socket.socket(socket.AF_UNIX); s.connect({daemon!r}); f = s.makefile('rwb')
        def rq(l):
            f.write((l + '\\n').encode()); f.flush(); return f.readline().decode()
        sess = rq('HELLO client=victim pid=%d' % os.getpid()).split('session=')[1].split()[0]
        print(rq('ACQUIRE session=%s devices=0 queues=32' % sess), flush=True)
        while True:
            rq('HEARTBEAT lease=2'); time.sleep(0.2)
        """)
    child = subprocess.Popen([sys.executable, "-c", code], stdout=subprocess.PIPE)
    assert child.stdout.readline().decode().startswith("OK")
    c = Client(daemon)
    assert c.kv("LIST")["free_queues"].startswith("0,")
    child.kill()  # the client dies holding a lease (a host process, no GPU involved)
    child.wait()
    deadline = time.time() + 5
    while time.time() < deadline and c.kv("STATUS")["leases"] != "0":
        time.sleep(0.1)
    assert c.kv("STATUS")["leases"] == "0"
    assert c.kv("LIST")["free_queues"] == "32,32"


def test_daemon_device_acl_by_accelerator():
    out = core().daemon_handle_request_selftest(
        ["HELLO client=a pid=0 accel=0", "HELLO client=b pid=0 accel=1", "HELLO client=c pid=0",
         "ACQUIRE session=1 devices=1 queues=4", "ACQUIRE session=2 devices=1 queues=4",
         "ACQUIRE session=3 devices=0 queues=4", "ACQUIRE session=3 devices=0,1 queues=4", "LIST"],
        [{"id": 0, "mount": "/m0", "queues": 64}, {"id": 1, "mount": "/m1", "queues": 64, "accelerators": [1, 2]}])
    assert out[3].startswith("ERR") and "PERMISSION_DENIED" in out[3] and "accelerator 0" in out[3]
    assert out[4].startswith("OK")  # accelerator 1 is on device 1's list
    assert out[5].startswith("OK")  # device 0 has no list: any accelerator
    assert out[6].startswith("ERR") and "PERMISSION_DENIED" in out[6]  # all-or-nothing
    assert "accelerators=*,1+2" in out[7] and "free_queues=60,60" in out[7]


def test_daemon_reads_accelerator_lists(tmp_path):
    if not os.path.exists(DAEMON):
        pytest.skip("tutti_daemon not built")
    sock = str(tmp_path / "acl.sock")
    cfg = tmp_path / "daemon.yaml"
    cfg.write_text(textwrap.dedent(f"""
        service: {{socket: {sock}}}
        devices:
          - {{id: 0, kind: emulated, mount: {tmp_path}/nvme0, queues: 8, accelerators: [3]}}
        """))
    p = subprocess.Popen([DAEMON, "--config", str(cfg)], stderr=subprocess.PIPE)
    try:
        for _ in range(100):
            if os.path.exists(sock):
                break
            time.sleep(0.05)
        c = Client(sock)
        assert c.kv("LIST")["accelerators"] == "3"
        s_other = c.kv(f"HELLO client=x pid={os.getpid()} accel=1")["session"]
        assert "PERMISSION_DENIED" in c(f"ACQUIRE session={s_other} devices=0 queues=2")
        s_mine = c.kv(f"HELLO client=y pid={os.getpid()} accel=3")["session"]
        assert c.kv(f"ACQUIRE session={s_mine} devices=0 queues=2")["lease"]
    finally:
        p.send_signal(signal.SIGTERM)
        p.wait(timeout=10)


def test_daemon_reads_tutti_schema(tmp_path):
    if not os.path.exists(DAEMON):
        pytest.skip("tutti_daemon not built")
    sock = str(tmp_path / "t.sock")
    cfg = tmp_path / "nvme_daemon.yaml"
    cfg.write_text(textwrap.dedent(f"""
        service: {{socket: {sock}}}
        grpc: {{endpoint: "127.0.0.1:50051"}}
        accelerators:
          - {{accel_id: 0, view_root: {tmp_path}/gpu0}}
        nvmes:
          - device_id: 0
            pci_addr: "0000:08:00.0"
            backing_mount_path: {tmp_path}/nvme0
            namespace_id: 1
            kernel_ioq_cap: 32
            allowed_accel_ids: [0]
            auto_mount: true
          - device_id: 1
            pci_addr: "0000:4b:00.0"
            backing_mount_path: {tmp_path}/nvme1
            namespace_id: 1
            kernel_ioq_cap: 32
            allowed_accel_ids: [1]
            auto_mount: true
        queue_pool: {{default_per_client: 16, max_per_client: 24}}
        lease: {{heartbeat_interval_sec: 10, timeout_sec: 30}}
        unmount_retry: {{interval_ms: 1000, max: 30}}
        """))
    p = subprocess.Popen([DAEMON, "--config", str(cfg)], stderr=subprocess.PIPE)
    try:
        for _ in range(100):
            if os.path.exists(sock):
                break
            time.sleep(0.05)
        c = Client(sock)
        lst = c.kv("LIST")
        assert lst["devices"] == "0,1" and lst["kinds"] == "nvme,nvme" and lst["accelerators"] == "0,1"
        assert lst["free_queues"] == "64,64" and lst["mounts"].endswith("nvme1")  # kernel_ioq_cap is not a budget
        s0 = c.kv(f"HELLO client=g0 pid={os.getpid()} accel=0")["session"]
        assert "RESOURCE_EXHAUSTED" in c(f"ACQUIRE session={s0} devices=0 queues=30")  # above max_per_client
        assert "PERMISSION_DENIED" in c(f"ACQUIRE session={s0} devices=1 queues=8")
        c.kv(f"ACQUIRE session={s0} devices=0 queues=0")  # 0: the pool's default
        assert c.kv("LIST")["free_queues"] == "48,64"
    finally:
        p.send_signal(signal.SIGTERM)
        p.wait(timeout=10)


def _kv(rsp):
    assert rsp.startswith("OK"), rsp
    from urllib.parse import unquote
    return {k: unquote(v) for k, v in (t.split("=", 1) for t in rsp.split()[1:])}


def test_daemon_service_surface_connect_slices_and_resources():
    devs = [{"id": 0, "mount": "/mnt/nvme 0", "queues": 32, "accelerators": [0], "pci": "0000:08:00.0",
             "chrdev": "/dev/ssnvme0", "lba_bytes": 4096},
            {"id": 1, "mount": "/mnt/nvme1", "queues": 32, "accelerators": [0, 1]},
            {"id": 2, "mount": "/mnt/nvme2", "queues": 32, "available": False, "diagnostic": "mount: no superblock"}]
    accs = [{"accel_id": 0, "view_root": "/run/tutti/gpu0"}, {"accel_id": 1, "view_root": "/run/tutti/gpu1"}]
    out = core().daemon_handle_request_selftest(
        ["LIST_DEVICES", "LIST_ACCELERATORS",
         "CONNECT device=0 accel=0 queues=8 pid=0",
         "ACQUIRE_SLICES accel=1 selection=allowed queues=4 pid=0",
         "ACQUIRE_SLICES accel=0 selection=striped queues=4 pid=0",
         "ACQUIRE_SLICES accel=1 selection=explicit devices=0 queues=4 pid=0",
         "CONNECT device=2 accel=0 queues=4 pid=0",
         "LIST_RESOURCES", "HEARTBEAT allocation_id=1", "DISCONNECT allocation_id=1",
         "ACQUIRE_SLICES accel=1 selection=striped queues=4 pid=0", "STATUS"], devs, accs)
    lst = _kv(out[0])
    assert lst["devices"] == "3" and lst["d0.pci_addr"] == "0000:08:00.0" and lst["d0.snvme_dev_path"] == "/dev/ssnvme0"
    assert lst["d0.blk_size_log"] == "12" and lst["d0.backing_mount_path"] == "/mnt/nvme 0"  # spaces survive
    assert lst["d1.allowed_gpus"] == "0:/run/tutti/gpu0/nvme1;1:/run/tutti/gpu1/nvme1"
    acc = _kv(out[1])
    assert acc["accelerators"] == "2" and acc["a1.view_root"] == "/run/tutti/gpu1"
    con = _kv(out[2])  # the reference's ConnectResponse fields
    assert con["allocation_id"] == "2" and con["granted_queues"] == "8" and con["mount_path"] == "/run/tutti/gpu0/nvme0"
    assert con["snvme_dev_path"] == "/dev/ssnvme0" and con["blk_size"] == "4096" and con["lease_timeout_sec"] == "30"
    sl = _kv(out[3])  # accelerator 1 may use device 1 only
    assert sl["slices"] == "1" and sl["s0.device_id"] == "1" and sl["s0.view_path"] == "/run/tutti/gpu1/nvme1"
    st = _kv(out[4])  # striped over the available drives accelerator 0 may use (2 is unavailable)
    assert st["slices"] == "2" and st["s0.device_id"] == "0" and st["s1.device_id"] == "1"
    assert out[5].startswith("ERR") and "PERMISSION_DENIED" in out[5]
    assert out[6].startswith("ERR") and "unavailable" in out[6] and "no superblock" in out[6]
    res = _kv(out[7])
    assert res["resources"] == "3" and res["r2.available"] == "false" and res["r2.available_queues"] == "0"
    assert res["r0.reserved_queues"] == "12" and res["r0.controller_queue_capacity"] == "32"
    assert out[8].startswith("ERR")  # allocation 1 does not exist (ids count sessions too)
    assert out[9].startswith("ERR")
    assert out[10].startswith("ERR") and "RESOURCE_EXHAUSTED" in out[10]  # one drive cannot be striped
    assert _kv(out[11])["leases"] == "3"


def test_daemon_connect_and_disconnect_close_their_session():
    out = core().daemon_handle_request_selftest(
        ["CONNECT device=0 accel=0 queues=16 pid=0", "LIST", "DISCONNECT allocation_id=2", "LIST",
         "DISCONNECT allocation_id=2"],
        [{"id": 0, "mount": "/m0", "queues": 32}])
    assert _kv(out[0])["allocation_id"] == "2"
    assert _kv(out[1])["free_queues"] == "16"
    assert _kv(out[2])["success"] == "true"
    assert _kv(out[3])["free_queues"] == "32"
    assert out[4].startswith("ERR") and "NOT_FOUND" in out[4]


def test_daemon_builds_accelerator_view_roots(tmp_path):
    if not os.path.exists(DAEMON):
        pytest.skip("tutti_daemon not built")
    sock = str(tmp_path / "v.sock")
    (tmp_path / "gpu0").mkdir()
    (tmp_path / "gpu0" / "nvme1").symlink_to("/stale/target")  # replaced
    (tmp_path / "gpu0" / "keep.txt").write_text("x")  # left alone
    cfg = tmp_path / "daemon.yaml"
    cfg.write_text(textwrap.dedent(f"""
        service: {{socket: {sock}}}
        accelerators:
          - {{accel_id: 0, view_root: {tmp_path}/gpu0}}
          - {{accel_id: 1, view_root: {tmp_path}/gpu1}}
        nvmes:
          - {{device_id: 0, backing_mount_path: {tmp_path}/nvme0, allowed_accel_ids: [0]}}
          - {{device_id: 1, backing_mount_path: {tmp_path}/nvme1, allowed_accel_ids: [0, 1]}}
        """))
    p = subprocess.Popen([DAEMON, "--config", str(cfg)], stderr=subprocess.PIPE)
    try:
        for _ in range(100):
            if os.path.exists(sock):
                break
            time.sleep(0.05)
        assert os.readlink(tmp_path / "gpu0" / "nvme0") == f"{tmp_path}/nvme0"
        assert os.readlink(tmp_path / "gpu0" / "nvme1") == f"{tmp_path}/nvme1"
        assert os.readlink(tmp_path / "gpu1" / "nvme1") == f"{tmp_path}/nvme1"
        assert not (tmp_path / "gpu1" / "nvme0").exists()
        assert (tmp_path / "gpu0" / "keep.txt").read_text() == "x"
        c = Client(sock)
        sl = c.kv("ACQUIRE_SLICES accel=1 selection=allowed queues=4 pid=%d" % os.getpid())
        assert sl["slices"] == "1" and sl["s0.view_path"] == f"{tmp_path}/gpu1/nvme1"
        res = c.kv("LIST_RESOURCES")
        assert res["r0.available"] == "true"  # no block device configured: mounted outside the daemon
    finally:
        p.send_signal(signal.SIGTERM)
        p.wait(timeout=10)
