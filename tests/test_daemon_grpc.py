"""Tutti's gRPC NvmeService over this daemon: the gateway against the real tutti_daemon binary,
called the way a Tutti client calls it (service/method paths, message field numbers)."""
import os
import signal
import subprocess
import textwrap
import time

import pytest

grpc = pytest.importorskip("grpc")

from tutti_b200 import daemon_grpc as dg  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DAEMON = os.path.join(ROOT, "tutti_b200", "bin", "tutti_daemon")
M = dg.messages


@pytest.fixture
def gateway(tmp_path):
    if not os.path.exists(DAEMON):
        pytest.skip("tutti_daemon not built")
    sock = str(tmp_path / "d.sock")
    cfg = tmp_path / "daemon.yaml"
    cfg.write_text(textwrap.dedent(f"""
        service: {{socket: {sock}}}
        accelerators:
          - {{accel_id: 0, view_root: {tmp_path}/gpu0}}
          - {{accel_id: 1, view_root: {tmp_path}/gpu1}}
        nvmes:
          - {{device_id: 0, backing_mount_path: {tmp_path}/nvme0, pci_addr: "0000:1b:00.0", allowed_accel_ids: [0]}}
          - {{device_id: 1, backing_mount_path: {tmp_path}/nvme1, allowed_accel_ids: [0, 1]}}
        """))
    p = subprocess.Popen([DAEMON, "--config", str(cfg)], stderr=subprocess.PIPE)
    for _ in range(200):
        if os.path.exists(sock):
            break
        time.sleep(0.05)
    server, port = dg.serve(sock, "127.0.0.1:0")
    channel = grpc.insecure_channel(f"127.0.0.1:{port}")
    try:
        yield channel, tmp_path
    finally:
        channel.close()
        server.stop(1)
        p.send_signal(signal.SIGTERM)
        p.wait(timeout=10)


def test_messages_keep_tuttis_wire_format():
    # field numbers decide the bytes: ConnectResponse.granted_queues is field 10, error_message 99
    r = M["ConnectResponse"](allocation_id="7", granted_queues=4, error_message="x")
    assert r.SerializeToString() == b"\x0a\x017" + b"\x50\x04" + b"\x9a\x06\x01x"
    req = M["AcquireNvmeSlicesRequest"](accel_id=1, selection=2, device_ids=[0, 1])
    assert req.SerializeToString() == b"\x08\x01\x10\x02\x1a\x02\x00\x01"  # packed repeated int32
    assert dg.method_path("AcquireNvmeSlices") == "/nvmeservice.NvmeService/AcquireNvmeSlices"


def test_gateway_serves_the_nvme_service(gateway):
    channel, tmp = gateway
    devs = dg.stub(channel, "ListDevices")(M["Empty"](), timeout=10)
    assert [d.device_id for d in devs.devices] == [0, 1]
    assert devs.devices[0].pci_addr == "0000:1b:00.0" and devs.devices[0].page_size == 4096
    assert [(g.cuda_device, g.mount_path) for g in devs.devices[1].allowed_gpus] == \
        [(0, f"{tmp}/gpu0/nvme1"), (1, f"{tmp}/gpu1/nvme1")]
    acc = dg.stub(channel, "ListAccelerators")(M["Empty"](), timeout=10)
    assert [(a.accel_id, a.view_root) for a in acc.accelerators] == [(0, f"{tmp}/gpu0"), (1, f"{tmp}/gpu1")]

    con = dg.stub(channel, "Connect")(M["ConnectRequest"](device_id=0, cuda_device=0, num_queues=4,
                                                           client_pid=os.getpid()), timeout=10)
    assert con.error_message == "" and con.allocation_id and con.granted_queues == 4
    assert con.mount_path == f"{tmp}/gpu0/nvme0" and con.lease_timeout_sec > 0
    denied = dg.stub(channel, "Connect")(M["ConnectRequest"](device_id=0, cuda_device=1, num_queues=4,
                                                              client_pid=os.getpid()), timeout=10)
    assert "PERMISSION_DENIED" in denied.error_message and not denied.allocation_id

    res = dg.stub(channel, "ListNvmeResources")(M["Empty"](), timeout=10)
    r0 = res.resources[0]
    assert r0.reserved_queues == 4 and r0.available and list(r0.allowed_accel_ids) == [0]
    assert list(res.resources[1].allowed_accel_ids) == [0, 1]

    sl = dg.stub(channel, "AcquireNvmeSlices")(M["AcquireNvmeSlicesRequest"](
        accel_id=0, selection=M["AcquireNvmeSlicesRequest"].DESCRIPTOR.fields_by_name["selection"]
        .enum_type.values_by_name["NVME_SELECTION_STRIPED"].number, queues_per_controller=2,
        client_pid=os.getpid()), timeout=10)
    assert sl.error_message == "" and [s.device_id for s in sl.slices] == [0, 1]
    assert [s.view_path for s in sl.slices] == [f"{tmp}/gpu0/nvme0", f"{tmp}/gpu0/nvme1"]
    assert all(s.granted_queues == 2 and s.accel_id == 0 for s in sl.slices)

    # the heartbeat stream echoes each allocation; an unknown one is revoked
    beats = list(dg.stub(channel, "Heartbeat")(iter([M["HeartbeatMsg"](allocation_id=con.allocation_id),
                                                      M["HeartbeatMsg"](allocation_id="999")]), timeout=10))
    kind = M["AdminNotice"].DESCRIPTOR.enum_types_by_name["Kind"].values_by_name
    assert beats[0].allocation_id == con.allocation_id and beats[0].notice.kind == kind["NONE"].number
    assert beats[0].timestamp_ns > 0 and beats[1].notice.kind == kind["LEASE_REVOKED"].number

    rel = dg.stub(channel, "Release")(M["ReleaseRequest"](allocation_id=sl.allocation_id), timeout=10)
    assert rel.success and not rel.already_released
    again = dg.stub(channel, "Release")(M["ReleaseRequest"](allocation_id=sl.allocation_id), timeout=10)
    assert not again.success and again.already_released
    bye = dg.stub(channel, "Disconnect")(M["DisconnectRequest"](allocation_id=con.allocation_id), timeout=10)
    assert bye.success
    res = dg.stub(channel, "ListNvmeResources")(M["Empty"](), timeout=10)
    assert all(r.reserved_queues == 0 for r in res.resources)


def test_gateway_reports_a_daemon_that_is_gone(tmp_path):
    server, port = dg.serve(str(tmp_path / "missing.sock"), "127.0.0.1:0")
    channel = grpc.insecure_channel(f"127.0.0.1:{port}")
    try:
        with pytest.raises(grpc.RpcError) as e:
            dg.stub(channel, "ListDevices")(M["Empty"](), timeout=10)
        assert e.value.code() == grpc.StatusCode.UNAVAILABLE
    finally:
        channel.close()
        server.stop(1)
