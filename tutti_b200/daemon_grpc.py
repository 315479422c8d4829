"""gRPC front end of the device-manager daemon: Tutti's ``nvmeservice.NvmeService``.

Clients written against Tutti's NVMe service (package ``nvmeservice``, service
``NvmeService``: ListDevices, Connect, Disconnect, Heartbeat (bidirectional
stream), ListAccelerators, ListNvmeResources, AcquireNvmeSlices, Release)
talk to this gateway unchanged: the messages are declared here with the same
names, field numbers and types, so the bytes on the wire are the same. Each
call is translated to the daemon's line protocol on its UNIX socket
(``tutti_daemon``: LIST_DEVICES, CONNECT, ...), which keeps the queue ledger,
leases and reaper; the gateway holds no state of its own.

    python -m tutti_b200 daemon-grpc --socket /run/tutti/daemon.sock --listen 127.0.0.1:50051

Errors the daemon reports come back in the response's ``error_message`` field
(Connect, AcquireNvmeSlices, Disconnect, Release), as a LEASE_REVOKED notice
(Heartbeat), or as a gRPC status (the list calls). The message classes are
built at import from a descriptor assembled in code (no generated stubs).
Parity: reference csrc/device_manager/nvme/nvmeservice/src/nvmeservice.proto
(the service and message contract) and nvmeservice_server.h (the server).
"""
from __future__ import annotations

import os
import socket
import threading
import time
from concurrent import futures

from google.protobuf import descriptor_pb2, descriptor_pool, message_factory

PACKAGE = "nvmeservice"
SERVICE = "NvmeService"

_F = descriptor_pb2.FieldDescriptorProto
_SCALAR = {"int32": _F.TYPE_INT32, "uint32": _F.TYPE_UINT32, "uint64": _F.TYPE_UINT64, "string": _F.TYPE_STRING,
           "bool": _F.TYPE_BOOL}

# message -> [(field, number, type, repeated)]; a type that is not a scalar names a message or an enum
_MESSAGES = {
    "Empty": [],
    "AllowedGpu": [("cuda_device", 1, "int32", False), ("mount_path", 2, "string", False)],
    "DeviceInfo": [("device_id", 1, "int32", False), ("pci_addr", 2, "string", False),
                   ("snvme_dev_path", 3, "string", False), ("namespace_id", 4, "uint32", False),
                   ("page_size", 5, "uint32", False), ("blk_size", 6, "uint32", False),
                   ("blk_size_log", 7, "uint32", False), ("queue_depth", 8, "uint32", False),
                   ("dstrd", 9, "uint32", False), ("max_user_qid", 11, "uint32", False),
                   ("max_queues_per_group", 12, "uint32", False), ("allowed_gpus", 13, "AllowedGpu", True)],
    "DeviceListResponse": [("devices", 1, "DeviceInfo", True)],
    "ConnectRequest": [("device_id", 1, "int32", False), ("cuda_device", 2, "int32", False),
                       ("num_queues", 3, "int32", False), ("client_pid", 4, "uint32", False)],
    "ConnectResponse": [("allocation_id", 1, "string", False), ("pci_addr", 2, "string", False),
                        ("snvme_dev_path", 3, "string", False), ("granted_queues", 10, "int32", False),
                        ("namespace_id", 20, "uint32", False), ("page_size", 21, "uint32", False),
                        ("blk_size", 22, "uint32", False), ("blk_size_log", 23, "uint32", False),
                        ("queue_depth", 24, "uint32", False), ("dstrd", 25, "uint32", False),
                        ("max_data_size", 26, "uint64", False), ("heartbeat_interval_sec", 30, "uint32", False),
                        ("lease_timeout_sec", 31, "uint32", False), ("mount_path", 32, "string", False),
                        ("error_message", 99, "string", False)],
    "DisconnectRequest": [("allocation_id", 1, "string", False), ("client_pid", 2, "uint32", False)],
    "DisconnectResponse": [("success", 1, "bool", False), ("error_message", 2, "string", False)],
    "AdminNotice": [("kind", 1, "AdminNotice.Kind", False), ("seconds_remaining", 2, "uint32", False),
                    ("message", 3, "string", False)],
    "HeartbeatMsg": [("allocation_id", 1, "string", False), ("timestamp_ns", 2, "uint64", False),
                     ("notice", 3, "AdminNotice", False)],
    "AcceleratorInfo": [("accel_id", 1, "int32", False), ("view_root", 2, "string", False)],
    "AcceleratorListResponse": [("accelerators", 1, "AcceleratorInfo", True)],
    "NvmeResource": [("device_id", 1, "int32", False), ("pci_bdf", 2, "string", False),
                     ("chrdev_minor", 3, "int32", False), ("chrdev_path", 4, "string", False),
                     ("block_path", 5, "string", False), ("backing_mount_path", 6, "string", False),
                     ("namespace_id", 7, "uint32", False), ("page_size", 8, "uint32", False),
                     ("logical_block_size", 9, "uint32", False), ("logical_block_size_log", 10, "uint32", False),
                     ("queue_depth", 11, "uint32", False), ("dstrd", 12, "uint32", False),
                     ("max_data_size", 14, "uint64", False), ("max_user_qid", 15, "uint32", False),
                     ("kernel_io_qps", 16, "uint32", False), ("controller_queue_capacity", 17, "uint32", False),
                     ("max_queues_per_group", 18, "uint32", False), ("reserved_queues", 19, "uint32", False),
                     ("available_queues", 20, "uint32", False), ("allowed_accel_ids", 21, "int32", True),
                     ("available", 22, "bool", False), ("diagnostic", 23, "string", False),
                     ("heartbeat_interval_sec", 24, "uint32", False), ("lease_timeout_sec", 25, "uint32", False)],
    "NvmeResourceListResponse": [("resources", 1, "NvmeResource", True)],
    "AcquireNvmeSlicesRequest": [("accel_id", 1, "int32", False), ("selection", 2, "NvmeSelectionMode", False),
                                 ("device_ids", 3, "int32", True), ("queues_per_controller", 4, "int32", False),
                                 ("client_pid", 5, "uint32", False)],
    "NvmeSlice": [("device_id", 1, "int32", False), ("accel_id", 2, "int32", False), ("pci_bdf", 3, "string", False),
                  ("chrdev_minor", 4, "int32", False), ("chrdev_path", 5, "string", False),
                  ("block_path", 6, "string", False), ("backing_mount_path", 7, "string", False),
                  ("view_path", 8, "string", False), ("namespace_id", 9, "uint32", False),
                  ("page_size", 10, "uint32", False), ("logical_block_size", 11, "uint32", False),
                  ("logical_block_size_log", 12, "uint32", False), ("queue_depth", 13, "uint32", False),
                  ("dstrd", 14, "uint32", False), ("max_data_size", 16, "uint64", False),
                  ("controller_queue_capacity", 17, "uint32", False), ("granted_queues", 18, "uint32", False),
                  ("max_queues_per_group", 19, "uint32", False), ("allowed_accel_ids", 20, "int32", True),
                  ("heartbeat_interval_sec", 21, "uint32", False), ("lease_timeout_sec", 22, "uint32", False)],
    "AcquireNvmeSlicesResponse": [("allocation_id", 1, "string", False), ("slices", 2, "NvmeSlice", True),
                                  ("error_message", 99, "string", False)],
    "ReleaseRequest": [("allocation_id", 1, "string", False)],
    "ReleaseResponse": [("success", 1, "bool", False), ("already_released", 2, "bool", False),
                        ("error_message", 3, "string", False)],
}
_ENUMS = {"NvmeSelectionMode": [("NVME_SELECTION_ALLOWED", 0), ("NVME_SELECTION_EXPLICIT", 1),
                                ("NVME_SELECTION_STRIPED", 2)]}
_NESTED_ENUMS = {"AdminNotice": {"Kind": [("NONE", 0), ("LEASE_EXPIRING", 1), ("LEASE_REVOKED", 2)]}}

# method -> (request, response, client streaming, server streaming)
METHODS = {
    "ListDevices": ("Empty", "DeviceListResponse", False, False),
    "Connect": ("ConnectRequest", "ConnectResponse", False, False),
    "Disconnect": ("DisconnectRequest", "DisconnectResponse", False, False),
    "Heartbeat": ("HeartbeatMsg", "HeartbeatMsg", True, True),
    "ListAccelerators": ("Empty", "AcceleratorListResponse", False, False),
    "ListNvmeResources": ("Empty", "NvmeResourceListResponse", False, False),
    "AcquireNvmeSlices": ("AcquireNvmeSlicesRequest", "AcquireNvmeSlicesResponse", False, False),
    "Release": ("ReleaseRequest", "ReleaseResponse", False, False),
}


def _file_descriptor() -> descriptor_pb2.FileDescriptorProto:
    fd = descriptor_pb2.FileDescriptorProto(name="tutti_nvmeservice.proto", package=PACKAGE, syntax="proto3")
    for name, values in _ENUMS.items():
        e = fd.enum_type.add(name=name)
        for vn, num in values:
            e.value.add(name=vn, number=num)
    for name, fields in _MESSAGES.items():
        m = fd.message_type.add(name=name)
        for en, values in _NESTED_ENUMS.get(name, {}).items():
            e = m.enum_type.add(name=en)
            for vn, num in values:
                e.value.add(name=vn, number=num)
        for fname, num, ftype, repeated in fields:
            f = m.field.add(name=fname, number=num,
                            label=_F.LABEL_REPEATED if repeated else _F.LABEL_OPTIONAL)
            if ftype in _SCALAR:
                f.type = _SCALAR[ftype]
            elif ftype in _ENUMS or "." in ftype:
                f.type = _F.TYPE_ENUM
                f.type_name = f".{PACKAGE}.{ftype}"
            else:
                f.type = _F.TYPE_MESSAGE
                f.type_name = f".{PACKAGE}.{ftype}"
    svc = fd.service.add(name=SERVICE)
    for mname, (req, rsp, cs, ss) in METHODS.items():
        svc.method.add(name=mname, input_type=f".{PACKAGE}.{req}", output_type=f".{PACKAGE}.{rsp}",
                       client_streaming=cs, server_streaming=ss)
    return fd


_POOL = descriptor_pool.DescriptorPool()
_POOL.Add(_file_descriptor())
messages = {name: message_factory.GetMessageClass(_POOL.FindMessageTypeByName(f"{PACKAGE}.{name}"))
            for name in _MESSAGES}


def method_path(name: str) -> str:
    return f"/{PACKAGE}.{SERVICE}/{name}"


# -- the daemon's line protocol ------------------------------------------------------------
def _enc(v) -> str:
    out = []
    for ch in str(v):
        out.append(f"%{ord(ch):02X}" if ch in "% \t\n\r" else ch)
    return "".join(out)


def _dec(v: str) -> str:
    out, i = [], 0
    while i < len(v):
        h = v[i + 1:i + 3]
        if v[i] == "%" and len(h) == 2 and all(c in "0123456789abcdefABCDEF" for c in h):
            out.append(chr(int(h, 16)))
            i += 3
        else:
            out.append(v[i])
            i += 1
    return "".join(out)


class DaemonError(RuntimeError):
    """The daemon answered ERR (the message is its status)."""


class DaemonLink:
    """One connection to tutti_daemon's UNIX socket, one request at a time."""

    def __init__(self, path: str, timeout_s: float = 10.0):
        self.path, self.timeout_s = path, timeout_s
        self._mu = threading.Lock()
        self._sock = None
        self._file = None

    def _connect(self):
        s = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        s.settimeout(self.timeout_s)
        s.connect(self.path)
        self._sock, self._file = s, s.makefile("rwb")

    def call(self, verb: str, **kv) -> dict:
        line = " ".join([verb] + [f"{k}={_enc(v)}" for k, v in kv.items() if v is not None]) + "\n"
        with self._mu:
            for attempt in (0, 1):  # one reconnect if the daemon restarted
                try:
                    if self._file is None:
                        self._connect()
                    self._file.write(line.encode())
                    self._file.flush()
                    rsp = self._file.readline().decode()
                    if not rsp:
                        raise ConnectionError("daemon closed the connection")
                    break
                except OSError:
                    self.close_locked()
                    if attempt:
                        raise
        rsp = rsp.strip()
        if rsp.startswith("ERR"):
            raise DaemonError(rsp[4:] if len(rsp) > 3 else "error")
        out = {}
        for tok in rsp.split()[1:]:
            k, _, v = tok.partition("=")
            out[k] = _dec(v)
        return out

    def close_locked(self) -> None:
        for x in (self._file, self._sock):
            try:
                if x is not None:
                    x.close()
            except OSError:
                pass
        self._sock = self._file = None

    def close(self) -> None:
        with self._mu:
            self.close_locked()


def _int(d: dict, k: str, default: int = 0) -> int:
    try:
        return int(d.get(k, default))
    except ValueError:
        return default


def _ids(v: str) -> list[int]:
    if not v or v == "*":
        return []
    return [int(x) for x in v.split(",") if x]


def _log2(v: int) -> int:
    return max(0, v.bit_length() - 1)


class NvmeServiceGateway:
    """The NvmeService methods over a DaemonLink (register with ``add_to_server``)."""

    def __init__(self, link: DaemonLink):
        self.link = link

    # -- lists -------------------------------------------------------------------------
    def ListDevices(self, request, context):
        d = self.link.call("LIST_DEVICES")
        out = messages["DeviceListResponse"]()
        for i in range(_int(d, "devices")):
            p = f"d{i}."
            di = out.devices.add(device_id=_int(d, p + "device_id"), pci_addr=d.get(p + "pci_addr", ""),
                                 snvme_dev_path=d.get(p + "snvme_dev_path", ""),
                                 namespace_id=_int(d, p + "namespace_id", 1), page_size=_int(d, p + "page_size", 4096),
                                 blk_size=_int(d, p + "blk_size", 512), blk_size_log=_int(d, p + "blk_size_log", 9),
                                 queue_depth=_int(d, p + "queue_depth"), dstrd=_int(d, p + "dstrd"),
                                 max_user_qid=_int(d, p + "max_user_qid"),
                                 max_queues_per_group=_int(d, p + "max_queues_per_group"))
            for entry in filter(None, d.get(p + "allowed_gpus", "").split(";")):
                gpu, _, mount = entry.partition(":")
                di.allowed_gpus.add(cuda_device=int(gpu), mount_path=mount)
        return out

    def ListAccelerators(self, request, context):
        d = self.link.call("LIST_ACCELERATORS")
        out = messages["AcceleratorListResponse"]()
        for i in range(_int(d, "accelerators")):
            out.accelerators.add(accel_id=_int(d, f"a{i}.accel_id"), view_root=d.get(f"a{i}.view_root", ""))
        return out

    def ListNvmeResources(self, request, context):
        d = self.link.call("LIST_RESOURCES")
        out = messages["NvmeResourceListResponse"]()
        hb, lt = _int(d, "heartbeat_interval_sec"), _int(d, "lease_timeout_sec")
        for i in range(_int(d, "resources")):
            p = f"r{i}."
            lba = _int(d, p + "blk_size", 512)
            out.resources.add(
                device_id=_int(d, p + "device_id"), pci_bdf=d.get(p + "pci_addr", ""),
                chrdev_minor=_int(d, p + "chrdev_minor", -1), chrdev_path=d.get(p + "snvme_dev_path", ""),
                block_path=d.get(p + "block_path", ""), backing_mount_path=d.get(p + "backing_mount_path", ""),
                namespace_id=_int(d, p + "namespace_id", 1), page_size=_int(d, p + "page_size", 4096),
                logical_block_size=lba, logical_block_size_log=_log2(lba), queue_depth=_int(d, p + "queue_depth"),
                dstrd=_int(d, p + "dstrd"), max_data_size=_int(d, p + "max_data_size"),
                max_user_qid=_int(d, p + "max_user_qid"),
                controller_queue_capacity=_int(d, p + "controller_queue_capacity"),
                max_queues_per_group=_int(d, p + "max_queues_per_group"),
                reserved_queues=_int(d, p + "reserved_queues"), available_queues=_int(d, p + "available_queues"),
                allowed_accel_ids=_ids(d.get(p + "allowed_accel_ids", "")),
                available=d.get(p + "available", "true") == "true", diagnostic=d.get(p + "diagnostic", ""),
                heartbeat_interval_sec=hb, lease_timeout_sec=lt)
        return out

    # -- allocations -------------------------------------------------------------------
    def Connect(self, request, context):
        out = messages["ConnectResponse"]()
        try:
            d = self.link.call("CONNECT", device_id=request.device_id, accel=request.cuda_device,
                               queues=request.num_queues, pid=request.client_pid)
        except DaemonError as e:
            out.error_message = str(e)
            return out
        lba = _int(d, "blk_size", 512)
        out.allocation_id = d.get("allocation_id", "")
        out.pci_addr, out.snvme_dev_path = d.get("pci_addr", ""), d.get("snvme_dev_path", "")
        out.granted_queues = _int(d, "granted_queues")
        out.namespace_id, out.page_size = _int(d, "namespace_id", 1), _int(d, "page_size", 4096)
        out.blk_size, out.blk_size_log = lba, _log2(lba)
        out.queue_depth, out.dstrd = _int(d, "queue_depth"), _int(d, "dstrd")
        out.max_data_size = _int(d, "max_data_size")
        out.heartbeat_interval_sec, out.lease_timeout_sec = _int(d, "heartbeat_interval_sec"), _int(d, "lease_timeout_sec")
        out.mount_path = d.get("mount_path", "")
        return out

    def AcquireNvmeSlices(self, request, context):
        out = messages["AcquireNvmeSlicesResponse"]()
        mode = {0: "allowed", 1: "explicit", 2: "striped"}.get(int(request.selection), "allowed")
        try:
            d = self.link.call("ACQUIRE_SLICES", accel=request.accel_id, selection=mode,
                               devices=",".join(str(x) for x in request.device_ids) or None,
                               queues=request.queues_per_controller, pid=request.client_pid)
        except DaemonError as e:
            out.error_message = str(e)
            return out
        out.allocation_id = d.get("allocation_id", "")
        hb, lt = _int(d, "heartbeat_interval_sec"), _int(d, "lease_timeout_sec")
        for i in range(_int(d, "slices")):
            p = f"s{i}."
            lba = _int(d, p + "blk_size", 512)
            out.slices.add(
                device_id=_int(d, p + "device_id"), accel_id=_int(d, p + "accel_id", request.accel_id),
                pci_bdf=d.get(p + "pci_addr", ""), chrdev_minor=_int(d, p + "chrdev_minor", -1),
                chrdev_path=d.get(p + "snvme_dev_path", ""), block_path=d.get(p + "block_path", ""),
                backing_mount_path=d.get(p + "backing_mount_path", ""), view_path=d.get(p + "view_path", ""),
                namespace_id=_int(d, p + "namespace_id", 1), page_size=_int(d, p + "page_size", 4096),
                logical_block_size=lba, logical_block_size_log=_log2(lba), queue_depth=_int(d, p + "queue_depth"),
                dstrd=_int(d, p + "dstrd"), max_data_size=_int(d, p + "max_data_size"),
                controller_queue_capacity=_int(d, p + "controller_queue_capacity"),
                granted_queues=_int(d, p + "granted_queues"),
                max_queues_per_group=_int(d, p + "max_queues_per_group"),
                allowed_accel_ids=_ids(d.get(p + "allowed_accel_ids", "")), heartbeat_interval_sec=hb,
                lease_timeout_sec=lt)
        return out

    def _end(self, verb: str, allocation_id: str):
        try:
            self.link.call(verb, allocation_id=allocation_id)
            return True, False, ""
        except DaemonError as e:
            return False, "NOT_FOUND" in str(e), str(e)

    def Disconnect(self, request, context):
        ok, _gone, msg = self._end("DISCONNECT", request.allocation_id)
        return messages["DisconnectResponse"](success=ok, error_message=msg)

    def Release(self, request, context):
        ok, gone, msg = self._end("RELEASE", request.allocation_id)
        return messages["ReleaseResponse"](success=ok, already_released=gone, error_message="" if gone else msg)

    def Heartbeat(self, request_iterator, context):
        revoked = messages["AdminNotice"].Kind.Value("LEASE_REVOKED")
        for msg in request_iterator:
            out = messages["HeartbeatMsg"](allocation_id=msg.allocation_id, timestamp_ns=time.time_ns())
            try:
                self.link.call("HEARTBEAT", allocation_id=msg.allocation_id)
            except DaemonError as e:
                out.notice.kind = revoked
                out.notice.message = str(e)
            yield out

    # -- registration --------------------------------------------------------------------
    def handlers(self):
        import grpc

        table = {}
        for name, (req, rsp, cs, ss) in METHODS.items():
            fn = self._wrap(getattr(self, name))
            de, se = messages[req].FromString, messages[rsp].SerializeToString
            if cs and ss:
                table[name] = grpc.stream_stream_rpc_method_handler(fn, request_deserializer=de, response_serializer=se)
            else:
                table[name] = grpc.unary_unary_rpc_method_handler(fn, request_deserializer=de, response_serializer=se)
        return grpc.method_handlers_generic_handler(f"{PACKAGE}.{SERVICE}", table)

    @staticmethod
    def _wrap(fn):
        import grpc

        def call(request, context):
            try:
                return fn(request, context)
            except DaemonError as e:
                context.abort(grpc.StatusCode.FAILED_PRECONDITION, str(e))
            except OSError as e:
                context.abort(grpc.StatusCode.UNAVAILABLE, f"tutti_daemon unreachable: {e}")

        return call


def serve(socket_path: str, listen: str = "127.0.0.1:50051", workers: int = 8):
    """Start the gateway; returns (grpc server, bound port). ``server.stop(grace)`` ends it."""
    import grpc

    server = grpc.server(futures.ThreadPoolExecutor(max_workers=workers))
    gw = NvmeServiceGateway(DaemonLink(socket_path))
    server.add_generic_rpc_handlers((gw.handlers(),))
    port = server.add_insecure_port(listen)
    if port == 0:
        raise OSError(f"cannot listen on {listen}")
    server.start()
    return server, port


def stub(channel, name: str):
    """A client callable for method ``name`` on ``channel`` (tests and tools; Tutti's stubs work as well)."""
    req, rsp, cs, ss = METHODS[name]
    de, se = messages[rsp].FromString, messages[req].SerializeToString
    if cs and ss:
        return channel.stream_stream(method_path(name), request_serializer=se, response_deserializer=de)
    return channel.unary_unary(method_path(name), request_serializer=se, response_deserializer=de)


def main(argv=None) -> int:
    import argparse

    p = argparse.ArgumentParser(prog="python -m tutti_b200 daemon-grpc")
    p.add_argument("--socket", required=True, help="tutti_daemon's UNIX socket")
    p.add_argument("--listen", default="127.0.0.1:50051")
    args = p.parse_args(argv)
    if not os.path.exists(args.socket):
        print(f"error: no daemon socket at {args.socket}")
        return 1
    server, port = serve(args.socket, args.listen)
    print(f"nvmeservice.NvmeService on {args.listen.rsplit(':', 1)[0]}:{port} -> {args.socket}", flush=True)
    try:
        server.wait_for_termination()
    except KeyboardInterrupt:
        server.stop(2)
    return 0
