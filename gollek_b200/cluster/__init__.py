"""Cluster plane: node roles and the KV-cache hand-off RPC between prefill and decode nodes.

The service keeps the reference's wire contract — package ``tech.kayys.gollek.cluster.proto``,
service ``GollekInternal`` with ``HandoffCache`` and ``Ping``, and its message field numbers
(inference/gollek-cluster/src/main/proto/gollek_internal.proto:9-44) — so nodes of either
implementation can talk. The schema is built in code (no protoc step). Unlike the reference's
acknowledging stub (…/cluster/CacheHandoffService.java:27-54), the receiving node reconstitutes
the sequence: ``block_data`` carries the packed KV blocks ``[L, n, 2, Hk, block_size, head_dim]``
and ``metadata`` the prompt/first tokens, sampling parameters and tensor layout; the decode node
scatters the blocks into its own pool (``engine.disagg.import_sequence``) and continues decoding.

Node roles follow ``NodeRole`` (…/cluster/NodeRole.java:8-43): PREFILL, DECODE, BOTH, GATEWAY,
selected by ``GOLLEK_CLUSTER_ROLE`` (the reference's ``gollek.cluster.role``).
"""
from __future__ import annotations

import enum
import json
import os
import queue
import threading
from concurrent import futures
from typing import Callable, Optional

import torch

from google.protobuf import descriptor_pb2, descriptor_pool, message_factory

PACKAGE = "tech.kayys.gollek.cluster.proto"
SERVICE = f"{PACKAGE}.GollekInternal"
MAX_MESSAGE = 2 ** 31 - 1


class NodeRole(enum.Enum):
    PREFILL = "PREFILL"
    DECODE = "DECODE"
    BOTH = "BOTH"
    GATEWAY = "GATEWAY"

    @property
    def can_prefill(self) -> bool:
        return self in (NodeRole.PREFILL, NodeRole.BOTH)

    @property
    def can_decode(self) -> bool:
        return self in (NodeRole.DECODE, NodeRole.BOTH)

    @staticmethod
    def from_env(default: str = "BOTH") -> "NodeRole":
        return NodeRole(os.environ.get("GOLLEK_CLUSTER_ROLE", default).upper())


def _build_messages():
    F = descriptor_pb2.FieldDescriptorProto
    fd = descriptor_pb2.FileDescriptorProto(name="gollek_b200_internal.proto", package=PACKAGE, syntax="proto3")

    def msg(name, fields):
        m = fd.message_type.add(name=name)
        for fname, num, ftype, label, tname in fields:
            f = m.field.add(name=fname, number=num, type=ftype, label=label)
            if tname:
                f.type_name = tname
        return m

    opt, rep = F.LABEL_OPTIONAL, F.LABEL_REPEATED
    req = msg("CacheHandoffRequest", [("request_id", 1, F.TYPE_STRING, opt, None),
                                      ("model_id", 2, F.TYPE_STRING, opt, None),
                                      ("prompt_token_count", 3, F.TYPE_INT32, opt, None),
                                      ("block_ids", 4, F.TYPE_INT32, rep, None),
                                      ("block_data", 5, F.TYPE_BYTES, opt, None),
                                      ("metadata", 6, F.TYPE_MESSAGE, rep,
                                       f".{PACKAGE}.CacheHandoffRequest.MetadataEntry")])
    entry = req.nested_type.add(name="MetadataEntry")
    entry.field.add(name="key", number=1, type=F.TYPE_STRING, label=opt)
    entry.field.add(name="value", number=2, type=F.TYPE_STRING, label=opt)
    entry.options.map_entry = True
    msg("CacheHandoffResponse", [("success", 1, F.TYPE_BOOL, opt, None),
                                 ("error_message", 2, F.TYPE_STRING, opt, None),
                                 ("decode_node_id", 3, F.TYPE_STRING, opt, None)])
    msg("PingRequest", [("source_node_id", 1, F.TYPE_STRING, opt, None)])
    msg("PingResponse", [("node_id", 1, F.TYPE_STRING, opt, None), ("role", 2, F.TYPE_STRING, opt, None),
                         ("ready", 3, F.TYPE_BOOL, opt, None)])
    svc = fd.service.add(name="GollekInternal")
    svc.method.add(name="HandoffCache", input_type=f".{PACKAGE}.CacheHandoffRequest",
                   output_type=f".{PACKAGE}.CacheHandoffResponse")
    svc.method.add(name="Ping", input_type=f".{PACKAGE}.PingRequest", output_type=f".{PACKAGE}.PingResponse")
    pool = descriptor_pool.DescriptorPool()
    pool.Add(fd)
    get = lambda n: message_factory.GetMessageClass(pool.FindMessageTypeByName(f"{PACKAGE}.{n}"))  # noqa: E731
    return (get("CacheHandoffRequest"), get("CacheHandoffResponse"), get("PingRequest"), get("PingResponse"))


CacheHandoffRequest, CacheHandoffResponse, PingRequest, PingResponse = _build_messages()

_DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def handoff_to_proto(h) -> "CacheHandoffRequest":
    """``engine.disagg.KVHandoff`` → wire message (KV bytes go through host memory)."""
    kv = h.kv.detach().contiguous()
    meta = {"prompt_token_ids": json.dumps(h.prompt_token_ids), "output_token_ids": json.dumps(h.output_token_ids),
            "params": json.dumps(h.params), "block_size": str(h.block_size), "kv_shape": json.dumps(list(kv.shape)),
            "kv_dtype": str(kv.dtype).replace("torch.", ""), "lora_id": str(h.lora_id)}
    return CacheHandoffRequest(request_id=h.request_id, model_id=h.model_id,
                               prompt_token_count=len(h.prompt_token_ids),
                               block_ids=list(range(kv.shape[1])),
                               block_data=kv.cpu().view(torch.uint8).numpy().tobytes(), metadata=meta)


def proto_to_handoff(req, device: Optional[torch.device] = None):
    from ..engine.disagg import KVHandoff
    m = dict(req.metadata)
    shape = json.loads(m["kv_shape"])
    dt = _DTYPES[m["kv_dtype"]]
    kv = torch.frombuffer(bytearray(req.block_data), dtype=torch.uint8).view(dt).view(*shape)
    if device is not None:
        kv = kv.to(device)
    return KVHandoff(req.request_id, req.model_id, json.loads(m["prompt_token_ids"]),
                     json.loads(m["output_token_ids"]), json.loads(m["params"]), int(m["block_size"]), kv,
                     int(m.get("lora_id", "0")))


class HandoffServer:
    """gRPC ``GollekInternal`` endpoint of a decode (or BOTH) node. Received hand-offs are queued;
    the node's engine loop imports them between steps (``drain``), never concurrently with a step."""

    def __init__(self, node_id: str, role: NodeRole = NodeRole.DECODE, port: int = 0, host: str = "127.0.0.1",
                 ready: Callable[[], bool] = lambda: True, max_workers: int = 4):
        import grpc
        self.node_id, self.role, self.ready = node_id, role, ready
        self.inbox: "queue.Queue" = queue.Queue()
        opts = [("grpc.max_receive_message_length", MAX_MESSAGE), ("grpc.max_send_message_length", MAX_MESSAGE)]
        self.server = grpc.server(futures.ThreadPoolExecutor(max_workers=max_workers), options=opts)
        handlers = {
            "HandoffCache": grpc.unary_unary_rpc_method_handler(
                self._handoff, request_deserializer=CacheHandoffRequest.FromString,
                response_serializer=CacheHandoffResponse.SerializeToString),
            "Ping": grpc.unary_unary_rpc_method_handler(
                self._ping, request_deserializer=PingRequest.FromString,
                response_serializer=PingResponse.SerializeToString),
        }
        self.server.add_generic_rpc_handlers((grpc.method_handlers_generic_handler(SERVICE, handlers),))
        self.port = self.server.add_insecure_port(f"{host}:{port}")
        self.address = f"{host}:{self.port}"

    def start(self) -> "HandoffServer":
        self.server.start()
        return self

    def stop(self, grace: float = 0.5) -> None:
        self.server.stop(grace)

    def _ping(self, req, ctx):
        return PingResponse(node_id=self.node_id, role=self.role.value, ready=bool(self.ready()))

    def _handoff(self, req, ctx):
        if not self.role.can_decode:
            return CacheHandoffResponse(success=False, error_message=f"node role {self.role.value} does not decode",
                                        decode_node_id=self.node_id)
        try:
            done = threading.Event()
            box = {}
            self.inbox.put((req, done, box))
            if not done.wait(timeout=60.0):
                return CacheHandoffResponse(success=False, error_message="decode node did not import in time",
                                            decode_node_id=self.node_id)
            err = box.get("error")
            return CacheHandoffResponse(success=err is None, error_message=err or "", decode_node_id=self.node_id)
        except Exception as e:  # report, never crash the RPC thread
            return CacheHandoffResponse(success=False, error_message=str(e), decode_node_id=self.node_id)

    def drain(self, engine) -> int:
        """Import queued hand-offs into ``engine`` (call from the engine's thread between steps)."""
        from ..engine.disagg import import_sequence
        n = 0
        while True:
            try:
                req, done, box = self.inbox.get_nowait()
            except queue.Empty:
                return n
            try:
                import_sequence(engine, proto_to_handoff(req, engine.kv_cache.device))
                n += 1
            except Exception as e:
                box["error"] = str(e)
            finally:
                done.set()


class HandoffClient:
    def __init__(self, address: str, timeout: float = 120.0):
        import grpc
        opts = [("grpc.max_receive_message_length", MAX_MESSAGE), ("grpc.max_send_message_length", MAX_MESSAGE)]
        self.channel = grpc.insecure_channel(address, options=opts)
        self.timeout = timeout
        self._handoff = self.channel.unary_unary(f"/{SERVICE}/HandoffCache",
                                                 request_serializer=CacheHandoffRequest.SerializeToString,
                                                 response_deserializer=CacheHandoffResponse.FromString)
        self._ping = self.channel.unary_unary(f"/{SERVICE}/Ping", request_serializer=PingRequest.SerializeToString,
                                              response_deserializer=PingResponse.FromString)

    def ping(self, source: str = "") -> "PingResponse":
        return self._ping(PingRequest(source_node_id=source), timeout=self.timeout)

    def send(self, handoff) -> "CacheHandoffResponse":
        return self._handoff(handoff_to_proto(handoff), timeout=self.timeout)

    def close(self) -> None:
        self.channel.close()


class RemoteHandoff:
    """Prefill-node side of cross-node disaggregation: install as ``engine.handoff_hook`` of a
    PREFILL engine whose requests carry their full ``max_tokens`` in ``full_params``."""

    def __init__(self, engine, client: HandoffClient):
        self.engine, self.client = engine, client
        self.full_params = {}
        self.sent = 0
        self.failed = []
        engine.handoff_hook = self

    def __call__(self, seq) -> bool:
        import dataclasses
        from ..engine.disagg import export_sequence
        full = self.full_params.pop(seq.request_id, None)
        if full is None or len(seq.output_token_ids) >= full.max_tokens:
            return False
        h = export_sequence(self.engine, seq)
        h.params = dataclasses.asdict(full)
        r = self.client.send(h)
        if not r.success:
            self.failed.append((seq.request_id, r.error_message))
            return False
        self.sent += 1
        return True
