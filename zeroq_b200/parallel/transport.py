"""ZeroMQ control plane (reference ``src/transport.py``).

On one NVSwitch node every byte of training data moves over NVLink (NCCL or
this framework's peer-memory kernels).  This module is the control plane for
multi-node or multi-job setups: registration, heartbeats and failure detection,
barriers, and a small CPU data plane (tensor send/recv, naive all-reduce, the
ring of :class:`zeroq_b200.parallel.gradient_sync.RingAllReduce`).

Class and message names follow the reference: ``TransportCoordinator``
(ROUTER + PUB sockets, :197-427), ``TransportWorker`` (DEALER, SUB, PULL, and
one PUSH per peer, :430-793), ``GradientCompressor`` (Top-K with error feedback,
:94-167), ``serialize_tensor``/``deserialize_tensor`` and ``create_transport``.

Differences, all deliberate:

* Tensors travel as a JSON header plus raw bytes (``serialize_tensor``); nothing
  received from the network is unpickled.
* Heartbeats use their own DEALER socket, so a heartbeat reply can never be
  consumed by a barrier waiting on the control socket.
* Barriers carry a generation number, so a late release of barrier ``g`` cannot
  release barrier ``g+1``.
* ``recv_gradient``/``recv_chunk`` raise ``TimeoutError`` instead of returning
  ``None`` (``recv_gradient(..., raise_on_timeout=False)`` keeps the old
  behaviour).
* ``fault_injector`` (tests only) can drop or delay outgoing data messages.
"""

from __future__ import annotations

import json
import struct
import threading
import time
import zlib
from dataclasses import dataclass
from enum import Enum
from typing import Any, Callable, Dict, Optional, Tuple, Union

import torch

try:
    import zmq

    HAS_ZMQ = True
except ImportError:  # pragma: no cover
    HAS_ZMQ = False


class MessageType(Enum):
    REGISTER = "register"
    HEARTBEAT = "heartbeat"
    HEARTBEAT_ACK = "heartbeat_ack"
    NODE_LIST = "node_list"
    SHUTDOWN = "shutdown"
    BARRIER = "barrier"
    BARRIER_ACK = "barrier_ack"
    GRADIENT = "gradient"
    GRADIENT_ACK = "gradient_ack"
    PARAM_REQUEST = "param_request"
    PARAM_RESPONSE = "param_response"
    REDUCE_SCATTER = "reduce_scatter"
    ALL_GATHER = "all_gather"
    RING_SEND = "ring_send"
    RING_RECV_ACK = "ring_recv_ack"


@dataclass
class NodeInfo:
    node_id: str
    hostname: str
    port: int
    rank: int
    gpus: int
    last_heartbeat: float = 0.0
    is_alive: bool = True

    @property
    def address(self) -> str:
        return f"tcp://{self.hostname}:{self.port}"


@dataclass
class TransportConfig:
    bind_address: str = "0.0.0.0"
    coordinator_host: str = "localhost"
    coordinator_port: int = 5555
    data_port_start: int = 5560
    heartbeat_interval_ms: int = 5000
    heartbeat_timeout_ms: int = 15000
    recv_timeout_ms: int = 30000
    send_timeout_ms: int = 30000
    high_water_mark: int = 1000
    tcp_buffer_size: int = 4 * 1024 * 1024
    compress_threshold: int = 1024 * 1024
    use_compression: bool = True


# ----------------------------------------------------------------------------
# Tensor codec and compression
# ----------------------------------------------------------------------------

_DTYPES = {str(d): d for d in (torch.float32, torch.float16, torch.bfloat16, torch.float64,
                                torch.int64, torch.int32, torch.int16, torch.int8, torch.uint8,
                                torch.bool)}


def serialize_tensor(tensor: torch.Tensor) -> bytes:
    """``[u32 header length][JSON header][raw little-endian bytes]``."""
    t = tensor.detach().contiguous().cpu()
    header = json.dumps({"shape": list(t.shape), "dtype": str(t.dtype)}).encode()
    raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
    return struct.pack("<I", len(header)) + header + raw


def deserialize_tensor(data: bytes, device: Union[str, torch.device] = "cpu") -> torch.Tensor:
    (hlen,) = struct.unpack_from("<I", data, 0)
    header = json.loads(data[4:4 + hlen].decode())
    dtype = _DTYPES.get(header["dtype"])
    if dtype is None:
        raise ValueError(f"unsupported dtype {header['dtype']!r}")
    payload = bytearray(data[4 + hlen:])
    if not payload:
        return torch.empty(header["shape"], dtype=dtype, device=device)
    t = torch.frombuffer(payload, dtype=torch.uint8).view(dtype).reshape(header["shape"])
    return t.clone().to(device)


class GradientCompressor:
    """Top-K magnitude sparsification with error feedback; values sent as fp16."""

    def __init__(self, compression_ratio: float = 0.01):
        self.compression_ratio = compression_ratio
        self.error_feedback: Dict[int, torch.Tensor] = {}

    def compress(self, tensor: torch.Tensor, param_id: int
                 ) -> Tuple[torch.Tensor, torch.Tensor, Dict[str, Any]]:
        if param_id in self.error_feedback:
            tensor = tensor + self.error_feedback[param_id]
        flat = tensor.reshape(-1)
        k = max(1, int(flat.numel() * self.compression_ratio))
        _, idx = torch.topk(flat.abs(), k)
        vals = flat[idx]
        residual = flat.clone()
        residual[idx] = 0
        self.error_feedback[param_id] = residual.view(tensor.shape)
        meta = {"shape": list(tensor.shape), "numel": tensor.numel(), "k": k,
                "dtype": str(tensor.dtype)}
        return vals.to(torch.float16), idx, meta

    def decompress(self, values: torch.Tensor, indices: torch.Tensor, metadata: Dict[str, Any],
                   device: Union[str, torch.device] = "cpu") -> torch.Tensor:
        flat = torch.zeros(metadata["numel"], dtype=torch.float32, device=device)
        flat[indices.to(device)] = values.to(device=device, dtype=torch.float32)
        return flat.view(metadata["shape"])


def _require_zmq():
    if not HAS_ZMQ:
        raise ImportError("pyzmq is required for the multi-node transport")


# ----------------------------------------------------------------------------
# Coordinator
# ----------------------------------------------------------------------------

class TransportCoordinator:
    """Registers nodes, tracks heartbeats, releases barriers, publishes the node list."""

    def __init__(self, config: Optional[TransportConfig] = None):
        _require_zmq()
        self.config = config or TransportConfig()
        self.context = zmq.Context()
        self.nodes: Dict[str, NodeInfo] = {}
        self.rank_to_node: Dict[int, str] = {}
        self.next_rank = 0
        self._barrier_arrivals: Dict[int, set] = {}
        self.router_socket = None
        self.pub_socket = None
        self._running = False
        self._lock = threading.Lock()
        self._heartbeat_thread: Optional[threading.Thread] = None
        self._loop_thread: Optional[threading.Thread] = None
        self.on_node_dead: Optional[Callable[[NodeInfo], None]] = None

    def start(self, background: bool = False):
        self.router_socket = self.context.socket(zmq.ROUTER)
        self.router_socket.setsockopt(zmq.RCVHWM, self.config.high_water_mark)
        self.router_socket.setsockopt(zmq.SNDHWM, self.config.high_water_mark)
        self.router_socket.setsockopt(zmq.LINGER, 0)
        self.router_socket.bind(f"tcp://{self.config.bind_address}:{self.config.coordinator_port}")
        self.pub_socket = self.context.socket(zmq.PUB)
        self.pub_socket.setsockopt(zmq.LINGER, 0)
        self.pub_socket.bind(f"tcp://{self.config.bind_address}:{self.config.coordinator_port + 1}")
        self._running = True
        self._heartbeat_thread = threading.Thread(target=self._heartbeat_monitor, daemon=True)
        self._heartbeat_thread.start()
        if background:
            self._loop_thread = threading.Thread(target=self.run, daemon=True)
            self._loop_thread.start()

    def stop(self):
        if not self._running:
            return
        self._running = False
        try:
            self.pub_socket.send_json({"type": MessageType.SHUTDOWN.value})
        except Exception:
            pass
        if self._loop_thread is not None:
            self._loop_thread.join(timeout=2.0)
        for s in (self.router_socket, self.pub_socket):
            if s is not None:
                s.close(0)
        self.context.term()

    def run(self):
        while self._running:
            try:
                if self.router_socket.poll(timeout=50):
                    frames = self.router_socket.recv_multipart()
                    identity, body = frames[0], frames[-1]
                    msg = json.loads(body.decode())
                    reply = self._handle_message(identity, msg)
                    self.router_socket.send_multipart([identity, b"", json.dumps(reply).encode()])
            except zmq.ZMQError:
                if self._running:
                    time.sleep(0.01)
            except Exception as e:  # keep serving other nodes
                if self._running:
                    print(f"[Coordinator] error: {e!r}")

    def alive_count(self) -> int:
        return sum(1 for n in self.nodes.values() if n.is_alive)

    def _handle_message(self, identity: bytes, msg: dict) -> dict:
        t = msg.get("type")
        if t == MessageType.REGISTER.value:
            return self._handle_register(msg)
        if t == MessageType.HEARTBEAT.value:
            return self._handle_heartbeat(msg)
        if t == MessageType.BARRIER.value:
            return self._handle_barrier(msg)
        return {"status": "error", "message": f"Unknown message type: {t}"}

    def _handle_register(self, msg: dict) -> dict:
        with self._lock:
            nid = msg["node_id"]
            if nid in self.nodes:
                node = self.nodes[nid]
                node.last_heartbeat = time.time()
                node.is_alive = True
                node.port = msg.get("port", node.port)
            else:
                node = NodeInfo(node_id=nid, hostname=msg["hostname"], port=msg["port"],
                                rank=self.next_rank, gpus=msg.get("gpus", 1),
                                last_heartbeat=time.time())
                self.next_rank += 1
                self.nodes[nid] = node
                self.rank_to_node[node.rank] = nid
            self._broadcast_node_list()
            return {"status": "ok", "rank": node.rank, "world_size": self.alive_count()}

    def _handle_heartbeat(self, msg: dict) -> dict:
        with self._lock:
            node = self.nodes.get(msg["node_id"])
            if node is None:
                return {"status": "error", "message": "Node not registered"}
            node.last_heartbeat = time.time()
            revived = not node.is_alive
            node.is_alive = True
            if revived:
                self._broadcast_node_list()
            return {"status": "ok", "type": MessageType.HEARTBEAT_ACK.value}

    def _handle_barrier(self, msg: dict) -> dict:
        with self._lock:
            gen = int(msg.get("gen", 0))
            arrived = self._barrier_arrivals.setdefault(gen, set())
            arrived.add(msg["node_id"])
            alive = {nid for nid, n in self.nodes.items() if n.is_alive}
            if alive and alive.issubset(arrived):
                del self._barrier_arrivals[gen]
                self.pub_socket.send_json({"type": MessageType.BARRIER_ACK.value, "gen": gen})
                return {"status": "ok", "released": True, "gen": gen}
            return {"status": "ok", "released": False, "waiting": len(arrived), "gen": gen}

    def _broadcast_node_list(self):
        nodes = {nid: {"hostname": n.hostname, "port": n.port, "rank": n.rank, "gpus": n.gpus}
                 for nid, n in self.nodes.items() if n.is_alive}
        self.pub_socket.send_json({"type": MessageType.NODE_LIST.value, "nodes": nodes,
                                   "world_size": len(nodes)})

    def _heartbeat_monitor(self):
        period = self.config.heartbeat_interval_ms / 1000.0
        timeout = self.config.heartbeat_timeout_ms / 1000.0
        while self._running:
            time.sleep(min(period, timeout / 4))
            now = time.time()
            dead = []
            with self._lock:
                for n in self.nodes.values():
                    if n.is_alive and now - n.last_heartbeat > timeout:
                        n.is_alive = False
                        dead.append(n)
                if dead:
                    # a dead node can no longer hold up a barrier
                    alive = {nid for nid, n in self.nodes.items() if n.is_alive}
                    for gen, arrived in list(self._barrier_arrivals.items()):
                        if alive and alive.issubset(arrived):
                            del self._barrier_arrivals[gen]
                            self.pub_socket.send_json({"type": MessageType.BARRIER_ACK.value,
                                                       "gen": gen})
                    self._broadcast_node_list()
            for n in dead:
                if self.on_node_dead is not None:
                    self.on_node_dead(n)


# ----------------------------------------------------------------------------
# Worker
# ----------------------------------------------------------------------------

class TransportWorker:
    """One node's side of the control plane plus a CPU tensor data plane."""

    def __init__(self, node_id: str, hostname: str, config: Optional[TransportConfig] = None,
                 local_gpus: int = 1):
        _require_zmq()
        self.node_id = node_id
        self.hostname = hostname
        self.config = config or TransportConfig()
        self.local_gpus = local_gpus
        self.context = zmq.Context()
        self.rank = -1
        self.world_size = 0
        self.peers: Dict[int, NodeInfo] = {}
        self.dealer_socket = None
        self._hb_socket = None
        self._dealer_lock = threading.Lock()
        self.sub_socket = None
        self._sub_lock = threading.Lock()
        self.peer_sockets: Dict[int, Any] = {}
        self._send_lock = threading.Lock()
        self.recv_socket = None
        self.data_port = -1
        self._running = False
        self._heartbeat_thread = None
        self._recv_thread = None
        self._lock = threading.Lock()
        self._recv_cv = threading.Condition(self._lock)
        self._recv_buffer: Dict[Any, Dict[int, torch.Tensor]] = {}
        self._barrier_gen = 0
        self._released_gens: set = set()
        self.compressor = GradientCompressor()
        self.fault_injector: Optional[Callable[[dict], Optional[float]]] = None
        self.heartbeat_enabled = True

    # -- setup ---------------------------------------------------------------
    def _dealer(self, identity: str):
        s = self.context.socket(zmq.DEALER)
        s.setsockopt(zmq.IDENTITY, identity.encode())
        s.setsockopt(zmq.RCVTIMEO, self.config.recv_timeout_ms)
        s.setsockopt(zmq.SNDTIMEO, self.config.send_timeout_ms)
        s.setsockopt(zmq.LINGER, 0)
        s.connect(f"tcp://{self.config.coordinator_host}:{self.config.coordinator_port}")
        return s

    def _request(self, sock, msg: dict) -> dict:
        sock.send_multipart([b"", json.dumps(msg).encode()])
        frames = sock.recv_multipart()
        return json.loads(frames[-1].decode())

    def connect(self) -> bool:
        self.dealer_socket = self._dealer(self.node_id)
        self._hb_socket = self._dealer(self.node_id + "#hb")
        self.sub_socket = self.context.socket(zmq.SUB)
        self.sub_socket.setsockopt(zmq.SUBSCRIBE, b"")
        self.sub_socket.setsockopt(zmq.LINGER, 0)
        self.sub_socket.connect(f"tcp://{self.config.coordinator_host}:{self.config.coordinator_port + 1}")
        self.recv_socket = self.context.socket(zmq.PULL)
        self.recv_socket.setsockopt(zmq.RCVHWM, self.config.high_water_mark)
        self.recv_socket.setsockopt(zmq.LINGER, 0)
        base = self.config.data_port_start + zlib.adler32(self.node_id.encode()) % 1000
        for attempt in range(1000):
            try:
                self.recv_socket.bind(f"tcp://{self.config.bind_address}:{base + attempt}")
                self.data_port = base + attempt
                break
            except zmq.ZMQError:
                continue
        else:
            return False
        try:
            with self._dealer_lock:
                resp = self._request(self.dealer_socket, {
                    "type": MessageType.REGISTER.value, "node_id": self.node_id,
                    "hostname": self.hostname, "port": self.data_port, "gpus": self.local_gpus})
        except zmq.ZMQError:
            return False
        if resp.get("status") != "ok":
            return False
        self.rank = int(resp["rank"])
        self.world_size = int(resp["world_size"])
        self._running = True
        self._heartbeat_thread = threading.Thread(target=self._heartbeat_loop, daemon=True)
        self._heartbeat_thread.start()
        self._recv_thread = threading.Thread(target=self._receive_loop, daemon=True)
        self._recv_thread.start()
        self.poll_broadcasts(timeout_sec=0.5)
        return True

    def disconnect(self):
        self._running = False
        for t in (self._heartbeat_thread, self._recv_thread):
            if t is not None:
                t.join(timeout=2.0)
        for s in list(self.peer_sockets.values()) + [self.dealer_socket, self._hb_socket,
                                                     self.sub_socket, self.recv_socket]:
            if s is not None:
                s.close(0)
        self.peer_sockets.clear()
        self.context.term()

    # -- background threads --------------------------------------------------
    def _heartbeat_loop(self):
        period = self.config.heartbeat_interval_ms / 1000.0 / 2
        while self._running:
            time.sleep(period)
            if not self.heartbeat_enabled:
                continue
            try:
                self._request(self._hb_socket, {"type": MessageType.HEARTBEAT.value,
                                                "node_id": self.node_id})
            except zmq.ZMQError:
                pass  # the coordinator's timeout notices a silent node

    def _receive_loop(self):
        while self._running:
            try:
                if self.recv_socket.poll(timeout=50):
                    header, payload = self.recv_socket.recv_multipart()
                    self._handle_peer_message(json.loads(header.decode()), payload)
            except zmq.ZMQError:
                pass
            except Exception as e:
                print(f"[Worker {self.node_id}] receive error: {e!r}")

    def _handle_peer_message(self, hdr: dict, payload: bytes):
        t = hdr.get("type")
        if t == MessageType.GRADIENT.value:
            key = ("grad", hdr["param_id"])
        elif t == MessageType.RING_SEND.value:
            key = ("ring", tuple(hdr["tag"]), tuple(hdr["chunk"]))
        else:
            return
        tensor = deserialize_tensor(payload)
        with self._recv_cv:
            self._recv_buffer.setdefault(key, {})[int(hdr["src_rank"])] = tensor
            self._recv_cv.notify_all()

    # -- node list / barrier -------------------------------------------------
    def update_peers(self, nodes: Dict[str, dict]):
        with self._lock:
            live_ranks = set()
            for nid, info in nodes.items():
                if nid == self.node_id:
                    continue
                r = int(info["rank"])
                live_ranks.add(r)
                if r not in self.peers:
                    self.peers[r] = NodeInfo(node_id=nid, hostname=info["hostname"],
                                             port=int(info["port"]), rank=r,
                                             gpus=int(info.get("gpus", 1)))
                    s = self.context.socket(zmq.PUSH)
                    s.setsockopt(zmq.SNDHWM, self.config.high_water_mark)
                    s.setsockopt(zmq.LINGER, 0)
                    s.connect(self.peers[r].address)
                    self.peer_sockets[r] = s
            for r in list(self.peers):
                self.peers[r].is_alive = r in live_ranks

    def _on_broadcast(self, msg: dict):
        t = msg.get("type")
        if t == MessageType.NODE_LIST.value:
            self.update_peers(msg["nodes"])
            self.world_size = int(msg["world_size"])
        elif t == MessageType.BARRIER_ACK.value:
            self._released_gens.add(int(msg.get("gen", 0)))
        elif t == MessageType.SHUTDOWN.value:
            self._running = False

    def poll_broadcasts(self, timeout_sec: float = 0.0):
        end = time.time() + timeout_sec
        with self._sub_lock:
            while True:
                remaining = max(0.0, end - time.time())
                if not self.sub_socket.poll(timeout=int(remaining * 1000)):
                    break
                self._on_broadcast(self.sub_socket.recv_json())
                if time.time() >= end:
                    break

    def barrier(self, timeout_sec: float = 60.0) -> bool:
        """Block until every live node reached this barrier; ``False`` on timeout."""
        gen = self._barrier_gen
        self._barrier_gen += 1
        with self._dealer_lock:
            resp = self._request(self.dealer_socket, {"type": MessageType.BARRIER.value,
                                                      "node_id": self.node_id, "gen": gen})
        if resp.get("released"):
            return True
        end = time.time() + timeout_sec
        while time.time() < end:
            if gen in self._released_gens:
                self._released_gens.discard(gen)
                return True
            self.poll_broadcasts(timeout_sec=min(0.05, max(0.0, end - time.time())))
        return gen in self._released_gens

    # -- data plane ----------------------------------------------------------
    def _send(self, dst_rank: int, header: dict, tensor: torch.Tensor):
        if dst_rank not in self.peer_sockets:
            self.poll_broadcasts(timeout_sec=0.2)
        if dst_rank not in self.peer_sockets:
            raise ValueError(f"No connection to rank {dst_rank}")
        if self.fault_injector is not None:
            delay = self.fault_injector(header)
            if delay is None:
                return  # dropped
            if delay > 0:
                time.sleep(delay)
        with self._send_lock:
            self.peer_sockets[dst_rank].send_multipart(
                [json.dumps(header).encode(), serialize_tensor(tensor)])

    def _recv(self, key, src_rank: int, timeout_sec: float, raise_on_timeout: bool = True):
        end = time.time() + timeout_sec
        with self._recv_cv:
            while True:
                slot = self._recv_buffer.get(key)
                if slot is not None and src_rank in slot:
                    t = slot.pop(src_rank)
                    if not slot:
                        del self._recv_buffer[key]
                    return t
                remaining = end - time.time()
                if remaining <= 0:
                    if raise_on_timeout:
                        raise TimeoutError(f"[Worker {self.node_id}] no message {key} "
                                           f"from rank {src_rank} within {timeout_sec}s")
                    return None
                self._recv_cv.wait(timeout=min(remaining, 0.05))

    def send_gradient(self, tensor: torch.Tensor, param_id: int, dst_rank: int,
                      compress: bool = False):
        self._send(dst_rank, {"type": MessageType.GRADIENT.value, "param_id": int(param_id),
                              "src_rank": self.rank}, tensor)

    def recv_gradient(self, param_id: int, src_rank: int, timeout_sec: float = 30.0,
                      raise_on_timeout: bool = True) -> Optional[torch.Tensor]:
        return self._recv(("grad", int(param_id)), src_rank, timeout_sec, raise_on_timeout)

    def send_chunk(self, dst_rank: int, tag, chunk_id, tensor: torch.Tensor):
        self._send(dst_rank, {"type": MessageType.RING_SEND.value, "tag": list(tag),
                              "chunk": list(chunk_id), "src_rank": self.rank}, tensor)

    def recv_chunk(self, src_rank: int, tag, chunk_id, timeout_sec: float = 30.0) -> torch.Tensor:
        return self._recv(("ring", tuple(tag), tuple(chunk_id)), src_rank, timeout_sec)

    def all_reduce(self, tensor: torch.Tensor, param_id: int, op: str = "sum") -> torch.Tensor:
        """Naive all-reduce: send to every peer, sum what comes back."""
        peers = sorted(self.peer_sockets)
        for r in peers:
            self.send_gradient(tensor, param_id, r)
        out = tensor.clone()
        for r in peers:
            out += self.recv_gradient(param_id, r, timeout_sec=self.config.recv_timeout_ms / 1000)
        if op == "mean":
            out /= max(1, self.world_size)
        return out


def create_transport(role: str, node_id: str, hostname: str = "localhost",
                     coordinator_host: str = "localhost", coordinator_port: int = 5555,
                     local_gpus: int = 1):
    cfg = TransportConfig(coordinator_host=coordinator_host, coordinator_port=coordinator_port)
    if role == "coordinator":
        return TransportCoordinator(cfg)
    if role == "worker":
        return TransportWorker(node_id=node_id, hostname=hostname, config=cfg,
                               local_gpus=local_gpus)
    raise ValueError(f"Unknown role: {role}")


__all__ = ["MessageType", "NodeInfo", "TransportConfig", "TransportCoordinator",
           "TransportWorker", "GradientCompressor", "serialize_tensor",
           "deserialize_tensor", "create_transport"]
