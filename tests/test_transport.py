"""ZeroMQ control plane, ring all-reduce, compression, accumulation (reference
tests/test_transport.py).  Failures are made on the host: a worker that stops
heartbeating, a message the test drops, a barrier nobody completes."""

import socket
import threading
import time

import pytest
import torch

import zeroq_b200 as zq
from zeroq_b200.parallel.gradient_sync import (GradientAccumulator, GradSyncConfig, RingAllReduce,
                                               SyncMode, TorchDistributedSync)
from zeroq_b200.parallel.transport import (GradientCompressor, TransportConfig,
                                           TransportCoordinator, TransportWorker,
                                           deserialize_tensor, serialize_tensor)


def _port_pair() -> int:
    for _ in range(50):
        s1, s2 = socket.socket(), socket.socket()
        try:
            s1.bind(("127.0.0.1", 0))
            p = s1.getsockname()[1]
            s2.bind(("127.0.0.1", p + 1))
            return p
        except OSError:
            continue
        finally:
            s1.close()
            s2.close()
    raise RuntimeError("no free port pair")


def _cluster(n, hb_ms=200, timeout_ms=1000):
    port = _port_pair()
    cfg = TransportConfig(bind_address="127.0.0.1", coordinator_host="127.0.0.1",
                          coordinator_port=port, data_port_start=20000 + (port % 20000),
                          heartbeat_interval_ms=hb_ms, heartbeat_timeout_ms=timeout_ms,
                          recv_timeout_ms=5000, send_timeout_ms=5000)
    coord = TransportCoordinator(cfg)
    coord.start(background=True)
    workers = [TransportWorker(f"node{i}", "127.0.0.1", cfg) for i in range(n)]
    for w in workers:
        assert w.connect()
    deadline = time.time() + 5
    while time.time() < deadline and not all(len(w.peer_sockets) == n - 1 for w in workers):
        for w in workers:
            w.poll_broadcasts(0.05)
    for w in workers:
        w.world_size = n
    return coord, workers


def _shutdown(coord, workers):
    for w in workers:
        w.disconnect()
    coord.stop()


class TestSerialization:
    @pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16, torch.int64])
    def test_roundtrip(self, dtype):
        t = (torch.randn(3, 5, 7) * 10).to(dtype)
        assert torch.equal(deserialize_tensor(serialize_tensor(t)), t)

    def test_large_and_empty(self):
        t = torch.randn(1_000_000)
        assert torch.equal(deserialize_tensor(serialize_tensor(t)), t)
        e = torch.empty(0, 4)
        assert deserialize_tensor(serialize_tensor(e)).shape == (0, 4)


class TestCompression:
    def test_topk(self):
        c = GradientCompressor(0.1)
        g = torch.randn(1000)
        vals, idx, meta = c.compress(g, 0)
        assert vals.dtype == torch.float16 and meta["k"] == 100
        out = c.decompress(vals, idx, meta, "cpu")
        top = g.abs().topk(100).indices
        assert torch.allclose(out[top], g[top], atol=1e-2)

    def test_error_feedback(self):
        c = GradientCompressor(0.01)
        g = torch.randn(1000)
        vals, idx, meta = c.compress(g, 7)
        resid = c.error_feedback[7]
        assert torch.allclose(resid.view(-1)[idx], torch.zeros(len(idx)))
        assert torch.allclose(resid.sum() + g[idx].sum(), g.sum(), atol=1e-4)


class TestAccumulator:
    def test_single_process(self):
        acc = GradientAccumulator(TorchDistributedSync())
        acc.accumulate(0, torch.ones(3))
        acc.accumulate(0, torch.ones(3))
        out = acc.sync_and_clear()
        assert torch.equal(out[0], torch.full((3,), 2.0))

    def test_local_sgd(self):
        acc = GradientAccumulator(TorchDistributedSync(),
                                  GradSyncConfig(mode=SyncMode.LOCAL_SGD, local_steps=3))
        assert [acc.should_sync() for _ in range(3)] == [False, False, True]

    def test_create_gradient_sync(self):
        assert isinstance(zq.create_gradient_sync("nccl"), TorchDistributedSync)
        with pytest.raises(ValueError):
            zq.create_gradient_sync("ring")


class TestControlPlane:
    def test_register_barrier_ring_allreduce(self):
        coord, ws = _cluster(3)
        try:
            assert sorted(w.rank for w in ws) == [0, 1, 2]
            results = [None] * 3

            def body(i):
                assert ws[i].barrier(timeout_sec=5)
                ring = RingAllReduce(ws[i], GradSyncConfig(timeout_sec=10))
                t = torch.arange(10, dtype=torch.float32) + ws[i].rank
                results[i] = ring.all_reduce(t, param_id=1)

            th = [threading.Thread(target=body, args=(i,)) for i in range(3)]
            [t.start() for t in th]
            [t.join(30) for t in th]
            expect = torch.arange(10, dtype=torch.float32) * 3 + 3
            for r in results:
                assert torch.equal(r, expect)
        finally:
            _shutdown(coord, ws)

    def test_naive_allreduce(self):
        coord, ws = _cluster(2)
        try:
            out = [None, None]

            def body(i):
                out[i] = ws[i].all_reduce(torch.full((4,), float(ws[i].rank + 1)), param_id=3)

            th = [threading.Thread(target=body, args=(i,)) for i in range(2)]
            [t.start() for t in th]
            [t.join(30) for t in th]
            assert torch.equal(out[0], torch.full((4,), 3.0)) and torch.equal(out[0], out[1])
        finally:
            _shutdown(coord, ws)

    def test_dead_node_detected_by_heartbeat_timeout(self):
        coord, ws = _cluster(2, hb_ms=100, timeout_ms=600)
        dead = []
        coord.on_node_dead = lambda n: dead.append(n.node_id)
        try:
            ws[1].heartbeat_enabled = False  # the node goes silent
            deadline = time.time() + 5
            while time.time() < deadline and not dead:
                time.sleep(0.05)
            assert dead == ["node1"]
            assert coord.alive_count() == 1
            ws[1].heartbeat_enabled = True   # a new heartbeat revives it
            deadline = time.time() + 5
            while time.time() < deadline and coord.alive_count() != 2:
                time.sleep(0.05)
            assert coord.alive_count() == 2
        finally:
            _shutdown(coord, ws)

    def test_barrier_timeout_returns_false(self):
        coord, ws = _cluster(2)
        try:
            assert ws[0].barrier(timeout_sec=0.5) is False  # node1 never arrives
        finally:
            _shutdown(coord, ws)

    def test_dropped_message_raises_timeout(self):
        coord, ws = _cluster(2)
        try:
            ws[0].fault_injector = lambda hdr: None  # drop everything node0 sends
            ws[0].send_gradient(torch.ones(3), param_id=9, dst_rank=ws[1].rank)
            with pytest.raises(TimeoutError):
                ws[1].recv_gradient(9, ws[0].rank, timeout_sec=0.5)
            assert ws[1].recv_gradient(9, ws[0].rank, timeout_sec=0.2, raise_on_timeout=False) is None
        finally:
            _shutdown(coord, ws)

    def test_ring_chunk_loss_is_an_error(self):
        coord, ws = _cluster(2)
        try:
            ws[0].fault_injector = lambda hdr: None
            ring = RingAllReduce(ws[1], GradSyncConfig(timeout_sec=0.5))
            with pytest.raises(TimeoutError):
                ring.all_reduce(torch.ones(8), param_id=2)
        finally:
            _shutdown(coord, ws)
