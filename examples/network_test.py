#!/usr/bin/env python
"""ZeroMQ link check between two hosts: tensor round trips, latency and bandwidth.

Counterpart of the reference's ``simple_network_test.py``.  The server echoes
every tensor back doubled; the client checks the values and reports the
round-trip time per size (and a GPU round trip when CUDA is present).

    python examples/network_test.py --role server --port 5556
    python examples/network_test.py --role client --server-host head --port 5556
    python examples/network_test.py --role local          # both ends in one process
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from zeroq_b200.parallel.transport import deserialize_tensor, serialize_tensor  # noqa: E402

SIZES = (1 << 10, 1 << 16, 1 << 20, 1 << 24)  # elements (fp32)


def run_server(port: int, rounds: int, ready: threading.Event = None):
    import zmq

    ctx = zmq.Context()
    sock = ctx.socket(zmq.REP)
    sock.setsockopt(zmq.LINGER, 10000)  # let the last (large) reply leave before close
    sock.bind(f"tcp://*:{port}")
    if ready is not None:
        ready.set()
    try:
        for _ in range(rounds):
            t = deserialize_tensor(sock.recv())
            sock.send(serialize_tensor(t * 2))
    finally:
        sock.close()
        ctx.term()


def run_client(host: str, port: int, reps: int) -> list:
    import zmq

    ctx = zmq.Context()
    sock = ctx.socket(zmq.REQ)
    sock.setsockopt(zmq.LINGER, 0)
    sock.setsockopt(zmq.RCVTIMEO, 60000)
    sock.connect(f"tcp://{host}:{port}")
    results = []
    try:
        devices = ["cpu"] + (["cuda"] if torch.cuda.is_available() else [])
        for dev in devices:
            for n in SIZES:
                x = torch.arange(n, dtype=torch.float32, device=dev) % 1000
                times = []
                for _ in range(reps):
                    t0 = time.perf_counter()
                    sock.send(serialize_tensor(x.cpu()))
                    y = deserialize_tensor(sock.recv(), device=dev)
                    times.append(time.perf_counter() - t0)
                    if not torch.equal(y, x * 2):
                        raise RuntimeError(f"corrupted round trip at {n} elements on {dev}")
                best = min(times)
                results.append({"device": dev, "elements": n, "bytes": 4 * n,
                                "rtt_ms": round(best * 1e3, 3),
                                "gbit_s": round(2 * 4 * n * 8 / best / 1e9, 3)})
                print(json.dumps(results[-1]), flush=True)
    finally:
        sock.close(0)
        ctx.term()
    return results


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--role", choices=["server", "client", "local"], required=True)
    p.add_argument("--server-host", default="localhost")
    p.add_argument("--port", type=int, default=5556)
    p.add_argument("--reps", type=int, default=3)
    args = p.parse_args(argv)
    rounds = len(SIZES) * args.reps * (2 if torch.cuda.is_available() else 1)
    if args.role == "server":
        run_server(args.port, rounds)
        return 0
    if args.role == "client":
        run_client(args.server_host, args.port, args.reps)
        return 0
    ready = threading.Event()
    t = threading.Thread(target=run_server, args=(args.port, rounds, ready), daemon=True)
    t.start()
    ready.wait(10)
    run_client("127.0.0.1", args.port, args.reps)
    t.join(10)
    return 0


if __name__ == "__main__":
    sys.exit(main())
