"""Multi-node runner: ZeroMQ control plane + per-GPU worker processes.

Command-line parity with the reference's ``run_distributed.py`` (``--role
coordinator|worker|both``, ``--coordinator host:port``, ``--gpus``, ``--script``,
``--backend``, ``--gradient-compression``, ``--hierarchical-sync``,
``--verbose``, ``--dry-run``); see ``run_distributed.py:42-375`` there.

    python -m zeroq_b200.run_distributed --role coordinator --port 5555
    python -m zeroq_b200.run_distributed --role worker --coordinator head:5555 --gpus 0,1,2,3 \\
        --expected-world 8 --script train.py
    python -m zeroq_b200.run_distributed --role both --gpus 0,1 --script train.py

Each worker process registers with the coordinator (which assigns ranks in
arrival order), waits until ``--expected-world`` nodes are registered (when
given), passes a control-plane barrier, and builds the gradient-sync backend:

* ``nccl`` / ``gloo``: ``torch.distributed`` is initialised with the
  coordinator-assigned rank and world size over TCP at ``--dist-addr``
  (default: the coordinator host) and ``--dist-port``;
* ``ring``: the ZeroMQ ring all-reduce of the transport (CPU data plane);
* ``--hierarchical-sync``: NCCL inside the node plus the ring between nodes.

The training script is executed with the globals ``RANK``, ``WORLD_SIZE``,
``LOCAL_RANK``, ``DEVICE``, ``GRAD_SYNC`` and ``TRANSPORT`` set, and its
``main()`` is called if it defines one.  Inside one 8×B200 node prefer
``torchrun`` with NCCL (the data plane is NVLink); this runner is the
cross-node control plane.
"""

from __future__ import annotations

import argparse
import datetime
import importlib.util
import os
import signal
import socket
import sys
import threading
import time
from typing import List, Optional, Tuple

import torch
import torch.multiprocessing as mp

from .parallel.gradient_sync import GradSyncConfig, create_gradient_sync
from .parallel.transport import TransportConfig, TransportCoordinator, TransportWorker


def parse_args(argv=None):
    p = argparse.ArgumentParser(description="zeroq_b200 distributed runner",
                                formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--role", choices=["coordinator", "worker", "both"], default="worker")
    p.add_argument("--host", default=socket.gethostname(), help="this node's hostname")
    p.add_argument("--port", type=int, default=5555, help="coordinator port (PUB socket at port+1)")
    p.add_argument("--coordinator", default="localhost:5555", help="coordinator host:port")
    p.add_argument("--gpus", default="0", help="comma-separated GPU ids, one worker each")
    p.add_argument("--gpus-per-node", type=int, default=None)
    p.add_argument("--script", default=None, help="training script to execute in each worker")
    p.add_argument("--config", default=None, help="JSON config passed to the script as CONFIG_PATH")
    p.add_argument("--backend", choices=["nccl", "gloo", "ring"], default="nccl")
    p.add_argument("--gradient-compression", action="store_true")
    p.add_argument("--hierarchical-sync", action="store_true")
    p.add_argument("--expected-world", type=int, default=0,
                   help="wait until this many workers registered before the first barrier")
    p.add_argument("--dist-addr", default=None, help="torch.distributed rendezvous host")
    p.add_argument("--dist-port", type=int, default=29531)
    p.add_argument("--timeout", type=float, default=120.0, help="registration/barrier timeout (s)")
    p.add_argument("--verbose", action="store_true")
    p.add_argument("--dry-run", action="store_true")
    return p.parse_args(argv)


def get_gpu_list(gpu_str: str) -> List[int]:
    if not gpu_str:
        return [0]
    return [int(g.strip()) for g in gpu_str.split(",") if g.strip()]


def get_coordinator_address(addr: str) -> Tuple[str, int]:
    if ":" in addr:
        host, port = addr.rsplit(":", 1)
        return host, int(port)
    return addr, 5555


def run_coordinator(args, stop_event: Optional[threading.Event] = None):
    """Serve registration, heartbeats and barriers until SIGINT/SIGTERM or ``stop_event``."""
    cfg = TransportConfig(bind_address="0.0.0.0", coordinator_port=args.port)
    coord = TransportCoordinator(cfg)
    coord.start(background=True)
    print(f"[coordinator] listening on {args.host}:{args.port}", flush=True)
    stop_event = stop_event or threading.Event()
    if threading.current_thread() is threading.main_thread():
        for sig in (signal.SIGINT, signal.SIGTERM):
            signal.signal(sig, lambda *_: stop_event.set())
    try:
        while not stop_event.is_set():
            stop_event.wait(0.2)
    finally:
        coord.stop()
    print("[coordinator] stopped", flush=True)


def _wait_for_world(worker: TransportWorker, n: int, timeout: float) -> bool:
    end = time.time() + timeout
    while time.time() < end:
        if worker.world_size >= n:
            return True
        worker.poll_broadcasts(timeout_sec=0.1)
    return worker.world_size >= n


def run_worker(args, local_rank: int = 0, local_size: int = 1) -> int:
    gpus = get_gpu_list(args.gpus)
    gpu_id = gpus[local_rank] if local_rank < len(gpus) else local_rank
    if torch.cuda.is_available():
        torch.cuda.set_device(gpu_id)
        device = torch.device("cuda", gpu_id)
    else:
        device = torch.device("cpu")
    host, port = get_coordinator_address(args.coordinator)
    node_id = f"{args.host}-gpu{gpu_id}-{os.getpid()}"
    worker = TransportWorker(node_id=node_id, hostname=args.host,
                             config=TransportConfig(coordinator_host=host, coordinator_port=port),
                             local_gpus=local_size)
    if not worker.connect():
        print(f"[worker {node_id}] could not register with {host}:{port}", flush=True)
        return 1
    if args.expected_world and not _wait_for_world(worker, args.expected_world, args.timeout):
        print(f"[worker {node_id}] only {worker.world_size} of {args.expected_world} workers "
              f"registered", flush=True)
        worker.disconnect()
        return 1
    if not worker.barrier(timeout_sec=args.timeout):
        print(f"[worker {node_id}] barrier timeout", flush=True)
        worker.disconnect()
        return 1
    rank, world = worker.rank, worker.world_size
    if args.verbose:
        print(f"[worker {node_id}] rank {rank}/{world} on {device}", flush=True)

    use_dist = args.backend in ("nccl", "gloo") or args.hierarchical_sync
    if use_dist:
        backend = args.backend if args.backend in ("nccl", "gloo") else "nccl"
        if backend == "nccl" and not torch.cuda.is_available():
            backend = "gloo"
        addr = args.dist_addr or host
        torch.distributed.init_process_group(
            backend, init_method=f"tcp://{addr}:{args.dist_port}", rank=rank, world_size=world,
            timeout=datetime.timedelta(seconds=args.timeout))
    mode = "hierarchical" if args.hierarchical_sync else ("ring" if args.backend == "ring" else "nccl")
    grad_sync = create_gradient_sync(mode=mode, transport=worker,
                                     config=GradSyncConfig(compress=args.gradient_compression))
    rc = 0
    try:
        if args.script:
            spec = importlib.util.spec_from_file_location("zeroq_training_script", args.script)
            mod = importlib.util.module_from_spec(spec)
            mod.RANK, mod.WORLD_SIZE, mod.LOCAL_RANK = rank, world, local_rank
            mod.DEVICE, mod.GRAD_SYNC, mod.TRANSPORT = device, grad_sync, worker
            mod.CONFIG_PATH = args.config
            spec.loader.exec_module(mod)
            if hasattr(mod, "main"):
                out = mod.main()
                rc = int(out) if isinstance(out, int) else 0
        else:
            print(f"[worker {node_id}] ready: rank {rank}/{world}, device {device}, "
                  f"peers {sorted(worker.peers)}", flush=True)
        worker.barrier(timeout_sec=args.timeout)  # finish together
    finally:
        if use_dist and torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()
        worker.disconnect()
    return rc


def _worker_entry(local_rank: int, args, local_size: int, results):
    results[local_rank] = run_worker(args, local_rank, local_size)


def spawn_local_workers(args) -> int:
    n = len(get_gpu_list(args.gpus))
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    procs = [ctx.Process(target=_worker_entry, args=(i, args, n, results)) for i in range(n)]
    for p in procs:
        p.start()
    for p in procs:
        p.join()
    codes = [results.get(i, p.exitcode or 1) for i, p in enumerate(procs)]
    manager.shutdown()
    return max([abs(c) for c in codes] + [0])


def run_both(args) -> int:
    stop = threading.Event()
    t = threading.Thread(target=run_coordinator, args=(args, stop), daemon=True)
    t.start()
    time.sleep(0.5)
    args.coordinator = f"localhost:{args.port}"
    if not args.expected_world:
        args.expected_world = len(get_gpu_list(args.gpus))
    try:
        return spawn_local_workers(args)
    finally:
        stop.set()
        t.join(timeout=5.0)


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.verbose or args.dry_run:
        print(f"role={args.role} host={args.host} port={args.port} coordinator={args.coordinator} "
              f"gpus={args.gpus} backend={args.backend} hierarchical={args.hierarchical_sync} "
              f"compression={args.gradient_compression}", flush=True)
    if args.dry_run:
        print("dry run: configuration valid", flush=True)
        return 0
    if args.role == "coordinator":
        run_coordinator(args)
        return 0
    if args.role == "worker":
        if len(get_gpu_list(args.gpus)) > 1:
            return spawn_local_workers(args)
        return run_worker(args)
    return run_both(args)


if __name__ == "__main__":
    sys.exit(main())
