"""The multi-node runner on CPU: coordinator + 2 workers, gloo and ZeroMQ ring backends."""

import os
import socket
import subprocess
import sys
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = textwrap.dedent('''
    import os, torch
    def main():
        t = torch.full((8,), float(RANK + 1))
        if GRAD_SYNC.__class__.__name__ == "RingAllReduce":
            out = GRAD_SYNC.all_reduce(t, param_id=7)
        else:
            GRAD_SYNC.all_reduce(t)  # in place
            out = t
        with open(os.path.join(os.environ["ZQ_OUT"], f"rank{RANK}.txt"), "w") as f:
            f.write(f"{WORLD_SIZE} {out[0].item()} {DEVICE}")
        return 0
''')


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.distributed
@pytest.mark.parametrize("backend", ["gloo", "ring"])
def test_runner_both_roles_two_workers(tmp_path, backend):
    script = tmp_path / "train.py"
    script.write_text(SCRIPT)
    env = dict(os.environ, ZQ_OUT=str(tmp_path), CUDA_VISIBLE_DEVICES="", PYTHONPATH=ROOT)
    port = _free_port()
    cmd = [sys.executable, os.path.join(ROOT, "run_distributed.py"), "--role", "both",
           "--host", "127.0.0.1", "--gpus", "0,1", "--port", str(port), "--backend", backend,
           "--dist-addr", "127.0.0.1", "--dist-port", str(_free_port()), "--timeout", "60",
           "--script", str(script)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=240)
    assert r.returncode == 0, r.stdout + r.stderr
    got = sorted((tmp_path / f"rank{i}.txt").read_text().split() for i in range(2))
    for world, value, dev in got:
        assert world == "2" and float(value) == 3.0 and dev == "cpu"


def test_runner_dry_run():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "run_distributed.py"), "--dry-run",
                        "--role", "both", "--gpus", "0,1"], capture_output=True, text=True,
                       timeout=120, env=dict(os.environ, PYTHONPATH=ROOT))
    assert r.returncode == 0 and "configuration valid" in r.stdout
