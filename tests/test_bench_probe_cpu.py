"""bench.py --probe a2a (the NCCL all-to-all comparison of the expert-parallel
dispatch) runs its plumbing on CPU: two gloo ranks, one JSON line from rank 0."""
import json
import os
import socket
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_a2a_probe_on_gloo():
    cmd = ["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           f"--master-port={_port()}", os.path.join(ROOT, "bench.py"), "--probe", "a2a",
           "--probe-mb", "1"]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    p = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [json.loads(l) for l in p.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1 and lines[0]["probe"] == "a2a" and lines[0]["world"] == 2
    assert lines[0]["ms"] > 0
