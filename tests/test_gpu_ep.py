"""Expert parallelism on 2 GPUs against the single-GPU layer
(tests/ep_worker.py, one process per GPU over NCCL): routing, per-slot expert
outputs and shared outputs bit-identical; combined outputs bit-identical
when both runs use the same router kernel, else within 1e-6 relative.
Skipped with fewer than two GPUs."""
import os
import socket
import subprocess
import sys

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("transport", ["peer", "nccl"])
def test_expert_parallel_matches_single_gpu(transport):
    """peer: rows and outputs as peer-memory stores into fixed slabs (all
    cases). nccl: the same slabs over NCCL for the small cases and the
    host-sized exchange for the large one."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    if transport == "nccl":
        env["HF_EP_NCCL_ONLY"] = "1"
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           f"--master-port={_port()}", os.path.join(HERE, "ep_worker.py")]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True)
    lines = [l for l in p.stdout.splitlines() if l.startswith("EPRESULT")]
    errs = [l for l in (p.stdout + p.stderr).splitlines()
            if "Error" in l or "error" in l or "EPRESULT" in l]
    assert p.returncode == 0, "\n".join(errs[-60:])
    assert len(lines) == 2, p.stdout[-2000:]


def test_expert_parallel_recovery():
    """tests/ep_recovery_worker.py on 2 GPUs (NVLS off): all ranks agree on the
    NCCL transport when one rank cannot map its peers, and a forward skipped by
    one rank ends in HF_ERR_TIMEOUT on the other (bounded waits, 1 ms), after
    which hf_moe_ep_resync on both makes the next forward correct again."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           f"--master-port={_port()}", os.path.join(HERE, "ep_recovery_worker.py")]
    p = subprocess.run(cmd, env=env, capture_output=True, text=True)
    lines = [l for l in p.stdout.splitlines() if l.startswith("EPRECOVERY")]
    errs = [l for l in (p.stdout + p.stderr).splitlines()
            if "Error" in l or "error" in l or "EPRECOVERY" in l]
    assert p.returncode == 0, "\n".join(errs[-60:])
    assert len(lines) == 2, p.stdout[-2000:]
