"""Row-sharded tensor parallelism on 2+ GPUs: one rank per GPU over NCCL
(tests/tp_gpu_worker.py), assembled outputs against the unsharded oracle.
Skipped when fewer than two GPUs are visible (the single-GPU suite covers the
kernel itself)."""

import os
import socket
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.gpu
def test_tp_sharded_plan_matches_oracle(cuda):
    import torch

    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two or more GPUs")
    world = 8 if n >= 8 else (4 if n >= 4 else 2)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(HERE, "tp_gpu_worker.py")]
    r = subprocess.run(cmd, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    assert r.returncode == 0, r.stdout[-4000:]
    assert f"tp parity world={world}: ok" in r.stdout
