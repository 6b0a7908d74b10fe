"""Multi-GPU group training (eb_engine_join + eb_train) on two GPUs: every
rank's result equals a lone engine's bit for bit. Needs two GPUs; skipped
otherwise. The ranks run as child processes under torch.distributed.run."""

import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def gpu_count():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(gpu_count() < 2, reason="needs two GPUs")
def test_group_training_equals_one_engine():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port()),
           os.path.join(HERE, "_group_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, cwd=os.path.dirname(HERE), env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("group training equals the lone engine") == 2
