"""Multi-GPU parity tests, run as child processes under torchrun (one process per GPU) when the box has at least
two GPUs; skipped otherwise. NVLS is off in NCCL for these runs (NCCL_NVLS_ENABLE=0)."""

import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _ngpu():
    import torch
    return torch.cuda.device_count()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _torchrun(script, n, *args, timeout=600):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", TORCH_NCCL_ASYNC_ERROR_HANDLING="1")
    cmd = ["timeout", "-k", "60", str(timeout), sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", f"--master-port={_port()}", os.path.join(HERE, script),
           *args]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    return r.returncode, r.stdout + r.stderr


@pytest.mark.parametrize("n", [2])
def test_lm_head_row_split_argmax(n):
    if _ngpu() < n:
        pytest.skip(f"needs {n} GPUs")
    rc, out = _torchrun("mgpu_lm_head.py", n, "--fail-test")
    assert rc == 0, out[-4000:]
    assert '"failures": 0' in out and '"failure_test": "ok"' in out, out[-4000:]


@pytest.mark.parametrize("n", [2])
def test_moe_expert_parallel(n):
    if _ngpu() < n:
        pytest.skip(f"needs {n} GPUs")
    rc, out = _torchrun("mgpu_moe.py", n, "--fail-test")
    assert rc == 0, out[-4000:]
    assert '"failures": 0' in out and '"failure_test": "ok"' in out, out[-4000:]
