"""Tensor parallelism on 2 GPUs against the single-GPU model (runs
tests/tp_check.py with one process per GPU; skipped with fewer than 2 GPUs),
once with the peer-memory exchange and once with NCCL for every exchange."""
import socket
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _gpus():
    import torch

    return torch.cuda.device_count()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("mode", ["peer", "nccl"])
@pytest.mark.parametrize("name", ["llama_q8", "qwen2_mix"])
def test_tensor_parallel_matches_single_gpu(tmp_path, name, mode):
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    cmd = ["timeout", "-k", "30", "540", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           str(ROOT / "tests" / "tp_check.py"), name, str(tmp_path / f"{name}.gguf")]
    r = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, env={**__import__("os").environ,
                                                                          "NCCL_NVLS_ENABLE": "0",
                                                                          "PRANA_TP_ALLREDUCE": mode})
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
