"""Tensor-parallel Dream path on 2 (and, where present, 4 and 8) GPUs: one process per GPU through
torch.distributed.run, NCCL all-reduce of the o_proj / down_proj partials. The checks run in
tp_worker.py; this wrapper launches the group under a hard timeout and reports its output."""
from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_dream_matches_whole_model(world):
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
           str(ROOT / "tests" / "tp_worker.py")]
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    proc = subprocess.run(cmd, cwd=str(ROOT), env=env, capture_output=True, text=True)
    print(proc.stdout[-4000:])
    print(proc.stderr[-4000:])
    assert proc.returncode == 0
