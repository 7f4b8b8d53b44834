"""Expert parallelism over NCCL: the EP layer equals the single-GPU layer bit for
bit on every rank (tests/ep_gpu_worker.py, one process per GPU), on two GPUs and,
so that a one-GPU run covers the same code, as a single rank."""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _run_workers(n: int, port: int) -> None:
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr", "127.0.0.1", "--master-port", str(port),
           str(ROOT / "tests" / "ep_gpu_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-3000:]
    for rank in range(n):
        assert f"EP-OK {rank} of {n}" in out, out[-3000:]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_two_gpus_matches_single_gpu():
    _run_workers(2, 29561)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_ep_one_rank_matches_single_gpu():
    """The CUDA expert-parallel path (owner grouping by the align kernel, the
    per-slot forward, the row-mapped combine) in a one-rank NCCL group: every
    all-to-all is a copy to itself, and the result equals the layer bit for bit."""
    _run_workers(1, 29562)
