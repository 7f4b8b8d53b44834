"""Expert parallelism over NVLink peer memory (hexmoe_ep_*): on every rank the EP
layer equals the single-GPU layer's per-slot rows put through the EP combine, bit
for bit (tests/ep_gpu_worker.py, one process per GPU), on two GPUs and, so that a
one-GPU run covers the same kernels, as a single rank (which must equal the plain
layer bit for bit).  NCCL only carries the one-time IPC handle exchange."""

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
    """The expert-parallel kernels (plan, dispatch to itself, ragged align and
    mapped gather, pre-summed return, combine) as a single rank: the result
    equals the single-GPU layer bit for bit."""
    _run_workers(1, 29562)
