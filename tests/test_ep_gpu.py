"""Expert parallelism over NVLink peer memory (hexmoe_ep_*): on every rank the EP
layer equals the plain single-GPU layer bit for bit (tests/ep_gpu_worker.py, one
process per GPU), on two GPUs and, so that a one-GPU run covers the same
kernels, as a single rank.  NCCL only carries the one-time IPC handle
exchange."""

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
    mapped gather, the down GEMM's routed per-slot stores, combine) as a single
    rank: the result equals the single-GPU layer bit for bit."""
    _run_workers(1, 29562)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_ep_bounded_wait_runs_out_and_the_context_recovers():
    """A wait on a flag that nothing sets ends by itself: combine right after
    dispatch (the experts phase that would raise the return flag skipped) gives
    up after its bounded wait (2 s) with the timeout bit in the device error
    word, and the kernels return.  Running the skipped phase then completes the
    same epoch, and the next forward is correct again.  One rank, one GPU."""
    import ctypes
    import sys
    import time
    sys.path.insert(0, str(ROOT / "blackhole-harness_b200"))
    from blackhole_b200 import _lib
    from blackhole_b200 import hex_data as hd
    from blackhole_b200.ep import EPMoE, ExpertShard, shard_tiers
    from blackhole_b200.hex_moe import HexTier, device_status, layer_for

    dev = torch.device("cuda", 0)
    E, H, I, K, T = 8, 256, 256, 2, 24
    L = hd.synth_layer(E, H, I, "mixed", 32, seed=9, device=dev)
    tiers = [HexTier(t["bits"], t["experts"], t["gate_proj"], t["up_proj"], t["down_proj"]).prepare(E)
             for t in shard_tiers(L.tiers, ExpertShard(E, 0, 1))]
    ep = EPMoE(ExpertShard(E, 0, 1), tiers, block_m=16, max_tokens=T, topk=K, hidden=H)
    w, ids = hd.synth_routing(T, E, K, seed=10, device=dev)
    x = hd.synth_x(T, H, seed=11, device=dev)
    device_status(0, clear=True)
    want = ep(x, w, ids)
    assert torch.equal(want, layer_for(tiers).forward(x, w, ids, 16))
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ws = ep._workspace(16)
    out = torch.empty_like(want)
    L_ = _lib.lib
    _lib.check(L_.hexmoe_ep_dispatch(ep._ctx, x.data_ptr(), _lib.BF16, T, w.data_ptr(), ids.data_ptr(), _lib.I64, st))
    t0 = time.monotonic()
    _lib.check(L_.hexmoe_ep_combine(ep._ctx, T, out.data_ptr(), _lib.BF16, st))   # nothing raises the return flag
    torch.cuda.synchronize()
    waited = time.monotonic() - t0
    status = device_status(0, clear=True)
    assert status & 1, f"the wait should have run out (status {status})"
    assert 1.5 < waited < 30, waited
    # the skipped phase completes the epoch; its combine and the next forward are correct
    _lib.check(L_.hexmoe_ep_experts(ep._ctx, ep._layer.handle, 16, ws.data_ptr(), ws.numel(), st))
    _lib.check(L_.hexmoe_ep_combine(ep._ctx, T, out.data_ptr(), _lib.BF16, st))
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    assert torch.equal(ep(x, w, ids), want)
    assert device_status(0, clear=True) == 0
    ep.close()
