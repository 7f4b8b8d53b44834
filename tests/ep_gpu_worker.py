"""One rank of the multi-GPU expert-parallel check (launched by test_ep_gpu.py with
torchrun, one process per GPU, NCCL): the EP layer on this rank's tokens must equal
the single-GPU layer on the same tokens bit for bit.  Prints "EP-OK <rank> ..." on
success."""

from __future__ import annotations

import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT / "blackhole-harness_b200")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main() -> int:
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    try:
        from blackhole_b200 import hex_data as hd
        from blackhole_b200.ep import EPMoE, ExpertShard, shard_tiers
        from blackhole_b200.hex_moe import HexTier, hex_moe

        E, H, I, K = 16, 512, 256, 4
        L = hd.synth_layer(E, H, I, "mixed", 128, seed=5, device=dev)
        mk = lambda ts: [HexTier(t["bits"], t["experts"], t["gate_proj"], t["up_proj"], t["down_proj"]).prepare(E)  # noqa: E731
                         for t in ts]
        full = mk(L.tiers)
        shard = ExpertShard(E, rank, world)
        ep = EPMoE(shard, mk(shard_tiers(L.tiers, shard)), block_m=16)
        for T, zipf in ((48 + 16 * rank, None), (96, 1.2), (0 if rank == world - 1 else 8, None)):
            w, ids = hd.synth_routing(T, E, K, seed=11 + rank, zipf=zipf, device=dev)
            x = hd.synth_x(T, H, seed=21 + rank, device=dev)
            got = ep(x, w, ids)
            # the single-GPU layer, one slot per row (the EP path's arithmetic), then the same combine
            want_slots = hex_moe(x.repeat_interleave(K, 0), w.reshape(-1, 1), ids.reshape(-1, 1), full,
                                 {"BLOCK_M": 16})
            want = ep.combine_fn(want_slots, T, K) if T else want_slots
            torch.cuda.synchronize()
            if not torch.equal(got, want):
                print(f"EP-MISMATCH rank {rank} T={T} max diff {(got.float() - want.float()).abs().max().item()}",
                      flush=True)
                return 1
            ref = hex_moe(x, w, ids, full)          # the plain single-GPU layer: same up to combine order
            if T and not torch.allclose(got.float(), ref.float(), rtol=2e-2, atol=1e-2):
                print(f"EP-TOL rank {rank} T={T}", flush=True)
                return 1
        print(f"EP-OK {rank} of {world}", flush=True)
        return 0
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
