"""One rank of the multi-GPU expert-parallel check (launched by test_ep_gpu.py with
torchrun, one process per GPU).  The hexmoe_ep_* path (peer-memory dispatch,
local experts whose down GEMM stores every slot's row into its source rank's
buffer, the single-GPU combine) on this rank's tokens must equal the plain
single-GPU layer bit for bit at every world size, with the tcgen05 GEMM (tile
height 16) and with the small-batch kernel (tile height 8).  A CUDA-graph
replay of the EP forward must give the eager result.  Prints "EP-OK <rank> of
<world>" on success."""

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
    ep = None
    try:
        from blackhole_b200 import hex_data as hd
        from blackhole_b200.ep import EPMoE, ExpertShard, reference_combine, shard_tiers
        from blackhole_b200.hex_moe import HexTier, device_status, layer_for

        device_status(local, clear=True)
        E, H, I, K, BM = 16, 512, 256, 4, 16
        L = hd.synth_layer(E, H, I, "mixed", 128, seed=5, device=dev)
        mk = lambda ts: [HexTier(t["bits"], t["experts"], t["gate_proj"], t["up_proj"], t["down_proj"]).prepare(E)  # noqa: E731
                         for t in ts]
        full = layer_for(mk(L.tiers))
        shard = ExpertShard(E, rank, world)
        # tile height 8: the small-batch kernel picks its tile height (and so the
        # order of its fp32 step-group sums) from the tile count; from 264 tokens
        # at top-4 on up both this rank's single-GPU call and the EP slot space
        # take the tallest tiles, so the two agree bit for bit
        ep8 = EPMoE(shard, mk(shard_tiers(L.tiers, shard)), block_m=8, max_tokens=320, topk=K, hidden=H)
        try:
            for T in (264 + 8 * rank, 320):
                w, ids = hd.synth_routing(T, E, K, seed=31 + rank + T, device=dev)
                x = hd.synth_x(T, H, seed=41 + rank + T, device=dev)
                got = ep8(x, w, ids)
                ref = full.forward(x, w, ids, 8)
                if not torch.equal(got, ref):
                    print(f"EP-MISMATCH-BM8 rank {rank} T={T} max diff {(got.float() - ref.float()).abs().max().item()}",
                          flush=True)
                    return 1
        finally:
            ep8.close()
        ep = EPMoE(shard, mk(shard_tiers(L.tiers, shard)), block_m=BM, max_tokens=128, topk=K, hidden=H)
        cases = ((48 + 16 * rank, None), (96, 1.2), (0 if rank == world - 1 else 8, None), (128, None))
        for T, zipf in cases:
            w, ids = hd.synth_routing(T, E, K, seed=11 + rank + T, zipf=zipf, device=dev)
            x = hd.synth_x(T, H, seed=21 + rank + T, device=dev)
            got = ep(x, w, ids)
            torch.cuda.synchronize()
            if T == 0:
                if got.shape != (0, H):
                    print(f"EP-SHAPE rank {rank}", flush=True)
                    return 1
                continue
            y = full.forward_slots(x, w, ids, BM)
            want = reference_combine(y, ids, shard, x.dtype)
            ref = full.forward(x, w, ids, BM)       # the plain single-GPU layer
            if not (torch.equal(got, want) and torch.equal(got, ref)):
                print(f"EP-MISMATCH rank {rank} T={T} max diff {(got.float() - ref.float()).abs().max().item()}",
                      flush=True)
                return 1
        # the EP forward captured in a CUDA graph (no host synchronisation inside)
        T = 64
        w, ids = hd.synth_routing(T, E, K, seed=77 + rank, device=dev)
        x = hd.synth_x(T, H, seed=78 + rank, device=dev)
        eager = ep(x, w, ids)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ep(x, w, ids)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = ep(x, w, ids)
        for _ in range(2):
            g.replay()
            torch.cuda.synchronize()
            if not torch.equal(out, eager):
                print(f"EP-GRAPH rank {rank}", flush=True)
                return 1
        del g
        err = device_status(local, clear=True)
        if err:
            print(f"EP-DEVERR rank {rank} word {err}", flush=True)
            return 1
        print(f"EP-OK {rank} of {world}", flush=True)
        return 0
    finally:
        if ep is not None:
            ep.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
