"""Expert parallelism (blackhole_b200.ep) on CPU ranks over gloo, world sizes 2, 3,
5 and 8, with the C oracle standing in for each rank's local experts.

The reference has no multi-GPU path (its plugin refuses expert parallelism), so
the bar is the single-process computation: every slot computed alone at top-1
and rounded to the activation dtype (as the single-GPU layer's per-slot rows),
then per token the fp32 sum of its slots in top-k order rounded once (the
single-GPU layer's combine, ep.reference_combine).  EP must reproduce that bit
for bit at every world size, and the oracle's moe_reference within the layer
tolerance.  The same host protocol (one row per token and destination rank out,
one row per slot back) is what the hexmoe_ep_* kernels run on GPUs.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from helpers import np_tiers, rel_err, within

E, H, I, K, BLOCK = 12, 256, 128, 4, 32


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(seed=3):
    from blackhole_b200 import hex_data as hd
    return hd.synth_layer(E, H, I, "mixed", BLOCK, seed=seed)


def _tokens(rank: int, T: int, zipf=None):
    from blackhole_b200 import hex_data as hd
    w, ids = hd.synth_routing(T, E, K, seed=100 + rank, zipf=zipf)
    x = hd.synth_x(T, H, seed=200 + rank)
    return x, w, ids


def _per_slot_rows(x, w, ids, tiers_np) -> torch.Tensor:
    """Every slot alone at top-1 (weighted, rounded to bf16): the single-GPU
    layer's per-slot rows [T * k, H], in one process."""
    import hexoracle
    T, k = ids.shape
    layer = hexoracle.Layer(tiers_np, E, H, I, BLOCK)
    xs = np.repeat(x.float().numpy(), k, axis=0)
    y = layer.forward(xs, w.reshape(-1, 1).numpy(), ids.reshape(-1, 1).numpy())
    return torch.from_numpy(hexoracle.round_bf16(y)).to(torch.bfloat16)


def _worker(rank: int, world: int, port: int, T_of, zipf, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import hexoracle

        from blackhole_b200.ep import EPMoE, ExpertShard, shard_tiers
        shard = ExpertShard(E, rank, world)
        L = _layer()
        local_np = np_tiers(shard_tiers(L.tiers, shard))
        local = hexoracle.Layer(local_np, E, H, I, BLOCK) if local_np else None
        lo, hi = shard.local_range

        def expert_fn(xr, wr, ir):
            assert int(ir.min()) >= lo and int(ir.max()) < hi, "slot routed to a rank that does not own it"
            y = local.forward(xr.float().numpy(), wr.reshape(-1, 1).numpy(), ir.reshape(-1, 1).numpy())
            return torch.from_numpy(hexoracle.round_bf16(y)).to(torch.bfloat16)

        ep = EPMoE(shard, expert_fn=expert_fn)
        x, w, ids = _tokens(rank, T_of[rank], zipf)
        out = ep(x, w, ids)
        out_q.put((rank, out.float().numpy()))
    except BaseException as e:  # noqa: BLE001
        out_q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def _run(world: int, T_of: list[int], zipf=None) -> dict:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, T_of, zipf, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, val = q.get(timeout=240)
        res[rank] = val
    for p in procs:
        p.join(timeout=60)
    for r, v in res.items():
        assert not isinstance(v, str), f"rank {r} failed: {v}"
    return res


@pytest.mark.parametrize("world,T_of,zipf", [
    (2, [24, 17], None),
    (3, [16, 0, 9], 1.2),          # a rank with no tokens; skewed routing
    (5, [7, 5, 0, 3, 6], None),    # E=12 over 5 ranks: rank 4 owns no experts
    (8, [4, 3, 5, 0, 2, 6, 1, 3], 1.2),   # eight ranks, as on one B200 node: ranks 6 and 7 own none
])
def test_ep_matches_single_process(oracle, world, T_of, zipf):
    res = _run(world, T_of, zipf)
    L = _layer()
    full_np = np_tiers(L.tiers)
    for r in range(world):
        x, w, ids = _tokens(r, T_of[r], zipf)
        got = res[r]
        assert got.shape == (T_of[r], H)
        if T_of[r] == 0:
            continue
        from blackhole_b200.ep import ExpertShard, reference_combine
        per_slot = reference_combine(_per_slot_rows(x, w, ids, full_np), ids, ExpertShard(E, r, world),
                                     torch.bfloat16).float().numpy()
        assert np.array_equal(got, per_slot), rel_err(got, per_slot)
        want = oracle.moe_reference(x.float().numpy(), w.numpy(), ids.numpy(), full_np, E, BLOCK)
        assert within(got, want), rel_err(got, want)


def _bad_id_worker(rank: int, world: int, port: int, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from blackhole_b200.ep import EPMoE, ExpertShard
        ep = EPMoE(ExpertShard(E, rank, world), expert_fn=lambda xr, wr, ir: xr)
        x, w, ids = _tokens(rank, 6)
        if rank == 1:
            ids = ids.clone()
            ids[2, 1] = E                      # out of range on this rank only
        try:
            ep(x, w, ids)
            out_q.put((rank, "no error"))
        except ValueError as e:
            out_q.put((rank, str(e)))
    finally:
        dist.destroy_process_group()


def test_out_of_range_id_raises_on_every_rank():
    """On CPU ranks a bad expert id on one rank ends the call with ValueError on
    every rank, before any token row moves (the flag rides on the count
    exchange).  The GPU path has no host exchange: it drops the slot and sets
    the device error word."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_bad_id_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "topk_ids out of range"
    assert res[0] == "topk_ids out of range on another rank"


def test_shard_tiers_partition_the_experts():
    from blackhole_b200.ep import ExpertShard, shard_tiers
    L = _layer()
    for world in (1, 2, 3, 5):
        seen = []
        for r in range(world):
            sh = ExpertShard(E, r, world)
            lo, hi = sh.local_range
            for t in shard_tiers(L.tiers, sh):
                ex = t["experts"].tolist()
                assert all(lo <= e < hi for e in ex)
                full = next(ft for ft in L.tiers if ft["bits"] == t["bits"])
                pos = [full["experts"].tolist().index(e) for e in ex]
                for p in ("gate_proj", "up_proj", "down_proj"):
                    for q in ("idx", "block_scale", "expert_scale", "levels"):
                        assert torch.equal(t[p][q], full[p][q][pos])
                seen += ex
        assert sorted(seen) == list(range(E))


def test_expert_shard_ownership():
    from blackhole_b200.ep import ExpertShard
    sh = ExpertShard(96, 3, 8)
    assert sh.per_rank == 12 and sh.local_range == (36, 48)
    assert sh.owner(torch.tensor([0, 11, 12, 95])).tolist() == [0, 0, 1, 7]
    sh = ExpertShard(10, 3, 4)                 # uneven: 3, 3, 3, 1
    assert sh.local_range == (9, 10)


def test_plan_dispatch_rows_and_slots():
    """One row per (token, owner rank) in token order; slots in (token, j) order."""
    from blackhole_b200.ep import ExpertShard, plan_dispatch
    ids = torch.tensor([[0, 5, 1], [7, 6, 2], [3, 4, 5]])        # E=8 over 4 ranks: 2 experts each
    p = plan_dispatch(ids, ExpertShard(8, 0, 4))
    assert [r.tolist() for r in p.rows] == [[0], [1, 2], [0, 2], [1]]
    assert p.pos.tolist() == [[0, -1, 0, -1], [-1, 0, -1, 0], [-1, 1, 1, -1]]
    assert [list(zip(t.tolist(), j.tolist())) for t, j in p.slots] == [
        [(0, 0), (0, 2)], [(1, 2), (2, 0)], [(0, 1), (2, 1), (2, 2)], [(1, 0), (1, 1)]]


@pytest.mark.parametrize("world", [1, 3, 8])
def test_reference_combine_is_the_layer_combine(world):
    """At any world size the EP combine is the single-GPU combine (slots in j
    order, fp32, rounded once)."""
    from blackhole_b200.ep import ExpertShard, reference_combine
    g = torch.Generator().manual_seed(3)
    T, k = 9, 4
    y = torch.randn(T * k, 16, generator=g).to(torch.bfloat16)
    ids = torch.randint(0, 12, (T, k), generator=g)
    want = y.view(T, k, 16).float()
    acc = want[:, 0]
    for j in range(1, k):
        acc = acc + want[:, j]
    got = reference_combine(y, ids, ExpertShard(12, world - 1, world), torch.bfloat16)
    assert torch.equal(got, acc.to(torch.bfloat16))


def _leaving_worker(rank: int, world: int, port: int, out_q):
    """Rank 1 takes part in one forward and then leaves (exits between steps);
    rank 0's next forward must fail with an error, not hang."""
    import time
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    from blackhole_b200.ep import EPMoE, ExpertShard
    ep = EPMoE(ExpertShard(E, rank, world), expert_fn=lambda xr, wr, ir: xr)
    x, w, ids = _tokens(rank, 6)
    ep(x, w, ids)
    if rank == 1:
        out_q.put((rank, "left"))
        out_q.close()
        out_q.join_thread()             # the message is out; then no goodbye: the process is simply gone
        os._exit(0)
    t0 = time.monotonic()
    try:
        ep(x, w, ids)
        out_q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001  (gloo raises RuntimeError subclasses)
        out_q.put((rank, f"raised after {time.monotonic() - t0:.1f}s: {type(e).__name__}"))
    out_q.close()
    out_q.join_thread()
    os._exit(0)


def test_rank_that_leaves_fails_the_others_within_the_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=30)
    assert res[1] == "left"
    assert res[0].startswith("raised after"), res[0]
    assert float(res[0].split()[2].rstrip("s:")) < 60


def _mismatch_worker(rank: int, world: int, port: int, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from blackhole_b200.ep import EPMoE, ExpertShard
        ep = EPMoE(ExpertShard(E, rank, world), expert_fn=lambda xr, wr, ir: xr)
        x, w, ids = _tokens(rank, 5)
        if rank == 1:
            x = x[:, : H // 2].contiguous()          # this rank's rows are narrower than everyone else's
        try:
            ep(x, w, ids)
            out_q.put((rank, "no error"))
        except ValueError as e:
            out_q.put((rank, str(e)))
    finally:
        dist.destroy_process_group()


def test_ranks_that_disagree_on_shapes_raise_on_every_rank():
    """A rank whose rows have another width fails the call on every rank, in the
    count exchange, before any row moves."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_mismatch_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert all(v.startswith("ranks disagree on hidden / topk") for v in res.values()), res
