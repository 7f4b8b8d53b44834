"""Expert parallelism for the HEX MoE layer over a torch.distributed process group.

The reference plugin refuses expert and tensor parallelism
(runtime/blackhole_runtime/vllm_hex.py:101-102) and runs one GPU; this module is
the multi-GPU path for the prefill configs.  Experts are sharded contiguously
over the ranks (rank r owns global experts [r * P, (r + 1) * P), P =
ceil(E / world)) and each rank holds only its experts' HEX tiers.

Forward for the T tokens of this rank (global expert ids in topk_ids):
  1. the S = T * k slots (t, j), grouped by the rank that owns expert
     topk_ids[t, j] (stable, so each rank's slots keep their order);
  2. an all-to-all of the per-rank slot counts, then of the slots' token rows
     (in the activation dtype), expert ids and top-k weights;
  3. the local experts on the received rows: the layer at top-1, each row with
     its own weight, so every row comes back as w * down(silu(gate x) * up x)
     rounded to the activation dtype, exactly as the single-GPU layer rounds
     each slot before its combine;
  4. an all-to-all of those rows back to the ranks they came from;
  5. out[t] = the k returned rows of token t summed in fp32 and rounded (the
     layer's own combine kernel on the GPU).
Each slot goes through the same arithmetic as in the single-GPU layer, so the
result equals the single-GPU output bit for bit (at the same block_m).  Traffic
per rank: 2 x S x H activation rows plus 8 bytes of metadata per slot.

Collectives: plain all-to-alls (NCCL on GPUs).  The first carries each rank's
slot count per destination and its argument-error flag, read on the host once
(the counts set the split lists; a bad call raises on every rank before any
data moves).  Every rank runs the same collectives in the same order, including
ranks with no tokens and calls that end in an argument error.  On the GPU the
local experts run as the layer's phases without its top-1 combine, and the
returned rows are summed in slot order through a row map (hexmoe_combine_rows)
instead of being copied back into slot order first.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist

PROJ = ("gate_proj", "up_proj", "down_proj")


@dataclass(frozen=True)
class ExpertShard:
    """Which global experts a rank owns."""
    num_experts: int
    rank: int
    world: int

    @property
    def per_rank(self) -> int:
        return -(-self.num_experts // self.world)

    @property
    def local_range(self) -> tuple[int, int]:
        lo = min(self.rank * self.per_rank, self.num_experts)
        return lo, min(lo + self.per_rank, self.num_experts)

    def owner(self, ids: torch.Tensor) -> torch.Tensor:
        return torch.div(ids, self.per_rank, rounding_mode="floor")


def shard_tiers(tiers: list, shard: ExpertShard) -> list:
    """The tiers restricted to this rank's experts (tier dicts of the HEX parts, or
    unprepared HexTier objects): every part stacked over experts keeps only the
    local experts' slices, in the same order; tiers with none are dropped."""
    lo, hi = shard.local_range
    out = []
    for t in tiers:
        is_dict = isinstance(t, dict)
        experts = torch.as_tensor(t["experts"] if is_dict else t.experts)
        keep = torch.nonzero((experts >= lo) & (experts < hi)).flatten()
        if keep.numel() == 0:
            continue
        projs = {p: {q: torch.as_tensor(v).index_select(0, keep.to(torch.as_tensor(v).device))
                     for q, v in (t[p] if is_dict else getattr(t, p)).items()} for p in PROJ}
        ex = experts.index_select(0, keep)
        if is_dict:
            out.append({"bits": t["bits"], "experts": ex, **projs})
        else:
            out.append(type(t)(t.bits, ex, projs["gate_proj"], projs["up_proj"], projs["down_proj"]))
    return out


ExpertFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]
CombineFn = Callable[[torch.Tensor, int, int], torch.Tensor]


def _sum_combine(y: torch.Tensor, T: int, k: int) -> torch.Tensor:
    """The combine of the CUDA layer on any device: slots added in order in fp32."""
    yv = y.view(T, k, -1)
    acc = yv[:, 0].float()
    for j in range(1, k):
        acc = acc + yv[:, j].float()
    return acc.to(y.dtype)


class EPMoE:
    """The HEX MoE layer with experts sharded over `group`.

    local_tiers: this rank's prepared HexTier list (from shard_tiers(...) then
    HexTier.prepare(num_experts)); expert_fn / combine_fn replace the CUDA layer
    (tests run the host logic on CPU ranks with the oracle as expert_fn).
    block_m: tile height of the local layer (0 = by the received slot count).
    The down GEMM's accumulation order depends on it (two accumulators for
    block_m <= 64), so EP equals a single-GPU run bit for bit at the same block_m."""

    def __init__(self, shard: ExpertShard, local_tiers: list | None = None, group=None,
                 expert_fn: ExpertFn | None = None, combine_fn: CombineFn | None = None, block_m: int = 0):
        self.shard = shard
        self.block_m = block_m
        self.group = group
        self.local_tiers = local_tiers
        self._layer = None
        self._cuda = expert_fn is None        # the CUDA layer (else injected functions, e.g. on CPU ranks)
        if expert_fn is None:
            if local_tiers is None:
                raise ValueError("EPMoE needs the local tiers or an expert_fn")
            from blackhole_b200.hex_moe import layer_for
            # a rank may own no experts (more ranks than experts allow): it only
            # sends its tokens out and combines what comes back
            self._layer = layer_for(local_tiers) if local_tiers else None
            expert_fn = self._local_phases
        self.expert_fn = expert_fn
        self.combine_fn = combine_fn or _sum_combine

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int]) -> None:
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def _by_owner(self, owner: torch.Tensor) -> torch.Tensor:
        """Slot ids ordered by owner rank, stable (slots of one rank keep their
        order): on the GPU the layer's own align with the ranks as the experts and
        runs of one slot, elsewhere a stable sort (the same order)."""
        if owner.is_cuda and owner.numel():
            from blackhole_b200.hex_moe import align
            sid, _, _ = align(owner.to(torch.int32), self.shard.world, 1)
            return sid[:owner.numel()].to(torch.int64)
        return torch.argsort(owner, stable=True)

    def _local_phases(self, xr: torch.Tensor, wr: torch.Tensor, ir: torch.Tensor) -> torch.Tensor:
        """The local experts on the received rows, one slot per row: the layer
        forward up to the per-slot rows (weighted, rounded to the activation
        dtype) in one call, so the layer's top-1 combine (a copy) is skipped."""
        n = xr.shape[0]
        return self._layer.forward_slots(xr, wr.reshape(n, 1), ir.reshape(n, 1), self.block_m)

    def forward(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
        if x.dim() != 2 or topk_ids.dim() != 2 or topk_weights.shape != topk_ids.shape or x.shape[0] != topk_ids.shape[0]:
            raise ValueError("x [T, H], topk_weights and topk_ids [T, k] expected")
        T, k = topk_ids.shape
        H = x.shape[1]
        dev = x.device
        world, E = self.shard.world, self.shard.num_experts
        ids = topk_ids.reshape(-1).to(torch.int64)
        w = topk_weights.reshape(-1).to(torch.float32)
        # 1. per destination rank: slot count and this rank's argument-error flag,
        #    exchanged in one all-to-all and read on the host once, so a bad call
        #    fails on every rank before any data moves
        bad = ((ids < 0) | (ids >= E)).any().to(torch.int64)
        owner = self.shard.owner(ids.clamp(0, max(E - 1, 0)))
        # (torch.bincount would read its input's maximum on the host: a second sync)
        send_counts = (owner.unsqueeze(1) == torch.arange(world, device=dev)).sum(0, dtype=torch.int64)
        info = torch.stack([send_counts, bad.expand(world)], 1).contiguous()
        recv_info = torch.empty_like(info)
        dist.all_to_all_single(recv_info, info, group=self.group)
        host = torch.cat([send_counts, recv_info.reshape(-1)]).tolist()
        sc, rc, flags = host[:world], host[world::2], host[world + 1::2]
        if any(flags):
            mine = flags[dist.get_rank(self.group)]
            raise ValueError("topk_ids out of range" if mine else "topk_ids out of range on another rank")
        n_recv = sum(rc)
        order = self._by_owner(owner)
        # 2. token rows, ids and weights of the slots, grouped by owner
        send_x = x.index_select(0, torch.div(order, k, rounding_mode="floor"))
        recv_x = torch.empty(n_recv, H, dtype=x.dtype, device=dev)
        self._a2a(recv_x, send_x, rc, sc)
        # expert id (high word) and top-k weight bits (low word) of each slot, one int64
        meta = ((ids << 32) | (w.view(torch.int32).to(torch.int64) & 0xFFFFFFFF)).index_select(0, order)
        recv_meta = torch.empty(n_recv, dtype=torch.int64, device=dev)
        self._a2a(recv_meta, meta, rc, sc)
        recv_ids = (recv_meta >> 32).to(torch.int32)
        recv_w = (recv_meta & 0xFFFFFFFF).to(torch.int32).view(torch.float32)
        # 3. local experts, one slot per row
        out_dt = x.dtype if x.dtype in (torch.bfloat16, torch.float16) else torch.bfloat16
        if n_recv:
            if self._cuda and self._layer is None:
                raise RuntimeError("slots were routed to a rank that holds no experts")
            y_recv = self.expert_fn(recv_x, recv_w, recv_ids).to(out_dt).contiguous()
        else:
            y_recv = torch.empty(0, H, dtype=out_dt, device=dev)
        # 4. rows back to their source rank, in the order they were sent
        back = torch.empty(T * k, H, dtype=out_dt, device=dev)
        self._a2a(back, y_recv, sc, rc)
        if T == 0:
            return torch.empty(0, H, dtype=x.dtype, device=dev)
        # 5. combine the k slots of each token: slot order[i] came back as row i
        if self._cuda:
            from blackhole_b200.hex_moe import combine_rows
            rows = torch.empty(T * k, dtype=torch.int32, device=dev)
            rows.index_copy_(0, order, torch.arange(T * k, dtype=torch.int32, device=dev))
            return combine_rows(back, T, k, rows, out_dtype=x.dtype)
        y = torch.empty_like(back)
        y.index_copy_(0, order, back)
        return self.combine_fn(y, T, k).to(x.dtype)

    __call__ = forward
