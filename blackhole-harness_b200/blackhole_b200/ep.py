"""Expert parallelism for the HEX MoE layer: experts sharded over the ranks of one node.

The reference plugin refuses expert and tensor parallelism
(runtime/blackhole_runtime/vllm_hex.py:101-102) and runs one GPU; this module is
the multi-GPU path for the prefill configs.  Experts are sharded contiguously
over the ranks (rank r owns global experts [r * P, (r + 1) * P), P =
ceil(E / world)) and each rank holds only its experts' HEX tiers.

Forward for the T tokens of this rank (global expert ids in topk_ids):
  1. dispatch: each token row goes once to every rank that owns at least one
     of its k experts (not once per slot), with one record per slot (row,
     expert, top-k weight) in the token's j order;
  2. experts: each rank runs its experts on the received slots, one slot per
     row at top-1, giving w * down(silu(gate x) * up x) rounded to the row
     dtype per slot, exactly as the single-GPU layer rounds each slot;
  3. return: every slot's row goes back to its source rank, to the place of
     slot (t, j) there;
  4. combine: out[t] = the k slot rows of token t summed in j order in fp32,
     rounded once: the single-GPU layer's combine.
So the output equals the single-GPU layer's bit for bit, for any number of
ranks.

On GPUs (EPMoE with local tiers) the four steps are the library's hexmoe_ep_*
kernels over CUDA-IPC peer memory: stores straight into the owner's region over
NVLink (the return from the down GEMM's own epilogue; the token rows pulled by
their owners from the source's region), epoch flags instead of host
synchronisation, so a forward can be captured in a CUDA graph.  The only collective on the host is the one-time
exchange of the IPC handles at construction.  An expert id outside 0..E-1 is
dropped and sets the device error word (hexmoe_device_status) on the GPU path.

On CPU ranks (EPMoE with an expert_fn, e.g. the oracle over gloo in the tests)
the same protocol runs over torch all-to-alls with the counts read on the host;
there a bad expert id raises ValueError on every rank before any row moves.
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


@dataclass
class DispatchPlan:
    """Where this rank's tokens go (the host form of the device plan).

    pos[t, d]   row position of token t in the list sent to rank d, -1 = none
    rows[d]     tokens sent to rank d, in token order
    slots[d]    (token, j) of the slots sent to rank d, ordered by (token, j)
    """
    pos: torch.Tensor
    rows: list
    slots: list


def plan_dispatch(ids: torch.Tensor, shard: ExpertShard) -> DispatchPlan:
    """Rows and slots per destination rank, stable in token order and j order
    (what ep_plan_kernel computes on the device).  ids: valid global ids [T, k]."""
    T, k = ids.shape
    owner = shard.owner(ids)                                          # [T, k]
    pos = torch.full((T, shard.world), -1, dtype=torch.int64)
    rows, slots = [], []
    for d in range(shard.world):
        mine = owner == d                                             # [T, k]
        has = mine.any(1)
        tok = torch.nonzero(has).flatten()
        pos[tok, d] = torch.arange(tok.numel())
        rows.append(tok)
        t_idx, j_idx = torch.nonzero(mine, as_tuple=True)             # row-major: (t, j) order
        slots.append((t_idx, j_idx))
    return DispatchPlan(pos, rows, slots)


def _row_dtype(dt: torch.dtype) -> torch.dtype:
    return dt if dt in (torch.bfloat16, torch.float16) else torch.bfloat16


class EPMoE:
    """The HEX MoE layer with experts sharded over `group` (one rank per GPU).

    GPU path: local_tiers is this rank's prepared HexTier list (from
    shard_tiers(...) then HexTier.prepare(num_experts)); an empty list on a rank
    that owns no experts.  max_tokens, topk and hidden fix the shared buffers at
    construction (every rank must pass the same values: the buffers of all
    ranks have one layout); construction exchanges the IPC handles over `group`
    and so is collective.  Then every rank must make the same sequence of
    forward calls.  close() (collective) frees the buffers.

    CPU path: expert_fn(x_rows, weights, ids) -> per-slot rows (rounded to the
    row dtype) replaces the local layer; the protocol runs over torch
    all-to-alls (the tests run it on gloo ranks with the oracle as expert_fn).
    block_m: tile height of the local layer (0 = automatic)."""

    def __init__(self, shard: ExpertShard, local_tiers: list | None = None, group=None,
                 expert_fn: ExpertFn | None = None, block_m: int = 0, max_tokens: int = 4096, topk: int = 8,
                 hidden: int | None = None, row_dtype: torch.dtype = torch.bfloat16):
        self.shard = shard
        self.block_m = block_m
        self.group = group
        self.expert_fn = expert_fn
        self.local_tiers = local_tiers
        self._ctx = None
        self._ws = {}
        self._layer = None
        if expert_fn is not None:
            return
        if local_tiers is None:
            raise ValueError("EPMoE needs the local tiers (possibly empty) or an expert_fn")
        from blackhole_b200 import _lib
        from blackhole_b200.hex_moe import layer_for
        self._lib = _lib
        if local_tiers:
            self._layer = layer_for(local_tiers)
            if hidden is not None and hidden != self._layer.H:
                raise ValueError(f"hidden {hidden} differs from the local tiers' {self._layer.H}")
            hidden = self._layer.H
            self.device = self._layer.device
        else:
            if hidden is None:
                raise ValueError("a rank without experts must be given `hidden`")
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.hidden, self.topk, self.max_tokens = int(hidden), int(topk), int(max_tokens)
        if row_dtype not in (torch.bfloat16, torch.float16):
            raise ValueError("rows travel as bf16 or fp16")
        self.row_dtype = row_dtype
        import ctypes
        h = ctypes.c_void_p()
        rdt = _lib.BF16 if row_dtype == torch.bfloat16 else _lib.F16
        with torch.cuda.device(self.device):
            _lib.check(_lib.lib.hexmoe_ep_init(shard.rank, shard.world, shard.num_experts, self.hidden, self.topk,
                                               self.max_tokens, rdt, ctypes.byref(h)), "hexmoe_ep_init")
            self._ctx = h
            if shard.world > 1:
                # every rank must build the same buffer layout: agree on it before mapping anything
                on_dev = dist.get_backend(group) == "nccl"
                cfg = torch.tensor([self.max_tokens, self.topk, self.hidden, rdt, shard.num_experts],
                                   dtype=torch.int64)
                cfg_t = cfg.to(self.device) if on_dev else cfg
                cfgs = [torch.empty_like(cfg_t) for _ in range(shard.world)]
                dist.all_gather(cfgs, cfg_t, group=group)
                if any(not torch.equal(c.cpu(), cfg) for c in cfgs):
                    _lib.lib.hexmoe_ep_destroy(h)
                    self._ctx = None
                    raise ValueError("EPMoE: ranks disagree on max_tokens / topk / hidden / row dtype / experts: "
                                     f"{[c.cpu().tolist() for c in cfgs]}")
                mine = torch.empty(_lib.EP_HANDLE_BYTES, dtype=torch.uint8)
                _lib.check(_lib.lib.hexmoe_ep_handle(h, mine.data_ptr()), "hexmoe_ep_handle")
                t = mine.to(self.device) if on_dev else mine
                got = [torch.empty_like(t) for _ in range(shard.world)]
                dist.all_gather(got, t, group=group)
                allh = torch.cat([g.cpu() for g in got]).contiguous()
                _lib.check(_lib.lib.hexmoe_ep_connect(h, allh.data_ptr()), "hexmoe_ep_connect")

    # ------------------------------------------------------------------ GPU
    def _workspace(self, bm: int) -> torch.Tensor | None:
        if self._layer is None:
            return None
        ws = self._ws.get(bm)
        if ws is None:
            n = self._lib.lib.hexmoe_ep_workspace_bytes(self._ctx, self._layer.handle, bm)
            ws = self._ws[bm] = torch.empty(n, dtype=torch.uint8, device=self.device)
        return ws

    def _forward_device(self, x: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, events=None) -> torch.Tensor:
        _lib = self._lib
        T, k = ids.shape
        if k != self.topk or x.shape[1] != self.hidden:
            raise ValueError(f"this context was built for top-{self.topk} and hidden {self.hidden}")
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the context's max_tokens {self.max_tokens}")
        if x.dtype == torch.float32 and self.row_dtype != torch.bfloat16:
            raise ValueError("fp32 activations need bf16 rows")
        if x.dtype not in (torch.float32, self.row_dtype):
            raise ValueError(f"activations {x.dtype} do not match the rows' {self.row_dtype}")
        from blackhole_b200.hex_moe import _DT, _aligned, _stream
        x = _aligned(x)
        w = _aligned(w.to(torch.float32))
        ids = _aligned(ids if ids.dtype in (torch.int32, torch.int64) else ids.long())
        out = torch.empty(T, self.hidden, dtype=x.dtype, device=x.device)
        ws = self._workspace(self.block_m)
        st = _stream(self.device)
        ids_dt = _lib.I64 if ids.dtype == torch.int64 else _lib.I32
        wsp, wsn = (ws.data_ptr(), ws.numel()) if ws is not None else (None, 0)
        lay = self._layer.handle if self._layer else None
        with torch.cuda.device(self.device):
            if events is None:
                rc = _lib.lib.hexmoe_ep_forward(self._ctx, lay, x.data_ptr(), _DT[x.dtype], T, w.data_ptr(),
                                                ids.data_ptr(), ids_dt, out.data_ptr(), _DT[out.dtype], self.block_m,
                                                wsp, wsn, st)
                _lib.check(rc, "hexmoe_ep_forward")
                return out
            # the three phases apart, with events[0..3] recorded around them
            cur = torch.cuda.current_stream(self.device)
            events[0].record(cur)
            _lib.check(_lib.lib.hexmoe_ep_dispatch(self._ctx, x.data_ptr(), _DT[x.dtype], T, w.data_ptr(),
                                                   ids.data_ptr(), ids_dt, st), "hexmoe_ep_dispatch")
            events[1].record(cur)
            _lib.check(_lib.lib.hexmoe_ep_experts(self._ctx, lay, self.block_m, wsp, wsn, st), "hexmoe_ep_experts")
            events[2].record(cur)
            _lib.check(_lib.lib.hexmoe_ep_combine(self._ctx, T, out.data_ptr(), _DT[out.dtype], st),
                       "hexmoe_ep_combine")
            events[3].record(cur)
        return out

    def close(self) -> None:
        """Collective: waits for every rank, then frees this rank's buffers."""
        if self._ctx is None:
            return
        torch.cuda.synchronize(self.device)
        if self.shard.world > 1:
            dist.barrier(group=self.group)
        self._lib.lib.hexmoe_ep_destroy(self._ctx)
        self._ctx = None
        self._ws.clear()

    def __del__(self):
        ctx = getattr(self, "_ctx", None)
        if ctx is not None and self.shard.world == 1:
            self._lib.lib.hexmoe_ep_destroy(ctx)
            self._ctx = None

    # ------------------------------------------------------------------ CPU ranks
    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int]) -> None:
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def _forward_host(self, x: torch.Tensor, w: torch.Tensor, ids: torch.Tensor) -> torch.Tensor:
        T, k = ids.shape
        H = x.shape[1]
        world, E = self.shard.world, self.shard.num_experts
        rdt = _row_dtype(x.dtype)
        ids = ids.to(torch.int64)
        w = w.to(torch.float32)
        bad = bool(((ids < 0) | (ids >= E)).any())
        plan = plan_dispatch(ids.clamp(0, max(E - 1, 0)), self.shard)
        # 1. rows, slots, this rank's error flag, hidden and top-k per destination, read on
        #    the host: a bad id or ranks that disagree on the shapes fail on every rank
        #    before any row moves
        info = torch.tensor([[len(plan.rows[d]), len(plan.slots[d][0]), int(bad), H, k] for d in range(world)],
                            dtype=torch.int64)
        recv_info = torch.empty_like(info)
        dist.all_to_all_single(recv_info, info, group=self.group)
        if bool((recv_info[:, 3] != H).any() | (recv_info[:, 4] != k).any()):
            raise ValueError(f"ranks disagree on hidden / topk: {recv_info[:, 3:].tolist()}")
        if bool(recv_info[:, 2].any()) or bad:
            raise ValueError("topk_ids out of range" if bad else "topk_ids out of range on another rank")
        sent_rows = [len(r) for r in plan.rows]
        sent_slots = [len(s[0]) for s in plan.slots]
        got_rows, got_slots = recv_info[:, 0].tolist(), recv_info[:, 1].tolist()
        # 2. one row per (token, destination); one record per slot: (row at the destination, expert, weight bits)
        send_x = torch.cat([x[r].to(rdt) for r in plan.rows]) if T else x.new_zeros(0, H, dtype=rdt)
        recv_x = torch.empty(sum(got_rows), H, dtype=rdt)
        self._a2a(recv_x, send_x, got_rows, sent_rows)
        recs = []
        for d, (t_idx, j_idx) in enumerate(plan.slots):
            wbits = w[t_idx, j_idx].view(torch.int32).to(torch.int64)
            recs.append(torch.stack([plan.pos[t_idx, d], ids[t_idx, j_idx], wbits], 1))
        send_rec = torch.cat(recs) if recs else torch.zeros(0, 3, dtype=torch.int64)
        recv_rec = torch.empty(sum(got_slots), 3, dtype=torch.int64)
        self._a2a(recv_rec, send_rec, got_slots, sent_slots)
        # 3. the local experts, one slot per row
        row_base = torch.tensor([0] + got_rows[:-1], dtype=torch.int64).cumsum(0)
        src_of_slot = torch.repeat_interleave(torch.arange(world), torch.tensor(got_slots))
        row = row_base[src_of_slot] + recv_rec[:, 0]
        e = recv_rec[:, 1]
        wr = recv_rec[:, 2].to(torch.int32).view(torch.float32)
        y = self.expert_fn(recv_x[row], wr, e).to(rdt) if row.numel() else torch.empty(0, H, dtype=rdt)
        # 4. every slot's row back to its source, in the order the source sent the slots
        ret = torch.empty(sum(sent_slots), H, dtype=rdt)
        self._a2a(ret, y.contiguous(), sent_slots, got_slots)
        per = torch.zeros(T, k, H, dtype=torch.float32)
        base = 0
        for t_idx, j_idx in plan.slots:
            per[t_idx, j_idx] = ret[base:base + t_idx.numel()].float()
            base += t_idx.numel()
        # 5. the single-GPU combine: the k slot rows in j order, fp32, rounded once
        out = torch.zeros(T, H, dtype=torch.float32)
        for j in range(k):
            out = out + per[:, j]
        return out.to(x.dtype)

    # ------------------------------------------------------------------ entry
    def forward(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                events=None) -> torch.Tensor:
        """events (GPU path, optional): four torch.cuda.Event recorded before
        dispatch, before experts, before combine and after it."""
        if x.dim() != 2 or topk_ids.dim() != 2 or topk_weights.shape != topk_ids.shape or x.shape[0] != topk_ids.shape[0]:
            raise ValueError("x [T, H], topk_weights and topk_ids [T, k] expected")
        if self.expert_fn is not None:
            return self._forward_host(x, topk_weights, topk_ids)
        return self._forward_device(x, topk_weights, topk_ids, events)

    __call__ = forward


def reference_combine(y_slots: torch.Tensor, ids: torch.Tensor, shard: ExpertShard, out_dtype) -> torch.Tensor:
    """What EPMoE returns, from the single-GPU layer's per-slot rows y [T * k, H]
    (hexmoe_forward_slots): per token the fp32 sum of its k slot rows in j
    order, rounded once to out_dtype, which is the single-GPU layer's own
    combine whatever the sharding (`shard` and the ids only fix the shapes).
    Any device."""
    T, k = ids.shape
    yv = y_slots.view(T, k, -1).float()
    out = torch.zeros(T, yv.shape[2], dtype=torch.float32, device=y_slots.device)
    for j in range(k):
        out = out + yv[:, j]
    return out.to(out_dtype)
