"""HEX fused MoE on B200 (sm_100a): the drop-in for runtime/blackhole_runtime/hex_moe.py.

Same names, argument meaning and exceptions as the reference module
(OliverVillson/BlackHole-Harness, runtime/blackhole_runtime/hex_moe.py): HexTier
(174-198), align (201-222), direct (228-237), plan (248-257), default_config
(264-283), hex_moe_fused (304-325), dequant_all (328-346), hex_moe_dequant
(357-371), hex_moe (374-382), PARTS (39).  What runs underneath is libhexmoe.so:

  hex_moe / hex_moe_fused   one C call (hexmoe_forward): the stable align plan,
                            the tcgen05 gate/up grouped GEMM with SwiGLU, the
                            down grouped GEMM with the top-k weight, the combine.
                            No host synchronisation, so CUDA graphs capture it.
  path="dequant"            the same fused path: the sm_100a kernel decodes each
                            weight tile once into tensor memory, so a bf16 copy
                            of every expert in HBM (the reference's prefill path)
                            would only add traffic.  Accepted for compatibility.
  config / align_mode       config["BLOCK_M"] sets the tile height (tokens per
                            expert tile): 8 runs the small-batch (decode)
                            kernels, 16/32/64/128 the tcgen05 grouped GEMM;
                            the other keys and align_mode are accepted and have
                            no effect.
  dequant_all / align       hexmoe_dequant (bit-exact) / hexmoe_align (stable,
                            equal to the reference output bit for bit).

Inputs must be CUDA tensors on an sm_100 device; there is no CPU path.
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass, field

import torch

from blackhole_b200 import _lib

PARTS = ("idx", "block_scale", "expert_scale", "levels")
HEX_BLOCK = 32
TILE = 128          # rows of a weight tile and granule of the padded kernel layout

DIRECT_MAX = int(os.environ.get("BLACKHOLE_HEX_DIRECT_MAX", "32"))      # slots: 4 tokens at top-8
DEQUANT_MIN = int(os.environ.get("BLACKHOLE_HEX_DEQUANT_MIN", "1024"))  # kept for API compatibility

_DT = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _round_up(v: int, m: int) -> int:
    return (v + m - 1) // m * m


def _aligned(t: torch.Tensor, align: int = 16) -> torch.Tensor:
    t = t.contiguous()
    if t.data_ptr() % align:
        t = t.clone()
    return t


@dataclass
class HexTier:
    """One tier of a MoE layer: experts sharing one index width, stacked in the HEX layout."""
    bits: int
    experts: torch.Tensor              # int global expert ids [n]
    gate_proj: dict                    # {"idx", "block_scale", "expert_scale", "levels"}
    up_proj: dict
    down_proj: dict
    lookup: torch.Tensor | None = None  # int32 [num_experts]: local index in this tier or -1
    block: int = 0                     # fp8 scale block (32 = layout, or 128); set by prepare
    kernel_parts: dict = field(default_factory=dict)   # per projection, the parts the kernels read

    def prepare(self, num_experts: int) -> "HexTier":
        """Kernel-ready views (uint32 words as int32, f32 scales/levels) and the global -> local
        expert map, as the reference; plus the kernel layout: the parts themselves whenever the
        shapes are multiples of 128 (every production shape), else a zero-padded copy."""
        if self.bits not in (3, 4):
            raise ValueError(f"HEX tier bits must be 3 or 4, got {self.bits}")
        for p in (self.gate_proj, self.up_proj, self.down_proj):
            if p["idx"].dtype == torch.uint32:
                p["idx"] = p["idx"].view(torch.int32)
            p["expert_scale"] = p["expert_scale"].float().reshape(-1).contiguous()
            p["levels"] = p["levels"].float().contiguous()
            for k in ("idx", "block_scale"):
                p[k] = p[k].contiguous()
        dev = self.gate_proj["idx"].device
        n = len(self.experts)
        lk = torch.full((num_experts,), -1, dtype=torch.int32, device=dev)
        lk[self.experts.to(dev).long()] = torch.arange(n, dtype=torch.int32, device=dev)
        self.lookup = lk
        self.experts = self.experts.to(dev).to(torch.int32)
        I, H = self.dims()
        nblk = self.gate_proj["block_scale"].shape[-1]
        if H % nblk or H // nblk not in (32, 128):
            raise ValueError(f"block_scale has {nblk} blocks for {H} inputs (block must be 32 or 128)")
        self.block = H // nblk
        for name, (rows, cols) in (("gate_proj", (I, H)), ("up_proj", (I, H)), ("down_proj", (H, I))):
            p = getattr(self, name)
            if tuple(p["idx"].shape) != (n, rows, cols // HEX_BLOCK * self.bits):
                raise ValueError(f"{name}.idx shape {tuple(p['idx'].shape)} != {(n, rows, cols // 32 * self.bits)}")
            if tuple(p["block_scale"].shape) != (n, rows, cols // self.block):
                raise ValueError(f"{name}.block_scale shape {tuple(p['block_scale'].shape)}")
            if p["levels"].shape != (n, 2 ** self.bits) or p["expert_scale"].numel() != n:
                raise ValueError(f"{name}: levels / expert_scale do not match {n} experts of {self.bits} bits")
            self.kernel_parts[name] = self._kernel_layout(p, rows, cols)
        return self

    def dims(self) -> tuple[int, int]:
        """(I, H) of this tier: gate_proj is [I, H]."""
        _, I, nw = self.gate_proj["idx"].shape
        return I, nw // self.bits * HEX_BLOCK

    def _kernel_layout(self, p: dict, rows: int, cols: int) -> dict:
        rp, cp = _round_up(rows, TILE), _round_up(cols, TILE)
        idx, bs = p["idx"], p["block_scale"]
        if (rp, cp) != (rows, cols):
            n = idx.shape[0]
            pi = torch.zeros(n, rp, cp // HEX_BLOCK * self.bits, dtype=idx.dtype, device=idx.device)
            pi[:, :rows, : idx.shape[2]] = idx
            pb = torch.zeros(n, rp, cp // self.block, dtype=bs.dtype, device=bs.device)
            pb[:, :rows, : bs.shape[2]] = bs
            idx, bs = pi, pb
        return {"idx": _aligned(idx), "block_scale": _aligned(bs), "expert_scale": _aligned(p["expert_scale"]),
                "levels": _aligned(p["levels"]), "rows_pad": rp, "cols_pad": cp}


def _parts_struct(kp: dict) -> _lib.Parts:
    return _lib.Parts(_ptr(kp["idx"]), _ptr(kp["block_scale"]), _ptr(kp["expert_scale"]), _ptr(kp["levels"]))


class _Layer:
    """A C-ABI layer handle over prepared tiers (owns the device expert map)."""

    def __init__(self, tiers: list[HexTier]):
        if not tiers or len(tiers) > _lib.MAX_TIERS:
            raise ValueError(f"1..{_lib.MAX_TIERS} tiers expected, got {len(tiers)}")
        t0 = tiers[0]
        if t0.lookup is None:
            raise ValueError("tiers must be prepared (HexTier.prepare) before use")
        self.E = t0.lookup.numel()
        self.I, self.H = t0.dims()
        self.block = t0.block
        dev = t0.gate_proj["idx"].device
        if dev.type != "cuda":
            raise ValueError("blackhole_b200 runs on CUDA (sm_100a) only; the tiers are on " + str(dev))
        self.device = dev
        d = _lib.LayerDesc()
        d.num_experts, d.hidden, d.inter, d.block, d.num_tiers = self.E, self.H, self.I, self.block, len(tiers)
        d.hidden_pad = t0.kernel_parts["gate_proj"]["cols_pad"]
        d.inter_pad = t0.kernel_parts["gate_proj"]["rows_pad"]
        self.keep = []
        for i, t in enumerate(tiers):
            if t.dims() != (self.I, self.H) or t.block != self.block or t.lookup.numel() != self.E:
                raise ValueError("all tiers of a layer must share E, H, I and the scale block")
            ct = d.tiers[i]
            ct.bits, ct.n, ct.experts = t.bits, len(t.experts), _ptr(t.experts)
            ct.gate = _parts_struct(t.kernel_parts["gate_proj"])
            ct.up = _parts_struct(t.kernel_parts["up_proj"])
            ct.down = _parts_struct(t.kernel_parts["down_proj"])
            self.keep.append(t)
        self.desc = d
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("the first hex_moe call on a set of tiers builds the layer (a synchronous tiled copy "
                               "of the index streams); make it before CUDA graph capture")
        with torch.cuda.device(dev):
            self.expert_map = torch.empty(self.E, dtype=torch.int32, device=dev)
            _lib.check(_lib.lib.hexmoe_build_expert_map(ctypes.byref(d), _ptr(self.expert_map), _stream(dev)),
                       "hexmoe_build_expert_map")
            d.expert_map = _ptr(self.expert_map)
            h = ctypes.c_void_p()
            _lib.check(_lib.lib.hexmoe_layer_create(ctypes.byref(d), ctypes.byref(h)), "hexmoe_layer_create")
        self.handle = h

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            _lib.lib.hexmoe_layer_destroy(h)
            self.handle = None

    def forward(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                block_m: int = 0) -> torch.Tensor:
        if x.device != self.device:
            raise ValueError(f"x is on {x.device}, the experts on {self.device}")
        if x.dim() != 2 or x.shape[1] != self.H:
            raise ValueError(f"x must be [T, {self.H}], got {tuple(x.shape)}")
        if x.dtype not in _DT:
            raise ValueError(f"unsupported activation dtype {x.dtype}")
        T, k = topk_ids.shape
        if topk_weights.shape != (T, k) or x.shape[0] != T:
            raise ValueError("topk_weights / topk_ids / x disagree on T or k")
        x = _aligned(x)
        w = _aligned(topk_weights.to(torch.float32))
        ids = topk_ids if topk_ids.dtype in (torch.int32, torch.int64) else topk_ids.long()
        ids = _aligned(ids)
        ids_dt = _lib.I64 if ids.dtype == torch.int64 else _lib.I32
        out = torch.empty(T, self.H, dtype=x.dtype, device=x.device)
        if T == 0:
            return out
        xdt = _DT[x.dtype]
        nbytes = _lib.lib.hexmoe_forward_workspace_bytes(self.handle, T, k, block_m, xdt)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
        with torch.cuda.device(x.device):
            rc = _lib.lib.hexmoe_forward(self.handle, _ptr(x), xdt, T, k, _ptr(w), _ptr(ids), ids_dt, _ptr(out), xdt,
                                         block_m, _ptr(ws), nbytes, _stream(x.device))
        _lib.check(rc, "hexmoe_forward")
        return out


    def forward_slots(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                      block_m: int = 0) -> torch.Tensor:
        """forward() without the combine: the weighted per-slot rows [T * k, H]
        (16-bit: x's dtype, bf16 for fp32 x), in slot order (hexmoe_forward_slots)."""
        T, k = topk_ids.shape
        if x.device != self.device or x.dim() != 2 or x.shape != (T, self.H) or topk_weights.shape != (T, k):
            raise ValueError("x [T, H] on the layer's device, topk_weights / topk_ids [T, k] expected")
        if x.dtype not in _DT:
            raise ValueError(f"unsupported activation dtype {x.dtype}")
        x = _aligned(x)
        w = _aligned(topk_weights.to(torch.float32))
        ids = _aligned(topk_ids if topk_ids.dtype in (torch.int32, torch.int64) else topk_ids.long())
        y = torch.empty(T * k, self.H, dtype=torch.float16 if x.dtype == torch.float16 else torch.bfloat16,
                        device=x.device)
        if T == 0:
            return y
        xdt = _DT[x.dtype]
        nbytes = _lib.lib.hexmoe_forward_workspace_bytes(self.handle, T, k, block_m, xdt)
        ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
        with torch.cuda.device(x.device):
            rc = _lib.lib.hexmoe_forward_slots(self.handle, _ptr(x), xdt, T, k, _ptr(w), _ptr(ids),
                                               _lib.I64 if ids.dtype == torch.int64 else _lib.I32, _ptr(y), block_m,
                                               _ptr(ws), nbytes, _stream(x.device))
        _lib.check(rc, "hexmoe_forward_slots")
        return y

    # -- the phases of forward(), for callers that time or drive them apart
    def plan(self, topk_ids: torch.Tensor, block_m: int):
        return align(topk_ids.reshape(-1), self.E, block_m)

    def max_blocks(self, slots: int, block_m: int) -> int:
        return -(-slots // block_m) + min(self.E, slots)

    def gather(self, x: torch.Tensor, k: int, plan, block_m: int, xs: torch.Tensor | None = None) -> torch.Tensor:
        """Plan-ordered activation rows (16-bit; bf16 for fp32 x)."""
        sid, _, npp = plan
        T = x.shape[0]
        dt = torch.bfloat16 if x.dtype == torch.float32 else x.dtype
        if xs is None:
            xs = torch.empty(self.max_blocks(T * k, block_m) * block_m, self.H, dtype=dt, device=x.device)
        with torch.cuda.device(x.device):
            rc = _lib.lib.hexmoe_gather(_ptr(x), _DT[x.dtype], T, self.H, k, self.E, _ptr(sid), _ptr(npp), block_m,
                                        _ptr(xs), _stream(x.device))
        _lib.check(rc, "hexmoe_gather")
        return xs

    def gate_up(self, xs: torch.Tensor, T: int, k: int, plan, block_m: int,
                act: torch.Tensor | None = None) -> torch.Tensor:
        sid, eid, npp = plan
        if act is None:
            act = torch.empty(self.max_blocks(T * k, block_m) * block_m, self.desc.inter_pad, dtype=xs.dtype,
                              device=xs.device)
        with torch.cuda.device(xs.device):
            rc = _lib.lib.hexmoe_gate_up(self.handle, _ptr(xs), _DT[xs.dtype], T, k, _ptr(sid), _ptr(eid), _ptr(npp),
                                         block_m, _ptr(act), _stream(xs.device))
        _lib.check(rc, "hexmoe_gate_up")
        return act

    def down(self, act: torch.Tensor, topk_weights: torch.Tensor, plan, block_m: int,
             y: torch.Tensor | None = None) -> torch.Tensor:
        sid, eid, npp = plan
        T, k = topk_weights.shape
        if y is None:
            y = torch.empty(T * k, self.H, dtype=act.dtype, device=act.device)
        with torch.cuda.device(act.device):
            rc = _lib.lib.hexmoe_down(self.handle, _ptr(act), _DT[act.dtype], T, k, _ptr(topk_weights), _ptr(sid),
                                      _ptr(eid), _ptr(npp), block_m, _ptr(y), _stream(act.device))
        _lib.check(rc, "hexmoe_down")
        return y

    def combine(self, y: torch.Tensor, T: int, k: int, out_dtype=None) -> torch.Tensor:
        out = torch.empty(T, self.H, dtype=out_dtype or y.dtype, device=y.device)
        with torch.cuda.device(y.device):
            rc = _lib.lib.hexmoe_combine(_ptr(y), _DT[y.dtype], T, k, self.H, _ptr(out), _DT[out.dtype],
                                         _stream(y.device))
        _lib.check(rc, "hexmoe_combine")
        return out

    def combine_rows(self, y: torch.Tensor, T: int, k: int, rows: torch.Tensor, out_dtype=None) -> torch.Tensor:
        """out[t] = sum_j y[rows[t*k + j]]: see combine_rows()."""
        return combine_rows(y, T, k, rows, out_dtype)


def combine_rows(y: torch.Tensor, T: int, k: int, rows: torch.Tensor, out_dtype=None) -> torch.Tensor:
    """out[t] = sum_j y[rows[t*k + j]] (hexmoe_combine_rows): the layer's combine
    of per-slot rows held in another order; needs no layer.  y [R, H] 16-bit,
    rows int32 [T * k]."""
    if not y.is_cuda:
        raise ValueError("combine_rows runs on CUDA only")
    if rows.dtype != torch.int32 or rows.numel() != T * k:
        raise ValueError("rows must be int32 [T * k]")
    if y.dtype not in (torch.bfloat16, torch.float16) or y.dim() != 2:
        raise ValueError("y must be a bf16 / fp16 [rows, H] tensor")
    out = torch.empty(T, y.shape[1], dtype=out_dtype or y.dtype, device=y.device)
    y, rows = _aligned(y), rows.contiguous()
    with torch.cuda.device(y.device):
        rc = _lib.lib.hexmoe_combine_rows(_ptr(y), _DT[y.dtype], y.shape[0], T, k, y.shape[1], _ptr(rows), _ptr(out),
                                          _DT[out.dtype], _stream(y.device))
    _lib.check(rc, "hexmoe_combine_rows")
    return out


def auto_block_m(slots: int, num_experts: int, hidden: int = 0) -> int:
    """The block_m hexmoe_forward picks when given 0 (api.cu auto_block_m): the
    small-batch kernels (8) while an expert averages at most 8 slots (and the
    hidden size is a multiple of 64), else the smallest of 16/32/64/128 covering
    the mean slots per expert."""
    avg = -(-slots // max(num_experts, 1))
    for bm in ((8, 16, 32, 64) if hidden % 64 == 0 else (16, 32, 64)):
        if avg <= bm:
            return bm
    return 128


def _layer(tiers: list[HexTier]) -> _Layer:
    key = tuple((id(t), _ptr(t.kernel_parts["gate_proj"]["idx"])) for t in tiers)
    cache = tiers[0].__dict__.setdefault("_b200_layers", {})
    L = cache.get(key)
    if L is None:
        L = cache[key] = _Layer(tiers)
    return L


def layer_for(tiers: list[HexTier]) -> _Layer:
    """The (cached) C-ABI layer handle of prepared tiers, with the phase calls
    plan / gate_up / down / combine of hex_moe_fused."""
    return _layer(tiers)


def align(ids: torch.Tensor, n: int, block_m: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Group slots by expert, each expert's run padded to block_m, without a host sync.
    ids: int [S] global expert ids. Returns sorted slot ids int32 [B * block_m] (S = padding),
    the expert of every block int32 [B] (-1 = unused) and the padded length int32 [1]."""
    if not ids.is_cuda:
        raise ValueError("align runs on CUDA only")
    ids = ids.reshape(-1)
    if ids.dtype not in (torch.int32, torch.int64):
        ids = ids.long()
    ids = ids.contiguous()
    S = ids.numel()
    max_blocks = -(-S // block_m) + min(n, S)
    sid = torch.empty(max_blocks * block_m, dtype=torch.int32, device=ids.device)
    eid = torch.empty(max_blocks, dtype=torch.int32, device=ids.device)
    npp = torch.empty(1, dtype=torch.int32, device=ids.device)
    nws = _lib.lib.hexmoe_align_workspace_bytes(S, n)
    ws = torch.empty(nws, dtype=torch.uint8, device=ids.device) if nws else None
    with torch.cuda.device(ids.device):
        rc = _lib.lib.hexmoe_align(_ptr(ids), _lib.I64 if ids.dtype == torch.int64 else _lib.I32, S, n, block_m,
                                   _ptr(sid), _ptr(eid), _ptr(npp), _ptr(ws) if nws else None, nws,
                                   _stream(ids.device))
    _lib.check(rc, "hexmoe_align")
    return sid, eid, npp


_DIRECT: dict = {}


def direct(ids: torch.Tensor, block_m: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """One block per slot (few slots: no sorting at all). Same outputs as align()."""
    S = ids.numel()
    key = (S, block_m, ids.device)
    if key not in _DIRECT:
        s = torch.full((S, block_m), S, dtype=torch.int32, device=ids.device)
        s[:, 0] = torch.arange(S, dtype=torch.int32, device=ids.device)
        _DIRECT[key] = (s.reshape(-1), torch.full((1,), S * block_m, dtype=torch.int32, device=ids.device))
    sid, npp = _DIRECT[key]
    return sid, ids.reshape(-1).to(torch.int32), npp


def plan(ids: torch.Tensor, n: int, block_m: int, mode: str = "auto"):
    """(sorted slot ids, block experts, padded length) in the reference's plan format."""
    if mode == "direct" or (mode == "auto" and ids.numel() <= DIRECT_MAX):
        return direct(ids, block_m)
    return align(ids, n, block_m)


def default_config(slots: int, n_out: int, n_in: int, glu: bool) -> dict:
    """Tile choice by slot count (BLOCK_M = tokens per expert tile, the UMMA N side).
    BLACKHOLE_HEX_TILES="BM,..." overrides BLOCK_M as in the reference."""
    env = os.environ.get("BLACKHOLE_HEX_TILES")
    if env:
        v = [int(t) for t in env.split(",")]
        return {"BLOCK_M": v[0], "BLOCK_N": TILE, "BLOCK_K": TILE}
    if slots <= 512:
        bm = 16
    elif slots <= 4096:
        bm = 64
    else:
        bm = 128
    return {"BLOCK_M": bm, "BLOCK_N": TILE, "BLOCK_K": TILE}


def _block_m(config: dict | None) -> int:
    if not config:
        env = os.environ.get("BLACKHOLE_HEX_TILES")
        return int(env.split(",")[0]) if env else 0
    bm = int(config.get("BLOCK_M", 0))
    return bm if bm in (8, 16, 32, 64, 128) else 0


def hex_moe_fused(x, topk_weights, topk_ids, tiers: list[HexTier], config: dict | None = None,
                  align_mode: str = "auto") -> torch.Tensor:
    """Routed-expert output [T, H] through the fused HEX kernels."""
    if align_mode not in ("auto", "torch", "vllm", "direct"):
        raise ValueError(f"unknown align_mode {align_mode!r}")
    return _layer(tiers).forward(x, topk_weights, topk_ids, _block_m(config))


def dequant_all(tiers: list[HexTier], dtype=torch.bfloat16) -> tuple[torch.Tensor, torch.Tensor]:
    """All experts as stacks: w13 [E, 2I, H] (gate rows, then up) and w2 [E, H, I]."""
    t0 = tiers[0]
    E = t0.lookup.numel()
    I, H = t0.dims()
    dev = t0.gate_proj["idx"].device
    if dev.type != "cuda":
        raise ValueError("dequant_all runs on CUDA only")
    if dtype not in _DT:
        raise ValueError(f"unsupported dtype {dtype}")
    w13 = torch.empty(E, 2 * I, H, dtype=dtype, device=dev)
    w2 = torch.empty(E, H, I, dtype=dtype, device=dev)
    with torch.cuda.device(dev):
        for t in tiers:
            n = len(t.experts)
            for name, out, row_off, (rows, cols) in (("gate_proj", w13, 0, (I, H)), ("up_proj", w13, I, (I, H)),
                                                     ("down_proj", w2, 0, (H, I))):
                kp = t.kernel_parts[name]
                parts = _parts_struct(kp)
                rc = _lib.lib.hexmoe_dequant(ctypes.byref(parts), t.bits, t.block, n, rows, cols, kp["rows_pad"],
                                             kp["cols_pad"], _ptr(t.experts), _ptr(out), _DT[dtype], out.stride(0),
                                             out.stride(1), row_off, _stream(dev))
                _lib.check(rc, "hexmoe_dequant")
    return w13, w2


def hex_moe_dequant(x, topk_weights, topk_ids, tiers: list[HexTier]) -> torch.Tensor:
    """Routed-expert output [T, H]; on sm_100a the fused kernels are the prefill path too."""
    return hex_moe_fused(x, topk_weights, topk_ids, tiers)


def hex_moe(x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor, tiers: list[HexTier],
            config: dict | None = None, path: str = "auto") -> torch.Tensor:
    """Routed-expert output [T, H] of a SwiGLU MoE layer whose experts are HEX tiers (prepared).
    path: "auto", "fused" or "dequant" (all three run the fused sm_100a kernels)."""
    if path not in ("auto", "fused", "dequant"):
        raise ValueError(f"unknown path {path!r}")
    return hex_moe_fused(x, topk_weights, topk_ids, tiers, config)


def route_topk(logits: torch.Tensor, k: int, renormalize: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """softmax(logits) -> top-k (ties: lower id) -> optional renormalisation, on the device.
    Returns (weights f32 [T, k], ids int32 [T, k])."""
    if not logits.is_cuda:
        raise ValueError("route_topk runs on CUDA only")
    if logits.dtype not in _DT:
        raise ValueError(f"unsupported logits dtype {logits.dtype}")
    logits = _aligned(logits)
    T, E = logits.shape
    w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    ids = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    with torch.cuda.device(logits.device):
        rc = _lib.lib.hexmoe_route_topk(_ptr(logits), _DT[logits.dtype], T, E, k, int(renormalize), _ptr(w),
                                        _ptr(ids), _stream(logits.device))
    _lib.check(rc, "hexmoe_route_topk")
    return w, ids


def device_status(device=None, clear: bool = True) -> int:
    """The device error word (bounded-wait timeouts, bad expert ids); synchronises the device."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    return _lib.device_status(dev.index or 0, clear)
