"""CPU oracle for the HEX fused-MoE path (numpy front end of hex_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() and by
bench.py's CPU-baseline leg, as the checker.  The product (blackhole_b200,
libhexmoe.so) never imports it.

Every function restates a piece of the reference (OliverVillson/BlackHole-Harness):
  fp8 / fp8_table    blackhole/anatomy/hex.py:199-203
  dequant            blackhole/anatomy/hex.py:180-204 (== hex_ref.py:24-46)
  pack / unpack      runtime/blackhole_runtime/hex_ref.py:49-61, hex.py:136-166
  align              runtime/blackhole_runtime/hex_moe.py:201-222
  moe_reference      runtime/blackhole_runtime/hex_ref.py:77-94
Pinned against tests/golden/*.npz, which tests/golden/make_golden.py wrote by
running the Python reference itself.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libhexoracle.so"
HEX_BLOCK = 32

_lib = None


def build(force: bool = False) -> Path:
    """Compile hex_oracle.c into libhexoracle.so (gcc, OpenMP)."""
    if force or not LIB.exists() or LIB.stat().st_mtime < (HERE / "hex_oracle.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB))
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        I32 = ctypes.c_int32
        L.hexo_fp8.restype = ctypes.c_float
        L.hexo_fp8.argtypes = [ctypes.c_uint8]
        L.hexo_fp8_table.argtypes = [P]
        L.hexo_dequant.argtypes = [P, P, P, P, I64, I64, I64, I64, I64, ctypes.c_int, ctypes.c_int, P]
        L.hexo_pack.argtypes = [P, I64, I64, ctypes.c_int, P]
        L.hexo_unpack.argtypes = [P, I64, I64, ctypes.c_int, P]
        L.hexo_align.restype = I64
        L.hexo_align.argtypes = [P, I64, I64, I64, P, P, P]
        L.hexo_moe_reference.argtypes = [P, I64, I64, I64, I64, I64, P, P, I64, P, I32, I32, I32, P, P, P]
        L.hexo_threads.restype = ctypes.c_int
        L.hexo_threads.argtypes = [ctypes.c_int]
        _lib = L
    return _lib


def _p(a: np.ndarray) -> ctypes.c_void_p:
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return ctypes.c_void_p(a.ctypes.data)


def fp8(code: int) -> float:
    return float(lib().hexo_fp8(code))


def fp8_table() -> np.ndarray:
    out = np.zeros(256, np.float32)
    lib().hexo_fp8_table(_p(out))
    return out


def pack(codes: np.ndarray, bits: int) -> np.ndarray:
    """[..., cols] codes -> [..., cols/32*bits] uint32 HEX bit stream."""
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    *lead, cols = codes.shape
    rows = int(np.prod(lead)) if lead else 1
    out = np.zeros((*lead, cols // HEX_BLOCK * bits), np.uint32)
    lib().hexo_pack(_p(codes), rows, cols, bits, _p(out))
    return out


def unpack(words: np.ndarray, bits: int, cols: int) -> np.ndarray:
    words = np.ascontiguousarray(words, dtype=np.uint32)
    *lead, _ = words.shape
    rows = int(np.prod(lead)) if lead else 1
    out = np.zeros((*lead, cols), np.uint8)
    lib().hexo_unpack(_p(words), rows, cols, bits, _p(out))
    return out


def dequant(parts: dict, bits: int, block: int = HEX_BLOCK, rows: int | None = None,
            cols: int | None = None) -> np.ndarray:
    """fp32 weights [n, rows, cols] of a stacked projection (parts as numpy arrays:
    idx uint32/int32 [n, rows_pad, cols_pad/32*bits], block_scale uint8, expert_scale
    f32 [n], levels f32 [n, 2^bits])."""
    idx = np.ascontiguousarray(parts["idx"]).view(np.uint32)
    bs = np.ascontiguousarray(parts["block_scale"], dtype=np.uint8)
    es = np.ascontiguousarray(parts["expert_scale"], dtype=np.float32).reshape(-1)
    lev = np.ascontiguousarray(parts["levels"], dtype=np.float32)
    n, rows_pad, nw = idx.shape
    cols_pad = nw // bits * HEX_BLOCK
    rows = rows_pad if rows is None else rows
    cols = cols_pad if cols is None else cols
    assert bs.shape == (n, rows_pad, cols_pad // block), (bs.shape, block)
    out = np.zeros((n, rows, cols), np.float32)
    lib().hexo_dequant(_p(idx), _p(bs), _p(es), _p(lev), n, rows, cols, rows_pad, cols_pad, bits, block,
                       _p(out))
    return out


def align(ids: np.ndarray, n: int, block_m: int):
    """(sorted_ids int32, expert_ids int32, npp int32[1]) exactly as the reference align()."""
    ids = np.ascontiguousarray(ids, dtype=np.int64).reshape(-1)
    S = ids.size
    max_blocks = -(-S // block_m) + min(n, S)
    sid = np.zeros(max(max_blocks * block_m, 1), np.int32)[: max_blocks * block_m]
    eid = np.zeros(max(max_blocks, 1), np.int32)[:max_blocks]
    npp = np.zeros(1, np.int32)
    sid = np.ascontiguousarray(sid)
    eid = np.ascontiguousarray(eid)
    r = lib().hexo_align(_p(ids), S, n, block_m, _p(sid) if sid.size else None, _p(eid) if eid.size else None,
                         _p(npp))
    if r < 0:
        raise ValueError("align: expert id out of range")
    return sid, eid, npp


class _Proj(ctypes.Structure):
    _fields_ = [("idx", ctypes.c_void_p), ("bs", ctypes.c_void_p), ("es", ctypes.c_void_p),
                ("lev", ctypes.c_void_p)]


class _Tier(ctypes.Structure):
    _fields_ = [("bits", ctypes.c_int32), ("n", ctypes.c_int32), ("experts", ctypes.c_void_p),
                ("gate", _Proj), ("up", _Proj), ("down", _Proj)]


ACT_DTYPES = {"float32": 0, "bfloat16": 1, "float16": 2}


class Layer:
    """Numpy copy of a tiered HEX layer for the oracle (keeps the arrays alive)."""

    def __init__(self, tiers: list[dict], num_experts: int, hidden: int, inter: int, block: int = HEX_BLOCK):
        self.E, self.H, self.I, self.block = num_experts, hidden, inter, block
        self.keep = []
        self.ctiers = (_Tier * len(tiers))()
        for ti, t in enumerate(tiers):
            bits = int(t["bits"])
            ex = np.ascontiguousarray(np.asarray(t["experts"]), dtype=np.int64).reshape(-1)
            self.keep.append(ex)
            ct = self.ctiers[ti]
            ct.bits, ct.n, ct.experts = bits, ex.size, ex.ctypes.data
            for proj in ("gate_proj", "up_proj", "down_proj"):
                p = t[proj]
                arrs = (np.ascontiguousarray(np.asarray(p["idx"])).view(np.uint32),
                        np.ascontiguousarray(np.asarray(p["block_scale"]), dtype=np.uint8),
                        np.ascontiguousarray(np.asarray(p["expert_scale"]), dtype=np.float32).reshape(-1),
                        np.ascontiguousarray(np.asarray(p["levels"]), dtype=np.float32))
                self.keep.extend(arrs)
                setattr(ct, proj.split("_")[0], _Proj(*(a.ctypes.data for a in arrs)))
            gi = np.asarray(t["gate_proj"]["idx"])
            self.I_pad = gi.shape[1]
            self.H_pad = gi.shape[2] // bits * HEX_BLOCK
        self.ntiers = len(tiers)
        self._wcache = None
        self._filled = ctypes.c_int32(0)

    def forward(self, x: np.ndarray, topk_w: np.ndarray, topk_ids: np.ndarray, act_dtype: str = "bfloat16",
                cache_weights: bool = False) -> np.ndarray:
        """moe_reference: fp32 [T, H].  x given as float32 values (already in the
        activation dtype's grid); act_dtype is the dtype h is rounded to."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        w = np.ascontiguousarray(topk_w, dtype=np.float32)
        ids = np.ascontiguousarray(topk_ids, dtype=np.int64)
        T, k = ids.shape
        out = np.zeros((T, self.H), np.float32)
        wc = None
        if cache_weights:
            if self._wcache is None:
                bufs = []
                for ti in range(self.ntiers):
                    n = self.ctiers[ti].n
                    bufs += [np.zeros(n * self.I * self.H, np.float32) for _ in range(3)]
                self._wcache = bufs
                self._wptrs = (ctypes.c_void_p * len(bufs))(*(b.ctypes.data for b in bufs))
            wc = self._wptrs
        lib().hexo_moe_reference(_p(x), T, self.H, self.I, self.H_pad, self.I_pad, _p(w), _p(ids), k,
                                 ctypes.cast(self.ctiers, ctypes.c_void_p), self.ntiers, self.block,
                                 ACT_DTYPES[act_dtype], _p(out), ctypes.cast(wc, ctypes.c_void_p) if wc else None,
                                 ctypes.byref(self._filled))
        return out


def moe_reference(x, topk_w, topk_ids, tiers: list[dict], num_experts: int, block: int = HEX_BLOCK,
                  act_dtype: str = "bfloat16") -> np.ndarray:
    """One-shot moe_reference (hex_ref.py:77-94) on numpy tiers."""
    gi = np.asarray(tiers[0]["gate_proj"]["idx"])
    bits = int(tiers[0]["bits"])
    H = x.shape[1]
    I = gi.shape[1]
    layer = Layer(tiers, num_experts, H, I, block)
    return layer.forward(x, topk_w, topk_ids, act_dtype)


def round_bf16(a: np.ndarray) -> np.ndarray:
    """float32 -> nearest-even bf16 values, still as float32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def set_threads(n: int | None = None) -> int:
    """OpenMP threads the oracle uses (default: all host cores); returns the count."""
    return int(lib().hexo_threads(int(n or os.cpu_count() or 1)))
