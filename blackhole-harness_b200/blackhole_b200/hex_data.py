"""Seeded synthetic HEX layers, routings and activations (tests and benchmarks).

No dataset is involved anywhere on this path: the reference benchmarks random
HEX experts (runtime/blackhole_runtime/hex_check.py:28-46) and the layer configs
below restate its headline shapes.  The value distributions follow the configs
of the benchmark this package is measured on:

  levels        per expert, Phi^-1((l + 0.5) / L) * 0.02 + N(0, 0.002) per level,
                sorted, rounded to fp16, stored float32
  indices       uniform over the L levels; generated as uniform random idx words
                (packing is a bijection of 32*bits code bits onto `bits` words,
                so uniform words are uniform codes)
  block scales  |N(1, 0.1)| per (row, `block` inputs), rounded to fp8 e4m3 codes
  expert scale  1.0
  x             N(0, 1) in the activation dtype
  router        logits N(0, 1) [T, E] (+ log(1 / r^s) per expert for a Zipf(s)
                skew over a seeded rank permutation) -> softmax -> top-k ->
                renormalised (Qwen3 norm_topk_prob)

Everything draws from torch.Generator objects seeded per tensor, on the device
asked for (CPU results are identical on every machine with the same torch).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

HEX_BLOCK = 32

# The layer shapes of the benchmark configs (E experts, hidden H, moe_intermediate I, top-k).
CONFIGS = {
    "cfg1": dict(E=8, H=256, I=512, k=2, T=(64,), bits="4", block=128),
    "cfg2": dict(E=96, H=2048, I=768, k=8, T=(1, 8, 32, 64), bits="3", block=128),
    "cfg3": dict(E=96, H=2048, I=768, k=8, T=(4096, 16384), bits="mixed", block=128),
    "cfg4": dict(E=128, H=4096, I=1536, k=8, T=(8192,), bits="mixed", block=128),
    "cfg5": dict(E=96, H=2048, I=768, k=8, T=(32768,), bits="3", block=128, zipf=1.2),
}


def _gen(seed: int, device) -> torch.Generator:
    dev = torch.device(device)
    return torch.Generator(device=dev).manual_seed(int(seed))


def pack(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """[..., cols] codes in [0, 2**bits) -> [..., cols/32*bits] uint32 words: one
    little-endian bit stream per block of 32 inputs, value j at bits j*bits.."""
    *lead, n = codes.shape
    x = codes.to(torch.int64).reshape(*lead, n // HEX_BLOCK, HEX_BLOCK)
    words = torch.zeros(*lead, n // HEX_BLOCK, bits, dtype=torch.int64, device=codes.device)
    for j in range(HEX_BLOCK):
        lo = j * bits
        w, sh = divmod(lo, 32)
        words[..., w] |= (x[..., j] << sh) & 0xFFFFFFFF
        spill = sh + bits - 32
        if spill > 0:
            words[..., w + 1] |= x[..., j] >> (bits - spill)
    return (words - (words >= 2 ** 31).to(torch.int64) * 2 ** 32).to(torch.int32).reshape(*lead, -1).view(
        torch.uint32)


def fp8_codes(v: torch.Tensor) -> torch.Tensor:
    """float values -> fp8 e4m3 codes (uint8), nearest, as torch's float8_e4m3fn cast."""
    return v.to(torch.float32).to(torch.float8_e4m3fn).view(torch.uint8)


def synth_levels(n: int, bits: int, seed: int, device="cpu") -> torch.Tensor:
    L = 2 ** bits
    g = _gen(seed, "cpu")
    q = torch.tensor([math.sqrt(2.0) * torch.erfinv(torch.tensor(2.0 * ((l + 0.5) / L) - 1.0)).item()
                      for l in range(L)], dtype=torch.float64)
    lev = q[None, :] * 0.02 + torch.randn(n, L, generator=g, dtype=torch.float64) * 0.002
    lev = torch.sort(lev, dim=-1).values.to(torch.float16).to(torch.float32)
    return lev.to(device)


def synth_parts(n: int, rows: int, cols: int, bits: int, block: int = 128, seed: int = 0,
                device="cpu") -> dict:
    """One projection of n experts in the HEX layout (block 32 or 128 scales)."""
    assert cols % block == 0 and cols % HEX_BLOCK == 0
    g = _gen(seed, device)
    words = torch.randint(-2 ** 31, 2 ** 31, (n, rows, cols // HEX_BLOCK * bits), generator=g,
                          dtype=torch.int64, device=device).to(torch.int32).view(torch.uint32)
    s = torch.randn(n, rows, cols // block, generator=g, device=device, dtype=torch.float32).mul_(0.1).add_(1.0).abs_()
    return {"idx": words, "block_scale": fp8_codes(s),
            "expert_scale": torch.ones(n, dtype=torch.float32, device=device),
            "levels": synth_levels(n, bits, seed + 7919, device)}


def expand_block_scale(bs: torch.Tensor, block: int) -> torch.Tensor:
    """Scale codes at `block` inputs -> the same scales at the layout's 32-input block
    (each code repeated block/32 times along the input axis; dequantized weights are
    unchanged)."""
    return bs.repeat_interleave(block // HEX_BLOCK, dim=-1).contiguous()


@dataclass
class SynthLayer:
    E: int
    H: int
    I: int
    block: int
    tiers: list            # [{"bits", "experts", "gate_proj", "up_proj", "down_proj"}] (not prepared)


def synth_layer(E: int, H: int, I: int, bits="3", block: int = 128, seed: int = 0, device="cpu") -> SynthLayer:
    """Tiers of a synthetic layer: bits "3", "4", or "mixed" (a seeded half of the
    experts 4-bit, the rest 3-bit, as two tiers, 16-level tier first)."""
    perm = torch.randperm(E, generator=_gen(seed, "cpu"))
    if bits == "mixed":
        groups = [(perm[: E // 2].sort().values, 4), (perm[E // 2:].sort().values, 3)]
    else:
        groups = [(torch.arange(E), int(bits))]
    tiers = []
    for ti, (ids, b) in enumerate(groups):
        n = len(ids)
        parts = [synth_parts(n, o, i, b, block, seed + 1000 * ti + 10 * j, device)
                 for j, (o, i) in enumerate(((I, H), (I, H), (H, I)))]
        tiers.append({"bits": b, "experts": ids.to(torch.int32).to(device), "gate_proj": parts[0],
                      "up_proj": parts[1], "down_proj": parts[2]})
    return SynthLayer(E, H, I, block, tiers)


def synth_routing(T: int, E: int, k: int, seed: int = 0, zipf: float | None = None, device="cpu",
                  renormalize: bool = True):
    """(topk_weights f32 [T, k], topk_ids int64 [T, k]) from N(0,1) router logits."""
    g = _gen(seed, "cpu")
    logits = torch.randn(T, E, generator=g, dtype=torch.float32)
    if zipf:
        rank = torch.randperm(E, generator=g).to(torch.float32) + 1.0
        logits = logits + torch.log(1.0 / rank ** zipf)[None, :]
    p = torch.softmax(logits, dim=-1)
    w, ids = torch.topk(p, k, dim=-1)
    if renormalize:
        w = w / w.sum(-1, keepdim=True)
    return w.to(device), ids.to(torch.int64).to(device)


def synth_x(T: int, H: int, seed: int = 0, dtype=torch.bfloat16, device="cpu") -> torch.Tensor:
    g = _gen(seed, "cpu")
    return torch.randn(T, H, generator=g, dtype=torch.float32).to(dtype).to(device)


def tier_bytes(bits: int, H: int, I: int, block: int) -> int:
    """HBM bytes of one expert's three HEX projections (idx + scales + levels + scales)."""
    return 3 * H * I * bits // 8 + 3 * H * I // block + 3 * 4 * 2 ** bits + 3 * 4
