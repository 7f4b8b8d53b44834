"""HEX checkpoint folders (the "blackhole-hex" layout) straight into the layer.

A folder holds safetensors files whose routed-expert tensors are named

    <prefix>.tier<L>.experts                  int32 [n]: the tier's global expert ids
    <prefix>.tier<L>.<proj>.<part>            the HEX parts stacked over those n experts

with proj in gate_proj / up_proj / down_proj, part in idx / block_scale /
expert_scale / levels and L the levels per table (8: 3-bit codes, 16: 4-bit),
plus a config.json whose quantization_config.quant_method is "blackhole-hex".
That is the contract of the reference's serving plugin and tools
(runtime/blackhole_runtime/vllm_hex.py:1-20 and :32, check_folder.py:22-44,
convert.py:32-56); every other tensor of the folder is ignored here.

    read_tiers(folder)          {prefix: {L: {"experts", gate_proj, up_proj, down_proj}}}
    layer_tiers(tiers, E, dev)  the prepared HexTier list of one MoE layer
    check_folder(folder, ...)   the checks of check_folder.py:47-93 on this build:
                                every expert held by exactly one tier, consistent
                                shapes, and the fused layer against
                                reference_moe (hex_ref.moe_reference restated in
                                torch over format_dequant, which decodes the
                                stored parts itself), as check_folder.py:86-90
    save_folder(folder, ...)    writes a folder in the same layout (synthetic
                                checkpoints for tests and benchmarks)

    python -m blackhole_b200.folder <folder> [--device cuda] [--layers N] [--no-kernel]

prints the check as one JSON line and exits 1 on any problem.
"""

from __future__ import annotations

import argparse
import json
import re
import sys
from pathlib import Path

import torch

PROJ = ("gate_proj", "up_proj", "down_proj")
PART = ("idx", "block_scale", "expert_scale", "levels")
QUANT_METHOD = "blackhole-hex"
_NAME = re.compile(r"^(?P<pre>.+)\.tier(?P<L>\d+)\.(?:experts|(?P<proj>gate_proj|up_proj|down_proj)\.(?P<part>idx|"
                   r"block_scale|expert_scale|levels))$")


def read_tiers(folder: str | Path) -> dict[str, dict[int, dict]]:
    """Every HEX tier of the folder's safetensors files, by layer prefix and table size."""
    from safetensors import safe_open
    out: dict[str, dict[int, dict]] = {}
    files = sorted(Path(folder).glob("*.safetensors"))
    for f in files:
        with safe_open(str(f), framework="pt") as h:
            for name in h.keys():
                m = _NAME.match(name)
                if not m:
                    continue
                tier = out.setdefault(m["pre"], {}).setdefault(int(m["L"]), {})
                if m["proj"]:
                    tier.setdefault(m["proj"], {})[m["part"]] = h.get_tensor(name)
                else:
                    tier["experts"] = h.get_tensor(name)
    return out


def _bits(levels_per_table: int) -> int:
    if levels_per_table not in (8, 16):
        raise ValueError(f"tier{levels_per_table}: HEX tables have 8 or 16 levels")
    return levels_per_table.bit_length() - 1


def tier_problems(prefix: str, tiers: dict[int, dict], num_experts: int | None) -> list[str]:
    """What keeps one layer's tiers from loading (empty when they load)."""
    problems = []
    for L, t in sorted(tiers.items()):
        missing = [f"{p}.{q}" for p in PROJ for q in PART if q not in t.get(p, {})]
        if "experts" not in t:
            missing.append("experts")
        if missing:
            problems.append(f"{prefix}.tier{L}: missing {', '.join(missing)}")
        if L not in (8, 16):
            problems.append(f"{prefix}.tier{L}: HEX tables have 8 or 16 levels")
    if problems:
        return problems
    seen = torch.cat([t["experts"].reshape(-1).long() for t in tiers.values()])
    n = num_experts if num_experts else int(seen.max()) + 1
    if sorted(seen.tolist()) != list(range(n)):
        problems.append(f"{prefix}: the tiers hold experts {sorted(seen.tolist())[:6]}..., "
                        f"expected each of 0..{n - 1} exactly once")
    dims = set()
    for L, t in tiers.items():
        nt = t["experts"].numel()
        for p in PROJ:
            for q in PART:
                if t[p][q].shape[0] != nt:
                    problems.append(f"{prefix}.tier{L}.{p}.{q}: {t[p][q].shape[0]} experts stacked, "
                                    f"the tier lists {nt}")
        bits = _bits(L)
        g, d = t["gate_proj"]["idx"], t["down_proj"]["idx"]
        I, H = g.shape[1], g.shape[2] * 32 // bits
        if t["up_proj"]["idx"].shape != g.shape or tuple(d.shape[1:]) != (H, I * bits // 32):
            problems.append(f"{prefix}.tier{L}: gate/up [I, H] and down [H, I] shapes disagree")
        dims.add((I, H))
    if len(dims) > 1:
        problems.append(f"{prefix}: tiers disagree on (I, H): {sorted(dims)}")
    return problems


def layer_tiers(tiers: dict[int, dict], num_experts: int, device) -> list:
    """One layer's tiers (read_tiers()[prefix]) as prepared HexTier objects on
    `device`, the 16-level tier first (the order of vllm_hex.py:123-134)."""
    from blackhole_b200.hex_moe import HexTier
    dev = torch.device(device)
    out = []
    for L, t in sorted(tiers.items(), reverse=True):
        parts = [{q: t[p][q].to(dev) for q in PART} for p in PROJ]
        out.append(HexTier(_bits(L), t["experts"].to(dev).to(torch.int32), *parts).prepare(num_experts))
    return out


def _fp8_values(device) -> torch.Tensor:
    """The 256 fp8 e4m3 scale codes as HEX reads them (blackhole/anatomy/hex.py:199-203):
    exponent field 0 is m/8 * 2^-6, every other field (1 + m/8) * 2^(e-7), the
    all-ones codes included (+-480, not NaN)."""
    c = torch.arange(256, device=device)
    e, m = (c >> 3) & 15, (c & 7).to(torch.float32)
    v = torch.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * torch.exp2((e - 7).to(torch.float32)))
    return torch.where(c >= 128, -v, v)


def format_dequant(parts: dict, bits: int, experts: torch.Tensor) -> torch.Tensor:
    """fp32 weights [len(experts), rows, cols] of local experts `experts` of one
    stacked projection, decoded from the stored parts by the format's own rule
    (blackhole/anatomy/hex.py:180-204): per 32-input block `bits` little-endian
    words, code j at bits [j*bits, j*bits + bits); W = levels[code] * (fp8(scale)
    * expert_scale), fp32 products.  The folder check's reference arithmetic: it
    shares no code with the kernels it checks."""
    idx = parts["idx"].index_select(0, experts)
    n, rows, nw = idx.shape
    words = idx.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    nblk = nw // bits
    words = words.reshape(n, rows, nblk, bits)
    lo = torch.arange(32, device=idx.device) * bits
    wi, sh = lo // 32, lo % 32
    v = words[..., wi] >> sh
    spill = (sh + bits > 32)
    nxt = words[..., torch.clamp(wi + 1, max=bits - 1)] << (32 - sh)
    v = torch.where(spill, v | nxt, v)
    codes = (v & ((1 << bits) - 1)).reshape(n, rows, nblk * 32)
    lev = parts["levels"].index_select(0, experts).float()
    vals = torch.gather(lev, 1, codes.reshape(n, -1)).reshape(n, rows, -1)
    bs = parts["block_scale"].index_select(0, experts).to(torch.int64)
    block = nblk * 32 // bs.shape[2]
    s = _fp8_values(idx.device)[bs] * parts["expert_scale"].float().reshape(-1).index_select(0, experts)[:, None, None]
    return vals * s.repeat_interleave(block, dim=2)


def reference_moe(x: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, tiers: dict[int, dict]) -> torch.Tensor:
    """moe_reference (runtime/blackhole_runtime/hex_ref.py:77-94) over a folder
    layer's tiers: per routed expert its weights by format_dequant, h = silu(x Wg^T)
    * (x Wu^T) in fp32 rounded to x's dtype, out += w * (h Wd^T) in fp32."""
    xf = x.float()
    out = torch.zeros(x.shape[0], x.shape[1], dtype=torch.float32, device=x.device)
    for L, t in tiers.items():
        bits = _bits(L)
        ex = t["experts"].reshape(-1).to(x.device).long()
        for local in range(ex.numel()):
            tok, slot = torch.nonzero(ids == ex[local], as_tuple=True)
            if tok.numel() == 0:
                continue
            li = torch.tensor([local], device=x.device)
            g, u, d = (format_dequant({q: v.to(x.device) for q, v in t[p].items()}, bits, li)[0] for p in PROJ)
            a = xf[tok]
            h = (torch.nn.functional.silu(a @ g.T) * (a @ u.T)).to(x.dtype).float()
            out.index_add_(0, tok, (h @ d.T) * w[tok, slot].float()[:, None])
    return out


def _natural(s: str) -> list:
    return [int(p) if p.isdigit() else p for p in re.split(r"(\d+)", s)]


def check_folder(folder: str | Path, device: str = "cuda", layers: int = 0, tokens: int = 5,
                 run_kernel: bool = True) -> dict:
    """The folder check: config, every layer's tiers, and (run_kernel) the fused
    layer on `tokens` random tokens and routings per layer (the first `layers`
    layers; 0 = all) against reference_moe, relative max error within 2e-2
    (bf16 activations; check_folder.py:86-90)."""
    folder = Path(folder)
    problems: list[str] = []
    cfg_path = folder / "config.json"
    cfg = json.loads(cfg_path.read_text()) if cfg_path.exists() else {}
    if not cfg:
        problems.append("no config.json")
    q = cfg.get("quantization_config") or {}
    if cfg and q.get("quant_method") != QUANT_METHOD:
        problems.append(f"quantization_config.quant_method is {q.get('quant_method')!r}, not {QUANT_METHOD!r}")
    tc = cfg.get("text_config") or cfg
    E = next((tc[k] for k in ("num_experts", "num_local_experts", "n_routed_experts") if isinstance(tc.get(k), int)),
             None)
    k = int(tc.get("num_experts_per_tok") or 2)
    all_tiers = read_tiers(folder)
    if not all_tiers:
        problems.append("no HEX tiers (<prefix>.tier<L>.*) in the safetensors files")
    worst, checked = 0.0, 0
    for li, prefix in enumerate(sorted(all_tiers, key=_natural)):
        tiers = all_tiers[prefix]
        p = tier_problems(prefix, tiers, E)
        problems += p
        if p or not run_kernel or (layers and checked >= layers):
            continue
        from blackhole_b200.hex_moe import hex_moe
        n = E or int(torch.cat([t["experts"].reshape(-1) for t in tiers.values()]).max()) + 1
        run = layer_tiers(tiers, n, device)
        I, H = run[0].dims()
        g = torch.Generator().manual_seed(li)
        kk = min(k, n)
        ids = torch.stack([torch.randperm(n, generator=g)[:kk] for _ in range(tokens)]).to(device)
        w = torch.softmax(torch.randn(tokens, kk, generator=g), -1).to(device)
        x = torch.randn(tokens, H, generator=g).to(torch.bfloat16).to(device)
        got = hex_moe(x, w, ids, run).float()
        want = reference_moe(x, w, ids, tiers)
        worst = max(worst, float((got - want).abs().max() / (want.abs().max() + 1e-12)))
        checked += 1
    if checked and worst >= 2e-2:
        problems.append(f"the fused layer differs from moe_reference over the format's dequantization by "
                        f"{worst:.1e} (tolerance 2e-2)")
    return {"layers": len(all_tiers), "checked": checked, "kernel_rel": worst, "problems": problems,
            "ok": not problems}


def save_folder(folder: str | Path, layers: dict[str, list[dict]], config: dict, shard_bytes: int = 1 << 30) -> None:
    """Writes `layers` ({prefix: [tier dicts with "bits", "experts" and the three
    projections' parts]}) as a blackhole-hex folder: safetensors shards of at
    most shard_bytes and config.json (quant_method set)."""
    from safetensors.torch import save_file
    folder = Path(folder)
    folder.mkdir(parents=True, exist_ok=True)
    tensors = {}
    for prefix, tiers in layers.items():
        for t in tiers:
            L = 1 << int(t["bits"])
            tensors[f"{prefix}.tier{L}.experts"] = torch.as_tensor(t["experts"]).to(torch.int32).cpu().contiguous()
            for p in PROJ:
                for q in PART:
                    tensors[f"{prefix}.tier{L}.{p}.{q}"] = torch.as_tensor(t[p][q]).cpu().contiguous()
    shard, size, n = {}, 0, 0
    for name in sorted(tensors, key=_natural):
        t = tensors[name]
        if shard and size + t.numel() * t.element_size() > shard_bytes:
            save_file(shard, str(folder / f"model-{n:05d}.safetensors"), metadata={"format": "pt"})
            shard, size, n = {}, 0, n + 1
        shard[name] = t
        size += t.numel() * t.element_size()
    if shard:
        save_file(shard, str(folder / f"model-{n:05d}.safetensors"), metadata={"format": "pt"})
    cfg = dict(config)
    qc = dict(cfg.get("quantization_config") or {})
    qc["quant_method"] = QUANT_METHOD
    qc.setdefault("version", 1)
    cfg["quantization_config"] = qc
    (folder / "config.json").write_text(json.dumps(cfg, indent=1))


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description="check a blackhole-hex folder on this build's kernels")
    ap.add_argument("folder")
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--layers", type=int, default=0, help="layers to run the kernel on (0 = all)")
    ap.add_argument("--tokens", type=int, default=5)
    ap.add_argument("--no-kernel", action="store_true", help="structural checks only (no GPU needed)")
    a = ap.parse_args(argv)
    r = check_folder(a.folder, a.device, a.layers, a.tokens, run_kernel=not a.no_kernel)
    print(json.dumps(r))
    return 0 if r["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
