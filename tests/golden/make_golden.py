"""Write the golden vectors under tests/golden/ by running the Python reference.

Run in a container that has the reference tree (OliverVillson/BlackHole-Harness)
checked out; the GPU test box never runs this script, it only reads its output:

    REF=/path/to/BlackHole-Harness python tests/golden/make_golden.py

What is recorded (all small; inputs are stored whenever the reference generated
them, and regenerated from a recorded seed + sha256 when this package's seeded
generator made them):

  fp8_kat.npz        the reference hex_dequant of every fp8 code (levels 1, scale 1)
  pack.npz           reference pack() of seeded codes, 3 and 4 bits
  align.npz          reference align() on fixed and seeded id vectors
  dequant_*.npz      reference hex_dequant of reference random_parts (bits 3, 4)
  moe_ref*.npz       reference moe_reference on the shapes of the reference's own
                     test (E=12, H=128, I=64, k=4, T in 1/3/40), fp32 and bf16 x
  moe_cfg1.npz       reference moe_reference on the tiny benchmark config (cfg1:
                     E=8, H=256, I=512, top-2, 64 tokens, 4-bit, block-128 scales
                     expanded to the layout's block 32), inputs from hex_data
  triton_interp.npz  the reference Triton fused kernel under TRITON_INTERPRET=1
                     (fp32 x: the interpreter is exact there)
"""

from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")
if "REF" not in os.environ:
    sys.exit("make_golden.py: set REF to the root of a BlackHole-Harness checkout (the reference implementation)")
REF = Path(os.environ["REF"])
sys.path[:0] = [str(REF / "runtime"), str(REF)]
HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1] / "blackhole-harness_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
from blackhole_runtime.hex_moe import HexTier, align, hex_moe_fused  # noqa: E402
from blackhole_runtime.hex_ref import hex_dequant, moe_reference, pack, random_parts  # noqa: E402

from blackhole_b200 import hex_data as hd  # noqa: E402

PARTS = ("idx", "block_scale", "expert_scale", "levels")


def digest(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(np.ascontiguousarray(t.cpu().numpy() if isinstance(t, torch.Tensor) else t).tobytes())
    return h.hexdigest()


def np_(t):
    t = t.cpu()
    if t.dtype == torch.uint32:
        t = t.view(torch.int32)
    if t.dtype == torch.bfloat16:
        t = t.float()
    return t.numpy()


def save(name, **arrays):
    np.savez_compressed(HERE / name, **arrays)
    print(f"wrote {name}: " + ", ".join(f"{k}{list(np.shape(v))}" for k, v in arrays.items()))


def fp8_kat():
    # 256 rows of one 32-input block, all codes 0 (level 1.0), row r scaled by fp8 code r
    words = torch.zeros(1, 256, 3, dtype=torch.int32).view(torch.uint32)
    bs = torch.arange(256, dtype=torch.int64).to(torch.uint8).reshape(1, 256, 1)
    lv = torch.ones(1, 8, dtype=torch.float32)
    W = hex_dequant(words, bs, torch.ones(1), lv, 3)                          # [1, 256, 32]
    save("fp8_kat.npz", table=np_(W[0, :, 0]))


def pack_case():
    out = {}
    g = torch.Generator().manual_seed(11)
    for bits in (3, 4):
        c = torch.randint(0, 2 ** bits, (3, 7, 96), generator=g)
        out[f"codes{bits}"] = c.to(torch.uint8).numpy()
        out[f"words{bits}"] = np_(pack(c, bits))
    save("pack.npz", **out)


def align_case():
    out = {}
    cases = [("fixed", torch.tensor([2, 0, 0, 2, 2, 1, 3, 0]), 4, 4)]
    g = torch.Generator().manual_seed(5)
    for S, n, bm in ((1, 12, 16), (7, 12, 4), (40, 12, 16), (300, 96, 16), (512, 96, 64), (1000, 8, 128),
                     (64, 3, 16), (2048, 128, 32)):
        cases.append((f"r{S}_{n}_{bm}", torch.randint(0, n, (S,), generator=g), n, bm))
    cases.append(("one_expert", torch.full((33,), 5), 8, 16))
    cases.append(("skip", torch.tensor([7, 7, 0, 7, 0, 7, 7, 7, 7, 7, 7, 7, 7, 7, 7, 7, 7, 7, 7]), 9, 16))
    for name, ids, n, bm in cases:
        sid, eid, npp = align(ids, n, bm)
        out[f"{name}_ids"] = ids.numpy().astype(np.int64)
        out[f"{name}_meta"] = np.array([n, bm], np.int64)
        out[f"{name}_sid"] = np_(sid)
        out[f"{name}_eid"] = np_(eid)
        out[f"{name}_npp"] = np_(npp)
    save("align.npz", **out)


def dequant_case():
    for bits in (3, 4):
        p = random_parts(3, 20, 96, bits, seed=40 + bits)
        W = hex_dequant(*(p[q] for q in PARTS), bits)
        save(f"dequant_b{bits}.npz", **{q: np_(p[q]) for q in PARTS}, W=np_(W))


def make_tiers(E, H, I, split, bits, seed):
    """The reference test's tier builder (runtime/tests/test_hex_moe.py:19-29)."""
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(E, generator=g)
    groups = [perm[:split], perm[split:]] if split else [perm]
    tiers = []
    for i, (ids, b) in enumerate(zip(groups, bits)):
        n = len(ids)
        tiers.append({"bits": b, "experts": ids,
                      "gate_proj": random_parts(n, I, H, b, seed=seed + 10 * i + 1),
                      "up_proj": random_parts(n, I, H, b, seed=seed + 10 * i + 2),
                      "down_proj": random_parts(n, H, I, b, seed=seed + 10 * i + 3)})
    return tiers


def routing(T, E, k, seed):
    g = torch.Generator().manual_seed(seed)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    w = torch.softmax(torch.randn(T, k, generator=g), -1)
    return ids, w


def flat_tiers(tiers):
    out = {}
    for ti, t in enumerate(tiers):
        out[f"t{ti}_bits"] = np.array(t["bits"])
        out[f"t{ti}_experts"] = t["experts"].numpy().astype(np.int64)
        for proj in ("gate_proj", "up_proj", "down_proj"):
            for q in PARTS:
                out[f"t{ti}_{proj}_{q}"] = np_(t[proj][q])
    out["ntiers"] = np.array(len(tiers))
    return out


def moe_ref_cases():
    E, H, I, k = 12, 128, 64, 4
    for T, split in ((1, 0), (3, 5), (40, 4)):
        tiers = make_tiers(E, H, I, split, (4, 3) if split else (3,), seed=T)
        ids, w = routing(T, E, k, seed=T)
        g = torch.Generator().manual_seed(100 + T)
        x32 = torch.randn(T, H, generator=g) * 0.5
        xb = x32.to(torch.bfloat16)
        ref32 = moe_reference(x32, w, ids, tiers)
        refb = moe_reference(xb, w, ids, tiers)
        save(f"moe_ref_T{T}.npz", **flat_tiers(tiers), x32=np_(x32), xbf16=np_(xb), w=np_(w),
             ids=ids.numpy().astype(np.int64), E=np.array(E), out_f32=np_(ref32), out_bf16=np_(refb))


def moe_cfg1():
    c = hd.CONFIGS["cfg1"]
    E, H, I, k, T, block = c["E"], c["H"], c["I"], c["k"], c["T"][0], c["block"]
    L = hd.synth_layer(E, H, I, c["bits"], block, seed=1)
    w, ids = hd.synth_routing(T, E, k, seed=2)
    x = hd.synth_x(T, H, seed=3)
    ref_tiers = []
    dig = []
    for t in L.tiers:
        dig.append(digest(*(t[p][q] for p in ("gate_proj", "up_proj", "down_proj") for q in PARTS), t["experts"]))
        rt = {"bits": t["bits"], "experts": t["experts"].long()}
        for p in ("gate_proj", "up_proj", "down_proj"):
            rt[p] = dict(t[p])
            rt[p]["block_scale"] = hd.expand_block_scale(t[p]["block_scale"], block)
        ref_tiers.append(rt)
    ref = moe_reference(x, w, ids, ref_tiers)
    Wg0 = hex_dequant(*(ref_tiers[0]["gate_proj"][q] for q in PARTS), ref_tiers[0]["bits"])
    save("moe_cfg1.npz", tier_digests=np.array(dig), x_digest=np.array(digest(x.float())),
         route_digest=np.array(digest(w, ids)), out_bf16=np_(ref),
         gate0_rows=np_(Wg0[:, :4]), gate0_sum=np.array(float(Wg0.double().sum())),
         seeds=np.array([1, 2, 3]))


def triton_interp():
    E, H, I, k, T = 12, 128, 64, 4, 3
    tiers = make_tiers(E, H, I, 5, (4, 3), seed=7)
    ids, w = routing(T, E, k, seed=7)
    g = torch.Generator().manual_seed(77)
    x = torch.randn(T, H, generator=g) * 0.5
    run = [HexTier(t["bits"], t["experts"], *(dict(t[p]) for p in ("gate_proj", "up_proj", "down_proj"))).prepare(E)
           for t in tiers]
    small = {"BLOCK_M": 16, "BLOCK_N": 32, "BLOCK_K": 32, "num_warps": 4, "num_stages": 1}
    got = hex_moe_fused(x, w, ids, run, small, align_mode="torch")
    save("triton_interp.npz", **flat_tiers(tiers), x32=np_(x), w=np_(w), ids=ids.numpy().astype(np.int64),
         E=np.array(E), out=np_(got), ref=np_(moe_reference(x, w, ids, tiers)))


if __name__ == "__main__":
    torch.set_num_threads(os.cpu_count() or 1)
    fp8_kat()
    pack_case()
    align_case()
    dequant_case()
    moe_ref_cases()
    moe_cfg1()
    triton_interp()
