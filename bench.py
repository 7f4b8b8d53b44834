"""Benchmark of the HEX fused-MoE layer on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--no-extras]

Headline workload: the prefill config that runs on 1, 2, 4 and 8 GPUs (cfg3): a
Qwen3-30B-A3B REAP-25% MoE layer, 96 experts, hidden 2048, moe_intermediate 768,
top-8, SwiGLU, half the experts (seeded) 4-bit / 16-level and half 3-bit /
8-level HEX with fp8 e4m3 scales per 128 inputs, 4096 tokens per GPU.  At N=1
one step is the single-GPU layer (hexmoe_forward: align plan, gather, gate/up
GEMM with SwiGLU, down GEMM with the top-k weight, combine); at N>1 it is the
expert-parallel layer (hexmoe_ep_forward: experts sharded 96/N per GPU, token
rows pulled by their experts' GPUs over NVLink peer memory, every slot's output
row stored back into its home GPU by the down GEMM), value = all ranks' tokens
over the slowest rank's time.
Synthetic seeded data (blackhole_b200.hex_data): no dataset exists on this
path.  Steps are replayed from a CUDA graph with inputs in HBM, timed with CUDA
events on the launching stream; between timed steps a 256 MiB buffer is
written and a second one read (cold L2, 126 MB, holding no dirty lines that the
step would have to write back: a decode step follows other layers' weight reads,
which leave clean lines).  `e2e` is the same step through the public API
(hex_moe / EPMoE) with the inputs copied from pinned host memory and the
output copied back inside the timed region.  `roofline` is for the dominant
kernel, the gate/up grouped GEMM of the 1-GPU layer, timed alone (tensor-bound).

Other objects of the line: `decode` (cfg2: all-3-bit, T = 64 with the decode
roofline against HBM, and the 1/8/32/64 sweep), `prefill_T16384` (cfg3 at
16384 tokens on one GPU), `cfg4_slice` (one GPU's share of cfg4 at 8 GPUs: 16
experts of H=4096, I=1536, 1024 tokens routed over them), `quantize` (the GPU
HEX quantizer on 96 matrices of 768 x 2048 against the numpy restatement of the
reference's quantize on one); at N>1 `ep` (per-phase
times, per-rank expert time, and a bit-exactness check of rank 0's output),
`cfg4_ep` and `cfg5_ep` (cfg4: 128 experts of H=4096, 8192 tokens over the
GPUs, 16 experts per GPU at N=8; cfg5: Zipf-skewed routing, 32768 tokens over
the GPUs; each with per-rank expert time).  `cpu_baseline`: the oracle (a C restatement of the reference's
moe_reference) on the host cores over a bounded sample of the headline.
`gpu_reference`: the reference's own Triton hex_moe on the same GPU, when a copy
of it is installed under baseline/_ref.

--impl reference times the reference's CPU implementation of the path (the
oracle port of hex_ref.moe_reference, all host threads) on the headline config;
each step is a bounded sample: a fixed slice of the batch's tokens through every
expert, dequantized per call as moe_reference does.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT / "blackhole-harness_b200"), str(ROOT / "oracle")]

METRIC = "HEX MoE layer tokens/s (decode & prefill) and % of HBM / bf16 roofline, 1/2/4/8 B200"
E, H, I, K_TOP, BLOCK = 96, 2048, 768, 8, 128
T_PREFILL = 4096
FLUSH_BYTES = 256 << 20


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


class Clocks:
    """SM clock and throttle-reason sampling (NVML) on a thread, each sample time-
    stamped, so the samples inside a timed window can be picked out afterwards."""
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index: int):
        import threading
        self.samples = []
        self.stop_ev = threading.Event()
        self.thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001  (no NVML: no clock record)
            self.nv = None
            return
        self.thread = threading.Thread(target=self._run, daemon=True)
        self.thread.start()

    def _run(self):
        nv = self.nv
        pw, i = 0.0, 0
        while not self.stop_ev.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                if i % 10 == 0:     # the power query is the slow one: every tenth sample
                    pw = nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
                self.samples.append((time.perf_counter(), sm, rs, pw))
                i += 1
            except Exception:  # noqa: BLE001
                pass
            self.stop_ev.wait(0.0002)

    def stop(self, window: tuple[float, float] | None = None) -> dict | None:
        """Summary of the samples (those inside `window` = (t0, t1) perf_counter
        seconds, when given and any fall inside it)."""
        if self.thread is None:
            return None
        self.stop_ev.set()
        self.thread.join(timeout=2)
        smp = self.samples
        if window:
            inside = [s for s in smp if window[0] <= s[0] <= window[1]]
            smp = inside or smp
        if not smp:
            return None
        sm = [s[1] for s in smp]
        loaded = [x for x in sm if x > 0.5 * self.max_mhz] or sm
        reasons = sorted({name for _, _, rs, _ in smp for bit, name in self.REASONS.items() if rs & bit})
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(sm), "power_w_max": max(s[3] for s in smp)}


def graphed(fn):
    """Capture fn (a launch sequence with no host synchronisation) into a CUDA graph."""
    import torch
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def time_steps(fn, steps: int, flush, stream) -> list[float]:
    """ms of each of `steps` calls of fn, CUDA events on `stream`, L2 flushed before each."""
    import torch
    times = []
    for _ in range(steps):
        flush()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        times.append((a, b))
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in times]


def max_over_ranks(ms: float, world: int, dev) -> float:
    if world == 1:
        return ms
    import torch
    import torch.distributed as dist
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def build_tiers(layer_tiers, num_experts: int):
    from blackhole_b200.hex_moe import HexTier
    return [HexTier(t["bits"], t["experts"], t["gate_proj"], t["up_proj"], t["down_proj"]).prepare(num_experts)
            for t in layer_tiers]


def weight_bytes(tiers_bits: dict, block: int, H_: int, I_: int, projections: int = 3) -> float:
    """HBM bytes of `projections` HEX projections of each routed expert (bits -> count)."""
    total = 0.0
    for bits, n in tiers_bits.items():
        per = projections * (H_ * I_ * bits / 8 + H_ * I_ / block + 4 * 2 ** bits + 4)
        total += per * n
    return total


def routed_bits(L, ids) -> dict:
    used = set(ids.reshape(-1).tolist())
    out = {}
    for t in L.tiers:
        n = sum(1 for e in t["experts"].tolist() if e in used)
        out[t["bits"]] = out.get(t["bits"], 0) + n
    return out


def moe_flops(tokens: int, k: int, H_: int, I_: int, projections: int = 3) -> float:
    """Algorithmic FLOPs of the routed experts: 2 * slots * projections * H * I (padding not counted)."""
    return 2.0 * tokens * k * projections * H_ * I_


# ---------------------------------------------------------------------------- CPU (oracle) arms
def _oracle_layer(L, keep_experts=None):
    """hexoracle.Layer over a synthetic layer's tiers (numpy views)."""
    import numpy as np
    import torch

    import hexoracle
    tiers = []
    for t in L.tiers:
        d = {"bits": t["bits"], "experts": t["experts"].cpu().numpy().astype(np.int64)}
        for p in ("gate_proj", "up_proj", "down_proj"):
            d[p] = {q: (v.view(torch.int32) if v.dtype == torch.uint32 else v).cpu().numpy() for q, v in t[p].items()}
        tiers.append(d)
    return hexoracle.Layer(tiers, L.E, L.H, L.I, L.block)


def headline_inputs(rank: int = 0, T: int = T_PREFILL, device="cpu"):
    from blackhole_b200 import hex_data as hd
    w, ids = hd.synth_routing(T, E, K_TOP, seed=5 + 1000 * rank, device=device)
    x = hd.synth_x(T, H, seed=6 + 1000 * rank, device=device)
    return x, w, ids


def cpu_baseline(sample_tokens: int = 32, reps: int = 2) -> dict:
    """The oracle (C port of hex_ref.moe_reference) on this host's cores, on a bounded
    sample of the headline workload: `sample_tokens` of the 4096 tokens through
    the layer, every expert dequantized per call as the reference does."""
    import hexoracle
    from blackhole_b200 import hex_data as hd
    threads = hexoracle.set_threads(os.cpu_count())
    L = hd.synth_layer(E, H, I, "mixed", BLOCK, seed=3)
    x, w, ids = headline_inputs()
    xs, ws, ids_s = x[:sample_tokens].float().numpy(), w[:sample_tokens].numpy(), ids[:sample_tokens].numpy()
    layer = _oracle_layer(L)
    layer.forward(xs, ws, ids_s)                        # warm-up (page-in)
    t0 = time.perf_counter()
    for _ in range(reps):
        layer.forward(xs, ws, ids_s)
    dt = (time.perf_counter() - t0) / reps
    layer.forward(xs, ws, ids_s, cache_weights=True)    # fills the dequantized cache
    t1 = time.perf_counter()
    for _ in range(reps):
        layer.forward(xs, ws, ids_s, cache_weights=True)
    dt_mm = (time.perf_counter() - t1) / reps
    return {"value": sample_tokens / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{sample_tokens} of the {T_PREFILL} cfg3 prefill tokens per call (top-{K_TOP}, all {E} mixed "
                      "3/4-bit experts dequantized every call as hex_ref.moe_reference does)",
            "seconds_per_call": dt, "matmul_only_tokens_per_s": sample_tokens / dt_mm}


def reference_arm(args) -> None:
    """--impl reference: the reference's CPU path (oracle port of moe_reference) on
    the host cores, on the headline config; rank 0 alone."""
    import hexoracle
    from blackhole_b200 import hex_data as hd
    if int(os.environ.get("RANK", "0")) != 0:
        return
    threads = hexoracle.set_threads(os.cpu_count())
    L = hd.synth_layer(E, H, I, "mixed", BLOCK, seed=3)
    x, w, ids = headline_inputs()
    layer = _oracle_layer(L)
    per = 32
    slices = T_PREFILL // per

    def step(s):
        sl = slice((s % slices) * per, (s % slices + 1) * per)
        layer.forward(x[sl].float().numpy(), w[sl].numpy(), ids[sl].numpy())

    for s in range(args.warmup):
        step(s)
    secs = 0.0
    for s in range(args.steps):
        t0 = time.perf_counter()
        step(s)
        secs += time.perf_counter() - t0
    value = per * args.steps / secs
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": secs / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": f"cfg3 prefill: E={E} H={H} I={I} top-{K_TOP}, mixed 3/4-bit HEX, fp8 block-{BLOCK} "
                                   f"scales, {T_PREFILL} tokens", "tokens": T_PREFILL, "parallelism": "host cores"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"each step: {per} of the {T_PREFILL} tokens (a rotating slice) through all {E} "
                                       "experts, dequantized and multiplied as hex_ref.moe_reference"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- one-GPU measurements
def gate_up_alone(layer, x, w, ids, bm: int, steps: int, flush, stream):
    """ms per launch of the gate/up grouped GEMM alone (graph-replayed, L2 flushed)."""
    T, k = ids.shape
    plan = layer.plan(ids, bm)
    xs = layer.gather(x, k, plan, bm)
    act = layer.gate_up(xs, T, k, plan, bm)
    g = graphed(lambda: layer.gate_up(xs, T, k, plan, bm, act))
    for _ in range(3):
        g.replay()
    ms = time_steps(g.replay, steps, flush, stream)
    return sum(ms) / len(ms)


def layer_step_ms(layer, x, w, ids, bm: int, steps: int, flush, stream, warmup: int = 3) -> float:
    g = graphed(lambda: layer.forward(x, w, ids, bm))
    for _ in range(warmup):
        g.replay()
    ms = time_steps(g.replay, steps, flush, stream)
    return sum(ms) / len(ms)


def prefill_one_gpu(dev, layer, T: int, steps: int, flush, stream, pk, seed: int = 50) -> dict:
    from blackhole_b200 import hex_data as hd
    w, ids = hd.synth_routing(T, E, K_TOP, seed=seed, device=dev)
    x = hd.synth_x(T, H, seed=seed + 1, device=dev)
    t = layer_step_ms(layer, x, w, ids, 128, steps, flush, stream)
    fl = moe_flops(T, K_TOP, H, I)
    return {"workload": f"cfg3 prefill: E={E} H={H} I={I} top-{K_TOP}, mixed 3/4-bit HEX, fp8 block-{BLOCK} scales, "
                        f"T={T}, 1 GPU", "tokens_per_s": T / (t * 1e-3), "ms": t, "TFLOPs": fl / t / 1e9,
            "bf16_frac": fl / t / 1e9 / pk["bf16_tflops"]}


def decode_block(dev, steps: int, flush, stream, pk) -> dict:
    """cfg2 decode: all-3-bit 96-expert layer, T = 64 (roofline against HBM: the
    gate/up kernel alone and the whole layer), and the 1/8/32/64 sweep."""
    from blackhole_b200 import hex_data as hd
    from blackhole_b200.hex_moe import layer_for
    L = hd.synth_layer(E, H, I, "3", BLOCK, seed=0, device=dev)
    layer = layer_for(build_tiers(L.tiers, E))
    from blackhole_b200.hex_moe import auto_block_m
    out = {"workload": f"cfg2 decode: E={E} H={H} I={I} top-{K_TOP}, 3-bit/8-level HEX, fp8 block-{BLOCK} scales, "
                       "1 GPU, automatic tile height (8: the small-batch kernels, up to 8 slots per expert)",
           "sweep": {}}
    for T in (1, 8, 32, 64):
        w, ids = hd.synth_routing(T, E, K_TOP, seed=1 if T == 64 else 10 + T, device=dev)
        x = hd.synth_x(T, H, seed=2 if T == 64 else 20 + T, device=dev)
        bm = auto_block_m(T * K_TOP, E)
        t = layer_step_ms(layer, x, w, ids, bm, steps, flush, stream)
        rb = routed_bits(L, ids.cpu())
        byts = weight_bytes(rb, BLOCK, H, I) + 2 * T * H * 2 + T * K_TOP * 12
        out["sweep"][f"T={T}"] = {"tokens_per_s": T / (t * 1e-3), "us": t * 1e3, "experts_routed": sum(rb.values()),
                                  "block_m": bm, "GBps": byts / t / 1e6, "hbm_frac": byts / t / 1e6 / pk["hbm_gbs"]}
        if T == 64:
            gu = gate_up_alone(layer, x, w, ids, bm, steps, flush, stream)
            gu_bytes = weight_bytes(rb, BLOCK, H, I, projections=2) + T * K_TOP * (H + I) * 2
            out.update({"tokens": T, "tokens_per_s": T / (t * 1e-3), "ms": t, "experts_routed": sum(rb.values()),
                        "block_m": bm,
                        "roofline": {"bound": "hbm", "kernel": "gate/up grouped GEMM (hex_decode_kernel<GLU> at block_m 8)",
                                     "ms": gu,
                                     "algorithmic_bytes": gu_bytes, "achieved": gu_bytes / gu / 1e6,
                                     "peak": pk["hbm_gbs"], "unit": "GB/s",
                                     "frac": gu_bytes / gu / 1e6 / pk["hbm_gbs"],
                                     "peak_src": pk["src"] + " (hbm_gbs)",
                                     "traffic": read_traffic("gate_up_cfg2_T64_dram_bytes"),
                                     "layer_bytes": byts, "layer_achieved_gbs": byts / t / 1e6,
                                     "layer_frac": byts / t / 1e6 / pk["hbm_gbs"]}})
    return out


def cfg4_slice(dev, steps: int, flush, stream, pk) -> dict:
    """One GPU's share of cfg4 at 8 GPUs: 16 of the 128 experts (H=4096, I=1536,
    mixed 3/4-bit, block-128 scales) with 1024 tokens routed top-8 over them."""
    from blackhole_b200 import hex_data as hd
    from blackhole_b200.hex_moe import layer_for
    E4, H4, I4, T4 = 16, 4096, 1536, 1024
    L = hd.synth_layer(E4, H4, I4, "mixed", BLOCK, seed=44, device=dev)
    layer = layer_for(build_tiers(L.tiers, E4))
    w, ids = hd.synth_routing(T4, E4, K_TOP, seed=45, device=dev)
    x = hd.synth_x(T4, H4, seed=46, device=dev)
    t = layer_step_ms(layer, x, w, ids, 128, steps, flush, stream)
    fl = moe_flops(T4, K_TOP, H4, I4)
    return {"workload": "cfg4 per-GPU slice: 16 experts H=4096 I=1536 top-8 over them, mixed 3/4-bit, 1024 tokens",
            "tokens_per_s": T4 / (t * 1e-3), "ms": t, "TFLOPs": fl / t / 1e9, "bf16_frac": fl / t / 1e9 / pk["bf16_tflops"]}


def quantize_block(dev, steps: int, flush, stream, pk) -> dict:
    """The GPU HEX quantizer (hexmoe_quantize) on a stack shaped as cfg2's gate
    projections (96 experts of 768 x 2048, 8 levels, 128-input scale blocks,
    the reference's 2^17-value fit sample), against the reference algorithm
    restated in numpy (oracle/hexquant.py) on one of the matrices."""
    import torch

    import hexquant
    from blackhole_b200.quant import quantize_stack
    g = torch.Generator(device="cpu").manual_seed(81)
    W = (torch.randn(E, I, H, generator=g) * 0.02).to(dev)
    quantize_stack(W[:2], 8, BLOCK)                     # warm-up (and the cub sort's first launch)
    torch.cuda.synchronize()
    ms = time_steps(lambda: quantize_stack(W, 8, BLOCK), max(3, steps // 4), flush, stream)
    t = sum(ms) / len(ms)
    w0 = W[0].cpu().numpy()
    t0 = time.perf_counter()
    hexquant.quantize(w0, 8, BLOCK)
    cpu_s = time.perf_counter() - t0
    nbytes = W.numel() * 4
    return {"workload": f"quantize {E} matrices of {I}x{H} (cfg2 gate projections), 8 levels, fp8 block-{BLOCK} scales, "
                        "k-means on the reference's 2^17-value sample, 20 iterations",
            "ms": t, "matrices_per_s": E / (t * 1e-3), "input_GBps": nbytes / t / 1e6,
            "cpu_numpy_s_per_matrix": cpu_s, "cpu_numpy_matrices_per_s": 1.0 / cpu_s}


def read_traffic(key: str):
    """DRAM bytes per launch of a kernel from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get(key)
        except (ValueError, AttributeError):
            return None
    return None


# ---------------------------------------------------------------------------- expert parallelism
def make_ep(dev, rank: int, world: int, L, num_experts: int, hidden: int, max_tokens: int):
    from blackhole_b200.ep import EPMoE, ExpertShard, shard_tiers
    shard = ExpertShard(num_experts, rank, world)
    local = build_tiers(shard_tiers(L.tiers, shard), num_experts)
    return EPMoE(shard, local, block_m=128, max_tokens=max_tokens, topk=K_TOP, hidden=hidden), shard


def ep_phases(ep, x, w, ids, dev, world: int, reps: int = 5) -> dict:
    """Per-phase ms (dispatch / experts / combine) of eager EP forwards, this rank's
    mean, and every rank's expert-phase ms (all ranks take part)."""
    import torch
    import torch.distributed as dist
    acc = torch.zeros(3, dtype=torch.float64)
    for _ in range(reps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ep(x, w, ids, events=ev)
        torch.cuda.synchronize()
        acc += torch.tensor([ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]), ev[2].elapsed_time(ev[3])],
                            dtype=torch.float64)
    mine = (acc / reps).to(dev)
    every = [torch.zeros_like(mine) for _ in range(world)]
    dist.all_gather(every, mine)
    per_rank = [[round(float(v), 4) for v in t.cpu()] for t in every]
    return {"dispatch_ms": float(mine[0]), "experts_ms": float(mine[1]), "combine_ms": float(mine[2]),
            "per_rank_dispatch_experts_combine_ms": per_rank}


def ep_run(dev, rank: int, world: int, L, num_experts: int, hidden: int, inter: int, T: int, steps: int, flush,
           stream, pk, seed: int, zipf=None, label: str = "") -> tuple[dict, object]:
    """One EP workload: max-over-ranks ms per graph-replayed step and phase times."""
    import torch
    import torch.distributed as dist

    from blackhole_b200 import hex_data as hd
    ep, shard = make_ep(dev, rank, world, L, num_experts, hidden, T)
    w, ids = hd.synth_routing(T, num_experts, K_TOP, seed=seed + 1000 * rank, zipf=zipf, device=dev)
    x = hd.synth_x(T, hidden, seed=seed + 1 + 1000 * rank, device=dev)
    for _ in range(2):
        ep(x, w, ids)
    g = graphed(lambda: ep(x, w, ids))
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    ms = time_steps(g.replay, steps, flush, stream)
    step = max_over_ranks(sum(ms) / len(ms), world, dev)
    ph = ep_phases(ep, x, w, ids, dev, world)
    fl = moe_flops(T * world, K_TOP, hidden, inter)
    res = {"workload": label, "tokens_per_s": world * T / (step * 1e-3), "ms": step, "TFLOPs": fl / step / 1e9,
           "bf16_frac_per_gpu": fl / world / step / 1e9 / pk["bf16_tflops"], "scaling": "weak", **ph}
    del g
    torch.cuda.synchronize()
    return res, (ep, shard, x, w, ids)


def ep_bit_check(L, ep_state, got) -> dict:
    """Rank 0: `got`, the EP output of its tokens (from a forward every rank
    made), against the plain single-GPU layer on the same tokens (bit for bit,
    and the max abs difference)."""
    import torch

    from blackhole_b200.hex_moe import layer_for
    ep, shard, x, w, ids = ep_state
    full = layer_for(build_tiers(L.tiers, L.E))
    plain = full.forward(x, w, ids, 128)
    torch.cuda.synchronize()
    d = (got.float() - plain.float()).abs()
    return {"bit_equal_single_gpu_layer": bool(torch.equal(got, plain)), "tokens_checked": int(x.shape[0]),
            "max_abs_err_vs_single_gpu_layer": float(d.max())}


# ---------------------------------------------------------------------------- the reference's GPU kernel
def gpu_reference(dev, steps: int, flush, stream) -> dict:
    """The reference's own Triton path (runtime/blackhole_runtime/hex_moe.py, an
    unmodified copy installed under baseline/_ref) on the same GPU and the same
    synthetic layers and routings: hex_moe(path="fused") replayed from a CUDA
    graph (as its hex_check.timeit does) and path="dequant" (its prefill path:
    every expert to bf16, then vLLM's fused_experts) eagerly, L2 flushed between
    steps.  Its layout fixes 32-input scale blocks, so the block-128 codes are
    repeated 4x along the inputs (identical weights).  Context only: nothing of
    this repository runs on this path."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "blackhole_runtime" / "hex_moe.py").exists():
        return {"unavailable": "the reference runtime is not installed under baseline/_ref"}
    import torch
    sys.path.insert(0, str(ref))
    try:
        from blackhole_runtime import hex_moe as rh
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"import failed: {type(e).__name__}: {e}"}
    from blackhole_b200 import hex_data as hd
    out = {"source": "baseline/_ref/blackhole_runtime/hex_moe.py (reference, unmodified)"}

    def ref_tiers(L):
        ts = []
        for t in L.tiers:
            parts = []
            for p in ("gate_proj", "up_proj", "down_proj"):
                d = {q: v.clone() for q, v in t[p].items()}
                d["block_scale"] = hd.expand_block_scale(d["block_scale"], L.block)
                parts.append(d)
            ts.append(rh.HexTier(t["bits"], t["experts"].clone(), *parts).prepare(L.E))
        return ts

    def timed(fn, graph: bool) -> float:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        run = graphed(fn).replay if graph else fn
        return sum(time_steps(run, steps, flush, stream)) / steps

    cases = (("cfg3_prefill_T4096", "mixed", 3, T_PREFILL, (("fused", True), ("dequant", False))),
             ("cfg2_decode_T64", "3", 0, 64, (("fused", True),)))
    for name, bits, seed, T, paths in cases:
        try:
            L = hd.synth_layer(E, H, I, bits, BLOCK, seed=seed, device=dev)
            tiers = ref_tiers(L)
            if T == T_PREFILL:
                x, w, ids = headline_inputs(0, T, dev)
            else:
                w, ids = hd.synth_routing(T, E, K_TOP, seed=1, device=dev)
                x = hd.synth_x(T, H, seed=2, device=dev)
            res = {}
            for path, graph in paths:
                try:
                    ms = timed(lambda: rh.hex_moe(x, w, ids, tiers, path=path), graph)
                    res[path] = {"ms": ms, "tokens_per_s": T / (ms * 1e-3)}
                except Exception as e:  # noqa: BLE001
                    res[path] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
            out[name] = res
            del tiers, L
            torch.cuda.empty_cache()
        except Exception as e:  # noqa: BLE001
            out[name] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    return out


# ---------------------------------------------------------------------------- main
def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=("b200", "reference"))
    ap.add_argument("--no-extras", action="store_true", help="headline, e2e and roofline only")
    ap.add_argument("--profile", nargs="?", const="prefill", choices=("prefill", "decode"),
                    help="a few eager steps only (for ncu): the headline prefill layer, or the cfg2 T=64 decode layer")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        reference_arm(args)
        return

    import torch
    import torch.distributed as dist

    from blackhole_b200.hex_moe import device_status, hex_moe, layer_for
    from blackhole_b200 import hex_data as hd

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        os.environ.setdefault("NCCL_DEBUG", "WARN")     # stdout carries the JSON line only
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    pk = peaks()
    stream = torch.cuda.current_stream(dev)
    flush_buf = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)
    flush_read = torch.ones(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def flush():
        flush_buf.fill_(rank & 0xFF)
        flush_read.sum()

    if args.profile == "decode":
        from blackhole_b200.hex_moe import auto_block_m
        Ld = hd.synth_layer(E, H, I, "3", BLOCK, seed=0, device=dev)
        lay_d = layer_for(build_tiers(Ld.tiers, E))
        wd, idd = hd.synth_routing(64, E, K_TOP, seed=1, device=dev)
        xd = hd.synth_x(64, H, seed=2, device=dev)
        for _ in range(args.warmup):
            lay_d.forward(xd, wd, idd, auto_block_m(64 * K_TOP, E))
        torch.cuda.synchronize()
        return

    # ---- the headline step: cfg3 prefill, 4096 tokens per GPU
    T = T_PREFILL
    L3 = hd.synth_layer(E, H, I, "mixed", BLOCK, seed=3, device=dev)
    x, w, ids = headline_inputs(rank, T, dev)
    layer, tiers3, ep, shard = None, None, None, None
    if world == 1:
        tiers3 = build_tiers(L3.tiers, E)
        layer = layer_for(tiers3)

        def step_fn():
            return layer.forward(x, w, ids, 128)
        launches = 7       # align (count, plan, scatter), gather, gate/up, down, combine
        par = "1 GPU"
    else:
        ep, shard = make_ep(dev, rank, world, L3, E, H, T)

        def step_fn():
            return ep(x, w, ids)
        launches = 12      # plan, send, wait, align x3, gather, gate/up, down, return, wait, combine
        par = f"expert parallel x{world}: {E // world} experts per GPU, token rows over NVLink peer memory"
    if args.profile:
        for _ in range(args.warmup):
            step_fn()
        torch.cuda.synchronize()
        return
    clocks = Clocks(local)
    for _ in range(args.warmup):
        step_fn()
    g_step = graphed(step_fn)
    for _ in range(args.warmup):
        g_step.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    ms = time_steps(g_step.replay, args.steps, flush, stream)
    t1 = time.perf_counter()
    clk = clocks.stop(window=(t0, t1))
    step_ms = max_over_ranks(sum(ms) / len(ms), world, dev)
    value = world * T / (step_ms * 1e-3)

    # ---- e2e through the public API: pinned host inputs in, output back, each step
    xh, wh, ih = x.cpu().pin_memory(), w.cpu().pin_memory(), ids.cpu().pin_memory()
    oh = torch.empty(T, H, dtype=x.dtype).pin_memory()

    def e2e_step():
        xd = xh.to(dev, non_blocking=True)
        wd = wh.to(dev, non_blocking=True)
        idd = ih.to(dev, non_blocking=True)
        out = hex_moe(xd, wd, idd, tiers3, {"BLOCK_M": 128}) if world == 1 else ep(xd, wd, idd)
        oh.copy_(out, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2e_ms = time_steps(e2e_step, args.steps, flush, stream)
    e2e_step_ms = max_over_ranks(sum(e2e_ms) / len(e2e_ms), world, dev)
    h2d = xh.numel() * xh.element_size() + wh.numel() * 4 + ih.numel() * ih.element_size()
    d2h = oh.numel() * oh.element_size()

    extras = {}
    # ---- expert parallelism: phases, per-rank expert time, rank 0's bit check (all ranks take part)
    if world > 1:
        got = ep(x, w, ids)
        torch.cuda.synchronize()
        ph = ep_phases(ep, x, w, ids, dev, world)
        extras["ep"] = {"workload": f"cfg3 prefill, {E // world} experts and {T} tokens per GPU", **ph}
        if rank == 0:
            extras["ep"]["check"] = ep_bit_check(L3, (ep, shard, x, w, ids), got)
        if not args.no_extras:
            L4 = hd.synth_layer(128, 4096, 1536, "mixed", BLOCK, seed=44, device=dev)
            r4, st4 = ep_run(dev, rank, world, L4, 128, 4096, 1536, 8192 // world, args.steps, flush, stream, pk, 61,
                             label=f"cfg4: 128 experts H=4096 I=1536 top-8 mixed 3/4-bit, {128 // world} per GPU, "
                                   f"8192 tokens ({8192 // world} per GPU)")
            st4[0].close()
            del L4, st4
            L5 = hd.synth_layer(E, H, I, "3", BLOCK, seed=9, device=dev)
            r5, st5 = ep_run(dev, rank, world, L5, E, H, I, 32768 // world, args.steps, flush, stream, pk, 71,
                             zipf=1.2, label=f"cfg5: 96 experts 3-bit, Zipf(1.2) routing skew, 32768 tokens "
                                             f"({32768 // world} per GPU), {E // world} experts per GPU")
            st5[0].close()
            del L5, st5
            extras["cfg4_ep"], extras["cfg5_ep"] = r4, r5
            torch.cuda.empty_cache()

    # ---- the dominant kernel alone: gate/up grouped GEMM of the one-GPU layer (rank 0)
    roof = None
    if rank == 0:
        if layer is None:
            tiers3 = build_tiers(L3.tiers, E)
            layer = layer_for(tiers3)
        gu = gate_up_alone(layer, x, w, ids, 128, args.steps, flush, stream)
        gfl = moe_flops(T, K_TOP, H, I, projections=2)
        roof = {"bound": "tensor", "kernel": "hex_gemm_kernel<GLU> (gate/up), cfg3 T=4096, 1 GPU",
                "achieved": gfl / gu / 1e9, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": gfl / gu / 1e9 / pk["bf16_tflops"], "traffic": read_traffic("gate_up_cfg3_T4096_dram_bytes"),
                "peak_src": pk["src"] + " (bf16_tflops, burst: the kernel is timed alone)", "ms": gu,
                "algorithmic_flops": gfl}
        if world == 1:
            fl = moe_flops(T, K_TOP, H, I)
            roof.update({"layer_TFLOPs": fl / step_ms / 1e9, "layer_frac": fl / step_ms / 1e9 / pk["bf16_tflops"]})
        if world == 1 and not args.no_extras:
            extras["decode"] = decode_block(dev, max(args.steps, 10), flush, stream, pk)
            extras["prefill_T16384"] = prefill_one_gpu(dev, layer, 16384, max(5, args.steps // 2), flush, stream, pk)
            extras["cfg4_slice"] = cfg4_slice(dev, max(5, args.steps // 2), flush, stream, pk)
            try:
                extras["quantize"] = quantize_block(dev, args.steps, flush, stream, pk)
            except Exception as e:  # noqa: BLE001  (reported, not required)
                extras["quantize"] = {"error": f"{type(e).__name__}: {e}"}
            torch.cuda.empty_cache()
            try:
                extras["cpu_baseline"] = cpu_baseline()
            except Exception as e:  # noqa: BLE001  (the baseline is reported, not required)
                extras["cpu_baseline"] = {"value": None, "error": f"{type(e).__name__}: {e}"}
            extras["gpu_reference"] = gpu_reference(dev, max(5, args.steps // 2), flush, stream)
    err = device_status(local)
    del g_step
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"cfg3 prefill: E={E} H={H} I={I} top-{K_TOP}, SwiGLU, mixed 3/4-bit HEX (half the "
                                   f"experts each), fp8 e4m3 block-{BLOCK} scales, {T} tokens per GPU",
                       "tokens": T, "block_m": 128, "parallelism": par,
                       "l2": "flushed between timed steps (256 MiB written, then 256 MiB read)", "timed_wall_s": t1 - t0},
            "e2e": {"value": world * T / (e2e_step_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_step_ms},
            "gpu_launches": launches * args.steps, "roofline": roof, "clocks": clk, "device_error_word": err,
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    if ep is not None:
        ep.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
