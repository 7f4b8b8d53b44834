"""Benchmark of the HEX fused-MoE layer on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T] [--impl b200|reference]

Workload (the metric's decode config, on one GPU): a Qwen3-30B-A3B REAP-25% MoE
layer, 96 experts, hidden 2048, moe_intermediate 768, top-8, SwiGLU, every
expert 3-bit / 8-level HEX with fp8 e4m3 scales per 128 inputs, T = 64 tokens
(the largest point of the 1/8/32/64 decode sweep; the other points are
reported under "sweep").  Synthetic seeded data (blackhole_b200.hex_data): no
dataset exists on this path.

One step = one layer forward (align plan, gate/up GEMM with SwiGLU, down GEMM
with the top-k weight, combine) over one batch already in HBM, timed with CUDA
events on the launching stream; a 256 MiB buffer is written between timed
steps so every step starts with a cold L2 (126 MB).  `e2e` is the same step
through the public API (blackhole_b200.hex_moe.hex_moe) with the inputs copied
from pinned host memory and the output copied back inside the timed region.
`roofline` is for the dominant kernel (the gate/up grouped GEMM), timed alone
the same way.  `cpu_baseline` times the CPU oracle (a C restatement of the
reference's torch moe_reference) on this host.

Multi-GPU (torchrun, one process per GPU): the decode path does not shard
(replicas only): each rank runs its own batch, `value` is the sum of all ranks'
tokens over the slowest rank's time (max over ranks), scaling "weak".

--impl reference times the reference's CPU implementation of the path (the
oracle port of hex_ref.moe_reference, all host threads) on the same metric; each
step is a bounded sample: the experts of one eighth of the layer, with their
routed slots, dequantized and multiplied as moe_reference does per call;
tokens are counted as slots processed / top-k.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path[:0] = [str(ROOT / "blackhole-harness_b200"), str(ROOT / "oracle")]

METRIC = "HEX MoE layer tokens/s (decode & prefill) and % of HBM / bf16 roofline, 1/2/4/8 B200"
E, H, I, K_TOP, BLOCK = 96, 2048, 768, 8, 128
FLUSH_BYTES = 256 << 20


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "src": "fallback"}


class Clocks:
    """SM clock and throttle-reason sampling (NVML, back to back: a few hundred µs per
    sample) during the timed region."""
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
                self.samples.append((sm, rs, pw))
                i += 1
            except Exception:  # noqa: BLE001
                pass
            self.stop_ev.wait(0.0001)

    def stop(self) -> dict | None:
        if self.thread is None:
            return None
        self.stop_ev.set()
        self.thread.join(timeout=2)
        if not self.samples:
            return None
        sm = [s[0] for s in self.samples]
        loaded = [x for x in sm if x > 0.5 * self.max_mhz] or sm
        reasons = sorted({name for _, rs, _ in self.samples for bit, name in self.REASONS.items() if rs & bit})
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(sm), "power_w_max": max(s[2] for s in self.samples)}


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


def build_layer(device, seed=0, bits="3", E_=E, H_=H, I_=I, block=BLOCK):
    import torch

    from blackhole_b200 import hex_data as hd
    from blackhole_b200.hex_moe import HexTier
    L = hd.synth_layer(E_, H_, I_, bits, block, seed=seed, device=device)
    tiers = [HexTier(t["bits"], t["experts"], t["gate_proj"], t["up_proj"], t["down_proj"]).prepare(E_)
             for t in L.tiers]
    torch.cuda.synchronize(device)
    return L, tiers


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


def time_steps(fn, steps: int, flush, stream) -> list[float]:
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


def cpu_baseline(sample_experts: int = 12, T: int = 64, seed: int = 0) -> dict:
    """The oracle (C port of hex_ref.moe_reference) on this host's cores, on a bounded
    sample of the workload: the routed slots of `sample_experts` of the 96 experts,
    dequantized and multiplied per call as the reference does."""
    import numpy as np
    import torch

    import hexoracle
    from blackhole_b200 import hex_data as hd
    threads = hexoracle.set_threads(os.cpu_count())
    L = hd.synth_layer(E, H, I, "3", BLOCK, seed=seed)
    w, ids = hd.synth_routing(T, E, K_TOP, seed=seed + 1)
    x = hd.synth_x(T, H, seed=seed + 2).float().numpy()
    t = L.tiers[0]
    keep = list(range(sample_experts))
    sub = {"bits": 3, "experts": np.array(keep, np.int64)}
    for p in ("gate_proj", "up_proj", "down_proj"):
        sub[p] = {q: (v[keep].view(torch.int32) if v.dtype == torch.uint32 else v[keep]).numpy()
                  for q, v in t[p].items()}
    slots = int(np.isin(ids.numpy(), keep).sum())
    layer = hexoracle.Layer([sub], E, H, I, BLOCK)
    layer.forward(x, w.numpy(), ids.numpy())               # warm-up (page-in)
    t0 = time.perf_counter()
    reps = 2
    for _ in range(reps):
        layer.forward(x, w.numpy(), ids.numpy())
    dt = (time.perf_counter() - t0) / reps
    tok = slots / K_TOP
    layer.forward(x, w.numpy(), ids.numpy(), cache_weights=True)     # fills the dequantized cache
    t1 = time.perf_counter()
    layer.forward(x, w.numpy(), ids.numpy(), cache_weights=True)
    layer.forward(x, w.numpy(), ids.numpy(), cache_weights=True)
    dt_mm = time.perf_counter() - t1
    return {"value": tok / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"T={T} decode batch, the {slots} slots routed to {sample_experts} of {E} experts per call "
                      f"({tok:.1f} token-equivalents), weights dequantized every call as hex_ref.moe_reference does",
            "seconds_per_call": dt, "matmul_only_tokens_per_s": tok / (dt_mm / 2 if dt_mm > 0 else 1)}


def reference_arm(args) -> None:
    """--impl reference: the reference's CPU path (oracle port) on the host cores."""
    import numpy as np
    import torch

    import hexoracle
    from blackhole_b200 import hex_data as hd
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = hexoracle.set_threads(os.cpu_count())
    T = args.tokens
    L = hd.synth_layer(E, H, I, "3", BLOCK, seed=0)
    w, ids = hd.synth_routing(T, E, K_TOP, seed=1)
    x = hd.synth_x(T, H, seed=2).float().numpy()
    t = L.tiers[0]
    groups = 8
    per = E // groups
    layers, tok = [], []
    for g in range(groups):
        keep = list(range(g * per, (g + 1) * per))
        sub = {"bits": 3, "experts": np.array(keep, np.int64)}
        for p in ("gate_proj", "up_proj", "down_proj"):
            sub[p] = {q: (v[keep].view(torch.int32) if v.dtype == torch.uint32 else v[keep]).numpy()
                      for q, v in t[p].items()}
        layers.append(hexoracle.Layer([sub], E, H, I, BLOCK))
        tok.append(float(np.isin(ids.numpy(), keep).sum()) / K_TOP)
    for s in range(args.warmup):
        layers[s % groups].forward(x, w.numpy(), ids.numpy())
    done, secs = 0.0, 0.0
    for s in range(args.steps):
        t0 = time.perf_counter()
        layers[s % groups].forward(x, w.numpy(), ids.numpy())
        secs += time.perf_counter() - t0
        done += tok[s % groups]
    value = done / secs
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": secs / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": f"cfg2 decode: E={E} H={H} I={I} top-{K_TOP}, 3-bit HEX, fp8 block-{BLOCK} "
                                   f"scales, T={T}", "tokens": T, "parallelism": "host cores"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": f"each step: the slots of {per} of {E} experts (one eighth of the layer, "
                                       "rotating), dequantized and multiplied as hex_ref.moe_reference"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--impl", default="b200", choices=("b200", "reference"))
    ap.add_argument("--no-extras", action="store_true", help="skip the sweep, prefill and CPU baseline")
    ap.add_argument("--profile", action="store_true", help="a few launches only (for ncu)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        reference_arm(args)
        return

    import torch
    import torch.distributed as dist

    from blackhole_b200 import hex_data as hd
    from blackhole_b200.hex_moe import device_status, hex_moe, layer_for

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        os.environ.setdefault("NCCL_DEBUG", "WARN")     # stdout carries the JSON line only
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    T = args.tokens
    L, tiers = build_layer(dev, seed=0)
    layer = layer_for(tiers)
    w, ids = hd.synth_routing(T, E, K_TOP, seed=1 + 1000 * rank)
    x = hd.synth_x(T, H, seed=2 + 1000 * rank, device=dev)
    w, ids = w.to(dev), ids.to(dev)
    stream = torch.cuda.current_stream(dev)
    flush_buf = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=dev)

    def flush():
        flush_buf.fill_(rank & 0xFF)

    bm = 16 if T <= 64 else 128     # align block height: decode batches / prefill

    def step_eager():
        layer.forward(x, w, ids, bm)

    if args.profile:
        for _ in range(args.warmup):
            step_eager()
        plan = layer.plan(ids, bm)
        xs = layer.gather(x, K_TOP, plan, bm)
        act = layer.gate_up(xs, T, K_TOP, plan, bm)
        layer.down(act, w, plan, bm)
        torch.cuda.synchronize()
        return

    for _ in range(args.warmup):
        step_eager()
    g_step = graphed(step_eager)
    step = g_step.replay
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = Clocks(local)
    torch.cuda.synchronize()
    t_wall = time.perf_counter()
    ms = time_steps(step, args.steps, flush, stream)
    t_wall = time.perf_counter() - t_wall
    clk = clocks.stop()
    step_ms = sum(ms) / len(ms)
    if world > 1:
        tt = torch.tensor([sum(ms)], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        step_ms = float(tt) / len(ms)
        dist.barrier()
    value = world * T / (step_ms * 1e-3)

    # ---- e2e through the public API: pinned host inputs in, output back, each step
    xh = x.cpu().pin_memory()
    wh = w.cpu().pin_memory()
    ih = ids.cpu().pin_memory()
    oh = torch.empty(T, H, dtype=x.dtype).pin_memory()

    def e2e_step():
        xd = xh.to(dev, non_blocking=True)
        wd = wh.to(dev, non_blocking=True)
        idd = ih.to(dev, non_blocking=True)
        out = hex_moe(xd, wd, idd, tiers, {"BLOCK_M": bm})
        oh.copy_(out, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    e2e_ms = time_steps(e2e_step, args.steps, flush, stream)
    e2e_step_ms = sum(e2e_ms) / len(e2e_ms)
    if world > 1:
        tt = torch.tensor([sum(e2e_ms)], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_step_ms = float(tt) / len(e2e_ms)
    h2d = xh.numel() * xh.element_size() + wh.numel() * 4 + ih.numel() * 8
    d2h = oh.numel() * oh.element_size()

    # ---- dominant kernel alone: the gate/up grouped GEMM
    plan = layer.plan(ids, bm)
    xs = layer.gather(x, K_TOP, plan, bm)
    act = layer.gate_up(xs, T, K_TOP, plan, bm)
    g_gu = graphed(lambda: layer.gate_up(xs, T, K_TOP, plan, bm, act))
    for _ in range(args.warmup):
        g_gu.replay()
    gu_ms = time_steps(g_gu.replay, args.steps, flush, stream)
    gu = sum(gu_ms) / len(gu_ms)
    rb = routed_bits(L, ids.cpu())
    U = sum(rb.values())
    gu_bytes = weight_bytes(rb, BLOCK, H, I, projections=2) + T * K_TOP * (H + I) * 2   # weights, token rows, act
    layer_bytes = weight_bytes(rb, BLOCK, H, I, projections=3) + 2 * T * H * 2 + T * K_TOP * 12
    pk = peaks()
    err = device_status(local)

    extras = {}
    if world > 1 and not args.no_extras:
        extras["prefill_ep"] = run_ep_prefill(dev, rank, world, flush, stream, pk)   # every rank takes part
    if not args.no_extras and rank == 0:
        extras.update(run_extras(dev, L, tiers, layer, flush, stream, args, pk, cpu=world == 1))

    if rank != 0:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    launches = 5 * args.steps   # align, gather, gate/up, down, combine per step
    traffic = read_traffic()
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"cfg2 decode: E={E} H={H} I={I} top-{K_TOP}, SwiGLU, 3-bit/8-level HEX, "
                               f"fp8 e4m3 block-{BLOCK} scales, T={T} tokens per GPU", "tokens": T,
                   "experts_routed": U, "block_m": bm, "parallelism": f"replicas x{world}" if world > 1 else "1 GPU",
                   "l2": "flushed between timed steps (256 MiB write)", "timed_wall_s": t_wall},
        "e2e": {"value": world * T / (e2e_step_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": e2e_step_ms},
        "gpu_launches": launches,
        "roofline": {"bound": "hbm", "kernel": "hex_gemm_kernel<GLU> (gate/up)", "achieved": gu_bytes / gu / 1e6,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": gu_bytes / gu / 1e6 / pk["hbm_gbs"],
                     "traffic": traffic, "peak_src": pk["src"] + " (hbm_gbs, burst)", "ms": gu,
                     "algorithmic_bytes": gu_bytes,
                     "layer_achieved_gbs": layer_bytes / step_ms / 1e6,
                     "layer_frac": layer_bytes / step_ms / 1e6 / pk["hbm_gbs"], "layer_bytes": layer_bytes},
        "clocks": clk, "device_error_word": err,
    }
    line.update(extras)
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_ep_prefill(dev, rank: int, world: int, flush, stream, pk, T: int = 4096, steps: int = 5) -> dict:
    """cfg3 prefill with expert parallelism: the 96 experts (mixed 3/4-bit) sharded
    over the ranks, T tokens per rank routed to their owners by all-to-all
    (blackhole_b200.ep), max-over-ranks time per step."""
    import torch
    import torch.distributed as dist

    from blackhole_b200 import hex_data as hd
    from blackhole_b200.ep import EPMoE, ExpertShard, shard_tiers
    from blackhole_b200.hex_moe import HexTier
    Lm = hd.synth_layer(E, H, I, "mixed", BLOCK, seed=0, device=dev)
    shard = ExpertShard(E, rank, world)
    local = [HexTier(t["bits"], t["experts"], t["gate_proj"], t["up_proj"], t["down_proj"]).prepare(E)
             for t in shard_tiers(Lm.tiers, shard)]
    del Lm
    ep = EPMoE(shard, local)
    w, ids = hd.synth_routing(T, E, K_TOP, seed=7 + 1000 * rank, device=dev)
    x = hd.synth_x(T, H, seed=8 + 1000 * rank, device=dev)
    for _ in range(2):
        ep(x, w, ids)
    torch.cuda.synchronize()
    dist.barrier()
    ms = time_steps(lambda: ep(x, w, ids), steps, flush, stream)
    tt = torch.tensor([sum(ms)], device=dev)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    step_ms = float(tt) / steps
    flops = 2.0 * world * T * K_TOP * 3 * H * I
    return {"workload": f"cfg3 prefill with expert parallelism: E={E} H={H} I={I} top-{K_TOP}, mixed 3/4-bit HEX, "
                        f"{E // world} experts and {T} tokens per GPU, NCCL all-to-all dispatch/combine",
            "tokens_per_s": world * T / (step_ms * 1e-3), "ms": step_ms, "TFLOPs": flops / (step_ms * 1e-3) / 1e12,
            "bf16_frac_per_gpu": flops / world / (step_ms * 1e-3) / 1e12 / pk["bf16_tflops"], "scaling": "weak"}


def read_traffic():
    """DRAM bytes per launch of the gate/up kernel from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get("gate_up_cfg2_T64_dram_bytes")
        except (ValueError, AttributeError):
            return None
    return None


def run_extras(dev, L, tiers, layer, flush, stream, args, pk, cpu: bool = True) -> dict:
    import torch

    from blackhole_b200 import hex_data as hd
    from blackhole_b200.hex_moe import layer_for
    out = {"sweep": {}}
    steps = max(5, args.steps // 2)
    for T in (1, 8, 32, 64):
        w, ids = hd.synth_routing(T, E, K_TOP, seed=10 + T)
        x = hd.synth_x(T, H, seed=20 + T, device=dev)
        w, ids = w.to(dev), ids.to(dev)
        g = graphed(lambda: layer.forward(x, w, ids, 16))
        for _ in range(3):
            g.replay()
        ms = time_steps(g.replay, steps, flush, stream)
        t = sum(ms) / len(ms)
        rb = routed_bits(L, ids.cpu())
        byts = weight_bytes(rb, BLOCK, H, I) + 2 * T * H * 2 + T * K_TOP * 12
        out["sweep"][f"T={T}"] = {"tokens_per_s": T / (t * 1e-3), "us": t * 1e3, "experts_routed": sum(rb.values()),
                                  "GBps": byts / t / 1e6, "hbm_frac": byts / t / 1e6 / pk["hbm_gbs"]}
    # prefill: cfg3 (mixed 3/4-bit, 96 experts), T = 4096, one GPU
    del tiers
    L3, t3 = build_layer(dev, seed=3, bits="mixed")
    lay3 = layer_for(t3)
    T = 4096
    w, ids = hd.synth_routing(T, E, K_TOP, seed=5)
    x = hd.synth_x(T, H, seed=6, device=dev)
    w, ids = w.to(dev), ids.to(dev)
    g3 = graphed(lambda: lay3.forward(x, w, ids, 128))
    for _ in range(3):
        g3.replay()
    ms = time_steps(g3.replay, steps, flush, stream)
    t = sum(ms) / len(ms)
    flops = 2.0 * T * K_TOP * 3 * H * I
    plan = lay3.plan(ids, 128)
    xs = lay3.gather(x, K_TOP, plan, 128)
    act = lay3.gate_up(xs, T, K_TOP, plan, 128)
    g3u = graphed(lambda: lay3.gate_up(xs, T, K_TOP, plan, 128, act))
    g3u.replay()
    gms = time_steps(g3u.replay, steps, flush, stream)
    g = sum(gms) / len(gms)
    gflops = 2.0 * T * K_TOP * 2 * H * I
    out["prefill"] = {"workload": "cfg3 prefill: E=96 H=2048 I=768 top-8, mixed 3/4-bit HEX (half each), "
                                  "fp8 block-128 scales, T=4096, 1 GPU",
                      "tokens_per_s": T / (t * 1e-3), "ms": t, "TFLOPs": flops / t / 1e9,
                      "bf16_frac": flops / t / 1e9 / pk["bf16_tflops"],
                      "gate_up_ms": g, "gate_up_TFLOPs": gflops / g / 1e9,
                      "gate_up_bf16_frac": gflops / g / 1e9 / pk["bf16_tflops"]}
    del lay3, t3, L3, act, xs, g3, g3u
    torch.cuda.empty_cache()
    if cpu:   # rank 0 at N=1 only
        try:
            out["cpu_baseline"] = cpu_baseline()
        except Exception as e:  # noqa: BLE001  (the baseline is reported, not required)
            out["cpu_baseline"] = {"value": None, "error": f"{type(e).__name__}: {e}"}
    return out


if __name__ == "__main__":
    main()
