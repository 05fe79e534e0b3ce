"""Benchmark: MoE decode µs/token over the 48-layer qwen4exp MoE stack.

Default (N=1): BASELINE config 2 -- 48 independent seeded layers (hidden 2048,
inter 512, 512 experts, top-10, shared expert, IQ4_XS; ~41 GB resident),
batch-1 decode, one token per step, a fresh synthetic x per step.  A step is
one replay of the CUDA graph of the whole stack.

  value     device time per token (CUDA events around K steps, max over ranks),
            inputs already in HBM
  e2e       the same through the public API with host buffers: per step the
            pinned host x is copied in, the stack runs, the fp32 output is read
            back and the host waits for it
  roofline  the dominant kernel -- the single-launch stack kernel when it
            applies (one token, unsharded), else gate|up + SwiGLU: its
            algorithmic bytes per launch / its average duration from CUDA
            events in this run
  cpu_baseline  the CPU oracle (a restatement of reference/model.py:387-417
            with cold IQ4_XS dequant) on a bounded sample of layers, scaled
            to 48 layers

N > 1 (torchrun): the stack sharded over N GPUs (--variant B by default:
intermediate rows; A: expert ids), one NCCL all-reduce per layer inside the
graph; the metric stays µs per token (total work fixed: "strong" scaling).

`--impl reference` times the CPU oracle port with every host thread on the
same metric (rank 0 only).
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
sys.path.insert(0, str(ROOT))

METRIC = "MoE decode µs/token (48 layers, batch 1); achieved HBM GB/s vs 8 TB/s peak"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per layer of the single-launch stack
# kernel, from one ncu capture of a 2-layer stack of the same shape; traffic grows with the layer
# count, so a launch of n layers moves n times this.
STACK_TRAFFIC_PER_LAYER_B = (45_254_656 + 178_688) // 2


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(f"/tmp/qmoe_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict | None:
        if self.proc is None or not self.path.exists():
            return None
        rows = []
        for line in self.path.read_text().splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), f[5:9]))
            except ValueError:
                continue
        self.path.unlink(missing_ok=True)
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------
# CPU baseline and the reference arm: the oracle port of the reference's CPU MoE
# (test infrastructure, used here only as the timed CPU arm).  Neither loads
# the product library: the weights are the same device-family bytes, rebuilt
# on the host by the oracle's own restatement of the generator.

C2_SHAPES = dict(hidden=2048, inter=512, n_experts=512, top_k=10, shared_inter=512, weight_std=0.02)


def reference_stack(n_layers: int, seed: int = 0):
    from oracle import synth_family

    shapes = synth_family.Shapes(**C2_SHAPES)
    return shapes, [synth_family.FamilyLayer(shapes, l, seed) for l in range(n_layers)]


def reference_xs(shapes, first: int, n: int, tokens: int = 1):
    from oracle import synth_family

    return [synth_family.synth_x(shapes.hidden, tokens, 1000 + i) for i in range(first, first + n)]


def cpu_baseline(n_layers: int, budget_s: float, warm_steps: int = 2) -> dict:
    """The CPU reference on a bounded sample of the bench's own workload: `warm_steps` untimed
    decode steps of the 48-layer stack (fresh x each, as the GPU arm), then timed steps until
    `budget_s` of CPU work (at least 3); median seconds per step."""
    from oracle import moe_ref, synth_family

    shapes, layers = reference_stack(n_layers)
    cache = synth_family.RowCache()
    synth_family.run_steps(layers, reference_xs(shapes, 0, warm_steps), shapes.top_k, cache)
    times: list[float] = []
    i = warm_steps
    t_end = time.perf_counter() + budget_s
    while len(times) < 3 or time.perf_counter() < t_end:
        times += synth_family.run_steps(layers, reference_xs(shapes, i, 1), shapes.top_k, cache)
        i += 1
    return {
        "value": round(statistics.median(times) * 1e6, 1), "unit": "us/token", "cores": moe_ref.threads(),
        "kind": "port",
        "sample": f"{len(times)} timed decode steps of the {n_layers}-layer stack (fresh x per step, after "
                  f"{warm_steps} untimed), the oracle port of reference/model.py:387-417 with the reference's "
                  f"row cache (LRU, 24 GiB): experts missing from it are dequantised in the step; median",
        "row_cache_hit_rate": round(cache.hits / max(1, cache.hits + cache.misses), 3),
    }


def physical_gpu(local_rank: int) -> int:
    """nvidia-smi index of this process's GPU (CUDA_VISIBLE_DEVICES remaps)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    ids = [v.strip() for v in vis.split(",") if v.strip()]
    if local_rank < len(ids) and ids[local_rank].isdigit():
        return int(ids[local_rank])
    return local_rank


def load_pkg():
    import __graft_entry__

    return __graft_entry__.load_package()


# ---------------------------------------------------------------------------

def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--tokens", type=int, default=1, help="tokens per step (1 = decode; 4/8 = verify)")
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--variant", default="B", choices=["A", "B"])
    ap.add_argument("--exchange", default="auto", choices=["auto", "kernel", "nccl"],
                    help="N>1: partial sums exchanged inside the stack kernel over NVLink, or NCCL per layer")
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU-baseline sampling")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the config-4 prefill timings")
    ap.add_argument("--no-verify", action="store_true", help="skip the config-3 verify-chunk timings")
    ap.add_argument("--no-formats", action="store_true", help="skip the checkpoint-format block timings")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))

    pkg = load_pkg()
    cfg = pkg.MoEConfig(n_layers=args.layers)
    shard = pkg.Shard(args.variant, rank, world) if world > 1 else pkg.Shard()
    M = args.tokens

    layers = [pkg.synth_device_layer(cfg, l, seed=0, shard=shard, device=dev) for l in range(cfg.n_layers)]
    torch.cuda.synchronize(dev)
    if world > 1:
        from importlib import import_module

        dist_mod = import_module(pkg.__name__ + ".dist")
        exchange = args.exchange
        if exchange == "auto":
            exchange = "kernel" if M == 1 and dist_mod.kernel_exchange_supported(layers) else "nccl"
        stack = dist_mod.ShardedMoEStack(layers, max_tokens=max(M, 1), exchange=exchange)
        out_buf = stack.act
    else:
        stack = pkg.MoEStack(layers, max_tokens=max(M, 1))
        out_buf = stack.out

    n_x = args.warmup + args.steps
    xs = torch.stack([pkg.synth_x(cfg, M, seed=1000 + i) for i in range(n_x)]).to(dev)   # [n, M, D] bf16
    g = stack.graph(M)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    # ---- device-resident timing ----
    for i in range(args.warmup):
        stack.x_in[:M].copy_(xs[i])
        g.replay()
    barrier()
    torch.cuda.synchronize(dev)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(physical_gpu(local_rank)) as clk:
        barrier()
        torch.cuda.synchronize(dev)
        start.record()
        for i in range(args.steps):
            stack.x_in[:M].copy_(xs[args.warmup + i])
            g.replay()
        stop.record()
        torch.cuda.synchronize(dev)
        barrier()
    ms = start.elapsed_time(stop)
    clocks = clk.summary()

    # ---- end to end: pinned host in, host read of the result each step ----
    x_host = [xs[i].cpu().pin_memory() for i in range(n_x)]
    out_host = torch.empty(M, cfg.hidden, dtype=torch.float32).pin_memory()
    for i in range(args.warmup):
        stack.x_in[:M].copy_(x_host[i], non_blocking=True)
        g.replay()
        out_host.copy_(out_buf[:M], non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
    barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        stack.x_in[:M].copy_(x_host[args.warmup + i], non_blocking=True)
        g.replay()
        out_host.copy_(out_buf[:M], non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
    e1.record()
    torch.cuda.synchronize(dev)
    ms_e2e = e0.elapsed_time(e1)
    # The workspace status word after every timed step (0, or the first QMOE_ERR_* a kernel
    # recorded, e.g. a bounded wait that ran out): a nonzero value makes the timings invalid.
    device_status = stack.ws.read_status()

    # ---- per-kernel durations for the roofline (eager, events per stage) ----
    stage = stage_timings(pkg, layers, xs[0], M, dev)
    prefill = prefill_timings(pkg, layers[0], cfg, dev) if world == 1 and not args.no_prefill else None
    verify = verify_timings(pkg, layers, cfg, dev) if world == 1 and M == 1 and not args.no_verify else None
    formats = formats_timings(pkg, cfg, dev) if world == 1 and M == 1 and not args.no_formats else None

    if world > 1:
        t = torch.tensor([ms, ms_e2e, float(device_status != 0)], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e, any_bad = t.tolist()
        device_status = device_status or int(any_bad)
        # Every CUDA graph holding NCCL work is released before the process group is destroyed
        # (a live one makes destroy_process_group wait forever).
        torch.cuda.synchronize(dev)
        del g
        stack.release()
        import gc

        gc.collect()

    if rank == 0:
        hbm, hbm_kind = peaks()
        ms_step = ms / args.steps
        us_tok = ms_step * 1000.0 / M
        bytes_tok = cfg.n_layers * cfg.layer_expert_bytes() / max(world, 1) if M == 1 else None
        single = stack.single_launch(M) if world == 1 else stack.exchange == "kernel"
        if single:
            # one persistent launch per step: its bytes are the whole stack's (this rank's slice on N > 1)
            rl_kernel, rl_bytes, rl_us = "stack_kernel", bytes_tok, ms_step * 1000.0
            rl_traffic = STACK_TRAFFIC_PER_LAYER_B * cfg.n_layers if world == 1 else None
        else:
            rl_kernel = "gateup_swiglu"
            rl_bytes = (cfg.top_k + (1 if shard.has_shared() else 0)) * 2 * shard.dims(cfg).inter_local \
                * cfg.gate_up_row_bytes
            rl_us = stage["gateup_us"]
            rl_traffic = None
        rl_gbs = rl_bytes / (rl_us * 1e-6) / 1e9
        line = {
            "metric": METRIC, "value": round(us_tok, 3), "unit": "us/token", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": False, "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "iq4xs weights, bf16 activations, fp32 accumulate",
            "data": "synthetic: seeded N(0,0.02) weights quantised to IQ4_XS, x ~ N(0,1) bf16, fresh x per step",
            "config": {
                "workload": f"BASELINE config {'2' if M == 1 else '3'}: {cfg.n_layers}-layer MoE stack, "
                            f"{M} token(s)/step, hidden {cfg.hidden}, inter {cfg.inter}, {cfg.n_experts} experts, "
                            f"top-{cfg.top_k} + shared",
                "tokens_per_step": M, "layers": cfg.n_layers,
                "parallelism": (f"variant {args.variant} x{world}, " + (
                    "partial rows exchanged inside the stack kernel over NVLink" if single else
                    "NCCL all-reduce per layer")) if world > 1 else "1 GPU",
                "l2": "inputs larger than L2: ~1.08 GB of weights read per token vs 126 MB L2",
            },
            "e2e": {"value": round(ms_e2e / args.steps * 1000.0 / M, 3), "unit": "us/token",
                    "h2d_bytes_per_step": M * cfg.hidden * 2, "d2h_bytes_per_step": M * cfg.hidden * 4},
            "gpu_launches": (1 if single else 3 * cfg.n_layers) * args.steps,
            "roofline": {
                "kernel": rl_kernel, "bound": "hbm", "achieved": round(rl_gbs, 1), "peak": hbm,
                "peak_kind": hbm_kind, "unit": "GB/s", "frac": round(rl_gbs / hbm, 4), "traffic": rl_traffic,
                "bytes_per_launch": rl_bytes, "avg_launch_us": round(rl_us, 3),
                "frac_of_nominal_8tbs": round(rl_gbs / NOMINAL_HBM_GBS, 4),
            },
            "per_layer_path_stage_us": {k: round(v, 3) for k, v in stage.items()},
            "prefill_config4": prefill,
            "verify_config3": verify,
            "formats_block": formats,
            "clocks": clocks,
            "device_status": device_status,
        }
        if bytes_tok:
            gbs = bytes_tok / (us_tok * 1e-6) / 1e9
            line["step_hbm"] = {
                "expert_bytes_per_token": bytes_tok, "achieved_gbs": round(gbs, 1),
                "frac_of_8tbs": round(gbs / NOMINAL_HBM_GBS, 4), f"frac_of_{hbm_kind}": round(gbs / hbm, 4),
                "bytes_with_router": bytes_tok + cfg.n_layers * (cfg.router_bytes + cfg.hidden * 4),
            }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg.n_layers, budget_s=args.cpu_budget)
        print(json.dumps(line), flush=True)

    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def verify_timings(pkg, layers, cfg, dev, tokens=(4, 8), steps: int = 10, warmup: int = 3) -> list:
    """the config-2 stack with M = 4 and 8 tokens per step (speculative verify;
    each token routes on its own, the per-layer kernels share the experts the tokens have in
    common), one CUDA graph per step, inputs resident.  Bytes = expected distinct experts per layer
    512 (1 - (1 - 10/512)^M) x expert bytes + shared, x 48.  A failure is reported, not raised."""
    import torch

    hbm = peaks()[0]
    out = []
    for M in tokens:
        try:
            stack = pkg.MoEStack(layers, max_tokens=M)
            xs = [pkg.synth_x(cfg, M, seed=7000 + i).to(dev) for i in range(warmup + steps)]
            g = stack.graph(M)
            for i in range(warmup):
                stack.x_in[:M].copy_(xs[i])
                g.replay()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(steps):
                stack.x_in[:M].copy_(xs[warmup + i])
                g.replay()
            e1.record()
            torch.cuda.synchronize(dev)
            status = stack.ws.read_status()
            us = e0.elapsed_time(e1) * 1000.0 / steps
            uniq = cfg.n_experts * (1.0 - (1.0 - cfg.top_k / cfg.n_experts) ** M)
            expert_b = cfg.gate_up_row_bytes * 2 * cfg.inter + cfg.hidden * cfg.down_row_bytes
            nbytes = cfg.n_layers * (uniq * expert_b + cfg.shared_bytes)
            gbs = nbytes / (us * 1e-6) / 1e9
            out.append({"tokens": M, "us_per_step": round(us, 2), "us_per_token": round(us / M, 2),
                        "launches_per_step": 4 * cfg.n_layers, "expected_experts_per_layer": round(uniq, 1),
                        "bytes_per_step": round(nbytes), "achieved_gbs": round(gbs, 1),
                        "frac_of_measured_hbm": round(gbs / hbm, 4), "device_status": status})
            del g, stack
        except Exception as exc:  # noqa: BLE001 -- a sub-measurement reports its failure in the line
            out.append({"tokens": M, "error": f"{type(exc).__name__}: {exc}"[:300]})
    return out


def prefill_timings(pkg, layer, cfg, dev, chunks=(128, 2048), steps: int = 10, warmup: int = 3) -> list:
    """one layer, chunks of T tokens (x ~ N(0,1) bf16) through the chunked-prefill
    path (router GEMM + top-k + grouping + tcgen05 grouped GEMMs).  Device time per chunk from CUDA
    events, split into routing and experts; bytes = the IQ4_XS rows of the experts the chunk touches
    (+ router), FLOPs = 2 x T x (k + 1) x (2I x D + D x I)."""
    import torch

    peaks_all = {}
    pp = ROOT / "MEASURED_PEAKS.json"
    if pp.exists():
        try:
            peaks_all = json.loads(pp.read_text())
        except ValueError:
            peaks_all = {}
    hbm = float(peaks_all.get("hbm_gbs", FALLBACK_HBM_GBS))
    tflops_peak = float(peaks_all.get("bf16_tflops", 1590.0))
    ml = pkg.MoELayer(layer)
    out = []
    for T in chunks:
        xs = [pkg.synth_x(cfg, T, seed=5000 + i).to(dev) for i in range(warmup + steps)]
        ids, _, _ = ml.prefill_route(xs[0])
        uniq = int(torch.unique(ids).numel())
        for i in range(warmup):
            ml.prefill(xs[i])
        torch.cuda.synchronize(dev)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record()
        for i in range(steps):
            ml.prefill(xs[warmup + i])
        ev[1].record()
        torch.cuda.synchronize(dev)
        us = ev[0].elapsed_time(ev[1]) * 1000.0 / steps
        # routing alone (router GEMM + top-k), to split the time
        ev[0].record()
        for i in range(steps):
            ml.prefill_route(xs[warmup + i])
        ev[1].record()
        torch.cuda.synchronize(dev)
        us_route = ev[0].elapsed_time(ev[1]) * 1000.0 / steps
        expert_b = cfg.gate_up_row_bytes * 2 * cfg.inter + cfg.hidden * cfg.down_row_bytes
        nbytes = (uniq + 1) * expert_b + cfg.router_bytes
        flops = 2.0 * T * (cfg.top_k + 1) * (2 * cfg.inter * cfg.hidden + cfg.hidden * cfg.inter)
        out.append({
            "tokens": T, "us_per_chunk": round(us, 2), "tokens_per_s": round(T / (us * 1e-6), 1),
            "us_routing": round(us_route, 2), "us_experts": round(us - us_route, 2),
            "experts_touched": uniq, "bytes": nbytes, "achieved_gbs": round(nbytes / (us * 1e-6) / 1e9, 1),
            "frac_of_measured_hbm": round(nbytes / (us * 1e-6) / 1e9 / hbm, 4),
            "tflops": round(flops / (us * 1e-6) / 1e12, 2),
            "frac_of_measured_bf16": round(flops / (us * 1e-6) / 1e12 / tflops_peak, 4),
        })
        del xs
    return out


def formats_timings(pkg, cfg, dev, tokens=(1, 4), n_layers: int = 4, steps: int = 24, warmup: int = 4) -> list:
    """The MoE block on the real checkpoint's format mix (IQ3_S gate|up, IQ4_NL down, IQ3_S gate|up
    and Q8_0 down of the shared expert; tt/plan.py:90-103) at the config's dimensions, through the C
    ABI (`qmoe_moe_block_formats`).  Weights are random block bytes with a fixed fp16 scale, made on
    the device (4 layers, 3 GB, rotated per step so each step reads its experts from HBM); bytes =
    the rows of the k routed experts and the shared expert + the router."""
    import torch

    bb = {8: 34, 20: 18, 21: 110}
    bv = {8: 32, 20: 32, 21: 256}
    E, D, I, Ish = cfg.n_experts, cfg.hidden, cfg.inter, cfg.shared_inter
    gen = torch.Generator(device=dev)
    gen.manual_seed(77)

    def blocks(fmt, rows, vals):
        nb = rows * vals // bv[fmt]
        t = torch.randint(0, 256, (nb, bb[fmt]), dtype=torch.uint8, device=dev, generator=gen)
        t[:, 0:2] = torch.full((nb, 1), 2e-4, dtype=torch.float16, device=dev).view(torch.uint8)
        return t.view(rows, vals // bv[fmt] * bb[fmt])

    lays = []
    for _ in range(n_layers):
        lays.append(dict(
            router=torch.randn(E, D, device=dev, generator=gen) * 0.02,
            gate_vec=torch.randn(D, device=dev, generator=gen) * 0.02,
            gate_up=blocks(21, E * 2 * I, D).view(E, 2 * I, -1), down=blocks(20, E * D, I).view(E, D, -1),
            sh_gate_up=blocks(21, 2 * Ish, D), sh_down=blocks(8, D, Ish)))
    fmts = (21, 20, 21, 8)
    row_b = 2 * I * (D // 256 * 110) + D * (I // 32 * 18)
    sh_b = 2 * Ish * (D // 256 * 110) + D * (Ish // 32 * 34)
    hbm = peaks()[0]
    out = []
    for M in tokens:
        xs = [(torch.randn(M, D, device=dev, generator=gen)).to(torch.bfloat16) for _ in range(warmup + steps)]

        def run(i):
            L = lays[i % n_layers]
            return pkg.moe_block_formats(xs[i], L["router"], L["gate_vec"], L["gate_up"], L["down"],
                                         L["sh_gate_up"], L["sh_down"], fmts, cfg.top_k)

        for i in range(warmup):
            run(i)
        touched = 0
        for i in range(steps):
            L = lays[(warmup + i) % n_layers]
            logits = xs[warmup + i].float() @ L["router"].t()
            touched += int(torch.unique(logits.topk(cfg.top_k, dim=-1).indices).numel())
        torch.cuda.synchronize(dev)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record()
        for i in range(steps):
            run(warmup + i)
        ev[1].record()
        torch.cuda.synchronize(dev)
        us = ev[0].elapsed_time(ev[1]) * 1000.0 / steps
        nbytes = touched / steps * row_b + sh_b + E * D * 4
        gbs = nbytes / (us * 1e-6) / 1e9
        out.append({"tokens": M, "us_per_layer": round(us, 2), "bytes_per_layer": int(nbytes),
                    "achieved_gbs": round(gbs, 1), "frac_of_measured_hbm": round(gbs / hbm, 4),
                    "launches_per_layer": 3})
        del xs
    del lays
    torch.cuda.empty_cache()
    return out


def stage_timings(pkg, layers, x, M: int, dev, reps: int = 10) -> dict:
    """Average device time of each stage launch of the per-layer path (route, gate|up, down through
    their C entry points), every layer's call of a stage captured in one CUDA graph and replayed
    `reps` times; CUDA events around the replays on the launching stream."""
    import torch

    mls = [pkg.MoELayer(l, max_tokens=max(M, 1)) for l in layers]
    x = x.contiguous()
    routed = [ml.route(x) for ml in mls]
    hs = [ml.gate_up(x, r[0]) for ml, r in zip(mls, routed)]
    stages = {
        "route_us": lambda: [ml.route(x) for ml in mls],
        "gateup_us": lambda: [ml.gate_up(x, r[0]) for ml, r in zip(mls, routed)],
        "down_us": lambda: [ml.down(h, r[0], r[1], r[2]) for ml, r, h in zip(mls, routed, hs)],
    }
    out = {}
    for name, fn in stages.items():
        fn()
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        g.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        out[name] = e0.elapsed_time(e1) * 1000.0 / reps / len(mls)
        del g
    return out


def run_reference_arm(args, rank: int, world: int) -> None:
    """The reference's CPU implementation of the path (the oracle port), timed on this host's cores
    with every thread, on the GPU arm's config: the same 48 device-family layers (rebuilt on the host,
    no product library loaded), the same fresh x per step, one token per step; W untimed steps, then
    K timed ones, each a whole 48-layer decode step.  Rank 0 only."""
    if rank != 0:
        return
    from oracle import moe_ref, synth_family

    t_setup = time.perf_counter()
    shapes, layers = reference_stack(args.layers)
    cache = synth_family.RowCache()
    setup_s = time.perf_counter() - t_setup
    M = args.tokens
    synth_family.run_steps(layers, reference_xs(shapes, 0, args.warmup, M), shapes.top_k, cache)
    times = synth_family.run_steps(layers, reference_xs(shapes, args.warmup, args.steps, M), shapes.top_k, cache)
    us_tok = statistics.median(times) * 1e6 / M
    line = {
        "metric": METRIC, "value": round(us_tok, 1), "unit": "us/token", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(statistics.median(times) * 1e3, 3),
        "higher_is_better": False, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "impl": "reference", "dtype": "iq4xs weights dequantised to fp32, fp32 activations and compute",
        "data": "synthetic: the GPU arm's device-family weights (seed 0) rebuilt on the host, x ~ N(0,1) "
                "bf16, fresh x per step (the GPU arm's seeds)",
        "config": {
            "workload": f"BASELINE config {'2' if M == 1 else '3'}: {args.layers}-layer MoE stack, {M} token(s)/step, "
                        f"hidden {shapes.hidden}, inter {shapes.inter}, {shapes.n_experts} experts, "
                        f"top-{shapes.top_k} + shared",
            "tokens_per_step": M, "layers": args.layers,
        },
        "cpu_baseline": {
            "value": round(us_tok, 1), "unit": "us/token", "cores": moe_ref.threads(), "kind": "port",
            "sample": f"{args.steps} whole decode steps (after {args.warmup} untimed), median; the oracle port "
                      "of reference/model.py:387-417 with the reference's LRU row cache (24 GiB); generating "
                      "expert bytes not yet held is excluded (the reference reads them from its checkpoint)",
        },
        "e2e": {"value": round(us_tok, 1), "unit": "us/token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "step_seconds": {"median": round(statistics.median(times), 4), "min": round(min(times), 4),
                         "max": round(max(times), 4), "mean": round(statistics.mean(times), 4)},
        "row_cache_hit_rate": round(cache.hits / max(1, cache.hits + cache.misses), 3),
        "setup_seconds": round(setup_s + sum(l.gen_seconds for l in layers), 1),
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
