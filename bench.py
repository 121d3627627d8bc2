"""Benchmark: Qwen3-0.6B-shaped greedy decode (bf16) on B200.

Workload (batch 32 per GPU): random-init weights
~N(0, 0.02) of the Qwen3-0.6B shape, a prompt of 512 random token ids per
sequence, then 256 greedy decode steps with the KV cache.  One bench step =
one such request batch: prefill (untimed for `value`) + 255 decode steps
replayed as a CUDA graph (timed).  Weights (1.19 GB) and KV cache are far
larger than L2, so no L2 flush is needed between steps.

  value  = decode tokens/s (all ranks): batch * 255 * steps / max-over-ranks
           of the summed decode time (CUDA events on the launch stream).
  e2e    = tokens/s through the public API Qwen3.generate(host ids) -- prompt
           H2D copy, prefill, 256 decode steps, result D2H copy all timed.
  roofline = the decode linear kernel (dominant: streams every weight once per
           step), timed alone as a CUDA-graph replay of all 113 linear
           launches of one step; bytes = weights + activations.
  cpu_baseline = the fp32 PyTorch-eager oracle (the reference's eager
           formulation) decoding a bounded sample on the host cores.

Multi-GPU: one process per GPU (torchrun), each rank decodes its own batch
of 32 (weak scaling); no collective on the data path (barriers and the
max-over-ranks timing reduction only).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tokens/sec (Qwen3-0.6B shape) at 1/2/4/8 B200; per-op % of HBM/TC roofline"
PROMPT, GEN = 512, 256


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """Samples nvidia-smi every 200 ms while the timed region runs."""

    def __init__(self, index: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap,utilization.gpu")
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(index), f"--query-gpu={q}",
                                       "--format=csv,noheader,nounits", "-lms", "200"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        rows = []
        for line in Path(self.f.name).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 8:
                rows.append(parts)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        load = [r for r in rows if r[7].isdigit() and int(r[7]) > 0] or rows
        reasons = sorted({names[i] for r in rows for i in range(4) if r[3 + i] == "Active"})

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[0]) for r in load if num(r[0]) is not None]
        mx = [num(r[1]) for r in rows if num(r[1]) is not None]
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def dist_setup(n):
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- CPU baseline
def cpu_decode_rate(batch: int, steps: int, ctx: int, threads: int | None = None) -> dict:
    """fp32 eager oracle decode on the host: KV cache pre-filled with random
    rows up to `ctx` (stands in for the prompt), then `steps` greedy steps."""
    from oracle import model as OM
    from torchplusplus_b200.llmops.qwen3 import Qwen3Config
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = Qwen3Config()
    sd = OM.random_state_dict(cfg)
    g = torch.Generator().manual_seed(1)
    kc = [torch.randn(batch, cfg.n_kv_heads, ctx + steps + 1, cfg.head_dim, generator=g)
          for _ in range(cfg.n_layers)]
    vc = [torch.randn_like(k) for k in kc]
    tok = torch.randint(0, cfg.vocab_size, (batch,), generator=g)
    tok = OM.decode_step_cached(sd, cfg, tok, kc, vc, ctx)  # warm-up
    t0 = time.perf_counter()
    for i in range(steps):
        tok = OM.decode_step_cached(sd, cfg, tok, kc, vc, ctx + 1 + i)
    dt = time.perf_counter() - t0
    return {"value": batch * steps / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"fp32 eager oracle, batch {batch}, {steps} decode steps at context "
                      f"{ctx + 1}..{ctx + steps} (KV cache pre-filled with random rows), "
                      f"{threads} threads, {dt:.1f} s"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    b = cpu_decode_rate(args.batch, args.cpu_steps, PROMPT)
    line = {"impl": "reference", "metric": METRIC, "value": b["value"], "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "qwen3-0.6b-shape greedy decode",
                                            "batch": args.batch, "prompt": PROMPT, "gen": GEN,
                                            "device": "host CPU"},
            "cpu_baseline": {k: b[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": b["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm
def linear_roofline(eng, reps: int = 20) -> dict:
    """Times the decode linear kernel alone: all 4*L + 1 linear launches of one
    decode step captured in a graph and replayed; algorithmic bytes = weights
    + x + y (+ residual) per launch."""
    from torchplusplus_b200 import ops
    B = eng.batch_size
    byts = 0
    calls = []
    for L in eng.layers:
        calls += [(eng.x, L["wqkv_f"], "none", None, eng.qkv.view(B, -1), True),
                  (eng.o.view(B, -1), L["wo"], "none", eng.x, eng.x, False),
                  (eng.x, L["wgu_f"], "swiglu", None, eng.ff, True),
                  (eng.ff, L["wdown"], "none", eng.x, eng.x, False)]
    calls.append((eng.x, eng.lm_head_f, "none", None, eng.logits, True))
    for x, w, act, r, y, nrm in calls:
        byts += w.numel() * 2 + x.numel() * 2 + y.numel() * 2 * (2 if r is not None else 1)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for x, w, act, r, y, nrm in calls:
                if nrm:
                    ops.rmsnorm_linear(x, w, 1e-6, act=act, out=y)
                else:
                    ops.linear(x, w, act=act, residual=r, out=y)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / reps
    return {"bytes_per_step": byts, "launches": len(calls), "seconds": t,
            "bytes_per_launch": byts / len(calls), "avg_launch_s": t / len(calls)}


def run_ours(args, rank, world, local):
    from torchplusplus_b200 import _native as N
    from torchplusplus_b200.llmops.qwen3 import Qwen3, Qwen3Config
    dev = torch.device("cuda", local)
    cfg = Qwen3Config()
    model = Qwen3(cfg, device=dev).init_weights(0.02, seed=0)
    B = args.batch
    cap = PROMPT + GEN
    eng = model.engine(B, cap)
    g = torch.Generator().manual_seed(100 + rank)
    prompts = [torch.randint(0, cfg.vocab_size, (B, PROMPT), generator=g)
               for _ in range(args.warmup + args.steps)]
    st = torch.cuda.current_stream()
    nrep = GEN - 1

    def one(ids, timed):
        eng.prefill(ids)
        if eng.graph is None:
            eng.capture()
        if not timed:
            eng.decode(nrep)
            return 0.0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        eng.decode(nrep)
        e1.record(st)
        e1.synchronize()
        return e0.elapsed_time(e1) / 1e3

    for i in range(args.warmup):
        one(prompts[i], False)
    torch.cuda.synchronize()
    clocks = Clocks(local)
    barrier(world)
    torch.cuda.synchronize()
    tot = 0.0
    for i in range(args.steps):
        tot += one(prompts[args.warmup + i], True)
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop()
    tmax = max_over_ranks(tot, world)
    tokens_all = B * nrep * args.steps * world
    value = tokens_all / tmax

    # ---- end to end through the public API (host ids in, host ids out)
    e2e_iters = max(1, min(args.steps, 3))
    host = [torch.randint(0, cfg.vocab_size, (B, PROMPT), generator=g).pin_memory()
            for _ in range(e2e_iters)]
    model.generate(host[0], max_new_token=GEN, sampling_strategy="greedy").cpu()  # warm
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for h in host:
        out = model.generate(h, max_new_token=GEN, sampling_strategy="greedy").cpu()
    torch.cuda.synchronize()
    te = max_over_ranks((time.perf_counter() - t0) / e2e_iters, world)
    e2e = {"value": B * GEN * world / te, "unit": "tokens/s",
           "h2d_bytes_per_step": B * PROMPT * 8, "d2h_bytes_per_step": out.numel() * 8,
           "seconds_per_request": te}

    # ---- roofline of the dominant kernel, batch-1 decode rate
    rl = linear_roofline(eng)
    peak, peak_kind = peaks()
    achieved = rl["bytes_per_launch"] / rl["avg_launch_s"] / 1e9
    roofline = {"kernel": "linear_skinny_kernel (all decode-step linears incl. LM head)",
                "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": f"hbm_gbs of {peak_kind}",
                "traffic": None, "bytes_per_launch": rl["bytes_per_launch"],
                "avg_launch_us": rl["avg_launch_s"] * 1e6,
                "step_linear_time_us": rl["seconds"] * 1e6}
    extra = {}
    if rank == 0 and not args.skip_b1:
        e1 = model.engine(1, cap)
        e1.prefill(prompts[0][:1])
        e1.capture()
        e1.decode(8)
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        e1.decode(nrep)
        a1.record()
        a1.synchronize()
        extra["batch1_decode_tokens_per_s"] = nrep / (a0.elapsed_time(a1) / 1e3)
        model._engine = None

    if rank != 0:
        return
    cpu = cpu_decode_rate(B, args.cpu_steps, PROMPT) if world == 1 and not args.skip_cpu else None
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": tmax / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init weights, uniform random prompt ids)",
            "config": {"workload": "qwen3-0.6b-shape greedy decode (config 4)",
                       "model": "Qwen3-0.6B shape: 28L, E1024, 16q/8kv x128, SwiGLU 3072, V151936",
                       "batch_per_gpu": B, "global_batch": B * world, "prompt": PROMPT,
                       "gen_tokens": GEN, "timed": f"{nrep} graph-replayed decode steps per step",
                       "parallelism": f"replicas x{world} (batch-sharded, no collective)",
                       "l2": "inputs larger than L2 (1.19 GB weights + KV per step)"},
            "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "clocks": clk,
            "gpu_launches": (eng.launches_per_step or 0) * nrep * args.steps,
            "launches_per_decode_step": eng.launches_per_step,
            "tpp_launches_total": N.launch_count(), **extra}
    print(json.dumps(line), flush=True)


def main():
    global GEN
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--cpu-steps", type=int, default=4)
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-b1", action="store_true")
    ap.add_argument("--gen", type=int, default=GEN,
                    help="tokens generated per request (profiling runs use fewer)")
    args = ap.parse_args()
    GEN = args.gen
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", 0))
        run_reference(args, rank, int(os.environ.get("WORLD_SIZE", 1)))
        return
    rank, world, local = dist_setup(args.gpus)
    with torch.inference_mode():
        run_ours(args, rank, world, local)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
