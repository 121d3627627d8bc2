"""Benchmark: Qwen3-0.6B-shaped greedy decode (bf16) on B200.

Workload (the Qwen3-0.6B-shaped decode configuration, batch 32 per GPU): random-init weights
~N(0, 0.02) of the Qwen3-0.6B shape, a prompt of 512 random token ids per
sequence, then 256 greedy decode steps with the KV cache.  One bench step =
one such request batch: prefill (untimed for `value`) + 255 decode steps
replayed as a CUDA graph (timed).  Weights (1.19 GB) and KV cache are far
larger than L2, so no L2 flush is needed between steps.

  value  = decode tokens/s (all ranks): batch * 255 * steps / max-over-ranks
           of the summed decode time (CUDA events on the launch stream).
  e2e    = tokens/s through the public API Qwen3.generate(host ids) -- prompt
           H2D copy, prefill, 256 decode steps, result D2H copy all timed.
  roofline = the decode linear kernels (dominant: stream every weight once per
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
# The CPU sample decodes at the middle of the GPU arm's context span
# (513..767): its per-token cost grows with the context, so the mean context
# stands in for the whole span.
CPU_CTX = PROMPT + GEN // 2 - 2


# Measured DRAM traffic of the decode linears (ncu dram__bytes_read.sum +
# dram__bytes_write.sum on `bench.py --one-op decode_linears`), kept as one
# machine-readable line in the committed kernel summary; None when absent.
TRAFFIC_SUMMARY = ROOT / "profiles" / "decode_linears_traffic_qwen3_b32.md"


def linear_traffic_per_launch() -> float | None:
    """Mean DRAM bytes per launch over one decode step's linear launches
    (4 per layer x 28 + LM head), from the summary's `traffic_bytes_per_launch:`."""
    try:
        for line in TRAFFIC_SUMMARY.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


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
    from torchplusplus_b200 import replicas
    return replicas.max_over_ranks(x, world, "cuda")


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
    b = cpu_decode_rate(args.batch, args.cpu_steps, CPU_CTX)
    line = {"impl": "reference", "metric": METRIC, "value": b["value"], "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "qwen3-0.6b-shape greedy decode",
                                            "batch": args.batch, "prompt": PROMPT, "gen": GEN,
                                            "device": "host CPU"},
            "cpu_baseline": {k: b[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "value_scope": "the host CPU of the box: does not grow with n_gpus",
            "e2e": {"value": b["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU arm
def linear_roofline(eng, reps: int = 20) -> dict:
    """Times the decode linear kernels alone: all (4*L + 1) x lanes linear
    launches of one decode step captured in a graph (one stream) and replayed;
    algorithmic bytes = weights + x + y (+ residual) per launch."""
    from torchplusplus_b200 import ops
    byts = 0
    calls = []
    for ln in eng.lanes:  # each lane (sub-batch) reads every weight once
        n, x = ln["n"], ln["x"]
        for L in eng.layers:
            calls += [(x, L["wqkv_f"], "none", None, ln["qkv"].view(n, -1), True),
                      (ln["o"].view(n, -1), L["wo"], "none", x, x, False),
                      (x, L["wgu_f"], "swiglu", None, ln["ff"], True),
                      (ln["ff"], L["wdown"], "none", x, x, False)]
        calls.append((x, eng.lm_head_f, "none", None, ln["logits"], True))
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


def _time_graph(fn_list, reps: int = 5) -> float:
    """Captures the callables (one launch sequence) in a CUDA graph, replays it
    `reps` times and returns seconds per replay (CUDA events)."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for f in fn_list:
            f()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for f in fn_list:
                f()
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 1e3 / reps


def per_op(hbm_peak: float, tc_peak: float) -> dict:
    """Per-op achieved throughput on the op-level configurations (1: RMSNorm +
    Linear+SiLU, 2: RoPE + causal GQA prefill, 3: decode GEMVs, 5: SWA decode).

    Each op is launched over enough distinct input copies that the bytes
    touched per replay exceed L2 (126 MB), so every launch streams from HBM;
    the time per launch is the graph replay time / launches."""
    from torchplusplus_b200 import ops
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    res = {}

    def rnd(*shape, dtype=torch.float16, std=1.0, mean=0.0):
        return (torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * std + mean).to(dtype)

    def copies(nbytes):
        return max(1, min(64, int(2 * 126e6 // max(nbytes, 1)) + 1))

    def rec(name, t, work, unit):
        if unit == "GB/s":
            ach = work / t / 1e9
            res[name] = {"us": t * 1e6, "achieved": ach, "unit": unit, "frac_hbm": ach / hbm_peak}
        else:
            ach = work / t / 1e12
            res[name] = {"us": t * 1e6, "achieved": ach, "unit": unit, "frac_tc": ach / tc_peak}

    # config 1: RMSNorm [2048, 1024] fp16, then Linear+SiLU 2048x3072x1024
    nb = 2 * 2 * 2048 * 1024 + 2 * 1024
    n = copies(nb)
    xs = [rnd(2048, 1024) for _ in range(n)]
    ys = [torch.empty_like(xs[0]) for _ in range(n)]
    w = rnd(1024, mean=1.0, std=0.1)
    t = _time_graph([lambda i=i: ops.rmsnorm(xs[i], w, 1e-6, out=ys[i]) for i in range(n)]) / n
    rec("cfg1_rmsnorm_2048x1024_f16", t, nb, "GB/s")
    W = rnd(3072, 1024, std=0.02)
    yl = torch.empty(2048, 3072, device=dev, dtype=torch.float16)
    t = _time_graph([lambda: ops.linear(xs[0], W, act="silu", out=yl)] * 10) / 10
    rec("cfg1_linear_silu_2048x3072x1024_f16", t, 2 * 2048 * 3072 * 1024, "TFLOP/s")
    del xs, ys

    # config 2: RoPE on Q [4,16,2048,128] + K [4,8,2048,128]; causal GQA prefill
    q = rnd(4, 16, 2048, 128)
    k = rnd(4, 8, 2048, 128)
    cos, sin = (torch.cos(torch.arange(2048 * 128, device=dev).view(2048, 128) * 1e-3).half(),
                torch.sin(torch.arange(2048 * 128, device=dev).view(2048, 128) * 1e-3).half())
    nb = 2 * 2 * (q.numel() + k.numel())
    t = _time_graph([lambda: ops.qkrope(q, k, cos, sin)] * 5) / 5
    rec("cfg2_qkrope_B4_S2048_Hq16_Hk8_D128_f16", t, nb, "GB/s")
    qa = rnd(4, 2048, 16, 128)
    ka = rnd(4, 2048, 8, 128)
    va = rnd(4, 2048, 8, 128)
    oa = torch.empty_like(qa)
    t = _time_graph([lambda: ops.attention(qa, ka, va, causal=True, out=oa)] * 5) / 5
    rec("cfg2_attention_causal_gqa_B4_S2048_f16", t, 4 * 4 * 16 * 2048 * 2048 * 128 / 2, "TFLOP/s")
    del q, k, qa, ka, va, oa

    # config 3: decode GEMV sweep (batch 1) and fused Linear+SiLU at M = 1, 32
    for K_, N_ in ((1024, 2048), (1024, 3072), (3072, 1024), (1024, 151936)):
        nb = 2 * (N_ * K_ + K_ + N_)
        n = copies(nb)
        Ws = [rnd(N_, K_, std=0.02) for _ in range(n)]
        x1 = rnd(K_)
        t = _time_graph([lambda i=i: ops.hgemv(Ws[i], x1) for i in range(n)]) / n
        rec(f"cfg3_hgemv_K{K_}_N{N_}_f16", t, nb, "GB/s")
        del Ws
    for M_ in (1, 32):
        nb = 2 * (3072 * 1024 + M_ * 1024 + M_ * 3072)
        n = copies(nb)
        Ws = [rnd(3072, 1024, std=0.02) for _ in range(n)]
        xm = rnd(M_, 1024)
        t = _time_graph([lambda i=i: ops.linear(xm, Ws[i], act="silu") for i in range(n)]) / n
        rec(f"cfg3_linear_silu_M{M_}_K1024_N3072_f16", t, nb, "GB/s")
        del Ws

    # decode linears at batch 32 (bf16 activations), bf16 weights vs fp8
    # weights (tpp_linear_fp8): LM head, gate/up (SwiGLU), qkv; several weight
    # copies rotate so every launch streams from HBM.  Algorithmic bytes =
    # weights + scales + x + y.
    for rows_, K_, act_, name_ in ((151936, 1024, "none", "lm_head"),
                                   (6144, 1024, "swiglu", "gate_up"),
                                   (4096, 1024, "none", "qkv")):
        n_out = rows_ // 2 if act_ == "swiglu" else rows_
        io = 2 * 32 * (K_ + n_out)
        xm = rnd(32, K_, dtype=torch.bfloat16)
        n = copies(rows_ * K_)
        Ws = [rnd(rows_, K_, std=0.02, dtype=torch.bfloat16) for _ in range(n)]
        t = _time_graph([lambda i=i: ops.linear(xm, Ws[i], act=act_) for i in range(n)]) / n
        rec(f"decode_{name_}_M32_bf16_weights", t, 2 * rows_ * K_ + io, "GB/s")
        Fs = [ops.Fp8Weight(W, act_) for W in Ws]
        del Ws
        t = _time_graph([lambda i=i: ops.linear_fp8(xm, Fs[i]) for i in range(len(Fs))]) / len(Fs)
        rec(f"decode_{name_}_M32_fp8_weights", t, rows_ * K_ + 4 * rows_ + io, "GB/s")
        del Fs

    # on-device sampling of a decode step's logits (batch 32, Qwen3 vocabulary):
    # algorithmic bytes = one read of the logits
    lg = rnd(32, 151936, dtype=torch.bfloat16, std=3.0)
    cnt = torch.arange(32, dtype=torch.int32, device=dev)
    tok = torch.empty(32, dtype=torch.int64, device=dev)
    t = _time_graph([lambda: ops.argmax(lg, out=tok)] * 10) / 10
    rec("decode_argmax_B32_V151936_bf16", t, lg.numel() * 2, "GB/s")
    t = _time_graph([lambda: ops.sample(lg, 0.8, 0, 0.9, 1, counters=cnt, out=tok)] * 10) / 10
    rec("decode_sample_top_p0.9_B32_V151936_bf16", t, lg.numel() * 2, "GB/s")
    del lg

    # config 5: sliding-window GQA decode, B64, Hq16/Hkv8, D128, window 4096, bf16
    for L in (1024, 4096, 16384, 32768):
        B = 64
        kc = rnd(B, 8, L, 128, dtype=torch.bfloat16)
        vc = rnd(B, 8, L, 128, dtype=torch.bfloat16)
        qd = rnd(B, 16, 128, dtype=torch.bfloat16)
        od = torch.empty_like(qd)
        sl = torch.full((B,), L, dtype=torch.int32, device=dev)
        ws = torch.empty(max(16, ops.decode_workspace_bytes(B, 16, L, 128)), dtype=torch.uint8,
                         device=dev)
        nb = B * (2 * min(L, 4096) * 8 * 128 * 2 + 2 * 16 * 128 * 2)
        t = _time_graph([lambda: ops.attention_decode(qd, kc, vc, sl, L, window_left=4095,
                                                      out=od, workspace=ws)] * 10) / 10
        rec(f"cfg5_swa_decode_B64_L{L}_w4096_bf16", t, nb, "GB/s")
        if L == 4096:
            # the same keys in a paged cache: 64-key blocks scattered over a pool
            nblk = L // 64
            perm = torch.randperm(B * nblk, device=dev)
            table = perm.view(B, nblk).to(torch.int32)
            kp = torch.empty(B * nblk, 8, 64, 128, dtype=torch.bfloat16, device=dev)
            vp = torch.empty_like(kp)
            ops.kv_append_paged(kc, vc, kp, vp, table, start_pos=0)
            t = _time_graph([lambda: ops.attention_decode_paged(qd, kp, vp, table, sl, L,
                                                                window_left=4095, out=od,
                                                                workspace=ws)] * 10) / 10
            rec(f"cfg5_swa_decode_paged_B64_L{L}_w4096_bf16", t, nb, "GB/s")
            del kp, vp
        del kc, vc
    torch.cuda.synchronize()
    return res


ONE_OPS = ("rmsnorm", "linear_silu", "qkrope", "attention_prefill", "prefill_attn_d64",
           "hgemv_lm_head", "hgemv_k1024_n3072", "decode_linears", "decode_attention",
           "qk_norm_rope_cache", "swa_decode", "argmax", "sample", "embedding", "lm_head_fp8",
           "decode_step_b1")


def one_op(name: str, reps: int) -> dict:
    """Builds one op's operands at its benchmark shape and launches it `reps`
    times (no graph, synchronised): the small, self-contained command the
    per-kernel ncu captures run on (a few GB on the device at most)."""
    from torchplusplus_b200 import ops
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape, dtype=torch.float16, std=1.0, mean=0.0):
        return (torch.randn(*shape, generator=g, device=dev, dtype=torch.float32) * std
                + mean).to(dtype)
    bf = torch.bfloat16
    fn = None
    if name == "rmsnorm":                      # config 1
        x, w = rnd(2048, 1024), rnd(1024, mean=1.0, std=0.1)
        y = torch.empty_like(x)
        fn = lambda: ops.rmsnorm(x, w, 1e-6, out=y)  # noqa: E731
    elif name == "linear_silu":                # config 1
        x, W = rnd(2048, 1024), rnd(3072, 1024, std=0.02)
        y = torch.empty(2048, 3072, device=dev, dtype=torch.float16)
        fn = lambda: ops.linear(x, W, act="silu", out=y)  # noqa: E731
    elif name == "qkrope":                     # config 2
        q, k = rnd(4, 16, 2048, 128), rnd(4, 8, 2048, 128)
        cos, sin = rnd(2048, 128), rnd(2048, 128)
        fn = lambda: ops.qkrope(q, k, cos, sin)  # noqa: E731
    elif name == "attention_prefill":          # config 2 (tcgen05 kernel, D 128)
        q, k, v = rnd(4, 2048, 16, 128), rnd(4, 2048, 8, 128), rnd(4, 2048, 8, 128)
        o = torch.empty_like(q)
        fn = lambda: ops.attention(q, k, v, causal=True, out=o)  # noqa: E731
    elif name == "prefill_attn_d64":           # register-tile kernel (head dim 64)
        q, k, v = rnd(4, 2048, 16, 64), rnd(4, 2048, 8, 64), rnd(4, 2048, 8, 64)
        o = torch.empty_like(q)
        fn = lambda: ops.attention(q, k, v, causal=True, out=o)  # noqa: E731
    elif name == "hgemv_lm_head":              # config 3, K 1024 N 151936
        W, x = rnd(151936, 1024, std=0.02), rnd(1024)
        fn = lambda: ops.hgemv(W, x)  # noqa: E731
    elif name == "hgemv_k1024_n3072":          # config 3
        W, x = rnd(3072, 1024, std=0.02), rnd(1024)
        fn = lambda: ops.hgemv(W, x)  # noqa: E731
    elif name == "decode_linears":   # one Qwen3 layer's projections + LM head, 32 tokens
        x, o, ff = rnd(32, 1024, dtype=bf), rnd(32, 2048, dtype=bf), rnd(32, 3072, dtype=bf)
        wqkv, wo = rnd(4096, 1024, std=0.02, dtype=bf), rnd(1024, 2048, std=0.02, dtype=bf)
        wgu, wd = rnd(6144, 1024, std=0.02, dtype=bf), rnd(1024, 3072, std=0.02, dtype=bf)
        wh = rnd(151936, 1024, std=0.02, dtype=bf)
        qkv, r = torch.empty(32, 4096, device=dev, dtype=bf), x.clone()
        lg = torch.empty(32, 151936, device=dev, dtype=bf)

        def fn():
            ops.rmsnorm_linear(x, wqkv, 1e-6, out=qkv)
            ops.linear(o, wo, residual=r, out=r)
            ops.rmsnorm_linear(x, wgu, 1e-6, act="swiglu", out=ff)
            ops.linear(ff, wd, residual=r, out=r)
            ops.rmsnorm_linear(x, wh, 1e-6, out=lg)
    elif name in ("decode_attention", "qk_norm_rope_cache"):   # Qwen3 layer, 32 tokens
        B, Hq, Hkv, D, cap, pos = 32, 16, 8, 128, 768, 640
        qkv = rnd(B, 1, (Hq + 2 * Hkv) * D, dtype=bf)
        qn, kn = rnd(D, mean=1.0, std=0.1, dtype=bf), rnd(D, mean=1.0, std=0.1, dtype=bf)
        from torchplusplus_b200.dlops.rope import compute_rope_params
        cos, sin = compute_rope_params(D, 1e6, cap, device=dev)
        kc, vc = rnd(B, Hkv, cap, D, dtype=bf), rnd(B, Hkv, cap, D, dtype=bf)
        p = torch.full((B,), pos, dtype=torch.int32, device=dev)
        sl = p + 1
        o = torch.empty(B, Hq, D, device=dev, dtype=bf)
        ws = torch.empty(max(16, ops.decode_workspace_bytes(B, Hq, cap, D)), dtype=torch.uint8,
                         device=dev)
        if name == "decode_attention":
            fn = lambda: ops.attention_decode_qkv(  # noqa: E731
                qkv, qn, kn, 1e-6, cos, sin, p, kc, vc, sl, cap, Hq, Hkv, out=o, workspace=ws)
        else:
            q = torch.empty(B, 1, Hq, D, device=dev, dtype=bf)
            fn = lambda: ops.qk_norm_rope_cache(qkv, qn, kn, 1e-6, cos, sin, p, kc,  # noqa: E731
                                                vc, Hq, Hkv, q_out=q)
    elif name == "swa_decode":                 # config 5 at L 4096 (1 GB of cache)
        B, L = 64, 4096
        kc, vc = rnd(B, 8, L, 128, dtype=bf), rnd(B, 8, L, 128, dtype=bf)
        q = rnd(B, 16, 128, dtype=bf)
        o = torch.empty_like(q)
        sl = torch.full((B,), L, dtype=torch.int32, device=dev)
        fn = lambda: ops.attention_decode(q, kc, vc, sl, L, window_left=4095, out=o)  # noqa: E731
    elif name in ("argmax", "sample"):         # decode step's logits, 32 x 151936
        lg = rnd(32, 151936, dtype=bf, std=3.0)
        cnt = torch.arange(32, dtype=torch.int32, device=dev)
        tok = torch.empty(32, dtype=torch.int64, device=dev)
        if name == "argmax":
            fn = lambda: ops.argmax(lg, out=tok)  # noqa: E731
        else:
            fn = lambda: ops.sample(lg, 0.8, 0, 0.9, 1, counters=cnt, out=tok)  # noqa: E731
    elif name == "embedding":                  # 32 token rows of the Qwen3 table
        tab = rnd(151936, 1024, dtype=bf, std=0.02)
        ids = torch.randint(0, 151936, (32,), device=dev)
        y = torch.empty(32, 1024, device=dev, dtype=bf)
        fn = lambda: ops.embedding(ids, tab, out=y)  # noqa: E731
    elif name == "lm_head_fp8":                # fp8 LM head, 32 tokens
        W = ops.Fp8Weight(rnd(151936, 1024, std=0.02, dtype=bf))
        x = rnd(32, 1024, dtype=bf)
        y = torch.empty(32, 151936, device=dev, dtype=bf)
        fn = lambda: ops.linear_fp8(x, W, eps=1e-6, out=y)  # noqa: E731
    elif name == "decode_step_b1":   # persistent one-kernel decode step, batch 1, context 640
        from torchplusplus_b200.llmops.engine import DecodeEngine
        from torchplusplus_b200.llmops.qwen3 import Qwen3, Qwen3Config
        cfg = Qwen3Config()
        model = Qwen3(cfg, device=dev).init_weights(0.02, seed=0)
        ids = torch.randint(0, cfg.vocab_size, (1, 640), generator=torch.Generator().manual_seed(1))
        with torch.inference_mode():
            eng = DecodeEngine(model, 1, 640 + 64 * reps + 8, persistent=True)
            if eng.persistent is None:
                raise SystemExit("decode_step_b1: the persistent step is unavailable")
            eng.prefill(ids)

        def fn():
            with torch.inference_mode():
                eng.step_eager()
    else:
        raise SystemExit(f"--one-op: unknown op {name!r}; one of {', '.join(ONE_OPS)}")
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    assert ops.device_error() == 0
    return {"one_op": name, "reps": reps, "us_per_rep": e0.elapsed_time(e1) * 1e3 / reps}


def torchpp_comparator(model, prompt_ids, cap: int, nrep: int) -> dict:
    """The reference's own CUDA decode path (baseline/torchpp_gpu.py: torchpp's
    sm_100a extensions + flash_attn + cuBLAS, fp16, eager) at batch 1 and 32,
    run in a subprocess on this GPU, next to this engine on the same fp16
    model shape and decode length."""
    from torchplusplus_b200.llmops.qwen3 import Qwen3, Qwen3Config
    out = {}
    for bsz in (1, 32):
        try:
            r = subprocess.run([sys.executable, str(ROOT / "baseline" / "torchpp_gpu.py"),
                                "--batch", str(bsz), "--prompt", str(PROMPT), "--gen", str(GEN)],
                               capture_output=True, text=True, timeout=600,
                               env={**os.environ, "CUDA_VISIBLE_DEVICES":
                                    os.environ.get("CUDA_VISIBLE_DEVICES", "0")})
            lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
            out[f"torchpp_cuda_batch{bsz}"] = json.loads(lines[-1]) if lines else \
                {"unavailable": (r.stderr or "no output").strip().splitlines()[-1][:300]}
        except (subprocess.TimeoutExpired, OSError) as e:
            out[f"torchpp_cuda_batch{bsz}"] = {"unavailable": f"{type(e).__name__}: {e}"}
    # this engine on the same fp16 model (the reference's kernels are fp16-only)
    m16 = Qwen3(Qwen3Config(dtype=torch.float16),
                device=model.out_head.weight.device).init_weights(0.02, seed=0)
    for bsz in (1, 32):
        e = m16.engine(bsz, cap)
        e.prefill(prompt_ids[:bsz])
        e.capture()
        e.decode(8)
        e.prefill(prompt_ids[:bsz])
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        e.decode(nrep)
        a1.record()
        a1.synchronize()
        out[f"ours_f16_batch{bsz}_decode_tokens_per_s"] = bsz * nrep / (a0.elapsed_time(a1) / 1e3)
        m16._engine = None
    for bsz in (1, 32):
        ref = out[f"torchpp_cuda_batch{bsz}"].get("decode_tokens_per_s")
        if ref:
            out[f"ratio_batch{bsz}"] = out[f"ours_f16_batch{bsz}_decode_tokens_per_s"] / ref
    del m16
    torch.cuda.empty_cache()
    return out


def strong_scaling(model, prompt_ids, cap: int, nrep: int, world: int) -> dict:
    """Fixed global work split over the ranks (no collective): the decode at
    global batch 32 (32 / N sequences per GPU) and the SWA decode attention at
    global batch 64 (64 / N per GPU, cache length 16384, window 4096).
    Aggregate throughput = global work / max-over-ranks device time."""
    from torchplusplus_b200 import ops
    out = {}
    bs = max(1, 32 // world)
    e = model.engine(bs, cap)
    e.prefill(prompt_ids[:bs])
    e.capture()
    e.decode(8)
    e.prefill(prompt_ids[:bs])
    torch.cuda.synchronize()
    barrier(world)
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record()
    e.decode(nrep)
    a1.record()
    a1.synchronize()
    t = max_over_ranks(a0.elapsed_time(a1) / 1e3, world)
    out["decode_global_batch32"] = {"per_gpu_batch": bs, "tokens_per_s": bs * world * nrep / t,
                                    "ms_per_decode_step": t / nrep * 1e3}
    model._engine = None
    del e
    B, L = max(1, 64 // world), 16384
    g = torch.Generator(device="cuda").manual_seed(7)
    kc = torch.randn(B, 8, L, 128, generator=g, device="cuda", dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    q = torch.randn(B, 16, 128, generator=g, device="cuda", dtype=torch.bfloat16)
    o = torch.empty_like(q)
    sl = torch.full((B,), L, dtype=torch.int32, device="cuda")
    ws = torch.empty(max(16, ops.decode_workspace_bytes(B, 16, L, 128)), dtype=torch.uint8,
                     device="cuda")
    barrier(world)
    t = max_over_ranks(_time_graph([lambda: ops.attention_decode(
        q, kc, vc, sl, L, window_left=4095, out=o, workspace=ws)] * 10) / 10, world)
    nb = B * world * (2 * 4096 * 8 * 128 * 2 + 2 * 16 * 128 * 2)
    out["swa_decode_global_batch64_L16384"] = {"per_gpu_batch": B, "us": t * 1e6,
                                               "aggregate_GBps": nb / t / 1e9}
    del kc, vc
    torch.cuda.empty_cache()
    return out


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
    roofline = {"kernel": "decode linears: linear_xs_kernel (qkv, o, gate/up, down) and "
                          "linear_skinny_kernel (LM head), 113 launches per step",
                "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                "frac": achieved / peak, "peak_source": f"hbm_gbs of {peak_kind}",
                "traffic": linear_traffic_per_launch(),
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the same "
                                  "kernels at the same shapes (--one-op decode_linears), "
                                  "weighted to one step's 113 launches",
                "bytes_per_launch": rl["bytes_per_launch"],
                "avg_launch_us": rl["avg_launch_s"] * 1e6,
                "step_linear_time_us": rl["seconds"] * 1e6}
    extra = {}
    if rank == 0 and not args.skip_b1:
        # batch 1: the persistent one-kernel step (the default at batch 1)
        # and the launch-per-phase graph beside it
        for key, pers in (("batch1_decode_tokens_per_s", None),
                          ("batch1_launch_graph_decode_tokens_per_s", False)):
            model._engine = None
            model.decode_persistent = pers
            e1 = model.engine(1, cap)
            e1.prefill(prompts[0][:1])
            e1.capture()
            e1.decode(8)
            e1.prefill(prompts[0][:1])  # back to the prompt: nrep steps fill the capacity
            torch.cuda.synchronize()
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record()
            e1.decode(nrep)
            a1.record()
            a1.synchronize()
            extra[key] = nrep / (a0.elapsed_time(a1) / 1e3)
            if pers is None:
                extra["batch1_persistent_step"] = e1.persistent is not None
            del e1
        model.decode_persistent = None
        model._engine = None
    if rank == 0 and not args.skip_fp8:
        # the same decode with fp8 (e4m3, per-row scale) copies of the
        # projection and LM-head weights (weight_format="fp8") or of the LM
        # head alone ("fp8_head"); reported beside, not as, the headline (the
        # reference's weights are bf16)
        for fmt, bsz in (("fp8", B), ("fp8", 1), ("fp8_head", B), ("fp8_head", 1)):
            ef = model.engine(bsz, cap, weight_format=fmt)
            ef.prefill(prompts[0][:bsz])
            ef.capture()
            ef.decode(8)
            ef.prefill(prompts[0][:bsz])
            torch.cuda.synchronize()
            a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a0.record()
            ef.decode(nrep)
            a1.record()
            a1.synchronize()
            extra[f"{fmt}_weights_batch{bsz}_decode_tokens_per_s"] = \
                bsz * nrep / (a0.elapsed_time(a1) / 1e3)
            model._engine = None
            del ef

    if not args.skip_strong:
        extra["strong_scaling"] = strong_scaling(model, prompts[0], cap, nrep, world)
    if rank == 0 and not args.skip_torchpp:
        extra["gpu_comparator"] = torchpp_comparator(model, prompts[0], cap, nrep)
    lps = eng.launches_per_step or 0
    ops_res = None
    if rank == 0 and not args.skip_ops:
        model._engine = None
        del eng
        torch.cuda.empty_cache()
        import json as _j
        peaks_d = _j.loads((ROOT / "MEASURED_PEAKS.json").read_text()) \
            if (ROOT / "MEASURED_PEAKS.json").exists() else {"bf16_tflops": 1590.0}
        ops_res = per_op(peak, float(peaks_d.get("bf16_tflops", 1590.0)))
    if rank != 0:
        return
    cpu = cpu_decode_rate(B, args.cpu_steps, CPU_CTX) if world == 1 and not args.skip_cpu else None
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
            "gpu_launches": lps * nrep * args.steps,
            "launches_per_decode_step": lps,
            "tpp_launches_total": N.launch_count(), "per_op": ops_res, **extra}
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
    ap.add_argument("--skip-ops", action="store_true", help="skip the per-op roofline table")
    ap.add_argument("--skip-fp8", action="store_true", help="skip the fp8-weights decode lines")
    ap.add_argument("--skip-strong", action="store_true",
                    help="skip the fixed-global-batch (strong scaling) lines")
    ap.add_argument("--skip-torchpp", action="store_true",
                    help="skip the reference's CUDA-path comparator (baseline/torchpp_gpu.py)")
    ap.add_argument("--gen", type=int, default=GEN,
                    help="tokens generated per request (profiling runs use fewer)")
    ap.add_argument("--one-op", default=None, choices=ONE_OPS,
                    help="launch one op at its benchmark shape --reps times and exit "
                         "(the command per-kernel ncu captures run on)")
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    GEN = args.gen
    if args.one_op:
        torch.cuda.set_device(0)
        with torch.inference_mode():
            print(json.dumps(one_op(args.one_op, args.reps)), flush=True)
        return
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
