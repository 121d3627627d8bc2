"""DecodeEngine: the whole greedy decode step of a Qwen3-shaped model as ONE
CUDA graph of sm_100a kernels, with every buffer static and the sampled token
fed back on the device.

Per step and layer (5 kernels): RMSNorm+QKV linear (norm fused into the
GEMM) -> decode attention with the q/k norm, RoPE and KV-cache write of the
new token fused in (split-KV merged in a cluster) -> o-proj linear with the
residual add in its epilogue -> RMSNorm+gate/up linear with the SwiGLU
product in its epilogue -> down linear with the residual add in its
epilogue.  Then RMSNorm+LM-head
linear -> argmax -> decode_advance (token history, positions).  Nothing
returns to the host between steps.

This replaces the reference's per-token Python loop (torchpp/llmops/llm.py:
263-282), which issues ~20 launches per layer from Python, copies the whole
cache per step (kvcache.py:106-107) and synchronises on token.item()
(llm.py:212).
"""
from __future__ import annotations

import os
from typing import List, Optional

import torch

from .. import _native as N
from .. import ops
from ..replicas import shard
from .kvcache import KVCache


class DecodeEngine:
    """`lanes` > 1 splits the batch into that many independent sub-batches
    whose decode steps are recorded as parallel branches of the one CUDA
    graph (each weight is then read once per lane); the default is one lane
    (see the measurement noted below)."""

    def __init__(self, model, batch_size: int, max_seq_len: int, lanes: int | None = None,
                 weight_format: str = "native", persistent: bool | None = None):
        cfg = model.cfg
        dev = model.out_head.weight.device
        self.model = model
        self.cfg = cfg
        self.batch_size = B = batch_size
        self.max_seq_len = max_seq_len
        self.device = dev
        dt = cfg.dtype
        self.Hq, self.Hkv, self.D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        self.eps = 1e-6
        self.layers = []
        # The decode step runs each RMSNorm inside the following projection
        # (tpp_rmsnorm_linear), with the norm weight folded into that
        # projection's matrix once here.  These folded copies belong to the
        # engine; rebuild the engine after changing the model's weights.
        for blk in model.transformer_blocs:
            a = blk.attn
            n1, n2 = blk.rms_norm1.weight.detach(), blk.rms_norm2.weight.detach()
            self.layers.append(dict(
                n1=n1, n2=n2,
                wqkv=a._qkv.get(a.Wq.weight, a.Wk.weight, a.Wv.weight),
                wqkv_f=ops.fold_rmsnorm_weight(a._qkv.get(a.Wq.weight, a.Wk.weight, a.Wv.weight), n1),
                qn=a.q_norm.weight.detach() if a.q_norm is not None else None,
                kn=a.k_norm.weight.detach() if a.k_norm is not None else None,
                wo=a.out_projection.weight.detach(),
                wgu=blk.ffn.gate_up_weight(),
                wgu_f=ops.fold_rmsnorm_weight(blk.ffn.gate_up_weight(), n2),
                wdown=blk.ffn.linear_layer2.weight.detach()))
        self.nf = model.final_rmsnorm.weight.detach()
        self.lm_head = model.out_head.weight.detach()
        self.lm_head_f = ops.fold_rmsnorm_weight(self.lm_head, self.nf)
        self.emb = model.tok_embed.weight.detach()
        self.cos, self.sin = model.cos, model.sin
        if self.cos.shape[0] < max_seq_len:
            raise ValueError("max_seq_len exceeds the model's rotary table")
        self.caches: List[KVCache] = [
            KVCache(max_seq_len, self.Hkv, self.D, dt, dev, batch_size=B)
            for _ in range(cfg.n_layers)]
        E, W = cfg.embed_dim, (self.Hq + 2 * self.Hkv) * self.D

        def z(*s, d=dt):
            return torch.zeros(*s, dtype=d, device=dev)
        self.tokens = z(B, d=torch.int64)
        self.positions = z(B, d=torch.int32)
        self.seqlens = z(B, d=torch.int32)
        self.out_ids = z(B, max_seq_len, d=torch.int64)
        self.logits = z(B, cfg.vocab_size)
        if lanes is None:
            # measured on B200 (Qwen3-0.6B shape, 32 sequences): one lane 1265 us
            # a step, two lanes of 16 1313 us (the branches overlap only ~40%:
            # each lane's kernels plus their early-starting successors do not
            # all fit the SMs), so one lane unless asked
            lanes = 1
        self.lanes = []
        for i in range(max(1, min(lanes, B))):
            b0, n = shard(B, i, max(1, min(lanes, B)))
            sl = slice(b0, b0 + n)
            nws = ops.decode_workspace_bytes(n, self.Hq, max_seq_len, self.D)
            self.lanes.append(dict(
                b=sl, n=n,
                tokens=self.tokens[sl], positions=self.positions[sl],
                seqlens=self.seqlens[sl], out_ids=self.out_ids[sl],
                logits=self.logits[sl],
                x=z(n, E), qkv=z(n, 1, W), q=z(n, 1, self.Hq, self.D),
                o=z(n, self.Hq, self.D), ff=z(n, cfg.hidden_dim),
                ws=torch.empty(max(nws, 16), dtype=torch.uint8, device=dev),
                k=[c.k_cache[sl] for c in self.caches], v=[c.v_cache[sl] for c in self.caches]))
        # q/k norm + RoPE + KV append inside the decode-attention launch (head
        # dims 64 / 128 with fp16 RoPE tables); otherwise a separate kernel.
        self.fuse_qk_attention = self.D in (64, 128) and self.cos.dtype == torch.float16
        # Optional parallel graph branch warming L2 with each layer's
        # o/gate-up/down weights while its attention runs.  Off: measured
        # slower on B200 (1166 vs 1095 us a step for the Qwen3-0.6B shape at
        # batch 32 -- the fork costs the chain its programmatic launch edge
        # and the prefetches compete with the K/V stream).
        self.l2_warm = False
        # None = greedy; else dict(temperature, top_k, top_p, seed) (set_sampling)
        self.sampling: Optional[dict] = None
        self._graph_sampling: Optional[dict] = None
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.launches_per_step: int | None = None
        self.prompt_len = 0
        self._pos = 0  # host copy of the next write position (all sequences)
        # weight_format "fp8": the decode step's projections and LM head run
        # on e4m3 copies of the (norm-folded) weights with per-row scales
        # (tpp_linear_fp8, half the weight bytes); "fp8_head": only the LM
        # head (the one decode linear that is bandwidth-bound, so the only one
        # fp8 makes faster on B200; the per-layer projections are latency-
        # bound).  Prefill keeps the model's own weights.  Lanes of up to 32
        # sequences.
        if weight_format not in ("native", "fp8", "fp8_head"):
            raise ValueError("weight_format must be 'native', 'fp8' or 'fp8_head'")
        self.weight_format = weight_format
        self.lm_head_f8 = None
        if weight_format != "native":
            if max(ln["n"] for ln in self.lanes) > 32:
                raise ValueError("fp8 decode weights serve lanes of at most 32 sequences")
            self.lm_head_f8 = ops.Fp8Weight(self.lm_head_f)
        # batch 1, native weights: the whole step as one persistent
        # cooperative kernel (tpp_decode_step_persistent) unless turned off
        # (persistent=False or TPP_PERSISTENT=0).  Qwen3-0.6B shape, context
        # ~640: ~580 us a step against ~865 us for the launch-per-phase graph.
        self.persistent = None
        if persistent is None:
            persistent = os.environ.get("TPP_PERSISTENT", "1") != "0"
        if persistent and B == 1 and weight_format == "native" and \
                self.cos.dtype == torch.float16:
            try:
                self.persistent = ops.PersistentDecode(
                    [dict(wqkv=L["wqkv_f"], qn=L["qn"], kn=L["kn"], wo=L["wo"], wgu=L["wgu_f"],
                          wdown=L["wdown"], kc=c.k_cache[0], vc=c.v_cache[0])
                     for L, c in zip(self.layers, self.caches)],
                    self.emb, self.lm_head_f, self.cos, self.sin, self.Hq, self.Hkv, self.D,
                    max_seq_len, self.eps)
            except ValueError:
                self.persistent = None
        if weight_format == "fp8":
            for L in self.layers:
                L["f8"] = dict(qkv=ops.Fp8Weight(L["wqkv_f"]), o=ops.Fp8Weight(L["wo"]),
                               gu=ops.Fp8Weight(L["wgu_f"], "swiglu"),
                               down=ops.Fp8Weight(L["wdown"]))

    # ------------------------------------------------------------ one step
    def _step_lane(self, ln: dict, warm: Optional[torch.cuda.Stream] = None) -> None:
        if self.persistent is not None and self.sampling is None:
            self.persistent.step(self.tokens, self.positions, self.seqlens, self.out_ids[0],
                                 self.logits[0])
            return
        # several lanes run side by side as graph branches: each plans its
        # grids for its share of the SMs
        nl = len(self.lanes)
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        ops.set_sm_budget(sms // nl if nl > 1 else 0)
        try:
            self._step_lane_launches(ln, warm)
        finally:
            ops.set_sm_budget(0)

    def _step_lane_launches(self, ln: dict, warm: Optional[torch.cuda.Stream]) -> None:
        n, Hq, Hkv, D = ln["n"], self.Hq, self.Hkv, self.D
        x = ln["x"]
        ops.embedding(ln["tokens"], self.emb, out=x)
        for L, kc, vc in zip(self.layers, ln["k"], ln["v"]):
            f8 = L.get("f8")
            if f8 is not None:
                ops.linear_fp8(x, f8["qkv"], eps=self.eps, out=ln["qkv"].view(n, -1))
            else:
                ops.rmsnorm_linear(x, L["wqkv_f"], self.eps, out=ln["qkv"].view(n, -1))
            if warm is not None:
                # parallel branch: pull this layer's remaining weights into L2
                # while attention runs
                ev = torch.cuda.Event()
                ev.record(torch.cuda.current_stream())
                warm.wait_event(ev)
                with torch.cuda.stream(warm):
                    for w in (L["wo"], L["wgu_f"], L["wdown"]):
                        ops.l2_prefetch(w)
            if self.fuse_qk_attention:
                ops.attention_decode_qkv(ln["qkv"], L["qn"], L["kn"], self.eps, self.cos,
                                         self.sin, ln["positions"], kc, vc, ln["seqlens"],
                                         self.max_seq_len, Hq, Hkv, out=ln["o"],
                                         workspace=ln["ws"])
            else:
                ops.qk_norm_rope_cache(ln["qkv"], L["qn"], L["kn"], self.eps, self.cos,
                                       self.sin, ln["positions"], kc, vc, Hq, Hkv,
                                       q_out=ln["q"])
                ops.attention_decode(ln["q"].view(n, Hq, D), kc, vc, ln["seqlens"],
                                     self.max_seq_len, out=ln["o"], workspace=ln["ws"])
            if f8 is not None:
                ops.linear_fp8(ln["o"].view(n, Hq * D), f8["o"], residual=x, out=x)
                ops.linear_fp8(x, f8["gu"], eps=self.eps, out=ln["ff"])
                ops.linear_fp8(ln["ff"], f8["down"], residual=x, out=x)
            else:
                ops.linear(ln["o"].view(n, Hq * D), L["wo"], residual=x, out=x)
                ops.rmsnorm_linear(x, L["wgu_f"], self.eps, act="swiglu", out=ln["ff"])
                ops.linear(ln["ff"], L["wdown"], residual=x, out=x)
        if self.lm_head_f8 is not None:
            ops.linear_fp8(x, self.lm_head_f8, eps=self.eps, out=ln["logits"])
        else:
            ops.rmsnorm_linear(x, self.lm_head_f, self.eps, out=ln["logits"])
        self._pick(ln["logits"], ln["positions"], ln["tokens"])
        ops.decode_advance(ln["tokens"], ln["out_ids"], ln["positions"], ln["seqlens"])

    def _pick(self, logits: torch.Tensor, counters: torch.Tensor, out: torch.Tensor) -> None:
        """Next token per row: argmax, or an on-device draw (temperature /
        top-k / top-p) keyed by the row's position, so each graph replay
        draws afresh."""
        if self.sampling is None:
            ops.argmax(logits, out=out)
        else:
            sp = self.sampling
            ops.sample(logits, sp["temperature"], sp["top_k"], sp["top_p"], sp["seed"],
                       counters=counters, out=out)

    def _step(self) -> None:
        for ln in self.lanes:
            self._step_lane(ln)

    def set_sampling(self, temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0,
                     seed: int = 0) -> None:
        """Sample instead of argmax (None-equivalent: set_greedy).  The decode
        graph is re-recorded when the setting changes."""
        self.sampling = dict(temperature=float(temperature), top_k=int(top_k),
                             top_p=float(top_p), seed=int(seed))

    def set_greedy(self) -> None:
        self.sampling = None

    def step_eager(self) -> None:
        """One decode step launched directly (no graph); used by tests."""
        self._advance(1)
        self._step()

    def capture(self) -> None:
        """Records one decode step into a CUDA graph (the capture does not
        execute it); with several lanes each lane is a parallel branch."""
        main = torch.cuda.Stream(self.device)
        main.wait_stream(torch.cuda.current_stream(self.device))
        side = [torch.cuda.Stream(self.device) for _ in self.lanes]
        with torch.cuda.stream(main):
            n0 = N.launch_count()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=main):
                if len(self.lanes) == 1:
                    warm = torch.cuda.Stream(self.device) if self.l2_warm else None
                    if warm is not None:
                        warm.wait_stream(main)
                    self._step_lane(self.lanes[0], warm)
                    if warm is not None:
                        main.wait_stream(warm)
                else:
                    fork = torch.cuda.Event()
                    fork.record(main)
                    for s, ln in zip(side, self.lanes):
                        s.wait_event(fork)
                        with torch.cuda.stream(s):
                            self._step_lane(ln)
                    for s in side:
                        main.wait_stream(s)
            self.launches_per_step = N.launch_count() - n0
        torch.cuda.current_stream(self.device).wait_stream(main)
        self.graph = g
        self._graph_sampling = None if self.sampling is None else dict(self.sampling)

    # ------------------------------------------------------------ prefill
    @torch.inference_mode()
    def prefill(self, input_ids: torch.Tensor) -> None:
        """Runs the prompt through the model (tensor-core GEMMs + flash
        attention, writing the caches) and samples the first new token."""
        B, S = input_ids.shape
        if B != self.batch_size or S >= self.max_seq_len:
            raise ValueError("prompt does not fit the engine's batch / capacity")
        ids = input_ids.to(self.device, non_blocking=True)
        for c in self.caches:
            c.cache_len = 0
        x = ops.embedding(ids, self.emb)
        for blk, c in zip(self.model.transformer_blocs, self.caches):
            x = blk(x, self.cos, self.sin, c, 0)
        h = ops.rmsnorm(x[:, -1], self.nf, self.eps)
        ops.linear(h, self.lm_head, out=self.logits)
        self._pick(self.logits, torch.full((B,), S - 1, dtype=torch.int32, device=self.device),
                   self.tokens)
        self.out_ids[:, :S].copy_(ids)
        self.out_ids[:, S].copy_(self.tokens)
        self.positions.fill_(S)
        self.seqlens.fill_(S + 1)
        self.prompt_len = S
        self._pos = S

    def _advance(self, steps: int) -> None:
        # every step writes one K/V row at the current position and the next
        # output id after it; the device does not bound-check those writes
        if self._pos + steps > self.max_seq_len - 1:
            raise ValueError(f"{steps} more decode steps from position {self._pos} exceed the "
                             f"engine's capacity of {self.max_seq_len} (prefill again first)")
        self._pos += steps

    def decode(self, steps: int) -> None:
        self._advance(steps)
        if self.graph is None or self._graph_sampling != self.sampling:
            self.capture()
        for _ in range(steps):
            self.graph.replay()

    @torch.inference_mode()
    def generate(self, input_ids: torch.Tensor, max_new_token: int,
                 eos_token_id: Optional[int] = None,
                 stop_token_ids: Optional[list] = None, check_every: int = 16) -> torch.Tensor:
        B, S = input_ids.shape
        if S + max_new_token > self.max_seq_len:
            raise ValueError("prompt + max_new_token exceeds the engine capacity")
        self.prefill(input_ids)
        stops = set(stop_token_ids or [])
        if eos_token_id is not None:
            stops.add(eos_token_id)
        remaining = max_new_token - 1
        done = 0
        while remaining > 0:
            n = min(remaining, check_every) if stops else remaining
            self.decode(n)
            remaining -= n
            done += n
            if stops:
                cur = self.out_ids[:, S:S + 1 + done].cpu()
                hit = torch.zeros(B, dtype=torch.bool)
                for t in stops:
                    hit |= (cur == t).any(dim=1)
                if bool(hit.all()):
                    break
        return self.out_ids[:, :S + 1 + done]
