"""Parity at the exact shapes the benchmark times, against the fp32 CPU oracle.

- Config 4: the Qwen3-0.6B-shaped model (28 layers, width 1024, 16/8 heads of
  128, SwiGLU 3072, vocab 151936, bf16, weights ~N(0, 0.02)) served by the
  decode engine at batch 32 with a 512-token prompt -- the engine, launch plans
  and CUDA graph the headline number comes from.  The prefill's last-position
  logits and three teacher-forced graph-replayed decode steps are compared
  with oracle/model.py on a subset of the 32 rows (rows are independent; the
  GPU still runs all 32).  The decode steps start from the engine's own
  prefilled KV cache, so each step is checked on its own.
- Config 2: RoPE on Q [4,16,2048,128] / K [4,8,2048,128] and causal GQA
  prefill attention at B4 S2048 Hq16 Hkv8 D128, fp16.
- Config 5: sliding-window (4096) GQA decode, B64 Hq16 Hkv8 D128 bf16, at
  cache lengths 16k and 32k (contiguous) and 4k (paged, shuffled blocks).

Kernel tolerance (the suite's): max |err| <= 2e-2 * max(1, |ref|) against the
fp32 oracle, mean |err| <= 1e-3 against the oracle rounded once to the output
dtype.  Model tolerance (logits of the 28-layer bf16 model): the same
formulation evaluated eagerly with every module output stored in bf16 -- the
reference's own eager model at the model's dtype (oracle/model.py with
store_dtype) -- differs from the fp32 oracle by ~3.6e-2 max (relative) and
~6e-3 mean on these logits, from bf16 storage alone.  The engine must be at
least as close to the fp32 oracle as that: its max and mean errors at most
1.25x the bf16 eager formulation's (+1e-3).  Every token the engine picks must
also be an argmax of the fp32 oracle's logits up to 2e-2 * max(1, |logit|).
"""
import pytest
import torch

from oracle import model as OM
from oracle import ops as O
from torchplusplus_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda"

MAX_ABS = 2e-2
MEAN_ABS = 1e-3
MODEL_SLACK = 1.25     # engine error / bf16 eager error (both against fp32)


def _errs(y, ref):
    """(max |err| / max(1, |ref|), mean |err|) of y against the fp32 ref."""
    y = y.detach().float().cpu()
    ref = ref.float()
    assert y.shape == ref.shape, (y.shape, ref.shape)
    assert torch.isfinite(y).all()
    return ((y - ref).abs() / ref.abs().clamp(min=1.0)).max().item(), \
        (y - ref).abs().mean().item()


def _check(y, ref, what=""):
    dt = y.dtype
    y = y.detach().float().cpu()
    ref = ref.float()
    assert y.shape == ref.shape, (y.shape, ref.shape)
    assert torch.isfinite(y).all()
    mx = ((y - ref).abs() / ref.abs().clamp(min=1.0)).max().item()
    mean = (y - ref.to(dt).float()).abs().mean().item()
    assert mx <= MAX_ABS and mean <= MEAN_ABS, f"{what}: max {mx:.3g} mean {mean:.3g}"


def _check_model(y, ref32, ref16, what=""):
    """Engine logits y vs the fp32 oracle, bounded by the bf16 eager
    formulation's own distance from it."""
    gm, ga = _errs(y, ref32)
    em, ea = _errs(ref16, ref32)
    assert gm <= MODEL_SLACK * em + 1e-3 and ga <= MODEL_SLACK * ea + 1e-3, \
        f"{what}: engine max {gm:.3g} mean {ga:.3g}; bf16 eager max {em:.3g} mean {ea:.3g}"


# ------------------------------------------------------------------ config 4
ROWS = [0, 13, 31]      # rows of the 32-sequence batch compared with the oracle


@pytest.fixture(scope="module")
def qwen3_0p6b():
    from torchplusplus_b200.llmops.qwen3 import Qwen3, Qwen3Config
    cfg = Qwen3Config()
    torch.manual_seed(0)
    m = Qwen3(cfg, device=DEV).init_weights(0.02, seed=0)
    sd = {k: v.detach().float().cpu() for k, v in m.state_dict().items()}
    ids = torch.randint(0, cfg.vocab_size, (32, 512), generator=torch.Generator().manual_seed(4))
    yield m, sd, ids
    m._engine = None
    del m
    torch.cuda.empty_cache()


@pytest.mark.parametrize("weight_format", ["native", "fp8_head"])
def test_config4_engine_prefill_and_decode_match_oracle(qwen3_0p6b, weight_format):
    m, sd, ids = qwen3_0p6b
    cfg = m.cfg
    eng = m.engine(32, 576, weight_format=weight_format)
    f = dict(sd)
    if weight_format == "fp8_head":
        # the LM head runs on the e4m3 copy of (final-norm-folded) weights:
        # the oracle uses its dequantized value, with the norm weight folded
        f["out_head.weight"] = eng.lm_head_f8.dequantize().float().cpu()
        f["final_rmsnorm.weight"] = torch.ones_like(f["final_rmsnorm.weight"])
    with torch.inference_mode():
        eng.prefill(ids)
        torch.cuda.synchronize()
        pre = eng.logits[ROWS].float().cpu()
        # snapshot the prefilled cache rows of the compared sequences
        kc = [c.k_cache[ROWS, :, :515].float().cpu() for c in eng.caches]
        vc = [c.v_cache[ROWS, :, :515].float().cpu() for c in eng.caches]
        steps = []
        for _ in range(3):
            eng.decode(1)           # graph replay: the benchmarked step
            steps.append(eng.logits[ROWS].float().cpu())
        out_ids = eng.out_ids[ROWS, :516].cpu()
    assert ops.device_error() == 0
    # prefill: the unfused bf16 LM head on the final-norm output (native head
    # in both formats; fp8 applies to the decode step)
    ref = OM.forward(sd, cfg, ids[ROWS], last_only=True)[:, 0]
    ref16 = OM.forward(sd, cfg, ids[ROWS], last_only=True, store_dtype=torch.bfloat16)[:, 0]
    _check_model(pre, ref, ref16, "prefill logits")
    # teacher-forced decode steps from the engine's cache and tokens
    kc, vc = [t.clone() for t in kc], [t.clone() for t in vc]     # writable outside inference
    kc16, vc16 = [t.clone() for t in kc], [t.clone() for t in vc]
    for t, lg in enumerate(steps):
        pos = 512 + t
        tok = out_ids[:, pos]
        ref = OM.decode_logits_cached(f, cfg, tok, kc, vc, pos)
        ref16 = OM.decode_logits_cached(f, cfg, tok, kc16, vc16, pos, store_dtype=torch.bfloat16)
        _check_model(lg, ref, ref16, f"decode step {t}")
        picked = ref.gather(1, out_ids[:, pos + 1][:, None])[:, 0]
        best = ref.max(1).values
        assert bool((picked >= best - MAX_ABS * best.abs().clamp(min=1.0)).all()), t


# ------------------------------------------------------------------ config 2
def test_config2_rope_and_causal_gqa_prefill_match_oracle():
    g = torch.Generator().manual_seed(20)
    B, S, Hq, Hkv, D = 4, 2048, 16, 8, 128
    q = torch.randn(B, Hq, S, D, generator=g).half()
    k = torch.randn(B, Hkv, S, D, generator=g).half()
    v = torch.randn(B, S, Hkv, D, generator=g).half()
    cos, sin = O.compute_rope_params(D, 1e6, S)
    qr = ops.rope(q.to(DEV), cos.to(DEV), sin.to(DEV))
    kr = ops.rope(k.to(DEV), cos.to(DEV), sin.to(DEV))
    _check(qr, O.rope(q, cos, sin), what="rope q")
    _check(kr, O.rope(k, cos, sin), what="rope k")
    # attention on the rotated tensors, [B,S,H,D] views as the GQA module passes
    o = ops.attention(qr.transpose(1, 2), kr.transpose(1, 2), v.to(DEV), causal=True)
    qh, kh = qr.transpose(1, 2).cpu(), kr.transpose(1, 2).cpu()
    o = o.cpu()
    G = Hq // Hkv
    for b in range(B):
        for h in range(Hkv):
            hs = slice(h * G, (h + 1) * G)
            ref = O.attention(qh[b:b + 1, :, hs], kh[b:b + 1, :, h:h + 1],
                              v[b:b + 1, :, h:h + 1], causal=True)
            _check(o[b:b + 1, :, hs], ref, what=f"attention b{b} kv{h}")


# ------------------------------------------------------------------ config 5
def _swa_oracle(q, kc, vc, lens, window):
    """Oracle over each sequence's last `window` keys only (copied to the host)."""
    B = q.shape[0]
    out = []
    for b in range(B):
        L = int(lens[b])
        lo = max(0, L - window)
        ks = kc[b:b + 1, :, lo:L].float().cpu()
        vs = vc[b:b + 1, :, lo:L].float().cpu()
        out.append(O.attention_decode(q[b:b + 1].cpu(), ks, vs, torch.tensor([L - lo]),
                                      window_left=window - 1))
    return torch.cat(out)


@pytest.mark.parametrize("L", [16384, 32768])
def test_config5_swa_decode_long_cache_matches_oracle(L):
    B, Hq, Hkv, D, W = 64, 16, 8, 128, 4096
    g = torch.Generator(device=DEV).manual_seed(L)
    kc = torch.randn(B, Hkv, L, D, generator=g, device=DEV, dtype=torch.bfloat16)
    vc = torch.randn(B, Hkv, L, D, generator=g, device=DEV, dtype=torch.bfloat16)
    q = torch.randn(B, Hq, D, generator=g, device=DEV, dtype=torch.bfloat16)
    # the benchmarked case (every sequence full) plus a few ragged lengths
    lens = [L] * B
    lens[5], lens[17], lens[40], lens[63] = L - 1, W - 3, 1, L - W - 77
    sl = torch.tensor(lens, dtype=torch.int32, device=DEV)
    y = ops.attention_decode(q, kc, vc, sl, L, window_left=W - 1)
    _check(y, _swa_oracle(q, kc, vc, lens, W), what=f"swa L{L}")
    del kc, vc
    torch.cuda.empty_cache()


def test_config5_swa_decode_paged_matches_oracle():
    B, Hq, Hkv, D, W, L = 64, 16, 8, 128, 4096, 4096
    g = torch.Generator(device=DEV).manual_seed(5)
    kc = torch.randn(B, Hkv, L, D, generator=g, device=DEV, dtype=torch.bfloat16)
    vc = torch.randn(B, Hkv, L, D, generator=g, device=DEV, dtype=torch.bfloat16)
    q = torch.randn(B, Hq, D, generator=g, device=DEV, dtype=torch.bfloat16)
    nblk = L // 64
    perm = torch.randperm(B * nblk, generator=g, device=DEV)
    table = perm.view(B, nblk).to(torch.int32)
    kp = torch.empty(B * nblk, Hkv, 64, D, dtype=torch.bfloat16, device=DEV)
    vp = torch.empty_like(kp)
    ops.kv_append_paged(kc, vc, kp, vp, table, start_pos=0)
    lens = [L] * B
    lens[3], lens[30] = 65, L - 63
    sl = torch.tensor(lens, dtype=torch.int32, device=DEV)
    y = ops.attention_decode_paged(q, kp, vp, table, sl, L, window_left=W - 1)
    _check(y, _swa_oracle(q, kc, vc, lens, W), what="swa paged L4096")
