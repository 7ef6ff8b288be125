"""GPU parity of the fused one-token attention kernels against plain PyTorch fp32.

* hc_attn_decode (RoPE, KV-cache write, grouped-query attention over
  positions 0..pos; the reference's LlamaAttention for one token,
  engine.py:100-125, :130-158) against an fp32 restatement, for several
  positions and head groupings, including a position outside the cache.
* hc_fp8_gemv_ex (input_layernorm fused before the q/k/v GEMV, the residual
  fused after the o GEMV) against fp32 torch on the same e4m3 weights.
* DesdemonaEngine one-token steps through the fused kernels against the same
  steps through the torch attention path.
"""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def N():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import hc_native
    return hc_native


def _rope_tables(cap, half=64, theta=500000.0):
    inv = 1.0 / (theta ** (torch.arange(half, device="cuda").float() / half))
    ang = torch.arange(cap, device="cuda").float()[:, None] * inv[None, :]
    return torch.cos(ang).contiguous(), torch.sin(ang).contiguous()


def _rot(x, c, s):
    d = x.shape[-1] // 2
    a, b = x[..., :d], x[..., d:]
    return torch.cat((a * c - b * s, a * s + b * c), dim=-1)


def _reference(qkv, kc, vc, cos, sin, pos, nq, nkv):
    """fp32: rotated q / k, the new k / v at pos, softmax(q k^T / sqrt(128)) v."""
    D = 128
    q = qkv[:nq * D].float().view(nq, D)
    k = qkv[nq * D:(nq + nkv) * D].float().view(nkv, D)
    v = qkv[(nq + nkv) * D:].view(nkv, D)
    c, s = cos[pos], sin[pos]
    q, k = _rot(q, c, s), _rot(k, c, s)
    kc, vc = kc.clone(), vc.clone()
    kc[:, pos] = k.half()
    vc[:, pos] = v
    g = nq // nkv
    keys = kc[:, :pos + 1].float().repeat_interleave(g, dim=0)          # [nq, n, D]
    vals = vc[:, :pos + 1].float().repeat_interleave(g, dim=0)
    sc = torch.einsum("hd,hnd->hn", q, keys) / math.sqrt(D)
    out = torch.einsum("hn,hnd->hd", torch.softmax(sc, dim=-1), vals)
    return out.reshape(-1), kc, vc


@pytest.mark.parametrize("nq,nkv", [(32, 8), (8, 8), (16, 2)])
@pytest.mark.parametrize("pos", [0, 5, 100, 767])
def test_attn_decode_matches_fp32(N, nq, nkv, pos):
    cap, D = 768, 128
    g = torch.Generator(device="cuda").manual_seed(pos * 7 + nq)
    qkv = torch.randn((nq + 2 * nkv) * D, generator=g, device="cuda").half()
    kc = torch.randn(nkv, cap, D, generator=g, device="cuda").half()
    vc = torch.randn(nkv, cap, D, generator=g, device="cuda").half()
    cos, sin = _rope_tables(cap)
    ref, kref, vref = _reference(qkv, kc, vc, cos, sin, pos, nq, nkv)
    out = torch.empty(nq * D, dtype=torch.float16, device="cuda")
    st = N.new_status("cuda")
    p = torch.tensor([pos], dtype=torch.int64, device="cuda")
    for _ in range(2):
        kw, vw = kc.clone(), vc.clone()
        N.check(N.lib.hc_attn_decode(N.ptr(qkv), N.ptr(cos), N.ptr(sin), N.ptr(p), N.ptr(kw), N.ptr(vw), cap, nq,
                                     nkv, D, N.ptr(out), N.ptr(st), N.stream_handle()), "hc_attn_decode")
        torch.cuda.synchronize()
        N.read_status(st, "hc_attn_decode")
        rel = ((out.float() - ref).norm() / ref.norm()).item()
        assert rel < 2e-3, rel               # fp16 output; fp32 softmax
        assert torch.equal(vw, vref)
        dk = (kw.float() - kref.float()).abs().max().item()
        assert dk <= 2e-3 * max(1.0, kref.float().abs().max().item()), dk     # one fp16 rounding apart at most


def test_attn_decode_position_outside_cache(N):
    cap, D, nq, nkv = 64, 128, 8, 2
    qkv = torch.randn((nq + 2 * nkv) * D, device="cuda").half()
    kc = torch.zeros(nkv, cap, D, dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    cos, sin = _rope_tables(cap)
    out = torch.zeros(nq * D, dtype=torch.float16, device="cuda")
    st = N.new_status("cuda")
    p = torch.tensor([cap], dtype=torch.int64, device="cuda")
    N.check(N.lib.hc_attn_decode(N.ptr(qkv), N.ptr(cos), N.ptr(sin), N.ptr(p), N.ptr(kc), N.ptr(vc), cap, nq, nkv,
                                 D, N.ptr(out), N.ptr(st), N.stream_handle()), "hc_attn_decode")
    torch.cuda.synchronize()
    assert int(st.item()) & N.HC_ERR_RANGE
    assert int(kc.count_nonzero()) == 0 and int(out.count_nonzero()) == 0
    # argument errors come back as HC_ERR_ARG
    assert N.lib.hc_attn_decode(N.ptr(qkv), N.ptr(cos), N.ptr(sin), N.ptr(p), N.ptr(kc), N.ptr(vc), cap, nq, nkv,
                                64, N.ptr(out), N.ptr(st), N.stream_handle()) == N.HC_ERR_ARG
    for bad_nq, bad_nkv in ((12, 8), (32, 2)):       # not a multiple / more than 8 query heads a group
        assert N.lib.hc_attn_decode(N.ptr(qkv), N.ptr(cos), N.ptr(sin), N.ptr(p), N.ptr(kc), N.ptr(vc), cap, bad_nq,
                                    bad_nkv, D, N.ptr(out), N.ptr(st), N.stream_handle()) == N.HC_ERR_ARG


def test_fp8_gemv_ex_norm_and_residual(N):
    H, rows = 4096, 6144
    g = torch.Generator(device="cuda").manual_seed(3)
    w8 = (torch.randn(rows, H, generator=g, device="cuda") * 0.02).to(torch.float8_e4m3fn)
    x = (torch.randn(H, generator=g, device="cuda") * 3).half()
    nw = (1.0 + 0.1 * torch.randn(H, generator=g, device="cuda")).half()
    eps = 1e-5
    y = torch.empty(rows, dtype=torch.float16, device="cuda")
    N.check(N.lib.hc_fp8_gemv_ex(N.ptr(w8.view(torch.uint8)), None, rows, H, N.ptr(x), N.ptr(nw), eps, None,
                                 N.ptr(y), N.stream_handle()), "hc_fp8_gemv_ex")
    xf = x.float()
    xn = (xf * torch.rsqrt(xf.pow(2).mean() + eps) * nw.float()).half().float()
    ref = w8.float() @ xn
    assert ((y.float() - ref).norm() / ref.norm()).item() < 2e-3
    # residual: y = r + W x (in place on r as well)
    r = torch.randn(H, generator=g, device="cuda").half()
    wo = (torch.randn(H, H, generator=g, device="cuda") * 0.02).to(torch.float8_e4m3fn)
    a = torch.randn(H, generator=g, device="cuda").half()
    y2 = torch.empty(H, dtype=torch.float16, device="cuda")
    N.check(N.lib.hc_fp8_gemv_ex(N.ptr(wo.view(torch.uint8)), None, H, H, N.ptr(a), None, 0.0, N.ptr(r),
                                 N.ptr(y2), N.stream_handle()), "hc_fp8_gemv_ex")
    ref2 = r.float() + wo.float() @ a.float()
    assert ((y2.float() - ref2).norm() / ref2.norm()).item() < 2e-3
    r2 = r.clone()
    N.check(N.lib.hc_fp8_gemv_ex(N.ptr(wo.view(torch.uint8)), None, H, H, N.ptr(a), None, 0.0, N.ptr(r2),
                                 N.ptr(r2), N.stream_handle()), "hc_fp8_gemv_ex")
    assert torch.equal(r2, y2)
    # a residual that partly overlaps y is refused
    buf = torch.empty(2 * H, dtype=torch.float16, device="cuda")
    assert N.lib.hc_fp8_gemv_ex(N.ptr(wo.view(torch.uint8)), None, H, H, N.ptr(a), None, 0.0, N.ptr(buf),
                                N.ptr(buf) + 2, N.stream_handle()) == N.HC_ERR_ARG


def test_engine_fused_attention_matches_torch_attention():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import engine
    import hc_synth
    from predictor import PredictorRegistry
    L, H, vocab, nq, nkv = 2, 4096, 512, 32, 8
    syn = hc_synth.make_stack(n_layers=L, inter=2048, hot_frac=0.2, rank=64, activation="silu", act_on_both=False,
                              seed=5)
    g = torch.Generator(device="cuda").manual_seed(9)
    shared = {}
    for li in range(L):
        for name, rows in (("q_proj", H), ("k_proj", nkv * 128), ("v_proj", nkv * 128), ("o_proj", H)):
            shared[f"layer_{li:03d}.{name}"] = (torch.randn(rows, H, generator=g, device="cuda") * 0.02).to(
                torch.float8_e4m3fn)
        shared[f"layer_{li:03d}.input_layernorm"] = (1 + 0.1 * torch.randn(H, generator=g, device="cuda")).half()
        shared[f"layer_{li:03d}.post_attention_layernorm"] = syn.norms[li].half()
    shared["embed_tokens"] = torch.randn(vocab, H, generator=g, device="cuda").half()
    shared["lm_head"] = (torch.randn(vocab, H, generator=g, device="cuda") * 0.02).half()
    shared["final_norm"] = torch.ones(H, dtype=torch.float16, device="cuda")
    cfg = {"hidden_dim": H, "intermediate_dim": 2048, "num_layers": L, "vocab_size": vocab,
           "num_attention_heads": nq, "num_key_value_heads": nkv, "rope_theta": 500000.0, "rms_norm_eps": 1e-5,
           "hidden_act": "silu", "act_on_both": False, "max_position_embeddings": 256, "num_experts": 1}
    reg = PredictorRegistry.__new__(PredictorRegistry)
    reg.device = "cuda"
    reg.predictors = {(li, 0): p for li, p in enumerate(syn.predictors)}
    eng = engine.DesdemonaEngine.from_parts(cfg, shared, syn.store, syn.hot, reg, device="cuda", max_seq_len=256)
    assert all(a.fused_decode for a in eng.attention_layers)
    prompt = torch.randint(0, vocab, (1, 40), generator=torch.Generator().manual_seed(1)).cuda()
    outs = {}
    for fused in (True, False):
        eng.fused_attention = fused
        cache = eng.new_cache(1, 64)
        eng.forward(prompt, cache)                   # prefill: torch attention in both runs
        toks = [3, 17, 200, 45]
        logits = []
        for t in toks:                               # eager one-token steps
            lg, cache = eng.forward(torch.tensor([[t]], device="cuda"), cache)
            logits.append(lg[0, -1].float())
        # and through the captured graph
        eng._graph = None
        logits.append(eng.decode_step(torch.tensor([9], device="cuda"), cache)[0].float().clone())
        torch.cuda.synchronize()
        eng.check()
        outs[fused] = (torch.stack(logits), cache.k.clone(), cache.v.clone())
    la, lb = outs[True][0], outs[False][0]
    rel = ((la - lb).norm(dim=1) / lb.norm(dim=1)).max().item()
    assert rel < 1e-2, rel
    n = 40 + 5
    dk = ((outs[True][1][:, :, :, :n].float() - outs[False][1][:, :, :, :n].float()).norm() /
          outs[False][1][:, :, :, :n].float().norm()).item()
    assert dk < 5e-3, dk
    eng.close()
