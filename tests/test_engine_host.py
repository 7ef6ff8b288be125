"""CPU checks of the engine's host-side pieces (no kernel launches): nucleus
sampling (engine.py:493-511), the RoPE tables and rotation (engine.py:130-158)
and the preallocated KV cache's reference-style (k, v) views."""
import numpy as np
import torch


def test_sample_greedy_and_nucleus_keep_set():
    import engine
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(3, 50, generator=g)
    assert torch.equal(engine._sample(logits, 0.0, 0.9), logits.argmax(-1))
    # a nucleus smaller than the top probability keeps only the top token
    peaked = torch.zeros(1, 10)
    peaked[0, 7] = 10.0
    for _ in range(20):
        assert int(engine._sample(peaked, 1.0, 0.5)) == 7
    # kept set = tokens whose preceding cumulative mass is below top_p: never sample outside it
    probs = torch.tensor([[0.4, 0.3, 0.2, 0.1]])
    lg = probs.log()
    seen = set()
    torch.manual_seed(1)
    for _ in range(300):
        seen.add(int(engine._sample(lg, 1.0, 0.65)))
    assert seen == {0, 1}          # 0 (before: 0.0) and 1 (before: 0.4) are kept, 2 (before: 0.7) is not


def test_rope_tables_and_rotation():
    import engine
    cos, sin = engine.build_rope_cache(64, 128, 500000.0)
    half = 64
    inv = 1.0 / (500000.0 ** (np.arange(half) / half))
    ang = np.arange(64)[:, None] * inv[None, :]
    assert np.allclose(cos.numpy(), np.cos(ang), atol=2e-5)     # fp32 angles, as the reference builds them
    assert np.allclose(sin.numpy(), np.sin(ang), atol=2e-5)
    x = torch.randn(2, 4, 5, 128, dtype=torch.float64)
    r = engine._rotate(x, cos[:5].double(), sin[:5].double())
    a, b = x[..., :half].numpy(), x[..., half:].numpy()
    c, s = np.cos(ang[:5]), np.sin(ang[:5])
    assert np.allclose(r[..., :half].numpy(), a * c - b * s, atol=1e-6)
    assert np.allclose(r[..., half:].numpy(), a * s + b * c, atol=1e-6)
    # a rotation keeps each (i, i + half) pair's length
    assert torch.allclose(r[..., :half] ** 2 + r[..., half:] ** 2, x[..., :half] ** 2 + x[..., half:] ** 2)


def test_kv_cache_views():
    import engine
    c = engine.KVCache(3, 1, 8, 16, 128, "cpu")
    assert len(c) == 3
    c.length = 5
    k, v = c[1]
    assert k.shape == (1, 8, 5, 128) and v.shape == (1, 8, 5, 128)
    assert k.shape[2] == c.length          # the reference reads past_len as kv[0][0].shape[2]
