"""Generate the golden fixtures in this directory by running the REFERENCE's own code.

Run once, in a container where the reference checkout is available:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py <reference checkout dir>

Nothing at test time imports the reference; tests read only the files written
here.  What is produced (all from reference code paths, seeds fixed):

* ``quant.npz``          quantize_int4 / dequantize_int4 on edge-case vectors
                         (splitter.py:81-124).
* ``split/``             a real split written by ``splitter.split_dense``
                         (splitter.py:129-302) for a stub 2-layer model with
                         H=4096, I=40, hot_count=8 (cold_weights.bin,
                         cold_index.npy, hot_weights/layer_*.pt, split_config.json).
                         Model loading is stubbed (no network / no checkpoint).
* ``store_reads.npz``    ColdWeightStore.read_neurons on that split
                         (splitter.py:354-403), incl. absent / repeated ids.
* ``unsorted/``          the reference test fixture's cold file
                         (tests/common.py:31-104: unsorted ids, N(0,1) values)
                         plus read-backs.
* ``predictors/``        one NeuronPredictor.save file (predictor.py:83-90),
                         rank 16, for layer 0 of the split.
* ``predictor.npz``      predict_mask / forward outputs (predictor.py:70-79).
* ``ffn.npz``            engine.sparse_ffn (engine.py:173-209) for SwiGLU and
                         dReLU, and SparseFFNLayer.forward / _cold_ids_for
                         (engine.py:274-312) with the predictor registry.
* ``engine.npz``         the reference's DesdemonaEngine (engine.py:317-511)
                         on a split of the 2-layer Llama-geometry stub of
                         stub_models.py written by the reference's split_dense:
                         prefill logits, greedy generate() tokens, the logits of
                         every decode step with the cache, the cold ids each
                         layer fetched, and the split's small files
                         (split_config.json, cold_index.npy, a digest of
                         cold_weights.bin).  ``make_golden.py <ref> engine``
                         regenerates only this file.
"""

from __future__ import annotations

import json
import os
import shutil
import sys
import tempfile
import types
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _stub_model(seed: int, n_layers: int, H: int, I: int, act: str, model_type: str):
    """A stand-in for AutoModelForCausalLM.from_pretrained(..., torch_dtype=fp16):
    only the attributes split_dense reads (splitter.py:151-183, :195-198, :265-289)."""
    g = torch.Generator().manual_seed(seed)
    lin = lambda o, i, std=0.02: types.SimpleNamespace(
        weight=types.SimpleNamespace(data=(torch.randn(o, i, generator=g) * std).half()))
    norm = lambda n: types.SimpleNamespace(
        weight=types.SimpleNamespace(data=(1.0 + 0.1 * torch.randn(n, generator=g)).half()))
    layers = []
    for _ in range(n_layers):
        attn = types.SimpleNamespace(q_proj=lin(8, 8), k_proj=lin(8, 8), v_proj=lin(8, 8), o_proj=lin(8, 8))
        mlp = types.SimpleNamespace(gate_proj=lin(I, H), up_proj=lin(I, H), down_proj=lin(H, I))
        layers.append(types.SimpleNamespace(self_attn=attn, mlp=mlp,
                                            input_layernorm=norm(H), post_attention_layernorm=norm(H)))
    inner = types.SimpleNamespace(layers=layers, embed_tokens=lin(16, H), norm=norm(H))
    cfg = types.SimpleNamespace(hidden_size=H, num_hidden_layers=n_layers, intermediate_size=I,
                                vocab_size=16, num_attention_heads=32, num_key_value_heads=8,
                                rope_theta=10000.0, rms_norm_eps=1e-5, hidden_act=act,
                                model_type=model_type, max_position_embeddings=256)
    return types.SimpleNamespace(config=cfg, model=inner, lm_head=lin(16, H))


def main(ref_dir: str):
    sys.path.insert(0, ref_dir)
    import splitter  # noqa: E402  (reference)
    import predictor as ref_predictor  # noqa: E402
    import engine as ref_engine  # noqa: E402

    torch.manual_seed(0)
    H = splitter.HIDDEN_DIM

    # ---------------------------------------------------------------- quant
    vecs = {
        "randn3": torch.randn(4096) * 3.0,
        "randn002": torch.randn(4096) * 0.02,
        "zeros": torch.zeros(4096),
        "extreme": torch.tensor([100.0, -100.0, 50.0, -50.0] * 32),
        "short100": torch.randn(100),
        "ties": (torch.arange(4096, dtype=torch.float32) % 15 - 7) * 0.5,
    }
    q = {}
    for name, v in vecs.items():
        packed, scales = splitter.quantize_int4(v)
        n = v.numel()
        q[f"{name}_x"] = v.numpy()
        q[f"{name}_packed"] = np.frombuffer(packed, np.uint8).copy()
        q[f"{name}_scales"] = scales.numpy()
        q[f"{name}_deq"] = splitter.dequantize_int4(packed, scales, n).numpy()
        q[f"{name}_deq16"] = splitter.dequantize_int4(packed, scales.half().float(), n).numpy()
    np.savez_compressed(HERE / "quant.npz", **q)

    # ---------------------------------------------------------------- split
    n_layers, I, hot_count = 2, 40, 8
    stub = _stub_model(1, n_layers, H, I, "silu", "llama")
    splitter.AutoModelForCausalLM = types.SimpleNamespace(from_pretrained=lambda *a, **k: stub)
    work = Path(tempfile.mkdtemp())
    gen = torch.Generator().manual_seed(2)
    profile = {"layers": {str(li): {"expert_0": torch.rand(I, generator=gen).tolist()}
                          for li in range(n_layers)}}
    (work / "profile.json").write_text(json.dumps(profile))
    splitter.split_dense("stub-model", str(work / "profile.json"), str(work / "split"), hot_count=hot_count)
    out_split = HERE / "split"
    if out_split.exists():
        shutil.rmtree(out_split)
    (out_split / "hot_weights").mkdir(parents=True)
    for f in ("cold_weights.bin", "cold_index.npy", "split_config.json"):
        shutil.copy(work / "split" / f, out_split / f)
    for li in range(n_layers):
        f = f"layer_{li:03d}_expert_000.pt"
        shutil.copy(work / "split" / "hot_weights" / f, out_split / "hot_weights" / f)
    # the post-attention norms live in shared.pt (splitter.py:179); keep only those
    shared = torch.load(work / "split" / "hot_weights" / "shared.pt")
    norms = {f"layer_{li:03d}.post_attention_layernorm": shared[f"layer_{li:03d}.post_attention_layernorm"]
             for li in range(n_layers)}
    np.savez_compressed(out_split / "norms.npz", **{k: v.float().numpy() for k, v in norms.items()})

    cfg = json.loads((out_split / "split_config.json").read_text())
    store = splitter.ColdWeightStore(str(out_split / "cold_weights.bin"),
                                     str(out_split / "cold_index.npy"), cfg)
    hot0 = torch.load(out_split / "hot_weights" / "layer_000_expert_000.pt")
    cold_ids0 = [i for i in range(I) if i not in set(hot0["neuron_ids"].tolist())]
    reads = {}
    req_lists = {
        "l0_all": cold_ids0[:8],
        "l0_mixed": [cold_ids0[5], 9999, cold_ids0[0], cold_ids0[5], hot0["neuron_ids"][0].item(), cold_ids0[-1]],
        "l1_rev": list(reversed([i for i in range(I) if i not in set(
            torch.load(out_split / "hot_weights" / "layer_001_expert_000.pt")["neuron_ids"].tolist())]))[:7],
    }
    for name, ids in req_lists.items():
        li = 0 if name.startswith("l0") else 1
        r = store.read_neurons(li, 0, ids)
        reads[f"{name}_ids"] = np.asarray(ids, np.int64)
        reads[f"{name}_gate"], reads[f"{name}_up"], reads[f"{name}_down"] = (t.numpy() for t in r)
    reads["none_ids"] = np.asarray([9999, 10000], np.int64)
    reads["none_is_none"] = np.asarray([store.read_neurons(0, 0, [9999, 10000]) is None])
    np.savez_compressed(HERE / "store_reads.npz", **reads)

    # ------------------------------------------------ reference test fixture file
    sys.path.insert(0, ref_dir)
    from tests.common import build_synthetic_cold_file  # reference fixture
    uns = HERE / "unsorted"
    if uns.exists():
        shutil.rmtree(uns)
    ub, ui, ucfg, truth = build_synthetic_cold_file(str(uns), num_layers=2, n_cold=8, seed=3)
    tr = {}
    for (li, nid), v in truth.items():
        tr[f"{li}_{nid}_gate"] = v["gate"].numpy()
        tr[f"{li}_{nid}_up"] = v["up"].numpy()
        tr[f"{li}_{nid}_down"] = v["down"].numpy()
    np.savez_compressed(uns / "truth.npz", **tr)
    (uns / "config.json").write_text(json.dumps(ucfg))

    # ---------------------------------------------------------------- predictor
    pdir = HERE / "predictors"
    if pdir.exists():
        shutil.rmtree(pdir)
    pdir.mkdir()
    torch.manual_seed(4)
    pred = ref_predictor.NeuronPredictor(H, I, rank=16)
    with torch.no_grad():
        pred.up.bias.mul_(20.0)  # spread the logits so the set is mixed
    pred.save(str(pdir / "layer_000_expert_000.pt"))
    xs = torch.randn(16, H)
    xs[3] = 0.0
    with torch.no_grad():
        probs = pred(xs)
        mask = pred.predict_mask(xs, 0.5)
        mask_hi = pred.predict_mask(xs, 0.7)
    reg = ref_predictor.PredictorRegistry(str(pdir), device="cpu")
    with torch.no_grad():
        reg_mask = reg.predict(0, 0, xs[:4].half())
    np.savez_compressed(HERE / "predictor.npz", x=xs.numpy(), probs=probs.numpy(),
                        mask=mask.numpy(), mask_07=mask_hi.numpy(),
                        reg_mask_fp16_in=reg_mask.numpy(),
                        reg_missing_is_none=np.asarray([reg.predict(1, 0, xs[:1]) is None]))

    # ---------------------------------------------------------------- FFN
    ffn = {}
    torch.manual_seed(5)
    x16 = torch.randn(2, H).half()
    hot_f16 = (hot0["gate"].half(), hot0["up"].half(), hot0["down"].half())
    cg, cu, cd = store.read_neurons(0, 0, cold_ids0)
    ffn["x16"] = x16.float().numpy()
    for tag, act, both in (("swiglu", "silu", False), ("drelu", "relu", True)):
        y = ref_engine.sparse_ffn(x16, act, both, *hot_f16, cg, cu, cd)
        ffn[f"sparse_{tag}"] = y.float().numpy()
        y_hot = ref_engine.sparse_ffn(x16, act, both, *hot_f16, None, None, None)
        ffn[f"sparse_{tag}_hotonly"] = y_hot.float().numpy()
    ffn["sparse_empty"] = ref_engine.sparse_ffn(x16, "silu", False, None, None, None, None, None, None).float().numpy()

    # SparseFFNLayer with the predictor registry (engine.py:212-312)
    pex = ThreadPoolExecutor(2)
    xin = (torch.randn(1, 1, H) * 2).half()
    ffn["layer_x"] = xin.float().numpy()
    for tag, act, both in (("swiglu", "silu", False), ("drelu", "relu", True)):
        lcfg = dict(cfg, hidden_act=act, act_on_both=both)
        layer = ref_engine.SparseFFNLayer(0, str(out_split / "hot_weights"), store, reg, lcfg,
                                          torch.device("cpu"), pex,
                                          ffn_norm_weight=norms["layer_000.post_attention_layernorm"])
        with torch.no_grad():
            xn = layer.input_layernorm(xin)
            ids = layer._cold_ids_for(xn)
            y = layer(xin)
        ffn[f"layer_{tag}_ids"] = np.asarray(ids, np.int64)
        ffn[f"layer_{tag}_y"] = y.float().numpy()
        ffn[f"layer_{tag}_xn"] = xn.float().numpy()
        layer_np = ref_engine.SparseFFNLayer(0, str(out_split / "hot_weights"), store, None, lcfg,
                                             torch.device("cpu"), pex,
                                             ffn_norm_weight=norms["layer_000.post_attention_layernorm"])
        with torch.no_grad():
            ffn[f"layer_{tag}_nopred_ids"] = np.asarray(layer_np._cold_ids_for(xn), np.int64)
            ffn[f"layer_{tag}_nopred_y"] = layer_np(xin).float().numpy()
    pex.shutdown()
    np.savez_compressed(HERE / "ffn.npz", **ffn)
    store.close()
    shutil.rmtree(work)
    print("golden fixtures written to", HERE)


def engine_main(ref_dir: str):
    """engine.npz: the reference's own engine, run on the CPU in fp16."""
    import hashlib
    sys.path.insert(0, ref_dir)
    sys.path.insert(0, str(HERE))
    import splitter  # noqa: E402  (reference)
    import predictor as ref_predictor  # noqa: E402
    import engine as ref_engine  # noqa: E402
    import stub_models as SM  # noqa: E402

    n_layers, inter, hot_count, vocab = 2, 64, 16, 64
    stub = SM.engine_stub_model(11, n_layers, inter, vocab)
    splitter.AutoModelForCausalLM = types.SimpleNamespace(from_pretrained=lambda *a, **k: stub)
    work = Path(tempfile.mkdtemp())
    (work / "profile.json").write_text(json.dumps(SM.engine_stub_profile(12, n_layers, inter)))
    splitter.split_dense("engine-stub", str(work / "profile.json"), str(work / "split"), hot_count=hot_count)
    pdir = work / "predictors"
    pdir.mkdir()
    for li in range(n_layers):
        p = ref_predictor.NeuronPredictor(SM.H, inter, rank=16)
        down, up, bias = SM.engine_stub_predictor_params(li, 13, inter, 16)
        with torch.no_grad():
            p.down.weight.copy_(down)
            p.up.weight.copy_(up)
            p.up.bias.copy_(bias)
        p.save(str(pdir / f"layer_{li:03d}_expert_000.pt"))

    fetched = []                           # (layer, ids) of every cold read, in order
    orig_read = splitter.ColdWeightStore.read_neurons

    def recording_read(self, layer_idx, expert_idx, neuron_ids):
        fetched.append((layer_idx, list(neuron_ids)))
        return orig_read(self, layer_idx, expert_idx, neuron_ids)
    splitter.ColdWeightStore.read_neurons = recording_read

    eng = ref_engine.DesdemonaEngine(str(work / "split"), str(pdir), device="cpu", n_threads=2, max_seq_len=64)
    g = torch.Generator().manual_seed(14)
    prompt = torch.randint(0, vocab, (1, 12), generator=g)
    out = {"prompt": prompt.numpy()}
    with torch.inference_mode():
        logits, kv = eng.forward(prompt)
        out["prefill_logits"] = logits[0].float().numpy()
        n_prefill = len(fetched)
        tokens = eng.generate(prompt, max_new_tokens=8, temperature=0.0)
        out["greedy_tokens"] = np.asarray(tokens, np.int64)
        # teacher-forced decode: the logits of each generated token's step, with the cache
        logits, kv = eng.forward(prompt)
        steps = [logits[0, -1].float().numpy()]
        fetch_steps = []
        for t in tokens[:-1]:
            k0 = len(fetched)
            logits, kv = eng.forward(torch.tensor([[t]]), kv)
            steps.append(logits[0, -1].float().numpy())
            fetch_steps.append(fetched[k0:])
    out["decode_logits"] = np.stack(steps)
    for li in range(n_layers):
        out[f"prefill_fetch_l{li}"] = np.asarray(fetched[li][1] if fetched[li][0] == li else [], np.int64)
    out["decode_fetch"] = np.asarray([[len(ids) for (_, ids) in st] for st in fetch_steps], np.int64)
    out["n_prefill_reads"] = np.asarray([n_prefill])
    split = work / "split"
    out["split_config"] = np.frombuffer((split / "split_config.json").read_bytes(), np.uint8)
    out["cold_index"] = np.load(split / "cold_index.npy")
    out["cold_sha256"] = np.frombuffer(hashlib.sha256((split / "cold_weights.bin").read_bytes()).digest(), np.uint8)
    hot0 = torch.load(split / "hot_weights" / "layer_000_expert_000.pt")
    out["hot0_ids"] = hot0["neuron_ids"].numpy()
    out["hot0_gate_bytes"] = hot0["gate"].view(torch.uint8).numpy()
    shared = torch.load(split / "hot_weights" / "shared.pt")
    out["shared_keys"] = np.asarray(sorted(shared.keys()))
    out["shared_q0_sha256"] = np.frombuffer(hashlib.sha256(
        shared["layer_000.q_proj"].view(torch.uint8).numpy().tobytes()).digest(), np.uint8)
    eng.close()
    splitter.ColdWeightStore.read_neurons = orig_read
    np.savez_compressed(HERE / "engine.npz", **out)
    shutil.rmtree(work)
    print("engine fixture written to", HERE / "engine.npz")


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HC_REFERENCE_DIR")
    if not ref:
        raise SystemExit("usage: make_golden.py <reference checkout dir> [engine]  (or set HC_REFERENCE_DIR)")
    if len(sys.argv) > 2 and sys.argv[2] == "engine":
        engine_main(ref)
    else:
        main(ref)
        engine_main(ref)
