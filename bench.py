"""Benchmark of the B200 hot/cold sparse-FFN decode path.

Default workload (the metric's 32-layer stack):
32-layer dReLU FFN stack, hidden 4096 / intermediate 14336, 20% hot FP8 /
80% cold INT4 records, rank-64 predictor per layer (N(0, 0.02) weights,
sigmoid >= 0.5 fetch set, engine lookahead), batch-1 decode.  One step = one
pass of 256 synthetic N(0,1) tokens, each decoded through all 32 layers.

Printed (rank 0, one JSON line): tokens/s with inputs resident in HBM
(`value`), the same through the public API with host buffers (`e2e`), the
roofline of the dominant kernel (hc_ffn_stack), the CPU reference leg, the
config-2 cold dequant microbench, and the SM clocks seen while timing.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "hot-cold-neural-split-openinfer2_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "sparse-FFN decode tokens/s (32L, 4096/14336) + cold dequant GB/s vs HBM peak"
H, INTER, LAYERS, RANK, TOKENS = 4096, 14336, 32, 64, 256
N_HOT = int(0.2 * INTER)
HOT_BYTES = 3 * H                       # fp8 gate row + up row + down column
COLD_BYTES = 3 * (H // 2) + 192         # INT4 payload + fp16 scales (6336 B)
PRED_BYTES = 4 * (RANK * H + INTER * RANK + INTER)
WORKLOAD = ("configs[2]: 32-layer dReLU sparse-FFN stack 4096/14336, hot 20% FP8 e4m3 (direct cast), cold 80% INT4 "
            "records (reference on-disk layout), rank-64 predictor N(0,0.02) w/ bias, sigmoid>=0.5 fetch set with "
            "engine lookahead; batch-1 decode of 256 N(0,1) tokens per step")


def _peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms while timing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(gpu_index)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            return None
        mhz, maxes, reasons = [], [], set()
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm, smax = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            mhz.append(sm)
            maxes.append(smax)
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"),
                               parts[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not mhz:
            return None
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": max(maxes), "samples": len(mhz),
                "reasons": sorted(reasons)}


def _physical_gpu(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            return int(vis.split(",")[local])
        except (ValueError, IndexError):
            return local
    return local


TRAFFIC_JSON = os.path.join(REPO, "profiles", "ffn_stack_traffic.json")


def _profile_traffic():
    """DRAM bytes per hc_ffn_stack launch, from the committed ncu summary
    (profiles/ffn_stack_traffic.json: dram__bytes_read.sum + write.sum of a
    capture, scaled to one 32-layer launch)."""
    try:
        with open(TRAFFIC_JSON) as f:
            return float(json.load(f)["traffic_bytes_per_launch"])
    except (OSError, KeyError, ValueError):
        return None


# ----------------------------------------------------------------------------
# CPU reference leg (the oracle's restatement of the reference's CPU path)
# ----------------------------------------------------------------------------
def cpu_reference(steps: int, warmup: int, layers_per_step: int = 2, budget_s: float = 20.0):
    import torch
    from oracle import hotcold_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    layers = [O.make_cpu_layer(1000 + i) for i in range(layers_per_step)]
    g = torch.Generator().manual_seed(2)
    times, fetched = [], []
    t_start = time.perf_counter()
    for s in range(warmup + steps):
        x = torch.randn(H, generator=g)
        t0 = time.perf_counter()
        for L in layers:
            x, n = O.ref_layer_cpu(L, x)
            fetched.append(n)
        dt = time.perf_counter() - t0
        if s >= warmup:
            times.append(dt)
        if time.perf_counter() - t_start > budget_s and len(times) >= 1:
            break
    per_layer = sum(times) / (len(times) * layers_per_step)
    tok_s = 1.0 / (per_layer * LAYERS)
    # read_neurons alone (splitter.py:354-403 through the port), 256 seeded ids per call
    store = layers[0]["store"]
    rng = __import__("numpy").random.default_rng(7)
    tab = store.record_index_table(0)
    present = __import__("numpy").nonzero(tab >= 0)[0]
    ids = rng.choice(present, size=min(256, len(present)), replace=False).tolist()
    n_read, t_read = 0, 0.0
    while t_read < 2.0:
        t0 = time.perf_counter()
        store.read_neurons(0, 0, ids)
        t_read += time.perf_counter() - t0
        n_read += len(ids)
    return {"value": tok_s, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "read_neurons_per_s": n_read / t_read,
            "sample": f"{len(times)} token(s) x {layers_per_step} of 32 layers (same geometry/seeds class, "
                      f"~{int(statistics.mean(fetched))} cold neurons fetched per layer), timed per layer and "
                      f"scaled to 32 layers",
            "s_per_layer": per_layer, "steps_timed": len(times), "layers_per_step": layers_per_step}


def run_reference(args):
    ws, rank, _ = _dist()
    if rank != 0:
        return
    ref = cpu_reference(args.steps, args.warmup, layers_per_step=2, budget_s=120.0)
    # a step is what was timed: one token through the sampled layers; the
    # tokens/s value scales that time to all 32 layers
    line = {"metric": METRIC, "impl": "reference", "value": ref["value"], "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": ref["steps_timed"], "warmup": args.warmup,
            "ms_per_step": 1000.0 * ref["s_per_layer"] * ref["layers_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic",
            "config": {"workload": WORKLOAD, "layers": LAYERS, "hidden": H, "inter": INTER, "batch": 1,
                       "timed_layers_per_step": ref["layers_per_step"],
                       "note": "one step = one token through 2 sampled layers on the host cores; value scales "
                               "the measured time per layer to 32 layers"},
            "cpu_baseline": {k: ref[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": ref["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------
def cold_dequant_bench(store, reps: int = 5, ks=(256, 1024, 4096, 8192)):
    """gather K seeded-random records per layer for all 32
    layers, dequantised to bf16 (6336 B read + 24576 B written per neuron).
    With a store in pinned host memory the records cross PCIe (`read_gbs`)."""
    import torch
    peak, _ = _peaks()
    out = {}
    g = torch.Generator(device=store.device).manual_seed(7)
    nrec = int(store.n_rec_host.min())
    for K in ks:
        rec = torch.randint(0, nrec, (store.n_layers, K), generator=g, device=store.device, dtype=torch.int32)
        buf = torch.empty(3, store.n_layers, K, H, dtype=torch.bfloat16, device=store.device)
        for _ in range(2):
            store.gather_layers(range(store.n_layers), rec, out=buf, out_dtype=torch.bfloat16)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            store.gather_layers(range(store.n_layers), rec, out=buf, out_dtype=torch.bfloat16)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        neurons = K * store.n_layers
        gbs = neurons * (COLD_BYTES + 3 * H * 2) / (ms * 1e-3) / 1e9
        out[str(K)] = {"ms": round(ms, 4), "neurons_per_s": neurons / (ms * 1e-3), "gbs": round(gbs, 1),
                       "frac": round(gbs / peak, 4),
                       "read_gbs": round(neurons * COLD_BYTES / (ms * 1e-3) / 1e9, 1)}
        del buf
    store.check()
    return out


def batched_decode_bench(syn, steps: int, warmup: int, batches=(1, 8, 32, 64), shard=None):
    """configs[4] on one GPU: the 32-layer stack for B tokens at once with
    per-token Bernoulli(0.1) masks unioned per layer (BatchStack: hc_union_cold_layers
    + hc_ffn_batch_layer per layer, tcgen05 tensor-core GEMMs), captured in one
    CUDA graph per batch size; B = 1 runs the fused batch-1 stack kernel.
    ``shard=(rank, size)`` (every rank calls this): each GPU streams its share
    of every layer and the partial outputs are summed by one exchange kernel
    per layer (hc_xchg_sum: NVLink stores, bounded waits), captured in the same
    CUDA graph; times are the max over ranks.  `value` is device-resident;
    `e2e` adds the pinned host->device copy of the B inputs and the
    device->host copy of the outputs to every step."""
    import torch
    import hc_synth
    peak, _ = _peaks()
    import torch.distributed as dist
    bst = syn.batch_stack(max_batch=max(batches), shard=shard)
    dev = syn.store.device
    stream = torch.cuda.Stream(device=dev)
    out = {}
    for B in batches:
        masks = hc_synth.bernoulli_words(LAYERS, B, INTER, 0.1, seed=2, device=dev)
        gen = torch.Generator(device="cpu").manual_seed(200 + B)
        x_host = torch.randn(B, H, generator=gen).pin_memory()
        y_host = torch.empty(B, H).pin_memory()
        x_in = x_host.to(dev)
        y = torch.empty(B, H, device=dev)
        bst.forward(x_in, masks=masks, out=y)                   # first call outside capture
        torch.cuda.synchronize()
        # B = 1 on one GPU runs the fused stack (one cooperative launch per token):
        # launched directly; everything else replays one captured graph per step
        # (the sharded exchange is a plain kernel with bounded waits, no library
        # collective)
        g = None
        sharded = shard is not None and shard[1] > 1
        if B > 1 or sharded:
            g = torch.cuda.CUDAGraph()
            stream.wait_stream(torch.cuda.current_stream())
            try:
                with torch.cuda.stream(stream):
                    with torch.cuda.graph(g, stream=stream):
                        bst.forward(x_in, masks=masks, out=y)
            except RuntimeError as e:       # a collective that cannot be captured: launch eagerly
                print(f"batched decode B={B}: graph capture failed ({str(e)[:120]}); eager launches", file=sys.stderr)
                g = None
            torch.cuda.current_stream().wait_stream(stream)
        step = g.replay if g is not None else (lambda: bst.forward(x_in, masks=masks, out=y))
        union = float(bst.count.float().mean().item())
        for _ in range(max(warmup, 3)):
            step()
        torch.cuda.synchronize()
        if sharded:
            dist.barrier()                      # the ranks start the timed steps together
            torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            step()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        e0.record()
        for _ in range(steps):
            x_in.copy_(x_host, non_blocking=True)
            step()
            y_host.copy_(y, non_blocking=True)
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = e0.elapsed_time(e1) / steps
        bst.check()
        if shard is not None and shard[1] > 1:
            t = torch.tensor([ms, e2e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms, e2e_ms = (float(v) for v in t.tolist())
        # algorithmic bytes of one step: every hot neuron and every record of
        # each layer's union once, plus the B hidden states in and out per layer
        step_bytes = LAYERS * (N_HOT * HOT_BYTES + union * COLD_BYTES + 2 * B * H * 4)
        gbs = step_bytes / (ms * 1e-3) / 1e9
        n_gpu = shard[1] if shard is not None else 1
        out[str(B)] = {"tokens_per_s": round(B / (ms * 1e-3), 1), "ms_per_step": round(ms, 4),
                       "e2e_tokens_per_s": round(B / (e2e_ms * 1e-3), 1),
                       "union_records_per_layer": round(union, 1),
                       "union_frac": round(union / (INTER - N_HOT), 4),
                       "algorithmic_gbs": round(gbs, 1), "frac": round(gbs / (peak * n_gpu), 4),
                       "graph": g is not None}
        del g
    bst.close()
    return out


def pinned_tier_bench(syn, pstore, tokens: int = 8):
    """configs[2] with cold_weights.bin in pinned host memory (the reference's
    tiering, splitter.py:307-330): per layer the predicted records cross PCIe
    into the store's staging buffer (hc_union_cold + hc_cold_stage), then the
    layer's stack launch, which also predicts the next layer's set.  Timed
    with CUDA events over ``tokens`` decode tokens after one warm-up token."""
    import torch
    import engine
    dev = pstore.device
    st = engine.FFNStack(pstore, syn.hot, syn.norms, syn.predictors, syn.activation, syn.act_on_both, syn.eps,
                         inter=syn.inter)
    g = torch.Generator(device=dev).manual_seed(5)
    xs = torch.randn(tokens + 1, H, device=dev, generator=g)
    ys = torch.empty_like(xs)
    st.forward(xs[tokens], out=ys[tokens])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for t in range(tokens):
        st.forward(xs[t], out=ys[t])
    e1.record()
    torch.cuda.synchronize()
    st.check()
    ms = e0.elapsed_time(e1)
    staged = 0
    for t in range(tokens):                      # the records each token fetched (untimed replay)
        st.forward(xs[t], out=ys[t])
        staged += int(st.active_counts().sum())
    rec_read = 6352                              # bytes of a record the kernels read
    return {"workload": "configs[2] (32L dReLU 4096/14336, rank-64 predictors), cold store in pinned host memory",
            "tokens": tokens, "tokens_per_s": round(tokens / (ms / 1e3), 2), "ms_per_token": round(ms / tokens, 3),
            "staged_records_per_token": round(staged / tokens, 1),
            "bus_gbs": round(staged * rec_read / (ms * 1e-3) / 1e9, 2),
            "hbm_staging_bytes": int(pstore.stage_bytes()),
            "launches_per_token": 2 + 3 * LAYERS}     # layer 0 predictor (2), per layer union + stage + stack


def config0_quality(dev):
    """one 4096/14336 SwiGLU layer, hot 20% FP8 with per-row absmax
    scales, cold 80% INT4, one N(0, 1) token, Bernoulli(0.1) active cold mask,
    run through the fused stack kernel; the hot+cold output against the dense
    fp32 FFN over the same neurons (hot + active cold), computed in float64 on
    the host as the checker.  The reference reports 9.5-17.5% for its
    mixed-precision split against fp32 (its BENCHMARKS.md:41)."""
    import numpy as np
    import torch
    import hc_synth
    syn = hc_synth.make_stack(n_layers=1, inter=INTER, hot_frac=0.2, activation="silu", act_on_both=False, seed=0,
                              row_scale=True, predictors=False, keep_dense=True, device=dev)
    masks = hc_synth.bernoulli_words(1, 1, INTER, 0.1, seed=2, device=dev)[:, 0].contiguous()
    x0 = torch.randn(H, device=dev, generator=torch.Generator(device=dev).manual_seed(1))
    st = syn.stack(with_predictors=False)
    y = st.forward(x0, masks=masks).double().cpu().numpy()
    st.check()
    gate, up, down, hot_ids = (t.numpy().astype(np.float64) for t in syn.extra["dense"][0])
    from splitter import words_to_bits
    active = words_to_bits(masks[0], INTER) & words_to_bits(st.fetch[0], INTER)
    ids = np.concatenate([hot_ids.astype(np.int64), np.nonzero(active)[0]])
    x = x0.double().cpu().numpy()
    xn = x / np.sqrt(np.mean(x * x) + syn.eps)
    g, u = gate[ids] @ xn, up[ids] @ xn
    dense = (g / (1.0 + np.exp(-g)) * u) @ down[:, ids].T
    rel = float(np.linalg.norm((y - x) - dense) / np.linalg.norm(dense))
    return {"workload": "configs[0]: 1 SwiGLU layer 4096/14336, hot 20% FP8 e4m3 with per-row absmax scale, cold 80% "
                        "INT4 records, 1 N(0,1) token, Bernoulli(0.1) active cold mask",
            "neurons": int(len(ids)), "cold_active": int(active.sum()),
            "rel_l2_vs_dense_fp32": round(rel, 4),
            "reference_figure": "9.5-17.5% (mixed FP8/INT4 split vs fp32, reference BENCHMARKS.md:41)"}


def full_decode_bench(dev, prompt_len: int = 512, new_tokens: int = 256, layers: int = LAYERS):
    """Llama-3.1-8B geometry (32 layers, hidden 4096, 32 query / 8
    key-value heads, vocab 128256, SwiGLU 14336 split 20% FP8 hot / 80% INT4
    cold, rank-64 predictor per layer), random-init weights, through
    DesdemonaEngine.generate: a 512-token prompt of uniform random ids, 256
    greedy tokens.  Attention is fp16 torch code (prefill) and the FP8 GEMV
    (decode steps); each decode step is one CUDA graph replay."""
    import torch
    import engine
    import hc_synth
    from predictor import PredictorRegistry
    vocab, nq, nkv = 128256, 32, 8
    syn = hc_synth.make_stack(n_layers=layers, inter=INTER, hot_frac=0.2, rank=RANK, activation="silu",
                              act_on_both=False, seed=3, device=dev)
    g = torch.Generator(device=dev).manual_seed(33)
    shared = {}
    for li in range(layers):
        for name, rows in (("q_proj", H), ("k_proj", nkv * 128), ("v_proj", nkv * 128), ("o_proj", H)):
            shared[f"layer_{li:03d}.{name}"] = (torch.randn(rows, H, generator=g, device=dev) * 0.02).to(
                torch.float8_e4m3fn)
        shared[f"layer_{li:03d}.input_layernorm"] = torch.ones(H, dtype=torch.float16, device=dev)
        shared[f"layer_{li:03d}.post_attention_layernorm"] = syn.norms[li].half()
    shared["embed_tokens"] = torch.randn(vocab, H, generator=g, device=dev).half()
    shared["lm_head"] = (torch.randn(vocab, H, generator=g, device=dev) * 0.02).half()
    shared["final_norm"] = torch.ones(H, dtype=torch.float16, device=dev)
    cfg = {"hidden_dim": H, "intermediate_dim": INTER, "num_layers": layers, "vocab_size": vocab,
           "num_attention_heads": nq, "num_key_value_heads": nkv, "rope_theta": 500000.0, "rms_norm_eps": 1e-5,
           "hidden_act": "silu", "act_on_both": False, "max_position_embeddings": 8192, "num_experts": 1}
    reg = PredictorRegistry.__new__(PredictorRegistry)
    reg.device = str(dev)
    reg.predictors = {(li, 0): p for li, p in enumerate(syn.predictors)}
    eng = engine.DesdemonaEngine.from_parts(cfg, shared, syn.store, syn.hot, reg, device=dev,
                                            max_seq_len=prompt_len + new_tokens)
    del shared
    prompt = torch.randint(0, vocab, (1, prompt_len), generator=torch.Generator().manual_seed(34))
    eng.generate(prompt.to(dev), max_new_tokens=8, temperature=0.0)        # warm-up: graph capture, workspaces
    torch.cuda.synchronize()
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    e0.record()
    logits, cache = eng.forward(prompt.to(dev), eng.new_cache(1, prompt_len + new_tokens))
    e1.record()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e0b = torch.cuda.Event(enable_timing=True)
    e0b.record()
    out = eng.generate(prompt, max_new_tokens=new_tokens, temperature=0.0)   # host prompt ids, host token list
    e2.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    eng.check()
    prefill_ms = e0.elapsed_time(e1)
    total_ms = e0b.elapsed_time(e2)
    decode_ms = total_ms - prefill_ms
    return {"workload": "configs[3]: Llama-3.1-8B geometry (32L, 32q/8kv heads, vocab 128256), SwiGLU 4096/14336 "
                        "20% FP8 hot / 80% INT4 cold with rank-64 predictors (random init), 512-token random prompt, "
                        "256 greedy tokens through DesdemonaEngine.generate",
            "tokens": len(out), "generate_tokens_per_s": round(len(out) / (total_ms / 1e3), 1),
            "decode_tokens_per_s": round((len(out) - 1) / (decode_ms / 1e3), 1),
            "prefill_ms": round(prefill_ms, 2), "generate_ms": round(total_ms, 2), "generate_wall_s": round(wall, 3),
            "note": "generate() timed end to end on the device (prefill + 255 graph-replayed decode steps + "
                    "sampling + one device-to-host read of the tokens); decode = generate - prefill"}


def run_gpu(args):
    import torch
    import torch.distributed as dist

    import engine
    import hc_native as N
    import hc_synth

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", init_method="env://", timeout=__import__("datetime").timedelta(seconds=120),
                                device_id=dev)
    syn = hc_synth.make_stack(n_layers=LAYERS, inter=INTER, hot_frac=0.2, rank=RANK, activation="relu",
                              act_on_both=True, seed=0, device=dev)
    # N > 1: every layer's neurons are split over the GPUs (tensor parallelism,
    # one in-kernel exchange of the partial output per layer); all ranks decode
    # the same tokens, so the job's throughput is one rank's tokens/s
    tp = engine.TPGroup(device=dev) if ws > 1 else None
    st = syn.stack(tp=tp)
    gen = torch.Generator(device="cpu").manual_seed(100)
    x_host = torch.randn(TOKENS, H, generator=gen).pin_memory()
    x_dev = x_host.to(dev)
    y_host = torch.empty(TOKENS, H).pin_memory()
    y_dev = torch.empty(TOKENS, H, device=dev)
    pred0 = st.pred0_in_kernel()      # layer 0's predictor inside the stack kernel
    launches_per_token = 1 if pred0 else 3          # fused stack (+ 2 predictor launches otherwise)

    def step_resident():
        for t in range(TOKENS):
            st.forward(x_dev[t], out=y_dev[t])

    # fetched cold neurons per token (deterministic: same tokens, same masks)
    if ws > 1:
        dist.barrier()
        torch.cuda.synchronize()
    own = slice(st.words_lo, st.words_lo + st.words_n)
    fetched = []
    for t in range(TOKENS):
        st.forward(x_dev[t], out=y_dev[t])
        m = (st.masks[:, own] & st.fetch[:, own]).cpu().numpy().astype("uint32")
        fetched.append(int(sum(bin(int(w)).count("1") for w in m.reshape(-1))))
    st.check()
    mean_fetched = sum(fetched) / len(fetched)          # this GPU's share, summed over the 32 layers
    # algorithmic bytes of one hc_ffn_stack launch on this GPU (one token, 32
    # layers): its hot neurons, its fetched cold records, every predictor's
    # W_down and its share of W_up / bias, x and y
    n_hot_local = sum(h.n for h in st.hot) / LAYERS
    share = st.words_n / st.words
    pred_local = 4 * (RANK * H) + share * 4 * (INTER * RANK + INTER)
    stack_bytes = (LAYERS * n_hot_local * HOT_BYTES + mean_fetched * COLD_BYTES
                   + (LAYERS if pred0 else LAYERS - 1) * pred_local + 2 * LAYERS * H * 4)
    token_bytes = stack_bytes + (0 if pred0 else PRED_BYTES)     # + layer-0 predictor launches

    for _ in range(max(args.warmup, 3)):
        step_resident()
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()

    stream = torch.cuda.current_stream()
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(TOKENS)]
          for _ in range(args.steps)]
    sampler = ClockSampler(_physical_gpu(local)) if rank == 0 else None
    t_begin, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t_begin.record(stream)
    for s in range(args.steps):
        evs = ev[s]
        for t in range(TOKENS):
            if not pred0:
                st.first_mask(x_dev[t])
            evs[t][0].record(stream)
            st.launch(x_dev[t], 2 if pred0 else False, None, y_dev[t])
            evs[t][1].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize()
    stack_ms = sum(a.elapsed_time(b) for evs in ev for a, b in evs)
    elapsed_ms = t_begin.elapsed_time(t_end)
    clocks = sampler.stop() if sampler else None
    st.check()
    if ws > 1:
        t = torch.tensor([elapsed_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    tokens_all = TOKENS * args.steps            # the ranks decode the same tokens together
    value = tokens_all / (elapsed_ms / 1e3)
    ms_per_step = elapsed_ms / args.steps

    # e2e: the public API with host buffers (pinned H2D of the step's tokens,
    # D2H of the step's outputs) inside the timed region
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for s in range(args.steps):
        st.decode_host(x_host, y_host)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if ws > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = tokens_all / (e2e_ms / 1e3)

    peak, peak_kind = _peaks()
    avg_stack_ms = stack_ms / (args.steps * TOKENS)
    achieved = stack_bytes / (avg_stack_ms * 1e-3) / 1e9
    traffic = _profile_traffic()
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                "kernel": "hc_ffn_stack (ffn_stack_kernel)", "algorithmic_bytes_per_launch": int(stack_bytes),
                "avg_launch_ms": round(avg_stack_ms, 5),
                "token_frac": round(token_bytes * value / 1e9 / peak, 4)}
    if ws > 1:
        roofline["traffic"] = None          # the committed capture is of the one-GPU launch
    line = None
    bd_tp = None
    if ws > 1:
        dist.barrier()
        torch.cuda.synchronize()
        tp.close()
        # configs[4] across the GPUs: B = 64, every layer's neurons sharded, one NCCL all-reduce per layer
        # (every rank takes the same path; a failure is reported in the line instead of losing it)
        try:
            bd_tp = batched_decode_bench(syn, args.steps, args.warmup, batches=(64,), shard=(rank, ws))
        except Exception as e:          # noqa: BLE001 -- reported, not hidden
            bd_tp = {"error": f"{type(e).__name__}: {str(e)[:160]}"}
    if rank == 0:
        dq = cold_dequant_bench(syn.store) if ws == 1 else None
        dq_pinned = None
        pt = None
        if ws == 1:
            # the same gather with the cold file image in pinned host memory (PCIe-bound)
            from splitter import ColdWeightStore
            pstore = ColdWeightStore(syn.store.image, syn.cold_index, {"hidden_dim": H, "intermediate_dim": INTER},
                                     device=dev, source="pinned")
            dq_pinned = cold_dequant_bench(pstore, reps=3, ks=(256, 1024, 4096))
            for v in dq_pinned.values():
                v.pop("frac", None)            # bound by PCIe, not HBM
            try:
                pt = pinned_tier_bench(syn, pstore)
            except Exception as e:          # noqa: BLE001 -- reported in the line, not hidden
                pt = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
            del pstore
        bd = batched_decode_bench(syn, args.steps, args.warmup) if ws == 1 else None
        cpu = cpu_reference(4, 0, layers_per_step=2, budget_s=25.0) if ws == 1 else None
        q0 = config0_quality(dev) if ws == 1 else None
        fd = None
        if ws == 1:
            try:
                fd = full_decode_bench(dev)
            except Exception as e:          # noqa: BLE001 -- reported in the line, not hidden
                fd = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
        line = {"metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "e4m3/int4 weights, fp32 accumulate",
                "data": "synthetic",
                "config": {"workload": WORKLOAD, "layers": LAYERS, "hidden": H, "inter": INTER, "hot": N_HOT,
                           "rank": RANK, "batch": 1, "tokens_per_step": TOKENS,
                           "cold_fetched_per_token": round(mean_fetched, 1),
                           "cold_fetched_frac": round(mean_fetched / (LAYERS * (INTER - N_HOT)), 4),
                           "l2": "no flush: each token streams ~2.4 GB of weights, far above the 126 MB L2",
                           "parallelism": (f"tp{ws}: neurons of every layer split over {ws} GPUs, one in-kernel "
                                           "NVLink exchange of the 16 KB partial output per layer") if ws > 1
                           else "single GPU"},
                "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s",
                        "h2d_bytes_per_step": TOKENS * H * 4, "d2h_bytes_per_step": TOKENS * H * 4},
                "gpu_launches": args.steps * TOKENS * launches_per_token,
                "roofline": roofline,
                "clocks": clocks}
        if cpu is not None:
            line["cpu_baseline"] = {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
        if q0 is not None:
            line["config0_quality"] = q0
        if fd is not None:
            line["full_decode"] = fd
        if bd is not None:
            line["batched_decode"] = {"workload": "configs[4] on 1 GPU: 32L 4096/14336 stack, B tokens, per-token "
                                                  "Bernoulli(0.1) masks unioned per layer, tcgen05 GEMMs",
                                      "unit": "tokens/s", "peak": peak, "by_B": bd}
        if bd_tp is not None:
            line["batched_decode"] = {"workload": f"configs[4] on {ws} GPUs: 32L 4096/14336 stack, B tokens, "
                                                  "per-token Bernoulli(0.1) masks unioned per layer; every layer's "
                                                  f"hot neurons and cold records split over {ws} GPUs, one "
                                                  "exchange kernel (NVLink stores into the peers' buffers) per "
                                                  "layer summing the [B, 4096] partial outputs, CUDA graph",
                                      "unit": "tokens/s (whole job)", "peak": peak, "by_B": bd_tp}
        if dq is not None:
            line["cold_dequant"] = {"unit": "GB/s", "peak": peak, "bytes_per_neuron": COLD_BYTES + 3 * H * 2,
                                    "layers": LAYERS, "out_dtype": "bf16", "by_K": dq}
            if cpu is not None:
                # the same read (record lookup + 3 x dequantize_int4 per neuron) on the host cores, same run
                rate = cpu["read_neurons_per_s"]
                line["cold_dequant"]["cpu_read_neurons_per_s"] = round(rate, 1)
                line["cold_dequant"]["cpu_sample"] = "read_neurons of 256 seeded ids per call, repeated for 2 s"
                for v in dq.values():
                    v["vs_cpu"] = round(v["neurons_per_s"] / rate, 1)
        if pt is not None:
            line["pinned_tier"] = pt
        if dq_pinned is not None:
            line["cold_dequant_pinned"] = {"unit": "GB/s", "source": "pinned host memory read over PCIe by the "
                                           "gather kernel; read_gbs = 6336 B per neuron / time",
                                           "layers": LAYERS, "out_dtype": "bf16", "by_K": dq_pinned}
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    return line


# ----------------------------------------------------------------------------
# Profiling targets (small cases for ncu captures, launch lists and traces)
# ----------------------------------------------------------------------------
def run_profile(args):
    """One kernel of the path on a seeded synthetic model, through the public
    API, for ncu captures and device traces (nothing is skipped inside a
    launch).  Targets: stack (hc_ffn_stack; --masks-p P gives Bernoulli(P)
    fetch sets instead of the predictors), gather (hc_cold_gather_dequant),
    predictor (hc_predictor_forward), batch (hc_ffn_batch_layer, B tokens).
    --trace prints the stack kernel's per-phase table (device timestamps)."""
    import torch
    import hc_synth
    ws, rank, local = _dist()
    tp = None
    if ws > 1:
        import torch.distributed as dist
        import engine
        torch.cuda.set_device(local)
        dist.init_process_group("gloo")
        tp = engine.TPGroup()
    what = args.profile_target
    if what == "engine":
        # configs[3] alone: DesdemonaEngine.generate (the bench line's full_decode field)
        print(json.dumps(full_decode_bench(torch.device("cuda"))))
        print("profile target done")
        return
    syn = hc_synth.make_stack(n_layers=args.layers, inter=args.inter, activation="relu", act_on_both=True, seed=0,
                              predictors=what not in ("gather", "batch") and args.masks_p <= 0)
    if what == "stack":
        st = syn.stack(tp=tp)
        if tp is not None:
            dist.barrier()
            torch.cuda.synchronize()
        x = torch.randn(args.tokens, H, generator=torch.Generator().manual_seed(1)).cuda()   # same on every rank
        masks = None
        if args.masks_p > 0:
            masks = hc_synth.bernoulli_words(args.layers, 1, args.inter, args.masks_p, seed=2)[:, 0].contiguous()
        trace = torch.zeros(args.layers, st.grid, 40, dtype=torch.int64, device="cuda") if args.trace else None
        for t in range(args.tokens):
            if trace is not None:
                trace.zero_()          # keep the last token's stamps and waits
            if masks is not None:
                st.masks.copy_(masks)
                st.launch(x[t], True, None, None, trace)
            elif st.pred0_in_kernel():
                st.launch(x[t], 2, None, None, trace)      # layer 0's predictor inside the kernel
            else:
                st.first_mask(x[t])
                st.launch(x[t], False, None, None, trace)
        torch.cuda.synchronize()
        st.check()
        if trace is not None and rank == 0:
            fetched = int(st.active_counts().sum())
            print(f"stack trace: {args.layers} layers, {fetched / args.layers:.0f} cold records per layer")
            for k, (mean, mx) in st.trace_summary(trace).items():
                print(f"  {k:28s} mean {mean:9.2f}   max {mx:9.2f}")
        if trace is not None and tp is not None:
            # across GPUs: per layer, local sum seen (max over CTAs, event 32), slice pushed
            # (max over the pushing CTAs, event 36) and peers' words seen (max over CTAs, 35)
            tr = trace.cpu()
            allt = [None] * ws
            dist.all_gather_object(allt, tr)
            if rank == 0:
                seen = torch.stack([a[:, :, 32].max(dim=1).values for a in allt]).double() / 1e3
                push = torch.stack([a[:, :32, 36].max(dim=1).values for a in allt]).double() / 1e3
                got = torch.stack([a[:-1, :, 35].max(dim=1).values for a in allt]).double() / 1e3
                skew = (seen.max(dim=0).values - seen.min(dim=0).values)[:-1]
                print(f"  cross-GPU: local-sum skew between GPUs (us) mean {float(skew.mean()):.2f} "
                      f"max {float(skew.max()):.2f}")
                if ws == 2:
                    # transit each way includes the clock offset with opposite signs: the mean cancels it
                    t01 = got[1] - push[0][:-1]
                    t10 = got[0] - push[1][:-1]
                    print(f"  cross-GPU: last push -> peer's last CTA saw it (us), offset-free mean "
                          f"{float(((t01 + t10) / 2).mean()):.2f}; each way {float(t01.mean()):.2f} / "
                          f"{float(t10.mean()):.2f}")
                late = (seen.max(dim=0).values - seen)[:, :-1]
                print(f"  cross-GPU: per GPU mean lateness behind the last GPU (us) "
                      f"{[round(float(v), 2) for v in late.mean(dim=1)]}")
        if tp is not None:
            dist.barrier()
            tp.close()
            dist.destroy_process_group()
    elif what == "batch":
        # per-token Bernoulli(0.1) masks unioned per layer; --tokens batched steps
        bst = syn.batch_stack(max_batch=max(args.batch, 1), dense_min_batch=args.dense_min_batch)
        masks = hc_synth.bernoulli_words(args.layers, args.batch, args.inter, 0.1, seed=2)
        x = torch.randn(args.batch, H, generator=torch.Generator().manual_seed(1)).cuda()
        for _ in range(args.tokens):
            bst.forward(x, masks=masks)
        torch.cuda.synchronize()
        bst.check()
    elif what == "gather":
        store = syn.store
        g = torch.Generator(device="cuda").manual_seed(7)
        rec = torch.randint(0, int(store.n_rec_host.min()), (store.n_layers, args.k), generator=g, device="cuda",
                            dtype=torch.int32)
        out = torch.empty(3, store.n_layers, args.k, H, dtype=torch.bfloat16, device="cuda")
        for _ in range(args.tokens):
            store.gather_layers(range(store.n_layers), rec, out=out, out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
        store.check()
    else:
        p = syn.predictors[0]
        x = torch.randn(args.tokens, H, device="cuda")
        for t in range(args.tokens):
            p.predict_words(x[t:t + 1], norm_w=syn.norms[0], eps=syn.eps)
        torch.cuda.synchronize()
    print("profile target done")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    # profiling targets (not a bench line): one kernel on a small synthetic case
    ap.add_argument("--profile-target", choices=["stack", "gather", "predictor", "batch", "engine"], default=None)
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--inter", type=int, default=INTER)
    ap.add_argument("--tokens", type=int, default=3)
    ap.add_argument("--k", type=int, default=4096, help="records per layer (--profile-target gather)")
    ap.add_argument("--batch", type=int, default=64, help="tokens per batched step (--profile-target batch)")
    ap.add_argument("--dense-min-batch", type=int, default=8)
    ap.add_argument("--masks-p", type=float, default=0.0, help="stack: Bernoulli(P) fetch sets instead of predictors")
    ap.add_argument("--trace", action="store_true", help="stack: print the per-phase table of the device trace")
    args = ap.parse_args()
    if args.profile_target:
        run_profile(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
