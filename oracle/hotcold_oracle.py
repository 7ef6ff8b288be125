"""CPU oracle for the per-token hot/cold sparse-FFN path.

TEST INFRASTRUCTURE ONLY.  This module is a numpy restatement of the
reference's algorithm (Hot-Cold-Neural-Split-OpenInfer2: ``splitter.py``,
``predictor.py``, ``engine.py``).  It is imported by ``tests/``, by
``__graft_entry__.smoke()`` and by the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` -- always as the checker or the timed CPU baseline, never
as part of the product path.  The product (the CUDA library and its Python
host side) never imports it.

Parity is pinned: ``tests/golden/`` holds vectors produced by running the
reference's own code (``tests/golden/make_golden.py``), and
``tests/test_oracle_golden.py`` checks every function below against them.

Every function cites the reference ``file:line`` it restates.
"""

from __future__ import annotations

import struct
from typing import Optional, Sequence

import numpy as np

# ---------------------------------------------------------------------------
# Format constants (splitter.py:57-76)
# ---------------------------------------------------------------------------
HIDDEN_DIM = 4096
ALIGN_BYTES = 64
PAGE_ALIGN = 4096
VEC_BYTES = HIDDEN_DIM // 2                       # 2048
GROUP_SIZE = 128
N_GROUPS = HIDDEN_DIM // GROUP_SIZE               # 32
SCALE_BYTES_PER_VEC = N_GROUPS * 2                # 64
SCALE_BYTES_TOTAL = SCALE_BYTES_PER_VEC * 3       # 192
RAW_RECORD = 2 + VEC_BYTES * 3 + SCALE_BYTES_TOTAL          # 6338
NEURON_RECORD_BYTES = ((RAW_RECORD + ALIGN_BYTES - 1) // ALIGN_BYTES) * ALIGN_BYTES  # 6400
SECTION_HEADER_BYTES = 16                         # struct '<HHIq' (splitter.py:230, :342)


# ---------------------------------------------------------------------------
# INT4 quantisation (splitter.py:81-124)
# ---------------------------------------------------------------------------
def quantize_int4_rows(x: np.ndarray, group_size: int = GROUP_SIZE):
    """Vectorised ``quantize_int4`` over the rows of ``x`` (splitter.py:81-108).

    x: float32 [R, N].  Returns (packed uint8 [R, ceil(N/2)], scales float32
    [R, ceil(N/group)]).  Per row this is byte-identical to the reference:
    scale = max(absmax, 1e-8) / 7 in fp32 (true division), q =
    round_half_even(x / scale) clamped to [-8, 7], element 2i in the low
    nibble and 2i+1 in the high nibble.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None, :]
    R, N = x.shape
    assert N % group_size == 0 or N < group_size, (N, group_size)
    if N % group_size != 0:                                   # splitter.py:93-95
        pad = group_size - (N % group_size)
        x = np.concatenate([x, np.zeros((R, pad), np.float32)], axis=1)
    groups = x.reshape(R, -1, group_size)                      # splitter.py:97
    absmax = np.abs(groups).max(axis=2)
    scales = np.maximum(absmax, np.float32(1e-8)) / np.float32(7.0)   # splitter.py:98
    scales = scales.astype(np.float32)
    q = np.round(groups / scales[:, :, None])                  # splitter.py:99
    q = np.clip(q, -8, 7).astype(np.int8).reshape(R, -1)[:, :N]
    if N % 2 != 0:                                             # splitter.py:102-103
        q = np.concatenate([q, np.zeros((R, 1), np.int8)], axis=1)
    lo = q[:, 0::2].view(np.uint8) & 0x0F                      # splitter.py:104
    hi = (q[:, 1::2].view(np.uint8) & 0x0F) << 4               # splitter.py:105
    packed = (lo | hi).astype(np.uint8)
    return packed, scales


def quantize_int4(vec: np.ndarray, group_size: int = GROUP_SIZE):
    """Single-vector form of :func:`quantize_int4_rows` (splitter.py:81)."""
    packed, scales = quantize_int4_rows(np.asarray(vec, np.float32)[None, :], group_size)
    return packed[0].tobytes(), scales[0]


def dequantize_int4(packed: bytes, scales: np.ndarray, N: int,
                    group_size: int = GROUP_SIZE) -> np.ndarray:
    """Inverse of quantize_int4 for one vector (splitter.py:111-124).

    Low nibble first, nibbles 8..15 map to -8..-1, multiplied in fp32 by the
    group scale repeated over its group.  q*s is exact in fp32.
    """
    arr = np.frombuffer(packed, dtype=np.uint8)
    lo = (arr & 0x0F).astype(np.int8)
    hi = ((arr >> 4) & 0x0F).astype(np.int8)
    flat = np.stack([lo, hi], axis=1).reshape(-1)[:N].astype(np.float32)
    flat = np.where(flat > 7, flat - 16, flat).astype(np.float32)
    n_groups = (N + group_size - 1) // group_size
    s = np.repeat(np.asarray(scales, np.float32)[:n_groups], group_size)[:N]
    return (flat * s).astype(np.float32)


def dequantize_int4_rows(packed: np.ndarray, scales: np.ndarray, N: int,
                         group_size: int = GROUP_SIZE) -> np.ndarray:
    """Row-vectorised :func:`dequantize_int4` (same arithmetic, splitter.py:111-124)."""
    packed = np.asarray(packed, np.uint8)
    R = packed.shape[0]
    lo = (packed & 0x0F).astype(np.int16)
    hi = ((packed >> 4) & 0x0F).astype(np.int16)
    flat = np.stack([lo, hi], axis=2).reshape(R, -1)[:, :N]
    flat = np.where(flat > 7, flat - 16, flat).astype(np.float32)
    n_groups = (N + group_size - 1) // group_size
    s = np.repeat(np.asarray(scales, np.float32)[:, :n_groups], group_size, axis=1)[:, :N]
    return (flat * s).astype(np.float32)


def int4_roundtrip_rows(w: np.ndarray) -> np.ndarray:
    """INT4 weights with FP16-rounded scales, as stored on disk
    (tests/common.py:68-81 of the reference applies the same rounding)."""
    packed, scales = quantize_int4_rows(w)
    s16 = scales.astype(np.float16).astype(np.float32)
    return dequantize_int4_rows(packed, s16, w.shape[1])


# ---------------------------------------------------------------------------
# Cold file format (splitter.py:186-262; reader splitter.py:307-407)
# ---------------------------------------------------------------------------
def build_records(nids: np.ndarray, gate: np.ndarray, up: np.ndarray,
                  down_cols: np.ndarray) -> np.ndarray:
    """Pack neuron records exactly as split_dense's inner loop (splitter.py:234-248).

    nids: [n] ids; gate/up: [n, H] fp32 rows; down_cols: [n, H] fp32 (the
    down_proj column of each neuron, i.e. down[:, nid]).  Returns uint8
    [n, NEURON_RECORD_BYTES].
    """
    n = len(nids)
    H = gate.shape[1]
    assert H == HIDDEN_DIM
    rec = np.zeros((n, NEURON_RECORD_BYTES), np.uint8)
    rec[:, 0:2] = np.asarray(nids, np.uint16).reshape(n, 1).view(np.uint8).reshape(n, 2)
    off = 2
    scales16 = []
    for mat in (gate, up, down_cols):
        p, s = quantize_int4_rows(np.asarray(mat, np.float32))
        rec[:, off:off + VEC_BYTES] = p
        off += VEC_BYTES
        scales16.append(s.astype(np.float16))
    for s16 in scales16:
        rec[:, off:off + SCALE_BYTES_PER_VEC] = s16.view(np.uint8).reshape(n, SCALE_BYTES_PER_VEC)
        off += SCALE_BYTES_PER_VEC
    return rec


def build_cold_file(layers: Sequence[tuple]) -> tuple[bytes, np.ndarray]:
    """Assemble cold_weights.bin + cold_index (splitter.py:188-262).

    layers: per layer (nids, gate_rows, up_rows, down_cols), or a precomputed
    records array ``(n, records_uint8)``.  Returns (file_bytes, cold_index
    uint64 [L, 1, 2]).
    """
    L = len(layers)
    cold_index = np.zeros((L, 1, 2), np.uint64)
    chunks = []
    cursor = 0
    for li, item in enumerate(layers):
        if len(item) == 2:
            n_cold, recs = item
        else:
            nids, g, u, d = item
            recs = build_records(np.asarray(nids), g, u, d)
            n_cold = len(nids)
        section_start = cursor
        header = struct.pack("<HHIq", li, 0, n_cold, 0)        # splitter.py:230
        chunks.append(header)
        cursor += len(header)
        body = np.ascontiguousarray(recs).tobytes()
        chunks.append(body)
        cursor += len(body)
        rem = cursor % PAGE_ALIGN                                # splitter.py:250-254
        if rem:
            pad = PAGE_ALIGN - rem
            chunks.append(b"\x00" * pad)
            cursor += pad
        cold_index[li, 0] = (section_start, n_cold)              # splitter.py:256
    return b"".join(chunks), cold_index


class ColdStoreOracle:
    """Restatement of ``ColdWeightStore`` (splitter.py:307-407).

    ``buf`` holds the whole cold_weights.bin.  Lookups follow the reference:
    the section is scanned once into an id -> offset dict (later duplicates
    overwrite earlier ones, splitter.py:345-349), absent ids are skipped
    (:371-372) and None is returned for an empty section or no match
    (:366-367, :397-398).
    """

    def __init__(self, buf, cold_index: np.ndarray, config: dict):
        self.buf = memoryview(bytes(buf)) if not isinstance(buf, memoryview) else buf
        self.index = np.asarray(cold_index)
        self.H = config["hidden_dim"]
        self._cache: dict = {}

    def section_offsets(self, layer_idx: int, expert_idx: int = 0):
        key = (layer_idx, expert_idx)
        if key in self._cache:
            return self._cache[key]
        off, n_cold = (int(v) for v in self.index[layer_idx, expert_idx])
        if n_cold == 0:
            return None
        cur = off + SECTION_HEADER_BYTES
        table = {}
        for _ in range(n_cold):
            nid = struct.unpack_from("<H", self.buf, cur)[0]
            table[nid] = cur
            cur += NEURON_RECORD_BYTES
        self._cache[key] = table
        return table

    def read_neurons(self, layer_idx: int, expert_idx: int, neuron_ids):
        table = self.section_offsets(layer_idx, expert_idx)
        if table is None:
            return None
        g_rows, u_rows, d_rows = [], [], []
        for nid in neuron_ids:
            if nid not in table:
                continue
            off = table[nid] + 2
            sc = off + 3 * VEC_BYTES
            s = np.frombuffer(self.buf[sc:sc + SCALE_BYTES_TOTAL], np.float16).astype(np.float32)
            g_rows.append(dequantize_int4(self.buf[off:off + VEC_BYTES], s[0:32], self.H))
            u_rows.append(dequantize_int4(self.buf[off + VEC_BYTES:off + 2 * VEC_BYTES], s[32:64], self.H))
            d_rows.append(dequantize_int4(self.buf[off + 2 * VEC_BYTES:off + 3 * VEC_BYTES], s[64:96], self.H))
        if not g_rows:
            return None
        return np.stack(g_rows), np.stack(u_rows), np.stack(d_rows, axis=1)

    def record_index_table(self, layer_idx: int, table_size: int = 65536) -> np.ndarray:
        """nid -> record index (-1 when absent), last duplicate wins (splitter.py:345-349)."""
        off, n_cold = (int(v) for v in self.index[layer_idx, 0])
        t = np.full(table_size, -1, np.int32)
        if n_cold == 0:
            return t
        base = off + SECTION_HEADER_BYTES
        raw = np.frombuffer(self.buf, np.uint8, count=n_cold * NEURON_RECORD_BYTES, offset=base)
        nids = raw.reshape(n_cold, NEURON_RECORD_BYTES)[:, 0:2].copy().view(np.uint16).reshape(-1)
        t[nids] = np.arange(n_cold, dtype=np.int32)      # numpy fancy assign: last wins
        return t


# ---------------------------------------------------------------------------
# FP8 e4m3 (the reference casts with torch: splitter.py:223-225)
# ---------------------------------------------------------------------------
def e4m3_decode_table() -> np.ndarray:
    """float32 value of every e4m3fn byte (bias 7, no infinities, 0x7F/0xFF NaN)."""
    t = np.zeros(256, np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 0x7
        if e == 0xF and m == 0x7:
            t[b] = np.nan
        elif e == 0:
            t[b] = s * (m / 8.0) * 2.0 ** -6
        else:
            t[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3 = e4m3_decode_table()


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3fn bytes with torch's cast (round-to-nearest-even,
    |x| > 448 -> NaN), which is what splitter.py:223-225 uses."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.float8_e4m3fn)
    return t.view(torch.uint8).numpy()


def e4m3_decode(b: np.ndarray) -> np.ndarray:
    return E4M3[np.asarray(b, np.uint8)]


# ---------------------------------------------------------------------------
# Predictor (predictor.py:55-96, :435-456) and cold-id selection (engine.py:274-283)
# ---------------------------------------------------------------------------
def predictor_logits(x: np.ndarray, w_down: np.ndarray, w_up: np.ndarray,
                     bias: np.ndarray):
    """Exact (float64) logits of ``up(down(x))`` (predictor.py:70-75) and a
    rigorous bound on the fp32 rounding error of any summation order.

    Returns (logits64, bound64); |fp32 logit - logits64| <= bound for a
    standard fp32 dot-product evaluation of either layer.
    """
    x = np.asarray(x, np.float64)
    wd = np.asarray(w_down, np.float64)
    wu = np.asarray(w_up, np.float64)
    b = np.asarray(bias, np.float64)
    z = x @ wd.T                                        # [.., R]
    u = 2.0 ** -24
    Kd, Ku = wd.shape[1], wu.shape[1]
    gd = Kd * u / (1 - Kd * u)
    gu = (Ku + 1) * u / (1 - (Ku + 1) * u)
    zerr = gd * (np.abs(x) @ np.abs(wd).T)              # |fl(z) - z|
    logits = z @ wu.T + b
    bound = gu * (np.abs(z) + zerr) @ np.abs(wu).T + gu * np.abs(b) + zerr @ np.abs(wu).T
    return logits, bound


def predictor_mask_fp32(x, w_down, w_up, bias, threshold: float = 0.5):
    """predict_mask in fp32 through torch, as the reference evaluates it
    (predictor.py:70-79: sigmoid(up(down(x))) >= threshold)."""
    import torch
    import torch.nn.functional as F
    xt = torch.as_tensor(np.asarray(x, np.float32))
    z = F.linear(xt, torch.as_tensor(np.asarray(w_down, np.float32)))
    lg = F.linear(z, torch.as_tensor(np.asarray(w_up, np.float32)),
                  torch.as_tensor(np.asarray(bias, np.float32)))
    return (torch.sigmoid(lg) >= threshold).numpy()


def cold_ids_for(mask: Optional[np.ndarray], hot_ids, inter_dim: int) -> list:
    """engine.py:274-283: ascending nonzero ids of the mask minus the hot ids;
    without a predictor every non-hot id."""
    hot = set(int(i) for i in np.asarray(hot_ids).tolist())
    if mask is not None:
        ids = np.nonzero(np.asarray(mask).reshape(-1))[0].tolist()
        return [i for i in ids if i not in hot]
    return [i for i in range(inter_dim) if i not in hot]


# ---------------------------------------------------------------------------
# FFN (engine.py:163-209) and the layer wrapper (engine.py:285-312)
# ---------------------------------------------------------------------------
def gated_act(g, u, activation: str, act_on_both: bool):
    """engine.py:163-170: relu if activation=='relu' else silu; act(g)*act(u)
    when act_on_both (dReLU) else act(g)*u (SwiGLU)."""
    if activation == "relu":
        act = lambda v: np.maximum(v, 0.0)
    else:
        act = lambda v: v / (1.0 + np.exp(-v))
    return act(g) * act(u) if act_on_both else act(g) * u


def sparse_ffn(x, activation, act_on_both, gate_hot, up_hot, down_hot,
               gate_cold, up_cold, down_cold) -> np.ndarray:
    """engine.py:173-209 in float64: hot half + cold half, exact by linearity.

    gate_*/up_*: [n, H]; down_*: [H, n] (reference layouts)."""
    x = np.asarray(x, np.float64)
    out = np.zeros_like(x)
    any_part = False
    for g_w, u_w, d_w in ((gate_hot, up_hot, down_hot), (gate_cold, up_cold, down_cold)):
        if g_w is None or np.asarray(g_w).shape[0] == 0:
            continue
        g = x @ np.asarray(g_w, np.float64).T
        u = x @ np.asarray(u_w, np.float64).T
        out = out + gated_act(g, u, activation, act_on_both) @ np.asarray(d_w, np.float64).T
        any_part = True
    return out if any_part else np.zeros_like(x)


def rmsnorm(x, w, eps: float):
    """torch.nn.RMSNorm (engine.py:247, :289, :295): x * rsqrt(mean(x^2)+eps) * w."""
    x = np.asarray(x, np.float64)
    r = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    return x * r * np.asarray(w, np.float64)


def ffn_layer(x, norm_w, eps, activation, act_on_both, hot, cold_rows):
    """SparseFFNLayer.forward (engine.py:292-312) for [B, H] input: RMSNorm,
    hot + selected cold neurons, residual.  ``hot`` = (gate[n,H], up[n,H],
    down[H,n]) decoded; ``cold_rows`` = (gate[m,H], up[m,H], down[H,m]) or None."""
    xn = rmsnorm(x, norm_w, eps)
    gc, uc, dc = cold_rows if cold_rows is not None else (None, None, None)
    return np.asarray(x, np.float64) + sparse_ffn(xn, activation, act_on_both,
                                                  hot[0], hot[1], hot[2], gc, uc, dc)


# ---------------------------------------------------------------------------
# Checker helpers for the fused stack (engine.py:292-312 per layer, with the
# predictor lookahead of engine.py:421-438)
# ---------------------------------------------------------------------------
def predictor_mask_banded(x, w_down, w_up, bias, logit_thr: float, norm_w=None, eps: float = 1e-5,
                          input_rel_err: float = 8 * 2.0 ** -24):
    """(mask, ambiguous): mask = exact logit >= logit_thr, where the input is
    RMSNorm(x) when ``norm_w`` is given; ``ambiguous`` marks neurons whose
    exact logit lies within the fp32 evaluation error bound of the
    threshold (any correct fp32 implementation may decide them either way).
    ``input_rel_err`` covers the rounding of the normalised input itself."""
    xin = rmsnorm(x, norm_w, eps) if norm_w is not None else np.asarray(x, np.float64)
    lg, bound = predictor_logits(xin, w_down, w_up, bias)
    dz = input_rel_err * (np.abs(xin) @ np.abs(np.asarray(w_down, np.float64)).T)
    bound = bound + dz @ np.abs(np.asarray(w_up, np.float64)).T
    bound = 2.0 * bound + 1e-12
    return lg >= logit_thr, np.abs(lg - logit_thr) <= bound


def mask_from_words(words, n: int) -> np.ndarray:
    """uint32/int32 words -> bool [n] (bit j of word w = id 32w + j)."""
    w = np.asarray(words).astype(np.int64) & 0xFFFFFFFF
    bits = ((w[:, None] >> np.arange(32)) & 1).astype(bool).reshape(-1)
    return bits[:n]


def words_from_mask(mask) -> np.ndarray:
    m = np.asarray(mask, bool)
    n = m.size
    pad = np.zeros(((n + 31) // 32) * 32, bool)
    pad[:n] = m
    w = (pad.reshape(-1, 32).astype(np.int64) << np.arange(32)).sum(axis=1)
    return w.astype(np.uint32).view(np.int32)


def ffn_layer_from_records(x, norm_w, eps, activation, act_on_both, hot, store: "ColdStoreOracle",
                           layer_idx: int, fetch_ids):
    """One SparseFFNLayer.forward in float64 with the cold rows read through
    the oracle store (read_neurons semantics), given the fetch id list."""
    rows = store.read_neurons(layer_idx, 0, list(fetch_ids)) if len(fetch_ids) else None
    return ffn_layer(np.asarray(x, np.float64).reshape(1, -1), norm_w, eps, activation, act_on_both, hot, rows)[0]


# ---------------------------------------------------------------------------
# Timed CPU baseline: the reference's per-layer CPU path on synthetic data
# ---------------------------------------------------------------------------
def make_cpu_layer(seed: int, inter: int = 14336, hot_frac: float = 0.2, rank: int = 64, std: float = 0.02):
    """One synthetic layer built on the CPU only (numpy / torch CPU): hot FP8
    by direct cast (splitter.py:221-226), cold INT4 records
    (splitter.py:228-256), predictor N(0, std), norm weight 1."""
    import torch
    g = torch.Generator().manual_seed(seed)
    H = HIDDEN_DIM
    gate = torch.randn(inter, H, generator=g) * std
    up = torch.randn(inter, H, generator=g) * std
    down = torch.randn(H, inter, generator=g) * std
    perm = torch.randperm(inter, generator=g)
    n_hot = int(hot_frac * inter)
    hot_ids = np.sort(perm[:n_hot].numpy())
    is_hot = np.zeros(inter, bool)
    is_hot[hot_ids] = True
    cold_ids = np.nonzero(~is_hot)[0]
    recs = build_records(cold_ids, gate.numpy()[cold_ids], up.numpy()[cold_ids], down.numpy()[:, cold_ids].T)
    buf, index = build_cold_file([(len(cold_ids), recs)])
    f8 = lambda t: t.to(torch.float8_e4m3fn).to(torch.float32)
    layer = {
        "hot_ids": hot_ids,
        "gate_hot": f8(gate[hot_ids]), "up_hot": f8(up[hot_ids]), "down_hot": f8(down[:, hot_ids]),
        "store": ColdStoreOracle(buf, index, {"hidden_dim": H}),
        "w_down": torch.randn(rank, H, generator=g) * std,
        "w_up": torch.randn(inter, rank, generator=g) * std,
        "b_up": torch.randn(inter, generator=g) * std,
        "norm": torch.ones(H),
        "inter": inter,
    }
    return layer


def ref_layer_cpu(layer: dict, x, activation: str = "relu", act_on_both: bool = True, eps: float = 1e-5):
    """SparseFFNLayer.forward on the CPU as the reference runs it
    (engine.py:292-312): torch RMSNorm; predict_mask (predictor.py:77);
    _cold_ids_for's Python filter (engine.py:280-281); read_neurons through
    the per-neuron store port (splitter.py:354-403); sparse_ffn in fp32 torch
    (engine.py:173-209); residual.  Returns (y, n_cold_fetched)."""
    import torch
    import torch.nn.functional as F
    x = torch.as_tensor(x, dtype=torch.float32).reshape(1, -1)
    xn = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * layer["norm"]
    probs = torch.sigmoid(F.linear(F.linear(xn, layer["w_down"]), layer["w_up"], layer["b_up"]))
    mask = probs >= 0.5
    hot = set(layer["hot_ids"].tolist())
    ids = [i for i in mask[0].nonzero(as_tuple=True)[0].tolist() if i not in hot]
    rows = layer["store"].read_neurons(0, 0, ids)
    act = F.relu if activation == "relu" else F.silu
    gated = (lambda g, u: act(g) * act(u)) if act_on_both else (lambda g, u: act(g) * u)
    g = F.linear(xn, layer["gate_hot"])
    u = F.linear(xn, layer["up_hot"])
    out = F.linear(gated(g, u), layer["down_hot"])
    if rows is not None:
        cg, cu, cd = (torch.from_numpy(r) for r in rows)
        out = out + F.linear(gated(F.linear(xn, cg), F.linear(xn, cu)), cd)
    return (x + out)[0], len(ids)
