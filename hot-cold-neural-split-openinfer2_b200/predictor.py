"""B200 drop-in for the inference half of the reference's ``predictor.py``.

``NeuronPredictor`` keeps the reference's module layout (``down``:
Linear(hidden -> rank, no bias), ``up``: Linear(rank -> inter)) and its
``save``/``load`` file format (predictor.py:55-96), so the reference's trained
predictor files load unchanged.  ``forward``/``predict_mask`` run the fused
CUDA predictor (two launches, no host sync).  ``PredictorRegistry`` mirrors
predictor.py:413-462.

The mask decision equals the reference's ``torch.sigmoid(logit) >=
threshold`` for the same fp32 logit: :func:`logit_threshold` finds, once per
threshold, the smallest fp32 logit whose torch sigmoid reaches it, and the
kernel compares logits against that value.
"""
from __future__ import annotations

import functools
from pathlib import Path
from typing import Optional

import numpy as np
import torch
import torch.nn as nn

import hc_native as N


def _f32_key(v: float) -> int:
    """Order-preserving integer image of an fp32 value."""
    i = int(np.array([v], np.float32).view(np.int32)[0])
    return i if i >= 0 else -(i & 0x7FFFFFFF)


def _f32_from_keys(keys: np.ndarray) -> np.ndarray:
    keys = np.asarray(keys, np.int64)
    bits = np.where(keys >= 0, keys, (-keys) | 0x80000000).astype(np.uint32)
    return bits.view(np.float32)


def _torch_sigmoid_ge(vals: np.ndarray, threshold: float) -> np.ndarray:
    # evaluate like the reference does: a vector-width fp32 tensor through
    # torch.sigmoid (its scalar tail path may round differently)
    v = torch.from_numpy(np.ascontiguousarray(vals, np.float32))
    pad = (-v.numel()) % 64 + 64
    v = torch.cat([v, v[-1:].expand(pad)])
    return (torch.sigmoid(v) >= threshold).numpy()[: len(vals)]


@functools.lru_cache(maxsize=64)
def logit_threshold(threshold: float) -> float:
    """Smallest fp32 z such that every fp32 logit >= z satisfies the
    reference's ``torch.sigmoid(logit) >= threshold`` (and none below it,
    checked over a window of 8193 neighbouring values); +inf if no value
    passes, -inf if every value does."""
    ge = lambda v: bool(_torch_sigmoid_ge(np.array([v], np.float32), threshold)[0])
    if ge(float("-inf")):
        return float("-inf")
    if not ge(float("inf")):
        return float("inf")
    lo, hi = _f32_key(-np.finfo(np.float32).max), _f32_key(np.finfo(np.float32).max)
    while hi - lo > 1:                       # invariant: not ge(lo), ge(hi)
        mid = (lo + hi) // 2
        if ge(float(_f32_from_keys(np.array([mid]))[0])):
            hi = mid
        else:
            lo = mid
    # torch's fp32 sigmoid need not be monotone in the last ulp: take the
    # upper edge of any mixed window around the crossing
    keys = np.arange(hi - 4096, hi + 4097, dtype=np.int64)
    vals = _f32_from_keys(keys)
    ok = _torch_sigmoid_ge(vals, threshold)
    fail = np.nonzero(~ok)[0]
    first = fail[-1] + 1 if fail.size else 0
    return float(vals[min(first, len(vals) - 1)])


class NeuronPredictor(nn.Module):
    """Low-rank activation predictor (predictor.py:55-96) on the fused kernel."""

    def __init__(self, hidden_dim: int, intermediate_dim: int, rank: int = 64):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.intermediate_dim = intermediate_dim
        self.rank = rank
        self.down = nn.Linear(hidden_dim, rank, bias=False)
        self.up = nn.Linear(rank, intermediate_dim, bias=True)
        self._ws: Optional[torch.Tensor] = None
        self._ws_batch = 0
        self._w_down_t: Optional[torch.Tensor] = None
        self._status: Optional[torch.Tensor] = None

    # -- kernel plumbing ---------------------------------------------------
    def _workspace(self, batch: int) -> torch.Tensor:
        dev = self.down.weight.device
        if self._ws is None or self._ws_batch < batch or self._ws.device != dev:
            nbytes = int(N.lib.hc_predictor_workspace_bytes(batch, self.rank, self.intermediate_dim))
            self._ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
            self._ws_batch = batch
        return self._ws

    def _launch(self, x: torch.Tensor, threshold: float, want_probs: bool = False, want_logits: bool = False,
                norm_w: Optional[torch.Tensor] = None, eps: float = 0.0, fetch_bits=None, table=None,
                ids_out=None, rec_out=None, count_out=None, mask_out=None):
        w_down = self.down.weight
        N.require_cuda(w_down, x)
        if w_down.dtype != torch.float32:
            raise TypeError("NeuronPredictor weights must be float32 (the reference stores them in fp32)")
        lead = x.shape[:-1]
        x2 = x.reshape(-1, self.hidden_dim).to(torch.float32).contiguous()
        B = x2.shape[0]
        I = self.intermediate_dim
        words = (I + 31) // 32
        if mask_out is None:
            mask_out = torch.empty(B, words, dtype=torch.int32, device=x.device)
        probs = torch.empty(B, I, dtype=torch.float32, device=x.device) if want_probs else None
        logits = torch.empty(B, I, dtype=torch.float32, device=x.device) if want_logits else None
        thr = logit_threshold(float(threshold))
        if self._status is None or self._status.device != x.device:
            self._status = N.new_status(x.device)
        status = self._status
        for b0 in range(0, B, 64):
            nb = min(64, B - b0)
            ws = self._workspace(nb)
            N.check(N.lib.hc_predictor_forward(
                N.ptr(x2[b0:b0 + nb]), nb, N.ptr(norm_w), float(eps), N.ptr(w_down.data),
                N.ptr(self.up.weight.data), N.ptr(self.up.bias.data), self.rank, I, thr,
                N.ptr(mask_out[b0:b0 + nb]),
                N.ptr(probs[b0:b0 + nb]) if probs is not None else None,
                N.ptr(logits[b0:b0 + nb]) if logits is not None else None,
                N.ptr(fetch_bits) if b0 == 0 else None, N.ptr(table), N.ptr(ids_out), N.ptr(rec_out),
                N.ptr(count_out), N.ptr(ws), N.ptr(status), N.stream_handle()), "hc_predictor_forward")
        return lead, mask_out, probs, logits

    # -- reference interface ---------------------------------------------
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """Probability each neuron activates: sigmoid(up(down(x))) (predictor.py:70-75)."""
        lead, _, probs, _ = self._launch(x, 0.5, want_probs=True)
        return probs.reshape(*lead, self.intermediate_dim)

    def predict_mask(self, x: torch.Tensor, threshold: float = 0.5) -> torch.Tensor:
        """Boolean mask of predicted-active neurons (predictor.py:77-79)."""
        lead, words, _, _ = self._launch(x, threshold)
        return unpack_mask(words, self.intermediate_dim).reshape(*lead, self.intermediate_dim)

    def logits(self, x: torch.Tensor) -> torch.Tensor:
        lead, _, _, lg = self._launch(x, 0.5, want_logits=True)
        return lg.reshape(*lead, self.intermediate_dim)

    def predict_words(self, x: torch.Tensor, threshold: float = 0.5, norm_w=None, eps: float = 0.0,
                      mask_out=None) -> torch.Tensor:
        """Packed uint32 mask words [B, ceil(I/32)] (bit j of word w = id 32w+j)."""
        return self._launch(x, threshold, norm_w=norm_w, eps=eps, mask_out=mask_out)[1]

    def predict_ids(self, x: torch.Tensor, fetch_bits: torch.Tensor, table: Optional[torch.Tensor] = None,
                    threshold: float = 0.5, norm_w=None, eps: float = 0.0):
        """Ascending ids of (mask & fetch_bits) for row 0 of ``x`` -- the list
        SparseFFNLayer._cold_ids_for builds (engine.py:274-283) -- plus their
        record indices, all on the device: (ids int32 [I], recs int32 [I],
        count int32 [1]); only the first ``count`` entries are valid."""
        dev = x.device
        I = self.intermediate_dim
        ids = torch.empty(I, dtype=torch.int32, device=dev)
        recs = torch.empty(I, dtype=torch.int32, device=dev) if table is not None else None
        count = torch.zeros(1, dtype=torch.int32, device=dev)
        self._launch(x[..., :].reshape(-1, self.hidden_dim)[:1], threshold, norm_w=norm_w, eps=eps,
                     fetch_bits=fetch_bits, table=table, ids_out=ids, rec_out=recs, count_out=count)
        return ids, recs, count

    def down_t(self) -> torch.Tensor:
        """W_down transposed to [hidden][rank] (the fused stack kernel's layout)."""
        if self._w_down_t is None or self._w_down_t.device != self.down.weight.device:
            self._w_down_t = self.down.weight.data.t().contiguous()
        return self._w_down_t

    # -- serialisation (predictor.py:83-96, same format) -------------------
    def save(self, path: str):
        torch.save({
            "hidden_dim": self.hidden_dim,
            "intermediate_dim": self.intermediate_dim,
            "rank": self.rank,
            "state_dict": self.state_dict(),
        }, path)

    @classmethod
    def load(cls, path: str, device: str = "cuda") -> "NeuronPredictor":
        ckpt = torch.load(path, map_location=device)
        model = cls(ckpt["hidden_dim"], ckpt["intermediate_dim"], ckpt["rank"])
        model.load_state_dict(ckpt["state_dict"])
        return model.to(device).eval()


def unpack_mask(words: torch.Tensor, n: int) -> torch.Tensor:
    """int32 words [B, W] -> bool [B, n] on the same device."""
    w = words.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(32, device=words.device, dtype=torch.int64)
    bits = ((w.unsqueeze(-1) >> shifts) & 1).bool()
    return bits.reshape(words.shape[0], -1)[:, :n]


class PredictorRegistry:
    """All per-layer predictors resident on the device (predictor.py:413-462)."""

    def __init__(self, predictor_dir: str, device: str = "cuda"):
        self.predictors: dict[tuple[int, int], NeuronPredictor] = {}
        self.device = device
        for f in sorted(Path(predictor_dir).glob("layer_*_expert_*.pt")):
            parts = f.stem.split("_")
            self.predictors[(int(parts[1]), int(parts[3]))] = NeuronPredictor.load(str(f), device)

    def predict(self, layer_idx: int, expert_idx: int, hidden_state: torch.Tensor,
                threshold: float = 0.5) -> Optional[torch.Tensor]:
        """Boolean mask of predicted-active neurons, or None when the layer has
        no predictor (predictor.py:435-456)."""
        p = self.predictors.get((layer_idx, expert_idx))
        if p is None:
            return None
        with torch.no_grad():
            return p.predict_mask(hidden_state.to(torch.float32), threshold)

    def get(self, layer_idx: int, expert_idx: int = 0) -> Optional[NeuronPredictor]:
        return self.predictors.get((layer_idx, expert_idx))

    def vram_usage_mb(self) -> float:
        total = 0
        for p in self.predictors.values():
            total += sum(par.numel() * par.element_size() for par in p.parameters())
        return total / 1e6
