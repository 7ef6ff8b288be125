"""Seeded synthetic models in the reference's split format, built on the GPU.

Random-init weights stand in for the checkpoints the reference splits (there
is no network here).  ``make_stack`` follows the benchmark configurations:

* gate/up [I, H] and down [H, I] ~ N(0, 0.02) fp32 per layer;
* hot set = the first ``hot_frac`` of a seeded random ranking (the stand-in
  for the profile's frequency top-k, splitter.py:201-206), ids ascending;
* hot -> FP8 e4m3 by direct cast (splitter.py:223-225; optional per-neuron
  absmax scales), cold -> INT4 records written by the GPU splitter in the
  exact on-disk layout (splitter.py:228-262);
* per-layer predictor hidden -> rank -> I with W ~ N(0, 0.02), bias ~ N(0,
  0.02) (predictor.py:66-67 geometry), RMSNorm weights = 1.

The returned :class:`SynthStack` keeps the host-side copies a checker needs.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch

from engine import BatchStack, FFNStack, HotNeurons
from predictor import NeuronPredictor
from splitter import HIDDEN_DIM, ColdWeightStore, build_cold_image, build_records, hot_from_dense


@dataclass
class SynthStack:
    store: ColdWeightStore
    hot: list
    norms: list
    predictors: list
    cold_index: np.ndarray
    inter: int
    activation: str
    act_on_both: bool
    eps: float
    seed: int
    image: Optional[torch.Tensor] = None
    extra: dict = field(default_factory=dict)

    def stack(self, grid: int = 0, threshold: float = 0.5, with_predictors: bool = True, tp=None) -> FFNStack:
        preds = self.predictors if with_predictors else [None] * len(self.hot)
        return FFNStack(self.store, self.hot, self.norms, preds, self.activation, self.act_on_both, self.eps,
                        threshold, grid=grid, inter=self.inter, tp=tp)

    def batch_stack(self, threshold: float = 0.5, with_predictors: bool = False, max_batch: int = 64,
                    dense_min_batch: int = 8, single_token_stack: bool = True, shard=None,
                    group=None) -> BatchStack:
        preds = self.predictors if with_predictors else None
        return BatchStack(self.store, self.hot, self.norms, preds, self.activation, self.act_on_both, self.eps,
                          threshold, inter=self.inter, max_batch=max_batch, dense_min_batch=dense_min_batch,
                          single_token_stack=single_token_stack, shard=shard, group=group)


def make_stack(n_layers: int = 32, inter: int = 14336, hot_frac: float = 0.2, rank: int = 64,
               activation: str = "relu", act_on_both: bool = True, seed: int = 0, device="cuda",
               std: float = 0.02, row_scale: bool = False, predictors: bool = True, eps: float = 1e-5,
               norm_std: float = 0.0, keep_dense: bool = False) -> SynthStack:
    dev = torch.device(device)
    H = HIDDEN_DIM
    n_hot = int(hot_frac * inter)
    sections, hot, norms, preds = [], [], [], []
    dense = []
    for li in range(n_layers):
        g = torch.Generator(device=dev).manual_seed(seed * 1000 + li)
        gate = torch.randn(inter, H, generator=g, device=dev) * std
        up = torch.randn(inter, H, generator=g, device=dev) * std
        down = torch.randn(H, inter, generator=g, device=dev) * std
        rank_perm = torch.randperm(inter, generator=g, device=dev)
        hot_ids = torch.sort(rank_perm[:n_hot]).values
        is_hot = torch.zeros(inter, dtype=torch.bool, device=dev)
        is_hot[hot_ids] = True
        cold_ids = torch.nonzero(~is_hot).flatten()
        hg, hu, hd, hs = hot_from_dense(gate, up, down, hot_ids, row_scale=row_scale)
        hot.append(HotNeurons(hot_ids, hg, hu, hd, hs, dev))
        sections.append(build_records(cold_ids, gate[cold_ids], up[cold_ids], down[:, cold_ids].t().contiguous()))
        if norm_std > 0:
            norms.append(1.0 + norm_std * torch.randn(H, generator=g, device=dev))
        else:
            norms.append(torch.ones(H, device=dev))
        if predictors:
            p = NeuronPredictor(H, inter, rank).to(dev)
            with torch.no_grad():
                p.down.weight.copy_(torch.randn(rank, H, generator=g, device=dev) * std)
                p.up.weight.copy_(torch.randn(inter, rank, generator=g, device=dev) * std)
                p.up.bias.copy_(torch.randn(inter, generator=g, device=dev) * std)
            preds.append(p.eval())
        else:
            preds.append(None)
        if keep_dense:
            dense.append((gate.cpu(), up.cpu(), down.cpu(), hot_ids.cpu()))
        del gate, up, down
    image, index = build_cold_image(sections, device=dev)
    del sections
    cfg = {"hidden_dim": H, "intermediate_dim": inter}
    store = ColdWeightStore(image, index, cfg, device=dev)
    out = SynthStack(store, hot, norms, preds, index, inter, activation, act_on_both, eps, seed, image)
    if keep_dense:
        out.extra["dense"] = dense
    return out


def bernoulli_words(n_layers: int, batch: int, inter: int, p: float = 0.1, seed: int = 2, device="cuda"):
    """Per-token Bernoulli(p) active masks as packed int32 words [L, B, W]
    (bit j of word w = neuron 32w + j), drawn on the device from ``seed``."""
    dev = torch.device(device)
    W = (inter + 31) // 32
    g = torch.Generator(device=dev).manual_seed(seed)
    bits = torch.zeros(n_layers, batch, W * 32, dtype=torch.int64, device=dev)
    bits[..., :inter] = (torch.rand(n_layers, batch, inter, generator=g, device=dev) < p).to(torch.int64)
    shifts = torch.arange(32, dtype=torch.int64, device=dev)
    words = (bits.view(n_layers, batch, W, 32) << shifts).sum(dim=-1)
    return (words - ((words >> 31) << 32)).to(torch.int32)      # two's-complement view of the u32 words
