"""B200 drop-in for the runtime half of the reference's ``splitter.py``.

* Format constants: identical to the reference (splitter.py:57-76).
* :class:`ColdWeightStore`: same constructor and ``read_neurons`` contract as
  the reference (splitter.py:307-407).  The whole ``cold_weights.bin`` image
  is uploaded unchanged to HBM (or kept in pinned host memory), a device
  table maps neuron ids to records, and a CUDA kernel gathers and
  dequantises the requested records in one launch.
* A GPU splitter (:func:`quantize_int4_rows`, :func:`build_records`,
  :func:`build_cold_image`, :func:`hot_from_dense`) that writes byte-identical
  records from device-resident weights, replacing the reference's
  per-vector Python loop (splitter.py:186-262), and :func:`split_dense`, the
  reference's split-dense entry point (splitter.py:129-302) on top of it:
  the same split directory, file for file.

Everything that computes runs on CUDA; there is no CPU fallback.
"""
from __future__ import annotations

import json
import struct
from pathlib import Path
from typing import Optional, Sequence

import numpy as np
import torch

import hc_native as N

# ─── Format constants (splitter.py:57-76) ──────────────────────────────────
HIDDEN_DIM = 4096
ALIGN_BYTES = 64
PAGE_ALIGN = 4096
HOT_COUNT_DENSE = 4096
_VEC_BYTES = HIDDEN_DIM // 2
_GROUP_SIZE = 128
_N_GROUPS = HIDDEN_DIM // _GROUP_SIZE
_SCALE_BYTES_PER_VEC = _N_GROUPS * 2
_SCALE_BYTES_TOTAL = _SCALE_BYTES_PER_VEC * 3
_RAW_RECORD = 2 + _VEC_BYTES * 3 + _SCALE_BYTES_TOTAL
NEURON_RECORD_BYTES = ((_RAW_RECORD + ALIGN_BYTES - 1) // ALIGN_BYTES) * ALIGN_BYTES
SECTION_HEADER_BYTES = 16
RECORD_READ_BYTES = 6352           # payload rounded up to 16: what the kernels read


def _words(n: int) -> int:
    return (n + 31) // 32


def bits_to_words(flags, n: int) -> torch.Tensor:
    """bool [n] -> int32 words with bit j of word w = flag of id 32w + j."""
    bits = np.zeros(_words(n) * 32, bool)
    bits[:n] = np.asarray(flags, bool)[:n]
    w = np.packbits(bits.reshape(-1, 32), axis=1, bitorder="little").view("<u4").reshape(-1)
    return torch.from_numpy(w.astype(np.uint32).view(np.int32).copy())


def words_to_bits(words, n: int) -> np.ndarray:
    """Inverse of :func:`bits_to_words` (accepts a tensor or array)."""
    w = np.asarray(words.cpu() if isinstance(words, torch.Tensor) else words).astype(np.int64) & 0xFFFFFFFF
    b = np.unpackbits(w.astype("<u4").view(np.uint8).reshape(-1, 4), axis=1, bitorder="little")
    return b.reshape(-1)[:n].astype(bool)


# ─── Cold weight reader (splitter.py:307-407) ───────────────────────────────
class ColdWeightStore:
    """Device-resident cold store with the reference's interface.

    ``ColdWeightStore(cold_bin, cold_index, config)`` loads the file image to
    ``device`` (``source="device"``, HBM) or to pinned host memory read over
    the bus by the same kernel (``source="pinned"``).  ``read_neurons`` keeps
    the reference's contract (splitter.py:354-403): (gate [N,H], up [N,H],
    down [H,N]) for the present ids in request order, absent ids skipped,
    ``None`` for an empty section or no match.  Tensors are returned on the
    store's device in ``out_dtype`` (fp32 by default, the reference's dtype);
    ``down`` is the transposed view of a neuron-major buffer.
    """

    def __init__(self, cold_bin: str, cold_index: str, config: dict, device="cuda",
                 source: str = "device", out_dtype: torch.dtype = torch.float32):
        self.config = config
        self.index = np.load(cold_index) if isinstance(cold_index, str) else np.asarray(cold_index)
        if self.index.ndim != 3 or self.index.shape[2] != 2:
            raise ValueError(f"cold_index must have shape (L, E, 2), got {self.index.shape}")
        self.H = config["hidden_dim"]
        self.I = config.get("intermediate_dim", config.get("expert_inter_dim"))
        if self.H != HIDDEN_DIM:
            raise ValueError(f"cold records are sized for hidden_dim {HIDDEN_DIM}, config says {self.H}")
        self.device = torch.device(device)
        self.out_dtype = out_dtype
        if isinstance(cold_bin, (bytes, bytearray, memoryview)):
            data = np.frombuffer(cold_bin, dtype=np.uint8)
        elif isinstance(cold_bin, torch.Tensor):
            data = None
            image = cold_bin
        else:
            data = np.fromfile(cold_bin, dtype=np.uint8)
        if data is not None:
            image = torch.from_numpy(data.copy() if not data.flags.writeable else data)
        self.image_bytes = int(image.numel())
        L = self.index.shape[0]
        offs = self.index[:, 0, 0].astype(np.int64)
        ncold = self.index[:, 0, 1].astype(np.int64)
        for li in range(L):
            if ncold[li] == 0:
                continue
            if offs[li] % 16 != 0:
                raise ValueError(f"layer {li}: section offset {offs[li]} is not 16-byte aligned")
            end = offs[li] + SECTION_HEADER_BYTES + (ncold[li] - 1) * NEURON_RECORD_BYTES + RECORD_READ_BYTES
            if end > self.image_bytes:
                raise ValueError(f"layer {li}: cold_index points past the end of cold_weights.bin "
                                 f"({end} > {self.image_bytes} bytes)")
        if source == "device":
            self.image = image.to(self.device) if image.device != self.device else image
        elif source == "pinned":
            self.image = image.cpu().pin_memory()
        else:
            raise ValueError("source must be 'device' or 'pinned'")
        self.source = source
        self.n_layers = L
        self.sec_off = torch.from_numpy(offs).to(self.device)
        self.n_rec = torch.from_numpy(ncold.astype(np.int32)).to(self.device)
        self.n_rec_host = ncold.astype(np.int32)
        self.status = N.new_status(self.device)
        self.table = torch.empty(L, N.TABLE_SIZE, dtype=torch.int32, device=self.device)
        with torch.cuda.device(self.device):
            N.check(N.lib.hc_build_record_table(N.ptr(self.image), self.image_bytes, N.ptr(self.sec_off),
                                                N.ptr(self.n_rec), L, int(ncold.max(initial=0)),
                                                N.ptr(self.table), N.ptr(self.status), N.stream_handle()),
                    "hc_build_record_table")
        self.table_host = self.table.cpu().numpy()          # host copy for list requests
        N.read_status(self.status, "hc_build_record_table")
        # kept for interface parity with the reference (filled on first access)
        self._offset_cache: dict = {}
        self._staging = None

    # -- reference interface ------------------------------------------------
    def _section_table(self, layer_idx: int, expert_idx: int):
        key = (layer_idx, expert_idx)
        cached = self._offset_cache.get(key)
        if cached is not None:
            return cached
        _, n_cold = self.index[layer_idx, expert_idx]
        if n_cold == 0:
            return None
        self._offset_cache[key] = self.table_host[layer_idx]
        return self._offset_cache[key]

    def read_neurons(self, layer_idx: int, expert_idx: int, neuron_ids):
        """splitter.py:354-403 on the GPU (see class docstring)."""
        tab = self._section_table(layer_idx, expert_idx)
        if tab is None:
            return None
        ids = np.asarray(list(neuron_ids) if not isinstance(neuron_ids, np.ndarray) else neuron_ids,
                         dtype=np.int64).reshape(-1)
        ok = (ids >= 0) & (ids < N.TABLE_SIZE)
        rec = np.full(ids.shape, -1, np.int32)
        rec[ok] = tab[ids[ok]]
        rec = rec[rec >= 0]
        if rec.size == 0:
            return None
        rec_t = torch.from_numpy(rec).pin_memory().to(self.device, non_blocking=True)
        g, u, d = self.read_records(layer_idx, rec_t)
        return g, u, d.t()

    def close(self):
        self.image = None
        self.table = None
        self._staging = None

    # -- device-side interface --------------------------------------------
    def read_records(self, layer_idx: int, rec_idx: torch.Tensor, count: Optional[torch.Tensor] = None,
                     out_dtype: Optional[torch.dtype] = None, out: Optional[torch.Tensor] = None):
        """Gather + dequantise records ``rec_idx`` (device int32 [K]) of one
        layer into neuron-major (gate, up, down) [K, H] tensors.  ``count``
        (device int32 [1]) limits the rows written without a host sync."""
        return tuple(self.gather_layers(torch.as_tensor([layer_idx]), rec_idx.view(1, -1), count, out_dtype, out)[:, 0])

    def gather_layers(self, layers, rec_idx: torch.Tensor, count: Optional[torch.Tensor] = None,
                      out_dtype: Optional[torch.dtype] = None, out: Optional[torch.Tensor] = None):
        """Batched gather over several layers in one launch.

        layers: host sequence/tensor of layer ids [Lb]; rec_idx: device int32
        [Lb, K]; returns (or fills ``out``) [3, Lb, K, H] = gate/up/down."""
        dt = out_dtype or self.out_dtype
        code = {torch.float32: N.HC_F32, torch.bfloat16: N.HC_BF16}.get(dt)
        if code is None:
            raise ValueError("out_dtype must be float32 or bfloat16")
        layers = torch.as_tensor(layers, dtype=torch.long).reshape(-1)
        N.require_cuda(rec_idx)
        rec_idx = rec_idx.to(torch.int32).contiguous()
        Lb, K = rec_idx.shape
        if layers.numel() == self.n_layers and bool((layers == torch.arange(self.n_layers)).all()):
            so, nr = self.sec_off, self.n_rec
        else:
            li = layers.to(self.device)
            so, nr = self.sec_off[li].contiguous(), self.n_rec[li].contiguous()
        if out is None:
            out = torch.empty(3, Lb, K, self.H, dtype=dt, device=self.device)
        N.check(N.lib.hc_cold_gather_dequant(N.ptr(self.image), self.image_bytes, N.ptr(so), N.ptr(nr), Lb,
                                             N.ptr(rec_idx), K, N.ptr(count), code, N.ptr(out[0]),
                                             N.ptr(out[1]), N.ptr(out[2]), N.ptr(self.status),
                                             N.stream_handle()), "hc_cold_gather_dequant")
        return out

    def check(self):
        """Raise if a kernel flagged an error (synchronises)."""
        N.read_status(self.status, "ColdWeightStore")

    def section_records(self, layer_idx: int) -> torch.Tensor:
        """View of the first record of a layer's section (for the fused FFN):
        device memory, or pinned host memory for ``source="pinned"``."""
        off = int(self.index[layer_idx, 0, 0])
        return self.image[off + SECTION_HEADER_BYTES:]

    def stage_bytes(self) -> int:
        """Size of a device buffer that holds any one section's records at
        their own offsets (record r at r * 6400)."""
        return max(int(self.n_rec_host.max(initial=0)), 1) * NEURON_RECORD_BYTES

    def staging(self) -> torch.Tensor:
        """The store's device staging buffer (:meth:`stage_bytes`, allocated on
        first use): the section a fused kernel reads for a layer whose
        records :meth:`fetch_masked` fetched.  Every stack over this store
        shares it, so their launches must stay in one stream's order."""
        if self._staging is None:
            n = max(int(self.n_rec_host.max(initial=0)), 1)
            self._staging = torch.empty(self.stage_bytes(), dtype=torch.uint8, device=self.device)
            self._stage_rec = torch.empty(n, dtype=torch.int32, device=self.device)
            self._stage_count = torch.zeros(1, dtype=torch.int32, device=self.device)
        return self._staging

    def fetch_masked(self, layer_idx: int, words: torch.Tensor, fetch_bits: torch.Tensor, inter: int,
                     batch: int = 1) -> torch.Tensor:
        """Fetch the records of layer ``layer_idx`` whose ids are set in
        ``words`` (int32 mask words, [batch][ceil(inter/32)] rows: their
        union) and in ``fetch_bits`` into :meth:`staging`, on the device (no
        host sync).  Returns the staging buffer."""
        dst = self.staging()
        W = (inter + 31) // 32
        n = max(int(self.n_rec_host[layer_idx]), 1)
        N.check(N.lib.hc_union_cold(N.ptr(words), batch, words.stride(0) if words.dim() > 1 else W, inter,
                                    N.ptr(fetch_bits), N.ptr(self.table[layer_idx]), N.ptr(self._stage_rec),
                                    N.ptr(self._stage_count), N.stream_handle()), "hc_union_cold")
        self.stage_records(layer_idx, self._stage_rec[:n], dst, self._stage_count)
        return dst

    def stage_records(self, layer_idx: int, rec_idx: torch.Tensor, dst: torch.Tensor,
                      count: Optional[torch.Tensor] = None):
        """The per-layer fetch of the cold tier: copy the raw records
        ``rec_idx`` (device int32 [K]; the first ``count[0]`` entries when a
        device ``count`` is given) of layer ``layer_idx`` from the store
        (pinned host memory over the bus, or HBM) to the same offsets of the
        device buffer ``dst`` (uint8, at least :meth:`stage_bytes`).  Bad
        indices flag HC_ERR_RANGE in :meth:`check`; asynchronous."""
        N.require_cuda(rec_idx, dst)
        if rec_idx.dtype != torch.int32 or not rec_idx.is_contiguous():
            raise ValueError("rec_idx must be a contiguous int32 tensor")
        src = self.section_records(layer_idx)
        N.check(N.lib.hc_cold_stage(N.ptr(src), src.numel(), N.ptr(rec_idx), N.ptr(count), rec_idx.numel(),
                                    int(self.n_rec_host[layer_idx]), N.ptr(dst), dst.numel(), N.ptr(self.status),
                                    N.stream_handle()), "hc_cold_stage")

    def fetch_bits(self, layer_idx: int, hot_ids, inter: Optional[int] = None) -> torch.Tensor:
        """uint32 words: bit i set iff id i has a record and is not hot -- the
        ids engine.py:281 can fetch (hot ids are filtered out there and
        read_neurons drops ids without a record)."""
        inter = inter or self.I
        has = self.table_host[layer_idx, :inter] >= 0
        if hot_ids is not None and len(hot_ids):
            h = np.asarray(hot_ids, np.int64)
            h = h[(h >= 0) & (h < inter)]
            has[h] = False
        return bits_to_words(has, inter).to(self.device)


# ─── GPU splitter: identical bytes from device-resident weights ───────────────
def quantize_int4_rows(x: torch.Tensor, group_size: int = _GROUP_SIZE):
    """Row-wise quantize_int4 (splitter.py:81-108) on the GPU.

    x: float32 [R, N] CUDA tensor, N % group_size == 0.  Returns (packed uint8
    [R, N/2], scales fp32 [R, N/group]).  Uses true division by a tensor
    divisor, as the reference's CPU code does, so bytes are identical."""
    N.require_cuda(x)
    x = x.float()
    R, n = x.shape
    if n % group_size:
        raise ValueError("row length must be a multiple of the group size")
    g = x.view(R, n // group_size, group_size)
    absmax = g.abs().amax(dim=2).clamp(min=1e-8)
    scales = absmax / torch.full_like(absmax, 7.0)
    q = torch.round(g / scales.unsqueeze(2)).clamp_(-8, 7).to(torch.int8).view(R, n)
    lo = q[:, 0::2].view(torch.uint8) & 0x0F
    hi = (q[:, 1::2].view(torch.uint8) & 0x0F) << 4
    return (lo | hi), scales


def build_records(nids: torch.Tensor, gate: torch.Tensor, up: torch.Tensor, down_cols: torch.Tensor) -> torch.Tensor:
    """Neuron records exactly as split_dense writes them (splitter.py:234-248).

    nids [n]; gate/up/down_cols [n, H] fp32 on the GPU (down_cols[i] is
    down[:, nid_i]).  Returns uint8 [n, NEURON_RECORD_BYTES] on the GPU."""
    n = gate.shape[0]
    rec = torch.zeros(n, NEURON_RECORD_BYTES, dtype=torch.uint8, device=gate.device)
    nid = nids.to(device=gate.device, dtype=torch.int64)
    rec[:, 0] = (nid & 0xFF).to(torch.uint8)          # '<H' little-endian id
    rec[:, 1] = ((nid >> 8) & 0xFF).to(torch.uint8)
    off = 2
    s16 = []
    for m in (gate, up, down_cols):
        p, s = quantize_int4_rows(m)
        rec[:, off:off + _VEC_BYTES] = p
        off += _VEC_BYTES
        s16.append(s.to(torch.float16))
    for s in s16:
        rec[:, off:off + _SCALE_BYTES_PER_VEC] = s.view(torch.uint8).view(n, _SCALE_BYTES_PER_VEC)
        off += _SCALE_BYTES_PER_VEC
    return rec


def build_cold_image(sections: Sequence[torch.Tensor], device="cuda"):
    """Assemble a cold_weights.bin image (splitter.py:228-262) from per-layer
    record tensors [n_l, 6400].  Returns (uint8 image on `device`, cold_index
    numpy uint64 [L, 1, 2])."""
    L = len(sections)
    index = np.zeros((L, 1, 2), np.uint64)
    sizes = []
    cursor = 0
    for li, recs in enumerate(sections):
        n = int(recs.shape[0])
        start = cursor
        cursor += SECTION_HEADER_BYTES + n * NEURON_RECORD_BYTES
        cursor += (-cursor) % PAGE_ALIGN
        index[li, 0] = (start, n)
        sizes.append((start, n))
    image = torch.zeros(cursor, dtype=torch.uint8, device=device)
    for li, (start, n) in enumerate(sizes):
        hdr = torch.frombuffer(bytearray(struct.pack("<HHIq", li, 0, n, 0)), dtype=torch.uint8)
        image[start:start + SECTION_HEADER_BYTES] = hdr.to(device)
        if n:
            body = sections[li].reshape(-1)
            image[start + SECTION_HEADER_BYTES:start + SECTION_HEADER_BYTES + body.numel()] = body.to(device)
    return image, index


def hot_from_dense(gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor, hot_ids: torch.Tensor,
                   row_scale: bool = False):
    """Hot FP8 tensors of split_dense (splitter.py:221-226): direct e4m3 cast
    of gate[hot], up[hot], down[:, hot].  With ``row_scale`` each neuron's
    three vectors get an absmax/448 scale first (stored separately, fp32
    [n_hot, 3]); without it the scales are 1 and the bytes equal the
    reference's."""
    g, u, d = gate[hot_ids].float(), up[hot_ids].float(), down[:, hot_ids].float().t()
    scales = None
    if row_scale:
        s = torch.stack([t.abs().amax(dim=1) for t in (g, u, d)], dim=1).clamp(min=1e-12)
        scales = s / torch.full_like(s, 448.0)
        g, u, d = g / scales[:, 0:1], u / scales[:, 1:2], d / scales[:, 2:3]
    return (g.to(torch.float8_e4m3fn), u.to(torch.float8_e4m3fn), d.t().to(torch.float8_e4m3fn), scales)


# ─── split_dense (splitter.py:129-302) ────────────────────────────────────────
def _load_base_model(base_model, trust_remote_code: bool):
    """The model object split_dense reads: passed in directly, or loaded from a
    path the way the reference does (fp16 on the CPU, splitter.py:151-154)."""
    if not isinstance(base_model, (str, Path)):
        return base_model
    from transformers import AutoModelForCausalLM      # only needed for a checkpoint path
    return AutoModelForCausalLM.from_pretrained(str(base_model), torch_dtype=torch.float16, device_map="cpu",
                                                trust_remote_code=trust_remote_code)


def split_dense(base_model, profile_path: str, output_dir: str, hot_count: int = HOT_COUNT_DENSE,
                trust_remote_code: bool = False, device="cuda") -> dict:
    """The reference's split-dense step (splitter.py:129-302) on the GPU.

    ``base_model`` is a checkpoint path (loaded like the reference: fp16 on
    the CPU) or an already loaded causal-LM object with the same attributes
    (``config``, ``model.layers[i].self_attn/mlp/norms``, ``model.embed_tokens``,
    ``model.norm``, ``lm_head``).  Writes the same artefacts into
    ``output_dir`` -- ``hot_weights/shared.pt``,
    ``hot_weights/layer_XXX_expert_000.pt``, ``cold_weights.bin``,
    ``cold_index.npy`` and ``split_config.json`` -- with the same contents:
    weights taken at fp16 as the reference loads them, hot neurons = top
    ``hot_count`` of the profile's ``expert_0`` frequencies (torch.topk on the
    host, as the reference), hot FP8 by direct cast, cold records quantised on
    the GPU by :func:`build_records` (byte-identical to the reference's
    per-vector loop).  Raises ValueError where the reference does (hidden size
    other than 4096, a layer without usable frequencies).  Returns the config
    dict."""
    out = Path(output_dir)
    hot_dir = out / "hot_weights"
    hot_dir.mkdir(parents=True, exist_ok=True)
    with open(profile_path) as f:
        profile = json.load(f)
    model = _load_base_model(base_model, trust_remote_code)
    hf = model.config
    if hf.hidden_size != HIDDEN_DIM:
        raise ValueError(f"Base model hidden_size={hf.hidden_size} but the cold-record binary layout is sized for "
                         f"{HIDDEN_DIM}")
    dev = torch.device(device)
    f16 = lambda w: w.data.to(torch.float16) if hasattr(w, "data") else torch.as_tensor(w).to(torch.float16)
    layers = model.model.layers
    num_layers = hf.num_hidden_layers
    inter_dim = hf.intermediate_size

    shared = {}
    for li, layer in enumerate(layers):
        for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
            w = f16(getattr(layer.self_attn, name).weight)
            shared[f"layer_{li:03d}.{name}"] = w.to(dev).to(torch.float8_e4m3fn).cpu()
        shared[f"layer_{li:03d}.input_layernorm"] = f16(layer.input_layernorm.weight).cpu()
        shared[f"layer_{li:03d}.post_attention_layernorm"] = f16(layer.post_attention_layernorm.weight).cpu()
    shared["embed_tokens"] = f16(model.model.embed_tokens.weight).cpu()
    shared["lm_head"] = f16(model.lm_head.weight).cpu()
    shared["final_norm"] = f16(model.model.norm.weight).cpu()
    torch.save(shared, str(hot_dir / "shared.pt"))
    del shared

    cold_index = np.zeros((num_layers, 1, 2), dtype=np.uint64)
    total_hot = total_cold = 0
    cursor = 0
    with open(out / "cold_weights.bin", "wb") as cold_f:
        for li in range(num_layers):
            mlp = layers[li].mlp
            gate = f16(mlp.gate_proj.weight).to(dev).float()          # (I, H)
            up = f16(mlp.up_proj.weight).to(dev).float()              # (I, H)
            down = f16(mlp.down_proj.weight).to(dev).float()          # (H, I)
            I = gate.shape[0]
            freq_list = profile["layers"].get(str(li), {}).get("expert_0", [])
            if not freq_list or len(freq_list) != I:
                raise ValueError(f"profile has no usable expert_0 frequencies for layer {li} "
                                 f"(got {len(freq_list)}, need {I})")
            top = torch.topk(torch.tensor(freq_list), min(hot_count, I)).indices
            hot_mask = torch.zeros(I, dtype=torch.bool)
            hot_mask[top] = True
            hot_ids = hot_mask.nonzero(as_tuple=True)[0]
            cold_ids = (~hot_mask).nonzero(as_tuple=True)[0]
            total_hot += len(hot_ids)
            total_cold += len(cold_ids)
            hd = hot_ids.to(dev)
            torch.save({"neuron_ids": hot_ids,
                        "gate": gate[hd].to(torch.float8_e4m3fn).cpu(),
                        "up": up[hd].to(torch.float8_e4m3fn).cpu(),
                        "down": down[:, hd].to(torch.float8_e4m3fn).cpu()},
                       str(hot_dir / f"layer_{li:03d}_expert_000.pt"))
            cd = cold_ids.to(dev)
            start = cursor
            cold_f.write(struct.pack("<HHIq", li, 0, len(cold_ids), 0))
            cursor += SECTION_HEADER_BYTES
            # records in chunks (bounded device memory), in cold-id order
            for c0 in range(0, len(cold_ids), 4096):
                ids = cd[c0:c0 + 4096]
                rec = build_records(ids, gate[ids], up[ids], down[:, ids].t().contiguous())
                cold_f.write(rec.cpu().numpy().tobytes())
                cursor += rec.numel()
            pad = (-cursor) % PAGE_ALIGN
            if pad:
                cold_f.write(b"\x00" * pad)
                cursor += pad
            cold_index[li, 0] = (start, len(cold_ids))
            del gate, up, down
    np.save(str(out / "cold_index.npy"), cold_index)
    config = {
        "base_model": str(base_model) if isinstance(base_model, (str, Path)) else getattr(hf, "_name_or_path", ""),
        "hidden_dim": hf.hidden_size,
        "intermediate_dim": inter_dim,
        "expert_inter_dim": inter_dim,
        "num_experts": 1,
        "num_layers": num_layers,
        "vocab_size": hf.vocab_size,
        "num_attention_heads": hf.num_attention_heads,
        "num_key_value_heads": hf.num_key_value_heads,
        "rope_theta": getattr(hf, "rope_theta", 10000.0),
        "rms_norm_eps": hf.rms_norm_eps,
        "hidden_act": hf.hidden_act,
        "act_on_both": getattr(hf, "model_type", "") == "bamboo",
        "max_position_embeddings": hf.max_position_embeddings,
        "hot_count": hot_count,
        "total_hot_neurons": int(total_hot),
        "total_cold_neurons": int(total_cold),
        "hot_fraction": total_hot / max(total_hot + total_cold, 1),
        "cold_file_bytes": cursor,
        "neuron_record_bytes": NEURON_RECORD_BYTES,
        "page_align": PAGE_ALIGN,
    }
    with open(out / "split_config.json", "w") as f:
        json.dump(config, f, indent=2)
    return config
