"""ctypes binding of libhotcold.so (the C ABI declared in include/hotcold.h).

This is the only module that touches the native library.  Importing it never
compiles anything; a missing library raises ImportError, and every compute
helper requires CUDA tensors -- there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

import torch

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libhotcold.so")

HC_OK = 0
HC_ERR_ARG = 1
HC_ERR_CUDA = 2
HC_ERR_RANGE = 4
HC_ERR_TIMEOUT = 8
HC_ERR_UNSUPPORTED = 16

HC_F32, HC_BF16, HC_F16 = 0, 1, 2
HC_ACT_SILU, HC_ACT_RELU = 0, 1
ABI_VERSION = 3

TABLE_SIZE = 65536


class HotColdError(RuntimeError):
    """A libhotcold call (or a kernel's device status word) reported an error."""

    def __init__(self, where: str, status: int):
        self.status = int(status)
        super().__init__(f"{where}: {status_string(self.status)} (status {self.status})")


c_p = ctypes.c_void_p
c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_f = ctypes.c_float


class LayerDesc(ctypes.Structure):
    """Mirror of ``hc_layer_desc`` (include/hotcold.h)."""

    _fields_ = [
        ("hot", c_p), ("hot_scale", c_p), ("norm_w", c_p), ("cold_records", c_p),
        ("table", c_p), ("fetch_bits", c_p), ("pred_w_down_t", c_p), ("pred_w_up", c_p),
        ("pred_b_up", c_p), ("n_hot", c_i32), ("n_records", c_i32), ("inter", c_i32), ("rank", c_i32),
    ]


_SIGS = {
    "hc_version": (c_i32, []),
    "hc_status_string": (ctypes.c_char_p, [c_i32]),
    "hc_device_sm_count": (c_i32, []),
    "hc_build_record_table": (c_i32, [c_p, c_i64, c_p, c_p, c_i32, c_i32, c_p, c_p, c_p]),
    "hc_map_ids": (c_i32, [c_p, c_i32, c_p, c_p, c_p, c_p, c_p]),
    "hc_cold_gather_dequant": (c_i32, [c_p, c_i64, c_p, c_p, c_i32, c_p, c_i32, c_p, c_i32,
                                       c_p, c_p, c_p, c_p, c_p]),
    "hc_cold_stage": (c_i32, [c_p, c_i64, c_p, c_p, c_i32, c_i32, c_p, c_i64, c_p, c_p]),
    "hc_predictor_workspace_bytes": (c_i64, [c_i32, c_i32, c_i32]),
    "hc_predictor_forward": (c_i32, [c_p, c_i32, c_p, c_f, c_p, c_p, c_p, c_i32, c_i32, c_f, c_p, c_p, c_p,
                                     c_p, c_p, c_p, c_p, c_p, c_p, c_p, c_p]),
    "hc_predictor_forward_static": (c_i32, [c_p, c_i32, c_p, c_f, c_p, c_p, c_p, c_i32, c_i32, c_f, c_p, c_p, c_p,
                                            c_p, c_p, c_p, c_p, c_p, c_p, c_p]),
    "hc_ffn_stack_grid": (c_i32, []),
    "hc_ffn_stack_workspace_bytes": (c_i64, [c_i32, c_i32]),
    "hc_ffn_stack": (c_i32, [c_p, c_i32, c_i32, c_p, c_p, c_i32, c_p, c_p, c_f, c_i32, c_i32, c_f,
                             c_i32, c_p, c_p, c_p, c_p]),
    "hc_tp_buffer_bytes": (c_i64, [c_i32]),
    "hc_ffn_stack_tp": (c_i32, [c_p, c_i32, c_i32, c_p, c_p, c_i32, c_p, c_p, c_f, c_i32, c_i32, c_f,
                                c_i32, c_p, c_p, c_p, c_p, c_p]),
    "hc_tp_alloc": (c_i32, [c_i64, c_p]),
    "hc_tp_free": (c_i32, [c_p]),
    "hc_ipc_get_handle": (c_i32, [c_p, c_p]),
    "hc_ipc_open": (c_i32, [c_p, c_p]),
    "hc_ipc_close": (c_i32, [c_p]),
    "hc_union_cold": (c_i32, [c_p, c_i32, c_i64, c_i32, c_p, c_p, c_p, c_p, c_p]),
    "hc_union_cold_layers": (c_i32, [c_p, c_i32, c_i64, c_i32, c_i64, c_i32, c_p, c_p, c_p, c_i64, c_p, c_p, c_i64,
                                     c_p]),
    "hc_ffn_batch_workspace_bytes": (c_i64, [c_i32]),
    "hc_batch_set_trace": (c_i32, [c_p, c_p]),
    "hc_ffn_batch_layer": (c_i32, [c_p, c_p, c_p, c_i32, c_p, c_p, c_i32, c_p, c_f, c_i32, c_i32, c_p, c_p, c_p]),
    "hc_ffn_batch_layer_partial": (c_i32, [c_p, c_p, c_p, c_i32, c_p, c_p, c_i32, c_p, c_f, c_i32, c_i32, c_p, c_p, c_p,
                                           c_p]),
    "hc_batch_pack_bytes": (c_i64, [c_i32, c_i32]),
    "hc_batch_pack": (c_i32, [c_p, c_p, c_p]),
    "hc_fp8_gemv": (c_i32, [c_p, c_p, c_i64, c_i32, c_p, c_p, c_p]),
    "hc_fp8_gemv_ex": (c_i32, [c_p, c_p, c_i64, c_i32, c_p, c_p, ctypes.c_float, c_p, c_p, c_p]),
    "hc_attn_decode": (c_i32, [c_p, c_p, c_p, c_p, c_p, c_p, c_i32, c_i32, c_i32, c_i32, c_p, c_p, c_p]),
    "hc_xchg_buffer_bytes": (c_i64, [c_i32, c_i64]),
    "hc_xchg_sum": (c_i32, [c_p, c_i64, c_p, c_i64, c_p, c_p, c_p]),
}


class TPDesc(ctypes.Structure):
    """Mirror of hc_tp_desc (include/hotcold.h)."""
    _fields_ = [("size", ctypes.c_int32), ("rank", ctypes.c_int32), ("words_lo", ctypes.c_int32),
                ("words_n", ctypes.c_int32), ("peer_buf", ctypes.c_void_p), ("seq_base", ctypes.c_uint32),
                ("wait_ns", ctypes.c_uint64), ("predict_last", ctypes.c_int32),
                ("io_f16", ctypes.c_int32)]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libhotcold.so is not built ({LIB_PATH}); run hc_build.py (or __graft_entry__.build())")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.hc_version() != ABI_VERSION:
        raise ImportError(f"libhotcold.so ABI {lib.hc_version()} != expected {ABI_VERSION}; rebuild it")
    return lib


lib = _load()


def exported_symbols():
    return sorted(_SIGS)


def status_string(status: int) -> str:
    return lib.hc_status_string(int(status)).decode()


def check(status: int, where: str):
    if status != HC_OK:
        raise HotColdError(where, status)


def ptr(t) -> int | None:
    """Device (or pinned host) address of a tensor; None passes NULL."""
    if t is None:
        return None
    return t.data_ptr()


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("hotcold: this operation runs only on CUDA tensors (no CPU fallback)")


def stream_handle(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def new_status(device) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device)


def read_status(status: torch.Tensor, where: str):
    v = int(status.item())
    if v != 0:
        raise HotColdError(where, v)


def layer_desc_array(descs, device) -> torch.Tensor:
    """Pack a list of LayerDesc into a device byte tensor (hc_layer_desc[])."""
    arr = (LayerDesc * len(descs))(*descs)
    raw = bytes(ctypes.string_at(ctypes.addressof(arr), ctypes.sizeof(arr)))
    host = torch.frombuffer(bytearray(raw), dtype=torch.uint8)
    return host.to(device)
