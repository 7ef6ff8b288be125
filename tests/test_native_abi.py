"""CPU checks of the C ABI and the host-side logic (no kernel launches)."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "hotcold.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^HC_API\s+[\w\s\*]+?\b(hc_\w+)\s*\(", src, flags=re.M)))


def test_header_declares_entry_points():
    names = _declared()
    for n in ("hc_cold_gather_dequant", "hc_predictor_forward", "hc_ffn_stack", "hc_build_record_table"):
        assert n in names


def test_library_exports_every_declared_symbol():
    import hc_native as N
    lib = ctypes.CDLL(N.LIB_PATH)
    for n in _declared():
        assert hasattr(lib, n), f"{n} declared in include/hotcold.h but not exported"
    assert set(_declared()) == set(N.exported_symbols()), "ctypes signatures out of sync with the header"


def test_version_and_status_strings():
    import hc_native as N
    assert N.lib.hc_version() == N.ABI_VERSION
    assert N.status_string(0) == "ok"
    assert "range" in N.status_string(N.HC_ERR_RANGE)
    assert "wait" in N.status_string(N.HC_ERR_TIMEOUT)
    assert N.lib.hc_predictor_workspace_bytes(1, 64, 14336) > 0
    assert N.lib.hc_ffn_stack_workspace_bytes(148, 14336) >= 3 * 4096 * 4   # rotating layer accumulators
    assert N.lib.hc_ffn_stack_workspace_bytes(0, 14336) == -1


@pytest.mark.skipif(torch.cuda.is_available(), reason="CPU-only host check")
def test_no_device_is_reported_not_faulted():
    import hc_native as N
    assert N.lib.hc_device_sm_count() == -1


def test_argument_errors_are_reported_without_a_device():
    """Host-side argument validation returns HC_ERR_ARG before any CUDA call."""
    import hc_native as N
    assert N.lib.hc_cold_gather_dequant(None, 0, None, None, 1, None, 4, None, 0, None, None, None, None,
                                        None) == N.HC_ERR_ARG
    assert N.lib.hc_predictor_forward(None, 1, None, 0.0, None, None, None, 64, 100, 0.0, None, None, None,
                                      None, None, None, None, None, None, None, None) == N.HC_ERR_ARG
    assert N.lib.hc_ffn_stack(None, 1, 64, None, None, 0, None, None, 1e-5, 0, 0, 0.0, 0, None, None,
                              None, None) == N.HC_ERR_ARG
    # masks_given is 0 (row 0 given), 1 (all given) or 2 (layer 0 predicted in the kernel); checked
    # before any device work, so fake aligned pointers suffice here
    fake = 256
    assert N.lib.hc_ffn_stack(fake, 1, 64, fake, fake, 3, fake, None, 1e-5, 0, 0, 0.0, 0, fake, fake,
                              None, None) == N.HC_ERR_ARG
    assert N.lib.hc_ffn_stack(fake, 1, 64, fake, fake, -1, fake, None, 1e-5, 0, 0, 0.0, 0, fake, fake,
                              None, None) == N.HC_ERR_ARG
    assert N.lib.hc_map_ids(None, -1, None, None, None, None, None) == N.HC_ERR_ARG
    # the allocation-free predictor checks its arguments before it touches its device array:
    # non-positive sizes and missing pointers are argument errors, as for every other entry point
    for batch, rank in ((0, 64), (-1, 64), (1, 0), (1, -8)):
        assert N.lib.hc_predictor_forward_static(fake, batch, None, 0.0, fake, fake, fake, rank, 1024, 0.0, fake,
                                                 None, None, None, None, None, None, None, None,
                                                 None) == N.HC_ERR_ARG, (batch, rank)
    assert N.lib.hc_predictor_forward_static(None, 1, None, 0.0, fake, fake, fake, 64, 1024, 0.0, fake, None,
                                             None, None, None, None, None, None, None, None) == N.HC_ERR_ARG
    assert N.lib.hc_predictor_forward_static(fake, 1, None, 0.0, fake, fake, fake, 64, 1024, 0.0, None, None,
                                             None, None, None, None, None, None, None, None) == N.HC_ERR_ARG
    # an unaligned input row is rejected too (x + 4 bytes)
    assert N.lib.hc_predictor_forward_static(fake + 4, 1, None, 0.0, fake, fake, fake, 64, 1024, 0.0, fake, None,
                                             None, None, None, None, None, None, None, None) == N.HC_ERR_ARG
    assert N.lib.hc_union_cold(None, 1, 32, 1024, None, None, None, None, None) == N.HC_ERR_ARG
    assert N.lib.hc_union_cold_layers(None, 2, 0, 1, 32, 1024, None, None, None, 0, None, None, 0,
                                      None) == N.HC_ERR_ARG
    assert N.lib.hc_ffn_batch_layer(None, None, None, 4, None, None, 0, None, 1e-5, 0, 0, None, None,
                                    None) == N.HC_ERR_ARG
    assert N.lib.hc_ffn_batch_layer_partial(None, None, None, 4, None, None, 0, None, 1e-5, 0, 0, None, None,
                                            None, None) == N.HC_ERR_ARG
    assert N.lib.hc_batch_pack(None, None, None) == N.HC_ERR_ARG
    # record staging: missing buffers or status, negative sizes, a list without indices, misaligned addresses
    a16, st = 1 << 20, 1 << 21                    # never dereferenced: every call below fails its checks
    assert N.lib.hc_cold_stage(None, 64, a16, None, 1, 1, a16, 64, st, None) == N.HC_ERR_ARG
    assert N.lib.hc_cold_stage(a16, 64, a16, None, 1, 1, None, 64, st, None) == N.HC_ERR_ARG
    assert N.lib.hc_cold_stage(a16, 64, a16, None, 1, 1, a16, 64, None, None) == N.HC_ERR_ARG
    assert N.lib.hc_cold_stage(a16, 64, a16, None, -1, 1, a16, 64, st, None) == N.HC_ERR_ARG
    assert N.lib.hc_cold_stage(a16, -1, a16, None, 1, 1, a16, 64, st, None) == N.HC_ERR_ARG
    assert N.lib.hc_cold_stage(a16, 64, None, None, 1, 1, a16, 64, st, None) == N.HC_ERR_ARG
    assert N.lib.hc_cold_stage(a16 + 8, 64, a16, None, 1, 1, a16, 64, st, None) == N.HC_ERR_ARG
    assert N.lib.hc_cold_stage(a16, 64, a16, None, 1, 1, a16 + 4, 64, st, None) == N.HC_ERR_ARG
    assert N.lib.hc_cold_stage(a16, 64, None, None, 0, 1, a16, 64, st, None) == N.HC_OK     # nothing to copy
    # packed copy: 16 KB per hot gate/up step, 8.5 KB per cold one, 8 / 4.1 KB per down step
    assert N.lib.hc_batch_pack_bytes(2867, 11469) >= (23 * 64 * 16384 + 90 * 64 * 8704 + 32 * 46 * 8192
                                                      + 32 * 180 * 4224)
    assert N.lib.hc_ffn_batch_workspace_bytes(0) == -1
    # workspace grows with the neuron count it must hold (activations, partial sums)
    assert N.lib.hc_ffn_batch_workspace_bytes(14336) > N.lib.hc_ffn_batch_workspace_bytes(1024) > 0


def test_logit_threshold_reproduces_torch_sigmoid_decision():
    from predictor import logit_threshold
    for p in (0.5, 0.7, 0.3, 0.9, 0.01):
        z = logit_threshold(p)
        t = torch.tensor([z], dtype=torch.float32)
        below = torch.nextafter(t, torch.tensor([-float("inf")]))
        assert bool(torch.sigmoid(t)[0] >= p)
        assert not bool(torch.sigmoid(below)[0] >= p)
    assert logit_threshold(0.0) == float("-inf")
    assert logit_threshold(1.5) == float("inf")
    # a dense sweep around the 0.5 threshold agrees with torch exactly
    z = logit_threshold(0.5)
    grid = torch.linspace(-1e-6, 1e-6, 20001, dtype=torch.float32)
    assert torch.equal(grid >= z, torch.sigmoid(grid) >= 0.5)


def test_mask_word_packing_roundtrip():
    from splitter import bits_to_words, words_to_bits
    from oracle import hotcold_oracle as O
    rng = np.random.default_rng(0)
    for n in (1, 31, 32, 40, 14336, 14337):
        m = rng.random(n) < 0.3
        w = bits_to_words(m, n)
        assert w.dtype == torch.int32 and w.numel() == (n + 31) // 32
        assert np.array_equal(words_to_bits(w, n), m)
        assert np.array_equal(O.mask_from_words(w.numpy(), n), m)
        assert np.array_equal(O.words_from_mask(m), w.numpy())


def test_layer_desc_layout_matches_c_struct():
    import hc_native as N
    # 9 pointers + 4 int32 = 88 bytes, pointer-aligned
    assert ctypes.sizeof(N.LayerDesc) == 9 * 8 + 4 * 4
    assert N.LayerDesc.n_hot.offset == 72


def test_tensor_parallel_host_pieces():
    import hc_native as N
    from engine import split_range
    # every unit lands on exactly one rank, in order
    for n, size in ((448, 2), (448, 8), (2867, 8), (5, 8)):
        got = [split_range(n, r, size) for r in range(size)]
        assert got[0][0] == 0 and got[-1][1] == n
        assert all(got[i][1] == got[i + 1][0] for i in range(size - 1))
    # hc_tp_desc layout: 4 int32, a pointer, a uint32, a uint64 wait limit, an int32 flag
    assert ctypes.sizeof(N.TPDesc) == 48 and N.TPDesc.peer_buf.offset == 16 and N.TPDesc.seq_base.offset == 24
    assert N.TPDesc.wait_ns.offset == 32 and N.TPDesc.predict_last.offset == 40 and N.TPDesc.io_f16.offset == 44
    assert N.lib.hc_tp_buffer_bytes(8) == 256 + 3 * 8 * 4096 * 8      # (seq, value) words
    assert N.lib.hc_tp_buffer_bytes(0) == -1 and N.lib.hc_tp_buffer_bytes(9) == -1
