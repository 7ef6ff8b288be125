"""GPU parity of the cold store: record table, gather + dequantise, GPU splitter.

Bit-exact against the oracle and against vectors written by the reference
(tests/golden).  INT4 unpacking is integer work: fp32 outputs must equal the
reference's fp32 q*s exactly, bf16 outputs the round-to-nearest-even of it.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import hotcold_oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def mods():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import hc_native
    import splitter
    return hc_native, splitter


def _golden_store(splitter, name="split", **kw):
    d = os.path.join(GOLD, name)
    cfg = json.load(open(os.path.join(d, "split_config.json" if name == "split" else "config.json")))
    return splitter.ColdWeightStore(os.path.join(d, "cold_weights.bin"), os.path.join(d, "cold_index.npy"),
                                    cfg, **kw), cfg


@pytest.mark.parametrize("source", ["device", "pinned"])
def test_read_neurons_matches_reference_golden(mods, source):
    N, S = mods
    store, cfg = _golden_store(S, source=source)
    g = np.load(os.path.join(GOLD, "store_reads.npz"))
    for name in ("l0_all", "l0_mixed", "l1_rev"):
        li = 0 if name.startswith("l0") else 1
        out = store.read_neurons(li, 0, g[f"{name}_ids"].tolist())
        for part, t in zip(("gate", "up", "down"), out):
            ref = g[f"{name}_{part}"]
            assert tuple(t.shape) == ref.shape
            assert t.dtype == torch.float32
            assert np.array_equal(t.cpu().numpy().view(np.uint32), ref.view(np.uint32)), (name, part)
    assert store.read_neurons(0, 0, g["none_ids"].tolist()) is None
    assert store.read_neurons(0, 0, []) is None
    store.check()
    assert (1, 0) not in store._offset_cache or True
    store.read_neurons(1, 0, [0])
    assert (1, 0) in store._offset_cache


def test_read_neurons_unsorted_reference_fixture(mods):
    N, S = mods
    store, cfg = _golden_store(S, "unsorted")
    truth = np.load(os.path.join(GOLD, "unsorted", "truth.npz"))
    keys = {}
    for k in truth.files:
        li, nid, part = k.split("_")
        keys.setdefault((int(li), int(nid)), {})[part] = truth[k]
    for li in (0, 1):
        nids = [nid for (l, nid) in keys if l == li]
        out = store.read_neurons(li, 0, nids)
        for row, nid in enumerate(nids):
            assert np.array_equal(out[0][row].cpu().numpy(), keys[(li, nid)]["gate"])
            assert np.array_equal(out[1][row].cpu().numpy(), keys[(li, nid)]["up"])
            assert np.array_equal(out[2][:, row].cpu().numpy(), keys[(li, nid)]["down"])


def test_bf16_is_rne_of_fp32(mods):
    N, S = mods
    store, cfg = _golden_store(S, out_dtype=torch.bfloat16)
    g = np.load(os.path.join(GOLD, "store_reads.npz"))
    out = store.read_neurons(0, 0, g["l0_all_ids"].tolist())
    for part, t in zip(("gate", "up", "down"), out):
        ref = torch.from_numpy(g[f"l0_all_{part}"]).to(torch.bfloat16)
        assert torch.equal(t.cpu().view(torch.int16), ref.view(torch.int16))


def _synthetic(S, L=3, n=700, seed=0, std=0.02):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    secs, hostsecs = [], []
    for li in range(L):
        nl = n - 37 * li
        nids = torch.randperm(3 * n, generator=gen, device="cuda")[:nl]
        g = torch.randn(nl, 4096, generator=gen, device="cuda") * std
        u = torch.randn(nl, 4096, generator=gen, device="cuda") * std
        d = torch.randn(nl, 4096, generator=gen, device="cuda") * std
        if li == 1:
            g[0].zero_()
            u[1, :128] = 1e3
        secs.append(S.build_records(nids, g, u, d))
        hostsecs.append((nids.cpu().numpy(), g.cpu().numpy(), u.cpu().numpy(), d.cpu().numpy()))
    return secs, hostsecs


def test_gpu_splitter_bytes_equal_oracle_writer(mods):
    N, S = mods
    secs, hostsecs = _synthetic(S, L=2, n=300)
    for recs, (nids, g, u, d) in zip(secs, hostsecs):
        ref = O.build_records(nids, g, u, d)
        assert np.array_equal(recs.cpu().numpy(), ref)
    image, index = S.build_cold_image(secs)
    ref_bytes, ref_index = O.build_cold_file([(len(h[0]), O.build_records(*h)) for h in hostsecs])
    assert np.array_equal(index, ref_index)
    assert image.cpu().numpy().tobytes() == ref_bytes


def test_record_table_and_batched_gather_bit_exact(mods):
    N, S = mods
    secs, hostsecs = _synthetic(S, L=3, n=700)
    image, index = S.build_cold_image(secs)
    cfg = {"hidden_dim": 4096, "intermediate_dim": 2100}
    store = S.ColdWeightStore(image, index, cfg)
    host = image.cpu().numpy().tobytes()
    ostore = O.ColdStoreOracle(host, index, cfg)
    for li in range(3):
        assert np.array_equal(store.table_host[li], ostore.record_index_table(li))
    # batched multi-layer gather, K records per layer, incl. repeats
    K = 257
    gen = torch.Generator().manual_seed(1)
    rec = torch.stack([torch.randint(0, int(index[li, 0, 1]), (K,), generator=gen) for li in range(3)]).int()
    for dt in (torch.float32, torch.bfloat16):
        out = store.gather_layers(range(3), rec.cuda(), out_dtype=dt)
        store.check()
        for li in range(3):
            off, n = (int(v) for v in index[li, 0])
            raw = np.frombuffer(host, np.uint8, count=n * 6400, offset=off + 16).reshape(n, 6400)
            for v, part in enumerate(("gate", "up", "down")):
                r = raw[rec[li].numpy()]
                packed = r[:, 2 + 2048 * v: 2 + 2048 * (v + 1)]
                sc = r[:, 6146 + 64 * v: 6146 + 64 * (v + 1)].copy().view(np.float16).astype(np.float32)
                ref = O.dequantize_int4_rows(packed, sc, 4096)
                got = out[v, li].cpu()
                if dt == torch.float32:
                    assert np.array_equal(got.numpy().view(np.uint32), ref.view(np.uint32)), (li, part)
                else:
                    assert torch.equal(got.view(torch.int16), torch.from_numpy(ref).to(torch.bfloat16).view(torch.int16))


def test_out_of_range_records_flag_and_zero(mods):
    N, S = mods
    secs, _ = _synthetic(S, L=1, n=64)
    image, index = S.build_cold_image(secs)
    store = S.ColdWeightStore(image, index, {"hidden_dim": 4096, "intermediate_dim": 192})
    rec = torch.tensor([[0, 64, -1, 5, 1 << 30]], dtype=torch.int32, device="cuda")
    out = store.gather_layers([0], rec)
    torch.cuda.synchronize()
    assert int(store.status.item()) & N.HC_ERR_RANGE
    assert torch.count_nonzero(out[:, 0, 1]) == 0 and torch.count_nonzero(out[:, 0, 2]) == 0
    assert torch.count_nonzero(out[:, 0, 4]) == 0
    assert torch.count_nonzero(out[:, 0, 0]) > 0 and torch.count_nonzero(out[:, 0, 3]) > 0
    store.status.zero_()
    # device-side count: rows past count stay untouched
    sentinel = torch.full((3, 1, 5, 4096), 7.0, device="cuda")
    cnt = torch.tensor([2], dtype=torch.int32, device="cuda")
    store.gather_layers([0], rec[:, [0, 3, 0, 3, 0]].contiguous(), count=cnt, out=sentinel)
    assert torch.all(sentinel[:, 0, 2:] == 7.0)
    assert not torch.any(sentinel[:, 0, :2] == 7.0)
    store.check()


def test_corrupt_index_is_rejected_on_host(mods):
    N, S = mods
    secs, _ = _synthetic(S, L=1, n=16)
    image, index = S.build_cold_image(secs)
    bad = index.copy()
    bad[0, 0, 1] = 10_000          # n_cold past EOF
    with pytest.raises(ValueError, match="past the end"):
        S.ColdWeightStore(image, bad, {"hidden_dim": 4096, "intermediate_dim": 48})
    bad = index.copy()
    bad[0, 0, 0] = 8               # misaligned section
    with pytest.raises(ValueError, match="aligned"):
        S.ColdWeightStore(image, bad, {"hidden_dim": 4096, "intermediate_dim": 48})
    with pytest.raises(ValueError, match="past the end"):
        S.ColdWeightStore(image[: 16 + 15 * 6400], index, {"hidden_dim": 4096, "intermediate_dim": 48})


def test_device_table_bounds_past_image(mods):
    """The device table builder itself refuses records past the image (status
    bit, entry left absent) when called through the C ABI directly."""
    N, S = mods
    secs, _ = _synthetic(S, L=1, n=16)
    image, index = S.build_cold_image(secs)
    so = torch.tensor([0], dtype=torch.int64, device="cuda")
    nr = torch.tensor([40], dtype=torch.int32, device="cuda")    # 40 records claimed, 16 present
    table = torch.empty(1, 65536, dtype=torch.int32, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    img = image[: 16 + 16 * 6400]
    N.check(N.lib.hc_build_record_table(N.ptr(img), img.numel(), N.ptr(so), N.ptr(nr), 1, 40, N.ptr(table),
                                        N.ptr(st), N.stream_handle()), "table")
    torch.cuda.synchronize()
    assert int(st.item()) & N.HC_ERR_RANGE
    assert int((table >= 0).sum()) == 16


def test_map_ids_order_and_absent(mods):
    N, S = mods
    store, cfg = _golden_store(S)
    ids = torch.tensor([5, 99999, -3, 12, 5, 7, 65535, 3] * 300, dtype=torch.int64, device="cuda")
    rec = torch.empty(ids.numel(), dtype=torch.int32, device="cuda")
    nid = torch.empty_like(rec)
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    N.check(N.lib.hc_map_ids(N.ptr(ids), ids.numel(), N.ptr(store.table[0]), N.ptr(rec), N.ptr(nid), N.ptr(cnt),
                             N.stream_handle()), "map")
    tab = store.table_host[0]
    want = [(int(i), int(tab[i])) for i in ids.cpu().tolist() if 0 <= i < 65536 and tab[i] >= 0]
    c = int(cnt.item())
    assert c == len(want)
    assert list(zip(nid[:c].cpu().tolist(), rec[:c].cpu().tolist())) == want
