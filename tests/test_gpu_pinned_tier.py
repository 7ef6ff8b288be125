"""GPU parity of the cold tier kept in pinned host memory.

The reference keeps cold_weights.bin outside the GPU and reads only the
neurons each layer fetches (ColdWeightStore, splitter.py:307-330, :354-403;
the 8 GB VRAM design of README.md:3-9).  Here ``ColdWeightStore(...,
source="pinned")`` keeps the file image in pinned host memory; before a layer
runs, its fetched records cross the bus into one device staging buffer
(hc_cold_stage) at their own record offsets, and the fused kernels read that
buffer as the layer's section.

* hc_cold_stage copies exactly the listed records (bytes equal to the
  image's), honours a device-side count, leaves other records untouched and
  flags a bad index with HC_ERR_RANGE;
* the batch-1 stack over the pinned store matches the float64 oracle layer by
  layer (rel-L2 <= 1e-3, the stack's bar) with the predictor lookahead, and
  equals the HBM-resident stack on given sets;
* the batched layer kernels over the pinned store match the oracle (2e-3, the
  batched bar).
The engine over a pinned store is covered in test_gpu_engine.py.
"""
import numpy as np
import pytest
import torch

from oracle import hotcold_oracle as O

pytestmark = pytest.mark.gpu
REC = 6400          # record stride (splitter.py:76)
READ = 6352         # bytes of a record the kernels read (id, three INT4 fields, scales, rounded to 16)


@pytest.fixture(scope="module")
def M():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import engine
    import hc_native
    import hc_synth
    import predictor
    import splitter
    return engine, hc_native, hc_synth, splitter, predictor


def _pinned(M, syn):
    splitter = M[3]
    cfg = {"hidden_dim": 4096, "intermediate_dim": syn.inter}
    store = splitter.ColdWeightStore(syn.image, syn.cold_index, cfg, source="pinned")
    assert store.source == "pinned" and not store.image.is_cuda and store.image.is_pinned()
    return store


def _section(syn, l):
    off = int(syn.cold_index[l, 0, 0]) + 16
    return syn.image[off:off + int(syn.cold_index[l, 0, 1]) * REC]


def test_stage_records_copies_listed_records(M):
    engine, N, hc_synth, splitter, predictor = M
    syn = hc_synth.make_stack(n_layers=2, inter=512, hot_frac=0.25, seed=31, predictors=False)
    ps = _pinned(M, syn)
    n = int(syn.cold_index[1, 0, 1])
    src = _section(syn, 1)
    dst = torch.full((ps.stage_bytes(),), 0xAB, dtype=torch.uint8, device="cuda")
    picks = [5, 0, 17, n - 1]
    ps.stage_records(1, torch.tensor(picks, dtype=torch.int32, device="cuda"), dst)
    ps.check()
    for r in picks:
        assert torch.equal(dst[r * REC:r * REC + READ], src[r * REC:r * REC + READ]), f"record {r}"
        assert bool((dst[r * REC + READ:(r + 1) * REC] == 0xAB).all())      # the pad is not read
    assert bool((dst[1 * REC:2 * REC] == 0xAB).all())                        # unlisted records untouched
    # a device-side count limits the list
    dst.fill_(0xAB)
    cnt = torch.tensor([2], dtype=torch.int32, device="cuda")
    ps.stage_records(1, torch.tensor(picks, dtype=torch.int32, device="cuda"), dst, count=cnt)
    ps.check()
    assert torch.equal(dst[5 * REC:5 * REC + READ], src[5 * REC:5 * REC + READ])
    assert torch.equal(dst[0:READ], src[0:READ])
    assert bool((dst[17 * REC:18 * REC] == 0xAB).all())
    # an index outside the section: skipped and flagged, the rest still copied
    dst.fill_(0xAB)
    ps.stage_records(1, torch.tensor([3, n, -1], dtype=torch.int32, device="cuda"), dst)
    with pytest.raises(N.HotColdError) as e:
        ps.check()
    assert e.value.status == N.HC_ERR_RANGE
    ps.status.zero_()
    assert torch.equal(dst[3 * REC:3 * REC + READ], src[3 * REC:3 * REC + READ])
    # argument errors are found on the host, before any device work
    with pytest.raises(N.HotColdError):
        ps.stage_records(1, torch.tensor([0], dtype=torch.int32, device="cuda"), dst[1:])   # misaligned
    with pytest.raises(ValueError):
        ps.stage_records(1, torch.tensor([0], dtype=torch.int64, device="cuda"), dst)


@pytest.mark.parametrize("act,both", [("relu", True), ("silu", False)])
def test_stack_over_pinned_store_lookahead(M, act, both):
    """forward() over a pinned store: layer 0's set from the separate predictor
    launches, then per layer the staging copy and one launch that computes the
    layer and predicts the next layer's set (the lookahead order of the
    whole-stack launch)."""
    engine, N, hc_synth, splitter, predictor = M
    import test_gpu_stack as TS
    syn = hc_synth.make_stack(n_layers=4, inter=1024, hot_frac=0.2, rank=64, activation=act, act_on_both=both,
                              seed=11, norm_std=0.1)
    ps = _pinned(M, syn)
    st = engine.FFNStack(ps, syn.hot, syn.norms, syn.predictors, syn.activation, syn.act_on_both, syn.eps,
                         inter=syn.inter)
    assert st.pinned
    x0 = torch.randn(4096, device="cuda", generator=torch.Generator(device="cuda").manual_seed(3))
    x_hist = torch.empty(4, 4096, device="cuda")
    out = st.forward(x0, x_hist=x_hist)
    st.check()
    ps.check()
    assert torch.equal(out, x_hist[-1])
    masks = st.masks.cpu().numpy()
    assert sum(int(np.count_nonzero(O.mask_from_words(masks[l] & st.fetch[l].cpu().numpy(), 1024)))
               for l in range(4)) > 0
    n_flip = TS._check_stack((engine, hc_synth, predictor, splitter), syn, st, x0, x_hist, masks, True)
    assert n_flip <= 4


def test_stack_over_pinned_store_equals_hbm_store(M):
    """Given sets: the pinned tier and the HBM-resident store give the same
    layer outputs within the kernel's bar.  Two runs of the stack differ by
    about 1e-4: the cold pool's order (which CTA's planner publishes first)
    decides the grouping of records, and the cold down columns are summed in
    fp32 with a bias of ~1000 per element that is removed once per layer."""
    engine, N, hc_synth, splitter, predictor = M
    syn = hc_synth.make_stack(n_layers=3, inter=2048, hot_frac=0.2, rank=64, activation="silu",
                              act_on_both=False, seed=12, predictors=False, norm_std=0.1)
    import test_gpu_stack as TS
    ps = _pinned(M, syn)
    words = hc_synth.bernoulli_words(3, 1, 2048, p=0.3, seed=7)[:, 0]
    x0 = torch.randn(4096, device="cuda", generator=torch.Generator(device="cuda").manual_seed(4))
    h_dev = torch.empty(3, 4096, device="cuda")
    h_pin = torch.empty(3, 4096, device="cuda")
    syn.stack().forward(x0, masks=words, x_hist=h_dev)
    st = engine.FFNStack(ps, syn.hot, syn.norms, [None] * 3, syn.activation, syn.act_on_both, syn.eps,
                         inter=syn.inter)
    st.forward(x0, masks=words, x_hist=h_pin)
    st.check()
    ps.check()
    xs = [x0] + [h_dev[l] for l in range(3)]
    for l in range(3):
        d_dev = (h_dev[l] - xs[l]).double()
        d_pin = (h_pin[l] - xs[l]).double()
        assert (d_pin - d_dev).norm().item() <= TS.TOL * d_dev.norm().item(), f"layer {l}"
    TS._check_stack((engine, hc_synth, predictor, splitter), syn, st, x0, h_pin, words.cpu().numpy(), False)


@pytest.mark.parametrize("B", [5, 40])
def test_batch_stack_over_pinned_store(M, B):
    engine, N, hc_synth, splitter, predictor = M
    import test_gpu_batch as TB
    syn = hc_synth.make_stack(n_layers=2, inter=1024, hot_frac=0.2, rank=64, activation="silu",
                              act_on_both=False, seed=21, norm_std=0.1, predictors=False)
    ps = _pinned(M, syn)
    bst = engine.BatchStack(ps, syn.hot, syn.norms, None, syn.activation, syn.act_on_both, syn.eps,
                            inter=syn.inter, max_batch=64)
    assert bst.pinned and all(p is None for p in bst.packed)          # gathered mode, no packed copies
    words, bits = TB._bernoulli_masks(2, B, syn.inter, 0.1, seed=B)
    x0 = torch.randn(B, 4096, device="cuda", generator=torch.Generator(device="cuda").manual_seed(B))
    x_hist = torch.empty(2, B, 4096, device="cuda")
    out = bst.forward(x0, masks=torch.from_numpy(words), x_hist=x_hist)
    bst.check()
    ps.check()
    assert torch.equal(out, x_hist[-1])
    union = [TB._union_ids(bst, bits[l].numpy(), l) for l in range(2)]
    assert bst.union_counts().tolist() == [len(u) for u in union]
    TB._check_layers(syn, bst, x0, x_hist, union)
