"""GPU parity of the fused predictor (predictor.py:55-96, :413-462) and the
ordered cold-id selection (engine.py:274-283).

The mask is compared exactly wherever the exact (float64) logit is further
from the threshold than the fp32 rounding bound of any evaluation order; the
neurons inside that band ("ambiguous") are reported and must be rare.
"""
import os

import numpy as np
import pytest
import torch

from oracle import hotcold_oracle as O

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def P():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import predictor
    return predictor


def test_golden_predictor_file_masks(P):
    p = P.NeuronPredictor.load(os.path.join(GOLD, "predictors", "layer_000_expert_000.pt"), device="cuda")
    g = np.load(os.path.join(GOLD, "predictor.npz"))
    x = torch.from_numpy(g["x"]).cuda()
    m = p.predict_mask(x, 0.5).cpu().numpy()
    wd, wu, b = (t.detach().cpu().numpy() for t in (p.down.weight, p.up.weight, p.up.bias))
    _, amb = O.predictor_mask_banded(g["x"], wd, wu, b, P.logit_threshold(0.5))
    assert np.array_equal(m[~amb], g["mask"][~amb])
    assert amb.sum() <= 1
    m7 = p.predict_mask(x, 0.7).cpu().numpy()
    _, amb7 = O.predictor_mask_banded(g["x"], wd, wu, b, P.logit_threshold(0.7))
    assert np.array_equal(m7[~amb7], g["mask_07"][~amb7])
    probs = p(x).cpu().numpy()
    assert np.abs(probs - g["probs"]).max() < 2e-6
    reg = P.PredictorRegistry(os.path.join(GOLD, "predictors"), device="cuda")
    x16 = x[:4].half()
    rm = reg.predict(0, 0, x16).cpu().numpy()
    _, amb16 = O.predictor_mask_banded(x16.float().cpu().numpy(), wd, wu, b, P.logit_threshold(0.5))
    assert np.array_equal(rm[~amb16], g["reg_mask_fp16_in"][~amb16])
    assert reg.predict(1, 0, x[:1]) is None
    assert reg.vram_usage_mb() > 0


@pytest.mark.parametrize("inter,rank,batch", [(14336, 64, 1), (14336, 64, 3), (1000, 16, 70), (4096, 128, 2)])
def test_masks_probs_vs_exact_logits(P, inter, rank, batch):
    torch.manual_seed(inter + rank + batch)
    p = P.NeuronPredictor(4096, inter, rank).cuda()
    with torch.no_grad():
        for t in (p.down.weight, p.up.weight, p.up.bias):
            t.normal_(0, 0.02)
    x = torch.randn(batch, 4096, device="cuda")
    m = p.predict_mask(x).cpu().numpy()
    wd, wu, b = (t.detach().cpu().numpy() for t in (p.down.weight, p.up.weight, p.up.bias))
    exact, amb = O.predictor_mask_banded(x.cpu().numpy(), wd, wu, b, P.logit_threshold(0.5))
    assert np.array_equal(m[~amb], exact[~amb])      # outside the rigorous rounding band: exact
    assert (m != exact).mean() < 1e-3                # actual flips inside the band are rare
    lg = p.logits(x).cpu().numpy()
    assert np.array_equal(m, lg >= P.logit_threshold(0.5))   # mask == thresholded kernel logits
    ref_lg, bound = O.predictor_logits(x.cpu().numpy(), wd, wu, b)
    assert np.all(np.abs(lg - ref_lg) <= 2 * bound + 1e-9)
    # torch CPU (the reference's own arithmetic) agrees outside the band
    tm = O.predictor_mask_fp32(x.cpu().numpy(), wd, wu, b)
    assert np.array_equal(m[~amb], tm[~amb])


def test_predict_ids_matches_cold_ids_for(P):
    """Ordered, hot-filtered, record-present id list on device."""
    torch.manual_seed(7)
    inter = 14336
    p = P.NeuronPredictor(4096, inter, 64).cuda()
    with torch.no_grad():
        for t in (p.down.weight, p.up.weight, p.up.bias):
            t.normal_(0, 0.02)
    hot = np.sort(np.random.default_rng(0).choice(inter, 2867, replace=False))
    fetchable = np.ones(inter, bool)
    fetchable[hot] = False
    fetchable[::97] = False                           # ids without a record are skipped
    import splitter
    fb = splitter.bits_to_words(fetchable, inter).cuda()
    table = torch.full((65536,), -1, dtype=torch.int32, device="cuda")
    table[:inter] = torch.arange(inter, dtype=torch.int32, device="cuda") * 3
    x = torch.randn(1, 4096, device="cuda")
    nw = 1.0 + 0.1 * torch.randn(4096, device="cuda")
    ids, recs, cnt = p.predict_ids(x, fb, table, norm_w=nw, eps=1e-5)
    c = int(cnt.item())
    wd, wu, b = (t.detach().cpu().numpy() for t in (p.down.weight, p.up.weight, p.up.bias))
    exact, amb = O.predictor_mask_banded(x.cpu().numpy(), wd, wu, b, P.logit_threshold(0.5),
                                         norm_w=nw.cpu().numpy(), eps=1e-5)
    got = ids[:c].cpu().numpy()
    assert np.all(np.diff(got) > 0), "ascending (nonzero order)"
    assert np.array_equal(recs[:c].cpu().numpy(), got * 3)
    want = set(np.nonzero(exact[0] & fetchable)[0].tolist())
    band = set(np.nonzero(amb[0])[0].tolist())
    assert set(got.tolist()) - band == want - band
    # the reference's list semantics on the same mask
    m = p.predict_mask(torch.from_numpy(O.rmsnorm(x.cpu().numpy(), nw.cpu().numpy(), 1e-5)).float().cuda())
    ref_ids = O.cold_ids_for(m[0].cpu().numpy() & fetchable, [], inter)
    assert set(ref_ids) - band == set(got.tolist()) - band


def test_save_load_roundtrip(P, tmp_path):
    p = P.NeuronPredictor(4096, 256, 32).cuda()
    path = str(tmp_path / "layer_003_expert_000.pt")
    p.save(path)
    q = P.NeuronPredictor.load(path, device="cuda")
    x = torch.randn(5, 4096, device="cuda")
    assert torch.equal(p(x), q(x))
    reg = P.PredictorRegistry(str(tmp_path), device="cuda")
    assert (3, 0) in reg.predictors


def test_cpu_tensors_fail_loudly(P):
    p = P.NeuronPredictor(4096, 64, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        p(torch.randn(1, 4096))
