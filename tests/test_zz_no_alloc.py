"""The allocation-free predictor entry point, checked against the workspace one.

hc_predictor_forward_static serves callers that cannot allocate device
memory (a process whose allocator is frozen after start-up, an embedded
runtime, a plugin host that owns all allocations): its scratch is a fixed
array inside the library instead of a caller workspace.  This file is named
to run last so that a failure here never hides the other tests' results.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def N():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import hc_native
    return hc_native


def _weights(seed, inter, rank):
    g = torch.Generator(device="cuda").manual_seed(seed)
    wd = torch.randn(rank, 4096, generator=g, device="cuda") * 0.02
    wu = torch.randn(inter, rank, generator=g, device="cuda") * 0.02
    b = torch.randn(inter, generator=g, device="cuda") * 0.02
    return wd, wu, b


def _outputs(batch, inter, dev):
    words = (inter + 31) // 32
    return (torch.empty(batch, words, dtype=torch.int32, device=dev),
            torch.empty(batch, inter, dtype=torch.float32, device=dev),
            torch.empty(inter, dtype=torch.int32, device=dev),
            torch.zeros(1, dtype=torch.int32, device=dev))


def test_static_scratch_matches_workspace_entry_point(N):
    from predictor import logit_threshold
    import splitter
    inter, rank, batch = 14336, 64, 4
    wd, wu, b = _weights(3, inter, rank)
    x = torch.randn(batch, 4096, device="cuda")
    nw = 1.0 + 0.1 * torch.randn(4096, device="cuda")
    fetch = splitter.bits_to_words(torch.rand(inter) < 0.8, inter).cuda()
    thr = logit_threshold(0.5)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    s = N.stream_handle()

    ws = torch.zeros(int(N.lib.hc_predictor_workspace_bytes(batch, rank, inter)), dtype=torch.uint8, device="cuda")
    m0, p0, i0, c0 = _outputs(batch, inter, "cuda")
    N.check(N.lib.hc_predictor_forward(N.ptr(x), batch, N.ptr(nw), 1e-5, N.ptr(wd), N.ptr(wu), N.ptr(b), rank, inter,
                                       thr, N.ptr(m0), N.ptr(p0), None, N.ptr(fetch), None, N.ptr(i0), None,
                                       N.ptr(c0), N.ptr(ws), N.ptr(st), s), "workspace entry point")
    for call in range(2):        # two calls in a row share the static scratch
        m1, p1, i1, c1 = _outputs(batch, inter, "cuda")
        N.check(N.lib.hc_predictor_forward_static(N.ptr(x), batch, N.ptr(nw), 1e-5, N.ptr(wd), N.ptr(wu), N.ptr(b),
                                                  rank, inter, thr, N.ptr(m1), N.ptr(p1), None, N.ptr(fetch), None,
                                                  N.ptr(i1), None, N.ptr(c1), N.ptr(st), s), f"static call {call}")
        torch.cuda.synchronize()
        assert torch.equal(m1, m0), f"mask words differ on call {call}"
        assert torch.allclose(p1, p0, rtol=0, atol=1e-6), f"probabilities differ on call {call}"
        n = int(c0.item())
        assert int(c1.item()) == n and torch.equal(i1[:n], i0[:n]), f"active id list differs on call {call}"
    assert int(st.item()) == 0


def test_static_scratch_rejects_sizes_beyond_its_limit(N):
    inter, rank, batch = 1024, 128, 8        # batch * rank = 1024 > 512
    wd, wu, b = _weights(4, inter, rank)
    x = torch.randn(batch, 4096, device="cuda")
    m, p, i, c = _outputs(batch, inter, "cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    r = N.lib.hc_predictor_forward_static(N.ptr(x), batch, None, 0.0, N.ptr(wd), N.ptr(wu), N.ptr(b), rank, inter,
                                          0.0, N.ptr(m), N.ptr(p), None, None, None, None, None, None, N.ptr(st),
                                          N.stream_handle())
    assert r == N.HC_ERR_UNSUPPORTED
