"""A bounded device wait that runs out, on one GPU.

The tensor-parallel stack waits, per layer, for every peer GPU's partial
output (words tagged with the exchange number, stored over NVLink).  Here the
"peer" exchange buffer is a second local allocation whose kernel never runs,
so no tagged word ever reaches this GPU's buffer, and the wait limit is 5 ms:
the first layer boundary's wait expires on every CTA.
The launch must come back on its own with HC_ERR_TIMEOUT in the status word,
leave its workspace counters clean, and the context must stay usable: a
normal launch right after it passes the oracle parity check.  Nothing here
faults or hangs the GPU: every wait in the kernel is bounded and the copies
in flight are drained before the CTAs exit.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

from oracle import hotcold_oracle as O

pytestmark = pytest.mark.gpu


class _LocalPeers:
    """Exchange buffers of a two-GPU group faked on one GPU: rank 0's own
    buffer plus a 'peer' buffer that nothing ever writes to."""

    def __init__(self, N):
        self.N = N
        self.size, self.rank, self.seq = 2, 0, 0
        nbytes = int(N.lib.hc_tp_buffer_bytes(2))
        self.bufs = []
        for _ in range(2):
            b = ctypes.c_void_p()
            N.check(N.lib.hc_tp_alloc(nbytes, ctypes.byref(b)), "hc_tp_alloc")
            self.bufs.append(b.value)
        self.peer_buf = torch.tensor(self.bufs, dtype=torch.int64, device="cuda")

    def close(self):
        for b in self.bufs:
            self.N.lib.hc_tp_free(b)
        self.bufs = []


def test_peer_wait_expires_and_context_stays_usable():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import engine
    import hc_native as N
    import hc_synth
    import splitter
    L, inter = 2, 2048
    syn = hc_synth.make_stack(n_layers=L, inter=inter, hot_frac=0.2, activation="silu", act_on_both=False,
                              seed=41, predictors=False)
    g = torch.Generator().manual_seed(3)
    masks = torch.stack([splitter.bits_to_words((torch.rand(inter, generator=g) < 0.1).numpy(), inter)
                         for _ in range(L)]).cuda()
    x0 = torch.randn(4096, device="cuda", generator=torch.Generator(device="cuda").manual_seed(4))

    peers = _LocalPeers(N)
    try:
        st = engine.FFNStack(syn.store, syn.hot, syn.norms, [None] * L, syn.activation, syn.act_on_both, syn.eps,
                             inter=inter, tp=peers, wait_ns=5_000_000)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        st.forward(x0, masks=masks)
        torch.cuda.synchronize()
        took = time.perf_counter() - t0
        status = int(st.status.item())
        assert status & N.HC_ERR_TIMEOUT, f"status {status}: the peer wait did not report a timeout"
        assert took < 1.0, f"the timed-out launch took {took:.2f} s (limit 5 ms per wait)"
        # the kernel leaves its barrier / claim counters and layer accumulators zeroed for the next launch
        head = st.ws[:256].view(torch.int32)
        assert int(head.count_nonzero()) == 0, "workspace counters left set after the timeout"
        yacc = st.ws[256:256 + 3 * 4096 * 4].view(torch.float32)
        assert int(yacc.count_nonzero()) == 0, "layer accumulators left set after the timeout"
    finally:
        torch.cuda.synchronize()
        peers.close()

    # the context is still usable: a normal launch passes the oracle check layer by layer
    st1 = syn.stack(with_predictors=False)
    hist = torch.empty(L, 4096, device="cuda")
    st1.forward(x0, masks=masks, x_hist=hist)
    torch.cuda.synchronize()
    st1.check()
    ostore = O.ColdStoreOracle(syn.store.image.cpu().numpy().tobytes(), syn.cold_index, {"hidden_dim": 4096})
    xs = [x0.double().cpu().numpy()] + [hist[l].double().cpu().numpy() for l in range(L)]
    for l in range(L):
        ids = np.nonzero(O.mask_from_words(masks[l].cpu().numpy(), inter)
                         & O.mask_from_words(st1.fetch[l].cpu().numpy(), inter))[0]
        hg, hu, hd = (t.double().cpu().numpy() for t in syn.hot[l].decoded())
        ref = O.ffn_layer_from_records(xs[l], syn.norms[l].cpu().numpy(), syn.eps, syn.activation, syn.act_on_both,
                                       (hg, hu, hd), ostore, l, ids.tolist())
        rel = np.linalg.norm((xs[l + 1] - xs[l]) - (ref - xs[l])) / np.linalg.norm(ref - xs[l])
        assert rel < 1e-3, f"layer {l} after the timeout: rel-L2 {rel:.2e}"
