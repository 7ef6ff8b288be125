"""Host logic of the neuron-sharded (tensor-parallel) paths, on CPU: two
gloo ranks, no GPU.

Each rank takes its share of a layer exactly as the GPU paths do
(``engine.split_range`` over the hot list and over the section's records,
``FFNStack._hot_share``), computes the FFN over its share with the float64
oracle, and the partial outputs are summed with an all-reduce.  The shares
must partition the layer, and the summed partials must equal the whole
layer's FFN (down_proj is linear in the neuron dimension, engine.py:184-188).
"""
import os
import socket

import numpy as np
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "hot-cold-neural-split-openinfer2_b200")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(seed, n_hot, n_rec, H=4096):
    g = torch.Generator().manual_seed(seed)
    hot = [torch.randn(n_hot, H, generator=g) * 0.02 for _ in range(2)] + [torch.randn(H, n_hot, generator=g) * 0.02]
    cold = [torch.randn(n_rec, H, generator=g) * 0.02 for _ in range(2)] + [torch.randn(H, n_rec, generator=g) * 0.02]
    x = torch.randn(3, H, generator=g)
    sel = torch.rand(n_rec, generator=g) < 0.4          # the batch's union over the section's records
    return hot, cold, x, sel


def _worker(rank, world, port, out):
    import sys
    sys.path.insert(0, PKG)
    sys.path.insert(0, REPO)
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    import engine
    from oracle import hotcold_oracle as O
    n_hot, n_rec = 37, 53
    hot, cold, x, sel = _layer(11, n_hot, n_rec)
    hn = engine.HotNeurons(torch.arange(n_hot) * 3, hot[0].to(torch.float8_e4m3fn), hot[1].to(torch.float8_e4m3fn),
                           hot[2].to(torch.float8_e4m3fn), device="cpu")
    share = engine.FFNStack._hot_share(hn, engine._Share(rank, world))
    r0, r1 = engine.split_range(n_rec, rank, world)
    # this rank's hot neurons (decoded FP8) and its union records, float64 oracle
    g_h, u_h, d_h = (t.double().numpy() for t in share.decoded())
    keep = np.nonzero(sel.numpy()[r0:r1])[0] + r0
    gc, uc, dc = cold[0].double().numpy()[keep], cold[1].double().numpy()[keep], cold[2].double().numpy()[:, keep]
    part = O.sparse_ffn(x.double().numpy(), "relu", True, g_h, u_h, d_h, gc, uc, dc)
    t = torch.from_numpy(part).contiguous()
    dist.all_reduce(t)
    ids = [None] * world
    dist.all_gather_object(ids, (share.ids.tolist(), (r0, r1)))
    if rank == 0:
        g_a, u_a, d_a = (t_.double().numpy() for t_ in hn.decoded())
        keep_a = np.nonzero(sel.numpy())[0]
        whole = O.sparse_ffn(x.double().numpy(), "relu", True, g_a, u_a, d_a, cold[0].double().numpy()[keep_a],
                             cold[1].double().numpy()[keep_a], cold[2].double().numpy()[:, keep_a])
        torch.save({"sum": t, "whole": torch.from_numpy(whole), "shares": ids}, out)
    dist.barrier()
    dist.destroy_process_group()


def test_shards_partition_the_layer_and_partials_sum_to_it(tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "r.pt")
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    r = torch.load(out)
    hot_ids = sorted(i for ids, _ in r["shares"] for i in ids)
    assert hot_ids == [3 * k for k in range(37)]                       # every hot neuron exactly once
    ranges = [rng for _, rng in r["shares"]]
    assert ranges[0][0] == 0 and ranges[-1][1] == 53
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))      # records: contiguous, disjoint
    err = (r["sum"] - r["whole"]).norm() / r["whole"].norm()
    assert err < 1e-12, err
