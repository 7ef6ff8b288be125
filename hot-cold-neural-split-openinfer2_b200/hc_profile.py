"""Profiling driver: run one kernel of the path on a seeded synthetic model.

Used as the target of ncu captures (small cases) and launch lists:

    python hc_profile.py --what stack --layers 4 --tokens 3
    python hc_profile.py --what gather --layers 4 --k 4096
    python hc_profile.py --what predictor --tokens 3
    python hc_profile.py --what batch --layers 2 --batch 64 --tokens 3

Everything runs through the public API; nothing is skipped inside a launch.
"""
from __future__ import annotations

import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--what", choices=["stack", "gather", "predictor", "batch"], default="stack")
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--inter", type=int, default=14336)
    ap.add_argument("--tokens", type=int, default=3)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--grid", type=int, default=0)
    ap.add_argument("--batch", type=int, default=64, help="tokens per batched step (--what batch)")
    ap.add_argument("--dense-min-batch", type=int, default=8, help="smallest batch run in the packed dense mode")
    ap.add_argument("--trace", action="store_true", help="print per-phase durations from the device trace")
    args = ap.parse_args()

    import torch
    import hc_synth

    # under torchrun (WORLD_SIZE > 1) the stack runs tensor-parallel, one GPU per rank
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    tp = None
    if world > 1:
        import torch.distributed as dist
        import engine
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("gloo")
        tp = engine.TPGroup()
    syn = hc_synth.make_stack(n_layers=args.layers, inter=args.inter, activation="relu", act_on_both=True, seed=0,
                              predictors=args.what not in ("gather", "batch"))
    if args.what == "stack":
        st = syn.stack(grid=args.grid, tp=tp)
        if tp is not None:
            dist.barrier()
            torch.cuda.synchronize()
        x = torch.randn(args.tokens, 4096, generator=torch.Generator().manual_seed(1)).cuda()   # same on every rank
        trace = torch.zeros(args.layers, st.grid, 40, dtype=torch.int64, device="cuda") if args.trace else None
        for t in range(args.tokens):
            if trace is not None:
                trace.zero_()          # keep the last token's stamps and waits
            if st.pred0_in_kernel():
                st.launch(x[t], 2, None, None, trace)      # layer 0's predictor inside the kernel
            else:
                st.first_mask(x[t])
                st.launch(x[t], False, None, None, trace)
        torch.cuda.synchronize()
        st.check()
        if trace is not None and rank == 0:
            for k, (mean, mx) in st.trace_summary(trace).items():
                print(f"  {k:18s} mean {mean:9.2f} us   max {mx:9.2f} us")
        if tp is not None:
            dist.barrier()
            tp.close()
            dist.destroy_process_group()
    elif args.what == "batch":
        # per-token Bernoulli(0.1) masks unioned per layer; --tokens batched steps
        bst = syn.batch_stack(max_batch=max(args.batch, 1), dense_min_batch=args.dense_min_batch)
        masks = hc_synth.bernoulli_words(args.layers, args.batch, args.inter, 0.1, seed=2)
        x = torch.randn(args.batch, 4096, generator=torch.Generator().manual_seed(1)).cuda()
        for _ in range(args.tokens):
            bst.forward(x, masks=masks)
        torch.cuda.synchronize()
        bst.check()
    elif args.what == "gather":
        store = syn.store
        g = torch.Generator(device="cuda").manual_seed(7)
        rec = torch.randint(0, int(store.n_rec_host.min()), (store.n_layers, args.k), generator=g, device="cuda",
                            dtype=torch.int32)
        out = torch.empty(3, store.n_layers, args.k, 4096, dtype=torch.bfloat16, device="cuda")
        for _ in range(args.tokens):
            store.gather_layers(range(store.n_layers), rec, out=out, out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
        store.check()
    else:
        p = syn.predictors[0]
        x = torch.randn(args.tokens, 4096, device="cuda")
        for t in range(args.tokens):
            p.predict_words(x[t:t + 1], norm_w=syn.norms[0], eps=syn.eps)
        torch.cuda.synchronize()
    print("profile target done")


if __name__ == "__main__":
    main()
