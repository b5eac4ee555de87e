"""Time verify passes of a synthetic 35B-shaped model with a chosen number of
layers (the counterpart of the reference's ``gguf_verify_bench`` at model
level).

    python -m inferq_b200.pass_bench --layers 4 --k 4 --ctx 64 --passes 3

Prints the device time per pass (CUDA events, graph replays) and the
per-stage event profile.  With ``--eager`` every pass runs as separate
launches with per-stage events (the stage profiler), which is the form a
kernel profiler should capture: launch order per pass is embed, then per
layer its projections, mixer, MoE, then the LM head and the accept kernels.
"""
from __future__ import annotations

import argparse

import numpy as np


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--k", type=int, default=4)
    ap.add_argument("--ctx", type=int, default=64)
    ap.add_argument("--passes", type=int, default=3)
    ap.add_argument("--eager", action="store_true", help="stage profiler on (separate launches, events)")
    ap.add_argument("--seed", type=int, default=2)
    args = ap.parse_args()

    import torch

    from . import synth
    from .model import Model, State
    cfg = synth.qwen36_35b()
    cfg.num_hidden_layers = args.layers
    model = Model(cfg, synth.generate(cfg, seed=args.seed, device="cuda"))
    rng = np.random.default_rng(0)
    st = State(model, args.ctx + args.k * (args.passes + 2) + 8)
    am, _, _ = st.forward(rng.integers(0, cfg.vocab_size, args.ctx))
    toks = [int(am[-1])] + [int(t) for t in rng.integers(0, cfg.vocab_size, args.k - 1)]
    st.set_profiling(args.eager)
    st.verify(toks)  # warm-up (and graph capture when not eager)
    stream = torch.cuda.ExternalStream(st.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.passes):
        st.verify(toks)
    e1.record(stream)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / args.passes * 1e3
    print(f"{args.layers} layers, k={args.k}, ctx {args.ctx}: {us:.0f} us per verify pass"
          f"{' (eager, stage events)' if args.eager else ''}")
    if args.eager:
        for name, (n, t) in sorted(st.profile().items(), key=lambda kv: -kv[1][1]):
            print(f"  {name:16s} {n:5d} x  {t / max(n, 1):8.1f} us")


if __name__ == "__main__":
    main()
