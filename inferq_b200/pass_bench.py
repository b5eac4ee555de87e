"""Time verify passes of a synthetic 35B-shaped model with a chosen number of
layers (the counterpart of the reference's ``gguf_verify_bench`` at model
level).

    python -m inferq_b200.pass_bench --layers 4 --k 4 --ctx 64 --passes 3
    python -m inferq_b200.pass_bench --layers 8 --wide 512 --ctx 512 --passes 1 --nvtx

Prints the device time per pass (CUDA events, graph replays) and the
per-stage event profile.  ``--wide ROWS`` times instead the wide prefill pass
(iq_forward of ROWS rows) on the same shapes with every matrix Q8_0 (the
wide pass's dtype set), each pass from the state image of a ``--ctx``-token
prefill.  ``--nvtx`` brackets the timed passes in an NVTX range ("passes"),
so a profiler can capture exactly their launches.  With ``--eager`` every pass runs as separate
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
    ap.add_argument("--wide", type=int, default=0, help="time the wide pass over this many rows instead")
    ap.add_argument("--nvtx", action="store_true", help="NVTX range 'passes' around the timed passes")
    args = ap.parse_args()

    import torch

    from . import synth
    from .model import Model, State
    cfg = synth.qwen36_35b()
    cfg.num_hidden_layers = args.layers
    if args.wide:
        from . import quants as Q
        cfg.dtypes = {"default": Q.Q8_0, "router": Q.F32}
    model = Model(cfg, synth.generate(cfg, seed=args.seed, device="cuda"))
    rng = np.random.default_rng(0)
    stream = None
    if args.wide:
        st = State(model, args.ctx + args.wide + 8)
        st.forward(rng.integers(0, cfg.vocab_size, args.ctx))
        img = st.export_image()
        toks = rng.integers(0, cfg.vocab_size, args.wide)
        st.import_image(img)
        st.forward(toks)  # warm-up
        stream = torch.cuda.ExternalStream(st.stream())
        total = 0.0
        if args.nvtx:
            torch.cuda.nvtx.range_push("passes")
        for _ in range(args.passes):
            st.import_image(img)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            st.forward(toks)
            e1.record(stream)
            torch.cuda.synchronize()
            total += e0.elapsed_time(e1)
        if args.nvtx:
            torch.cuda.nvtx.range_pop()
        us = total / args.passes * 1e3
        print(f"{args.layers} layers Q8_0, wide pass of {args.wide} rows at ctx {args.ctx}: {us:.0f} us "
              f"({args.wide / us * 1e6:.0f} tok/s)")
        return
    st = State(model, args.ctx + args.k * (args.passes + 2) + 8)
    am, _, _ = st.forward(rng.integers(0, cfg.vocab_size, args.ctx))
    toks = [int(am[-1])] + [int(t) for t in rng.integers(0, cfg.vocab_size, args.k - 1)]
    st.set_profiling(args.eager)
    st.verify(toks)  # warm-up (and graph capture when not eager)
    stream = torch.cuda.ExternalStream(st.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if args.nvtx:
        torch.cuda.nvtx.range_push("passes")
    e0.record(stream)
    for _ in range(args.passes):
        st.verify(toks)
    e1.record(stream)
    torch.cuda.synchronize()
    if args.nvtx:
        torch.cuda.nvtx.range_pop()
    us = e0.elapsed_time(e1) / args.passes * 1e3
    print(f"{args.layers} layers, k={args.k}, ctx {args.ctx}: {us:.0f} us per verify pass"
          f"{' (eager, stage events)' if args.eager else ''}")
    if args.eager:
        for name, (n, t) in sorted(st.profile().items(), key=lambda kv: -kv[1][1]):
            print(f"  {name:16s} {n:5d} x  {t / max(n, 1):8.1f} us")


if __name__ == "__main__":
    main()
