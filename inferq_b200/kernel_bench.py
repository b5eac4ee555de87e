"""Time one quantized matrix x k-row product on the GPU (the counterpart of
the reference's ``gguf_matmul_bench``).

    python -m inferq_b200.kernel_bench --dtype Q6_K --rows 248320 --cols 2048 --k 4

Weights are seeded random N(0, 0.02) blocks generated on the device; the
input rows are quantized and multiplied through iq_matrix_forward_device.
Prints device time per call (CUDA events) and achieved weight GB/s.
"""
from __future__ import annotations

import argparse

import torch

from . import _lib
from . import quants as Q


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--dtype", default="Q6_K", choices=["Q4_K", "Q5_K", "Q6_K", "Q8_0"])
    ap.add_argument("--rows", type=int, default=248320)
    ap.add_argument("--cols", type=int, default=2048)
    ap.add_argument("--k", type=int, default=4)
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    dt = {"Q4_K": Q.Q4_K, "Q5_K": Q.Q5_K, "Q6_K": Q.Q6_K, "Q8_0": Q.Q8_0}[args.dtype]
    g = torch.Generator(device="cuda").manual_seed(0)
    w = Q.encode(torch.randn(args.rows, args.cols, device="cuda", generator=g) * 0.02, dt)
    m = _lib.Matrix(dt, w, args.rows, args.cols)
    del w
    L = _lib.lib()
    x = torch.randn(args.k, args.cols, device="cuda", generator=g)
    y = torch.empty(args.k, args.rows, device="cuda")
    st = torch.cuda.current_stream()
    for _ in range(3):
        _lib.check(L.iq_matrix_forward_device(m._h, x.data_ptr(), args.k, y.data_ptr(), st.cuda_stream))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.iters):
        L.iq_matrix_forward_device(m._h, x.data_ptr(), args.k, y.data_ptr(), st.cuda_stream)
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / args.iters * 1e3
    nbytes = Q.row_bytes(dt, args.cols) * args.rows
    print(f"{args.dtype} {args.rows}x{args.cols} k={args.k}: {us:.1f} us/call (quantize + GEMV), "
          f"{nbytes / us / 1e3:.0f} GB/s of weights")


if __name__ == "__main__":
    main()
