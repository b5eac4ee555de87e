"""Time one quantized matrix x k-row product on the GPU (the counterpart of
the reference's ``gguf_matmul_bench``).

    python -m inferq_b200.kernel_bench --dtype Q6_K --rows 248320 --cols 2048 --k 4

Weights are seeded random N(0, 0.02) blocks generated on the device; the
input rows are quantized and multiplied through iq_matrix_forward_device.
Prints device time per call (CUDA events) and achieved weight GB/s.

    python -m inferq_b200.kernel_bench --dtype Q8_0 --rows 8192 --cols 2048 --wide 512

times the tensor-core wide product (iq_matrix_forward_wide) over 512 input
rows instead and prints its rate as 2*rows*cols*n operations per second
against the measured dense bf16 GEMM peak.
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
    ap.add_argument("--wide", type=int, default=0, help="input rows for the wide (tensor-core) product")
    args = ap.parse_args()
    dt = {"Q4_K": Q.Q4_K, "Q5_K": Q.Q5_K, "Q6_K": Q.Q6_K, "Q8_0": Q.Q8_0}[args.dtype]
    g = torch.Generator(device="cuda").manual_seed(0)
    w = Q.encode(torch.randn(args.rows, args.cols, device="cuda", generator=g) * 0.02, dt)
    m = _lib.Matrix(dt, w, args.rows, args.cols)
    del w
    L = _lib.lib()
    if args.wide:
        return wide(m, args, g)
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


def wide(m, args, g):
    import json
    from pathlib import Path
    x = torch.randn(args.wide, args.cols, device="cuda", generator=g)
    for _ in range(3):
        y = m.forward_wide(x)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(args.iters):
        m.forward_wide(x)
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / args.iters * 1e3
    tops = 2.0 * args.rows * args.cols * args.wide / us / 1e6
    peaks = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"
    peak = json.loads(peaks.read_text())["bf16_tflops"] if peaks.exists() else 1590.0
    print(f"{args.dtype} {args.rows}x{args.cols} wide n={args.wide}: {us:.1f} us/call (quantize + product), "
          f"{tops:.0f} TOP/s = {tops / peak:.3f} of the measured bf16 GEMM peak {peak:.0f}")
    del y


if __name__ == "__main__":
    main()
