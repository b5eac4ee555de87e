"""Benchmark of the speculative-verify hot path (BASELINE.json metric).

Workload: Qwen3.6-35B-A3B-shaped random-init Q4_K_M
checkpoint (seeded; weights N(0, 0.02), Zipf-biased routers), context 1024.
One step = one speculative verification pass of k=4 rows (seed + 3 drafts)
with on-device greedy accept, DeltaNet rollback and KV truncation.  Drafts
are the target's own greedy continuation with a seeded 30% of draft tokens
corrupted, which fixes the acceptance rate.

value      committed (accepted + authoritative) tokens per second, all ranks,
           timed with CUDA events on the pass stream (inputs resident)
e2e        the same steps timed on the host clock through the C ABI
           (iq_verify: host tokens in, host result out, per step)
roofline   algorithmic bytes of a verify pass (weights read once, measured
           expert union, KV + DeltaNet state traffic) over the pass time,
           against the measured HBM copy bandwidth
cpu_baseline  the CPU restatement of the reference (oracle/, a port of
           inferq's arithmetic; the Rust reference cannot be built here)
           timed on a bounded sample and scaled to one k=4 pass

Run: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
Under torchrun each rank runs its own replica on its own GPU (weak scaling);
the job value is the sum of committed tokens over the slowest rank's time.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "accepted tok/s (bs=1, MTP+verify) Qwen3.6-35B-A3B Q4_K_M; verify µs at k=4"
K_ROWS = 4
CTX = 1024
CORRUPT = 0.30


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ep", action="store_true",
                    help="with N > 1: one sequence, experts split over the ranks (expert parallelism) "
                         "instead of N independent replicas")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def read_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi samples during the timed region."""

    def __init__(self, index: int):
        self.path = Path(f"/tmp/iq_clocks_{os.getpid()}.csv")
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(index), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait()
        rows = []
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) == 7:
                rows.append(f)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[0]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[3 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(rows[0][1]), "reasons": reasons,
                "samples": len(rows)}


def pass_bytes(cfg, union, ctx: int, k: int) -> float:
    """Algorithmic bytes of one verify pass (every weight byte read once)."""
    from inferq_b200 import quants as Q
    H = cfg.hidden_size
    rb = lambda kind, rows, cols: rows * Q.row_bytes(cfg.dtype(kind), cols)
    nk, nv, dk, dv = (cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_key_head_dim,
                      cfg.linear_value_head_dim)
    conv_dim, vdim = 2 * nk * dk + nv * dv, nv * dv
    nh, nkv, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    E, F, Fs = cfg.num_experts, cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size
    dn = (rb("attn_qkv", conv_dim, H) + rb("attn_gate", vdim, H) + 2 * rb("ssm_ba", nv, H) +
          rb("ssm_out", H, vdim) + 2 * 4 * (nv * dk * dv + conv_dim * (cfg.linear_conv_kernel_dim - 1)) +
          4 * conv_dim * cfg.linear_conv_kernel_dim)
    att = (rb("attn_q", 2 * nh * hd, H) + rb("attn_k", nkv * hd, H) + rb("attn_v", nkv * hd, H) +
           rb("attn_output", H, nh * hd) + 2 * 4 * nkv * hd * (ctx + k))
    expert = rb("exp_gate", F, H) + rb("exp_up", F, H) + rb("exp_down", H, F)
    shared = rb("sh_gate", Fs, H) + rb("sh_up", Fs, H) + rb("sh_down", H, Fs)
    router = 4 * (E + 1) * H
    total = 0.0
    for l in range(cfg.num_hidden_layers):
        total += att if cfg.layer_is_full(l) else dn
        total += router + shared + float(union[l]) * expert
    total += rb("output", cfg.vocab_size, H) + k * Q.row_bytes(cfg.dtype("token_embd"), H)
    return total


def gemv_bytes(cfg, union, k: int) -> float:
    """Weight bytes the quantized GEMV kernel streams in one verify pass."""
    from inferq_b200 import quants as Q
    H = cfg.hidden_size
    rb = lambda kind, rows, cols: rows * Q.row_bytes(cfg.dtype(kind), cols)
    nk, nv, dk, dv = (cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_key_head_dim,
                      cfg.linear_value_head_dim)
    conv_dim, vdim = 2 * nk * dk + nv * dv, nv * dv
    nh, nkv, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    F, Fs = cfg.moe_intermediate_size, cfg.shared_expert_intermediate_size
    dn = rb("attn_qkv", conv_dim, H) + rb("attn_gate", vdim, H) + 2 * rb("ssm_ba", nv, H) + rb("ssm_out", H, vdim)
    att = (rb("attn_q", 2 * nh * hd, H) + rb("attn_k", nkv * hd, H) + rb("attn_v", nkv * hd, H) +
           rb("attn_output", H, nh * hd))
    expert = rb("exp_gate", F, H) + rb("exp_up", F, H) + rb("exp_down", H, F)
    shared = rb("sh_gate", Fs, H) + rb("sh_up", Fs, H) + rb("sh_down", H, Fs)
    total = 0.0
    for l in range(cfg.num_hidden_layers):
        total += att if cfg.layer_is_full(l) else dn
        total += shared + float(union[l]) * expert
    return total + rb("output", cfg.vocab_size, H)


GEMV_STAGES = ("dn.proj", "dn.out", "attn.proj", "attn.out", "moe.gate_up", "moe.down", "head.lm_head")


def build_model(cfg, device, ep_rank=0, ep_world=1):
    from inferq_b200 import synth
    from inferq_b200.model import Model
    if ep_world > 1:
        from inferq_b200 import ep
        return Model(cfg, synth.generate(cfg, seed=0, device=device), ep_rank=ep_rank, ep_world=ep_world,
                     nccl_id=ep.shared_unique_id())
    return Model(cfg, synth.generate(cfg, seed=0, device=device))


def mtp_timing(state, cfg, hidden_row, seed_token, draft_vocab=32768, depth=3, reps=10):
    """Device time of an MTP draft call (depth steps, vocabulary-prefix head)
    and of the catch-up of one committed row; untimed by the main line."""
    import torch
    t = []
    for i in range(reps + 2):
        pos = state.mtp_position
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        state.mtp_draft(seed_token, hidden_row, depth, min(draft_vocab, cfg.vocab_size))
        t1 = time.perf_counter()
        state.mtp_sync(pos, hidden_row, [seed_token], hidden_row[None])
        t2 = time.perf_counter()
        if i >= 2:
            t.append((t1 - t0, t2 - t1))
    d = np.median(np.array(t), axis=0)
    return {"draft_us_per_call": d[0] * 1e6, "depth": depth, "draft_vocab": min(draft_vocab, cfg.vocab_size),
            "sync_us_one_row": d[1] * 1e6, "timing": "host clock around the C-ABI call (synchronizing)"}


def wide_timing(rows=8192, cols=2048, n=512, reps=10):
    """The tensor-core wide product (prefill-shaped: n input rows through one
    projection of the 35B width), Q8_0, Q4_K and Q6_K, timed with CUDA events:
    quantize + expand + product per call, and the rate against the measured
    dense bf16 peak."""
    import torch

    from inferq_b200 import _lib
    from inferq_b200 import quants as Q
    peaks = ROOT / "MEASURED_PEAKS.json"
    bf16 = json.loads(peaks.read_text()).get("bf16_tflops") if peaks.exists() else 1590.0
    out = {"shape": f"{rows}x{cols}, {n} input rows", "kernel": "wide_q80_kernel / wide_q4k_kernel / wide_q6k_kernel "
           "(tcgen05, exact block dots)"}
    for name, dt in (("q8_0", Q.Q8_0), ("q4_k", Q.Q4_K), ("q6_k", Q.Q6_K)):
        g = torch.Generator(device="cuda").manual_seed(5)
        w = Q.encode(torch.randn(rows, cols, device="cuda", generator=g) * 0.02, dt)
        m = _lib.Matrix(dt, w, rows, cols)
        del w
        x = torch.randn(n, cols, device="cuda", generator=g)
        for _ in range(3):
            m.forward_wide(x)
        st = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            m.forward_wide(x)
        e1.record(st)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) / reps * 1e3
        tops = 2.0 * rows * cols * n / us / 1e6
        out[name] = {"us": us, "int_tops": tops, "frac_of_bf16_peak": tops / bf16}
        del m
    return out


def greedy_continuation(model, prompt, n):
    from inferq_b200.model import State
    s = State(model, CTX + n + 16)
    am, _, _ = s.forward(prompt)
    out = [int(am[-1])]
    for _ in range(n):
        a, _, _ = s.forward([out[-1]])
        out.append(int(a[0]))
    return out


def cpu_baseline_sample(cfg_full, budget_s: float = 20.0):
    """Time the oracle on a bounded sample: one row through 4 of the 40
    layers (3 DeltaNet + 1 attention, full widths) and the full LM head,
    scaled to a k=4 verify pass of the 40-layer model."""
    import torch
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    from inferq_b200 import synth
    c = synth.qwen36_35b()
    c.num_hidden_layers = 4
    c.mtp_num_hidden_layers = 0
    tensors = [synth.Tensor(t.name, t.dtype, t.shape, t.data.cpu()) for t in
               synth.generate(c, seed=0, device="cuda" if torch.cuda.is_available() else "cpu")]
    om = oracle.OracleModel(c, tensors)
    st = om.state(64)
    st.forward([1])  # warm-up (first touches of the weights)
    t0 = time.time()
    rows = 0
    while True:
        st.forward([2 + rows], logits=True)
        rows += 1
        if time.time() - t0 > budget_s / 4 or rows >= 4:
            break
    per_row_4l = (time.time() - t0) / rows
    # split per-row time into layers and head with a head-only timing
    t1 = time.time()
    h = np.random.default_rng(0).standard_normal(c.hidden_size).astype(np.float32)
    lm = [t for t in tensors if t.name == "output.weight"][0]
    oracle.qmatvec(lm.dtype, lm.data.numpy(), c.vocab_size, c.hidden_size, h)
    t_head = time.time() - t1
    t_layers4 = max(per_row_4l - t_head, 0.0)
    per_row_full = t_head + t_layers4 * (cfg_full.num_hidden_layers / 4)
    return {"per_row_s": per_row_full, "pass_s": per_row_full * K_ROWS, "cores": os.cpu_count(),
            "sample": f"{rows} row(s) through 4 of 40 layers (full widths) + full LM head, "
                      f"scaled x10 per layer and x{K_ROWS} rows to one k={K_ROWS} pass"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from inferq_b200 import synth
    cfg = synth.qwen36_35b()
    results = [cpu_baseline_sample(cfg, budget_s=10.0) for _ in range(max(1, min(args.steps, 3)))]
    pass_s = float(np.median([r["pass_s"] for r in results]))
    # expected committed tokens per k=4 step with each draft corrupted
    # independently at 30%: 1 + 0.7 + 0.7^2 + 0.7^3
    committed_per_step = sum((1 - CORRUPT) ** i for i in range(K_ROWS))
    v = committed_per_step / pass_s
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": world,
            "steps": len(results), "warmup": 1, "ms_per_step": pass_s * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8xq4/q6 dot, f32 accumulate",
            "data": "synthetic (seeded random-init weights)",
            "config": {"workload": "qwen3.6-35b-a3b q4_k_m verify k=4 ctx=1024, 30% corrupted greedy drafts",
                       "verify_us_k4": pass_s * 1e6},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": results[0]["cores"], "kind": "port",
                             "sample": results[0]["sample"]},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    import torch
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from inferq_b200 import synth
    from inferq_b200.model import State
    cfg = synth.qwen36_35b()
    ep_mode = args.ep and world > 1
    model = build_model(cfg, "cuda", rank if ep_mode else 0, world if ep_mode else 1)
    rng = np.random.default_rng(1234)
    prompt = rng.integers(0, cfg.vocab_size, CTX)
    n_tokens = (args.warmup + args.steps) * K_ROWS + 8
    greedy = greedy_continuation(model, prompt, n_tokens)
    state = State(model, CTX + n_tokens + 16)
    _, _, prompt_hidden = state.forward(prompt, hidden=True)
    state.mtp_sync(0, None, prompt, prompt_hidden)
    corrupt = np.random.default_rng(7)
    out = [greedy[0]]

    def step():
        drafts = [greedy[len(out) + i] if corrupt.random() >= CORRUPT else int(corrupt.integers(cfg.vocab_size))
                  for i in range(K_ROWS - 1)]
        (acc, auth, com), _, _ = state.verify([out[-1]] + drafts)
        out.extend(drafts[:acc])
        out.append(auth)
        return com

    for _ in range(args.warmup):
        step()
    stream = torch.cuda.ExternalStream(state.stream())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    unions = []
    launches0 = state.launch_count()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    t0 = time.perf_counter()
    e0.record(stream)
    committed = 0
    torch.cuda.nvtx.range_push("verify_steps")
    for _ in range(args.steps):
        committed += step()
        unions.append(state.union_sizes())
    torch.cuda.nvtx.range_pop()
    e1.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    clk = clocks.stop()
    dev_s = e0.elapsed_time(e1) / 1e3
    launches = state.launch_count() - launches0
    assert out[:len(out)] == greedy[:len(out)], "speculative output diverged from greedy"
    if world > 1:
        t = torch.tensor([dev_s, wall, committed], device="cuda", dtype=torch.float64)
        mx = t.clone()
        torch.distributed.all_reduce(mx[:2], op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(t[2:], op=torch.distributed.ReduceOp.SUM)
        # replicas: every rank commits its own sequence; EP: all ranks commit the same one
        dev_s, wall, committed_all = float(mx[0]), float(mx[1]), float(t[2]) / (world if ep_mode else 1)
    else:
        committed_all = committed
    # per-stage profile (separate, untimed) for the roofline of the GEMVs
    state.set_profiling(True)
    for _ in range(3):
        step()
    prof = state.profile()
    state.set_profiling(False)
    mtp = None
    if not ep_mode:  # MTP drafting cost at this context (one GPU), after everything timed
        _, _, hrow = state.forward([out[-1]], hidden=True)
        mtp = mtp_timing(state, cfg, hrow[0], int(out[-1]))
    wide = None
    if rank == 0 and not ep_mode:
        try:
            wide = wide_timing()
        except Exception as e:  # reported, never required
            wide = {"failed": str(e)}
    if rank != 0:
        return
    per_seq = 1 if ep_mode else world  # sequences the job ran
    union = np.mean(np.stack(unions), axis=0)
    pos = CTX + len(out)
    alg_bytes = pass_bytes(cfg, union, pos, K_ROWS)
    ms_step = dev_s / args.steps * 1e3
    peak, peak_kind = read_peaks()
    pass_gbs = alg_bytes / (ms_step / 1e3) / 1e9
    # dominant kernel: the quantized GEMV (every projection, expert and the
    # LM head); its launches timed with CUDA events in the per-stage run
    qmv_us = sum(v[1] for k, v in prof.items() if k in GEMV_STAGES) / 3
    qmv_launches = sum(v[0] for k, v in prof.items() if k in GEMV_STAGES) / 3
    g_bytes = gemv_bytes(cfg, union, K_ROWS)
    achieved = g_bytes / (qmv_us / 1e6) / 1e9 if qmv_us else None
    prof_total = sum(v[1] for v in prof.values()) / 3
    traffic = None
    tpath = ROOT / "profiles" / "traffic.json"
    if tpath.exists():  # ncu DRAM bytes / algorithmic bytes of the GEMV launches, times this pass's bytes
        ratio = json.loads(tpath.read_text()).get("qmv_traffic_over_algorithmic")
        traffic = ratio * gemv_bytes(cfg, union, K_ROWS) if ratio else None
    cpu = None
    if not args.no_cpu_baseline:
        try:
            cb = cpu_baseline_sample(cfg)
            cpu = {"value": (committed_all / args.steps / per_seq) / cb["pass_s"], "unit": "tok/s",
                   "cores": cb["cores"], "kind": "port", "sample": cb["sample"]}
        except Exception as e:  # the baseline is reported, never required
            cpu = {"value": None, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
                   "sample": f"failed: {e}"}
    line = {
        "metric": METRIC, "value": committed_all / dev_s, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong" if ep_mode else "weak", "vs_baseline": None, "dtype": "int8xq4/q6 dot, f32 accumulate",
        "data": "synthetic (seeded random-init Q4_K_M weights, Zipf router bias)",
        "config": {"workload": "qwen3.6-35b-a3b q4_k_m verify k=4 ctx=1024, 30% corrupted greedy drafts",
                   "verify_us_k4": ms_step * 1e3, "committed_per_step": committed_all / args.steps / per_seq,
                   "expert_union_mean": float(union.mean()), "pass_bytes": alg_bytes,
                   "l2": "weights (23.6 GB) exceed L2; no flush needed",
                   "parallelism": f"ep{world} (experts split, NCCL sum of routed outputs per MoE layer)"
                   if ep_mode else f"replicas x{world}",
                   "mtp": mtp,
                   "wide": wide,
                   "pass_roofline": {"achieved_gbs": pass_gbs, "frac": pass_gbs / peak,
                                     "scope": "whole verify pass: algorithmic bytes / device-timed pass"}},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak if achieved else None, "traffic": traffic, "peak_kind": peak_kind,
                     "traffic_scope": "DRAM bytes of the pass's GEMV launches (ncu ratio x weight bytes)",
                     "kernel": "qmv_kernel", "scope": "weight bytes of the pass's GEMV launches / their "
                     "event-timed durations (per-stage run, PDL off)",
                     "gemv_bytes_per_pass": g_bytes, "gemv_us_per_pass": qmv_us,
                     "gemv_launches_per_pass": qmv_launches,
                     "share_of_pass": qmv_us / prof_total if prof_total else None},
        "cpu_baseline": cpu,
        "e2e": {"value": committed_all / wall, "unit": "tok/s", "h2d_bytes_per_step": 4 * K_ROWS,
                "d2h_bytes_per_step": 16},
        "gpu_launches": int(launches),
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
