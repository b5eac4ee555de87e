"""Expert parallelism on two GPUs: every rank's logits equal one GPU's, bit
for bit (verify pass, greedy accept, and a plain forward), for a
world-size-2 expert split with the NCCL exchange inside the pass; and the
wide prefill pass under the same split (IQ_WIDE_EP, set in the child
processes only) equal to the one-GPU wide pass."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, wide=False):
    if wide:
        os.environ["IQ_WIDE_EP"] = "1"  # before the library reads it
    import torch.distributed as dist
    from inferq_b200 import ep, synth
    from inferq_b200 import quants as Q
    from inferq_b200.model import Model, State
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = synth.mini_35b()
        if wide:  # every dense matrix of a wide-capable dtype
            cfg.dtypes = dict(cfg.dtypes, attn_output=Q.Q6_K)
        tensors = list(synth.generate(cfg, seed=9))
        nid = ep.shared_unique_id()
        model = Model(cfg, tensors, ep_rank=rank, ep_world=world, nccl_id=nid)
        prompt = np.random.default_rng(1).integers(0, cfg.vocab_size, 130 if wide else 10)
        st = State(model, 256)
        am, lg, _ = st.forward(prompt, logits=True)
        drafts = [int(am[-1]), 5, 17, 3]
        (acc, auth, com), vl, _ = st.verify(drafts, logits=True)
        single = None
        if rank == 0:
            one = Model(cfg, tensors)
            s1 = State(one, 256)
            _, lg1, _ = s1.forward(prompt, logits=True)
            r1, vl1, _ = s1.verify(drafts, logits=True)
            single = (lg1.view(np.uint32), vl1.view(np.uint32), r1)
        q.put((rank, (lg.view(np.uint32), vl.view(np.uint32), (acc, auth, com)), single))
    finally:
        dist.destroy_process_group()


def _run_pair(wide):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, wide)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    single = None
    for _ in procs:
        r, res, s = q.get(timeout=600)
        got[r] = res
        single = s if s is not None else single
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in (0, 1):
        lg, vl, res = got[r]
        assert np.array_equal(lg, single[0]), r
        assert np.array_equal(vl, single[1]), r
        assert res == single[2], r


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_expert_parallel_matches_one_gpu_bitwise():
    _run_pair(wide=False)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_wide_pass_under_expert_parallelism_matches_one_gpu_bitwise():
    """130 prompt rows take the wide pass (512-row chunk, experts grouped per
    expert, only this rank's experts, one NCCL sum of the routed slots per
    MoE layer), then a verify pass continues from its state."""
    _run_pair(wide=True)
