"""Host logic of expert parallelism, on CPU with world_size-2 gloo groups.

* the loader's expert ranges (iq_ep_expert_range, which the loader itself
  calls) partition [0, E) into equal contiguous ranges;
* rank 0's NCCL unique id reaches every rank intact;
* the exchange's exactness: routed slots that are nonzero on their owner
  only, summed over the ranks, equal the owner's values bit for bit (the
  property that keeps expert-parallel results identical to one GPU's).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from inferq_b200 import ep


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, fn, *args):
    port = _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fn, args)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in procs:
        r, res = q.get(timeout=120)
        out[r] = res
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return [out[r] for r in range(world)]


def _worker(rank, world, port, q, fn, args):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q.put((rank, fn(rank, world, *args)))
    finally:
        dist.destroy_process_group()


def _share_id(rank, world):
    return ep.shared_unique_id()


def _exchange(rank, world, seed):
    rng = np.random.default_rng(seed)
    E, slots, H = 16, 12, 64
    experts = rng.integers(0, E, slots)            # the expert of each routed slot
    full = rng.standard_normal((slots, H)).astype(np.float32) * 3
    full[0] = -0.0 * full[0] - 1e-30               # tiny and negative values too
    lo, hi = ep.expert_range(E, rank, world)
    mine = np.where(((experts >= lo) & (experts < hi))[:, None], full, np.float32(0))
    t = torch.from_numpy(mine.copy())
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return full.view(np.uint32), t.numpy().view(np.uint32)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("E", [256, 512])
def test_expert_ranges_partition_the_experts(world, E):
    covered = []
    for r in range(world):
        lo, hi = ep.expert_range(E, r, world)
        assert (lo, hi) == (r * E // world, (r + 1) * E // world)
        covered.extend(range(lo, hi))
    assert covered == list(range(E))
    with pytest.raises(ValueError):
        ep.expert_range(10, 0, 4)
    with pytest.raises(ValueError):
        ep.expert_range(E, world, world)


def test_the_library_refuses_what_does_not_divide():
    import ctypes
    from inferq_b200 import _lib
    L = _lib.lib()
    lo, hi = ctypes.c_int32(), ctypes.c_int32()
    for E, r, w in ((10, 0, 4), (256, 2, 2), (256, -1, 2), (0, 0, 1)):
        assert L.iq_ep_expert_range(ctypes.c_int64(E), r, w, ctypes.byref(lo), ctypes.byref(hi)) != 0


def test_unique_id_reaches_every_rank():
    a, b = _run(2, _share_id)
    assert len(a) == 128 and a == b


@pytest.mark.parametrize("seed", [0, 1])
def test_owner_only_sum_is_exact(seed):
    for full, summed in _run(2, _exchange, seed):
        assert np.array_equal(full, summed)
