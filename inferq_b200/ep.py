"""Host side of expert parallelism (one process per GPU).

Experts are split into contiguous ranges, rank r keeping
[r*E/world, (r+1)*E/world) (the library's loader uses the same rule);
every other weight is replicated.  The ranks share one NCCL unique id
(created by rank 0 through the library, broadcast by the host's own process
group, gloo or NCCL) and the library builds its communicator from it.  After
each MoE layer the library sums the routed expert outputs over the ranks;
each slot is nonzero on its owner only, so the sum is exact and every rank's
results equal a single GPU's bit for bit.
"""
from __future__ import annotations

import ctypes

from . import _lib


def expert_range(num_experts: int, rank: int, world: int) -> tuple[int, int]:
    """Experts [lo, hi) resident on `rank` of `world`: the loader's own rule
    (iq_ep_expert_range, host only)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"invalid rank {rank} of {world}")
    if num_experts % world:
        raise ValueError(f"{num_experts} experts do not divide over {world} ranks")
    L = _lib.lib()
    L.iq_ep_expert_range.restype = ctypes.c_int
    L.iq_ep_expert_range.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                     ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32)]
    lo, hi = ctypes.c_int32(), ctypes.c_int32()
    _lib.check(L.iq_ep_expert_range(num_experts, rank, world, ctypes.byref(lo), ctypes.byref(hi)))
    return lo.value, hi.value


def unique_id() -> bytes:
    """A fresh 128-byte NCCL unique id (call on one rank only)."""
    L = _lib.lib()
    L.iq_nccl_unique_id.restype = ctypes.c_int
    L.iq_nccl_unique_id.argtypes = [ctypes.c_void_p]
    buf = ctypes.create_string_buffer(128)
    _lib.check(L.iq_nccl_unique_id(buf))
    return buf.raw


def shared_unique_id(group=None) -> bytes:
    """Rank 0's unique id on every rank of the torch.distributed group."""
    import torch.distributed as dist
    obj = [unique_id() if dist.get_rank(group) == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    return obj[0]
