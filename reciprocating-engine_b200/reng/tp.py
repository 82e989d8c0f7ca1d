"""Tensor parallelism on the host side: the reference's TpGenerator
(crates/reng-model/src/lib.rs:3245-3355) and the process-level pieces of
`reng-tp` (crates/reng-model/src/bin/tp.rs).

One process per GPU.  Rank 0 creates the NCCL unique id (the reference
passes its HCCL id through a handshake file, hccl.rs:580-637; here it goes
through the torch.distributed store of the job) and every rank builds its
shard of the model: the library copies rank r's query/KV heads, MLP columns
and the matching o_proj / down_proj column windows from the full weights
(LlamaWeights::shard, lib.rs:1155-1243).  The all-reduces after o_proj and
down_proj run inside the captured decode step.  Every rank computes the same
argmax; `check_agreement` is the coordinator's rule that all ranks produced
the same ids (bin/tp.rs:604-675).
"""
import ctypes as C

import numpy as np

from . import _lib
from .model import Engine


def share_unique_id(dist, group=None):
    """Rank 0's ncclUniqueId, broadcast to every rank (128 bytes)."""
    obj = [None]
    if dist.get_rank(group) == 0 if group is not None else dist.get_rank() == 0:
        buf = (C.c_uint8 * 128)()
        _lib.call("reng_tp_unique_id", buf)
        obj = [bytes(buf)]
    dist.broadcast_object_list(obj, src=0, group=group)
    uid = obj[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise RuntimeError("tensor-parallel handshake: bad unique id")
    return bytes(uid)


def check_agreement(ids, dist, group=None):
    """Raise if the ranks did not produce identical ids (the reference's
    coordinator check); returns the ids otherwise."""
    ids = np.ascontiguousarray(ids, np.uint32).reshape(-1)
    world = dist.get_world_size(group)
    gathered = [None] * world
    dist.all_gather_object(gathered, ids.tolist(), group=group)
    for r, g in enumerate(gathered):
        if g != gathered[0]:
            first = next(i for i, (a, b) in enumerate(zip(g, gathered[0])) if a != b) \
                if len(g) == len(gathered[0]) else min(len(g), len(gathered[0]))
            raise RuntimeError("rank %d disagrees with rank 0 at id %d" % (r, first))
    return ids


class TpGenerator:
    """B sequences decoded tensor-parallel (reng-model TpGenerator)."""

    def __init__(self, w, cfg, rank, world, nccl_id, batch=1, capacity=1024, device=None, fp8=None):
        cfg.shard(rank, world)  # the reference's divisibility rule, as a ValueError
        self.rank, self.world = rank, world
        self.engine = Engine(cfg, w, batch=batch, capacity=capacity,
                             device=rank if device is None else device,
                             tp_rank=rank, tp_world=world, nccl_id=nccl_id, fp8=fp8)

    def batch(self):
        return self.engine.batch

    def position(self, b):
        return self.engine.position(b)

    def reset(self, b=-1):
        self.engine.reset(b)

    def prefill(self, b, ids):
        """Append ids to slot b; returns the greedy next id."""
        return self.engine.prefill(b, ids)[0]

    def generate(self, seeds, n):
        return [int(x) for x in self.engine.decode(seeds, n).reshape(-1)]

    def close(self):
        self.engine.close()
