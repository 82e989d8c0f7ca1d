"""Tensor-parallel host logic on CPU: two gloo ranks exchange the NCCL unique
id through the process group, and the rank-agreement check of the
reference's coordinator (crates/reng-model/src/bin/tp.rs:604-675) passes on
equal ids and names the first disagreeing id otherwise."""
import os
import socket

import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "reciprocating-engine_b200"))
    import torch.distributed as dist
    from reng.tp import check_agreement, share_unique_id
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        uid = share_unique_id(dist)
        ok = check_agreement([5, 6, 7], dist)
        res = {"uid": uid.hex(), "ok": list(map(int, ok))}
        try:
            check_agreement([5, 6, 7 + rank], dist)
            res["disagree"] = None
        except RuntimeError as e:
            res["disagree"] = str(e)
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_two_ranks_share_the_unique_id_and_check_agreement(reng_lib):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert out[0]["uid"] == out[1]["uid"] and len(out[0]["uid"]) == 256
    assert out[0]["ok"] == [5, 6, 7]
    assert "rank 1 disagrees with rank 0 at id 2" in out[0]["disagree"]


def test_tp_generator_refuses_an_indivisible_world():
    import sys
    from reng.config import smollm2_135m
    from reng.tp import TpGenerator
    with pytest.raises(ValueError):
        TpGenerator({}, smollm2_135m(), 0, 2, b"\0" * 128)
