"""Tensor-parallel decode on 2 GPUs (skipped with fewer): every rank holds
its shard, the o_proj/down_proj partials are all-reduced over NCCL inside the
captured step, all ranks produce the same ids (the reference's coordinator
rule, crates/reng-model/src/bin/tp.rs:604-675), and those ids follow the f32
host forward of the full model under teacher forcing (near-tie margin 0.5),
with the prompt's last logits within cosine 0.999 of it.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg(bias):
    from reng.config import LlamaConfig
    return LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                       num_attention_heads=4, num_key_value_heads=2, head_dim_=64, vocab_size=1024,
                       rms_norm_eps=1e-5, rope_theta=10000.0, attention_bias=bias,
                       model_type="qwen2" if bias else "llama")


def _worker(rank, port, bias, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "reciprocating-engine_b200"))
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from reng.synth import prompt_ids
        from reng.tp import TpGenerator, check_agreement, share_unique_id
        from reng.weights import random_weights
        cfg = _cfg(bias)
        w = random_weights(cfg, seed=21)
        uid = share_unique_id(dist)
        g = TpGenerator(w, cfg, rank, WORLD, uid, batch=1, capacity=64, device=rank)
        prompt = prompt_ids(13, cfg.vocab_size, seed=2)
        last = g.engine.prefill(0, prompt, last_logits=True)
        nxt = last[0]
        ids = g.generate([nxt], 12)
        check_agreement([nxt] + ids, dist)
        q.put((rank, {"nxt": nxt, "ids": ids, "last": last[1]}))
        g.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bias", [False, True])
def test_tensor_parallel_decode_on_two_gpus(reng_lib, bias):
    import torch
    if torch.cuda.device_count() < WORLD:
        pytest.skip("needs %d GPUs" % WORLD)
    import torch.multiprocessing as mp
    from test_decode_gpu import check_greedy, cosine, oracle_for
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, port, bias, q)) for r in range(WORLD)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=600) for _ in ps)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert out[0]["ids"] == out[1]["ids"] and out[0]["nxt"] == out[1]["nxt"]
    cfg = _cfg(bias)
    w = random_weights(cfg, seed=21)
    prompt = prompt_ids(13, cfg.vocab_size, seed=2)
    seq = np.concatenate([prompt, [out[0]["nxt"]], out[0]["ids"][:-1]]).astype(np.uint32)
    sin, cos = rope_caches_for(cfg, 64)
    want = oracle_for(cfg, w).forward(seq, sin, cos, logits_from=prompt.size - 1)
    assert cosine(out[0]["last"], want[0]) >= 0.999
    check_greedy([out[0]["nxt"]] + out[0]["ids"], want)
