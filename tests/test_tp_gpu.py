"""Tensor-parallel decode on 2 GPUs (skipped with fewer): every rank holds
its shard, the o_proj/down_proj partials are all-reduced inside the captured
step (the fused peer all-reduce over NVLink for decode steps, NCCL for the
prefill blocks; NCCL throughout with RENG_TP_P2P=0), decode steps shard the
LM head by vocabulary and swap argmax keys (the logits entry point runs the
whole head and must agree on every rank), all ranks produce the same ids (the reference's coordinator rule, crates/reng-model/src/bin/tp.rs:
604-675), and those ids follow the f32 host forward of the full model under
teacher forcing (near-tie margin 0.5), with the prompt's last logits within
cosine 0.999 of it.
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


def _cfg(bias, hidden=256):
    from reng.config import LlamaConfig
    return LlamaConfig(hidden_size=hidden, intermediate_size=512, num_hidden_layers=2,
                       num_attention_heads=4, num_key_value_heads=2, head_dim_=64, vocab_size=1024,
                       rms_norm_eps=1e-5, rope_theta=10000.0, attention_bias=bias,
                       model_type="qwen2" if bias else "llama")


def _worker(rank, port, bias, hidden, batch, p2p, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "reciprocating-engine_b200"))
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ["RENG_TP_P2P"] = "1" if p2p else "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from reng.synth import prompt_ids
        from reng.tp import TpGenerator, check_agreement, share_unique_id
        from reng.weights import random_weights
        cfg = _cfg(bias, hidden)
        w = random_weights(cfg, seed=21)
        uid = share_unique_id(dist)
        g = TpGenerator(w, cfg, rank, WORLD, uid, batch=batch, capacity=64, device=rank)
        kind = g.engine.tp_exchange()
        prompt = prompt_ids(13, cfg.vocab_size, seed=2)
        last = g.engine.prefill(0, prompt, last_logits=True)
        for b in range(1, batch):  # the other slots decode the same prompt
            g.engine.prefill(b, prompt)
        nxt = last[0]
        ids = np.array(g.generate([nxt] * batch, 12)).reshape(12, batch)
        check_agreement([nxt] + [int(x) for x in ids.reshape(-1)], dist)
        # one more step through the logits entry point (the whole LM head
        # on every rank, while decode steps shard it over the ranks)
        lg, nx = g.engine.step_logits(ids[-1])
        q.put((rank, {"nxt": nxt, "ids": [int(x) for x in ids[:, 0]], "rows": ids.tolist(), "last": last[1],
                      "kind": kind, "step_logits": lg, "step_next": nx.tolist()}))
        g.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bias,hidden,batch,p2p", [(False, 320, 1, True), (True, 256, 1, True),
                                                   (False, 256, 3, True), (False, 256, 4, True),
                                                   (False, 320, 1, False)])
def test_tensor_parallel_decode_on_two_gpus(reng_lib, bias, hidden, batch, p2p):
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
    ps = [ctx.Process(target=_worker, args=(r, port, bias, hidden, batch, p2p, q)) for r in range(WORLD)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=600) for _ in ps)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert out[0]["rows"] == out[1]["rows"] and out[0]["nxt"] == out[1]["nxt"]
    assert out[0]["kind"] == out[1]["kind"] == (2 if p2p else 1)
    assert np.array_equal(out[0]["step_logits"], out[1]["step_logits"])
    assert out[0]["step_next"] == out[1]["step_next"]
    assert out[0]["step_next"] == [int(x) for x in np.argmax(out[0]["step_logits"], axis=1)]
    cfg = _cfg(bias, hidden)
    w = random_weights(cfg, seed=21)
    prompt = prompt_ids(13, cfg.vocab_size, seed=2)
    seq = np.concatenate([prompt, [out[0]["nxt"]], out[0]["ids"][:-1]]).astype(np.uint32)
    sin, cos = rope_caches_for(cfg, 64)
    want = oracle_for(cfg, w).forward(seq, sin, cos, logits_from=prompt.size - 1)
    assert cosine(out[0]["last"], want[0]) >= 0.999
    check_greedy([out[0]["nxt"]] + out[0]["ids"], want)


def test_peer_exchange_reports_a_missing_peer(reng_lib):
    """The exchange's failure path on one GPU: rank 1 of the group never
    answers, the kernel's bounded waits give up (2 s), the call reports
    RENG_E_TIMEOUT, and the device keeps working (a model decodes after)."""
    from reng._lib import RENG_E_TIMEOUT, lib
    from reng.model import Engine
    from reng.weights import random_weights
    assert lib().reng_tp_peer_wait_check(0) == RENG_E_TIMEOUT
    cfg = _cfg(False)
    e = Engine(cfg, random_weights(cfg, seed=5), batch=1, capacity=32)
    nxt = e.prefill(0, np.arange(5, dtype=np.uint32))[0]
    assert e.decode([nxt], 3).shape == (3, 1)
    e.close()
