"""Tensor-parallel decode on 2, 4 and 8 GPUs (each world skipped when the box
has fewer): every rank holds its shard, the o_proj/down_proj partials are
all-reduced inside the captured step (the fused peer all-reduce over NVLink
for decode steps, NCCL for the prefill blocks; NCCL throughout with
RENG_TP_P2P=0), decode steps shard the LM head by vocabulary and swap argmax
keys (the logits entry point runs the whole head and must agree on every
rank), all ranks produce the same ids (the reference's coordinator rule,
crates/reng-model/src/bin/tp.rs:604-675), and those ids follow the f32 host
forward of the full model under teacher forcing (near-tie margin 0.5), with
the prompt's last logits within cosine 0.999 of it.

FP8 models quantize each rank's shard on its device: q/k/v/gate/up rows are
whole rows (the same scales as one GPU), o_proj/down_proj column windows get
one scale per row and window; the oracle runs on those dequantized shards.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg(world, bias, hidden, shape):
    from reng.config import LlamaConfig, llama31_8b
    if shape == "llama8b":
        c = llama31_8b()
        c.num_hidden_layers = 2
        return c
    # 8 KV heads shard at every world up to 8
    return LlamaConfig(hidden_size=hidden, intermediate_size=1024, num_hidden_layers=2,
                       num_attention_heads=16, num_key_value_heads=8, head_dim_=64, vocab_size=1024,
                       rms_norm_eps=1e-5, rope_theta=10000.0, attention_bias=bias,
                       model_type="qwen2" if bias else "llama")


def _weights(cfg, shape, device):
    from reng.weights import random_weights
    if shape == "llama8b":  # generated on the device (same values on every B200)
        return random_weights(cfg, seed=21, device=device, layers=2)
    return random_weights(cfg, seed=21)


def _worker(rank, world, port, case, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "reciprocating-engine_b200"))
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ["RENG_TP_P2P"] = "1" if case["p2p"] else "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from reng.synth import prompt_ids
        from reng.tp import TpGenerator, check_agreement, share_unique_id
        cfg = _cfg(world, case["bias"], case["hidden"], case["shape"])
        w = _weights(cfg, case["shape"], "cuda:%d" % rank)
        uid = share_unique_id(dist)
        batch = case["batch"]
        g = TpGenerator(w, cfg, rank, world, uid, batch=batch, capacity=64, device=rank,
                        fp8=("e4m3", "pcs") if case["fp8"] else None)
        del w
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


CASES = [
    dict(bias=False, hidden=512, batch=1, p2p=True, fp8=False, shape="small"),
    dict(bias=True, hidden=512, batch=4, p2p=True, fp8=False, shape="small"),
    dict(bias=False, hidden=512, batch=1, p2p=False, fp8=False, shape="small"),
    dict(bias=False, hidden=512, batch=3, p2p=True, fp8=True, shape="small"),
    dict(bias=False, hidden=4096, batch=1, p2p=True, fp8=False, shape="llama8b"),
]


def _case_id(c):
    return "%s-b%d%s%s%s" % (c["shape"], c["batch"], "-bias" if c["bias"] else "",
                             "-p2p" if c["p2p"] else "-nccl", "-fp8" if c["fp8"] else "")


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("case", CASES, ids=_case_id)
def test_tensor_parallel_decode(reng_lib, world, case):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    import torch.multiprocessing as mp
    from test_decode_gpu import check_greedy, cosine, oracle_for
    from test_fp8_decode_gpu import dequantized
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=900) for _ in ps)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(1, world):
        assert out[r]["rows"] == out[0]["rows"] and out[r]["nxt"] == out[0]["nxt"], r
        assert out[r]["kind"] == out[0]["kind"]
        assert np.array_equal(out[r]["step_logits"], out[0]["step_logits"]), r
        assert out[r]["step_next"] == out[0]["step_next"], r
    assert out[0]["kind"] == (2 if case["p2p"] else 1)
    assert out[0]["step_next"] == [int(x) for x in np.argmax(out[0]["step_logits"], axis=1)]
    cfg = _cfg(world, case["bias"], case["hidden"], case["shape"])
    w = _weights(cfg, case["shape"], "cuda:0")
    if case["fp8"]:
        w = dequantized(w, windows=world)
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
    from test_decode_gpu import small_cfg
    assert lib().reng_tp_peer_wait_check(0) == RENG_E_TIMEOUT
    cfg = small_cfg()
    e = Engine(cfg, random_weights(cfg, seed=5), batch=1, capacity=32)
    nxt = e.prefill(0, np.arange(5, dtype=np.uint32))[0]
    assert e.decode([nxt], 3).shape == (3, 1)
    e.close()
