"""Decode parity at the benchmark's own shapes against the f32 host forward.

1. Llama-3.1-8B at full depth (32 layers, the bench workload): a 32-layer
   bf16 stack accumulates rounding that a 2-layer model cannot show.  The
   reference's own full-depth gate is `reng-generate --ref` (teacher-forced
   greedy ids under a 0.5-logit near-tie margin,
   crates/reng-model/src/bin/generate.rs:47-59, 156-188); its hardware tests
   bound per-position logits by rel-L2 0.05 (cache_test.rs:437); the north
   star adds last-position cosine >= 0.999.
2. Qwen2.5-32B widths (hidden 5120, 40/8 heads, hd 128,
   q/k/v bias, intermediate 27648, vocab 152064, eps 1e-6, theta 1e6),
   layer-truncated to 2 layers, after a 4096-token prompt: GQA with 5 query
   heads per KV group over a KV-heavy cache (position >= 4096), at batch 1
   and batch 8 (slots alternate between two prompts).
"""
import numpy as np
import pytest

from test_decode_gpu import COS_MIN, REL_L2_MAX, check_greedy, cosine, oracle_for, rel_l2

pytestmark = pytest.mark.gpu


def _device_weights(cfg, seed, layers=None):
    from reng.weights import random_weights
    return random_weights(cfg, seed=seed, device="cuda:0", layers=layers)


@pytest.mark.parametrize("batch", [1, 8])
def test_llama8b_full_depth_matches_the_oracle(reng_lib, batch):
    import torch
    from reng.config import llama31_8b
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    cfg = llama31_8b()
    w = _device_weights(cfg, seed=3)
    cap = 64
    e = Engine(cfg, w, batch=batch, capacity=cap)
    prompts = [prompt_ids(16 + b % 3, cfg.vocab_size, seed=40 + b) for b in range(batch)]
    seeds, last = [], {}
    check = sorted({0, batch - 1})
    for b in range(batch):
        nxt, ll, _ = e.prefill(b, prompts[b], last_logits=b in check)
        seeds.append(nxt)
        last[b] = ll
    ids = e.decode(seeds, 8)
    e.close()
    orc = oracle_for(cfg, w)  # host copy of all 32 layers
    del w
    torch.cuda.empty_cache()
    sin, cos = rope_caches_for(cfg, cap)
    for b in check:
        seq = np.concatenate([prompts[b], [seeds[b]], ids[:-1, b]]).astype(np.uint32)
        want = orc.forward(seq, sin, cos, logits_from=prompts[b].size - 1)
        assert cosine(last[b], want[0]) >= COS_MIN, (b, cosine(last[b], want[0]))
        assert rel_l2(last[b], want[0]) < REL_L2_MAX, (b, rel_l2(last[b], want[0]))
        check_greedy([seeds[b]] + [int(x) for x in ids[:, b]], want)


def test_qwen32b_widths_after_a_4096_token_prompt(reng_lib):
    import torch
    from reng.config import qwen25_32b
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    cfg = qwen25_32b()
    cfg.num_hidden_layers = 2
    w = _device_weights(cfg, seed=8, layers=2)
    n_prompt, steps = 4096, 16
    cap = n_prompt + steps + 16
    prompts = [prompt_ids(n_prompt, cfg.vocab_size, seed=61), prompt_ids(n_prompt, cfg.vocab_size, seed=62)]
    runs = []  # (prompt index, last logits or None, seed, ids)
    e = Engine(cfg, w, batch=1, capacity=cap)
    nxt, ll, _ = e.prefill(0, prompts[0], last_logits=True)
    runs.append((0, ll, nxt, [int(x) for x in e.decode([nxt], steps)[:, 0]]))
    e.close()
    B = 8
    e = Engine(cfg, w, batch=B, capacity=cap)
    seeds, lasts = [], []
    for b in range(B):
        nxt, ll, _ = e.prefill(b, prompts[b % 2], last_logits=b < 2)
        seeds.append(nxt)
        lasts.append(ll)
    ids = e.decode(seeds, steps)
    e.close()
    for b in range(B):
        runs.append((b % 2, lasts[b], seeds[b], [int(x) for x in ids[:, b]]))
    orc = oracle_for(cfg, w)
    del w
    torch.cuda.empty_cache()
    sin, cos = rope_caches_for(cfg, cap)
    cache = {}
    for p, ll, seed, out in runs:
        seq = tuple(int(x) for x in np.concatenate([prompts[p], [seed], out[:-1]]))
        if seq not in cache:  # one f32 forward per distinct sequence (~4k tokens each)
            cache[seq] = orc.forward(np.asarray(seq, np.uint32), sin, cos, logits_from=n_prompt - 1)
        want = cache[seq]
        if ll is not None:
            assert cosine(ll, want[0]) >= COS_MIN, (p, cosine(ll, want[0]))
            assert rel_l2(ll, want[0]) < REL_L2_MAX, (p, rel_l2(ll, want[0]))
        check_greedy([seed] + out, want)
