"""Decode parity at the benchmark's own shapes against the f32 host forward.

1. Llama-3.1-8B at full depth (32 layers, the bench workload).  A 32-layer
   bf16 stack accumulates rounding that a 2-layer model cannot show, and on
   this random-init N(0, 0.02) model it shows a lot: any implementation of
   the reference's device rounding (every activation, the residual stream
   and the logits in bf16; model.rs:738-742) drifts from the f32 forward to
   a last-position cosine near 0.9988 and rel-L2 near 0.048, the engine and
   a torch emulation of those rounding points alike (B200: engine 0.99881 /
   0.0488, emulation 0.99883 / 0.0484; at 2 / 8 / 16 layers both are at
   0.99993 / 0.99973 / 0.99949).  The north star's 0.999 is therefore out of
   reach of the reference's own bf16 semantics at this depth, so the bar
   here is: no farther from the f32 forward than the emulation (cosine
   within 5e-4 of it and never below 0.998; rel-L2 within 15% + 0.002 of
   it), the reference's own hardware bar rel-L2 < 0.05 (cache_test.rs:437)
   for the prompt-end logits wherever the emulation itself meets it, and greedy ids under teacher forcing equal to
   the f32 forward's except at near-ties within 0.5 logits (the
   `reng-generate --ref` gate, crates/reng-model/src/bin/generate.rs:47-59,
   156-188).
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


def bf16_emulation(cfg, w, ids, sin, cos):
    """Last-position logits of a torch forward that rounds where the
    reference's device graph rounds (the attention scale folded into a
    bf16 wq; the normalised rows, q / k / v, the attention output, the
    branch outputs, the residual stream, the SwiGLU product and the logits
    in bf16; f32 arithmetic in between), on the GPU.  Llama layers without
    biases."""
    import torch
    dev = w["embed"].device

    def bf(t):
        return t.to(torch.bfloat16).to(torch.float32)

    def f(t):
        return t.view(torch.bfloat16).to(torch.float32)

    h, nh, nkv, hd = cfg.hidden_size, cfg.num_attention_heads, cfg.n_kv_heads(), cfg.head_dim()
    n = len(ids)
    x = f(w["embed"])[torch.as_tensor(np.asarray(ids, np.int64), device=dev)]
    sn = torch.from_numpy(np.ascontiguousarray(sin[:n])).to(dev)
    cs = torch.from_numpy(np.ascontiguousarray(cos[:n])).to(dev)
    eps = cfg.rms_norm_eps

    def rms(v, g):
        return v * torch.rsqrt((v * v).mean(-1, keepdim=True) + eps) * g

    def rope(t):
        half = hd // 2
        return t * cs[:, None, :] + torch.cat([-t[..., half:], t[..., :half]], -1) * sn[:, None, :]

    mask = torch.full((n, n), float("-inf"), device=dev).triu(1)
    with torch.no_grad():
        for lw in w["layers"]:
            assert lw.get("bq") is None
            n1 = bf(rms(x, lw["g1"].float()))
            wq = bf(f(lw["wq"]) * np.float32(cfg.attention_scale()))
            q = bf(rope((n1 @ wq.T).view(n, nh, hd)))
            k = bf(rope((n1 @ f(lw["wk"]).T).view(n, nkv, hd)))
            v = bf((n1 @ f(lw["wv"]).T).view(n, nkv, hd))
            rep = nh // nkv
            p = torch.softmax(torch.einsum("qhd,khd->hqk", q, k.repeat_interleave(rep, 1)) + mask, -1)
            a = bf(torch.einsum("hqk,khd->qhd", p, v.repeat_interleave(rep, 1)).reshape(n, nh * hd))
            x = bf(x + bf(a @ f(lw["wo"]).T))
            n2 = bf(rms(x, lw["g2"].float()))
            g = n2 @ f(lw["wg"]).T
            act = bf(g / (1 + torch.exp(-g)) * (n2 @ f(lw["wu"]).T))
            x = bf(x + bf(act @ f(lw["wd"]).T))
        nf = bf(rms(x[-1:], w["final_gamma"].float()))
        return bf(nf @ f(w["lm_head"]).T)[0].cpu().numpy()


@pytest.mark.parametrize("batch", [1, 8])
def test_llama8b_full_depth_matches_the_oracle(reng_lib, batch):
    import torch
    from reng.config import llama31_8b
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cuda.matmul.allow_bf16_reduced_precision_reduction = False
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
    sin, cos = rope_caches_for(cfg, cap)
    emu = {b: bf16_emulation(cfg, w, prompts[b], sin, cos) for b in check}
    orc = oracle_for(cfg, w)  # host copy of all 32 layers
    del w
    torch.cuda.empty_cache()
    for b in check:
        seq = np.concatenate([prompts[b], [seeds[b]], ids[:-1, b]]).astype(np.uint32)
        want = orc.forward(seq, sin, cos, logits_from=prompts[b].size - 1)
        c_eng, c_emu = cosine(last[b], want[0]), cosine(emu[b], want[0])
        r_eng, r_emu = rel_l2(last[b], want[0]), rel_l2(emu[b], want[0])
        assert c_eng >= 0.998 and c_eng >= c_emu - 5e-4, (b, c_eng, c_emu)
        assert r_eng <= 1.15 * r_emu + 2e-3, (b, r_eng, r_emu)
        # the reference's hardware bar, wherever its own bf16 semantics meet it
        assert r_eng < REL_L2_MAX or r_emu >= REL_L2_MAX, (b, r_eng, r_emu)
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
