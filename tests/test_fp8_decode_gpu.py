"""FP8-E4M3 weight-only decode against the f32 host forward
on the dequantized weights.

The model quantizes every projection on the device at create time with the
config-0 quantizer (E4M3, per-output-channel absmax scales, backoff 1.0,
Gaudi-range saturation).  The oracle quantizes the same matrices with its
restatement of reng-fp8 (bit-identical codes and scales, see
tests/test_fp8_gpu.py) and runs the f32 forward on `Quantized::dequantize_bf16`
of them (crates/reng-fp8/src/lib.rs:328-345).  Norms, embedding and LM head
stay bf16 (reng-model/src/lib.rs:1058-1065).  Same bars as the bf16 path.
"""
import numpy as np
import pytest

from test_decode_gpu import check_greedy, check_rows, cosine, oracle_for, rel_l2, small_cfg

pytestmark = pytest.mark.gpu


def dequantized(w, windows=1):
    """The weights dict with every projection replaced by its E4M3 per-channel
    round trip in bf16, as the oracle quantizer computes it.  windows > 1:
    o_proj and down_proj are quantized per column window, as each rank of a
    tensor-parallel model quantizes its own window (one scale per row and
    window); the row-split matrices keep whole-row scales."""
    import oracle
    from reng.synth import f32_to_bf16_bits
    from reng.weights import to_host
    h = to_host(w)
    out = {"embed": h["embed"], "lm_head": h["lm_head"], "final_gamma": h["final_gamma"], "layers": []}
    for lw in h["layers"]:
        d = dict(lw)
        for k in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
            parts = []
            for win in np.split(lw[k], windows if k in ("wo", "wd") else 1, axis=1):
                win = np.ascontiguousarray(win)
                rows, cols = win.shape
                codes, scales, _ = oracle.quantize(win, rows, cols, oracle.E4M3, oracle.PCS)
                parts.append(f32_to_bf16_bits(oracle.dequantize(codes, scales, rows, cols, oracle.E4M3))
                             .reshape(rows, cols))
            d[k] = np.concatenate(parts, axis=1)
        out["layers"].append(d)
    return out


@pytest.mark.parametrize("bias", [False, True])
def test_fp8_prefill_and_decode_match_the_dequantized_oracle(reng_lib, bias):
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = small_cfg(bias=bias)
    w = random_weights(cfg, seed=31)
    e = Engine(cfg, w, batch=1, capacity=96, fp8=("e4m3", "pcs"))
    prompt = prompt_ids(19, cfg.vocab_size, seed=4)
    _, _, allg = e.prefill(0, prompt, all_logits=True)
    sin, cos = rope_caches_for(cfg, 96)
    orc = oracle_for(cfg, dequantized(w))
    check_rows(allg, orc.forward(prompt, sin, cos), "fp8 prefill")
    nxt = int(np.argmax(allg[-1]))
    ids = [int(x) for x in e.decode([nxt], 16)[:, 0]]
    seq = np.concatenate([prompt, [nxt], ids[:-1]]).astype(np.uint32)
    check_greedy([nxt] + ids, orc.forward(seq, sin, cos, logits_from=prompt.size - 1))
    e.close()


def test_fp8_batched_decode(reng_lib):
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = small_cfg()
    w = random_weights(cfg, seed=32)
    B = 8
    e = Engine(cfg, w, batch=B, capacity=64, fp8=("e4m3", "pcs"))
    prompts = [prompt_ids(9 + b % 3, cfg.vocab_size, seed=50 + b) for b in range(B)]
    seeds = [e.prefill(b, prompts[b])[0] for b in range(B)]
    ids = e.decode(seeds, 8)
    sin, cos = rope_caches_for(cfg, 64)
    orc = oracle_for(cfg, dequantized(w))
    for b in range(B):
        seq = np.concatenate([prompts[b], [seeds[b]], ids[:-1, b]]).astype(np.uint32)
        check_greedy([seeds[b]] + list(ids[:, b]), orc.forward(seq, sin, cos, logits_from=prompts[b].size - 1))
    e.close()


def test_fp8_llama8b_widths_two_layers(reng_lib):
    from reng.config import llama31_8b
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = llama31_8b()
    w = random_weights(cfg, seed=5, layers=2)
    cfg.num_hidden_layers = 2
    e = Engine(cfg, w, batch=1, capacity=64, fp8=("e4m3", "pcs"))
    prompt = prompt_ids(10, cfg.vocab_size, seed=6)
    nxt, last, _ = e.prefill(0, prompt, last_logits=True)
    ids = [int(x) for x in e.decode([nxt], 5)[:, 0]]
    sin, cos = rope_caches_for(cfg, 64)
    seq = np.concatenate([prompt, [nxt], ids[:-1]]).astype(np.uint32)
    want = oracle_for(cfg, dequantized(w)).forward(seq, sin, cos, logits_from=prompt.size - 1)
    assert cosine(last, want[0]) >= 0.999 and rel_l2(last, want[0]) < 0.05
    check_greedy([nxt] + ids, want)
    e.close()


@pytest.mark.parametrize("bias", [False, True])
def test_fp8_gemm_prefill_block(reng_lib, bias):
    """A 300-row FP8 prefill block runs on the tcgen05 GEMM (two N-tiles):
    the E4M3 codes are copied into shared memory, converted to bf16 there
    by the epilogue warps while the MMAs run, and the per-row scale is
    applied in the epilogue; every row's logits against the f32 forward on
    the dequantized weights."""
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = small_cfg(bias=bias)
    w = random_weights(cfg, seed=33)
    e = Engine(cfg, w, batch=1, capacity=320, fp8=("e4m3", "pcs"))
    prompt = prompt_ids(300, cfg.vocab_size, seed=7)
    _, _, allg = e.prefill(0, prompt, all_logits=True)
    e.close()
    sin, cos = rope_caches_for(cfg, 320)
    check_rows(allg, oracle_for(cfg, dequantized(w)).forward(prompt, sin, cos), "fp8 GEMM prefill")


@pytest.mark.parametrize("B", [16, 24])
def test_fp8_wide_batch_decode(reng_lib, B):
    """FP8 decode above the GEMV's 8 rows: the step's projections run on the
    FP8 GEMM (codes converted in shared memory); staggered prompts, greedy
    ids against the teacher-forced f32 forward on the dequantized weights."""
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = small_cfg()
    w = random_weights(cfg, seed=34)
    e = Engine(cfg, w, batch=B, capacity=64, fp8=("e4m3", "pcs"))
    prompts = [prompt_ids(9 + b % 5, cfg.vocab_size, seed=80 + b) for b in range(B)]
    seeds = [e.prefill(b, prompts[b])[0] for b in range(B)]
    ids = e.decode(seeds, 8)
    e.close()
    sin, cos = rope_caches_for(cfg, 64)
    orc = oracle_for(cfg, dequantized(w))
    for b in range(B):
        seq = np.concatenate([prompts[b], [seeds[b]], ids[:-1, b]]).astype(np.uint32)
        check_greedy([seeds[b]] + list(ids[:, b]), orc.forward(seq, sin, cos, logits_from=prompts[b].size - 1))


def test_fp8_llama8b_widths_gemm_prefill(reng_lib):
    """The FP8 GEMM at Llama-8B widths (2 layers): a 280-token prompt as one
    block, the last row's logits and the greedy continuation."""
    from reng.config import llama31_8b
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = llama31_8b()
    w = random_weights(cfg, seed=8, layers=2)
    cfg.num_hidden_layers = 2
    e = Engine(cfg, w, batch=1, capacity=320, fp8=("e4m3", "pcs"))
    prompt = prompt_ids(280, cfg.vocab_size, seed=9)
    nxt, last, _ = e.prefill(0, prompt, last_logits=True)
    ids = [int(x) for x in e.decode([nxt], 4)[:, 0]]
    e.close()
    sin, cos = rope_caches_for(cfg, 320)
    seq = np.concatenate([prompt, [nxt], ids[:-1]]).astype(np.uint32)
    want = oracle_for(cfg, dequantized(w)).forward(seq, sin, cos, logits_from=prompt.size - 1)
    assert cosine(last, want[0]) >= 0.999 and rel_l2(last, want[0]) < 0.05
    check_greedy([nxt] + ids, want)
