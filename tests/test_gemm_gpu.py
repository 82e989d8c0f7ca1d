"""The tcgen05 GEMM (steps of more than 8 rows) against float64 sums of the
same bf16 values, and the model paths that run on it: decode at batch 16 /
64 and prefill blocks of up to 1024 rows against the f32 host forward.

GEMM bar: every output within 1e-4 x sum_k |x_k w_k| of the exact sum (the
products of two bf16 are exact in f32; only the f32 accumulation order
differs, a layout or descriptor mistake gives O(1) errors).
"""
import numpy as np
import pytest

from test_decode_gpu import COS_MIN, REL_L2_MAX, check_greedy, check_rows, cosine, oracle_for, rel_l2, small_cfg

pytestmark = pytest.mark.gpu


def bf16_bits(a):
    from reng.synth import f32_to_bf16_bits
    return f32_to_bf16_bits(np.asarray(a, np.float32))


def bits_to_f64(b):
    return (b.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


# splits: 0 = the engine's plan; s > 0 = a cluster of s CTAs per 128-row
# super-tile adding their partials over shared memory; s < 0 = -s plain CTAs
# adding theirs through global scratch, the last to arrive in split order
@pytest.mark.parametrize("rows,K,M,splits", [
    (128, 64, 16, 1),        # one CTA, one k chunk
    (256, 512, 9, 1),        # M padded to N = 16
    (200, 200, 33, 0),       # ragged rows (16-row tiles, 128-row super-tiles) and K (zero fill past K)
    (384, 1024, 64, 3),      # split K, a cluster of 3 adding over shared memory
    (384, 1024, 24, -3),     # split K, 3 plain CTAs adding through global scratch
    (300, 1000, 8, -5),      # ragged rows and K, 5 plain splits
    (1000, 576, 256, 0),     # N = 256, the widest MMA
    (4096, 4096, 64, 0),     # Llama-8B o_proj widths, automatic splits
    (4096, 14336, 8, 0),     # Llama-8B down_proj at batch 8: plain splits
    (512, 2048, 40, -4),     # plain splits at N = 48
    (128, 4096, 32, 8),      # one super-tile split 8 ways in a cluster
    (8192, 520, 24, 0),      # 64 super-tiles, ragged K: an odd chunk count (units of 2 chunks and of 1)
    (2048, 2048, 256, 0),    # N = 256 with split K
    (256, 1000, 48, 3),      # ragged K with a cluster: per-chunk activation copies
    (1000, 576, 1024, 0),    # four N-tiles of 256 rows, ragged super-tiles
    (384, 1000, 700, 0),     # three N-tiles, the last of 188 rows; ragged K
    (256, 2048, 300, 2),     # two N-tiles, each a cluster of 2 K splits
    (6144, 512, 1024, 0),    # 48 super-tiles x 4 N-tiles: two waves of CTAs
    (6144, 520, 900, 0),     # the same with a ragged last N-tile and ragged K
])
def test_gemm_matches_exact_sums(reng_lib, rows, K, M, splits):
    from reng.gemm import gemm_bf16
    rng = np.random.default_rng(rows * 7 + K + M)
    w = bf16_bits(rng.standard_normal((rows, K)) * 0.05)
    x = bf16_bits(rng.standard_normal((M, K)))
    y, _ = gemm_bf16(w, x, splits=splits)
    wf, xf = bits_to_f64(w), bits_to_f64(x)
    want = xf @ wf.T
    bound = 1e-4 * (np.abs(xf) @ np.abs(wf).T) + 1e-30
    err = np.abs(y.astype(np.float64) - want)
    assert np.all(err <= bound), (float(err.max()), int(np.argmax(err - bound)))


def test_gemm_rejects_bad_shapes(reng_lib):
    from reng._lib import RengError
    from reng.gemm import gemm_bf16
    w = np.zeros((16, 64), np.uint16)
    with pytest.raises(RengError):
        gemm_bf16(w, np.zeros((1025, 64), np.uint16))       # more than 1024 rows
    with pytest.raises(RengError):
        gemm_bf16(np.zeros((16, 60), np.uint16), np.zeros((4, 60), np.uint16))  # K % 8 != 0


@pytest.mark.parametrize("batch", [16, 64])
def test_wide_batch_decode(reng_lib, batch):
    from reng.model import BatchedGenerator
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = small_cfg()
    w = random_weights(cfg, seed=40)
    cap = 64
    g = BatchedGenerator(w, cfg, batch, capacity=cap)
    prompts = [prompt_ids(5 + (b % 7), cfg.vocab_size, seed=200 + b) for b in range(batch)]
    seeds = [g.prefill_id(b, prompts[b]) for b in range(batch)]
    n = 8
    ids = np.array(g.generate(seeds, n)).reshape(n, batch)
    sin, cos = rope_caches_for(cfg, cap)
    orc = oracle_for(cfg, w)
    for b in range(0, batch, max(1, batch // 16)):
        assert g.position(b) == prompts[b].size + n
        seq = np.concatenate([prompts[b], [seeds[b]], ids[:-1, b]]).astype(np.uint32)
        want = orc.forward(seq, sin, cos, logits_from=prompts[b].size - 1)
        check_greedy([seeds[b]] + list(ids[:, b]), want)
    g.close()


def test_wide_batch_step_logits(reng_lib):
    """All 24 rows of one decode step through the GEMM (bias model)."""
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = small_cfg(bias=True)
    w = random_weights(cfg, seed=41)
    B = 24
    e = Engine(cfg, w, batch=B, capacity=48)
    prompts = [prompt_ids(3 + b % 5, cfg.vocab_size, seed=300 + b) for b in range(B)]
    seeds = [e.prefill(b, prompts[b])[0] for b in range(B)]
    lg, nxt = e.step_logits(seeds)
    sin, cos = rope_caches_for(cfg, 48)
    orc = oracle_for(cfg, w)
    for b in range(B):
        seq = np.concatenate([prompts[b], [seeds[b]]]).astype(np.uint32)
        want = orc.forward(seq, sin, cos, logits_from=prompts[b].size)
        check_rows(lg[b:b + 1], want, "step row %d" % b)
        assert int(nxt[b]) == int(np.argmax(lg[b]))
    e.close()


@pytest.mark.parametrize("n", [300, 37, 700, 1100])
def test_long_prefill_in_gemm_blocks(reng_lib, n):
    """Prefill blocks of up to 1024 rows (+ the rest) with every row's
    logits: the GEMMs run N-tiles of 256 activation rows (700 rows: a last
    N-tile of 188; 1100: a full block of four N-tiles, then 76 rows)."""
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = small_cfg(bias=True)
    w = random_weights(cfg, seed=42)
    cap = max(320, n + 16)
    e = Engine(cfg, w, batch=1, capacity=cap)
    prompt = prompt_ids(n, cfg.vocab_size, seed=8)
    nxt, last, allg = e.prefill(0, prompt, last_logits=True, all_logits=True)
    sin, cos = rope_caches_for(cfg, cap)
    want = oracle_for(cfg, w).forward(prompt, sin, cos)
    check_rows(allg, want, "prefill")
    assert np.array_equal(last, allg[-1])
    assert nxt == int(np.argmax(allg[-1]))
    e.close()


def test_prefill_last_row_head_matches_all_rows(reng_lib):
    """The prefill without all_logits runs the LM head on the last row only."""
    from reng.model import Engine
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = small_cfg()
    w = random_weights(cfg, seed=43)
    prompt = prompt_ids(70, cfg.vocab_size, seed=9)
    a = Engine(cfg, w, batch=1, capacity=96)
    b = Engine(cfg, w, batch=1, capacity=96)
    n1, last1, _ = a.prefill(0, prompt, last_logits=True)
    n2, last2, allg = b.prefill(0, prompt, last_logits=True, all_logits=True)
    assert n1 == n2
    assert cosine(last1, last2) > 0.9999 and rel_l2(last1, last2) < 1e-2
    a.close()
    b.close()


def test_llama8b_widths_batch64_two_layers(reng_lib):
    """Llama-3.1-8B widths at batch 64 (the BASELINE batch-64 shape) on a
    layer-truncated model; a few rows checked against the f32 forward."""
    from reng.config import llama31_8b
    from reng.model import BatchedGenerator
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = llama31_8b()
    w = random_weights(cfg, seed=3, layers=2)
    cfg.num_hidden_layers = 2
    B, cap = 64, 32
    g = BatchedGenerator(w, cfg, B, capacity=cap)
    prompts = [prompt_ids(4 + b % 5, cfg.vocab_size, seed=400 + b) for b in range(B)]
    seeds = [g.prefill_id(b, prompts[b]) for b in range(B)]
    n = 4
    ids = np.array(g.generate(seeds, n)).reshape(n, B)
    sin, cos = rope_caches_for(cfg, cap)
    orc = oracle_for(cfg, w)
    for b in (0, 21, 63):
        seq = np.concatenate([prompts[b], [seeds[b]], ids[:-1, b]]).astype(np.uint32)
        want = orc.forward(seq, sin, cos, logits_from=prompts[b].size - 1)
        check_greedy([seeds[b]] + list(ids[:, b]), want)
    g.close()
