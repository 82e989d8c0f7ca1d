"""Prefill-block attention on the tensor cores (csrc/attn_prefill.cu) against
the f32 host forward and against the per-row attention kernel it replaces
for prefill blocks (RENG_FLASH_PREFILL=0).

A tile packs a KV group's query heads times 128 / heads-per-group positions
into the MMA's 128 rows, so the shapes cover 2, 3, 4 and 5 heads per group
(tiles of 128, 126, 128 and 125 rows) at head_dim 64 and 128.  Each prompt
runs as one block and, with RENG_PREFILL_ROWS=256, as several 256-row blocks
whose later blocks start mid-tile (the causal mask inside a key tile, keys
of earlier blocks read back from the cache).
"""
import numpy as np
import pytest

from test_decode_gpu import check_rows, cosine, oracle_for, rel_l2

pytestmark = pytest.mark.gpu

SHAPES = [
    # hidden, heads, kv heads, head_dim, prompt
    (256, 4, 2, 64, 300),
    (512, 8, 2, 128, 300),
    (640, 10, 2, 128, 530),
    (576, 9, 3, 64, 270),
]


def _cfg(hidden, nh, nkv, hd):
    from reng.config import LlamaConfig
    return LlamaConfig(hidden_size=hidden, intermediate_size=2 * hidden, num_hidden_layers=2,
                       num_attention_heads=nh, num_key_value_heads=nkv, head_dim_=hd, vocab_size=1024,
                       rms_norm_eps=1e-5, rope_theta=10000.0, tie_word_embeddings=False, model_type="llama")


@pytest.mark.parametrize("rows", [None, 256])
@pytest.mark.parametrize("hidden,nh,nkv,hd,n", SHAPES)
def test_flash_prefill_matches_the_oracle_and_the_per_row_kernel(reng_lib, monkeypatch, hidden, nh, nkv, hd, n,
                                                                 rows):
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = _cfg(hidden, nh, nkv, hd)
    w = random_weights(cfg, seed=70 + hd + nh)
    prompt = prompt_ids(n, cfg.vocab_size, seed=3)
    cap = n + 16

    def run():
        e = Engine(cfg, w, batch=1, capacity=cap)
        _, _, allg = e.prefill(0, prompt, all_logits=True)
        nxt = int(np.argmax(allg[-1]))
        ids = e.decode([nxt], 4)[:, 0]
        e.close()
        return allg, [nxt] + [int(x) for x in ids]

    if rows:
        monkeypatch.setenv("RENG_PREFILL_ROWS", str(rows))
    monkeypatch.delenv("RENG_FLASH_PREFILL", raising=False)
    flash, ids_flash = run()
    monkeypatch.setenv("RENG_FLASH_PREFILL", "0")
    per_row, ids_row = run()
    sin, cos = rope_caches_for(cfg, cap)
    want = oracle_for(cfg, w).forward(prompt, sin, cos)
    check_rows(flash, want, "flash prefill")
    # the two kernels differ only in f32 summation order and the bf16 P
    for i in range(n):
        assert cosine(flash[i], per_row[i]) >= 0.9999, (i, cosine(flash[i], per_row[i]))
    assert rel_l2(flash, per_row.astype(np.float64)) < 0.01


def test_flash_prefill_long_prompt_in_several_blocks(reng_lib):
    """1500 tokens: a 1024-row block, then 476 rows walking 12 key tiles."""
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = _cfg(512, 8, 2, 128)
    w = random_weights(cfg, seed=91)
    prompt = prompt_ids(1500, cfg.vocab_size, seed=5)
    e = Engine(cfg, w, batch=1, capacity=1536)
    _, last, _ = e.prefill(0, prompt, last_logits=True)
    e.close()
    sin, cos = rope_caches_for(cfg, 1536)
    want = oracle_for(cfg, w).forward(prompt, sin, cos, logits_from=1499)[0]
    assert cosine(last, want) >= 0.999 and rel_l2(last, want) < 0.05
