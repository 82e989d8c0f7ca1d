"""Qwen3's per-head q/k RMSNorm on the engine: the q/k/v
launch writes raw q and k (identity rotation), k_qk_norm normalises each
head, applies the gains (the attention scale riding on the q gain) and
rotates; prefill logits and greedy decode against the f32 oracle's q/k-norm
layer (oracle/forward_oracle.c, pinned to transformers' Qwen3ForCausalLM)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_qwen3_qk_norm_matches_the_oracle(reng_lib, oracle_lib):
    import oracle
    from test_decode_gpu import check_greedy, check_rows
    from reng.config import LlamaConfig
    from reng.model import Generator
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = LlamaConfig.from_dict(dict(hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                     num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                                     vocab_size=1024, rms_norm_eps=1e-6, rope_theta=10000.0,
                                     tie_word_embeddings=False, model_type="qwen3"))
    w = random_weights(cfg, seed=17)
    rng = np.random.default_rng(17)
    for lw in w["layers"]:
        lw["qn"] = (1.0 + 0.2 * rng.standard_normal(64)).astype(np.float32)
        lw["kn"] = (1.0 + 0.2 * rng.standard_normal(64)).astype(np.float32)
    orc = oracle.Model.for_config(cfg, w)
    sin, cos = rope_caches_for(cfg, 128)
    ids = prompt_ids(19, cfg.vocab_size, seed=9)
    g = Generator(w, cfg, capacity=128)
    check_rows(g.feed_all(ids), orc.forward(ids, sin, cos), "qwen3 prefill")
    g.reset()
    nxt = g.feed_id(ids)
    out = g.generate(nxt, 12)
    seq = np.concatenate([ids, [nxt], out[:-1]]).astype(np.uint32)
    check_greedy([nxt] + out, orc.forward(seq, sin, cos, logits_from=ids.size - 1))
    g.close()
