"""The f32 forward oracle against HF transformers (the reference's
tools/oracle method) on the committed golden logits (Llama, Qwen2, Qwen3),
plus its own invariants: causality and prefix consistency (a longer prompt
does not change earlier positions' logits)."""
import os

import numpy as np
import pytest

from conftest import GOLDEN


def load():
    z = np.load(os.path.join(GOLDEN, "forward_golden.npz"))
    return {k: z[k] for k in z.files}


def oracle_model(z, bias, qk_norm=False):
    import oracle
    from reng.config import LlamaConfig
    cfg = LlamaConfig(hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=2, num_key_value_heads=1, head_dim_=64, vocab_size=256,
                      rms_norm_eps=1e-5, rope_theta=10000.0, attention_bias=bias)
    layers = []
    for l in range(2):
        lw = {k: z["l%d_%s" % (l, k)] for k in ("wq", "wk", "wv", "wo", "wg", "wu", "wd", "g1", "g2")}
        if bias:
            lw.update({k: z["l%d_%s" % (l, k)] for k in ("bq", "bk", "bv")})
        if qk_norm:
            lw.update({k: z["l%d_%s" % (l, k)] for k in ("qn", "kn")})
        layers.append(lw)
    width = 64 if qk_norm else 0
    c = dict(hidden=128, inter=256, n_layers=2, n_heads=2, n_kv_heads=1, head_dim=64, vocab=256,
             eps=1e-5, attn_scale=cfg.attention_scale(), has_bias=int(bias), qn_width=width,
             kn_width=width)
    return cfg, oracle.Model(c, layers, z["final_gamma"], z["lm_head"], z["embed"])


@pytest.mark.parametrize("arch,bias,qk_norm", [("llama", False, False), ("qwen2", True, False),
                                               ("qwen3", False, True)])
def test_oracle_matches_transformers(oracle_lib, arch, bias, qk_norm):
    """qwen3: per-head q/k RMSNorm before RoPE, the attention scale on the
    q norm gain instead of wq (the reference's layer_cpu,
    crates/reng-synapse/src/model.rs:2962-3006)."""
    from reng.rope import rope_caches_for
    z = load()
    cfg, m = oracle_model(z, bias, qk_norm)
    sin, cos = rope_caches_for(cfg, 64)
    got = m.forward(z["ids"], sin, cos)
    want = z["logits_" + arch]
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err < 1e-5, err
    assert np.array_equal(got.argmax(-1), want.argmax(-1))
    assert np.max(np.abs(got - want)) < 1e-4


def test_oracle_is_causal_and_prefix_consistent(oracle_lib):
    from reng.rope import rope_caches_for
    z = load()
    cfg, m = oracle_model(z, False)
    sin, cos = rope_caches_for(cfg, 64)
    full = m.forward(z["ids"], sin, cos)
    part = m.forward(z["ids"][:10], sin, cos)
    assert np.allclose(full[:10], part, rtol=0, atol=1e-5)
    tail = m.forward(z["ids"], sin, cos, logits_from=20)
    assert np.allclose(full[20:], tail, rtol=0, atol=1e-6)
