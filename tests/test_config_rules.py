"""The reference's own unit tests of its config and RoPE rules
(crates/reng-model/src/lib.rs:3361-4160), restated against reng.config /
reng.rope with the same known answers: the RoPE scaling types, Phi-3's
legacy names and partial rotation, load-time refusal of incomplete
scalings, the longrope capacity warning, the multimodal Gemma-3 flattening,
Granite's multipliers, the Gemma layer kinds and the trained-context warning."""
import json

import numpy as np
import pytest


def cfg_of(d):
    from reng.config import LlamaConfig
    return LlamaConfig.from_dict(d)


def scaling(d):
    from reng.config import RopeScaling
    keys = RopeScaling.__dataclass_fields__
    r = RopeScaling(**{k: v for k, v in d.items() if k in keys and k != "rope_type"})
    r.rope_type = d.get("rope_type", d.get("type"))
    return r


def test_llama3_scaling_moves_only_low_frequencies():
    """lib.rs:3362-3378: dim 0 untouched, the last pair divided by 8."""
    from reng.rope import rope_caches_partial
    s = scaling(dict(rope_type="llama3", factor=8.0, low_freq_factor=1.0, high_freq_factor=4.0,
                     original_max_position_embeddings=8192))
    sa, _ = rope_caches_partial(2, 128, 128, 500000.0, None, 2)
    sb, _ = rope_caches_partial(2, 128, 128, 500000.0, s, 2)
    assert sa[1, 0] == sb[1, 0]
    assert abs(np.arcsin(sa[1, 63]) / np.arcsin(sb[1, 63]) - 8.0) < 1e-3


def test_linear_scaling_divides_every_frequency():
    """lib.rs:3385-3396 (Gemma-3-4B global layers)."""
    from reng.rope import rope_spec
    a, _ = rope_spec(256, 1e6, None, 16)
    b, af = rope_spec(256, 1e6, scaling(dict(rope_type="linear", factor=8.0)), 16)
    assert af == 1.0 and b[0] == np.float32(0.125)
    assert np.all(np.abs(a / b - 8.0) < 1e-4)


def test_yarn_ramps_between_the_correction_dims():
    """lib.rs:3398-3433 (DeepSeek-V2-Lite): correction range (10, 23), the
    mscale pair cancels, dim 13 at 0.01838, 0.1 ln(40) + 1 without it."""
    from reng.rope import rope_spec
    s = scaling(dict(rope_type="yarn", factor=40, original_max_position_embeddings=4096,
                     beta_fast=32, beta_slow=1, mscale=0.707, mscale_all_dim=0.707))
    a, _ = rope_spec(64, 1e4, None, 16)
    b, af = rope_spec(64, 1e4, s, 16)
    assert af == 1.0
    assert np.array_equal(a[:11], b[:11])
    assert np.all(np.abs(a[23:32] / b[23:32] - 40.0) < 1e-3)
    assert abs(b[13] - 0.01838) < 2e-5
    c, af2 = rope_spec(64, 1e4, scaling(dict(rope_type="yarn", factor=40,
                                               original_max_position_embeddings=4096)), 16)
    assert abs(af2 - 1.3688885) < 1e-5 and np.array_equal(c, b)


def test_longrope_picks_the_factors_by_length_and_scales_the_tables():
    """lib.rs:3435-3475 (Phi-3.5-mini shape): short factors up to the
    pretraining length, long past it, attention factor sqrt(1 + 5/12)."""
    from reng.rope import rope_caches_partial, rope_spec
    short = [1.0 + i / 48.0 for i in range(48)]
    s = scaling(dict(type="longrope", short_factor=short, long_factor=[2.0] * 48,
                     original_max_position_embeddings=4096, max_position_embeddings=131072))
    assert s.rope_type == "longrope"
    base, _ = rope_spec(96, 1e4, None, 4096)
    af = np.sqrt(np.float32(17.0) / np.float32(12.0))
    for n in (1, 300, 4096):
        inv, a = rope_spec(96, 1e4, s, n)
        assert abs(a - af) < 1e-6
        assert np.all(np.abs(base / np.float32(short) - inv) < 1e-7), n
    for n in (4097, 4500):
        inv, a = rope_spec(96, 1e4, s, n)
        assert abs(a - af) < 1e-6 and np.all(np.abs(base / 2.0 - inv) < 1e-7)
    sin, cos = rope_caches_partial(2, 96, 96, 1e4, s, 4097)
    assert abs(cos[0, 0] - af) < 1e-6 and sin[0, 0] == 0.0
    assert abs(sin[1, 0] - np.sin(np.float32(0.5)) * af) < 1e-6
    s.attention_factor = 1.0
    assert rope_spec(96, 1e4, s, 8)[1] == 1.0


def phi_config(factor="0.75", n=48, heads=24, kv=8, typ="longrope", **extra):
    d = {"model_type": "phi3", "hidden_size": 3072, "intermediate_size": 8192,
         "num_hidden_layers": 32, "num_attention_heads": heads, "num_key_value_heads": kv,
         "rms_norm_eps": 1e-5, "vocab_size": 200064, "partial_rotary_factor": float(factor),
         "max_position_embeddings": 131072, "original_max_position_embeddings": 4096,
         "rope_scaling": {"type": typ, "short_factor": [1.0] * n, "long_factor": [1.0] * n}}
    d.update(extra)
    return d


def test_phi3_config_lengths_and_legacy_type_names():
    """lib.rs:3481-3520: "su" means longrope, lengths come from the top
    level, Phi-4-mini rotates 96 of 128 dims, bad widths are refused."""
    c = cfg_of(phi_config(factor="1.0", heads=32, kv=32, typ="su"))
    s = c.rope_scaling
    assert s.rope_type == "longrope" and s.original_max_position_embeddings == 4096
    assert s.max_position_embeddings == 131072 and c.weight_prefix is None and c.rotary_dim() == 96
    c = cfg_of(phi_config())
    assert (c.head_dim(), c.rotary_dim()) == (128, 96)
    with pytest.raises(ValueError):
        cfg_of(phi_config(factor="0.2"))          # 25 rotated dims: no whole pair count
    with pytest.raises(ValueError, match="rotary pairs"):
        cfg_of(phi_config(factor="1.0"))          # 48 factors for 64 rotary pairs


def llama_with(sc):
    return {"model_type": "llama", "hidden_size": 4096, "intermediate_size": 11008,
            "num_hidden_layers": 2, "num_attention_heads": 32, "rms_norm_eps": 1e-5,
            "vocab_size": 32000, "rope_scaling": sc}


def test_a_scaling_without_its_parameters_is_refused_at_load():
    """lib.rs:3533-3582."""
    from reng.rope import rope_caches_for
    for sc in ({"rope_type": "linear"}, {"rope_type": "yarn"},
               {"rope_type": "llama3", "factor": 8.0},
               {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0},
               {"rope_type": "longrope", "original_max_position_embeddings": 4096}):
        with pytest.raises(ValueError, match=r"rope_scaling\."):
            cfg_of(llama_with(sc))
    for sc in ({"rope_type": "linear", "factor": 8.0},
               {"rope_type": "yarn", "factor": 40.0, "original_max_position_embeddings": 4096},
               {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                "original_max_position_embeddings": 8192}):
        assert rope_caches_for(cfg_of(llama_with(sc)), 4)[1].shape == (4, 128)
    c = cfg_of(llama_with({"rope_type": "dynamic", "factor": 8.0}))   # ignored, not refused
    assert rope_caches_for(c, 2)[1][0, 0] == 1.0


def test_a_cache_capacity_past_the_pretraining_length_is_reported():
    """lib.rs:3584-3611."""
    from reng.rope import rope_caches_for
    d = phi_config(factor="1.0", heads=32, kv=32)
    d["rope_scaling"]["long_factor"] = [2.0] * 48
    c = cfg_of(d)
    assert c.longrope_capacity_warning(1024) is None and c.longrope_capacity_warning(4096) is None
    msg = c.longrope_capacity_warning(8192)
    assert "8192" in msg and "4096" in msg
    assert abs(rope_caches_for(c, 4096)[1][1, 0] / rope_caches_for(c, 8192)[1][1, 0] - 1.0) > 1e-3
    ll = cfg_of(llama_with({"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                            "high_freq_factor": 4.0, "original_max_position_embeddings": 8192}))
    assert ll.longrope_capacity_warning(1 << 20) is None


def test_multimodal_gemma3_config_flattens_to_its_text_config():
    """lib.rs:3972-4011 (google/gemma-3-4b-pt's config shape)."""
    from reng.rope import rope_caches_for, rope_local_caches_for
    c = cfg_of({"architectures": ["Gemma3ForConditionalGeneration"], "model_type": "gemma3",
                "text_config": {"hidden_size": 2560, "intermediate_size": 10240,
                                "model_type": "gemma3_text", "num_hidden_layers": 34,
                                "rope_scaling": {"factor": 8.0, "rope_type": "linear"},
                                "sliding_window": 1024},
                "vision_config": {"hidden_size": 1152, "model_type": "siglip_vision_model"}})
    assert c.weight_prefix == "language_model.model." and c.model_type == "gemma3_text"
    assert c.is_gemma() and c.tied()
    assert (c.hidden_size, c.num_hidden_layers) == (2560, 34)
    assert (c.num_attention_heads, c.n_kv_heads(), c.head_dim()) == (8, 4, 256)
    assert (c.vocab_size, c.rope_theta, c.rope_local_base_freq) == (262208, 1e6, 1e4)
    assert c.rms_norm_eps == 1e-6 and c.activation() == "gelu_tanh"
    assert c.attention_scale() == 0.0625 and c.max_position_embeddings == 131072
    assert [li for li in range(34) if not c.sliding(li)] == [5, 11, 17, 23, 29]
    assert c.layer_window(0) == 1024 and c.layer_window(5) is None
    # the linear factor lands on the global table only
    _, cos = rope_caches_for(c, 4)
    _, cos_l = rope_local_caches_for(c, 4)
    assert abs(cos[1, 0] - np.cos(np.float32(0.125))) < 1e-6
    assert abs(cos_l[1, 0] - np.cos(np.float32(1.0))) < 1e-6
    with pytest.raises(ValueError):
        cfg_of({"model_type": "gemma3"})


def test_granite_multipliers_parse_and_default():
    """lib.rs:4014-4036."""
    base = {"hidden_size": 64, "intermediate_size": 128, "num_hidden_layers": 1,
            "num_attention_heads": 4, "rms_norm_eps": 1e-5, "vocab_size": 16}
    ll = cfg_of(base)
    for k in ("embedding_multiplier", "attention_multiplier", "residual_multiplier", "logits_scaling"):
        assert ll.raw.get(k) is None
    assert not ll.raw.get("mlp_bias") and ll.attention_scale() == 0.25
    g = cfg_of(dict(base, embedding_multiplier=12.0, attention_multiplier=0.015625,
                    residual_multiplier=0.22, logits_scaling=8.0, mlp_bias=False,
                    attention_bias=False, rope_scaling=None))
    assert g.embed_scale() == 12.0 and g.attention_scale() == 0.015625
    assert g.raw["residual_multiplier"] == 0.22 and g.raw["logits_scaling"] == 8.0
    assert g.rope_scaling is None


def test_gemma_layer_kinds_tables_and_defaults():
    """lib.rs:4038-4130: Gemma-3-270m's explicit layer_types, Gemma-3-1B's
    pattern, Gemma-2's alternation and softcaps, the Llama defaults."""
    from reng.rope import rope_caches_for, rope_local_caches_for
    base = {"hidden_size": 640, "intermediate_size": 2048, "num_attention_heads": 4,
            "num_key_value_heads": 1, "head_dim": 256, "rms_norm_eps": 1e-6, "vocab_size": 262144,
            "rope_theta": 1000000.0, "rope_local_base_freq": 10000.0, "sliding_window": 512,
            "query_pre_attn_scalar": 256, "hidden_activation": "gelu_pytorch_tanh"}
    types = ["full_attention" if (i + 1) % 6 == 0 else "sliding_attention" for i in range(18)]
    g270 = cfg_of(dict(base, model_type="gemma3_text", num_hidden_layers=18,
                       _sliding_window_pattern=6, layer_types=types))
    assert g270.is_gemma() and g270.tied() and g270.activation() == "gelu_tanh"
    assert g270.attention_scale() == 0.0625
    assert abs(g270.embed_scale() - np.sqrt(np.float32(640))) < 1e-6
    assert [li for li in range(18) if not g270.sliding(li)] == [5, 11, 17]
    assert g270.layer_window(0) == 512 and g270.layer_window(5) is None
    assert g270.local_rope(0) and not g270.local_rope(5)
    g1b = cfg_of(dict(base, model_type="gemma3_text", num_hidden_layers=26, sliding_window_pattern=6))
    assert [li for li in range(26) if not g1b.sliding(li)] == [5, 11, 17, 23]
    sin, _ = rope_caches_for(g1b, 16)
    sin_l, _ = rope_local_caches_for(g1b, 16)
    assert sin_l.shape == (16, 256)
    assert abs(np.arcsin(sin_l[13, 1]) - np.arcsin(sin[13, 1]) - 0.43) < 0.02
    g2 = cfg_of(dict(base, model_type="gemma2", num_hidden_layers=26))
    assert [li for li in range(6) if g2.sliding(li)] == [0, 2, 4]
    assert not g2.local_rope(0) and rope_local_caches_for(g2, 4) is None
    assert g2.attn_softcap() is None
    g2 = cfg_of(dict(base, model_type="gemma2", num_hidden_layers=26,
                     final_logit_softcapping=30.0, attn_logit_softcapping=50.0))
    assert g2.attn_softcap() == 50.0 and g2.final_softcap() == 30.0
    assert g270.attn_softcap() is None and g270.final_softcap() is None
    ll = cfg_of({"hidden_size": 64, "intermediate_size": 128, "num_hidden_layers": 2,
                 "num_attention_heads": 4, "rms_norm_eps": 1e-5, "vocab_size": 16, "hidden_act": "silu"})
    assert not ll.is_gemma() and not ll.tied() and not ll.sliding(0)
    assert ll.activation() == "silu" and ll.embed_scale() == 1.0 and ll.layer_window(0) is None
    assert rope_local_caches_for(ll, 4) is None
    with pytest.raises(ValueError, match="activation"):
        cfg_of({"hidden_size": 64, "intermediate_size": 128, "num_hidden_layers": 2,
                "num_attention_heads": 4, "rms_norm_eps": 1e-5, "vocab_size": 16, "hidden_act": "gelu"})


def test_config_round_trips_through_json(tmp_path):
    """to_dict keeps the family keys, so a saved config parses to the same rules."""
    from reng.config import LlamaConfig
    g = cfg_of({"hidden_size": 640, "intermediate_size": 2048, "num_attention_heads": 4,
                "num_key_value_heads": 1, "head_dim": 256, "vocab_size": 1024, "num_hidden_layers": 6,
                "model_type": "gemma2", "attn_logit_softcapping": 50.0, "sliding_window": 512,
                "query_pre_attn_scalar": 256, "hidden_activation": "gelu_pytorch_tanh"})
    h = LlamaConfig.from_json(json.dumps(g.to_dict()))
    assert [h.layer_window(i) for i in range(6)] == [g.layer_window(i) for i in range(6)]
    assert (h.attn_softcap(), h.attention_scale(), h.tied()) == (50.0, 0.0625, True)


def test_trained_context_warns_only_past_it():
    """lib.rs:4791-4807."""
    c = cfg_of({"model_type": "llama", "hidden_size": 4096, "intermediate_size": 14336,
                "num_hidden_layers": 32, "num_attention_heads": 32, "num_key_value_heads": 8,
                "rms_norm_eps": 1e-5, "vocab_size": 128256, "max_position_embeddings": 131072,
                "rope_scaling": {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                 "high_freq_factor": 4.0, "original_max_position_embeddings": 8192}})
    assert c.trained_context() == 131072 and c.original_context() == 8192
    assert c.context_warning(131072) is None
    w = c.context_warning(131073)
    assert "131072" in w and "rope scaling" in w
    bare = cfg_of({"hidden_size": 64, "intermediate_size": 128, "num_hidden_layers": 1,
                   "num_attention_heads": 4, "rms_norm_eps": 1e-5, "vocab_size": 16})
    assert bare.trained_context() is None and bare.context_warning(1000000) is None


def test_conversions_and_position_zero():
    """lib.rs:4406-4436: small integers and powers of two survive bf16, f16
    reads as the reference's conversion, position 0 is the identity rotation,
    argmax_rows picks the first maximum of each row."""
    from reng.model import argmax_rows
    from reng.rope import rope_caches_partial
    from reng.synth import bf16_bits_to_f32, f32_to_bf16_bits
    v = np.array([0.0, 1.0, -2.0, 0.5, 256.0, -0.125], np.float32)
    assert np.array_equal(bf16_bits_to_f32(f32_to_bf16_bits(v)), v)
    h = np.array([0x3C00, 0xC000, 0x0000, 0x3555], np.uint16).view(np.float16).astype(np.float32)
    assert h[0] == 1.0 and h[1] == -2.0 and h[2] == 0.0 and abs(h[3] - 0.33325) < 1e-4
    sin, cos = rope_caches_partial(2, 4, 4, 10000.0)
    assert np.all(sin[0] == 0.0) and np.all(cos[0] == 1.0) and np.any(sin[1] != 0.0)
    assert argmax_rows(np.array([[0.1, 0.9, 0.3], [2.0, -1.0, 0.0]], np.float32)) == [1, 0]
