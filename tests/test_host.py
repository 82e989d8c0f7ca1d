"""Host-side pieces of the reng-model mirror (CPU only): config.json parsing,
RoPE tables against the reference's transformers fixture, the safetensors
loader, the tensor-parallel shard rule, the RENG_FP8 switch and argmax."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN


def test_rope_tables_match_the_transformers_reference():
    """crates/reng-model/src/lib.rs:3849-3969 on rope_reference.json."""
    from reng.config import LlamaConfig
    from reng.rope import rope_caches_for, rope_head_perm, rope_spec
    with open(os.path.join(GOLDEN, "rope_reference.json")) as f:
        fx = json.load(f)
    assert fx["transformers"].startswith("5")
    want = ["phi35-short", "phi35-long", "phi35-long-short-table", "phi4mini-short",
            "phi4mini-long", "gemma3-4b-global", "gemma3-4b-local", "yarn-dsv2lite",
            "yarn-kimi-k2", "yarn-dsv4-flash"]
    assert sorted(c["name"] for c in fx["cases"]) == sorted(want)

    def rel(a, b):
        return abs(float(a) - float(b)) / max(abs(float(b)), np.finfo(np.float64).tiny)

    for c in fx["cases"]:
        cfg = LlamaConfig.from_dict(c["config"])
        hd, rd, local = cfg.head_dim(), cfg.rotary_dim(), c["table"] == "local"
        assert (hd, rd) == (c["head_dim"], c["rotary_dim"]), c["name"]
        if local:
            inv, af = rope_spec(rd, cfg.rope_local_base_freq or 1e4, None, c["table_len"])
        else:
            inv, af = rope_spec(rd, cfg.rope_theta, cfg.rope_scaling, c["seq_len"])
        assert rel(af, c["attention_factor"]) < 1e-6, c["name"]
        assert len(inv) == len(c["inv_freq"])
        for i, (e, r) in enumerate(zip(inv, c["inv_freq"])):
            assert rel(e, r) < 1e-6, (c["name"], i, e, r)
        if local:
            from reng.rope import rope_caches_partial
            sin, cos = rope_caches_partial(c["table_len"], hd, rd, cfg.rope_local_base_freq or 1e4,
                                           None, c["table_len"])
        else:
            sin, cos = rope_caches_for(cfg, c["table_len"], c["seq_len"])
        assert cos.shape == (c["table_len"], hd)
        perm = rope_head_perm(hd, rd)
        for row, p in enumerate(c["positions"]):
            for d in range(hd):
                src = perm[d]
                if src < rd:
                    j = src % (rd // 2)
                    ae = np.float32(p) * np.float32(inv[j])
                    ar = np.float32(p) * np.float32(c["inv_freq"][j])
                    slack = abs(float(ae) - float(ar)) * c["attention_factor"]
                    rc, rs = c["cos"][row][src], c["sin"][row][src]
                else:
                    slack, rc, rs = 0.0, 1.0, 0.0
                tol = 1e-6 + slack + abs(af - c["attention_factor"]) + 2e-7 * p
                assert abs(float(cos[p, d]) - rc) < tol, (c["name"], p, d, cos[p, d], rc)
                assert abs(float(sin[p, d]) - rs) < tol, (c["name"], p, d, sin[p, d], rs)


def test_baseline_shapes():
    from reng.config import llama31_8b, qwen25_32b, smollm2_135m
    s, l, q = smollm2_135m(), llama31_8b(), qwen25_32b()
    # active params as reng-ceiling counts them (embedding excluded, head included)
    assert s.active_params() == 134_479_872
    assert l.active_params() == 7_504_658_432
    assert q.active_params() == 31_984_189_440
    assert s.kv_bytes_per_token() == 23_040
    assert l.kv_bytes_per_token() == 131_072
    assert q.kv_bytes_per_token() == 262_144
    assert l.attention_scale() == np.float32(1.0) / np.sqrt(np.float32(128))


def test_shard_divides_heads_and_intermediate():
    from reng.config import llama31_8b, smollm2_135m
    c = llama31_8b().shard(1, 4)
    assert (c.num_attention_heads, c.n_kv_heads(), c.intermediate_size, c.head_dim()) == \
        (8, 2, 3584, 128)
    with pytest.raises(ValueError):
        smollm2_135m().shard(0, 2)  # 9 heads / 3 kv heads do not shard
    with pytest.raises(ValueError):
        llama31_8b().shard(4, 4)


def test_config_json_round_trip_and_safetensors_loader(tmp_path):
    from reng.config import LlamaConfig
    from reng.weights import load_weights, random_weights, save_checkpoint
    cfg = LlamaConfig(hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim_=16, vocab_size=96,
                      rms_norm_eps=1e-6, rope_theta=1e6, attention_bias=True, model_type="qwen2")
    w = random_weights(cfg, seed=5)
    save_checkpoint(str(tmp_path), cfg, w)
    cfg2 = LlamaConfig.load(str(tmp_path))
    assert (cfg2.hidden_size, cfg2.n_kv_heads(), cfg2.head_dim(), cfg2.rope_theta, cfg2.has_bias()) \
        == (64, 2, 16, 1e6, True)
    w2 = load_weights(str(tmp_path), cfg2)
    for l in range(2):
        for k in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
            assert np.array_equal(np.asarray(w2["layers"][l][k]), w["layers"][l][k]), (l, k)
        for k in ("g1", "g2", "bq", "bk", "bv"):
            assert np.array_equal(w2["layers"][l][k], w["layers"][l][k]), (l, k)
    assert np.array_equal(w2["embed"], w["embed"]) and np.array_equal(w2["lm_head"], w["lm_head"])
    # a missing tensor is an error, not a silent zero
    from reng.weights import write_safetensors
    write_safetensors(str(tmp_path / "model.safetensors"), {"x": ("F32", np.zeros(1, np.float32))})
    with pytest.raises(ValueError):
        load_weights(str(tmp_path), cfg2)


def test_qk_norm_gains_round_trip_and_are_refused_by_the_engine(tmp_path):
    """q/k norm gains (Qwen3's [head_dim] form) survive save/load as the
    reference reads them (crates/reng-model/src/lib.rs:1607-1609); an
    engine given them refuses, whatever the model_type says, instead of
    decoding without the norm."""
    from reng.config import LlamaConfig
    from reng.model import Engine
    from reng.weights import load_weights, random_weights, save_checkpoint
    cfg = LlamaConfig(hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim_=16, vocab_size=96,
                      rms_norm_eps=1e-6, rope_theta=1e6, model_type="qwen3")
    w = random_weights(cfg, seed=6)
    rng = np.random.default_rng(6)
    for lw in w["layers"]:
        lw["qn"] = rng.standard_normal(16).astype(np.float32)
        lw["kn"] = rng.standard_normal(16).astype(np.float32)
    save_checkpoint(str(tmp_path), cfg, w)
    w2 = load_weights(str(tmp_path), LlamaConfig.load(str(tmp_path)))
    for l in range(2):
        for k in ("qn", "kn"):
            assert np.array_equal(w2["layers"][l][k], w["layers"][l][k]), (l, k)
    as_llama = LlamaConfig.from_dict(dict(cfg.to_dict(), model_type="llama"))
    assert as_llama.unsupported(capacity=64) == []
    with pytest.raises(ValueError, match="q/k RMSNorm"):
        Engine(as_llama, w2, capacity=64)
    # a plain Llama checkpoint loads without them
    del w["layers"][0]["qn"], w["layers"][0]["kn"], w["layers"][1]["qn"], w["layers"][1]["kn"]
    save_checkpoint(str(tmp_path / "plain"), as_llama, w)
    w3 = load_weights(str(tmp_path / "plain"), as_llama)
    assert all("qn" not in lw and "kn" not in lw for lw in w3["layers"])


def test_fp8_switch_grammar():
    from reng.model import fp8_switch
    assert fp8_switch(None) is None
    assert fp8_switch("0") is None and fp8_switch("off") is None
    assert fp8_switch("1") == ("e4m3", "pcs")
    assert fp8_switch("e5m2:hw") == ("e5m2", "hw")
    assert fp8_switch("E4M3:unit") == ("e4m3", "unit")
    assert fp8_switch(None, flag=True) == ("e4m3", "pcs")
    for bad in ("fp4", "e4m3:bogus", "e4m3:pcs:x"):
        with pytest.raises(ValueError):
            fp8_switch(bad)


def test_argmax_rows_picks_the_first_max():
    from reng.model import argmax_rows
    assert argmax_rows([[1.0, 3.0, 3.0, 2.0], [0.0, -1.0, 0.0, np.nan]]) == [1, 0]


def test_fp8_format_enums_mirror_the_reference():
    from reng.fp8 import Fp8Format, Scaling
    assert Fp8Format.E4M3.max_finite_code == 0x77 and Fp8Format.E5M2.max_finite_code == 0x7b
    assert Fp8Format.from_name("hf8") is Fp8Format.E4M3 and Fp8Format.from_name("f8") is Fp8Format.E5M2
    assert Fp8Format.from_name("fp4") is None
    assert Scaling.from_name("per-channel") is Scaling.PerChannel and Scaling.from_name("x") is None


def test_engine_refuses_what_its_kernels_do_not_compute():
    """Configs the loader parses but the engine's decoder does not run are
    refused before any device work, with the features named (the reference
    refuses activations and MLP biases it has no node for,
    crates/reng-model/src/lib.rs:318-330, :1479)."""
    from reng.config import LlamaConfig, llama31_8b, qwen25_32b, smollm2_135m
    from reng.model import Engine
    base = {"hidden_size": 256, "intermediate_size": 512, "num_hidden_layers": 2,
            "num_attention_heads": 4, "num_key_value_heads": 2, "vocab_size": 1024}
    for c in (llama31_8b(), qwen25_32b(), smollm2_135m(), LlamaConfig.from_dict(dict(base, model_type="llama")),
              LlamaConfig.from_dict(dict(base, model_type="qwen2", sliding_window=4096, use_sliding_window=False))):
        assert c.unsupported(capacity=8192) == []
    cases = [
        (dict(base, model_type="qwen3"), "model_type qwen3"),
        (dict(base, model_type="olmo2"), "model_type olmo2"),
        (dict(base, model_type="llama", hidden_act="gelu_pytorch_tanh"), "activation"),
        (dict(base, model_type="llama", partial_rotary_factor=0.5), "partial rotary"),
        (dict(base, model_type="llama", mlp_bias=True), "mlp_bias"),
        (dict(base, model_type="granite", embedding_multiplier=12.0), "embedding_multiplier"),
        (dict(base, model_type="mistral", sliding_window=1024), "sliding window"),
        ({"model_type": "gemma3", "text_config": {}}, "model_type gemma3_text"),
    ]
    for d, what in cases:
        cfg = LlamaConfig.from_dict(d)
        miss = cfg.unsupported(capacity=4096)
        assert any(what in m for m in miss), (d, miss)
        with pytest.raises(ValueError, match="does not run"):
            Engine(cfg, {"embed": np.zeros((1, 1), np.uint16)}, capacity=4096)
    # a sliding window at or above the capacity attends exactly as full attention
    assert LlamaConfig.from_dict(dict(base, model_type="mistral", sliding_window=4096)).unsupported(4096) == []
