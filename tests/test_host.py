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


def test_qk_norm_gains_round_trip(tmp_path):
    """q/k norm gains (Qwen3's [head_dim] form) survive save/load as the
    reference reads them (crates/reng-model/src/lib.rs:1607-1609); the
    engine computes the norm wherever a layer carries them, whatever the
    model_type says (tests/test_qk_norm_gpu.py)."""
    from reng.config import LlamaConfig
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
    # an explicit off value wins over the flag (a wrapper's --fp8 can be
    # turned off from the environment)
    assert fp8_switch("off", flag=True) is None and fp8_switch("", flag=True) is None
    # settings in any order, ':' or ',' separated, with a backoff in (0, 1]
    c = fp8_switch("hw,e5m2")
    assert c == ("e5m2", "hw") and c.backoff == 1.0
    c = fp8_switch("pcs,backoff=0.5")
    assert c == ("e4m3", "pcs") and c.backoff == 0.5
    for bad in ("fp4", "e4m3:bogus", "e4m3:pcs:x", "backoff=2", "backoff=0", "backoff=x"):
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
        (dict(base, model_type="olmo2"), "model_type olmo2"),
        (dict(base, model_type="llama", hidden_act="gelu_pytorch_tanh"), "activation"),
        (dict(base, model_type="llama", mlp_bias=True), "mlp_bias"),
        (dict(base, model_type="gemma2", attn_logit_softcapping=50.0), "attn_logit_softcapping"),
        (dict(base, model_type="mistral", sliding_window=1024), "sliding window"),
        ({"model_type": "gemma3", "text_config": {}}, "model_type gemma3_text"),
    ]
    for d, what in cases:
        cfg = LlamaConfig.from_dict(d)
        miss = cfg.unsupported(capacity=4096)
        assert any(what in m for m in miss), (d, miss)
        with pytest.raises(ValueError, match="does not run"):
            Engine(cfg, {"embed": np.zeros((1, 1), np.uint16)}, capacity=4096)
    # Granite's multipliers (folded by the loader) and a partial rotation run
    for d in (dict(base, model_type="granite", embedding_multiplier=12.0, residual_multiplier=0.25,
                   attention_multiplier=0.0625, logits_scaling=8.0),
              dict(base, model_type="phi3", partial_rotary_factor=0.5)):
        assert LlamaConfig.from_dict(d).unsupported(capacity=4096) == [], d
    # a sliding window at or above the capacity attends exactly as full attention
    assert LlamaConfig.from_dict(dict(base, model_type="mistral", sliding_window=4096)).unsupported(4096) == []


def _raw_safetensors(path, parts):
    """A safetensors file of (name, dtype, shape, bytes) packed back to back
    with no padding between tensors, so a one-byte U8 tensor puts the next
    one on an odd offset (as in large real checkpoints)."""
    import json as _json
    import struct as _struct
    header, data = {}, b""
    for name, dt, shape, raw in parts:
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [len(data), len(data) + len(raw)]}
        data += raw
    hb = _json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(_struct.pack("<Q", len(hb)) + hb + data)


def test_mapped_views_odd_offsets_and_conversions(tmp_path):
    """The reference's loader test (crates/reng-model/src/lib.rs:4163-4215):
    an aligned bf16 tensor is a view of the mapped file (no copy), one on an
    odd byte offset still reads its own values, f32 tensors convert to bf16
    (round to nearest even) and bf16 reads back as f32."""
    from reng.synth import f32_to_bf16_bits
    from reng.weights import SafeTensors, _as_bf16, _as_f32
    a = f32_to_bf16_bits(np.arange(6, dtype=np.float32) * 0.5).reshape(2, 3)
    c = f32_to_bf16_bits(np.array([-1.0, 2.0], np.float32))
    d = np.array([0.25, -8.0], np.float32)
    p = str(tmp_path / "model.safetensors")
    _raw_safetensors(p, [("a", "BF16", (2, 3), a.tobytes()), ("b", "U8", (1,), b"\x07"),
                         ("c", "BF16", (2,), c.tobytes()), ("d", "F32", (2,), d.tobytes())])
    st = SafeTensors(p)
    va = _as_bf16(st, "a")
    assert va.shape == (2, 3) and np.array_equal(va, a)
    assert not va.flags.owndata                       # a view of the map, not a copy
    vc = _as_bf16(st, "c")
    assert (st._base + st.header["c"]["data_offsets"][0]) % 2 == 1
    assert np.array_equal(vc, c)
    assert np.array_equal(_as_bf16(st, "d"), f32_to_bf16_bits(d))
    assert np.array_equal(_as_f32(st, "d"), d) and _as_f32(st, "a")[1, 0] == 1.5


def test_loader_reads_a_checkpoint_with_odd_offsets(tmp_path):
    """Every tensor of a small Llama checkpoint on an odd byte: the loaded
    weights equal the aligned checkpoint's."""
    from reng.config import LlamaConfig
    from reng.weights import load_weights, random_weights, save_checkpoint
    cfg = LlamaConfig(hidden_size=32, intermediate_size=64, num_hidden_layers=1,
                      num_attention_heads=2, num_key_value_heads=1, head_dim_=16, vocab_size=40,
                      model_type="llama")
    w = random_weights(cfg, seed=9)
    save_checkpoint(str(tmp_path / "a"), cfg, w)
    ref = load_weights(str(tmp_path / "a"), cfg)
    from reng.weights import SafeTensors
    st = SafeTensors(str(tmp_path / "a" / "model.safetensors"))
    parts = []
    for name in st.names():
        parts.append(("pad." + name, "U8", (1,), b"\x00"))
        v = st.view(name)
        parts.append((name, st.dtype(name), v.shape, np.ascontiguousarray(v).tobytes()))
    (tmp_path / "b").mkdir()
    _raw_safetensors(str(tmp_path / "b" / "model.safetensors"), parts)
    import shutil
    shutil.copy(str(tmp_path / "a" / "config.json"), str(tmp_path / "b" / "config.json"))
    odd = load_weights(str(tmp_path / "b"), cfg)
    for k in ("wq", "wk", "wv", "wo", "wg", "wu", "wd", "g1", "g2"):
        assert np.array_equal(odd["layers"][0][k], ref["layers"][0][k]), k
    assert np.array_equal(odd["embed"], ref["embed"]) and np.array_equal(odd["lm_head"], ref["lm_head"])


def test_the_engine_scales_its_embedding_table_like_the_gather():
    """bf16(f32(e) * f32(m)) per element, the same bits from a host array and
    a torch tensor (the device path's arithmetic, run here on CPU)."""
    import torch
    from reng.model import _scaled_table
    from reng.synth import bf16_bits_to_f32, f32_to_bf16_bits
    e = f32_to_bf16_bits(np.random.default_rng(2).standard_normal((16, 32)).astype(np.float32) * 0.02)
    want = f32_to_bf16_bits(bf16_bits_to_f32(e) * np.float32(12.0))
    assert np.array_equal(_scaled_table(e, 12.0), want)
    t = torch.from_numpy(e.view(np.int16).copy())
    got = _scaled_table(t, 12.0)
    assert got.dtype == torch.int16 and np.array_equal(got.numpy().view(np.uint16), want)


def test_qk_norm_forms(monkeypatch):
    """Qwen3's per-head q/k norm is a config the engine runs; the whole-row
    form (OLMo-2) is refused before any device work."""
    from reng.config import LlamaConfig
    from reng.model import Engine
    base = {"hidden_size": 64, "intermediate_size": 128, "num_hidden_layers": 1,
            "num_attention_heads": 4, "num_key_value_heads": 2, "head_dim": 16, "vocab_size": 32,
            "model_type": "qwen3"}
    cfg = LlamaConfig.from_dict(base)
    assert cfg.unsupported(capacity=64) == []
    wide = {"qn": np.ones(64, np.float32), "kn": np.ones(32, np.float32)}
    with pytest.raises(ValueError, match="whole-row q/k norm"):
        Engine(cfg, {"layers": [wide], "embed": np.zeros((1, 1), np.uint16)}, capacity=64)