"""The loader (reng.weights.load_weights) and the f32 forward oracle
against HF transformers for the decoder families past Llama / Qwen2 /
Qwen3, on the committed fixture of tests/golden/make_family_golden.py.

Each case writes the family's checkpoint in its own HF layout, parses
its config.json with LlamaConfig, loads it with the reference's family
rules (crates/reng-model/src/lib.rs:1477-1688) and runs the oracle with
the per-layer settings of layer_views (lib.rs:2630-2707); the logits must
match transformers' f32 eager forward to f32 rounding.  The engine
refuses these families (`LlamaConfig.unsupported`); this pins the checker
their kernels will be held to."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

FAMILIES = ("granite", "olmo2", "gemma2", "gemma3_text", "phi3", "mistral", "smollm3")


@pytest.fixture(scope="module")
def golden():
    z = np.load(os.path.join(GOLDEN, "family_golden.npz"))
    return {k: z[k] for k in z.files}


def write_checkpoint(z, fam, d):
    from reng.weights import write_safetensors
    cfg = json.loads(str(z[fam + "|config"]))
    os.makedirs(d, exist_ok=True)
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f)
    t = {}
    for k, a in z.items():
        if k.startswith(fam + "|") and k not in (fam + "|config", fam + "|logits"):
            t[k.split("|", 1)[1]] = ("BF16" if a.dtype == np.uint16 else "F32", a)
    write_safetensors(os.path.join(d, "model.safetensors"), t)
    return cfg


def family_oracle(z, fam, d):
    import oracle
    from reng.config import LlamaConfig
    from reng.weights import load_weights
    write_checkpoint(z, fam, d)
    cfg = LlamaConfig.load(d)
    w = load_weights(d, cfg)
    return cfg, w, oracle.Model.for_config(cfg, w)


def run(cfg, m, ids):
    from reng.rope import rope_caches_for, rope_local_caches_for
    sin, cos = rope_caches_for(cfg, len(ids))
    loc = rope_local_caches_for(cfg, len(ids))
    kw = {} if loc is None else {"sin_local": loc[0], "cos_local": loc[1]}
    return m.forward(ids, sin, cos, **kw)


@pytest.mark.parametrize("fam", FAMILIES)
def test_family_oracle_matches_transformers(oracle_lib, golden, fam, tmp_path):
    cfg, _, m = family_oracle(golden, fam, str(tmp_path))
    got = run(cfg, m, golden["ids"])
    want = golden[fam + "|logits"]
    err = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert err < 2e-5, (fam, err)
    assert np.array_equal(got.argmax(-1), want.argmax(-1)), fam


def test_family_rules_as_parsed(golden, tmp_path):
    """The per-family settings the oracle ran with are the reference's
    (lib.rs:268-420, 697-712)."""
    from reng.config import LlamaConfig
    got = {}
    for fam in FAMILIES:
        d = tmp_path / fam
        d.mkdir()
        write_checkpoint(golden, fam, str(d))
        got[fam] = LlamaConfig.load(str(d))
    g2, g3 = got["gemma2"], got["gemma3_text"]
    assert [g2.layer_window(i) for i in range(2)] == [8, None]
    assert [g3.local_rope(i) for i in range(2)] == [True, False]
    assert g2.attn_softcap() == 1.0 and g3.attn_softcap() is None
    assert g2.tied() and g2.activation() == "gelu_tanh"
    assert g2.embed_scale() == pytest.approx(8.0) and g2.attention_scale() == 0.25
    gr = got["granite"]
    assert gr.attention_scale() == 0.125 and gr.embed_scale() == 12.0
    assert got["olmo2"].post_norm() and not got["mistral"].post_norm()
    assert got["mistral"].window() == 8 and got["phi3"].window() == 8
    assert got["phi3"].rotary_dim() == 8
    assert [got["smollm3"].use_rope(i) for i in range(2)] == [True, False]
    # the engine runs Granite (multipliers folded by the loader), partial
    # rotation and NoPE layers; it refuses the rest, and Phi-3 here for its
    # window of 8 below the capacity
    for fam, c in got.items():
        assert bool(c.unsupported(capacity=64)) == (fam not in ("granite", "smollm3")), \
            (fam, c.unsupported(capacity=64))
    assert got["phi3"].unsupported(capacity=8) == []


def test_loader_family_tensors(golden, tmp_path):
    """What the loader makes of each layout: Phi-3's fused tensors split
    into row blocks, Gemma's gains plus one and final gain over the cap,
    Granite's folds exact at power-of-two multipliers."""
    from reng.synth import bf16_bits_to_f32
    _, w, _ = family_oracle(golden, "phi3", str(tmp_path / "p"))
    qkv = golden["phi3|model.layers.0.self_attn.qkv_proj.weight"]
    assert np.array_equal(w["layers"][0]["wv"], qkv[64 + 32:])
    _, w, _ = family_oracle(golden, "gemma2", str(tmp_path / "g"))
    assert np.array_equal(w["layers"][1]["g_post_mlp"],
                          golden["gemma2|model.layers.1.post_feedforward_layernorm.weight"] + 1.0)
    assert np.allclose(w["final_gamma"], (golden["gemma2|model.norm.weight"] + 1.0) / 2.0,
                       rtol=0, atol=0)
    assert w["lm_head"] is w["embed"]
    _, w, _ = family_oracle(golden, "granite", str(tmp_path / "r"))
    wo = golden["granite|model.layers.0.self_attn.o_proj.weight"]
    assert np.array_equal(bf16_bits_to_f32(w["layers"][0]["wo"]), bf16_bits_to_f32(wo) * 0.25)
    lm = golden["granite|lm_head.weight"]
    assert np.array_equal(bf16_bits_to_f32(w["lm_head"]), bf16_bits_to_f32(lm) / 8.0)


def test_partial_rotation_permutes_q_and_k_alike(golden, tmp_path):
    """Phi-3 with partial_rotary_factor 0.5: the loader moves q/k head dims
    into the kernel's pair order (rope_head_perm, lib.rs:2231-2251); the
    permutation leaves every q.k product unchanged without RoPE."""
    from reng.rope import rope_head_perm
    from reng.synth import bf16_bits_to_f32
    _, w, _ = family_oracle(golden, "phi3", str(tmp_path))
    perm = rope_head_perm(16, 8)
    assert perm[:4] == [0, 1, 2, 3] and perm[8:12] == [4, 5, 6, 7]
    qkv = bf16_bits_to_f32(golden["phi3|model.layers.0.self_attn.qkv_proj.weight"])
    x = np.random.default_rng(0).standard_normal(64).astype(np.float32)
    q_hf, k_hf = qkv[:64] @ x, qkv[64:96] @ x
    q, k = bf16_bits_to_f32(w["layers"][0]["wq"]) @ x, bf16_bits_to_f32(w["layers"][0]["wk"]) @ x
    # head 0 of q against KV head 0
    assert np.allclose(q[:16] @ k[:16], q_hf[:16] @ k_hf[:16], rtol=1e-5)
    assert not np.array_equal(q[:16], q_hf[:16])
