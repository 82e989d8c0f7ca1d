"""Golden logits that pin the loader and the f32 forward oracle to HF
transformers for the decoder families beyond Llama / Qwen2 / Qwen3.

The reference's loader and host forward (crates/reng-model/src/lib.rs:
268-420 and 1477-1688, crates/reng-synapse/src/model.rs:2903-3138) take
Granite's four multipliers, OLMo-2's post-norm and whole-row q/k norms,
Gemma-2's GELU-tanh, four norms, zero-centred gains, sqrt(hidden)
embedding scale, score and logit softcaps and alternating sliding layers,
Gemma-3's per-head q/k norms and local RoPE table, Phi-3's fused
qkv_proj / gate_up_proj and partial rotation, Mistral's sliding window
and SmolLM3's NoPE layers.  For each, this script writes a seeded random
checkpoint in the family's own HF layout (config.json + model.safetensors),
runs transformers' f32 eager forward on it, and stores the config, the
stored tensors, the prompt ids and the logits in
tests/golden/family_golden.npz (keys "<family>|<tensor name>").

    python tests/golden/make_family_golden.py

Run in the build container (transformers is not needed on the GPU box; the
fixture is committed).  Every scale the reference folds into a bf16 weight
(the attention scale into wq, Granite's residual multiplier into o/down
and 1/logits_scaling into the head) is a power of two here, so the folds
are exact and the oracle must agree with transformers to f32 rounding.
"""
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "reciprocating-engine_b200"))

H, I, L, NH, NKV, HD, V = 64, 128, 2, 4, 2, 16, 128
TOKENS = 24
WINDOW = 8

BASE = dict(hidden_size=H, intermediate_size=I, num_hidden_layers=L, num_attention_heads=NH,
            num_key_value_heads=NKV, vocab_size=V, rms_norm_eps=1e-5, rope_theta=10000.0,
            max_position_embeddings=256, tie_word_embeddings=False, bos_token_id=1,
            eos_token_id=2, pad_token_id=0)

FAMILIES = {
    "granite": dict(BASE, model_type="granite", embedding_multiplier=12.0,
                    attention_multiplier=0.125, residual_multiplier=0.25, logits_scaling=8.0,
                    attention_bias=False, mlp_bias=False, hidden_act="silu"),
    "olmo2": dict(BASE, model_type="olmo2", attention_bias=False, rms_norm_eps=1e-6,
                  hidden_act="silu"),
    "gemma2": dict(BASE, model_type="gemma2", head_dim=HD, query_pre_attn_scalar=HD,
                   sliding_window=WINDOW, attn_logit_softcapping=1.0, final_logit_softcapping=2.0,
                   hidden_activation="gelu_pytorch_tanh", hidden_act="gelu_pytorch_tanh",
                   rms_norm_eps=1e-6, tie_word_embeddings=True),
    "gemma3_text": dict(BASE, model_type="gemma3_text", head_dim=HD, query_pre_attn_scalar=HD,
                        sliding_window=WINDOW, hidden_activation="gelu_pytorch_tanh",
                        layer_types=["sliding_attention", "full_attention"],
                        rope_theta=1000000.0, rope_local_base_freq=10000.0, rms_norm_eps=1e-6,
                        final_logit_softcapping=None, attn_logit_softcapping=None,
                        tie_word_embeddings=True),
    "phi3": dict(BASE, model_type="phi3", partial_rotary_factor=0.5, sliding_window=WINDOW,
                 hidden_act="silu", original_max_position_embeddings=256),
    "mistral": dict(BASE, model_type="mistral", head_dim=HD, sliding_window=WINDOW,
                    hidden_act="silu"),
    "smollm3": dict(BASE, model_type="smollm3", no_rope_layers=[1, 0], use_sliding_window=False,
                    hidden_act="silu", attention_bias=False, mlp_bias=False),
}


def checkpoint(fam, cfg, rng):
    """{name: (safetensors dtype, array)} in the family's own HF layout."""
    from reng.synth import f32_to_bf16_bits
    gemma = fam.startswith("gemma")
    qd, kvd = NH * HD, NKV * HD

    def mat(r, c, std=0.05):
        return ("BF16", f32_to_bf16_bits(rng.standard_normal((r, c)).astype(np.float32) * std))

    def gain(n):
        # Gemma stores zero-centred gains (applied as 1 + w)
        c = 0.0 if gemma else 1.0
        return ("F32", (c + 0.1 * rng.standard_normal(n)).astype(np.float32))

    t = {"model.embed_tokens.weight": mat(V, H, 0.5)}
    for l in range(L):
        p = "model.layers.%d." % l
        if fam == "phi3":
            t[p + "self_attn.qkv_proj.weight"] = mat(qd + 2 * kvd, H)
            t[p + "mlp.gate_up_proj.weight"] = mat(2 * I, H)
        else:
            t[p + "self_attn.q_proj.weight"] = mat(qd, H)
            t[p + "self_attn.k_proj.weight"] = mat(kvd, H)
            t[p + "self_attn.v_proj.weight"] = mat(kvd, H)
            t[p + "mlp.gate_proj.weight"] = mat(I, H)
            t[p + "mlp.up_proj.weight"] = mat(I, H)
        t[p + "self_attn.o_proj.weight"] = mat(H, qd)
        t[p + "mlp.down_proj.weight"] = mat(H, I)
        if fam == "olmo2":
            t[p + "post_attention_layernorm.weight"] = gain(H)
            t[p + "post_feedforward_layernorm.weight"] = gain(H)
            t[p + "self_attn.q_norm.weight"] = gain(qd)
            t[p + "self_attn.k_norm.weight"] = gain(kvd)
        elif gemma:
            for n in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                      "post_feedforward_layernorm"):
                t[p + n + ".weight"] = gain(H)
            if fam == "gemma3_text":
                t[p + "self_attn.q_norm.weight"] = gain(HD)
                t[p + "self_attn.k_norm.weight"] = gain(HD)
        else:
            t[p + "input_layernorm.weight"] = gain(H)
            t[p + "post_attention_layernorm.weight"] = gain(H)
    t["model.norm.weight"] = gain(H)
    if not cfg.get("tie_word_embeddings"):
        t["lm_head.weight"] = mat(V, H, 0.2)
    return t


def main():
    import torch
    import transformers
    from transformers import AutoConfig, AutoModelForCausalLM

    from reng.weights import write_safetensors

    rng = np.random.default_rng(20261202)
    ids = rng.integers(0, V, TOKENS).astype(np.uint32)
    out = {"ids": ids}
    for fam, cfg in FAMILIES.items():
        t = checkpoint(fam, cfg, rng)
        with tempfile.TemporaryDirectory() as d:
            with open(os.path.join(d, "config.json"), "w") as f:
                json.dump(cfg, f)
            write_safetensors(os.path.join(d, "model.safetensors"), t)
            hc = AutoConfig.from_pretrained(d)
            m = AutoModelForCausalLM.from_pretrained(d, config=hc, torch_dtype=torch.float32,
                                                     attn_implementation="eager")
            m.eval()
            with torch.no_grad():
                lg = m(torch.tensor(ids[None, :].astype(np.int64))).logits[0].numpy()
        out[fam + "|config"] = np.array(json.dumps(cfg))
        for name, (dt, a) in t.items():
            out[fam + "|" + name] = a
        out[fam + "|logits"] = lg.astype(np.float32)
        print(fam, type(m).__name__, "logits", lg.shape, "max |l| %.3f" % np.abs(lg).max())
    out["meta"] = np.array(["transformers " + transformers.__version__, "torch " + torch.__version__])
    np.savez_compressed(os.path.join(HERE, "family_golden.npz"), **out)
    print("wrote family_golden.npz, %d arrays" % len(out))


if __name__ == "__main__":
    main()
