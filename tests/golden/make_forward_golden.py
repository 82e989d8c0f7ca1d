"""Golden logits that pin the f32 forward oracle to HF transformers.

The reference's external oracle (tools/oracle/oracle.py) runs a checkpoint
through transformers' AutoModelForCausalLM in f32 and records the logits.
This script does the same on seeded random weights written as a
config.json + model.safetensors pair, for a Llama decoder, a Qwen2
decoder (q/k/v biases) and a Qwen3 decoder (per-head q/k RMSNorm, no
biases), and stores the weights (bf16 bits), the prompt ids and the
transformers logits in tests/golden/forward_golden.npz.  The Qwen3 norm
gains are drawn after everything else, so the Llama / Qwen2 arrays do not
depend on them.

    python tests/golden/make_forward_golden.py

Run in the build container (transformers is not needed on the GPU box; the
fixture is committed).  head_dim 64 keeps the attention scale 1/8 exact, so
folding it into the bf16 wq (the reference's scaled_wq) loses nothing and
the oracle must agree with transformers to f32 rounding.
"""
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "reciprocating-engine_b200"))

CFG = dict(hidden_size=128, intermediate_size=256, num_hidden_layers=2,
           num_attention_heads=2, num_key_value_heads=1, head_dim=64, vocab_size=256,
           rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=512,
           tie_word_embeddings=False, hidden_act="silu")
TOKENS = 24


def main():
    import torch
    from transformers import LlamaForCausalLM, Qwen2ForCausalLM, Qwen3ForCausalLM

    from reng.config import LlamaConfig as RCfg
    from reng.synth import bf16_bits_to_f32, f32_to_bf16_bits
    from reng.weights import save_checkpoint

    rng = np.random.default_rng(20261201)
    h, I, V = CFG["hidden_size"], CFG["intermediate_size"], CFG["vocab_size"]
    hd, nh, nkv = CFG["head_dim"], CFG["num_attention_heads"], CFG["num_key_value_heads"]

    def mat(r, c):
        return f32_to_bf16_bits(rng.standard_normal((r, c)).astype(np.float32) * 0.05)

    layers = []
    for _ in range(CFG["num_hidden_layers"]):
        layers.append({
            "wq": mat(nh * hd, h), "wk": mat(nkv * hd, h), "wv": mat(nkv * hd, h),
            "wo": mat(h, nh * hd), "wg": mat(I, h), "wu": mat(I, h), "wd": mat(h, I),
            "g1": (1.0 + 0.1 * rng.standard_normal(h)).astype(np.float32),
            "g2": (1.0 + 0.1 * rng.standard_normal(h)).astype(np.float32),
            "bq": (0.05 * rng.standard_normal(nh * hd)).astype(np.float32),
            "bk": (0.05 * rng.standard_normal(nkv * hd)).astype(np.float32),
            "bv": (0.05 * rng.standard_normal(nkv * hd)).astype(np.float32),
        })
    embed = mat(V, h)
    lm = mat(V, h)
    fg = (1.0 + 0.1 * rng.standard_normal(h)).astype(np.float32)
    ids = rng.integers(0, V, TOKENS).astype(np.uint32)

    norms = [{"qn": (1.0 + 0.2 * rng.standard_normal(hd)).astype(np.float32),
              "kn": (1.0 + 0.2 * rng.standard_normal(hd)).astype(np.float32)}
             for _ in layers]

    out = {"ids": ids, "embed": embed, "lm_head": lm, "final_gamma": fg}
    for l, lw in enumerate(layers):
        for k, v in list(lw.items()) + list(norms[l].items()):
            out["l%d_%s" % (l, k)] = v
    classes = {"llama": LlamaForCausalLM, "qwen2": Qwen2ForCausalLM, "qwen3": Qwen3ForCausalLM}
    for arch, cls in classes.items():
        with tempfile.TemporaryDirectory() as d:
            rc = RCfg.from_dict(dict(CFG, model_type=arch, attention_bias=arch == "qwen2"))
            ls = []
            for l, lw in enumerate(layers):
                x = {k: v for k, v in lw.items() if arch == "qwen2" or not k.startswith("b")}
                if arch == "qwen3":
                    x.update(norms[l])
                ls.append(x)
            save_checkpoint(d, rc, {"layers": ls, "embed": embed, "lm_head": lm, "final_gamma": fg})
            m = cls.from_pretrained(d, torch_dtype=torch.float32, attn_implementation="eager")
            m.eval()
            with torch.no_grad():
                lg = m(torch.tensor(ids[None, :].astype(np.int64))).logits[0].numpy()
        out["logits_" + arch] = lg.astype(np.float32)
    import transformers
    out["meta"] = np.array(["transformers " + transformers.__version__, "torch " + torch.__version__])
    np.savez_compressed(os.path.join(HERE, "forward_golden.npz"), **out)
    print("wrote forward_golden.npz", {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
