"""First-principles decode / prefill ceilings on B200 (reng-ceiling's role).

Mirrors crates/reng-ceiling/src/lib.rs: `HardwareSpec` (lib.rs:15-52),
`Precision` (:55-105), the model-shape byte and parameter counts (:107-207),
`prefill_ceiling` / `decode_ceiling` (:236-311), and the tensor-parallel
strategy of strategy.rs:770-843 (body/N + replicated head + KV/N per card,
plus two all-reduces per layer).  Decode is HBM-bound (weight + KV bytes
over bandwidth), prefill tensor-bound (causal FLOPs over peak).

B200 figures: the spec sheet (HBM3e 8 TB/s, 2.25 PFLOP/s dense bf16,
4.5 dense fp8, 180 GB, NVLink 5 900 GB/s per direction) and, when
MEASURED_PEAKS.json is present, the measured copy bandwidth and cuBLAS bf16
rate of this pool's B200s.

    python -m reng.ceiling [--model llama-3.1-8b] [--batch 1] [--ctx 192] [--cards 1]
"""
import json
import os
from dataclasses import dataclass


@dataclass
class HardwareSpec:
    name: str
    flops_bf16: float
    flops_fp16: float
    flops_fp8: float
    flops_fp32: float
    hbm_bytes: int
    hbm_bw: float
    sram_bytes: int
    link_bw: float      # per direction: PCIe for Gaudi2, NVLink for B200

    @staticmethod
    def b200():
        return HardwareSpec("B200 (spec)", 2.25e15, 2.25e15, 4.5e15, 80e12,
                            183_359 * 1024 * 1024, 8.0e12, 126 * 1024 * 1024, 900e9)

    @staticmethod
    def b200_measured(path=None):
        """The spec with the measured HBM copy bandwidth and bf16 GEMM rate."""
        if path is None:
            path = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(
                os.path.abspath(__file__)))), "MEASURED_PEAKS.json")
        hw = HardwareSpec.b200()
        try:
            with open(path) as f:
                p = json.load(f)
        except OSError:
            return hw
        hw.name = "B200 (measured)"
        hw.hbm_bw = float(p["hbm_gbs"]) * 1e9
        hw.flops_bf16 = hw.flops_fp16 = float(p["bf16_tflops"]) * 1e12
        hw.flops_fp8 = 2 * hw.flops_bf16
        return hw

    @staticmethod
    def gaudi2():
        """The reference's own card (lib.rs:39-52), for comparisons."""
        return HardwareSpec("Gaudi2 (HL-225)", 432e12, 432e12, 865e12, 45e12,
                            98_304 * 1024 * 1024, 2.45e12, 48 * 1024 * 1024, 32e9)


WEIGHT_BYTES = {"fp32": 4.0, "bf16": 2.0, "fp16": 2.0, "fp8": 1.0, "int8": 1.0, "int4": 0.5}


def compute_flops(prec, hw):
    return {"fp8": hw.flops_fp8, "fp32": hw.flops_fp32, "fp16": hw.flops_fp16}.get(prec, hw.flops_bf16)


@dataclass
class ModelShape:
    name: str
    layers: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ff: int
    vocab: int
    tied_embeddings: bool = False

    @staticmethod
    def from_config(cfg, name="model"):
        return ModelShape(name, cfg.num_hidden_layers, cfg.hidden_size, cfg.num_attention_heads,
                          cfg.n_kv_heads(), cfg.head_dim(), cfg.intermediate_size, cfg.vocab_size,
                          cfg.tie_word_embeddings)

    def q_dim(self):
        return self.n_heads * self.head_dim

    def kv_dim(self):
        return self.n_kv_heads * self.head_dim

    def attn_params_per_layer(self):
        return self.hidden * self.q_dim() + 2 * self.hidden * self.kv_dim() + self.q_dim() * self.hidden

    def mlp_params_per_layer(self):
        return 3 * self.hidden * self.ff

    def head_params(self):
        return self.hidden * self.vocab

    def body_params(self):
        return self.layers * (self.attn_params_per_layer() + self.mlp_params_per_layer())

    def active_params(self):
        """Params touched per token; the embedding (a lookup) excluded."""
        return self.body_params() + self.head_params()

    def total_params(self):
        emb = self.hidden * self.vocab
        return self.body_params() + (emb if self.tied_embeddings else emb + self.head_params())

    def kv_bytes_per_token(self, kv="bf16"):
        return 2.0 * self.kv_dim() * self.layers * WEIGHT_BYTES[kv]


@dataclass
class Ceiling:
    latency_s: float
    tokens_per_s: float
    bottleneck: str
    compute_time_s: float
    memory_time_s: float
    arithmetic_intensity: float
    bytes: float
    flops: float


def _ceiling(flops, bytes_, peak, bw, tokens):
    ct, mt = flops / peak, bytes_ / bw
    lat = max(ct, mt)
    return Ceiling(lat, tokens / lat, "compute" if ct >= mt else "hbm", ct, mt, flops / bytes_, bytes_, flops)


def prefill_ceiling(hw, m, prec="bf16", kv="bf16", batch=1, seq_len=1024):
    b, s = float(batch), float(seq_len)
    active = float(m.active_params())
    linear = 2.0 * active * b * s
    attn = 4.0 * m.layers * b * m.n_heads * (s * (s + 1.0) / 2.0) * m.head_dim
    bytes_ = active * WEIGHT_BYTES[prec] + 2.0 * b * s * m.kv_bytes_per_token(kv)
    return _ceiling(linear + attn, bytes_, compute_flops(prec, hw), hw.hbm_bw, b * s)


def decode_ceiling(hw, m, prec="bf16", kv="bf16", batch=1, ctx_len=192):
    b, ctx = float(batch), float(ctx_len)
    active = float(m.active_params())
    flops = 2.0 * active * b + 4.0 * m.layers * b * m.n_heads * ctx * m.head_dim
    bytes_ = active * WEIGHT_BYTES[prec] + b * ctx * m.kv_bytes_per_token(kv)
    return _ceiling(flops, bytes_, compute_flops(prec, hw), hw.hbm_bw, b)


def tensor_parallel(hw, m, cards, batch=1, ctx_len=192, prec="bf16", kv="bf16",
                    all_reduce_s=None):
    """Per-card decode ceiling of Megatron TP over `cards` GPUs: projections
    split, LM head replicated, KV split, two all-reduces of hidden x batch x 4
    bytes per layer.  all_reduce_s(bytes) defaults to latency 0 + bytes over
    the per-direction link bandwidth (a lower bound)."""
    n = float(cards)
    wb = WEIGHT_BYTES[prec]
    body = m.body_params() * wb
    head = m.head_params() * wb if prec != "fp8" else m.head_params() * 2.0
    kvb = batch * ctx_len * m.kv_bytes_per_token(kv)
    card_bytes = body / n + head + kvb / n
    ar_bytes = m.hidden * batch * 4
    ar = all_reduce_s(ar_bytes) if all_reduce_s else (0.0 if cards == 1 else ar_bytes / hw.link_bw)
    coll = 0.0 if cards == 1 else 2.0 * m.layers * ar
    mem = card_bytes / hw.hbm_bw
    step = mem + coll
    divisible = (m.n_heads % cards == 0 and m.n_kv_heads % cards == 0 and m.ff % cards == 0)
    return {"cards": cards, "card_bytes": card_bytes, "memory_s": mem, "collective_s": coll,
            "step_s": step, "tokens_per_s": batch / step, "shardable": divisible}


def main():
    import argparse
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from reng.config import SHAPES
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3.1-8b")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=192)
    ap.add_argument("--prec", default="bf16")
    ap.add_argument("--cards", type=int, default=1)
    a = ap.parse_args()
    m = ModelShape.from_config(SHAPES[a.model](), a.model)
    for hw in (HardwareSpec.b200(), HardwareSpec.b200_measured(), HardwareSpec.gaudi2()):
        d = decode_ceiling(hw, m, a.prec, "bf16", a.batch, a.ctx)
        p = prefill_ceiling(hw, m, a.prec, "bf16", 1, 1024)
        tp = tensor_parallel(hw, m, a.cards, a.batch, a.ctx, a.prec)
        print("%-18s decode b%d ctx %d: %.4g GB/step, %.1f tok/s (%s);  prefill 1024: %.0f tok/s (%s);"
              "  tp%d: %.1f tok/s" % (hw.name, a.batch, a.ctx, d.bytes / 1e9, d.tokens_per_s, d.bottleneck,
                                      p.tokens_per_s, p.bottleneck, a.cards, tp["tokens_per_s"]))


if __name__ == "__main__":
    main()
