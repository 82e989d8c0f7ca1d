"""reng-ceiling formulas (crates/reng-ceiling/src/lib.rs:184-311,
strategy.rs:770-843) and the CachePlan, against the byte counts of the
BASELINE shapes and the reference's own ceiling tests (lib.rs:485-640)."""
import pytest


def shapes():
    from reng.ceiling import ModelShape
    from reng.config import llama31_8b, qwen25_32b, smollm2_135m
    return {n: ModelShape.from_config(f(), n) for n, f in
            (("s", smollm2_135m), ("l", llama31_8b), ("q", qwen25_32b))}


def test_decode_bytes_per_step_of_the_baseline_configs():
    from reng.ceiling import HardwareSpec, decode_ceiling
    hw = HardwareSpec.b200()
    m = shapes()
    for key, b, ctx, gb in (("s", 1, 192, 0.273), ("s", 8, 192, 0.304), ("s", 64, 192, 0.552),
                            ("l", 1, 192, 15.034), ("l", 8, 192, 15.211), ("l", 64, 192, 16.620),
                            ("q", 1, 4224, 65.08), ("q", 8, 4224, 72.83), ("q", 64, 4224, 134.8)):
        c = decode_ceiling(hw, m[key], "bf16", "bf16", b, ctx)
        assert c.bottleneck == "hbm"
        assert abs(c.bytes / 1e9 - gb) / gb < 2e-3, (key, b, c.bytes / 1e9, gb)
    # 8 TB/s spec: Llama-8B b1 at ctx 192 -> 532 tok/s
    assert round(decode_ceiling(hw, m["l"], batch=1, ctx_len=192).tokens_per_s) == 532


def test_tensor_parallel_card_bytes():
    from reng.ceiling import HardwareSpec, tensor_parallel
    hw = HardwareSpec.b200()
    l = shapes()["l"]
    for cards, gb in ((2, 8.04), (4, 4.55), (8, 2.80)):
        tp = tensor_parallel(hw, l, cards, batch=1, ctx_len=192)
        assert abs(tp["card_bytes"] / 1e9 - gb) < 0.01, (cards, tp["card_bytes"])
        assert tp["shardable"] and tp["collective_s"] > 0
    assert not tensor_parallel(hw, shapes()["s"], 2)["shardable"]  # 9 heads / 3 KV heads


def test_reference_ceiling_properties():
    from reng.ceiling import HardwareSpec, ModelShape, decode_ceiling, prefill_ceiling
    for hw in (HardwareSpec.gaudi2(), HardwareSpec.b200()):
        m = ModelShape("dense_7b", 32, 4096, 32, 32, 128, 11008, 32000)
        assert decode_ceiling(hw, m, batch=1, ctx_len=2048).bottleneck == "hbm"
        p = prefill_ceiling(hw, m, seq_len=8192)
        assert p.bottleneck == "compute" and p.arithmetic_intensity > 100
        s = 131072
        c = prefill_ceiling(hw, m, seq_len=s)
        linear = 2.0 * m.active_params() * s
        attn = 4.0 * m.layers * m.n_heads * (s * (s + 1) / 2) * m.head_dim
        assert abs(c.latency_s - (linear + attn) / hw.flops_bf16) / c.latency_s < 1e-9
        d16 = decode_ceiling(hw, m, "bf16", "bf16", 1, 512)
        d4 = decode_ceiling(hw, m, "int4", "bf16", 1, 512)
        assert d4.tokens_per_s > 2 * d16.tokens_per_s


def test_cache_plan_fits_and_refuses():
    from reng.config import llama31_8b, qwen25_32b
    from reng.plan import CachePlan
    p = CachePlan.new(llama31_8b(), batch=64)
    assert p.bytes_per_position_per_layer() == 4096
    p.check(1024)
    cap = p.max_capacity()
    assert p.fits(cap) and not p.fits(cap + 1)
    with pytest.raises(ValueError, match="does not fit"):
        p.check(cap + 1)
    q = CachePlan.new(qwen25_32b(), batch=64)
    q.check(4352)                                   # the Qwen b64 4096+256 config
    assert CachePlan.new(qwen25_32b(), weights="fp8").weight_bytes < q.weight_bytes


def test_cache_plan_counts_the_engines_work_buffers():
    """The plan's work buffers are the engine's: 1024-row prefill blocks,
    whose bf16 logits dominate (Llama-8B: 1024 x 128256 x 2 = 263 MB)."""
    from reng.config import llama31_8b
    from reng.plan import BLOCK_ROWS, CachePlan
    cfg = llama31_8b()
    p = CachePlan.new(cfg, batch=1)
    work = p.transient_bytes_at(0)
    logits = BLOCK_ROWS * cfg.vocab_size * 2
    assert logits < work < logits + (200 << 20)
    assert p.transient_bytes_at(1000) - work == 1000 * 4   # the id ring: one u32 per step and slot
