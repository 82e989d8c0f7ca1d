"""GPU parity of the decode path against the f32 host forward (the oracle).

The reference's bar (crates/reng-synapse/src/bin/cache_test.rs:437,
batch_test.rs:487; tools/oracle method): per-position logits within rel-L2
0.05 of the f32 forward, last-position cosine >= 0.999, and greedy ids equal
to the oracle's except at bf16 near-ties, where the engine's pick must be
within MARGIN logits of the oracle's best (generate.rs:30, default 0.5).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

COS_MIN = 0.999
REL_L2_MAX = 0.05
MARGIN = 0.5


def small_cfg(bias=False, **kw):
    from reng.config import LlamaConfig
    d = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
             num_key_value_heads=2, head_dim_=64, vocab_size=1024, rms_norm_eps=1e-5,
             rope_theta=10000.0, tie_word_embeddings=False, attention_bias=bias,
             model_type="qwen2" if bias else "llama")
    d.update(kw)
    return LlamaConfig(**d)


def oracle_for(cfg, w):
    import oracle
    from reng.weights import to_host
    h = to_host(w)
    c = dict(hidden=cfg.hidden_size, inter=cfg.intermediate_size, n_layers=len(h["layers"]),
             n_heads=cfg.num_attention_heads, n_kv_heads=cfg.n_kv_heads(), head_dim=cfg.head_dim(),
             vocab=cfg.vocab_size, eps=cfg.rms_norm_eps, attn_scale=cfg.attention_scale(),
             has_bias=int(cfg.has_bias()))
    return oracle.Model(c, h["layers"], h["final_gamma"], h["lm_head"], h["embed"])


def cosine(a, b):
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def rel_l2(got, want):
    return float(np.linalg.norm(got.astype(np.float64) - want) / np.linalg.norm(want))


def check_rows(got, want, what):
    for i in range(want.shape[0]):
        assert rel_l2(got[i], want[i]) < REL_L2_MAX, (what, i, rel_l2(got[i], want[i]))
        assert cosine(got[i], want[i]) >= COS_MIN, (what, i, cosine(got[i], want[i]))
        gi = int(np.argmax(got[i]))
        wi = int(np.argmax(want[i]))
        if gi != wi:
            assert want[i][wi] - want[i][gi] < MARGIN, (what, i, gi, wi)


def check_greedy(ids_engine, oracle_logits):
    """ids_engine[t] is the engine's pick after position t; oracle_logits[t]
    the f32 logits there (teacher-forced on the engine's own ids)."""
    ties = 0
    for t, e in enumerate(ids_engine):
        best = int(np.argmax(oracle_logits[t]))
        if best != e:
            gap = oracle_logits[t][best] - oracle_logits[t][e]
            assert gap < MARGIN, (t, e, best, gap)
            ties += 1
    return ties


@pytest.fixture(scope="module")
def lib(reng_lib):
    return reng_lib


@pytest.mark.parametrize("bias", [False, True])
def test_prefill_logits_match_the_oracle(lib, bias):
    from reng.model import Generator
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = small_cfg(bias=bias)
    w = random_weights(cfg, seed=7)
    ids = prompt_ids(21, cfg.vocab_size, seed=3)
    g = Generator(w, cfg, capacity=128)
    got = g.feed_all(ids)
    sin, cos = rope_caches_for(cfg, 128)
    want = oracle_for(cfg, w).forward(ids, sin, cos)
    check_rows(got, want, "prefill")
    assert g.position() == ids.size
    g.close()


def test_greedy_decode_matches_the_teacher_forced_oracle(lib):
    from reng.model import Generator
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = small_cfg()
    w = random_weights(cfg, seed=11)
    prompt = prompt_ids(17, cfg.vocab_size, seed=5)
    g = Generator(w, cfg, capacity=128)
    nxt = g.feed_id(prompt)
    out = g.generate(nxt, 24)
    assert g.position() == prompt.size + 24
    seq = np.concatenate([prompt, [nxt], out[:-1]]).astype(np.uint32)
    sin, cos = rope_caches_for(cfg, 128)
    want = oracle_for(cfg, w).forward(seq, sin, cos, logits_from=prompt.size - 1)
    check_greedy([nxt] + out, want)
    # reset replays the same ids (the stale cache is masked by the position)
    g.reset()
    assert g.position() == 0
    assert g.feed_id(prompt) == nxt
    assert g.generate(nxt, 24) == out
    g.close()


@pytest.mark.parametrize("ring", ["1", "0"])
def test_long_context_decode_attention(lib, monkeypatch, ring):
    """Decode attention over 1100+ cached positions: the TMA-ring kernel
    (engines of 2048+ positions run it) and the per-row kernel, each against
    the f32 forward teacher-forced on the engine's ids; 2 query heads per
    group at head_dim 64, 8 key slices of ~140 keys (3 tiles each)."""
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    monkeypatch.setenv("RENG_ATTN_RING", ring)
    cfg = small_cfg(bias=True)
    w = random_weights(cfg, seed=13)
    cap = 1200
    prompt = prompt_ids(1100, cfg.vocab_size, seed=6)
    e = Engine(cfg, w, batch=1, capacity=cap)
    nxt, _, _ = e.prefill(0, prompt)
    seq = list(prompt) + [nxt]
    got = []
    for _ in range(6):
        lg, n = e.step_logits([seq[-1]])
        got.append(lg[0])
        seq.append(int(n[0]))
    ids = [int(x) for x in e.decode([seq[-1]], 8)[:, 0]]
    e.close()
    sin, cos = rope_caches_for(cfg, cap)
    orc = oracle_for(cfg, w)
    want = orc.forward(np.array(seq[:-1], np.uint32), sin, cos, logits_from=prompt.size)
    check_rows(np.array(got), want, "step")
    full = np.array(seq + ids[:-1], np.uint32)
    want2 = orc.forward(full, sin, cos, logits_from=len(seq) - 1)
    check_greedy(ids, want2)


def test_decode_step_logits_match(lib):
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = small_cfg(bias=True)
    w = random_weights(cfg, seed=2)
    prompt = prompt_ids(9, cfg.vocab_size, seed=1)
    e = Engine(cfg, w, batch=1, capacity=64)
    nxt, _, _ = e.prefill(0, prompt)
    seq = list(prompt) + [nxt]
    got = []
    for _ in range(6):
        lg, n = e.step_logits([seq[-1]])
        got.append(lg[0])
        seq.append(int(n[0]))
    sin, cos = rope_caches_for(cfg, 64)
    want = oracle_for(cfg, w).forward(np.array(seq[:-1], np.uint32), sin, cos,
                                      logits_from=prompt.size)
    check_rows(np.array(got), want, "step")
    e.close()


@pytest.mark.parametrize("batch", [2, 8])
def test_batched_decode_with_staggered_prompts(lib, batch):
    from reng.model import BatchedGenerator
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = small_cfg()
    w = random_weights(cfg, seed=4)
    cap = 96
    g = BatchedGenerator(w, cfg, batch, capacity=cap)
    prompts = [prompt_ids(12 - (b % 3), cfg.vocab_size, seed=100 + b) for b in range(batch)]
    seeds = [g.prefill_id(b, prompts[b]) for b in range(batch)]
    n = 10
    ids = np.array(g.generate(seeds, n)).reshape(n, batch)
    sin, cos = rope_caches_for(cfg, cap)
    orc = oracle_for(cfg, w)
    for b in range(batch):
        assert g.position(b) == prompts[b].size + n
        seq = np.concatenate([prompts[b], [seeds[b]], ids[:-1, b]]).astype(np.uint32)
        want = orc.forward(seq, sin, cos, logits_from=prompts[b].size - 1)
        check_greedy([seeds[b]] + list(ids[:, b]), want)
    g.close()


def test_smollm2_shape_full_depth(lib):
    from reng.config import smollm2_135m
    from reng.model import Generator
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = smollm2_135m()
    w = random_weights(cfg, seed=0)
    prompt = prompt_ids(32, cfg.vocab_size, seed=0)
    g = Generator(w, cfg, capacity=256)
    last = g.feed(prompt)
    nxt = int(np.argmax(last))
    out = g.generate(nxt, 16)
    seq = np.concatenate([prompt, [nxt], out[:-1]]).astype(np.uint32)
    sin, cos = rope_caches_for(cfg, 256)
    want = oracle_for(cfg, w).forward(seq, sin, cos, logits_from=prompt.size - 1)
    assert cosine(last, want[0]) >= COS_MIN
    check_greedy([nxt] + out, want)
    g.close()


def test_llama8b_shape_two_layers(lib):
    """The Llama-3.1-8B widths (hidden 4096, GQA 32/8, hd 128, inter 14336,
    vocab 128256) on a layer-truncated model."""
    from reng.config import llama31_8b
    from reng.model import Generator
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = llama31_8b()
    w = random_weights(cfg, seed=1, layers=2)
    cfg.num_hidden_layers = 2
    prompt = prompt_ids(12, cfg.vocab_size, seed=9)
    g = Generator(w, cfg, capacity=128)
    last = g.feed(prompt)
    nxt = int(np.argmax(last))
    out = g.generate(nxt, 6)
    seq = np.concatenate([prompt, [nxt], out[:-1]]).astype(np.uint32)
    sin, cos = rope_caches_for(cfg, 128)
    want = oracle_for(cfg, w).forward(seq, sin, cos, logits_from=prompt.size - 1)
    assert cosine(last, want[0]) >= COS_MIN
    assert rel_l2(last, want[0]) < REL_L2_MAX
    check_greedy([nxt] + out, want)
    g.close()


def test_errors_are_reported_not_aborted(lib):
    from reng._lib import RengError
    from reng.model import Engine
    from reng.weights import random_weights
    cfg = small_cfg()
    w = random_weights(cfg, seed=1)
    e = Engine(cfg, w, batch=1, capacity=16)
    with pytest.raises(RengError):
        e.prefill(0, np.arange(17, dtype=np.uint32))       # overflows the capacity
    with pytest.raises(RengError):
        e.prefill(0, np.array([cfg.vocab_size], np.uint32))  # id out of range
    with pytest.raises(RengError):
        e.prefill(1, np.array([1], np.uint32))              # no such slot
    e.prefill(0, np.arange(10, dtype=np.uint32))
    with pytest.raises(RengError):
        e.decode([1], 7)                                    # 10 + 7 > 16
    assert e.position(0) == 10
    e.close()


@pytest.mark.parametrize("batch,fp8", [(8, False), (3, False), (8, True), (2, False)])
def test_register_fragment_gemv_equals_shared_memory_gemv(lib, monkeypatch, batch, fp8):
    """At 2..8 rows the Llama-8B-width q/k/v, o_proj and gate/up projections
    (and the LM head) run on the register-fragment GEMV (gemv8.cu).  It
    splits k over the warps and adds their slices in the same order as the
    shared-memory GEMV (RENG_GEMV8=0), so the layers' outputs are
    bit-identical; with RENG_GEMV8=0 the bf16 LM head at 4..8 rows runs on
    the tcgen05 GEMM, and at 2 rows the shared-memory GEMV splits k over 4
    warps, not 8: f32 sums in another order there (logits within 1% of the
    row's largest, the same greedy ids)."""
    from reng.config import llama31_8b
    from reng.model import Engine
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = llama31_8b()
    w = random_weights(cfg, seed=3, layers=2)
    cfg.num_hidden_layers = 2
    q = ("e4m3", "pcs") if fp8 else None
    monkeypatch.setenv("RENG_GEMV8", "0")
    ref = Engine(cfg, w, batch=batch, capacity=64, fp8=q)
    monkeypatch.delenv("RENG_GEMV8")
    eng = Engine(cfg, w, batch=batch, capacity=64, fp8=q)
    # prompt lengths 3..9 and 11: no prefill block of 2 rows (FP8 prefill
    # runs 8-row blocks; at 2 rows the two paths split k differently)
    prompts = [prompt_ids(3 + b if b < 7 else 11, cfg.vocab_size, seed=70 + b) for b in range(batch)]
    seeds = [ref.prefill(b, prompts[b])[0] for b in range(batch)]
    assert seeds == [eng.prefill(b, prompts[b])[0] for b in range(batch)]
    ids = list(seeds)
    for _ in range(3):
        la, na = ref.step_logits(ids)
        lb, nb = eng.step_logits(ids)
        if 3 <= batch < 4 or fp8:
            assert np.array_equal(la, lb)
        else:  # the same f32 dot products summed in another order, then rounded to bf16
            for b in range(batch):
                assert np.max(np.abs(la[b] - lb[b])) <= 2e-2 * np.max(np.abs(la[b]))
                assert cosine(la[b], lb[b]) > 0.9999
                if na[b] != nb[b]:  # only at a near-tie
                    assert abs(la[b][na[b]] - la[b][nb[b]]) < 0.1
        if 3 <= batch < 4 or fp8:
            assert np.array_equal(na, nb)
        ids = [int(x) for x in na]
    assert np.array_equal(eng.decode(ids, 3), ref.decode(ids, 3))
    ref.close()
    eng.close()


FAMILY_CASES = {
    # Granite: every multiplier, folded by the loader (residual into o/down,
    # 1/logits_scaling into the head), attention scale into wq, embedding
    # scale at the gather
    "granite": dict(model_type="granite", embedding_multiplier=12.0, attention_multiplier=0.0625,
                    residual_multiplier=0.25, logits_scaling=8.0),
    # Phi-3 with half the head dims rotated: q/k head dims permuted into the
    # kernels' pair order, identity RoPE entries on the pass-through pairs
    "phi3": dict(model_type="phi3", partial_rotary_factor=0.5),
    # SmolLM3: layer 1 applies no rotary embedding (the q/k/v launch
    # rotates with the identity table there)
    "smollm3": dict(model_type="smollm3", no_rope_layers=[1, 0], use_sliding_window=False),
}


@pytest.mark.parametrize("fam", sorted(FAMILY_CASES))
def test_loaded_family_checkpoint_matches_the_oracle(lib, fam, tmp_path):
    """A checkpoint of the family written in its HF layout, read back by
    load_weights: prefill logits and greedy decode on the engine against
    the f32 oracle with the reference's per-family settings
    (oracle.Model.for_config, pinned to transformers for these families)."""
    import oracle
    from reng.config import LlamaConfig
    from reng.model import Generator
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import load_weights, random_weights, save_checkpoint
    d = dict(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
             num_key_value_heads=2, head_dim=64, vocab_size=1024, rms_norm_eps=1e-5,
             rope_theta=10000.0, tie_word_embeddings=False, max_position_embeddings=4096)
    d.update(FAMILY_CASES[fam])
    cfg0 = LlamaConfig.from_dict(d)
    save_checkpoint(str(tmp_path), cfg0, random_weights(cfg0, seed=31))
    cfg = LlamaConfig.load(str(tmp_path))
    assert cfg.unsupported(capacity=128) == []
    w = load_weights(str(tmp_path), cfg)
    orc = oracle.Model.for_config(cfg, w)
    sin, cos = rope_caches_for(cfg, 128)
    ids = prompt_ids(19, cfg.vocab_size, seed=8)
    g = Generator(w, cfg, capacity=128)
    check_rows(g.feed_all(ids), orc.forward(ids, sin, cos), fam + " prefill")
    g.reset()
    nxt = g.feed_id(ids)
    out = g.generate(nxt, 12)
    seq = np.concatenate([ids, [nxt], out[:-1]]).astype(np.uint32)
    check_greedy([nxt] + out, orc.forward(seq, sin, cos, logits_from=ids.size - 1))
    g.close()
