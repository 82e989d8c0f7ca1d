"""The command-line tools end to end on a small checkpoint written in the
HF layout (config.json + model.safetensors), against references the f32
host forward writes in the formats the reference's tools read
(tools/oracle/generate.py's `generated` + per-step top candidates for
`reng-generate --ref`; `argmax` / `last_logits` / `last_top5` for
`reng-prefill --ref`)."""
import json
import os

import numpy as np
import pytest

from test_decode_gpu import oracle_for, small_cfg

pytestmark = pytest.mark.gpu

PROMPT = [5, 17, 300, 2, 999, 41, 7]


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory, reng_lib):
    from reng.weights import random_weights, save_checkpoint
    d = str(tmp_path_factory.mktemp("ckpt"))
    cfg = small_cfg()
    w = random_weights(cfg, seed=44)
    save_checkpoint(d, cfg, w)
    return d, cfg, w


def _oracle_generate_ref(cfg, w, prompt, n, path):
    """Greedy f32 generation with each step's top candidates (the
    generate.py reference format)."""
    from reng.rope import rope_caches_for
    orc = oracle_for(cfg, w)
    sin, cos = rope_caches_for(cfg, len(prompt) + n + 1)
    seq, gen, steps = list(prompt), [], []
    for _ in range(n):
        lg = orc.forward(np.asarray(seq, np.uint32), sin, cos, logits_from=len(seq) - 1)[0]
        order = np.argsort(-lg.astype(np.float64), kind="stable")[:8]
        steps.append({"top1": int(order[0]), "top2": int(order[1]),
                      "margin": float(lg[order[0]] - lg[order[1]]),
                      "top_ids": [int(x) for x in order], "top_logits": [float(lg[x]) for x in order]})
        gen.append(int(order[0]))
        seq.append(int(order[0]))
    with open(path, "w") as f:
        json.dump({"prompt": list(prompt), "generated": gen, "steps": steps}, f)
    return gen


def test_generate_teacher_forced_against_the_oracle(ckpt, tmp_path, capsys):
    from reng import cli
    d, cfg, w = ckpt
    ref = str(tmp_path / "ref.json")
    _oracle_generate_ref(cfg, w, PROMPT, 8, ref)
    out = str(tmp_path / "out.json")
    assert cli.generate_main([d, out, "8", "--ref", ref, "--capacity", "64"] + [str(x) for x in PROMPT]) == 0
    assert "PASS" in capsys.readouterr().out
    doc = json.load(open(out))
    assert doc["teacher_forced"] is True and doc["kv_cache"] is True
    assert doc["prompt"] == PROMPT and len(doc["generated"]) == 8 and len(doc["step_seconds"]) == 8


def test_generate_free_running_batch_and_recompute(ckpt, tmp_path):
    from reng import cli
    d, cfg, w = ckpt
    ref = str(tmp_path / "ref.json")
    want = _oracle_generate_ref(cfg, w, PROMPT, 6, ref)
    out = str(tmp_path / "out.json")
    ids = [str(x) for x in PROMPT]
    assert cli.generate_main([d, out, "6", "--batch", "3", "--capacity", "64"] + ids) == 0
    doc = json.load(open(out))
    assert doc["batch"] == 3 and all(s == doc["sequences"][0] for s in doc["sequences"])
    out2 = str(tmp_path / "out2.json")
    assert cli.generate_main([d, out2, "6", "--recompute"] + ids) == 0
    doc2 = json.load(open(out2))
    assert doc2["kv_cache"] is False
    # both follow the f32 greedy ids unless a step is a near-tie there
    steps = json.load(open(ref))["steps"]
    for gen in (doc["generated"], doc2["generated"]):
        for t, (g, e) in enumerate(zip(gen, want)):
            if g != e:
                assert cli.RefStep(steps[t]).near_tie(g, 0.5), (t, g, e)
                break


def test_prefill_against_the_oracle(ckpt, tmp_path, capsys):
    from reng import cli
    from reng.rope import rope_caches_for
    d, cfg, w = ckpt
    prompt = PROMPT * 5
    sin, cos = rope_caches_for(cfg, len(prompt))
    lg = oracle_for(cfg, w).forward(np.asarray(prompt, np.uint32), sin, cos)
    ref = str(tmp_path / "ref.json")
    with open(ref, "w") as f:
        json.dump({"argmax": [int(x) for x in np.argmax(lg, 1)], "last_logits": [float(x) for x in lg[-1]],
                   "last_top5": [int(x) for x in np.argsort(-lg[-1].astype(np.float64), kind="stable")[:5]]}, f)
    out = str(tmp_path / "out.json")
    assert cli.main(["prefill", d, out, "--ref", ref, "--rows", "16"] + [str(x) for x in prompt]) == 0
    assert "PASS" in capsys.readouterr().out
    doc = json.load(open(out))
    assert doc["tokens"] == len(prompt) and len(doc["argmax"]) == len(prompt)
    assert len(doc["last_logits"]) == cfg.vocab_size and len(doc["last_top5"]) == 5


def test_fp8_quantize_report(ckpt, capsys):
    from reng import cli
    d, cfg, _ = ckpt
    assert cli.fp8_quantize_main([d, "--per-matrix", "--layers", "2"]) == 0
    text = capsys.readouterr().out
    assert "projection bytes" in text and "fp8: 14 matrices" in text
    assert sum(1 for ln in text.splitlines() if ln.startswith("  l")) == 14


def test_fp8_generate_runs_e4m3(ckpt, tmp_path, monkeypatch):
    from reng import cli
    d, _, _ = ckpt
    out = str(tmp_path / "out.json")
    assert cli.generate_main([d, out, "4", "--fp8"] + [str(x) for x in PROMPT]) == 0
    assert len(json.load(open(out))["generated"]) == 4
    monkeypatch.setenv("RENG_FP8", "e5m2")
    assert cli.main(["generate", d, out, "4"] + [str(x) for x in PROMPT]) == 1


def test_bench_writes_the_chart_entries(ckpt, tmp_path):
    from reng import cli
    d, _, _ = ckpt
    out = str(tmp_path / "bench.json")
    assert cli.bench_main([d, out, "--prompt", "32", "--new", "16", "--batch", "2", "--warmup", "1",
                           "--capacity", "64"]) == 0
    doc = json.load(open(out))
    assert [e["unit"] for e in doc] == ["tok/s", "%", "tok/s", "%"]
    assert doc[2]["name"].endswith("decode tok/s (b2)") and doc[2]["value"] > 0


def test_tp_two_ranks_agree(ckpt, tmp_path, capsys):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from reng import cli
    d, _, _ = ckpt
    out = str(tmp_path / "tp.json")
    rc = cli.tp_main([d, "6"] + [str(x) for x in PROMPT] +
                     ["--modules", "0,1", "--batch", "2", "--bench", "8", "--out", out, "--timeout", "600"])
    text = capsys.readouterr().out
    assert rc == 0, text[-3000:]
    assert "VERDICT: PASS" in text and "all 2 ranks agree" in text
    doc = json.load(open(out))
    assert doc["world"] == 2 and doc["ranks_agree"] and len(doc["sequences"]) == 2
    assert doc["bench"]["exchange_ms"] > 0
