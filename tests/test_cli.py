"""The command-line tools' host logic on the CPU (reng.cli): argument
grammar and refusals of crates/reng-model/src/bin/*.rs, the generation loop
(free-running, teacher-forced, recompute) over a stand-in engine, the
reference comparison verdicts, the prefill report, the bench prompt and
hash, and the reng-tp coordinator's rank check (tp.rs:790-900 restated)."""
import json

import numpy as np
import pytest

from reng import cli
from reng.cli import UsageError


class FakeEngine:
    """The Engine calls the loops make, with a deterministic next-id rule:
    the next id after a sequence is (sum of its ids * 31 + slot) % 97."""

    def __init__(self, batch):
        self.batch = batch
        self.seqs = [[] for _ in range(batch)]
        self.decode_calls = 0

    def _next(self, b):
        return (sum(self.seqs[b]) * 31 + b) % 97

    def reset(self, slot=-1):
        for b in range(self.batch) if slot < 0 else [slot]:
            self.seqs[b] = []

    def prefill(self, slot, ids, last_logits=False, all_logits=False):
        self.seqs[slot] += [int(x) for x in ids]
        return self._next(slot), None, None

    def decode(self, seeds, n):
        self.decode_calls += 1
        out = np.zeros((n, self.batch), np.uint32)
        cur = list(seeds)
        for t in range(n):
            for b in range(self.batch):
                self.seqs[b].append(int(cur[b]))
                cur[b] = self._next(b)
                out[t, b] = cur[b]
        return out


def _gen_args(**kw):
    a = {"batch": 1, "n_new": 6, "ids": [3, 4, 5], "recompute": False, "margin": 0.5}
    a.update(kw)
    return a


def _greedy(ids, n, slot=0):
    seq, out = list(ids), []
    for _ in range(n):
        nx = (sum(seq) * 31 + slot) % 97
        out.append(nx)
        seq.append(nx)
    return out


def test_generate_grammar():
    a = cli.parse_generate(["m", "o.json", "8", "--ref", "r.json", "--margin", "0.25", "--capacity", "64",
                            "--batch", "2", "--recompute", "1", "2", "3"], env=None)
    assert (a["dir"], a["out"], a["n_new"], a["ref"], a["margin"]) == ("m", "o.json", 8, "r.json", 0.25)
    assert (a["capacity"], a["batch"], a["recompute"], a["ids"], a["fp8"]) == (64, 2, True, [1, 2, 3], None)
    assert cli.parse_generate(["m", "o", "2", "--fp8", "7"], env=None)["fp8"] == ("e4m3", "pcs")
    assert cli.parse_generate(["m", "o", "2", "7"], env="1")["fp8"] == ("e4m3", "pcs")
    with pytest.raises(UsageError, match="unknown flag --bogus"):
        cli.parse_generate(["m", "o", "2", "--bogus", "1", "7"], env=None)
    with pytest.raises(UsageError, match="usage"):
        cli.parse_generate(["m", "o", "2"], env=None)
    with pytest.raises(UsageError, match="n_new"):
        cli.parse_generate(["m", "o", "x", "1"], env=None)
    with pytest.raises(UsageError, match="token id"):
        cli.parse_generate(["m", "o", "2", "a"], env=None)
    # a format the engine does not run is refused, never run as bf16
    with pytest.raises(UsageError, match="e4m3"):
        cli.parse_generate(["m", "o", "2", "7"], env="e5m2")
    with pytest.raises(UsageError, match="neither a format"):
        cli.parse_generate(["m", "o", "2", "7"], env="e9m9")
    with pytest.raises(UsageError, match="backoff 1"):
        cli.parse_generate(["m", "o", "2", "7"], env="backoff=0.5")
    # an explicit off value turns a wrapper's --fp8 off
    assert cli.parse_generate(["m", "o", "2", "--fp8", "7"], env="0")["fp8"] is None


def test_free_running_generation_uses_one_decode_call():
    e = FakeEngine(1)
    doc, fails = cli.run_generate(_gen_args(), e, out=lambda *_: None)
    assert fails == [] and e.decode_calls == 1
    assert doc["generated"] == _greedy([3, 4, 5], 6)
    assert doc["prompt"] == [3, 4, 5] and doc["teacher_forced"] is False and doc["kv_cache"] is True
    assert len(doc["step_seconds"]) == 6 and "sequences" not in doc


def test_batched_generation_writes_every_sequence():
    e = FakeEngine(3)
    doc, _ = cli.run_generate(_gen_args(batch=3), e, out=lambda *_: None)
    assert doc["batch"] == 3 and len(doc["sequences"]) == 3
    for b in range(3):
        assert doc["sequences"][b] == _greedy([3, 4, 5], 6, slot=b)


def test_recompute_prefills_the_whole_sequence_each_step():
    e = FakeEngine(1)
    doc, _ = cli.run_generate(_gen_args(recompute=True), e, out=lambda *_: None)
    assert e.decode_calls == 0 and doc["kv_cache"] is False
    assert doc["generated"] == _greedy([3, 4, 5], 6)


def test_teacher_forcing_counts_near_ties_and_divergences():
    # the engine's pick at step t scores prompt ++ ref[..t] (teacher forcing)
    ref_gen, want = [], []
    for t in range(4):
        pick = (sum([3, 4, 5] + ref_gen) * 31) % 97
        want.append(pick)
        # the reference disagrees at step 1 within the margin (a near-tie)
        # and at step 3 by far (a divergence)
        ref_gen.append((pick + {1: 1, 3: 2}.get(t, 0)) % 97)
    steps = [{"top1": g, "top2": g, "margin": 3.0, "top_ids": [g], "top_logits": [5.0]} for g in ref_gen]
    steps[1] = {"top1": ref_gen[1], "top2": want[1], "margin": 0.1,
                "top_ids": [ref_gen[1], want[1]], "top_logits": [5.0, 4.9]}
    ref = cli.Reference({"generated": ref_gen, "steps": steps})
    lines = []
    doc, fails = cli.run_generate(_gen_args(n_new=10), FakeEngine(1), ref, out=lines.append)
    # teacher forcing: at step t the engine scored prompt ++ ref[..t]
    assert doc["teacher_forced"] is True and len(doc["generated"]) == 4
    assert doc["generated"] == want
    assert any("near-tie" in ln for ln in lines) and any("DIVERGE" in ln for ln in lines)
    assert len(fails) == 1 and fails[0].startswith("step 3")
    assert any("1 near-tie" in ln and "1 diverge" in ln for ln in lines)


def test_near_tie_rules():
    old = cli.RefStep({"top1": 5, "top2": 6, "margin": 0.3})
    assert old.near_tie(6, 0.5) and not old.near_tie(7, 0.5) and not old.near_tie(6, 0.2)
    new = cli.RefStep({"top1": 5, "top2": 6, "margin": 0.3, "top_ids": [5, 6, 9],
                       "top_logits": [2.0, 1.7, 1.6]})
    assert new.near_tie(9, 0.5) and not new.near_tie(9, 0.3) and not new.near_tie(4, 10.0)


def test_prefill_grammar_and_report():
    a = cli.parse_prefill(["m", "o.json", "--cached", "--rows", "64", "--ref", "r.json", "5", "6"], env=None)
    assert (a["cached"], a["rows"], a["ref"], a["ids"]) == (True, 64, "r.json", [5, 6])
    with pytest.raises(UsageError, match="no token ids"):
        cli.parse_prefill(["m", "o.json", "--cached"], env=None)
    rng = np.random.default_rng(0)
    logits = rng.standard_normal((4, 50)).astype(np.float32)
    doc, err = cli.prefill_report(logits, 4, 0.5, out=lambda *_: None)
    assert err is None and doc["tokens"] == 4 and doc["prefill_seconds"] == 0.5
    assert doc["argmax"] == [int(x) for x in np.argmax(logits, 1)]
    assert doc["last_top5"] == [int(x) for x in np.argsort(-logits[-1])[:5]]
    assert len(doc["last_logits"]) == 50
    ref = {"argmax": doc["argmax"], "last_logits": doc["last_logits"], "last_top5": doc["last_top5"]}
    assert cli.prefill_report(logits, 4, 0.5, ref, out=lambda *_: None)[1] is None
    bad = dict(ref, last_logits=list(-logits[-1].astype(float)))
    assert "diverges" in cli.prefill_report(logits, 4, 0.5, bad, out=lambda *_: None)[1]


def test_fp8_quantize_grammar():
    a = cli.parse_fp8_quantize(["m"], env=None)
    assert a["fp8"] == ("e4m3", "pcs") and a["layers"] == 1 and not a["per_matrix"]
    a = cli.parse_fp8_quantize(["m", "--fp8", "e5m2,hw,backoff=0.5", "--per-matrix", "--layers", "3"], env=None)
    assert a["fp8"] == ("e5m2", "hw") and a["backoff"] == 0.5 and a["per_matrix"] and a["layers"] == 3
    assert cli.parse_fp8_quantize(["m"], env="e5m2:unit")["fp8"] == ("e5m2", "unit")
    with pytest.raises(UsageError, match="turns the fp8 switch off"):
        cli.parse_fp8_quantize(["m"], env="off")
    with pytest.raises(UsageError, match="comes first"):
        cli.parse_fp8_quantize(["--per-matrix", "m"], env=None)
    with pytest.raises(UsageError, match="unknown flag"):
        cli.parse_fp8_quantize(["m", "--bogus"], env=None)


def test_bench_grammar_prompt_and_hash():
    a = cli.parse_bench(["m", "o.json", "--batch", "8", "--new", "32"], env=None)
    assert (a["batch"], a["new"], a["prompt"], a["capacity"], a["warmup"]) == (8, 32, 128, 1024, 4)
    with pytest.raises(UsageError, match="capacity"):
        cli.parse_bench(["m", "o", "--prompt", "1000", "--new", "100"], env=None)
    with pytest.raises(UsageError, match="stagger"):
        cli.parse_bench(["m", "o", "--prompt", "4", "--stagger", "5"], env=None)
    with pytest.raises(UsageError, match="unknown flag"):
        cli.parse_bench(["m", "o", "--bogus", "5"], env=None)
    assert cli.bench_prompt(3, 1000) == [13, 7932 % 1000, (2 * 7919 + 13) % 1000]
    assert len(cli.bench_prompt(10, 1000, b=3, stagger=4)) == 7
    # FNV-1a 64 over little-endian u32 bytes, against a direct byte loop
    data = b"".join(int(x).to_bytes(4, "little") for x in [1, 2, 70000])
    h = 0xcbf29ce484222325
    for byte in data:
        h = ((h ^ byte) * 0x100000001b3) % (1 << 64)
    assert cli.fnv1a64([1, 2, 70000]) == h
    assert cli.fnv1a64([]) == 0xcbf29ce484222325


def test_tp_grammar(tmp_path):
    pf = tmp_path / "p.json"
    pf.write_text(json.dumps({"prompt": [9, 8]}))
    o = cli.parse_tp(["m", "12", "1", "--modules", "0,1", "--batch", "4", "--bench", "16",
                      "--prompt-file", str(pf), "--out", "o.json"], env=None)
    assert (o["dir"], o["n_new"], o["modules"], o["batch"], o["bench"]) == ("m", 12, [0, 1], 4, 16)
    assert o["ids"] == [9, 8, 1] and o["out"] == "o.json" and o["rank"] is None
    w = cli.parse_tp(["m", "12", "1", "--rank", "1", "--world", "2", "--module", "1", "--dir", "/x"], env=None)
    assert (w["rank"], w["world"], w["module"], w["hand_dir"]) == (1, 2, 1, "/x")
    with pytest.raises(UsageError, match="--modules"):
        cli.parse_tp(["m", "12", "1"], env=None)
    with pytest.raises(UsageError):
        cli.parse_tp(["m", "12", "1", "--modules", "0", "--bogus", "3"], env=None)


def _rank_doc(seqs):
    return {"prompt": [1, 2, 3], "generated": seqs[0], "sequences": seqs, "batch": len(seqs),
            "teacher_forced": False, "step_ms": [1.0]}


def test_coordinator_rank_check():
    a, b = [10, 11, 12], [20, 21, 22]
    ok, lines = cli.compare_ranks([_rank_doc([a, b, a, b])] * 2)
    assert ok and lines[0] == "generated ids: [10, 11, 12]"
    assert lines[1] == "coordinator: all 2 ranks agree (4 sequences of 3 ids)"
    ok, lines = cli.compare_ranks([_rank_doc([a, b]), _rank_doc([a, [20, 21, 23]])])
    assert not ok and "rank 1 disagrees with rank 0 on sequence 1" in lines[-1]
    ok, lines = cli.compare_ranks([_rank_doc([a]), None])
    assert not ok and "no ids from rank(s) [1]" in lines[0]


def test_entry_point_reports_errors_with_status_1(capsys):
    assert cli.main(["generate", "m", "o"]) == 1
    assert "usage: reng-generate" in capsys.readouterr().err
    assert cli.main(["nope"]) == 1
