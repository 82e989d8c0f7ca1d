"""The reference's command-line tools over this engine, with their flags and
JSON outputs (crates/reng-model/src/bin/*.rs):

    reng-generate <model_dir> <out.json> <n_new> [--ref <ref.json>] [--margin <f32>]
                  [--rows <n>] [--decode-rows <n>] [--capacity <n>] [--recompute]
                  [--batch <n>] [--fp8] <id> [<id> ...]                     (generate.rs)
    reng-prefill  <model_dir> <out.json> [--ref <ref.json>] [--fp8] [--cached]
                  [--rows <n>] [--batch <n>] <id> [<id> ...]                 (prefill.rs)
    reng-fp8-quantize <model_dir> [--fp8 <spec>] [--per-matrix] [--layers <n>] (fp8_quantize.rs)
    reng-bench    <model_dir> <out.json> [--prompt <n>] [--new <n>] [--rows <n>]
                  [--decode-rows <n>] [--capacity <n>] [--warmup <n>] [--batch <n>]
                  [--stagger <k>] [--fp8]                                   (bench.rs)
    reng-tp       <model_dir> <n_new> [<id> ...] --modules 0,1 [--prompt-file <json>]
                  [--ref <ref.json>] [--margin <f32>] [--rows <n>] [--capacity <n>]
                  [--batch <n>] [--bench <tokens>] [--out <out.json>] [--timeout <s>]
                  [--fp8]                                                   (tp.rs)

Installed as console scripts (pyproject.toml), or run as
`python -m reng.cli <generate|prefill|fp8-quantize|bench|tp> ...`.

Differences from the reference, each a consequence of the device: the
engine always prefills through its KV cache in blocks of `--rows` (there is
no one-recipe prefill to fall back from, so `--cached` is accepted and
changes nothing); `--decode-rows` is accepted for compatibility (decode
always runs one row per slot); `--batch` is accepted by generate and prefill
as well (every slot takes the prompt, as reng-tp's `--batch`); FP8 weights
are E4M3 with per-channel scales (the engine's device format: another
`RENG_FP8` format is refused, never run as something else), and reng-tp
accepts `--fp8` because each rank quantizes its own shard on its device.
reng-tp's `--ifname` / `--no-numa` (HCCL sideband interface, NUMA binding)
have no counterpart: NCCL picks its transport itself.  Errors print one
line to stderr and exit with status 1, as the reference's `Result` mains do.
"""
import json
import os
import sys
import time

import numpy as np

DEFAULT_MARGIN = 0.5      # generate.rs:30
DEFAULT_ROWS = 256        # generate.rs:31
DEFAULT_CAPACITY = 1024   # generate.rs:33


class UsageError(Exception):
    pass


FROM_ENV = object()  # the `env` default of the parsers: read RENG_FP8 (None: unset)


# ----------------------------------------------------------------- shared --

class RefStep:
    """One step of a generate.py reference (generate.rs:36-60)."""

    def __init__(self, d):
        self.top1 = int(d.get("top1", 0))
        self.top2 = int(d.get("top2", 0))
        self.margin = float(d.get("margin", float("nan")))
        self.top_ids = [int(x) for x in d.get("top_ids", [])]
        self.top_logits = [float(x) for x in d.get("top_logits", [])]

    def near_tie(self, tok, margin):
        """Whether `tok` is within `margin` logits of the reference's best."""
        if not self.top_ids:
            return self.margin < margin and tok in (self.top1, self.top2)
        best = self.top_logits[0]
        return any(t == tok and best - l < margin for t, l in zip(self.top_ids, self.top_logits))


class Reference:
    def __init__(self, d):
        self.generated = [int(x) for x in d["generated"]]
        self.steps = [RefStep(s) for s in d.get("steps", [])]
        self.prompt = [int(x) for x in d.get("prompt", [])]

    @staticmethod
    def load(path):
        try:
            with open(path) as f:
                return Reference(json.load(f))
        except (OSError, ValueError, KeyError) as e:
            raise UsageError("%s: %s" % (path, e))


def verdict(ref, step, last, margin, secs, tally, failures, out=print):
    """Compare the engine's pick at `step` with the reference (generate.rs:
    150-190): a match, a near-tie (counted) or a divergence (recorded)."""
    want = ref.generated[step]
    s = ref.steps[step] if step < len(ref.steps) else None
    if last == want:
        v = "match"
    elif s is not None and s.near_tie(last, margin):
        tally["near_ties"] += 1
        v = "near-tie"
    else:
        failures.append("step %d: got %d, want %d%s" % (
            step, last, want, " (ref margin %.3f)" % s.margin if s is not None else ""))
        v = "DIVERGE"
    out("step %d: engine %d  ref %d  margin %.3f  %s  (%.1f ms)" % (
        step, last, want, s.margin if s is not None else float("nan"), v, secs * 1e3))


def parse_fp8(args, env=FROM_ENV):
    """The `--fp8` flag and the RENG_FP8 variable (take_fp8_flag +
    fp8_switch, reng-model lib.rs:1693-1782).  Returns (args without the
    flag, None or (format, scheme)); a format the engine cannot run is an
    error, not a silent bf16 run."""
    from .model import fp8_switch
    flag = "--fp8" in args
    rest = [a for a in args if a != "--fp8"]
    env = os.environ.get("RENG_FP8") if env is FROM_ENV else env
    try:
        sw = fp8_switch(env, flag)
    except ValueError as e:
        raise UsageError(str(e))
    if sw is not None and (sw != ("e4m3", "pcs") or sw.backoff != 1.0):
        raise UsageError("RENG_FP8 %s: this engine's FP8 weights are e4m3 with per-channel "
                         "scales (pcs) and backoff 1" % (sw,))
    return rest, sw


def take_opts(args, start, spec, usage):
    """Flags from args[start:] while they start with '--' (a value after
    each, except the names in spec['bool']).  Returns (opts, next index)."""
    opts, i = {}, start
    while i < len(args) and args[i].startswith("--"):
        name = args[i][2:]
        if name in spec.get("bool", ()):
            opts[name] = True
            i += 1
            continue
        if name not in spec["value"]:
            raise UsageError("unknown flag %s\n%s" % (args[i], usage))
        if i + 1 >= len(args):
            raise UsageError(usage)
        opts[name] = args[i + 1]
        i += 2
    return opts, i


def num(opts, name, default, kind=int, minimum=None):
    if name not in opts:
        return default
    try:
        v = kind(opts[name])
    except ValueError as e:
        raise UsageError("%s: %s" % (name, e))
    if minimum is not None and v < minimum:
        raise UsageError("--%s needs a number of at least %s" % (name, minimum))
    return v


def parse_ids(words):
    try:
        ids = [int(w) for w in words]
    except ValueError as e:
        raise UsageError("token id: %s" % e)
    if any(x < 0 or x >= 1 << 32 for x in ids):
        raise UsageError("token id out of range")
    return ids


def load_model(model_dir):
    from .config import LlamaConfig
    from .weights import load_weights
    t0 = time.perf_counter()
    cfg = LlamaConfig.load(model_dir)
    w = load_weights(model_dir, cfg)
    return cfg, w, time.perf_counter() - t0


def fp8_report_line(cfg, w, fp8):
    """The reference prints its quantization report when FP8 is on
    (generate.rs:207-212); the engine itself quantizes on the device at
    create time with the same rules."""
    from . import fp8 as f
    _, rep = f.quantize_model(w, cfg)
    return "fp8 %s:%s: %s" % (fp8[0], fp8[1], rep)


def write_json(path, obj, pretty=False):
    try:
        with open(path, "w") as fh:
            fh.write(json.dumps(obj, indent=2 if pretty else None))
    except OSError as e:
        raise UsageError("%s: %s" % (path, e))


def top5(row):
    """Indices of the five largest logits, best first (prefill.rs:33-41)."""
    return [int(i) for i in np.argsort(-np.asarray(row, np.float64), kind="stable")[:5]]


def cosine(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-12))


_ROWS_SAVED = []


def _set_rows(rows):
    """RENG_PREFILL_ROWS = --rows when below the reference's default of 256
    (the library reads it at every prefill; at the default the engine runs
    its own blocks of up to 1024 rows); `_run` puts the old value back when
    the command ends, so later engines of the process keep their default."""
    if rows < DEFAULT_ROWS:
        _ROWS_SAVED.append(os.environ.get("RENG_PREFILL_ROWS"))
        os.environ["RENG_PREFILL_ROWS"] = str(rows)


def _restore_rows():
    while _ROWS_SAVED:
        old = _ROWS_SAVED.pop()
        if old is None:
            os.environ.pop("RENG_PREFILL_ROWS", None)
        else:
            os.environ["RENG_PREFILL_ROWS"] = old


# --------------------------------------------------------------- generate --

GEN_USAGE = ("usage: reng-generate <model_dir> <out.json> <n_new> [--ref <ref.json>] [--margin <f32>] "
             "[--rows <n>] [--decode-rows <n>] [--capacity <n>] [--recompute] [--batch <n>] [--fp8] "
             "<id> [<id> ...]")


def parse_generate(argv, env=FROM_ENV):
    args, fp8 = parse_fp8(list(argv), env)
    if len(args) < 4:
        raise UsageError(GEN_USAGE)
    try:
        n_new = int(args[2])
    except ValueError as e:
        raise UsageError("n_new: %s" % e)
    opts, i = take_opts(args, 3, {"value": ("ref", "margin", "rows", "decode-rows", "capacity", "batch"),
                                  "bool": ("recompute",)}, GEN_USAGE)
    ids = parse_ids(args[i:])
    if not ids:
        raise UsageError("no token ids given")
    return {"dir": args[0], "out": args[1], "n_new": n_new, "ref": opts.get("ref"),
            "margin": num(opts, "margin", DEFAULT_MARGIN, float),
            "rows": num(opts, "rows", DEFAULT_ROWS, int, 1),
            "decode_rows": num(opts, "decode-rows", 1, int, 1),
            "capacity": num(opts, "capacity", DEFAULT_CAPACITY, int, 1),
            "batch": num(opts, "batch", 1, int, 1),
            "recompute": bool(opts.get("recompute")), "fp8": fp8, "ids": ids}


def run_generate(a, engine, ref=None, out=print):
    """The generation loop of generate.rs:252-316 over an engine object
    (reng.model.Engine or a stand-in with prefill / decode / reset):
    free-running (one prefill, then the rest of the tokens from one device
    decode call), teacher-forced against `ref` (every step feeds the
    reference's token and compares the engine's pick), or `recompute`
    (every step prefills the whole sequence again into a reset slot).
    Returns (json dict, failures)."""
    B = a["batch"]
    n_new = min(a["n_new"], len(ref.generated)) if ref is not None else a["n_new"]
    prompt = list(a["ids"])
    ids = list(prompt)
    generated = [[] for _ in range(B)]
    step_secs, failures = [], []
    tally = {"near_ties": 0}
    pending = 0
    step = 0
    t_start = time.perf_counter()
    while step < n_new:
        t0 = time.perf_counter()
        if ref is None and step > 0 and not a["recompute"]:
            # the device decode loop: every remaining token from one call
            seeds = [generated[b][-1] for b in range(B)]
            run = engine.decode(seeds, n_new - step)  # [n, B]
            per = (time.perf_counter() - t0) / run.shape[0]
            for row in run:
                step_secs.append(per)
                for b in range(B):
                    generated[b].append(int(row[b]))
                out("step %d: next id %d  (%.1f ms, device loop)" % (step, int(row[0]), per * 1e3))
                step += 1
            break
        if a["recompute"]:
            engine.reset(-1)
            picks = [engine.prefill(b, ids)[0] for b in range(B)]
        else:
            picks = [engine.prefill(b, ids[pending:])[0] for b in range(B)]
        pending = len(ids)
        per = time.perf_counter() - t0
        if step == 0:
            out("first token %.2fs after start" % (time.perf_counter() - t_start))
        step_secs.append(per)
        for b in range(B):
            generated[b].append(int(picks[b]))
        last = int(picks[0])
        if ref is None:
            out("step %d: next id %d  (%.1f ms)" % (step, last, per * 1e3))
            ids.append(last)
        else:
            for b in range(B):
                verdict(ref, step, int(picks[b]), a["margin"], per, tally, failures,
                        out=out if b == 0 else (lambda *_: None))
            ids.append(ref.generated[step])
        step += 1
    doc = {"prompt": prompt, "generated": generated[0], "teacher_forced": ref is not None,
           "kv_cache": not a["recompute"], "step_seconds": step_secs}
    if B > 1:
        doc["batch"] = B
        doc["sequences"] = generated
    out("generated ids: %s" % generated[0])
    if ref is not None:
        exact = sum(1 for g, w in zip(generated[0], ref.generated) if g == w)
        out("vs reference: %d/%d exact, %d near-tie (ref margin < %s), %d diverge" % (
            exact, n_new, tally["near_ties"], a["margin"], len(failures)))
    return doc, failures


def generate_main(argv=None):
    from .model import Engine
    from .plan import CachePlan
    a = parse_generate(sys.argv[1:] if argv is None else argv)
    ref = Reference.load(a["ref"]) if a["ref"] else None
    n_new = min(a["n_new"], len(ref.generated)) if ref is not None else a["n_new"]
    cfg, w, load_s = load_model(a["dir"])
    if a["fp8"]:
        print(fp8_report_line(cfg, w, a["fp8"]))
    print("loaded weights in %.2fs" % load_s)
    plan = CachePlan.new(cfg, batch=a["batch"], weights="fp8" if a["fp8"] else "bf16")
    cap = a["capacity"]
    if a["recompute"]:
        cap = max(cap, len(a["ids"]) + n_new)
    else:
        print(plan.summary(cap))
    msg = cfg.context_warning(len(a["ids"]) + n_new)
    if msg:
        print(msg, file=sys.stderr)
        print(msg)
    if len(a["ids"]) + n_new > cap:
        raise UsageError("a prompt of %d tokens plus %d new tokens exceeds the cache capacity %d "
                         "(--capacity); this model holds up to %d positions"
                         % (len(a["ids"]), n_new, cap, plan.max_capacity()))
    t0 = time.perf_counter()
    _set_rows(a["rows"])
    eng = Engine(cfg, w, batch=a["batch"], capacity=cap, fp8=a["fp8"])
    print("created cached model (rows %d, batch %d, capacity %d): %.2fs"
          % (a["rows"], a["batch"], cap, time.perf_counter() - t0))
    try:
        doc, failures = run_generate(a, eng, ref)
    finally:
        eng.close()
    write_json(a["out"], doc)
    if ref is not None:
        if failures:
            raise UsageError("generation diverges from reference: " + "; ".join(failures))
        print("PASS")
    return 0


# ---------------------------------------------------------------- prefill --

PRE_USAGE = ("usage: reng-prefill <model_dir> <out.json> [--ref <ref.json>] [--fp8] [--cached] "
             "[--rows <n>] [--batch <n>] <id> [<id> ...]")


def parse_prefill(argv, env=FROM_ENV):
    args, fp8 = parse_fp8(list(argv), env)
    if len(args) < 3:
        raise UsageError(PRE_USAGE)
    opts, i = take_opts(args, 2, {"value": ("ref", "rows", "batch"), "bool": ("cached",)}, PRE_USAGE)
    ids = parse_ids(args[i:])
    if not ids:
        raise UsageError("no token ids given")
    return {"dir": args[0], "out": args[1], "ref": opts.get("ref"), "fp8": fp8,
            "cached": bool(opts.get("cached")), "rows": num(opts, "rows", DEFAULT_ROWS, int, 1),
            "batch": num(opts, "batch", 1, int, 1), "ids": ids}


def prefill_report(logits, tokens, secs, ref=None, out=print):
    """The prefill JSON (prefill.rs:201-211) and, against a reference, the
    verdict (prefill.rs:213-235: last-position top-1 equal, cosine > 0.98,
    argmax agreeing on >= 80% of positions).  Returns (json dict, error or
    None)."""
    am = [int(x) for x in np.argmax(logits, axis=1)]
    last = logits[-1]
    t5 = top5(last)
    out("argmax: %s" % am)
    out("last top5: %s" % t5)
    doc = {"argmax": am, "last_logits": [float(x) for x in last], "last_top5": t5, "tokens": tokens,
           "prefill_seconds": secs}
    err = None
    if ref is not None:
        agree = sum(1 for x, y in zip(am, ref["argmax"]) if x == y)
        cos = cosine(last, ref["last_logits"])
        top1 = t5[0] == ref["last_top5"][0]
        out("vs reference: argmax agree %d/%d, last-position top1 %s, last-logits cosine %.4f, ref top5 %s"
            % (agree, tokens, "MATCH" if top1 else "DIFFER", cos, ref["last_top5"]))
        if top1 and cos > 0.98 and agree * 10 >= tokens * 8:
            out("PASS")
        else:
            err = "engine diverges from reference: agree %d/%d, cosine %s" % (agree, tokens, cos)
    return doc, err


def prefill_main(argv=None):
    from .model import Engine
    from .plan import CachePlan
    a = parse_prefill(sys.argv[1:] if argv is None else argv)
    cfg, w, load_s = load_model(a["dir"])
    if a["fp8"]:
        print(fp8_report_line(cfg, w, a["fp8"]))
    print("loaded %d layers, hidden %d, inter %d, heads %d/%d kv, head_dim %d, vocab %d in %.2fs" % (
        cfg.num_hidden_layers, cfg.hidden_size, cfg.intermediate_size, cfg.num_attention_heads,
        cfg.n_kv_heads(), cfg.head_dim(), cfg.vocab_size, load_s))
    tokens = len(a["ids"])
    msg = cfg.context_warning(tokens)
    if msg:
        print(msg, file=sys.stderr)
        print(msg)
    plan = CachePlan.new(cfg, batch=a["batch"], weights="fp8" if a["fp8"] else "bf16")
    print(plan.summary(tokens))
    plan.check(tokens)
    host = 4.0 * cfg.vocab_size * tokens
    if host > 8e9:
        msg = ("warning: %d positions of f32 logits are %.1f GB of host memory in one allocation "
               "(%d bytes a token)" % (tokens, host / 1e9, 4 * cfg.vocab_size))
        print(msg, file=sys.stderr)
        print(msg)
    _set_rows(a["rows"])
    eng = Engine(cfg, w, batch=a["batch"], capacity=tokens, fp8=a["fp8"])
    try:
        t0 = time.perf_counter()
        _, _, logits = eng.prefill(0, a["ids"], all_logits=True)
        for b in range(1, a["batch"]):
            eng.prefill(b, a["ids"])
        dt = time.perf_counter() - t0
    finally:
        eng.close()
    rows = min(a["rows"], DEFAULT_ROWS)
    print("prefill of %d tokens (cached, %d blocks of %d): %.2fs" % (tokens, -(-tokens // rows), rows, dt))
    ref = None
    if a["ref"]:
        try:
            with open(a["ref"]) as f:
                ref = json.load(f)
        except (OSError, ValueError) as e:
            raise UsageError("%s: %s" % (a["ref"], e))
    doc, err = prefill_report(logits, tokens, dt, ref)
    write_json(a["out"], doc)
    if err:
        raise UsageError(err)
    return 0


# ----------------------------------------------------------- fp8-quantize --

FP8Q_USAGE = "usage: reng-fp8-quantize <model_dir> [--fp8 <spec>] [--per-matrix] [--layers <n>]"


def parse_fp8_quantize(argv, env=FROM_ENV):
    """fp8_quantize.rs:30-84: RENG_FP8 first, `--fp8 <spec>` overrides it; an
    off value is an error (the binary has nothing else to do)."""
    from .model import fp8_switch
    argv = list(argv)
    if not argv:
        raise UsageError(FP8Q_USAGE)
    if argv[0].startswith("-"):
        raise UsageError("the model directory comes first, not %r\n%s" % (argv[0], FP8Q_USAGE))
    env = os.environ.get("RENG_FP8") if env is FROM_ENV else env
    try:
        spec = fp8_switch(env, True)
    except ValueError as e:
        raise UsageError(str(e))
    if spec is None:
        raise UsageError("RENG_FP8=%s turns the fp8 switch off and reng-fp8-quantize does nothing else; "
                         "unset it or pass --fp8 <spec>" % (env or ""))
    a = {"dir": argv[0], "fp8": spec, "backoff": spec.backoff, "per_matrix": False, "layers": 1}
    i = 1
    while i < len(argv):
        if argv[i] == "--per-matrix":
            a["per_matrix"] = True
            i += 1
        elif argv[i] in ("--fp8", "--layers"):
            if i + 1 >= len(argv):
                raise UsageError(FP8Q_USAGE)
            v = argv[i + 1]
            if argv[i] == "--fp8":
                a["fp8"], a["backoff"] = _fp8_spec(v)
            else:
                try:
                    a["layers"] = int(v)
                except ValueError as e:
                    raise UsageError("--layers: %s" % e)
            i += 2
        else:
            raise UsageError("unknown flag %s\n%s" % (argv[i], FP8Q_USAGE))
    return a


def _fp8_spec(v):
    """A --fp8 spec, in the RENG_FP8 grammar (format, scheme, backoff=<f32>)."""
    from .model import fp8_switch
    try:
        sw = fp8_switch(v, True)
    except ValueError as e:
        raise UsageError(str(e))
    if sw is None:
        raise UsageError("--fp8 %s: that switch is off" % v)
    return sw, sw.backoff


def fp8_quantize_main(argv=None):
    from . import fp8 as f
    a = parse_fp8_quantize(sys.argv[1:] if argv is None else argv)
    cfg, w, load_s = load_model(a["dir"])
    print("%s: %d layers, hidden %d, intermediate %d, loaded in %.2f s"
          % (a["dir"], cfg.num_hidden_layers, cfg.hidden_size, cfg.intermediate_size, load_s))
    fmt, sch = f.Fp8Format.from_name(a["fp8"][0]), f.Scaling.from_name(a["fp8"][1])
    backoff = a["backoff"]
    print("fp8 scheme: %s:%s backoff %s" % (a["fp8"][0], a["fp8"][1], backoff))
    layers, rep = f.quantize_model(w, cfg, fmt, sch, backoff)
    print("fp8: %s" % rep)
    gib = float(1 << 30)
    after = rep.fp8_bytes + rep.scale_bytes
    print("projection bytes: %.3f GiB -> %.3f GiB (%.2fx, %.3f GiB saved)" % (
        rep.bf16_bytes / gib, after / gib, rep.bf16_bytes / max(after, 1), (rep.bf16_bytes - after) / gib))
    if a["per_matrix"]:
        for li, layer in enumerate(layers[:a["layers"]]):
            for name in f.PROJECTIONS:
                q = layer[name]
                src = np.asarray(w["layers"][li][name], np.uint16).reshape(-1)
                errs = f.sample_row_errors(src, q, f.FP8_ERROR_ROWS)
                mean = sum(e.mean_rel for e in errs) / max(len(errs), 1)
                mx = max([0.0] + [e.max_rel for e in errs])
                absmax = float(np.max(f.row_absmax(src, q.rows, q.cols)))
                print("  l%d %-3s [%d, %d] bias %d absmax %.4f mean_rel %.4f max_rel %.4f"
                      % (li, name[1:], q.rows, q.cols, q.exp_bias, absmax, mean, mx))
    return 0


# ------------------------------------------------------------------ bench --

BENCH_USAGE = ("usage: reng-bench <model_dir> <out.json> [--prompt <tokens>] [--new <tokens>] [--rows <n>] "
               "[--decode-rows <n>] [--capacity <n>] [--warmup <steps>] [--batch <n>] [--stagger <k>] [--fp8]")


def parse_bench(argv, env=FROM_ENV):
    args, fp8 = parse_fp8(list(argv), env)
    if len(args) < 2:
        raise UsageError(BENCH_USAGE)
    a = {"dir": args[0], "out": args[1], "prompt": 128, "new": 64, "rows": 256, "decode_rows": 1,
         "capacity": 1024, "warmup": 4, "batch": 1, "stagger": 0, "fp8": fp8}
    keys = {"--prompt": "prompt", "--new": "new", "--rows": "rows", "--decode-rows": "decode_rows",
            "--capacity": "capacity", "--warmup": "warmup", "--batch": "batch", "--stagger": "stagger"}
    i = 2
    while i + 1 < len(args):
        if args[i] not in keys:
            raise UsageError("unknown flag %s" % args[i])
        try:
            a[keys[args[i]]] = int(args[i + 1])
        except ValueError as e:
            raise UsageError("%s: %s" % (args[i], e))
        i += 2
    if i != len(args):
        raise UsageError(BENCH_USAGE)
    if a["prompt"] < 1 or a["new"] < 1:
        raise UsageError("--prompt and --new must be at least 1")
    if a["stagger"] > a["prompt"]:
        raise UsageError("stagger must leave every sequence at least one prompt token")
    if a["prompt"] + a["new"] > a["capacity"]:
        raise UsageError("prompt + new must fit the cache capacity")
    return a


def fnv1a64(ids):
    """FNV-1a over the ids' little-endian bytes (bench.rs:106-112)."""
    h = 0xcbf29ce484222325
    for x in ids:
        for byte in int(x).to_bytes(4, "little"):
            h = ((h ^ byte) * 0x100000001b3) & 0xFFFFFFFFFFFFFFFF
    return h


def bench_prompt(n, vocab, b=0, stagger=0):
    """bench.rs:165-180: (i * 7919 + 13) % vocab; with --stagger k sequence
    b is its own stream, b % k tokens shorter."""
    if stagger == 0:
        return [(i * 7919 + 13) % vocab for i in range(n)]
    m = n - b % stagger
    return [(i * 7919 + 13 + b * 7) % vocab for i in range(m)]


def bench_main(argv=None):
    from . import ceiling
    from .model import Engine
    from .plan import CachePlan
    t_start = time.perf_counter()
    a = parse_bench(sys.argv[1:] if argv is None else argv)
    cfg, w, load_s = load_model(a["dir"])
    if a["fp8"]:
        print(fp8_report_line(cfg, w, a["fp8"]))
    print("loaded weights in %.2fs" % load_s)
    B = max(a["batch"], 1)
    plan = CachePlan.new(cfg, batch=B, weights="fp8" if a["fp8"] else "bf16")
    print(plan.summary(a["capacity"]))
    msg = cfg.context_warning(a["prompt"] + a["new"])
    if msg:
        print(msg, file=sys.stderr)
        print(msg)
    plan.check(a["capacity"])
    name = os.path.basename(os.path.normpath(a["dir"]))
    t0 = time.perf_counter()
    _set_rows(a["rows"])
    eng = Engine(cfg, w, batch=B, capacity=a["capacity"], fp8=a["fp8"])
    print("%s: %d layers, hidden %d, vocab %d; created batch %d / rows %d / capacity %d in %.2fs (device decode loop)"
          % (name, cfg.num_hidden_layers, cfg.hidden_size, cfg.vocab_size, B, a["rows"], a["capacity"],
             time.perf_counter() - t0))
    first = None
    try:
        prompts = [bench_prompt(a["prompt"], cfg.vocab_size, b, a["stagger"]) for b in range(B)]
        for _ in range(a["warmup"]):
            eng.reset(-1)
            nx = [eng.prefill(b, prompts[b])[0] for b in range(B)]
            if first is None:
                first = time.perf_counter() - t_start
            eng.decode(nx, 1)
        eng.reset(-1)
        t1 = time.perf_counter()
        nx = [eng.prefill(b, prompts[b])[0] for b in range(B)]
        prefill_s = (time.perf_counter() - t1) / B
        if first is None:
            first = time.perf_counter() - t_start
        t2 = time.perf_counter()
        ids = eng.decode(nx, a["new"])
        decode_s = time.perf_counter() - t2
    finally:
        eng.close()
    flat = [int(x) for x in ids.T.reshape(-1)] if B > 1 else [int(x) for x in ids[:, 0]]
    step_ms = decode_s / a["new"] * 1e3
    prefill_tps = a["prompt"] / prefill_s
    decode_tps = B * a["new"] / decode_s
    print("decode ids: %d ids step by step, fnv1a64 %016x, first %s" % (len(flat), fnv1a64(flat), flat[:8]))
    print("first token %.2fs after start (weights loaded in %.2fs)" % (first, load_s))
    hw = ceiling.HardwareSpec.b200_measured()
    shape = ceiling.ModelShape.from_config(cfg, name)
    ctx = a["prompt"] + a["new"] // 2
    prec = "fp8" if a["fp8"] else "bf16"
    c_pre = ceiling.prefill_ceiling(hw, shape, "bf16", "bf16", 1, a["prompt"])
    c_dec = ceiling.decode_ceiling(hw, shape, prec, "bf16", B, ctx)
    pre_pct = 100.0 * prefill_tps / c_pre.tokens_per_s
    dec_pct = 100.0 * decode_tps / c_dec.tokens_per_s
    print("prefill %d tokens: %.4fs = %.0f tok/s  (ceiling %.0f tok/s, %s) = %.2f%%"
          % (a["prompt"], prefill_s, prefill_tps, c_pre.tokens_per_s, c_pre.bottleneck, pre_pct))
    print("decode %d tokens x batch %d at ctx ~%d: %.1f tok/s, mean step %.2f ms  (ceiling %.0f tok/s, %s) = %.2f%%"
          % (a["new"], B, ctx, decode_tps, step_ms, c_dec.tokens_per_s, c_dec.bottleneck, dec_pct))

    def entry(n, unit, value, extra):
        return {"name": "%s %s" % (name, n), "unit": unit, "value": value, "extra": extra}

    doc = [entry("prefill tok/s (b1)", "tok/s", prefill_tps,
                 "%d tokens; ceiling %.0f tok/s" % (a["prompt"], c_pre.tokens_per_s)),
           entry("prefill % of ceiling (b1)", "%", pre_pct, "%s bound" % c_pre.bottleneck),
           entry("decode tok/s (b%d)" % B, "tok/s", decode_tps,
                 "ctx ~%d; mean step %.2f ms; ceiling %.0f tok/s" % (ctx, step_ms, c_dec.tokens_per_s)),
           entry("decode %% of ceiling (b%d)" % B, "%", dec_pct, "%s bound" % c_dec.bottleneck)]
    write_json(a["out"], doc, pretty=True)
    print("wrote %s" % a["out"])
    return 0


# --------------------------------------------------------------------- tp --

TP_USAGE = ("usage: reng-tp <model_dir> <n_new> [<id>...] --modules 0,1 [--prompt-file <json>] "
            "[--ref <ref.json>] [--margin <f32>] [--rows <n>] [--capacity <n>] [--batch <n>] "
            "[--bench <tokens>] [--out <out.json>] [--timeout <s>] [--fp8]")
DEFAULT_TIMEOUT_S = 3600


def parse_tp(argv, env=FROM_ENV):
    """tp.rs:124-240: positional model dir, n_new and ids mixed with flags;
    worker-only flags --rank / --world / --module / --dir."""
    args, fp8 = parse_fp8(list(argv), env)
    o = {"fp8": fp8, "modules": [], "prompt_file": None, "ref": None, "margin": DEFAULT_MARGIN,
         "rows": DEFAULT_ROWS, "capacity": DEFAULT_CAPACITY, "batch": 1, "bench": 0, "out": None,
         "timeout": DEFAULT_TIMEOUT_S, "rank": None, "world": 0, "module": 0, "hand_dir": None}
    pos = []
    i = 0
    intval = {"--rows": "rows", "--capacity": "capacity", "--batch": "batch", "--bench": "bench",
              "--rank": "rank", "--world": "world", "--module": "module"}
    while i < len(args):
        x = args[i]
        if not x.startswith("--"):
            pos.append(x)
            i += 1
            continue
        if i + 1 >= len(args):
            raise UsageError(TP_USAGE)
        v = args[i + 1]
        try:
            if x == "--modules":
                o["modules"] = [int(m) for m in v.split(",") if m.strip()]
            elif x in intval:
                o[intval[x]] = int(v)
            elif x == "--margin":
                o["margin"] = float(v)
            elif x == "--timeout":
                o["timeout"] = float(v)
            elif x == "--prompt-file":
                o["prompt_file"] = v
            elif x == "--ref":
                o["ref"] = v
            elif x == "--out":
                o["out"] = v
            elif x == "--dir":
                o["hand_dir"] = v
            else:
                raise UsageError(TP_USAGE)
        except ValueError:
            raise UsageError(TP_USAGE)
        i += 2
    if len(pos) < 2:
        raise UsageError(TP_USAGE)
    o["dir"] = pos[0]
    try:
        o["n_new"] = int(pos[1])
    except ValueError:
        raise UsageError(TP_USAGE)
    o["ids"] = parse_ids(pos[2:])
    o["batch"] = max(o["batch"], 1)
    if o["rank"] is None and not o["modules"]:
        raise UsageError("--modules is required\n" + TP_USAGE)
    if o["prompt_file"]:
        try:
            with open(o["prompt_file"]) as f:
                pf = json.load(f)
            o["ids"] = [int(x) for x in pf["prompt"]] + o["ids"]
        except (OSError, ValueError, KeyError) as e:
            raise UsageError("%s: %s" % (o["prompt_file"], e))
    if not o["ids"]:
        raise UsageError("no token ids given")
    return o


def compare_ranks(docs):
    """The coordinator's check (tp.rs:604-675): every rank wrote its ids,
    and every rank's sequences equal rank 0's.  Returns (ok, lines)."""
    lines = []
    if any(d is None for d in docs):
        missing = [r for r, d in enumerate(docs) if d is None]
        return False, ["coordinator: no ids from rank(s) %s" % missing]
    first = docs[0]
    lines.append("generated ids: %s" % first["generated"])
    for r, d in enumerate(docs[1:], 1):
        if d["sequences"] != first["sequences"]:
            for b, (x, y) in enumerate(zip(d["sequences"], first["sequences"])):
                if x != y:
                    lines.append("coordinator: rank %d disagrees with rank 0 on sequence %d: %s against %s"
                                 % (r, b, x, y))
                    break
            else:
                lines.append("coordinator: rank %d wrote %d sequences, rank 0 %d"
                             % (r, len(d["sequences"]), len(first["sequences"])))
            return False, lines
    lines.append("coordinator: all %d ranks agree (%d sequences of %d ids)"
                 % (len(docs), len(first["sequences"]), len(first["generated"])))
    return True, lines


def _wait_file(path, timeout, poll=0.05):
    t0 = time.time()
    while not os.path.exists(path):
        if time.time() - t0 > timeout:
            raise UsageError("timed out after %.0f s waiting for %s" % (timeout, path))
        time.sleep(poll)


def tp_worker(o):
    """One rank: joins through the hand-shake directory (rank 0 writes the
    NCCL unique id to id.bin, the others wait for it: hccl.rs:580-637),
    builds its shard, prefills every slot with the prompt, generates (or is
    teacher-forced), writes rank<r>.ids and, with --bench, times decode
    steps and the partial exchange on every rank at once."""
    import ctypes as C
    from . import _lib
    from .model import Engine
    r, W, d = o["rank"], o["world"], o["hand_dir"]
    idp = os.path.join(d, "id.bin")
    if r == 0:
        buf = (C.c_uint8 * 128)()
        _lib.call("reng_tp_unique_id", buf)
        tmp = idp + ".tmp"
        with open(tmp, "wb") as f:
            f.write(bytes(buf))
        os.replace(tmp, idp)
    _wait_file(idp, o["timeout"])
    with open(idp, "rb") as f:
        uid = f.read()
    cfg, w, load_s = load_model(o["dir"])
    cfg.shard(r, W)
    ref = Reference.load(o["ref"]) if o["ref"] else None
    n_new = min(o["n_new"], len(ref.generated)) if ref is not None else o["n_new"]
    cap = max(o["capacity"], len(o["ids"]) + n_new + o["bench"] + 1)
    B = o["batch"]
    quiet = r != 0
    say = (lambda *x: None) if quiet else print
    _set_rows(o["rows"])
    eng = Engine(cfg, w, batch=B, capacity=cap, device=o["module"], tp_rank=r, tp_world=W,
                 nccl_id=uid, fp8=o["fp8"])
    try:
        a = {"batch": B, "n_new": n_new, "ids": o["ids"], "recompute": False, "margin": o["margin"]}
        doc, failures = run_generate(a, eng, ref, out=say)
        seqs = doc.get("sequences", [doc["generated"]])
        ids_doc = {"prompt": o["ids"], "generated": doc["generated"], "sequences": seqs, "batch": B,
                   "teacher_forced": ref is not None, "step_ms": [s * 1e3 for s in doc["step_seconds"]]}
        write_json(os.path.join(d, "rank%d.ids" % r), ids_doc)
        same = sum(1 for s in seqs if s == seqs[0])
        if same != B:
            raise UsageError("rank %d: %d of %d sequences produced sequence 0's ids" % (r, same, B))
        if o["bench"] > 0:
            eng.reset(-1)
            nx = [eng.prefill(b, o["ids"])[0] for b in range(B)]
            t0 = time.perf_counter()
            eng.decode(nx, o["bench"])
            step_ms = (time.perf_counter() - t0) / o["bench"] * 1e3
            xms = eng.time_exchange(iters=64)
            per_layer = 2 * xms
            say("bench: %d steps x batch %d: %.3f ms a step (%.1f tok/s); exchange %.2f us each, "
                "%.3f ms a step (%d per step, %.0f%% of the step)"
                % (o["bench"], B, step_ms, B * 1e3 / step_ms, xms * 1e3, per_layer * cfg.num_hidden_layers,
                   2 * cfg.num_hidden_layers, 100 * per_layer * cfg.num_hidden_layers / step_ms))
            write_json(os.path.join(d, "rank%d.bench" % r),
                       {"step_ms": step_ms, "exchange_ms": xms, "layers": cfg.num_hidden_layers, "batch": B})
        if ref is not None and failures:
            raise UsageError("generation diverges from reference: " + "; ".join(failures))
    finally:
        eng.close()
    return 0


def tp_coordinate(o, argv):
    """Spawns one worker per module in rank order, waits (bounded by
    --timeout), compares the ranks' ids, prints the verdict and writes
    --out (tp.rs:240-330, 604-790)."""
    import shutil
    import subprocess
    import tempfile
    W = len(o["modules"])
    d = tempfile.mkdtemp(prefix="reng-tp-%d-" % os.getpid())
    procs = []
    try:
        for r, m in enumerate(o["modules"]):
            cmd = [sys.executable, "-m", "reng.cli", "tp"] + list(argv) + [
                "--rank", str(r), "--world", str(W), "--module", str(m), "--dir", d]
            env = dict(os.environ)
            env["PYTHONPATH"] = os.path.dirname(os.path.dirname(os.path.abspath(__file__))) + \
                (os.pathsep + env["PYTHONPATH"] if env.get("PYTHONPATH") else "")
            procs.append(subprocess.Popen(cmd, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                                          text=True))
        t0 = time.time()
        outs = [None] * W
        codes = [None] * W
        for r, p in enumerate(procs):
            left = max(1.0, o["timeout"] - (time.time() - t0))
            try:
                outs[r], _ = p.communicate(timeout=left)
                codes[r] = p.returncode
            except subprocess.TimeoutExpired:
                for q in procs:
                    q.kill()
                outs[r], _ = p.communicate()
                codes[r] = "timeout"
        for r in range(W):
            for line in (outs[r] or "").splitlines():
                print("[r%d] %s" % (r, line))
        docs = []
        for r in range(W):
            try:
                with open(os.path.join(d, "rank%d.ids" % r)) as f:
                    docs.append(json.load(f))
            except (OSError, ValueError):
                docs.append(None)
        ok, lines = compare_ranks(docs)
        for line in lines:
            print(line)
        bad = [(r, c) for r, c in enumerate(codes) if c != 0]
        for r, c in bad:
            print("coordinator: rank %d exited with %s" % (r, c))
        verdict_ok = ok and not bad
        if o["out"] and docs[0] is not None:
            out = dict(docs[0])
            out["world"] = W
            out["modules"] = o["modules"]
            out["ranks_agree"] = ok
            try:
                with open(os.path.join(d, "rank0.bench")) as f:
                    out["bench"] = json.load(f)
            except (OSError, ValueError):
                pass
            write_json(o["out"], out)
        print("VERDICT: %s" % ("PASS" if verdict_ok else "FAIL"))
        return 0 if verdict_ok else 1
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
        if not os.environ.get("RENG_TP_KEEP_DIR"):
            shutil.rmtree(d, ignore_errors=True)


def tp_main(argv=None):
    argv = sys.argv[1:] if argv is None else list(argv)
    o = parse_tp(argv)
    if o["rank"] is not None:
        if o["hand_dir"] is None or o["world"] < 1:
            raise UsageError(TP_USAGE)
        return tp_worker(o)
    return tp_coordinate(o, argv)


# ------------------------------------------------------------ entry points --

def _run(fn, argv=None):
    from ._lib import RengError
    try:
        return fn(argv)
    except (UsageError, ValueError, OSError, RengError) as e:
        print("Error: %s" % e, file=sys.stderr)
        return 1
    finally:
        _restore_rows()


def generate():
    sys.exit(_run(generate_main))


def prefill():
    sys.exit(_run(prefill_main))


def fp8_quantize():
    sys.exit(_run(fp8_quantize_main))


def bench():
    sys.exit(_run(bench_main))


def tp():
    sys.exit(_run(tp_main))


COMMANDS = {"generate": generate_main, "prefill": prefill_main, "fp8-quantize": fp8_quantize_main,
            "bench": bench_main, "tp": tp_main}


def main(argv=None):
    argv = sys.argv[1:] if argv is None else list(argv)
    if not argv or argv[0] not in COMMANDS:
        print("usage: python -m reng.cli {%s} ..." % "|".join(COMMANDS), file=sys.stderr)
        return 1
    return _run(COMMANDS[argv[0]], argv[1:])


if __name__ == "__main__":
    sys.exit(main())
