"""Decode throughput of the B200 path on the BASELINE workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--model llama-3.1-8b|qwen2.5-32b|smollm2-135m] [--batch B]
                    [--weights bf16|fp8] [--prompt 128] [--extras b8,b64,fp8]

Workload (the north-star config): Llama-3.1-8B-shaped
decoder, random-init N(0, 0.02) bf16 weights generated on the device (no
checkpoint), a 128-token uniform-random prompt, then greedy decode at batch 1.
A step is one decode token for every slot: the whole model's weights stream
from HBM once (15 GB > L2, so no step is served from L2).  N > 1 runs the
same model tensor-parallel over N GPUs (strong scaling: the tokens are the
same, the per-GPU work shrinks).

Prints ONE JSON line (rank 0).  `value` is device-timed (CUDA events on the
decode stream around K steps, inputs already in HBM, max over ranks); `e2e`
is the same steps through the public C ABI with host buffers (seed upload and
id readback inside the timed region); `roofline` is the dominant kernel
(gate/up projection) against the measured HBM copy bandwidth; `parity` is a
check made before the timed region: a 2-layer model with the workload's
widths, run the same way (same batch, weights kind and tensor-parallel world),
against the f32 host forward (cosine of the prompt's last logits, greedy ids
under teacher forcing with the 0.5-logit near-tie rule), plus the timed run's
ids compared across ranks; `cpu_baseline` is the CPU restatement of the
reference's f32 host forward on this box's cores; `extra` holds the same
decode measurement at batch 8 and 64 and with FP8 weights at batch 1
(1 GPU, Llama shape), so one run covers BASELINE's b1/b8/b64 metric.
"""
import argparse
import copy
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "reciprocating-engine_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

HBM_FALLBACK_GBS = 6650.0
COS_MIN = 0.999    # last-position cosine against the f32 forward (north star)
MARGIN = 0.5       # near-tie margin in logits (crates/reng-model/src/bin/generate.rs:30)

# dram__bytes_read.sum + dram__bytes_write.sum per launch of the roofline
# kernel, from one ncu capture of that kernel on B200 (same shapes), keyed
# by (model, batch, weights); absent: null in the JSON line
MEASURED_TRAFFIC = {
    ("llama-3.1-8b", 1, "bf16"): 239.2e6,  # gate/up GEMV: 234.95 MB read + 3.8-4.8 MB written (mean of 2)
}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK_GBS, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.p = None

    def start(self):
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.Q,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        try:
            out, _ = self.p.communicate(timeout=5)
        except Exception:
            self.p.kill()
            out = ""
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# --------------------------------------------------------------- CPU arm --

_CPU_MODELS = {}


def cpu_sample(cfg, tokens=32, layers=2, threads=0, seed=0):
    """One timed sample of the oracle (CPU f32 forward restating the
    reference's model_forward_cpu) on a layer-truncated model of the
    workload's widths: per-layer time and LM-head time over `tokens`
    teacher-forced tokens, scaled to the full depth.  The sample model is
    built once per shape (weight generation is not timed).  Returns (tok/s,
    cores, sample description)."""
    import oracle
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    key = (cfg.hidden_size, cfg.intermediate_size, cfg.num_attention_heads, cfg.vocab_size, layers, tokens, seed)
    if key not in _CPU_MODELS:
        w = random_weights(cfg, seed=seed, layers=layers)
        base = dict(hidden=cfg.hidden_size, inter=cfg.intermediate_size, n_heads=cfg.num_attention_heads,
                    n_kv_heads=cfg.n_kv_heads(), head_dim=cfg.head_dim(), vocab=cfg.vocab_size,
                    eps=cfg.rms_norm_eps, attn_scale=cfg.attention_scale(), has_bias=int(cfg.has_bias()))
        _CPU_MODELS[key] = (
            oracle.Model(dict(base, n_layers=layers), w["layers"], w["final_gamma"], w["lm_head"], w["embed"]),
            oracle.Model(dict(base, n_layers=0), [], w["final_gamma"], w["lm_head"], w["embed"]),
            rope_caches_for(cfg, tokens), prompt_ids(tokens, cfg.vocab_size, seed=seed))
    m_layers, m_head, (sin, cos), ids = _CPU_MODELS[key]
    cores = oracle.lib().orc_max_threads() if threads <= 0 else threads
    t0 = time.perf_counter()
    m_layers.forward(ids, sin, cos, logits_from=tokens, threads=threads)
    t1 = time.perf_counter()
    m_head.forward(ids, sin, cos, logits_from=0, threads=threads)
    t2 = time.perf_counter()
    t_full = (t1 - t0) / layers * cfg.num_hidden_layers + (t2 - t1)
    sample = ("f32 host forward (oracle/forward_oracle.c, OpenMP) of a %d-layer model with the "
              "workload's widths over %d teacher-forced tokens (a batched forward, not "
              "token-by-token decode); per-layer time x %d layers + LM head" % (layers, tokens, cfg.num_hidden_layers))
    return tokens / t_full, cores, sample


def cpu_measure(cfg, tokens, warmup, reps):
    """`warmup` untimed samples, then the median of `reps` samples: the same
    procedure for the reference arm and for the cpu_baseline key, so the
    two agree within noise."""
    for _ in range(warmup):
        cpu_sample(cfg, tokens=tokens)
    vals = []
    cores, sample = 0, ""
    for _ in range(reps):
        v, cores, sample = cpu_sample(cfg, tokens=tokens)
        vals.append(v)
    return statistics.median(vals), cores, sample + "; median of %d samples after %d warm-up" % (reps, warmup)


def run_reference(args, cfg):
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    v, cores, sample = cpu_measure(cfg, args.cpu_tokens, args.warmup, args.steps)
    line = {
        "impl": "reference", "metric": "decode tok/s (b%d)" % args.batch, "value": v,
        "unit": "tok/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "strong" if ws > 1 else "weak", "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (random-init N(0,0.02) bf16 weights, uniform-random prompt ids)",
        "config": workload_config(args, ws),
        "cpu_baseline": {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference is Rust for Intel Gaudi2 (no cargo/rustc or Gaudi here); its CPU "
                "path is run as the oracle's C restatement",
    }
    print(json.dumps(line), flush=True)


def workload_config(args, ws):
    return {"workload": "%s%s decode b%d, prompt %d, %d greedy steps%s" % (
        args.model, " fp8" if args.weights == "fp8" else "", args.batch, args.prompt, args.steps,
        ", tensor-parallel %d" % ws if ws > 1 else ""),
        "model": args.model, "batch": args.batch, "prompt": args.prompt, "weights": args.weights,
        "parallelism": "tp%d" % ws if ws > 1 else "single"}


# ------------------------------------------------------------- helpers --

def step_bytes(cfg, B, weights, ws, ctx):
    """Algorithmic HBM bytes of one decode step on one rank: the rank's
    projections (bf16 or E4M3 + one f32 scale per output row), the LM head
    (replicated), and every slot's KV prefix of this rank's heads (the
    reng-ceiling decode formula, crates/reng-ceiling/src/lib.rs:184-207)."""
    head = cfg.hidden_size * cfg.vocab_size
    body = cfg.active_params() - head
    wb = 1 if weights == "fp8" else 2
    rows_per_layer = (cfg.q_dim() + 2 * cfg.n_kv_heads() * cfg.head_dim() + cfg.hidden_size +
                      2 * cfg.intermediate_size + cfg.hidden_size)
    scales = 4 * rows_per_layer * cfg.num_hidden_layers if weights == "fp8" else 0
    return (wb * body + scales) / ws + 2 * head + B * ctx * cfg.kv_bytes_per_token() / ws


def new_unique_id(ws, rank):
    """A fresh NCCL unique id from rank 0 for each tensor-parallel model."""
    if ws == 1:
        return None
    import ctypes as C
    import torch.distributed as dist
    from reng import _lib
    buf = (C.c_uint8 * 128)()
    if rank == 0:
        _lib.call("reng_tp_unique_id", buf)
    obj = [bytes(buf)]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]


def ranks_agree(arr, ws):
    """True when every rank holds the same integer array (all-gather)."""
    if ws == 1:
        return True
    import torch.distributed as dist
    got = [None] * ws
    dist.all_gather_object(got, [int(x) for x in arr.reshape(-1)])
    return all(g == got[0] for g in got)


def dequantized_host(h, ws):
    """Host weights with every projection replaced by its E4M3 per-channel
    round trip in bf16, quantized the way a rank of a `ws`-way model
    quantizes its shard: q/k/v/gate/up by whole rows (a row's scale is the
    same in any row split), o_proj/down_proj per column window (each rank
    quantizes its own window, so a row has one scale per window)."""
    import numpy as np
    import oracle
    from reng.synth import f32_to_bf16_bits
    out = {"embed": h["embed"], "lm_head": h["lm_head"], "final_gamma": h["final_gamma"], "layers": []}
    for lw in h["layers"]:
        d = dict(lw)
        for k in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
            m = lw[k]
            rows, cols = m.shape
            nwin = ws if k in ("wo", "wd") else 1
            parts = []
            for win in np.split(m, nwin, axis=1):
                win = np.ascontiguousarray(win)
                c = win.shape[1]
                codes, scales, _ = oracle.quantize(win, rows, c, oracle.E4M3, oracle.PCS)
                parts.append(f32_to_bf16_bits(oracle.dequantize(codes, scales, rows, c, oracle.E4M3)).reshape(rows, c))
            d[k] = np.concatenate(parts, axis=1)
        out["layers"].append(d)
    return out


def parity_check(args, cfg, local, rank, ws):
    """The workload's path on a 2-layer model with its widths, against the
    f32 host forward on rank 0 (the reference's tools/oracle method and its
    hardware tests' bar, crates/reng-synapse/src/bin/cache_test.rs:437):
    prompt-end logits cosine >= 0.999; greedy ids equal to the oracle's
    under teacher forcing except where the oracle's top-1 leads the engine's
    pick by less than 0.5; every rank's ids identical (the reference's
    coordinator rule, crates/reng-model/src/bin/tp.rs:604-675).  Slots 0
    and B-1 are checked against the oracle; every slot's ids across ranks."""
    import numpy as np
    import torch
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.synth import prompt_ids
    from reng.weights import random_weights, to_host
    dev = torch.device("cuda", local)
    B = args.batch
    pc = copy.deepcopy(cfg)
    pc.num_hidden_layers = 2
    w = random_weights(pc, seed=args.seed + 7, device=dev, layers=2)
    uid = new_unique_id(ws, rank)
    fp8 = ("e4m3", "pcs") if args.weights == "fp8" else None
    steps, cap = 8, 64
    eng = Engine(pc, w, batch=B, capacity=cap, device=local, tp_rank=rank, tp_world=ws, nccl_id=uid, fp8=fp8)
    prompts = [prompt_ids(12 + b % 5, pc.vocab_size, seed=100 + b) for b in range(B)]
    check = sorted({0, B - 1})
    seeds, last = [], {}
    for b in range(B):
        nxt, ll, _ = eng.prefill(b, prompts[b], last_logits=b in check)
        seeds.append(nxt)
        if ll is not None:
            last[b] = ll
    ids = eng.decode(seeds, steps)
    eng.close()
    agree = ranks_agree(np.concatenate([np.asarray(seeds, np.uint32), ids.reshape(-1)]), ws)
    res = None
    if rank == 0:
        import oracle
        h = to_host(w)
        if fp8:
            h = dequantized_host(h, ws)
        c = dict(hidden=pc.hidden_size, inter=pc.intermediate_size, n_layers=2,
                 n_heads=pc.num_attention_heads, n_kv_heads=pc.n_kv_heads(), head_dim=pc.head_dim(),
                 vocab=pc.vocab_size, eps=pc.rms_norm_eps, attn_scale=pc.attention_scale(),
                 has_bias=int(pc.has_bias()))
        orc = oracle.Model(c, h["layers"], h["final_gamma"], h["lm_head"], h["embed"])
        sin, cos = rope_caches_for(pc, cap)
        worst_cos, ties, mismatch = 1.0, 0, []
        for b in check:
            seq = np.concatenate([prompts[b], [seeds[b]], ids[:-1, b]]).astype(np.uint32)
            want = orc.forward(seq, sin, cos, logits_from=prompts[b].size - 1).astype(np.float64)
            got = last[b].astype(np.float64)
            worst_cos = min(worst_cos, float(got @ want[0] / (np.linalg.norm(got) * np.linalg.norm(want[0]))))
            for t, e in enumerate([seeds[b]] + [int(x) for x in ids[:, b]]):
                best = int(np.argmax(want[t]))
                if best != e:
                    gap = float(want[t][best] - want[t][e])
                    if gap < MARGIN:
                        ties += 1
                    else:
                        mismatch.append((b, t, e, best, round(gap, 4)))
        res = {"model": "%s widths, 2 layers%s, batch %d%s" % (
                   args.model, ", fp8-e4m3 weights (oracle on the dequantized shards)" if fp8 else "", B,
                   ", tensor-parallel %d" % ws if ws > 1 else ""),
               "oracle": "oracle/forward_oracle.c f32 host forward, teacher-forced on the engine's ids",
               "slots_checked": check, "steps": steps, "cosine_min": worst_cos,
               "near_ties": ties, "mismatches": mismatch, "ranks_agree": agree,
               "pass": bool(worst_cos >= COS_MIN and not mismatch and agree)}
    del w
    torch.cuda.empty_cache()
    return res


def decode_measure(eng, args, B, prompt, dev, ws, rank, local, with_e2e=True, with_clocks=True):
    """Warm-up, then the device-timed K steps (max over ranks) and, with
    `with_e2e`, the same K steps through the host-buffer C-ABI call."""
    import numpy as np
    import torch
    import torch.distributed as dist

    def fresh():
        eng.reset(-1)
        return [eng.prefill(b, prompt)[0] for b in range(B)]

    st = torch.cuda.Stream(device=dev)
    clocks = Clocks(local) if with_clocks else None
    if clocks:
        # sampled from before the warm-up to the end of the timed steps: a
        # timed region of tens of ms would otherwise fall between samples
        clocks.start()
        time.sleep(0.3)
    seeds = fresh()
    eng.decode(seeds, args.warmup)
    seeds = fresh()
    seeds_d = torch.tensor(seeds, dtype=torch.int32, device=dev)
    out_d = torch.empty((args.steps, B), dtype=torch.int32, device=dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    if ws > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with torch.cuda.stream(st):
        torch.cuda.nvtx.range_push("decode_timed")  # the range launch-list captures select
        e0.record(st)
        eng.decode_device(seeds_d, args.steps, out_d, st.cuda_stream)
        e1.record(st)
        torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    clk = clocks.stop() if clocks else None
    if clk is not None:
        clk["window"] = "warm-up and timed decode steps"
    if ws > 1:
        dist.barrier()
    t = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if ws > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    ids_value = out_d.cpu().numpy().astype(np.uint32)
    res = {"ms": ms, "clocks": clk, "ids": ids_value}
    if with_e2e:
        seeds = fresh()
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ids_e2e = eng.decode(seeds, args.steps)
        e2e_s = time.perf_counter() - t0
        te = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
        if ws > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        res["e2e_s"] = float(te.item())
        res["same"] = bool(np.array_equal(ids_value, ids_e2e))
    res["ranks_agree"] = ranks_agree(ids_value, ws)
    return res


# --------------------------------------------------------------- GPU arm --

def run_ours(args, cfg):
    import torch
    import torch.distributed as dist
    from reng import _lib
    from reng.model import Engine
    from reng.synth import prompt_ids
    from reng.weights import random_weights

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev,
                                timeout=__import__("datetime").timedelta(seconds=300))
    _lib.lib()
    peak, peak_kind = peaks()

    parity = parity_check(args, cfg, local, rank, ws) if not args.no_parity else None

    w = random_weights(cfg, seed=args.seed, device=dev)
    torch.cuda.synchronize()
    cap = max(args.prompt + args.warmup + 2 * args.steps + 8, args.prefill)
    fp8 = ("e4m3", "pcs") if args.weights == "fp8" else None
    eng = Engine(cfg, w, batch=args.batch, capacity=cap, device=local, tp_rank=rank,
                 tp_world=ws, nccl_id=new_unique_id(ws, rank), fp8=fp8)
    extras = [x for x in args.extras.split(",") if x] if ws == 1 else []
    if not extras:
        del w
        w = None
    torch.cuda.empty_cache()
    B = args.batch
    prompt = prompt_ids(args.prompt, cfg.vocab_size, seed=args.seed)

    r = decode_measure(eng, args, B, prompt, dev, ws, rank, local)
    ms = r["ms"]
    # ---- per-kernel timing for the roofline (resets the slots) ----
    eng.reset(-1)
    seeds = [eng.prefill(b, prompt)[0] for b in range(B)]
    eng.decode(seeds, args.steps // 2)
    kt = eng.time_kernels(iters=max(32, cfg.num_hidden_layers))
    kpl = eng.last_times().kernels_per_step
    xchg = None
    if ws > 1:
        # every rank times the exchange together (it waits on its peers)
        dist.barrier()
        xchg = eng.time_exchange(iters=2 * cfg.num_hidden_layers)
    # ---- prefill of a long prompt through the C ABI (host ids in, next id out) ----
    pf = None
    if args.prefill > 0:
        long_prompt = prompt_ids(args.prefill, cfg.vocab_size, seed=args.seed + 1)
        runs = []
        for i in range(3):
            eng.reset(0)
            if ws > 1:
                dist.barrier()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            eng.prefill(0, long_prompt)
            runs.append(time.perf_counter() - t0)
        tp_ = torch.tensor([statistics.median(runs[1:])], dtype=torch.float64, device=dev)
        if ws > 1:
            dist.all_reduce(tp_, op=dist.ReduceOp.MAX)
        pf_s = float(tp_.item())
        n_att = cfg.num_hidden_layers * cfg.num_attention_heads * cfg.head_dim()
        flops = 2 * cfg.active_params() * args.prefill + 4 * n_att * args.prefill * (args.prefill + 1) / 2
        pf = {"tokens": args.prefill, "tok_s": args.prefill / pf_s, "ms": pf_s * 1e3,
              "tflops": flops / pf_s / 1e12 / ws,
              "timing": "wall clock around reng_model_prefill (median of 2 after 1 warm-up), max over ranks; "
                        "tflops per GPU from the reng-ceiling prefill formula (crates/reng-ceiling/src/lib.rs:264-289)"}
    exchange = eng.tp_exchange()
    eng.close()

    # ---- the rest of BASELINE's metric on one GPU: b8, b64, FP8 weights ----
    extra = {}
    for x in extras:
        if x.startswith("b") and x[1:].isdigit():
            xb, xw, xf = int(x[1:]), args.weights, fp8
        elif x == "fp8":
            xb, xw, xf = 1, "fp8", ("e4m3", "pcs")
        else:
            continue
        e = Engine(cfg, w, batch=xb, capacity=cap, device=local, fp8=xf)
        rx = decode_measure(e, args, xb, prompt, dev, ws, rank, local, with_e2e=False, with_clocks=False)
        e.close()
        torch.cuda.empty_cache()
        ctx = args.prompt + args.steps // 2
        bx = step_bytes(cfg, xb, xw, 1, ctx)
        gbs = bx / (rx["ms"] / 1e3 / args.steps) / 1e9
        extra["%s_b%d" % (xw, xb)] = {
            "tok_s": args.steps * xb / (rx["ms"] / 1e3), "ms_per_step": rx["ms"] / args.steps,
            "step_roofline": {"bytes_per_step": bx, "achieved_gbs": gbs, "frac_of_measured": gbs / peak,
                              "frac_of_8tbs_spec": gbs / 8000.0}}
    w = None

    if rank == 0:
        tokens = args.steps * B
        value = tokens / (ms / 1e3)
        ctx = args.prompt + args.steps // 2
        bytes_step = step_bytes(cfg, B, args.weights, ws, ctx)
        wb = 1 if args.weights == "fp8" else 2
        h, inter = cfg.hidden_size, cfg.intermediate_size // ws
        gu_bytes = 2 * inter * h * wb + (8 * inter if args.weights == "fp8" else 0) + B * h * 2 + B * inter * 2
        achieved = gu_bytes / (kt["gate_up"] / 1e3) / 1e9
        step_gbs = bytes_step / (ms / 1e3 / args.steps) / 1e9
        conf = workload_config(args, ws)
        conf.update({
            "tp_exchange": {0: "none", 1: "ncclAllReduce", 2: "fused peer all-reduce (NVLink stores)"}[exchange],
            "l2": "inputs larger than L2 (weights %.1f GB streamed per step)" % (bytes_step / 1e9)})
        line = {
            "metric": "decode tok/s (b%d)" % B, "value": value, "unit": "tok/s",
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if ws > 1 else "weak", "vs_baseline": None,
            "dtype": "bf16" if args.weights == "bf16" else "fp8-e4m3 weights, bf16 activations",
            "data": "synthetic (random-init N(0,0.02) bf16 weights, uniform-random prompt ids)",
            "config": conf,
            "clocks": r["clocks"],
            "e2e": {"value": tokens / r["e2e_s"], "unit": "tok/s", "h2d_bytes_per_step": 4 * B / args.steps,
                    "d2h_bytes_per_step": 4 * B, "ids_equal_device_run": r["same"]},
            "gpu_launches": kpl * args.steps,
            "parity": parity,
            "timed_ids_ranks_agree": r["ranks_agree"],
            "roofline": {"bound": "hbm", "kernel": ("gemv<SWIGLU> gate/up" if B <= 8 or args.weights == "fp8"
                                                    else "rmsnorm rows + tcgen05 gemm<SWIGLU> gate/up")
                         + (" (layer-cycled, this rank's 1/%d of the columns)" % ws if ws > 1 else " (layer-cycled)"),
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         # ncu traffic was captured for the whole matrix on one GPU
                         "traffic": MEASURED_TRAFFIC.get((args.model, B, args.weights)) if ws == 1 else None,
                         "bytes_per_launch": gu_bytes},
            "step_roofline": {"bytes_per_step": bytes_step, "achieved_gbs": step_gbs,
                              "frac_of_measured": step_gbs / peak,
                              "frac_of_8tbs_spec": step_gbs / 8000.0},
            "kernel_ms": kt,
        }
        if xchg is not None:
            per_step = 2 * cfg.num_hidden_layers * xchg
            line["exchange"] = {
                "ms_per_launch": xchg, "launches_per_step": 2 * cfg.num_hidden_layers,
                "ms_per_step": per_step, "share_of_step": per_step / (ms / args.steps),
                "bytes_per_launch_per_peer": 4 * B * cfg.hidden_size,
                "timing": "CUDA events around back-to-back exchange launches on every rank at once "
                          "(reng_model_time_exchange), rank 0"}
        if pf is not None:
            line["prefill"] = pf
        if extra:
            line["extra"] = extra
        if not args.no_cpu and ws == 1:
            v, cores, sample = cpu_measure(cfg, args.cpu_tokens, 1, 5)
            line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port",
                                    "sample": sample}
        if args.fp8 and ws == 1:
            line["fp8_quant"] = fp8_quant_bench(dev)
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def fp8_quant_bench(dev, iters=4):
    """Config 0: bf16 [4096, 4096] -> E4M3 per-channel, GB/s of algorithmic
    bytes (2 B in + 1 B out per element + 4 B per row), device-timed over a
    rotation of matrices larger than L2 together.  The 16 quantize calls of
    a rotation are captured once in a CUDA graph (each call's C-ABI launch
    as issued by the Python wrapper) and the graph is replayed, so the time
    is the device's, not the host loop's."""
    import torch
    from reng import fp8
    from reng.synth import fp8_config0_matrix
    import numpy as np
    rows = cols = 4096
    w = torch.from_numpy(fp8_config0_matrix(rows, cols, seed=0).view(np.int16)).to(dev)
    n = 16  # 16 x 48 MB > L2
    ws = [w.clone() for _ in range(n)]
    codes = [torch.empty((rows, cols), dtype=torch.uint8, device=dev) for _ in range(n)]
    scales = [torch.empty(rows, dtype=torch.float32, device=dev) for _ in range(n)]
    for i in range(n):
        fp8.quantize_device(ws[i], rows, cols, 0, 0, codes=codes[i], scales=scales[i])
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(n):
            fp8.quantize_device(ws[i], rows, cols, 0, 0, codes=codes[i], scales=scales[i])
    g.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        g.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / (iters * n)
    del g
    b = rows * cols * 3 + rows * 4
    peak, kind = peaks()
    return {"matrix": "bf16 [4096,4096] N(0,0.02) 0.1% x50 -> e4m3 pcs", "ms": ms,
            "gbs": b / (ms / 1e3) / 1e9, "frac": b / (ms / 1e3) / 1e9 / peak, "peak_kind": kind}


def run_profile(args, cfg):
    """The small case of the ncu captures (one GPU, a few GB on the device):
    a layer-truncated model of the workload's widths (`--layers`), then
      * each kernel kind alone on the model's stream `--iters` times,
        cycling over the layers (reng_model_time_kernels; not with
        --no-kinds), after `--ctx` prompt tokens in every slot,
      * with --rows R: the same at a prefill block of R rows of slot 0
        (after a --ctx prompt), attention in its prefill form,
      * with --decode-steps N: a 16-token prompt in every slot and N greedy
        steps through the step graph (device ms per step),
      * with --quant N: N config-0 FP8 quantizations (bf16 [4096, 4096] ->
        E4M3 per-channel) on device buffers,
      * with --gemm shapes: the tcgen05 GEMM alone (reng_gemm_bf16) on
        random bf16 of those shapes, --iters launches.
    Prints one JSON line of device times; no bench line."""
    import torch
    from reng import fp8 as f
    from reng.model import Engine
    from reng.synth import fp8_config0_matrix, prompt_ids
    from reng.weights import random_weights
    torch.cuda.set_device(0)
    rep = {"model": args.model, "layers": args.layers, "batch": args.batch, "weights": args.weights}
    if args.gemm:
        import numpy as np
        from reng.gemm import gemm_bf16
        out = []
        for spec in args.gemm.split(";"):
            rows, K, M = (int(v) for v in spec.split(","))
            rng = np.random.default_rng(1)
            w = rng.integers(0x3c00, 0x3c80, size=(rows, K), dtype=np.uint16)  # bf16 in [1, 2)
            x = rng.integers(0x3c00, 0x3c80, size=(M, K), dtype=np.uint16)
            _, ms = gemm_bf16(w, x, splits=0, iters=args.iters)
            out.append({"rows": rows, "K": K, "M": M, "us": round(ms * 1e3, 2),
                        "weight_gbs": round(rows * K * 2 / (ms / 1e3) / 1e9, 1)})
        rep = {"gemm": out, "timing": "reng_gemm_bf16 alone, %d back-to-back launches after one (CUDA "
                                      "events, launch overhead included, weights resident in L2 when they fit)" % args.iters}
        print(json.dumps(rep))
        return
    if args.quant > 0:
        import numpy as np
        w = torch.from_numpy(fp8_config0_matrix(4096, 4096, seed=0).view(np.int16)).cuda()
        codes = torch.empty((4096, 4096), dtype=torch.uint8, device="cuda")
        scales = torch.empty(4096, dtype=torch.float32, device="cuda")
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        f.quantize_device(w, 4096, 4096, 0, 0, codes=codes, scales=scales)
        e0.record()
        for _ in range(args.quant):
            f.quantize_device(w, 4096, 4096, 0, 0, codes=codes, scales=scales)
        e1.record()
        torch.cuda.synchronize()
        rep["quant_us"] = round(e0.elapsed_time(e1) * 1e3 / args.quant, 2)
        print(json.dumps(rep))
        return
    cfg.num_hidden_layers = args.layers
    w = random_weights(cfg, seed=0, device="cuda", layers=args.layers)
    fp8 = ("e4m3", "pcs") if args.weights == "fp8" else None
    e = Engine(cfg, w, batch=args.batch, capacity=args.capacity, fp8=fp8)
    del w
    if args.ctx > 0:  # every slot holds a prompt, so attention reads a real context
        p = prompt_ids(args.ctx, cfg.vocab_size, seed=2)
        for b in range(args.batch):
            e.prefill(b, p)
        rep["ctx"] = args.ctx
    if args.kinds:
        rep["kernel_us"] = {k: round(v * 1e3, 2) for k, v in e.time_kernels(args.iters).items()}
    if args.rows > 0:  # the kinds at a prefill block of --rows rows (after the --ctx prompt)
        if args.ctx > 0 and args.kinds:  # the decode timing reset the slots
            e.prefill(0, prompt_ids(args.ctx, cfg.vocab_size, seed=2))
        rep["prefill_rows"] = args.rows
        rep["prefill_kernel_us"] = {k: round(v * 1e3, 2) for k, v in e.time_kernels(args.iters, rows=args.rows).items()}
    if args.decode_steps > 0:
        p = prompt_ids(16, cfg.vocab_size, seed=1)
        seeds = [e.prefill(b, p)[0] for b in range(args.batch)]
        e.decode(seeds, max(1, args.decode_steps))
        t = e.last_times()
        rep["decode"] = {"steps": t.steps, "ms_per_step": round(t.device_ms / t.steps, 4),
                         "kernels_per_step": t.kernels_per_step}
    print(json.dumps(rep))
    e.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="llama-3.1-8b")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--weights", default="bf16", choices=["bf16", "fp8"],
                    help="fp8: projections quantized E4M3 per channel at load (config 3)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--prefill", type=int, default=1024,
                    help="also time a prefill of this many prompt tokens (0: skip)")
    ap.add_argument("--extras", default=None,
                    help="comma list of extra 1-GPU decode measurements: bN (batch N, same weights "
                         "kind), fp8 (FP8 weights at batch 1); default b8,b64,fp8 for the Llama shape")
    ap.add_argument("--cpu-tokens", type=int, default=32)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--no-fp8", dest="fp8", action="store_false",
                    help="skip the FP8 quantizer line")
    pg = ap.add_argument_group("profiling (--profile: the small case of the ncu captures, no bench line)")
    pg.add_argument("--profile", action="store_true")
    pg.add_argument("--layers", type=int, default=2, help="depth of the profiled model")
    pg.add_argument("--iters", type=int, default=4, help="launches per kernel kind")
    pg.add_argument("--capacity", type=int, default=256)
    pg.add_argument("--ctx", type=int, default=0, help="prompt tokens prefilled in every slot before the kernel timing")
    pg.add_argument("--rows", type=int, default=0, help="also time each kernel kind at a prefill block of this many rows")
    pg.add_argument("--decode-steps", type=int, default=0)
    pg.add_argument("--no-kinds", dest="kinds", action="store_false")
    pg.add_argument("--quant", type=int, default=0, help="FP8 quantizations of the config-0 matrix")
    pg.add_argument("--gemm", default="", help="rows,K,M[;rows,K,M...]: the tcgen05 GEMM alone on these shapes")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.extras is None:
        args.extras = "b8,b64,fp8" if args.model == "llama-3.1-8b" and args.batch == 1 else ""
    from reng.config import SHAPES
    cfg = SHAPES[args.model]()
    if args.profile:
        run_profile(args, cfg)
    elif args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_ours(args, cfg)


if __name__ == "__main__":
    main()
