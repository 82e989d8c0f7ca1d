"""Device times of the decode step's kernels, for profiling.

    python -m reng.profile_kernels [--model llama-3.1-8b] [--layers 2] [--batch 1]
                                   [--iters 4] [--decode 0] [--trace] [--no-kinds]

Builds a layer-truncated model of a BASELINE shape (random-init weights on the
device), then
  * times each per-projection kernel kind alone on the model's stream,
    cycling over the layers (reng_model_time_kernels; skipped with
    --no-kinds),
  * with --decode N: prefills a 16-token prompt into every slot and runs N
    greedy decode steps (the step's CUDA graph: the persistent step kernel
    when the shape allows it), reporting the device ms per step,
  * with --trace: the phase timeline of one step of the persistent kernel
    (reng_model_trace_step), summarised per phase kind.
Used as the small-case command of the ncu captures summarised under
profiles/ (one kernel, a few launches, a few GB on the device).
"""
import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def trace_summary(rows):
    """Mean per phase kind of (duration, arrival spread, barrier, first and
    last arrival), microseconds."""
    import numpy as np
    kinds = {}
    for i, (name, start, first, last, staged, loop) in enumerate(rows):
        k = "".join(ch for ch in name if not ch.isdigit())
        nxt = rows[i + 1][1] if i + 1 < len(rows) else last
        kinds.setdefault(k, []).append((nxt - start, last - first, nxt - last, first - start, last - start,
                                        staged - start if staged else 0.0, loop - start if loop else 0.0))
    out = {}
    for k, v in kinds.items():
        a = np.array(v).mean(0)
        out[k] = {"n": len(v), "us": round(a[0], 2), "spread_us": round(a[1], 2), "barrier_us": round(a[2], 2),
                  "first_done_us": round(a[3], 2), "last_done_us": round(a[4], 2),
                  "cta0_staged_us": round(a[5], 2), "cta0_loop_done_us": round(a[6], 2)}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3.1-8b")
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--iters", type=int, default=4)
    ap.add_argument("--capacity", type=int, default=256)
    ap.add_argument("--decode", type=int, default=0, help="decode steps to run through the step graph")
    ap.add_argument("--trace", action="store_true", help="phase timeline of one persistent step")
    ap.add_argument("--no-kinds", dest="kinds", action="store_false", help="skip the per-kind kernel timing")
    a = ap.parse_args()
    from reng.config import SHAPES
    from reng.model import Engine
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = SHAPES[a.model]()
    cfg.num_hidden_layers = a.layers
    w = random_weights(cfg, seed=0, device="cuda", layers=a.layers)
    e = Engine(cfg, w, batch=a.batch, capacity=a.capacity)
    del w
    rep = {"model": a.model, "layers": a.layers, "batch": a.batch}
    if a.kinds:
        rep["kernel_us"] = {k: round(v * 1e3, 2) for k, v in e.time_kernels(a.iters).items()}
    if a.decode > 0 or a.trace:
        p = prompt_ids(16, cfg.vocab_size, seed=1)
        seeds = [e.prefill(b, p)[0] for b in range(a.batch)]
        e.decode(seeds, max(1, a.decode))
        t = e.last_times()
        rep["decode"] = {"steps": t.steps, "ms_per_step": round(t.device_ms / t.steps, 4),
                         "kernels_per_step": t.kernels_per_step}
        if a.trace:
            rows = e.trace_step()
            rep["trace"] = {"step_us": round(rows[-1][3], 1), "phases": trace_summary(rows)}
    print(json.dumps(rep))
    e.close()


if __name__ == "__main__":
    main()
