"""Per-kernel device times of the decode step (reng_model_time_kernels).

    python -m reng.profile_kernels [--model llama-3.1-8b] [--layers 2] [--batch 1] [--iters 4]

Builds a layer-truncated model of a BASELINE shape (random-init weights on the
device), then times each kernel kind of the decode step alone on the model's
stream, cycling over the layers.  Used as the small-case command of the ncu
captures summarised under profiles/ (one kernel kind, a few launches, a few
GB on the device).
"""
import argparse
import json
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3.1-8b")
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--iters", type=int, default=4)
    ap.add_argument("--capacity", type=int, default=256)
    a = ap.parse_args()
    from reng.config import SHAPES
    from reng.model import Engine
    from reng.weights import random_weights
    cfg = SHAPES[a.model]()
    cfg.num_hidden_layers = a.layers
    w = random_weights(cfg, seed=0, device="cuda", layers=a.layers)
    e = Engine(cfg, w, batch=a.batch, capacity=a.capacity)
    print(json.dumps({"model": a.model, "layers": a.layers, "batch": a.batch,
                      "kernel_us": {k: round(v * 1e3, 2) for k, v in e.time_kernels(a.iters).items()}}))
    e.close()


if __name__ == "__main__":
    main()
