"""N-card decode strategies on B200 with this engine's measured floors
(the role of crates/reng-ceiling/src/strategy.rs: data, tensor, pipeline,
hybrid and expert plans, judged on one stream or on every card summed).

A plan's decode step on one card is modelled as

    step = bytes on the card / HBM rate + kernels x launch floor + exchanges

where all three terms come from measurements of this engine on this pool's
B200s rather than from spec sheets:

* HBM rate and launch floor: a least-squares line through the per-kernel
  device times of the four projection GEMVs of a Llama-8B batch-1 step
  (bytes streamed against microseconds, `LAUNCH_FIT` below): the slope is
  the streaming rate a projection reaches, the intercept the fixed cost of
  one kernel boundary (the time from one kernel's last CTA to the next
  kernel streaming at full rate, plus its tail).
* Exchanges: the peer all-reduce of decode steps (`CollectiveFloor`), each
  including its own kernel.  At world 2 the measured TP2 step (2.227 ms,
  Llama-8B b1) leaves 3.2 us per exchange once the card's bytes at the
  fitted rate and its 162 projection kernels at the fitted floor are taken
  out; other worlds and sizes add the bytes each rank pushes, (W - 1) x
  message, at the pool's measured 770 GB/s peer copy rate.  The table is
  overridable from JSON like the reference's.

Unlike the reference (which replicates the LM head on every rank), this
engine shards the head by vocabulary in tensor-parallel decode; `tensor`
plans follow the engine, `head="replicated"` gives the reference's split.
Pipeline, hybrid and expert plans are projections: the engine has no
pipeline stages or MoE layers, so those rows say so (`projected`).

    python -m reng.strategy [--model llama-3.1-8b] [--cards 8] [--batch 8] [--ctx 192]
"""
import json
import math
from dataclasses import dataclass, field

from .ceiling import HardwareSpec, ModelShape, WEIGHT_BYTES

# Per-kernel device times of the batch-1 projection GEMVs (Llama-3.1-8B
# widths, B200, bench.py kernel_ms): (algorithmic bytes, microseconds).
LAUNCH_FIT = [
    (6144 * 4096 * 2, 12.64),      # q/k/v
    (4096 * 4096 * 2, 9.85),       # o_proj
    (2 * 14336 * 4096 * 2, 40.26),  # gate/up
    (4096 * 14336 * 2, 25.02),     # down_proj
]

PEER_COPY_BPS = 770e9   # measured peer copy per direction on this pool
# measured: (TP2 Llama-8B b1 step 2.2266 ms - 7.515 GB per card at the fitted
# rate - 162 kernels at the fitted floor) / 64 exchanges
WORLD2_EXCHANGE_S = 3.24e-6


def fit_launch(points=LAUNCH_FIT):
    """(seconds per byte, seconds per kernel) of the least-squares line."""
    n = len(points)
    xs = [float(b) for b, _ in points]
    ys = [t * 1e-6 for _, t in points]
    mx, my = sum(xs) / n, sum(ys) / n
    sxx = sum((x - mx) ** 2 for x in xs)
    sxy = sum((x - mx) * (y - my) for x, y in zip(xs, ys))
    slope = sxy / sxx
    return slope, my - slope * mx


@dataclass
class CollectiveFloor:
    """Seconds one decode exchange costs (its kernel included), per world
    and message size (log-linear between tabulated sizes)."""
    source: str
    worlds: dict = field(default_factory=dict)  # world -> [(bytes, seconds)]

    @staticmethod
    def measured():
        worlds = {}
        for w in (2, 4, 8):
            worlds[w] = [(b, WORLD2_EXCHANGE_S + (w - 1) * b / PEER_COPY_BPS)
                         for b in (16 * 1024, 128 * 1024, 1 << 20, 16 << 20)]
        return CollectiveFloor("B200: world 2 measured (TP2 Llama-8B step); worlds 4 and 8 and larger "
                               "messages add (W-1) x bytes at the measured 770 GB/s peer copy rate", worlds)

    @staticmethod
    def from_json(text):
        d = json.loads(text)
        return CollectiveFloor(d.get("source", "json"),
                               {int(w): sorted((int(b), float(s)) for b, s in pts) for w, pts in d["worlds"].items()})

    def exchange_s(self, world, nbytes):
        if world <= 1:
            return 0.0
        key = min(self.worlds, key=lambda w: (abs(w - world), -w))
        pts = self.worlds[key]
        if nbytes <= pts[0][0]:
            return pts[0][1]
        if nbytes >= pts[-1][0]:
            return pts[-1][1] * nbytes / pts[-1][0]
        for (b0, s0), (b1, s1) in zip(pts, pts[1:]):
            if b0 <= nbytes <= b1:
                t = (math.log(nbytes) - math.log(b0)) / (math.log(b1) - math.log(b0))
                return s0 + t * (s1 - s0)
        return pts[-1][1]


@dataclass
class Rate:
    tokens_per_s: float
    step_s: float
    memory_s: float
    launch_s: float
    collective_s: float


@dataclass
class Plan:
    strategy: str
    cards: int
    batch: int
    rejected: str = None
    single_stream: Rate = None
    aggregate: Rate = None
    resident_bytes_per_card: float = 0.0
    projected: bool = False
    notes: list = field(default_factory=list)

    def admissible(self):
        return self.rejected is None

    def rate(self, objective):
        return self.single_stream if objective == "single-stream" else self.aggregate


@dataclass
class Scenario:
    """The model, precision and decode shape every plan is judged at."""
    hw: HardwareSpec
    model: ModelShape
    batch: int = 1          # per replica, for the aggregate objective
    ctx: int = 192          # context the KV cache is charged at
    prec: str = "bf16"
    kv: str = "bf16"
    floor: CollectiveFloor = None
    head: str = "sharded"   # tensor-parallel LM head: "sharded" (this engine) or "replicated"

    def __post_init__(self):
        if self.floor is None:
            self.floor = CollectiveFloor.measured()
        self.s_per_byte, self.launch_s = fit_launch()

    def body_bytes(self):
        return self.model.body_params() * WEIGHT_BYTES[self.prec]

    def head_bytes(self):  # the LM head stays bf16 with FP8 projections
        return self.model.head_params() * (2.0 if self.prec == "fp8" else WEIGHT_BYTES[self.prec])

    def kv_bytes(self, batch):
        return batch * self.ctx * self.model.kv_bytes_per_token(self.kv)

    def exchange_bytes(self, batch):
        return self.model.hidden * batch * 4

    def card_step(self, card_bytes, kernels, exchanges, world, batch):
        mem = card_bytes * self.s_per_byte
        launch = kernels * self.launch_s
        coll = exchanges * self.floor.exchange_s(world, self.exchange_bytes(batch))
        step = mem + launch + coll
        return Rate(batch / step, step, mem, launch, coll)


def _kernels(m):
    """Projection-class kernels per decode step: embed, 5 per layer, LM head
    (the exchanges are charged by the collective floor)."""
    return 2 + m.layers * 5


def data_parallel(s, cards):
    m = s.model
    one = s.card_step(s.body_bytes() + s.head_bytes() + s.kv_bytes(1), _kernels(m), 0, 1, 1)
    b = s.card_step(s.body_bytes() + s.head_bytes() + s.kv_bytes(s.batch), _kernels(m), 0, 1, s.batch)
    agg = Rate(cards * b.tokens_per_s, b.step_s, b.memory_s, b.launch_s, 0.0)
    resident = s.body_bytes() + s.head_bytes() + s.kv_bytes(s.batch)
    p = Plan("data", cards, s.batch, single_stream=one, aggregate=agg, resident_bytes_per_card=resident,
             notes=["%d independent replicas (bench.py --gpus N replicas of a whole model)" % cards])
    if resident > s.hw.hbm_bytes:
        p.rejected = "the model does not fit one card (%.1f GB)" % (resident / 1e9)
    return p


def tensor_parallel(s, cards):
    m = s.model
    n = float(cards)
    head = s.head_bytes() / n if (s.head == "sharded" and cards > 1) else s.head_bytes()

    def rate(batch):
        card = s.body_bytes() / n + head + s.kv_bytes(batch) / n
        ex = 2 * m.layers if cards > 1 else 0
        return s.card_step(card, _kernels(m), ex, cards, batch)

    one, b = rate(1), rate(s.batch)
    p = Plan("tensor", cards, s.batch, single_stream=one, aggregate=b,
             resident_bytes_per_card=s.body_bytes() / n + s.head_bytes() + s.kv_bytes(s.batch) / n,
             notes=["heads and MLP columns split, %s LM head, two peer all-reduces per layer" % s.head])
    why = []
    if m.n_heads % cards or m.n_kv_heads % cards:
        why.append("%d/%d heads do not split over %d" % (m.n_heads, m.n_kv_heads, cards))
    if m.ff % cards or (m.ff // cards) % 8:
        why.append("intermediate %d does not split over %d in 8-row steps" % (m.ff, cards))
    if cards > 8:
        why.append("the peer exchange runs up to 8 ranks (one NVLink domain)")
    if p.resident_bytes_per_card > s.hw.hbm_bytes:
        why.append("does not fit (%.1f GB per card)" % (p.resident_bytes_per_card / 1e9))
    if why:
        p.rejected = "; ".join(why)
    return p


def pipeline_parallel(s, cards):
    """Consecutive layers per card; one activation hand-off per boundary
    (charged as a world-2 exchange plus a kernel).  A single stream visits
    every stage in turn; the aggregate keeps `cards` micro-batches in
    flight, so the slowest stage sets the rate."""
    m = s.model
    n = max(1, cards)
    per = [m.layers // n + (1 if i < m.layers % n else 0) for i in range(n)]
    lb = s.body_bytes() / m.layers

    def stage(l, last, batch):
        return s.card_step(l * lb + (s.head_bytes() if last else 0.0) + s.kv_bytes(batch) * l / m.layers,
                           5 * l + (2 if last else 0), 0, 1, batch)

    def total(batch):
        st = [stage(l, i == n - 1, batch) for i, l in enumerate(per)]
        hand = (n - 1) * (s.launch_s + s.floor.exchange_s(2, s.exchange_bytes(batch)))
        return st, hand

    st1, h1 = total(1)
    step1 = sum(r.step_s for r in st1) + h1
    one = Rate(1.0 / step1, step1, sum(r.memory_s for r in st1), sum(r.launch_s for r in st1), h1)
    stb, hb = total(s.batch)
    worst = max(r.step_s for r in stb) + (hb / max(1, n - 1) if n > 1 else 0.0)
    agg = Rate(s.batch / worst, worst, max(r.memory_s for r in stb), max(r.launch_s for r in stb), hb)
    p = Plan("pipeline", cards, s.batch, single_stream=one, aggregate=agg, projected=True,
             resident_bytes_per_card=max(per) * lb + s.head_bytes() + n * s.kv_bytes(s.batch) * max(per) / m.layers,
             notes=["projection: the engine has no pipeline stages"])
    if p.resident_bytes_per_card > s.hw.hbm_bytes:
        p.rejected = "does not fit (%.1f GB on the busiest stage)" % (p.resident_bytes_per_card / 1e9)
    return p


def hybrid(s, replicas, world):
    t = tensor_parallel(s, world)
    agg = Rate(replicas * t.aggregate.tokens_per_s, t.aggregate.step_s, t.aggregate.memory_s,
               t.aggregate.launch_s, t.aggregate.collective_s)
    return Plan("dp%d x tp%d" % (replicas, world), replicas * world, s.batch, rejected=t.rejected,
                single_stream=t.single_stream, aggregate=agg, resident_bytes_per_card=t.resident_bytes_per_card,
                notes=["%d replicas of a %d-way tensor-parallel model" % (replicas, world)])


def expert_parallel(s, cards):
    return Plan("expert", cards, s.batch, rejected="dense model: no routed experts", projected=True,
                notes=["the engine has no mixture-of-experts layer"])


def plans(s, cards):
    out = [data_parallel(s, cards), tensor_parallel(s, cards), pipeline_parallel(s, cards)]
    for w in (2, 4, 8):
        if 1 < w < cards and cards % w == 0:
            out.append(hybrid(s, cards // w, w))
    out.append(expert_parallel(s, cards))
    return out


def choose(s, cards, objective="single-stream"):
    """The best admissible plan for the objective; built plans before
    projections on ties."""
    ok = [p for p in plans(s, cards) if p.admissible()]
    if not ok:
        return None
    return max(ok, key=lambda p: (p.rate(objective).tokens_per_s, not p.projected))


def main():
    import argparse
    import os
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from reng.config import SHAPES
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3.1-8b")
    ap.add_argument("--cards", type=int, default=8)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--ctx", type=int, default=192)
    ap.add_argument("--prec", default="bf16")
    ap.add_argument("--head", default="sharded", choices=["sharded", "replicated"])
    ap.add_argument("--floor-json", default=None, help="a CollectiveFloor table to use instead")
    a = ap.parse_args()
    m = ModelShape.from_config(SHAPES[a.model](), a.model)
    floor = CollectiveFloor.from_json(open(a.floor_json).read()) if a.floor_json else None
    s = Scenario(HardwareSpec.b200_measured(), m, a.batch, a.ctx, a.prec, floor=floor, head=a.head)
    print("%s on %d x %s, %s, ctx %d; floors: %.2f TB/s streaming, %.2f us per kernel; %s" % (
        a.model, a.cards, s.hw.name, a.prec, a.ctx, 1e-12 / s.s_per_byte, s.launch_s * 1e6, s.floor.source))
    print("%-14s %12s %14s %10s  %s" % ("plan", "b1 tok/s", "b%d agg tok/s" % a.batch, "GB/card", "status"))
    for p in plans(s, a.cards):
        one = "%.1f" % p.single_stream.tokens_per_s if p.single_stream else "-"
        agg = "%.0f" % p.aggregate.tokens_per_s if p.aggregate else "-"
        st = ("rejected: " + p.rejected) if p.rejected else ("projection" if p.projected else "built")
        print("%-14s %12s %14s %10.1f  %s" % (p.strategy, one, agg, p.resident_bytes_per_card / 1e9, st))
    for obj in ("single-stream", "aggregate"):
        c = choose(s, a.cards, obj)
        print("best %s: %s" % (obj, c.strategy if c else "none"))


if __name__ == "__main__":
    main()
