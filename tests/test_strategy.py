"""The N-card strategy model (reng/strategy.py, the role of reng-ceiling's
strategy.rs): its floors reproduce the measured decode steps it was fitted
on, and its plans keep the invariants of the reference's module (replicas
scale the aggregate, tensor splits refuse non-divisible head counts, a
pipeline does not speed up one stream, choices follow the objective)."""
import json
import os
import sys

import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                "reciprocating-engine_b200"))


@pytest.fixture(scope="module")
def mods():
    from reng import ceiling, strategy
    from reng.config import SHAPES
    return ceiling, strategy, SHAPES


def scenario(mods, model="llama-3.1-8b", batch=1, ctx=160, **kw):
    ceiling, strategy, SHAPES = mods
    m = ceiling.ModelShape.from_config(SHAPES[model](), model)
    return strategy.Scenario(ceiling.HardwareSpec.b200_measured(), m, batch, ctx, **kw)


def test_floors_reproduce_the_measured_steps(mods):
    """Llama-8B b1 on this pool's B200s (bench.py): 3.16 ms per step on one
    GPU, 2.227 ms at TP2 with the peer all-reduce and the sharded LM head;
    the model, charged at a 160-position context, is within 2% of both."""
    _, strategy, _ = mods
    s = scenario(mods)
    one = strategy.tensor_parallel(s, 1).single_stream.step_s
    two = strategy.tensor_parallel(s, 2).single_stream.step_s
    assert abs(one - 3.160e-3) / 3.160e-3 < 0.02
    assert abs(two - 2.227e-3) / 2.227e-3 < 0.02
    spb, floor = strategy.fit_launch()
    assert 6.0e12 < 1.0 / spb < 7.5e12       # the projections' streaming rate
    assert 3e-6 < floor < 8e-6              # one kernel boundary


def test_replicas_scale_the_aggregate_not_the_stream(mods):
    _, strategy, _ = mods
    s = scenario(mods, batch=8)
    d1, d8 = strategy.data_parallel(s, 1), strategy.data_parallel(s, 8)
    assert d8.single_stream.tokens_per_s == pytest.approx(d1.single_stream.tokens_per_s)
    assert d8.aggregate.tokens_per_s == pytest.approx(8 * d1.aggregate.tokens_per_s)


def test_tensor_parallel_speeds_one_stream_up_and_shards_bytes(mods):
    _, strategy, _ = mods
    s = scenario(mods)
    rates = [strategy.tensor_parallel(s, n).single_stream.tokens_per_s for n in (1, 2, 4, 8)]
    assert rates == sorted(rates)
    t8 = strategy.tensor_parallel(s, 8)
    assert t8.admissible()
    rep = strategy.tensor_parallel(scenario(mods, head="replicated"), 8)
    assert rep.single_stream.tokens_per_s < t8.single_stream.tokens_per_s   # the engine shards the head


def test_non_divisible_heads_are_refused(mods):
    _, strategy, _ = mods
    s = scenario(mods, model="smollm2-135m")
    for n in (2, 4, 8):
        assert not strategy.tensor_parallel(s, n).admissible()
    assert strategy.choose(s, 8, "single-stream").strategy == "data"


def test_pipeline_does_not_speed_up_one_stream(mods):
    _, strategy, _ = mods
    s = scenario(mods, batch=8)
    p = strategy.pipeline_parallel(s, 4)
    assert p.projected
    assert p.single_stream.tokens_per_s <= strategy.data_parallel(s, 4).single_stream.tokens_per_s * 1.001
    assert p.aggregate.tokens_per_s > strategy.data_parallel(s, 1).aggregate.tokens_per_s


def test_choices_follow_the_objective(mods):
    _, strategy, _ = mods
    s = scenario(mods, batch=8)
    assert strategy.choose(s, 8, "single-stream").strategy == "tensor"
    assert strategy.choose(s, 8, "aggregate").strategy == "data"
    assert not strategy.expert_parallel(s, 8).admissible()


def test_collective_floor_from_json_and_interpolation(mods):
    _, strategy, _ = mods
    f = strategy.CollectiveFloor.from_json(json.dumps(
        {"source": "test", "worlds": {"2": [[1024, 1e-6], [1048576, 5e-6]]}}))
    assert f.exchange_s(1, 4096) == 0.0
    assert f.exchange_s(2, 512) == 1e-6
    mid = f.exchange_s(2, 32768)
    assert 1e-6 < mid < 5e-6
    assert f.exchange_s(4, 1048576) == 5e-6          # nearest tabulated world
    m = strategy.CollectiveFloor.measured()
    assert m.exchange_s(8, 16384) > m.exchange_s(2, 16384)
