"""Continuous batching (reng/serve.py) on CPU, over a stand-in engine with
the slot semantics of `Engine` / the reference's BatchedModel: independent
slots, `prefill` returns the next greedy id, `decode(seeds, n)` advances
every slot n positions and returns [n, batch] ids, and running past the
KV capacity is an error (crates/reng-model/src/lib.rs:3204-3235).  Its
next id is a hash of the slot's whole history, so any mix-up of slots,
seeds or positions changes the ids.  The property: every request gets
exactly the ids it would get alone, cut at its EOS or limit."""
import numpy as np
import pytest


class SlotEngine:
    def __init__(self, batch, capacity, vocab=61):
        self.batch, self.capacity, self.vocab = batch, capacity, vocab
        self.hist = [[] for _ in range(batch)]
        self.decode_calls = []

    @staticmethod
    def next_id(h, vocab):
        acc = 7
        for i, t in enumerate(h):
            acc = (acc * 1000003 + (t + 1) * (i + 3)) % 2147483647
        return acc % vocab

    def reset(self, b=-1):
        for s in (range(self.batch) if b < 0 else [b]):
            self.hist[s] = []

    def position(self, b=0):
        return len(self.hist[b])

    def prefill(self, b, ids):
        if not ids:
            raise ValueError("empty prompt")
        if len(self.hist[b]) + len(ids) > self.capacity:
            raise ValueError("cache overflow")
        self.hist[b] += list(ids)
        return self.next_id(self.hist[b], self.vocab), None, None

    def decode(self, seeds, n):
        if len(seeds) != self.batch or n < 1:
            raise ValueError("bad decode")
        if any(len(h) + n > self.capacity for h in self.hist):
            raise ValueError("cache overflow")
        self.decode_calls.append(n)
        out = np.empty((n, self.batch), np.uint32)
        cur = list(seeds)
        for j in range(n):
            for b in range(self.batch):
                self.hist[b].append(cur[b])
                cur[b] = self.next_id(self.hist[b], self.vocab)
                out[j, b] = cur[b]
        return out


def alone(prompt, max_new, eos, vocab=61):
    h = list(prompt)
    out = [SlotEngine.next_id(h, vocab)]
    while out[-1] not in eos and len(out) < max_new:
        h.append(out[-1])
        out.append(SlotEngine.next_id(h, vocab))
    return out


@pytest.fixture
def mods():
    from reng.serve import ContinuousBatcher, Request
    return ContinuousBatcher, Request


@pytest.mark.parametrize("batch,chunk,capacity", [(4, 8, 96), (1, 1, 64), (8, 5, 70), (3, 32, 80)])
def test_every_request_gets_its_own_greedy_ids(mods, batch, chunk, capacity):
    ContinuousBatcher, Request = mods
    rng = np.random.default_rng(batch * 100 + chunk)
    eng = SlotEngine(batch, capacity)
    cb = ContinuousBatcher(eng, chunk=chunk)
    reqs = []
    for i in range(25):
        p = rng.integers(0, 61, int(rng.integers(1, 20))).tolist()
        reqs.append(Request(p, int(rng.integers(1, 40)), eos=(3, 17), rid=i))
    done = cb.run(reqs)
    assert sorted(r.rid for r in done) == list(range(25))
    for r in reqs:
        want = alone(r.prompt, r.max_new, (3, 17))
        assert r.output == want, r.rid
        assert r.finish == ("eos" if want[-1] in (3, 17) else "length")
    assert all(n <= chunk for n in eng.decode_calls)
    assert 0.0 < cb.occupancy() <= 1.0


def test_a_request_that_stops_on_its_first_id_frees_the_slot_at_once(mods):
    ContinuousBatcher, Request = mods
    eng = SlotEngine(2, 64)
    first = alone([5, 6, 7], 1, ())[0]
    cb = ContinuousBatcher(eng, chunk=4)
    r0 = cb.submit(Request([5, 6, 7], 10, eos=(first,)))
    r1 = cb.submit(Request([1, 2], 12))
    r2 = cb.submit(Request([9], 12))
    done = cb.step()
    assert r0 in done and r0.output == [first] and r0.finish == "eos"
    assert cb.slots[0] is r1 and cb.slots[1] is r2      # r1 took r0's slot in the same round
    assert eng.decode_calls == [4]
    cb.run()
    assert r1.output == alone([1, 2], 12, ()) and r2.output == alone([9], 12, ())


def test_limits_are_never_overrun_and_idle_slots_never_overflow(mods):
    """Long run at a small capacity: chunks are cut to the fewest steps any
    active request needs, and idle slots restart before they run out."""
    ContinuousBatcher, Request = mods
    eng = SlotEngine(4, 24)
    cb = ContinuousBatcher(eng, chunk=16)
    reqs = [Request([i % 61 + 1] * (1 + i % 5), 1 + (7 * i) % 19, rid=i) for i in range(60)]
    cb.run(reqs)
    for r in reqs:
        assert len(r.output) == r.max_new
        assert r.output == alone(r.prompt, r.max_new, ())


def test_equal_requests_keep_every_slot_busy(mods):
    ContinuousBatcher, Request = mods
    eng = SlotEngine(4, 128)
    cb = ContinuousBatcher(eng, chunk=8)
    cb.run([Request([i + 1, i + 2], 33) for i in range(8)])
    assert cb.occupancy() == pytest.approx(1.0)
    assert sum(eng.decode_calls) == 2 * 32


def test_requests_that_cannot_fit_are_refused(mods):
    ContinuousBatcher, Request = mods
    cb = ContinuousBatcher(SlotEngine(2, 16), chunk=4)
    with pytest.raises(ValueError):
        cb.submit(Request([], 4))
    with pytest.raises(ValueError):
        cb.submit(Request([1], 0))
    with pytest.raises(ValueError):
        cb.submit(Request(list(range(10)), 7))
    with pytest.raises(ValueError):
        ContinuousBatcher(SlotEngine(2, 16), chunk=0)
    assert cb.pending() == 0


@pytest.mark.gpu
def test_continuous_batching_on_the_engine_matches_the_oracle(reng_lib, oracle_lib):
    """Over the CUDA engine (4 slots): every request's ids are the greedy
    ids of the f32 oracle teacher-forced on them, up to near-ties, whatever
    slot and neighbours it ran with."""
    from test_decode_gpu import check_greedy, oracle_for, small_cfg
    from reng.model import Engine
    from reng.rope import rope_caches_for
    from reng.serve import ContinuousBatcher, Request
    from reng.synth import prompt_ids
    from reng.weights import random_weights
    cfg = small_cfg()
    w = random_weights(cfg, seed=21)
    eng = Engine(cfg, w, batch=4, capacity=96)
    cb = ContinuousBatcher(eng, chunk=6)
    reqs = [Request(prompt_ids(3 + 2 * i, cfg.vocab_size, seed=40 + i).tolist(), 4 + 3 * (i % 5), rid=i)
            for i in range(9)]
    done = cb.run(reqs)
    assert sorted(r.rid for r in done) == list(range(9))
    sin, cos = rope_caches_for(cfg, 96)
    orc = oracle_for(cfg, w)
    for r in reqs:
        assert len(r.output) == r.max_new
        seq = np.array(list(r.prompt) + r.output[:-1], np.uint32)
        want = orc.forward(seq, sin, cos, logits_from=len(r.prompt) - 1)
        check_greedy(r.output, want)
    eng.close()
