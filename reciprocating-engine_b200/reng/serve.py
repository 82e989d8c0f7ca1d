"""Continuous batching over the engine's slots.

The reference's batched loop runs every slot for a fixed `n` steps; a
sequence that finishes early (EOS) keeps advancing on its own output, and
the caller drops its later ids or restarts the slot with `reset` and a new
prefill (crates/reng-synapse/src/batched.rs:36-43; BatchedGenerator::generate,
crates/reng-model/src/lib.rs:3204-3235).  `ContinuousBatcher` is that caller:
it keeps a queue of requests, prefills each into a free slot, runs the slots
in lockstep chunks of decode steps, cuts every sequence at its EOS id or its
token limit, and hands the freed slot to the next request.  Outputs are the
same greedy ids a request would get alone (the engine's slots are
independent); only how the steps are batched changes.

The engine is anything with the `Engine` calls the scheduler uses:
`batch`, `capacity`, `reset(slot)`, `position(slot)`,
`prefill(slot, ids) -> (next_id, ...)` and `decode(seeds, n) -> [n, batch]`.
"""
import collections
from dataclasses import dataclass, field
from typing import List, Optional, Sequence


@dataclass
class Request:
    """One generation: `prompt` ids, at most `max_new` generated ids, cut
    after the first id in `eos` (which is kept, as the last output id)."""
    prompt: Sequence[int]
    max_new: int
    eos: Sequence[int] = ()
    rid: object = None
    output: List[int] = field(default_factory=list)
    finish: Optional[str] = None       # "eos" or "length" once done

    def done(self):
        return self.finish is not None

    def _take(self, ids):
        """Append generated ids until EOS or the limit; returns True when done."""
        for t in ids:
            if self.finish is not None:
                break
            self.output.append(int(t))
            if int(t) in self.eos:
                self.finish = "eos"
            elif len(self.output) >= self.max_new:
                self.finish = "length"
        return self.finish is not None


class ContinuousBatcher:
    """Requests in, finished requests out, over one engine's `batch` slots.

    `chunk` bounds the decode steps between scheduling points: a sequence
    that stops inside a chunk wastes at most `chunk - 1` steps of its slot,
    and a waiting request waits at most one chunk for a slot.  Each chunk is
    also cut to the fewest steps any active slot still needs, so a token
    limit never overruns, and to the room left in the KV cache."""

    def __init__(self, engine, chunk=16):
        if chunk < 1:
            raise ValueError("chunk must be >= 1")
        self.engine = engine
        self.chunk = int(chunk)
        self.batch = int(engine.batch)
        self.capacity = int(engine.capacity)
        self.queue = collections.deque()
        self.slots: List[Optional[Request]] = [None] * self.batch
        self.seeds = [0] * self.batch
        self.steps = 0          # decode steps run (each advances every slot)
        self.useful = 0         # of those slot-steps, the ones that produced kept ids

    def submit(self, req):
        if len(req.prompt) == 0:
            raise ValueError("empty prompt")
        if req.max_new < 1:
            raise ValueError("max_new must be >= 1")
        if len(req.prompt) + req.max_new > self.capacity:
            raise ValueError("prompt %d + max_new %d exceeds the capacity %d"
                             % (len(req.prompt), req.max_new, self.capacity))
        self.queue.append(req)
        return req

    def pending(self):
        return len(self.queue) + sum(r is not None for r in self.slots)

    def _admit(self, finished):
        for b in range(self.batch):
            while self.slots[b] is None and self.queue:
                req = self.queue.popleft()
                self.engine.reset(b)
                nxt = self.engine.prefill(b, list(req.prompt))[0]
                if req._take([nxt]):
                    finished.append(req)     # stopped on its first id: slot stays free
                    continue
                self.slots[b] = req
                self.seeds[b] = int(nxt)

    def step(self):
        """One scheduling round: fill free slots, run one chunk, collect.
        Returns the requests that finished in it."""
        finished = []
        self._admit(finished)
        active = [b for b in range(self.batch) if self.slots[b] is not None]
        if not active:
            return finished
        need = min(self.slots[b].max_new - len(self.slots[b].output) for b in active)
        # every slot advances, idle ones too: idle slots restart at 0 when
        # they would run out of room, active ones always have it (their
        # prompt + max_new fits)
        n = max(1, min(self.chunk, need))
        for b in range(self.batch):
            if self.slots[b] is None and self.engine.position(b) + n > self.capacity:
                self.engine.reset(b)
                self.seeds[b] = 0
        room = min(self.capacity - self.engine.position(b) for b in range(self.batch))
        n = max(1, min(n, room))
        ids = self.engine.decode(self.seeds, n)
        self.steps += n
        for b in range(self.batch):
            col = [int(t) for t in ids[:, b]]
            self.seeds[b] = col[-1]
            req = self.slots[b]
            if req is None:
                continue
            before = len(req.output)
            if req._take(col):
                finished.append(req)
                self.slots[b] = None
            self.useful += len(req.output) - before
        return finished

    def run(self, requests=()):
        """Submit `requests`, step until every request is done; returns all
        finished requests in completion order."""
        for r in requests:
            self.submit(r)
        out = []
        while self.pending():
            out.extend(self.step())
        return out

    def occupancy(self):
        """Kept ids per slot-step so far (1.0 = no slot ever idle or wasted)."""
        return self.useful / float(max(1, self.steps * self.batch))
