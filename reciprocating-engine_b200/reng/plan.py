"""CachePlan: device-memory plan of a model (reng-model's CachePlan,
crates/reng-model/src/lib.rs:2366-2599), for this engine's HBM layout.

The engine keeps one KV cache of `batch` slots x `capacity` positions per
layer (K and V, bf16: `2 * n_kv_heads * head_dim * 2` bytes per position per
layer; no second buffer, since decode writes the cache in place), the packed
weights (the checkpoint's bytes, FP8 codes + one f32 scale per output row
when quantized), the embedding table, and work buffers of a few MB.  As in
the reference, `check` refuses a capacity that does not fit with an error
that says by how much, and `max_capacity` finds the largest that does.
"""
from dataclasses import dataclass


@dataclass
class CachePlan:
    layers: int
    n_kv_heads: int
    head_dim: int
    hidden: int
    inter: int
    vocab: int
    batch: int
    weight_bytes: int
    device_bytes: int = 183_359 * 1024 * 1024  # B200 HBM (nvidia-smi total)
    reserve_bytes: int = 2 << 30               # context, graphs, work buffers, allocator slack

    @staticmethod
    def new(cfg, batch=1, weights="bf16", device_bytes=None, world=1):
        h, hd = cfg.hidden_size, cfg.head_dim()
        nkv = cfg.n_kv_heads() // world
        qd = cfg.q_dim() // world
        inter = cfg.intermediate_size // world
        per_layer = h * qd * 2 + 2 * h * nkv * hd + 3 * h * inter
        rows = qd + 2 * nkv * hd + h + 2 * inter + h
        if weights == "fp8":
            body = cfg.num_hidden_layers * (per_layer + 4 * rows)
        else:
            body = cfg.num_hidden_layers * per_layer * 2
        emb = cfg.vocab_size * h * 2
        wbytes = body + 2 * emb  # LM head (packed) + embedding table, bf16
        p = CachePlan(cfg.num_hidden_layers, nkv, hd, h, inter, cfg.vocab_size, batch, wbytes)
        if device_bytes is not None:
            p.device_bytes = device_bytes
        return p

    def bytes_per_position_per_layer(self):
        return 2 * self.n_kv_heads * self.head_dim * 2

    def bytes_per_position(self):
        return self.bytes_per_position_per_layer() * self.layers

    def cache_bytes_at(self, capacity):
        return self.bytes_per_position() * self.batch * capacity

    def transient_bytes_at(self, capacity):
        """Work buffers: activations of <= 8 rows, logits, norm partials,
        argmax partials and the id ring."""
        rows = 8
        return (rows * (self.hidden * 2 * 2 + self.inter * 2 + self.vocab * 2) + (capacity + 1) * self.batch * 4
                + (1 << 20))

    def total_bytes_at(self, capacity):
        return self.weight_bytes + self.cache_bytes_at(capacity) + self.transient_bytes_at(capacity) + \
            self.reserve_bytes

    def fits(self, capacity):
        return self.total_bytes_at(capacity) <= self.device_bytes

    def max_capacity(self):
        lo, hi = 0, 1 << 24
        while lo < hi:
            mid = (lo + hi + 1) // 2
            if self.fits(mid):
                lo = mid
            else:
                hi = mid - 1
        return lo

    def summary(self, capacity):
        return ("weights %.2f GB + KV %.2f GB (%d slots x %d positions x %d B) + work %.2f GB + reserve %.2f GB "
                "= %.2f of %.2f GB" % (self.weight_bytes / 1e9, self.cache_bytes_at(capacity) / 1e9, self.batch,
                                        capacity, self.bytes_per_position(),
                                        self.transient_bytes_at(capacity) / 1e9, self.reserve_bytes / 1e9,
                                        self.total_bytes_at(capacity) / 1e9, self.device_bytes / 1e9))

    def check(self, capacity):
        if not self.fits(capacity):
            over = self.total_bytes_at(capacity) - self.device_bytes
            raise ValueError("capacity %d does not fit: %s; %.2f GB over, at most %d positions"
                             % (capacity, self.summary(capacity), over / 1e9, self.max_capacity()))
