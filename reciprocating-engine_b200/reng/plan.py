"""CachePlan: device-memory plan of a model (reng-model's CachePlan,
crates/reng-model/src/lib.rs:2366-2599), for this engine's HBM layout.

The engine keeps one KV cache of `batch` slots x `capacity` positions per
layer (K and V, bf16: `2 * n_kv_heads * head_dim * 2` bytes per position per
layer; no second buffer, since decode writes the cache in place), the packed
weights (the checkpoint's bytes, FP8 codes + one f32 scale per output row
when quantized), the embedding table, and work buffers sized for a prefill
block of BLOCK_ROWS rows (at Llama-8B widths ~0.4 GB, most of it the block's
bf16 logits).  As in
the reference, `check` refuses a capacity that does not fit with an error
that says by how much, and `max_capacity` finds the largest that does.
"""
from dataclasses import dataclass

BLOCK_ROWS = 1024     # rows of a prefill block: the engine's work buffers (kBlockRows)
SS_STRIDE = 512       # RMS partials per row (kSsStride)
GEMM_PARTS = 2 * 148 * 128 * 64  # GEMM split-K f32 partials (2 x SMs x 128 x 64)


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
    q_dim: int = 0       # query width (heads x head_dim); 0: the hidden size
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
        p = CachePlan(cfg.num_hidden_layers, nkv, hd, h, inter, cfg.vocab_size, batch, wbytes, q_dim=qd)
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
        """Work buffers, as the engine allocates them (csrc/model.cu): per
        block row the residual stream and its normalised copy, q and the
        attention output, the SwiGLU activation, bf16 logits, f32 partials
        of tensor parallelism, RMS partials, row bookkeeping and argmax keys;
        the GEMM split-K partials; the id ring of `capacity + 1` steps."""
        qd = self.q_dim or self.hidden
        per_row = (2 * self.hidden * 2 + 2 * qd * 2 + self.inter * 2 + self.vocab * 2 + self.hidden * 4
                   + SS_STRIDE * 4 + 3 * 4 + 8)
        return BLOCK_ROWS * per_row + GEMM_PARTS * 4 + (capacity + 1) * self.batch * 4 + (1 << 20)

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
