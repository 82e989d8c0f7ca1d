"""The reference's generator API over libreng_cuda.

`Engine` owns one `reng_model` (the C ABI object that replaces
reng_synapse::CachedModel / BatchedModel / tp::TpModel).  `Generator`,
`BatchedGenerator` and `TpGenerator` mirror reng-model's generators
(crates/reng-model/src/lib.rs:2807-3355) method for method: `feed`,
`feed_all`, `feed_id`, `generate`, `reset`, `position`, `prefill`,
`prefill_id`, `step`, `step_ids`, `batch`.  Where the reference panics
(empty input, cache overflow) these raise ValueError; device failures raise
reng._lib.RengError.
"""
import ctypes as C
import os

import numpy as np

from . import _lib
from .rope import rope_caches_for
from .weights import MATS


def _ptr(x):
    if x is None:
        return None
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    return x.data_ptr()


def _numel(x):
    return x.size if isinstance(x, np.ndarray) else x.numel()


def _is_device(w):
    x = w["embed"]
    return not isinstance(x, np.ndarray)


class Fp8Config(tuple):
    """(format, scheme) of the FP8 switch, with its backoff as an attribute
    (reng-model's Fp8Config, lib.rs:1693-1721); equal to the plain pair."""

    def __new__(cls, fmt="e4m3", scheme="pcs", backoff=1.0):
        t = super().__new__(cls, (fmt, scheme))
        t.backoff = backoff
        return t

    def __str__(self):
        return "%s/%s backoff %s" % (self[0], self[1], self.backoff)


def fp8_switch(value, flag=False):
    """The FP8 switch of reng-model (fp8_switch, lib.rs:1723-1782): `value` is
    RENG_FP8 (None when unset) and `flag` whether --fp8 was given.  Unset:
    the flag decides (the defaults, E4M3 per-channel, backoff 1).  An empty
    value, 0, off, false or no turns it off even with the flag; 1, on, true,
    yes mean the defaults; anything else is a list of settings separated by
    ':' or ',', each a format (e4m3, e5m2), a scale scheme (pcs, hw, unit)
    or backoff=<f32> in (0, 1].  A word that is none of these raises
    ValueError, so a typo never runs as bf16."""
    import re
    from .fp8 import Fp8Format, Scaling
    if value is None:
        return Fp8Config() if flag else None
    v = value.strip().lower()
    if v in ("", "0", "off", "false", "no"):
        return None
    if v in ("1", "on", "true", "yes"):
        return Fp8Config()
    fmt, sch, backoff = "e4m3", "pcs", 1.0
    for word in re.split("[:,]", v):
        word = word.strip()
        if not word:
            continue
        if Fp8Format.from_name(word) is not None:
            fmt = Fp8Format.from_name(word).short_name
        elif Scaling.from_name(word) is not None:
            sch = Scaling.from_name(word).short_name
        elif word.startswith("backoff="):
            try:
                backoff = float(np.float32(word[len("backoff="):]))
            except ValueError:
                raise ValueError("RENG_FP8: %r is not a number" % word) from None
            if not 0.0 < backoff <= 1.0:
                raise ValueError("RENG_FP8: backoff %s must lie in (0, 1]" % backoff)
        else:
            raise ValueError("RENG_FP8: %r is neither a format (e4m3, e5m2), a scale scheme "
                             "(pcs, hw, unit) nor backoff=<f32>" % word)
    return Fp8Config(fmt, sch, backoff)


def _scaled_table(t, s):
    """bf16 bits of bf16(f32(t) * f32(s)), host array or device tensor."""
    if isinstance(t, np.ndarray):
        from .synth import bf16_bits_to_f32, f32_to_bf16_bits
        return f32_to_bf16_bits(bf16_bits_to_f32(t) * np.float32(s))
    import torch
    f = t.view(torch.bfloat16).to(torch.float32) * torch.tensor(np.float32(s), device=t.device)
    return f.to(torch.bfloat16).view(t.dtype)


class Engine:
    def __init__(self, cfg, w, batch=1, capacity=1024, device=0, tp_rank=0, tp_world=1,
                 nccl_id=None, fp8=None):
        missing = cfg.unsupported(capacity)
        layers = w.get("layers", ())
        qk = any(lw.get(k) is not None for lw in layers for k in ("qn", "kn"))
        # q/k norm: Qwen3's per-head form runs (k_qk_norm); OLMo-2's
        # whole-row form has no kernel
        if qk and not all(lw.get(k) is not None and _numel(lw[k]) == cfg.head_dim()
                          for lw in layers for k in ("qn", "kn")):
            missing = missing + ["whole-row q/k norm"]
        if any(lw.get(k) is not None for lw in layers for k in ("g_post_attn", "g_post_mlp")):
            missing = missing + ["branch-output norms"]
        if missing:
            raise ValueError("this engine does not run %s" % ", ".join(missing))
        # q/k/v biases where the checkpoint has them, as the reference's
        # optional biases (crates/reng-model/src/lib.rs:1604-1606, 1628)
        has = [[lw.get(k) is not None for k in ("bq", "bk", "bv")] for lw in layers]
        if any(any(b) != all(b) for b in has) or len({all(b) for b in has}) > 1:
            raise ValueError("q/k/v biases must be all present or all absent in every layer")
        with_bias = bool(has) and all(has[0])
        warn = cfg.longrope_capacity_warning(capacity)
        if warn:  # as the reference's generators do at construction (lib.rs:2870, 3059, 3272)
            import sys
            print(warn, file=sys.stderr)
        self.cfg = cfg
        self.batch = batch
        self.capacity = capacity
        self.vocab = cfg.vocab_size
        dev = _is_device(w)
        mem = _lib.RENG_MEM_DEVICE if dev else _lib.RENG_MEM_HOST
        sin, cos = rope_caches_for(cfg, capacity)
        keep = [sin, cos]
        if dev:
            import torch
            d = w["embed"].device
            sin_t = torch.from_numpy(sin).to(d)
            cos_t = torch.from_numpy(cos).to(d)
            keep += [sin_t, cos_t]
            sin_p, cos_p = sin_t.data_ptr(), cos_t.data_ptr()
            torch.cuda.synchronize(d)
        else:
            sin_p, cos_p = sin.ctypes.data, cos.ctypes.data
        n = len(w["layers"])
        arr = (_lib.LayerWeights * n)()
        for i, lw in enumerate(w["layers"]):
            arr[i].no_rope = 0 if cfg.use_rope(i) else 1  # NoPE layers rotate nothing
            for k in MATS + ("g1", "g2", "bq", "bk", "bv", "qn", "kn"):
                x = lw.get(k)
                if x is None:
                    continue
                if isinstance(x, np.ndarray):
                    x = np.ascontiguousarray(x)
                    keep.append(x)
                setattr(arr[i], k, _ptr(x))
        desc = _lib.ModelDesc()
        desc.hidden = cfg.hidden_size
        desc.inter = cfg.intermediate_size
        desc.n_layers = n
        desc.n_heads = cfg.num_attention_heads
        desc.n_kv_heads = cfg.n_kv_heads()
        desc.head_dim = cfg.head_dim()
        desc.vocab = cfg.vocab_size
        desc.eps = cfg.rms_norm_eps
        desc.attn_scale = cfg.attention_scale()
        desc.has_qkv_bias = 1 if with_bias else 0
        desc.qk_norm = 1 if qk else 0
        desc.weights = _lib.RENG_WEIGHTS_BF16 if fp8 is None else _lib.RENG_WEIGHTS_FP8_E4M3
        desc.batch = batch
        desc.capacity = capacity
        desc.tp_rank = tp_rank
        desc.tp_world = tp_world
        desc.device = device
        idbuf = None
        if nccl_id is not None:
            idbuf = (C.c_uint8 * 128).from_buffer_copy(bytes(nccl_id))
            desc.nccl_id = C.addressof(idbuf)
        fg = w["final_gamma"]
        if isinstance(fg, np.ndarray):
            fg = np.ascontiguousarray(fg, np.float32)
            keep.append(fg)
        emb = w["embed"]
        lm = w["lm_head"]
        es = cfg.embed_scale()
        if es != 1.0:
            # the gather's factor (Granite's embedding_multiplier): one f32
            # product per element rounded to bf16, the value the reference's
            # host gather hands its bf16 device graph (embed_tokens,
            # crates/reng-model/src/lib.rs:2286-2305); a scaled copy, so a
            # tied LM head keeps the table as stored
            emb = _scaled_table(emb, es)
        if isinstance(emb, np.ndarray):
            emb = np.ascontiguousarray(emb)
            keep.append(emb)
        if isinstance(lm, np.ndarray):
            lm = np.ascontiguousarray(lm)
            keep.append(lm)
        h = C.c_void_p()
        _lib.call("reng_model_create", C.byref(desc), arr, _ptr(emb), _ptr(lm), _ptr(fg),
                  sin_p, cos_p, mem, C.byref(h))
        self.h = h
        del keep

    def close(self):
        if getattr(self, "h", None) is not None and self.h.value:
            _lib.lib().reng_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    # ------------------------------------------------------------- calls --
    def prefill(self, slot, ids, last_logits=False, all_logits=False):
        ids = np.ascontiguousarray(ids, np.uint32).reshape(-1)
        if ids.size == 0:
            raise ValueError("empty prompt")
        nxt = C.c_uint32(0)
        ll = np.empty(self.vocab, np.float32) if last_logits else None
        al = np.empty((ids.size, self.vocab), np.float32) if all_logits else None
        _lib.call("reng_model_prefill", self.h, slot, ids.ctypes.data, ids.size, C.byref(nxt),
                  _ptr(ll), _ptr(al))
        return int(nxt.value), ll, al

    def decode(self, seeds, n):
        seeds = np.ascontiguousarray(seeds, np.uint32).reshape(-1)
        if seeds.size != self.batch:
            raise ValueError("%d seeds for batch %d" % (seeds.size, self.batch))
        if n < 1:
            raise ValueError("n must be >= 1")
        out = np.empty((n, self.batch), np.uint32)
        _lib.call("reng_model_decode", self.h, seeds.ctypes.data, n, out.ctypes.data)
        return out

    def decode_device(self, seeds_dev, n, out_dev, stream):
        _lib.call("reng_model_decode_device", self.h, seeds_dev.data_ptr(), n, out_dev.data_ptr(),
                  stream)

    def step_logits(self, ids):
        ids = np.ascontiguousarray(ids, np.uint32).reshape(-1)
        if ids.size != self.batch:
            raise ValueError("%d ids for batch %d" % (ids.size, self.batch))
        logits = np.empty((self.batch, self.vocab), np.float32)
        nxt = np.empty(self.batch, np.uint32)
        _lib.call("reng_model_step_logits", self.h, ids.ctypes.data, logits.ctypes.data,
                  nxt.ctypes.data)
        return logits, nxt

    def reset(self, slot=-1):
        _lib.call("reng_model_reset", self.h, slot)

    def position(self, slot=0):
        p = C.c_int(0)
        _lib.call("reng_model_position", self.h, slot, C.byref(p))
        return p.value

    def device_bytes(self):
        b = C.c_uint64(0)
        _lib.call("reng_model_device_bytes", self.h, C.byref(b))
        return b.value

    def time_kernels(self, iters=64, rows=0):
        """Mean ms per launch of each kernel kind (qkv, attn, o, gate_up,
        down, lm_head) at the decode rows (rows=0) or at a prefill block of
        `rows` rows of slot 0; resets every slot afterwards."""
        out = np.zeros(6, np.float32)
        _lib.call("reng_model_time_kernels_rows", self.h, rows, iters, out.ctypes.data)
        return dict(zip(("qkv", "attn", "o_proj", "gate_up", "down", "lm_head"),
                        (float(x) for x in out)))

    def time_exchange(self, iters=64):
        """Mean ms of one partial exchange (tensor-parallel models; every
        rank calls it at the same time); resets every slot afterwards."""
        out = C.c_float(0.0)
        _lib.call("reng_model_time_exchange", self.h, iters, C.byref(out))
        return float(out.value)

    def last_times(self):
        t = _lib.StepTimes()
        _lib.call("reng_model_last_times", self.h, C.byref(t))
        return t

    def tp_exchange(self):
        """0 none (world 1), 1 NCCL all-reduce, 2 the fused peer all-reduce."""
        k = C.c_int(0)
        _lib.call("reng_model_tp_exchange", self.h, C.byref(k))
        return int(k.value)


class Generator:
    """One sequence (reng-model Generator, lib.rs:2807-3023)."""

    def __init__(self, w, cfg, rows=256, decode_rows=1, capacity=1024, device=0):
        self.cfg = cfg
        self.rows = rows
        self.engine = Engine(cfg, w, batch=1, capacity=capacity, device=device)

    def position(self):
        return self.engine.position(0)

    def device_loop(self):
        return True

    def reset(self):
        self.engine.reset(0)

    def feed(self, ids):
        """Append ids and return the last position's logits."""
        return self.engine.prefill(0, ids, last_logits=True)[1]

    def feed_all(self, ids):
        return self.engine.prefill(0, ids, all_logits=True)[2]

    def feed_id(self, ids):
        if os.environ.get("RENG_HOST_ARGMAX", "0") not in ("", "0"):
            return int(argmax_rows(self.feed(ids)[None, :])[0])
        return self.engine.prefill(0, ids)[0]

    def generate(self, seed, n):
        if n < 1:
            raise ValueError("n must be >= 1")
        return [int(x) for x in self.engine.decode([seed], n)[:, 0]]

    def close(self):
        self.engine.close()


class BatchedGenerator:
    """B sequences in lockstep (reng-model BatchedGenerator, lib.rs:3031-3237)."""

    def __init__(self, w, cfg, batch, rows=256, capacity=1024, device=0):
        self.cfg = cfg
        self.engine = Engine(cfg, w, batch=batch, capacity=capacity, device=device)

    def batch(self):
        return self.engine.batch

    def device_loop(self):
        return True

    def position(self, b):
        return self.engine.position(b)

    def reset(self, b=-1):
        self.engine.reset(b)

    def prefill(self, b, ids):
        return self.engine.prefill(b, ids, last_logits=True)[1]

    def prefill_id(self, b, ids):
        return self.engine.prefill(b, ids)[0]

    def step(self, ids):
        return self.engine.step_logits(ids)[0]

    def step_ids(self, ids):
        return [int(x) for x in self.engine.step_logits(ids)[1]]

    def generate(self, seeds, n):
        return [int(x) for x in self.engine.decode(seeds, n).reshape(-1)]

    def close(self):
        self.engine.close()


def argmax_rows(logits):
    """First index of the max of each row (reng-model argmax_rows, lib.rs:2309-2321)."""
    logits = np.asarray(logits, np.float32)
    out = []
    for row in logits:
        best, bi = -np.inf, 0
        # vectorised form of the strict '>' scan: the first maximal index,
        # NaN never selected
        r = np.where(np.isnan(row), -np.inf, row)
        m = r.max()
        if m > best:
            bi = int(np.flatnonzero(r == m)[0])
        out.append(bi)
    return out
