"""TEST INFRASTRUCTURE ONLY: ctypes binding of the CPU oracle (oracle/lib/liboracle.so).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module, and only as the checker / the timed CPU restatement of the
reference.  See fp8_oracle.c and forward_oracle.c for what is restated.
"""
import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "lib", "liboracle.so")

E4M3, E5M2 = 0, 1
PCS, HW, UNIT = 0, 1, 2

_lib = None


class Cfg(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("inter", C.c_int32), ("n_layers", C.c_int32),
                ("n_heads", C.c_int32), ("n_kv_heads", C.c_int32), ("head_dim", C.c_int32),
                ("vocab", C.c_int32), ("eps", C.c_float), ("attn_scale", C.c_float),
                ("has_bias", C.c_int32), ("qn_width", C.c_int32), ("kn_width", C.c_int32),
                ("post_norm", C.c_int32), ("act", C.c_int32), ("attn_softcap", C.c_float),
                ("final_softcap", C.c_float)]


LAYER_ARRAYS = ("wq", "wk", "wv", "wo", "wg", "wu", "wd", "g1", "g2", "bq", "bk", "bv", "qn", "kn",
                "g_post_attn", "g_post_mlp")
LAYER_INTS = ("window", "no_rope", "local_rope")


class Layer(C.Structure):
    _fields_ = ([(n, C.c_void_p) for n in LAYER_ARRAYS] +
                [(n, C.c_int32) for n in LAYER_INTS])


def build():
    """Compile the oracle with its Makefile (gcc, OpenMP)."""
    import subprocess
    r = subprocess.run(["make", "-C", HERE], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + r.stdout + r.stderr)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = C.CDLL(LIB)
        P = C.c_void_p
        L.orc_fp8_encode.argtypes = [C.c_float, C.c_int]
        L.orc_fp8_encode.restype = C.c_uint8
        L.orc_fp8_decode.argtypes = [C.c_uint8, C.c_int]
        L.orc_fp8_decode.restype = C.c_float
        L.orc_fp8_quantize.argtypes = [P, C.c_int64, C.c_int64, C.c_int, C.c_int, C.c_float,
                                       C.c_int, P, P, P]
        L.orc_fp8_quantize.restype = C.c_int
        L.orc_row_errors.argtypes = [P, C.c_int64, C.c_int64, P, P, C.c_int, P, P]
        L.orc_row_errors.restype = None
        L.orc_row_absmax.argtypes = [P, C.c_int64, C.c_int64, P]
        L.orc_row_absmax.restype = None
        L.orc_fp8_dequantize.argtypes = [P, P, C.c_int64, C.c_int64, C.c_int, P]
        L.orc_fp8_dequantize.restype = None
        L.orc_choose_exp_bias.argtypes = [C.c_float, C.c_int]
        L.orc_choose_exp_bias.restype = C.c_uint32
        L.orc_split.argtypes = [C.c_int64, C.c_int64]
        L.orc_split.restype = C.c_int
        L.orc_max_finite.argtypes = [C.c_int]
        L.orc_max_finite.restype = C.c_float
        L.orc_f32_to_bf16.argtypes = [C.c_float]
        L.orc_f32_to_bf16.restype = C.c_uint16
        L.orc_embed.argtypes = [P, C.c_int, P, C.c_int, C.c_float, P]
        L.orc_embed.restype = None
        L.orc_forward.argtypes = [P, P, P, P, P, P, P, P, P, C.c_int, C.c_int, P, C.c_int]
        L.orc_forward.restype = C.c_int
        L.orc_max_threads.argtypes = []
        L.orc_max_threads.restype = C.c_int
        L.orc_encode_checksum.argtypes = [C.c_uint64, C.c_uint64, C.c_int, C.c_int]
        L.orc_encode_checksum.restype = C.c_uint64
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def encode(x, fmt):
    return int(lib().orc_fp8_encode(float(x), fmt))


def decode(code, fmt):
    return float(lib().orc_fp8_decode(int(code), fmt))


def f32_to_bf16(x):
    return int(lib().orc_f32_to_bf16(float(x)))


def quantize(w, rows, cols, fmt, scaling, backoff=1.0, threads=0):
    """reng_fp8::quantize_with restated: returns (codes u8 [rows*cols], scales f32, exp_bias)."""
    w = np.ascontiguousarray(w, dtype=np.uint16).reshape(-1)
    assert w.size == rows * cols
    codes = np.empty(rows * cols, np.uint8)
    scales = np.empty(rows, np.float32)
    bias = C.c_uint32(0)
    rc = lib().orc_fp8_quantize(_p(w), rows, cols, fmt, scaling, backoff, threads, _p(codes),
                                _p(scales), C.byref(bias))
    if rc != 0:
        raise ValueError("oracle quantize rejected the arguments")
    return codes, scales, int(bias.value)


def row_errors(w, codes, scales, rows, cols, fmt):
    w = np.ascontiguousarray(w, dtype=np.uint16).reshape(-1)
    codes = np.ascontiguousarray(codes, dtype=np.uint8).reshape(-1)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    mean = np.empty(rows, np.float32)
    mx = np.empty(rows, np.float32)
    lib().orc_row_errors(_p(w), rows, cols, _p(codes), _p(scales), fmt, _p(mean), _p(mx))
    return mean, mx


def dequantize(codes, scales, rows, cols, fmt):
    codes = np.ascontiguousarray(codes, dtype=np.uint8).reshape(-1)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    out = np.empty(rows * cols, np.float32)
    lib().orc_fp8_dequantize(_p(codes), _p(scales), rows, cols, fmt, _p(out))
    return out


def encode_checksum(lo, hi, fmt, threads=0):
    """Checksum of the oracle's codes for every f32 bit pattern in [lo, hi)."""
    return int(lib().orc_encode_checksum(lo, hi, fmt, threads))


class Model:
    """Holds numpy weights of a decoder and runs the f32 forward oracle."""

    def __init__(self, cfg, layers, final_gamma, lm_head, embed):
        # cfg: dict with hidden, inter, n_layers, n_heads, n_kv_heads, head_dim, vocab,
        # eps, attn_scale, and optionally has_bias, qn_width / kn_width (q / k
        # norm part widths), post_norm, act (0 SiLU, 1 GELU-tanh), attn_softcap,
        # final_softcap, embed_scale (absent = the Llama behaviour).
        # layers: list of dicts of numpy arrays (LAYER_ARRAYS) and ints
        # (LAYER_INTS: window, no_rope, local_rope).
        self.cfg = cfg
        self._keep = []
        self.c = Cfg(cfg["hidden"], cfg["inter"], cfg["n_layers"], cfg["n_heads"],
                     cfg["n_kv_heads"], cfg["head_dim"], cfg["vocab"], cfg["eps"],
                     cfg["attn_scale"], int(cfg.get("has_bias", 0)), int(cfg.get("qn_width", 0)),
                     int(cfg.get("kn_width", 0)), int(cfg.get("post_norm", 0)),
                     int(cfg.get("act", 0)), float(cfg.get("attn_softcap") or 0.0),
                     float(cfg.get("final_softcap") or 0.0))
        self.embed_scale = float(cfg.get("embed_scale", 1.0))
        for key, width in (("qn", self.c.qn_width), ("kn", self.c.kn_width)):
            for lw in layers:
                g = lw.get(key)
                if width and (g is None or np.asarray(g).size != width):
                    raise ValueError("%s_width %d needs a [%d] %s gain in every layer"
                                     % (key, width, width, key))
        arr = (Layer * len(layers))()
        for i, lw in enumerate(layers):
            for name in LAYER_ARRAYS:
                a = lw.get(name)
                if a is None:
                    continue
                a = np.ascontiguousarray(a)
                self._keep.append(a)
                setattr(arr[i], name, a.ctypes.data)
            for name in LAYER_INTS:
                setattr(arr[i], name, int(lw.get(name) or 0))
        self.layers = arr
        self.final_gamma = np.ascontiguousarray(final_gamma, np.float32)
        self.lm_head = np.ascontiguousarray(lm_head, np.uint16)
        self.embed = np.ascontiguousarray(embed, np.uint16)

    @classmethod
    def for_config(cls, cfg, w):
        """The oracle of a host LlamaConfig and its loaded weights, with the
        per-layer settings of the reference's layer_views
        (crates/reng-model/src/lib.rs:2630-2707): attention scale, window,
        RoPE use and table, activation, softcaps, post-norm, embed scale."""
        layers = []
        for li, lw in enumerate(w["layers"]):
            d = dict(lw)
            d["window"] = cfg.layer_window(li) or 0
            d["no_rope"] = 0 if cfg.use_rope(li) else 1
            d["local_rope"] = 1 if cfg.local_rope(li) else 0
            layers.append(d)
        l0 = w["layers"][0] if w["layers"] else {}

        def width(k):
            return int(np.asarray(l0[k]).size) if l0.get(k) is not None else 0

        c = dict(hidden=cfg.hidden_size, inter=cfg.intermediate_size, n_layers=len(layers),
                 n_heads=cfg.num_attention_heads, n_kv_heads=cfg.n_kv_heads(),
                 head_dim=cfg.head_dim(), vocab=cfg.vocab_size, eps=cfg.rms_norm_eps,
                 attn_scale=cfg.attention_scale(), has_bias=int(l0.get("bq") is not None),
                 qn_width=width("qn"), kn_width=width("kn"), post_norm=int(cfg.post_norm()),
                 act=1 if cfg.activation() == "gelu_tanh" else 0,
                 attn_softcap=cfg.attn_softcap() or 0.0, final_softcap=cfg.final_softcap() or 0.0,
                 embed_scale=cfg.embed_scale())
        return cls(c, layers, w["final_gamma"], w["lm_head"], w["embed"])

    def forward(self, ids, sin, cos, logits_from=0, threads=0, sin_local=None, cos_local=None):
        """Logits [len(ids) - logits_from, vocab] of a causal forward over ids
        (sin_local / cos_local: the table of layers with local_rope)."""
        ids = np.ascontiguousarray(ids, np.uint32)
        n = ids.size
        h = self.cfg["hidden"]
        x = np.empty((n, h), np.float32)
        lib().orc_embed(_p(self.embed), h, _p(ids), n, self.embed_scale, _p(x))
        sin = np.ascontiguousarray(sin[:n], np.float32)
        cos = np.ascontiguousarray(cos[:n], np.float32)
        if sin_local is not None:
            sin_local = np.ascontiguousarray(sin_local[:n], np.float32)
            cos_local = np.ascontiguousarray(cos_local[:n], np.float32)
        out = np.empty((n - logits_from, self.cfg["vocab"]), np.float32)
        rc = lib().orc_forward(C.byref(self.c), self.layers, _p(self.final_gamma),
                               _p(self.lm_head), _p(sin), _p(cos), _p(sin_local), _p(cos_local),
                               _p(x), n, logits_from, _p(out), threads)
        if rc != 0:
            raise ValueError("oracle forward rejected the arguments")
        return out
