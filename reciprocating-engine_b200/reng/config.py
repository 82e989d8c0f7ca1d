"""`LlamaConfig`: the config.json contract of the reference's loader.

Mirrors crates/reng-model/src/lib.rs: `LlamaConfig` (lib.rs:84-193),
`from_json` (lib.rs:488-618), `n_kv_heads` / `head_dim` / `rotary_dim` /
`q_dim` / `attention_scale` (lib.rs:666-705) and `shard` (lib.rs:725-742),
and the per-family rules of lib.rs:268-420 (windows, Gemma sliding layers
and softcaps, embedding scale, post-norm).  The engine runs the Llama /
Qwen2 / Mistral decoder and Granite / Phi-3 checkpoints as loaded, and
refuses the rest (`unsupported`); the loader and the f32 oracle take every
family the reference's host forward does.  A
multimodal Gemma-3 config parses through its `text_config`.
"""
import copy
import json
import math
import os
from dataclasses import dataclass, field
from typing import Optional


# Gemma3TextConfig's defaults for the keys a multimodal config.json leaves out
GEMMA3_TEXT_DEFAULTS = {
    "model_type": "gemma3_text", "vocab_size": 262208, "hidden_size": 2304,
    "intermediate_size": 9216, "num_hidden_layers": 26, "num_attention_heads": 8,
    "num_key_value_heads": 4, "head_dim": 256, "hidden_activation": "gelu_pytorch_tanh",
    "max_position_embeddings": 131072, "rms_norm_eps": 1e-6, "tie_word_embeddings": True,
    "query_pre_attn_scalar": 256, "sliding_window": 4096, "sliding_window_pattern": 6,
    "rope_theta": 1000000.0, "rope_local_base_freq": 10000.0,
}


# Gemma text model types: zero-centred norm gains, sqrt(hidden) embedding
# scale, GELU-tanh, per-layer sliding windows, tied head by default
GEMMA_TYPES = ("gemma2", "gemma3_text")


@dataclass
class RopeScaling:
    rope_type: Optional[str] = None
    factor: Optional[float] = None
    low_freq_factor: Optional[float] = None
    high_freq_factor: Optional[float] = None
    original_max_position_embeddings: Optional[int] = None
    max_position_embeddings: Optional[int] = None
    attention_factor: Optional[float] = None
    beta_fast: Optional[float] = None
    beta_slow: Optional[float] = None
    mscale: Optional[float] = None
    mscale_all_dim: Optional[float] = None
    truncate: Optional[bool] = None
    short_factor: Optional[list] = None
    long_factor: Optional[list] = None


@dataclass
class LlamaConfig:
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    vocab_size: int
    num_key_value_heads: Optional[int] = None
    head_dim_: Optional[int] = None
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    rope_scaling: Optional[RopeScaling] = None
    partial_rotary_factor: Optional[float] = None
    tie_word_embeddings: bool = False
    attention_bias: bool = False
    model_type: Optional[str] = None
    max_position_embeddings: Optional[int] = None
    hidden_act: str = "silu"
    rope_local_base_freq: Optional[float] = None
    weight_prefix: Optional[str] = None
    raw: dict = field(default_factory=dict, repr=False)

    # ----------------------------------------------------------- parsing --
    @staticmethod
    def from_dict(d):
        """from_json's rules (lib.rs:488-618): a multimodal Gemma-3 config
        flattens to its text_config completed with Gemma3TextConfig's
        defaults; rope_scaling gets the top-level lengths; Phi-3's legacy
        "su"/"yarn" types mean longrope."""
        d = dict(d)
        if d.get("model_type") == "gemma3":
            if not isinstance(d.get("text_config"), dict):
                raise ValueError("config.json: gemma3 without text_config")
            t = dict(GEMMA3_TEXT_DEFAULTS)
            t.update(d["text_config"])
            d = t
            prefix = "language_model.model."
        else:
            prefix = None
        rp = d.get("rope_parameters")
        rope_theta = d.get("rope_theta")
        rs = d.get("rope_scaling")
        if isinstance(rp, dict):  # transformers 5 "rope_parameters" form
            rope_theta = rope_theta if rope_theta is not None else rp.get("rope_theta")
            if rs is None and rp.get("rope_type", "default") != "default":
                rs = rp
        scaling = None
        if isinstance(rs, dict):
            rtype = rs.get("rope_type", rs.get("type"))
            if d.get("model_type") == "phi3" and rtype in ("su", "yarn"):
                rtype = "longrope"
            max_pos = d.get("max_position_embeddings")
            orig = d.get("original_max_position_embeddings")
            if orig is None:
                orig = rs.get("original_max_position_embeddings", max_pos)
            scaling = RopeScaling(
                rope_type=rtype, factor=rs.get("factor"),
                low_freq_factor=rs.get("low_freq_factor"),
                high_freq_factor=rs.get("high_freq_factor"),
                original_max_position_embeddings=orig, max_position_embeddings=max_pos,
                attention_factor=rs.get("attention_factor"),
                beta_fast=rs.get("beta_fast"), beta_slow=rs.get("beta_slow"),
                mscale=rs.get("mscale"), mscale_all_dim=rs.get("mscale_all_dim"),
                truncate=rs.get("truncate"),
                short_factor=rs.get("short_factor"), long_factor=rs.get("long_factor"))
        for k in ("hidden_size", "intermediate_size", "num_hidden_layers",
                  "num_attention_heads", "vocab_size"):
            if k not in d:
                raise ValueError("config.json: missing %s" % k)
        mt = d.get("model_type")
        cfg = LlamaConfig(
            hidden_size=int(d["hidden_size"]), intermediate_size=int(d["intermediate_size"]),
            num_hidden_layers=int(d["num_hidden_layers"]),
            num_attention_heads=int(d["num_attention_heads"]), vocab_size=int(d["vocab_size"]),
            num_key_value_heads=d.get("num_key_value_heads"), head_dim_=d.get("head_dim"),
            rms_norm_eps=float(d.get("rms_norm_eps", 1e-6)),
            rope_theta=float(rope_theta if rope_theta is not None else 10000.0),
            rope_scaling=scaling, partial_rotary_factor=d.get("partial_rotary_factor"),
            tie_word_embeddings=bool(d.get("tie_word_embeddings", mt in GEMMA_TYPES)),
            attention_bias=bool(d.get("attention_bias", mt == "qwen2")),
            model_type=mt, max_position_embeddings=d.get("max_position_embeddings"),
            hidden_act=d.get("hidden_activation") or d.get("hidden_act") or "silu",
            rope_local_base_freq=d.get("rope_local_base_freq"), weight_prefix=prefix, raw=d)
        if cfg.partial_rotary_factor is not None:
            f, rd = float(cfg.partial_rotary_factor), cfg.rotary_dim()
            if not (0.0 < f <= 1.0) or rd == 0 or rd % 2:
                raise ValueError("config.json: partial_rotary_factor %r rotates %d of %d head dims"
                                 % (f, rd, cfg.head_dim()))
        cfg._check_scaling()
        cfg.activation()
        return cfg

    def _check_scaling(self):
        """Every parameter the rope type's table needs, and longrope's one
        factor per rotary pair, refused at load as the reference does
        (lib.rs:553-612, after transformers' validate_rope)."""
        s = self.rope_scaling
        if s is None:
            return
        t = s.rope_type or "default"

        def need(name, have):
            if not have:
                raise ValueError("config.json: rope_scaling.%s is required by rope_type %s" % (name, t))

        factor = s.factor is not None or (s.max_position_embeddings is not None and
                                          s.original_max_position_embeddings is not None)
        orig = s.original_max_position_embeddings is not None
        if t == "llama3":
            need("factor", s.factor is not None)
            need("low_freq_factor", s.low_freq_factor is not None)
            need("high_freq_factor", s.high_freq_factor is not None)
            need("original_max_position_embeddings", orig)
        elif t == "linear":
            need("factor", s.factor is not None)
        elif t == "yarn":
            need("factor", factor)
            need("original_max_position_embeddings", orig)
        elif t == "longrope":
            need("factor", factor)
            need("original_max_position_embeddings", orig)
            need("short_factor", s.short_factor is not None)
            need("long_factor", s.long_factor is not None)
            half = self.rotary_dim() // 2
            for name, lst in (("short_factor", s.short_factor), ("long_factor", s.long_factor)):
                if len(lst) != half:
                    raise ValueError("config.json: rope_scaling.%s has %d entries for %d rotary pairs"
                                     % (name, len(lst), half))

    def longrope_capacity_warning(self, capacity):
        """The warning a cached run deserves when its capacity, past the
        pretraining length, makes every position read longrope's long
        factors (lib.rs:445-458); None otherwise."""
        s = self.rope_scaling
        if s is None or s.rope_type != "longrope" or s.original_max_position_embeddings is None:
            return None
        orig = int(s.original_max_position_embeddings)
        if capacity <= orig:
            return None
        return ("rope_scaling: cache capacity %d is past the pretraining length %d, so the longrope "
                "long factors serve every position; size the cache to the run's length to match "
                "transformers" % (capacity, orig))

    @staticmethod
    def from_json(text):
        return LlamaConfig.from_dict(json.loads(text))

    # ----------------------------------------------------------- context --
    def trained_context(self):
        """max_position_embeddings when positive (lib.rs:627-629)."""
        n = self.max_position_embeddings
        return int(n) if n else None

    def original_context(self):
        """The pre-scaling context a rope_scaling states (lib.rs:636-641)."""
        s = self.rope_scaling
        n = None if s is None else s.original_max_position_embeddings
        return int(n) if n else None

    def context_warning(self, positions):
        """A warning when `positions` runs past the trained context, else
        None (lib.rs:646-663)."""
        trained = self.trained_context()
        if trained is None or positions <= trained:
            return None
        o = self.original_context()
        scaled = (" (rope scaling stretches a %d-position model to %d)" % (o, trained)
                  if o is not None and o < trained else "")
        return ("warning: %d positions exceed this model's trained context of %d%s; the engine will "
                "run it, but the rotary embeddings are extrapolating and the output past position %d "
                "is not what the checkpoint was trained to produce" % (positions, trained, scaled, trained))

    # ------------------------------------------------------ family rules --
    # crates/reng-model/src/lib.rs:268-420 and :697-712, read from the
    # config.json keys this dataclass keeps in `raw`.
    def _opt(self, key):
        v = (self.raw or {}).get(key)
        return None if v is None else v

    def is_gemma(self):
        """gemma2 / gemma3_text (lib.rs:290-292)."""
        return self.model_type in GEMMA_TYPES

    def post_norm(self):
        """OLMo-2 normalises the branch outputs, not the inputs (lib.rs:707-712)."""
        return self.model_type == "olmo2"

    def tied(self):
        return bool(self.tie_word_embeddings)

    def embed_scale(self):
        """Factor on the gathered embedding rows, f32 (lib.rs:303-312):
        Gemma's sqrt(hidden) times Granite's embedding_multiplier."""
        import numpy as np
        g = np.sqrt(np.float32(self.hidden_size)) if self.is_gemma() else np.float32(1.0)
        m = self._opt("embedding_multiplier")
        return float(np.float32(g) * np.float32(1.0 if m is None else m))

    def activation(self):
        """"silu" or "gelu_tanh"; anything else is an error (lib.rs:319-331)."""
        name = self.hidden_act or "silu"
        if name == "silu":
            return "silu"
        if name == "gelu_pytorch_tanh":
            return "gelu_tanh"
        raise ValueError("config.json: activation %s is not supported" % name)

    def window(self):
        """The model-wide sliding window (lib.rs:275-287): Phi-3 and Mistral
        always, Qwen2/Qwen3 only with use_sliding_window true."""
        w = self._opt("sliding_window")
        w = int(w) if w else None
        if self.model_type in ("phi3", "mistral"):
            return w
        if self.model_type in ("qwen2", "qwen3") and self._opt("use_sliding_window") is True:
            return w
        return None

    def sliding(self, li):
        """Whether Gemma layer li is a sliding-attention layer (lib.rs:337-350)."""
        if not self.is_gemma():
            return False
        types = self._opt("layer_types")
        if types is not None:
            return li < len(types) and types[li] == "sliding_attention"
        pattern = 2 if self.model_type == "gemma2" else int(self._opt("sliding_window_pattern") or 6)
        return (li + 1) % pattern != 0

    def layer_window(self, li):
        """Layer li's window (lib.rs:356-366)."""
        if not self.is_gemma():
            return self.window()
        if not self.sliding(li):
            return None
        w = self._opt("sliding_window")
        return int(w) if w else None

    def attn_softcap(self):
        """Gemma-2's attn_logit_softcapping (lib.rs:370-377)."""
        c = self._opt("attn_logit_softcapping")
        return float(c) if self.model_type == "gemma2" and c is not None and c > 0 else None

    def final_softcap(self):
        c = self._opt("final_logit_softcapping")
        return float(c) if c is not None and c > 0 else None

    def local_rope(self, li):
        """Gemma-3 sliding layers read the local RoPE table (lib.rs:387-390)."""
        return self.model_type == "gemma3_text" and self.sliding(li)

    def use_rope(self, li):
        """False on SmolLM3's NoPE layers (no_rope_layers[li] == 0)."""
        v = self._opt("no_rope_layers")
        return v is None or li >= len(v) or v[li] != 0

    # ------------------------------------------------------ engine support --
    # the families whose layers are this engine's decoder as loaded: Granite
    # once load_weights has folded its multipliers into the weights (the
    # embedding one is applied at the gather), Phi-3 once its partial
    # rotation is permuted into the kernels' pair order, SmolLM3 with its
    # NoPE layers rotating nothing
    ENGINE_TYPES = (None, "llama", "qwen2", "qwen3", "mistral", "granite", "phi3", "smollm3")

    def unsupported(self, capacity=None):
        """What this engine's kernels do not compute for this config (empty
        when it runs as written).  The reference parses more families than
        its device graph covers and refuses what it has no node for
        (`activation`, lib.rs:318-330; `mlp_bias`, :1479); this engine does
        the same for the features outside the decoder it runs, instead of
        computing a plain Llama in their place.  It runs weights in the form
        load_weights gives them: Granite's residual multiplier and
        1/logits_scaling folded in, a partial rotation's q/k head dims in
        pair order (the RoPE tables carry the identity on the pass-through
        pairs)."""
        out = []
        raw = self.raw or {}
        if self.model_type not in self.ENGINE_TYPES:
            out.append("model_type %s" % self.model_type)
        if (self.hidden_act or "silu") != "silu":
            out.append("activation %s" % self.hidden_act)
        if raw.get("mlp_bias"):
            out.append("mlp_bias")
        for k in ("final_logit_softcapping", "attn_logit_softcapping", "query_pre_attn_scalar"):
            if raw.get(k) is not None:
                out.append(k)
        if raw.get("qk_norm") or raw.get("use_qk_norm"):
            out.append("q/k RMSNorm")
        win = self.window()
        if win and capacity is not None and capacity > win:
            out.append("sliding window %d below the capacity %d" % (win, capacity))
        return out

    @staticmethod
    def load(model_dir):
        with open(os.path.join(model_dir, "config.json")) as f:
            return LlamaConfig.from_json(f.read())

    def to_dict(self):
        d = dict(self.raw) if self.raw else {}
        d.update({
            "hidden_size": self.hidden_size, "intermediate_size": self.intermediate_size,
            "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads, "vocab_size": self.vocab_size,
            "num_key_value_heads": self.n_kv_heads(), "head_dim": self.head_dim(),
            "rms_norm_eps": self.rms_norm_eps, "rope_theta": self.rope_theta,
            "tie_word_embeddings": self.tie_word_embeddings, "hidden_act": self.hidden_act,
            "model_type": self.model_type or "llama",
        })
        if self.model_type == "qwen2" or self.attention_bias:
            d["attention_bias"] = self.attention_bias
        return d

    # ---------------------------------------------------------- geometry --
    def n_kv_heads(self):
        return int(self.num_key_value_heads or self.num_attention_heads)

    def head_dim(self):
        return int(self.head_dim_ or self.hidden_size // self.num_attention_heads)

    def rotary_dim(self):
        hd = self.head_dim()
        if self.partial_rotary_factor is None:
            return hd
        return int(hd * float(self.partial_rotary_factor))

    def q_dim(self):
        return self.num_attention_heads * self.head_dim()

    def attention_scale(self):
        """The softmax scale on q.k, as an f32 (lib.rs:697-705): Granite's
        attention_multiplier, else Gemma's 1/sqrt(query_pre_attn_scalar),
        else 1/sqrt(head_dim)."""
        import numpy as np
        m = self._opt("attention_multiplier")
        if m is not None:
            return float(np.float32(m))
        s = self._opt("query_pre_attn_scalar")
        base = np.float32(s) if s is not None else np.float32(self.head_dim())
        return float(np.float32(1.0) / np.sqrt(base))

    def has_bias(self):
        return bool(self.attention_bias)

    def shard(self, rank, world):
        """The config of one tensor-parallel shard (lib.rs:725-742)."""
        if not (world >= 1 and 0 <= rank < world):
            raise ValueError("rank %d of %d" % (rank, world))
        nkv = self.n_kv_heads()
        if (self.num_attention_heads % world or nkv % world or self.intermediate_size % world):
            raise ValueError("heads %d / kv heads %d / intermediate %d are not divisible by %d"
                             % (self.num_attention_heads, nkv, self.intermediate_size, world))
        c = copy.deepcopy(self)
        c.head_dim_ = self.head_dim()
        c.num_attention_heads = self.num_attention_heads // world
        c.num_key_value_heads = nkv // world
        c.intermediate_size = self.intermediate_size // world
        return c

    def active_params(self):
        """Params touched per token: attention + MLP per layer + LM head
        (reng-ceiling active_params, crates/reng-ceiling/src/lib.rs:184-207)."""
        h, hd = self.hidden_size, self.head_dim()
        attn = h * self.q_dim() * 2 + h * self.n_kv_heads() * hd * 2
        mlp = 3 * h * self.intermediate_size
        return self.num_hidden_layers * (attn + mlp) + h * self.vocab_size

    def kv_bytes_per_token(self, kv_bytes=2):
        return 2 * self.n_kv_heads() * self.head_dim() * self.num_hidden_layers * kv_bytes


# The BASELINE shapes (random-init weights; synthetic config.json contents).
def smollm2_135m():
    return LlamaConfig(hidden_size=576, intermediate_size=1536, num_hidden_layers=30,
                       num_attention_heads=9, num_key_value_heads=3, head_dim_=64,
                       vocab_size=49152, rms_norm_eps=1e-5, rope_theta=100000.0,
                       tie_word_embeddings=True, model_type="llama")


def llama31_8b():
    return LlamaConfig(hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                       num_attention_heads=32, num_key_value_heads=8, head_dim_=128,
                       vocab_size=128256, rms_norm_eps=1e-5, rope_theta=500000.0,
                       tie_word_embeddings=False, model_type="llama")


def qwen25_32b():
    return LlamaConfig(hidden_size=5120, intermediate_size=27648, num_hidden_layers=64,
                       num_attention_heads=40, num_key_value_heads=8, head_dim_=128,
                       vocab_size=152064, rms_norm_eps=1e-6, rope_theta=1000000.0,
                       tie_word_embeddings=False, attention_bias=True, model_type="qwen2")


SHAPES = {"smollm2-135m": smollm2_135m, "llama-3.1-8b": llama31_8b, "qwen2.5-32b": qwen25_32b}
