"""Decoder weights: the checkpoint loader of reng-model and seeded random init.

`load_weights(dir)` mirrors crates/reng-model/src/lib.rs:1477-1688: it maps
`model.safetensors` (or the shards of `model.safetensors.index.json`) and
returns bf16 views without copying (the reference's `Bf16Slice`,
lib.rs:755-999) where no family rule rewrites a tensor, with q/k/v biases
and q/k norm gains when present (lib.rs:1605-1630) and the embedding as the
LM head when the embeddings are tied (lib.rs:1666-1674).  Tensor names are
the HF ones of the families the reference loads.

A weights object is a dict:
  {"layers": [{"wq","wk","wv","wo","wg","wu","wd": bf16 bits [out, in] (u16),
               "g1","g2": f32 [hidden], "bq","bk","bv": f32 or absent,
               "qn","kn","g_post_attn","g_post_mlp": f32 or absent}],
   "embed": u16 [vocab, hidden], "lm_head": u16 [vocab, hidden],
   "final_gamma": f32 [hidden]}
with numpy arrays (host) or torch tensors on a CUDA device (device memory).
"""
import json
import mmap
import os
import struct

import numpy as np

from .synth import bf16_bits_to_f32, f32_to_bf16_bits

NAMES = {
    "wq": "self_attn.q_proj.weight", "wk": "self_attn.k_proj.weight",
    "wv": "self_attn.v_proj.weight", "wo": "self_attn.o_proj.weight",
    "wg": "mlp.gate_proj.weight", "wu": "mlp.up_proj.weight", "wd": "mlp.down_proj.weight",
    "g1": "input_layernorm.weight", "g2": "post_attention_layernorm.weight",
    "bq": "self_attn.q_proj.bias", "bk": "self_attn.k_proj.bias", "bv": "self_attn.v_proj.bias",
    "qn": "self_attn.q_norm.weight", "kn": "self_attn.k_norm.weight",
}
MATS = ("wq", "wk", "wv", "wo", "wg", "wu", "wd")
VECS = ("g1", "g2", "bq", "bk", "bv", "qn", "kn")

_DT = {"BF16": (np.uint16, 2), "F32": (np.float32, 4), "F16": (np.float16, 2)}


class SafeTensors:
    """A memory-mapped safetensors file: name -> numpy view (no copy)."""

    def __init__(self, path):
        self.path = path
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        (n,) = struct.unpack("<Q", self._mm[:8])
        self.header = json.loads(self._mm[8:8 + n].decode())
        self.header.pop("__metadata__", None)
        self._base = 8 + n

    def names(self):
        return list(self.header)

    def dtype(self, name):
        return self.header[name]["dtype"]

    def shape(self, name):
        return tuple(self.header[name]["shape"])

    def view(self, name):
        h = self.header[name]
        if h["dtype"] not in _DT:
            raise ValueError("%s: dtype %s is not supported" % (name, h["dtype"]))
        dt, _ = _DT[h["dtype"]]
        a, b = h["data_offsets"]
        arr = np.frombuffer(self._mm, dtype=dt, count=(b - a) // np.dtype(dt).itemsize,
                            offset=self._base + a)
        return arr.reshape(h["shape"])


def write_safetensors(path, tensors):
    """Write {name: (dtype_str, numpy array)} as a safetensors file."""
    header, off, blobs = {}, 0, []
    for name, (dt, arr) in tensors.items():
        raw = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in blobs:
            f.write(b)


def _as_bf16(st, name):
    dt = st.dtype(name)
    v = st.view(name)
    if dt == "BF16":
        return v
    return f32_to_bf16_bits(v.astype(np.float32))


def _as_f32(st, name):
    dt = st.dtype(name)
    v = st.view(name)
    if dt == "BF16":
        return bf16_bits_to_f32(v).reshape(v.shape)
    return v.astype(np.float32)


def scale_bf16(w, s):
    """bf16(f32(w) * s), round to nearest even (the reference's scale_bf16,
    crates/reng-synapse/src/lib.rs:61-69): a scaled copy of bf16 bits."""
    return f32_to_bf16_bits(bf16_bits_to_f32(np.asarray(w)) * np.float32(s))


def permute_head_rows(m, hd, perm):
    """Rows of every hd-row head block reordered: row e of a block is the
    block's row perm[e] (lib.rs:2253-2275); works for matrices and vectors."""
    m = np.asarray(m)
    blocks = m.reshape((m.shape[0] // hd, hd) + m.shape[1:])
    return np.ascontiguousarray(blocks[:, perm].reshape(m.shape))


def _open(model_dir):
    idx = os.path.join(model_dir, "model.safetensors.index.json")
    if os.path.exists(idx):
        with open(idx) as f:
            wm = json.load(f)["weight_map"]
        sts = {fn: SafeTensors(os.path.join(model_dir, fn)) for fn in set(wm.values())}
        return {name: sts[fn] for name, fn in wm.items()}
    st = SafeTensors(os.path.join(model_dir, "model.safetensors"))
    return {n: st for n in st.names()}


def load_weights(model_dir, cfg):
    """Map the checkpoint of `model_dir` (reng-model load_weights,
    crates/reng-model/src/lib.rs:1477-1688).  Per family, as the reference:
    Phi-3's fused qkv_proj / gate_up_proj split into row blocks; Gemma's
    zero-centred gains applied as 1 + w, its four norms (pre-norms g1 / g2,
    branch-output norms g_post_attn / g_post_mlp) and a final norm carrying
    1 / final softcap; OLMo-2's branch-output norms as g1 / g2; optional
    q/k/v biases and q/k norm gains; a partial rotation's q/k head dims put
    in the kernel's pair order (rope_head_perm); Granite's residual
    multiplier folded into o_proj / down_proj and 1 / logits_scaling into
    the LM head's own copy (scale_bf16).  The embedding stays as stored
    (its scale is applied at the gather)."""
    from .rope import rope_head_perm
    raw = cfg.raw or {}
    if raw.get("mlp_bias"):
        raise ValueError("mlp_bias is not supported")
    where = _open(model_dir)

    def get(name, kind, shape):
        if name not in where:
            raise ValueError("checkpoint lacks %s" % name)
        st = where[name]
        if tuple(st.shape(name)) != tuple(shape):
            raise ValueError("%s: shape %s, expected %s" % (name, st.shape(name), shape))
        return _as_bf16(st, name) if kind == "bf16" else _as_f32(st, name)

    h, hd = cfg.hidden_size, cfg.head_dim()
    qd, kvd, inter, V = cfg.q_dim(), cfg.n_kv_heads() * hd, cfg.intermediate_size, cfg.vocab_size
    pre = cfg.weight_prefix or "model."
    gemma, post = cfg.is_gemma(), cfg.post_norm()

    def plus_one(v):
        return (v + np.float32(1.0)).astype(np.float32) if gemma else v

    perm = rope_head_perm(hd, cfg.rotary_dim()) if cfg.rotary_dim() < hd else None
    rmul = raw.get("residual_multiplier")
    embed = get(pre + "embed_tokens.weight", "bf16", (V, h))
    layers = []
    for l in range(cfg.num_hidden_layers):
        p = "%slayers.%d." % (pre, l)

        def opt(name, lens):
            n = p + name
            if n not in where:
                return None
            shp = where[n].shape(n)
            if len(shp) != 1 or shp[0] not in lens:
                raise ValueError("%s: shape %s, expected one of %s" % (n, shp, lens))
            return _as_f32(where[n], n)

        lw = {}
        if p + "self_attn.qkv_proj.weight" in where:
            qkv = get(p + "self_attn.qkv_proj.weight", "bf16", (qd + 2 * kvd, h))
            lw["wq"], lw["wk"], lw["wv"] = qkv[:qd], qkv[qd:qd + kvd], qkv[qd + kvd:]
        else:
            lw["wq"] = get(p + NAMES["wq"], "bf16", (qd, h))
            lw["wk"] = get(p + NAMES["wk"], "bf16", (kvd, h))
            lw["wv"] = get(p + NAMES["wv"], "bf16", (kvd, h))
        if p + "mlp.gate_up_proj.weight" in where:
            gu = get(p + "mlp.gate_up_proj.weight", "bf16", (2 * inter, h))
            lw["wg"], lw["wu"] = gu[:inter], gu[inter:]
        else:
            lw["wg"] = get(p + NAMES["wg"], "bf16", (inter, h))
            lw["wu"] = get(p + NAMES["wu"], "bf16", (inter, h))
        lw["wo"] = get(p + NAMES["wo"], "bf16", (h, qd))
        lw["wd"] = get(p + NAMES["wd"], "bf16", (h, inter))
        if rmul is not None:
            lw["wo"], lw["wd"] = scale_bf16(lw["wo"], rmul), scale_bf16(lw["wd"], rmul)

        def g(name):
            return plus_one(get(p + name, "f32", (h,)))

        if gemma:
            lw["g1"], lw["g2"] = g("input_layernorm.weight"), g("pre_feedforward_layernorm.weight")
            lw["g_post_attn"] = g("post_attention_layernorm.weight")
            lw["g_post_mlp"] = g("post_feedforward_layernorm.weight")
        elif post:
            lw["g1"] = g("post_attention_layernorm.weight")
            lw["g2"] = g("post_feedforward_layernorm.weight")
        else:
            lw["g1"], lw["g2"] = g("input_layernorm.weight"), g("post_attention_layernorm.weight")
        for k, lens in (("bq", (qd,)), ("bk", (kvd,)), ("bv", (kvd,))):
            v = opt(NAMES[k], lens)
            if v is not None:
                lw[k] = v
        for k, lens in (("qn", (hd, qd)), ("kn", (hd, kvd))):
            # per head (Qwen3, Gemma-3) or over the whole projection (OLMo-2),
            # lib.rs:1607-1609
            v = opt(NAMES[k], lens)
            if v is not None:
                lw[k] = plus_one(v)
        if perm is not None:
            for k in ("wq", "wk", "bq", "bk", "qn", "kn"):
                if k in lw:
                    lw[k] = permute_head_rows(lw[k], hd, perm)
        layers.append(lw)
    fg = plus_one(get(pre + "norm.weight", "f32", (h,)))
    cap = cfg.final_softcap()
    if cap is not None:
        # Gemma-2: tanh(logits / cap) * cap, the division on the final gain
        fg = (fg / np.float32(cap)).astype(np.float32)
    outer = pre[:-len("model.")] if pre.endswith("model.") else ""
    heads = [outer + "lm_head.weight"] + (["lm_head.weight"] if outer else [])
    head = next((n for n in heads if n in where), None)
    if head is not None:
        lm = get(head, "bf16", (V, h))
    elif cfg.tied():
        lm = embed
    else:
        raise ValueError("lm_head.weight missing and embeddings are not tied")
    ls = raw.get("logits_scaling")
    if ls is not None:
        lm = scale_bf16(lm, np.float32(1.0) / np.float32(ls))
    return {"layers": layers, "embed": embed, "lm_head": lm, "final_gamma": fg}


def save_checkpoint(model_dir, cfg, w):
    """Write config.json + model.safetensors of host weights `w` (for tests)."""
    os.makedirs(model_dir, exist_ok=True)
    with open(os.path.join(model_dir, "config.json"), "w") as f:
        json.dump(cfg.to_dict(), f, indent=1)
    t = {}
    for l, lw in enumerate(w["layers"]):
        for k in MATS:
            t["model.layers.%d.%s" % (l, NAMES[k])] = ("BF16", np.asarray(lw[k]))
        for k in VECS:
            if lw.get(k) is not None:
                t["model.layers.%d.%s" % (l, NAMES[k])] = ("F32", np.asarray(lw[k], np.float32))
    t["model.embed_tokens.weight"] = ("BF16", np.asarray(w["embed"]))
    if not cfg.tie_word_embeddings:
        t["lm_head.weight"] = ("BF16", np.asarray(w["lm_head"]))
    t["model.norm.weight"] = ("F32", np.asarray(w["final_gamma"], np.float32))
    write_safetensors(os.path.join(model_dir, "model.safetensors"), t)


def random_weights(cfg, seed=0, device="cpu", std=0.02, layers=None):
    """Seeded random init: projections and embedding N(0, std) in bf16, norm
    gains 1.0, biases N(0, std).  device="cpu" gives numpy arrays, a CUDA
    device gives torch tensors in HBM (generated there).  `layers` limits
    the depth (a layer-truncated model of the same widths)."""
    import torch
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    h, hd = cfg.hidden_size, cfg.head_dim()
    qd, kvd, inter, V = cfg.q_dim(), cfg.n_kv_heads() * hd, cfg.intermediate_size, cfg.vocab_size
    L = cfg.num_hidden_layers if layers is None else layers

    def mat(r, c):
        t = torch.empty((r, c), dtype=torch.float32, device=dev)
        t.normal_(0.0, std, generator=gen)
        b = t.to(torch.bfloat16).view(torch.int16)
        return b.numpy().view(np.uint16) if dev.type == "cpu" else b

    def vec(n, fill=None):
        t = torch.empty(n, dtype=torch.float32, device=dev)
        if fill is None:
            t.normal_(0.0, std, generator=gen)
        else:
            t.fill_(fill)
        return t.numpy() if dev.type == "cpu" else t

    layers_out = []
    for _ in range(L):
        lw = {"wq": mat(qd, h), "wk": mat(kvd, h), "wv": mat(kvd, h), "wo": mat(h, qd),
              "wg": mat(inter, h), "wu": mat(inter, h), "wd": mat(h, inter),
              "g1": vec(h, 1.0), "g2": vec(h, 1.0)}
        if cfg.has_bias():
            lw.update({"bq": vec(qd), "bk": vec(kvd), "bv": vec(kvd)})
        layers_out.append(lw)
    embed = mat(V, h)
    lm = embed if cfg.tie_word_embeddings else mat(V, h)
    return {"layers": layers_out, "embed": embed, "lm_head": lm, "final_gamma": vec(h, 1.0)}


def to_host(w):
    """numpy copies of a weights dict (torch tensors are brought to the host)."""
    def conv(x):
        if x is None:
            return None
        if isinstance(x, np.ndarray):
            return x
        t = x.detach().cpu()
        if t.dtype == torch_int16():
            return t.numpy().view(np.uint16)
        return t.numpy()
    out = {"layers": [{k: conv(v) for k, v in lw.items()} for lw in w["layers"]],
           "embed": conv(w["embed"]), "final_gamma": conv(w["final_gamma"])}
    out["lm_head"] = out["embed"] if w["lm_head"] is w["embed"] else conv(w["lm_head"])
    return out


def torch_int16():
    import torch
    return torch.int16
