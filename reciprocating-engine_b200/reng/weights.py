"""Decoder weights: the checkpoint loader of reng-model and seeded random init.

`load_weights(dir)` mirrors crates/reng-model/src/lib.rs:1477-1688: it maps
`model.safetensors` (or the shards of `model.safetensors.index.json`) and
returns bf16 views without copying (the reference's `Bf16Slice`,
lib.rs:755-999), with q/k/v biases when present (lib.rs:1605-1630) and the
embedding as the LM head when the embeddings are tied (lib.rs:1666-1674).
Tensor names are the HF Llama / Qwen2 ones.

A weights object is a dict:
  {"layers": [{"wq","wk","wv","wo","wg","wu","wd": bf16 bits [out, in] (u16),
               "g1","g2": f32 [hidden], "bq","bk","bv": f32 or absent}],
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


def load_weights(model_dir, cfg):
    """Map the checkpoint of `model_dir` (reng-model load_weights)."""
    idx = os.path.join(model_dir, "model.safetensors.index.json")
    files = {}
    if os.path.exists(idx):
        with open(idx) as f:
            wm = json.load(f)["weight_map"]
        for name, fn in wm.items():
            files.setdefault(fn, None)
        sts = {fn: SafeTensors(os.path.join(model_dir, fn)) for fn in files}
        where = {name: sts[fn] for name, fn in wm.items()}
    else:
        st = SafeTensors(os.path.join(model_dir, "model.safetensors"))
        where = {n: st for n in st.names()}

    def get(name, kind, shape):
        if name not in where:
            raise ValueError("checkpoint lacks %s" % name)
        st = where[name]
        if tuple(st.shape(name)) != tuple(shape):
            raise ValueError("%s: shape %s, expected %s" % (name, st.shape(name), shape))
        return _as_bf16(st, name) if kind == "bf16" else _as_f32(st, name)

    h, hd = cfg.hidden_size, cfg.head_dim()
    qd, kvd, inter = cfg.q_dim(), cfg.n_kv_heads() * hd, cfg.intermediate_size
    shapes = {"wq": (qd, h), "wk": (kvd, h), "wv": (kvd, h), "wo": (h, qd), "wg": (inter, h),
              "wu": (inter, h), "wd": (h, inter), "g1": (h,), "g2": (h,), "bq": (qd,),
              "bk": (kvd,), "bv": (kvd,)}
    layers = []
    for l in range(cfg.num_hidden_layers):
        lw = {}
        for k in MATS:
            lw[k] = get("model.layers.%d.%s" % (l, NAMES[k]), "bf16", shapes[k])
        for k in ("g1", "g2"):
            lw[k] = get("model.layers.%d.%s" % (l, NAMES[k]), "f32", shapes[k])
        if cfg.has_bias():
            for k in ("bq", "bk", "bv"):
                lw[k] = get("model.layers.%d.%s" % (l, NAMES[k]), "f32", shapes[k])
        for k, full in (("qn", qd), ("kn", kvd)):
            # optional q/k norm gains: [head_dim] per head (Qwen3) or the whole
            # projection row (OLMo-2), as reng-model reads them
            # (crates/reng-model/src/lib.rs:1607-1609)
            name = "model.layers.%d.%s" % (l, NAMES[k])
            if name in where:
                n = where[name].shape(name)
                lw[k] = get(name, "f32", (hd,) if tuple(n) == (hd,) else (full,))
        layers.append(lw)
    embed = get("model.embed_tokens.weight", "bf16", (cfg.vocab_size, h))
    if cfg.tie_word_embeddings or "lm_head.weight" not in where:
        lm = embed
    else:
        lm = get("lm_head.weight", "bf16", (cfg.vocab_size, h))
    fg = get("model.norm.weight", "f32", (h,))
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
