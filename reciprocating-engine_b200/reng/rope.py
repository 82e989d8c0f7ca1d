"""RoPE tables of reng-model (crates/reng-model/src/lib.rs:1968-2276).

`rope_spec` (lib.rs:2015-2143) computes the inverse frequencies and the
attention factor with the config's rope_scaling (llama3, linear, yarn,
longrope; anything else keeps the default table), in f32 as the reference
does; `rope_caches_partial` (lib.rs:2188-2216) builds the [positions,
head_dim] sin/cos tables in the kernel's rotate-half pair order.
"""
import math

import numpy as np

F = np.float32


def rope_spec(rotary_dim, theta, scaling=None, seq_len=0):
    half = rotary_dim // 2
    theta = F(theta)
    inv = np.array([np.power(theta, F(F(-2.0) * F(i) / F(rotary_dim)), dtype=F)
                    for i in range(half)], F)
    af = F(1.0)
    if scaling is None:
        return inv, float(af)
    rtype = scaling.rope_type or "default"

    def orig():
        if scaling.original_max_position_embeddings is None:
            raise ValueError("this rope scaling needs original_max_position_embeddings in rope_scaling")
        return F(scaling.original_max_position_embeddings)

    def factor_or_ratio():
        if scaling.factor is not None:
            return F(scaling.factor)
        return F(F(scaling.max_position_embeddings) / orig())

    two_pi = F(2.0) * F(math.pi)
    if rtype == "llama3":
        factor, low, high = F(scaling.factor), F(scaling.low_freq_factor), F(scaling.high_freq_factor)
        o = orig()
        low_w, high_w = F(o / low), F(o / high)
        for i in range(half):
            f = inv[i]
            wl = F(two_pi / f)
            if wl > low_w:
                inv[i] = F(f / factor)
            elif wl >= high_w:
                smooth = F(F(F(o / wl) - low) / F(high - low))
                inv[i] = F(F(F(F(1.0) - smooth) * f) / factor + F(smooth * f))
    elif rtype == "linear":
        inv = (inv / F(scaling.factor)).astype(F)
    elif rtype == "yarn":
        o = orig()
        factor = factor_or_ratio()

        def mscale(scale, m):
            return F(1.0) if scale <= 1.0 else F(F(F(0.1) * F(m)) * F(np.log(F(scale))) + F(1.0))

        if scaling.attention_factor is not None:
            af = F(scaling.attention_factor)
        elif scaling.mscale and scaling.mscale_all_dim:
            af = F(mscale(factor, scaling.mscale) / mscale(factor, scaling.mscale_all_dim))
        else:
            af = mscale(factor, 1.0)
        bf = F(scaling.beta_fast) if scaling.beta_fast else F(32.0)
        bs = F(scaling.beta_slow) if scaling.beta_slow else F(1.0)
        dim = F(rotary_dim)

        def corr(rot):
            return F(F(dim * F(np.log(F(o / F(F(rot * F(2.0)) * F(math.pi)))))) /
                     F(F(2.0) * F(np.log(theta))))

        lo, hi = corr(bf), corr(bs)
        if scaling.truncate is None or scaling.truncate:
            lo, hi = F(math.floor(lo)), F(math.ceil(hi))
        lo = F(max(lo, F(0.0)))
        hi = F(min(hi, F(dim - F(1.0))))
        if lo == hi:
            hi = F(hi + F(0.001))
        for i in range(half):
            ramp = F(min(max(F(F(F(i) - lo) / F(hi - lo)), F(0.0)), F(1.0)))
            f = inv[i]
            inv[i] = F(F(F(f / factor) * ramp) + F(f * F(F(1.0) - ramp)))
    elif rtype == "longrope":
        if scaling.original_max_position_embeddings is None:
            raise ValueError("this rope scaling needs original_max_position_embeddings in rope_scaling")
        olen = int(scaling.original_max_position_embeddings)
        factor = factor_or_ratio()
        if scaling.attention_factor is not None:
            af = F(scaling.attention_factor)
        elif factor <= 1.0:
            af = F(1.0)
        else:
            af = F(np.sqrt(F(F(1.0) + F(F(np.log(factor)) / F(np.log(F(olen)))))))
        ext = scaling.long_factor if seq_len > olen else scaling.short_factor
        if ext is None or len(ext) != half:
            raise ValueError("longrope: the factor list has %s values but the head rotates %d pairs"
                             % (None if ext is None else len(ext), half))
        inv = np.array([F(inv[i] / F(ext[i])) for i in range(half)], F)
    return inv, float(af)


def rope_caches_partial(tokens, head_dim, rotary_dim, theta, scaling=None, seq_len=None):
    """(sin, cos) f32 [tokens, head_dim]: sin(p * inv_freq[d % half]) * af, the
    identity (cos 1, sin 0) on pass-through pairs of a partial rotation."""
    if rotary_dim > head_dim or rotary_dim % 2:
        raise ValueError("rotary width %d of %d" % (rotary_dim, head_dim))
    if seq_len is None:
        seq_len = tokens
    half, rot_half = head_dim // 2, rotary_dim // 2
    inv, af = rope_spec(rotary_dim, theta, scaling, seq_len)
    af = F(af)
    sin = np.zeros((tokens, head_dim), F)
    cos = np.ones((tokens, head_dim), F)
    p = np.arange(tokens, dtype=F)[:, None]
    j = np.arange(head_dim) % half
    rot = j < rot_half
    ang = (p * inv[np.minimum(j, rot_half - 1)][None, :]).astype(F)
    sin[:, rot] = (np.sin(ang[:, rot]) * af).astype(F)
    cos[:, rot] = (np.cos(ang[:, rot]) * af).astype(F)
    return sin, cos


def rope_head_perm(head_dim, rotary_dim):
    """Engine dim e of a head holds HF dim perm[e] (lib.rs:2231-2254)."""
    half, rot_half = head_dim // 2, rotary_dim // 2
    pas = half - rot_half
    out = []
    for e in range(head_dim):
        j, second = e % half, e >= half
        if j < rot_half:
            out.append(j + (rot_half if second else 0))
        else:
            out.append(rotary_dim + (j - rot_half) + (pas if second else 0))
    return out


def rope_caches_for(cfg, positions, seq_len=None):
    """The global table pair of a config for `positions` rows (lib.rs:394-420)."""
    return rope_caches_partial(positions, cfg.head_dim(), cfg.rotary_dim(), cfg.rope_theta,
                               cfg.rope_scaling, positions if seq_len is None else seq_len)


def rope_local_caches_for(cfg, positions):
    """The local table pair (Gemma-3 sliding layers): rope_local_base_freq,
    default 1e4, without rope_scaling (lib.rs:411-420); None when no layer
    reads it."""
    if not any(cfg.local_rope(li) for li in range(cfg.num_hidden_layers)):
        return None
    theta = cfg.rope_local_base_freq if cfg.rope_local_base_freq is not None else 1e4
    return rope_caches_partial(positions, cfg.head_dim(), cfg.rotary_dim(), theta, None, positions)
