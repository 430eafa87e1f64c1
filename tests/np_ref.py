"""Independent float64 numpy restatement of the MoE path (test infrastructure).

A second, from-scratch statement of the same semantics as oracle/moe_oracle.c,
used only to cross-check the C oracle on small cases. Citations are to the
reference tree (nanguoyu/minirun-app).
"""
from __future__ import annotations

import numpy as np


def bf16_to_f32(a):
    return (np.asarray(a, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16r(a):
    return bf16_to_f32(f32_to_bf16(np.asarray(a, np.float32)))


def unpack(packed, bits):
    """MLX affine: element j of a row at bit (j % (32/bits))*bits of word j // (32/bits)."""
    per = 32 // bits
    shifts = (np.arange(per, dtype=np.uint32) * bits)
    q = (packed[..., :, None] >> shifts) & np.uint32((1 << bits) - 1)
    return q.reshape(packed.shape[:-1] + (packed.shape[-1] * per,))


def dequant64(packed, scales, biases, bits, group):
    """w = scale*q + bias (AffineWeights.swift:44, :328-342), float64."""
    q = unpack(packed, bits).astype(np.float64)
    s = np.repeat(bf16_to_f32(scales).astype(np.float64), group, axis=-1)
    z = np.repeat(bf16_to_f32(biases).astype(np.float64), group, axis=-1)
    return s * q + z


def gather_mm(x_bf16, w, ids):
    """out[t,j] = W[ids[t,j]] . x[t] (AffineWeights.swift:283-318) -> bf16."""
    x = bf16_to_f32(x_bf16).astype(np.float64)
    Wd = dequant64(w.packed, w.scales, w.biases, w.bits, w.group)
    T, k = ids.shape
    out = np.empty((T, k, Wd.shape[-2]), np.float32)
    for t in range(T):
        for j in range(k):
            out[t, j] = (Wd[ids[t, j]] @ x[t]).astype(np.float32)
    return f32_to_bf16(out), out


def router(logits, k, scoring="sigmoid", bias=None, renorm="eps", eps=1e-20, scale=1.0):
    """Selection of MoE.swift:98-150 / DeepSeekV4Routing.swift:124-280 /
    QwenMoEModel.swift:82-131."""
    l = logits.astype(np.float64)
    if scoring == "sigmoid":
        s = 1.0 / (1.0 + np.exp(-l))
    elif scoring == "softmax":
        e = np.exp(l - l.max(axis=1, keepdims=True))
        s = e / e.sum(axis=1, keepdims=True)
    else:
        s = np.sqrt(np.maximum(l, 0) + np.log1p(np.exp(-np.abs(l))))
    s = s.astype(np.float32)
    ch = s if bias is None else (s + bias.astype(np.float32)).astype(np.float32)
    T, E = s.shape
    ids = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    margins = np.empty(T)
    for t in range(T):
        order = sorted(range(E), key=lambda e: (-float(ch[t, e]), e))
        ids[t] = order[:k]
        w[t] = s[t, order[:k]]
        kth, rej = float(ch[t, order[k - 1]]), float(ch[t, order[k]])
        sc = max(abs(kth), abs(rej))
        margins[t] = (kth - rej) / sc if sc > 0 else 0.0
    den = np.zeros(T, np.float32)
    for j in range(k):
        den = (den + w[:, j]).astype(np.float32)
    if renorm == "plain":
        w = (w / den[:, None]).astype(np.float32)
    elif renorm == "eps" and k > 1:
        w = (w / (den + np.float32(eps))[:, None]).astype(np.float32)
    return ids, (w * np.float32(scale)).astype(np.float32), margins


def sigmoid32(g):
    return (1.0 / (1.0 + np.exp(-g.astype(np.float64)))).astype(np.float32)


def router_hashed(logits, table, token_ids, scoring="sqrt_softplus", renorm="plain", eps=1e-20,
                  scale=1.0):
    """The .tokenHash choice (DeepSeekV4Routing.swift:231-256): experts from
    the table row of each token id, weights = the scores at those experts."""
    l = logits.astype(np.float64)
    if scoring == "sigmoid":
        s = 1.0 / (1.0 + np.exp(-l))
    elif scoring == "softmax":
        e = np.exp(l - l.max(axis=1, keepdims=True))
        s = e / e.sum(axis=1, keepdims=True)
    else:
        s = np.sqrt(np.maximum(l, 0) + np.log1p(np.exp(-np.abs(l))))
    s = s.astype(np.float32)
    ids = table[token_ids].astype(np.int32)
    w = np.take_along_axis(s, ids, axis=1).astype(np.float32)
    T, k = ids.shape
    den = np.zeros(T, np.float32)
    for j in range(k):
        den = (den + w[:, j]).astype(np.float32)
    if renorm == "plain":
        w = (w / den[:, None]).astype(np.float32)
    elif renorm == "eps" and k > 1:
        w = (w / (den + np.float32(eps))[:, None]).astype(np.float32)
    return ids, (w * np.float32(scale)).astype(np.float32)


def layer(Lw, x_bf16, hashed=None):
    """Router -> routed (weight before w2, DeepSeekV4ExpertBackend.swift:311-342)
    -> shared (DeepSeekV4HashFFN.swift:223-255) -> sum. hashed = (table,
    token_ids) routes by token id instead."""
    c = Lw.cfg
    x64 = bf16_to_f32(x_bf16).astype(np.float64)
    r64 = bf16_to_f32(Lw.router_w).astype(np.float64)
    logits = (x64 @ r64.T).astype(np.float32)
    if hashed is None:
        ids, w, m = router(logits, c.top_k, c.scoring, Lw.correction_bias, c.renorm,
                           c.renorm_eps, c.routed_scale)
    else:
        ids, w = router_hashed(logits, hashed[0], hashed[1], c.scoring, c.renorm, c.renorm_eps,
                               c.routed_scale)
        m = None
    gb, _ = gather_mm(x_bf16, Lw.gate, ids)
    ub, _ = gather_mm(x_bf16, Lw.up, ids)
    g = bf16_to_f32(gb)
    u = bf16_to_f32(ub)
    if c.swiglu_limit > 0:
        g = np.minimum(g, np.float32(c.swiglu_limit))
        u = np.clip(u, -np.float32(c.swiglu_limit), np.float32(c.swiglu_limit))
    T, k = ids.shape
    if not c.weight_after_down:
        a = (g * sigmoid32(g)).astype(np.float32)
        a = (a * u).astype(np.float32)
        a = (a * w[:, :, None]).astype(np.float32)
        h = f32_to_bf16(a)
    else:
        sg = bf16r(sigmoid32(g))
        a = bf16r(g * sg)
        h = f32_to_bf16(a * u)
    db, _ = gather_mm(h.reshape(T * k, -1), Lw.down, ids.reshape(T * k, 1))
    d = bf16_to_f32(db).reshape(T, k, -1)
    acc = np.zeros((T, d.shape[-1]), np.float32)
    for j in range(k):
        acc = (acc + (d[:, j] * w[:, j:j + 1] if c.weight_after_down else d[:, j])).astype(
            np.float32)
    if not c.weight_after_down:
        acc = bf16r(acc)
    if Lw.sgate is not None:
        sg_w = dequant64(Lw.sgate.packed, Lw.sgate.scales, Lw.sgate.biases, Lw.sgate.bits,
                         Lw.sgate.group)
        su_w = dequant64(Lw.sup.packed, Lw.sup.scales, Lw.sup.biases, Lw.sup.bits, Lw.sup.group)
        sd_w = dequant64(Lw.sdown.packed, Lw.sdown.scales, Lw.sdown.biases, Lw.sdown.bits,
                         Lw.sdown.group)
        sgv = bf16r((x64 @ sg_w.T).astype(np.float32))
        suv = bf16r((x64 @ su_w.T).astype(np.float32))
        if c.swiglu_limit > 0:
            sgv = np.minimum(sgv, np.float32(c.swiglu_limit))
            suv = np.clip(suv, -np.float32(c.swiglu_limit), np.float32(c.swiglu_limit))
        sa = ((sgv * sigmoid32(sgv)).astype(np.float32) * suv).astype(np.float32)
        sd = (sa.astype(np.float64) @ sd_w.T).astype(np.float32)
        acc = (acc + sd).astype(np.float32)
    return f32_to_bf16(acc), acc, ids, w, m
