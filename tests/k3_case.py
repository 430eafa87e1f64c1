"""Seeded K3 latent-MoE blocks for the tests: the oracle's description
(oracle/k3_oracle.Block) and, on a GPU, the same weights as minirun_moe.K3MoE."""
import numpy as np

from oracle import k3_oracle as K
from oracle import oracle as O


def _exp_for(inn):
    # e8m0 exponents putting |w| near 1 / sqrt(in) (e2m1 magnitudes average ~2.2)
    c = int(round(127 - np.log2(2.2 * np.sqrt(inn))))
    return c - 1, c + 1


def _dense(seed, out, inn):
    bits = O.gen_normal_bf16(seed, out * inn, 1.0 / np.sqrt(inn)).reshape(out, inn)
    return bits, O.bf16_to_f32(bits)


def make(seed=1, E=32, H=1024, Lt=512, I=512, S=512, k=4, mx_proj=False, norm=True,
         linear_beta=25.0, renormalize=True, scale=1.0):
    """Returns (oracle Block, dict of raw arrays for the GPU side)."""
    rng = np.random.default_rng(seed)
    raw = {}
    gb, gf = _dense(seed * 10 + 1, E, H)
    raw["gate"] = gb
    bias = (rng.standard_normal(E) * 0.05).astype(np.float32)
    raw["bias"] = bias

    def proj(tag, out, inn, s):
        if mx_proj:
            lo, hi = _exp_for(inn)
            m = O.gen_mxfp4(s, 0, out, inn, lo, hi)
            raw[tag] = m
            return K.Proj(mx=m)
        b, f = _dense(s, out, inn)
        raw[tag] = b
        return K.Proj(dense=f)

    down = proj("down", Lt, H, seed * 10 + 2)
    up = proj("up", H, Lt, seed * 10 + 3)
    nw = (1.0 + 0.1 * rng.standard_normal(Lt)).astype(np.float32) if norm else None
    raw["norm"] = nw
    lo, hi = _exp_for(Lt)
    w1 = O.gen_mxfp4(seed * 10 + 4, E, I, Lt, lo, hi)
    w3 = O.gen_mxfp4(seed * 10 + 5, E, I, Lt, lo, hi)
    lo2, hi2 = _exp_for(I)
    w2 = O.gen_mxfp4(seed * 10 + 6, E, Lt, I, lo2, hi2)
    raw.update(w1=w1, w3=w3, w2=w2)
    shared = None
    if S:
        shared = (proj("sg", S, H, seed * 10 + 7), proj("su", S, H, seed * 10 + 8),
                  proj("sd", H, S, seed * 10 + 9))
    B = K.Block(gf, bias, k, renormalize, scale, down, up, nw, 1e-5, w1, w3, w2, shared, 4.0,
                linear_beta)
    return B, raw


def x_for(seed, T, H):
    return np.random.default_rng(seed + 1000).standard_normal((T, H)).astype(np.float32)


def to_gpu(B, raw, dev):
    import torch

    import minirun_moe as M

    def t_bf16(bits):
        return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(
            torch.bfloat16).to(dev)

    def mx(m):
        return M.MXFP4Weights(torch.from_numpy(np.ascontiguousarray(m.packed).view(np.int32)).to(dev),
                              torch.from_numpy(np.ascontiguousarray(m.scales)).to(dev))

    def proj(tag):
        v = raw[tag]
        return M.K3Projection(mx(v) if isinstance(v, O.Mxfp4) else t_bf16(v))

    shared = (proj("sg"), proj("su"), proj("sd")) if B.shared is not None else None
    norm = None if raw["norm"] is None else torch.from_numpy(raw["norm"]).to(dev)
    return M.K3MoE(t_bf16(raw["gate"]), torch.from_numpy(raw["bias"]).to(dev), proj("down"),
                   proj("up"), norm, mx(raw["w1"]), mx(raw["w3"]), mx(raw["w2"]), shared,
                   B.top_k, B.renormalize, B.scale, B.eps, B.beta, B.linear_beta)
