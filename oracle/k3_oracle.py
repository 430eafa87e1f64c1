"""CPU restatement of K3's latent MoE block, composed from the C oracle's
MXFP4 products and router.

TEST INFRASTRUCTURE ONLY: the checker for ``mr_k3_moe_forward``; imported by
tests/ only, never by the product package.

Follows K3MoE.forward (Sources/ModelAdapters/Operators/MoE.swift:219-272):
fp32 router logits of the full hidden state (:80-83), K3Router.select
(:98-150), the latent down projection, the gate (w1) and up (w3) gathers,
K3Activation.situ (Operators/Activations.swift:31-47), the down gather (w2)
per (token, slot), the fp32 weighted slot sum (:250-253), K3Norm.rms
(Operators/Normalization.swift:15-19), the up projection and the shared
expert K3MLP on the original hidden state. Dot products are exact in
float64 and rounded to fp32 (the reference's fp32 matmuls round each sum);
the elementwise steps run in fp32 in the reference's evaluation order.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import oracle as O


@dataclass
class Proj:
    dense: np.ndarray | None = None   # fp32 values [out, in]
    mx: O.Mxfp4 | None = None         # single MXFP4 matrix

    def __call__(self, x: np.ndarray) -> np.ndarray:
        if self.mx is not None:
            return O.mxfp4_mm_f32(x, self.mx)
        return (x.astype(np.float64) @ self.dense.astype(np.float64).T).astype(np.float32)


@dataclass
class Block:
    gate_w: np.ndarray        # [E, H] fp32 values
    bias: np.ndarray          # [E] fp32
    top_k: int
    renormalize: bool
    scale: float
    down: Proj                # [latent, H]
    up: Proj                  # [H, latent]
    norm: np.ndarray | None   # [latent] fp32 values
    eps: float
    w1: O.Mxfp4
    w3: O.Mxfp4
    w2: O.Mxfp4
    shared: tuple[Proj, Proj, Proj] | None
    beta: float
    linear_beta: float | None


def situ(g: np.ndarray, u: np.ndarray, beta: float, linear_beta: float | None) -> np.ndarray:
    """(tanh(g / beta) * beta) * sigmoid(g) * (tanh(u / lb) * lb), fp32."""
    g = g.astype(np.float32)
    u = u.astype(np.float32)
    b = np.float32(beta)
    sig = (np.float32(1) / (np.float32(1) + np.exp(-g))).astype(np.float32)
    a = (np.tanh(g / b) * b * sig).astype(np.float32)
    if linear_beta:
        lb = np.float32(linear_beta)
        u = (np.tanh(u / lb) * lb).astype(np.float32)
    return (a * u).astype(np.float32)


def rms(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = x.astype(np.float32)
    ms = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    return (w.astype(np.float32) * (x * (1.0 / np.sqrt(ms + eps)).astype(np.float32))).astype(
        np.float32)


def forward(B: Block, x: np.ndarray):
    """Returns (out fp32 [T, H], ids [T, k], weights [T, k], margins [T])."""
    x = np.ascontiguousarray(x, np.float32)
    T = x.shape[0]
    k = B.top_k
    logits = (x.astype(np.float64) @ B.gate_w.astype(np.float64).T).astype(np.float32)
    ids, w, margins, _ = O.router_select(logits, k, "sigmoid", B.bias,
                                         "eps" if B.renormalize else "none", 1e-20, B.scale)
    latent = B.down(x)
    g = O.mxfp4_gather_mm_f32(latent, B.w1, ids)
    u = O.mxfp4_gather_mm_f32(latent, B.w3, ids)
    act = situ(g, u, B.beta, B.linear_beta)
    I = act.shape[-1]
    eo = O.mxfp4_gather_mm_f32(act.reshape(T * k, I), B.w2,
                               ids.reshape(T * k, 1)).reshape(T, k, -1)
    rs = np.zeros((T, eo.shape[-1]), np.float32)
    for j in range(k):  # slot order, fp32
        rs = (rs + (eo[:, j] * w[:, j:j + 1]).astype(np.float32)).astype(np.float32)
    normed = rms(rs, B.norm, B.eps) if B.norm is not None else rs
    out = B.up(normed)
    if B.shared is not None:
        sg, su, sd = B.shared
        out = (out + sd(situ(sg(x), su(x), B.beta, B.linear_beta))).astype(np.float32)
    return out, ids, w, margins
