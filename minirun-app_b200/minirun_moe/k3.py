"""K3's latent MoE block — the host mirror of K3MoE / K3Projection / K3MLP
(Sources/ModelAdapters/Operators/MoE.swift:152-272, Linear.swift:19-57,
Activations.swift:15-47) over libminirun_moe's C ABI.

``K3MoE.forward`` runs the whole block in one call (``mr_k3_moe_forward``):
router on the full hidden state (fp32 logits, sigmoid, correction bias for
the choice only), latent down projection, MXFP4 gate/up gathers in the
latent, situ, the down gather per (token, slot), the fp32 weighted slot sum,
RMSNorm in the latent, the up projection, plus the shared expert on the
original hidden state. Everything is fp32, as the reference pins it.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib as L
from .bridge import AffineBridgeError, Context, Selection, _ptr, _stream
from .moe import RouterConfig
from .mxfp4 import MXFP4Weights, mxfp4_mm_f32

_DENSE_DTYPES = {torch.bfloat16: L.MR_DTYPE_BF16, torch.float32: L.MR_DTYPE_F32}


class K3Projection:
    """``K3Projection`` (Linear.swift:19-45): a dense bf16/fp32 ``[out, in]``
    weight or a single MXFP4 matrix."""

    def __init__(self, weight: torch.Tensor | MXFP4Weights):
        if isinstance(weight, MXFP4Weights):
            if weight.experts is not None:
                raise AffineBridgeError("a K3 projection is a single matrix, not a stack")
            self.out_features, self.in_features = weight.out_features, weight.in_features
        else:
            if weight.dim() != 2 or weight.dtype not in _DENSE_DTYPES:
                raise AffineBridgeError("a dense K3 projection is a bf16 or fp32 [out, in] matrix")
            weight = weight.contiguous()
            self.out_features, self.in_features = weight.shape
        self.weight = weight

    @property
    def is_quantized(self) -> bool:
        return isinstance(self.weight, MXFP4Weights)

    def c(self) -> L.mr_k3_projection:
        if self.is_quantized:
            return L.mr_k3_projection(L.MR_K3_PROJ_MXFP4, None, 0, 0, 0, self.weight.desc())
        return L.mr_k3_projection(L.MR_K3_PROJ_DENSE, self.weight.data_ptr(),
                                  _DENSE_DTYPES[self.weight.dtype], self.out_features,
                                  self.in_features, L.mr_mxfp4_desc())

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """``callAsFunction`` (Linear.swift:24-29): fp32 in, fp32 out."""
        if self.is_quantized:
            return mxfp4_mm_f32(x, self.weight)
        return dense_mm_f32(x, self.weight)


def dense_mm_f32(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """``k3Linear(x, W)`` (Linear.swift:47-57): fp32 x, bf16/fp32 W [out, in]."""
    if x.dim() != 2 or x.dtype != torch.float32 or x.shape[1] != weight.shape[1]:
        raise AffineBridgeError("x must be fp32 [tokens, inFeatures]")
    x = x.contiguous()
    weight = weight.contiguous()
    out = torch.empty((x.shape[0], weight.shape[0]), dtype=torch.float32, device=x.device)
    ctx = Context.get(x.device.index)
    ctx.check("mr_dense_mm_f32", L.load().mr_dense_mm_f32(
        ctx.handle, _ptr(x), x.shape[0], _ptr(weight), _DENSE_DTYPES[weight.dtype],
        weight.shape[0], weight.shape[1], _ptr(out), C.c_void_p(_stream())))
    return out


def situ(x: torch.Tensor, beta: float, linear_beta: float | None) -> torch.Tensor:
    """``K3Activation.situ`` (Activations.swift:15-47) on ``[..., 2d]`` =
    concat(gate, up)."""
    if x.dtype != torch.float32 or x.shape[-1] % 2:
        raise AffineBridgeError("situ takes fp32 [..., 2d]")
    d = x.shape[-1] // 2
    xf = x.contiguous().reshape(-1, 2 * d)
    out = torch.empty((xf.shape[0], d), dtype=torch.float32, device=x.device)
    ctx = Context.get(x.device.index)
    ctx.check("mr_k3_situ", L.load().mr_k3_situ(
        ctx.handle, _ptr(xf), xf.shape[0], d, beta, linear_beta or 0.0, _ptr(out),
        C.c_void_p(_stream())))
    return out.reshape(*x.shape[:-1], d)


@dataclass
class K3MoE:
    """``K3MoE.Weights`` (MoE.swift:168-201) plus the block's config values.

    ``w1``/``w3``: MXFP4 stacks ``[E, inter, latent]``; ``w2``: ``[E, latent,
    inter]``; ``shared``: (gate, up, down) projections or None."""
    gate_weight: torch.Tensor          # [E, hidden] bf16 / fp32
    correction_bias: torch.Tensor      # [E] fp32
    routed_down: K3Projection          # [latent, hidden]
    routed_up: K3Projection            # [hidden, latent]
    routed_norm: torch.Tensor | None   # [latent] bf16 / fp32, None: latent_moe_use_norm false
    w1: MXFP4Weights
    w3: MXFP4Weights
    w2: MXFP4Weights
    shared: tuple[K3Projection, K3Projection, K3Projection] | None
    top_k: int
    renormalize: bool = True
    routed_scaling_factor: float = 1.0
    rms_norm_eps: float = 1e-5
    situ_beta: float = 4.0
    situ_linear_beta: float | None = 25.0

    def c(self) -> L.mr_k3_moe:
        E = self.gate_weight.shape[0]
        self._router = RouterConfig.k3(E, self.top_k, self.renormalize,
                                       self.routed_scaling_factor,
                                       self.correction_bias.float().contiguous())
        hidden, latent = self.routed_down.in_features, self.routed_down.out_features
        inter = self.w1.out_features
        S = self.shared[0].out_features if self.shared else 0
        none = L.mr_k3_projection()
        sh = [p.c() for p in self.shared] if self.shared else [none, none, none]
        norm = self.routed_norm
        return L.mr_k3_moe(
            self._router.c(), self.gate_weight.data_ptr(), _DENSE_DTYPES[self.gate_weight.dtype],
            self.routed_down.c(), self.routed_up.c(), 0 if norm is None else norm.data_ptr(),
            _DENSE_DTYPES[norm.dtype] if norm is not None else 0, self.rms_norm_eps,
            self.w1.desc(), self.w3.desc(), self.w2.desc(), sh[0], sh[1], sh[2], hidden,
            latent, inter, S, self.situ_beta, self.situ_linear_beta or 0.0)

    def validate(self) -> tuple[int, str]:
        buf = C.create_string_buffer(256)
        c = self.c()
        return L.load().mr_k3_moe_validate(C.byref(c), buf, 256), buf.value.decode()

    def forward(self, x: torch.Tensor) -> tuple[torch.Tensor, Selection]:
        """``K3MoE.forward`` (MoE.swift:219-272): fp32 [T, hidden] -> fp32
        [T, hidden] and the router's selection (ids, weights)."""
        if x.dim() != 2 or x.dtype != torch.float32:
            raise AffineBridgeError("x must be fp32 [tokens, hidden]")
        x = x.contiguous()
        T = x.shape[0]
        hidden = self.routed_down.in_features
        out = torch.empty((T, hidden), dtype=torch.float32, device=x.device)
        ids = torch.empty((T, self.top_k), dtype=torch.int32, device=x.device)
        w = torch.empty((T, self.top_k), dtype=torch.float32, device=x.device)
        c = self.c()
        ctx = Context.get(x.device.index)
        ctx.check("mr_k3_moe_forward", L.load().mr_k3_moe_forward(
            ctx.handle, C.byref(c), _ptr(x), T, _ptr(out), _ptr(ids), _ptr(w),
            C.c_void_p(_stream())))
        return out, Selection(ids, w, None, None)
