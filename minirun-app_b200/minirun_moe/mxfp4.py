"""MXFP4 weights and matmuls — the host mirror of Sources/MLXBridge/
MXFP4Weights.swift and MXFP4Matmul.swift over libminirun_moe's C ABI.

OCP MX FP4: e2m1 codes, eight per uint32 word with element 0 in the low
nibble (the byte image of a compressed-tensors checkpoint's uint8 stream),
one e8m0 exponent per 32 input elements, ``w = e2m1 * 2**(e - 127)``, no
bias. The arithmetic runs in the CUDA library; there is no CPU path.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from .bridge import Context, _check_x, _from_ptr, _ptr, _stream

_PACKED_DTYPES = (torch.int32, torch.uint32)


class MXFP4BridgeError(ValueError):
    """Packed MXFP4 operands do not describe a usable tensor
    (MXFP4Weights.swift:8-32): reported with the shapes involved."""


class MXFP4Weights:
    """Packed MXFP4 weights in checkpoint byte layout (MXFP4Weights.swift:65-140).

    ``packed``: uint32 (or int32 bit pattern) ``[experts?, out, in/8]``;
    ``scales``: uint8 e8m0 ``[experts?, out, in/32]``.
    """

    group_size = 32
    bits = 4

    def __init__(self, packed: torch.Tensor, scales: torch.Tensor):
        # The checks and messages of MXFP4Weights.init (:86-140), in its order.
        if packed.dtype not in _PACKED_DTYPES:
            raise MXFP4BridgeError(
                "packed MXFP4 weights must be .uint32 (the little-endian reinterpretation of "
                f"the checkpoint's uint8 stream), got {packed.dtype}")
        if scales.dtype != torch.uint8:
            raise MXFP4BridgeError(f"MXFP4 e8m0 scales must be .uint8, got {scales.dtype}")
        ps, ss = list(packed.shape), list(scales.shape)
        if not (len(ps) == len(ss) and len(ps) in (2, 3)):
            raise MXFP4BridgeError(
                f"packed {ps} and scales {ss} must both be rank 2 (one matrix) or rank 3 (an "
                "expert stack), and must agree")
        experts = ps[0] if len(ps) == 3 else None
        if experts is not None and ss[0] != experts:
            raise MXFP4BridgeError(
                f"expert count differs: packed has {experts}, scales has {ss[0]}")
        out_features = ps[-2]
        if ss[-2] != out_features:
            raise MXFP4BridgeError(
                f"row count differs: packed has {out_features}, scales has {ss[-2]}")
        in_features = ps[-1] * 8
        if in_features % self.group_size != 0:
            raise MXFP4BridgeError(
                f"inFeatures {in_features} is not a multiple of groupSize {self.group_size}; "
                "partial final groups are not supported")
        groups = in_features // self.group_size
        if ss[-1] != groups:
            raise MXFP4BridgeError(
                f"group count differs: {in_features} input features need {groups} scales per "
                f"row, got {ss[-1]}")
        for t in (packed, scales):
            if not t.is_contiguous():
                raise MXFP4BridgeError("MXFP4 tensors must be contiguous")
        self.packed, self.scales = packed, scales
        self.experts = experts
        self.out_features, self.in_features = out_features, in_features
        self._keepalive = None

    @staticmethod
    def adopting(packed_ptr: int, scales_ptr: int, out_features: int, in_features: int,
                 experts: int | None = None, device: int | None = None,
                 keepalive=None) -> "MXFP4Weights":
        """Wrap two device buffers without copying (MXFP4Weights.swift:207-237).
        The caller keeps the memory alive (``keepalive`` is held for it)."""
        pshape = [out_features, in_features // 8]
        sshape = [out_features, in_features // 32]
        if experts:
            pshape, sshape = [experts] + pshape, [experts] + sshape
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        w = MXFP4Weights(_from_ptr(packed_ptr, pshape, torch.int32, dev),
                         _from_ptr(scales_ptr, sshape, torch.uint8, dev))
        w._keepalive = keepalive
        return w

    def desc(self) -> L.mr_mxfp4_desc:
        return L.mr_mxfp4_desc(self.packed.data_ptr(), self.scales.data_ptr(),
                               self.experts or 0, self.out_features, self.in_features)

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.packed, self.scales))


def mxfp4_validate(weights: MXFP4Weights) -> tuple[int, str]:
    """Host-only validation through the C ABI (no GPU needed)."""
    buf = C.create_string_buffer(256)
    d = weights.desc()
    st = L.load().mr_mxfp4_validate(C.byref(d), buf, 256)
    return st, buf.value.decode()


def mxfp4_mm(x: torch.Tensor, weights: MXFP4Weights) -> torch.Tensor:
    """``y = x . W^T`` with W in checkpoint layout (MXFP4Matmul.swift:17-34)."""
    if weights.experts is not None:
        raise MXFP4BridgeError("mxfp4MM needs a single matrix; use mxfp4GatherMM for a stack")
    _check_x(x, weights.in_features)
    x = x.contiguous()
    out = torch.empty((x.shape[0], weights.out_features), dtype=torch.bfloat16, device=x.device)
    ctx = Context.get(x.device.index)
    d = weights.desc()
    ctx.check("mr_mxfp4_mm", L.load().mr_mxfp4_mm(
        ctx.handle, _ptr(x), x.shape[0], C.byref(d), _ptr(out), C.c_void_p(_stream())))
    return out


def mxfp4_gather_mm(x: torch.Tensor, weights: MXFP4Weights, rhs_indices: torch.Tensor,
                    sorted_indices: bool = False) -> torch.Tensor:
    """``out[t, j, :] = W[rhs_indices[t, j]] . x[t, :]`` (MXFP4Matmul.swift:74-112).

    Takes plain ``[tokens, inFeatures]`` x, as the reference does, so the
    slot-as-token broadcast mistake cannot be expressed. ``sorted_indices``
    is accepted for API parity and changes nothing: the device plan groups
    columns by expert whatever the order."""
    if weights.experts is None:
        raise MXFP4BridgeError(
            "mxfp4GatherMM needs a stacked MXFP4Weights; use mxfp4MM for a single matrix")
    _check_x(x, weights.in_features)
    if rhs_indices.dim() != 2 or rhs_indices.shape[0] != x.shape[0]:
        raise MXFP4BridgeError(
            "rhsIndices must be [tokens, expertsPerToken] matching x's token count")
    x = x.contiguous()
    ids = rhs_indices.to(device=x.device, dtype=torch.int32).contiguous()
    T, k = ids.shape
    out = torch.empty((T, k, weights.out_features), dtype=torch.bfloat16, device=x.device)
    ctx = Context.get(x.device.index)
    d = weights.desc()
    ctx.check("mr_mxfp4_gather_mm", L.load().mr_mxfp4_gather_mm(
        ctx.handle, _ptr(x), T, _ptr(ids), k, C.byref(d), _ptr(out), C.c_void_p(_stream())))
    return out


def _check_xf(x: torch.Tensor, in_features: int) -> None:
    if x.dim() != 2 or x.dtype != torch.float32 or x.shape[1] != in_features or not x.is_cuda:
        raise MXFP4BridgeError(f"x must be a CUDA fp32 [tokens, {in_features}] tensor")


def mxfp4_mm_f32(x: torch.Tensor, weights: MXFP4Weights) -> torch.Tensor:
    """``mxfp4MM`` with fp32 x: fp32 out (MXFP4Matmul.swift:7-8)."""
    if weights.experts is not None:
        raise MXFP4BridgeError("mxfp4MM needs a single matrix; use mxfp4GatherMM for a stack")
    _check_xf(x, weights.in_features)
    x = x.contiguous()
    out = torch.empty((x.shape[0], weights.out_features), dtype=torch.float32, device=x.device)
    ctx = Context.get(x.device.index)
    d = weights.desc()
    ctx.check("mr_mxfp4_mm_f32", L.load().mr_mxfp4_mm_f32(
        ctx.handle, _ptr(x), x.shape[0], C.byref(d), _ptr(out), C.c_void_p(_stream())))
    return out


def mxfp4_gather_mm_f32(x: torch.Tensor, weights: MXFP4Weights,
                        rhs_indices: torch.Tensor) -> torch.Tensor:
    """``mxfp4GatherMM`` with fp32 x: fp32 ``[tokens, k, out]``."""
    if weights.experts is None:
        raise MXFP4BridgeError(
            "mxfp4GatherMM needs a stacked MXFP4Weights; use mxfp4MM for a single matrix")
    _check_xf(x, weights.in_features)
    if rhs_indices.dim() != 2 or rhs_indices.shape[0] != x.shape[0]:
        raise MXFP4BridgeError(
            "rhsIndices must be [tokens, expertsPerToken] matching x's token count")
    x = x.contiguous()
    ids = rhs_indices.to(device=x.device, dtype=torch.int32).contiguous()
    T, k = ids.shape
    out = torch.empty((T, k, weights.out_features), dtype=torch.float32, device=x.device)
    ctx = Context.get(x.device.index)
    d = weights.desc()
    ctx.check("mr_mxfp4_gather_mm_f32", L.load().mr_mxfp4_gather_mm_f32(
        ctx.handle, _ptr(x), T, _ptr(ids), k, C.byref(d), _ptr(out), C.c_void_p(_stream())))
    return out


def mxfp4_dequantize(weights: MXFP4Weights) -> torch.Tensor:
    """Dense fp32 ``e2m1 * 2**(e-127)`` (MXFP4Matmul.swift:114-136), exact.
    Validation only."""
    shape = ([weights.experts] if weights.experts else []) + [weights.out_features,
                                                             weights.in_features]
    out = torch.empty(shape, dtype=torch.float32, device=weights.packed.device)
    ctx = Context.get(weights.packed.device.index)
    d = weights.desc()
    ctx.check("mr_mxfp4_dequantize", L.load().mr_mxfp4_dequantize(
        ctx.handle, C.byref(d), _ptr(out), C.c_void_p(_stream())))
    return out
