"""CUDA bridge: the reference's MLXBridge affine op API over the C ABI.

Python mirror of `Sources/MLXBridge/AffineWeights.swift` (nanguoyu/minirun-app):
``AffineWeights`` (:65-157) with ``adopting`` (:171-198), ``expert_stack`` /
``expert`` (:207-229), ``affine_mm`` (:239-254), ``affine_gather_mm``
(:283-318) and ``affine_dequantize`` (:328-342). Device memory is held in
torch tensors (plumbing only); every computation is a call into
libminirun_moe.so on torch's current CUDA stream.
"""
from __future__ import annotations

import ctypes as C
import threading
from dataclasses import dataclass

import torch

from . import _lib as L


class AffineBridgeError(ValueError):
    """Packed affine operands do not describe a usable tensor
    (AffineWeights.swift:8-38): reported with the shapes involved, never
    padded, reshaped or truncated."""


class MoeError(RuntimeError):
    """A C-ABI call returned a non-OK mr_status."""

    def __init__(self, fn: str, status: int, message: str):
        self.status = status
        self.message = message
        text = L.load().mr_status_string(status).decode()
        super().__init__(f"{fn}: {text} ({status}): {message}")


_SCALE_DTYPES = {torch.bfloat16: L.MR_DTYPE_BF16, torch.float16: L.MR_DTYPE_F16,
                 torch.float32: L.MR_DTYPE_F32}
_PACKED_DTYPES = (torch.int32, torch.uint32)


class Context:
    """One mr_ctx per (host thread, device), as the C ABI requires."""

    _local = threading.local()

    def __init__(self, device: int):
        lib = L.load()
        h = C.c_void_p()
        st = lib.mr_ctx_create(device, C.byref(h))
        if st != L.MR_OK:
            raise MoeError("mr_ctx_create", st, "cannot create a context on device %d" % device)
        self.handle = h
        self.device = device

    def __del__(self):
        try:
            if getattr(self, "handle", None):
                L.load().mr_ctx_destroy(self.handle)
                self.handle = None
        except Exception:
            pass

    @classmethod
    def get(cls, device: int | None = None) -> "Context":
        if device is None:
            device = torch.cuda.current_device()
        cache = getattr(cls._local, "ctx", None)
        if cache is None:
            cache = cls._local.ctx = {}
        if device not in cache:
            cache[device] = Context(device)
        return cache[device]

    def check(self, fn: str, status: int) -> None:
        if status != L.MR_OK:
            raise MoeError(fn, status, L.load().mr_last_error(self.handle).decode())

    def sync_check(self, stream: int | None = None) -> int:
        """Synchronise the stream and raise on a set device error word."""
        bits = C.c_uint32(0)
        st = L.load().mr_ctx_check(self.handle, C.c_void_p(stream or _stream()), C.byref(bits))
        self.check("mr_ctx_check", st)
        return bits.value

    def reserve(self, max_tokens, top_k, experts, hidden, inter) -> None:
        self.check("mr_ctx_reserve", L.load().mr_ctx_reserve(
            self.handle, max_tokens, top_k, experts, hidden, inter))

    KERNEL_PATHS = {"auto": 0, "register": 1, "tma": 2, "umma": 3, "v2": 4}

    def set_kernel_path(self, path: str) -> None:
        self.check("mr_ctx_set_kernel_path", L.load().mr_ctx_set_kernel_path(
            self.handle, self.KERNEL_PATHS[path]))

    KERNEL_CLASSES = ("router_logits", "topk_plan", "gate_up", "down_combine", "exchange",
                      "combine")

    def profile(self, enable: bool) -> None:
        self.check("mr_ctx_profile", L.load().mr_ctx_profile(self.handle, int(enable)))

    def profile_read(self) -> dict[str, tuple[float, int]]:
        """{kernel class: (total ms, launches)} since the last read."""
        n = len(self.KERNEL_CLASSES)
        ms = (C.c_double * n)()
        cnt = (C.c_int64 * n)()
        self.check("mr_ctx_profile_read", L.load().mr_ctx_profile_read(self.handle, ms, cnt, n))
        return {k: (ms[i], cnt[i]) for i, k in enumerate(self.KERNEL_CLASSES)}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> C.c_void_p:
    return C.c_void_p(0 if t is None else t.data_ptr())


class AffineWeights:
    """Packed MLX affine weights (AffineWeights.swift:40-157).

    ``packed``: uint32 (or int32 bit pattern) ``[experts?, out, in*bits/32]``;
    ``scales``/``biases``: ``[experts?, out, in/group]`` in one floating dtype.
    ``w = scale*q + bias``; element j of a row sits at bit
    ``(j % (32/bits))*bits`` of word ``j // (32/bits)``.
    """

    def __init__(self, packed: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                 group_size: int, bits: int):
        # The checks and messages of AffineWeights.init (:84-157).
        if packed.dtype not in _PACKED_DTYPES:
            raise AffineBridgeError(
                "packed affine weights must be .uint32 (the little-endian reinterpretation "
                f"of the checkpoint's stream), got {packed.dtype}")
        if scales.dtype not in _SCALE_DTYPES:
            raise AffineBridgeError(
                "affine scales must be a floating-point type — .bfloat16 for this checkpoint, "
                f".float16 or .float32 for others — got {scales.dtype}")
        if scales.dtype != biases.dtype:
            raise AffineBridgeError(
                f"scales are {scales.dtype} but biases are {biases.dtype}; MLX emits both in "
                "one dtype")
        ps, ss = list(packed.shape), list(scales.shape)
        if ss != list(biases.shape):
            raise AffineBridgeError(
                f"scales {ss} and biases {list(biases.shape)} must have one shape")
        if not (len(ps) == len(ss) and len(ps) in (2, 3)):
            raise AffineBridgeError(
                f"packed {ps} and scales {ss} must both be rank 2 (one matrix) or rank 3 (an "
                "expert stack), and must agree")
        if not (bits > 0 and 32 % bits == 0):
            raise AffineBridgeError(f"bits {bits} must divide 32 for the uint32 packing")
        if group_size <= 0:
            raise AffineBridgeError("group size must be positive")
        experts = ps[0] if len(ps) == 3 else None
        if experts is not None and ss[0] != experts:
            raise AffineBridgeError(
                f"expert count differs: packed has {experts}, scales has {ss[0]}")
        out_features = ps[-2]
        if ss[-2] != out_features:
            raise AffineBridgeError(
                f"row count differs: packed has {out_features}, scales has {ss[-2]}")
        in_features = ps[-1] * (32 // bits)
        if in_features % group_size != 0:
            raise AffineBridgeError(
                f"inFeatures {in_features} is not a multiple of the group size {group_size}; "
                "partial final groups are not supported")
        groups = in_features // group_size
        if ss[-1] != groups:
            raise AffineBridgeError(
                f"group count differs: {in_features} input features at group size "
                f"{group_size} need {groups} scales per row, got {ss[-1]}")
        for t in (packed, scales, biases):
            if not t.is_contiguous():
                raise AffineBridgeError("affine tensors must be contiguous")
        self.packed, self.scales, self.biases = packed, scales, biases
        self.group_size, self.bits = group_size, bits
        self.experts = experts
        self.out_features, self.in_features = out_features, in_features
        self._keepalive = None

    @staticmethod
    def adopting(packed_ptr: int, scales_ptr: int, biases_ptr: int, scale_dtype: torch.dtype,
                 out_features: int, in_features: int, group_size: int, bits: int,
                 experts: int | None = None, device: int | None = None,
                 keepalive=None) -> "AffineWeights":
        """Wrap three device buffers without copying (AffineWeights.swift:171-198).
        The caller keeps the memory alive (``keepalive`` is held for it)."""
        words = in_features * bits // 32
        groups = in_features // group_size
        pshape = [experts, out_features, words] if experts else [out_features, words]
        sshape = [experts, out_features, groups] if experts else [out_features, groups]
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        packed = _from_ptr(packed_ptr, pshape, torch.int32, dev)
        scales = _from_ptr(scales_ptr, sshape, scale_dtype, dev)
        biases = _from_ptr(biases_ptr, sshape, scale_dtype, dev)
        w = AffineWeights(packed, scales, biases, group_size, bits)
        w._keepalive = keepalive
        return w

    def expert_stack(self, index: int) -> "AffineWeights":
        """Expert ``index`` as a stack of one (keeps the leading axis, :207-217)."""
        if self.experts is None or not (0 <= index < self.experts):
            raise AffineBridgeError(
                f"expert {index} requested from a stack of {self.experts or 'none'}")
        return AffineWeights(self.packed[index:index + 1], self.scales[index:index + 1],
                             self.biases[index:index + 1], self.group_size, self.bits)

    def expert(self, index: int) -> "AffineWeights":
        """Expert ``index`` as a standalone matrix, no copy (:220-229)."""
        if self.experts is None or not (0 <= index < self.experts):
            raise AffineBridgeError(
                f"expert {index} requested from a stack of {self.experts or 'none'}")
        return AffineWeights(self.packed[index], self.scales[index], self.biases[index],
                             self.group_size, self.bits)

    def desc(self) -> L.mr_affine_desc:
        return L.mr_affine_desc(self.packed.data_ptr(), self.scales.data_ptr(),
                                self.biases.data_ptr(), self.experts or 0, self.out_features,
                                self.in_features, self.group_size, self.bits,
                                _SCALE_DTYPES[self.scales.dtype])

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.packed, self.scales, self.biases))


def _from_ptr(ptr: int, shape, dtype, device) -> torch.Tensor:
    """A tensor view of caller-owned device memory (no copy)."""
    numel = 1
    for s in shape:
        numel *= s
    itemsize = torch.empty((), dtype=dtype).element_size()

    class _Holder:
        __cuda_array_interface__ = {
            "shape": (numel * itemsize,), "typestr": "|u1", "data": (ptr, False), "version": 3}

    raw = torch.as_tensor(_Holder(), device=device)
    return raw.view(dtype).view(shape)


def _check_x(x: torch.Tensor, in_features: int) -> None:
    if x.dim() != 2:
        raise AffineBridgeError(
            "x must be [tokens, inFeatures]; this function inserts the broadcast axes itself")
    if x.dtype != torch.bfloat16:
        raise AffineBridgeError(f"x must be bfloat16, got {x.dtype}")
    if x.shape[1] != in_features:
        raise AffineBridgeError(f"x has {x.shape[1]} features, weights expect {in_features}")
    if not x.is_cuda:
        raise AffineBridgeError("x must be a CUDA tensor")


def affine_mm(x: torch.Tensor, weights: AffineWeights) -> torch.Tensor:
    """``y = x . W^T`` with W in checkpoint layout (AffineWeights.swift:239-254)."""
    if weights.experts is not None:
        raise AffineBridgeError("affineMM needs a single matrix; use affineGatherMM for a stack")
    _check_x(x, weights.in_features)
    x = x.contiguous()
    out = torch.empty((x.shape[0], weights.out_features), dtype=torch.bfloat16, device=x.device)
    ctx = Context.get(x.device.index)
    d = weights.desc()
    ctx.check("mr_affine_mm", L.load().mr_affine_mm(
        ctx.handle, _ptr(x), x.shape[0], C.byref(d), _ptr(out), C.c_void_p(_stream())))
    return out


def affine_gather_mm(x: torch.Tensor, weights: AffineWeights, rhs_indices: torch.Tensor,
                     sorted_indices: bool = False) -> torch.Tensor:
    """``out[t, j, :] = W[rhs_indices[t, j]] . x[t, :]`` (AffineWeights.swift:283-318).

    ``sorted_indices`` is accepted for API parity; the device plan groups
    columns by expert whatever the order, so it changes nothing here."""
    if weights.experts is None:
        raise AffineBridgeError(
            "affineGatherMM needs a stacked AffineWeights; use affineMM for a single matrix")
    _check_x(x, weights.in_features)
    if rhs_indices.dim() != 2 or rhs_indices.shape[0] != x.shape[0]:
        raise AffineBridgeError(
            "rhsIndices must be [tokens, expertsPerToken] matching x's token count")
    x = x.contiguous()
    ids = rhs_indices.to(device=x.device, dtype=torch.int32).contiguous()
    T, k = ids.shape
    out = torch.empty((T, k, weights.out_features), dtype=torch.bfloat16, device=x.device)
    ctx = Context.get(x.device.index)
    d = weights.desc()
    ctx.check("mr_affine_gather_mm", L.load().mr_affine_gather_mm(
        ctx.handle, _ptr(x), T, _ptr(ids), k, C.byref(d), _ptr(out), C.c_void_p(_stream())))
    return out


def affine_dequantize(weights: AffineWeights) -> torch.Tensor:
    """Dense fp32 ``scale*q + bias`` (AffineWeights.swift:328-342). Validation only."""
    shape = ([weights.experts] if weights.experts else []) + [weights.out_features,
                                                             weights.in_features]
    out = torch.empty(shape, dtype=torch.float32, device=weights.packed.device)
    ctx = Context.get(weights.packed.device.index)
    d = weights.desc()
    ctx.check("mr_affine_dequantize", L.load().mr_affine_dequantize(
        ctx.handle, C.byref(d), _ptr(out), C.c_void_p(_stream())))
    return out


def validate_desc(weights: AffineWeights) -> tuple[int, str]:
    """Host-only validation through the C ABI (no GPU needed)."""
    buf = C.create_string_buffer(256)
    d = weights.desc()
    st = L.load().mr_affine_validate(C.byref(d), buf, 256)
    return st, buf.value.decode()


@dataclass
class Selection:
    """Router output (MoE.swift:64-75, DeepSeekV4Routing.swift:79-87):
    ``ids`` [T, k] int32 in descending choice order, ``weights`` [T, k] fp32,
    ``margins`` [T] fp32 (kth − first rejected) / max(|kth|, |rejected|)."""
    ids: torch.Tensor
    weights: torch.Tensor
    margins: torch.Tensor | None
    logits: torch.Tensor | None = None
