"""HBM expert cache under a byte budget (mr_cache_* in the C ABI).

The device replacement of StorageCore's buffer pool / tile reader on the
expert path (Sources/StorageCore/BufferPool.swift:279-531,
TileReader.swift:216-340): routed experts live in host memory (pinned) and
are copied into least-recently-used HBM slots when the router selects them.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from .bridge import AffineBridgeError, AffineWeights, Context, _ptr, _stream
from .moe import RouterConfig

_SCALE_DTYPES = {torch.bfloat16: L.MR_DTYPE_BF16, torch.float16: L.MR_DTYPE_F16,
                 torch.float32: L.MR_DTYPE_F32}


class CachedLayer:
    """A MoE layer whose routed experts come from an ExpertCache: router and
    shared expert on the device, routed experts described by shape only."""

    def __init__(self, router_w: torch.Tensor, router: RouterConfig, hidden: int, inter: int,
                 bits: int, group: int = 64, scale_dtype: torch.dtype = torch.bfloat16,
                 shared: tuple[AffineWeights, AffineWeights, AffineWeights] | None = None,
                 swiglu_limit: float = 0.0, weight_placement: str = "before_down"):
        if weight_placement not in ("before_down", "after_down"):
            raise AffineBridgeError(f"unknown weight placement {weight_placement!r}")
        self.router_w = router_w.contiguous()
        self.router = router
        self.shared = shared
        self.hidden, self.inter = hidden, inter
        E = router.experts
        c = L.mr_moe_layer()
        c.hidden, c.inter = hidden, inter
        c.shared_inter = shared[0].out_features if shared else 0
        c.router = router.c()
        c.router_w = self.router_w.data_ptr()
        sd = _SCALE_DTYPES[scale_dtype]
        c.gate = L.mr_affine_desc(0, 0, 0, E, inter, hidden, group, bits, sd)
        c.up = L.mr_affine_desc(0, 0, 0, E, inter, hidden, group, bits, sd)
        c.down = L.mr_affine_desc(0, 0, 0, E, hidden, inter, group, bits, sd)
        c.expert_table = 0
        if shared:
            c.shared_gate, c.shared_up, c.shared_down = (s.desc() for s in shared)
        c.swiglu_limit = float(swiglu_limit)
        c.weight_placement = (L.MR_WEIGHT_BEFORE_DOWN if weight_placement == "before_down"
                              else L.MR_WEIGHT_AFTER_DOWN)
        self._c = c


def _host_arrays(w: AffineWeights, e: int):
    """(packed, scales, biases) of expert e as pinned host tensors."""
    return tuple(t[e].contiguous().cpu().pin_memory() for t in (w.packed, w.scales, w.biases))


class ExpertCache:
    """floor(budget_bytes / slot_bytes) expert slots on `device`."""

    def __init__(self, device: int, budget_bytes: int, slot_bytes: int):
        self.ctx = Context.get(device)
        h = C.c_void_p()
        self.ctx.check("mr_cache_create", L.load().mr_cache_create(
            self.ctx.handle, int(budget_bytes), int(slot_bytes), C.byref(h)))
        self.handle = h
        self._keep = {}  # host arrays must outlive their registration

    @staticmethod
    def slot_bytes_for(gate: AffineWeights, up: AffineWeights, down: AffineWeights) -> int:
        n = 0
        for w in (gate, up, down):
            for t in (w.packed, w.scales, w.biases):
                n += (t[0].numel() * t.element_size() + 255) // 256 * 256
        return n

    def register(self, layer: int, expert: int, arrays) -> None:
        """arrays: ((packed, scales, biases) of gate, up, down), host tensors."""
        hst = L.mr_expert_host()
        for p, (pk, sc, bi) in enumerate(arrays):
            hst.packed[p], hst.scales[p], hst.biases[p] = (pk.data_ptr(), sc.data_ptr(),
                                                           bi.data_ptr())
            hst.packed_bytes[p] = pk.numel() * pk.element_size()
            hst.scale_bytes[p] = sc.numel() * sc.element_size()
        self.ctx.check("mr_cache_register",
                       L.load().mr_cache_register(self.handle, layer, expert, C.byref(hst)))
        self._keep[(layer, expert)] = arrays

    def register_layer(self, layer: int, gate: AffineWeights, up: AffineWeights,
                       down: AffineWeights) -> None:
        """Copy a device-resident stack to pinned host memory, one expert at a time."""
        for e in range(gate.experts):
            self.register(layer, e, tuple(_host_arrays(w, e) for w in (gate, up, down)))

    def stats(self) -> dict:
        s = L.mr_cache_stats()
        st = L.load().mr_cache_get_stats(self.handle, C.byref(s))
        if st != L.MR_OK:
            raise AffineBridgeError("cache stats unavailable")
        return {k: getattr(s, k) for k, _ in L.mr_cache_stats._fields_}

    POLICIES = {"lru": 0, "none": 1, "pinned_hot_set": 2}

    def set_policy(self, policy: str, hot: list[tuple[int, int]] | None = None) -> None:
        """"lru" (default), "none" (retain nothing), or "pinned_hot_set" with
        `hot` = [(layer, expert), ...] the only experts admitted
        (BufferPool.swift CachePolicy)."""
        hot = hot or []
        lay = (C.c_int32 * max(1, len(hot)))(*[h[0] for h in hot])
        exp = (C.c_int32 * max(1, len(hot)))(*[h[1] for h in hot])
        st = L.load().mr_cache_set_policy(self.handle, self.POLICIES[policy], lay, exp, len(hot))
        if st != L.MR_OK:
            raise AffineBridgeError(f"cache policy {policy!r} refused")

    def prefetch(self, layer_id: int, experts) -> None:
        """Start copying these experts of `layer_id` into the cache (returns
        before the copies finish; the forward that uses them waits)."""
        ids = [int(e) for e in experts]
        arr = (C.c_int32 * max(1, len(ids)))(*ids)
        self.ctx.check("mr_cache_prefetch", L.load().mr_cache_prefetch(
            self.handle, layer_id, arr, len(ids), C.c_void_p(_stream())))

    def forward(self, layer_id: int, layer: CachedLayer, x: torch.Tensor,
                out: torch.Tensor | None = None, ids: torch.Tensor | None = None) -> torch.Tensor:
        if x.dim() != 2 or x.shape[1] != layer.hidden or x.dtype != torch.bfloat16:
            raise AffineBridgeError(f"input must be a [tokens, {layer.hidden}] bfloat16 matrix")
        x = x.contiguous()
        if out is None:
            out = torch.empty((x.shape[0], layer.hidden), dtype=torch.bfloat16, device=x.device)
        self.ctx.check("mr_moe_layer_forward_cached", L.load().mr_moe_layer_forward_cached(
            self.ctx.handle, self.handle, layer_id, C.byref(layer._c), _ptr(x), x.shape[0],
            _ptr(out), _ptr(ids), C.c_void_p(_stream())))
        return out

    def close(self) -> None:
        if self.handle:
            L.load().mr_cache_destroy(self.handle)
            self.handle = None
