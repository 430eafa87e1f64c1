"""Expert parallelism over one process per GPU (mr_ep_* in the C ABI).

Rank r of `world` holds routed experts [r*E/world, (r+1)*E/world); the router
and the shared expert are replicated. A forward all-gathers the ranks' tokens,
routes all of them (identically on every rank), runs this rank's experts over
the pairs routed to them, sums per token, and reduce-scatters the sums back to
the tokens' home ranks, where the shared expert and the combine run (NCCL over
NVLink, on the caller's stream). The reference runs experts in one process
(RoutedExpertBackend.gather, Sources/ModelAdapters/Operators/MoE.swift:22-51);
this is its multi-GPU form.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from .bridge import AffineBridgeError, Context, MoeError, _ptr, _stream
from .moe import MoELayer


class MoELayerShard(MoELayer):
    """This rank's shard of a MoE layer: gate/up/down stacks hold
    router.experts / world experts; router and shared expert are whole."""

    def __init__(self, world: int, *args, **kwargs):
        self.world = int(world)
        super().__init__(*args, **kwargs)

    def validate(self) -> tuple[int, str]:
        E = self.router.experts
        for name, w in (("gate", self.gate), ("up", self.up), ("down", self.down)):
            if (w.experts or 0) * self.world != E:
                return L.MR_ERR_INVALID_ARGUMENT, (
                    f"{name} stack holds {w.experts} experts; a shard of {E} experts over "
                    f"{self.world} ranks holds {E // self.world if E % self.world == 0 else '?'}")
        # the shard is checked as the layer it belongs to
        full = L.mr_moe_layer.from_buffer_copy(self._c)
        for d in (full.gate, full.up, full.down):
            d.experts = E
        buf = C.create_string_buffer(256)
        return L.load().mr_moe_layer_validate(C.byref(full), buf, 256), buf.value.decode()

    def forward(self, *a, **k):
        raise AffineBridgeError("a layer shard runs through ExpertGroup.forward")


def unique_id() -> bytes:
    """A new group id (rank 0 makes it; every rank needs the same bytes)."""
    buf = C.create_string_buffer(128)
    st = L.load().mr_ep_unique_id(buf)
    if st != L.MR_OK:
        raise MoeError("mr_ep_unique_id", st, "NCCL unavailable")
    return buf.raw


class ExpertGroup:
    """One rank of an expert-parallel group. With torch.distributed
    initialised, rank 0's id is broadcast to the others; otherwise pass
    `uid` (the same bytes on every rank)."""

    def __init__(self, device: int, rank: int, world: int, uid: bytes | None = None):
        if uid is None:
            import torch.distributed as dist
            box = [unique_id() if rank == 0 else None]
            dist.broadcast_object_list(box, src=0)
            uid = box[0]
        self.rank, self.world, self.device = rank, world, device
        self.ctx = Context.get(device)
        h = C.c_void_p()
        idbuf = C.create_string_buffer(uid, 128)
        self.ctx.check("mr_ep_create",
                       L.load().mr_ep_create(self.ctx.handle, idbuf, rank, world, C.byref(h)))
        self.handle = h

    def set_fused(self, fused: bool) -> None:
        """True (default): the down GEMV stores routed partials into their
        home ranks' buffers over NVLink and the home rank combines them in slot
        order (bit-identical to one GPU); False: NCCL reduce-scatter of
        per-token sums. Every rank must choose the same."""
        self.ctx.check("mr_ep_set_fused", L.load().mr_ep_set_fused(self.handle, 1 if fused else 0))

    MODES = {"allgather": 0, "nccl": 1, "alltoall": 2}

    def set_mode(self, mode: str) -> None:
        """"allgather" (default): NCCL all-gather of the tokens, fused peer
        combine; "nccl": all-gather + NCCL reduce-scatter; "alltoall": each
        rank routes its own tokens and stores their rows into the ranks that
        hold their experts (peer memory), fused peer combine. Every rank must
        choose the same."""
        self.ctx.check("mr_ep_set_mode", L.load().mr_ep_set_mode(self.handle, self.MODES[mode]))

    PLACEMENTS = {"contiguous": 0, "strided": 1}

    def set_placement(self, placement: str) -> None:
        """"contiguous" (default): rank r holds experts [r*E/N, (r+1)*E/N);
        "strided": experts r, r+N, r+2N, ... (build the shard with
        synth.synth_layer(..., shard=(r, N), strided=True) or the same
        expert order). Every rank must choose the same."""
        self.ctx.check("mr_ep_set_placement",
                       L.load().mr_ep_set_placement(self.handle, self.PLACEMENTS[placement]))

    def set_capacity(self, max_tokens: int) -> None:
        """All-to-all mode: each rank may then pass 0..max_tokens tokens per
        forward (0: every rank passes the same T). Every rank the same."""
        self.ctx.check("mr_ep_set_capacity",
                       L.load().mr_ep_set_capacity(self.handle, int(max_tokens)))

    def forward(self, shard: MoELayerShard, x: torch.Tensor, out: torch.Tensor | None = None,
                ids: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's T tokens in, their layer outputs out (same T on all
        ranks, or 0..capacity with set_capacity in the all-to-all mode)."""
        if shard.world != self.world:
            raise AffineBridgeError(f"shard of {shard.world} ranks used in a {self.world}-rank group")
        if x.dim() != 2 or x.shape[1] != shard.hidden or x.dtype != torch.bfloat16:
            raise AffineBridgeError(f"input must be a [tokens, {shard.hidden}] bfloat16 matrix")
        x = x.contiguous()
        T = x.shape[0]
        if out is None:
            out = torch.empty((T, shard.hidden), dtype=torch.bfloat16, device=x.device)
        self.ctx.check("mr_moe_layer_forward_ep", L.load().mr_moe_layer_forward_ep(
            self.ctx.handle, self.handle, C.byref(shard._c), _ptr(x), T, _ptr(out), _ptr(ids),
            C.c_void_p(_stream())))
        return out

    def close(self) -> None:
        if self.handle:
            L.load().mr_ep_destroy(self.handle)
            self.handle = None
