"""Seeded synthetic layers on the device (the benchmark configurations).

Counter-based SplitMix64 (Sources/StorageCore/Generator/SplitMix64.swift:13-50
in the reference) keyed by (seed, layer, tensor kind, expert, projection), so
any tensor of any layer is reproducible without generating the ones before it:
  * packed words: word i = 32-bit half (i & 1) of value(seed, i // 2), i.e.
    codes uniform over 0..2^bits-1;
  * scales: bf16(|N(0, 0.02)|), biases: bf16(-2^(bits-1) * scale);
  * activations x: bf16(N(0, 1)); router weight: bf16(N(0, 1/1024)).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import math

import torch

from . import _lib as L
from .bridge import AffineWeights, Context, _stream
from .ep import MoELayerShard
from .moe import MoELayer, RouterConfig

KIND_X, KIND_ROUTER, KIND_CODES, KIND_SCALES, KIND_BIAS = 1, 2, 3, 4, 5
PROJ_GATE, PROJ_UP, PROJ_DOWN = 0, 1, 2


@dataclass(frozen=True)
class LayerSpec:
    """Geometry and routing of one MoE layer (BASELINE.json `configs`)."""
    name: str
    hidden: int
    experts: int
    top_k: int
    inter: int
    shared_inter: int
    bits: int = 4
    group: int = 64
    scoring: str = "sigmoid"
    renorm: str = "eps"
    renorm_eps: float = 1e-20
    routed_scale: float = 1.0
    swiglu_limit: float = 0.0
    weight_after_down: bool = False
    zipf_beta: float = 0.0
    seed: int = 0x4D524E00

    def proj_bytes(self, out: int, inn: int) -> int:
        return out * inn * self.bits // 8 + 2 * 2 * out * (inn // self.group)

    def expert_bytes(self, inter: int | None = None) -> int:
        i = self.inter if inter is None else inter
        return 2 * self.proj_bytes(i, self.hidden) + self.proj_bytes(self.hidden, i)

    def router_bytes(self) -> int:
        return self.experts * self.hidden * 2


CONFIGS = {
    0: LayerSpec("config0-tiny", 1024, 16, 2, 512, 512, seed=0x4D524E00),
    1: LayerSpec("config1-dsv3", 7168, 256, 8, 2048, 2048, routed_scale=2.5, seed=0x4D524E01),
    "2b2": LayerSpec("config2-wide-2bit", 7168, 384, 8, 2048, 2048, bits=2, routed_scale=2.5,
                     seed=0x4D524E02),
    "2b8": LayerSpec("config2-wide-8bit", 7168, 384, 8, 2048, 2048, bits=8, routed_scale=2.5,
                     seed=0x4D524E12),
    3: LayerSpec("config3-prefill-zipf", 7168, 256, 8, 2048, 2048, routed_scale=2.5,
                 zipf_beta=0.25, seed=0x4D524E03),
}


def label(layer: int, kind: int, expert: int, proj: int) -> int:
    return int(L.load().mr_synth_label(layer, kind, expert, proj))


def derive(seed: int, lab: int) -> int:
    return int(L.load().mr_synth_derive(seed, lab))


def _ctx(device) -> Context:
    return Context.get(device.index)


def synth_words(seed: int, n: int, out: torch.Tensor) -> None:
    ctx = _ctx(out.device)
    ctx.check("mr_synth_words", L.load().mr_synth_words(
        ctx.handle, seed, n, C.c_void_p(out.data_ptr()), C.c_void_p(_stream())))


def synth_normal_bf16(seed: int, n: int, std: float, absval: bool, out: torch.Tensor) -> None:
    ctx = _ctx(out.device)
    ctx.check("mr_synth_normal_bf16", L.load().mr_synth_normal_bf16(
        ctx.handle, seed, n, std, int(absval), C.c_void_p(out.data_ptr()),
        C.c_void_p(_stream())))


def synth_biases(scales: torch.Tensor, bits: int, out: torch.Tensor) -> None:
    ctx = _ctx(out.device)
    ctx.check("mr_synth_affine_biases", L.load().mr_synth_affine_biases(
        ctx.handle, C.c_void_p(scales.data_ptr()), scales.numel(), bits,
        C.c_void_p(out.data_ptr()), C.c_void_p(_stream())))


def fill_affine(spec: LayerSpec, layer: int, expert: int, proj: int, packed: torch.Tensor,
                scales: torch.Tensor, biases: torch.Tensor) -> None:
    """Write one expert projection into preallocated (contiguous) views."""
    synth_words(derive(spec.seed, label(layer, KIND_CODES, expert, proj)), packed.numel(), packed)
    synth_normal_bf16(derive(spec.seed, label(layer, KIND_SCALES, expert, proj)),
                      scales.numel(), 0.02, True, scales)
    synth_biases(scales, spec.bits, biases)


def alloc_affine(experts: int | None, out: int, inn: int, bits: int, group: int,
                 device) -> AffineWeights:
    lead = [experts] if experts else []
    packed = torch.empty(lead + [out, inn * bits // 32], dtype=torch.int32, device=device)
    scales = torch.empty(lead + [out, inn // group], dtype=torch.bfloat16, device=device)
    biases = torch.empty_like(scales)
    return AffineWeights(packed, scales, biases, group, bits)


def zipf_bias(experts: int, beta: float, s: float = 1.1) -> list[float]:
    """beta*log(p_e), p_e ~ rank^-s with expert e at rank e+1."""
    p = [(r + 1) ** (-s) for r in range(experts)]
    tot = sum(p)
    return [beta * math.log(v / tot) for v in p]


def synth_layer(spec: LayerSpec, layer: int = 0, device=None,
                shard: tuple[int, int] | None = None, strided: bool = False) -> MoELayer:
    """The seeded layer; with ``shard=(rank, world)`` only that rank's routed
    experts [rank*E/world, (rank+1)*E/world) — or, with ``strided``, experts
    rank, rank+world, ... — (same seeds as in the full layer), as a
    MoELayerShard for the expert-parallel forward."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    H, E, I, S = spec.hidden, spec.experts, spec.inter, spec.shared_inter
    e0, e1 = 0, E
    if shard is not None:
        rank, world = shard
        if E % world:
            raise ValueError(f"{E} experts do not split over {world} ranks")
        e0, e1 = rank * E // world, (rank + 1) * E // world
    router_w = torch.empty((E, H), dtype=torch.bfloat16, device=dev)
    synth_normal_bf16(derive(spec.seed, label(layer, KIND_ROUTER, 0, 0)), E * H, 1.0 / 32.0,
                      False, router_w)
    gate = alloc_affine(e1 - e0, I, H, spec.bits, spec.group, dev)
    up = alloc_affine(e1 - e0, I, H, spec.bits, spec.group, dev)
    down = alloc_affine(e1 - e0, H, I, spec.bits, spec.group, dev)
    experts = range(e0, e1)
    if shard is not None and strided:
        experts = range(shard[0], E, shard[1])
    for i, e in enumerate(experts):
        for proj, w in ((PROJ_GATE, gate), (PROJ_UP, up), (PROJ_DOWN, down)):
            fill_affine(spec, layer, e, proj, w.packed[i], w.scales[i], w.biases[i])
    shared = None
    if S > 0:
        sg = alloc_affine(None, S, H, spec.bits, spec.group, dev)
        su = alloc_affine(None, S, H, spec.bits, spec.group, dev)
        sd = alloc_affine(None, H, S, spec.bits, spec.group, dev)
        for proj, w in ((PROJ_GATE, sg), (PROJ_UP, su), (PROJ_DOWN, sd)):
            fill_affine(spec, layer, E, proj, w.packed, w.scales, w.biases)
        shared = (sg, su, sd)
    bias = None
    if spec.zipf_beta > 0:
        bias = torch.tensor(zipf_bias(E, spec.zipf_beta), dtype=torch.float32, device=dev)
    router = RouterConfig(E, spec.top_k, spec.scoring, spec.renorm, spec.renorm_eps,
                          spec.routed_scale, bias)
    placement = "after_down" if spec.weight_after_down else "before_down"
    if shard is not None:
        return MoELayerShard(shard[1], router_w, gate, up, down, router, shared,
                             spec.swiglu_limit, placement)
    return MoELayer(router_w, gate, up, down, router, shared, spec.swiglu_limit, placement)


def synth_x(spec: LayerSpec, tokens: int, layer: int = 0, batch: int = 0,
            device=None, out: torch.Tensor | None = None) -> torch.Tensor:
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    if out is None:
        out = torch.empty((tokens, spec.hidden), dtype=torch.bfloat16, device=dev)
    synth_normal_bf16(derive(spec.seed, label(layer, KIND_X, batch, 0)), tokens * spec.hidden,
                      1.0, False, out)
    return out
