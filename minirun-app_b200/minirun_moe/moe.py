"""Router and MoE layer over the C ABI.

Mirrors, in the reference (nanguoyu/minirun-app):
  * K3Router.select (Sources/ModelAdapters/Operators/MoE.swift:77-150),
    DeepSeekV4Router.select (Operators/DeepSeekV4Routing.swift:100-280),
    QwenRouter.select (Model/QwenMoEModel.swift:74-131)   -> ``RouterConfig``,
    ``router_select``, ``router_select_logits``;
  * RoutedExpertBackend.gather/prefetch (Operators/MoE.swift:22-51) ->
    ``ResidentExpertBackend``;
  * DeepSeekV4MoEFFN router -> routed -> shared (Model/DeepSeekV4HashFFN.swift:
    75-106, 223-255), DeepSeekV4RoutedExperts.forward
    (Loading/DeepSeekV4ExpertBackend.swift:267-344) and QwenMoEBlock.forward
    (Model/QwenMoEModel.swift:312-362) -> ``MoELayer``.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib as L
from .bridge import (AffineBridgeError, AffineWeights, Context, MoeError, Selection, _ptr,
                     _stream, affine_gather_mm)

_SCORING = {"sigmoid": L.MR_SCORING_SIGMOID, "softmax": L.MR_SCORING_SOFTMAX,
            "sqrt_softplus": L.MR_SCORING_SQRT_SOFTPLUS}
_RENORM = {"none": L.MR_RENORM_NONE, "plain": L.MR_RENORM_PLAIN, "eps": L.MR_RENORM_EPS}


@dataclass
class RouterConfig:
    experts: int
    top_k: int
    scoring: str = "sigmoid"
    renorm: str = "eps"
    renorm_eps: float = 1e-20
    routed_scale: float = 1.0
    correction_bias: torch.Tensor | None = None  # [experts] fp32, steers choice only

    @staticmethod
    def k3(experts, top_k, renormalize=True, scale=1.0, correction_bias=None):
        """K3Router: sigmoid, bias for choice, /(sum + 1e-20) when k > 1 (MoE.swift:106-145)."""
        return RouterConfig(experts, top_k, "sigmoid", "eps" if renormalize else "none", 1e-20,
                            scale, correction_bias)

    @staticmethod
    def deepseek_v4(experts, top_k, normalize=True, scale=1.0, correction_bias=None):
        """DeepSeekV4Router: sqrt(softplus), plain renorm (DeepSeekV4Routing.swift:148-271)."""
        return RouterConfig(experts, top_k, "sqrt_softplus", "plain" if normalize else "none",
                            0.0, scale, correction_bias)

    @staticmethod
    def qwen(experts, top_k, norm_topk_prob=True):
        """QwenRouter: softmax first, top-k second, plain renorm (QwenMoEModel.swift:82-127)."""
        return RouterConfig(experts, top_k, "softmax", "plain" if norm_topk_prob else "none")

    def c(self) -> L.mr_router_config:
        if self.scoring not in _SCORING:
            raise AffineBridgeError(f"unknown scoring {self.scoring!r}")
        if self.renorm not in _RENORM:
            raise AffineBridgeError(f"unknown renorm {self.renorm!r}")
        b = self.correction_bias
        return L.mr_router_config(self.experts, self.top_k, _SCORING[self.scoring],
                                  _RENORM[self.renorm], self.renorm_eps, self.routed_scale,
                                  0 if b is None else b.data_ptr())

    def validate(self) -> tuple[int, str]:
        buf = C.create_string_buffer(256)
        c = self.c()
        return L.load().mr_router_config_validate(C.byref(c), buf, 256), buf.value.decode()


def _bias_ok(cfg: RouterConfig, device) -> None:
    b = cfg.correction_bias
    if b is not None:
        if b.dtype != torch.float32 or b.numel() != cfg.experts or b.device != device:
            raise AffineBridgeError(
                f"correction bias must be [{cfg.experts}] float32 on {device}")


def router_select(x: torch.Tensor, router_w: torch.Tensor, cfg: RouterConfig,
                  want_logits: bool = False) -> Selection:
    """fp32 logits of bf16 x and W_r, then the selection (see RouterConfig)."""
    if x.dim() != 2 or x.dtype != torch.bfloat16 or router_w.dtype != torch.bfloat16:
        raise AffineBridgeError("x [T, H] and router weight [E, H] must be bfloat16")
    if router_w.shape != (cfg.experts, x.shape[1]):
        raise AffineBridgeError(
            f"router weight must be [{cfg.experts}, {x.shape[1]}], got {list(router_w.shape)}")
    _bias_ok(cfg, x.device)
    x = x.contiguous()
    T = x.shape[0]
    dev = x.device
    ids = torch.empty((T, cfg.top_k), dtype=torch.int32, device=dev)
    w = torch.empty((T, cfg.top_k), dtype=torch.float32, device=dev)
    m = torch.empty((T,), dtype=torch.float32, device=dev)
    lg = torch.empty((T, cfg.experts), dtype=torch.float32, device=dev) if want_logits else None
    ctx = Context.get(dev.index)
    c = cfg.c()
    ctx.check("mr_router_select", L.load().mr_router_select(
        ctx.handle, _ptr(x), T, x.shape[1], _ptr(router_w.contiguous()), C.byref(c), _ptr(ids),
        _ptr(w), _ptr(m), _ptr(lg), C.c_void_p(_stream())))
    return Selection(ids, w, m, lg)


class TokenExpertMap:
    """DeepSeek V4's token -> experts table for its hash-routed layers
    (Operators/DeepSeekV4Routing.swift:4-64): int32 [vocab, k], validated on
    the host as the reference's initializer does, then kept on the device."""

    def __init__(self, table, experts: int, device=None):
        t = torch.as_tensor(table, dtype=torch.int32).contiguous().cpu()
        if t.dim() != 2:
            raise AffineBridgeError("token-to-expert table must be [vocabulary, expertsPerToken]")
        self.vocab, self.k = t.shape
        self.experts = experts
        buf = C.create_string_buffer(256)
        st = L.load().mr_token_map_validate(t.data_ptr(), self.vocab, self.k, experts, buf, 256)
        if st != L.MR_OK:
            raise AffineBridgeError(buf.value.decode())
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        self.table = t.to(dev)


def _hashed_args(cfg: RouterConfig, token_ids: torch.Tensor, token_map: TokenExpertMap, T: int):
    if token_map.k != cfg.top_k or token_map.experts != cfg.experts:
        raise AffineBridgeError("token-to-expert table geometry does not match this router")
    if token_ids.shape != (T,):
        raise AffineBridgeError(f"hash routing has {token_ids.numel()} token ids for {T} rows")
    return token_ids.to(torch.int32).contiguous()


def router_select_hashed(x: torch.Tensor, router_w: torch.Tensor, cfg: RouterConfig,
                         token_ids: torch.Tensor, token_map: TokenExpertMap,
                         want_logits: bool = False) -> Selection:
    """The .tokenHash choice of DeepSeekV4Router.select (:231-256): experts from
    the table, weights from the scores at those experts. No margins."""
    if x.dim() != 2 or x.dtype != torch.bfloat16 or router_w.dtype != torch.bfloat16:
        raise AffineBridgeError("x [T, H] and router weight [E, H] must be bfloat16")
    x = x.contiguous()
    T = x.shape[0]
    tok = _hashed_args(cfg, token_ids, token_map, T)
    dev = x.device
    ids = torch.empty((T, cfg.top_k), dtype=torch.int32, device=dev)
    w = torch.empty((T, cfg.top_k), dtype=torch.float32, device=dev)
    lg = torch.empty((T, cfg.experts), dtype=torch.float32, device=dev) if want_logits else None
    ctx = Context.get(dev.index)
    c = cfg.c()
    ctx.check("mr_router_select_hashed", L.load().mr_router_select_hashed(
        ctx.handle, _ptr(x), T, x.shape[1], _ptr(router_w.contiguous()), C.byref(c), _ptr(tok),
        _ptr(token_map.table), token_map.vocab, _ptr(ids), _ptr(w), _ptr(lg),
        C.c_void_p(_stream())))
    return Selection(ids, w, None, lg)


def router_select_logits(logits: torch.Tensor, cfg: RouterConfig) -> Selection:
    """The same selection from logits produced elsewhere (MoE.swift:98-150)."""
    if logits.dim() != 2 or logits.shape[1] != cfg.experts or logits.dtype != torch.float32:
        raise AffineBridgeError(
            f"router logits must be [tokens, {cfg.experts}] float32, got "
            f"{list(logits.shape)} {logits.dtype}")
    _bias_ok(cfg, logits.device)
    logits = logits.contiguous()
    T = logits.shape[0]
    dev = logits.device
    ids = torch.empty((T, cfg.top_k), dtype=torch.int32, device=dev)
    w = torch.empty((T, cfg.top_k), dtype=torch.float32, device=dev)
    m = torch.empty((T,), dtype=torch.float32, device=dev)
    ctx = Context.get(dev.index)
    c = cfg.c()
    ctx.check("mr_router_select_logits", L.load().mr_router_select_logits(
        ctx.handle, _ptr(logits), T, C.byref(c), _ptr(ids), _ptr(w), _ptr(m),
        C.c_void_p(_stream())))
    return Selection(ids, w, m)


class ResidentExpertBackend:
    """RoutedExpertBackend over resident stacks (MoE.swift:22-51,
    Loading/RoutedExpertBackends.swift:739-795): ``gather`` returns
    ``W[ids[t, j]] . x[t]`` as [T, k, out]; ``prefetch`` has nothing to do."""

    PROJECTIONS = ("w1", "w2", "w3")  # gate, down, up

    def __init__(self, layers: dict[int, dict[str, AffineWeights]]):
        self.layers = layers

    def gather(self, x: torch.Tensor, layer: int, projection: str,
               expert_ids: torch.Tensor) -> torch.Tensor:
        if projection not in self.PROJECTIONS:
            raise AffineBridgeError(f"unknown projection {projection!r}")
        return affine_gather_mm(x, self.layers[layer][projection], expert_ids)

    def prefetch(self, layer: int, projections, expert_ids) -> None:
        return None


class MoELayer:
    """One MoE layer: router -> routed experts -> shared expert -> sum, one
    C-ABI call (``mr_moe_layer_forward``)."""

    def __init__(self, router_w: torch.Tensor, gate: AffineWeights, up: AffineWeights,
                 down: AffineWeights, router: RouterConfig,
                 shared: tuple[AffineWeights, AffineWeights, AffineWeights] | None = None,
                 swiglu_limit: float = 0.0, weight_placement: str = "before_down",
                 expert_table: torch.Tensor | None = None):
        if weight_placement not in ("before_down", "after_down"):
            raise AffineBridgeError(f"unknown weight placement {weight_placement!r}")
        self.router_w = router_w.contiguous()
        self.gate, self.up, self.down = gate, up, down
        self.router = router
        self.shared = shared
        self.swiglu_limit = float(swiglu_limit)
        self.weight_placement = weight_placement
        self.expert_table = expert_table  # uint8 device tensor of mr_expert_ptrs[E]
        self.hidden = gate.in_features
        self.inter = gate.out_features
        self._c = self._build()
        st, why = self.validate()
        if st != L.MR_OK:
            raise AffineBridgeError(why) if st == L.MR_ERR_INVALID_ARGUMENT else MoeError(
                "mr_moe_layer_validate", st, why)

    def _build(self) -> L.mr_moe_layer:
        c = L.mr_moe_layer()
        c.hidden, c.inter = self.hidden, self.inter
        c.shared_inter = self.shared[0].out_features if self.shared else 0
        c.router = self.router.c()
        c.router_w = self.router_w.data_ptr()
        c.gate, c.up, c.down = self.gate.desc(), self.up.desc(), self.down.desc()
        c.expert_table = 0 if self.expert_table is None else self.expert_table.data_ptr()
        if self.shared:
            c.shared_gate, c.shared_up, c.shared_down = (s.desc() for s in self.shared)
        c.swiglu_limit = self.swiglu_limit
        c.weight_placement = (L.MR_WEIGHT_BEFORE_DOWN if self.weight_placement == "before_down"
                              else L.MR_WEIGHT_AFTER_DOWN)
        return c

    def validate(self) -> tuple[int, str]:
        buf = C.create_string_buffer(256)
        return L.load().mr_moe_layer_validate(C.byref(self._c), buf, 256), buf.value.decode()

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None,
                selection: bool = True) -> tuple[torch.Tensor, Selection | None]:
        if x.dim() != 2 or x.shape[1] != self.hidden or x.dtype != torch.bfloat16:
            raise AffineBridgeError(
                f"input must be a non-empty [tokens, {self.hidden}] bfloat16 matrix, got "
                f"{list(x.shape)} {x.dtype}")
        if self.router.correction_bias is not None:
            _bias_ok(self.router, x.device)
        x = x.contiguous()
        T = x.shape[0]
        dev = x.device
        if out is None:
            out = torch.empty((T, self.hidden), dtype=torch.bfloat16, device=dev)
        sel = None
        if selection:
            k = self.router.top_k
            sel = Selection(torch.empty((T, k), dtype=torch.int32, device=dev),
                            torch.empty((T, k), dtype=torch.float32, device=dev),
                            torch.empty((T,), dtype=torch.float32, device=dev))
        ctx = Context.get(dev.index)
        ctx.check("mr_moe_layer_forward", L.load().mr_moe_layer_forward(
            ctx.handle, C.byref(self._c), _ptr(x), T, _ptr(out),
            _ptr(sel.ids if sel else None), _ptr(sel.weights if sel else None),
            _ptr(sel.margins if sel else None), C.c_void_p(_stream())))
        return out, sel

    __call__ = forward

    def forward_hashed(self, x: torch.Tensor, token_ids: torch.Tensor,
                       token_map: TokenExpertMap,
                       out: torch.Tensor | None = None) -> tuple[torch.Tensor, Selection]:
        """The layer with token-hash routing (mr_moe_layer_forward_hashed)."""
        if x.dim() != 2 or x.shape[1] != self.hidden or x.dtype != torch.bfloat16:
            raise AffineBridgeError(f"input must be a non-empty [tokens, {self.hidden}] bfloat16 "
                                    "matrix")
        x = x.contiguous()
        T = x.shape[0]
        tok = _hashed_args(self.router, token_ids, token_map, T)
        dev = x.device
        if out is None:
            out = torch.empty((T, self.hidden), dtype=torch.bfloat16, device=dev)
        k = self.router.top_k
        sel = Selection(torch.empty((T, k), dtype=torch.int32, device=dev),
                        torch.empty((T, k), dtype=torch.float32, device=dev), None)
        ctx = Context.get(dev.index)
        ctx.check("mr_moe_layer_forward_hashed", L.load().mr_moe_layer_forward_hashed(
            ctx.handle, C.byref(self._c), _ptr(x), _ptr(tok), T, _ptr(token_map.table),
            token_map.vocab, _ptr(out), _ptr(sel.ids), _ptr(sel.weights),
            C.c_void_p(_stream())))
        return out, sel

    def forward_host(self, x_host: torch.Tensor, out_host: torch.Tensor,
                     ids_host: torch.Tensor | None = None, device: int | None = None) -> None:
        """Host arrays in, host arrays out (mr_moe_layer_forward_host), enqueued on
        the current stream; synchronise before reading ``out_host``."""
        for t in (x_host, out_host):
            if t.is_cuda or t.dtype != torch.bfloat16 or not t.is_contiguous():
                raise AffineBridgeError("host buffers must be contiguous CPU bfloat16 tensors")
        if x_host.shape != out_host.shape or x_host.shape[1] != self.hidden:
            raise AffineBridgeError(f"x and out must be [tokens, {self.hidden}]")
        ctx = Context.get(torch.cuda.current_device() if device is None else device)
        ctx.check("mr_moe_layer_forward_host", L.load().mr_moe_layer_forward_host(
            ctx.handle, C.byref(self._c), _ptr(x_host), x_host.shape[0], _ptr(out_host),
            _ptr(ids_host), C.c_void_p(_stream())))
