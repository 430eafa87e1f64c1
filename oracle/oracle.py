"""ctypes/numpy front end of the C oracle (oracle/moe_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker for the CUDA path. Imported by tests/,
``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg, never by the
product package.

Also holds the seeded description of the BASELINE configurations
(``CONFIGS``) and a numpy generator for them, built on the oracle's
SplitMix64 (Sources/StorageCore/Generator/SplitMix64.swift:13-50 in the
reference).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import threading
from dataclasses import dataclass, field

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libmoe_oracle.so")
_lib = None
_lock = threading.Lock()


def build() -> str:
    """Compile the oracle with its Makefile (gcc, OpenMP)."""
    env = dict(os.environ)
    env.pop("CC", None)
    subprocess.run(["make", "-s", "-C", _HERE], check=True, env=env)
    return _LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            src = os.path.join(_HERE, "moe_oracle.c")
            if not os.path.exists(_LIB_PATH) or (
                os.path.exists(src) and os.path.getmtime(src) > os.path.getmtime(_LIB_PATH)
            ):
                build()
            L = C.CDLL(_LIB_PATH)
            u64, i64, i32, f32, f64, vp = (
                C.c_uint64, C.c_int64, C.c_int32, C.c_float, C.c_double, C.c_void_p)
            L.mro_sm_mix.restype = u64
            L.mro_sm_mix.argtypes = [u64]
            L.mro_sm_value.restype = u64
            L.mro_sm_value.argtypes = [u64, u64]
            L.mro_sm_derive.restype = u64
            L.mro_sm_derive.argtypes = [u64, u64]
            L.mro_sm_stream.argtypes = [u64, i64, vp]
            L.mro_label.restype = u64
            L.mro_label.argtypes = [C.c_uint32] * 4
            L.mro_gen_words.argtypes = [u64, i64, vp]
            L.mro_gen_normal_bf16.argtypes = [u64, i64, f64, C.c_int, vp]
            L.mro_gen_biases.argtypes = [vp, i64, C.c_int, vp]
            L.mro_affine_validate.restype = C.c_int
            L.mro_affine_validate.argtypes = [vp, C.c_char_p, C.c_int]
            L.mro_pack.argtypes = [vp, i64, i64, C.c_int, vp]
            L.mro_unpack.argtypes = [vp, i64, i64, C.c_int, vp]
            L.mro_dequantize.argtypes = [vp, vp]
            L.mro_affine_mm.argtypes = [vp, i64, vp, i64, vp, vp]
            L.mro_affine_mm_f32.argtypes = [vp, i64, vp, i64, vp]
            L.mro_affine_gather_mm.restype = C.c_int
            L.mro_affine_gather_mm.argtypes = [vp, vp, i64, vp, i64, vp, vp]
            L.mro_e2m1_value.restype = f64
            L.mro_e2m1_value.argtypes = [C.c_int]
            L.mro_e8m0_value.restype = f64
            L.mro_e8m0_value.argtypes = [C.c_int]
            L.mro_mxfp4_validate.restype = C.c_int
            L.mro_mxfp4_validate.argtypes = [vp, C.c_char_p, C.c_int]
            L.mro_mxfp4_dequantize.argtypes = [vp, vp]
            L.mro_mxfp4_mm.argtypes = [vp, i64, vp, i64, vp, vp]
            L.mro_mxfp4_gather_mm.restype = C.c_int
            L.mro_mxfp4_gather_mm.argtypes = [vp, vp, i64, vp, i64, vp, vp]
            L.mro_mxfp4_mm_f32.argtypes = [vp, i64, vp, i64, vp]
            L.mro_mxfp4_gather_mm_f32.restype = C.c_int
            L.mro_mxfp4_gather_mm_f32.argtypes = [vp, vp, i64, vp, i64, vp]
            L.mro_router_logits.argtypes = [vp, vp, i64, i64, i64, vp]
            L.mro_router_select.restype = C.c_int
            L.mro_router_select.argtypes = [
                vp, i64, i64, i64, C.c_int, vp, C.c_int, f32, f32, vp, vp, vp, vp]
            L.mro_moe_layer_forward.restype = C.c_int
            L.mro_moe_layer_forward.argtypes = [vp, vp, i64, vp, vp, vp, vp, vp]
            L.mro_num_threads.restype = C.c_int
            L.mro_set_num_threads.argtypes = [C.c_int]
            _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


# ----------------------------------------------------------------- SplitMix64

def sm_mix(z: int) -> int:
    return int(lib().mro_sm_mix(z & (2**64 - 1)))


def sm_value(seed: int, index: int) -> int:
    return int(lib().mro_sm_value(seed, index))


def sm_derive(seed: int, label: int) -> int:
    return int(lib().mro_sm_derive(seed, label))


def sm_stream(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.uint64)
    lib().mro_sm_stream(seed, n, _p(out))
    return out


def label(layer: int, kind: int, expert: int, proj: int) -> int:
    return int(lib().mro_label(layer, kind, expert, proj))


KIND_X, KIND_ROUTER, KIND_CODES, KIND_SCALES, KIND_BIAS = 1, 2, 3, 4, 5
PROJ_GATE, PROJ_UP, PROJ_DOWN = 0, 1, 2


def gen_words(seed: int, n: int) -> np.ndarray:
    out = np.empty(n, np.uint32)
    lib().mro_gen_words(seed, n, _p(out))
    return out


def gen_normal_bf16(seed: int, n: int, std: float, absval: bool = False) -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().mro_gen_normal_bf16(seed, n, float(std), int(absval), _p(out))
    return out


def gen_biases(scales: np.ndarray, bits: int) -> np.ndarray:
    s = np.ascontiguousarray(scales, np.uint16)
    out = np.empty_like(s)
    lib().mro_gen_biases(_p(s), s.size, bits, _p(out))
    return out


# ---------------------------------------------------------------- bf16 (numpy)

def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.asarray(a, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


# ----------------------------------------------------------------- structures

class _Affine(C.Structure):
    _fields_ = [("packed", C.c_void_p), ("scales", C.c_void_p), ("biases", C.c_void_p),
                ("experts", C.c_int64), ("out", C.c_int64), ("in_", C.c_int64),
                ("group", C.c_int32), ("bits", C.c_int32), ("scale_dtype", C.c_int32)]


class _Layer(C.Structure):
    _fields_ = [("hidden", C.c_int64), ("experts", C.c_int64), ("top_k", C.c_int64),
                ("inter", C.c_int64), ("shared_inter", C.c_int64),
                ("scoring", C.c_int32), ("renorm", C.c_int32),
                ("renorm_eps", C.c_float), ("routed_scale", C.c_float),
                ("correction_bias", C.c_void_p), ("swiglu_limit", C.c_float),
                ("weight_after_down", C.c_int32), ("router_w", C.c_void_p),
                ("gate", _Affine), ("up", _Affine), ("down", _Affine),
                ("sgate", _Affine), ("sup", _Affine), ("sdown", _Affine)]


SCALE_DTYPES = {np.dtype(np.uint16): 0}  # bf16 bit patterns


@dataclass
class Affine:
    """MLX affine weights in numpy: packed uint32 [E?, out, in*bits/32];
    scales/biases [E?, out, in/group] as bf16 bit patterns (uint16),
    float16 or float32."""
    packed: np.ndarray
    scales: np.ndarray
    biases: np.ndarray
    group: int
    bits: int
    scale_dtype: int = 0  # 0 bf16 (uint16 bits), 1 f16, 2 f32

    @property
    def experts(self) -> int:
        return self.packed.shape[0] if self.packed.ndim == 3 else 0

    @property
    def out_features(self) -> int:
        return self.packed.shape[-2]

    @property
    def in_features(self) -> int:
        return self.packed.shape[-1] * (32 // self.bits)

    def c(self) -> _Affine:
        return _Affine(_p(self.packed), _p(self.scales), _p(self.biases), self.experts,
                       self.out_features, self.in_features, self.group, self.bits,
                       self.scale_dtype)

    def expert(self, e: int) -> "Affine":
        return Affine(self.packed[e], self.scales[e], self.biases[e], self.group, self.bits,
                      self.scale_dtype)

    def nbytes(self) -> int:
        return self.packed.nbytes + self.scales.nbytes + self.biases.nbytes


def affine_validate(w: Affine) -> tuple[int, str]:
    buf = C.create_string_buffer(256)
    cw = w.c()
    rc = lib().mro_affine_validate(C.byref(cw), buf, 256)
    return rc, buf.value.decode()


def pack(codes: np.ndarray, bits: int) -> np.ndarray:
    codes = np.ascontiguousarray(codes, np.uint8)
    rows, n = codes.reshape(-1, codes.shape[-1]).shape
    out = np.empty((rows, n * bits // 32), np.uint32)
    lib().mro_pack(_p(codes), rows, n, bits, _p(out))
    return out.reshape(codes.shape[:-1] + (n * bits // 32,))


def unpack(packed: np.ndarray, bits: int) -> np.ndarray:
    packed = np.ascontiguousarray(packed, np.uint32)
    rows, words = packed.reshape(-1, packed.shape[-1]).shape
    n = words * 32 // bits
    out = np.empty((rows, n), np.uint8)
    lib().mro_unpack(_p(packed), rows, n, bits, _p(out))
    return out.reshape(packed.shape[:-1] + (n,))


def dequantize(w: Affine) -> np.ndarray:
    shape = w.packed.shape[:-1] + (w.in_features,)
    out = np.empty(shape, np.float32)
    cw = w.c()
    lib().mro_dequantize(C.byref(cw), _p(out))
    return out


def affine_mm(x_bf16: np.ndarray, w: Affine, expert: int = 0):
    x = np.ascontiguousarray(x_bf16, np.uint16)
    T = x.shape[0]
    out = np.empty((T, w.out_features), np.uint16)
    f = np.empty((T, w.out_features), np.float32)
    cw = w.c()
    lib().mro_affine_mm(C.byref(cw), expert, _p(x), T, _p(out), _p(f))
    return out, f


def affine_gather_mm(x_bf16: np.ndarray, w: Affine, ids: np.ndarray):
    x = np.ascontiguousarray(x_bf16, np.uint16)
    ids = np.ascontiguousarray(ids, np.int32)
    T, k = ids.shape
    out = np.empty((T, k, w.out_features), np.uint16)
    f = np.empty((T, k, w.out_features), np.float32)
    cw = w.c()
    rc = lib().mro_affine_gather_mm(C.byref(cw), _p(x), T, _p(ids), k, _p(out), _p(f))
    if rc:
        raise ValueError("expert id out of range")
    return out, f


# ------------------------------------------------------------------ MXFP4

class _Mxfp4(C.Structure):
    _fields_ = [("packed", C.c_void_p), ("scales", C.c_void_p), ("experts", C.c_int64),
                ("out", C.c_int64), ("inn", C.c_int64)]


@dataclass
class Mxfp4:
    """MXFP4 weights: packed uint32 [E?, out, in/8], e8m0 uint8 [E?, out, in/32]."""
    packed: np.ndarray
    scales: np.ndarray

    @property
    def experts(self) -> int:
        return self.packed.shape[0] if self.packed.ndim == 3 else 0

    @property
    def out_features(self) -> int:
        return self.packed.shape[-2]

    @property
    def in_features(self) -> int:
        return self.packed.shape[-1] * 8

    def c(self) -> _Mxfp4:
        self.packed = np.ascontiguousarray(self.packed, np.uint32)
        self.scales = np.ascontiguousarray(self.scales, np.uint8)
        return _Mxfp4(self.packed.ctypes.data, self.scales.ctypes.data, self.experts,
                      self.out_features, self.in_features)


def e2m1_value(code: int) -> float:
    return lib().mro_e2m1_value(code)


def e8m0_value(e: int) -> float:
    return lib().mro_e8m0_value(e)


def mxfp4_validate(w: Mxfp4) -> tuple[int, str]:
    buf = C.create_string_buffer(256)
    cw = w.c()
    rc = lib().mro_mxfp4_validate(C.byref(cw), buf, 256)
    return rc, buf.value.decode()


def mxfp4_dequantize(w: Mxfp4) -> np.ndarray:
    out = np.empty(w.packed.shape[:-1] + (w.in_features,), np.float32)
    cw = w.c()
    lib().mro_mxfp4_dequantize(C.byref(cw), _p(out))
    return out


def mxfp4_mm(x_bf16: np.ndarray, w: Mxfp4, expert: int = 0):
    x = np.ascontiguousarray(x_bf16, np.uint16)
    T = x.shape[0]
    out = np.empty((T, w.out_features), np.uint16)
    f = np.empty((T, w.out_features), np.float32)
    cw = w.c()
    lib().mro_mxfp4_mm(C.byref(cw), expert, _p(x), T, _p(out), _p(f))
    return out, f


def mxfp4_gather_mm(x_bf16: np.ndarray, w: Mxfp4, ids: np.ndarray):
    x = np.ascontiguousarray(x_bf16, np.uint16)
    ids = np.ascontiguousarray(ids, np.int32)
    T, k = ids.shape
    out = np.empty((T, k, w.out_features), np.uint16)
    f = np.empty((T, k, w.out_features), np.float32)
    cw = w.c()
    rc = lib().mro_mxfp4_gather_mm(C.byref(cw), _p(x), T, _p(ids), k, _p(out), _p(f))
    if rc:
        raise ValueError("expert id out of range")
    return out, f


def mxfp4_mm_f32(x: np.ndarray, w: Mxfp4, expert: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty((x.shape[0], w.out_features), np.float32)
    cw = w.c()
    lib().mro_mxfp4_mm_f32(C.byref(cw), expert, _p(x), x.shape[0], _p(out))
    return out


def mxfp4_gather_mm_f32(x: np.ndarray, w: Mxfp4, ids: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    ids = np.ascontiguousarray(ids, np.int32)
    T, k = ids.shape
    out = np.empty((T, k, w.out_features), np.float32)
    cw = w.c()
    if lib().mro_mxfp4_gather_mm_f32(C.byref(cw), _p(x), T, _p(ids), k, _p(out)):
        raise ValueError("expert id out of range")
    return out


def gen_mxfp4(seed: int, experts: int, out: int, inn: int, e_lo: int = 117,
              e_hi: int = 128) -> Mxfp4:
    """Seeded MXFP4 stack (experts == 0: one matrix): uniform codes from the
    oracle's word stream, e8m0 exponents uniform in [e_lo, e_hi]."""
    E = max(experts, 1)
    words = gen_words(seed, E * out * inn // 8)
    ex = sm_stream(sm_derive(seed, 0xE8), E * out * inn // 32)
    scales = (e_lo + (ex % np.uint64(e_hi - e_lo + 1))).astype(np.uint8)
    shp = (experts,) if experts else ()
    return Mxfp4(words.reshape(shp + (out, inn // 8)), scales.reshape(shp + (out, inn // 32)))


def router_logits(x_bf16: np.ndarray, router_w: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x_bf16, np.uint16)
    w = np.ascontiguousarray(router_w, np.uint16)
    T, H = x.shape
    E = w.shape[0]
    out = np.empty((T, E), np.float32)
    lib().mro_router_logits(_p(x), _p(w), T, E, H, _p(out))
    return out


SCORING = {"sigmoid": 0, "softmax": 1, "sqrt_softplus": 2}
RENORM = {"none": 0, "plain": 1, "eps": 2}


def router_select(logits: np.ndarray, k: int, scoring: str = "sigmoid", bias=None,
                  renorm: str = "eps", eps: float = 1e-20, scale: float = 1.0):
    logits = np.ascontiguousarray(logits, np.float32)
    T, E = logits.shape
    ids = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    m = np.empty(T, np.float64)
    sc = np.empty((T, E), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    rc = lib().mro_router_select(_p(logits), T, E, k, SCORING[scoring], _p(b), RENORM[renorm],
                                 eps, scale, _p(ids), _p(w), _p(m), _p(sc))
    if rc:
        raise ValueError(f"router selection failed ({rc})")
    return ids, w, m, sc


# ------------------------------------------------------------------- configs

@dataclass(frozen=True)
class LayerConfig:
    """One MoE layer's geometry and routing (BASELINE.json `configs`)."""
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
    zipf_beta: float = 0.0  # > 0: correction bias beta*log(p_e), p_e ~ rank^-1.1
    seed: int = 0x4D524E00

    def expert_bytes(self, inter: int | None = None) -> int:
        i = self.inter if inter is None else inter
        proj = lambda o, n: o * n * self.bits // 8 + 2 * 2 * o * (n // self.group)
        return 2 * proj(i, self.hidden) + proj(self.hidden, i)


CONFIGS = {
    0: LayerConfig("config0-tiny", 1024, 16, 2, 512, 512, seed=0x4D524E00),
    1: LayerConfig("config1-dsv3", 7168, 256, 8, 2048, 2048, routed_scale=2.5,
                   seed=0x4D524E01),
    "2b2": LayerConfig("config2-wide-2bit", 7168, 384, 8, 2048, 2048, bits=2,
                       routed_scale=2.5, seed=0x4D524E02),
    "2b8": LayerConfig("config2-wide-8bit", 7168, 384, 8, 2048, 2048, bits=8,
                       routed_scale=2.5, seed=0x4D524E12),
    3: LayerConfig("config3-prefill-zipf", 7168, 256, 8, 2048, 2048, routed_scale=2.5,
                   zipf_beta=0.25, seed=0x4D524E03),
}


def zipf_bias(experts: int, beta: float, s: float = 1.1) -> np.ndarray:
    """beta*log(p_e) with p_e ~ rank^-s over a seeded permutation-free ranking
    (expert e has rank e+1)."""
    r = np.arange(1, experts + 1, dtype=np.float64)
    p = r ** (-s)
    p /= p.sum()
    return (beta * np.log(p)).astype(np.float32)


def gen_affine(seed: int, layer: int, expert: int, proj: int, out: int, inn: int,
               bits: int, group: int) -> Affine:
    words = gen_words(sm_derive(seed, label(layer, KIND_CODES, expert, proj)),
                      out * inn * bits // 32).reshape(out, inn * bits // 32)
    scales = gen_normal_bf16(sm_derive(seed, label(layer, KIND_SCALES, expert, proj)),
                             out * (inn // group), 0.02, True).reshape(out, inn // group)
    biases = gen_biases(scales, bits).reshape(scales.shape)
    return Affine(words, scales, biases, group, bits)


def _stack(parts: list[Affine]) -> Affine:
    return Affine(np.stack([p.packed for p in parts]), np.stack([p.scales for p in parts]),
                  np.stack([p.biases for p in parts]), parts[0].group, parts[0].bits)


@dataclass
class Layer:
    cfg: LayerConfig
    router_w: np.ndarray
    gate: Affine
    up: Affine
    down: Affine
    sgate: Affine | None
    sup: Affine | None
    sdown: Affine | None
    correction_bias: np.ndarray | None = None
    _keep: list = field(default_factory=list)

    def c(self) -> _Layer:
        c = self.cfg
        L = _Layer()
        L.hidden, L.experts, L.top_k, L.inter = c.hidden, c.experts, c.top_k, c.inter
        L.shared_inter = c.shared_inter if self.sgate is not None else 0
        L.scoring, L.renorm = SCORING[c.scoring], RENORM[c.renorm]
        L.renorm_eps, L.routed_scale = c.renorm_eps, c.routed_scale
        L.correction_bias = _p(self.correction_bias)
        L.swiglu_limit = c.swiglu_limit
        L.weight_after_down = int(c.weight_after_down)
        L.router_w = _p(self.router_w)
        L.gate, L.up, L.down = self.gate.c(), self.up.c(), self.down.c()
        if self.sgate is not None:
            L.sgate, L.sup, L.sdown = self.sgate.c(), self.sup.c(), self.sdown.c()
        return L


def gen_router_w(cfg: LayerConfig, layer: int = 0) -> np.ndarray:
    return gen_normal_bf16(sm_derive(cfg.seed, label(layer, KIND_ROUTER, 0, 0)),
                           cfg.experts * cfg.hidden, 1.0 / 32.0).reshape(cfg.experts, cfg.hidden)


def selected_experts(cfg: LayerConfig, x_bf16: np.ndarray, layer: int = 0) -> list[int]:
    """The routed experts the oracle's router picks for x (to generate only those)."""
    logits = router_logits(x_bf16, gen_router_w(cfg, layer))
    bias = zipf_bias(cfg.experts, cfg.zipf_beta) if cfg.zipf_beta > 0 else None
    ids, *_ = router_select(logits, cfg.top_k, cfg.scoring, bias, cfg.renorm, cfg.renorm_eps,
                            cfg.routed_scale)
    return sorted(set(ids.ravel().tolist()))


def gen_layer(cfg: LayerConfig, layer: int = 0, experts: list[int] | None = None) -> Layer:
    """Seeded weights of one layer. `experts` limits generation to a subset of
    routed experts (others are zero-filled, for oracle runs that only touch
    the selected ones)."""
    s = cfg.seed
    H, E, I, S = cfg.hidden, cfg.experts, cfg.inter, cfg.shared_inter
    router = gen_router_w(cfg, layer)

    def mk(e, proj, o, n):
        return gen_affine(s, layer, e, proj, o, n, cfg.bits, cfg.group)

    def stack(proj, o, n):
        # np.zeros is lazily committed: experts that are never generated cost
        # no resident memory
        w = Affine(np.zeros((E, o, n * cfg.bits // 32), np.uint32),
                   np.zeros((E, o, n // cfg.group), np.uint16),
                   np.zeros((E, o, n // cfg.group), np.uint16), cfg.group, cfg.bits)
        for e in (range(E) if experts is None else sorted(set(experts))):
            a = mk(e, proj, o, n)
            w.packed[e], w.scales[e], w.biases[e] = a.packed, a.scales, a.biases
        return w

    gate = stack(PROJ_GATE, I, H)
    up = stack(PROJ_UP, I, H)
    down = stack(PROJ_DOWN, H, I)
    sg = su = sd = None
    if S > 0:
        sg = mk(E, PROJ_GATE, S, H)
        su = mk(E, PROJ_UP, S, H)
        sd = mk(E, PROJ_DOWN, H, S)
    bias = zipf_bias(E, cfg.zipf_beta) if cfg.zipf_beta > 0 else None
    return Layer(cfg, router, gate, up, down, sg, su, sd, bias)


def gen_x(cfg: LayerConfig, tokens: int, layer: int = 0, batch: int = 0) -> np.ndarray:
    return gen_normal_bf16(sm_derive(cfg.seed, label(layer, KIND_X, batch, 0)),
                           tokens * cfg.hidden, 1.0).reshape(tokens, cfg.hidden)


def moe_layer_forward(L: Layer, x_bf16: np.ndarray):
    x = np.ascontiguousarray(x_bf16, np.uint16)
    T = x.shape[0]
    k, H = L.cfg.top_k, L.cfg.hidden
    out = np.empty((T, H), np.uint16)
    f = np.empty((T, H), np.float32)
    ids = np.empty((T, k), np.int32)
    w = np.empty((T, k), np.float32)
    m = np.empty(T, np.float64)
    cl = L.c()
    rc = lib().mro_moe_layer_forward(C.byref(cl), _p(x), T, _p(out), _p(f), _p(ids), _p(w),
                                     _p(m))
    if rc:
        raise ValueError(f"oracle layer forward failed ({rc})")
    return out, f, ids, w, m


def num_threads() -> int:
    return int(lib().mro_num_threads())


def set_num_threads(n: int) -> None:
    lib().mro_set_num_threads(n)
