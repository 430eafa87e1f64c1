"""Parity of the CUDA path (through the C ABI) with the CPU oracle.

Tolerances: top-k expert ids bit-exact, compared as
sets per token as the reference does (MoE.swift:59-61) — a flip is accepted
only where the oracle's relative margin shows a tie within fp32 summation
order (< 1e-5); layer outputs within 1e-2 relative L2 in bf16 (the checks
below are tighter where the arithmetic allows).
"""
import dataclasses
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
import minirun_moe as M
from minirun_moe import synth as S

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
REL_L2 = 1e-2          # BASELINE tolerance for layer outputs
TIE_MARGIN = 1e-5      # a top-k flip is only acceptable at a tie this close


def dev():
    return torch.device("cuda", 0)


def t_u16(a):  # numpy uint16 bf16 bits -> torch bf16 on the GPU
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev())


def n_u16(t):  # torch bf16 -> numpy uint16 bits
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


def to_dev(w: O.Affine, scale_dtype=torch.bfloat16) -> M.AffineWeights:
    packed = torch.from_numpy(np.ascontiguousarray(w.packed).view(np.int32)).to(dev())
    s, b = t_u16(w.scales), t_u16(w.biases)
    if scale_dtype != torch.bfloat16:
        s, b = s.to(scale_dtype), b.to(scale_dtype)
    return M.AffineWeights(packed, s, b, w.group, w.bits)


def oracle_with_scales(w: O.Affine, scale_dtype) -> O.Affine:
    """The same weights with scales stored as float16 / float32 (exact for
    these bf16 values: f16 holds them when in range, f32 always)."""
    s = torch.from_numpy(w.scales.view(np.int16)).view(torch.bfloat16)
    b = torch.from_numpy(w.biases.view(np.int16)).view(torch.bfloat16)
    if scale_dtype == torch.float16:
        return O.Affine(w.packed, s.half().view(torch.int16).numpy().view(np.uint16),
                        b.half().view(torch.int16).numpy().view(np.uint16), w.group, w.bits, 1)
    return O.Affine(w.packed, s.float().numpy(), b.float().numpy(), w.group, w.bits, 2)


@pytest.fixture(params=["auto", "register", "tma", "umma", "v2"])
def kernel_path(request):
    """Runs a test once per dequant-GEMV implementation."""
    ctx = M.Context.get(0)
    ctx.set_kernel_path(request.param)
    yield request.param
    ctx.set_kernel_path("auto")


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def assert_ids_match(gpu_ids, ref_ids, ref_margins):
    """Ids equal as sets per token; returns the number of tokens whose set
    differs at an oracle margin below TIE_MARGIN (excused ties)."""
    flips = 0
    for t in range(ref_ids.shape[0]):
        if set(gpu_ids[t].tolist()) != set(ref_ids[t].tolist()):
            assert abs(ref_margins[t]) < TIE_MARGIN, (t, gpu_ids[t], ref_ids[t], ref_margins[t])
            flips += 1
    return flips


# ------------------------------------------------------------------ affine ops

@pytest.mark.parametrize("bits", [2, 4, 8])
def test_gather_matches_golden(bits):
    g = np.load(os.path.join(GOLD, f"gather_b{bits}.npz"))
    w = to_dev(O.Affine(g["packed"], g["scales"], g["biases"], 64, bits))
    y = M.affine_gather_mm(t_u16(g["x"]), w, torch.from_numpy(g["ids"]).to(dev()))
    torch.cuda.synchronize()
    got = n_u16(y)
    ref = g["out"]
    assert got.shape == ref.shape
    assert rel_l2(O.bf16_to_f32(got), g["out_f32"]) < 2e-3
    assert np.mean(got == ref) > 0.97  # bf16 ties only differ in the last place


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("scale_dtype", [torch.float16, torch.float32])
def test_gather_scale_dtypes(bits, scale_dtype):
    E, out, inn, T, k = 5, 80, 448, 7, 3
    w = O._stack([O.gen_affine(21, 0, e, 1, out, inn, bits, 64) for e in range(E)])
    wo = oracle_with_scales(w, scale_dtype)
    x = O.gen_normal_bf16(5, T * inn, 1.0).reshape(T, inn)
    ids = np.random.default_rng(bits).integers(0, E, size=(T, k)).astype(np.int32)
    ref, reff = O.affine_gather_mm(x, wo, ids)
    y = M.affine_gather_mm(t_u16(x), to_dev(w, scale_dtype), torch.from_numpy(ids).to(dev()))
    assert rel_l2(O.bf16_to_f32(n_u16(y)), reff) < 2e-3


@pytest.mark.parametrize("T", [1, 3, 64, 130])
def test_affine_mm_matches_oracle(T):
    w = O.gen_affine(31, 0, 0, 2, 200, 1024, 4, 64)  # rows not a multiple of 128
    x = O.gen_normal_bf16(9, T * 1024, 1.0).reshape(T, 1024)
    ref, reff = O.affine_mm(x, w)
    y = M.affine_mm(t_u16(x), to_dev(w))
    assert rel_l2(O.bf16_to_f32(n_u16(y)), reff) < 2e-3


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_gather_both_paths_in1024(bits, kernel_path):
    """in = 1024 streams through the TMA kernel (whole 8-group stages)."""
    E, out, inn, T, k = 6, 200, 1024, 9, 4
    w = O._stack([O.gen_affine(81, 0, e, 2, out, inn, bits, 64) for e in range(E)])
    x = O.gen_normal_bf16(8, T * inn, 1.0).reshape(T, inn)
    ids = np.random.default_rng(bits + 10).integers(0, E, size=(T, k)).astype(np.int32)
    ref, reff = O.affine_gather_mm(x, w, ids)
    y = M.affine_gather_mm(t_u16(x), to_dev(w), torch.from_numpy(ids).to(dev()))
    assert rel_l2(O.bf16_to_f32(n_u16(y)), reff) < 2e-3


def test_gather_many_columns_per_expert():
    """More than 64 (token, slot) columns on one expert: several segments."""
    E, out, inn, T, k = 3, 64, 256, 50, 4
    w = O._stack([O.gen_affine(41, 0, e, 0, out, inn, 4, 64) for e in range(E)])
    x = O.gen_normal_bf16(3, T * inn, 1.0).reshape(T, inn)
    ids = np.zeros((T, k), np.int32)
    ids[:, 3] = 2
    ref, reff = O.affine_gather_mm(x, w, ids)
    y = M.affine_gather_mm(t_u16(x), to_dev(w), torch.from_numpy(ids).to(dev()))
    assert rel_l2(O.bf16_to_f32(n_u16(y)), reff) < 2e-3


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("scale_dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_staged_kernel_two_tile_segments(bits, scale_dtype):
    """The staged-activation kernel (path "v2") takes two 8-column mma tiles
    per segment once experts average more than 8 columns: each dequantised
    fragment feeds both tiles. Checked against the oracle, and a token's
    output must be bit-identical to its output in a small batch (one-tile
    segments), since every column goes through the same mma and fold."""
    ctx = M.Context.get(0)
    ctx.set_kernel_path("v2")
    try:
        E, out, inn, T, k = 3, 192, 1024, 40, 2  # Tk = 80 > 8E: 16-column segments
        w = O._stack([O.gen_affine(47, 0, e, 1, out, inn, bits, 64) for e in range(E)])
        wo = oracle_with_scales(w, scale_dtype) if scale_dtype != torch.bfloat16 else w
        x = O.gen_normal_bf16(13, T * inn, 1.0).reshape(T, inn)
        ids = np.random.default_rng(bits).integers(0, E, size=(T, k)).astype(np.int32)
        ref, reff = O.affine_gather_mm(x, wo, ids)
        wd = to_dev(w, scale_dtype)
        y = M.affine_gather_mm(t_u16(x), wd, torch.from_numpy(ids).to(dev()))
        assert rel_l2(O.bf16_to_f32(n_u16(y)), reff) < 2e-3
        small = M.affine_gather_mm(t_u16(x[:5]), wd, torch.from_numpy(ids[:5]).to(dev()))
        assert torch.equal(small, y[:5])
        ctx.sync_check()
    finally:
        ctx.set_kernel_path("auto")


@pytest.mark.parametrize("T", [1, 7, 40])
def test_f16_activation_form_wide_range(T):
    """Wide dynamic range through the default gather: each 64-element group
    of x at its own scale 2^[-60, 60], an all-zero group and a group of one
    nonzero element (one- and two-tile segments). The bf16 products are
    exact and the fold is per group, so every output stays within 1e-5 of
    sum |w||x| plus half a bf16 ulp of the exact value."""
    E, out, inn, k = 4, 160, 1024, 2
    w = O._stack([O.gen_affine(57, 0, e, 2, out, inn, 4, 64) for e in range(E)])
    rng = np.random.default_rng(T)
    xf = rng.standard_normal((T, inn)) * np.repeat(2.0 ** rng.integers(-60, 61, (T, inn // 64)),
                                                   64, axis=1)
    xf[:, 128:192] = 0.0
    xf[:, 256:320] = 0.0
    xf[:, 257] = 3.0
    x = O.f32_to_bf16(xf.astype(np.float32))
    ids = rng.integers(0, E, size=(T, k)).astype(np.int32)
    ref, reff = O.affine_gather_mm(x, w, ids)
    got = O.bf16_to_f32(n_u16(M.affine_gather_mm(t_u16(x), to_dev(w),
                                                 torch.from_numpy(ids).to(dev()))))
    dense = np.abs(O.dequantize(w).astype(np.float64))
    xa = np.abs(O.bf16_to_f32(x).astype(np.float64))
    bound = np.stack([np.stack([dense[ids[t, j]] @ xa[t] for j in range(k)]) for t in range(T)])
    err = np.abs(got.astype(np.float64) - reff)
    assert np.all(err <= 1e-5 * bound + np.abs(reff) * 2.0 ** -8), float(np.max(err / bound))
    M.Context.get(0).sync_check()


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_dequantize_exact(bits):
    w = O._stack([O.gen_affine(51, 0, e, 0, 32, 192, bits, 64) for e in range(3)])
    d = M.affine_dequantize(to_dev(w)).cpu().numpy()
    np.testing.assert_array_equal(d, O.dequantize(w))


def test_bad_expert_id_sets_device_error_without_fault():
    w = O._stack([O.gen_affine(61, 0, e, 0, 32, 128, 4, 64) for e in range(4)])
    x = t_u16(O.gen_normal_bf16(1, 2 * 128, 1.0).reshape(2, 128))
    ids = torch.tensor([[0, 4], [1, -1]], dtype=torch.int32, device=dev())
    M.affine_gather_mm(x, to_dev(w), ids)
    ctx = M.Context.get(0)
    with pytest.raises(M.MoeError, match="expert id out of range"):
        ctx.sync_check()
    assert ctx.sync_check() == 0  # the word was cleared; the context still works


# ------------------------------------------------------------------ router

@pytest.mark.parametrize("scoring,renorm,bias", [
    ("sigmoid", "eps", False), ("sigmoid", "eps", True), ("softmax", "plain", False),
    ("sqrt_softplus", "plain", True), ("sigmoid", "none", False)])
def test_router_variants(scoring, renorm, bias):
    T, E, H, k = 37, 96, 512, 6
    x = O.gen_normal_bf16(71, T * H, 1.0).reshape(T, H)
    rw = O.gen_normal_bf16(72, E * H, 1 / 32).reshape(E, H)
    b = np.random.default_rng(1).normal(0, 0.02, E).astype(np.float32) if bias else None
    logits = O.router_logits(x, rw)
    ids, w, m, _ = O.router_select(logits, k, scoring, b, renorm, 1e-20, 2.5)
    cfg = M.RouterConfig(E, k, scoring, renorm, 1e-20, 2.5,
                         None if b is None else torch.from_numpy(b).to(dev()))
    sel = M.router_select(t_u16(x), t_u16(rw), cfg, want_logits=True)
    np.testing.assert_allclose(sel.logits.cpu().numpy(), logits, rtol=1e-4, atol=1e-4)
    gi, gw = sel.ids.cpu().numpy(), sel.weights.cpu().numpy()
    assert_ids_match(gi, ids, m)
    same = np.all(gi == ids, axis=1)
    np.testing.assert_allclose(gw[same], w[same], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(sel.margins.cpu().numpy(), m, rtol=1e-3, atol=1e-5)


def test_router_config1_shape_bit_exact_ids():
    cfg = O.CONFIGS[1]
    T = 64
    x = O.gen_x(cfg, T)
    rw = O.gen_router_w(cfg)
    logits = O.router_logits(x, rw)
    ids, w, m, _ = O.router_select(logits, 8, "sigmoid", None, "eps", 1e-20, 2.5)
    sel = M.router_select(t_u16(x), t_u16(rw), M.RouterConfig(256, 8, routed_scale=2.5))
    assert_ids_match(sel.ids.cpu().numpy(), ids, m)


def test_router_select_logits_ties_lower_index():
    logits = torch.zeros((2, 16), dtype=torch.float32, device=dev())
    logits[:, [9, 3, 12]] = 1.0
    sel = M.router_select_logits(logits, M.RouterConfig(16, 2, renorm="none"))
    assert sel.ids.cpu().tolist() == [[3, 9], [3, 9]]
    assert sel.margins.cpu().tolist() == [0.0, 0.0]


# ------------------------------------------------------------------ layer

def gpu_layer_from_oracle(L: O.Layer) -> M.MoELayer:
    c = L.cfg
    shared = None
    if L.sgate is not None:
        shared = (to_dev(L.sgate), to_dev(L.sup), to_dev(L.sdown))
    bias = None if L.correction_bias is None else torch.from_numpy(L.correction_bias).to(dev())
    router = M.RouterConfig(c.experts, c.top_k, c.scoring, c.renorm, c.renorm_eps,
                            c.routed_scale, bias)
    return M.MoELayer(t_u16(L.router_w), to_dev(L.gate), to_dev(L.up), to_dev(L.down), router,
                      shared, c.swiglu_limit,
                      "after_down" if c.weight_after_down else "before_down")


def test_layer_config0_matches_golden(kernel_path):
    g = np.load(os.path.join(GOLD, "config0_T4.npz"))
    L = O.gen_layer(O.CONFIGS[0])
    layer = gpu_layer_from_oracle(L)
    out, sel = layer(t_u16(g["x"]))
    assert_ids_match(sel.ids.cpu().numpy(), g["ids"], g["margins"])
    np.testing.assert_allclose(sel.weights.cpu().numpy(), g["weights"], rtol=1e-5)
    err = rel_l2(O.bf16_to_f32(n_u16(out)), g["out_f32"])
    assert err < 5e-3, err
    M.Context.get(0).sync_check()


@pytest.mark.parametrize("variant", [dict(weight_after_down=True), dict(swiglu_limit=0.75),
                                     dict(shared_inter=0), dict(scoring="softmax",
                                                                renorm="plain")])
def test_layer_config0_variants(variant, kernel_path):
    cfg = dataclasses.replace(O.CONFIGS[0], **variant)
    L = O.gen_layer(cfg)
    if cfg.shared_inter == 0:
        L.sgate = L.sup = L.sdown = None
    x = O.gen_x(cfg, 9, batch=3)
    out, f, ids, w, m = O.moe_layer_forward(L, x)
    gout, sel = gpu_layer_from_oracle(L)(t_u16(x))
    assert_ids_match(sel.ids.cpu().numpy(), ids, m)
    err = rel_l2(O.bf16_to_f32(n_u16(gout)), f)
    assert err < 5e-3, err


@pytest.mark.parametrize("T", [1, 8])
def test_layer_config1_matches_oracle(T, kernel_path):
    cfg = O.CONFIGS[1]
    x = O.gen_x(cfg, T, batch=T)
    L = O.gen_layer(cfg, experts=O.selected_experts(cfg, x))
    out, f, ids, w, m = O.moe_layer_forward(L, x)
    layer = S.synth_layer(S.CONFIGS[1])          # all 256 experts, generated on the GPU
    gout, sel = layer(t_u16(x))
    assert_ids_match(sel.ids.cpu().numpy(), ids, m)
    err = rel_l2(O.bf16_to_f32(n_u16(gout)), f)
    assert err < 5e-3, err
    M.Context.get(0).sync_check()


def test_layer_config1_T64_matches_oracle():
    """The headline configuration itself: config 1 at T = 64 (all 64 tokens,
    ~230 distinct experts) on the default kernels against the oracle. Ids
    equal as sets per token; the tokens excused at a tie are counted and
    printed, and may only be the tokens whose oracle margin is below 1e-5."""
    cfg = O.CONFIGS[1]
    x = O.gen_x(cfg, 64, batch=64)
    L = O.gen_layer(cfg, experts=O.selected_experts(cfg, x))
    out, f, ids, w, m = O.moe_layer_forward(L, x)
    layer = S.synth_layer(S.CONFIGS[1])
    gout, sel = layer(t_u16(x))
    gids = sel.ids.cpu().numpy()
    flips = assert_ids_match(gids, ids, m)
    close = int(np.sum(np.abs(m) < TIE_MARGIN))
    err = rel_l2(O.bf16_to_f32(n_u16(gout)), f)
    print(f"config1 T=64: rel_l2={err:.3e} excused_flips={flips} "
          f"tokens_with_margin_below_{TIE_MARGIN:g}={close}")
    assert flips <= close
    assert err < 5e-3, err
    # tokens whose routing agrees are held to the same bound on their own rows
    same = [t for t in range(64) if set(gids[t].tolist()) == set(ids[t].tolist())]
    err_same = rel_l2(O.bf16_to_f32(n_u16(gout))[same], f[same])
    assert err_same < 5e-3, err_same
    M.Context.get(0).sync_check()


def test_layer_batch_invariance_config1_T64(kernel_path):
    """Each token's output depends only on that token (size-independent
    property at the full config-1 shape): a 64-token batch matches one-token
    calls — bit-identically on the register and staged kernels (every column
    goes through the same mma), and within fp32 summation order on the first
    TMA kernel, whose one-column items use fp32 FMAs instead of an mma tile."""
    layer = S.synth_layer(S.CONFIGS[1])
    x = S.synth_x(S.CONFIGS[1], 64, batch=7)
    out, sel = layer(x)
    for t in range(0, 64, 9):
        o1, s1 = layer(x[t:t + 1])
        assert torch.equal(s1.ids[0], sel.ids[t])
        if kernel_path in ("register", "v2", "auto"):
            assert torch.equal(o1[0], out[t])
        else:
            assert rel_l2(o1[0].float().cpu().numpy(), out[t].float().cpu().numpy()) < 2e-3
    M.Context.get(0).sync_check()


def test_layer_batch_invariance_config1_T512():
    """A 512-token batch (8 * 64: the 8-GPU weak-scaling group) runs the staged
    kernel with 16-column segments (two mma tiles); each token's output must
    still equal its one-token call bit for bit (routing weights included), as
    the expert-parallel path, whose ranks route their own tokens, relies on."""
    M.Context.get(0).set_kernel_path("auto")
    layer = S.synth_layer(S.CONFIGS[1])
    x = S.synth_x(S.CONFIGS[1], 512, batch=3)
    out, sel = layer(x)
    bad = []
    for t in (0, 1, 100, 257, 511):
        o1, s1 = layer(x[t:t + 1])
        assert torch.equal(s1.ids[0], sel.ids[t])
        assert torch.equal(s1.weights[0], sel.weights[t])  # routing is batch-invariant
        if not torch.equal(o1[0], out[t]):
            bad.append((t, rel_l2(o1[0].float().cpu().numpy(), out[t].float().cpu().numpy())))
    M.Context.get(0).sync_check()
    assert not bad, bad


def test_synth_matches_oracle_generator():
    cfg = O.CONFIGS[0]
    L = O.gen_layer(cfg)
    layer = S.synth_layer(S.CONFIGS[0])
    assert np.array_equal(n_u16(layer.router_w), L.router_w)
    for e in (0, 7, 15):
        assert np.array_equal(layer.gate.packed[e].cpu().numpy().view(np.uint32), L.gate.packed[e])
        assert np.array_equal(n_u16(layer.down.scales[e]), L.down.scales[e])
        assert np.array_equal(n_u16(layer.up.biases[e]), L.up.biases[e])
    assert np.array_equal(n_u16(layer.shared[2].scales), L.sdown.scales)
    assert np.array_equal(n_u16(S.synth_x(S.CONFIGS[0], 4)), O.gen_x(cfg, 4))


def test_expert_table_equals_stack():
    """Experts addressed through a device pointer table (the cache path) give
    bit-identical outputs to the contiguous stack on the same GEMV kernel
    (tables always stream with the register kernel)."""
    M.Context.get(0).set_kernel_path("register")
    from minirun_moe import _lib as LL
    import ctypes as C
    layer = S.synth_layer(S.CONFIGS[0])
    E = layer.router.experts
    table = (LL.mr_expert_ptrs * E)()
    for e in range(E):
        for p, w in enumerate((layer.gate, layer.up, layer.down)):
            table[e].packed[p] = w.packed[e].data_ptr()
            table[e].scales[p] = w.scales[e].data_ptr()
            table[e].biases[p] = w.biases[e].data_ptr()
    raw = bytes(table)
    t = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(dev())
    tl = M.MoELayer(layer.router_w, layer.gate, layer.up, layer.down, layer.router,
                    layer.shared, expert_table=t)
    x = S.synth_x(S.CONFIGS[0], 5, batch=2)
    a, _ = layer(x)
    b, _ = tl(x)
    M.Context.get(0).set_kernel_path("auto")
    assert torch.equal(a, b)


# ------------------------------------------------------ prefill-size batches

@pytest.mark.parametrize("variant", [dict(), dict(weight_after_down=True), dict(shared_inter=0),
                                     dict(bits=8), dict(swiglu_limit=0.75)])
def test_prefill_gemm_matches_oracle(variant):
    """T = 320 on config 0 (40 routed columns per expert on average) runs the
    tcgen05 grouped GEMM, which rounds each dequantised weight to bf16 as
    MLX's large-batch quantised matmul does: within the 1e-2 layer bound."""
    cfg = dataclasses.replace(O.CONFIGS[0], **variant)
    L = O.gen_layer(cfg)
    if cfg.shared_inter == 0:
        L.sgate = L.sup = L.sdown = None
    x = O.gen_x(cfg, 320, batch=5)
    out, f, ids, w, m = O.moe_layer_forward(L, x)
    gout, sel = gpu_layer_from_oracle(L)(t_u16(x))
    assert_ids_match(sel.ids.cpu().numpy(), ids, m)
    err = rel_l2(O.bf16_to_f32(n_u16(gout)), f)
    assert err < REL_L2, err
    M.Context.get(0).sync_check()
