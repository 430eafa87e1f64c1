"""The CPU oracle, pinned before it is trusted (no GPU needed).

1. SplitMix64 against the algorithm's published seed-0 outputs and the
   reference's own generator tests (Tests/StorageCoreTests/
   DeterministicContentTests.swift:6-53): value(seed, i) equals the stream,
   seeds and labels decorrelate, bits are balanced.
2. MLX affine packing against hand-computed words (kat.json).
3. Every oracle operator against an independent float64 numpy restatement
   (tests/np_ref.py).
4. The committed golden fixtures (tests/golden/) against the current oracle.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O
import np_ref as R

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def kat():
    with open(os.path.join(GOLD, "kat.json")) as f:
        return json.load(f)


def test_splitmix64_published_vectors():
    got = [int(v) for v in O.sm_stream(0, 3)]
    assert got == [int(h, 16) for h in kat()["splitmix64_seed0"]]


@pytest.mark.parametrize("seed", [0, 1, 42, 0xDEADBEEF, 2**64 - 1])
def test_splitmix64_value_equals_stream(seed):
    # DeterministicContentTests.swift:10-19
    stream = O.sm_stream(seed, 100)
    for i in range(100):
        assert O.sm_value(seed, i) == int(stream[i])


def test_splitmix64_derive_and_balance():
    # DeterministicContentTests.swift:22-46
    a = [O.sm_value(42, i) for i in range(64)]
    b = [O.sm_value(43, i) for i in range(64)]
    assert a != b
    assert O.sm_derive(42, 0) != O.sm_value(42, 0)
    assert O.sm_derive(42, 0) != O.sm_derive(42, 1)
    ones = sum(bin(O.sm_value(7, i)).count("1") for i in range(4096))
    assert abs(ones / (4096 * 64) - 0.5) < 0.02


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_pack_known_answer(bits):
    k = kat()
    codes = np.array(k[f"pack{bits}_codes"], np.uint8).reshape(1, -1)
    word = int(k[f"pack{bits}_word"], 16)
    assert int(O.pack(codes, bits)[0, 0]) == word
    assert O.unpack(np.array([[word]], np.uint32), bits).tolist() == codes.tolist()
    assert R.unpack(np.array([[word]], np.uint32), bits).tolist() == codes.tolist()


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_pack_roundtrip(bits):
    rng = np.random.default_rng(bits)
    codes = rng.integers(0, 2**bits, size=(7, 256), dtype=np.uint8)
    assert np.array_equal(O.unpack(O.pack(codes, bits), bits), codes)


def test_affine_validate_mirrors_reference():
    w = O.gen_affine(1, 0, 0, 0, 8, 128, 4, 64)
    assert O.affine_validate(w)[0] == 0
    bad = O.Affine(w.packed, w.scales, w.biases, 48, 4)  # 128 % 48 != 0
    rc, msg = O.affine_validate(bad)
    assert rc != 0 and "not a multiple of the group size" in msg
    rc, msg = O.affine_validate(O.Affine(w.packed, w.scales, w.biases, 64, 3))
    assert rc != 0 and "must divide 32" in msg


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_dequantize_matches_numpy(bits):
    w = O.gen_affine(5, 0, 1, 2, 16, 192, bits, 64)
    np.testing.assert_allclose(O.dequantize(w), R.dequant64(w.packed, w.scales, w.biases, bits,
                                                            64), rtol=0, atol=1e-6)


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_gather_matches_numpy(bits):
    E, out, inn, T, k = 5, 40, 320, 3, 4
    w = O._stack([O.gen_affine(11, 0, e, 0, out, inn, bits, 64) for e in range(E)])
    x = O.gen_normal_bf16(77, T * inn, 1.0).reshape(T, inn)
    ids = np.array([[4, 0, 4, 2], [1, 3, 0, 2], [2, 2, 2, 2]], np.int32)
    y, yf = O.affine_gather_mm(x, w, ids)
    ry, ryf = R.gather_mm(x, w, ids)
    np.testing.assert_allclose(yf, ryf, rtol=1e-6, atol=1e-5)
    assert np.mean(y == ry) > 0.999


def test_gather_rejects_bad_ids():
    w = O._stack([O.gen_affine(11, 0, e, 0, 8, 64, 4, 64) for e in range(2)])
    x = O.gen_normal_bf16(1, 64, 1.0).reshape(1, 64)
    with pytest.raises(ValueError):
        O.affine_gather_mm(x, w, np.array([[2]], np.int32))


@pytest.mark.parametrize("scoring,renorm", [("sigmoid", "eps"), ("softmax", "plain"),
                                            ("sqrt_softplus", "plain"), ("sigmoid", "none")])
def test_router_matches_numpy(scoring, renorm):
    rng = np.random.default_rng(3)
    logits = rng.normal(0, 2.5, size=(9, 64)).astype(np.float32)
    bias = rng.normal(0, 0.05, size=64).astype(np.float32)
    ids, w, m, _ = O.router_select(logits, 6, scoring, bias, renorm, 1e-20, 2.5)
    rid, rw, rm = R.router(logits, 6, scoring, bias, renorm, 1e-20, 2.5)
    assert np.array_equal(ids, rid)
    np.testing.assert_allclose(w, rw, rtol=1e-6)
    np.testing.assert_allclose(m, rm, rtol=1e-9, atol=1e-12)


def test_router_ties_go_to_lower_index():
    logits = np.zeros((1, 8), np.float32)
    logits[0, [6, 2, 5]] = 1.0
    ids, _, m, _ = O.router_select(logits, 2)
    assert ids.tolist() == [[2, 5]]
    assert m[0] == 0.0  # kth (5) and first rejected (6) tie


def test_router_plain_renorm_refuses_zero_sum():
    logits = np.full((1, 4), -1000.0, np.float32)  # softplus underflows to 0
    with pytest.raises(ValueError):
        O.router_select(logits, 2, "sqrt_softplus", None, "plain")


@pytest.mark.parametrize("after", [False, True])
def test_layer_matches_numpy(after):
    import dataclasses
    cfg = dataclasses.replace(O.CONFIGS[0], weight_after_down=after, swiglu_limit=0.0)
    L = O.gen_layer(cfg)
    x = O.gen_x(cfg, 3, batch=5)
    out, f, ids, w, m = O.moe_layer_forward(L, x)
    rout, rf, rids, rw, rm = R.layer(L, x)
    assert np.array_equal(ids, rids)
    np.testing.assert_allclose(w, rw, rtol=1e-6)
    rel = np.linalg.norm(f - rf) / np.linalg.norm(rf)
    assert rel < 1e-4, rel


def test_layer_swiglu_limit_matches_numpy():
    import dataclasses
    cfg = dataclasses.replace(O.CONFIGS[0], swiglu_limit=0.5)
    L = O.gen_layer(cfg)
    x = O.gen_x(cfg, 2)
    _, f, *_ = O.moe_layer_forward(L, x)
    _, rf, *_ = R.layer(L, x)
    assert np.linalg.norm(f - rf) / np.linalg.norm(rf) < 1e-4


def test_golden_config0_is_current():
    g = np.load(os.path.join(GOLD, "config0_T4.npz"))
    cfg = O.CONFIGS[0]
    L = O.gen_layer(cfg)
    x = O.gen_x(cfg, 4)
    assert np.array_equal(x, g["x"])
    assert np.array_equal(O.router_logits(x, L.router_w), g["logits"])
    out, f, ids, w, m = O.moe_layer_forward(L, x)
    assert np.array_equal(ids, g["ids"])
    assert np.array_equal(out, g["out"])
    np.testing.assert_array_equal(f, g["out_f32"])


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_golden_gather_is_current(bits):
    g = np.load(os.path.join(GOLD, f"gather_b{bits}.npz"))
    w = O.Affine(g["packed"], g["scales"], g["biases"], 64, bits)
    y, yf = O.affine_gather_mm(g["x"], w, g["ids"])
    assert np.array_equal(y, g["out"])


def test_config_tables_agree():
    """The product's seeded config table equals the oracle's."""
    import ast
    path = os.path.join(os.path.dirname(GOLD), "..", "minirun-app_b200", "minirun_moe",
                        "synth.py")
    src = open(path).read()
    tree = ast.parse(src)
    names = {n.args[0].value for n in ast.walk(tree)
             if isinstance(n, ast.Call) and getattr(n.func, "id", "") == "LayerSpec"
             and n.args and isinstance(n.args[0], ast.Constant)}
    assert names == {c.name for c in O.CONFIGS.values()}


def test_expert_bytes_match_survey():
    c = O.CONFIGS[1]
    assert c.expert_bytes() == 24_772_608
    assert O.CONFIGS[0].expert_bytes() == 884_736
    assert O.CONFIGS["2b2"].expert_bytes() == 13_762_560
    assert O.CONFIGS["2b8"].expert_bytes() == 46_792_704
