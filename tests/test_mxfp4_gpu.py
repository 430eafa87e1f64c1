"""MXFP4 on the GPU, through the C ABI, against the CPU oracle.

dequantize: bit-exact (e2m1 * 2^(e-127) is exact in fp32). The matmuls:
within 2e-3 relative L2 of the oracle's exact result and at least 97% of
the bf16 outputs bit-equal (fp32 summation order only moves ties); with a
wide dynamic range in x, every output within 1e-5 of sum |w||x| plus half a
bf16 ulp of the exact value.
"""
import numpy as np
import pytest
import torch

import minirun_moe as M
from minirun_moe import _lib as L
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def dev():
    return torch.device("cuda", 0)


def t_u16(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(dev())


def n_u16(t):
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)


def to_dev(w: O.Mxfp4) -> M.MXFP4Weights:
    packed = torch.from_numpy(np.ascontiguousarray(w.packed).view(np.int32)).to(dev())
    scales = torch.from_numpy(np.ascontiguousarray(w.scales)).to(dev())
    return M.MXFP4Weights(packed, scales)


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def check(got_u16, ref_u16, ref_f32):
    assert got_u16.shape == ref_u16.shape
    assert rel_l2(O.bf16_to_f32(got_u16), ref_f32) < 2e-3
    assert np.mean(got_u16 == ref_u16) > 0.97


def test_dequantize_exact_with_special_exponents():
    w = O.gen_mxfp4(11, 3, 40, 256, e_lo=0, e_hi=255)
    w.scales.reshape(-1)[:4] = [0, 1, 254, 255]
    ref = O.mxfp4_dequantize(w)
    got = M.mxfp4_dequantize(to_dev(w)).cpu().numpy()
    nan = np.isnan(ref)
    assert nan.any()
    np.testing.assert_array_equal(np.isnan(got), nan)
    np.testing.assert_array_equal(got[~nan], ref[~nan])
    one = O.Mxfp4(w.packed[1], w.scales[1])
    np.testing.assert_array_equal(M.mxfp4_dequantize(to_dev(one)).cpu().numpy(),
                                  O.mxfp4_dequantize(one))


@pytest.mark.parametrize("E,out,inn,T,k", [
    (8, 256, 512, 1, 4), (6, 200, 1024, 9, 4), (16, 512, 2048, 64, 6), (4, 96, 4096, 3, 2),
])
def test_gather_matches_oracle(E, out, inn, T, k):
    w = O.gen_mxfp4(20 + E, E, out, inn)
    x = O.gen_normal_bf16(7, T * inn, 1.0).reshape(T, inn)
    ids = np.random.default_rng(E + T).integers(0, E, size=(T, k)).astype(np.int32)
    ref, reff = O.mxfp4_gather_mm(x, w, ids)
    y = M.mxfp4_gather_mm(t_u16(x), to_dev(w), torch.from_numpy(ids).to(dev()))
    check(n_u16(y), ref, reff)


def test_gather_repeats_and_many_columns_per_expert():
    E, out, inn, T, k = 3, 64, 512, 50, 4
    w = O.gen_mxfp4(31, E, out, inn)
    x = O.gen_normal_bf16(3, T * inn, 1.0).reshape(T, inn)
    ids = np.zeros((T, k), np.int32)
    ids[:, 3] = 2
    ref, reff = O.mxfp4_gather_mm(x, w, ids)
    y = M.mxfp4_gather_mm(t_u16(x), to_dev(w), torch.from_numpy(ids).to(dev()))
    check(n_u16(y), ref, reff)


@pytest.mark.parametrize("T", [1, 5, 130])
def test_mm_matches_oracle(T):
    w = O.gen_mxfp4(41, 0, 200, 1024)
    x = O.gen_normal_bf16(9, T * 1024, 1.0).reshape(T, 1024)
    ref, reff = O.mxfp4_mm(x, w)
    y = M.mxfp4_mm(t_u16(x), to_dev(w))
    check(n_u16(y), ref, reff)


def test_wide_dynamic_range_activations():
    """Each 32-element half of x at its own scale 2^[-60, 60]: the per-half
    activation factor keeps every product exact."""
    E, out, inn, T, k = 4, 128, 1024, 6, 2
    w = O.gen_mxfp4(51, E, out, inn, e_lo=100, e_hi=140)
    rng = np.random.default_rng(5)
    xf = rng.standard_normal((T, inn)) * np.repeat(2.0 ** rng.integers(-60, 61, (T, inn // 32)),
                                                   32, axis=1)
    x = O.f32_to_bf16(xf.astype(np.float32))
    ids = rng.integers(0, E, size=(T, k)).astype(np.int32)
    ref, reff = O.mxfp4_gather_mm(x, w, ids)
    got = O.bf16_to_f32(n_u16(M.mxfp4_gather_mm(t_u16(x), to_dev(w),
                                                torch.from_numpy(ids).to(dev()))))
    dense = np.abs(O.mxfp4_dequantize(w).astype(np.float64))
    xa = np.abs(O.bf16_to_f32(x).astype(np.float64))
    bound = np.stack([np.stack([dense[ids[t, j]] @ xa[t] for j in range(k)]) for t in range(T)])
    err = np.abs(got.astype(np.float64) - reff)
    assert np.all(err <= 1e-5 * bound + np.abs(reff) * 2.0 ** -8), float(np.max(err / bound))


def test_batch_invariance_across_two_column_switch():
    """bf16 gathers take the two-column form while experts average at most
    two columns (Tk <= 2E) and the one-column form above. A token's output
    is bit-identical either way, also when a 32-element half spans a wide
    dynamic range (elements far below 2^-31 of the half's maximum fall into
    the f16 subnormal tail of the scaled activation)."""
    E, out, inn, k = 4, 128, 1024, 2
    w = O.gen_mxfp4(53, E, out, inn)
    rng = np.random.default_rng(11)
    xf = rng.standard_normal((5, inn)).astype(np.float32) * 2.0 ** -40
    xf[:, ::32] = rng.standard_normal((5, inn // 32)) * 64.0  # one large element per half
    x = t_u16(O.f32_to_bf16(xf.astype(np.float32)))
    ids = torch.from_numpy(rng.integers(0, E, size=(5, k)).astype(np.int32)).to(dev())
    wd = to_dev(w)
    small = M.mxfp4_gather_mm(x[:4], wd, ids[:4])  # Tk = 8 = 2E: two-column form
    large = M.mxfp4_gather_mm(x, wd, ids)          # Tk = 10: one-column form
    assert torch.equal(small, large[:4])


def test_nan_exponent_poisons_its_row_only():
    E, out, inn = 2, 64, 512
    w = O.gen_mxfp4(61, E, out, inn)
    w.scales[1, 5, 3] = 255
    x = O.gen_normal_bf16(2, inn, 1.0).reshape(1, inn)
    ids = np.array([[1, 0]], np.int32)
    y = O.bf16_to_f32(n_u16(M.mxfp4_gather_mm(t_u16(x), to_dev(w),
                                              torch.from_numpy(ids).to(dev()))))
    assert np.isnan(y[0, 0, 5]) and np.isfinite(np.delete(y[0, 0], 5)).all()
    assert np.isfinite(y[0, 1]).all()


def test_bad_expert_id_sets_device_error_without_fault():
    w = O.gen_mxfp4(71, 4, 64, 512)
    x = t_u16(O.gen_normal_bf16(1, 2 * 512, 1.0).reshape(2, 512))
    ids = torch.tensor([[0, 4], [1, -1]], dtype=torch.int32, device=dev())
    M.mxfp4_gather_mm(x, to_dev(w), ids)
    ctx = M.Context.get(0)
    with pytest.raises(M.MoeError, match="expert id out of range"):
        ctx.sync_check()
    assert ctx.sync_check() == 0


def test_unsupported_width_is_refused():
    w = O.gen_mxfp4(81, 2, 64, 96)  # valid MXFP4, not a whole 512-element stage
    x = t_u16(O.gen_normal_bf16(1, 96, 1.0).reshape(1, 96))
    with pytest.raises(M.MoeError) as e:
        M.mxfp4_gather_mm(x, to_dev(w), torch.zeros(1, 1, dtype=torch.int32, device=dev()))
    assert e.value.status == L.MR_ERR_UNSUPPORTED and "512" in e.value.message
    d = M.mxfp4_dequantize(to_dev(w)).cpu().numpy()  # dequantize takes any valid width
    np.testing.assert_array_equal(d, O.mxfp4_dequantize(w))
