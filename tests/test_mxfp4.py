"""MXFP4 on the CPU: the oracle pinned to the OCP MX element encodings and to
independent decoders, the host-side MXFP4Weights checks and the C-ABI
validator (no GPU).

Pins: the e2m1 values are the table of the OCP Microscaling Formats v1.0
specification and of transformers' MXFP4 integration (FP4_VALUES); e8m0 is
checked on all 256 codes against torch.float8_e8m0fnu; the oracle's
dequantize (element 0 in the low nibble, MXFP4Weights.swift:38-50) is checked
against transformers' gpt-oss block decoder on seeded blocks. The reference
holds no MXFP4 known-answer vectors of its own (its MLX arithmetic lives in
the un-vendored mlx-swift 0.31.4).
"""
import ctypes as C

import numpy as np
import pytest
import torch

import minirun_moe as M
from minirun_moe import _lib as L
from oracle import oracle as O

OCP_E2M1 = [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]


def test_e2m1_values_match_the_ocp_table():
    for c in range(16):
        v = O.e2m1_value(c)
        mag = OCP_E2M1[c & 7]
        assert abs(v) == mag and (np.signbit(v) == bool(c & 8)), (c, v)


def test_e2m1_values_match_transformers():
    mx = pytest.importorskip("transformers.integrations.mxfp4")
    assert [O.e2m1_value(c) for c in range(16)] == list(mx.FP4_VALUES)


def test_e8m0_values_match_torch():
    ref = torch.arange(256, dtype=torch.uint8).view(torch.float8_e8m0fnu).double().numpy()
    got = np.array([O.e8m0_value(e) for e in range(256)])
    np.testing.assert_array_equal(got[:255], ref[:255])
    assert np.isnan(got[255]) and np.isnan(ref[255])


def test_dequantize_matches_transformers_block_decoder():
    mx = pytest.importorskip("transformers.integrations.mxfp4")
    w = O.gen_mxfp4(3, 2, 24, 256, e_lo=100, e_hi=150)
    ref = O.mxfp4_dequantize(w)
    E, out, inn = 2, 24, 256
    blocks = torch.from_numpy(w.packed.view(np.uint8).reshape(E, out, inn // 32, 16).copy())
    scales = torch.from_numpy(w.scales.reshape(E, out, inn // 32).copy())
    dec = mx.convert_moe_packed_tensors(blocks, scales, dtype=torch.float32)
    np.testing.assert_array_equal(dec.transpose(1, 2).numpy(), ref)


def test_oracle_mm_matches_dense_float64():
    w = O.gen_mxfp4(4, 0, 40, 512)
    x = O.gen_normal_bf16(2, 3 * 512, 1.0).reshape(3, 512)
    out, f = O.mxfp4_mm(x, w)
    dense = O.mxfp4_dequantize(w).astype(np.float64)
    ref = O.bf16_to_f32(x).astype(np.float64) @ dense.T
    np.testing.assert_allclose(f, ref.astype(np.float32), rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(out, O.f32_to_bf16(f))


def test_oracle_gather_routes_each_slot():
    w = O.gen_mxfp4(5, 4, 16, 64)
    x = O.gen_normal_bf16(3, 2 * 64, 1.0).reshape(2, 64)
    ids = np.array([[3, 0], [3, 3]], np.int32)
    out, f = O.mxfp4_gather_mm(x, w, ids)
    dense = O.mxfp4_dequantize(w)
    for t in range(2):
        for j in range(2):
            ref, _ = O.mxfp4_mm(x[t:t + 1], O.Mxfp4(w.packed[ids[t, j]], w.scales[ids[t, j]]))
            np.testing.assert_array_equal(out[t, j], ref[0])
    with pytest.raises(ValueError):
        O.mxfp4_gather_mm(x, w, np.array([[4, 0], [0, 0]], np.int32))
    assert dense.shape == (4, 16, 64)


def _desc(experts, out, inn, packed=1, scales=1):
    return L.mr_mxfp4_desc(packed and 0x1000, scales and 0x2000, experts, out, inn)


@pytest.mark.parametrize("experts,out,inn,packed,scales,status,needle", [
    (4, 64, 512, 1, 1, L.MR_OK, ""),
    (0, 64, 96, 1, 1, L.MR_OK, ""),            # valid MXFP4 (the matmul needs in % 512)
    (4, 64, 100, 1, 1, L.MR_ERR_INVALID_ARGUMENT, "multiple of 8"),
    (4, 64, 48, 1, 1, L.MR_ERR_INVALID_ARGUMENT, "groupSize 32"),
    (-1, 64, 512, 1, 1, L.MR_ERR_INVALID_ARGUMENT, "positive"),
    (4, 0, 512, 1, 1, L.MR_ERR_INVALID_ARGUMENT, "positive"),
    (4, 64, 512, 0, 1, L.MR_ERR_INVALID_ARGUMENT, "non-NULL"),
    (4, 64, 512, 1, 0, L.MR_ERR_INVALID_ARGUMENT, "non-NULL"),
])
def test_c_abi_validator(experts, out, inn, packed, scales, status, needle):
    buf = C.create_string_buffer(256)
    d = _desc(experts, out, inn, packed, scales)
    assert L.load().mr_mxfp4_validate(C.byref(d), buf, 256) == status
    assert needle in buf.value.decode()
    rc, msg = O.mxfp4_validate(O.Mxfp4(np.zeros((1, 1), np.uint32), np.zeros((1, 1), np.uint8)))
    assert rc == 1 and "groupSize 32" in msg  # in = 8


def test_weights_wrapper_refusals():
    p = torch.zeros(2, 8, 64, dtype=torch.int32)
    s = torch.zeros(2, 8, 16, dtype=torch.uint8)
    w = M.MXFP4Weights(p, s)
    assert (w.experts, w.out_features, w.in_features) == (2, 8, 512)
    assert w.nbytes == p.numel() * 4 + s.numel()
    cases = [
        (p.float(), s, "must be .uint32"),
        (p, s.to(torch.int8), "must be .uint8"),
        (p, s[0], "rank 2"),
        (p, s[:1], "expert count differs"),
        (p, s[:, :4], "row count differs"),
        (p[..., :3].contiguous(), s[..., :1], "multiple of groupSize 32"),
        (p, s[..., :8], "group count differs"),
    ]
    for pk, sc, needle in cases:
        with pytest.raises(M.MXFP4BridgeError, match=needle):
            M.MXFP4Weights(pk, sc)
    one = M.MXFP4Weights(p[0], s[0])
    assert one.experts is None
    with pytest.raises(M.MXFP4BridgeError, match="stacked MXFP4Weights"):
        M.mxfp4_gather_mm(torch.zeros(1, 512, dtype=torch.bfloat16), one,
                          torch.zeros(1, 1, dtype=torch.int32))
    with pytest.raises(M.MXFP4BridgeError, match="single matrix"):
        M.mxfp4_mm(torch.zeros(1, 512, dtype=torch.bfloat16), w)
    st, msg = M.mxfp4_validate(w)
    assert st == L.MR_OK and msg == ""
