"""K3 latent MoE on the CPU: the oracle's pieces against their definitions,
and the C-ABI block validator (no GPU)."""
import ctypes as C

import numpy as np
import pytest

from minirun_moe import _lib as L
from oracle import k3_oracle as K
from oracle import oracle as O

import k3_case


def test_situ_matches_its_definition():
    rng = np.random.default_rng(0)
    g = (rng.standard_normal(4000) * 20).astype(np.float32)
    u = (rng.standard_normal(4000) * 40).astype(np.float32)
    gd, ud = g.astype(np.float64), u.astype(np.float64)
    ref = 4 * np.tanh(gd / 4) / (1 + np.exp(-gd)) * (25 * np.tanh(ud / 25))
    np.testing.assert_allclose(K.situ(g, u, 4.0, 25.0), ref, rtol=2e-6, atol=1e-6)
    ref_lin = 4 * np.tanh(gd / 4) / (1 + np.exp(-gd)) * ud
    np.testing.assert_allclose(K.situ(g, u, 4.0, None), ref_lin, rtol=2e-6, atol=1e-6)
    # the up branch saturates at +-25: not a SwiGLU
    assert abs(K.situ(np.float32([60]), np.float32([60]), 4.0, 25.0)[0] - 4 * 25 * np.tanh(2.4)) < 1e-3


def test_rms_norm_matches_its_definition():
    x = np.random.default_rng(1).standard_normal((3, 512)).astype(np.float32)
    w = np.linspace(0.5, 1.5, 512).astype(np.float32)
    ref = w * x / np.sqrt(np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True) + 1e-5)
    np.testing.assert_allclose(K.rms(x, w, 1e-5), ref, rtol=1e-6)


def test_oracle_block_composes_its_steps():
    B, _ = k3_case.make(seed=3, E=8, H=512, Lt=512, I=512, S=512, k=2)
    x = k3_case.x_for(3, 2, 512)
    out, ids, w, _ = K.forward(B, x)
    # routed part by hand for token 0
    t = 0
    lat = B.down(x[t:t + 1])
    rs = np.zeros(512, np.float64)
    for j in range(2):
        e = ids[t, j]
        g = O.mxfp4_mm_f32(lat, B.w1, e)
        u = O.mxfp4_mm_f32(lat, B.w3, e)
        a = K.situ(g, u, 4.0, 25.0)
        rs += w[t, j] * O.mxfp4_mm_f32(a, B.w2, e)[0]
    rs = K.rms(rs[None].astype(np.float32), B.norm, 1e-5)
    sg, su, sd = B.shared
    ref = B.up(rs) + sd(K.situ(sg(x[:1]), su(x[:1]), 4.0, 25.0))
    np.testing.assert_allclose(out[0], ref[0], rtol=1e-5, atol=1e-6)
    assert out.shape == (2, 512) and np.isfinite(out).all()


def _proj(out, inn, ptr=0x1000, dt=L.MR_DTYPE_BF16):
    return L.mr_k3_projection(L.MR_K3_PROJ_DENSE, ptr, dt, out, inn, L.mr_mxfp4_desc())


def _block(**kw):
    E, H, Lt, I, S, k = 16, 1024, 512, 512, 512, 4
    mx = lambda o, i: L.mr_mxfp4_desc(0x2000, 0x3000, E, o, i)
    r = L.mr_router_config(E, k, L.MR_SCORING_SIGMOID, L.MR_RENORM_EPS, 1e-20, 1.0, 0)
    b = L.mr_k3_moe(r, 0x4000, L.MR_DTYPE_BF16, _proj(Lt, H), _proj(H, Lt), 0x5000,
                    L.MR_DTYPE_F32, 1e-5, mx(I, Lt), mx(I, Lt), mx(Lt, I), _proj(S, H),
                    _proj(S, H), _proj(H, S), H, Lt, I, S, 4.0, 25.0)
    for key, v in kw.items():
        setattr(b, key, v)
    return b


@pytest.mark.parametrize("change,status,needle", [
    ({}, L.MR_OK, ""),
    ({"situ_beta": 0.0}, L.MR_ERR_INVALID_ARGUMENT, "situ beta"),
    ({"latent": 256}, L.MR_ERR_INVALID_ARGUMENT, "routed down"),
    ({"gate_weight": 0}, L.MR_ERR_INVALID_ARGUMENT, "router gate"),
    ({"norm_dtype": L.MR_DTYPE_F16}, L.MR_ERR_INVALID_ARGUMENT, "norm"),
    ({"shared_inter": 0}, L.MR_OK, ""),
    ({"inter": 256, "w1": L.mr_mxfp4_desc(0x2000, 0x3000, 16, 256, 512),
      "w3": L.mr_mxfp4_desc(0x2000, 0x3000, 16, 256, 512),
      "w2": L.mr_mxfp4_desc(0x2000, 0x3000, 16, 512, 256)}, L.MR_ERR_UNSUPPORTED, "512"),
])
def test_block_validator(change, status, needle):
    b = _block(**change)
    buf = C.create_string_buffer(256)
    assert L.load().mr_k3_moe_validate(C.byref(b), buf, 256) == status, buf.value
    assert needle in buf.value.decode()
    b = _block()
    b.router.scoring = L.MR_SCORING_SOFTMAX
    assert L.load().mr_k3_moe_validate(C.byref(b), buf, 256) == L.MR_ERR_INVALID_ARGUMENT
