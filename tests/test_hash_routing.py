"""Token-hash routing (DeepSeek V4's first layers,
Operators/DeepSeekV4Routing.swift:4-64, :231-256). CPU: the table checks of
DeepSeekV4TokenExpertMap.init, in the reference's order. GPU (marked): the
hashed layer against the numpy restatement — ids exactly the table rows,
weights the renormalised scores at them, outputs within the layer
tolerance — and an out-of-range token id reported through the error word."""
import ctypes as C
import dataclasses

import numpy as np
import pytest
import torch

import minirun_moe as M
from minirun_moe import _lib as L
import np_ref as R
from oracle import oracle as O


def _validate(table, experts):
    t = np.ascontiguousarray(table, np.int32)
    buf = C.create_string_buffer(256)
    st = L.load().mr_token_map_validate(t.ctypes.data, t.shape[0], t.shape[1], experts, buf, 256)
    return st, buf.value.decode()


def test_token_map_checks_in_reference_order():
    ok = np.array([[0, 1], [3, 2], [1, 0]])
    assert _validate(ok, 4) == (L.MR_OK, "")
    st, msg = _validate(np.array([[0, 1], [2, 7]]), 4)
    assert st == L.MR_ERR_INVALID_ARGUMENT and msg == "token 1 slot 1 names expert 7, outside 0..<4"
    st, msg = _validate(np.array([[0, 1], [2, 2]]), 4)
    assert msg == "token 1 names expert 2 more than once"
    # slot 1's range check precedes slot 2's duplicate check
    st, msg = _validate(np.array([[1, -1, 1]]), 4)
    assert msg == "token 0 slot 1 names expert -1, outside 0..<4"
    st, msg = _validate(np.array([[1, 1, -1]]), 4)
    assert msg == "token 0 names expert 1 more than once"
    with pytest.raises(M.AffineBridgeError, match="more than once"):
        M.TokenExpertMap(np.array([[3, 3]]), 4)


def _table(vocab, k, E, seed=5):
    rng = np.random.default_rng(seed)
    return np.stack([rng.permutation(E)[:k] for _ in range(vocab)]).astype(np.int32)


@pytest.mark.gpu
@pytest.mark.parametrize("variant", [dict(scoring="sqrt_softplus", renorm="plain",
                                          routed_scale=1.5),
                                     dict(scoring="sigmoid", renorm="eps")])
def test_hashed_layer_matches_reference(variant):
    cfg = dataclasses.replace(O.CONFIGS[0], **variant)
    Lw = O.gen_layer(cfg)
    vocab = 50
    table = _table(vocab, cfg.top_k, cfg.experts)
    tok = np.array([3, 49, 0, 17, 17, 8, 22, 31, 5], np.int64)
    x = O.gen_x(cfg, len(tok), batch=4)
    out, f, ids, w, _ = R.layer(Lw, x, hashed=(table, tok))
    from test_gpu_parity import gpu_layer_from_oracle, t_u16, n_u16, rel_l2
    layer = gpu_layer_from_oracle(Lw)
    tmap = M.TokenExpertMap(table, cfg.experts)
    tids = torch.from_numpy(tok.astype(np.int32)).cuda()
    gout, sel = layer.forward_hashed(t_u16(x), tids, tmap)
    assert np.array_equal(sel.ids.cpu().numpy(), table[tok])
    np.testing.assert_allclose(sel.weights.cpu().numpy(), w, rtol=1e-5, atol=1e-7)
    assert rel_l2(O.bf16_to_f32(n_u16(gout)), f) < 5e-3
    rs = M.router_select_hashed(t_u16(x), layer.router_w, layer.router, tids, tmap)
    assert torch.equal(rs.ids, sel.ids) and torch.equal(rs.weights, sel.weights)
    M.Context.get(0).sync_check()


@pytest.mark.gpu
def test_out_of_range_token_id_sets_the_error_word():
    cfg = dataclasses.replace(O.CONFIGS[0], scoring="sqrt_softplus", renorm="plain")
    Lw = O.gen_layer(cfg)
    from test_gpu_parity import gpu_layer_from_oracle, t_u16
    layer = gpu_layer_from_oracle(Lw)
    tmap = M.TokenExpertMap(_table(10, cfg.top_k, cfg.experts), cfg.experts)
    x = O.gen_x(cfg, 3, batch=1)
    ctx = M.Context.get(0)
    layer.forward_hashed(t_u16(x), torch.tensor([1, 10, 2], dtype=torch.int32).cuda(), tmap)
    with pytest.raises(M.MoeError) as e:
        ctx.sync_check()
    assert e.value.status == L.MR_ERR_DEVICE
