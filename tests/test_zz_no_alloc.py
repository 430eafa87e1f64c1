"""mr_affine_gather_mm_noalloc: the gather entry point that allocates nothing.

Collected last (file name) so that it also runs after every other test has
used the library; it must pass alone in a fresh process as well. The GPU test
calls the C ABI directly and compares with mr_affine_gather_mm, the existing
entry point, within the gather tests' tolerance, on two calls in a row with
different inputs (the scratch keeps the previous call's contents).
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from minirun_moe import _lib as L

REL_L2 = 2e-3  # the gather parity tests' bound
SCRATCH = 8 * 1024 * 1024  # MR_NOALLOC_SCRATCH_BYTES


def _desc(packed, scales, biases, experts, out, inn, bits):
    return L.mr_affine_desc(packed, scales, biases, experts, out, inn, 64, bits, 0)


def test_noalloc_rejects_sizes_beyond_scratch():
    """Host-side size check: refused before any device call, with the size."""
    lib = L.load()
    inn = 7168
    T = SCRATCH // (inn * 2) + 1  # permuted x alone exceeds the scratch
    d = _desc(16, 16, 16, 4, 2048, inn, 4)  # fake non-NULL pointers, never dereferenced
    msg = C.create_string_buffer(512)
    st = lib.mr_affine_gather_mm_noalloc(C.c_void_p(256), T, C.c_void_p(512), 8, C.byref(d),
                                         C.c_void_p(1024), None, msg, len(msg))
    assert st == 2  # MR_ERR_UNSUPPORTED
    text = msg.value.decode()
    assert "scratch" in text and str(SCRATCH) in text


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [4, 2, 8])
def test_noalloc_matches_gather_twice(bits):
    import torch
    import minirun_moe as M

    dev = torch.device("cuda", 0)
    E, out, inn = 8, 320, 1024
    w = O._stack([O.gen_affine(61, 0, e, 2, out, inn, bits, 64) for e in range(E)])
    packed = torch.from_numpy(np.ascontiguousarray(w.packed).view(np.int32)).to(dev)
    s = torch.from_numpy(np.ascontiguousarray(w.scales).view(np.int16)).view(torch.bfloat16).to(dev)
    b = torch.from_numpy(np.ascontiguousarray(w.biases).view(np.int16)).view(torch.bfloat16).to(dev)
    aw = M.AffineWeights(packed, s, b, 64, bits)
    d = aw.desc()
    lib = L.load()
    stream = torch.cuda.current_stream()

    def inputs(T, k, seed):
        x = O.gen_normal_bf16(seed, T * inn, 1.0).reshape(T, inn)
        ids = np.random.default_rng(seed).integers(0, E, size=(T, k)).astype(np.int32)
        xt = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).to(dev)
        return xt, torch.from_numpy(ids).to(dev), x, ids

    # two calls in a row: a larger one, then a smaller one that finds the
    # first call's plan and activations still in the scratch
    cases = [(37, 4, 11), (5, 3, 12)]
    got, want, exact = [], [], []
    for T, k, seed in cases:
        x, ids, xn, idn = inputs(T, k, seed)
        exact.append(O.affine_gather_mm(xn, w, idn)[1])  # the oracle's exact fp32 result
        y = torch.full((T, k, out), float("nan"), dtype=torch.bfloat16, device=dev)
        msg = C.create_string_buffer(512)
        st = lib.mr_affine_gather_mm_noalloc(C.c_void_p(x.data_ptr()), T,
                                             C.c_void_p(ids.data_ptr()), k, C.byref(d),
                                             C.c_void_p(y.data_ptr()),
                                             C.c_void_p(stream.cuda_stream), msg, len(msg))
        assert st == 0, msg.value.decode()
        got.append(y)
        want.append(M.affine_gather_mm(x, aw, ids))
    torch.cuda.synchronize()
    for g, r, e in zip(got, want, exact):
        g = g.float().cpu().numpy()
        r = r.float().cpu().numpy()
        assert np.isfinite(g).all()
        # against the CPU oracle directly, and against the existing entry point
        err = np.linalg.norm(g - e) / max(np.linalg.norm(e), 1e-30)
        assert err < REL_L2, err
        err = np.linalg.norm(g - r) / max(np.linalg.norm(r), 1e-30)
        assert err < REL_L2, err

    # later calls allocate nothing: device free memory is unchanged by them
    x, ids, _, _ = inputs(*cases[0])
    y = torch.empty((cases[0][0], cases[0][1], out), dtype=torch.bfloat16, device=dev)
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(dev)
    for _ in range(3):
        st = lib.mr_affine_gather_mm_noalloc(C.c_void_p(x.data_ptr()), cases[0][0],
                                             C.c_void_p(ids.data_ptr()), cases[0][1], C.byref(d),
                                             C.c_void_p(y.data_ptr()),
                                             C.c_void_p(stream.cuda_stream), None, 0)
        assert st == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(dev)
    assert free1 == free0


@pytest.mark.gpu
def test_noalloc_bad_id_leaves_its_rows_and_computes_the_rest():
    """An id outside [0, experts) cannot be reported (the entry point has no
    context to read an error word from): its output rows are left as they
    were, every other (token, slot) row is computed, and nothing faults."""
    import torch
    import minirun_moe as M

    dev = torch.device("cuda", 0)
    E, out, inn, T, k = 4, 192, 512, 3, 2
    w = O._stack([O.gen_affine(67, 0, e, 2, out, inn, 4, 64) for e in range(E)])
    packed = torch.from_numpy(np.ascontiguousarray(w.packed).view(np.int32)).to(dev)
    s = torch.from_numpy(np.ascontiguousarray(w.scales).view(np.int16)).view(torch.bfloat16).to(dev)
    b = torch.from_numpy(np.ascontiguousarray(w.biases).view(np.int16)).view(torch.bfloat16).to(dev)
    d = M.AffineWeights(packed, s, b, 64, 4).desc()
    xn = O.gen_normal_bf16(3, T * inn, 1.0).reshape(T, inn)
    idn = np.array([[0, 3], [E, 1], [2, -1]], np.int32)
    x = torch.from_numpy(xn.view(np.int16)).view(torch.bfloat16).to(dev)
    ids = torch.from_numpy(idn).to(dev)
    y = torch.full((T, k, out), float("nan"), dtype=torch.bfloat16, device=dev)
    lib = L.load()
    st = lib.mr_affine_gather_mm_noalloc(C.c_void_p(x.data_ptr()), T, C.c_void_p(ids.data_ptr()),
                                         k, C.byref(d), C.c_void_p(y.data_ptr()),
                                         C.c_void_p(torch.cuda.current_stream().cuda_stream),
                                         None, 0)
    assert st == 0
    torch.cuda.synchronize()
    g = y.float().cpu().numpy()
    good = [(0, 0), (0, 1), (1, 1), (2, 0)]
    ok_ids = np.where((idn >= 0) & (idn < E), idn, 0)
    ref = O.affine_gather_mm(xn, w, ok_ids.astype(np.int32))[1]
    for t, j in good:
        e = np.linalg.norm(g[t, j] - ref[t, j]) / np.linalg.norm(ref[t, j])
        assert e < REL_L2, (t, j, e)
    assert np.isnan(g[1, 0]).all() and np.isnan(g[2, 1]).all()
