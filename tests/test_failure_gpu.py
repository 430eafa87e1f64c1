"""Failure path of a bounded device wait, on one GPU, without a fault or hang.

The fused expert-parallel path ends with a home-rank kernel that waits for
every rank's step epoch with a bounded poll (ep_wait_combine_kernel). Here it
runs against a flag that nothing publishes, through the C-ABI test hook
mr_test_expire_ep_wait, with a short poll limit: the wait must expire, the
device error word must carry MR_DEVERR_TIMEOUT (read by mr_ctx_check), the
output must be zeros rather than stale values, and the context must stay
usable for ordinary work afterwards.
"""
import ctypes as C
import time

import pytest
import torch

import minirun_moe as M
from minirun_moe import _lib as L
from minirun_moe import synth as S

pytestmark = pytest.mark.gpu

MR_DEVERR_TIMEOUT = 0x8


def _expire(ctx, T, H, limit, out):
    st = L.load().mr_test_expire_ep_wait(ctx.handle, T, H, limit, C.c_void_p(out.data_ptr()),
                                         C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, L.load().mr_last_error(ctx.handle).decode()


def test_expired_wait_reports_timeout_and_writes_zeros():
    dev = torch.device("cuda", 0)
    ctx = M.Context.get(0)
    ctx.sync_check()
    T, H = 3, 7168
    out = torch.full((T, H), 1.5, dtype=torch.bfloat16, device=dev)  # stale values
    t0 = time.perf_counter()
    _expire(ctx, T, H, 2000, out)
    bits = C.c_uint32(0)
    st = L.load().mr_ctx_check(ctx.handle, C.c_void_p(torch.cuda.current_stream().cuda_stream),
                               C.byref(bits))
    dt = time.perf_counter() - t0
    assert st == 5  # MR_ERR_DEVICE
    assert bits.value & MR_DEVERR_TIMEOUT
    assert "bounded device wait expired" in L.load().mr_last_error(ctx.handle).decode()
    assert dt < 10.0  # 2000 polls of ~128 ns, not a hang
    assert torch.count_nonzero(out).item() == 0
    # the word was cleared by the check; the context still runs a layer
    assert ctx.sync_check() == 0
    layer = S.synth_layer(S.CONFIGS[0])
    y, sel = layer(S.synth_x(S.CONFIGS[0], 4))
    ctx.sync_check()
    assert torch.isfinite(y.float()).all()


def test_expired_wait_through_python_raises():
    ctx = M.Context.get(0)
    out = torch.empty((1, 512), dtype=torch.bfloat16, device="cuda:0")
    _expire(ctx, 1, 512, 64, out)
    with pytest.raises(M.MoeError, match="bounded device wait expired"):
        ctx.sync_check()
    assert ctx.sync_check() == 0


def test_spin_limit_is_validated():
    ctx = M.Context.get(0)
    out = torch.empty((1, 64), dtype=torch.bfloat16, device="cuda:0")
    lib = L.load()
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.mr_test_expire_ep_wait(ctx.handle, 1, 64, 0, C.c_void_p(out.data_ptr()), s) == 1
    assert lib.mr_test_expire_ep_wait(ctx.handle, 1, 64, (1 << 22) + 1,
                                      C.c_void_p(out.data_ptr()), s) == 1


def test_ep_init_and_mode_validate_arguments():
    """mr_ep_init refuses a missing communicator or an impossible rank before
    touching NCCL; mr_ep_set_mode refuses unknown modes."""
    ctx = M.Context.get(0)
    lib = L.load()
    h = C.c_void_p()
    assert lib.mr_ep_init(ctx.handle, None, 0, 2, C.byref(h)) == 1
    assert lib.mr_ep_init(ctx.handle, C.c_void_p(8), 2, 2, C.byref(h)) == 1
    assert lib.mr_ep_set_mode(None, 0) == 1
