"""The expert-parallel decomposition on CPU with 2 gloo ranks.

mr_moe_layer_forward_ep splits one MoE layer over ranks: all-gather the
ranks' tokens, route all of them, evaluate only the pairs whose expert lies in
this rank's range [r*E/N, (r+1)*E/N), sum them per token in slot order,
reduce-scatter the sums to the tokens' home ranks, then add the shared expert
and round there. This test runs exactly that sequence with torch.distributed
(gloo) collectives and the numpy restatement of the layer as the arithmetic,
and checks it against the one-process layer: the split loses nothing and
changes only the fp32 order of the routed-slot sums.
"""
import dataclasses
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_forward(L, x_own, rank, world):
    """One rank's part of the expert-parallel forward (numpy arithmetic)."""
    import np_ref as R
    c = L.cfg
    T = x_own.shape[0]
    # 1. all ranks' tokens, in rank order
    # (bf16 bit patterns travel as int32 pairs: gloo has no 16-bit integers)
    parts = [torch.empty((T, c.hidden // 2), dtype=torch.int32) for _ in range(world)]
    dist.all_gather(parts, torch.from_numpy(np.ascontiguousarray(x_own).view(np.int32)))
    x_all = torch.cat(parts).numpy().view(np.uint16)
    # 2. router over all tokens (identical on every rank)
    x64 = R.bf16_to_f32(x_all).astype(np.float64)
    logits = (x64 @ R.bf16_to_f32(L.router_w).astype(np.float64).T).astype(np.float32)
    ids, w, _ = R.router(logits, c.top_k, c.scoring, L.correction_bias, c.renorm,
                         c.renorm_eps, c.routed_scale)
    # 3. this rank's experts over the pairs routed to them
    E = c.experts
    lo, hi = rank * E // world, (rank + 1) * E // world
    local = (ids >= lo) & (ids < hi)
    NT, k = ids.shape
    gb, _ = R.gather_mm(x_all, L.gate, ids)
    ub, _ = R.gather_mm(x_all, L.up, ids)
    g, u = R.bf16_to_f32(gb), R.bf16_to_f32(ub)
    if not c.weight_after_down:
        a = ((g * R.sigmoid32(g)).astype(np.float32) * u).astype(np.float32)
        h = R.f32_to_bf16((a * w[:, :, None]).astype(np.float32))
    else:
        h = R.f32_to_bf16(R.bf16r(g * R.bf16r(R.sigmoid32(g))) * u)
    db, _ = R.gather_mm(h.reshape(NT * k, -1), L.down, ids.reshape(NT * k, 1))
    d = R.bf16_to_f32(db).reshape(NT, k, -1)
    # 4. per-token sum of the local slots, slot order
    part = np.zeros((NT, c.hidden), np.float32)
    for j in range(k):
        v = d[:, j] * w[:, j:j + 1] if c.weight_after_down else d[:, j]
        part = (part + np.where(local[:, j:j + 1], v, 0)).astype(np.float32)
    # 5. reduce-scatter: every token's sum over ranks, on its home rank
    t = torch.from_numpy(part)
    dist.all_reduce(t)
    acc = t.numpy()[rank * T:(rank + 1) * T].copy()
    # 6. home rank: rounding of the routed sum, shared expert, output
    if not c.weight_after_down:
        acc = R.bf16r(acc)
    if L.sgate is not None:
        xs = x64[rank * T:(rank + 1) * T]
        sgw = R.dequant64(L.sgate.packed, L.sgate.scales, L.sgate.biases, L.sgate.bits, 64)
        suw = R.dequant64(L.sup.packed, L.sup.scales, L.sup.biases, L.sup.bits, 64)
        sdw = R.dequant64(L.sdown.packed, L.sdown.scales, L.sdown.biases, L.sdown.bits, 64)
        sg = R.bf16r((xs @ sgw.T).astype(np.float32))
        su = R.bf16r((xs @ suw.T).astype(np.float32))
        sa = ((sg * R.sigmoid32(sg)).astype(np.float32) * su).astype(np.float32)
        acc = (acc + (sa.astype(np.float64) @ sdw.T).astype(np.float32)).astype(np.float32)
    return acc, ids[rank * T:(rank + 1) * T]


def _worker(rank, world, port, variant, queue):
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.dirname(HERE))
    from oracle import oracle as O
    import np_ref as R
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = dataclasses.replace(O.CONFIGS[0], **variant)
        L = O.gen_layer(cfg)
        if cfg.shared_inter == 0:
            L.sgate = L.sup = L.sdown = None
        T = 3
        x_all = O.gen_x(cfg, T * world, batch=11)
        acc, ids = _rank_forward(L, x_all[rank * T:(rank + 1) * T], rank, world)
        _, ref, ref_ids, _, _ = R.layer(L, x_all)
        ref = ref[rank * T:(rank + 1) * T]
        err = float(np.linalg.norm(acc - ref) / max(np.linalg.norm(ref), 1e-30))
        queue.put((rank, err, bool(np.array_equal(ids, ref_ids[rank * T:(rank + 1) * T]))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("variant", [{}, {"weight_after_down": True}, {"shared_inter": 0}])
def test_expert_parallel_decomposition_gloo(variant):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, variant, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    got = sorted(q.get(timeout=5) for _ in range(world))
    for rank, err, ids_ok in got:
        assert ids_ok, rank
        assert err < 1e-5, (rank, err)
