"""HBM expert cache (mr_moe_layer_forward_cached) on config-0 layers.

Config 4's contract: outputs are byte-identical whatever the budget. Three
seeded layers run a fixed sequence of calls under three budgets (everything
resident, 12 slots, 8 slots = one call's worst case); every output must be
bitwise equal across budgets and to the same layers' stacks on the same
GEMV kernel. Small budgets must miss and evict; a budget below one call's
distinct experts and an unregistered expert are refused with their status.
"""
import pytest
import torch

import minirun_moe as M
from minirun_moe import _lib as L
from minirun_moe import synth as S

pytestmark = pytest.mark.gpu
NL = 3
CALLS = [0, 1, 2, 0, 2, 1, 1, 0, 2]


def _setup():
    spec = S.CONFIGS[0]
    layers = [S.synth_layer(spec, layer=l, device=0) for l in range(NL)]
    cached = [M.CachedLayer(l.router_w, l.router, l.hidden, l.inter, spec.bits, spec.group,
                            torch.bfloat16, l.shared, l.swiglu_limit, l.weight_placement)
              for l in layers]
    xs = [S.synth_x(spec, 4, layer=c, batch=i, device=0) for i, c in enumerate(CALLS)]
    slot = M.ExpertCache.slot_bytes_for(layers[0].gate, layers[0].up, layers[0].down)
    return spec, layers, cached, xs, slot


def _run(layers, cached, xs, slot, n_slots):
    cache = M.ExpertCache(0, n_slots * slot, slot)
    try:
        for l, lay in enumerate(layers):
            cache.register_layer(l, lay.gate, lay.up, lay.down)
        outs = [cache.forward(c, cached[c], x).clone() for c, x in zip(CALLS, xs)]
        torch.cuda.synchronize()
        return outs, cache.stats()
    finally:
        cache.close()


def test_cache_outputs_byte_identical_across_budgets():
    spec, layers, cached, xs, slot = _setup()
    full, st_full = _run(layers, cached, xs, slot, NL * spec.experts)
    mid, st_mid = _run(layers, cached, xs, slot, 12)
    tiny, st_tiny = _run(layers, cached, xs, slot, 2 * 4)  # T * k distinct at most
    for a, b, c in zip(full, mid, tiny):
        assert torch.equal(a, b) and torch.equal(a, c)
    # the same layers' stacks through the same (table-capable) GEMV kernel
    ctx = M.Context.get(0)
    ctx.set_kernel_path("register")
    try:
        for c, x, o in zip(CALLS, xs, full):
            ref, _ = layers[c](x)
            assert torch.equal(ref, o)
    finally:
        ctx.set_kernel_path("auto")
    assert st_full["evictions"] == 0 and st_full["misses"] <= NL * spec.experts
    assert st_tiny["evictions"] > 0 and st_tiny["misses"] > st_full["misses"]
    assert st_tiny["bytes_copied"] > st_full["bytes_copied"]
    assert st_tiny["resident"] <= 8 and st_tiny["slots"] == 8
    ctx.sync_check()


def test_cache_refuses_small_budget_and_unknown_experts():
    spec, layers, cached, xs, slot = _setup()
    cache = M.ExpertCache(0, 1 * slot, slot)
    try:
        cache.register_layer(0, layers[0].gate, layers[0].up, layers[0].down)
        with pytest.raises(M.MoeError) as e:
            cache.forward(0, cached[0], xs[0])
        assert e.value.status == L.MR_ERR_BUDGET
    finally:
        cache.close()
    cache = M.ExpertCache(0, 64 * slot, slot)
    try:
        cache.register_layer(0, layers[0].gate, layers[0].up, layers[0].down)
        with pytest.raises(M.MoeError) as e:
            cache.forward(1, cached[1], xs[1])
        assert e.value.status == L.MR_ERR_STATE
    finally:
        cache.close()
    torch.cuda.synchronize()
