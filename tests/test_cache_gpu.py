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


def _routed(layer, x):
    _, sel = layer(x)
    return sorted(set(sel.ids.view(-1).tolist()))


def test_cache_policies_keep_outputs_and_follow_admission():
    """The three admission policies (BufferPool.swift CachePolicy) give the
    same bytes as LRU; NONE copies every routed expert on every call;
    PINNED_HOT_SET keeps its hot experts resident however many cold ones
    pass through, and admits nothing else."""
    spec, layers, cached, xs, slot = _setup()
    ref, _ = _run(layers, cached, xs, slot, NL * spec.experts)
    hot = [(0, e) for e in _routed(layers[0], xs[0])]
    for policy in ("none", "pinned_hot_set"):
        # the hot set plus one call's working set (T * k = 8 experts)
        cache = M.ExpertCache(0, (len(hot) + 8) * slot, slot)
        try:
            cache.set_policy(policy, hot if policy == "pinned_hot_set" else None)
            for l, lay in enumerate(layers):
                cache.register_layer(l, lay.gate, lay.up, lay.down)
            outs = []
            for c, x in zip(CALLS, xs):
                outs.append(cache.forward(c, cached[c], x).clone())
            torch.cuda.synchronize()
            st = cache.stats()
            for a, b in zip(ref, outs):
                assert torch.equal(a, b)
            n_routed = sum(len(_routed(layers[c], x)) for c, x in zip(CALLS, xs))
            if policy == "none":
                assert st["hits"] == 0 and st["misses"] == n_routed
            else:
                # every later call of layer 0 on the first call's experts hits
                first0 = [i for i, c in enumerate(CALLS) if c == 0]
                later = sum(len(set(_routed(layers[0], xs[i])) & {e for _, e in hot})
                            for i in first0[1:])
                assert st["hits"] >= later
                assert st["resident"] <= len(hot) + 8  # cold ones go back to free
        finally:
            cache.close()
    M.Context.get(0).sync_check()


def test_cache_prefetch_turns_misses_into_hits():
    """RoutedExpertBackend.prefetch: experts prefetched before a call are
    resident when it runs (hits, no new copies), and the outputs are the
    same bytes as without prefetch."""
    spec, layers, cached, xs, slot = _setup()
    ref, _ = _run(layers, cached, xs, slot, NL * spec.experts)
    cache = M.ExpertCache(0, NL * spec.experts * slot, slot)
    try:
        for l, lay in enumerate(layers):
            cache.register_layer(l, lay.gate, lay.up, lay.down)
        outs = []
        for c, x in zip(CALLS, xs):
            cache.prefetch(c, _routed(layers[c], x))
            before = cache.stats()
            outs.append(cache.forward(c, cached[c], x).clone())
            after = cache.stats()
            assert after["misses"] == before["misses"]  # all resident already
        torch.cuda.synchronize()
        st = cache.stats()
        assert st["prefetched"] > 0 and st["misses"] == 0
        for a, b in zip(ref, outs):
            assert torch.equal(a, b)
        with pytest.raises(M.MoeError):
            cache.prefetch(NL + 5, [0])  # unregistered
    finally:
        cache.close()
    M.Context.get(0).sync_check()
