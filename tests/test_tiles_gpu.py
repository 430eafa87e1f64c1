"""Routed experts streamed from MNRNTIL1 containers through the HBM cache.

Three seeded config-0 layers are written as expert containers (one per layer
and projection, one expert per tile, SHA-256 per tile), registered with an
ExpertCache by tile, and run through a fixed sequence of calls under three
budgets. Every output must be bitwise equal to the same layers' resident
stacks on the same (table-driven) GEMV kernel — the bytes took a different
road (file -> pinned staging -> slot) but are the same bytes — and small
budgets must miss, evict and re-read.
"""
import pytest
import torch

import minirun_moe as M
from minirun_moe import synth as S
from minirun_moe import tiles as TL

pytestmark = pytest.mark.gpu
NL = 3
CALLS = [0, 1, 2, 0, 2, 1, 1, 0, 2]


def _proj(w):
    return (w.packed, w.scales, w.biases, w.bits)


def test_expert_containers_feed_the_cache(tmp_path):
    spec = S.CONFIGS[0]
    layers = [S.synth_layer(spec, layer=l, device=0) for l in range(NL)]
    TL.write_expert_containers(str(tmp_path), {l: (_proj(lay.gate), _proj(lay.up),
                                                   _proj(lay.down))
                                               for l, lay in enumerate(layers)})
    cached = [M.CachedLayer(l.router_w, l.router, l.hidden, l.inter, spec.bits, spec.group,
                            torch.bfloat16, l.shared, l.swiglu_limit, l.weight_placement)
              for l in layers]
    xs = [S.synth_x(spec, 4, layer=c, batch=i, device=0) for i, c in enumerate(CALLS)]
    ec = TL.ExpertContainers(str(tmp_path))
    slot = ec.slot_bytes(0)
    assert slot == M.ExpertCache.slot_bytes_for(layers[0].gate, layers[0].up, layers[0].down)
    ctx = M.Context.get(0)
    results = []
    try:
        for n_slots in (NL * spec.experts, 12, 8):
            cache = M.ExpertCache(0, n_slots * slot, slot)
            try:
                for l in range(NL):
                    ec.register(cache, l)
                outs = [cache.forward(c, cached[c], x).clone() for c, x in zip(CALLS, xs)]
                torch.cuda.synchronize()
                results.append((outs, cache.stats()))
            finally:
                cache.close()
        ctx.set_kernel_path("register")
        try:
            refs = [layers[c](x)[0] for c, x in zip(CALLS, xs)]
        finally:
            ctx.set_kernel_path("auto")
        for outs, _ in results:
            for o, r in zip(outs, refs):
                assert torch.equal(o, r)
        full, tiny = results[0][1], results[2][1]
        assert full["evictions"] == 0 and tiny["evictions"] > 0
        assert tiny["bytes_copied"] > full["bytes_copied"] > 0
        ctx.sync_check()
    finally:
        ec.close()


def test_corrupted_tile_is_refused_on_the_miss(tmp_path):
    spec = S.CONFIGS[0]
    lay = S.synth_layer(spec, layer=0, device=0)
    TL.write_expert_containers(str(tmp_path), {0: (_proj(lay.gate), _proj(lay.up),
                                                   _proj(lay.down))})
    # flip one byte of every tile of the gate container (experts' codes)
    path = tmp_path / "layer000.w1.mnrntil"
    with TL.TileContainer(str(path)) as c:
        layout = c.layout
    with open(path, "r+b") as f:
        for t in range(layout.tile_count):
            f.seek(layout.first_tile_offset + t * layout.tile_stride + 100)
            b = f.read(1)
            f.seek(-1, 1)
            f.write(bytes([b[0] ^ 0x5A]))
    ec = TL.ExpertContainers(str(tmp_path))
    cached = M.CachedLayer(lay.router_w, lay.router, lay.hidden, lay.inter, spec.bits,
                           spec.group, torch.bfloat16, lay.shared, lay.swiglu_limit,
                           lay.weight_placement)
    slot = ec.slot_bytes(0)
    cache = M.ExpertCache(0, spec.experts * slot, slot)
    try:
        ec.register(cache, 0)
        with pytest.raises(M.MoeError) as e:
            cache.forward(0, cached, S.synth_x(spec, 4, layer=0, batch=0, device=0))
        assert "SHA-256" in str(e.value)
    finally:
        cache.close()
        ec.close()
    torch.cuda.synchronize()
