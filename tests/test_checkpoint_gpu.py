"""A layer loaded from a sharded safetensors checkpoint runs bit-identically
to the layer it was written from: the loader moves the stored bits to the
device unchanged (U32 codes, BF16 scales and biases viewed), through pinned
staging, with one projection's biases in another shard."""
import json

import numpy as np
import pytest
import torch

import minirun_moe as M
from minirun_moe import checkpoint as CK
from minirun_moe import synth as S

pytestmark = pytest.mark.gpu
PFX = "model.layers.3.mlp"


def _np(t):
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy().view(np.uint32)


def test_checkpoint_layer_matches_source_layer(tmp_path):
    spec = S.CONFIGS[0]
    lay = S.synth_layer(spec, layer=3, device=0)
    t1, t2 = {}, {}
    for proj, w in (("gate_proj", lay.gate), ("up_proj", lay.up), ("down_proj", lay.down)):
        base = f"{PFX}.switch_mlp.{proj}"
        t1[f"{base}.weight"] = ("U32", _np(w.packed))
        t1[f"{base}.scales"] = ("BF16", _np(w.scales))
        (t2 if proj == "down_proj" else t1)[f"{base}.biases"] = ("BF16", _np(w.biases))
    for proj, w in zip(("gate_proj", "up_proj", "down_proj"), lay.shared):
        for part, t in (("weight", w.packed), ("scales", w.scales), ("biases", w.biases)):
            t2[f"{PFX}.shared_expert.{proj}.{part}"] = ("U32" if part == "weight" else "BF16",
                                                         _np(t))
    t2[f"{PFX}.gate.weight"] = ("BF16", _np(lay.router_w))
    CK.write_safetensors(str(tmp_path / "a.safetensors"), t1)
    CK.write_safetensors(str(tmp_path / "b.safetensors"), t2)
    wm = {n: "a.safetensors" for n in t1}
    wm.update({n: "b.safetensors" for n in t2})
    json.dump({"weight_map": wm}, open(tmp_path / "model.safetensors.index.json", "w"))

    ck = M.Checkpoint(str(tmp_path))
    dev = torch.device("cuda", 0)
    gate, up, down = (ck.affine(f"{PFX}.switch_mlp.{p}", spec.group, spec.bits, stacked=True,
                                device=dev) for p in ("gate_proj", "up_proj", "down_proj"))
    shared = tuple(ck.affine(f"{PFX}.shared_expert.{p}", spec.group, spec.bits, device=dev)
                   for p in ("gate_proj", "up_proj", "down_proj"))
    router_w = ck.tensor(f"{PFX}.gate.weight", device=dev)
    loaded = M.MoELayer(router_w, gate, up, down, lay.router, shared, lay.swiglu_limit,
                        lay.weight_placement)
    for T in (1, 4, 16):
        x = S.synth_x(spec, T, layer=3, batch=T, device=0)
        a, ia = lay(x)
        b, ib = loaded(x)
        assert torch.equal(a, b) and torch.equal(ia.ids, ib.ids)
        assert torch.equal(ia.weights, ib.weights)
    torch.cuda.synchronize()
