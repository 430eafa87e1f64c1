"""Safetensors checkpoints on the CPU: a sharded checkpoint of the oracle's
config-0 layer whose down_proj biases sit in a different shard from its codes
(as in the reference's checkpoint, QwenCheckpoint.swift:100-106), loaded as
AffineWeights with the stored bits unchanged, and the header refusals of the
reference's reader (SafetensorsFile.swift:44-140)."""
import json

import numpy as np
import pytest
import torch

import minirun_moe as M
from minirun_moe import checkpoint as CK
from oracle import oracle as O

BASE = "model.layers.0.mlp.switch_mlp"


def _write_sharded(d):
    cfg = O.CONFIGS[0]
    lay = O.gen_layer(cfg)
    t1, t2 = {}, {}
    for proj, w in (("gate_proj", lay.gate), ("up_proj", lay.up), ("down_proj", lay.down)):
        t1[f"{BASE}.{proj}.weight"] = ("U32", w.packed)
        t1[f"{BASE}.{proj}.scales"] = ("BF16", w.scales)
        (t2 if proj == "down_proj" else t1)[f"{BASE}.{proj}.biases"] = ("BF16", w.biases)
    t2["model.layers.0.mlp.gate.weight"] = ("BF16", lay.router_w)
    CK.write_safetensors(str(d / "model-00001-of-00002.safetensors"), t1, {"format": "mlx"})
    CK.write_safetensors(str(d / "model-00002-of-00002.safetensors"), t2)
    wm = {n: "model-00001-of-00002.safetensors" for n in t1}
    wm.update({n: "model-00002-of-00002.safetensors" for n in t2})
    json.dump({"weight_map": wm}, open(d / "model.safetensors.index.json", "w"))
    return cfg, lay


def test_sharded_affine_tensors_load_bit_exact(tmp_path):
    cfg, lay = _write_sharded(tmp_path)
    ck = M.Checkpoint(str(tmp_path))
    assert ck.info(f"{BASE}.down_proj.biases").dtype == "BF16"
    for proj, w in (("gate_proj", lay.gate), ("up_proj", lay.up), ("down_proj", lay.down)):
        aw = ck.affine(f"{BASE}.{proj}", 64, 4, stacked=True)
        assert aw.experts == cfg.experts and aw.bits == 4
        assert aw.scales.dtype == torch.bfloat16  # viewed, not converted
        assert np.array_equal(aw.packed.numpy().view(np.uint32), w.packed)
        assert np.array_equal(aw.scales.view(torch.int16).numpy().view(np.uint16), w.scales)
        assert np.array_equal(aw.biases.view(torch.int16).numpy().view(np.uint16), w.biases)
    r = ck.tensor("model.layers.0.mlp.gate.weight")
    assert r.dtype == torch.bfloat16
    assert np.array_equal(r.view(torch.int16).numpy().view(np.uint16), lay.router_w)
    f = M.SafetensorsFile(str(tmp_path / "model-00001-of-00002.safetensors"))
    assert f.metadata == {"format": "mlx"}


def test_affine_refusals(tmp_path):
    _write_sharded(tmp_path)
    ck = M.Checkpoint(str(tmp_path))
    with pytest.raises(M.SafetensorsError, match="rank"):
        ck.affine(f"{BASE}.gate_proj", 64, 4, stacked=False)
    with pytest.raises(M.SafetensorsError, match="missing tensor"):
        ck.affine("model.layers.9.mlp.switch_mlp.gate_proj", 64, 4, stacked=True)
    a = np.zeros((2, 4, 4), np.uint16)
    CK.write_safetensors(str(tmp_path / "mix.safetensors"),
                         {"x.weight": ("U32", np.zeros((2, 4, 1), np.uint32)),
                          "x.scales": ("BF16", a), "x.biases": ("F16", a)})
    CK.write_safetensors(str(tmp_path / "i32.safetensors"),
                         {"y.weight": ("I32", np.zeros((2, 4, 1), np.int32)),
                          "y.scales": ("BF16", a), "y.biases": ("BF16", a)})
    for name, f in (("x", "mix"), ("y", "i32")):
        ck.weight_map.update({f"{name}.{p}": f"{f}.safetensors"
                              for p in ("weight", "scales", "biases")})
    with pytest.raises(M.SafetensorsError, match="scales are BF16 but biases are F16"):
        ck.affine("x", 64, 4, stacked=True)
    with pytest.raises(M.SafetensorsError, match="not U32"):
        ck.affine("y", 64, 4, stacked=True)


def _raw(path, header: dict, payload: bytes, hlen=None):
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write((len(h) if hlen is None else hlen).to_bytes(8, "little"))
        f.write(h)
        f.write(payload)


@pytest.mark.parametrize("header,payload,hlen,needle", [
    ({"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}}, b"\0" * 8, 1 << 40,
     "header claims"),
    ({"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 16]}}, b"\0" * 8, None,
     "payload is 8 bytes"),
    ({"a": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]}}, b"\0" * 8, None,
     "needs 12"),
    ({"a": {"dtype": "F8_E4M3", "shape": [8], "data_offsets": [0, 8]}}, b"\0" * 8, None,
     "unsupported dtype"),
    ({"a": {"dtype": "F32", "shape": [True], "data_offsets": [0, 4]}}, b"\0" * 4, None,
     "nonnegative integer"),
    ({"a": {"dtype": "F32", "shape": [-1], "data_offsets": [0, 4]}}, b"\0" * 4, None,
     "nonnegative integer"),
    ({"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},
      "b": {"dtype": "F32", "shape": [2], "data_offsets": [4, 12]}}, b"\0" * 12, None,
     "overlaps"),
    ({"a": {"dtype": "F32", "shape": [2]}}, b"\0" * 8, None, "well-formed"),
    ([1, 2], b"", None, "JSON object"),
])
def test_header_refusals(tmp_path, header, payload, hlen, needle):
    p = tmp_path / "bad.safetensors"
    _raw(p, header, payload, hlen)
    with pytest.raises(M.SafetensorsError, match=needle):
        M.SafetensorsFile(str(p))
    p.write_bytes(b"\x01\x02")
    with pytest.raises(M.SafetensorsError, match="shorter than the 8-byte"):
        M.SafetensorsFile(str(p))
