"""MNRNTIL1 tile containers on the CPU: SHA-256, the layout rules, the header
reader's refusals, and a round trip of the oracle's config-0 experts through
containers and a manifest.

The layout cases are the reference's own (Tests/StorageCoreTests/
MXFP4TileContainerTests.swift:38-88: the 512 x 1024 MXFP4 geometry and the
geometries it rejects); the refusals follow its reader (QuantizedTileContainer
.swift:811-1001: bad magic, unknown version, truncation, contradictory fields,
unknown feature bits) and its digest check (:1153-1181).
"""
import hashlib
import json
import os

import numpy as np
import pytest

from minirun_moe import _lib as L
from minirun_moe import tiles as TL
from oracle import oracle as O


def test_sha256_known_answers_and_hashlib():
    assert TL.sha256(b"").hex() == ("e3b0c44298fc1c149afbf4c8996fb924"
                                    "27ae41e4649b934ca495991b7852b855")
    assert TL.sha256(b"abc").hex() == ("ba7816bf8f01cfea414140de5dae2223"
                                       "b00361a396177a9cb410ff61f20015ad")
    msg = b"abcdbcdecdefdefgefghfghighijhijkijkljklmklmnlmnomnopnopq"
    assert TL.sha256(msg).hex() == ("248d6a61d20638b8e5c026930c3e6039"
                                    "a33ce45964ff2167f6ecedd419db06c1")
    rng = np.random.default_rng(7)
    for n in list(range(0, 130)) + [1 << 20]:
        d = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        assert TL.sha256(d) == hashlib.sha256(d).digest(), n


def _mx(rows, cols, tiles, **kw):
    return TL.layout_for(rows, cols, 32, 4, tiles, quant_mode=TL.MODE_MXFP4,
                         scale_dtype=TL.SCALE_E8M0, content_kind=TL.CONTENT_SYNTHETIC, **kw)


def test_layout_matches_the_geometry():
    lay = _mx(512, 1024, 6, seed=1)
    assert lay.packed_bytes == 512 * 1024 // 2
    assert lay.scale_bytes == 512 * 1024 // 32
    assert lay.scale_offset == lay.packed_bytes
    assert lay.tile_stride == lay.packed_bytes + lay.scale_bytes
    assert lay.first_tile_offset == TL.HEADER_BYTES
    assert lay.total_bytes == TL.HEADER_BYTES + 6 * lay.tile_stride
    assert lay.version == 1 and lay.feature_flags == 0 and lay.bias_bytes == 0
    for t in range(5):
        assert (lay.first_tile_offset + t * lay.tile_stride) % TL.ALIGN == 0
    assert lay.scale_offset % TL.ALIGN == 0


@pytest.mark.parametrize("rows,cols,tiles", [(512, 1000, 1), (8, 1024, 1), (256, 1024, 1),
                                             (0, 1024, 1), (512, 1024, 0)])
def test_unsupported_geometries_are_rejected(rows, cols, tiles):
    with pytest.raises(TL.TileContainerError) as e:
        _mx(rows, cols, tiles)
    assert e.value.status == L.MR_ERR_UNSUPPORTED


def test_affine_layout_is_version_2_with_biases_and_digests():
    lay = TL.layout_for(512, 1024, 64, 4, 16, digests=True)
    assert (lay.packed_bytes, lay.scale_bytes, lay.bias_bytes) == (262144, 16384, 16384)
    assert lay.version == 2
    assert lay.feature_flags == 1 | 2  # biases, tile digests
    assert lay.bias_offset == lay.scale_offset + 16384 and lay.tile_stride == 262144 + 2 * 16384
    with pytest.raises(TL.TileContainerError):  # affine scales are floats, not e8m0
        TL.layout_for(512, 1024, 64, 4, 1, scale_dtype=TL.SCALE_E8M0)
    with pytest.raises(TL.TileContainerError):  # 16384 / 32 digests fit a header
        TL.layout_for(512, 1024, 64, 4, 600, digests=True)


def test_block_scale_layout_is_version_3_padded():
    lay = TL.layout_for(256, 1024, 128, 8, 2, quant_mode=TL.MODE_FP8_BLOCK,
                        scale_dtype=TL.SCALE_E8M0, scale_block_rows=128)
    assert lay.version == 3 and lay.scale_bytes == 2 * 8
    assert lay.feature_flags == 4 | 8  # 2-D block scales, padded sub-regions
    assert lay.scale_region_bytes == TL.ALIGN and lay.bias_bytes == 0


def _expert_layers():
    cfg = O.CONFIGS[0]
    lay = O.gen_layer(cfg)
    proj = tuple((w.packed, w.scales, w.biases, w.bits) for w in (lay.gate, lay.up, lay.down))
    return cfg, lay, {0: proj}


def test_expert_containers_round_trip(tmp_path):
    cfg, lay, layers = _expert_layers()
    TL.write_expert_containers(str(tmp_path), layers)
    man = json.load(open(tmp_path / "manifest.json"))
    assert [c["projection"] for c in man["containers"]] == ["w1", "w3", "w2"]
    ec = TL.ExpertContainers(str(tmp_path))
    try:
        assert ec.layers() == [0] and ec.experts(0) == list(range(cfg.experts))
        for slot, w in zip(TL.PROJECTION_SLOTS, (lay.gate, lay.up, lay.down)):
            cont = ec.entries[(0, slot)].container
            assert cont.layout.version == 2 and cont.layout.content_kind == TL.CONTENT_CHECKPOINT
            for e in (0, 5, cfg.experts - 1):
                pk, sc, bi = cont.sub_regions(ec.entries[(0, slot)].tile_of_expert[e])
                assert pk.tobytes() == w.packed[e].tobytes()
                assert sc.tobytes() == w.scales[e].tobytes()
                assert bi.tobytes() == w.biases[e].tobytes()
        per = 0
        for w in (lay.gate, lay.up, lay.down):
            for a in (w.packed[0], w.scales[0], w.biases[0]):
                per += (a.nbytes + 255) // 256 * 256
        assert ec.slot_bytes(0) == per
    finally:
        ec.close()


def _one_container(path, **kw):
    cfg, lay, _ = _expert_layers()
    g = lay.gate
    tiles = [(g.packed[e], g.scales[e], g.biases[e]) for e in range(2)]
    return TL.write_container(str(path), tiles, rows=g.packed.shape[1],
                              cols=g.packed.shape[2] * 8, group_size=64, bits=4, **kw)


def _patch(path, off, data):
    with open(path, "r+b") as f:
        f.seek(off)
        f.write(data)


@pytest.mark.parametrize("off,data,status,needle", [
    (0, b"XNRNTIL1", L.MR_ERR_INVALID_ARGUMENT, "bad magic"),
    (8, (4).to_bytes(4, "little"), L.MR_ERR_INVALID_ARGUMENT, "not supported"),
    (32, (1).to_bytes(8, "little"), L.MR_ERR_INVALID_ARGUMENT, "contradict"),
    (92, (0x13).to_bytes(4, "little"), L.MR_ERR_INVALID_ARGUMENT, "feature flags"),
    (124, (1).to_bytes(4, "little"), L.MR_ERR_INVALID_ARGUMENT, "reserved"),
    (80, (0).to_bytes(4, "little"), L.MR_ERR_INVALID_ARGUMENT, "biases feature flag"),
])
def test_header_refusals(tmp_path, off, data, status, needle):
    p = tmp_path / "c.mnrntil"
    _one_container(p)
    TL.TileContainer(str(p)).close()
    _patch(p, off, data)
    with pytest.raises(TL.TileContainerError) as e:
        TL.TileContainer(str(p))
    assert e.value.status == status and needle in str(e.value), str(e.value)


def test_truncated_and_missing_files(tmp_path):
    p = tmp_path / "c.mnrntil"
    lay = _one_container(p)
    size = os.path.getsize(p)
    assert size == lay.total_bytes
    with open(p, "r+b") as f:
        f.truncate(size - 1)
    with pytest.raises(TL.TileContainerError) as e:
        TL.TileContainer(str(p))
    assert e.value.status == L.MR_ERR_IO and "truncated" in str(e.value)
    with open(p, "r+b") as f:
        f.truncate(TL.HEADER_BYTES)  # header only
    with pytest.raises(TL.TileContainerError) as e:
        TL.TileContainer(str(p))
    assert e.value.status == L.MR_ERR_IO
    with open(p, "r+b") as f:
        f.truncate(100)  # shorter than the header
    with pytest.raises(TL.TileContainerError) as e:
        TL.TileContainer(str(p))
    assert e.value.status == L.MR_ERR_IO
    with pytest.raises(TL.TileContainerError) as e:
        TL.TileContainer(str(tmp_path / "absent"))
    assert e.value.status == L.MR_ERR_IO


def test_tile_digest_mismatch_is_reported(tmp_path):
    p = tmp_path / "c.mnrntil"
    lay = _one_container(p)
    with TL.TileContainer(str(p)) as c:
        c.read(0)
        c.read(1)
        with pytest.raises(TL.TileContainerError) as e:
            c.read(2)
        assert e.value.status == L.MR_ERR_INVALID_ARGUMENT
    _patch(p, lay.first_tile_offset + lay.tile_stride + 12345, b"\xff")
    with TL.TileContainer(str(p)) as c:
        c.read(0)
        with pytest.raises(TL.TileContainerError) as e:
            c.read(1)
        assert e.value.status == L.MR_ERR_INTEGRITY
    with TL.TileContainer(str(p), verify=False) as c:
        assert c.read(1)[12345] == 0xff


def test_version_1_mxfp4_container_round_trip(tmp_path):
    p = tmp_path / "v1.mnrntil"
    rng = np.random.default_rng(3)
    tiles = [(rng.integers(0, 256, 262144, dtype=np.uint8), rng.integers(100, 141, 16384,
                                                                        dtype=np.uint8), None)
             for _ in range(2)]
    lay = TL.write_container(str(p), tiles, rows=512, cols=1024, group_size=32, bits=4,
                             quant_mode=TL.MODE_MXFP4, scale_dtype=TL.SCALE_E8M0,
                             content_kind=TL.CONTENT_SYNTHETIC, seed=9, digests=False)
    assert lay.version == 1
    with TL.TileContainer(str(p)) as c:
        assert c.layout.version == 1 and c.layout.seed == 9
        pk, sc, bi = c.sub_regions(1)
        assert pk.tobytes() == tiles[1][0].tobytes() and sc.tobytes() == tiles[1][1].tobytes()
        assert bi is None


def test_manifest_refusals(tmp_path):
    _, _, layers = _expert_layers()
    TL.write_expert_containers(str(tmp_path), layers)
    man = json.load(open(tmp_path / "manifest.json"))
    bad = json.loads(json.dumps(man))
    bad["containers"][0]["experts_per_tile"] = 2
    json.dump(bad, open(tmp_path / "manifest.json", "w"))
    with pytest.raises(TL.TileContainerError) as e:
        TL.ExpertContainers(str(tmp_path))
    assert e.value.status == L.MR_ERR_UNSUPPORTED
    bad = json.loads(json.dumps(man))
    bad["containers"][1]["in_features"] = 2048
    json.dump(bad, open(tmp_path / "manifest.json", "w"))
    with pytest.raises(TL.TileContainerError) as e:
        TL.ExpertContainers(str(tmp_path))
    assert "contradicts the manifest" in str(e.value)
    json.dump({"nothing": []}, open(tmp_path / "manifest.json", "w"))
    with pytest.raises(TL.TileContainerError):
        TL.ExpertContainers(str(tmp_path))
