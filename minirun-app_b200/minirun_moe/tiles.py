"""MNRNTIL1 quantized tile containers and expert sets stored in them.

The reference keeps routed experts on disk in its own container format
(Sources/StorageCore/Container/QuantizedTileContainer.swift): a 16 KiB header,
then tiles of output rows, each tile [packed | scales | biases] with every tile
and sub-region on a 16 KiB boundary, and optionally one SHA-256 per tile. A
directory of such containers plus a manifest (one container per layer and
projection, one expert per tile) is what its streamed expert backend reads
(Sources/ModelAdapters/Loading/QwenExpertBackends.swift:377-505).

Here the header is decoded and validated, tiles are read and digest-checked
by the native library (mr_tiles_*), and `ExpertContainers.register` hands the
tiles to the HBM expert cache, which reads each expert's three tiles into
pinned staging on a miss and copies them to its slot. `write_container` and
`write_expert_containers` produce the same files (the header comes from the
library's encoder, so writer and reader share one set of layout rules).
"""
from __future__ import annotations

import ctypes as C
import json
import os
from dataclasses import dataclass

import numpy as np

from . import _lib as L

ALIGN = 16384
HEADER_BYTES = 16384
MODE_MXFP4, MODE_AFFINE, MODE_FP8_BLOCK = 0, 1, 2
SCALE_E8M0, SCALE_F16, SCALE_BF16, SCALE_F32 = 0, 1, 2, 3
CONTENT_SYNTHETIC, CONTENT_CHECKPOINT = 0, 1
# container scale element type <-> the library's affine scale dtype
SCALE_TO_DTYPE = {SCALE_BF16: L.MR_DTYPE_BF16, SCALE_F16: L.MR_DTYPE_F16,
                  SCALE_F32: L.MR_DTYPE_F32}
DTYPE_TO_SCALE = {v: k for k, v in SCALE_TO_DTYPE.items()}
# manifest projection slots (QwenMoEConfig.swift:280-294): gate w1, up w3, down w2
PROJECTION_SLOTS = ("w1", "w3", "w2")


class TileContainerError(Exception):
    """A container or manifest the reader refuses; `status` is the mr_status."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def _msg(buf) -> str:
    return buf.value.decode(errors="replace")


def layout_for(rows: int, cols: int, group_size: int, bits: int, tile_count: int, *,
               quant_mode: int = MODE_AFFINE, scale_dtype: int = SCALE_BF16,
               scale_block_rows: int = 1, content_kind: int = CONTENT_CHECKPOINT,
               seed: int = 0, digests: bool = False) -> L.mr_tile_layout:
    """The layout a writer must produce for this geometry
    (QuantizedTileContainer.layout, :441-580); TileContainerError if the
    format rejects the geometry."""
    lay = L.mr_tile_layout()
    lay.rows, lay.cols, lay.group_size, lay.bits = rows, cols, group_size, bits
    lay.quant_mode, lay.scale_dtype = quant_mode, scale_dtype
    lay.scale_block_rows = scale_block_rows
    lay.content_kind, lay.seed = content_kind, seed
    msg = C.create_string_buffer(512)
    st = L.load().mr_tiles_layout_for(C.byref(lay), tile_count, 1 if digests else 0, msg, 512)
    if st != L.MR_OK:
        raise TileContainerError(st, _msg(msg))
    return lay


def sha256(data) -> bytes:
    """SHA-256 by the library's own implementation (the tile digest)."""
    a = np.ascontiguousarray(np.frombuffer(memoryview(data), dtype=np.uint8))
    out = (C.c_uint8 * 32)()
    L.load().mr_sha256(a.ctypes.data, a.nbytes, out)
    return bytes(out)


def _tile_bytes(lay: L.mr_tile_layout, packed, scales, biases) -> np.ndarray:
    t = np.zeros(lay.tile_stride, dtype=np.uint8)
    parts = [(0, packed, lay.packed_bytes), (lay.scale_offset, scales, lay.scale_bytes)]
    if lay.bias_bytes:
        parts.append((lay.bias_offset, biases, lay.bias_bytes))
    for off, data, n in parts:
        b = np.frombuffer(memoryview(np.ascontiguousarray(data)).cast("B"), dtype=np.uint8)
        if b.nbytes != n:
            raise TileContainerError(L.MR_ERR_INVALID_ARGUMENT,
                                     f"a sub-region is {b.nbytes} bytes, the layout says {n}")
        t[off:off + n] = b
    return t


def write_container(path: str, tiles, *, rows: int, cols: int, group_size: int, bits: int,
                    quant_mode: int = MODE_AFFINE, scale_dtype: int = SCALE_BF16,
                    content_kind: int = CONTENT_CHECKPOINT, seed: int = 0,
                    digests: bool = True) -> L.mr_tile_layout:
    """Write a container of `tiles`, each (packed, scales, biases) arrays of
    one tile's sub-regions (biases None without them). Returns the layout."""
    tiles = list(tiles)
    lay = layout_for(rows, cols, group_size, bits, len(tiles), quant_mode=quant_mode,
                     scale_dtype=scale_dtype, content_kind=content_kind, seed=seed,
                     digests=digests)
    blobs = [_tile_bytes(lay, *t) for t in tiles]
    table = np.zeros(max(1, 32 * len(tiles)), dtype=np.uint8)
    if digests:
        for i, b in enumerate(blobs):
            table[32 * i:32 * i + 32] = np.frombuffer(sha256(b), dtype=np.uint8)
    header = np.zeros(HEADER_BYTES, dtype=np.uint8)
    msg = C.create_string_buffer(512)
    st = L.load().mr_tiles_encode_header(C.byref(lay), table.ctypes.data if digests else None,
                                         header.ctypes.data, msg, 512)
    if st != L.MR_OK:
        raise TileContainerError(st, _msg(msg))
    with open(path, "wb") as f:
        f.write(header.tobytes())
        for b in blobs:
            f.write(b.tobytes())
    return lay


class TileContainer:
    """An open container (QuantizedTileContainer.open, :789-832)."""

    def __init__(self, path: str, verify: bool = True):
        self.path = path
        h = C.c_void_p()
        msg = C.create_string_buffer(1024)
        st = L.load().mr_tiles_open(path.encode(), 1 if verify else 0, C.byref(h), msg, 1024)
        if st != L.MR_OK:
            raise TileContainerError(st, _msg(msg))
        self.handle = h
        lay = L.mr_tile_layout()
        L.load().mr_tiles_get_layout(h, C.byref(lay))
        self.layout = lay

    def read(self, tile: int, out: np.ndarray | None = None) -> np.ndarray:
        """One whole tile (tile_stride bytes), digest-checked when verifying."""
        if out is None:
            out = np.empty(self.layout.tile_stride, dtype=np.uint8)
        msg = C.create_string_buffer(1024)
        st = L.load().mr_tiles_read(self.handle, tile, out.ctypes.data, out.nbytes, msg, 1024)
        if st != L.MR_OK:
            raise TileContainerError(st, _msg(msg))
        return out

    def sub_regions(self, tile: int):
        """(packed, scales, biases) byte arrays of one tile (biases None without)."""
        lay, t = self.layout, self.read(tile)
        biases = t[lay.bias_offset:lay.bias_offset + lay.bias_bytes] if lay.bias_bytes else None
        return (t[:lay.packed_bytes], t[lay.scale_offset:lay.scale_offset + lay.scale_bytes],
                biases)

    def close(self) -> None:
        if self.handle:
            L.load().mr_tiles_close(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


@dataclass
class _Entry:
    layer: int
    slot: str
    container: TileContainer
    out_features: int
    in_features: int
    tile_of_expert: dict


class ExpertContainers:
    """A directory of expert containers and its manifest.json: for each
    (layer, projection slot w1/w3/w2) one affine, checkpoint-derived
    container holding one whole expert per tile
    (QwenExpertBackends.swift:377-505, same manifest keys and checks)."""

    def __init__(self, directory: str, verify: bool = True):
        self.directory = directory
        path = os.path.join(directory, "manifest.json")
        try:
            root = json.load(open(path))
            records = root["containers"]
        except (OSError, ValueError, KeyError, TypeError) as e:
            raise TileContainerError(L.MR_ERR_INVALID_ARGUMENT,
                                     f"{path} has no 'containers' list ({e})") from None
        self.entries: dict[tuple[int, str], _Entry] = {}
        for rec in records:
            try:
                layer, slot, file = int(rec["layer"]), rec["projection"], rec["file"]
                out_f, in_f = int(rec["out_features_per_expert"]), int(rec["in_features"])
                per_tile, tiles = int(rec["experts_per_tile"]), rec["tiles"]
            except (KeyError, TypeError, ValueError):
                raise TileContainerError(L.MR_ERR_INVALID_ARGUMENT,
                                         f"malformed container record: {rec}") from None
            if slot not in PROJECTION_SLOTS:
                raise TileContainerError(L.MR_ERR_INVALID_ARGUMENT,
                                         f"unknown projection slot {slot!r}")
            if per_tile != 1:
                raise TileContainerError(
                    L.MR_ERR_UNSUPPORTED,
                    f"{file} packs {per_tile} experts per tile; this reader implements the "
                    "whole-expert geometry")
            cont = TileContainer(os.path.join(directory, file), verify)
            lay = cont.layout
            if lay.quant_mode != MODE_AFFINE:
                raise TileContainerError(L.MR_ERR_UNSUPPORTED, f"{file} is not an affine container")
            if lay.content_kind != CONTENT_CHECKPOINT:
                raise TileContainerError(L.MR_ERR_INVALID_ARGUMENT,
                                         f"{file} does not declare checkpoint-derived content")
            if (lay.rows, lay.cols) != (out_f, in_f):
                raise TileContainerError(
                    L.MR_ERR_INVALID_ARGUMENT,
                    f"{file}: header geometry {lay.rows}x{lay.cols} contradicts the manifest's "
                    f"{out_f}x{in_f}")
            tile_of = {}
            seen = set()
            for t in tiles:
                idx, members = int(t["tile"]), list(t["experts"])
                if len(members) != 1 or not 0 <= idx < lay.tile_count:
                    raise TileContainerError(L.MR_ERR_INVALID_ARGUMENT,
                                             f"malformed tile record in {file}: {t}")
                tile_of[int(members[0])] = idx
                seen.add(idx)
            if len(seen) != lay.tile_count:
                raise TileContainerError(L.MR_ERR_INVALID_ARGUMENT, f"{file}: a tile lists no expert")
            self.entries[(layer, slot)] = _Entry(layer, slot, cont, out_f, in_f, tile_of)

    def layers(self) -> list[int]:
        return sorted({k[0] for k in self.entries})

    def _triple(self, layer: int):
        try:
            return tuple(self.entries[(layer, s)] for s in PROJECTION_SLOTS)
        except KeyError:
            raise TileContainerError(L.MR_ERR_INVALID_ARGUMENT,
                                     f"layer {layer} lacks one of w1/w3/w2") from None

    def experts(self, layer: int) -> list[int]:
        return sorted(self._triple(layer)[0].tile_of_expert)

    def slot_bytes(self, layer: int) -> int:
        """Bytes of one expert in a cache slot (256-byte aligned arrays)."""
        n = 0
        for e in self._triple(layer):
            lay = e.container.layout
            n += (lay.packed_bytes + 255) // 256 * 256 + 2 * ((lay.scale_bytes + 255) // 256 * 256)
        return n

    def register(self, cache, layer: int) -> None:
        """Register every expert of `layer` with an ExpertCache, backed by the
        containers' tiles (the containers stay open while registered)."""
        trip = self._triple(layer)
        handles = (C.c_void_p * 3)(*(e.container.handle for e in trip))
        for ex in self.experts(layer):
            tiles = (C.c_int64 * 3)(*(e.tile_of_expert[ex] for e in trip))
            cache.ctx.check("mr_cache_register_tiles", L.load().mr_cache_register_tiles(
                cache.handle, layer, ex, handles, tiles))
            cache._keep[(layer, ex)] = self  # keep the containers alive

    def close(self) -> None:
        for e in self.entries.values():
            e.container.close()


def _np_bytes(t) -> np.ndarray:
    """A torch tensor or numpy array as host bytes."""
    if hasattr(t, "detach"):  # torch: reinterpret as bytes (bf16 has no numpy dtype)
        import torch
        t = t.detach().contiguous().cpu().reshape(-1).view(torch.uint8)
        return t.numpy().copy()
    return np.frombuffer(np.ascontiguousarray(t).tobytes(), dtype=np.uint8)


def write_expert_containers(directory: str, layers: dict, *, group_size: int = 64,
                            scale_dtype: int = SCALE_BF16, digests: bool = True) -> None:
    """Write `layers` {layer: (gate, up, down)} — each projection a stack of
    expert arrays (packed [E, out, in*bits/32] uint32, scales and biases
    [E, out, in/group]) given as (packed, scales, biases, bits) tuples of
    numpy arrays or torch tensors — as one container per (layer, projection)
    with one expert per tile, plus manifest.json."""
    os.makedirs(directory, exist_ok=True)
    records = []
    for layer, projs in sorted(layers.items()):
        for slot, (packed, scales, biases, bits) in zip(PROJECTION_SLOTS, projs):
            E, out_f = int(packed.shape[0]), int(packed.shape[1])
            in_f = int(packed.shape[2]) * 32 // bits
            tiles = [(_np_bytes(packed[e]), _np_bytes(scales[e]), _np_bytes(biases[e]))
                     for e in range(E)]
            file = f"layer{layer:03d}.{slot}.mnrntil"
            write_container(os.path.join(directory, file), tiles, rows=out_f, cols=in_f,
                            group_size=group_size, bits=bits, scale_dtype=scale_dtype,
                            digests=digests)
            records.append({"layer": layer, "projection": slot, "file": file,
                            "out_features_per_expert": out_f, "in_features": in_f,
                            "experts_per_tile": 1,
                            "tiles": [{"tile": e, "experts": [e]} for e in range(E)]})
    with open(os.path.join(directory, "manifest.json"), "w") as f:
        json.dump({"containers": records}, f, indent=1)
