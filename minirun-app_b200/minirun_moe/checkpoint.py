"""Safetensors checkpoints: the affine expert tensors of an MLX checkpoint.

Follows the reference's reader and sharded checkpoint
(Sources/ModelAdapters/Loading/SafetensorsFile.swift:22-330,
QwenCheckpoint.swift:19-164): the 8-byte header length and JSON header are
validated before any offset is used (well-formed records, non-negative
integer shapes and offsets, ranges inside the payload, byte counts equal to
shape x element size, no two tensors overlapping), the file is memory-mapped
so a tensor costs nothing until read, and a sharded checkpoint resolves each
tensor through `model.safetensors.index.json` on its own — the three parts of
a quantized linear may sit in different shards.

`Checkpoint.affine` returns the library's AffineWeights with the bytes as
they lie in the file: `U32` packed codes, and BF16/F16/F32 scales and biases
reinterpreted (viewed), never converted.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import dataclass

import numpy as np
import torch

from .bridge import AffineWeights

ITEM_SIZE = {"F32": 4, "I32": 4, "U32": 4, "BF16": 2, "F16": 2, "I16": 2, "U16": 2,
             "U8": 1, "I8": 1, "BOOL": 1, "F64": 8, "I64": 8, "U64": 8}
# host arrays of each dtype (BF16 as its 16-bit patterns)
_NP = {"F32": np.float32, "I32": np.int32, "U32": np.uint32, "BF16": np.uint16,
       "F16": np.float16, "I16": np.int16, "U16": np.uint16, "U8": np.uint8, "I8": np.int8,
       "BOOL": np.bool_, "F64": np.float64, "I64": np.int64, "U64": np.uint64}
_SCALE_TORCH = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32}


class SafetensorsError(ValueError):
    """A malformed file, a missing tensor or a dtype/shape the loader refuses."""


@dataclass(frozen=True)
class TensorInfo:
    name: str
    dtype: str
    shape: tuple
    offset: int      # absolute offset of the first byte in the file
    byte_count: int


def _nonneg_int(v, field: str) -> int:
    if isinstance(v, bool) or not isinstance(v, int) or v < 0:
        raise SafetensorsError(f"{field} is not a nonnegative integer")
    return v


class SafetensorsFile:
    """One .safetensors file, header validated, payload memory-mapped."""

    def __init__(self, path: str):
        self.path = path
        size = os.path.getsize(path)
        if size < 8:
            raise SafetensorsError(f"file is {size} bytes, shorter than the 8-byte header length")
        with open(path, "rb") as f:
            hlen = int.from_bytes(f.read(8), "little")
            if hlen <= 0 or 8 + hlen > size:
                raise SafetensorsError(
                    f"header claims {hlen} bytes, file has {size - 8} after the length field")
            raw = f.read(hlen)
        start = 8 + hlen
        payload = size - start
        try:
            root = json.loads(raw)
        except ValueError as e:
            raise SafetensorsError(f"header is not JSON ({e})") from None
        if not isinstance(root, dict):
            raise SafetensorsError("header is not a JSON object")
        self.metadata = {k: str(v) for k, v in (root.get("__metadata__") or {}).items()}
        self.tensors: dict[str, TensorInfo] = {}
        spans = []
        for name, ent in root.items():
            if name == "__metadata__":
                continue
            if (not isinstance(ent, dict) or not isinstance(ent.get("dtype"), str)
                    or not isinstance(ent.get("shape"), list)
                    or not isinstance(ent.get("data_offsets"), list)
                    or len(ent["data_offsets"]) != 2):
                raise SafetensorsError(f"entry '{name}' is not a well-formed tensor record")
            shape = tuple(_nonneg_int(v, f"tensor '{name}' shape[{i}]")
                          for i, v in enumerate(ent["shape"]))
            begin, end = (_nonneg_int(v, f"tensor '{name}' data_offsets[{i}]")
                          for i, v in enumerate(ent["data_offsets"]))
            if end < begin or end > payload:
                raise SafetensorsError(
                    f"tensor '{name}' spans [{begin}, {end}) but the payload is {payload} bytes")
            item = ITEM_SIZE.get(ent["dtype"])
            if item is None:
                raise SafetensorsError(f"tensor '{name}' has unsupported dtype {ent['dtype']}")
            # Python ints: a crafted shape cannot wrap to a small byte count
            need = math.prod(shape) * item
            if end - begin != need:
                raise SafetensorsError(
                    f"tensor '{name}' spans {end - begin} bytes, but shape {list(shape)} at "
                    f"{item} bytes per element needs {need}")
            self.tensors[name] = TensorInfo(name, ent["dtype"], shape, start + begin, end - begin)
            spans.append((begin, end, name))
        spans.sort()
        for (b0, e0, n0), (b1, e1, n1) in zip(spans, spans[1:]):
            if b1 < e0:
                raise SafetensorsError(
                    f"tensor '{n1}' range [{b1}, {e1}) overlaps tensor '{n0}' range [{b0}, {e0})")
        self._map = None

    def info(self, name: str) -> TensorInfo:
        try:
            return self.tensors[name]
        except KeyError:
            raise SafetensorsError(f"missing tensor '{name}'") from None

    def contains(self, name: str) -> bool:
        return name in self.tensors

    def array(self, name: str) -> np.ndarray:
        """The tensor as a read-only view of the mapped file (BF16 as uint16)."""
        info = self.info(name)
        if self._map is None:
            self._map = np.memmap(self.path, dtype=np.uint8, mode="r")
        raw = self._map[info.offset:info.offset + info.byte_count]
        return raw.view(_NP[info.dtype]).reshape(info.shape)


class Checkpoint:
    """A checkpoint directory: `model.safetensors.index.json` (weight_map:
    tensor -> shard) or a single `model.safetensors`. Shards open on first use."""

    def __init__(self, directory: str):
        self.directory = directory
        index = os.path.join(directory, "model.safetensors.index.json")
        if os.path.exists(index):
            try:
                self.weight_map = dict(json.load(open(index))["weight_map"])
            except (ValueError, KeyError, TypeError):
                raise SafetensorsError(f"{index} has no 'weight_map'") from None
        else:
            single = os.path.join(directory, "model.safetensors")
            if not os.path.exists(single):
                raise SafetensorsError(f"{directory} has neither an index nor model.safetensors")
            self.weight_map = {n: "model.safetensors" for n in SafetensorsFile(single).tensors}
        self._shards: dict[str, SafetensorsFile] = {}

    def _shard(self, name: str) -> SafetensorsFile:
        file = self.weight_map.get(name)
        if file is None:
            raise SafetensorsError(f"missing tensor '{name}'")
        if file not in self._shards:
            self._shards[file] = SafetensorsFile(os.path.join(self.directory, file))
        return self._shards[file]

    def contains(self, name: str) -> bool:
        return name in self.weight_map

    def info(self, name: str) -> TensorInfo:
        return self._shard(name).info(name)

    def array(self, name: str) -> np.ndarray:
        return self._shard(name).array(name)

    def tensor(self, name: str, device=None) -> torch.Tensor:
        """A float tensor as stored (BF16 viewed as bfloat16), on `device`."""
        info = self.info(name)
        host = torch.from_numpy(np.array(self.array(name)))
        if info.dtype in _SCALE_TORCH and info.dtype != "F32":
            host = host.view(_SCALE_TORCH[info.dtype])
        return host.to(device) if device is not None else host

    def affine(self, base: str, group_size: int, bits: int, stacked: bool = False,
               device=None) -> AffineWeights:
        """QwenCheckpoint.affine (:94-164): `{base}.weight` U32 codes,
        `{base}.scales` / `{base}.biases` in one float dtype, each resolved in
        its own shard; rank 3 (expert stack) when `stacked`."""
        pi, si, bi = (self.info(f"{base}.{p}") for p in ("weight", "scales", "biases"))
        if pi.dtype != "U32":
            raise SafetensorsError(f"tensor '{base}.weight' has dtype {pi.dtype}, not U32")
        if si.dtype != bi.dtype:
            raise SafetensorsError(f"{base}: scales are {si.dtype} but biases are {bi.dtype}")
        if si.dtype not in _SCALE_TORCH:
            raise SafetensorsError(f"tensor '{base}.scales' has unsupported dtype {si.dtype}")
        rank = 3 if stacked else 2
        if len(pi.shape) != rank:
            raise SafetensorsError(
                f"tensor '{base}.weight' has shape {list(pi.shape)}; expected rank {rank}")

        def host(name, dt):
            arr = self.array(name)  # read-only view of the mapped file
            if device is not None and torch.device(device).type == "cuda":
                # file -> pinned staging -> device, one copy each
                stage = torch.empty(arr.shape, pin_memory=True,
                                    dtype=torch.from_numpy(np.empty(0, arr.dtype)).dtype)
                stage.numpy()[...] = arr
                return stage.view(dt).to(device, non_blocking=True)
            t = torch.from_numpy(np.array(arr)).view(dt)  # a reinterpretation, never a conversion
            return t.to(device) if device is not None else t

        sd = _SCALE_TORCH[si.dtype]
        packed = host(f"{base}.weight", torch.int32)
        scales = host(f"{base}.scales", sd if si.dtype != "F32" else torch.float32)
        biases = host(f"{base}.biases", sd if si.dtype != "F32" else torch.float32)
        return AffineWeights(packed, scales, biases, group_size, bits)


def write_safetensors(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """Write {name: (dtype, array)} (arrays of any numpy dtype whose bytes are
    the tensor's, e.g. uint16 for BF16) as one .safetensors file."""
    header = {}
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    blobs, off = [], 0
    for name in sorted(tensors):
        dtype, arr = tensors[name]
        a = np.ascontiguousarray(arr)
        if dtype not in ITEM_SIZE:
            raise SafetensorsError(f"unsupported dtype {dtype}")
        b = a.tobytes()
        n = int(np.prod(a.shape, dtype=np.int64)) if a.shape else 1
        if len(b) != n * ITEM_SIZE[dtype]:
            raise SafetensorsError(f"'{name}': {len(b)} bytes do not hold {a.shape} {dtype}")
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)  # payload 8-byte aligned
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        for b in blobs:
            f.write(b)
