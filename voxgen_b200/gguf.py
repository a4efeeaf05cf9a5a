"""GGUF v3 writer and a small reader, used to build seeded synthetic BaseLM models.

The container has no VoxCPM2 GGUF files, so every model the tests and the bench run is
written here with the metadata keys and tensor names the reference loader expects:

* file layout: magic, version, tensor/metadata counts, metadata KVs, tensor infos, data
  region aligned to ``general.alignment`` (default 32) — the format parsed by
  ``load_summary`` (src/gguf.rs:222-286);
* tensor names and GGUF dims ``[cols, rows]`` as validated by ``validate_layer``
  (src/baselm.rs:215-247) and ``BaseLmConfig::from_gguf`` (:124-150);
* Q8_0 storage: 32-element blocks of ``{fp16 d, int8 qs[32]}`` = 34 bytes
  (src/gguf.rs:41-45).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from pathlib import Path
from typing import BinaryIO, Dict, List, Sequence, Tuple, Union

import numpy as np

GGUF_MAGIC = 0x46554747  # "GGUF" little-endian (src/gguf.rs:6)
DEFAULT_ALIGNMENT = 32   # src/gguf.rs:7

# GGML tensor types used by the BaseLM path (src/gguf.rs:31-33)
GGML_F32 = 0
GGML_F16 = 1
GGML_Q8_0 = 8

# GGUF metadata value types (read_meta_value, src/gguf.rs:190-220)
T_UINT8, T_INT8, T_UINT16, T_INT16, T_UINT32, T_INT32, T_FLOAT32, T_BOOL, T_STRING, \
    T_ARRAY, T_UINT64, T_INT64, T_FLOAT64 = range(13)

Q8_BLOCK = 32
Q8_BLOCK_BYTES = 34


class F32(float):
    """Marks a metadata value to be written as GGUF FLOAT32."""


class U32(int):
    """Marks a metadata value to be written as GGUF UINT32."""


MetaValue = Union[str, int, float, bool, F32, U32, list]


def storage_bytes(ggml_type: int, elements: int) -> int:
    """Bytes of a tensor in the GGUF data region (GgmlType::storage_bytes, src/gguf.rs:37-48)."""
    if ggml_type == GGML_F32:
        return elements * 4
    if ggml_type == GGML_F16:
        return elements * 2
    if ggml_type == GGML_Q8_0:
        if elements % Q8_BLOCK:
            raise ValueError(f"Q8_0 tensor has {elements} elements, not divisible by 32")
        return elements // Q8_BLOCK * Q8_BLOCK_BYTES
    raise ValueError(f"unsupported GGML tensor type {ggml_type}")


def q8_0_pack(d: np.ndarray, qs: np.ndarray) -> np.ndarray:
    """Packs per-block fp16 scales ``d[rows, cols/32]`` and int8 quants ``qs[rows, cols]``
    into the 34-byte GGML Q8_0 block stream (row-major blocks)."""
    rows, cols = qs.shape
    nb = cols // Q8_BLOCK
    assert d.shape == (rows, nb) and d.dtype == np.float16 and qs.dtype == np.int8
    out = np.empty((rows, nb, Q8_BLOCK_BYTES), dtype=np.uint8)
    out[:, :, 0:2] = d.view(np.uint8).reshape(rows, nb, 2)
    out[:, :, 2:] = qs.view(np.uint8).reshape(rows, nb, Q8_BLOCK)
    return out.reshape(-1)


def q8_0_unpack(raw: np.ndarray, rows: int, cols: int) -> Tuple[np.ndarray, np.ndarray]:
    """Inverse of :func:`q8_0_pack`: returns ``(d fp16[rows, cols/32], qs int8[rows, cols])``."""
    nb = cols // Q8_BLOCK
    blk = np.asarray(raw, dtype=np.uint8).reshape(rows, nb, Q8_BLOCK_BYTES)
    d = np.ascontiguousarray(blk[:, :, 0:2]).view(np.float16).reshape(rows, nb)
    qs = np.ascontiguousarray(blk[:, :, 2:]).view(np.int8).reshape(rows, cols)
    return d, qs


def q8_0_dequant(raw: np.ndarray, rows: int, cols: int) -> np.ndarray:
    """``float(d) * float(q)`` per element, exact in fp32 (embedding.comp:33-40)."""
    d, qs = q8_0_unpack(raw, rows, cols)
    return (np.repeat(d.astype(np.float32), Q8_BLOCK, axis=1) * qs.astype(np.float32))


@dataclass
class Tensor:
    name: str
    dims: Tuple[int, ...]          # GGUF order: dims[0] is the contiguous (column) extent
    ggml_type: int
    data: np.ndarray               # raw bytes (uint8) in GGUF storage order


@dataclass
class GgufFile:
    metadata: Dict[str, MetaValue] = field(default_factory=dict)
    tensors: List[Tensor] = field(default_factory=list)
    alignment: int = DEFAULT_ALIGNMENT

    def add(self, name: str, dims: Sequence[int], ggml_type: int, data: np.ndarray) -> None:
        raw = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        elements = int(np.prod(dims))
        if raw.size != storage_bytes(ggml_type, elements):
            raise ValueError(f"{name}: {raw.size} bytes for dims {dims} type {ggml_type}")
        self.tensors.append(Tensor(name, tuple(int(x) for x in dims), ggml_type, raw))


def _w_str(f: BinaryIO, s: str) -> None:
    b = s.encode("utf-8")
    f.write(struct.pack("<Q", len(b)))
    f.write(b)


def _w_value(f: BinaryIO, v: MetaValue) -> None:
    if isinstance(v, bool):
        f.write(struct.pack("<IB", T_BOOL, int(v)))
    elif isinstance(v, U32):
        f.write(struct.pack("<II", T_UINT32, int(v)))
    elif isinstance(v, F32):
        f.write(struct.pack("<If", T_FLOAT32, float(v)))
    elif isinstance(v, int):
        f.write(struct.pack("<IQ", T_UINT64, v)) if v >= 0 else f.write(struct.pack("<Iq", T_INT64, v))
    elif isinstance(v, float):
        f.write(struct.pack("<If", T_FLOAT32, v))
    elif isinstance(v, str):
        f.write(struct.pack("<I", T_STRING))
        _w_str(f, v)
    elif isinstance(v, list):
        f.write(struct.pack("<I", T_ARRAY))
        if all(isinstance(x, str) for x in v):
            f.write(struct.pack("<IQ", T_STRING, len(v)))
            for x in v:
                _w_str(f, x)
        else:
            f.write(struct.pack("<IQ", T_INT32, len(v)))
            for x in v:
                f.write(struct.pack("<i", int(x)))
    else:
        raise TypeError(f"unsupported metadata value {v!r}")


def write_gguf(path: Union[str, Path], g: GgufFile, version: int = 3) -> None:
    """Writes ``g`` as a GGUF file; tensor offsets are aligned to ``g.alignment``."""
    al = g.alignment
    offsets: List[int] = []
    off = 0
    for t in g.tensors:
        off = (off + al - 1) // al * al
        offsets.append(off)
        off += t.data.size
    meta = dict(g.metadata)
    if al != DEFAULT_ALIGNMENT:
        meta["general.alignment"] = U32(al)
    with open(path, "wb") as f:
        f.write(struct.pack("<IIQQ", GGUF_MAGIC, version, len(g.tensors), len(meta)))
        for k, v in meta.items():
            _w_str(f, k)
            _w_value(f, v)
        for t, o in zip(g.tensors, offsets):
            _w_str(f, t.name)
            f.write(struct.pack("<I", len(t.dims)))
            for dmn in t.dims:
                f.write(struct.pack("<Q", dmn))
            f.write(struct.pack("<IQ", t.ggml_type, o))
        pos = f.tell()
        data_start = (pos + al - 1) // al * al
        f.write(b"\0" * (data_start - pos))
        for t, o in zip(g.tensors, offsets):
            cur = f.tell() - data_start
            if o > cur:
                f.write(b"\0" * (o - cur))
            t.data.tofile(f)


@dataclass
class TensorInfo:
    name: str
    dims: Tuple[int, ...]
    ggml_type: int
    offset: int          # relative to the data region
    nbytes: int


@dataclass
class GgufSummary:
    path: Path
    version: int
    metadata: Dict[str, object]
    tensors: Dict[str, TensorInfo]
    data_offset: int

    def tensor_bytes(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        return np.fromfile(self.path, dtype=np.uint8, count=t.nbytes,
                           offset=self.data_offset + t.offset)

    def matrix_f32(self, name: str) -> np.ndarray:
        """Dequantised fp32 ``[rows, cols]`` (or ``[n]`` for vectors)."""
        t = self.tensors[name]
        raw = self.tensor_bytes(name)
        if len(t.dims) == 1:
            cols, rows = t.dims[0], 1
        else:
            cols, rows = t.dims[0], int(np.prod(t.dims[1:]))
        if t.ggml_type == GGML_F32:
            out = raw.view(np.float32).reshape(rows, cols)
        elif t.ggml_type == GGML_F16:
            out = raw.view(np.float16).astype(np.float32).reshape(rows, cols)
        else:
            out = q8_0_dequant(raw, rows, cols)
        return out.reshape(-1) if len(t.dims) == 1 else out


def read_gguf(path: Union[str, Path]) -> GgufSummary:
    """Parses header, metadata and tensor table (load_summary, src/gguf.rs:222-286)."""
    path = Path(path)
    f = open(path, "rb")

    def rd(n: int) -> bytes:
        b = f.read(n)
        if len(b) != n:
            raise ValueError("unexpected EOF while reading GGUF")
        return b

    def rs() -> str:
        (n,) = struct.unpack("<Q", rd(8))
        return rd(n).decode("utf-8")

    scal = {T_UINT8: "<B", T_INT8: "<b", T_UINT16: "<H", T_INT16: "<h", T_UINT32: "<I",
            T_INT32: "<i", T_FLOAT32: "<f", T_BOOL: "<B", T_UINT64: "<Q", T_INT64: "<q",
            T_FLOAT64: "<d"}

    def rv(ty: int):
        if ty in scal:
            fmt = scal[ty]
            (v,) = struct.unpack(fmt, rd(struct.calcsize(fmt)))
            return bool(v) if ty == T_BOOL else v
        if ty == T_STRING:
            return rs()
        if ty == T_ARRAY:
            ety, n = struct.unpack("<IQ", rd(12))
            return [rv(ety) for _ in range(n)]
        raise ValueError(f"unknown GGUF metadata value type {ty}")

    magic, version, n_t, n_kv = struct.unpack("<IIQQ", rd(24))
    if magic != GGUF_MAGIC:
        raise ValueError(f"{path} is not a GGUF file")
    meta: Dict[str, object] = {}
    for _ in range(n_kv):
        k = rs()
        (ty,) = struct.unpack("<I", rd(4))
        meta[k] = rv(ty)
    tensors: Dict[str, TensorInfo] = {}
    for _ in range(n_t):
        name = rs()
        (nd,) = struct.unpack("<I", rd(4))
        dims = struct.unpack(f"<{nd}Q", rd(8 * nd))
        ty, off = struct.unpack("<IQ", rd(12))
        tensors[name] = TensorInfo(name, tuple(dims), ty, off,
                                   storage_bytes(ty, int(np.prod(dims))))
    al = int(meta.get("general.alignment", DEFAULT_ALIGNMENT)) or 1
    pos = f.tell()
    f.close()
    return GgufSummary(path, version, meta, tensors, (pos + al - 1) // al * al)
