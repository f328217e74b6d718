"""GGUF v3 reader and streaming writer.

The layout follows llmdot's loader (src/Llmdot.Core/Loading/GgufReader.cs:8-126):
magic ``GGUF``, u32 version (>= 2), u64 tensor count, u64 metadata count,
typed key/value metadata, tensor infos (name, u32 n_dims, u64 dims, u32 ggml
type, u64 offset relative to the aligned data section), padding to
``general.alignment`` (default 32), tensor data.

The writer streams tensors one at a time so multi-GB synthetic models never
have to sit in host memory at once.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Sequence

import numpy as np

# GgufValueType (src/Llmdot.Core/Loading/GgufValueType.cs)
U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)

# GgmlType (src/Llmdot.Core/Loading/GgmlType.cs:3-27)
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_1 = 0, 1, 2, 3
GGML_Q5_0, GGML_Q5_1, GGML_Q8_0, GGML_Q8_1 = 6, 7, 8, 9
GGML_Q2_K, GGML_Q3_K, GGML_Q4_K, GGML_Q5_K, GGML_Q6_K = 10, 11, 12, 13, 14
GGML_BF16 = 25

TYPE_NAMES = {
    GGML_F32: "F32", GGML_F16: "F16", GGML_Q4_0: "Q4_0", GGML_Q4_1: "Q4_1",
    GGML_Q5_0: "Q5_0", GGML_Q5_1: "Q5_1", GGML_Q8_0: "Q8_0", GGML_Q8_1: "Q8_1",
    GGML_Q2_K: "Q2_K", GGML_Q3_K: "Q3_K", GGML_Q4_K: "Q4_K", GGML_Q5_K: "Q5_K",
    GGML_Q6_K: "Q6_K", GGML_BF16: "BF16",
}

# (elements per block, bytes per block): TensorSize.ByteCount, src/Llmdot.Core/Tensors/TensorSize.cs:7-24
BLOCK = {
    GGML_F32: (1, 4), GGML_F16: (1, 2), GGML_BF16: (1, 2),
    GGML_Q4_0: (32, 18), GGML_Q4_1: (32, 20), GGML_Q5_0: (32, 22), GGML_Q5_1: (32, 24),
    GGML_Q8_0: (32, 34), GGML_Q8_1: (32, 40),
    GGML_Q2_K: (256, 84), GGML_Q3_K: (256, 110), GGML_Q4_K: (256, 144),
    GGML_Q5_K: (256, 176), GGML_Q6_K: (256, 210),
}


def byte_count(ggml_type: int, n_elements: int) -> int:
    """TensorSize.ByteCount: raises for unsupported types like the reference."""
    if ggml_type not in BLOCK:
        raise NotImplementedError(f"Unsupported GGML type: {ggml_type}")
    be, bb = BLOCK[ggml_type]
    return n_elements // be * bb


@dataclass
class TensorInfo:
    name: str
    dims: List[int]          # ne0 (columns / in-features) first
    ggml_type: int
    offset: int = 0          # relative to the data section
    data_offset: int = 0     # absolute file offset (reader only)

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n if self.dims else 0

    @property
    def n_bytes(self) -> int:
        return byte_count(self.ggml_type, self.n_elements)


# --------------------------------------------------------------------------- writer

def _str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, v: Any) -> bytes:
    if vtype == U8:
        return struct.pack("<B", v)
    if vtype == I8:
        return struct.pack("<b", v)
    if vtype == U16:
        return struct.pack("<H", v)
    if vtype == I16:
        return struct.pack("<h", v)
    if vtype == U32:
        return struct.pack("<I", v)
    if vtype == I32:
        return struct.pack("<i", v)
    if vtype == F32:
        return struct.pack("<f", v)
    if vtype == BOOL:
        return struct.pack("<B", 1 if v else 0)
    if vtype == STR:
        return _str(v)
    if vtype == U64:
        return struct.pack("<Q", v)
    if vtype == I64:
        return struct.pack("<q", v)
    if vtype == F64:
        return struct.pack("<d", v)
    raise ValueError(vtype)


def _kv(key: str, vtype: int, v: Any, elem_type: Optional[int] = None) -> bytes:
    out = _str(key) + struct.pack("<I", vtype)
    if vtype == ARR:
        assert elem_type is not None
        out += struct.pack("<IQ", elem_type, len(v))
        if elem_type == STR:
            out += b"".join(_str(s) for s in v)
        elif elem_type == I32:
            out += np.asarray(v, dtype="<i4").tobytes()
        elif elem_type == F32:
            out += np.asarray(v, dtype="<f4").tobytes()
        else:
            out += b"".join(_value(elem_type, x) for x in v)
        return out
    return out + _value(vtype, v)


@dataclass
class Metadata:
    entries: List[bytes] = field(default_factory=list)

    def add(self, key: str, vtype: int, v: Any, elem_type: Optional[int] = None) -> "Metadata":
        self.entries.append(_kv(key, vtype, v, elem_type))
        return self


def write_gguf(path: str, metadata: Metadata, infos: Sequence[TensorInfo],
               produce: Callable[[TensorInfo], bytes], alignment: int = 32) -> None:
    """Write a GGUF v3 file.  ``produce(info)`` returns each tensor's raw bytes,
    called in order, so the caller can generate tensors lazily."""
    off = 0
    for t in infos:
        t.offset = off
        off += t.n_bytes
        off += (alignment - off % alignment) % alignment
    with open(path, "wb") as f:
        f.write(b"GGUF")
        f.write(struct.pack("<IQQ", 3, len(infos), len(metadata.entries)))
        for e in metadata.entries:
            f.write(e)
        for t in infos:
            f.write(_str(t.name))
            f.write(struct.pack("<I", len(t.dims)))
            f.write(struct.pack(f"<{len(t.dims)}Q", *t.dims))
            f.write(struct.pack("<IQ", t.ggml_type, t.offset))
        pos = f.tell()
        f.write(b"\0" * ((alignment - pos % alignment) % alignment))
        base = f.tell()
        for t in infos:
            data = produce(t)
            if len(data) != t.n_bytes:
                raise ValueError(f"{t.name}: produced {len(data)} bytes, expected {t.n_bytes}")
            cur = f.tell() - base
            if cur != t.offset:
                f.write(b"\0" * (t.offset - cur))
            f.write(data)
        end = f.tell() - base
        f.write(b"\0" * ((alignment - end % alignment) % alignment))


# --------------------------------------------------------------------------- reader

class GgufFile:
    """Parsed GGUF header; tensor bytes are served from a read-only memory map."""

    def __init__(self, path: str):
        self.path = path
        self.metadata: Dict[str, Any] = {}
        self.metadata_types: Dict[str, int] = {}
        self.tensors: Dict[str, TensorInfo] = {}
        self.order: List[str] = []
        with open(path, "rb") as f:
            buf = f.read(64 << 20)  # headers of our models are far below 64 MiB
            pos = 0

            def rd(fmt: str):
                nonlocal pos
                v = struct.unpack_from(fmt, buf, pos)
                pos += struct.calcsize(fmt)
                return v[0] if len(v) == 1 else v

            def rstr() -> str:
                nonlocal pos
                n = rd("<Q")
                s = buf[pos:pos + n].decode("utf-8")
                pos += n
                return s

            def rval(t: int):
                if t == STR:
                    return rstr()
                if t == ARR:
                    et, n = rd("<I"), rd("<Q")
                    return [rval(et) for _ in range(n)]
                fmt = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f",
                       BOOL: "<B", U64: "<Q", I64: "<q", F64: "<d"}[t]
                v = rd(fmt)
                return bool(v) if t == BOOL else v

            if buf[:4] != b"GGUF":
                raise ValueError("Invalid GGUF magic. Expected 'GGUF'.")
            pos = 4
            self.version = rd("<I")
            if self.version < 2:
                raise ValueError(f"Unsupported GGUF version: {self.version}")
            nt, nkv = rd("<Q"), rd("<Q")
            for _ in range(nkv):
                k = rstr()
                t = rd("<I")
                self.metadata[k] = rval(t)
                self.metadata_types[k] = t
            for _ in range(nt):
                name = rstr()
                nd = rd("<I")
                dims = [rd("<Q") for _ in range(nd)]
                gt, off = rd("<I"), rd("<Q")
                self.tensors[name] = TensorInfo(name, dims, gt, off)
                self.order.append(name)
            align = int(self.metadata.get("general.alignment", 32))
            self.data_start = pos + (align - pos % align) % align
        for t in self.tensors.values():
            t.data_offset = self.data_start + t.offset
        self._mm = np.memmap(path, dtype=np.uint8, mode="r")

    def tensor_bytes(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        return self._mm[t.data_offset:t.data_offset + t.n_bytes]
