"""GGUF v3 reader and writer (host side of the load/upload boundary).

``GgufFile`` mirrors the reference parser's public surface
(format/GgufFile.java:51-324): ``open``, ``version``, ``tensor_count``,
``metadata``, ``tensor_infos``, ``data_offset``, ``tensor_data`` and
``find_tensor``. Fields are tightly packed little-endian values; the tensor
data section starts at ``general.alignment`` (default 32) past the last
tensor info (format/GgufFile.java:138-139). Tensor data are exposed as
zero-copy ``memoryview`` slices of an ``mmap``; the CUDA library uploads
those bytes once.

``GgufWriter`` produces files the reference parser accepts; it is used to
write seeded random-init models for the benchmark and tests.
"""
from __future__ import annotations

import mmap
import os
import struct
from dataclasses import dataclass, field

MAGIC = 0x46554747  # "GGUF" little-endian (format/GgufFile.java:54)

# format/GgufTensorType.java:15-27 (code, bytes per block-or-element, label)
TENSOR_TYPES = {
    0: (4, "F32"), 1: (2, "F16"), 2: (18, "Q4_0"), 3: (20, "Q4_1"), 6: (22, "Q5_0"),
    7: (24, "Q5_1"), 8: (34, "Q8_0"), 9: (36, "Q8_1"), 10: (84, "Q2_K"), 11: (110, "Q3_K"),
    12: (148, "Q4_K"), 13: (180, "Q5_K"), 14: (210, "Q6_K"), 15: (260, "Q8_K"),
}
F32, F16, Q4_0, Q8_0, Q6_K = 0, 1, 2, 8, 14

# format/GgufMetadataValueType.java:11-23
U8, I8, U16, I16, U32, I32, F32V, BOOL, STR, ARR, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i",
           F32V: "<f", U64: "<Q", I64: "<q", F64: "<d"}


@dataclass
class GgufTensorInfo:
    """format/GgufTensorInfo.java:10-48."""
    name: str
    dims: tuple
    type: int
    offset: int

    def num_elements(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n

    def byte_size(self) -> int:
        per, _ = TENSOR_TYPES[self.type]
        elems = self.num_elements()
        if 2 <= self.type <= 15:
            blk = 256 if self.type >= 10 else 32
            return ((elems + blk - 1) // blk) * per
        return elems * per


class GgufMetadata(dict):
    """format/GgufMetadata.java:25-49 accessors."""

    def long_or_default(self, key, default):
        v = self.get(key)
        if v is None:
            return default
        if isinstance(v, bool) or not isinstance(v, (int, float)):
            raise TypeError(f"Metadata '{key}' is not a number")
        return int(v)

    def float_or_default(self, key, default):
        v = self.get(key)
        if v is None:
            return default
        if not isinstance(v, (int, float)):
            raise TypeError(f"Metadata '{key}' is not float-like")
        return float(v)

    def string_or_default(self, key, default):
        v = self.get(key)
        return default if v is None else str(v)


class GgufFile:
    """Read-only mmapped GGUF v3 file (format/GgufFile.java:97-166)."""

    def __init__(self, path: str):
        self._f = open(path, "rb")
        size = os.fstat(self._f.fileno()).st_size
        self._mm = mmap.mmap(self._f.fileno(), size, access=mmap.ACCESS_READ) if size else b""
        self.file_length = size
        buf = memoryview(self._mm) if size else memoryview(b"")
        self._buf = buf
        if size < 24:
            self.close()
            raise IOError("Not a GGUF file: too short")
        magic, version = struct.unpack_from("<II", buf, 0)
        if magic != MAGIC:
            self.close()
            raise IOError(f"Not a GGUF file: magic=0x{magic:x}")
        if version != 3:
            self.close()
            raise IOError(f"Unsupported GGUF version: {version} (AuraTensor supports v3)")
        self.version = version
        self.tensor_count, self.metadata_kv_count = struct.unpack_from("<QQ", buf, 8)
        pos = 24
        self.metadata = GgufMetadata()
        for _ in range(self.metadata_kv_count):
            key, pos = self._read_str(pos)
            (vt,), pos = struct.unpack_from("<i", buf, pos), pos + 4
            val, pos = self._read_value(vt, pos)
            self.metadata[key] = val
        self.tensor_infos = []
        for _ in range(self.tensor_count):
            name, pos = self._read_str(pos)
            (nd,), pos = struct.unpack_from("<i", buf, pos), pos + 4
            if nd < 1 or nd > 4:
                raise ValueError(f"Unsupported rank: {nd} ({name})")
            dims = struct.unpack_from(f"<{nd}q", buf, pos)
            pos += 8 * nd
            (tcode,), pos = struct.unpack_from("<i", buf, pos), pos + 4
            if tcode not in TENSOR_TYPES:
                raise ValueError(f"Unknown GGUF tensor type code: {tcode}")
            (off,), pos = struct.unpack_from("<q", buf, pos), pos + 8
            self.tensor_infos.append(GgufTensorInfo(name, tuple(dims), tcode, off))
        align = self.metadata.long_or_default("general.alignment", 32)
        self.data_offset = ((pos + align - 1) // align) * align

    @classmethod
    def open(cls, path: str) -> "GgufFile":
        return cls(path)

    def _read_str(self, pos):
        (n,) = struct.unpack_from("<q", self._buf, pos)
        if n < 0 or n > 0x7FFFFFFF:
            raise ValueError(f"Implausible string length: {n} at offset {pos}")
        pos += 8
        return bytes(self._buf[pos:pos + n]).decode("utf-8"), pos + n

    def _read_value(self, vt, pos):
        if vt in _SCALAR:
            fmt = _SCALAR[vt]
            (v,) = struct.unpack_from(fmt, self._buf, pos)
            return v, pos + struct.calcsize(fmt)
        if vt == BOOL:
            return self._buf[pos] != 0, pos + 1
        if vt == STR:
            return self._read_str(pos)
        if vt == ARR:
            (et,) = struct.unpack_from("<i", self._buf, pos)
            (n,) = struct.unpack_from("<q", self._buf, pos + 4)
            pos += 12
            if n < 0 or n > (1 << 26):
                raise ValueError(f"Implausible array length: {n}")
            out = []
            for _ in range(n):
                v, pos = self._read_value(et, pos)
                out.append(v)
            return out, pos
        raise ValueError(f"Unknown GGUF metadata value type: {vt}")

    def find_tensor(self, name: str):
        for t in self.tensor_infos:
            if t.name == name:
                return t
        return None

    def tensor_data(self, info: GgufTensorInfo) -> memoryview:
        n = info.byte_size()
        per, label = TENSOR_TYPES[info.type]
        if n <= 0 or per < 0:
            raise NotImplementedError(f"Gguf tensor type {label} for tensor '{info.name}'")
        start = self.data_offset + info.offset
        if start + n > self.file_length:
            raise ValueError(f"tensor '{info.name}' extends past end of file")
        return self._buf[start:start + n]

    # The reference's names (format/GgufFile.java:155,319): findTensor returns
    # null for an unknown name, tensorData the tensor's bytes in the mapping.
    findTensor = find_tensor
    tensorData = tensor_data

    def close(self):
        try:
            if isinstance(self._mm, mmap.mmap):
                self._buf.release()
                self._mm.close()
        except BufferError:
            pass  # slices still exported; the map is released when they are
        finally:
            self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


@dataclass
class GgufWriter:
    """Writes a GGUF v3 file: header, metadata, tensor infos, aligned data."""
    alignment: int = 32
    metadata: list = field(default_factory=list)
    tensors: list = field(default_factory=list)

    def add_kv(self, key: str, vtype: int, value) -> None:
        self.metadata.append((key, vtype, value))

    def add_tensor(self, name: str, dims, ggml_type: int, data) -> None:
        self.tensors.append((name, tuple(int(d) for d in dims), ggml_type, data))

    @staticmethod
    def _str(s: str) -> bytes:
        b = s.encode("utf-8")
        return struct.pack("<q", len(b)) + b

    def _value(self, vt, v) -> bytes:
        if vt in _SCALAR:
            return struct.pack(_SCALAR[vt], v)
        if vt == BOOL:
            return struct.pack("<B", 1 if v else 0)
        if vt == STR:
            return self._str(v)
        if vt == ARR:
            et, items = v
            return struct.pack("<iq", et, len(items)) + b"".join(self._value(et, x) for x in items)
        raise ValueError(vt)

    def write(self, path: str) -> None:
        meta = [("general.alignment", U32, self.alignment)] + self.metadata
        head = struct.pack("<IIQQ", MAGIC, 3, len(self.tensors), len(meta))
        body = bytearray()
        for k, vt, v in meta:
            body += self._str(k) + struct.pack("<i", vt) + self._value(vt, v)
        offs, off = [], 0
        for name, dims, tt, data in self.tensors:
            off = ((off + self.alignment - 1) // self.alignment) * self.alignment
            offs.append(off)
            off += len(memoryview(data).cast("B"))
        for (name, dims, tt, data), o in zip(self.tensors, offs):
            # GGUF stores the innermost dimension first.
            body += self._str(name) + struct.pack("<i", len(dims))
            body += struct.pack(f"<{len(dims)}q", *reversed(dims)) + struct.pack("<iq", tt, o)
        with open(path, "wb") as f:
            f.write(head)
            f.write(body)
            pos = len(head) + len(body)
            pad = (-pos) % self.alignment
            f.write(b"\0" * pad)
            cur = 0
            for (name, dims, tt, data), o in zip(self.tensors, offs):
                f.write(b"\0" * (o - cur))
                mv = memoryview(data).cast("B")
                f.write(mv)
                cur = o + len(mv)
