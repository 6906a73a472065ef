"""GGUF v3 container: a small reader and writer for the loader seam.

The reference reads GGUF in core/gguf (header/metadata/tensor index, src/reader.rs) and
sizes tensors with the type table of core/gguf/src/tensor.rs:18-57. Only what the decode
layer needs is here: metadata values, the tensor index and memory-mapped tensor bytes.
Layout (GGUF v3): magic "GGUF", u32 version, u64 tensor count, u64 metadata count, the
metadata key/values, the tensor infos (name, dims innermost-first, type, offset), then the
data section aligned to `general.alignment` (32 by default).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass

import numpy as np

MAGIC = 0x46554747
VERSION = 3
ALIGN = 32

(T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64) = range(13)
_SCALAR = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f",
           T_BOOL: "<?", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}

# ggml type id -> (name, elements per block, bytes per block)
GGML_TYPES = {0: ("F32", 1, 4), 1: ("F16", 1, 2), 12: ("Q4_K", 256, 144), 14: ("Q6_K", 256, 210)}


def tensor_nbytes(ggml_type: int, n_elements: int) -> int:
    name, be, bb = GGML_TYPES[ggml_type]
    if n_elements % be:
        raise ValueError(f"{n_elements} elements is not a whole number of {name} blocks")
    return n_elements // be * bb


@dataclass
class TensorInfo:
    name: str
    ne: tuple            # ggml dims, innermost first
    type: int
    offset: int          # from the start of the data section
    data: np.ndarray | None = None  # uint8 view of the bytes

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.ne:
            n *= d
        return n

    @property
    def nbytes(self) -> int:
        return tensor_nbytes(self.type, self.n_elements)


class GGUFReader:
    def __init__(self, path: str):
        self.path = path
        self.mm = np.memmap(path, dtype=np.uint8, mode="r")
        self.pos = 0
        magic, version = self._u("<I"), self._u("<I")
        if magic != MAGIC:
            raise ValueError(f"{path}: not a GGUF file")
        if version != VERSION:
            raise ValueError(f"{path}: GGUF version {version} (this reader handles 3)")
        n_t, n_kv = self._u("<Q"), self._u("<Q")
        self.metadata: dict = {}
        for _ in range(n_kv):
            key = self._str()
            self.metadata[key] = self._value(self._u("<I"))
        self.tensors: dict[str, TensorInfo] = {}
        for _ in range(n_t):
            name = self._str()
            nd = self._u("<I")
            ne = tuple(self._u("<Q") for _ in range(nd))
            ty = self._u("<I")
            off = self._u("<Q")
            self.tensors[name] = TensorInfo(name, ne, ty, off)
        align = int(self.metadata.get("general.alignment", ALIGN))
        start = (self.pos + align - 1) // align * align
        for t in self.tensors.values():
            t.data = self.mm[start + t.offset: start + t.offset + t.nbytes]

    def _u(self, fmt):
        n = struct.calcsize(fmt)
        v = struct.unpack_from(fmt, self.mm, self.pos)[0]
        self.pos += n
        return v

    def _str(self):
        n = self._u("<Q")
        s = bytes(self.mm[self.pos:self.pos + n]).decode()
        self.pos += n
        return s

    def _value(self, ty):
        if ty in _SCALAR:
            return self._u(_SCALAR[ty])
        if ty == T_STR:
            return self._str()
        if ty == T_ARR:
            et, n = self._u("<I"), self._u("<Q")
            return [self._value(et) for _ in range(n)]
        raise ValueError(f"unknown metadata type {ty}")

    def arch(self) -> str:
        return self.metadata["general.architecture"]

    def arch_value(self, suffix, default=None):
        return self.metadata.get(f"{self.arch()}.{suffix}", default)


class GGUFWriter:
    def __init__(self, path: str):
        self.path = path
        self.kv: list[tuple[str, int, object]] = []
        self.tensors: list[tuple[str, tuple, int, np.ndarray]] = []

    def add(self, key: str, value, ty: int | None = None):
        if ty is None:
            if isinstance(value, str):
                ty = T_STR
            elif isinstance(value, bool):
                ty = T_BOOL
            elif isinstance(value, int):
                ty = T_U32 if 0 <= value < 2 ** 32 else T_I64
            elif isinstance(value, float):
                ty = T_F32
            else:
                raise TypeError(f"cannot infer the GGUF type of {key}")
        self.kv.append((key, ty, value))

    def add_tensor(self, name: str, ne: tuple, ggml_type: int, data: np.ndarray):
        data = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
        n = 1
        for d in ne:
            n *= d
        if data.size != tensor_nbytes(ggml_type, n):
            raise ValueError(f"{name}: {data.size} bytes do not match dims {ne}")
        self.tensors.append((name, tuple(ne), ggml_type, data))

    @staticmethod
    def _s(s: str) -> bytes:
        b = s.encode()
        return struct.pack("<Q", len(b)) + b

    def _v(self, ty, v) -> bytes:
        if ty in _SCALAR:
            return struct.pack(_SCALAR[ty], v)
        if ty == T_STR:
            return self._s(v)
        raise TypeError("arrays are not written by this writer")

    def write(self):
        head = bytearray(struct.pack("<IIQQ", MAGIC, VERSION, len(self.tensors), len(self.kv)))
        for k, ty, v in self.kv:
            head += self._s(k) + struct.pack("<I", ty) + self._v(ty, v)
        off = 0
        offsets = []
        for name, ne, ty, data in self.tensors:
            offsets.append(off)
            head += self._s(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", d) for d in ne)
            head += struct.pack("<IQ", ty, off)
            off += (data.size + ALIGN - 1) // ALIGN * ALIGN
        pad = (-len(head)) % ALIGN
        with open(self.path, "wb") as f:
            f.write(head + b"\0" * pad)
            for (name, ne, ty, data), o in zip(self.tensors, offsets):
                f.write(data.tobytes())
                f.write(b"\0" * ((-data.size) % ALIGN))
