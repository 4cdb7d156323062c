"""A GGUF v2/v3 writer for tests: builds files with chosen metadata and tensors, and the raw
pieces to build malformed ones.

Follows the public layout of the format (ggml's gguf.h): "GGUF", u32 version, u64 tensor count,
u64 key/value count, the key/value pairs (string key, u32 value type, value), the tensor index
(string name, u32 rank, u64 dims fastest-varying first, u32 ggml type, u64 offset into the data
blob), padding to the alignment, the data blob with every tensor at an aligned offset. Strings
are a u64 length and the bytes; everything little-endian.
"""
from __future__ import annotations

import struct

# value types (gguf.h enum gguf_type)
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B",
        U64: "<Q", I64: "<q", F64: "<d"}


def gstr(s: str | bytes) -> bytes:
    b = s.encode() if isinstance(s, str) else s
    return struct.pack("<Q", len(b)) + b


def value(vtype: int, v) -> bytes:
    if vtype == STRING:
        return gstr(v)
    if vtype == ARRAY:
        elem, items = v
        out = struct.pack("<IQ", elem, len(items))
        return out + b"".join(value(elem, x) for x in items)
    return struct.pack(_FMT[vtype], int(v) if vtype not in (F32, F64) else v)


def kv(key: str, vtype: int, v) -> bytes:
    return gstr(key) + struct.pack("<I", vtype) + value(vtype, v)


def tensor_info(name: str, dims, type_id: int, offset: int) -> bytes:
    return gstr(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims) + \
        struct.pack("<IQ", type_id, offset)


def pad(n: int, a: int) -> int:
    return (n + a - 1) // a * a


class GgufWriter:
    def __init__(self, version: int = 3, alignment: int | None = None):
        self.version = version
        self.alignment = alignment or 32
        self.kvs: list[bytes] = []
        self.tensors: list[tuple[str, tuple, int, bytes]] = []
        if alignment is not None:
            self.add("general.alignment", U32, alignment)

    def add(self, key: str, vtype: int, v) -> "GgufWriter":
        self.kvs.append(kv(key, vtype, v))
        return self

    def add_tensor(self, name: str, dims, type_id: int, data: bytes) -> "GgufWriter":
        self.tensors.append((name, tuple(dims), type_id, bytes(data)))
        return self

    def build(self) -> tuple[bytes, int, list[int]]:
        """The file's bytes, the data blob's offset and each tensor's offset in the blob."""
        offs, o = [], 0
        for _, _, _, data in self.tensors:
            offs.append(o)
            o = pad(o + len(data), self.alignment)
        head = b"GGUF" + struct.pack("<IQQ", self.version, len(self.tensors), len(self.kvs))
        head += b"".join(self.kvs)
        head += b"".join(tensor_info(n, d, t, off) for (n, d, t, _), off in zip(self.tensors, offs))
        data_off = pad(len(head), self.alignment)
        blob = bytearray()
        for (_, _, _, data), off in zip(self.tensors, offs):
            blob += b"\0" * (off - len(blob)) + data
        blob += b"\0" * (pad(len(blob), self.alignment) - len(blob))
        return head + b"\0" * (data_off - len(head)) + bytes(blob), data_off, offs

    def write(self, path) -> tuple[int, list[int]]:
        raw, data_off, offs = self.build()
        with open(path, "wb") as f:
            f.write(raw)
        return data_off, offs
