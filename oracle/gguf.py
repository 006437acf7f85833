"""CPU restatement of the reference's GGUF reader — TEST INFRASTRUCTURE ONLY.

Follows ``src/gguf.rs`` of maximecb/bebelm step by step: ``parse`` (:301-341),
``read_value`` (:343-370), the little-endian bounds-checked ``Reader`` (:381-432),
``align_up`` (:372-378) and the ggml block table of ``src/tensor.rs:68-106``.
Plain Python over ``bytes`` (integers never overflow here, so element counts are the
mathematical products); it is the checker for the library's native reader
(``bebelm_gguf_*``) and is never called by the product.

``parse`` returns a dict (version, alignment, metadata, tensors, data_offset) or
raises :class:`GgufError` whose ``kind`` is the name of the reference's
``GgufError`` variant.
"""
from __future__ import annotations

import struct

DEFAULT_ALIGNMENT = 32  # src/gguf.rs:18

# src/tensor.rs:68-99: ggml type id -> (elements per block, bytes per block)
BLOCKS = {0: (1, 4), 1: (1, 2), 30: (1, 2), 28: (1, 8), 24: (1, 1), 25: (1, 2), 26: (1, 4), 27: (1, 8),
          2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 9: (32, 36),
          10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210), 15: (256, 292)}

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)  # src/gguf.rs:64-78


class GgufError(Exception):
    def __init__(self, kind: str, detail=None):
        super().__init__(f"{kind}: {detail}")
        self.kind = kind
        self.detail = detail


def byte_size(ty: int, n_elements: int):
    """GgmlType::byte_size (src/tensor.rs:101-106): None if unmodeled or not whole blocks."""
    b = BLOCKS.get(ty)
    if b is None or n_elements % b[0]:
        return None
    return n_elements // b[0] * b[1]


class _Reader:
    def __init__(self, buf: bytes):
        self.buf, self.pos = buf, 0

    def take(self, n: int) -> bytes:
        if self.pos + n > len(self.buf):
            raise GgufError("UnexpectedEof", (n, self.pos, len(self.buf)))
        s = self.buf[self.pos:self.pos + n]
        self.pos += n
        return s

    def unpack(self, fmt: str):
        return struct.unpack(fmt, self.take(struct.calcsize(fmt)))[0]

    def string(self) -> str:
        n = self.unpack("<Q")
        b = self.take(n)
        try:
            return b.decode("utf-8", errors="strict")
        except UnicodeDecodeError:
            raise GgufError("InvalidUtf8") from None


_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", U64: "<Q", I64: "<q", F64: "<d"}


def _value_type(v: int) -> int:
    if v > F64:
        raise GgufError("UnknownValueType", v)
    return v


def _read_value(r: _Reader, vt: int):
    """Returns (type, value); arrays are (ARRAY, (elem_type, [items]))."""
    if vt in _FMT:
        return vt, r.unpack(_FMT[vt])
    if vt == BOOL:
        return vt, r.unpack("<B") != 0
    if vt == STRING:
        return vt, r.string()
    et = _value_type(r.unpack("<I"))
    n = r.unpack("<Q")
    items = [_read_value(r, et)[1] for _ in range(n)]
    return vt, (et, items)


def _align_up(x: int, a: int) -> int:
    return x if a == 0 else -(-x // a) * a


def parse(buf: bytes) -> dict:
    r = _Reader(bytes(buf))
    magic = r.take(4)
    if magic != b"GGUF":
        raise GgufError("BadMagic", list(magic))
    version = r.unpack("<I")
    if version not in (2, 3):
        raise GgufError("UnsupportedVersion", version)
    tensor_count = r.unpack("<Q")
    kv_count = r.unpack("<Q")
    metadata = {}
    for _ in range(kv_count):
        key = r.string()
        vt = _value_type(r.unpack("<I"))
        metadata[key] = _read_value(r, vt)
    al = metadata.get("general.alignment")
    alignment = al[1] if al is not None and al[0] in (U32, U64) else DEFAULT_ALIGNMENT
    raw = []
    for _ in range(tensor_count):
        name = r.string()
        n_dims = r.unpack("<I")
        dims = [r.unpack("<Q") for _ in range(n_dims)]
        ty = r.unpack("<I")
        off = r.unpack("<Q")
        raw.append((name, dims, ty, off))
    data_offset = _align_up(r.pos, alignment)
    tensors = []
    for name, dims, ty, off in raw:
        n = 1
        for d in dims:
            n *= d
        nbytes = byte_size(ty, n)
        if nbytes is None:
            raise GgufError("UnknownTensorType", (name, ty))
        start = data_offset + off
        if start + nbytes > len(buf):
            raise GgufError("TensorOutOfBounds", name)
        tensors.append({"name": name, "dims": dims, "ggml_type": ty, "offset": off, "data_start": start,
                        "data_len": nbytes, "n_elements": n})
    return {"version": version, "alignment": alignment, "metadata": metadata, "tensors": tensors,
            "data_offset": data_offset}
