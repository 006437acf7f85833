"""Writes GGUF files for the tests, the way the reference's own tests build them
(src/gguf.rs:436-490 build_sample/header, src/config.rs:118-192 build_gguf): little-endian
header, key/value pairs, tensor table, padding to the alignment, tensor data."""
from __future__ import annotations

import struct

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
        I64: "<q", F64: "<d"}


def gstr(s) -> bytes:
    b = s.encode() if isinstance(s, str) else bytes(s)
    return struct.pack("<Q", len(b)) + b


def value(vt: int, v) -> bytes:
    if vt == STRING:
        return gstr(v)
    if vt == ARRAY:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(value(et, x) for x in items)
    return struct.pack(_FMT[vt], v)


def kv(key: str, vt: int, v) -> bytes:
    return gstr(key) + struct.pack("<I", vt) + value(vt, v)


def tensor_entry(name: str, dims, ggml_type: int, offset: int) -> bytes:
    return gstr(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims) + \
        struct.pack("<IQ", ggml_type, offset)


def build(kvs, tensors=(), alignment: int = 32, version: int = 3) -> bytes:
    """kvs: [(key, type, value)]; tensors: [(name, dims, ggml_type, data bytes)]. Tensor data
    is placed at `alignment`-aligned offsets of the data section, in order."""
    offs, off = [], 0
    for _, _, _, data in tensors:
        offs.append(off)
        off += len(data)
        off = -(-off // alignment) * alignment if alignment else off
    head = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(kvs))
    head += b"".join(kv(*x) for x in kvs)
    head += b"".join(tensor_entry(n, d, t, o) for (n, d, t, _), o in zip(tensors, offs))
    if alignment:
        head += b"\0" * (-len(head) % alignment)
    body = bytearray()
    for (_, _, _, data), o in zip(tensors, offs):
        body += b"\0" * (o - len(body))
        body += data
    return head + bytes(body)


ATTENTION_LAYERS = (2, 6, 10, 14, 18, 21)


def model_kvs(arch="lfm2moe", block_count=24, schedule=None):
    """The metadata config::validate checks (src/config.rs:50-96), as the real file has it."""
    if schedule is None:
        schedule = [8 if i in ATTENTION_LAYERS else 0 for i in range(24)]
    ints = [("lfm2moe.block_count", block_count), ("lfm2moe.embedding_length", 2048), ("lfm2moe.vocab_size", 128000),
            ("lfm2moe.attention.head_count", 32), ("lfm2moe.expert_count", 32), ("lfm2moe.expert_used_count", 4),
            ("lfm2moe.feed_forward_length", 7168), ("lfm2moe.expert_feed_forward_length", 1792),
            ("lfm2moe.leading_dense_block_count", 2), ("lfm2moe.shortconv.l_cache", 3)]
    return [(k, U32, v) for k, v in ints] + [
        ("general.architecture", STRING, arch), ("lfm2moe.rope.freq_base", F32, 5e6),
        ("lfm2moe.attention.layer_norm_rms_epsilon", F32, 1e-5),
        ("lfm2moe.attention.head_count_kv", ARRAY, (U32, list(schedule)))]
