"""A GGUF v3 writer for test fixtures: header, typed metadata and tensor infos
as crates/beacon-format/src/tests.rs builds them (build_test_gguf), then the
tensor data at general.alignment (32 unless set)."""
from __future__ import annotations

import struct

import numpy as np

# GGUF tensor type ids (crates/beacon-format/src/gguf/types.rs:8-29)
GGUF_TYPE = {"F32": 0, "F16": 1, "Q4_0": 2, "Q4_1": 3, "Q5_0": 6, "Q5_1": 7, "Q8_0": 8, "Q2_K": 10, "Q3_K": 11,
             "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "Q8_K": 15}
# metadata value types (types.rs:124-158)
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, v) -> bytes:
    if vtype == STRING:
        return _str(v)
    if vtype == ARRAY:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, x) for x in items)
    fmt = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
           I64: "<q", F64: "<d"}[vtype]
    return struct.pack(fmt, v)


class GgufBuilder:
    def __init__(self, version: int = 3, alignment: int = 32, pad_tensors: bool = True):
        self.version = version
        self.alignment = alignment
        self.pad_tensors = pad_tensors  # False: tensors back to back, as build_test_gguf writes them
        self.kv: list[tuple[str, int, object]] = []
        self.tensors: list[tuple[str, tuple, int, bytes]] = []

    def add_kv(self, key: str, vtype: int, value) -> "GgufBuilder":
        self.kv.append((key, vtype, value))
        return self

    def add_tensor(self, name: str, shape_row_major, gguf_type: str, data) -> "GgufBuilder":
        """shape in row-major order ([N, K]); written reversed, as GGUF stores dims."""
        self.tensors.append((name, tuple(shape_row_major), GGUF_TYPE[gguf_type],
                             np.ascontiguousarray(data).view(np.uint8).tobytes()))
        return self

    def build(self) -> bytes:
        out = bytearray(b"GGUF")
        out += struct.pack("<IQQ", self.version, len(self.tensors), len(self.kv))
        for key, vt, v in self.kv:
            out += _str(key) + struct.pack("<I", vt) + _value(vt, v)
        offset, blobs = 0, []
        for name, shape, t, blob in self.tensors:
            out += _str(name) + struct.pack("<I", len(shape))
            out += b"".join(struct.pack("<Q", d) for d in reversed(shape))
            out += struct.pack("<IQ", t, offset)
            pad = (-len(blob)) % self.alignment if self.pad_tensors else 0
            blobs.append(blob + bytes(pad))
            offset += len(blob) + pad
        out += bytes((-len(out)) % self.alignment)
        for b in blobs:
            out += b
        return bytes(out)

    def write(self, path) -> str:
        with open(path, "wb") as f:
            f.write(self.build())
        return str(path)


def llama_kv(b: GgufBuilder, hidden: int, layers: int, heads: int, kv_heads: int, ffn: int, vocab: int,
             ctx: int = 512, theta: float = 10000.0, eps: float = 1e-5) -> GgufBuilder:
    """The metadata of a Llama-architecture file (config_map.rs keys)."""
    b.add_kv("general.architecture", STRING, "llama")
    b.add_kv("llama.embedding_length", U32, hidden)
    b.add_kv("llama.block_count", U32, layers)
    b.add_kv("llama.attention.head_count", U32, heads)
    b.add_kv("llama.attention.head_count_kv", U32, kv_heads)
    b.add_kv("llama.feed_forward_length", U32, ffn)
    b.add_kv("llama.context_length", U32, ctx)
    b.add_kv("llama.rope.freq_base", F32, theta)
    b.add_kv("llama.attention.layer_norm_rms_epsilon", F32, eps)
    b.add_kv("llama.vocab_size", U32, vocab)
    return b
