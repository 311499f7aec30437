"""Builds GGUF file images for the tests (version 1..3 as the reference reads
them: u32 counts and dimensions in version 1, u64 from version 2, u64 string
lengths in every version; tensor data at the end of the tensor table rounded
up to 32 bytes, swamp-gguf/src/mmap.rs:33-91)."""
from __future__ import annotations

import struct

import numpy as np

# GGUF metadata value types (swamp-gguf/src/metadata.rs:197-219)
U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", U64: "<Q", I64: "<q",
           F64: "<d"}


def _s(b: bytes) -> bytes:
    return struct.pack("<Q", len(b)) + b


def _val(t: int, v) -> bytes:
    if t == BOOL:
        return struct.pack("<B", 1 if v else 0)
    if t == STR:
        return _s(v if isinstance(v, bytes) else v.encode())
    return struct.pack(_SCALAR[t], v)


def build(version: int = 3, kv=(), tensors=(), data: bytes | None = None, pad_to_data: bool = True) -> tuple:
    """kv: [(key, type, value)] with value a list for ARR as (elem_type, list);
    tensors: [(name, dims, dtype, relative offset)]. Returns (image, data
    offset)."""
    cw = "<Q" if version >= 2 else "<I"
    out = bytearray(b"GGUF" + struct.pack("<I", version) + struct.pack(cw, len(tensors)) + struct.pack(cw, len(kv)))
    for key, t, v in kv:
        out += _s(key if isinstance(key, bytes) else key.encode()) + struct.pack("<I", t)
        if t == ARR:
            et, vals = v
            out += struct.pack("<I", et) + struct.pack("<Q", len(vals))
            for e in vals:
                out += _val(et, e)
        else:
            out += _val(t, v)
    for name, dims, dt, off in tensors:
        out += _s(name if isinstance(name, bytes) else name.encode()) + struct.pack("<I", len(dims))
        for d in dims:
            out += struct.pack(cw, d)
        out += struct.pack("<I", dt) + struct.pack("<Q", off)
    data_offset = (len(out) + 31) // 32 * 32
    if pad_to_data:
        out += b"\0" * (data_offset - len(out))
    if data:
        out += data
    return bytes(out), data_offset


def model_file(weights: dict, version: int = 3, extra_kv=()) -> tuple:
    """A GGUF image holding raw Q4_0/Q4_K blocks: weights maps name ->
    (dtype, n_rows, n_cols, block bytes). Tensors are laid out in order, each
    at a 32-byte aligned relative offset. Returns (image, {name: relative
    offset})."""
    blob = bytearray()
    tens, offs = [], {}
    for name, (dt, n_rows, n_cols, raw) in weights.items():
        off = (len(blob) + 31) // 32 * 32
        blob += b"\0" * (off - len(blob))
        blob += np.ascontiguousarray(raw, np.uint8).tobytes()
        tens.append((name, (n_cols, n_rows), dt, off))
        offs[name] = off
    kv = [("general.architecture", STR, "llama"), ("general.alignment", U32, 32)] + list(extra_kv)
    img, _ = build(version, kv, tens, bytes(blob))
    return img, offs
