"""Test infrastructure only: a plain-Python restatement of the reference's
GGUF reader (swamp-gguf), the checker for the library's sg_gguf_* entry
points. Nothing on the product path imports it.

Follows, line by line:
  swamp-gguf/src/mmap.rs:33-91      GgufFile::parse (header, KV, tensor table,
                                     32-byte data alignment, absolute offsets)
  swamp-gguf/src/mmap.rs:111-118    tensor_raw_bytes (range check at access)
  swamp-gguf/src/metadata.rs:118-194 Reader (little-endian reads, u64-length
                                     strings decoded with from_utf8_lossy)
  swamp-gguf/src/metadata.rs:197-236 parse_metadata_value / _array
  swamp-gguf/src/dtype.rs:43-140    type ids, block sizes and block bytes
  swamp-gguf/src/tensor_info.rs:18-26 n_elems / nbytes
Errors are raised as GgufRefError with the reference's error kind
(error.rs): InvalidMagic, UnsupportedVersion, UnknownDType, Io (unexpected
end of file), InvalidTensor.
"""
from __future__ import annotations

import struct

ALIGN = 32  # mmap.rs:14 GGUF_ALIGNMENT
M64 = (1 << 64) - 1

# dtype.rs:43-75 (id -> (block size, block bytes)), dtype.rs:78-134
TYPES = {
    0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 9: (32, 40),
    10: (256, 84), 11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210), 15: (256, 292),
    16: (256, 66), 17: (256, 74), 18: (256, 98), 19: (256, 50), 20: (32, 18), 21: (256, 110), 22: (256, 82),
    23: (32, 136), 24: (1, 1), 25: (1, 2), 26: (1, 4), 27: (1, 8), 28: (1, 8), 29: (256, 56), 30: (1, 2),
}


class GgufRefError(Exception):
    def __init__(self, kind: str, detail: str = ""):
        super().__init__(f"{kind}: {detail}")
        self.kind = kind


class _Reader:
    """metadata.rs:118-194"""

    def __init__(self, data: bytes):
        self.d, self.pos = data, 0

    def take(self, n: int, what: str) -> bytes:
        if n > len(self.d) - self.pos:
            raise GgufRefError("Io", f"UnexpectedEof {what}")
        b = self.d[self.pos:self.pos + n]
        self.pos += n
        return b

    def u(self, n: int, what: str) -> int:
        return int.from_bytes(self.take(n, what), "little")

    def string(self) -> str:  # metadata.rs:185-191
        n = self.u(8, "read_u64")
        if n > len(self.d) - self.pos:
            raise GgufRefError("Io", "UnexpectedEof read_string")
        return self.take(n, "read_string").decode("utf-8", errors="replace")


def _value(r: _Reader, t: int):
    """metadata.rs:197-219 (one scalar value of type t)"""
    if t == 0:
        return r.u(1, "read_u8")
    if t == 1:
        return struct.unpack("<b", r.take(1, "read_u8"))[0]
    if t == 2:
        return r.u(2, "read_u16")
    if t == 3:
        return struct.unpack("<h", r.take(2, "read_u16"))[0]
    if t == 4:
        return r.u(4, "read_u32")
    if t == 5:
        return struct.unpack("<i", r.take(4, "read_u32"))[0]
    if t == 6:
        return struct.unpack("<f", r.take(4, "read_u32"))[0]
    if t == 7:
        return r.u(1, "read_u8") != 0
    if t == 8:
        return r.string()
    if t == 10:
        return r.u(8, "read_u64")
    if t == 11:
        return struct.unpack("<q", r.take(8, "read_u64"))[0]
    if t == 12:
        return struct.unpack("<d", r.take(8, "read_u64"))[0]
    raise GgufRefError("UnknownDType", str(t))


def parse(data: bytes) -> dict:
    """GgufFile::parse (mmap.rs:33-91). Returns {version, kv: {key: (type,
    elem_type, value)}, kv_order, tensors: [(name, shape, dtype, offset,
    nbytes)], data_offset}; offsets are absolute in the file."""
    r = _Reader(data)
    magic = r.take(4, "read_bytes")
    if magic != b"GGUF":
        raise GgufRefError("InvalidMagic", repr(magic))
    version = r.u(4, "read_u32")
    if version < 1 or version > 3:
        raise GgufRefError("UnsupportedVersion", str(version))
    cw = 8 if version >= 2 else 4
    n_t = r.u(cw, "count")
    n_kv = r.u(cw, "count")
    kv, order = {}, []
    for _ in range(n_kv):
        key = r.string()
        vt = r.u(4, "read_u32")
        if vt == 9:  # metadata.rs:208-214
            et = r.u(4, "read_u32")
            cnt = r.u(8, "read_u64")
            if et == 9 or et not in (0, 1, 2, 3, 4, 5, 6, 7, 8, 10, 11, 12):
                raise GgufRefError("UnknownDType", str(et))
            val = [_value(r, et) for _ in range(cnt)]
            kv[key] = (9, et, val)
        else:
            kv[key] = (vt, -1, _value(r, vt))
        order.append(key)
    tensors = []
    for _ in range(n_t):
        name = r.string()
        nd = r.u(4, "read_u32")
        shape = tuple(r.u(cw, "dim") for _ in range(nd))
        dt = r.u(4, "read_u32")
        if dt not in TYPES:
            raise GgufRefError("UnknownDType", str(dt))
        off = r.u(8, "read_u64")
        n = 1
        for d in shape:  # tensor_info.rs:19-21, u64 wrapping as in a release build
            n = (n * d) & M64
        bs, bb = TYPES[dt]
        nbytes = ((((n + bs - 1) & M64) // bs) * bb) & M64  # dtype.rs:136-140
        tensors.append([name, shape, dt, off, nbytes])
    data_offset = (r.pos + ALIGN - 1) // ALIGN * ALIGN  # mmap.rs:78-81
    for t in tensors:  # mmap.rs:84-89
        t[3] = (t[3] + data_offset) & M64
    return {"version": version, "kv": kv, "kv_order": order, "tensors": [tuple(t) for t in tensors],
            "data_offset": data_offset}


def tensor_raw_bytes(data: bytes, tensor: tuple) -> bytes:
    """mmap.rs:111-118: the tensor's bytes, or InvalidTensor when the range
    leaves the file."""
    _, _, _, off, nbytes = tensor
    if off > len(data) or nbytes > len(data) - off:
        raise GgufRefError("InvalidTensor", f"range {off}..{off + nbytes} outside {len(data)}")
    return data[off:off + nbytes]
