"""Generates the GGUF golden fixtures (tests/golden/gguf_*.gguf) and their
expected parse (tests/golden/gguf_expected.json).

The expected values are what the writer put in the file, so they pin both
the oracle (oracle/gguf_ref.py) and the library (sg_gguf_*): tensor names,
shapes, types, absolute offsets (data start = end of the tensor table
rounded up to 32, swamp-gguf/src/mmap.rs:78-89), byte sizes
(dtype.rs:136-140), and metadata with the reference's rules (last value of
a repeated key, invalid UTF-8 replaced by U+FFFD).

    python tests/golden/gen_gguf.py        # rewrites the fixtures
"""
from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
import gguf_writer as gw  # noqa: E402

TYPES_BYTES = {0: (1, 4), 2: (32, 18), 12: (256, 144), 14: (256, 210), 30: (1, 2)}


def fixture_all_types():
    kv = [
        ("general.architecture", gw.STR, "llama"),
        ("u8", gw.U8, 200), ("i8", gw.I8, -100), ("u16", gw.U16, 65000), ("i16", gw.I16, -30000),
        ("u32", gw.U32, 4000000000), ("i32", gw.I32, -2000000000), ("f32", gw.F32, 1.5),
        ("bool", gw.BOOL, True), ("u64", gw.U64, 18446744073709551615), ("i64", gw.I64, -9000000000000000000),
        ("f64", gw.F64, -2.25),
        ("arr.u8", gw.ARR, (gw.U8, [1, 2, 255])), ("arr.i32", gw.ARR, (gw.I32, [-1, 0, 7])),
        ("arr.f32", gw.ARR, (gw.F32, [0.5, -0.25])), ("arr.bool", gw.ARR, (gw.BOOL, [True, False])),
        ("arr.str", gw.ARR, (gw.STR, ["a", "", "tokén"])), ("arr.empty", gw.ARR, (gw.U32, [])),
        ("arr.f64", gw.ARR, (gw.F64, [3.0])), ("arr.u64", gw.ARR, (gw.U64, [1 << 40])),
        ("dup", gw.U32, 1), ("dup", gw.STR, "second"),
        (b"bad\xffkey", gw.STR, b"v\xc3\x28\xe2\x82\x28\xf0\x28\x8c\xbc"),
    ]
    tensors = [
        ("w.q4_0", (64, 2), 2, 0),        # 2 rows x 2 blocks x 18 B = 72 B
        ("w.q4_k", (256, 2), 12, 96),     # 2 x 144 = 288 B
        ("w.q6_k", (256, 1), 14, 384),    # 210 B
        ("t.f32.3d", (3, 2, 2), 0, 608),  # 48 B
        ("w.q4_0", (32, 1), 2, 672),      # a repeated name: lookups find the first
    ]
    data = bytes((i * 37 + 11) & 0xFF for i in range(704))
    return 3, kv, tensors, data


def fixture_v1():
    kv = [("general.architecture", gw.STR, "llama"), ("v1.count", gw.U32, 7)]
    tensors = [("blk.0.attn_q.weight", (64, 4), 2, 0), ("blk.0.ffn_up.weight", (256, 2), 12, 160)]
    return 1, kv, tensors, bytes(range(256)) * 2


def fixture_v2():
    kv = [("name", gw.STR, "x" * 33)]
    tensors = [("tok_embd", (5,), 30, 0)]
    return 2, kv, tensors, b"\x01\x02" * 8


FIXTURES = {"gguf_all_types_v3": fixture_all_types, "gguf_v1": fixture_v1, "gguf_v2": fixture_v2}


def jsonable(v):
    if isinstance(v, bytes):
        return v.decode("utf-8", errors="replace")
    if isinstance(v, (list, tuple)):
        return [jsonable(e) for e in v]
    return v


def expected(version, kv, tensors, data_offset):
    last = {}
    for key, t, v in kv:
        k = jsonable(key)
        if t == gw.ARR:
            last[k] = [t, v[0], jsonable(v[1])]
        else:
            last[k] = [t, -1, jsonable(v)]
    tens = []
    for name, dims, dt, off in tensors:
        n = 1
        for d in dims:
            n *= d
        bs, bb = TYPES_BYTES[dt]
        tens.append([name, list(dims), dt, off + data_offset, (n + bs - 1) // bs * bb])
    return {"version": version, "data_offset": data_offset, "tensors": tens, "kv": last,
            "kv_order": [jsonable(k) for k, _, _ in kv]}


def images():
    out = {}
    for name, fn in FIXTURES.items():
        version, kv, tensors, data = fn()
        img, data_offset = gw.build(version, kv, tensors, data)
        out[name] = (img, expected(version, kv, tensors, data_offset))
    return out


def main():
    exp = {}
    for name, (img, e) in images().items():
        with open(os.path.join(HERE, name + ".gguf"), "wb") as f:
            f.write(img)
        exp[name] = e
    with open(os.path.join(HERE, "gguf_expected.json"), "w") as f:
        json.dump(exp, f, indent=1, sort_keys=True)
    print("wrote", ", ".join(exp))


if __name__ == "__main__":
    main()
