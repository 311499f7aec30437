"""GGUF reader (sg_gguf_*, host-only) against the reference's rules.

The oracle (oracle/gguf_ref.py, a restatement of swamp-gguf/src/mmap.rs:33-91
and metadata.rs) and the library must both reproduce the golden fixtures
(tests/golden/gen_gguf.py: the expected parse is what the writer wrote), and
agree with each other on generated files, every truncation of a file, and
the reference's error cases.
"""
import json
import os
import random
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
sys.path.insert(0, os.path.join(HERE, "..", "oracle"))
sys.path.insert(0, os.path.join(HERE, "..", "llamanyon.rs_b200"))

import gen_gguf  # noqa: E402
import gguf_ref  # noqa: E402
import gguf_writer as gw  # noqa: E402
import swamp_gpu as sg  # noqa: E402

GOLDEN = os.path.join(HERE, "golden")


@pytest.fixture(scope="module")
def lib():
    return sg.load_library()


def lib_parse(lib, img: bytes) -> dict:
    f = sg.GgufFile(lib, data=img)
    try:
        kv = {}
        order = []
        for i in range(f.n_kv):
            key, val, t, et = f.kv_at(i)
            kv[key] = [t, et, val]
            order.append(key)
        return {"version": f.version, "data_offset": f.data_offset,
                "tensors": [[t.name, list(t.shape), t.dtype, t.offset, t.nbytes] for t in f.tensors],
                "kv": kv, "kv_order": order}
    finally:
        f.close()


def ref_parse(img: bytes) -> dict:
    p = gguf_ref.parse(img)
    kv = {k: [t, et, v] for k, (t, et, v) in p["kv"].items()}
    return {"version": p["version"], "data_offset": p["data_offset"],
            "tensors": [[n, list(s), d, o, b] for n, s, d, o, b in p["tensors"]], "kv": kv, "kv_order": p["kv_order"]}


def last_values(parsed: dict) -> dict:
    """the library lists every occurrence; a lookup returns the last one"""
    return {k: v for k, v in parsed["kv"].items()}


def test_golden_fixtures_are_the_generator_output():
    for name, (img, exp) in gen_gguf.images().items():
        with open(os.path.join(GOLDEN, name + ".gguf"), "rb") as f:
            assert f.read() == img, name
    with open(os.path.join(GOLDEN, "gguf_expected.json")) as f:
        saved = json.load(f)
    assert saved == json.loads(json.dumps({n: e for n, (_, e) in gen_gguf.images().items()}))


@pytest.mark.parametrize("name", sorted(gen_gguf.FIXTURES))
def test_golden_oracle_and_library(lib, name):
    with open(os.path.join(GOLDEN, name + ".gguf"), "rb") as f:
        img = f.read()
    with open(os.path.join(GOLDEN, "gguf_expected.json")) as f:
        exp = json.load(f)[name]
    for got in (ref_parse(img), lib_parse(lib, img)):
        assert got["version"] == exp["version"]
        assert got["data_offset"] == exp["data_offset"]
        assert got["tensors"] == exp["tensors"]
        assert got["kv_order"] == exp["kv_order"]
        assert json.loads(json.dumps(last_values(got))) == exp["kv"]


def test_library_lookups_follow_the_reference(lib):
    with open(os.path.join(GOLDEN, "gguf_all_types_v3.gguf"), "rb") as f:
        img = f.read()
    ref = gguf_ref.parse(img)
    f = sg.GgufFile(lib, data=img)
    try:
        # GgufFile::tensor: the first tensor of that name (mmap.rs:95-98)
        t = f.tensor("w.q4_0")
        assert t.index == 0 and t.shape == (64, 2)
        with pytest.raises(sg.SwampGpuError) as e:
            f.tensor("missing")
        assert e.value.code == sg.SG_ERR_NOT_FOUND
        # a repeated key keeps its last value (HashMap insert, mmap.rs:53-58)
        assert f.kv("dup") == "second"
        assert f.kv("u64") == 18446744073709551615 and f.kv("i64") == -9000000000000000000
        assert f.kv("arr.str") == ["a", "", "tokén"] and f.kv("arr.empty") == []
        with pytest.raises(sg.SwampGpuError) as e:
            f.kv("nope")
        assert e.value.code == sg.SG_ERR_NOT_FOUND
        for i, tr in enumerate(ref["tensors"]):
            assert f.tensor_raw_bytes(f.tensors[i]) == gguf_ref.tensor_raw_bytes(img, tr)
    finally:
        f.close()


def test_open_from_path(lib, tmp_path):
    with open(os.path.join(GOLDEN, "gguf_v1.gguf"), "rb") as f:
        img = f.read()
    p = tmp_path / "m.gguf"
    p.write_bytes(img)
    f = sg.GgufFile(lib, path=str(p))
    try:
        assert f.file_size == len(img) and f.version == 1
        assert [t.name for t in f.tensors] == ["blk.0.attn_q.weight", "blk.0.ffn_up.weight"]
        assert f.tensor_raw_bytes(f.tensors[1]) == gguf_ref.tensor_raw_bytes(img, gguf_ref.parse(img)["tensors"][1])
    finally:
        f.close()
    with pytest.raises(sg.SwampGpuError):
        sg.GgufFile(lib, path=str(tmp_path / "absent.gguf"))


def _outcome(fn):
    try:
        return ("ok", fn())
    except gguf_ref.GgufRefError as e:
        return ("err", e.kind)
    except sg.SwampGpuError as e:
        return ("err", e.code)


def test_every_truncation_agrees(lib):
    """Each prefix of a file either parses identically in both or fails in
    both (unexpected end of file)."""
    for name in sorted(gen_gguf.FIXTURES):
        with open(os.path.join(GOLDEN, name + ".gguf"), "rb") as f:
            img = f.read()
        for n in range(len(img) + 1):
            a = _outcome(lambda: ref_parse(img[:n]))
            b = _outcome(lambda: lib_parse(lib, img[:n]))
            assert a[0] == b[0], (name, n, a, b)
            if a[0] == "ok":
                assert a[1] == b[1], (name, n)
            else:
                assert b[1] == sg.SG_ERR_FORMAT


@pytest.mark.parametrize("img,kind", [
    (b"GGU", "Io"),
    (b"GGUX" + b"\3\0\0\0" + b"\0" * 16, "InvalidMagic"),
    (b"GGUF" + b"\0\0\0\0" + b"\0" * 16, "UnsupportedVersion"),
    (b"GGUF" + b"\4\0\0\0" + b"\0" * 16, "UnsupportedVersion"),
    (gw.build(3, [], [("t", (4,), 4, 0)])[0], "UnknownDType"),  # type 4 is not a ggml type
    (gw.build(3, [], [("t", (4,), 31, 0)])[0], "UnknownDType"),
])
def test_reference_error_cases(lib, img, kind):
    with pytest.raises(gguf_ref.GgufRefError) as e:
        gguf_ref.parse(img)
    assert e.value.kind == kind
    with pytest.raises(sg.SwampGpuError) as e2:
        sg.GgufFile(lib, data=img)
    assert e2.value.code == sg.SG_ERR_FORMAT


def _raw_kv(key: bytes, t: int, payload: bytes) -> bytes:
    import struct
    return struct.pack("<Q", len(key)) + key + struct.pack("<I", t) + payload


def test_unknown_metadata_types(lib):
    import struct
    head = b"GGUF" + struct.pack("<IQQ", 3, 0, 1)
    for payload in (_raw_kv(b"k", 13, b"\0" * 8),                                  # no such value type
                    _raw_kv(b"k", 9, struct.pack("<IQ", 9, 1) + b"\0" * 32),       # array of arrays
                    _raw_kv(b"k", 9, struct.pack("<IQ", 13, 1) + b"\0" * 8)):      # array of an unknown type
        img = head + payload
        with pytest.raises(gguf_ref.GgufRefError) as e:
            gguf_ref.parse(img)
        assert e.value.kind == "UnknownDType"
        with pytest.raises(sg.SwampGpuError) as e2:
            sg.GgufFile(lib, data=img)
        assert e2.value.code == sg.SG_ERR_FORMAT


def test_tensor_range_is_checked_on_access(lib):
    """A tensor whose bytes leave the file still parses (mmap.rs:84-89); its
    data access fails (mmap.rs:111-118)."""
    img, _ = gw.build(3, [], [("w", (64, 4), 2, 0), ("big", ((1 << 40) + 1, 1 << 30), 0, 0)], b"\0" * 144)
    ref = gguf_ref.parse(img)
    f = sg.GgufFile(lib, data=img)
    try:
        assert [t.nbytes for t in f.tensors] == [t[4] for t in ref["tensors"]]  # the second wraps in u64
        assert f.tensor_raw_bytes(f.tensors[0]) == gguf_ref.tensor_raw_bytes(img, ref["tensors"][0])
        with pytest.raises(gguf_ref.GgufRefError):
            gguf_ref.tensor_raw_bytes(img, ref["tensors"][1])
        with pytest.raises(sg.SwampGpuError) as e:
            f.tensor_raw_bytes(f.tensors[1])
        assert e.value.code == sg.SG_ERR_FORMAT
    finally:
        f.close()


def test_utf8_replacement_matches(lib):
    """Keys, string values and tensor names: invalid UTF-8 is replaced as
    Rust's from_utf8_lossy does, on random byte strings."""
    rng = random.Random(1234)
    pieces = [b"\xff", b"\xc3", b"\xc3\xa9", b"\xe2\x82", b"\xe2\x82\xac", b"\xed\xa0\x80", b"\xf0\x9f\x98\x80",
              b"\xf0\x9f", b"\xf4\x90\x80\x80", b"\x80", b"a", b"\xc0\xaf", b"\xe0\x80\xaf", b"\xf5"]
    for _ in range(200):
        s = b"".join(rng.choice(pieces) for _ in range(rng.randint(0, 8)))
        img, _ = gw.build(3, [(s, gw.STR, s), ("a", gw.ARR, (gw.STR, [s, s[:1]]))], [(s, (32,), 2, 0)], b"\0" * 32)
        a, b = ref_parse(img), lib_parse(lib, img)
        assert a == b, s


def test_random_files_agree(lib):
    rng = np.random.default_rng(7)
    types = [gw.U8, gw.I8, gw.U16, gw.I16, gw.U32, gw.I32, gw.F32, gw.BOOL, gw.STR, gw.U64, gw.I64, gw.F64]
    rand = {gw.U8: lambda: int(rng.integers(0, 256)), gw.I8: lambda: int(rng.integers(-128, 128)),
            gw.U16: lambda: int(rng.integers(0, 1 << 16)), gw.I16: lambda: int(rng.integers(-(1 << 15), 1 << 15)),
            gw.U32: lambda: int(rng.integers(0, 1 << 32)), gw.I32: lambda: int(rng.integers(-(1 << 31), 1 << 31)),
            gw.F32: lambda: float(np.float32(rng.standard_normal())), gw.BOOL: lambda: bool(rng.integers(0, 2)),
            gw.STR: lambda: "s" * int(rng.integers(0, 40)), gw.U64: lambda: int(rng.integers(0, 1 << 63)) * 2 + 1,
            gw.I64: lambda: int(rng.integers(-(1 << 62), 1 << 62)), gw.F64: lambda: float(rng.standard_normal())}
    for it in range(60):
        version = int(rng.integers(1, 4))
        kv = []
        for i in range(int(rng.integers(0, 12))):
            t = types[int(rng.integers(0, len(types)))]
            if rng.integers(0, 4) == 0:
                kv.append((f"k{i % 5}", gw.ARR, (t, [rand[t]() for _ in range(int(rng.integers(0, 5)))])))
            else:
                kv.append((f"k{i % 5}", t, rand[t]()))
        tens = []
        for i in range(int(rng.integers(0, 6))):
            dt = int(rng.choice([0, 1, 2, 12, 14, 30]))
            dims = tuple(int(rng.integers(1, 300)) for _ in range(int(rng.integers(1, 4))))
            if version == 1:
                dims = tuple(d % 1000 for d in dims)
            tens.append((f"t{i % 3}", dims, dt, int(rng.integers(0, 1 << 20))))
        img, _ = gw.build(version, kv, tens, b"\0" * int(rng.integers(0, 64)))
        a, b = ref_parse(img), lib_parse(lib, img)
        assert a == b, it


def test_register_needs_the_device_path_types(lib):
    """sg_gguf_register takes Q4_0, Q4_K and Q6_K matrices only; a supported
    tensor goes on to sg_weight_register, which without sg_init reports
    SG_ERR_NOT_INITIALIZED."""
    with open(os.path.join(GOLDEN, "gguf_all_types_v3.gguf"), "rb") as f:
        img = f.read()
    f = sg.GgufFile(lib, data=img)
    try:
        import ctypes
        h = ctypes.c_void_p()
        rc = lib.sg_gguf_register(f.handle, f.tensor("w.q6_k").index, 0, ctypes.byref(h))
        assert rc == -6  # supported type: sg_weight_register, not initialised
        rc = lib.sg_gguf_register(f.handle, f.tensor("t.f32.3d").index, 0, ctypes.byref(h))
        assert rc == -5
    finally:
        f.close()


# ---------------------------------------------------------------- GPU upload
# sg_gguf_register: from a GGUF file on disk to a resident device weight.

@pytest.mark.gpu
@pytest.mark.parametrize("version", [1, 3])
def test_gguf_register_parity(gpu, oracle, tmp_path, version):
    """Q4_0 and Q4_K matrices uploaded straight from a mapped GGUF file give
    bit-exact dequantized weights and GEMV/GEMM outputs within the parity
    bound of the oracle run on the file's raw blocks."""
    from conftest import SEED, reference_gate, reference_outputs
    shapes = {"blk.0.attn_q.weight": (2, 96, 256), "blk.0.ffn_down.weight": (12, 130, 512),
              "output.weight": (2, 40, 4096)}
    weights = {n: (dt, r, c, oracle.gen_weight(dt, SEED, 900 + i, r, c)) for i, (n, (dt, r, c)) in enumerate(shapes.items())}
    img, _ = gw.model_file(weights, version)
    path = tmp_path / "model.gguf"
    path.write_bytes(img)
    f = sg.GgufFile(gpu, path=str(path))
    try:
        rng = np.random.default_rng(5)
        for name, (dt, r, c, raw) in weights.items():
            t = f.tensor(name)
            assert (t.dtype, t.shape) == (dt, (c, r))
            assert f.tensor_raw_bytes(t) == np.ascontiguousarray(raw, np.uint8).tobytes()
            W = f.register(t)
            try:
                ref_deq = oracle.dequantize(dt, raw, r * c).reshape(r, c)
                assert np.array_equal(gpu.dequant(W).view(np.uint32), ref_deq.view(np.uint32))
                for B in (1, 5, 40):  # decode GEMV and prefill GEMM
                    x = rng.standard_normal((B, c)).astype(np.float32)
                    ref, l2 = reference_outputs(oracle, dt, raw, x, r, c)
                    reference_gate(gpu.linear(W, x), ref, l2)
            finally:
                W.free()
    finally:
        f.close()
