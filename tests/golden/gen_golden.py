"""Generate the golden fixtures under tests/golden/.

The reference (llamanyon.rs) is Rust and no Rust toolchain exists here, so the
reference itself cannot be executed. Its hot-path tests
(swamp-kernels/src/fused_gemv_q4k.rs:704-791) store no expected values: they
compare the dispatched kernel with the batched one on fixed inputs
(make_weight / make_x, K=256, rows 2/3/4/7). These fixtures pin the C oracle
(oracle/oracle.c) in two independent ways:

1. Known answers on the reference's own test inputs. With every nibble = 8
   and per-row-constant scales, each row of make_weight is one constant
   weight w_r = RN(RN(d*sc)*8 - RN(dmin*m)); the expected fp32 output is the
   reference's sequential sum, restated here with numpy float32 scalars (a
   separate implementation from the C oracle), and the exact rational value
   of the same sum is recorded beside it.
2. A second, vectorised numpy restatement of swamp-gguf's Q4_0 / Q4_K
   dequantizers (q4_0.rs:11-38, q4_k.rs:37-53,278-322) run on seeded random
   blocks, plus float32 sequential GEMVs, which the C oracle must reproduce
   bit for bit.

Run:  python tests/golden/gen_golden.py      (rewrites the .npz/.json files)
"""
from __future__ import annotations

import json
import os
import sys
from fractions import Fraction

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle  # noqa: E402

F32 = np.float32


# ---------------------------------------------------------------------------
# independent numpy restatement (vectorised; shares no code with oracle.c)
# ---------------------------------------------------------------------------

def np_f16(raw2: np.ndarray) -> np.ndarray:
    """little-endian binary16 -> float32 via numpy's IEEE half (exact)."""
    return raw2.view("<f2").astype(np.float32)


def np_dequant_q4_0(raw: np.ndarray, n: int) -> np.ndarray:
    blocks = raw[: (n // 32) * 18].reshape(-1, 18)
    d = np_f16(np.ascontiguousarray(blocks[:, 0:2]))[:, 0]
    nib = blocks[:, 2:18]
    q = np.empty((blocks.shape[0], 32), np.int32)
    q[:, 0::2] = nib & 0x0F          # element i even <- low nibble of byte i/2
    q[:, 1::2] = nib >> 4            # element i odd  <- high nibble
    return ((q - 8).astype(np.float32) * d[:, None]).astype(np.float32).reshape(-1)


def np_unpack_scales(sc: np.ndarray):
    sc = sc.astype(np.int32)
    scales = np.empty(sc.shape[:-1] + (8,), np.int32)
    mins = np.empty_like(scales)
    scales[..., 0:4] = sc[..., 0:4] & 63
    mins[..., 0:4] = sc[..., 4:8] & 63
    scales[..., 4:8] = (sc[..., 8:12] & 0xF) | ((sc[..., 0:4] >> 6) << 4)
    mins[..., 4:8] = (sc[..., 8:12] >> 4) | ((sc[..., 4:8] >> 6) << 4)
    return scales, mins


def np_dequant_q4k(raw: np.ndarray, n: int) -> np.ndarray:
    blocks = raw[: (n // 256) * 144].reshape(-1, 144)
    d = np_f16(np.ascontiguousarray(blocks[:, 0:2]))[:, 0]
    dmin = np_f16(np.ascontiguousarray(blocks[:, 2:4]))[:, 0]
    scales, mins = np_unpack_scales(blocks[:, 4:16])
    qs = blocks[:, 16:144].reshape(-1, 4, 32).astype(np.int32)
    q = np.empty((blocks.shape[0], 8, 32), np.int32)
    q[:, 0::2, :] = qs & 0xF       # sub-block 2p <- low nibbles of qs[32p..]
    q[:, 1::2, :] = qs >> 4        # sub-block 2p+1 <- high nibbles
    sv = (d[:, None] * scales.astype(np.float32)).astype(np.float32)
    mv = (dmin[:, None] * mins.astype(np.float32)).astype(np.float32)
    prod = (sv[:, :, None] * q.astype(np.float32)).astype(np.float32)
    return (prod - mv[:, :, None]).astype(np.float32).reshape(-1)


def np_dequant_q6k(raw: np.ndarray, n: int) -> np.ndarray:
    """q6_k.rs:22-57, vectorised: element 128h + 32m + l of a block takes the
    low nibble of ql[64h + l + 32(m&1)] (>> 4(m>>1)), the 2 bits
    (qh[32h + l] >> 2m) & 3, and w = d * sc[e/16] * (q - 32)."""
    blocks = raw[: (n // 256) * 210].reshape(-1, 210).astype(np.int32)
    d = np_f16(np.ascontiguousarray(raw[: (n // 256) * 210].reshape(-1, 210)[:, 208:210]))[:, 0]
    q = np.empty((blocks.shape[0], 256), np.int32)
    for h in range(2):
        for m in range(4):
            lo = (blocks[:, 64 * h + 32 * (m & 1): 64 * h + 32 * (m & 1) + 32] >> (4 * (m >> 1))) & 0xF
            hi = (blocks[:, 128 + 32 * h: 128 + 32 * h + 32] >> (2 * m)) & 3
            q[:, 128 * h + 32 * m: 128 * h + 32 * m + 32] = lo | (hi << 4)
    sc = blocks[:, 192:208].astype(np.uint8).view(np.int8).astype(np.float32)
    s16 = (d[:, None] * sc).astype(np.float32)                    # d * sc, exact
    w = (np.repeat(s16, 16, axis=1) * (q - 32).astype(np.float32)).astype(np.float32)
    return w.reshape(-1)


def np_gemv_q6k_scalar_order(w: np.ndarray, x: np.ndarray, n_rows: int, n_cols: int) -> np.ndarray:
    """fused_gemv_q6k_scalar (fused_gemv_q6k.rs:248-291): acc += w*x in f32,
    per block and half over l with the elements l, l+32, l+64, l+96."""
    deq = np_dequant_q6k(w, n_rows * n_cols).reshape(n_rows, n_cols)
    out = np.zeros(n_rows, np.float32)
    for r in range(n_rows):
        acc = F32(0.0)
        for blk in range(n_cols // 256):
            for h in range(2):
                base = blk * 256 + 128 * h
                for l in range(32):
                    for m in range(4):
                        k = base + l + 32 * m
                        acc = F32(acc + F32(deq[r, k] * x[k]))
        out[r] = acc
    return out


def np_seq_dot(w_row: np.ndarray, x: np.ndarray) -> np.float32:
    """acc += w*x in float32, left to right, products rounded before adding."""
    acc = F32(0.0)
    prods = (w_row.astype(np.float32) * x.astype(np.float32)).astype(np.float32)
    for p in prods:
        acc = F32(acc + p)
    return acc


def np_gemv_q4k_scalar_order(w: np.ndarray, x: np.ndarray, n_rows: int, n_cols: int) -> np.ndarray:
    """fused_gemv_q4k_scalar: the scalar kernel walks elements in dequant order
    (pair, even/odd, i), which equals ascending k, so the sequential sum over
    the dequantized row is the same float32 value."""
    deq = np_dequant_q4k(w, n_rows * n_cols).reshape(n_rows, n_cols)
    return np.array([np_seq_dot(deq[r], x) for r in range(n_rows)], np.float32)


def np_linear_q4_0(w, x, n_rows, n_cols):
    deq = np_dequant_q4_0(w, n_rows * n_cols).reshape(n_rows, n_cols)
    return np.array([np_seq_dot(deq[r], x) for r in range(n_rows)], np.float32)


def np_batched_scalar(w, xs, n_rows, n_cols):
    """batched_scalar (fused_gemv_q4k.rs:650-698): per 256-block a fresh f32
    acc over the block, then out += acc, blocks in ascending order."""
    deq = np_dequant_q4k(w, n_rows * n_cols).reshape(n_rows, n_cols)
    B = xs.shape[0]
    out = np.zeros((B, n_rows), np.float32)
    for blk in range(n_cols // 256):
        for r in range(n_rows):
            for t in range(B):
                acc = np_seq_dot(deq[r, blk * 256:(blk + 1) * 256], xs[t, blk * 256:(blk + 1) * 256])
                out[t, r] = F32(out[t, r] + acc)
    return out


# ---------------------------------------------------------------------------
# 1. the reference's own test inputs (make_weight / make_x), known answers
# ---------------------------------------------------------------------------

def kat_reference_tests():
    n_cols = 256
    x = oracle.make_x(n_cols)
    # make_x restated with numpy float32: (i%100) as f32 / 50 - 1
    x_np = np.array([F32(F32(i % 100) / F32(50.0)) - F32(1.0) for i in range(n_cols)], np.float32)
    assert np.array_equal(x, x_np)
    cases = []
    for n_rows in (2, 3, 4, 7):
        w = oracle.make_weight(n_rows)
        expect_seq = []
        expect_exact = []
        w_row_vals = []
        for r in range(n_rows):
            d32 = F32(F32(0.5) + F32(r) * F32(0.1))
            dm32 = F32(F32(0.1) + F32(r) * F32(0.05))
            d = F32(np.float16(d32))      # half::f16::from_f32 (RNE) then to_f32
            dm = F32(np.float16(dm32))
            sc = (r + 1) & 0x3F
            mn = (r + 2) & 0x3F
            sv = F32(d * F32(sc))
            mv = F32(dm * F32(mn))
            wv = F32(F32(sv * F32(8)) - mv)
            w_row_vals.append(float(wv))
            acc = F32(0)
            for k in range(n_cols):
                acc = F32(acc + F32(wv * x[k]))
            expect_seq.append(float(acc))
            exact = sum(Fraction(float(wv)) * Fraction(float(x[k])) for k in range(n_cols))
            expect_exact.append(float(exact))
        # the oracle must reproduce these bit-exactly
        deq = oracle.dequantize(oracle.DTYPE_Q4_K, w, n_rows * n_cols).reshape(n_rows, n_cols)
        assert np.array_equal(deq, np.repeat(np.array(w_row_vals, np.float32)[:, None], n_cols, 1))
        got = oracle.gemv_q4k_scalar(w, x, n_rows, n_cols)
        assert np.array_equal(got, np.array(expect_seq, np.float32)), (got, expect_seq)
        outs = np.zeros((1, n_rows), np.float32)
        oracle.gemv_q4k_batched_scalar(w, x[None].copy(), outs, n_rows, n_cols)
        # the reference test's own relation (|single - batched| < 0.01)
        assert np.all(np.abs(outs[0] - got) < 0.01)
        cases.append({
            "n_rows": n_rows,
            "n_cols": n_cols,
            "weight_hex": w.tobytes().hex(),
            "row_weight_value": w_row_vals,
            "expect_f32_sequential": expect_seq,
            "expect_exact_rational": expect_exact,
            "batched_b1_f32": [float(v) for v in outs[0]],
        })
    return {"x_make_x_256": [float(v) for v in x], "cases": cases,
            "source": "swamp-kernels/src/fused_gemv_q4k.rs:704-791 (make_q4k_block, make_weight, make_x)"}


# ---------------------------------------------------------------------------
# 2. hand-built Q4_0 known answers (no reference test exists for Q4_0)
# ---------------------------------------------------------------------------

def kat_q4_0():
    # two rows x 64 cols; row 0: d = 1.0, nibbles 0..15,0..15 (element order);
    # row 1: d = 2^-14 (smallest normal), descending nibbles; then a
    # subnormal scale block and a negative scale block.
    def block(d_bits: int, q: list[int]) -> bytes:
        b = bytearray(18)
        b[0] = d_bits & 0xFF
        b[1] = d_bits >> 8
        for j in range(16):
            b[2 + j] = q[2 * j] | (q[2 * j + 1] << 4)
        return bytes(b)

    ramp = [i % 16 for i in range(32)]
    down = [15 - (i % 16) for i in range(32)]
    rows = [
        block(0x3C00, ramp) + block(0x4000, down),          # d=1.0, d=2.0
        block(0x0400, down) + block(0x0001, ramp),          # d=2^-14, d=2^-24 (subnormal)
        block(0xBC00, ramp) + block(0x7BFF, [8] * 32),      # d=-1.0, d=65504 with q=8 -> 0
    ]
    raw = np.frombuffer(b"".join(rows), np.uint8).copy()
    n_rows, n_cols = 3, 64
    d_vals = [[1.0, 2.0], [2.0 ** -14, 2.0 ** -24], [-1.0, 65504.0]]
    q_vals = [[ramp, down], [down, ramp], [ramp, [8] * 32]]
    expect = np.array([[(q_vals[r][b][i] - 8) * d_vals[r][b] for b in range(2) for i in range(32)]
                       for r in range(n_rows)], np.float32)
    deq = oracle.dequantize(oracle.DTYPE_Q4_0, raw, n_rows * n_cols).reshape(n_rows, n_cols)
    assert np.array_equal(deq, expect)
    assert np.array_equal(np_dequant_q4_0(raw, n_rows * n_cols).reshape(n_rows, n_cols), expect)
    x = np.array([((i * 7) % 13 - 6) / 4.0 for i in range(n_cols)], np.float32)  # exact in f32
    exact = [float(sum(Fraction(float(expect[r, k])) * Fraction(float(x[k])) for k in range(n_cols)))
             for r in range(n_rows)]
    got = oracle.linear_q4_0(raw, x, n_rows, n_cols)
    seq = np_linear_q4_0(raw, x, n_rows, n_cols)
    assert np.array_equal(got, seq)
    return {"weight_hex": raw.tobytes().hex(), "n_rows": n_rows, "n_cols": n_cols,
            "dequant": expect.tolist(), "x": x.tolist(), "expect_f32_sequential": seq.tolist(),
            "expect_exact_rational": exact,
            "source": "swamp-gguf/src/quant/q4_0.rs:11-38 (semantics; the reference has no Q4_0 test)"}


# ---------------------------------------------------------------------------
# 3. seeded random blocks: dequant + reference fp32 GEMV, cross-checked
# ---------------------------------------------------------------------------

SEED = 0x5EED1A11


def random_fixtures():
    out = {}
    for name, dtype, n_rows, n_cols, B in (("q4_0", oracle.DTYPE_Q4_0, 48, 320, 3),
                                          ("q4k", oracle.DTYPE_Q4_K, 40, 512, 3)):
        w = oracle.gen_weight(dtype, SEED, 1, n_rows, n_cols)
        x = oracle.gen_x(SEED, 2, (B, n_cols))
        if dtype == oracle.DTYPE_Q4_0:
            deq_np = np_dequant_q4_0(w, n_rows * n_cols)
            ref_np = np.stack([np_linear_q4_0(w, x[b], n_rows, n_cols) for b in range(B)])
        else:
            deq_np = np_dequant_q4k(w, n_rows * n_cols)
            ref_np = np.stack([np_gemv_q4k_scalar_order(w, x[b], n_rows, n_cols) for b in range(B)])
            bat_np = np_batched_scalar(w, x, n_rows, n_cols)
            bat_c = np.zeros((B, n_rows), np.float32)
            oracle.gemv_q4k_batched_scalar(w, x, bat_c, n_rows, n_cols)
            assert np.array_equal(bat_np, bat_c)
            out[name + "_batched"] = bat_np
        deq_c = oracle.dequantize(dtype, w, n_rows * n_cols)
        assert np.array_equal(deq_np, deq_c)
        ref_c = oracle.reference_linear(dtype, w, x, n_rows, n_cols)
        assert np.array_equal(ref_np, ref_c)
        out[name + "_w"] = w
        out[name + "_x"] = x
        out[name + "_deq"] = deq_np.reshape(n_rows, n_cols)
        out[name + "_ref"] = ref_np
        out[name + "_shape"] = np.array([n_rows, n_cols, B], np.int64)
    return out


def q6k_create_test_data(n_rows: int, n_blocks: int) -> np.ndarray:
    """create_test_data (swamp-kernels/src/fused_gemv_q6k.rs:331-356)."""
    raw = np.zeros(n_rows * n_blocks * 210, np.uint8)
    for row in range(n_rows):
        for blk in range(n_blocks):
            b = (row * n_blocks + blk) * 210
            for i in range(128):
                raw[b + i] = (i & 0x0F) | ((((i + 128) & 0xFF) & 0x0F) << 4)
            for i in range(64):
                b0 = (i >> 4) & 3
                b1 = ((i + 64) >> 4) & 3
                b2 = (((i + 128) & 0xFF) >> 4) & 3
                b3 = (((i + 192) & 0xFF) >> 4) & 3
                raw[b + 128 + i] = b0 | (b1 << 2) | (b2 << 4) | (b3 << 6)
            for i in range(16):
                raw[b + 192 + i] = (row * 16 + i + 1) & 0x7F
            raw[b + 208] = 0x00
            raw[b + 209] = 0x38  # d = f16 0x3800 = 0.5
    return raw


def kat_q6k_reference_tests():
    """The reference's Q6_K test (fused_gemv_q6k.rs:358-376): create_test_data
    with 2 rows x 2 blocks, x[i] = sin(0.01 i) in f32 (here numpy's float32
    sin; Rust's may differ by an ulp, and the test's bound is loose), the
    scalar kernel against the dequantized dot."""
    n_rows, n_blocks = 2, 2
    n_cols = 256 * n_blocks
    raw = q6k_create_test_data(n_rows, n_blocks)
    x = np.sin(np.arange(n_cols, dtype=np.float32) * F32(0.01)).astype(np.float32)
    deq_np = np_dequant_q6k(raw, n_rows * n_cols).reshape(n_rows, n_cols)
    deq_c = oracle.dequantize(oracle.DTYPE_Q6_K, raw, n_rows * n_cols).reshape(n_rows, n_cols)
    assert np.array_equal(deq_np, deq_c)
    fused_np = np_gemv_q6k_scalar_order(raw, x, n_rows, n_cols)
    fused_c = oracle.gemv_q6k_scalar(raw, x, n_rows, n_cols)
    assert np.array_equal(fused_np, fused_c)
    dot_ref = [float(np.sum((deq_np[r] * x).astype(np.float32), dtype=np.float32)) for r in range(n_rows)]
    for r in range(n_rows):  # the reference test's own relation (:371-374)
        diff = abs(float(fused_np[r]) - dot_ref[r])
        assert diff < 1.0 or diff / max(abs(dot_ref[r]), 1.0) < 1e-4
    return {"n_rows": n_rows, "n_cols": n_cols, "weight_hex": raw.tobytes().hex(), "x": x.tolist(),
            "dequant_row0_first16": deq_np[0, :16].tolist(),
            "expect_f32_scalar_kernel": fused_np.tolist(), "dequant_dot_f32": dot_ref,
            "source": "swamp-kernels/src/fused_gemv_q6k.rs:331-376 (create_test_data, test_q6k_bitexact_vs_dequant_scalar)"}


def q6k_random_fixtures():
    n_rows, n_cols, B = 24, 512, 2
    w = oracle.gen_weight(oracle.DTYPE_Q6_K, SEED, 7, n_rows, n_cols)
    x = oracle.gen_x(SEED, 8, (B, n_cols))
    deq_np = np_dequant_q6k(w, n_rows * n_cols)
    assert np.array_equal(deq_np, oracle.dequantize(oracle.DTYPE_Q6_K, w, n_rows * n_cols))
    ref_np = np.stack([np_gemv_q6k_scalar_order(w, x[b], n_rows, n_cols) for b in range(B)])
    assert np.array_equal(ref_np, oracle.reference_linear(oracle.DTYPE_Q6_K, w, x, n_rows, n_cols))
    return {"q6k_w": w, "q6k_x": x, "q6k_deq": deq_np.reshape(n_rows, n_cols), "q6k_ref": ref_np,
            "q6k_shape": np.array([n_rows, n_cols, B], np.int64)}


def main():
    oracle.build()
    with open(os.path.join(HERE, "q6k_reference_tests.json"), "w") as f:
        json.dump(kat_q6k_reference_tests(), f, indent=1)
    np.savez_compressed(os.path.join(HERE, "q6k_small.npz"), seed=np.uint64(SEED), **q6k_random_fixtures())
    with open(os.path.join(HERE, "q4k_reference_tests.json"), "w") as f:
        json.dump(kat_reference_tests(), f, indent=1)
    with open(os.path.join(HERE, "q4_0_known_answers.json"), "w") as f:
        json.dump(kat_q4_0(), f, indent=1)
    np.savez_compressed(os.path.join(HERE, "random_small.npz"), seed=np.uint64(SEED), **random_fixtures())
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
