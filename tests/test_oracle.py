"""CPU tests: the oracle against the golden fixtures and the reference's own
test relations (swamp-kernels/src/fused_gemv_q4k.rs:742-790)."""
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


def test_f16_widening_exhaustive(oracle):
    """crate half 2.7.1 to_f32 is exact IEEE widening: all 65536 patterns."""
    bits = np.arange(65536, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([oracle.f16_to_f32(int(b)) for b in bits], np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_f16_narrowing_rne(oracle):
    rng = np.random.default_rng(1)
    vals = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-7, 1e-5, 1e-3, 1, 1e3, 6e4)])
    vals = np.concatenate([vals, np.float32([0.0, -0.0, 65504, 65520, 65519.99, 1e9, 5.96e-8, 2.98e-8, 2.99e-8])])
    want = vals.astype(np.float16).view(np.uint16)
    got = np.array([oracle.f32_to_f16(float(v)) for v in vals], np.uint16)
    assert np.array_equal(got, want)


def test_reference_test_fixtures_known_answers(oracle):
    """make_weight/make_x rows 2,3,4,7 (fused_gemv_q4k.rs:726-768)."""
    kat = json.load(open(os.path.join(GOLD, "q4k_reference_tests.json")))
    x = np.array(kat["x_make_x_256"], np.float32)
    assert np.array_equal(oracle.make_x(256), x)
    for case in kat["cases"]:
        n = case["n_rows"]
        w = np.frombuffer(bytes.fromhex(case["weight_hex"]), np.uint8).copy()
        assert np.array_equal(oracle.make_weight(n), w)
        got = oracle.gemv_q4k_scalar(w, x, n, 256)
        assert np.array_equal(got, np.array(case["expect_f32_sequential"], np.float32))
        # the reference test's relation: |single - batched| < 0.01 (:760-767)
        outs = np.zeros((1, n), np.float32)
        oracle.gemv_q4k_batched_scalar(w, x[None].copy(), outs, n, 256)
        assert np.all(np.abs(outs[0] - got) < 0.01)
        assert np.array_equal(outs[0], np.array(case["batched_b1_f32"], np.float32))
        # sequential f32 vs exact rational value
        ex = np.array(case["expect_exact_rational"])
        assert np.all(np.abs(got - ex) <= 1e-5 * np.abs(ex) + 1e-6)


def test_q4_0_known_answers(oracle):
    kat = json.load(open(os.path.join(GOLD, "q4_0_known_answers.json")))
    w = np.frombuffer(bytes.fromhex(kat["weight_hex"]), np.uint8).copy()
    n, k = kat["n_rows"], kat["n_cols"]
    deq = oracle.dequantize(oracle.DTYPE_Q4_0, w, n * k).reshape(n, k)
    assert np.array_equal(deq, np.array(kat["dequant"], np.float32))
    x = np.array(kat["x"], np.float32)
    assert np.array_equal(oracle.linear_q4_0(w, x, n, k), np.array(kat["expect_f32_sequential"], np.float32))


def test_random_fixtures_bit_exact(oracle):
    z = np.load(os.path.join(GOLD, "random_small.npz"))
    seed = int(z["seed"])
    for name, dtype in (("q4_0", oracle.DTYPE_Q4_0), ("q4k", oracle.DTYPE_Q4_K)):
        n, k, B = (int(v) for v in z[name + "_shape"])
        w = oracle.gen_weight(dtype, seed, 1, n, k)
        assert np.array_equal(w, z[name + "_w"]), "generator drifted"
        x = oracle.gen_x(seed, 2, (B, k))
        assert np.array_equal(x, z[name + "_x"])
        assert np.array_equal(oracle.dequantize(dtype, w, n * k).reshape(n, k), z[name + "_deq"])
        assert np.array_equal(oracle.reference_linear(dtype, w, x, n, k), z[name + "_ref"])


def test_unpack_scales_inverts_make_q4k_block(oracle):
    rng = np.random.default_rng(7)
    for _ in range(200):
        sc = rng.integers(0, 64, 8).astype(np.uint8)
        mn = rng.integers(0, 64, 8).astype(np.uint8)
        blk = oracle.make_q4k_block(0.5, 0.25, sc, mn, 3)
        s2, m2 = oracle.unpack_scales(blk[4:16])
        assert np.array_equal(s2, sc) and np.array_equal(m2, mn)


def test_q4k_element_order_pairs(oracle):
    """q4_k.rs:291-319: element 64p+i <- low nibble of qs[32p+i], 64p+32+i <- high."""
    sc = np.ones(8, np.uint8)
    mn = np.zeros(8, np.uint8)
    blk = oracle.make_q4k_block(1.0, 0.0, sc, mn, 0)
    for p in range(4):
        for i in range(32):
            blk[16 + 32 * p + i] = (i % 16) | (((i + 5) % 16) << 4)
    deq = oracle.dequantize(oracle.DTYPE_Q4_K, blk, 256)
    for p in range(4):
        for i in range(32):
            assert deq[64 * p + i] == i % 16
            assert deq[64 * p + 32 + i] == (i + 5) % 16


def test_dequant_buffer_too_small_and_partial(oracle):
    w = oracle.gen_weight(oracle.DTYPE_Q4_0, 3, 9, 1, 64)
    with pytest.raises(ValueError):
        oracle.dequantize(oracle.DTYPE_Q4_0, w[:20], 64)  # BufferTooSmall (q4_0.rs:15-19)
    full = oracle.dequantize(oracle.DTYPE_Q4_0, w, 64)
    part = oracle.dequantize(oracle.DTYPE_Q4_0, w, 40)  # partial last block (:28)
    assert np.array_equal(full[:40], part)


def test_forward_linear_partition_is_bit_exact(oracle):
    """Row partitioning over threads (linear.rs:31-45) changes nothing numerically."""
    for dtype, n, k in ((oracle.DTYPE_Q4_K, 37, 512), (oracle.DTYPE_Q4_0, 53, 320)):
        w = oracle.gen_weight(dtype, 11, 3, n, k)
        x = oracle.gen_x(11, 4, (k,))
        one = oracle.forward_linear(dtype, w, x, n, k, 1)
        for t in (2, 3, 6, 8, 64):
            assert np.array_equal(oracle.forward_linear(dtype, w, x, n, k, t), one)
        assert np.array_equal(one, oracle.reference_linear(dtype, w, x, n, k)[0])


def test_forward_linear_batch_matches_batched_kernel(oracle):
    n, k, B = 21, 768, 5
    w = oracle.gen_weight(oracle.DTYPE_Q4_K, 12, 3, n, k)
    xs = oracle.gen_x(12, 5, (B, k))
    got = oracle.forward_linear_batch(oracle.DTYPE_Q4_K, w, xs, n, k, 4)
    want = np.zeros((B, n), np.float32)
    oracle.gemv_q4k_batched_scalar(w, xs, want, n, k)
    assert np.array_equal(got, want)
    # and the batched order differs from the single-vector order only by rounding
    single = oracle.reference_linear(oracle.DTYPE_Q4_K, w, xs, n, k)
    assert np.all(np.abs(got - single) < 1e-3 * (np.abs(single) + 1))


def test_reference_outputs_batch_matches_per_token(oracle):
    """The full-size parity tests' fast reference (batched route on all host
    threads, ||w.*x||_2 from numpy) against the per-token one: Q4_0 bit for
    bit, Q4_K within rounding of the other summation order; the l2 norms
    agree to f64 rounding."""
    from conftest import reference_outputs, reference_outputs_batch
    for dtype, n, k, B in ((oracle.DTYPE_Q4_0, 2100, 352, 3), (oracle.DTYPE_Q4_K, 2050, 512, 4)):
        w = oracle.gen_weight(dtype, 13, 3, n, k)
        xs = oracle.gen_x(13, 5, (B, k))
        ref, l2 = reference_outputs(oracle, dtype, w, xs, n, k)
        ref_b, l2_b = reference_outputs_batch(oracle, dtype, w, xs, n, k)
        if dtype == oracle.DTYPE_Q4_0:
            assert np.array_equal(ref_b, ref)
        else:
            assert np.all(np.abs(ref_b - ref) <= 1e-5 * np.maximum(np.abs(ref), l2))
        assert np.allclose(l2_b, l2, rtol=1e-12, atol=0)


def test_generator_distributions(oracle):
    w = oracle.gen_weight(oracle.DTYPE_Q4_0, 5, 1, 64, 4096)
    blocks = w.reshape(-1, 18)
    d = blocks[:, :2].copy().view("<f2").astype(np.float32)[:, 0]
    assert d.min() >= 0.00099 and d.max() <= 0.01001
    nib = np.concatenate([blocks[:, 2:] & 15, blocks[:, 2:] >> 4]).ravel()
    counts = np.bincount(nib, minlength=16)
    assert counts.min() > 0.8 * counts.mean()
    x = oracle.gen_x(5, 2, (100000,))
    assert abs(float(x.mean())) < 0.02 and abs(float(x.std()) - 1) < 0.02
