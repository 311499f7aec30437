"""CPU tests of the timing-only restatements of the reference's SIMD Q4_K
paths (oracle/oracle_simd.c): each against a numpy model of the same
arithmetic, written from the reference's loops (fused_gemv_q4k.rs:101-317 for
VNNI, :325-392 for AVX2). These paths are not parity targets: the test checks
that the restatement computes what the reference's SIMD code computes, so that
timing it times the same work, and that it differs from the reference's
dequantized dot product (which is why it is labelled numerically divergent)."""
import numpy as np
import pytest

from conftest import SEED

Q4K = 12


def _blocks(oracle, w, n, k):
    nb = k // 256
    b = w.reshape(n, nb, 144)
    d = b[:, :, 0:2].copy().view(np.float16)[..., 0].astype(np.float32)
    dmin = b[:, :, 2:4].copy().view(np.float16)[..., 0].astype(np.float32)
    sc = np.zeros((n, nb, 8), np.float32)
    mn = np.zeros((n, nb, 8), np.float32)
    for r in range(n):
        for j in range(nb):
            s, m = oracle.unpack_scales(np.ascontiguousarray(b[r, j, 4:16]))
            sc[r, j], mn[r, j] = s & 0x3F, m & 0x3F
    return d, dmin, sc, mn, b[:, :, 16:].astype(np.int64)


def _avx2_model(oracle, w, x, n, k):
    d, dmin, sc, mn, qs = _blocks(oracle, w, n, k)
    out = np.zeros(n, np.float64)
    for blk in range(k // 256):
        xb = x[blk * 256:(blk + 1) * 256].astype(np.float64)
        for sb in range(8):
            q = qs[:, blk, sb * 16:(sb + 1) * 16]
            sv = (d[:, blk] * sc[:, blk, sb]).astype(np.float64)[:, None]
            mv = (dmin[:, blk] * mn[:, blk, sb]).astype(np.float64)[:, None]
            out += ((sv * (q & 15) - mv) * xb[sb * 32:sb * 32 + 16]).sum(1)
            out += ((sv * (q >> 4) - mv) * xb[sb * 32 + 16:sb * 32 + 32]).sum(1)
    return out


def _vnni_model(oracle, w, x, n, k):
    d, dmin, sc, mn, qs = _blocks(oracle, w, n, k)
    out = np.zeros(n, np.float64)
    for blk in range(k // 256):
        xb = x[blk * 256:(blk + 1) * 256]
        mx = np.float32(np.abs(xb).max())
        inv = np.float32(127) / mx if mx > 1e-6 else np.float32(0)
        scale = mx / np.float32(127) if mx > 1e-6 else np.float32(1)
        xi = np.zeros(256 + 32, np.int64)
        xi[:256] = np.rint(xb * inv).astype(np.int64)  # round to nearest even
        quire = np.zeros(n, np.int64)
        corr = np.zeros(n, np.float64)
        for sb in range(8):
            q = qs[:, blk, sb * 16:(sb + 1) * 16]
            wl, wh = (q & 15) + 120, (q >> 4) + 120  # ((nibble - 8) ^ 0x80) as u8
            xa, xc = xi[sb * 32:sb * 32 + 32], xi[sb * 32 + 16:sb * 32 + 48]
            quire += (wl * xa[:16]).sum(1) + (wh * xa[16:]).sum(1) + (wl * xc[:16]).sum(1) + (wh * xc[16:]).sum(1)
            sx = float(xi[sb * 32:sb * 32 + 32].sum()) * float(scale)
            sv = d[:, blk] * sc[:, blk, sb]
            mv = dmin[:, blk] * mn[:, blk, sb]
            corr += mv * sx + 136.0 * sx * sv
        out += quire * float(scale) - corr
    return out


@pytest.fixture
def case(oracle):
    n, k = 37, 1024
    return oracle.gen_weight(Q4K, SEED, 610, n, k), oracle.gen_x(SEED, 611, (k,)), n, k


def test_avx2_restatement(oracle, case):
    if oracle.simd_path() == "none":
        pytest.skip("CPU has neither AVX2+FMA nor AVX-512 VNNI")
    w, x, n, k = case
    got = oracle.gemv_q4k_simd("avx2", w, x, n, k)
    want = _avx2_model(oracle, w, x, n, k)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-3 * np.abs(want).max())
    ref = oracle.reference_linear(Q4K, w, x, n, k)[0]
    assert np.abs(got - ref).max() > 1e-2 * np.abs(ref).max()  # numerically divergent


def test_vnni_restatement(oracle, case):
    if oracle.simd_path() != "avx512-vnni":
        pytest.skip("CPU has no AVX-512 VNNI")
    w, x, n, k = case
    got = oracle.gemv_q4k_simd("avx512-vnni", w, x, n, k)
    want = _vnni_model(oracle, w, x, n, k)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4 * np.abs(want).max())
    ref = oracle.reference_linear(Q4K, w, x, n, k)[0]
    assert np.abs(got - ref).max() > 1e-2 * np.abs(ref).max()  # numerically divergent


@pytest.mark.parametrize("threads", [1, 3, 8])
def test_dispatched_row_partition(oracle, case, threads):
    """forward_linear's row split (linear.rs:31-45) leaves each row's result as
    the single-call kernel's."""
    if oracle.simd_path() == "none":
        pytest.skip("no SIMD path")
    w, x, n, k = case
    got, path = oracle.forward_linear_dispatched(w, x, n, k, threads)
    want = oracle.gemv_q4k_simd(path, w, x, n, k)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("threads", [1, 3, 8])
@pytest.mark.parametrize("batch", [1, 4, 5])
def test_fallback_gemv_token_split(oracle, threads, batch):
    """forward_linear_batch's non-Q4_K route (fallback_gemv, linear.rs:336-364)
    over Q4_0 bytes: tokens split over threads, each token the whole-tensor
    dispatched kernel, so every output row equals that kernel's single call on
    the same bytes."""
    if oracle.simd_path() == "none":
        pytest.skip("no SIMD path")
    n, k = 37, 512
    w = oracle.gen_weight(2, SEED, 40, n, k)  # Q4_0: 18 B per 32, read as 144 B per 256
    xs = oracle.gen_x(SEED, 41, (batch, k))
    outs, path = oracle.fallback_gemv_dispatched(w, xs, n, k, threads)
    for b in range(batch):
        # Q4_0 bytes read as Q4_K scales can decode to inf / NaN: NaN matches NaN
        assert np.array_equal(outs[b], oracle.gemv_q4k_simd(path, w, xs[b], n, k), equal_nan=True)
