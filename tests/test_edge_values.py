"""Edge values of the block formats through the GPU kernels, against the
oracle's restatement of the reference (q4_0.rs:24-35, q4_k.rs:291-319):
d and dmin of 0, f16 subnormals, +-inf and NaN, and blocks whose nibbles
are all 0 or all 15 with 6-bit scales and mins of 63.

Bars: dequantized weights bit-exact (a NaN matches a NaN: the GPU's multiply
returns the canonical NaN where the host keeps the operand's payload);
GEMV (every decode plan) and GEMM outputs non-finite exactly where the
reference's f32 sum is, and within the parity bound everywhere else.
"""
import numpy as np
import pytest

from conftest import SEED, reference_gate, reference_outputs

pytestmark = pytest.mark.gpu
Q40, Q4K = 2, 12
F16_SUB_MIN, F16_SUB_MAX, F16_MAX = 0x0001, 0x03FF, 0x7BFF
F16_INF, F16_NINF, F16_NAN = 0x7C00, 0xFC00, 0x7E01


def _le16(v):
    return np.array([v & 0xFF, v >> 8], np.uint8)


def q4_0_edges(oracle, k):
    """8 rows: d = 0; subnormal d; one +inf block; one -inf block; one NaN
    block; nibbles all 0; nibbles all 15 with the largest f16 d; random."""
    n = 8
    w = oracle.gen_weight(Q40, SEED, 600, n, k).copy()
    nb = k // 32
    blk = lambda r, b: w[(r * nb + b) * 18:(r * nb + b + 1) * 18]
    for b in range(nb):
        blk(0, b)[0:2] = _le16(0)
        blk(1, b)[0:2] = _le16(F16_SUB_MIN if b % 2 else F16_SUB_MAX)
        blk(5, b)[2:] = 0x00
        blk(6, b)[0:2] = _le16(F16_MAX)
        blk(6, b)[2:] = 0xFF
    blk(2, 1)[0:2] = _le16(F16_INF)
    blk(3, nb - 1)[0:2] = _le16(F16_NINF)
    blk(4, nb // 2)[0:2] = _le16(F16_NAN)
    return w, n


def q4_k_edges(oracle, k):
    """8 rows: d = dmin = 0; subnormal d and dmin; +inf d; +inf dmin with the
    block's mins 0 (inf * 0 = NaN in the reference); NaN d; nibbles all 15
    with scales and mins 63; nibbles all 0 with scales and mins 63; random."""
    n = 8
    w = oracle.gen_weight(Q4K, SEED, 601, n, k).copy()
    nb = k // 256
    blk = lambda r, b: w[(r * nb + b) * 144:(r * nb + b + 1) * 144]
    for b in range(nb):
        blk(0, b)[0:4] = 0
        blk(1, b)[0:2] = _le16(F16_SUB_MAX)
        blk(1, b)[2:4] = _le16(F16_SUB_MIN)
        blk(5, b)[4:16] = 0xFF   # every 6-bit scale and min = 63
        blk(5, b)[16:] = 0xFF
        blk(6, b)[4:16] = 0xFF
        blk(6, b)[16:] = 0x00
    blk(2, 0)[0:2] = _le16(F16_INF)
    blk(3, nb - 1)[2:4] = _le16(F16_INF)
    blk(3, nb - 1)[4:16] = 0x00  # scales and mins 0: d*sc*q = 0 * ... and dmin*m = inf*0
    blk(4, 0)[0:2] = _le16(F16_NAN)
    return w, n


CASES = [(Q40, 256, q4_0_edges), (Q40, 1024, q4_0_edges), (Q4K, 512, q4_k_edges), (Q4K, 2048, q4_k_edges)]


@pytest.mark.parametrize("dtype,k,make", CASES)
def test_edge_dequant_bit_exact(gpu, oracle, dtype, k, make):
    w, n = make(oracle, k)
    W = gpu.register(w, dtype, n, k)
    try:
        got = gpu.dequant(W)
        ref = oracle.dequantize(dtype, w, n * k).reshape(n, k)
        nan_g, nan_r = np.isnan(got), np.isnan(ref)
        assert np.array_equal(nan_g, nan_r)
        assert np.array_equal(got[~nan_g].view(np.uint32), ref[~nan_r].view(np.uint32))
        assert nan_r.any() and np.isinf(ref).any() and (ref == 0).any()  # the edges are present
    finally:
        W.free()


@pytest.mark.parametrize("batch", [1, 2, 4, 16, 32, 40])
@pytest.mark.parametrize("dtype,k,make", CASES)
def test_edge_linear(gpu, oracle, dtype, k, make, batch):
    w, n = make(oracle, k)
    x = oracle.gen_x(SEED, 602 + batch, (batch, k))
    W = gpu.register(w, dtype, n, k)
    try:
        y = gpu.linear(W, x)
        ref = oracle.reference_linear(dtype, w, x, n, k)
        bad = ~np.isfinite(ref)
        assert bad.any()
        assert np.array_equal(~np.isfinite(y), bad), (np.argwhere(~np.isfinite(y)), np.argwhere(bad))
        rows = [r for r in range(n) if not bad[:, r].any()]
        rb = oracle.row_bytes(dtype, k)
        sub = np.concatenate([w[r * rb:(r + 1) * rb] for r in rows])
        ref2, l2 = reference_outputs(oracle, dtype, sub, x, len(rows), k)
        reference_gate(y[:, rows], ref2, l2)
    finally:
        W.free()
