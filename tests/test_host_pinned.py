"""Host-pointer entry points (sg_linear, sg_linear_multi) with page-locked
rows from sg_host_alloc: x is copied to the device and y back by DMA straight
from and into the caller's arrays (one 2D copy each, strided rows allowed),
instead of through the library's staging buffer. Against the oracle
(forward_linear / forward_linear_batch, linear.rs:14-90,176-239) and against
the same call on ordinary (pageable) arrays, for the decode GEMV and the
prefill GEMM, with mixed pinned / pageable arguments and SG_FLAG_ACCUMULATE
(whose outputs always go through the staging buffer).
"""
import numpy as np
import pytest

from conftest import SEED, reference_gate, reference_outputs

pytestmark = pytest.mark.gpu
Q40, Q4K = 2, 12


def _close(a, b):
    # the decode GEMV sums rows shared by several CTAs with atomic adds in any
    # order, so two calls may differ in the last bits
    scale = float(np.abs(b).max()) + 1e-30
    assert float(np.abs(a - b).max()) <= 1e-6 * scale


@pytest.mark.parametrize("batch", [1, 4, 16, 40])
@pytest.mark.parametrize("dtype,n,k", [(Q40, 1000, 4096), (Q4K, 520, 2048)])
def test_pinned_rows(gpu, oracle, dtype, n, k, batch):
    raw = oracle.gen_weight(dtype, SEED, 900 + dtype, n, k)
    W = gpu.register(raw, dtype, n, k)
    try:
        x = oracle.gen_x(SEED, 901 + batch, (batch, k))
        ref, l2 = reference_outputs(oracle, dtype, raw, x, n, k)
        # x as a column slice of a wider pinned array (row stride k + 64)
        xw = gpu.host_array((batch, k + 64))
        xw[:] = 7.0
        xw[:, :k] = x
        xs = xw[:, :k]
        out = gpu.host_array((batch, n))
        out[:] = np.nan
        y = gpu.linear(W, xs, out=out)
        assert y is out or np.shares_memory(y, out)
        reference_gate(out, ref, l2)
        assert np.array_equal(xw[:, k:], np.full((batch, 64), 7.0, np.float32))  # x untouched
        pageable = gpu.linear(W, x)
        _close(out, pageable)
        # pinned x with a pageable out, and a pageable x with a pinned out
        y2 = gpu.linear(W, xs)
        _close(y2, pageable)
        out[:] = np.nan
        gpu.linear(W, x, out=out)
        _close(out, pageable)
        # accumulate: pinned x, outputs through the staging buffer
        y0 = oracle.gen_x(SEED, 902, (batch, n))
        acc = gpu.host_array((batch, n))
        acc[:] = y0
        gpu.linear(W, xs, accumulate_into=acc)
        reference_gate(acc - y0, ref, l2 + np.abs(y0))
    finally:
        W.free()


@pytest.mark.parametrize("dtype,k", [(Q40, 4096), (Q4K, 4096)])
def test_pinned_multi(gpu, oracle, dtype, k):
    rows = (600, 136, 256)
    raws = [oracle.gen_weight(dtype, SEED, 910 + i, r, k) for i, r in enumerate(rows)]
    Ws = [gpu.register(w, dtype, r, k) for w, r in zip(raws, rows)]
    try:
        x = oracle.gen_x(SEED, 913, (k,))
        xp = gpu.host_array((k,))
        xp[:] = x
        outs = [gpu.host_array((r,)) for r in rows]
        outs[1] = np.full(rows[1], np.nan, np.float32)  # one pageable output among pinned ones
        for o in outs:
            o[:] = np.nan
        got = gpu.linear_multi(Ws, xp, outs=outs)
        for g, o in zip(got, outs):
            assert np.shares_memory(g, o)
        sep = gpu.linear_multi(Ws, x)
        for w, r, o, s in zip(raws, rows, outs, sep):
            ref, l2 = reference_outputs(oracle, dtype, w, x[None], r, k)
            reference_gate(o[None], ref, l2)
            _close(o, s)
    finally:
        for W in Ws:
            W.free()


def test_out_argument_checked(gpu, oracle):
    k, n = 256, 8
    W = gpu.register(oracle.gen_weight(Q4K, SEED, 920, n, k), Q4K, n, k)
    try:
        import swamp_gpu as sg
        x = np.zeros((2, k), np.float32)
        with pytest.raises(sg.SwampGpuError):
            gpu.linear(W, x, out=np.zeros((2, n + 1), np.float32))
        with pytest.raises(sg.SwampGpuError):
            gpu.linear(W, x, out=np.zeros((2, n), np.float64))
        with pytest.raises(sg.SwampGpuError):
            gpu.linear(W, x, out=np.zeros((n, 2), np.float32).T)
    finally:
        W.free()
