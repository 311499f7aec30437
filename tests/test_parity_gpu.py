"""GPU parity tests: the CUDA path, called through the C ABI, against the CPU
oracle on identical seeded inputs.

Bars: dequantized weights bit-exact with swamp-gguf (q4_0.rs / q4_k.rs);
GEMV/GEMM outputs within |y-ref| <= 1e-3*max(|ref|, ||w.*x||_2) per element
of the reference's f32 result (conftest.reference_gate)."""
import os

import numpy as np
import pytest

from conftest import SEED, reference_gate, reference_outputs, reference_outputs_batch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
Q40, Q4K = 2, 12

SHAPES = [
    (Q40, 128, 256), (Q40, 200, 352), (Q40, 1, 32), (Q40, 77, 64), (Q40, 256, 1024),
    (Q4K, 128, 512), (Q4K, 300, 768), (Q4K, 7, 256), (Q4K, 129, 256),
]


def _weights(oracle, dtype, n, k, tid=1):
    return oracle.gen_weight(dtype, SEED, tid, n, k)


@pytest.mark.parametrize("dtype,n,k", SHAPES)
def test_dequant_bit_exact(gpu, oracle, dtype, n, k):
    w = _weights(oracle, dtype, n, k)
    W = gpu.register(w, dtype, n, k)
    try:
        got = gpu.dequant(W)
        ref = oracle.dequantize(dtype, w, n * k).reshape(n, k)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    finally:
        W.free()


def test_golden_fixtures_on_gpu(gpu, oracle):
    z = np.load(os.path.join(HERE, "golden", "random_small.npz"))
    for name, dtype in (("q4_0", Q40), ("q4k", Q4K)):
        n, k, B = (int(v) for v in z[name + "_shape"])
        W = gpu.register(z[name + "_w"], dtype, n, k)
        try:
            assert np.array_equal(gpu.dequant(W).view(np.uint32), z[name + "_deq"].view(np.uint32))
            x = z[name + "_x"]
            y = gpu.linear(W, x)
            _, l2 = reference_outputs(oracle, dtype, z[name + "_w"], x, n, k)
            reference_gate(y, z[name + "_ref"], l2)
        finally:
            W.free()


def test_reference_test_fixtures_on_gpu(gpu, oracle):
    """The reference's own make_weight/make_x inputs through swamp_fused_gemv_q4k's drop-in."""
    import json
    kat = json.load(open(os.path.join(HERE, "golden", "q4k_reference_tests.json")))
    x = np.array(kat["x_make_x_256"], np.float32)
    for case in kat["cases"]:
        n = case["n_rows"]
        w = np.frombuffer(bytes.fromhex(case["weight_hex"]), np.uint8).copy()
        y = gpu.fused_gemv_q4k(w, x, n, 256)
        ref = np.array(case["expect_f32_sequential"], np.float32)
        _, l2 = reference_outputs(oracle, Q4K, w, x, n, 256)
        reference_gate(y, ref, l2[0])
        assert np.all(np.abs(y - ref) < 0.01)  # the reference test's own bound (:765)


@pytest.mark.parametrize("batch", [1, 2, 3, 4, 5, 8, 13, 16, 17, 24, 31, 32])
@pytest.mark.parametrize("dtype,n,k", [(Q40, 300, 1024), (Q4K, 300, 1024), (Q40, 64, 96)])
def test_gemv_batches(gpu, oracle, dtype, n, k, batch):
    w = _weights(oracle, dtype, n, k, tid=3)
    x = oracle.gen_x(SEED, 100 + batch, (batch, k))
    W = gpu.register(w, dtype, n, k)
    try:
        y = gpu.linear(W, x)
        ref, l2 = reference_outputs(oracle, dtype, w, x, n, k)
        reference_gate(y, ref, l2)
    finally:
        W.free()


@pytest.mark.parametrize("batch", [33, 40, 64])
@pytest.mark.parametrize("dtype", [Q40, Q4K])
def test_prefill_batches(gpu, oracle, dtype, batch):
    n, k = 160, 512
    w = _weights(oracle, dtype, n, k, tid=4)
    x = oracle.gen_x(SEED, 200 + batch, (batch, k))
    W = gpu.register(w, dtype, n, k)
    try:
        y = gpu.linear(W, x)
        ref, l2 = reference_outputs(oracle, dtype, w, x, n, k)
        reference_gate(y, ref, l2)
    finally:
        W.free()


@pytest.mark.parametrize("dtype,n,k,m", [
    (Q40, 200, 352, 300),   # K % 64 == 32 (half-padded chunk), two token tiles, ragged last tile
    (Q40, 77, 64, 33),      # one chunk, ragged rows
    (Q4K, 129, 256, 257),   # one super-block, 257 tokens (one token in the second tile)
    (Q4K, 300, 768, 100),
])
def test_prefill_shapes(gpu, oracle, dtype, n, k, m):
    w = _weights(oracle, dtype, n, k, tid=6)
    x = oracle.gen_x(SEED, 300 + m, (m, k))
    W = gpu.register(w, dtype, n, k)
    try:
        y = gpu.linear(W, x)
        ref, l2 = reference_outputs(oracle, dtype, w, x, n, k)
        reference_gate(y, ref, l2)
    finally:
        W.free()


@pytest.mark.parametrize("dtype", [Q40, Q4K])
def test_prefill_device_strided_accumulate(gpu, oracle, dtype):
    """Device entry, batch > 32: padded leading dimensions, y += W x (split-K
    reduction onto existing values), and two calls in a row on one stream."""
    torch = pytest.importorskip("torch")
    n, k, m = 256, 2048, 40
    w = _weights(oracle, dtype, n, k, tid=21)
    x = oracle.gen_x(SEED, 21, (m, k))
    W = gpu.register(w, dtype, n, k)
    try:
        ldx, ldy = k + 4, n + 3
        xd = torch.zeros((m, ldx), dtype=torch.float32, device="cuda")
        xd[:, :k] = torch.from_numpy(x)
        y0 = torch.linspace(-2, 2, m * ldy, device="cuda").reshape(m, ldy)
        yd = y0.clone()
        gpu.linear_device(W, xd.data_ptr(), ldx, yd.data_ptr(), ldy, m, flags=2)  # SG_FLAG_ACCUMULATE
        gpu.linear_device(W, xd.data_ptr(), ldx, yd.data_ptr(), ldy, m, flags=2)
        torch.cuda.synchronize()
        got = (yd - y0).cpu().numpy()
        ref, l2 = reference_outputs(oracle, dtype, w, x, n, k)
        reference_gate(got[:, :n] / 2, ref, l2)
        assert np.array_equal(got[:, n:], np.zeros((m, ldy - n), np.float32))  # padding untouched
    finally:
        W.free()


def test_activation_ranges(gpu, oracle):
    """Large, tiny and mixed-magnitude activations (the f16 split is rescaled per column)."""
    n, k = 96, 512
    w = _weights(oracle, Q4K, n, k, tid=5)
    base = oracle.gen_x(SEED, 7, (4, k))
    x = np.stack([base[0] * 3e4, base[1] * 1e-6, base[2] * np.where(np.arange(k) % 7 == 0, 1e3, 1e-2), base[3]])
    x = x.astype(np.float32)
    W = gpu.register(w, Q4K, n, k)
    try:
        y = gpu.linear(W, x)
        ref, l2 = reference_outputs(oracle, Q4K, w, x, n, k)
        reference_gate(y, ref, l2)
        z = gpu.linear(W, np.zeros((2, k), np.float32))
        assert np.all(z == 0)
    finally:
        W.free()


@pytest.mark.parametrize("accumulate", [False, True])
@pytest.mark.parametrize("batch", [1, 16])
def test_gemv_shared_row_blocks(gpu, oracle, batch, accumulate):
    """4096 x 4096 runs 2048 chunks on one CTA per SM, so most row-blocks are
    shared by several CTAs (zeroed by the first, reduced into y by all);
    repeated calls must agree and match the reference, also when adding into
    a non-zero y."""
    n = k = 4096
    w = _weights(oracle, Q40, n, k, tid=30)
    x = oracle.gen_x(SEED, 31, (batch, k))
    W = gpu.register(w, Q40, n, k)
    try:
        ref, l2 = reference_outputs(oracle, Q40, w, x, n, k)
        y0 = np.linspace(-3, 3, batch * n).astype(np.float32).reshape(batch, n)
        for _ in range(3):
            y = gpu.linear(W, x, accumulate_into=y0.copy()) - y0 if accumulate else gpu.linear(W, x)
            reference_gate(y, ref, l2)
    finally:
        W.free()


def test_gemv_nonfinite_activation(gpu, oracle):
    """A non-finite x makes its token's outputs non-finite (as the reference's
    f32 sums do) and leaves the other tokens exact."""
    n, k = 200, 1024
    w = _weights(oracle, Q4K, n, k, tid=32)
    x = oracle.gen_x(SEED, 33, (3, k))
    x[1, 300] = np.inf
    x[2, 7] = np.nan
    W = gpu.register(w, Q4K, n, k)
    try:
        y = gpu.linear(W, x)
        assert not np.isfinite(y[1]).any() and not np.isfinite(y[2]).any()
        ref, l2 = reference_outputs(oracle, Q4K, w, x[:1], n, k)
        reference_gate(y[:1], ref, l2)
    finally:
        W.free()


def test_multi_and_accumulate(gpu, oracle):
    k = 512
    ws = [_weights(oracle, Q40, n, k, tid=10 + i) for i, n in enumerate((256, 64, 64))]
    Ws = [gpu.register(w, Q40, w.size // (k // 32 * 18), k) for w in ws]
    try:
        x = oracle.gen_x(SEED, 9, (k,))
        outs = gpu.linear_multi(Ws, x)
        for w, W, y in zip(ws, Ws, outs):
            ref, l2 = reference_outputs(oracle, Q40, w, x, W.n_rows, k)
            reference_gate(y, ref[0], l2[0])
        y0 = np.linspace(-1, 1, Ws[0].n_rows).astype(np.float32)
        yacc = gpu.linear(Ws[0], x, accumulate_into=y0.copy())
        ref, l2 = reference_outputs(oracle, Q40, ws[0], x, Ws[0].n_rows, k)
        reference_gate(yacc - y0, ref[0], l2[0])
    finally:
        for W in Ws:
            W.free()


def test_device_pointer_entry(gpu, oracle):
    torch = pytest.importorskip("torch")
    n, k, B = 384, 1024, 4
    w = _weights(oracle, Q4K, n, k, tid=20)
    x = oracle.gen_x(SEED, 21, (B, k))
    W = gpu.register(w, Q4K, n, k)
    try:
        xd = torch.from_numpy(x).cuda()
        yd = torch.full((B, n + 8), float("nan"), device="cuda")
        st = torch.cuda.current_stream().cuda_stream
        gpu.linear_device(W, xd.data_ptr(), k, yd.data_ptr(), n + 8, B, stream=st)
        torch.cuda.synchronize()
        y = yd[:, :n].cpu().numpy()
        assert torch.isnan(yd[:, n:]).all(), "wrote outside the requested rows"
        ref, l2 = reference_outputs(oracle, Q4K, w, x, n, k)
        reference_gate(y, ref, l2)
        dq = torch.empty((n, k), device="cuda")
        gpu.dequant_device(W, dq.data_ptr())
        torch.cuda.synchronize()
        assert np.array_equal(dq.cpu().numpy().view(np.uint32),
                              oracle.dequantize(Q4K, w, n * k).reshape(n, k).view(np.uint32))
    finally:
        W.free()


def test_host_validation_errors(gpu):
    import swamp_gpu
    w = np.zeros(144, np.uint8)
    with pytest.raises(swamp_gpu.SwampGpuError):
        gpu.register(w, 12, 1, 100)          # n_cols not a block multiple
    with pytest.raises(swamp_gpu.SwampGpuError):
        gpu.register(w, 3, 1, 256)           # unsupported dtype
    W = gpu.register(w, 12, 1, 256)
    try:
        assert gpu.linear(W, np.zeros((0, 256), np.float32)).shape == (0, 1)  # empty batch is a no-op
        with pytest.raises(swamp_gpu.SwampGpuError):
            gpu.linear(W, np.zeros(100, np.float32))  # shape mismatch (linear.rs:23)
    finally:
        W.free()
    gpu.synchronize()


@pytest.mark.parametrize("dtype,n,k,batch", [(Q40, 4096, 4096, 1), (Q40, 4096, 4096, 4), (Q4K, 1024, 4096, 2),
                                             (Q4K, 640, 2048, 9), (Q40, 300, 11008, 32)])
def test_gemv_graph_replay(gpu, oracle, dtype, n, k, batch):
    """One decode call captured alone in a CUDA graph and replayed with new
    activations: rows shared by several CTAs are handed over through flags
    that each launch sets and clears, so every replay must match the
    reference (y is poisoned with NaN before each replay)."""
    torch = pytest.importorskip("torch")
    w = _weights(oracle, dtype, n, k, tid=40)
    W = gpu.register(w, dtype, n, k)
    try:
        xd = torch.zeros((batch, k), dtype=torch.float32, device="cuda")
        yd = torch.zeros((batch, n), dtype=torch.float32, device="cuda")
        st = torch.cuda.Stream()
        with torch.cuda.stream(st):
            gpu.linear_device(W, xd.data_ptr(), k, yd.data_ptr(), n, batch, stream=st.cuda_stream)  # warm-up
        st.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            gpu.linear_device(W, xd.data_ptr(), k, yd.data_ptr(), n, batch, stream=st.cuda_stream)
        rows = np.arange(0, n, max(1, n // 97))
        rb = oracle.row_bytes(dtype, k)
        sub = np.concatenate([w[r * rb:(r + 1) * rb] for r in rows])
        for rep in range(6):
            x = oracle.gen_x(SEED, 41 + rep, (batch, k))
            xd.copy_(torch.from_numpy(x))
            yd.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
            y = yd.cpu().numpy()
            assert np.all(np.isfinite(y)), f"replay {rep}: rows left unwritten"
            ref, l2 = reference_outputs(oracle, dtype, sub, x, len(rows), k)
            reference_gate(y[:, rows], ref, l2)
        del g
    finally:
        W.free()


@pytest.mark.parametrize("batch", [1, 3, 16, 32])
def test_gemv_multi_device_shared(gpu, oracle, batch):
    """Three tensors sharing x in one call (the stacked Q/K/V pattern) with
    widths that make CTA ranges cross matrix boundaries; strided outputs."""
    torch = pytest.importorskip("torch")
    k = 2048
    ns = (1000, 136, 136)
    ws = [_weights(oracle, Q4K, n, k, tid=50 + i) for i, n in enumerate(ns)]
    Ws = [gpu.register(w, Q4K, n, k) for w, n in zip(ws, ns)]
    try:
        x = oracle.gen_x(SEED, 51, (batch, k))
        xd = torch.from_numpy(x).cuda()
        ys = [torch.full((batch, n + 5), float("nan"), device="cuda") for n in ns]
        gpu.linear_multi_device(Ws, xd.data_ptr(), k, [y.data_ptr() for y in ys], [n + 5 for n in ns], batch)
        torch.cuda.synchronize()
        for w, n, y in zip(ws, ns, ys):
            assert torch.isnan(y[:, n:]).all()
            ref, l2 = reference_outputs(oracle, Q4K, w, x, n, k)
            reference_gate(y[:, :n].cpu().numpy(), ref, l2)
    finally:
        for W in Ws:
            W.free()


# --------------------------------------------------------------- full sizes
def test_config0_q4_0_4096(gpu, oracle):
    n = k = 4096
    w = oracle.gen_weight(Q40, SEED, 0, n, k)
    x = oracle.gen_x(SEED, 1000, (k,))
    W = gpu.register(w, Q40, n, k)
    try:
        y = gpu.linear(W, x)
        ref, l2 = reference_outputs(oracle, Q40, w, x, n, k)
        reference_gate(y, ref[0], l2[0])
    finally:
        W.free()


@pytest.mark.parametrize("k,n", [(4096, 4096), (4096, 11008), (11008, 4096)])
@pytest.mark.parametrize("batch", [1, 4, 16])
def test_config1_llama2_layer_shapes(gpu, oracle, k, n, batch):
    w = oracle.gen_weight(Q40, SEED, 50 + n // 1000, n, k)
    x = oracle.gen_x(SEED, 2000 + batch, (batch, k))
    W = gpu.register(w, Q40, n, k)
    try:
        y = gpu.linear(W, x)
        ref, l2 = reference_outputs_batch(oracle, Q40, w, x, n, k)  # every row and token
        reference_gate(y, ref, l2)
    finally:
        W.free()


@pytest.mark.parametrize("k,n", [(4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096)])
def test_config2_q4k_prefill_512(gpu, oracle, k, n):
    M = 512
    w = oracle.gen_weight(Q4K, SEED, 70 + n // 1000, n, k)
    x = oracle.gen_x(SEED, 3000 + n, (M, k))
    W = gpu.register(w, Q4K, n, k)
    try:
        y = gpu.linear(W, x)
        tok = np.arange(0, M, 5)  # every row, every 5th token (the oracle's batched scalar kernel)
        ref, l2 = reference_outputs_batch(oracle, Q4K, w, x[tok], n, k)
        reference_gate(y[tok], ref, l2)
    finally:
        W.free()
