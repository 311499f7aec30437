"""Q6_K: oracle pinning (CPU) and the device path against it (GPU).

Oracle: swamp-gguf/src/quant/q6_k.rs:22-57 (dequant, the bit-exact bar) and
swamp-kernels/src/fused_gemv_q6k.rs:248-291 (scalar kernel of the engine's
Q6_K route, linear.rs:48-67: the reference f32 result), pinned by
tests/golden/gen_golden.py: an independent numpy restatement, and the
reference's own test input (create_test_data, :331-376)."""
import json
import os

import numpy as np
import pytest

from conftest import SEED, reference_gate, reference_outputs

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")
Q6K = 14


# ------------------------------------------------------------------- oracle

def test_reference_test_input_known_answers(oracle):
    kat = json.load(open(os.path.join(GOLD, "q6k_reference_tests.json")))
    n, k = kat["n_rows"], kat["n_cols"]
    w = np.frombuffer(bytes.fromhex(kat["weight_hex"]), np.uint8).copy()
    x = np.array(kat["x"], np.float32)
    got = oracle.gemv_q6k_scalar(w, x, n, k)
    assert np.array_equal(got, np.array(kat["expect_f32_scalar_kernel"], np.float32))
    deq = oracle.dequantize(Q6K, w, n * k).reshape(n, k)
    assert np.array_equal(deq[0, :16], np.array(kat["dequant_row0_first16"], np.float32))
    for r in range(n):  # the reference test's own relation (fused_gemv_q6k.rs:371-374)
        diff = abs(float(got[r]) - kat["dequant_dot_f32"][r])
        assert diff < 1.0 or diff / max(abs(kat["dequant_dot_f32"][r]), 1.0) < 1e-4


def test_random_fixtures_bit_exact(oracle):
    z = np.load(os.path.join(GOLD, "q6k_small.npz"))
    n, k, B = (int(v) for v in z["q6k_shape"])
    assert np.array_equal(oracle.dequantize(Q6K, z["q6k_w"], n * k).reshape(n, k).view(np.uint32),
                          z["q6k_deq"].view(np.uint32))
    assert np.array_equal(oracle.reference_linear(Q6K, z["q6k_w"], z["q6k_x"], n, k), z["q6k_ref"])


def test_dequant_extremes(oracle):
    """q = 0 and 63, scales -128 and 127, d = 1: w = sc * (q - 32), exact."""
    blk = np.zeros(210, np.uint8)
    blk[0:64] = 0xF0      # element l, m=0: low nibble 0; m=2: high nibble 15
    blk[64:128] = 0x0F    # second half, m=0 low nibble 15; m=2 high nibble 0
    blk[128:192] = 0b11001100
    blk[192:208] = np.array([-128, 127] * 8, np.int8).view(np.uint8)
    blk[208], blk[209] = 0x00, 0x3C  # d = 1.0
    deq = oracle.dequantize(Q6K, blk, 256)
    # element e: h = e/128, m = (e%128)/32, l = e%32; sc = sc[e/16]
    for e in range(256):
        h, m, l = e // 128, (e % 128) // 32, e % 32
        ql = int(blk[64 * h + l + 32 * (m & 1)])
        lo = (ql >> (4 * (m >> 1))) & 0xF
        hi = (int(blk[128 + 32 * h + l]) >> (2 * m)) & 3
        sc = -128 if (e // 16) % 2 == 0 else 127
        assert deq[e] == np.float32(sc * ((lo | (hi << 4)) - 32)), e


def test_engine_route_partition(oracle):
    """forward_linear's Q6_K branch (linear.rs:48-67) with several host
    threads equals the single-thread scalar kernel bit for bit."""
    n, k = 37, 768
    w = oracle.gen_weight(Q6K, SEED, 31, n, k)
    x = oracle.gen_x(SEED, 32, (k,))
    one = oracle.gemv_q6k_scalar(w, x, n, k)
    for th in (1, 3, 8):
        assert np.array_equal(oracle.forward_linear(Q6K, w, x, n, k, th), one)


def test_generator_covers_q6k_ranges(oracle):
    w = oracle.gen_weight(Q6K, SEED, 33, 64, 1024).reshape(-1, 210)
    sc = w[:, 192:208].view(np.int8)
    assert sc.min() < -100 and sc.max() > 100
    d = w[:, 208:210].copy().view("<f2").astype(np.float32)
    assert 0.001 <= d.min() and d.max() < 0.0101
    deq = oracle.dequantize(Q6K, w.reshape(-1), 64 * 1024)
    s16 = (np.repeat(d, 256, axis=1) * np.repeat(sc.astype(np.float32), 16, axis=1)).reshape(-1)
    nz = s16 != 0
    q = np.rint(deq[nz] / s16[nz]) + 32
    assert q.min() == 0 and q.max() == 63


def test_tp_shard_plan_on_q6k_blocks():
    import sys
    sys.path.insert(0, os.path.join(HERE, "..", "llamanyon.rs_b200"))
    import swamp_gpu as sg
    g = sg.SwampGpu()
    # row split takes whole 256-element blocks of every row
    assert g.tp_shard(Q6K, 100, 14336, sg.SG_TP_ROW, 8, 3) == (0, 100, 3 * 1792, 1792)
    with pytest.raises(sg.SwampGpuError):
        g.tp_shard(Q6K, 100, 300, 0, 1, 0)  # n_cols not a multiple of 256


# ---------------------------------------------------------------------- GPU

SHAPES = [(128, 256), (7, 256), (300, 768), (129, 1024)]


@pytest.mark.gpu
@pytest.mark.parametrize("n,k", SHAPES)
def test_dequant_bit_exact(gpu, oracle, n, k):
    w = oracle.gen_weight(Q6K, SEED, 40, n, k)
    W = gpu.register(w, Q6K, n, k)
    try:
        ref = oracle.dequantize(Q6K, w, n * k).reshape(n, k)
        assert np.array_equal(gpu.dequant(W).view(np.uint32), ref.view(np.uint32))
    finally:
        W.free()


@pytest.mark.gpu
def test_golden_on_gpu(gpu, oracle):
    z = np.load(os.path.join(GOLD, "q6k_small.npz"))
    n, k, B = (int(v) for v in z["q6k_shape"])
    W = gpu.register(z["q6k_w"], Q6K, n, k)
    try:
        assert np.array_equal(gpu.dequant(W).view(np.uint32), z["q6k_deq"].view(np.uint32))
        _, l2 = reference_outputs(oracle, Q6K, z["q6k_w"], z["q6k_x"], n, k)
        reference_gate(gpu.linear(W, z["q6k_x"]), z["q6k_ref"], l2)
    finally:
        W.free()
    kat = json.load(open(os.path.join(GOLD, "q6k_reference_tests.json")))
    w = np.frombuffer(bytes.fromhex(kat["weight_hex"]), np.uint8).copy()
    W = gpu.register(w, Q6K, kat["n_rows"], kat["n_cols"])
    try:
        x = np.array(kat["x"], np.float32)
        _, l2 = reference_outputs(oracle, Q6K, w, x, kat["n_rows"], kat["n_cols"])
        reference_gate(gpu.linear(W, x), np.array(kat["expect_f32_scalar_kernel"], np.float32), l2[0])
    finally:
        W.free()


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [1, 2, 3, 4, 8, 16, 17, 40, 300])
@pytest.mark.parametrize("n,k", [(300, 1024), (64, 256), (1000, 4096)])
def test_linear_batches(gpu, oracle, n, k, batch):
    """decode GEMV (1..16 tokens, CUDA cores) and prefill GEMM (more, tcgen05)"""
    w = oracle.gen_weight(Q6K, SEED, 41, n, k)
    x = oracle.gen_x(SEED, 500 + batch, (batch, k))
    W = gpu.register(w, Q6K, n, k)
    try:
        ref, l2 = reference_outputs(oracle, Q6K, w, x, n, k)
        reference_gate(gpu.linear(W, x), ref, l2)
    finally:
        W.free()


@pytest.mark.gpu
def test_multi_and_accumulate(gpu, oracle):
    """sg_linear_multi over two Q6_K tensors sharing x (output and ffn_down
    style), and out += W x."""
    k = 512
    wa = oracle.gen_weight(Q6K, SEED, 42, 96, k)
    wb = oracle.gen_weight(Q6K, SEED, 43, 80, k)
    W1, W2 = gpu.register(wa, Q6K, 96, k), gpu.register(wb, Q6K, 80, k)
    try:
        x = oracle.gen_x(SEED, 44, (k,))
        y1, y2 = gpu.linear_multi([W1, W2], x)
        for y, w, n in ((y1, wa, 96), (y2, wb, 80)):
            ref, l2 = reference_outputs(oracle, Q6K, w, x, n, k)
            reference_gate(y, ref[0], l2[0])
        base = oracle.gen_x(SEED, 45, (3, 80))
        xs = oracle.gen_x(SEED, 46, (3, k))
        got = gpu.linear(W2, xs, accumulate_into=base.copy())
        ref, l2 = reference_outputs(oracle, Q6K, wb, xs, 80, k)
        reference_gate(got - base, ref, l2)
    finally:
        W1.free()
        W2.free()


@pytest.mark.gpu
def test_noalloc_entry(gpu, oracle):
    import torch
    n, k = 700, 2048
    w = oracle.gen_weight(Q6K, SEED, 47, n, k)
    W = gpu.register(w, Q6K, n, k)
    try:
        for batch in (1, 16):
            x = oracle.gen_x(SEED, 48 + batch, (batch, k))
            xd = torch.from_numpy(x).cuda()
            yd = torch.full((batch, n), float("nan"), device="cuda")
            gpu.linear_device_noalloc(W, xd.data_ptr(), k, yd.data_ptr(), n, batch)
            torch.cuda.synchronize()
            ref, l2 = reference_outputs(oracle, Q6K, w, x, n, k)
            reference_gate(yd.cpu().numpy(), ref, l2)
    finally:
        W.free()


@pytest.mark.gpu
def test_gguf_register_q6k(gpu, oracle, tmp_path):
    import sys
    sys.path.insert(0, HERE)
    import gguf_writer as gw
    sys.path.insert(0, os.path.join(HERE, "..", "llamanyon.rs_b200"))
    import swamp_gpu as sg
    n, k = 200, 1024
    w = oracle.gen_weight(Q6K, SEED, 49, n, k)
    img, _ = gw.model_file({"output.weight": (Q6K, n, k, w)})
    p = tmp_path / "q6k.gguf"
    p.write_bytes(img)
    f = sg.GgufFile(gpu, path=str(p))
    try:
        t = f.tensor("output.weight")
        assert t.nbytes == n * k // 256 * 210
        W = f.register(t)
        try:
            assert np.array_equal(gpu.dequant(W).view(np.uint32),
                                  oracle.dequantize(Q6K, w, n * k).reshape(n, k).view(np.uint32))
        finally:
            W.free()
    finally:
        f.close()
