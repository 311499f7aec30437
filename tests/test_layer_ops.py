"""Decoder-layer operations on the device against the oracle.

Reference: swamp-engine/src/ops.rs (rmsnorm :188-201, init_rope_lut :20-38,
apply_rope_ufc :42-80, attention :82-186, silu/mul/add :203-220),
swamp-engine/src/cache.rs (PagedKVCache save / get and its tests :468-557),
sampler.rs:94-95 (greedy pick), executor.rs:416-418 (embedding row).

The reference holds no known-answer tests for these operations apart from
the KV cache's round trips and simd.rs's dot products; the oracle is pinned
by the hand-checkable cases below and otherwise by the source semantics.

Tolerances (written where used): RoPE, cache stores, residual add, argmax
and embedding rows are bit-exact. RMSNorm sums x^2 in a tree instead of a
running sum: relative 1e-4 (the running f32 sum of n squares is itself only
good to (n-1) * 2^-24 relative in the worst case). Attention sums in another
order and rescales split softmaxes: |out - ref| <= 1e-4 * max |v|. SiLU's
exp is CUDA's expf (within 2 ulp of libm's): relative 1e-6.
"""
import numpy as np
import pytest

from conftest import SEED

# ------------------------------------------------------------------ CPU pins


def test_synth_x_matches_oracle_generator():
    import swamp_gpu as sg
    import oracle
    g = sg.SwampGpu()
    for tid, n in ((1, 1), (2, 7), (3, 4096)):
        assert np.array_equal(g.synth_x(SEED, tid, (n,)), oracle.gen_x(SEED, tid, (n,)))


def test_rmsnorm_hand_case(oracle):
    x = np.array([3.0, 4.0], np.float32)
    w = np.array([1.0, 2.0], np.float32)
    inv = np.float32(1.0) / np.sqrt(np.float32(12.5) + np.float32(1e-5))
    assert np.array_equal(oracle.rmsnorm(x, w, 1e-5), np.array([x[0] * inv * w[0], x[1] * inv * w[1]], np.float32))


def test_rope_table_hand_values(oracle):
    """k = 0 has freq 1, so row m holds libm's cosf(m), sinf(m) (the functions
    Rust's f32::cos / sin call); row 0 is (1, 0); k = head_dim/4 has freq
    1 / powf(10000, 0.5) = 0.01."""
    import ctypes
    libm = ctypes.CDLL("libm.so.6")
    for f in ("cosf", "sinf", "powf"):
        getattr(libm, f).restype = ctypes.c_float
    libm.cosf.argtypes = libm.sinf.argtypes = [ctypes.c_float]
    libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    lut = oracle.rope_lut(128, 3)
    for m in range(3):
        assert lut[m, 0, 0] == np.float32(libm.cosf(float(m)))
        assert lut[m, 0, 1] == np.float32(libm.sinf(float(m)))
        assert abs(lut[m, 0, 0] - np.cos(m)) < 1e-7
    assert np.all(lut[0, :, 0] == 1.0) and np.all(lut[0, :, 1] == 0.0)
    freq = np.float32(1.0) / np.float32(libm.powf(10000.0, 0.5))
    assert lut[2, 32, 0] == np.float32(libm.cosf(float(np.float32(2.0) * freq)))


def test_rope_apply_clamps_position(oracle):
    lut = oracle.rope_lut(8, 4)
    q = oracle.gen_x(SEED, 5, (16,))
    k = oracle.gen_x(SEED, 6, (8,))
    a = oracle.rope_apply(q, k, 3, 2, 1, 8, 4, lut)
    b = oracle.rope_apply(q, k, 100, 2, 1, 8, 4, lut)  # ops.rs:54 pos.min(max_context - 1)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    z = oracle.rope_apply(q, k, 0, 2, 1, 8, 4, lut)   # angle 0: identity
    assert np.array_equal(z[0], q) and np.array_equal(z[1], k)


def test_attention_hand_cases(oracle):
    hd = 4
    v = np.arange(2 * hd, dtype=np.float32).reshape(1, 2, hd)
    k = np.zeros((1, 2, hd), np.float32)
    q = np.ones(2 * hd, np.float32)  # 2 query heads share the one KV head
    # one position: softmax = 1, out = v[0]
    out = oracle.attention(q, k[:, :1], v[:, :1], 1, 0, 2, 1, hd)
    assert np.array_equal(out, np.concatenate([v[0, 0], v[0, 0]]))
    # two positions with equal scores: p = 0.5 each
    out = oracle.attention(q, k, v, 2, 1, 2, 1, hd)
    assert np.array_equal(out[:hd], 0.5 * v[0, 0] + 0.5 * v[0, 1])
    # q_pos 0 with seq_len 2: position 1 is masked (ops.rs:145-147)
    out = oracle.attention(q, k, v, 2, 0, 2, 1, hd)
    assert np.array_equal(out[:hd], v[0, 0])


def test_argmax_rules(oracle):
    assert oracle.argmax(np.array([1, 5, 5, 2], np.float32)) == 2          # last of equal maxima
    assert oracle.argmax(np.array([0.0, -0.0], np.float32)) == 1           # -0 == +0
    assert oracle.argmax(np.array([-np.inf, -np.inf], np.float32)) == 1
    assert oracle.argmax(np.array([1, np.nan, 3], np.float32)) == -1       # the reference panics


def test_silu_mul_and_add(oracle):
    g = np.array([0.0, 1.0, -1.0, 20.0, -100.0], np.float32)
    u = np.array([1.0, 2.0, 3.0, 1.0, 1.0], np.float32)
    got = oracle.silu_mul(g, u)
    e = lambda t: np.float32(np.exp(np.float64(t)))
    assert got[0] == 0.0 and got[4] == 0.0
    assert abs(got[1] - np.float32(1.0 / (1.0 + e(-1.0))) * 2) <= 2e-7
    assert np.array_equal(oracle.add(u, g), u + g)


# ---------------------------------------------------------------------- GPU

def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(scope="module")
def ops(gpu):
    import swamp_gpu as sg
    return sg.LayerOps(gpu)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,n,k", [(2, 300, 320), (12, 129, 512), (14, 70, 768)])
def test_synth_blocks_match_oracle(gpu, oracle, dtype, n, k):
    raw = gpu.synth_blocks(dtype, SEED, 77, n, k)
    assert np.array_equal(raw, oracle.gen_weight(dtype, SEED, 77, n, k))
    W = gpu.synth_weight(dtype, SEED, 77, n, k)
    try:
        assert np.array_equal(gpu.dequant(W).view(np.uint32),
                              oracle.dequantize(dtype, raw, n * k).reshape(n, k).view(np.uint32))
    finally:
        W.free()


@pytest.mark.gpu
@pytest.mark.parametrize("n,rows", [(4096, 3), (5, 2), (14336, 1)])
def test_rmsnorm(gpu, oracle, ops, n, rows):
    import torch
    x = oracle.gen_x(SEED, 100 + n, (rows, n))
    w = (1 + 0.1 * oracle.gen_x(SEED, 101, (n,))).astype(np.float32)
    xd, wd = _t(x), _t(w)
    out = torch.full_like(xd, float("nan"))
    ops.rmsnorm(xd.data_ptr(), n, wd.data_ptr(), out.data_ptr(), n, n, rows, 1e-5)
    inplace = xd.clone()
    ops.rmsnorm(inplace.data_ptr(), n, wd.data_ptr(), inplace.data_ptr(), n, n, rows, 1e-5)
    got, got2 = out.cpu().numpy(), inplace.cpu().numpy()
    for r in range(rows):
        ref = oracle.rmsnorm(x[r], w, 1e-5)
        assert np.all(np.abs(got[r] - ref) <= 1e-4 * np.abs(ref) + 1e-30)
    assert np.array_equal(got, got2)


@pytest.mark.gpu
@pytest.mark.parametrize("hd,ctx", [(128, 300), (64, 17), (256, 5)])
def test_rope_table_bit_exact(gpu, oracle, hd, ctx):
    import swamp_gpu as sg
    r = sg.Rope(gpu, hd, ctx)
    try:
        assert np.array_equal(r.table().view(np.uint32), oracle.rope_lut(hd, ctx).view(np.uint32))
    finally:
        r.free()


@pytest.mark.gpu
def test_rope_kv_store_bit_exact(gpu, oracle, ops):
    import swamp_gpu as sg
    nq, nkv, hd, ctx, L, max_seq = 8, 2, 128, 40, 3, 64
    rope = sg.Rope(gpu, hd, ctx)
    cache = sg.KvCache(gpu, L, nkv, hd, max_seq, n_seqs=2)
    try:
        rows = 5
        pos = np.array([0, 7, 39, 45, 63], np.int32)  # 45, 63 past max_context: table row 39
        seq = np.array([0, 1, 1, 0, 1], np.int32)
        q = oracle.gen_x(SEED, 200, (rows, nq * hd))
        k = oracle.gen_x(SEED, 201, (rows, nkv * hd))
        v = oracle.gen_x(SEED, 202, (rows, nkv * hd))
        qd, kd, vd, pd, sd = _t(q), _t(k), _t(v), _t(pos), _t(seq)
        ops.rope_kv(rope, cache, 2, qd.data_ptr(), nq * hd, kd.data_ptr(), nkv * hd, vd.data_ptr(), nkv * hd,
                    pd.data_ptr(), sd.data_ptr(), rows, nq)
        gpu.synchronize()
        lut = oracle.rope_lut(hd, ctx)
        qg, kg = qd.cpu().numpy(), kd.cpu().numpy()
        for r in range(rows):
            qr, kr = oracle.rope_apply(q[r], k[r], int(pos[r]), nq, nkv, hd, ctx, lut)
            assert np.array_equal(qg[r].view(np.uint32), qr.view(np.uint32))
            assert np.array_equal(kg[r].view(np.uint32), kr.view(np.uint32))
            for h in range(nkv):
                kp, vp = cache.ptrs(int(seq[r]), 2, h)
                kc = _read_f32(kp + 4 * int(pos[r]) * hd, hd)
                vc = _read_f32(vp + 4 * int(pos[r]) * hd, hd)
                assert np.array_equal(kc, kr[h * hd:(h + 1) * hd])
                assert np.array_equal(vc, v[r, h * hd:(h + 1) * hd])
    finally:
        rope.free()
        cache.free()


def _read_f32(ptr, n):
    """Copy n floats at a raw device address to the host."""
    import torch
    torch.cuda.synchronize()
    return torch.as_tensor(_DevView(ptr, n), device="cuda").cpu().numpy()


class _DevView:
    """__cuda_array_interface__ over a raw device address (test helper)."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}


def _store(ops, cache, layer, k, v, pos, seq=None):
    """PagedKVCache::save_at without rotation."""
    rows = k.shape[0]
    kd, vd, pd = _t(k), _t(v), _t(np.asarray(pos, np.int32))
    sd = _t(np.asarray(seq, np.int32)) if seq is not None else None
    ops.rope_kv(None, cache, layer, 0, 0, kd.data_ptr(), k.shape[1], vd.data_ptr(), v.shape[1], pd.data_ptr(),
                sd.data_ptr() if sd is not None else None, rows, 0)


@pytest.mark.gpu
def test_reference_cache_tests(gpu, ops):
    """cache.rs:468-557 (basic_rw, multiple_pages, reset), on the device cache."""
    import swamp_gpu as sg
    # test_paged_cache_basic_rw: 2 layers, 4 kv heads, head_dim 64, 3 positions
    c = sg.KvCache(gpu, 2, 4, 64, 128)
    try:
        for pos in range(3):
            k = np.zeros((1, 4 * 64), np.float32)
            v = np.zeros((1, 4 * 64), np.float32)
            for h in range(4):
                k[0, h * 64] = pos * 100 + h
                v[0, h * 64] = pos * 1000 + h
            for l in range(2):
                _store(ops, c, l, k, v, [pos])
        gpu.synchronize()
        for l in range(2):
            for h in range(4):
                kp, vp = c.ptrs(0, l, h)
                for pos in range(3):
                    assert _read_f32(kp + 4 * pos * 64, 1)[0] == pos * 100 + h
                    assert _read_f32(vp + 4 * pos * 64, 1)[0] == pos * 1000 + h
    finally:
        c.free()
    # test_paged_cache_multiple_pages: 32 tokens (pages of 8 in the reference)
    c = sg.KvCache(gpu, 1, 1, 64, 1024)
    try:
        k = np.repeat(np.arange(32, dtype=np.float32)[:, None], 64, axis=1)
        _store(ops, c, 0, k, 2 * k, list(range(32)))
        gpu.synchronize()
        kp, vp = c.ptrs(0, 0, 0)
        kk = _read_f32(kp, 32 * 64).reshape(32, 64)
        vv = _read_f32(vp, 32 * 64).reshape(32, 64)
        assert np.array_equal(kk[:, 0], np.arange(32)) and np.array_equal(vv[:, 0], 2 * np.arange(32))
        # test_paged_cache_reset: position 0 written again
        _store(ops, c, 0, np.full((1, 64), 42.0, np.float32), np.full((1, 64), 42.0, np.float32), [0])
        gpu.synchronize()
        assert _read_f32(kp, 1)[0] == 42.0
    finally:
        c.free()


def _attention_case(gpu, oracle, ops, nq, nkv, hd, max_seq, rows_pos_seq, seq_lens=None):
    import torch
    import swamp_gpu as sg
    L, layer, n_seqs = 2, 1, 1 + max(s for _, s in rows_pos_seq)
    cache = sg.KvCache(gpu, L, nkv, hd, max_seq, n_seqs)
    try:
        K = oracle.gen_x(SEED, 300 + hd, (n_seqs, nkv, max_seq, hd))
        V = oracle.gen_x(SEED, 301 + hd, (n_seqs, nkv, max_seq, hd))
        for s in range(n_seqs):
            kk = np.ascontiguousarray(K[s].transpose(1, 0, 2).reshape(max_seq, nkv * hd))
            vv = np.ascontiguousarray(V[s].transpose(1, 0, 2).reshape(max_seq, nkv * hd))
            _store(ops, cache, layer, kk, vv, list(range(max_seq)), [s] * max_seq)
        rows = len(rows_pos_seq)
        pos = np.array([p for p, _ in rows_pos_seq], np.int32)
        seq = np.array([s for _, s in rows_pos_seq], np.int32)
        q = oracle.gen_x(SEED, 302, (rows, nq * hd))
        out = torch.full((rows, nq * hd + 4), float("nan"), device="cuda")
        qd, pd, sd = _t(q), _t(pos), _t(seq)
        sl = _t(np.asarray(seq_lens, np.int32)) if seq_lens is not None else None
        ops.attention(cache, layer, qd.data_ptr(), nq * hd, out.data_ptr(), nq * hd + 4, pd.data_ptr(),
                      sl.data_ptr() if sl is not None else None, sd.data_ptr(), rows, nq)
        gpu.synchronize()
        got = out.cpu().numpy()[:, :nq * hd]
        for r in range(rows):
            slen = int(seq_lens[r]) if seq_lens is not None else int(pos[r]) + 1
            ref = oracle.attention(q[r], K[seq[r]], V[seq[r]], slen, int(pos[r]), nq, nkv, hd)
            bound = 1e-4 * np.abs(V[seq[r]]).max()
            err = np.abs(got[r] - ref).max()
            assert err <= bound, (r, err, bound)
    finally:
        cache.free()


@pytest.mark.gpu
@pytest.mark.parametrize("nq,nkv,hd", [(32, 8, 128), (8, 8, 64), (16, 2, 256), (4, 1, 64)])
def test_attention_decode_rows(gpu, oracle, ops, nq, nkv, hd):
    # positions around the 128-position split boundaries, several sequences
    _attention_case(gpu, oracle, ops, nq, nkv, hd, 300,
                    [(0, 0), (1, 1), (127, 2), (128, 0), (129, 1), (255, 2), (299, 0)])


@pytest.mark.gpu
def test_attention_prefill_causal_and_seq_len(gpu, oracle, ops):
    # prefill rows of one sequence (q_pos = t, seq_len = t + 1), then rows
    # whose seq_len cuts below q_pos (valid_end = seq_len - 1, ops.rs:95)
    _attention_case(gpu, oracle, ops, 8, 2, 128, 200, [(t, 0) for t in range(0, 200, 7)])
    _attention_case(gpu, oracle, ops, 8, 2, 128, 200, [(150, 0), (150, 0), (10, 0)], seq_lens=[151, 40, 200])


@pytest.mark.gpu
def test_silu_mul_and_add_device(gpu, oracle, ops):
    import torch
    rows, n = 3, 14336
    g = 4 * oracle.gen_x(SEED, 400, (rows, n))
    u = oracle.gen_x(SEED, 401, (rows, n))
    gd, ud = _t(g), _t(u)
    ops.silu_mul(gd.data_ptr(), n, ud.data_ptr(), n, n, rows)
    got = gd.cpu().numpy()
    for r in range(rows):
        ref = oracle.silu_mul(g[r], u[r])
        assert np.all(np.abs(got[r] - ref) <= 1e-6 * np.abs(ref) + 1e-37)
    xd = _t(g)
    ops.add(xd.data_ptr(), n, ud.data_ptr(), n, n, rows)
    assert np.array_equal(xd.cpu().numpy(), g + u)
    # strided rows: only the first n of each ld are touched
    big = torch.zeros(rows, n + 8, device="cuda")
    ops.add(big.data_ptr(), n + 8, ud.data_ptr(), n, n, rows)
    b = big.cpu().numpy()
    assert np.array_equal(b[:, :n], u) and np.all(b[:, n:] == 0)
    # odd widths take the one-element path: same results
    n2 = 7
    g2, u2 = 4 * oracle.gen_x(SEED, 402, (rows, n2)), oracle.gen_x(SEED, 403, (rows, n2))
    g2d, u2d = _t(g2), _t(u2)
    ops.silu_mul(g2d.data_ptr(), n2, u2d.data_ptr(), n2, n2, rows)
    got2 = g2d.cpu().numpy()
    for r in range(rows):
        ref = oracle.silu_mul(g2[r], u2[r])
        assert np.all(np.abs(got2[r] - ref) <= 1e-6 * np.abs(ref) + 1e-37)
    x2d = _t(g2)
    ops.add(x2d.data_ptr(), n2, u2d.data_ptr(), n2, n2, rows)
    assert np.array_equal(x2d.cpu().numpy(), g2 + u2)


@pytest.mark.gpu
def test_argmax_device(gpu, oracle, ops):
    import torch
    V = 128256
    rows = [oracle.gen_x(SEED, 500 + i, (V,)) for i in range(3)]
    rows[1][[5, 77777, 128255]] = 9.0                      # ties: the last wins
    rows.append(np.full(V, -np.inf, np.float32))
    z = np.zeros(V, np.float32)
    z[10] = -0.0
    rows.append(z)                                         # all equal: the last
    n = oracle.gen_x(SEED, 510, (V,))
    n[4000] = np.nan
    rows.append(n)                                         # NaN: -1
    L = np.stack(rows)
    out = torch.full((len(rows),), -7, dtype=torch.int32, device="cuda")
    Ld = _t(L)
    ops.argmax(Ld.data_ptr(), V, V, len(rows), out.data_ptr())
    assert out.cpu().tolist() == [oracle.argmax(r) for r in rows]
    assert out.cpu().tolist()[1] == 128255 and out.cpu().tolist()[-1] == -1
    # calls of other shapes reuse the per-row state: results stay exact
    for shape in ((1, 5000), (2, 4096), (3, 1), (8, 128256), (1, 128256)):
        R, n = shape
        L2 = oracle.gen_x(SEED, 520 + n, (R, n))
        o2 = torch.full((R,), -7, dtype=torch.int32, device="cuda")
        L2d = _t(L2)
        ops.argmax(L2d.data_ptr(), n, n, R, o2.data_ptr())
        assert o2.cpu().tolist() == [oracle.argmax(r) for r in L2], shape


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [2, 12, 14])
def test_embed_rows_bit_exact(gpu, oracle, ops, dtype):
    import torch
    vocab, d = 1000, 512
    raw = oracle.gen_weight(dtype, SEED, 600, vocab, d)
    W = gpu.register(raw, dtype, vocab, d)
    try:
        table = oracle.dequantize(dtype, raw, vocab * d).reshape(vocab, d)
        toks = np.array([0, 999, 128, 129, 5, 5], np.int32)
        out = torch.full((len(toks), d + 4), float("nan"), device="cuda")
        td = _t(toks)
        ops.embed(W, td.data_ptr(), len(toks), out.data_ptr(), d + 4)
        gpu.synchronize()
        assert np.array_equal(out.cpu().numpy()[:, :d].view(np.uint32), table[toks].view(np.uint32))
    finally:
        W.free()


@pytest.mark.gpu
def test_device_index_out_of_range_is_reported(gpu, ops):
    """A token outside the table: the kernel skips the row, zero-fills it and
    flags the device; the next synchronize reports SG_ERR_DEVICE_FAULT."""
    import torch
    import swamp_gpu as sg
    W = gpu.synth_weight(12, SEED, 601, 300, 256)
    try:
        toks = _t(np.array([3, 300], np.int32))
        out = torch.full((2, 256), float("nan"), device="cuda")
        ops.embed(W, toks.data_ptr(), 2, out.data_ptr(), 256)
        with pytest.raises(sg.SwampGpuError) as e:
            gpu.synchronize()
        assert e.value.code == -7 and "out of range" in str(e.value)
        assert np.all(out.cpu().numpy()[1] == 0)
        gpu.synchronize()  # the flag was consumed
    finally:
        W.free()


@pytest.mark.gpu
def test_host_validation(gpu, ops):
    import swamp_gpu as sg
    with pytest.raises(sg.SwampGpuError):
        sg.KvCache(gpu, 1, 1, 6, 8)        # head_dim not a multiple of 4
    c = sg.KvCache(gpu, 1, 2, 96, 8)
    try:
        with pytest.raises(sg.SwampGpuError) as e:  # head_dim 96 has no attention kernel
            ops.attention(c, 0, 16, 192, 16, 192, 16, None, None, 1, 2)
        assert e.value.code == -5
    finally:
        c.free()
    c = sg.KvCache(gpu, 1, 2, 64, 8)
    try:
        with pytest.raises(sg.SwampGpuError) as e:  # 3 query heads over 2 KV heads
            ops.attention(c, 0, 16, 192, 16, 192, 16, None, None, 1, 3)
        assert e.value.code == -5
    finally:
        c.free()
    with pytest.raises(sg.SwampGpuError):
        ops.rmsnorm(16, 4, 16, 16, 4, 8, 1, 1e-5)  # ldx < n


@pytest.mark.gpu
@pytest.mark.parametrize("nq,nkv,hd,max_seq", [(32, 8, 128, 200), (8, 2, 64, 200), (16, 2, 256, 200),
                                               (8, 2, 64, 4300)])
def test_rope_attention_fused_matches_two_calls(gpu, oracle, ops, nq, nkv, hd, max_seq):
    """sg_rope_attention_device (one row per sequence) gives the same bits as
    sg_rope_kv_device + sg_attention_device, output and cache, at positions
    on and around the 64-position split edges (and past 64 splits), over two
    calls in a row."""
    import torch
    import swamp_gpu as sg
    L, ctx = 2, 150
    rope = sg.Rope(gpu, hd, ctx)
    caches = [sg.KvCache(gpu, L, nkv, hd, max_seq, n_seqs=6) for _ in range(2)]
    try:
        # shared history: positions 0..199 of every sequence, stored in both caches
        hist_k = oracle.gen_x(SEED, 700 + hd, (max_seq, nkv * hd))
        hist_v = oracle.gen_x(SEED, 701 + hd, (max_seq, nkv * hd))
        for c in caches:
            for s in range(6):
                _store(ops, c, 1, hist_k, hist_v, list(range(max_seq)), [s] * max_seq)
        plan = ([0, 63, 64, 65, 160, 199], [1, 127, 128, 129, 10, 198])
        if max_seq > 4096:
            plan = ([4290, 64, 4100, 0, 4160, 4299], [4291, 4095, 4096, 1, 2000, 4097])
        for call, pos in enumerate(plan):
            rows = len(pos)
            q = oracle.gen_x(SEED, 710 + call, (rows, nq * hd))
            k = oracle.gen_x(SEED, 711 + call, (rows, nkv * hd))
            v = oracle.gen_x(SEED, 712 + call, (rows, nkv * hd))
            pd = _t(np.array(pos, np.int32))
            sd = _t(np.array([5, 0, 3, 1, 2, 4], np.int32))
            # two-call form on cache 0
            q0, k0, v0 = _t(q), _t(k), _t(v)
            out0 = torch.full((rows, nq * hd), float("nan"), device="cuda")
            ops.rope_kv(rope, caches[0], 1, q0.data_ptr(), nq * hd, k0.data_ptr(), nkv * hd, v0.data_ptr(), nkv * hd,
                        pd.data_ptr(), sd.data_ptr(), rows, nq)
            ops.attention(caches[0], 1, q0.data_ptr(), nq * hd, out0.data_ptr(), nq * hd, pd.data_ptr(), None,
                          sd.data_ptr(), rows, nq)
            # fused form on cache 1
            q1, k1, v1 = _t(q), _t(k), _t(v)
            out1 = torch.full((rows, nq * hd), float("nan"), device="cuda")
            ops.rope_attention(rope, caches[1], 1, q1.data_ptr(), nq * hd, k1.data_ptr(), nkv * hd, v1.data_ptr(),
                               nkv * hd, out1.data_ptr(), nq * hd, pd.data_ptr(), sd.data_ptr(), rows, nq)
            gpu.synchronize()
            assert np.array_equal(out0.cpu().numpy().view(np.uint32), out1.cpu().numpy().view(np.uint32))
            assert np.array_equal(q1.cpu().numpy(), q) and np.array_equal(k1.cpu().numpy(), k)
            for s in range(6):
                for h in range(nkv):
                    a = [_read_f32(p, max_seq * hd) for p in caches[0].ptrs(s, 1, h)]
                    b = [_read_f32(p, max_seq * hd) for p in caches[1].ptrs(s, 1, h)]
                    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    finally:
        rope.free()
        for c in caches:
            c.free()


@pytest.mark.gpu
@pytest.mark.parametrize("nq,nkv,hd,n_seqs,n_tokens,seq_major", [(32, 8, 128, 1, 150, True), (8, 2, 64, 2, 77, False),
                                                                 (8, 8, 64, 2, 130, True), (16, 8, 128, 3, 40, False)])
def test_attention_prefill_matches_oracle(gpu, oracle, ops, nq, nkv, hd, n_seqs, n_tokens, seq_major):
    """sg_attention_prefill_device over all prompt positions (row layouts
    sequence-major and position-major) against the oracle's per-position
    attention (|out - ref| <= 1e-4 * max |v|) and the per-row kernel."""
    import torch
    import swamp_gpu as sg
    max_seq = 256
    cache = sg.KvCache(gpu, 2, nkv, hd, max_seq, n_seqs)
    try:
        K = oracle.gen_x(SEED, 800 + hd, (n_seqs, nkv, max_seq, hd))
        V = oracle.gen_x(SEED, 801 + hd, (n_seqs, nkv, max_seq, hd))
        for s in range(n_seqs):
            kk = np.ascontiguousarray(K[s].transpose(1, 0, 2).reshape(max_seq, nkv * hd))
            vv = np.ascontiguousarray(V[s].transpose(1, 0, 2).reshape(max_seq, nkv * hd))
            _store(ops, cache, 1, kk, vv, list(range(max_seq)), [s] * max_seq)
        rows = n_seqs * n_tokens
        rs_seq, rs_pos = (n_tokens, 1) if seq_major else (1, n_seqs)
        seq_of = np.empty(rows, np.int32)
        pos_of = np.empty(rows, np.int32)
        for s in range(n_seqs):
            for t in range(n_tokens):
                seq_of[s * rs_seq + t * rs_pos] = s
                pos_of[s * rs_seq + t * rs_pos] = t
        q = oracle.gen_x(SEED, 802, (rows, nq * hd))
        qd = _t(q)
        out = torch.full((rows, nq * hd), float("nan"), device="cuda")
        ops.attention_prefill(cache, 1, qd.data_ptr(), nq * hd, out.data_ptr(), nq * hd, n_seqs, n_tokens, rs_seq,
                              rs_pos, nq)
        out_rows = torch.full((rows, nq * hd), float("nan"), device="cuda")
        pd, sd = _t(pos_of), _t(seq_of)  # held until the kernel has run
        ops.attention(cache, 1, qd.data_ptr(), nq * hd, out_rows.data_ptr(), nq * hd, pd.data_ptr(), None,
                      sd.data_ptr(), rows, nq)
        gpu.synchronize()
        got, got_rows = out.cpu().numpy(), out_rows.cpu().numpy()
        for r in range(rows):
            s, t = int(seq_of[r]), int(pos_of[r])
            ref = oracle.attention(q[r], K[s], V[s], t + 1, t, nq, nkv, hd)
            bound = 1e-4 * np.abs(V[s]).max()
            assert np.abs(got[r] - ref).max() <= bound, (r, np.abs(got[r] - ref).max(), bound)
            assert np.abs(got[r] - got_rows[r]).max() <= bound
    finally:
        cache.free()


@pytest.mark.gpu
def test_prefill_and_fused_attention_reject_bad_shapes(gpu, ops):
    """Host-side checks of the prefill and decode-form attention: nothing is
    launched for shapes outside the cache or the kernels."""
    import swamp_gpu as sg
    c = sg.KvCache(gpu, 1, 2, 64, 32, n_seqs=2)
    r = sg.Rope(gpu, 64, 32)
    try:
        bad = [
            dict(n_seqs=3, n_tokens=8),    # more sequences than the cache holds
            dict(n_seqs=1, n_tokens=33),   # more positions than the cache holds
        ]
        for b in bad:
            with pytest.raises(sg.SwampGpuError):
                ops.attention_prefill(c, 0, 16, 256, 16, 256, b["n_seqs"], b["n_tokens"], 1, 1, 4)
        with pytest.raises(sg.SwampGpuError):  # 3 query heads over 2 KV heads
            ops.attention_prefill(c, 0, 16, 256, 16, 256, 1, 8, 1, 1, 3)
        with pytest.raises(sg.SwampGpuError):  # one row per sequence: 3 rows > 2 sequences
            ops.rope_attention(r, c, 0, 16, 256, 16, 128, 16, 128, 16, 256, 16, None, 3, 4)
        c256 = sg.KvCache(gpu, 1, 1, 256, 8)
        try:
            with pytest.raises(sg.SwampGpuError) as e:  # the prefill kernel covers head_dim 64 and 128
                ops.attention_prefill(c256, 0, 16, 256, 16, 256, 1, 4, 1, 1, 1)
            assert e.value.code == -5
        finally:
            c256.free()
    finally:
        r.free()
        c.free()


def test_oracle_attention_and_norm_against_float64(oracle):
    """The oracle's restatements against independent float64 numpy versions
    of the same formulas (ops.rs:82-201): attention within 1e-5 * max |v|,
    RMSNorm within 1e-5 relative, on GQA shapes and several positions."""
    nq, nkv, hd, T = 8, 2, 64, 40
    K = oracle.gen_x(SEED, 900, (nkv, T, hd)).astype(np.float32)
    V = oracle.gen_x(SEED, 901, (nkv, T, hd)).astype(np.float32)
    q = oracle.gen_x(SEED, 902, (nq * hd,))
    for pos in (0, 1, 17, 39):
        got = oracle.attention(q, K, V, pos + 1, pos, nq, nkv, hd)
        want = np.empty(nq * hd)
        for h in range(nq):
            kh, vh = K[h // (nq // nkv)].astype(np.float64), V[h // (nq // nkv)].astype(np.float64)
            s = kh[:pos + 1] @ q[h * hd:(h + 1) * hd].astype(np.float64) / np.sqrt(hd)
            p = np.exp(s - s.max())
            want[h * hd:(h + 1) * hd] = (p / p.sum()) @ vh[:pos + 1]
        assert np.abs(got - want).max() <= 1e-5 * np.abs(V).max(), pos
    x = oracle.gen_x(SEED, 903, (4096,))
    w = (1 + 0.1 * oracle.gen_x(SEED, 904, (4096,))).astype(np.float32)
    x64 = x.astype(np.float64)
    want = x64 / np.sqrt(np.mean(x64 * x64) + 1e-5) * w
    got = oracle.rmsnorm(x, w, 1e-5)
    assert np.all(np.abs(got - want) <= 1e-5 * np.abs(want) + 1e-30)
