"""ctypes bindings to the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY. Imported by tests/, by __graft_entry__.smoke() and by
bench.py's CPU-baseline / reference arm, always as the checker or the timed CPU
baseline, never as the thing measured or shipped. The product package
(llamanyon.rs_b200/) must not import this module.

Each wrapper names the reference function it restates (paths inside the
llamanyon.rs workspace); the C source carries the line citations.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

DTYPE_Q4_0 = 2
DTYPE_Q4_K = 12
DTYPE_Q6_K = 14
BLOCK = {DTYPE_Q4_0: 32, DTYPE_Q4_K: 256, DTYPE_Q6_K: 256}
BLOCK_BYTES = {DTYPE_Q4_0: 18, DTYPE_Q4_K: 144, DTYPE_Q6_K: 210}

_lib = None


def build() -> str:
    """Compile liboracle.so with the committed Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        build()
    L = ctypes.CDLL(LIB_PATH)
    P = ctypes.c_void_p
    i64 = ctypes.c_int64
    L.orc_f16_to_f32.argtypes = [ctypes.c_uint16]
    L.orc_f16_to_f32.restype = ctypes.c_float
    L.orc_f32_to_f16.argtypes = [ctypes.c_float]
    L.orc_f32_to_f16.restype = ctypes.c_uint16
    L.orc_dequantize.argtypes = [ctypes.c_int, P, ctypes.c_size_t, P, ctypes.c_size_t]
    L.orc_dequantize.restype = ctypes.c_int
    L.orc_q4k_unpack_scales.argtypes = [P, P, P]
    L.orc_gemv_q4k_scalar.argtypes = [P, P, P, i64, i64]
    L.orc_gemv_q4k_batched_scalar.argtypes = [P, P, P, i64, i64, i64]
    L.orc_gemv_q4k_multi.argtypes = [P, P, P, P, i64, i64]
    L.orc_swamp_fused_gemv_q4k.argtypes = [P, P, P, ctypes.c_int, ctypes.c_int]
    L.orc_linear_q4_0.argtypes = [P, P, P, i64, i64, P]
    L.orc_linear_q4_0.restype = ctypes.c_int
    L.orc_forward_linear.argtypes = [ctypes.c_int, P, P, P, i64, i64, ctypes.c_int]
    L.orc_forward_linear.restype = ctypes.c_int
    L.orc_forward_linear_batch.argtypes = [ctypes.c_int, P, P, P, i64, i64, i64, ctypes.c_int]
    L.orc_forward_linear_batch.restype = ctypes.c_int
    L.orc_make_q4k_block.argtypes = [ctypes.c_float, ctypes.c_float, P, P, ctypes.c_uint8, P]
    L.orc_make_weight.argtypes = [i64, P]
    L.orc_make_x.argtypes = [i64, P]
    L.orc_splitmix64.argtypes = [ctypes.c_uint64]
    L.orc_splitmix64.restype = ctypes.c_uint64
    L.orc_gen_q4_0.argtypes = [ctypes.c_uint64, ctypes.c_uint64, i64, i64, P, ctypes.c_int]
    L.orc_gen_q4k.argtypes = [ctypes.c_uint64, ctypes.c_uint64, i64, i64, P, ctypes.c_int]
    L.orc_gen_q6k.argtypes = [ctypes.c_uint64, ctypes.c_uint64, i64, i64, P, ctypes.c_int]
    L.orc_gemv_q6k_scalar.argtypes = [P, P, P, i64, i64]
    L.orc_gen_x.argtypes = [ctypes.c_uint64, ctypes.c_uint64, i64, P]
    L.orc_gemv_f64.argtypes = [ctypes.c_int, P, P, i64, i64, P, P, P]
    L.orc_gemv_f64.restype = ctypes.c_int
    f32 = ctypes.c_float
    L.orc_rmsnorm.argtypes = [P, P, P, i64, f32]
    L.orc_rope_lut.argtypes = [ctypes.c_int, i64, P]
    L.orc_rope_apply.argtypes = [P, P, i64, ctypes.c_int, ctypes.c_int, ctypes.c_int, i64, P]
    L.orc_attention.argtypes = [P, P, P, P, i64, i64, i64, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    L.orc_silu_mul.argtypes = [P, P, i64]
    L.orc_add.argtypes = [P, P, i64]
    L.orc_argmax.argtypes = [P, i64]
    L.orc_argmax.restype = i64
    L.orc_simd_path.restype = ctypes.c_int
    L.orc_gemv_q4k_vnni.argtypes = [P, P, P, i64, i64]
    L.orc_gemv_q4k_vnni.restype = ctypes.c_int
    L.orc_gemv_q4k_avx2.argtypes = [P, P, P, i64, i64]
    L.orc_gemv_q4k_avx2.restype = ctypes.c_int
    L.orc_forward_linear_dispatched.argtypes = [P, P, P, i64, i64, ctypes.c_int]
    L.orc_forward_linear_dispatched.restype = ctypes.c_int
    L.orc_fallback_gemv_dispatched.argtypes = [P, P, P, i64, i64, i64, ctypes.c_int]
    L.orc_fallback_gemv_dispatched.restype = ctypes.c_int
    _lib = L
    return L


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def row_bytes(dtype: int, n_cols: int) -> int:
    return n_cols // BLOCK[dtype] * BLOCK_BYTES[dtype]


def f16_to_f32(h: int) -> float:
    return float(lib().orc_f16_to_f32(h))


def f32_to_f16(f: float) -> int:
    return int(lib().orc_f32_to_f16(f))


def dequantize(dtype: int, raw: np.ndarray, n: int) -> np.ndarray:
    """swamp-gguf quant::dequantize for Q4_0 (q4_0.rs), Q4_K (q4_k.rs scalar)
    and Q6_K (q6_k.rs)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty(n, dtype=np.float32)
    rc = lib().orc_dequantize(dtype, _p(raw), raw.size, _p(out), n)
    if rc != 0:
        raise ValueError(f"orc_dequantize failed rc={rc}")
    return out


def unpack_scales(sc12: np.ndarray):
    sc12 = np.ascontiguousarray(sc12, dtype=np.uint8)
    s = np.empty(8, np.uint8)
    m = np.empty(8, np.uint8)
    lib().orc_q4k_unpack_scales(_p(sc12), _p(s), _p(m))
    return s, m


def gemv_q4k_scalar(w: np.ndarray, x: np.ndarray, n_rows: int, n_cols: int) -> np.ndarray:
    """fused_gemv_q4k_scalar (swamp-kernels/src/fused_gemv_q4k.rs:466-508)."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(n_rows, np.float32)
    lib().orc_gemv_q4k_scalar(_p(w), _p(x), _p(out), n_rows, n_cols)
    return out


def gemv_q4k_batched_scalar(w, xs: np.ndarray, outs: np.ndarray, n_rows, n_cols) -> np.ndarray:
    """batched_scalar (fused_gemv_q4k.rs:650-698): outs[t] += W x_t."""
    xs = np.ascontiguousarray(xs, np.float32)
    B = xs.shape[0]
    xp = (ctypes.c_void_p * B)(*[xs[t].ctypes.data for t in range(B)])
    op = (ctypes.c_void_p * B)(*[outs[t].ctypes.data for t in range(B)])
    lib().orc_gemv_q4k_batched_scalar(_p(w), ctypes.addressof(xp), ctypes.addressof(op), n_rows, n_cols, B)
    return outs


def gemv_q6k_scalar(w: np.ndarray, x: np.ndarray, n_rows: int, n_cols: int) -> np.ndarray:
    """fused_gemv_q6k_scalar (swamp-kernels/src/fused_gemv_q6k.rs:248-291),
    the engine's Q6_K route (linear.rs:48-67), with the exact f16 decode."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(n_rows, np.float32)
    lib().orc_gemv_q6k_scalar(_p(w), _p(x), _p(out), n_rows, n_cols)
    return out


def linear_q4_0(w, x, n_rows, n_cols) -> np.ndarray:
    """Engine Q4_0 route (swamp-engine/src/linear.rs:68-87)."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(n_rows, np.float32)
    rc = lib().orc_linear_q4_0(_p(w), _p(x), _p(out), n_rows, n_cols, None)
    if rc:
        raise ValueError(rc)
    return out


def reference_linear(dtype: int, w, x: np.ndarray, n_rows: int, n_cols: int) -> np.ndarray:
    """The reference's fp32 result for one token: the scalar Q4_K kernel or the
    engine's Q4_0 route. x may be 1-D (K) or 2-D (B, K)."""
    x = np.ascontiguousarray(x, np.float32)
    if x.ndim == 1:
        x = x[None]
    out = np.empty((x.shape[0], n_rows), np.float32)
    for b in range(x.shape[0]):
        if dtype == DTYPE_Q4_K:
            out[b] = gemv_q4k_scalar(w, x[b], n_rows, n_cols)
        elif dtype == DTYPE_Q6_K:
            out[b] = gemv_q6k_scalar(w, x[b], n_rows, n_cols)
        else:
            out[b] = linear_q4_0(w, x[b], n_rows, n_cols)
    return out


def forward_linear(dtype, w, x, n_rows, n_cols, n_threads) -> np.ndarray:
    """swamp-engine forward_linear (linear.rs:14-90) on n_threads host threads."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(n_rows, np.float32)
    rc = lib().orc_forward_linear(dtype, _p(w), _p(x), _p(out), n_rows, n_cols, n_threads)
    if rc:
        raise ValueError(rc)
    return out


SIMD_PATHS = {0: "none", 1: "avx2", 2: "avx512-vnni"}


def simd_path() -> str:
    """The SIMD path the reference's fused_gemv_q4k dispatcher
    (fused_gemv_q4k.rs:59-82) takes on this CPU."""
    return SIMD_PATHS[lib().orc_simd_path()]


def gemv_q4k_simd(path: str, w, x, n_rows, n_cols) -> np.ndarray:
    """The reference's SIMD Q4_K GEMV ("avx512-vnni": fused_gemv_q4k.rs:101-317,
    "avx2": :325-392), single-threaded. TIMING ONLY: these paths do not compute
    the reference's dequantized dot product (the VNNI path drops the sub-block
    scales from the integer quire and quantizes x to int8), so their outputs
    are not a parity target."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(n_rows, np.float32)
    fn = lib().orc_gemv_q4k_vnni if path == "avx512-vnni" else lib().orc_gemv_q4k_avx2
    if fn(_p(w), _p(x), _p(out), n_rows, n_cols):
        raise RuntimeError(f"{path} not supported on this CPU")
    return out


def forward_linear_dispatched(w, x, n_rows, n_cols, n_threads):
    """forward_linear's Q4_K arm (linear.rs:28-46) as the reference runs it on
    this CPU: rows over n_threads threads, each chunk through the dispatched
    SIMD kernel. TIMING ONLY (numerically divergent, see gemv_q4k_simd).
    Returns (out, path)."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(n_rows, np.float32)
    rc = lib().orc_forward_linear_dispatched(_p(w), _p(x), _p(out), n_rows, n_cols, n_threads)
    if rc < 1:
        raise RuntimeError("no SIMD path on this CPU")
    return out, SIMD_PATHS[rc]


def fallback_gemv_dispatched(w, xs: np.ndarray, n_rows, n_cols, n_threads):
    """forward_linear_batch's route for tensors that are not Q4_K
    (linear.rs:233-236 -> fallback_gemv, :336-364) as the reference runs it
    on this CPU: tokens over n_threads threads, each a whole-tensor
    dispatched fused_gemv_q4k. For Q4_0 bytes that is the reference's
    batched Q4_0 route. TIMING ONLY (the Q4_K kernel does not decode Q4_0).
    Returns (outs, path)."""
    xs = np.ascontiguousarray(xs, np.float32)
    B = xs.shape[0]
    outs = np.empty((B, n_rows), np.float32)
    xp = (ctypes.c_void_p * B)(*[xs[t].ctypes.data for t in range(B)])
    op = (ctypes.c_void_p * B)(*[outs[t].ctypes.data for t in range(B)])
    rc = lib().orc_fallback_gemv_dispatched(_p(w), ctypes.addressof(xp), ctypes.addressof(op), B, n_rows,
                                            n_cols, n_threads)
    if rc < 1:
        raise RuntimeError("no SIMD path on this CPU" if rc == -1 else f"orc_fallback_gemv_dispatched rc={rc}")
    return outs, SIMD_PATHS[rc]


def forward_linear_batch(dtype, w, xs: np.ndarray, n_rows, n_cols, n_threads) -> np.ndarray:
    """swamp-engine forward_linear_batch (linear.rs:176-239)."""
    xs = np.ascontiguousarray(xs, np.float32)
    B = xs.shape[0]
    outs = np.zeros((B, n_rows), np.float32)
    xp = (ctypes.c_void_p * B)(*[xs[t].ctypes.data for t in range(B)])
    op = (ctypes.c_void_p * B)(*[outs[t].ctypes.data for t in range(B)])
    rc = lib().orc_forward_linear_batch(dtype, _p(w), ctypes.addressof(xp), ctypes.addressof(op),
                                        B, n_rows, n_cols, n_threads)
    if rc < 0:
        raise ValueError(rc)
    return outs


def make_q4k_block(d, dmin, scales, mins, nibble_val) -> np.ndarray:
    out = np.empty(144, np.uint8)
    s = np.ascontiguousarray(scales, np.uint8)
    m = np.ascontiguousarray(mins, np.uint8)
    lib().orc_make_q4k_block(d, dmin, _p(s), _p(m), nibble_val, _p(out))
    return out


def make_weight(n_rows: int) -> np.ndarray:
    """Reference test fixture make_weight (fused_gemv_q4k.rs:726-736), K=256."""
    out = np.empty(n_rows * 144, np.uint8)
    lib().orc_make_weight(n_rows, _p(out))
    return out


def make_x(n_cols: int) -> np.ndarray:
    """Reference test fixture make_x (fused_gemv_q4k.rs:738-740)."""
    out = np.empty(n_cols, np.float32)
    lib().orc_make_x(n_cols, _p(out))
    return out


def gen_weight(dtype: int, seed: int, tensor_id: int, n_rows: int, n_cols: int,
               n_threads: int | None = None) -> np.ndarray:
    """Seeded raw GGUF blocks (row-major, n_rows*row_bytes)."""
    n_threads = n_threads or min(os.cpu_count() or 1, 64)
    out = np.empty(n_rows * row_bytes(dtype, n_cols), np.uint8)
    if dtype == DTYPE_Q4_0:
        lib().orc_gen_q4_0(seed, tensor_id, n_rows, n_cols, _p(out), n_threads)
    elif dtype == DTYPE_Q6_K:
        lib().orc_gen_q6k(seed, tensor_id, n_rows, n_cols, _p(out), n_threads)
    else:
        lib().orc_gen_q4k(seed, tensor_id, n_rows, n_cols, _p(out), n_threads)
    return out


def gen_x(seed: int, tensor_id: int, shape) -> np.ndarray:
    n = int(np.prod(shape))
    out = np.empty(n, np.float32)
    lib().orc_gen_x(seed, tensor_id, n, _p(out))
    return out.reshape(shape)


def gemv_f64(dtype, w, x, n_rows, n_cols):
    """fp64 dot of the dequantized weights plus sum|w x| and ||w*x||_2 per row."""
    x = np.ascontiguousarray(x, np.float32)
    o = np.empty(n_rows, np.float64)
    a = np.empty(n_rows, np.float64)
    l2 = np.empty(n_rows, np.float64)
    rc = lib().orc_gemv_f64(dtype, _p(w), _p(x), n_rows, n_cols, _p(o), _p(a), _p(l2))
    if rc:
        raise ValueError(rc)
    return o, a, l2


# ------------------------------------------------------------ decoder-layer ops

def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, np.float32)


def rmsnorm(x, w, eps: float) -> np.ndarray:
    """swamp-engine ops::rmsnorm (ops.rs:188-201) of one row."""
    x, w = _f32(x), _f32(w)
    out = np.empty_like(x)
    lib().orc_rmsnorm(_p(x), _p(w), _p(out), x.size, eps)
    return out


def rope_lut(head_dim: int, max_seq_len: int) -> np.ndarray:
    """ops::init_rope_lut (ops.rs:20-38): [max_seq_len][head_dim/2][cos, sin]."""
    out = np.empty((max_seq_len, head_dim // 2, 2), np.float32)
    lib().orc_rope_lut(head_dim, max_seq_len, _p(out))
    return out


def rope_apply(q, k, pos, n_q_heads, n_kv_heads, head_dim, max_context, lut):
    """ops::apply_rope_ufc (ops.rs:42-80) of one token; returns rotated copies."""
    q, k, lut = _f32(q).copy(), _f32(k).copy(), _f32(lut)
    lib().orc_rope_apply(_p(q), _p(k), pos, n_q_heads, n_kv_heads, head_dim, max_context, _p(lut))
    return q, k


def attention(q, k_cache, v_cache, seq_len, q_pos, n_heads, n_kv_heads, head_dim) -> np.ndarray:
    """ops::attention (ops.rs:82-186) of one token. k_cache / v_cache:
    [n_kv_heads][positions][head_dim] of this sequence and layer."""
    q, kc, vc = _f32(q), _f32(k_cache), _f32(v_cache)
    assert kc.shape == vc.shape and kc.shape[0] == n_kv_heads and kc.shape[2] == head_dim
    assert min(q_pos, seq_len - 1) < kc.shape[1]
    out = np.empty(n_heads * head_dim, np.float32)
    lib().orc_attention(_p(out), _p(q), _p(kc), _p(vc), kc.shape[1] * head_dim, seq_len, q_pos,
                        n_heads, n_kv_heads, head_dim)
    return out


def silu_mul(g, u) -> np.ndarray:
    """ops::silu then ops::mul_in_place (ops.rs:203-214)."""
    g, u = _f32(g).copy(), _f32(u)
    lib().orc_silu_mul(_p(g), _p(u), g.size)
    return g


def add(a, b) -> np.ndarray:
    """ops::add_in_place (ops.rs:216-220)."""
    a, b = _f32(a).copy(), _f32(b)
    lib().orc_add(_p(a), _p(b), a.size)
    return a


def argmax(logits) -> int:
    """Greedy pick: the sampler's max_by fallback (sampler.rs:94-95), the last
    of equal maxima; -1 for a row with a NaN (the reference panics)."""
    l = _f32(logits)
    return int(lib().orc_argmax(_p(l), l.size))
