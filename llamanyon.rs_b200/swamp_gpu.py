"""Python binding of libswamp_gpu.so (the C ABI in include/swamp_gpu.h).

Mirrors the reference's linear-layer interface (swamp-engine/src/linear.rs):
``forward_linear``, ``forward_linear_multi``, ``forward_linear_batch`` and
``forward_gemvs`` take a registered tensor (the GGUF TensorInfo + raw block
bytes) and f32 activations, with the same overwrite semantics and errors
raised as exceptions (the Rust functions return anyhow::Result). There is no
CPU fallback: if the shared library or a usable sm_100 GPU is missing, every
entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import weakref
from dataclasses import dataclass
from typing import Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libswamp_gpu.so")

SG_OK = 0
SG_DTYPE_Q4_0 = 2
SG_DTYPE_Q4_K = 12
SG_DTYPE_Q6_K = 14
SG_TP_REPLICATE, SG_TP_COLUMN, SG_TP_ROW = 0, 1, 2
SG_FLAG_DEVICE_PTRS = 0x1
SG_FLAG_ACCUMULATE = 0x2

BLOCK = {SG_DTYPE_Q4_0: 32, SG_DTYPE_Q4_K: 256, SG_DTYPE_Q6_K: 256}
BLOCK_BYTES = {SG_DTYPE_Q4_0: 18, SG_DTYPE_Q4_K: 144, SG_DTYPE_Q6_K: 210}

# every symbol include/swamp_gpu.h declares
EXPORTS = (
    "sg_init", "sg_get_unique_id", "sg_init_rank", "sg_shutdown", "sg_last_error", "sg_topology",
    "sg_weight_register", "sg_weight_free", "sg_tp_shard", "sg_weight_shard", "sg_linear", "sg_linear_multi",
    "sg_linear_device", "sg_linear_multi_device", "sg_linear_device_noalloc", "sg_dequant_f32", "sg_fused_gemv_q4k",
    "sg_synchronize", "sg_gguf_open", "sg_gguf_open_memory", "sg_gguf_close", "sg_gguf_header",
    "sg_gguf_find_tensor", "sg_gguf_tensor_info", "sg_gguf_tensor_data", "sg_gguf_find_kv", "sg_gguf_kv_info",
    "sg_gguf_kv_int", "sg_gguf_kv_float", "sg_gguf_kv_string", "sg_gguf_register",
    "sg_synth_weight", "sg_synth_blocks", "sg_synth_x",
    "sg_rope_create", "sg_rope_free", "sg_rope_table", "sg_kv_cache_create", "sg_kv_cache_free", "sg_kv_cache_ptr",
    "sg_rmsnorm_device", "sg_rope_kv_device", "sg_attention_device", "sg_rope_attention_device", "sg_attention_prefill_device", "sg_silu_mul_device", "sg_add_device",
    "sg_rmsnorm_linear_multi_device", "sg_silu_mul_linear_device",
    "sg_argmax_device", "sg_embed_device", "sg_allreduce_device", "sg_allreduce_path",
    "sg_host_alloc", "sg_host_free",
)
SG_ERR_FORMAT, SG_ERR_NOT_FOUND = -8, -9


class SwampGpuError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"swamp_gpu error {code}: {msg}")
        self.code = code


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    if not os.path.exists(path):
        raise SwampGpuError(-5, f"{path} is missing; run llamanyon.rs_b200/build_lib.py (no CPU fallback)")
    L = ctypes.CDLL(path)
    P, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    L.sg_init.argtypes = [i32]
    L.sg_get_unique_id.argtypes = [P]
    L.sg_init_rank.argtypes = [i32, i32, P, i32]
    L.sg_shutdown.argtypes = []
    L.sg_last_error.restype = ctypes.c_char_p
    L.sg_topology.argtypes = [P, P, P]
    L.sg_weight_register.argtypes = [P, i32, i64, i64, i32, P]
    L.sg_weight_free.argtypes = [P]
    L.sg_tp_shard.argtypes = [i32, i64, i64, i32, i32, i32, P, P, P, P]
    L.sg_weight_shard.argtypes = [P, i32, P, P, P, P]
    L.sg_linear.argtypes = [P, P, P, i32, i32]
    L.sg_linear_multi.argtypes = [P, i32, P, P, i32]
    L.sg_linear_device.argtypes = [P, P, i64, P, i64, i32, P, i32]
    L.sg_linear_multi_device.argtypes = [P, i32, P, i64, P, P, i32, P, i32]
    L.sg_rmsnorm_linear_multi_device.argtypes = [P, i32, P, i64, P, ctypes.c_float, P, P, i32, P, i32]
    L.sg_silu_mul_linear_device.argtypes = [P, P, i64, P, i64, P, i64, i32, P, i32]
    L.sg_linear_device_noalloc.argtypes = [P, P, i64, P, i64, i32, P, i32]
    L.sg_dequant_f32.argtypes = [P, P, i32]
    L.sg_fused_gemv_q4k.argtypes = [P, P, P, i32, i32]
    L.sg_synchronize.argtypes = []
    L.sg_gguf_open.argtypes = [ctypes.c_char_p, P]
    L.sg_gguf_open_memory.argtypes = [P, ctypes.c_size_t, P]
    L.sg_gguf_close.argtypes = [P]
    L.sg_gguf_header.argtypes = [P, P, P, P, P, P]
    L.sg_gguf_find_tensor.argtypes = [P, ctypes.c_char_p, P]
    L.sg_gguf_tensor_info.argtypes = [P, i64, P, P, P, P, i32, P, P]
    L.sg_gguf_tensor_data.argtypes = [P, i64, P, P]
    L.sg_gguf_find_kv.argtypes = [P, ctypes.c_char_p, P]
    L.sg_gguf_kv_info.argtypes = [P, i64, P, P, P, P]
    L.sg_gguf_kv_int.argtypes = [P, i64, i64, P]
    L.sg_gguf_kv_float.argtypes = [P, i64, i64, P]
    L.sg_gguf_kv_string.argtypes = [P, i64, i64, P, P]
    L.sg_gguf_register.argtypes = [P, i64, i32, P]
    u64, f32 = ctypes.c_uint64, ctypes.c_float
    L.sg_synth_weight.argtypes = [i32, u64, u64, i64, i64, i32, P]
    L.sg_synth_blocks.argtypes = [i32, u64, u64, i64, i64, P, i32]
    L.sg_synth_x.argtypes = [u64, u64, i64, P]
    L.sg_rope_create.argtypes = [i32, i32, P]
    L.sg_rope_free.argtypes = [P]
    L.sg_rope_table.argtypes = [P, P]
    L.sg_kv_cache_create.argtypes = [i32, i32, i32, i32, i32, P]
    L.sg_kv_cache_free.argtypes = [P]
    L.sg_kv_cache_ptr.argtypes = [P, i32, i32, i32, P, P]
    L.sg_rmsnorm_device.argtypes = [P, i64, P, P, i64, i32, i32, f32, P]
    L.sg_rope_kv_device.argtypes = [P, P, i32, P, i64, P, i64, P, i64, P, P, i32, i32, P]
    L.sg_attention_device.argtypes = [P, i32, P, i64, P, i64, P, P, P, i32, i32, P]
    L.sg_rope_attention_device.argtypes = [P, P, i32, P, i64, P, i64, P, i64, P, i64, P, P, i32, i32, P]
    L.sg_attention_prefill_device.argtypes = [P, i32, P, i64, P, i64, i32, i32, i64, i64, i32, P]
    L.sg_silu_mul_device.argtypes = [P, i64, P, i64, i32, i32, P]
    L.sg_add_device.argtypes = [P, i64, P, i64, i32, i32, P]
    L.sg_argmax_device.argtypes = [P, i64, i32, i32, P, P]
    L.sg_embed_device.argtypes = [P, P, i32, P, i64, P]
    L.sg_allreduce_device.argtypes = [P, i64, P]
    L.sg_allreduce_path.argtypes = [P]
    L.sg_host_alloc.argtypes = [ctypes.c_size_t, P]
    L.sg_host_free.argtypes = [P]
    for name in EXPORTS:
        getattr(L, name).restype = ctypes.c_char_p if name == "sg_last_error" else ctypes.c_int
    return L


def row_bytes(dtype: int, n_cols: int) -> int:
    return n_cols // BLOCK[dtype] * BLOCK_BYTES[dtype]


@dataclass
class TensorInfo:
    """swamp-gguf TensorInfo (tensor_info.rs:10-16): shape[0] = n_cols (K),
    shape[1] = n_rows (N)."""
    name: str
    shape: tuple
    dtype: int

    @property
    def n_cols(self) -> int:
        return int(self.shape[0])

    @property
    def n_rows(self) -> int:
        return int(self.shape[1])


class Weight:
    """A GGUF tensor resident on the GPU(s) (sg_weight_t)."""

    def __init__(self, lib: "SwampGpu", handle: int, dtype: int, n_rows: int, n_cols: int, tp_mode: int):
        self.lib, self.handle = lib, handle
        self.dtype, self.n_rows, self.n_cols, self.tp_mode = dtype, n_rows, n_cols, tp_mode

    def shard(self, local_device: int = 0):
        v = [ctypes.c_int64() for _ in range(4)]
        self.lib._check(self.lib.L.sg_weight_shard(self.handle, local_device, *[ctypes.byref(a) for a in v]))
        return tuple(int(a.value) for a in v)  # n_rows, n_cols, row0, col0

    def free(self):
        if self.handle:
            self.lib._check(self.lib.L.sg_weight_free(self.handle))
            self.handle = None


class SwampGpu:
    """One loaded libswamp_gpu.so with its init state."""

    def __init__(self, path: str = LIB_PATH):
        self.L = load_library(path)

    def _check(self, rc: int):
        if rc != SG_OK:
            raise SwampGpuError(rc, self.L.sg_last_error().decode(errors="replace"))

    def tp_shard(self, dtype: int, n_rows: int, n_cols: int, tp_mode: int, world: int, rank: int):
        """(row0, rows, col0, cols) of rank's slice; host-only, needs no GPU."""
        v = [ctypes.c_int64() for _ in range(4)]
        self._check(self.L.sg_tp_shard(dtype, n_rows, n_cols, tp_mode, world, rank, *[ctypes.byref(a) for a in v]))
        return tuple(a.value for a in v)

    # ---------------------------------------------------------- setup
    def init(self, n_gpus: int = 1):
        self._check(self.L.sg_init(n_gpus))
        return self

    def get_unique_id(self) -> bytes:
        buf = ctypes.create_string_buffer(128)
        self._check(self.L.sg_get_unique_id(buf))
        return buf.raw

    def init_rank(self, rank: int, world: int, uid: bytes | None, device: int):
        buf = ctypes.create_string_buffer(uid, 128) if uid is not None else None
        self._check(self.L.sg_init_rank(rank, world, buf, device))
        return self

    def shutdown(self):
        self._check(self.L.sg_shutdown())

    def topology(self):
        r, w, n = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
        self._check(self.L.sg_topology(ctypes.byref(r), ctypes.byref(w), ctypes.byref(n)))
        return r.value, w.value, n.value

    def synchronize(self):
        self._check(self.L.sg_synchronize())

    # --------------------------------------------------------- weights
    def register(self, blocks: np.ndarray, dtype: int, n_rows: int, n_cols: int,
                 tp_mode: int = SG_TP_REPLICATE) -> Weight:
        blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
        if dtype in BLOCK and blocks.size < n_rows * row_bytes(dtype, n_cols):
            raise SwampGpuError(-1, f"blocks hold {blocks.size} bytes, tensor needs {n_rows * row_bytes(dtype, n_cols)}")
        h = ctypes.c_void_p()
        self._check(self.L.sg_weight_register(blocks.ctypes.data, dtype, n_rows, n_cols, tp_mode, ctypes.byref(h)))
        return Weight(self, h.value, dtype, n_rows, n_cols, tp_mode)

    # --------------------------------------------------------- compute
    def host_array(self, shape, dtype=np.float32) -> np.ndarray:
        """A numpy array in page-locked host memory (sg_host_alloc), freed with
        its last view. xs and outs of linear / linear_multi held in such arrays
        are copied by DMA without the library's staging copy."""
        dt = np.dtype(dtype)
        n = int(np.prod(shape)) * dt.itemsize
        p = ctypes.c_void_p()
        self._check(self.L.sg_host_alloc(max(n, 1), ctypes.byref(p)))
        buf = (ctypes.c_ubyte * max(n, 1)).from_address(p.value)
        weakref.finalize(buf, self.L.sg_host_free, p.value)
        return np.frombuffer(buf, dtype=np.uint8, count=n).view(dt).reshape(shape)

    @staticmethod
    def _rows(a: np.ndarray, n: int):
        """Row pointers of a 2D float32 array whose rows are contiguous."""
        base, step = a.ctypes.data, a.strides[0]
        return (ctypes.c_void_p * n)(*[base + b * step for b in range(n)])

    @staticmethod
    def _out_rows(out: np.ndarray, shape) -> np.ndarray:
        if out.dtype != np.float32 or out.shape != shape or (out.ndim and out.strides[-1] != 4):
            raise SwampGpuError(-1, f"out must be float32 {shape} with contiguous rows")
        return out

    def linear(self, w: Weight, xs: np.ndarray, accumulate_into: np.ndarray | None = None,
               out: np.ndarray | None = None) -> np.ndarray:
        """outs[b] = W xs[b] (host arrays); xs is (K,) or (B, K), its rows may be
        strided (a column slice of a wider array). The result goes to `out`
        when given (float32, the shape of the result, contiguous rows; a
        column-split rank writes only its rows of it), else to a new array."""
        xs = np.asarray(xs, dtype=np.float32)
        single = xs.ndim == 1
        if single:
            xs = xs[None]
        if xs.ndim != 2 or xs.strides[1] != 4:
            xs = np.ascontiguousarray(xs)
        B = xs.shape[0]
        if xs.shape[1] < w.n_cols:
            raise SwampGpuError(-1, "forward_linear shape mismatch")  # linear.rs:23
        if accumulate_into is not None:
            outs = np.ascontiguousarray(accumulate_into, dtype=np.float32).reshape(B, w.n_rows)
            flags = SG_FLAG_ACCUMULATE
        elif out is not None:
            outs = self._out_rows(out, (w.n_rows,) if single else (B, w.n_rows))
            if single:
                outs = outs[None]
            flags = 0
        else:
            outs = np.zeros((B, w.n_rows), np.float32)
            flags = 0
        self._check(self.L.sg_linear(w.handle, self._rows(xs, B), self._rows(outs, B), B, flags))
        return outs[0] if single else outs

    def linear_multi(self, ws: Sequence[Weight], x: np.ndarray, outs: Sequence[np.ndarray] | None = None) -> list:
        """outs[i] = W_i x for one vector x; `outs` (float32 (n_rows_i,)
        arrays) receive the results when given."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if outs is None:
            outs = [np.zeros(w.n_rows, np.float32) for w in ws]
        else:
            if len(outs) != len(ws):
                raise SwampGpuError(-1, "one output per tensor")
            outs = [self._out_rows(o, (w.n_rows,)) for o, w in zip(outs, ws)]
        hp = (ctypes.c_void_p * len(ws))(*[w.handle for w in ws])
        op = (ctypes.c_void_p * len(ws))(*[o.ctypes.data for o in outs])
        self._check(self.L.sg_linear_multi(hp, len(ws), x.ctypes.data, op, 0))
        return list(outs)

    def linear_device(self, w: Weight, x_ptr: int, ldx: int, y_ptr: int, ldy: int, batch: int,
                      stream: int = 0, flags: int = 0):
        """Stream-ordered device call (pointers are raw device addresses)."""
        self._check(self.L.sg_linear_device(w.handle, x_ptr, ldx, y_ptr, ldy, batch, stream or None, flags))

    def linear_device_noalloc(self, w: Weight, x_ptr: int, ldx: int, y_ptr: int, ldy: int, batch: int,
                              stream: int = 0, flags: int = 0):
        """linear_device without any device allocation (decode batch 1..16)."""
        self._check(self.L.sg_linear_device_noalloc(w.handle, x_ptr, ldx, y_ptr, ldy, batch, stream or None, flags))

    def rmsnorm_linear_multi_device(self, ws: Sequence[Weight], x_ptr: int, ldx: int, norm_ptr: int, eps: float,
                                    y_ptrs: Sequence[int], ldys: Sequence[int], batch: int, stream: int = 0,
                                    flags: int = 0):
        """ys[i] = W_i rmsnorm(x) (RMSNorm fused into the decode GEMV's operand build)."""
        n = len(ws)
        hp = (ctypes.c_void_p * n)(*[w.handle for w in ws])
        yp = (ctypes.c_void_p * n)(*y_ptrs)
        lp = (ctypes.c_int64 * n)(*ldys)
        self._check(self.L.sg_rmsnorm_linear_multi_device(hp, n, x_ptr, ldx, norm_ptr, eps, yp, lp, batch,
                                                          stream or None, flags))

    def silu_mul_linear_device(self, w: Weight, g_ptr: int, ldg: int, u_ptr: int, ldu: int, y_ptr: int, ldy: int,
                               batch: int, stream: int = 0, flags: int = 0):
        """y = W (silu(g) * u) (SiLU-mul fused into the decode GEMV's operand build)."""
        self._check(self.L.sg_silu_mul_linear_device(w.handle, g_ptr, ldg, u_ptr, ldu, y_ptr, ldy, batch,
                                                     stream or None, flags))

    def linear_multi_device(self, ws: Sequence[Weight], x_ptr: int, ldx: int, y_ptrs: Sequence[int],
                            ldys: Sequence[int], batch: int, stream: int = 0, flags: int = 0):
        n = len(ws)
        hp = (ctypes.c_void_p * n)(*[w.handle for w in ws])
        yp = (ctypes.c_void_p * n)(*y_ptrs)
        lp = (ctypes.c_int64 * n)(*ldys)
        self._check(self.L.sg_linear_multi_device(hp, n, x_ptr, ldx, yp, lp, batch, stream or None, flags))

    def dequant(self, w: Weight) -> np.ndarray:
        out = np.empty((w.n_rows, w.n_cols), np.float32)
        self._check(self.L.sg_dequant_f32(w.handle, out.ctypes.data, 0))
        return out

    def dequant_device(self, w: Weight, dst_ptr: int):
        self._check(self.L.sg_dequant_f32(w.handle, dst_ptr, SG_FLAG_DEVICE_PTRS))

    def fused_gemv_q4k(self, w_raw: np.ndarray, x: np.ndarray, n_rows: int, n_cols: int) -> np.ndarray:
        """swamp_fused_gemv_q4k (fused_gemv_q4k.rs:799-823)."""
        w_raw = np.ascontiguousarray(w_raw, dtype=np.uint8)
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(n_rows, np.float32)
        self._check(self.L.sg_fused_gemv_q4k(w_raw.ctypes.data, x.ctypes.data, out.ctypes.data, n_rows, n_cols))
        return out


    def allreduce_device(self, buf_ptr: int, count: int, stream: int = 0):
        """In-place sum across the job's ranks (stream-ordered)."""
        self._check(self.L.sg_allreduce_device(buf_ptr, count, stream or None))

    def allreduce_path(self) -> str:
        v = ctypes.c_int()
        self._check(self.L.sg_allreduce_path(ctypes.byref(v)))
        return "peer" if v.value else "nccl"

    # ------------------------------------------------------- synthetic inputs
    def synth_weight(self, dtype: int, seed: int, tensor_id: int, n_rows: int, n_cols: int,
                     tp_mode: int = SG_TP_REPLICATE) -> Weight:
        """A seeded random-init tensor generated and registered on the device."""
        h = ctypes.c_void_p()
        self._check(self.L.sg_synth_weight(dtype, seed, tensor_id, n_rows, n_cols, tp_mode, ctypes.byref(h)))
        return Weight(self, h.value, dtype, n_rows, n_cols, tp_mode)

    def synth_blocks(self, dtype: int, seed: int, tensor_id: int, n_rows: int, n_cols: int) -> np.ndarray:
        """The GGUF bytes of that tensor (row-major), copied to the host."""
        out = np.empty(n_rows * row_bytes(dtype, n_cols), np.uint8)
        self._check(self.L.sg_synth_blocks(dtype, seed, tensor_id, n_rows, n_cols, out.ctypes.data, 0))
        return out

    def synth_x(self, seed: int, tensor_id: int, shape) -> np.ndarray:
        n = int(np.prod(shape))
        out = np.empty(n, np.float32)
        self._check(self.L.sg_synth_x(seed, tensor_id, n, out.ctypes.data))
        return out.reshape(shape)


class Rope:
    """init_rope_lut (swamp-engine/src/ops.rs:20-38), kept on the device."""

    def __init__(self, lib: SwampGpu, head_dim: int, max_context: int):
        self.lib, self.head_dim, self.max_context = lib, head_dim, max_context
        h = ctypes.c_void_p()
        lib._check(lib.L.sg_rope_create(head_dim, max_context, ctypes.byref(h)))
        self.handle = h.value

    def table(self) -> np.ndarray:
        out = np.empty((self.max_context, self.head_dim // 2, 2), np.float32)
        self.lib._check(self.lib.L.sg_rope_table(self.handle, out.ctypes.data))
        return out

    def free(self):
        if self.handle:
            self.lib._check(self.lib.L.sg_rope_free(self.handle))
            self.handle = None


class KvCache:
    """PagedKVCache (swamp-engine/src/cache.rs) of n_seqs sequences resident
    on the device: [seq][layer][kv_head][max_seq][head_dim] f32."""

    def __init__(self, lib: SwampGpu, n_layers: int, n_kv_heads: int, head_dim: int, max_seq: int, n_seqs: int = 1):
        self.lib = lib
        self.n_layers, self.n_kv_heads, self.head_dim, self.max_seq, self.n_seqs = (
            n_layers, n_kv_heads, head_dim, max_seq, n_seqs)
        h = ctypes.c_void_p()
        lib._check(lib.L.sg_kv_cache_create(n_layers, n_kv_heads, head_dim, max_seq, n_seqs, ctypes.byref(h)))
        self.handle = h.value

    def ptrs(self, seq: int, layer: int, kv_head: int):
        """Device addresses of position 0 of (seq, layer, kv_head) in K and V."""
        k, v = ctypes.c_void_p(), ctypes.c_void_p()
        self.lib._check(self.lib.L.sg_kv_cache_ptr(self.handle, seq, layer, kv_head, ctypes.byref(k), ctypes.byref(v)))
        return k.value, v.value

    def free(self):
        if self.handle:
            self.lib._check(self.lib.L.sg_kv_cache_free(self.handle))
            self.handle = None


class LayerOps:
    """The decoder layer's non-matmul operations (ops.rs, sampler.rs) on
    device pointers (ints: data_ptr() of CUDA tensors), stream-ordered;
    stream is a cudaStream_t as an int, 0/None for the default stream."""

    def __init__(self, lib: SwampGpu):
        self.lib, self.L = lib, lib.L

    def rmsnorm(self, x: int, ldx: int, weight: int, out: int, ldo: int, n: int, rows: int, eps: float,
                stream: int | None = None):
        self.lib._check(self.L.sg_rmsnorm_device(x, ldx, weight, out, ldo, n, rows, eps, stream or None))

    def rope_kv(self, rope: Rope | None, cache: KvCache, layer: int, q: int, ldq: int, k: int, ldk: int, v: int,
                ldv: int, pos: int, seq: int | None, rows: int, n_q_heads: int, stream: int | None = None):
        self.lib._check(self.L.sg_rope_kv_device(rope.handle if rope else None, cache.handle, layer, q or None, ldq,
                                                 k, ldk, v, ldv, pos, seq or None, rows, n_q_heads, stream or None))

    def attention(self, cache: KvCache, layer: int, q: int, ldq: int, out: int, ldo: int, pos: int,
                  seq_len: int | None, seq: int | None, rows: int, n_heads: int, stream: int | None = None):
        self.lib._check(self.L.sg_attention_device(cache.handle, layer, q, ldq, out, ldo, pos, seq_len or None,
                                                   seq or None, rows, n_heads, stream or None))

    def rope_attention(self, rope: Rope, cache: KvCache, layer: int, q: int, ldq: int, k: int, ldk: int, v: int,
                       ldv: int, out: int, ldo: int, pos: int, seq: int | None, rows: int, n_heads: int,
                       stream: int | None = None):
        """Decode form: RoPE, cache store and attention of one row per sequence."""
        self.lib._check(self.L.sg_rope_attention_device(rope.handle, cache.handle, layer, q, ldq, k, ldk, v, ldv, out,
                                                        ldo, pos, seq or None, rows, n_heads, stream or None))

    def attention_prefill(self, cache: KvCache, layer: int, q: int, ldq: int, out: int, ldo: int, n_seqs: int,
                          n_tokens: int, row_stride_seq: int, row_stride_pos: int, n_heads: int,
                          stream: int | None = None):
        """Causal attention of every prompt position of n_seqs sequences."""
        self.lib._check(self.L.sg_attention_prefill_device(cache.handle, layer, q, ldq, out, ldo, n_seqs, n_tokens,
                                                           row_stride_seq, row_stride_pos, n_heads, stream or None))

    def silu_mul(self, g: int, ldg: int, u: int, ldu: int, n: int, rows: int, stream: int | None = None):
        self.lib._check(self.L.sg_silu_mul_device(g, ldg, u, ldu, n, rows, stream or None))

    def add(self, x: int, ldx: int, y: int, ldy: int, n: int, rows: int, stream: int | None = None):
        self.lib._check(self.L.sg_add_device(x, ldx, y, ldy, n, rows, stream or None))

    def argmax(self, logits: int, ld: int, n: int, rows: int, out: int, stream: int | None = None):
        self.lib._check(self.L.sg_argmax_device(logits, ld, n, rows, out, stream or None))

    def embed(self, table: Weight, tokens: int, rows: int, out: int, ldo: int, stream: int | None = None):
        self.lib._check(self.L.sg_embed_device(table.handle, tokens, rows, out, ldo, stream or None))


# ---------------------------------------------------------------------------
# swamp-gguf GgufFile (mmap.rs:26-120) over sg_gguf_*
# ---------------------------------------------------------------------------

@dataclass
class GgufTensor:
    """swamp-gguf TensorInfo (tensor_info.rs:10-16) with its index in the
    file; offset is absolute in the file (mmap.rs:86-89)."""
    index: int
    name: str
    shape: tuple
    dtype: int
    offset: int
    nbytes: int


class GgufFile:
    """A GGUF file parsed by the library (host-only: no GPU or init needed,
    except for ``register``). Errors raise SwampGpuError (SG_ERR_FORMAT for a
    malformed file, SG_ERR_NOT_FOUND for a missing name or key)."""

    def __init__(self, gpu: "SwampGpu | ctypes.CDLL", path: str | None = None, data: bytes | None = None):
        self.L = gpu.L if isinstance(gpu, SwampGpu) else gpu
        self._gpu = gpu if isinstance(gpu, SwampGpu) else None
        self._data = data  # kept alive while the handle exists
        h = ctypes.c_void_p()
        if path is not None:
            rc = self.L.sg_gguf_open(os.fsencode(path), ctypes.byref(h))
        else:
            self._buf = ctypes.create_string_buffer(bytes(data), len(data)) if data else None
            rc = self.L.sg_gguf_open_memory(self._buf, len(data) if data else 0, ctypes.byref(h))
        self._check(rc)
        self.handle = h.value
        v, nt, nk, do, fs = (ctypes.c_uint32(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64())
        self._check(self.L.sg_gguf_header(self.handle, *[ctypes.byref(a) for a in (v, nt, nk, do, fs)]))
        self.version, self.data_offset, self.file_size = v.value, do.value, fs.value
        self.tensors = [self._tensor(i) for i in range(nt.value)]
        self.n_kv = nk.value

    def _check(self, rc: int):
        if rc != SG_OK:
            raise SwampGpuError(rc, self.L.sg_last_error().decode(errors="replace"))

    def _tensor(self, i: int) -> GgufTensor:
        name, dt, nd, off, nb = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int64(), ctypes.c_int64()
        dims = (ctypes.c_int64 * 64)()
        self._check(self.L.sg_gguf_tensor_info(self.handle, i, ctypes.byref(name), ctypes.byref(dt), ctypes.byref(nd),
                                               dims, 64, ctypes.byref(off), ctypes.byref(nb)))
        shape = tuple(int(dims[d]) & 0xFFFFFFFFFFFFFFFF for d in range(min(nd.value, 64)))
        return GgufTensor(i, name.value.decode(), shape, dt.value, off.value & 0xFFFFFFFFFFFFFFFF,
                          nb.value & 0xFFFFFFFFFFFFFFFF)

    def close(self):
        if self.handle:
            self._check(self.L.sg_gguf_close(self.handle))
            self.handle = None

    def tensor(self, name: str) -> GgufTensor:
        """GgufFile::tensor_or_err (mmap.rs:100-104)."""
        i = ctypes.c_int64()
        self._check(self.L.sg_gguf_find_tensor(self.handle, name.encode(), ctypes.byref(i)))
        return self.tensors[i.value]

    def tensor_raw_bytes(self, t: GgufTensor) -> bytes:
        """GgufFile::tensor_raw_bytes (mmap.rs:111-118)."""
        p, n = ctypes.c_void_p(), ctypes.c_int64()
        self._check(self.L.sg_gguf_tensor_data(self.handle, t.index, ctypes.byref(p), ctypes.byref(n)))
        return ctypes.string_at(p.value, n.value) if n.value else b""

    def kv(self, key: str):
        """Metadata value of key (the last occurrence): int, float, str, bool
        or a list of them for an array."""
        i = ctypes.c_int64()
        self._check(self.L.sg_gguf_find_kv(self.handle, key.encode(), ctypes.byref(i)))
        return self.kv_at(i.value)[1]

    def kv_at(self, index: int):
        key, t, et, cnt = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int(), ctypes.c_int64()
        self._check(self.L.sg_gguf_kv_info(self.handle, index, ctypes.byref(key), ctypes.byref(t), ctypes.byref(et),
                                           ctypes.byref(cnt)))
        et_ = et.value if t.value == 9 else t.value
        vals = [self._elem(index, e, et_) for e in range(cnt.value)]
        return key.value.decode(), (vals if t.value == 9 else vals[0]), t.value, et.value

    def _elem(self, index: int, e: int, t: int):
        if t in (6, 12):
            v = ctypes.c_double()
            self._check(self.L.sg_gguf_kv_float(self.handle, index, e, ctypes.byref(v)))
            return v.value
        if t == 8:
            p, n = ctypes.c_char_p(), ctypes.c_int64()
            self._check(self.L.sg_gguf_kv_string(self.handle, index, e, ctypes.byref(p), ctypes.byref(n)))
            return ctypes.string_at(p, n.value).decode()
        v = ctypes.c_int64()
        self._check(self.L.sg_gguf_kv_int(self.handle, index, e, ctypes.byref(v)))
        if t == 7:
            return bool(v.value)
        return v.value & 0xFFFFFFFFFFFFFFFF if t == 10 else v.value

    def register(self, t: GgufTensor, tp_mode: int = SG_TP_REPLICATE) -> Weight:
        """Upload a Q4_0/Q4_K matrix straight from the mapped file."""
        if self._gpu is None:
            raise SwampGpuError(-6, "register needs an initialised SwampGpu")
        h = ctypes.c_void_p()
        self._check(self.L.sg_gguf_register(self.handle, t.index, tp_mode, ctypes.byref(h)))
        return Weight(self._gpu, h.value, t.dtype, t.shape[1], t.shape[0], tp_mode)


# ---------------------------------------------------------------------------
# swamp-engine/src/linear.rs call shapes
# ---------------------------------------------------------------------------

def forward_linear(gpu: SwampGpu, tensor: Weight, x: np.ndarray, out: np.ndarray) -> None:
    """linear.rs:14-90: out[..n_rows] = W x (x has >= n_cols entries)."""
    if x.shape[0] < tensor.n_cols or out.shape[0] < tensor.n_rows:
        raise SwampGpuError(-1, "forward_linear shape mismatch")
    out[: tensor.n_rows] = gpu.linear(tensor, x[: tensor.n_cols])


def forward_linear_multi(gpu: SwampGpu, tensors: Sequence[Weight], x: np.ndarray, outputs: Sequence[np.ndarray]) -> None:
    """linear.rs:96-170: several tensors over one x; outputs overwritten."""
    res = gpu.linear_multi(tensors, x)
    for o, r in zip(outputs, res):
        o[: r.shape[0]] = r


def forward_linear_batch(gpu: SwampGpu, tensor: Weight, xs: Sequence[np.ndarray], outputs: Sequence[np.ndarray]) -> None:
    """linear.rs:176-239: batch of inputs; bs != outputs.len() is an error (:185-187)."""
    if len(xs) != len(outputs):
        raise SwampGpuError(-1, f"forward_linear_batch: {len(xs)} inputs != {len(outputs)} outputs")
    if len(xs) == 0:
        return
    res = gpu.linear(tensor, np.stack([np.asarray(x[: tensor.n_cols], np.float32) for x in xs]))
    for o, r in zip(outputs, res):
        o[: tensor.n_rows] = r


def forward_gemvs(gpu: SwampGpu, specs: Sequence[tuple]) -> None:
    """linear.rs:278-333: list of (tensor, x, out); outputs zero-filled then written."""
    for tensor, x, out in specs:
        forward_linear(gpu, tensor, x, out)
