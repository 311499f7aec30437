//! swamp-gpu: thin FFI to libswamp_gpu.so, the B200 (sm_100a) Q4_0 / Q4_K
//! quantized-linear path (declared in include/swamp_gpu.h).
//!
//! Replaces the reference crate's src/lib.rs (swamp-gpu/src/lib.rs:32-56 is
//! its loader): the library is opened once with libloading behind a
//! `OnceLock`, every entry returns an `int` status that becomes
//! `GpuError::Status` with the library's message, and there is no CPU
//! fallback (a missing library or GPU is an error, never a silent CPU path).
//!
//! swamp-engine routes its linears here under its `gpu` feature: see
//! `WeightCache` and `forward_linear*` below (the engine keys the cache on
//! `TensorInfo.offset`, as it re-reads the mmap on every call today,
//! swamp-engine/src/linear.rs:24).
#![allow(clippy::too_many_arguments)]

use libloading::{Library, Symbol};
use std::collections::HashMap;
use std::ffi::{c_void, CStr, CString};
use std::os::raw::{c_char, c_int};
use std::sync::{Mutex, OnceLock};
use thiserror::Error;
use tracing::info;

#[derive(Error, Debug, Clone)]
pub enum GpuError {
    #[error("CUDA/GPU not available: {0}")]
    NotAvailable(String),
    #[error("Library load failed: {0}")]
    LibLoad(String),
    #[error("Symbol lookup failed: {0}")]
    Symbol(String),
    #[error("swamp_gpu status {code}: {message}")]
    Status { code: i32, message: String },
}

impl From<libloading::Error> for GpuError {
    fn from(e: libloading::Error) -> Self {
        GpuError::Symbol(format!("{e:?}"))
    }
}

pub type Result<T> = std::result::Result<T, GpuError>;

// status codes and constants (include/swamp_gpu.h)
pub const SG_OK: c_int = 0;
pub const SG_ERR_DEVICE_FAULT: c_int = -7;
pub const SG_DTYPE_Q4_0: c_int = 2;
pub const SG_DTYPE_Q4_K: c_int = 12;
pub const SG_DTYPE_Q6_K: c_int = 14;
pub const SG_TP_REPLICATE: c_int = 0;
pub const SG_TP_COLUMN: c_int = 1;
pub const SG_TP_ROW: c_int = 2;
pub const SG_FLAG_DEVICE_PTRS: c_int = 0x1;
pub const SG_FLAG_ACCUMULATE: c_int = 0x2;

/// Opaque handles of the C ABI.
pub type SgWeight = *mut c_void;
pub type SgGguf = *mut c_void;
pub type SgRope = *mut c_void;
pub type SgKvCache = *mut c_void;
/// A `cudaStream_t` (null: CUDA's default stream).
pub type Stream = *mut c_void;

static GPU_LIB: OnceLock<Result<Library>> = OnceLock::new();

/// The library: $SWAMP_GPU_LIB at run time, else the one build.rs compiled
/// (feature `build-cuda`), else libswamp_gpu.so on the loader's path.
fn try_lib() -> Result<&'static Library> {
    let r = GPU_LIB.get_or_init(|| {
        let mut paths: Vec<String> = Vec::new();
        if let Ok(p) = std::env::var("SWAMP_GPU_LIB") {
            paths.push(p);
        }
        if let Some(p) = option_env!("SWAMP_GPU_LIB") {
            paths.push(p.to_string());
        }
        paths.push("libswamp_gpu.so".to_string());
        paths.push("./swamp-gpu/libswamp_gpu.so".to_string());
        for path in &paths {
            if let Ok(lib) = unsafe { Library::new(path) } {
                info!("libswamp_gpu loaded from {path}");
                return Ok(lib);
            }
        }
        Err(GpuError::LibLoad(format!("libswamp_gpu.so not found (tried {paths:?})")))
    });
    match r {
        Ok(lib) => Ok(lib),
        Err(e) => Err(e.clone()),
    }
}

macro_rules! sym {
    ($lib:expr, $name:literal, $ty:ty) => {{
        let s: Symbol<$ty> = unsafe { $lib.get(concat!($name, "\0").as_bytes())? };
        s
    }};
}

fn last_error(lib: &Library) -> String {
    match unsafe { lib.get::<unsafe extern "C" fn() -> *const c_char>(b"sg_last_error\0") } {
        Ok(f) => {
            let p = unsafe { f() };
            if p.is_null() {
                String::new()
            } else {
                unsafe { CStr::from_ptr(p) }.to_string_lossy().into_owned()
            }
        }
        Err(e) => format!("{e:?}"),
    }
}

fn check(lib: &Library, rc: c_int) -> Result<()> {
    if rc == SG_OK {
        return Ok(());
    }
    let message = last_error(lib);
    tracing::error!("swamp_gpu: {message}");
    Err(GpuError::Status { code: rc, message })
}

/// The library loads (a GPU is only touched by `init`).
pub fn gpu_available() -> bool {
    try_lib().is_ok()
}

// ------------------------------------------------------------------ setup

/// Single process, devices 0..n_gpus-1 (NCCL communicator over them for n > 1).
pub fn init(n_gpus: usize) -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_init", unsafe extern "C" fn(c_int) -> c_int);
    check(lib, unsafe { f(n_gpus as c_int) })
}

/// One process per GPU: rank 0 makes the id, the caller ships it to the others.
pub fn get_unique_id() -> Result<[u8; 128]> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_get_unique_id", unsafe extern "C" fn(*mut c_void) -> c_int);
    let mut id = [0u8; 128];
    check(lib, unsafe { f(id.as_mut_ptr() as *mut c_void) })?;
    Ok(id)
}

pub fn init_rank(rank: usize, world: usize, id: &[u8; 128], device: usize) -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_init_rank", unsafe extern "C" fn(c_int, c_int, *const c_void, c_int) -> c_int);
    check(lib, unsafe { f(rank as c_int, world as c_int, id.as_ptr() as *const c_void, device as c_int) })
}

pub fn shutdown() -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_shutdown", unsafe extern "C" fn() -> c_int);
    check(lib, unsafe { f() })
}

/// (rank, world, local devices)
pub fn topology() -> Result<(usize, usize, usize)> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_topology", unsafe extern "C" fn(*mut c_int, *mut c_int, *mut c_int) -> c_int);
    let (mut r, mut w, mut n) = (0, 0, 0);
    check(lib, unsafe { f(&mut r, &mut w, &mut n) })?;
    Ok((r as usize, w as usize, n as usize))
}

/// Wait for this process's devices; a kernel's bounded wait that gave up
/// comes back as `Status { code: SG_ERR_DEVICE_FAULT, .. }`.
pub fn synchronize() -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_synchronize", unsafe extern "C" fn() -> c_int);
    check(lib, unsafe { f() })
}

// ---------------------------------------------------------------- weights

/// Upload one GGUF tensor (its raw block bytes, row-major) and repack it on
/// the device; `tp` splits it across the job's ranks.
pub fn weight_register(raw: &[u8], dtype: c_int, n_rows: usize, n_cols: usize, tp: c_int) -> Result<SgWeight> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_weight_register",
                 unsafe extern "C" fn(*const c_void, c_int, i64, i64, c_int, *mut SgWeight) -> c_int);
    let mut w: SgWeight = std::ptr::null_mut();
    check(lib, unsafe { f(raw.as_ptr() as *const c_void, dtype, n_rows as i64, n_cols as i64, tp, &mut w) })?;
    Ok(w)
}

pub fn weight_free(w: SgWeight) -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_weight_free", unsafe extern "C" fn(SgWeight) -> c_int);
    check(lib, unsafe { f(w) })
}

/// (row0, rows, col0, cols) of rank's slice; host-only.
pub fn tp_shard(dtype: c_int, n_rows: usize, n_cols: usize, tp: c_int, world: usize, rank: usize)
                -> Result<(i64, i64, i64, i64)> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_tp_shard",
                 unsafe extern "C" fn(c_int, i64, i64, c_int, c_int, c_int, *mut i64, *mut i64, *mut i64, *mut i64)
                     -> c_int);
    let (mut r0, mut r, mut c0, mut c) = (0i64, 0i64, 0i64, 0i64);
    check(lib, unsafe {
        f(dtype, n_rows as i64, n_cols as i64, tp, world as c_int, rank as c_int, &mut r0, &mut r, &mut c0, &mut c)
    })?;
    Ok((r0, r, c0, c))
}

/// f32 host memory from sg_host_alloc (page-locked): `linear` / `linear_multi`
/// copy rows held here by DMA without the library's staging copy.
pub struct PinnedBuf {
    ptr: *mut f32,
    len: usize,
}

impl PinnedBuf {
    pub fn new(len: usize) -> Result<Self> {
        let lib = try_lib()?;
        let f = sym!(lib, "sg_host_alloc", unsafe extern "C" fn(usize, *mut *mut c_void) -> c_int);
        let mut p: *mut c_void = std::ptr::null_mut();
        check(lib, unsafe { f(len.max(1) * std::mem::size_of::<f32>(), &mut p) })?;
        unsafe { std::ptr::write_bytes(p as *mut f32, 0, len) };
        Ok(PinnedBuf { ptr: p as *mut f32, len })
    }
    pub fn as_slice(&self) -> &[f32] {
        unsafe { std::slice::from_raw_parts(self.ptr, self.len) }
    }
    pub fn as_mut_slice(&mut self) -> &mut [f32] {
        unsafe { std::slice::from_raw_parts_mut(self.ptr, self.len) }
    }
}

impl Drop for PinnedBuf {
    fn drop(&mut self) {
        if let Ok(lib) = try_lib() {
            if let Ok(f) = unsafe { lib.get::<unsafe extern "C" fn(*mut c_void) -> c_int>(b"sg_host_free\0") } {
                unsafe { f(self.ptr as *mut c_void) };
            }
        }
    }
}

// ---------------------------------------------------------------- compute

/// forward_linear / forward_linear_batch on host buffers: outs[b] = W xs[b]
/// (overwrite; SG_FLAG_ACCUMULATE adds).
pub fn linear(w: SgWeight, xs: &[&[f32]], outs: &mut [&mut [f32]], flags: c_int) -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_linear",
                 unsafe extern "C" fn(SgWeight, *const *const f32, *const *mut f32, c_int, c_int) -> c_int);
    if xs.len() != outs.len() {
        return Err(GpuError::Status { code: -1, message: "xs and outs differ in length".into() });
    }
    let xp: Vec<*const f32> = xs.iter().map(|x| x.as_ptr()).collect();
    let op: Vec<*mut f32> = outs.iter_mut().map(|o| o.as_mut_ptr()).collect();
    check(lib, unsafe { f(w, xp.as_ptr(), op.as_ptr(), xs.len() as c_int, flags) })
}

/// forward_linear_multi: several tensors sharing x (at most 4 per call).
pub fn linear_multi(ws: &[SgWeight], x: &[f32], outs: &mut [&mut [f32]], flags: c_int) -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_linear_multi",
                 unsafe extern "C" fn(*const SgWeight, c_int, *const f32, *const *mut f32, c_int) -> c_int);
    let op: Vec<*mut f32> = outs.iter_mut().map(|o| o.as_mut_ptr()).collect();
    check(lib, unsafe { f(ws.as_ptr(), ws.len() as c_int, x.as_ptr(), op.as_ptr(), flags) })
}

/// Device pointers, stream-ordered: x [batch][ldx], y [batch][ldy].
pub fn linear_device(w: SgWeight, x: *const f32, ldx: i64, y: *mut f32, ldy: i64, batch: usize, stream: Stream,
                     flags: c_int) -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_linear_device",
                 unsafe extern "C" fn(SgWeight, *const f32, i64, *mut f32, i64, c_int, Stream, c_int) -> c_int);
    check(lib, unsafe { f(w, x, ldx, y, ldy, batch as c_int, stream, flags) })
}

pub fn linear_multi_device(ws: &[SgWeight], x: *const f32, ldx: i64, ys: &[*mut f32], ldys: &[i64], batch: usize,
                           stream: Stream, flags: c_int) -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_linear_multi_device",
                 unsafe extern "C" fn(*const SgWeight, c_int, *const f32, i64, *const *mut f32, *const i64, c_int,
                                      Stream, c_int) -> c_int);
    check(lib, unsafe { f(ws.as_ptr(), ws.len() as c_int, x, ldx, ys.as_ptr(), ldys.as_ptr(), batch as c_int,
                          stream, flags) })
}

/// `linear_device` for callers that must never trigger a device allocation
/// (decode batch 1..16, within the library's fixed workspace).
pub fn linear_device_noalloc(w: SgWeight, x: *const f32, ldx: i64, y: *mut f32, ldy: i64, batch: usize,
                             stream: Stream, flags: c_int) -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_linear_device_noalloc",
                 unsafe extern "C" fn(SgWeight, *const f32, i64, *mut f32, i64, c_int, Stream, c_int) -> c_int);
    check(lib, unsafe { f(w, x, ldx, y, ldy, batch as c_int, stream, flags) })
}

/// The whole tensor dequantized to f32 [n_rows][n_cols] (bit-exact with swamp-gguf).
pub fn dequant_f32(w: SgWeight, dst: &mut [f32]) -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_dequant_f32", unsafe extern "C" fn(SgWeight, *mut f32, c_int) -> c_int);
    check(lib, unsafe { f(w, dst.as_mut_ptr(), 0) })
}

/// swamp_fused_gemv_q4k's drop-in (raw Q4_K bytes on every call; errors are reported).
pub fn fused_gemv_q4k(w_raw: &[u8], x: &[f32], out: &mut [f32], n_rows: usize, n_cols: usize) -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_fused_gemv_q4k",
                 unsafe extern "C" fn(*const u8, *const f32, *mut f32, c_int, c_int) -> c_int);
    check(lib, unsafe { f(w_raw.as_ptr(), x.as_ptr(), out.as_mut_ptr(), n_rows as c_int, n_cols as c_int) })
}

/// In-place sum across the job's ranks (one process per GPU).
pub fn allreduce_device(buf: *mut f32, count: usize, stream: Stream) -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_allreduce_device", unsafe extern "C" fn(*mut f32, i64, Stream) -> c_int);
    check(lib, unsafe { f(buf, count as i64, stream) })
}

// ------------------------------------------------------------------- GGUF

pub fn gguf_open(path: &std::path::Path) -> Result<SgGguf> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_gguf_open", unsafe extern "C" fn(*const c_char, *mut SgGguf) -> c_int);
    let c = CString::new(path.as_os_str().as_encoded_bytes())
        .map_err(|e| GpuError::Status { code: -1, message: e.to_string() })?;
    let mut g: SgGguf = std::ptr::null_mut();
    check(lib, unsafe { f(c.as_ptr(), &mut g) })?;
    Ok(g)
}

pub fn gguf_close(g: SgGguf) -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_gguf_close", unsafe extern "C" fn(SgGguf) -> c_int);
    check(lib, unsafe { f(g) })
}

/// Register a Q4_0 / Q4_K matrix of the file by tensor name.
pub fn gguf_register_by_name(g: SgGguf, name: &str, tp: c_int) -> Result<SgWeight> {
    let lib = try_lib()?;
    let find = sym!(lib, "sg_gguf_find_tensor", unsafe extern "C" fn(SgGguf, *const c_char, *mut i64) -> c_int);
    let reg = sym!(lib, "sg_gguf_register", unsafe extern "C" fn(SgGguf, i64, c_int, *mut SgWeight) -> c_int);
    let c = CString::new(name).map_err(|e| GpuError::Status { code: -1, message: e.to_string() })?;
    let mut idx: i64 = 0;
    check(lib, unsafe { find(g, c.as_ptr(), &mut idx) })?;
    let mut w: SgWeight = std::ptr::null_mut();
    check(lib, unsafe { reg(g, idx, tp, &mut w) })?;
    Ok(w)
}

// -------------------------------------------------------------- layer ops

pub fn rmsnorm_device(x: *const f32, ldx: i64, weight: *const f32, out: *mut f32, ldo: i64, n: usize, rows: usize,
                      eps: f32, stream: Stream) -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_rmsnorm_device",
                 unsafe extern "C" fn(*const f32, i64, *const f32, *mut f32, i64, c_int, c_int, f32, Stream) -> c_int);
    check(lib, unsafe { f(x, ldx, weight, out, ldo, n as c_int, rows as c_int, eps, stream) })
}

pub fn silu_mul_device(g: *mut f32, ldg: i64, u: *const f32, ldu: i64, n: usize, rows: usize, stream: Stream)
                       -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_silu_mul_device",
                 unsafe extern "C" fn(*mut f32, i64, *const f32, i64, c_int, c_int, Stream) -> c_int);
    check(lib, unsafe { f(g, ldg, u, ldu, n as c_int, rows as c_int, stream) })
}

/// `rmsnorm_device` then `linear_multi_device` on its rows as one call: at
/// decode batch the norm runs inside the GEMV's activation prep (the rows are
/// never written), bit-identical to the two calls.
pub fn rmsnorm_linear_multi_device(ws: &[SgWeight], x: *const f32, ldx: i64, norm_weight: *const f32, eps: f32,
                                   ys: &[*mut f32], ldys: &[i64], batch: usize, stream: Stream, flags: c_int)
                                   -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_rmsnorm_linear_multi_device",
                 unsafe extern "C" fn(*const SgWeight, c_int, *const f32, i64, *const f32, f32, *const *mut f32,
                                      *const i64, c_int, Stream, c_int) -> c_int);
    check(lib, unsafe { f(ws.as_ptr(), ws.len() as c_int, x, ldx, norm_weight, eps, ys.as_ptr(), ldys.as_ptr(),
                          batch as c_int, stream, flags) })
}

/// `silu_mul_device` then `linear_device` on its rows as one call (g and u
/// are not modified).
pub fn silu_mul_linear_device(w: SgWeight, g: *const f32, ldg: i64, u: *const f32, ldu: i64, y: *mut f32, ldy: i64,
                              batch: usize, stream: Stream, flags: c_int) -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_silu_mul_linear_device",
                 unsafe extern "C" fn(SgWeight, *const f32, i64, *const f32, i64, *mut f32, i64, c_int, Stream,
                                      c_int) -> c_int);
    check(lib, unsafe { f(w, g, ldg, u, ldu, y, ldy, batch as c_int, stream, flags) })
}

pub fn argmax_device(logits: *const f32, ld: i64, n: usize, rows: usize, out: *mut i32, stream: Stream)
                     -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_argmax_device",
                 unsafe extern "C" fn(*const f32, i64, c_int, c_int, *mut i32, Stream) -> c_int);
    check(lib, unsafe { f(logits, ld, n as c_int, rows as c_int, out, stream) })
}

pub fn rope_create(head_dim: usize, max_context: usize) -> Result<SgRope> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_rope_create", unsafe extern "C" fn(c_int, c_int, *mut SgRope) -> c_int);
    let mut r: SgRope = std::ptr::null_mut();
    check(lib, unsafe { f(head_dim as c_int, max_context as c_int, &mut r) })?;
    Ok(r)
}

pub fn kv_cache_create(n_layers: usize, n_kv_heads: usize, head_dim: usize, max_seq: usize, n_seqs: usize)
                       -> Result<SgKvCache> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_kv_cache_create",
                 unsafe extern "C" fn(c_int, c_int, c_int, c_int, c_int, *mut SgKvCache) -> c_int);
    let mut c: SgKvCache = std::ptr::null_mut();
    check(lib, unsafe {
        f(n_layers as c_int, n_kv_heads as c_int, head_dim as c_int, max_seq as c_int, n_seqs as c_int, &mut c)
    })?;
    Ok(c)
}

/// The decode step's RoPE + cache store + attention in one kernel; q, k and
/// v are column slices of one [q | k | v] row buffer of stride `ld`.
pub fn rope_attention_device(rope: SgRope, cache: SgKvCache, layer: usize, qkv: *const f32, ld: i64, d: i64,
                             kv: i64, att: *mut f32, pos: *const i32, seq: *const i32, rows: usize, n_heads: usize,
                             stream: Stream) -> Result<()> {
    let lib = try_lib()?;
    let f = sym!(lib, "sg_rope_attention_device",
                 unsafe extern "C" fn(SgRope, SgKvCache, c_int, *const f32, i64, *const f32, i64, *const f32, i64,
                                      *mut f32, i64, *const i32, *const i32, c_int, c_int, Stream) -> c_int);
    check(lib, unsafe {
        f(rope, cache, layer as c_int, qkv, ld, qkv.add(d as usize), ld, qkv.add((d + kv) as usize), ld, att, d, pos,
          seq, rows as c_int, n_heads as c_int, stream)
    })
}

// ------------------------------------------------------- engine routing

/// Registered weights keyed on the GGUF tensor's file offset
/// (TensorInfo.offset), so each tensor is uploaded once. The reference
/// engine calls from rayon workers (linear.rs:35); the cache is shared.
pub struct WeightCache {
    map: Mutex<HashMap<u64, usize>>, // offset -> SgWeight as an address (Send)
    tp: c_int,
}

impl WeightCache {
    /// `tp`: SG_TP_REPLICATE for one GPU; the engine's TP layout chooses
    /// column split for Q/K/V/gate/up and row split for O/down (use two caches).
    pub fn new(tp: c_int) -> Self {
        WeightCache { map: Mutex::new(HashMap::new()), tp }
    }

    pub fn get(&self, offset: u64, raw: &[u8], dtype: c_int, n_rows: usize, n_cols: usize) -> Result<SgWeight> {
        let mut m = self.map.lock().unwrap();
        if let Some(&w) = m.get(&offset) {
            return Ok(w as SgWeight);
        }
        let w = weight_register(raw, dtype, n_rows, n_cols, self.tp)?;
        m.insert(offset, w as usize);
        Ok(w)
    }
}

impl Drop for WeightCache {
    fn drop(&mut self) {
        if let Ok(m) = self.map.lock() {
            for &w in m.values() {
                let _ = weight_free(w as SgWeight);
            }
        }
    }
}

/// forward_linear (linear.rs:14-90) for a Q4_0 / Q4_K tensor: out = W x.
pub fn forward_linear(cache: &WeightCache, offset: u64, raw: &[u8], dtype: c_int, n_rows: usize, n_cols: usize,
                      x: &[f32], out: &mut [f32]) -> Result<()> {
    let w = cache.get(offset, raw, dtype, n_rows, n_cols)?;
    linear(w, &[x], &mut [out], 0)
}

/// forward_linear_batch (linear.rs:176-239): outs[b] = W xs[b] (zero-filled
/// first in the reference; overwrite here).
pub fn forward_linear_batch(cache: &WeightCache, offset: u64, raw: &[u8], dtype: c_int, n_rows: usize,
                            n_cols: usize, xs: &[&[f32]], outs: &mut [&mut [f32]]) -> Result<()> {
    let w = cache.get(offset, raw, dtype, n_rows, n_cols)?;
    linear(w, xs, outs, 0)
}

/// forward_linear_multi (linear.rs:96-170): several tensors, one x.
pub fn forward_linear_multi(cache: &WeightCache, tensors: &[(u64, &[u8], c_int, usize)], n_cols: usize, x: &[f32],
                            outs: &mut [&mut [f32]]) -> Result<()> {
    let mut ws = Vec::with_capacity(tensors.len());
    for &(offset, raw, dtype, n_rows) in tensors {
        ws.push(cache.get(offset, raw, dtype, n_rows, n_cols)?);
    }
    for (i, chunk) in ws.chunks(4).enumerate() {
        linear_multi(chunk, x, &mut outs[4 * i..4 * i + chunk.len()], 0)?;
    }
    Ok(())
}
