// sg_api.cu -- the C ABI of libswamp_gpu.so (declared in include/swamp_gpu.h).
//
// Host-side mirror of swamp-engine's linear dispatch (swamp-engine/src/linear.rs)
// for Q4_0/Q4_K, routed to the B200 kernels with no CPU fallback. Weight
// handles own device shards; tensor parallelism splits rows (SG_TP_COLUMN) or
// K (SG_TP_ROW, followed by an NCCL sum all-reduce over NVLink). NCCL is
// loaded lazily with dlopen("libnccl.so.2") only when more than one rank
// exists, so the single-GPU library has no NCCL dependency and shares the
// process's NCCL (e.g. torch's) when one is already loaded.
#include <dlfcn.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/swamp_gpu.h"
#include "sg_gemm.cuh"
#include "sg_gemv.cuh"
#include "sg_gemv_q6k.cuh"
#include "sg_peer.cuh"

// ---------------------------------------------------------------- NCCL shim
namespace {
typedef struct ncclComm* ncclComm_t;
typedef struct {
  char internal[128];
} ncclUniqueId;
typedef int ncclResult_t;
enum { kNcclUint8 = 1, kNcclInt32 = 2, kNcclFloat = 7, kNcclSum = 0, kNcclMin = 3 };

struct NcclApi {
  void* h = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommInitAll)(ncclComm_t*, int, const int*) = nullptr;
  ncclResult_t (*AllReduce)(const void*, void*, size_t, int, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  bool load(std::string& err) {
    if (h) return true;
    h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      err = "cannot dlopen libnccl.so.2";
      return false;
    }
#define SG_SYM(f, name)                                 \
  f = reinterpret_cast<decltype(f)>(dlsym(h, name));    \
  if (!f) {                                             \
    err = std::string("libnccl missing symbol ") + name; \
    return false;                                       \
  }
    SG_SYM(GetUniqueId, "ncclGetUniqueId");
    SG_SYM(CommInitRank, "ncclCommInitRank");
    SG_SYM(CommInitAll, "ncclCommInitAll");
    SG_SYM(AllReduce, "ncclAllReduce");
    SG_SYM(AllGather, "ncclAllGather");
    SG_SYM(GroupStart, "ncclGroupStart");
    SG_SYM(GroupEnd, "ncclGroupEnd");
    SG_SYM(CommDestroy, "ncclCommDestroy");
    SG_SYM(GetErrorString, "ncclGetErrorString");
#undef SG_SYM
    return true;
  }
};
NcclApi g_nccl;

// ------------------------------------------------------------------ state
struct DevState {
  int device = -1;
  int num_sms = 0;
  cudaStream_t stream = nullptr;
  ncclComm_t comm = nullptr;
  void* scratch = nullptr;  // activation scratch of the prefill GEMM (grows on demand)
  size_t scratch_bytes = 0;
  void* gemv_ws = nullptr;  // decode workspace for tensors wider than the static one
  size_t gemv_ws_bytes = 0;
  float* xbuf = nullptr;  // staging for host-pointer calls
  size_t xbuf_bytes = 0;
  float* ybuf = nullptr;
  size_t ybuf_bytes = 0;
  float* rbuf = nullptr;  // packed row-split partials of strided device outputs
  size_t rbuf_bytes = 0;
  float* attn_ws = nullptr;  // attention split partials (sg_attention_device)
  size_t attn_ws_bytes = 0;
  void* argmax_ws = nullptr;  // argmax chunk keys, row counters and NaN flags
  size_t argmax_ws_bytes = 0;
  int argmax_rows = 0;  // rows the argmax counters and flags cover
  float* hbuf = nullptr;  // pinned host staging
  size_t hbuf_bytes = 0;
  int* err_host = nullptr;  // pinned copy of the device error word (host-pointer calls)
  float* pbuf = nullptr;    // rows of a prologue (RMSNorm / SiLU-mul) run ahead of a GEMM or Q6_K call
  size_t pbuf_bytes = 0;
  uint8_t* upbuf[2] = {nullptr, nullptr};  // pinned double buffer of weight uploads
  cudaEvent_t upev[2] = {nullptr, nullptr};
  // peer all-reduce (one process per GPU, sg_peer.cuh): this rank's receive
  // buffer (values with their epochs, exported by CUDA IPC), the mappings of
  // every rank's, and the per-chunk epoch counters
  bool peer_on = false;
  void* peer_base = nullptr;
  uint32_t* peer_ctr = nullptr;
  uint32_t* peer_ctr2 = nullptr;  // the two-shot kernel's per-chunk epoch counters
  bool two_shot_on = false;
  SgPeerPtrs peer = {};
  void* peer_mapped[SG_PEER_MAX] = {};
};

struct Ctx {
  std::mutex mu;
  bool inited = false;
  int rank_base = 0;  // global rank of devs[0]
  int world = 1;
  std::vector<DevState> devs;
};
Ctx g_ctx;

thread_local std::string t_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  t_err = buf;
  return code;
}

#define CUDA_TRY(expr)                                                                          \
  do {                                                                                          \
    cudaError_t _e = (expr);                                                                    \
    if (_e != cudaSuccess) return fail(SG_ERR_CUDA, "%s: %s (%s:%d)", #expr, cudaGetErrorString(_e), \
                                       __FILE__, __LINE__);                                     \
  } while (0)

}  // namespace

struct Shard {
  int dev_idx = 0;
  int64_t row0 = 0, col0 = 0;
  SgDevWeight w = {};
};

struct sg_weight_s {
  int dtype = 0;
  int64_t n_rows = 0, n_cols = 0;
  int tp_mode = SG_TP_REPLICATE;
  std::vector<Shard> shards;  // one per local device
};

namespace {

int64_t block_of(int dtype) { return dtype == SG_DTYPE_Q4_0 ? 32 : 256; }
int64_t block_bytes(int dtype) { return dtype == SG_DTYPE_Q4_0 ? 18 : dtype == SG_DTYPE_Q4_K ? 144 : 210; }

// The slice of an n_rows x n_cols tensor that rank R of W holds: column split
// (SG_TP_COLUMN) takes rows [R*N/W, (R+1)*N/W); row split (SG_TP_ROW) takes
// whole blocks [R*nblk/W, (R+1)*nblk/W) of every row; replicate takes all.
// Returns SG_OK or SG_ERR_INVALID_ARG / SG_ERR_UNSUPPORTED with a message.
int shard_plan(int dtype, int64_t n_rows, int64_t n_cols, int tp_mode, int W, int R, int64_t* row0, int64_t* nr,
               int64_t* col0, int64_t* nc) {
  if (dtype != SG_DTYPE_Q4_0 && dtype != SG_DTYPE_Q4_K && dtype != SG_DTYPE_Q6_K)
    return fail(SG_ERR_UNSUPPORTED, "dtype %d not supported (Q4_0=2, Q4_K=12, Q6_K=14)", dtype);
  if (n_rows <= 0 || n_cols <= 0)
    return fail(SG_ERR_INVALID_ARG, "empty tensor %lld x %lld", (long long)n_rows, (long long)n_cols);
  const int64_t bs = block_of(dtype);
  if (n_cols % bs)
    return fail(SG_ERR_INVALID_ARG, "n_cols %lld not a multiple of %lld", (long long)n_cols, (long long)bs);
  if (tp_mode < SG_TP_REPLICATE || tp_mode > SG_TP_ROW) return fail(SG_ERR_INVALID_ARG, "bad tp_mode %d", tp_mode);
  if (W < 1 || R < 0 || R >= W) return fail(SG_ERR_INVALID_ARG, "rank %d of world %d", R, W);
  const int64_t nblk = n_cols / bs;
  if (tp_mode == SG_TP_ROW && nblk < W)
    return fail(SG_ERR_INVALID_ARG, "row split: %lld blocks < %d ranks", (long long)nblk, W);
  if (tp_mode == SG_TP_COLUMN && n_rows < W)
    return fail(SG_ERR_INVALID_ARG, "column split: %lld rows < %d ranks", (long long)n_rows, W);
  *row0 = 0;
  *col0 = 0;
  *nr = n_rows;
  *nc = n_cols;
  if (tp_mode == SG_TP_COLUMN) {
    *row0 = (int64_t)R * n_rows / W;
    *nr = (int64_t)(R + 1) * n_rows / W - *row0;
  } else if (tp_mode == SG_TP_ROW) {
    const int64_t b0 = (int64_t)R * nblk / W, b1 = (int64_t)(R + 1) * nblk / W;
    *col0 = b0 * bs;
    *nc = (b1 - b0) * bs;
  }
  return SG_OK;
}

int ensure_buf(void** p, size_t* have, size_t need) {
  if (*have >= need) return SG_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *have = 0;
  size_t sz = std::max(need, (size_t)1 << 20);
  if (cudaMalloc(p, sz) != cudaSuccess) {
    cudaGetLastError();
    return fail(SG_ERR_OOM, "cudaMalloc(%zu) failed", sz);
  }
  *have = sz;
  return SG_OK;
}

int ensure_host(DevState& d, size_t need) {
  if (d.hbuf_bytes >= need) return SG_OK;
  if (d.hbuf) cudaFreeHost(d.hbuf);
  d.hbuf = nullptr;
  d.hbuf_bytes = 0;
  size_t sz = std::max(need, (size_t)1 << 20);
  if (cudaMallocHost((void**)&d.hbuf, sz) != cudaSuccess) {
    cudaGetLastError();
    return fail(SG_ERR_OOM, "cudaMallocHost(%zu) failed", sz);
  }
  d.hbuf_bytes = sz;
  return SG_OK;
}

// ------------------------------------------------------- GEMV workspace
// The decode GEMV's workspace (sg_gemv.cuh): the activation images of a
// call. Up to kStaticWsCols columns at 16 tokens (wider at fewer tokens) it
// is a fixed array per device inside the library, so no decode call
// allocates; larger calls use a buffer that grows on demand. Every call
// rewrites what it reads, so no state carries over from one call to the
// next.
constexpr int64_t kStaticWsCols = 32768;
constexpr size_t kStaticWsBytes = gemv_mma::ws_bytes<2>(kStaticWsCols / 256);
static __device__ __align__(256) uint8_t g_gemv_ws[kStaticWsBytes];
std::mutex g_ws_mu;
void* g_ws_ptr[64] = {nullptr};

cudaError_t static_workspace(int device, void** out) {
  if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_ws_mu);
  if (!g_ws_ptr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_gemv_ws);
    if (e != cudaSuccess) return e;
    g_ws_ptr[device] = p;
  }
  *out = g_ws_ptr[device];
  return cudaSuccess;
}

// Host-pointer calls read the device error word in the same stream as their
// output (no extra synchronous copy per call): enqueue the read before the
// final synchronisation, check it after.
int read_error_async(DevState& d, cudaStream_t st) {
  if (!d.err_host && cudaMallocHost((void**)&d.err_host, 64) != cudaSuccess) {
    cudaGetLastError();
    d.err_host = nullptr;
    return fail(SG_ERR_OOM, "cudaMallocHost(64) failed");
  }
  CUDA_TRY(cudaMemcpyFromSymbolAsync(d.err_host, g_sg_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st));
  return SG_OK;
}

int check_device_error(DevState& d);

int error_after_sync(DevState& d) {
  if (d.err_host && *(volatile int*)d.err_host == 0) return SG_OK;
  return check_device_error(d);  // reads it again, clears it and reports
}

int check_device_error(DevState& d) {
  int v = 0;
  CUDA_TRY(cudaSetDevice(d.device));
  CUDA_TRY(cudaMemcpyFromSymbol(&v, g_sg_error, sizeof(int)));
  if (v != 0) {
    int z = 0;
    cudaMemcpyToSymbol(g_sg_error, &z, sizeof(int));
    return fail(SG_ERR_DEVICE_FAULT, "device %d: %s (code 0x%x)", d.device,
                v == 0x300 ? "a kernel read a position, token or sequence index out of range"
                           : v == 0x200 ? "a kernel was launched with bad arguments" : "a kernel wait gave up", v);
  }
  return SG_OK;
}

int init_devices(const std::vector<int>& devices, int rank_base, int world) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
    cudaGetLastError();
    return fail(SG_ERR_UNSUPPORTED, "no CUDA device (this library has no CPU fallback)");
  }
  g_ctx.devs.clear();
  for (int dev : devices) {
    if (dev < 0 || dev >= n) return fail(SG_ERR_INVALID_ARG, "device %d out of range (%d devices)", dev, n);
    cudaDeviceProp prop;
    CUDA_TRY(cudaGetDeviceProperties(&prop, dev));
    if (prop.major != 10)
      return fail(SG_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a (B200)", dev, prop.major,
                  prop.minor);
    DevState d;
    d.device = dev;
    d.num_sms = prop.multiProcessorCount;
    CUDA_TRY(cudaSetDevice(dev));
    CUDA_TRY(cudaStreamCreateWithFlags(&d.stream, cudaStreamNonBlocking));
    // bounded device waits: SG_WAIT_NS in the environment (nanoseconds,
    // 1 ms .. 60 s) replaces the built-in 4 s, e.g. for a test that lets a
    // wait run out
    unsigned long long wait_ns = SG_WAIT_NS;
    if (const char* e = std::getenv("SG_WAIT_NS")) {
      const unsigned long long v = strtoull(e, nullptr, 10);
      if (v >= 1000000ull && v <= 60000000000ull) wait_ns = v;
    }
    CUDA_TRY(cudaMemcpyToSymbol(g_sg_wait_ns, &wait_ns, sizeof wait_ns));
    g_ctx.devs.push_back(d);
  }
  g_ctx.rank_base = rank_base;
  g_ctx.world = world;
  return SG_OK;
}

void release_devices() {
  for (auto& d : g_ctx.devs) {
    cudaSetDevice(d.device);
    if (d.comm && g_nccl.CommDestroy) g_nccl.CommDestroy(d.comm);
    if (d.scratch) cudaFree(d.scratch);
    if (d.gemv_ws) cudaFree(d.gemv_ws);
    if (d.xbuf) cudaFree(d.xbuf);
    if (d.ybuf) cudaFree(d.ybuf);
    if (d.rbuf) cudaFree(d.rbuf);
    if (d.attn_ws) cudaFree(d.attn_ws);
    if (d.argmax_ws) cudaFree(d.argmax_ws);
    if (d.hbuf) cudaFreeHost(d.hbuf);
    if (d.err_host) cudaFreeHost(d.err_host);
    if (d.pbuf) cudaFree(d.pbuf);
    for (int i = 0; i < 2; ++i) {
      if (d.upbuf[i]) cudaFreeHost(d.upbuf[i]);
      if (d.upev[i]) cudaEventDestroy(d.upev[i]);
    }
    for (int p = 0; p < SG_PEER_MAX; ++p)
      if (d.peer_mapped[p]) cudaIpcCloseMemHandle(d.peer_mapped[p]);
    if (d.peer_base) cudaFree(d.peer_base);
    if (d.peer_ctr) cudaFree(d.peer_ctr);
    if (d.peer_ctr2) cudaFree(d.peer_ctr2);
    if (d.stream) cudaStreamDestroy(d.stream);
  }
  g_ctx.devs.clear();
  g_ctx.inited = false;
}

// ---------------------------------------------------------- the core launch
// y[b][*] (ldy) = W_shard x[b][*] (ldx) on one device, stream-ordered.
// the prologue's rows into out [batch][K] (sg_ops.cu: the same kernels as
// sg_rmsnorm_device / sg_silu_mul_device)
int apply_prologue(DevState& d, const SgGemvPrologue& pro, const float* x, int64_t ldx, int64_t K, int batch,
                   float* out, cudaStream_t st);

int run_linear(DevState& d, const SgDevWeight* const* ws, int n_w, const float* x, int64_t ldx,
               float* const* ys, const int64_t* ldys, int batch, cudaStream_t st, bool accumulate,
               const SgGemvPrologue* pro = nullptr) {
  const int64_t K = ws[0]->n_cols;
  if (((uintptr_t)x & 15) || (ldx & 3))
    return fail(SG_ERR_INVALID_ARG, "x must be 16-byte aligned with a row stride that is a multiple of 4 floats");
  if (pro && pro->kind != SG_PRO_NONE) {
    // the decode GEMV (Q4_0 / Q4_K, up to SG_GEMV_MAX_BATCH tokens) applies
    // the prologue on its own way in; anything else gets the rows first
    bool fused = batch <= SG_GEMV_MAX_BATCH;
    for (int i = 0; i < n_w; ++i) fused = fused && ws[i]->dtype != SG_DTYPE_Q6_K;
    if (!fused) {
      int rc = ensure_buf((void**)&d.pbuf, &d.pbuf_bytes, (size_t)batch * K * sizeof(float));
      if (rc) return rc;
      rc = apply_prologue(d, *pro, x, ldx, K, batch, d.pbuf, st);
      if (rc) return rc;
      x = d.pbuf;
      ldx = K;
      pro = nullptr;
    }
  }
  if (batch <= SG_GEMV_MAX_BATCH) {
    void* gws = nullptr;
    size_t gws_bytes = sg_gemv_scratch_bytes(K, batch);
    if (gws_bytes <= kStaticWsBytes) {
      CUDA_TRY(static_workspace(d.device, &gws));
      gws_bytes = kStaticWsBytes;
    } else {
      if (d.gemv_ws_bytes < gws_bytes) {
        if (d.gemv_ws) cudaFree(d.gemv_ws);
        d.gemv_ws = nullptr;
        d.gemv_ws_bytes = 0;
        if (cudaMalloc(&d.gemv_ws, gws_bytes) != cudaSuccess) {
          cudaGetLastError();
          return fail(SG_ERR_OOM, "cudaMalloc(%zu) failed", gws_bytes);
        }
        d.gemv_ws_bytes = gws_bytes;
      }
      gws = d.gemv_ws;
      gws_bytes = d.gemv_ws_bytes;
    }
    // one launch per run of consecutive same-dtype matrices (Q6_K: one per
    // matrix, on its own kernel)
    for (int i0 = 0; i0 < n_w;) {
      if (ws[i0]->dtype == SG_DTYPE_Q6_K) {
        if (batch <= SG_GEMV_Q6K_MAX_BATCH) {
          CUDA_TRY(sg_gemv_q6k(ws[i0], x, ldx, ys[i0], ldys[i0], batch, accumulate, d.num_sms, st));
        } else {
          const size_t need = sg_gemm_scratch_bytes(batch, K);
          int rc = need ? ensure_buf(&d.scratch, &d.scratch_bytes, need) : SG_OK;
          if (rc) return rc;
          CUDA_TRY(sg_gemm(ws[i0], x, ldx, ys[i0], ldys[i0], batch, accumulate, d.scratch, d.scratch_bytes,
                           d.num_sms, st));
        }
        ++i0;
        continue;
      }
      int i1 = i0 + 1;
      while (i1 < n_w && i1 - i0 < SG_GEMV_MAX_MATS && ws[i1]->dtype == ws[i0]->dtype) ++i1;
      SgGemvMat mats[SG_GEMV_MAX_MATS];
      for (int i = i0; i < i1; ++i) mats[i - i0] = {ws[i], ys[i], ldys[i]};
      CUDA_TRY(sg_gemv(mats, i1 - i0, x, ldx, batch, accumulate, gws, gws_bytes, d.num_sms, st, pro));
      i0 = i1;
    }
    return SG_OK;
  }
  // prefill GEMM: one launch per matrix
  for (int i = 0; i < n_w; ++i) {
    const size_t need = sg_gemm_scratch_bytes(batch, K);
    int rc = need ? ensure_buf(&d.scratch, &d.scratch_bytes, need) : SG_OK;
    if (rc) return rc;
    CUDA_TRY(sg_gemm(ws[i], x, ldx, ys[i], ldys[i], batch, accumulate, d.scratch, d.scratch_bytes, d.num_sms, st));
  }
  return SG_OK;
}

constexpr int64_t kPeerCap = (int64_t)kArChunk * kArMaxChunks;  // floats per slot
constexpr int64_t kPeerCap2 = kPeerCap / 2;                        // floats per two-shot part slot
constexpr int kAr2MaxChunks = (int)(kPeerCap2 / kAr2Chunk);

// -1: the size rule below; 0: never two-shot; 1: always (when set up)
int two_shot_mode() {
  static const int m = [] {
    const char* v = std::getenv("SG_AR_TWO_SHOT");
    return v ? (v[0] == '1' ? 1 : 0) : -1;
  }();
  return m;
}

// Sum all-reduce of `count` floats in place on this rank's device: the peer
// kernel when it is set up and the vector fits a slot, else NCCL.
// path: 0 by the rules below, 1 the one-shot peer kernel, 2 the two-shot one
int allreduce_rank(DevState& d, float* buf, size_t count, cudaStream_t st, int path = 0) {
  if (g_ctx.world <= 1 || count == 0) return SG_OK;
  const int tsm = two_shot_mode();
  const bool two = path == 2 || (path == 0 && d.two_shot_on &&
                                 (tsm == 1 || (tsm == -1 && g_ctx.world >= 4 && count >= ((size_t)1 << 17))));
  if (d.peer_on && two && (int64_t)count <= kPeerCap) {
    // large vectors on 4+ ranks: reduce-scatter + all-gather (each rank sends
    // 2 (W-1)/W of the vector instead of (W-1) times it)
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = sg_pdl_enabled() ? 1 : 0;
    const int64_t part = (((int64_t)count + g_ctx.world - 1) / g_ctx.world + 1) & ~(int64_t)1;
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3((unsigned)((part + kAr2Chunk - 1) / kAr2Chunk));
    c.blockDim = dim3(kAr2Threads);
    c.stream = st;
    c.attrs = attr;
    c.numAttrs = 1;
    CUDA_TRY(cudaLaunchKernelEx(&c, peer_allreduce2_kernel, (const float*)buf, buf, (int64_t)count, g_ctx.world,
                                g_ctx.rank_base, d.peer, d.peer_ctr2, part, kPeerCap2));
    return SG_OK;
  }
  if (d.peer_on && (int64_t)count <= kPeerCap) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = sg_pdl_enabled() ? 1 : 0;
    cudaLaunchConfig_t c = {};
    c.gridDim = dim3((unsigned)((count + kArChunk - 1) / kArChunk));
    c.blockDim = dim3(kArThreads);
    c.stream = st;
    c.attrs = attr;
    c.numAttrs = 1;
    CUDA_TRY(cudaLaunchKernelEx(&c, peer_allreduce_kernel, (const float*)buf, buf, (int64_t)count, g_ctx.world,
                                g_ctx.rank_base, d.peer, d.peer_ctr, kPeerCap));
    return SG_OK;
  }
  if (!g_nccl.AllReduce) return fail(SG_ERR_NCCL, "NCCL not initialised");
  ncclResult_t r = g_nccl.AllReduce(buf, buf, count, kNcclFloat, kNcclSum, d.comm, st);
  if (r) return fail(SG_ERR_NCCL, "ncclAllReduce: %s", g_nccl.GetErrorString(r));
  return SG_OK;
}

// Set up the peer all-reduce of a rank (collective: every rank calls it
// from sg_init_rank). Each rank allocates and zeroes its receive buffer,
// exports it, gathers every rank's handle over NCCL and maps the others;
// the ranks then agree (NCCL min) whether all of them succeeded, so that
// either every rank uses the peer kernel or every rank uses NCCL.
int peer_setup(DevState& d) {
  const int W = g_ctx.world, R = g_ctx.rank_base;
  int ok = W <= SG_PEER_MAX;
  const char* env = std::getenv("SG_PEER_ALLREDUCE");
  if (env && env[0] == '0') ok = 0;  // SG_PEER_ALLREDUCE=0: NCCL for every all-reduce
  // [2 parities][W ranks][kPeerCap / 2] words of {v0, epoch, v1, epoch}, then
  // the two-shot slots [2 parities][2 phases][W ranks][kPeerCap2 / 2]
  const size_t buf1_bytes = (size_t)2 * W * (kPeerCap / 2) * sizeof(uint4);
  const size_t buf_bytes = buf1_bytes + (size_t)2 * 2 * W * (kPeerCap2 / 2) * sizeof(uint4);
  cudaIpcMemHandle_t mine = {};
  if (ok && (cudaMalloc(&d.peer_base, buf_bytes) != cudaSuccess ||
             cudaMalloc((void**)&d.peer_ctr, kArMaxChunks * sizeof(uint32_t)) != cudaSuccess ||
             cudaMalloc((void**)&d.peer_ctr2, kAr2MaxChunks * sizeof(uint32_t)) != cudaSuccess ||
             cudaMemset(d.peer_ctr2, 0, kAr2MaxChunks * sizeof(uint32_t)) != cudaSuccess ||
             cudaMemset(d.peer_base, 0, buf_bytes) != cudaSuccess ||
             cudaMemset(d.peer_ctr, 0, kArMaxChunks * sizeof(uint32_t)) != cudaSuccess ||
             cudaDeviceSynchronize() != cudaSuccess || cudaIpcGetMemHandle(&mine, d.peer_base) != cudaSuccess)) {
    cudaGetLastError();
    ok = 0;
  }
  // gather the handles (64 bytes each) through a device buffer
  uint8_t* dev = nullptr;
  CUDA_TRY(cudaMalloc(&dev, (size_t)(W + 1) * sizeof(cudaIpcMemHandle_t)));
  std::vector<cudaIpcMemHandle_t> all(W);
  CUDA_TRY(cudaMemcpy(dev + (size_t)W * sizeof mine, &mine, sizeof mine, cudaMemcpyHostToDevice));
  ncclResult_t r = g_nccl.AllGather(dev + (size_t)W * sizeof mine, dev, sizeof mine, kNcclUint8, d.comm, d.stream);
  if (r) {
    cudaFree(dev);
    return fail(SG_ERR_NCCL, "ncclAllGather: %s", g_nccl.GetErrorString(r));
  }
  CUDA_TRY(cudaStreamSynchronize(d.stream));
  CUDA_TRY(cudaMemcpy(all.data(), dev, (size_t)W * sizeof mine, cudaMemcpyDeviceToHost));
  for (int p = 0; p < W && ok; ++p) {
    if (p == R) {
      d.peer.buf[p] = static_cast<uint4*>(d.peer_base);
      d.peer.buf2[p] = reinterpret_cast<uint4*>(static_cast<uint8_t*>(d.peer_base) + buf1_bytes);
    } else if (cudaIpcOpenMemHandle(&d.peer_mapped[p], all[p], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = 0;
      break;
    } else {
      d.peer.buf[p] = static_cast<uint4*>(d.peer_mapped[p]);
      d.peer.buf2[p] = reinterpret_cast<uint4*>(static_cast<uint8_t*>(d.peer_mapped[p]) + buf1_bytes);
    }
  }
  // every rank must take the same path
  int* dok = reinterpret_cast<int*>(dev);
  CUDA_TRY(cudaMemcpy(dok, &ok, sizeof ok, cudaMemcpyHostToDevice));
  r = g_nccl.AllReduce(dok, dok, 1, kNcclInt32, kNcclMin, d.comm, d.stream);
  CUDA_TRY(cudaStreamSynchronize(d.stream));
  CUDA_TRY(cudaMemcpy(&ok, dok, sizeof ok, cudaMemcpyDeviceToHost));
  if (r) {
    cudaFree(dev);
    return fail(SG_ERR_NCCL, "ncclAllReduce: %s", g_nccl.GetErrorString(r));
  }
  d.peer_on = ok != 0;
  if (d.peer_on) {
    // self-test: an all-reduce of small integers through each peer kernel
    // (one-shot, then two-shot), which must come out exact on every rank; a
    // wrong sum or a wait that gave up on any rank turns that kernel off for
    // the whole job (NCCL, or the one-shot kernel, instead)
    auto selftest = [&](int path, int64_t n) -> int {
      std::vector<float> h(n, (float)(R + 1));
      float* t = nullptr;
      int pass = cudaMalloc(&t, n * sizeof(float)) == cudaSuccess &&
                 cudaMemcpy(t, h.data(), n * sizeof(float), cudaMemcpyHostToDevice) == cudaSuccess;
      if (pass) pass = allreduce_rank(d, t, (size_t)n, d.stream, path) == SG_OK &&
                       cudaStreamSynchronize(d.stream) == cudaSuccess &&
                       cudaMemcpy(h.data(), t, n * sizeof(float), cudaMemcpyDeviceToHost) == cudaSuccess;
      const float want = (float)W * (W + 1) / 2;
      for (int64_t i = 0; pass && i < n; ++i) pass = h[i] == want;
      int err = 0;
      cudaMemcpyFromSymbol(&err, g_sg_error, sizeof(int));
      if (err) {
        pass = 0;
        const int z = 0;
        cudaMemcpyToSymbol(g_sg_error, &z, sizeof(int));
      }
      if (t) cudaFree(t);
      cudaGetLastError();
      return pass;
    };
    int pass[2];
    pass[0] = selftest(1, 2 * kArChunk + 3);
    pass[1] = pass[0] && selftest(2, 2 * (int64_t)W * kAr2Chunk + 3);
    CUDA_TRY(cudaMemcpy(dok, pass, sizeof pass, cudaMemcpyHostToDevice));
    r = g_nccl.AllReduce(dok, dok, 2, kNcclInt32, kNcclMin, d.comm, d.stream);
    CUDA_TRY(cudaStreamSynchronize(d.stream));
    CUDA_TRY(cudaMemcpy(pass, dok, sizeof pass, cudaMemcpyDeviceToHost));
    if (r) {
      cudaFree(dev);
      return fail(SG_ERR_NCCL, "ncclAllReduce: %s", g_nccl.GetErrorString(r));
    }
    if (!pass[0]) {
      std::fprintf(stderr, "swamp_gpu: the peer all-reduce self-test failed; using NCCL\n");
      d.peer_on = false;
    }
    d.two_shot_on = pass[0] && pass[1];
    if (pass[0] && !pass[1]) std::fprintf(stderr, "swamp_gpu: the two-shot all-reduce self-test failed; not used\n");
  }
  cudaFree(dev);
  return SG_OK;
}

int allreduce_local(const std::vector<float*>& bufs, size_t count) {
  if (g_ctx.world <= 1) return SG_OK;
  if (g_ctx.devs.size() == 1) return allreduce_rank(g_ctx.devs[0], bufs[0], count, g_ctx.devs[0].stream);
  if (!g_nccl.AllReduce) return fail(SG_ERR_NCCL, "NCCL not initialised");
  ncclResult_t r = g_nccl.GroupStart();
  for (size_t i = 0; i < g_ctx.devs.size() && r == 0; ++i) {
    DevState& d = g_ctx.devs[i];
    cudaSetDevice(d.device);
    r = g_nccl.AllReduce(bufs[i], bufs[i], count, kNcclFloat, kNcclSum, d.comm, d.stream);
  }
  ncclResult_t r2 = g_nccl.GroupEnd();
  if (r || r2) return fail(SG_ERR_NCCL, "ncclAllReduce: %s", g_nccl.GetErrorString(r ? r : r2));
  return SG_OK;
}

int validate_weight(sg_weight_t w) {
  if (!g_ctx.inited) return fail(SG_ERR_NOT_INITIALIZED, "sg_init not called");
  if (!w) return fail(SG_ERR_INVALID_ARG, "null weight handle");
  if (w->shards.size() != g_ctx.devs.size()) return fail(SG_ERR_INVALID_ARG, "weight registered under another init");
  return SG_OK;
}

// Rows rows[0..n) + off, `width` floats each, that sit in page-locked host
// memory one fixed stride apart (a caller's cudaHostAlloc or sg_host_alloc
// buffer): the copy engine moves them straight from or to the caller with one
// 2D copy instead of through the library's staging buffer. Returns that
// stride in floats, or 0 when the rows are pageable, ragged or overlapping.
int64_t pinned_stride(const float* const* rows, int n, int64_t off, int64_t width) {
  const uintptr_t base = (uintptr_t)rows[0];
  const intptr_t step = n > 1 ? (intptr_t)((uintptr_t)rows[1] - base) : (intptr_t)(width * sizeof(float));
  if (step % (intptr_t)sizeof(float) || step < (intptr_t)(width * sizeof(float))) return 0;
  for (int b = 2; b < n; ++b)
    if ((uintptr_t)rows[b] != base + (uintptr_t)step * (uintptr_t)b) return 0;
  const float* ends[2] = {rows[0] + off, rows[n - 1] + off + width - 1};
  for (const float* p : ends) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
      cudaGetLastError();
      return 0;
    }
    if (a.type != cudaMemoryTypeHost) return 0;
  }
  return (int64_t)(step / (intptr_t)sizeof(float));
}

// host-pointer linear over all local devices (also the multi form)
int linear_host(const sg_weight_t* ws, int n_w, const float* const* xs, float* const* outs, int batch, int flags) {
  const int64_t K = ws[0]->n_cols;
  const int tp = ws[0]->tp_mode;
  for (int i = 0; i < n_w; ++i) {
    int rc = validate_weight(ws[i]);
    if (rc) return rc;
    if (ws[i]->n_cols != K || ws[i]->dtype != ws[0]->dtype)
      return fail(SG_ERR_INVALID_ARG, "multi: tensors must share dtype and n_cols");
    if (ws[i]->tp_mode != tp) return fail(SG_ERR_INVALID_ARG, "multi: tensors must share tp_mode");
  }
  if (n_w > SG_GEMV_MAX_MATS) return fail(SG_ERR_INVALID_ARG, "at most %d tensors per multi call", SG_GEMV_MAX_MATS);
  const bool accumulate = (flags & SG_FLAG_ACCUMULATE) != 0;
  const size_t nd = g_ctx.devs.size();
  std::vector<std::vector<float*>> ydev(nd, std::vector<float*>(n_w));
  std::vector<std::vector<int64_t>> ld(nd, std::vector<int64_t>(n_w));
  // 1. stage inputs and launch on every local device
  for (size_t di = 0; di < nd; ++di) {
    DevState& d = g_ctx.devs[di];
    const Shard& s0 = ws[0]->shards[di];
    const int64_t kl = s0.w.n_cols, c0 = s0.col0;
    CUDA_TRY(cudaSetDevice(d.device));
    int64_t ytot = 0;
    for (int i = 0; i < n_w; ++i) ytot += (int64_t)batch * (tp == SG_TP_ROW ? ws[i]->n_rows : ws[i]->shards[di].w.n_rows);
    int rc = ensure_buf((void**)&d.xbuf, &d.xbuf_bytes, (size_t)batch * kl * sizeof(float));
    if (rc) return rc;
    rc = ensure_buf((void**)&d.ybuf, &d.ybuf_bytes, (size_t)ytot * sizeof(float));
    if (rc) return rc;
    const size_t hx = (size_t)batch * kl * sizeof(float);
    rc = ensure_host(d, std::max(hx, (size_t)ytot * sizeof(float)));
    if (rc) return rc;
    CUDA_TRY(cudaStreamSynchronize(d.stream));  // pinned staging reuse
    const int64_t xpitch = nd == 1 ? pinned_stride(xs, batch, c0, kl) : 0;
    if (xpitch) {
      CUDA_TRY(cudaMemcpy2DAsync(d.xbuf, (size_t)kl * sizeof(float), xs[0] + c0, (size_t)xpitch * sizeof(float),
                                 (size_t)kl * sizeof(float), (size_t)batch, cudaMemcpyHostToDevice, d.stream));
    } else {
      for (int b = 0; b < batch; ++b) memcpy(d.hbuf + (size_t)b * kl, xs[b] + c0, (size_t)kl * sizeof(float));
      CUDA_TRY(cudaMemcpyAsync(d.xbuf, d.hbuf, hx, cudaMemcpyHostToDevice, d.stream));
    }
    int64_t off = 0;
    const SgDevWeight* sw[SG_GEMV_MAX_MATS];
    for (int i = 0; i < n_w; ++i) {
      sw[i] = &ws[i]->shards[di].w;
      ydev[di][i] = d.ybuf + off;
      ld[di][i] = tp == SG_TP_ROW ? ws[i]->n_rows : sw[i]->n_rows;
      off += (int64_t)batch * ld[di][i];
    }
    rc = run_linear(d, sw, n_w, d.xbuf, kl, ydev[di].data(), ld[di].data(), batch, d.stream, false);
    if (rc) return rc;
  }
  // 2. row split: sum partial outputs across ranks
  if (tp == SG_TP_ROW && g_ctx.world > 1) {
    std::vector<float*> bufs(nd);
    size_t count = 0;
    for (int i = 0; i < n_w; ++i) count += (size_t)batch * ws[i]->n_rows;
    for (size_t di = 0; di < nd; ++di) bufs[di] = g_ctx.devs[di].ybuf;
    int rc = allreduce_local(bufs, count);
    if (rc) return rc;
  }
  // 3. copy back: column split -> every device its rows; otherwise device 0
  for (size_t di = 0; di < nd; ++di) {
    if (tp != SG_TP_COLUMN && di > 0) break;
    DevState& d = g_ctx.devs[di];
    CUDA_TRY(cudaSetDevice(d.device));
    // one device and no accumulation: outputs in page-locked memory are
    // written by the copy engine directly, the rest through the staging buffer
    int64_t tot = 0, staged = 0;
    int64_t opitch[SG_GEMV_MAX_MATS];
    for (int i = 0; i < n_w; ++i) {
      const int64_t r0 = tp == SG_TP_COLUMN ? ws[i]->shards[di].row0 : 0;
      opitch[i] = nd == 1 && !accumulate ? pinned_stride(outs + (size_t)i * batch, batch, r0, ld[di][i]) : 0;
      if (opitch[i]) {
        CUDA_TRY(cudaMemcpy2DAsync(outs[(size_t)i * batch] + r0, (size_t)opitch[i] * sizeof(float), d.ybuf + tot,
                                   (size_t)ld[di][i] * sizeof(float), (size_t)ld[di][i] * sizeof(float),
                                   (size_t)batch, cudaMemcpyDeviceToHost, d.stream));
      } else {
        staged = tot + (int64_t)batch * ld[di][i];
      }
      tot += (int64_t)batch * ld[di][i];
    }
    if (staged)  // the staged tensors lie within the first `staged` floats
      CUDA_TRY(cudaMemcpyAsync(d.hbuf, d.ybuf, (size_t)staged * sizeof(float), cudaMemcpyDeviceToHost, d.stream));
    int rc = read_error_async(d, d.stream);
    if (rc) return rc;
    CUDA_TRY(cudaStreamSynchronize(d.stream));
    rc = error_after_sync(d);
    if (rc) return rc;
    int64_t off = 0;
    for (int i = 0; i < n_w; ++i) {
      const Shard& s = ws[i]->shards[di];
      const int64_t r0 = tp == SG_TP_COLUMN ? s.row0 : 0;
      const int64_t nr = ld[di][i];
      if (opitch[i]) {
        off += (int64_t)batch * nr;
        continue;
      }
      for (int b = 0; b < batch; ++b) {
        float* dst = outs[(size_t)i * batch + b] + r0;
        const float* src = d.hbuf + off + (size_t)b * nr;
        if (accumulate)
          for (int64_t r = 0; r < nr; ++r) dst[r] += src[r];
        else
          memcpy(dst, src, (size_t)nr * sizeof(float));
      }
      off += (int64_t)batch * nr;
    }
  }
  for (size_t di = 1; di < nd; ++di) {
    cudaSetDevice(g_ctx.devs[di].device);
    CUDA_TRY(cudaStreamSynchronize(g_ctx.devs[di].stream));
    int rc = check_device_error(g_ctx.devs[di]);
    if (rc) return rc;
  }
  return SG_OK;
}

}  // namespace

// ====================================================================== ABI
extern "C" {

const char* sg_last_error(void) { return t_err.c_str(); }

int sg_init(int n_gpus) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  if (g_ctx.inited) return fail(SG_ERR_INVALID_ARG, "already initialised; call sg_shutdown first");
  if (n_gpus < 1) return fail(SG_ERR_INVALID_ARG, "n_gpus must be >= 1");
  std::vector<int> devs;
  for (int i = 0; i < n_gpus; ++i) devs.push_back(i);
  int rc = init_devices(devs, 0, n_gpus);
  if (rc) {
    release_devices();
    return rc;
  }
  if (n_gpus > 1) {
    std::string err;
    if (!g_nccl.load(err)) {
      release_devices();
      return fail(SG_ERR_NCCL, "%s", err.c_str());
    }
    std::vector<ncclComm_t> comms(n_gpus);
    ncclResult_t r = g_nccl.CommInitAll(comms.data(), n_gpus, devs.data());
    if (r) {
      release_devices();
      return fail(SG_ERR_NCCL, "ncclCommInitAll: %s", g_nccl.GetErrorString(r));
    }
    for (int i = 0; i < n_gpus; ++i) g_ctx.devs[i].comm = comms[i];
  }
  g_ctx.inited = true;
  return SG_OK;
}

int sg_get_unique_id(void* id128) {
  if (!id128) return fail(SG_ERR_INVALID_ARG, "null id buffer");
  std::string err;
  if (!g_nccl.load(err)) return fail(SG_ERR_NCCL, "%s", err.c_str());
  ncclUniqueId id;
  ncclResult_t r = g_nccl.GetUniqueId(&id);
  if (r) return fail(SG_ERR_NCCL, "ncclGetUniqueId: %s", g_nccl.GetErrorString(r));
  memcpy(id128, &id, sizeof id);
  return SG_OK;
}

int sg_init_rank(int rank, int world, const void* id128, int device) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  if (g_ctx.inited) return fail(SG_ERR_INVALID_ARG, "already initialised; call sg_shutdown first");
  if (world < 1 || rank < 0 || rank >= world) return fail(SG_ERR_INVALID_ARG, "bad rank %d / world %d", rank, world);
  if (world > 1 && !id128) return fail(SG_ERR_INVALID_ARG, "world > 1 needs the NCCL unique id");
  int rc = init_devices({device}, rank, world);
  if (rc) {
    release_devices();
    return rc;
  }
  if (world > 1) {
    std::string err;
    if (!g_nccl.load(err)) {
      release_devices();
      return fail(SG_ERR_NCCL, "%s", err.c_str());
    }
    ncclUniqueId id;
    memcpy(&id, id128, sizeof id);
    cudaSetDevice(device);
    ncclResult_t r = g_nccl.CommInitRank(&g_ctx.devs[0].comm, world, id, rank);
    if (r) {
      release_devices();
      return fail(SG_ERR_NCCL, "ncclCommInitRank: %s", g_nccl.GetErrorString(r));
    }
    g_ctx.world = world;
    g_ctx.rank_base = rank;
    rc = peer_setup(g_ctx.devs[0]);
    if (rc) {
      release_devices();
      return rc;
    }
  }
  g_ctx.inited = true;
  return SG_OK;
}

int sg_shutdown(void) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  for (auto& d : g_ctx.devs) {
    cudaSetDevice(d.device);
    cudaStreamSynchronize(d.stream);
  }
  release_devices();
  return SG_OK;
}

int sg_topology(int* rank, int* world, int* local_devices) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  if (!g_ctx.inited) return fail(SG_ERR_NOT_INITIALIZED, "sg_init not called");
  if (rank) *rank = g_ctx.rank_base;
  if (world) *world = g_ctx.world;
  if (local_devices) *local_devices = (int)g_ctx.devs.size();
  return SG_OK;
}

// Host blocks (any memory: a mapped GGUF file, pageable buffers) to the
// device: rows of `lrow` bytes at a stride of `row_bytes` are gathered into
// two pinned 8 MB buffers in turn, each copied asynchronously while the
// other is filled, so the copy runs at pinned-memory speed and overlaps the
// host gather.
namespace {
constexpr size_t kUploadChunk = 8u << 20;
cudaError_t upload_rows(DevState& d, uint8_t* dst, const uint8_t* src, size_t row_bytes, size_t lrow, int64_t nr) {
  for (int i = 0; i < 2; ++i) {
    if (!d.upbuf[i]) {
      cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&d.upbuf[i]), kUploadChunk, cudaHostAllocDefault);
      if (e != cudaSuccess) return e;
    }
    if (!d.upev[i]) {
      cudaError_t e = cudaEventCreateWithFlags(&d.upev[i], cudaEventDisableTiming);
      if (e != cudaSuccess) return e;
    }
  }
  if (lrow > kUploadChunk)  // a row wider than the staging buffer: one plain copy
    return cudaMemcpy2DAsync(dst, lrow, src, row_bytes, lrow, (size_t)nr, cudaMemcpyHostToDevice, d.stream);
  const int64_t rows_per = (int64_t)(kUploadChunk / lrow);
  int b = 0;
  for (int64_t r0 = 0; r0 < nr; r0 += rows_per, b ^= 1) {
    const int64_t n = std::min(rows_per, nr - r0);
    cudaError_t e = cudaEventSynchronize(d.upev[b]);  // this buffer's previous copy is done
    if (e != cudaSuccess) return e;
    uint8_t* buf = d.upbuf[b];
    if (row_bytes == lrow) {
      memcpy(buf, src + (size_t)r0 * row_bytes, (size_t)n * lrow);
    } else {
      for (int64_t r = 0; r < n; ++r) memcpy(buf + (size_t)r * lrow, src + (size_t)(r0 + r) * row_bytes, lrow);
    }
    e = cudaMemcpyAsync(dst + (size_t)r0 * lrow, buf, (size_t)n * lrow, cudaMemcpyHostToDevice, d.stream);
    if (e == cudaSuccess) e = cudaEventRecord(d.upev[b], d.stream);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// Fills a rank's raw GGUF block buffer on its device: rows [row0, row0+nr)
// and blocks [cb0, cb0+ncb) of every row, row-major with ncb*block_bytes per
// row. Host uploads and the on-device synthetic generator implement it.
struct RawFill {
  virtual cudaError_t fill(DevState& d, uint8_t* raw, int64_t row0, int64_t nr, int64_t cb0, int64_t ncb) = 0;
  virtual ~RawFill() {}
};

struct HostFill : RawFill {
  const uint8_t* blocks;
  size_t row_bytes, bb;
  cudaError_t fill(DevState& d, uint8_t* raw, int64_t row0, int64_t nr, int64_t cb0, int64_t ncb) override {
    return upload_rows(d, raw, blocks + (size_t)row0 * row_bytes + (size_t)cb0 * bb, row_bytes, (size_t)ncb * bb, nr);
  }
};

// Validate, shard, fill the raw blocks of each local shard on its device and
// repack them into the tile layout. Called with g_ctx.mu held.
int register_weight(RawFill& src, int dtype, int64_t n_rows, int64_t n_cols, int tp_mode, sg_weight_t* out) {
  if (!g_ctx.inited) return fail(SG_ERR_NOT_INITIALIZED, "sg_init not called");
  if (!out) return fail(SG_ERR_INVALID_ARG, "null pointer");
  const int W = g_ctx.world;
  for (int R = 0; R < W; ++R) {  // validates the arguments for every rank's slice
    int64_t r0, nr, c0, nc;
    const int rc = shard_plan(dtype, n_rows, n_cols, tp_mode, W, R, &r0, &nr, &c0, &nc);
    if (rc != SG_OK) return rc;
  }
  const int64_t bs = block_of(dtype), bb = block_bytes(dtype);
  auto* w = new sg_weight_s();
  w->dtype = dtype;
  w->n_rows = n_rows;
  w->n_cols = n_cols;
  w->tp_mode = tp_mode;
  int rc = SG_OK;
  for (size_t di = 0; di < g_ctx.devs.size() && rc == SG_OK; ++di) {
    DevState& d = g_ctx.devs[di];
    const int R = g_ctx.rank_base + (int)di;
    Shard s;
    s.dev_idx = (int)di;
    int64_t nr = n_rows, nc = n_cols;
    shard_plan(dtype, n_rows, n_cols, tp_mode, W, R, &s.row0, &nr, &s.col0, &nc);
    cudaSetDevice(d.device);
    if (sg_layout_alloc(&s.w, dtype, nr, nc)) {
      cudaGetLastError();
      rc = fail(SG_ERR_OOM, "device %d: cannot allocate %zu bytes for weights", d.device,
                sg_layout_bytes(dtype, nr, nc));
      break;
    }
    const size_t lrow = (size_t)(nc / bs) * bb;
    uint8_t* raw = nullptr;
    if (cudaMalloc(&raw, lrow * nr) != cudaSuccess) {
      cudaGetLastError();
      sg_layout_free(&s.w);
      rc = fail(SG_ERR_OOM, "device %d: cannot allocate upload staging", d.device);
      break;
    }
    cudaError_t e = src.fill(d, raw, s.row0, nr, s.col0 / bs, nc / bs);
    if (e == cudaSuccess) e = sg_layout_repack(&s.w, raw, d.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d.stream);
    cudaFree(raw);
    if (e != cudaSuccess) {
      sg_layout_free(&s.w);
      rc = fail(SG_ERR_CUDA, "upload/repack on device %d: %s", d.device, cudaGetErrorString(e));
      break;
    }
    w->shards.push_back(s);
  }
  if (rc != SG_OK) {
    for (auto& s : w->shards) {
      cudaSetDevice(g_ctx.devs[s.dev_idx].device);
      sg_layout_free(&s.w);
    }
    delete w;
    return rc;
  }
  *out = w;
  return SG_OK;
}
}  // namespace

int sg_weight_register(const void* host_blocks, int dtype, int64_t n_rows, int64_t n_cols, int tp_mode,
                       sg_weight_t* out) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  if (!host_blocks) return fail(SG_ERR_INVALID_ARG, "null pointer");
  HostFill f;
  f.blocks = static_cast<const uint8_t*>(host_blocks);
  f.bb = (size_t)block_bytes(dtype);
  f.row_bytes = (size_t)(n_cols / std::max<int64_t>(1, block_of(dtype))) * f.bb;
  return register_weight(f, dtype, n_rows, n_cols, tp_mode, out);
}

int sg_weight_free(sg_weight_t w) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  if (!w) return fail(SG_ERR_INVALID_ARG, "null weight handle");
  for (auto& s : w->shards) {
    if (s.dev_idx < (int)g_ctx.devs.size()) {
      cudaSetDevice(g_ctx.devs[s.dev_idx].device);
      cudaStreamSynchronize(g_ctx.devs[s.dev_idx].stream);
    }
    sg_layout_free(&s.w);
  }
  delete w;
  return SG_OK;
}

int sg_tp_shard(int dtype, int64_t n_rows, int64_t n_cols, int tp_mode, int world, int rank, int64_t* row0,
                int64_t* rows, int64_t* col0, int64_t* cols) {
  if (!row0 || !rows || !col0 || !cols) return fail(SG_ERR_INVALID_ARG, "null pointer");
  return shard_plan(dtype, n_rows, n_cols, tp_mode, world, rank, row0, rows, col0, cols);
}

int sg_weight_shard(sg_weight_t w, int local_device, int64_t* n_rows, int64_t* n_cols, int64_t* row0, int64_t* col0) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  int rc = validate_weight(w);
  if (rc) return rc;
  if (local_device < 0 || local_device >= (int)w->shards.size()) return fail(SG_ERR_INVALID_ARG, "bad local device");
  const Shard& s = w->shards[local_device];
  if (n_rows) *n_rows = s.w.n_rows;
  if (n_cols) *n_cols = s.w.n_cols;
  if (row0) *row0 = s.row0;
  if (col0) *col0 = s.col0;
  return SG_OK;
}

int sg_linear(sg_weight_t w, const float* const* xs, float* const* outs, int batch, int flags) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  int rc = validate_weight(w);
  if (rc) return rc;
  if (batch < 0) return fail(SG_ERR_INVALID_ARG, "negative batch");
  if (batch == 0) return SG_OK;  // forward_linear_batch with no inputs (linear.rs:184)
  if (!xs || !outs) return fail(SG_ERR_INVALID_ARG, "null xs/outs");
  for (int b = 0; b < batch; ++b)
    if (!xs[b] || !outs[b]) return fail(SG_ERR_INVALID_ARG, "null xs[%d]/outs[%d]", b, b);
  if (flags & SG_FLAG_DEVICE_PTRS) {
    if (g_ctx.devs.size() != 1) return fail(SG_ERR_INVALID_ARG, "device pointers need one device per process");
    // xs/outs are arrays of device pointers; contiguous [batch][K] layout required
    for (int b = 1; b < batch; ++b)
      if (xs[b] != xs[0] + (size_t)b * w->shards[0].w.n_cols)
        return fail(SG_ERR_INVALID_ARG, "device xs must be one contiguous [batch][n_cols] array");
    DevState& d = g_ctx.devs[0];
    const SgDevWeight* sw = &w->shards[0].w;
    const int64_t ldy = w->tp_mode == SG_TP_ROW ? w->n_rows : sw->n_rows;
    for (int b = 1; b < batch; ++b)
      if (outs[b] != outs[0] + (size_t)b * ldy)
        return fail(SG_ERR_INVALID_ARG, "device outs must be one contiguous [batch][rows] array");
    CUDA_TRY(cudaSetDevice(d.device));
    float* y0 = outs[0];
    rc = run_linear(d, &sw, 1, xs[0], sw->n_cols, &y0, &ldy, batch, d.stream, (flags & SG_FLAG_ACCUMULATE) != 0);
    if (rc) return rc;
    if (w->tp_mode == SG_TP_ROW && g_ctx.world > 1) {
      rc = allreduce_local({outs[0]}, (size_t)batch * ldy);
      if (rc) return rc;
    }
    CUDA_TRY(cudaStreamSynchronize(d.stream));
    return check_device_error(d);
  }
  return linear_host(&w, 1, xs, outs, batch, flags);
}

int sg_linear_multi(const sg_weight_t* ws, int n_weights, const float* x, float* const* outs, int flags) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  if (!ws || !x || !outs || n_weights < 1) return fail(SG_ERR_INVALID_ARG, "bad arguments");
  if (flags & SG_FLAG_DEVICE_PTRS) return fail(SG_ERR_INVALID_ARG, "use sg_linear_multi_device for device pointers");
  for (int i = 0; i < n_weights; ++i)
    if (!outs[i]) return fail(SG_ERR_INVALID_ARG, "null outs[%d]", i);
  const float* xs[1] = {x};
  // chunk into groups of SG_GEMV_MAX_MATS tensors sharing x
  for (int i0 = 0; i0 < n_weights; i0 += SG_GEMV_MAX_MATS) {
    const int n = std::min(SG_GEMV_MAX_MATS, n_weights - i0);
    int rc = linear_host(ws + i0, n, xs, outs + i0, 1, flags);
    if (rc) return rc;
  }
  return SG_OK;
}

int sg_linear_device(sg_weight_t w, const float* x, int64_t ldx, float* y, int64_t ldy, int batch, void* stream,
                     int flags) {
  const int64_t ldys[1] = {ldy};
  return sg_linear_multi_device(&w, 1, x, ldx, &y, ldys, batch, stream, flags);
}

int linear_multi_device_impl(const sg_weight_t* ws, int n_weights, const float* x, int64_t ldx, float* const* ys,
                             const int64_t* ldys, int batch, void* stream, int flags, const SgGemvPrologue* pro) {
  if (!ws || !x || !ys || !ldys || n_weights < 1 || n_weights > SG_GEMV_MAX_MATS)
    return fail(SG_ERR_INVALID_ARG, "bad arguments");
  if (g_ctx.devs.size() != 1) return fail(SG_ERR_INVALID_ARG, "device entry points need one device per process");
  if (batch < 0) return fail(SG_ERR_INVALID_ARG, "negative batch");
  if (batch == 0) return SG_OK;
  const bool acc = (flags & SG_FLAG_ACCUMULATE) != 0;
  const SgDevWeight* sw[SG_GEMV_MAX_MATS];
  for (int i = 0; i < n_weights; ++i) {
    int rc = validate_weight(ws[i]);
    if (rc) return rc;
    sw[i] = &ws[i]->shards[0].w;
    if (sw[i]->n_cols != sw[0]->n_cols || sw[i]->dtype != sw[0]->dtype || ws[i]->tp_mode != ws[0]->tp_mode)
      return fail(SG_ERR_INVALID_ARG, "multi: tensors must share dtype, n_cols and tp_mode");
    const int64_t need = ws[i]->tp_mode == SG_TP_ROW ? ws[i]->n_rows : sw[i]->n_rows;
    if (!ys[i] || ldys[i] < need) return fail(SG_ERR_INVALID_ARG, "y[%d]: ldy %lld < %lld rows", i, (long long)ldys[i], (long long)need);
  }
  if (ldx < sw[0]->n_cols) return fail(SG_ERR_INVALID_ARG, "ldx %lld < n_cols %lld", (long long)ldx, (long long)sw[0]->n_cols);
  DevState& d = g_ctx.devs[0];
  CUDA_TRY(cudaSetDevice(d.device));
  // a NULL stream is CUDA's default stream (the CUDA convention), not the
  // library's internal stream, so callers on the default stream stay ordered
  cudaStream_t st = (cudaStream_t)stream;
  if (ws[0]->tp_mode != SG_TP_ROW || g_ctx.world == 1)
    return run_linear(d, sw, n_weights, x, ldx, ys, ldys, batch, st, acc, pro);
  // Row split: every rank holds a partial sum of all n_rows outputs. They are
  // written packed ([batch][n_rows] per tensor, back to back) so that one
  // all-reduce covers the call, then copied into strided outputs if needed.
  // With SG_FLAG_ACCUMULATE rank 0 adds its partial onto y's current values
  // and the other ranks overwrite theirs, so the sum holds y once (every rank
  // passes the same y, e.g. a replicated residual stream).
  if (!g_nccl.AllReduce) return fail(SG_ERR_NCCL, "NCCL not initialised");
  const bool lead = g_ctx.rank_base == 0;
  bool packed = true;
  size_t count = 0;
  for (int i = 0; i < n_weights; ++i) {
    packed = packed && ldys[i] == ws[i]->n_rows && (i == 0 || ys[i] == ys[i - 1] + (size_t)batch * ws[i - 1]->n_rows);
    count += (size_t)batch * ws[i]->n_rows;
  }
  float* yp[SG_GEMV_MAX_MATS];
  int64_t lp[SG_GEMV_MAX_MATS];
  if (packed) {
    for (int i = 0; i < n_weights; ++i) {
      yp[i] = ys[i];
      lp[i] = ldys[i];
    }
  } else {
    int rc = ensure_buf((void**)&d.rbuf, &d.rbuf_bytes, count * sizeof(float));
    if (rc) return rc;
    size_t off = 0;
    for (int i = 0; i < n_weights; ++i) {
      yp[i] = d.rbuf + off;
      lp[i] = ws[i]->n_rows;
      off += (size_t)batch * ws[i]->n_rows;
    }
  }
  if (!packed && acc && lead)
    for (int i = 0; i < n_weights; ++i)
      CUDA_TRY(cudaMemcpy2DAsync(yp[i], (size_t)lp[i] * sizeof(float), ys[i], (size_t)ldys[i] * sizeof(float),
                                 (size_t)lp[i] * sizeof(float), batch, cudaMemcpyDeviceToDevice, st));
  int rc = run_linear(d, sw, n_weights, x, ldx, yp, lp, batch, st, acc && lead, pro);
  if (rc) return rc;
  rc = allreduce_rank(d, yp[0], count, st);
  if (rc) return rc;
  if (!packed)
    for (int i = 0; i < n_weights; ++i)
      CUDA_TRY(cudaMemcpy2DAsync(ys[i], (size_t)ldys[i] * sizeof(float), yp[i], (size_t)lp[i] * sizeof(float),
                                 (size_t)lp[i] * sizeof(float), batch, cudaMemcpyDeviceToDevice, st));
  return SG_OK;
}

int sg_linear_multi_device(const sg_weight_t* ws, int n_weights, const float* x, int64_t ldx, float* const* ys,
                           const int64_t* ldys, int batch, void* stream, int flags) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  return linear_multi_device_impl(ws, n_weights, x, ldx, ys, ldys, batch, stream, flags, nullptr);
}

int sg_rmsnorm_linear_multi_device(const sg_weight_t* ws, int n_weights, const float* x, int64_t ldx,
                                   const float* norm_weight, float eps, float* const* ys, const int64_t* ldys,
                                   int batch, void* stream, int flags) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  if (!norm_weight) return fail(SG_ERR_INVALID_ARG, "null norm weight");
  const SgGemvPrologue pro = {SG_PRO_RMSNORM, norm_weight, eps, nullptr, 0};
  return linear_multi_device_impl(ws, n_weights, x, ldx, ys, ldys, batch, stream, flags, &pro);
}

int sg_silu_mul_linear_device(sg_weight_t w, const float* g, int64_t ldg, const float* u, int64_t ldu, float* y,
                              int64_t ldy, int batch, void* stream, int flags) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  if (!u) return fail(SG_ERR_INVALID_ARG, "null pointer");
  int rc = validate_weight(w);
  if (rc) return rc;
  if (ldu < w->shards[0].w.n_cols)
    return fail(SG_ERR_INVALID_ARG, "ldu %lld < n_cols %lld", (long long)ldu, (long long)w->shards[0].w.n_cols);
  const SgGemvPrologue pro = {SG_PRO_SILU_MUL, nullptr, 0.f, u, ldu};
  const int64_t ldys[1] = {ldy};
  return linear_multi_device_impl(&w, 1, g, ldg, &y, ldys, batch, stream, flags, &pro);
}

int sg_dequant_f32(sg_weight_t w, float* dst, int flags) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  int rc = validate_weight(w);
  if (rc) return rc;
  if (!dst) return fail(SG_ERR_INVALID_ARG, "null dst");
  if (flags & SG_FLAG_DEVICE_PTRS) {
    if (g_ctx.devs.size() != 1) return fail(SG_ERR_INVALID_ARG, "device pointers need one device per process");
    DevState& d = g_ctx.devs[0];
    CUDA_TRY(cudaSetDevice(d.device));
    const SgDevWeight& s = w->shards[0].w;
    CUDA_TRY(sg_layout_dequant(&s, dst, s.n_cols, d.stream));
    CUDA_TRY(cudaStreamSynchronize(d.stream));
    return SG_OK;
  }
  for (size_t di = 0; di < w->shards.size(); ++di) {
    const Shard& sh = w->shards[di];
    if (w->tp_mode == SG_TP_REPLICATE && di > 0) break;
    DevState& d = g_ctx.devs[sh.dev_idx];
    CUDA_TRY(cudaSetDevice(d.device));
    const size_t n = (size_t)sh.w.n_rows * sh.w.n_cols;
    rc = ensure_buf((void**)&d.ybuf, &d.ybuf_bytes, n * sizeof(float));
    if (rc) return rc;
    CUDA_TRY(sg_layout_dequant(&sh.w, d.ybuf, sh.w.n_cols, d.stream));
    // place the shard into the full [n_rows][n_cols] host matrix
    CUDA_TRY(cudaMemcpy2DAsync(dst + (size_t)sh.row0 * w->n_cols + sh.col0, (size_t)w->n_cols * sizeof(float), d.ybuf,
                               (size_t)sh.w.n_cols * sizeof(float), (size_t)sh.w.n_cols * sizeof(float),
                               (size_t)sh.w.n_rows, cudaMemcpyDeviceToHost, d.stream));
    CUDA_TRY(cudaStreamSynchronize(d.stream));
  }
  return SG_OK;
}

int sg_fused_gemv_q4k(const uint8_t* w_raw, const float* x, float* out, int n_rows, int n_cols) {
  if (!w_raw || !x || !out) return fail(SG_ERR_INVALID_ARG, "null pointer");
  if (n_rows <= 0 || n_cols <= 0 || n_cols % 256) return fail(SG_ERR_INVALID_ARG, "n_cols %d not a positive multiple of 256", n_cols);
  sg_weight_t w = nullptr;
  int rc = sg_weight_register(w_raw, SG_DTYPE_Q4_K, n_rows, n_cols, SG_TP_REPLICATE, &w);
  if (rc) return rc;
  const float* xs[1] = {x};
  float* outs[1] = {out};
  rc = sg_linear(w, xs, outs, 1, 0);
  int rc2 = sg_weight_free(w);
  return rc ? rc : rc2;
}

int sg_allreduce_device(float* buf, int64_t count, void* stream) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  if (!g_ctx.inited) return fail(SG_ERR_NOT_INITIALIZED, "sg_init not called");
  if (g_ctx.devs.size() != 1) return fail(SG_ERR_INVALID_ARG, "device entry points need one device per process");
  if (count < 0 || (!buf && count)) return fail(SG_ERR_INVALID_ARG, "bad buffer");
  DevState& d = g_ctx.devs[0];
  CUDA_TRY(cudaSetDevice(d.device));
  return allreduce_rank(d, buf, (size_t)count, (cudaStream_t)stream);
}

int sg_allreduce_path(int* peer) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  if (!g_ctx.inited) return fail(SG_ERR_NOT_INITIALIZED, "sg_init not called");
  if (!peer) return fail(SG_ERR_INVALID_ARG, "null pointer");
  *peer = g_ctx.devs.size() == 1 && g_ctx.devs[0].peer_on ? 1 : 0;
  return SG_OK;
}

int sg_host_alloc(size_t bytes, void** out) {
  if (!out) return fail(SG_ERR_INVALID_ARG, "null pointer");
  *out = nullptr;
  if (bytes == 0) return SG_OK;
  if (cudaHostAlloc(out, bytes, cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();
    *out = nullptr;
    return fail(SG_ERR_OOM, "cudaHostAlloc(%zu) failed", bytes);
  }
  return SG_OK;
}

int sg_host_free(void* p) {
  if (p) CUDA_TRY(cudaFreeHost(p));
  return SG_OK;
}

int sg_synchronize(void) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  if (!g_ctx.inited) return fail(SG_ERR_NOT_INITIALIZED, "sg_init not called");
  for (auto& d : g_ctx.devs) {
    CUDA_TRY(cudaSetDevice(d.device));
    CUDA_TRY(cudaStreamSynchronize(d.stream));
    int rc = check_device_error(d);
    if (rc) return rc;
  }
  return SG_OK;
}

}  // extern "C"
