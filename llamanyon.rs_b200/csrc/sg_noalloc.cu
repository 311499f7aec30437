// sg_noalloc.cu -- sg_linear_device_noalloc: the decode GEMV (batch 1..16,
// device pointers) with its activation scratch in a fixed device array, so a
// call allocates no memory.
//
// The scratch is this file's static __device__ array below, sized for
// n_cols <= SG_NOALLOC_MAX_COLS. Its address is looked up once per device
// (cudaGetSymbolAddress, with that device current) on the first call that
// uses the device; later calls only launch kernels. Nothing in the array has
// to start at zero: every byte the kernels read is written earlier in the
// same call. The array is shared by all calls on a device, so two calls whose
// kernels overlap in time (different streams, no ordering between them) race
// on it.
#include <mutex>

#define SG_NOALLOC_MAX_COLS 16384

namespace noalloc {

constexpr size_t kUnits = (((size_t)SG_NOALLOC_MAX_COLS + 63) / 64 + gemv_tc::kUC - 1) / gemv_tc::kUC;
constexpr size_t kBytes = ((kUnits * gemv_tc::Cfg<16>::XU + 1023) / 1024) * 1024 + 1024;  // = sg_gemv_scratch_bytes

static __device__ __align__(256) uint8_t g_scratch[kBytes];

std::mutex g_mu;
void* g_ptr[64] = {nullptr};

// address of this device's scratch array (one lookup per device)
cudaError_t scratch_ptr(int device, void** out) {
  if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_ptr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) return e;
    g_ptr[device] = p;
  }
  *out = g_ptr[device];
  return cudaSuccess;
}

}  // namespace noalloc

int sg_linear_device_noalloc(sg_weight_t w, const float* x, int64_t ldx, float* y, int64_t ldy, int batch,
                             void* stream, int flags) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  int rc = validate_weight(w);
  if (rc) return rc;
  if (!x || !y) return fail(SG_ERR_INVALID_ARG, "null pointer");
  if (g_ctx.devs.size() != 1) return fail(SG_ERR_INVALID_ARG, "device entry points need one device per process");
  if (batch < 1 || batch > SG_GEMV_MAX_BATCH)
    return fail(SG_ERR_UNSUPPORTED, "sg_linear_device_noalloc: batch %d outside 1..%d", batch, SG_GEMV_MAX_BATCH);
  const SgDevWeight* sw = &w->shards[0].w;
  if (sw->n_cols > SG_NOALLOC_MAX_COLS)
    return fail(SG_ERR_UNSUPPORTED, "sg_linear_device_noalloc: n_cols %lld above the fixed scratch limit %d",
                (long long)sw->n_cols, SG_NOALLOC_MAX_COLS);
  if (sg_gemv_scratch_bytes(sw->n_cols) > noalloc::kBytes)
    return fail(SG_ERR_UNSUPPORTED, "sg_linear_device_noalloc: scratch %zu bytes above the fixed %zu",
                sg_gemv_scratch_bytes(sw->n_cols), noalloc::kBytes);
  const bool acc = (flags & SG_FLAG_ACCUMULATE) != 0;
  const bool row_split = w->tp_mode == SG_TP_ROW && g_ctx.world > 1;
  const int64_t need = w->tp_mode == SG_TP_ROW ? w->n_rows : sw->n_rows;
  if (ldy < need) return fail(SG_ERR_INVALID_ARG, "ldy %lld < %lld rows", (long long)ldy, (long long)need);
  if (ldx < sw->n_cols) return fail(SG_ERR_INVALID_ARG, "ldx %lld < n_cols %lld", (long long)ldx, (long long)sw->n_cols);
  if (row_split && (acc || ldy != w->n_rows))
    return fail(SG_ERR_UNSUPPORTED, "sg_linear_device_noalloc: a row-split tensor needs ldy == n_rows and no "
                                    "SG_FLAG_ACCUMULATE (its all-reduce runs in place)");
  if (((uintptr_t)x & 15) || (ldx & 3))
    return fail(SG_ERR_INVALID_ARG, "x must be 16-byte aligned with a row stride that is a multiple of 4 floats");
  DevState& d = g_ctx.devs[0];
  CUDA_TRY(cudaSetDevice(d.device));
  void* scratch = nullptr;
  CUDA_TRY(noalloc::scratch_ptr(d.device, &scratch));
  cudaStream_t st = (cudaStream_t)stream;
  SgGemvMat m = {sw, y, ldy};
  CUDA_TRY(sg_gemv(&m, 1, x, ldx, batch, acc, scratch, noalloc::kBytes, d.num_sms, st));
  if (row_split) {
    if (!g_nccl.AllReduce) return fail(SG_ERR_NCCL, "NCCL not initialised");
    const ncclResult_t r = g_nccl.AllReduce(y, y, (size_t)batch * w->n_rows, kNcclFloat, kNcclSum, d.comm, st);
    if (r) return fail(SG_ERR_NCCL, "ncclAllReduce: %s", g_nccl.GetErrorString(r));
  }
  return SG_OK;
}
