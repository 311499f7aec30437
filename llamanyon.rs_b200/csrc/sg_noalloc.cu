// sg_noalloc.cu -- sg_linear_device_noalloc: the decode GEMV (batch 1..16,
// device pointers) for callers that must never trigger a device allocation.
//
// The decode GEMV's workspace (the call's activations converted to the MMA
// operand layout, rewritten by every call) is the library's fixed per-device
// array (g_gemv_ws in sg_api.cu), sized for n_cols <= kStaticWsCols at 16
// tokens (more at fewer tokens), so a call only launches kernels. A row-split
// tensor's all-reduce is the peer kernel over the receive buffers that
// sg_init_rank mapped (vectors up to 512 Ki floats) or, with that kernel off
// or for longer vectors, ncclAllReduce. The workspace's address is looked up
// once per device on the first call that uses the device. The workspace is shared by all
// decode calls on a device, so two calls whose kernels overlap in time
// (different streams, no ordering between them) race on it.
constexpr int kNoallocMaxBatch = 16;

int sg_linear_device_noalloc(sg_weight_t w, const float* x, int64_t ldx, float* y, int64_t ldy, int batch,
                             void* stream, int flags) {
  std::lock_guard<std::mutex> lk(g_ctx.mu);
  int rc = validate_weight(w);
  if (rc) return rc;
  if (!x || !y) return fail(SG_ERR_INVALID_ARG, "null pointer");
  if (g_ctx.devs.size() != 1) return fail(SG_ERR_INVALID_ARG, "device entry points need one device per process");
  if (batch < 1 || batch > kNoallocMaxBatch)
    return fail(SG_ERR_UNSUPPORTED, "sg_linear_device_noalloc: batch %d outside the range 1..%d of the fixed workspace",
                batch, kNoallocMaxBatch);
  const SgDevWeight* sw = &w->shards[0].w;
  if (sw->dtype != SG_DTYPE_Q6_K && sg_gemv_scratch_bytes(sw->n_cols, batch) > kStaticWsBytes) {
    const long long limit = (long long)(kStaticWsBytes / sg_gemv_scratch_bytes(256, batch)) * 256;
    return fail(SG_ERR_UNSUPPORTED, "sg_linear_device_noalloc: n_cols %lld above %lld at batch %d (the fixed workspace)",
                (long long)sw->n_cols, limit, batch);
  }
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
  void* ws = nullptr;
  CUDA_TRY(static_workspace(d.device, &ws));
  cudaStream_t st = (cudaStream_t)stream;
  if (sw->dtype == SG_DTYPE_Q6_K) {  // no workspace: zeroes y and reduces K ranges in place
    CUDA_TRY(sg_gemv_q6k(sw, x, ldx, y, ldy, batch, acc, d.num_sms, st));
  } else {
    SgGemvMat m = {sw, y, ldy};
    CUDA_TRY(sg_gemv(&m, 1, x, ldx, batch, acc, ws, kStaticWsBytes, d.num_sms, st));
  }
  // the peer all-reduce kernel (receive buffers mapped by sg_init_rank) for
  // vectors within its slot, else ncclAllReduce
  return row_split ? allreduce_rank(d, y, (size_t)batch * w->n_rows, st) : SG_OK;
}
