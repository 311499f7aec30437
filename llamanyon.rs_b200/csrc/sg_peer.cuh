// sg_peer.cuh -- sum all-reduce of a row-split linear's outputs over NVLink
// peer memory, for one process per GPU.
//
// After a row-split (K-split) GEMV every rank holds a partial sum of all
// outputs; the reference design follows each such GEMV with an
// ncclAllReduce. Decode outputs are small (4096 x batch floats), where a
// collective library's launch and protocol latency dominates. This kernel
// does the exchange itself:
//
//   CTA c owns chunk c of the vector (kArChunk floats). It stores its chunk of
//   this rank's partial into slot [parity][rank] of every peer's receive
//   buffer (plain stores through CUDA IPC mappings, over NVLink), fences at
//   system scope and sets flag [parity][rank][c] = epoch in every peer. It
//   then waits (bounded) until every peer's flag [parity][peer][c] in its own
//   memory reaches the epoch and sums the slots in rank order, so every rank
//   computes the same float sum.
//
// Epochs: CTA c keeps a counter in this rank's memory; each call uses
// counter + 1 and stores it at the end, so the kernel needs no host argument
// that changes between calls and can be captured in a CUDA graph. All ranks
// make the same calls, so their counters stay equal. Slots and flags are
// double-buffered by the epoch's parity: a rank writes slot parity p for
// epoch e + 2 only after it saw every peer's chunk-c flag for epoch e + 1,
// which a peer sets only after its call for epoch e has completed, reads of
// slot p included.
#pragma once
#include "sg_common.cuh"

#define SG_PEER_MAX 8
constexpr int kArChunk = 2048;      // floats per CTA
constexpr int kArMaxChunks = 512;   // -> at most 1 Mi floats per call
constexpr int kArThreads = 256;

struct SgPeerPtrs {
  float* buf[SG_PEER_MAX];       // each rank's receive buffer: [2][world][cap]
  uint32_t* flags[SG_PEER_MAX];  // each rank's flags: [2][world][kArMaxChunks]
};

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// dst[i] = sum over ranks of src[i], i < count (dst may equal src).
__global__ void __launch_bounds__(kArThreads) peer_allreduce_kernel(const float* src, float* dst, int64_t count,
                                                                  int world, int rank, SgPeerPtrs pp,
                                                                  uint32_t* ctr, int64_t cap) {
  __shared__ uint32_t e_sh;
  pdl_launch_dependents();
  pdl_wait();  // src comes from the previous kernel
  const int c = blockIdx.x, tid = threadIdx.x;
  if (tid == 0) e_sh = ctr[c] + 1;
  __syncthreads();
  const uint32_t e = e_sh, par = e & 1u;
  const int64_t i0 = (int64_t)c * kArChunk, n = (count - i0 < kArChunk) ? count - i0 : (int64_t)kArChunk;
  const bool vec = ((count & 3) == 0) && (((uintptr_t)src & 15) == 0);
  // 1. this rank's chunk into slot [par][rank] of every peer (the peers in
  // an order that starts after this rank, so the ranks' stores spread over
  // the links)
  for (int j = 1; j < world; ++j) {
    const int p = (rank + j) % world;
    float* slot = pp.buf[p] + ((int64_t)par * world + rank) * cap + i0;
    if (vec) {
      for (int64_t i = 4 * tid; i < n; i += 4 * kArThreads)
        *reinterpret_cast<float4*>(slot + i) = *reinterpret_cast<const float4*>(src + i0 + i);
    } else {
      for (int64_t i = tid; i < n; i += kArThreads) slot[i] = src[i0 + i];
    }
  }
  // one system-scope fence after the CTA barrier orders every thread's
  // stores (the barrier makes them visible to thread 0) before the flags
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    for (int j = 1; j < world; ++j) {
      const int p = (rank + j) % world;
      *(volatile uint32_t*)(pp.flags[p] + ((int64_t)par * world + rank) * kArMaxChunks + c) = e;
    }
  }
  // 2. wait for every peer's chunk (one thread per peer polls its flag in
  // this rank's own memory, bounded)
  if (tid < world && tid != rank) {
    const uint32_t* f = pp.flags[rank] + ((int64_t)par * world + tid) * kArMaxChunks + c;
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys_u32(f) != e) {
      if (globaltimer_ns() - t0 > g_sg_wait_ns) {
        sg_set_error(SG_DEVERR_WAIT_TIMEOUT | 0x50);
        break;
      }
    }
  }
  __syncthreads();
  // 3. sum in rank order (the same float sum on every rank)
  const float* mine = pp.buf[rank] + (int64_t)par * world * cap + i0;
  for (int64_t i = tid; i < n; i += kArThreads) {
    float v = 0.f;
    for (int p = 0; p < world; ++p) v += p == rank ? src[i0 + i] : __ldcg(mine + (int64_t)p * cap + i);
    dst[i0 + i] = v;
  }
  if (tid == 0) ctr[c] = e;  // advance even after a timeout: the error is reported, epochs stay in step
}
