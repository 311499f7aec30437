// sg_peer.cuh -- sum all-reduce of a row-split linear's outputs over NVLink
// peer memory, for one process per GPU.
//
// After a row-split (K-split) GEMV every rank holds a partial sum of all
// outputs; the reference design follows each such GEMV with an
// ncclAllReduce. Decode outputs are small (4096 x batch floats), where a
// collective library's launch and protocol latency dominates. This kernel
// does the exchange itself, with no fence and no separate flag:
//
//   CTA c owns chunk c of the vector (kArChunk floats). Every value travels
//   with the call's epoch in the same 8-byte word (value bits, epoch): a
//   thread stores its pairs of values of this rank's partial as 16-byte
//   words {v0, e, v1, e} into slot [parity][rank] of every peer's receive
//   buffer (plain stores through CUDA IPC mappings, over NVLink). An aligned
//   8-byte store is seen whole or not at all, so a reader that finds the
//   epoch beside a value has the value. The same thread then reads its pairs
//   from every peer's slot in this rank's own memory, polling (bounded) until
//   both epochs match, and sums the ranks in rank order, so every rank
//   computes the same float sum. (A system-scope fence between the data and
//   a flag, or a release store of the flag, cost about 4 us per call.)
//
// Epochs: CTA c keeps a counter in this rank's memory; each call uses
// counter + 1 and stores it at the end, so the kernel needs no host argument
// that changes between calls and can be captured in a CUDA graph. All ranks
// make the same calls, so their counters stay equal. Slots are
// double-buffered by the epoch's parity: a rank writes slot parity p for
// epoch e + 2 only after it read every peer's chunk-c values of epoch e + 1,
// which a peer writes only after its call for epoch e has completed, reads of
// slot p included.
#pragma once
#include "sg_common.cuh"

#define SG_PEER_MAX 8
constexpr int kArChunk = 2048;      // floats per CTA
constexpr int kArMaxChunks = 256;   // -> at most 512 Ki floats per call (larger ones go to NCCL)
constexpr int kArThreads = 256;
constexpr int kArPairs = kArChunk / 2 / kArThreads;  // value pairs per thread

struct SgPeerPtrs {
  uint4* buf[SG_PEER_MAX];  // each rank's receive buffer: [2][world][cap / 2] of {v0, e, v1, e}
};

__device__ __forceinline__ void st_volatile_v4(uint4* p, uint4 v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_volatile_v4(const uint4* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
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
  const int64_t half = cap / 2;  // 16-byte words per slot
  // this thread's value pairs j = tid + k * kArThreads: elements i0 + 2j, i0 + 2j + 1
  float2 own[kArPairs];
#pragma unroll
  for (int k = 0; k < kArPairs; ++k) {
    const int64_t i = 2 * (int64_t)(tid + k * kArThreads);
    own[k] = make_float2(i < n ? src[i0 + i] : 0.f, i + 1 < n ? src[i0 + i + 1] : 0.f);
  }
  // 1. push: this rank's pairs into slot [par][rank] of every peer (the peers
  // in an order that starts after this rank, so the ranks' stores spread
  // over the links)
  for (int j = 1; j < world; ++j) {
    const int p = (rank + j) % world;
    uint4* slot = pp.buf[p] + ((int64_t)par * world + rank) * half + i0 / 2;
#pragma unroll
    for (int k = 0; k < kArPairs; ++k) {
      const int64_t w = tid + k * kArThreads;
      if (2 * w < n) st_volatile_v4(slot + w, make_uint4(__float_as_uint(own[k].x), e, __float_as_uint(own[k].y), e));
    }
  }
  // 2. pull: every peer's pairs from this rank's own buffer, each word
  // polled until it carries the epoch (bounded), summed in rank order
  const uint4* mine = pp.buf[rank] + (int64_t)par * world * half + i0 / 2;
  float2 sum[kArPairs];
#pragma unroll
  for (int k = 0; k < kArPairs; ++k) sum[k] = make_float2(0.f, 0.f);
  bool timed_out = false;
  for (int p = 0; p < world; ++p) {
#pragma unroll
    for (int k = 0; k < kArPairs; ++k) {
      const int64_t w = tid + k * kArThreads;
      if (2 * w >= n) continue;
      float2 v = own[k];
      if (p != rank) {
        const uint4* q = mine + (int64_t)p * half + w;
        uint4 u = ld_volatile_v4(q);
        if ((u.y != e || u.w != e) && !timed_out) {
          const uint64_t t0 = globaltimer_ns();
          do {
            u = ld_volatile_v4(q);
            if (globaltimer_ns() - t0 > g_sg_wait_ns) {
              sg_set_error(SG_DEVERR_WAIT_TIMEOUT | 0x50);
              timed_out = true;  // the sum is wrong; the error is reported and later waits are skipped
              break;
            }
          } while (u.y != e || u.w != e);
        }
        v = make_float2(__uint_as_float(u.x), __uint_as_float(u.z));
      }
      sum[k].x += v.x;
      sum[k].y += v.y;
    }
  }
#pragma unroll
  for (int k = 0; k < kArPairs; ++k) {
    const int64_t i = 2 * (int64_t)(tid + k * kArThreads);
    if (i < n) dst[i0 + i] = sum[k].x;
    if (i + 1 < n) dst[i0 + i + 1] = sum[k].y;
  }
  __syncthreads();               // every thread has used e_sh
  if (tid == 0) ctr[c] = e;      // advance even after a timeout: the error is reported, epochs stay in step
}
