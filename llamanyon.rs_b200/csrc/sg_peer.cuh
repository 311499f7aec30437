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
  uint4* buf[SG_PEER_MAX];   // each rank's receive buffer: [2][world][cap / 2] of {v0, e, v1, e}
  uint4* buf2[SG_PEER_MAX];  // each rank's two-shot slots: [2 parities][2 phases][world][cap2 / 2]
};

// Two-shot variant (reduce-scatter, then all-gather) for large vectors on
// many ranks, where the one-shot push sends each rank's whole vector to every
// peer: the vector is cut into `world` parts; CTA c owns offset c * kAr2Chunk
// of every part. Phase 1: this rank's slice of part j goes to rank j's
// phase-1 slot [rank]; rank j sums its part's slices in rank order. Phase 2:
// the sum goes to every rank's phase-2 slot [j], and every rank copies the
// parts out. Each rank sends 2 (world - 1) / world of the vector instead of
// (world - 1) times it. Values travel beside the epoch as in the one-shot
// kernel; slots alternate by parity with the same argument (a rank writes a
// parity-p slot for epoch e + 2 only after its call e + 1 completed, which
// needed every peer's phase-2 values of e + 1, which a peer sends only after
// its call e, reads included, completed).
constexpr int kAr2Chunk = 512;     // floats per CTA within a part
constexpr int kAr2Threads = 128;   // two value pairs per thread
constexpr int kAr2Pairs = kAr2Chunk / 2 / kAr2Threads;

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

__device__ __forceinline__ uint4 ll_pair(float2 v, uint32_t e) {
  return make_uint4(__float_as_uint(v.x), e, __float_as_uint(v.y), e);
}

// polls one {v0, e, v1, e} word until both epochs are e (bounded); on a timeout
// records the error and returns what it has
__device__ __forceinline__ float2 ll_wait(const uint4* q, uint32_t e, bool& timed_out) {
  uint4 u = ld_volatile_v4(q);
  if ((u.y != e || u.w != e) && !timed_out) {
    const uint64_t t0 = globaltimer_ns();
    do {
      u = ld_volatile_v4(q);
      if (globaltimer_ns() - t0 > g_sg_wait_ns) {
        sg_set_error(SG_DEVERR_WAIT_TIMEOUT | 0x51);
        timed_out = true;
        break;
      }
    } while (u.y != e || u.w != e);
  }
  return make_float2(__uint_as_float(u.x), __uint_as_float(u.z));
}

// dst[i] = sum over ranks of src[i], i < count (dst may equal src), two-shot.
// part: floats per part (count / world rounded up to even); cap2: the slot
// capacity in floats (>= part).
__global__ void __launch_bounds__(kAr2Threads) peer_allreduce2_kernel(const float* src, float* dst, int64_t count,
                                                                    int world, int rank, SgPeerPtrs pp,
                                                                    uint32_t* ctr, int64_t part, int64_t cap2) {
  __shared__ uint32_t e_sh;
  pdl_launch_dependents();
  pdl_wait();  // src comes from the previous kernel
  const int c = blockIdx.x, tid = threadIdx.x;
  if (tid == 0) e_sh = ctr[c] + 1;
  __syncthreads();
  const uint32_t e = e_sh, par = e & 1u;
  const int64_t o = (int64_t)c * kAr2Chunk;  // offset within a part
  const int64_t h2 = cap2 / 2;               // words per (parity, phase, rank) slot
  auto slot = [&](int owner, int phase, int from) -> uint4* {
    return pp.buf2[owner] + (((int64_t)par * 2 + phase) * world + from) * h2 + o / 2;
  };
  auto val = [&](int64_t i) -> float { return i < count ? src[i] : 0.f; };
  // pairs w = tid + k * kAr2Threads, elements o + 2w, o + 2w + 1 of a part
  bool timed_out = false;
  // phase 1: this rank's slice of every part j to rank j (own part kept)
  float2 own[kAr2Pairs];
  for (int jj = 0; jj < world; ++jj) {
    const int j = (rank + jj) % world;
    const int64_t base = (int64_t)j * part + o;
#pragma unroll
    for (int k = 0; k < kAr2Pairs; ++k) {
      const int64_t w = tid + k * kAr2Threads;
      if (o + 2 * w >= part) continue;
      const float2 v = make_float2(val(base + 2 * w), val(base + 2 * w + 1));
      if (j == rank) own[k] = v;
      else st_volatile_v4(slot(j, 0, rank) + w, ll_pair(v, e));
    }
  }
  // this rank's part: every rank's slice, summed in rank order; then to every rank
  float2 sum[kAr2Pairs];
#pragma unroll
  for (int k = 0; k < kAr2Pairs; ++k) sum[k] = make_float2(0.f, 0.f);
  for (int q = 0; q < world; ++q) {
#pragma unroll
    for (int k = 0; k < kAr2Pairs; ++k) {
      const int64_t w = tid + k * kAr2Threads;
      if (o + 2 * w >= part) continue;
      const float2 v = q == rank ? own[k] : ll_wait(slot(rank, 0, q) + w, e, timed_out);
      sum[k].x += v.x;
      sum[k].y += v.y;
    }
  }
  const int64_t mine = (int64_t)rank * part + o;
#pragma unroll
  for (int k = 0; k < kAr2Pairs; ++k) {
    const int64_t w = tid + k * kAr2Threads;
    if (o + 2 * w >= part) continue;
    for (int jj = 1; jj < world; ++jj) st_volatile_v4(slot((rank + jj) % world, 1, rank) + w, ll_pair(sum[k], e));
    const int64_t i = mine + 2 * w;
    if (i < count) dst[i] = sum[k].x;
    if (i + 1 < count) dst[i + 1] = sum[k].y;
  }
  // phase 2: the other parts' sums from their owners
  for (int jj = 1; jj < world; ++jj) {
    const int q = (rank + jj) % world;
#pragma unroll
    for (int k = 0; k < kAr2Pairs; ++k) {
      const int64_t w = tid + k * kAr2Threads;
      if (o + 2 * w >= part) continue;
      const float2 v = ll_wait(slot(rank, 1, q) + w, e, timed_out);
      const int64_t i = (int64_t)q * part + o + 2 * w;
      if (i < count) dst[i] = v.x;
      if (i + 1 < count) dst[i + 1] = v.y;
    }
  }
  __syncthreads();           // every thread has used e_sh
  if (tid == 0) ctr[c] = e;  // advance even after a timeout: the error is reported, epochs stay in step
}
