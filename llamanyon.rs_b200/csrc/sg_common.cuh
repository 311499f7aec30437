// sg_common.cuh -- shared device helpers for the swamp-gpu B200 kernels.
//
// Every spin-wait in these kernels is bounded: after g_sg_wait_ns of wall time
// (%globaltimer) the waiting thread records an error code in the per-device
// flag g_sg_error and returns false, and the caller abandons its loop. The
// host reads the flag after a call (SG_ERR_DEVICE_FAULT) instead of the GPU
// hanging.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define SG_DTYPE_Q4_0 2
#define SG_DTYPE_Q4_K 12
#define SG_DTYPE_Q6_K 14

// Device layout geometry (see sg_layout.cuh).
#define SG_RB_ROWS 128   // rows per row-block
#define SG_RT_ROWS 16    // rows per row-tile (mma M)
#define SG_CHUNK_K 64    // K elements per chunk
#define SG_CHUNK_QS 4096 // nibble bytes per (row-block, chunk)
#define SG_CHUNK_SC 512  // scale bytes per (row-block, chunk) (Q4_0 d / Q4_K scm)
#define SG_SB_DD 512     // Q4_K d|dmin bytes per (row-block, super-block)

// Error codes written to g_sg_error.
#define SG_DEVERR_WAIT_TIMEOUT 0x100
#define SG_DEVERR_BAD_ARGS 0x200

// The library is built as one translation unit (swamp_gpu.cu), so this is the
// single definition of the per-device error flag.
__device__ int g_sg_error = 0;

__device__ __forceinline__ void sg_set_error(int code) { atomicCAS(&g_sg_error, 0, code); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

// try_wait with a suspend-time hint: a waiting thread sleeps (it does not
// spin and issue) until the phase completes or the hint expires.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// non-blocking test of a phase (no suspend)
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: returns false (and records SG_DEVERR_WAIT_TIMEOUT | tag) if the
// phase with the given parity has not completed after SG_WAIT_NS nanoseconds
// of wall time (or after another thread already recorded an error).
//
// The poll loop touches nothing but the barrier and the SM's cycle counter:
// the global error flag and the wall clock are read only once a wait has
// lasted SG_WAIT_QUIET_CYCLES. A global load in the loop would take a
// microsecond while HBM is saturated by the weight stream, and a barrier
// that completes meanwhile would go unnoticed for that long.
#ifndef SG_WAIT_NS
#define SG_WAIT_NS 4000000000ull
#endif
// The limit in force, per device: SG_WAIT_NS unless the host set another one
// at initialisation (SG_WAIT_NS in the environment of sg_init / sg_init_rank).
__device__ unsigned long long g_sg_wait_ns = SG_WAIT_NS;
#ifndef SG_WAIT_QUIET_CYCLES
#define SG_WAIT_QUIET_CYCLES (1ll << 17)
#endif
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int tag) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long c0 = clock64();
  uint64_t t0 = 0;
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - c0 > SG_WAIT_QUIET_CYCLES) {  // a long wait: watch the error flag and the wall clock
      if (t0 == 0) t0 = globaltimer_ns();
      if (*(volatile int*)&g_sg_error != 0) return false;
      if (globaltimer_ns() - t0 > g_sg_wait_ns) break;
    }
  }
  sg_set_error(SG_DEVERR_WAIT_TIMEOUT | tag);
  return false;
}

// Drain wait used on the error path: waits (bounded, ignoring the error flag)
// for a phase whose asynchronous copies or MMAs are still in flight, so that
// none of them lands after the CTA has released its shared memory or TMEM.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > g_sg_wait_ns) return false;
  }
}

// ------------------------------------------------------------ bulk copies
// 1-D bulk async copy global -> shared, completion counted on an mbarrier.
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void bulk_g2s_evict_first(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                                     uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Per-thread asynchronous copies global -> shared (LSU path, no TMA unit).
// src_bytes < bytes zero-fills the rest (0 = all zeros, src not read).
__device__ __forceinline__ void cp_async16(void* dst_smem, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst_smem)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst_smem, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// wait until at most N of this thread's committed groups are still in flight
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 2-D tiled TMA load into this CTA only, completion on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void* dst_smem, const CUtensorMap* map, int c0, int c1,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst_smem)),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// 4-D tiled TMA load into this CTA only, completion on an mbarrier.
__device__ __forceinline__ void tma_load_4d(void* dst_smem, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];" ::"r"(smem_u32(dst_smem)),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Generic-proxy shared-memory writes -> visible to the async proxy (tensor core).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------ programmatic dependent launch
// Host switch: SG_PDL=0 in the environment launches every kernel without the
// programmatic-serialization attribute (plain stream order).
#include <cstdlib>
inline bool sg_pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("SG_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------------ misc
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));  // (a & b) | c
  return r;
}

// 64-bit flag store with release semantics at GPU scope, and a relaxed
// (volatile) load of it; pair the load with __threadfence() to acquire.
__device__ __forceinline__ void st_release_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_add_f32(float* addr, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, %1;\n\t"
      "selp.b32 %0, 1, 0, P;\n\t}"
      : "=r"(pred)
      : "r"(0xffffffffu));
  return pred != 0;
}
