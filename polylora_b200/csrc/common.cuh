// Shared device helpers for the sm_100a kernels: inline-PTX wrappers for
// mbarriers, TMA tensor loads, programmatic dependent launch, the bounded
// waits that every pipeline wait goes through, and 16-bit float conversions.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/polylora_b200.h"

namespace plora {

// Device status word of this library (one per device context).  Kernels OR
// PLORA_DEV_* bits into it; plora_device_status() reads and clears it.
__device__ int g_device_status;

__device__ __forceinline__ void raise_status(int bits) { atomicOr(&g_device_status, bits); }

// Upper bound of any single pipeline wait.  A correct launch never waits more
// than microseconds; after this the kernel records PLORA_DEV_WAIT_TIMEOUT and
// unwinds instead of spinning forever.  1 s unless plora_set_wait_limit_ns
// changed it (tests shorten it to make a wait expire; 0 expires every wait
// that is not already complete when first polled).
constexpr uint64_t kWaitLimitNs = 1000ull * 1000ull * 1000ull;  // 1 s
__device__ uint64_t g_wait_limit_ns = kWaitLimitNs;
__device__ __forceinline__ uint64_t wait_limit_ns() {
  return *reinterpret_cast<volatile uint64_t*>(&g_wait_limit_ns);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Non-blocking test of the phase with the given parity (try_wait may suspend
// the thread for a while before reporting an incomplete phase).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Longest time one try_wait may park the calling warp (ns).  A parked warp
// issues no instructions, so waiting roles leave the issue slots to the roles
// that move data; the phase completing wakes it earlier.
constexpr uint32_t kSuspendHintNs = 100u * 1000u;

__device__ __forceinline__ bool mbar_try_wait_parked(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return done != 0;
}

// Waits until the phase with the given parity of `bar` has completed.  Gives
// up when `abort_flag` (shared) is raised by another role or after
// wait_limit_ns(); on expiry raises the device status and the abort flag.
// Returns false when the caller must unwind.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort_flag) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t limit = wait_limit_ns();
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 >= limit) {
      *abort_flag = 1;
      raise_status(PLORA_DEV_WAIT_TIMEOUT);
      return false;
    }
    if (mbar_try_wait_parked(bar, parity)) return true;
  }
}

// Bounded wait that ignores the abort flag: used to let copies already issued
// land before the CTA exits.  Its limit is the fixed 1 s, not the settable
// wait limit: a copy in flight takes microseconds, and a shortened limit must
// not let a CTA exit while one still writes its shared memory.  Returns false
// on expiry (status raised).
__device__ __forceinline__ bool mbar_drain(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait_parked(bar, parity)) return true;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      raise_status(PLORA_DEV_WAIT_TIMEOUT);
      return false;
    }
  }
}

// Warp-uniform variant: every lane polls, and the warp proceeds only if all
// lanes saw the phase complete (so the .sync.aligned ldmatrix / mma that
// follow never diverge).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity,
                                               volatile int* abort_flag) {
  const bool ok = mbar_wait(bar, parity, abort_flag);
  return __all_sync(0xffffffffu, ok);
}

// Named barrier over `count` threads (id 1..15; id 0 is __syncthreads).
__device__ __forceinline__ void named_barrier(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// Counts the calling warp in at the named barrier without waiting for it.
__device__ __forceinline__ void named_barrier_arrive(int id, int count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Orders this thread's generic-proxy shared-memory accesses before its later
// async-proxy (TMA) operations on the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialisation may start before its predecessor in the stream has finished;
// griddep_wait() returns once that predecessor grid has completed and its
// memory is visible (at once for an ordinary launch).  griddep_launch()
// lets the next such kernel start as SMs free up.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Coherent (L2) loads for data that the grid before this one in the stream
// writes.  A programmatically launched kernel may start while that grid still
// runs; __ldg (a read-only load) may be scheduled above griddep_wait() and
// then read stale data, while these volatile loads stay after it.
__device__ __forceinline__ uint32_t ld_cg_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ int32_t ld_cg_i32(const int32_t* p) { return (int32_t)ld_cg_u32(p); }
__device__ __forceinline__ int64_t ld_cg_i64(const int64_t* p) {
  int64_t v;
  asm volatile("ld.global.cg.s64 %0, [%1];" : "=l"(v) : "l"(p));
  return v;
}
// The same ordering, cached in L1 as well: for data read by several warps of
// the CTA after griddep_wait() (the previous grid has completed by then).
__device__ __forceinline__ uint32_t ld_ca_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.ca.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// 4-D tiled TMA load (box starting at (0, 0, c2, c3)), completing on `bar`.
__device__ __forceinline__ void tma_load_4d_outer(uint32_t dst, const void* tmap, uint64_t* bar,
                                                  int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %3, %4, %5}], [%2];" ::"r"(dst),
      "l"(tmap), "r"(smem_u32(bar)), "r"(0), "r"(c2), "r"(c3)
      : "memory");
}

// 5-D tiled TMA load (box starting at (0, 0, 0, 0, c4)), completing on `bar`.
__device__ __forceinline__ void tma_load_5d_outer(uint32_t dst, const void* tmap, uint64_t* bar,
                                                  int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %3, %3, %3, %4}], [%2];" ::"r"(dst),
      "l"(tmap), "r"(smem_u32(bar)), "r"(0), "r"(c4)
      : "memory");
}

// ---------------------------------------------------------------- numerics
template <bool BF16>
struct Elem;
template <>
struct Elem<true> {
  using T = __nv_bfloat16;
  __device__ static __forceinline__ float to_f(uint16_t v) {
    return __uint_as_float(((uint32_t)v) << 16);
  }
  __device__ static __forceinline__ uint16_t from_f(float f) {
    __nv_bfloat16 h = __float2bfloat16_rn(f);
    return *reinterpret_cast<uint16_t*>(&h);
  }
};
template <>
struct Elem<false> {
  using T = __half;
  __device__ static __forceinline__ float to_f(uint16_t v) {
    __half h = *reinterpret_cast<__half*>(&v);
    return __half2float(h);
  }
  __device__ static __forceinline__ uint16_t from_f(float f) {
    __half h = __float2half_rn(f);
    return *reinterpret_cast<uint16_t*>(&h);
  }
};

// ---------------------------------------------------------------- segments
// Index of the slot whose token range [ss[s], ss[s+1]) contains position p
// (largest s with ss[s] <= p; ss is non-decreasing, ss[0] = 0).
__device__ __forceinline__ int slot_of_position(const int32_t* ss, int num_slots, int64_t p) {
  int lo = 0, hi = num_slots - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if ((int64_t)ss[mid] <= p)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

}  // namespace plora
