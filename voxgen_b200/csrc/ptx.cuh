// Inline-PTX helpers for sm_100a: mbarriers, bulk async copies (TMA engine,
// non-tensor, no multicast), programmatic dependent launch, L2 prefetch.
//
// Every wait here is bounded: it gives up after a wall-clock limit read from
// %globaltimer (and an iteration cap as a backstop) and returns false, so a
// kernel can record an error in its device flag and leave instead of hanging.
//
// A wait may be given the error word of a control block as its abort flag: it
// then gives up as soon as that word is nonzero, and the word after it holds
// the wall-clock limit in nanoseconds (0 = kWaitLimitNs), so a host can
// shorten every wait of a stream at run time.
#pragma once
#include <cstdint>

namespace vg {

// Limits of every bounded device-side wait.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
constexpr uint32_t kWaitMaxIters = 1u << 26;

// Device error flag bits (ctrl[kCtrlErr]).
enum : uint32_t {
  kErrConsumerWait = 1u,   // a warp gave up waiting for its bulk copy or a peer warp
  kErrDrainWait = 4u,      // bulk copies still in flight at kernel exit
  kErrBadToken = 8u,       // token id outside the vocabulary
  kErrPosition = 16u,      // position outside the KV cache
  kErrGridWait = 32u,      // a CTA gave up waiting at a grid barrier
  kErrPlan = 64u,          // launch parameters the kernel was not built for
};

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

// Wall-clock limit of a wait whose abort flag is a control block's error word
// (the limit is the next word; 0 or no flag: kWaitLimitNs). Read once, when a
// wait first fails its fast check.
__device__ __forceinline__ uint64_t wait_limit(const uint32_t *abort_flag) {
  const uint32_t ns = abort_flag ? ld_volatile_u32(abort_flag + 1) : 0u;
  return ns ? (uint64_t)ns : kWaitLimitNs;
}

// Waits for the phase with the given parity to complete; false on timeout, or
// as soon as *abort_flag (when given) is nonzero.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  const uint32_t *abort_flag = nullptr) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer(), lim = wait_limit(abort_flag);
  for (uint32_t it = 0; it < kWaitMaxIters; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 255u) {
      if (globaltimer() - t0 > lim) return false;
      if (abort_flag && ld_volatile_u32(abort_flag)) return false;
    }
  }
  return false;
}

// The same wait with a short sleep between polls, for a thread that is not on
// the critical path (the producer waiting for a free ring slot): it then
// leaves the issue slots of its SM sub-partition to the consumer warps.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t *bar, uint32_t parity,
                                                  const uint32_t *abort_flag = nullptr) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer(), lim = wait_limit(abort_flag);
  for (uint32_t it = 0; it < kWaitMaxIters; ++it) {
    __nanosleep(128);
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15u) == 15u) {
      if (globaltimer() - t0 > lim) return false;
      if (abort_flag && ld_volatile_u32(abort_flag)) return false;
    }
  }
  return false;
}

// Grid-wide barrier over a monotonically increasing 64-bit arrival counter:
// grid_arrive adds one arrival with release semantics at GPU scope (the
// caller first synchronises the arriving threads of its CTA); grid_wait spins
// (bounded, acquire) until the counter reaches target. Both are called by one
// thread per CTA; all CTAs of the grid must be resident (cooperative launch).
__device__ __forceinline__ void grid_arrive(unsigned long long *ctr) {
  asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(ctr) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool grid_wait(const unsigned long long *ctr, unsigned long long target,
                                          const uint32_t *abort_flag) {
  if (ld_acquire_u64(ctr) >= target) return true;
  const uint64_t t0 = globaltimer(), lim = wait_limit(abort_flag);
  for (uint32_t it = 0; it < kWaitMaxIters; ++it) {
    if (ld_acquire_u64(ctr) >= target) return true;
    if ((it & 63u) == 63u) {
      if (globaltimer() - t0 > lim) return false;
      if (abort_flag && ld_volatile_u32(abort_flag)) return false;
    }
  }
  return false;
}

// Orders this thread's earlier generic-proxy accesses (an acquire of other
// CTAs' writes included) before its later async-proxy ones (bulk copies).
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Bulk copy global -> shared (cp.async.bulk, TMA engine, no tensor map, no
// multicast). dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// The same copy with an L2 evict-first policy, for data read once per step
// (weights, cached K/V rows): it leaves L2 to the partial sums and vectors
// that other CTAs read back within the step. The batched step kernel streams
// with it (its split-K and attention partials otherwise stay dirty in L2 until
// the weight stream evicts them to DRAM); the single-stream kernel, whose
// partials are few, measured no gain from it.
__device__ __forceinline__ void bulk_g2s_stream(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .b64 pol;\n\t"
      "createpolicy.fractional.L2::evict_first.b64 pol, 1.0;\n\t"
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], pol;\n\t}"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch (PDL).
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void prefetch_l2(const void *p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Named barrier over `threads` threads (a multiple of 32), id 1..15.
__device__ __forceinline__ void named_bar(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Atomic add with acquire-release semantics at GPU scope; returns the old value.
__device__ __forceinline__ uint32_t atomic_add_acq_rel(uint32_t *p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void set_error(uint32_t *flag, uint32_t bits) {
  if (flag) atomicOr(flag, bits);
}

}  // namespace vg
