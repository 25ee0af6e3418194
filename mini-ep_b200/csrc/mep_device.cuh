// Device helpers: element conversions that mirror torch's CPU rounding,
// system-scope flag signalling with bounded waits.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include "mep_internal.h"

namespace mep {

template <typename T> struct Elt;
template <> struct Elt<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
  // value as the model dtype would hold it (identity for fp32)
  static __device__ __forceinline__ float round(float v) { return v; }
};
template <> struct Elt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float round(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
  }
};

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// A relaxed store at system scope: after a fence.acq_rel.sys by the same
// thread it is a release (one fence for several flags, where a loop of
// st.release would fence once per flag).
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Acquire-release fences. The step's flags are message passing (data
// written, then a flag raised; a waiter reads the flag with ld.acquire.sys,
// then the data), which needs no sequentially consistent order: these are
// lighter than __threadfence_system (fence.sc.sys).
__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

__device__ __forceinline__ void set_err(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// Step timeline (profiling, off unless the context's "timeline" option is
// set): %globaltimer stamps of each stage of a layer step, in nanoseconds.
// A stage's start is stamped by block 0 when it starts; its end is the
// latest end over the stage's CTAs (atomicMax, which needs no reset between
// steps because the timer only grows). Slot numbers are the MEP_TL_* values
// of include/miniep_b200.h.
__device__ __forceinline__ void tl_begin(uint64_t* tl, int slot) {
  if (tl && blockIdx.x == 0 && threadIdx.x == 0) tl[slot] = globaltimer_ns();
}
__device__ __forceinline__ void tl_mark(uint64_t* tl, int slot) {
  if (tl) atomicMax(reinterpret_cast<unsigned long long*>(tl) + slot, globaltimer_ns());
}
__device__ __forceinline__ void tl_end(uint64_t* tl, int slot) {
  if (threadIdx.x == 0) tl_mark(tl, slot);
}

// Spin until *flag has reached `target` (wrap-safe compare), for at most
// wc.timeout_ns. Gives up early when another wait already failed, so one
// missing peer costs one timeout rather than one per kernel. The error word
// lives in host memory: each read crosses PCIe, and thousands of waiting
// threads reading it often would compete with the step's host copies, so a
// thread reads it at most once per kErrPollNs. Returns true when the flag
// arrived.
constexpr unsigned long long kErrPollNs = 1000000ull;
__device__ __forceinline__ bool wait_flag(const uint32_t* flag, uint32_t target, int errcode,
                                          const WaitCfg& wc) {
  if ((int32_t)(ld_acquire_sys(flag) - target) >= 0) return true;
  const unsigned long long t0 = globaltimer_ns();
  unsigned long long next_err = t0 + kErrPollNs;
  for (uint32_t it = 0;; ++it) {
    if ((int32_t)(ld_acquire_sys(flag) - target) >= 0) return true;
    __nanosleep(64);
    if ((it & 255u) == 255u) {
      const unsigned long long now = globaltimer_ns();
      if (now >= next_err) {
        if (wc.err && *(volatile int*)wc.err != 0) return false;
        next_err = now + kErrPollNs;
      }
      if (now - t0 > wc.timeout_ns) {
        set_err(wc.err, errcode);
        return false;
      }
    }
  }
}

// ---- shared-memory mbarriers (completion of bulk / TMA copies, role hand-offs)
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
// Bounded parity wait on a CTA-local mbarrier: false after timeout_ns (or
// once *abort is set by another warp of the CTA that gave up).
__device__ __forceinline__ bool mbar_wait_for(uint64_t* b, uint32_t parity,
                                              unsigned long long timeout_ns,
                                              volatile int* abort) {
  if (mbar_try(b, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try(b, parity)) return true;
    if ((it & 63u) == 63u) {
      if (abort && *abort) return false;
      if (globaltimer_ns() - t0 > timeout_ns) {
        if (abort) *abort = 1;
        return false;
      }
    }
  }
}
// Bulk copy of `bytes` from global memory into this CTA's shared memory,
// completing (complete_tx) on mbarrier `bar`.
__device__ __forceinline__ void bulk_load_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Bulk copy of `bytes` from shared memory to global memory (local or a
// peer's), in the issuing thread's current bulk group.
__device__ __forceinline__ void bulk_store_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}

// inclusive prefix sum over the 32 lanes of a warp
__device__ __forceinline__ int warp_inclusive_scan(int v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += t;
  }
  return v;
}

__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

}  // namespace mep
