// common.cuh — shared device helpers for the sm_100a decode kernels: error reporting, mbarrier + bulk-copy
// (TMA, non-tensor) wrappers, the fp16 m16n8k16 MMA, programmatic-dependent-launch controls, small math.
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

namespace agxc {

constexpr int kNumSMs = 148;            // B200
constexpr unsigned kTokenUnset = 0xFFFFFFFFu;

// Error bits of the device error word (set by bounded waits that gave up, and by bounds checks).
constexpr unsigned kErrMbarTimeout = 1u << 0;
constexpr unsigned kErrBadToken = 1u << 1;
constexpr unsigned kErrBadPos = 1u << 2;
constexpr unsigned kErrGridTimeout = 1u << 3;  // a grid barrier of the persistent step gave up
constexpr unsigned kErrAbort = 1u << 4;        // a wait gave up: every other wait of the launch leaves too

// ----------------------------------------------------------------------------------------------- host errors
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

#define AGXC_CUDA(call)                                   \
  do {                                                    \
    cudaError_t _e = (call);                              \
    if (_e != cudaSuccess) return ::agxc::cuda_fail(_e, #call); \
  } while (0)

// ----------------------------------------------------------------------------------------------- device helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// The same with a suspend-time hint: a thread whose phase is not complete sleeps (issuing nothing) until the phase
// completes or about hint_ns pass.
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, unsigned parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// The launch trace (optional): per launch kTraceSlots {min, max} pairs over its CTAs of %globaltimer at CTA entry
// (slot 0), after the dependency wait (slot 1), at CTA exit (slot 2), and for the GEMV after its activation rows are
// staged (slot 3), after its last unit's epilogue (slot 4) and when its first weight chunk has landed (slot 5).
// `t` NULL = not traced.
constexpr int kTraceSlots = 6;
__device__ __forceinline__ void trace_mark(unsigned long long* t, int slot) {
  if (!t) return;
  const unsigned long long v = globaltimer_ns();
  atomicMin(t + 2 * slot, v);
  atomicMax(t + 2 * slot + 1, v);
}

// A bounded wait on an mbarrier phase: gives up after `limit_ns` of the global timer, sets kErrMbarTimeout in the
// error word and returns false. Every wait in this library is bounded; none spins forever.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity, unsigned* err,
                                                  uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (unsigned it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 63u && globaltimer_ns() - t0 > limit_ns) {
      if (err) atomicOr(err, kErrMbarTimeout);
      return false;
    }
  }
}

// The bounded wait for warps that share a scheduler with busy ones: between polls the thread sleeps until the phase
// completes (or 0.2 ms pass), so a waiting warp takes no issue slots from the warps still working.
__device__ __forceinline__ bool mbar_wait_quiet(uint64_t* bar, unsigned parity, unsigned* err,
                                                uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait_hint(bar, parity, 200000u)) return true;
    if (globaltimer_ns() - t0 > limit_ns) {
      if (err) atomicOr(err, kErrMbarTimeout);
      return false;
    }
  }
}

// One bulk (non-tensor TMA) copy global -> this CTA's shared memory, completing on `bar` with complete_tx bytes.
// src and dst 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// An L2 prefetch hint for a contiguous range (16-byte aligned, a multiple of 16 bytes).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Programmatic dependent launch: wait for the upstream kernel's completion and memory; let the downstream launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// A kernel that may start before its predecessor in the stream has finished (pdl != 0): it waits for it before any
// global memory access, and lets its own successor start.
__device__ __forceinline__ void pdl_enter(int pdl) {
  if (pdl) {
    pdl_wait();
    pdl_launch_dependents();
  }
}

// Launch with programmatic dependent launch allowed when pdl != 0 (the kernel calls pdl_enter / pdl_wait first).
template <typename... KArgs, typename... Args>
int launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, int pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  AGXC_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
  return 0;
}

// D = A B + C, m16n8k16, fp16 operands, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float& d0, float& d1, float& d2, float& d3, uint32_t a0, uint32_t a1,
                                          uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d0), "+f"(d1), "+f"(d2), "+f"(d3)
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ float scale_to_f32(uint16_t v, int sdt) {
  return sdt ? __uint_as_float(static_cast<uint32_t>(v) << 16) : __half2float(__ushort_as_half(v));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}

// Loads that bypass L1 (data another CTA of this grid wrote; L2 is the coherence point).
__device__ __forceinline__ float ld_cg(const float* p) { return __ldcg(p); }

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace agxc
