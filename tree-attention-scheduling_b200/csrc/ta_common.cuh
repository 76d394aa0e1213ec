// Shared device helpers for the tree-attention kernels (sm_100a only).
//
// Every wait on an mbarrier is bounded: after about a second the waiting thread
// records TA_ERR_TIMEOUT in the call's status word and gives up, so a lost
// completion can never hang the GPU.  Index checks on plan metadata record
// TA_ERR_BOUNDS and skip the access instead of trapping.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "tree_attn.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "tree-attention kernels target sm_100a only"
#endif

namespace ta {

// A wait on an mbarrier is declared lost after TA_WAIT_NS nanoseconds of the
// global timer (about a second: far above any legitimate wait in these
// kernels, short enough that a lost completion ends the kernel quickly).
constexpr uint64_t TA_WAIT_NS = 1000000000ull;

__device__ __forceinline__ void set_status(int32_t* status, int32_t bit) {
  if (status) atomicOr(status, bit);
}

// ---------------------------------------------------------------------------
// element types
template <typename T> struct Elem;
template <> struct Elem<__nv_bfloat16> {
  static constexpr int kCode = TA_DTYPE_BF16;
  __device__ __forceinline__ static float2 to_float2(uint32_t bits) {
    // bf16 -> f32 is exact: the bf16 bits are the high half of the f32.
    return make_float2(__uint_as_float(bits << 16), __uint_as_float(bits & 0xffff0000u));
  }
  __device__ __forceinline__ static float to_float(uint16_t bits) {
    return __uint_as_float(uint32_t(bits) << 16);
  }
  __device__ __forceinline__ static uint16_t from_float(float x) {
    __nv_bfloat16 h = __float2bfloat16_rn(x);
    return *reinterpret_cast<uint16_t*>(&h);
  }
  __device__ __forceinline__ static uint32_t pack2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct Elem<__half> {
  static constexpr int kCode = TA_DTYPE_F16;
  __device__ __forceinline__ static float2 to_float2(uint32_t bits) {
    __half2 h = *reinterpret_cast<__half2*>(&bits);
    return __half22float2(h);
  }
  __device__ __forceinline__ static float to_float(uint16_t bits) {
    __half h = *reinterpret_cast<__half*>(&bits);
    return __half2float(h);
  }
  __device__ __forceinline__ static uint16_t from_float(float x) {
    __half h = __float2half_rn(x);
    return *reinterpret_cast<uint16_t*>(&h);
  }
  __device__ __forceinline__ static uint32_t pack2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

// ---------------------------------------------------------------------------
// exp2 on the SFU: softmax runs in the log2 domain (scores are pre-scaled by
// log2(e)/sqrt(D)), the LSE is converted back to natural-log units on output.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float fast_log2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// ---------------------------------------------------------------------------
// shared-memory addresses and mbarriers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of phase `parity` of `bar` (for loops that poll several barriers).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that suspends the thread for at most about `ns` nanoseconds.
__device__ __forceinline__ bool mbar_try_wait_for(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for phase `parity` of `bar`.  Returns false (and records the
// timeout) if the phase did not complete within TA_WAIT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - start > TA_WAIT_NS) break;
  }
  set_status(status, TA_ERR_TIMEOUT);
  return false;
}

// 1-D bulk copy global -> shared, completing on `bar` (non-multicast).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// Warp transpose-reduction: lane l ends up with the sum over all lanes of
// v[l].  31 shuffles for 32 sums (versus 5 per sum for a plain butterfly).
__device__ __forceinline__ float warp_transpose_sum32(float (&v)[32], int lane) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = upper ? v[i] : v[i + off];
      const float keep = upper ? v[i + off] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
  return v[0];
}

// Sums of W values (W = 4, 8 or 16) over the 32 lanes by recursive halving:
// W - 1 + 5 - log2(W) shuffles.  Lane l returns the sum of v[l >> (5 - log2 W)].
template <int W>
__device__ __forceinline__ float warp_transpose_sum(const float (&in)[W], int lane) {
  float v[W];
#pragma unroll
  for (int i = 0; i < W; ++i) v[i] = in[i];
  int off = 16;
#pragma unroll
  for (int n = W; n > 1; n >>= 1, off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = upper ? v[i] : v[i + n / 2];
      const float keep = upper ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
#pragma unroll
  for (; off >= 1; off >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
  return v[0];
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, off));
  return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

// Programmatic dependent launch.  A segment kernel lets the next kernel of
// its stream start early (its CTAs are placed as SMs free up); a dependent
// waits, before touching what its predecessors wrote, until those have
// completed and their writes are visible.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launch `kernel` so that it may start before the previous kernel of `stream`
// completes (that kernel must have called pdl_trigger; the new one calls
// pdl_wait before it depends on it).
template <typename... Params, typename... Args>
cudaError_t launch_dependent(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace ta
