// Shared helpers for the llmyb sm_100a kernels: status codes, bf16 helpers,
// bounded device-side waits and warp reductions.
//
// Every exported entry point returns an int32 status: 0 on success, a
// cudaError_t value for CUDA failures (cudaErrorInvalidValue for bad
// arguments, as the reference engine does in llmy_cuda/src/llmy.cpp:216-218),
// or one of the LLMYB_E* codes below.  Kernels never allocate memory; every
// buffer, including scratch, is owned by the caller.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define LLMYB_OK 0
#define LLMYB_EINVAL 1            /* == cudaErrorInvalidValue */
#define LLMYB_EUNSUPPORTED 1001   /* shape outside what the kernel implements */
#define LLMYB_ETIMEOUT 1002       /* a device-side wait ran out (see dev_status) */

#define LLMYB_API extern "C" __attribute__((visibility("default")))

namespace llmyb {

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Host-side count of kernel launches issued by this library (diagnostics:
// lets a caller state how many of its kernels a step or a captured graph
// contains).  Incremented by every launch site through count_launch().
int64_t& launch_counter();
inline void count_launch(int n = 1) { launch_counter() += n; }

// Raise a kernel's dynamic shared-memory limit to at least `bytes` on the
// current device.  The attribute belongs to the (device, kernel) pair, so the
// largest value set is remembered per pair, under a lock: a process that
// drives several GPUs sets it on each, and concurrent host threads agree.
int32_t smem_limit_at_least(const void* kernel, int bytes);
template <typename K>
inline int32_t ensure_smem(K* kernel, int bytes) {
  return smem_limit_at_least(reinterpret_cast<const void*>(kernel), bytes);
}

inline int32_t launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LLMYB_OK : static_cast<int32_t>(e);
}

// Programmatic dependent launch.  A kernel launched by launch_pdl() may start
// while its predecessor in the stream is still running.  Before pdl_wait() it
// may only read data that no kernel still in flight writes: weights, or
// buffers last written two or more launches earlier (each kernel passes its
// own pdl_wait() before it triggers, so those writers have completed).
// pdl_wait() returns once the predecessor has completed and its writes are
// visible; pdl_trigger() then lets the successor launch.  For a kernel
// launched without the attribute both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

__device__ __forceinline__ float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float v) { return __float2bfloat16_rn(v); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&p);
}

__device__ __forceinline__ float2 unpack_bf16x2(uint32_t v) {
  __nv_bfloat162 p = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(p);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// silu(g) * u evaluated in fp32.  The reference applies
// torch.nn.functional.silu(gate) * up (model/layers/moe.py:75).
__device__ __forceinline__ float silu_mul(float g, float u) {
  return g / (1.0f + expf(-g)) * u;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// 2^x by the MUFU ex2 instruction (relative error about 2^-22; subnormal
// results flush to zero).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Upper bound for any spin-wait inside a kernel.  A legitimate wait in these
// kernels lasts microseconds; one second means a peer role has stopped.
constexpr uint64_t kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ void report_status(int32_t* dev_status, int32_t code) {
  if (dev_status != nullptr) atomicCAS(dev_status, 0, code);
}

}  // namespace llmyb
