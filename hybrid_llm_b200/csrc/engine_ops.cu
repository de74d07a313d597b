// Two stand-alone device entry points of the reference engine's C ABI
// (llmy_cuda/include/llmy.h:74-88):
//   llmyb_mhc_sinkhorn4      <- llmy_mhc_sinkhorn4 (the mHC mapping normaliser,
//                               model/layers/mhc.py:12-17)
//   llmyb_moe_selected_fp32  <- llmy_moe_selected_fp32 (one token through its k
//                               routed experts, fp32 weights)
// Both return an int32 status (LLMYB_EINVAL on bad arguments) and never
// allocate; the caller passes every buffer and the stream.
#include <cstdint>

#include "common.cuh"

namespace llmyb {
namespace {

// log(sum_i exp(v_i)) of four values, shifted by their maximum.
__device__ __forceinline__ float lse4(float a, float b, float c, float d) {
  const float m = fmaxf(fmaxf(a, b), fmaxf(c, d));
  return m + logf(expf(a - m) + expf(b - m) + expf(c - m) + expf(d - m));
}

// One thread per 4x4 matrix, all sixteen values in registers: `iters` rounds of
// row then column log-normalisation, then exp (mhc.py:12-17).  Each matrix is
// 64 contiguous bytes, read and written as four 16-byte vectors.
__global__ void __launch_bounds__(256) sinkhorn4_kernel(const float4* __restrict__ in,
                                                        float4* __restrict__ out,
                                                        int64_t matrices, int iters) {
  const int64_t m = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (m >= matrices) return;
  float a[4][4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const float4 v = in[m * 4 + r];
    a[r][0] = v.x;
    a[r][1] = v.y;
    a[r][2] = v.z;
    a[r][3] = v.w;
  }
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float l = lse4(a[r][0], a[r][1], a[r][2], a[r][3]);
#pragma unroll
      for (int c = 0; c < 4; ++c) a[r][c] -= l;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float l = lse4(a[0][c], a[1][c], a[2][c], a[3][c]);
#pragma unroll
      for (int r = 0; r < 4; ++r) a[r][c] -= l;
    }
  }
#pragma unroll
  for (int r = 0; r < 4; ++r)
    out[m * 4 + r] = make_float4(expf(a[r][0]), expf(a[r][1]), expf(a[r][2]), expf(a[r][3]));
}

// Dot product of one weight row with a vector, by a whole warp (lane-strided,
// 16-byte loads when both are 16-byte aligned), result in every lane.
__device__ __forceinline__ float warp_dot(const float* __restrict__ w, const float* __restrict__ v,
                                          int n, int lane) {
  float acc = 0.0f;
  if (((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(v)) & 15u) == 0 &&
      (n & 3) == 0) {
    const float4* w4 = reinterpret_cast<const float4*>(w);
    const float4* v4 = reinterpret_cast<const float4*>(v);
    for (int i = lane; i < n / 4; i += 32) {
      const float4 a = __ldg(w4 + i), b = __ldg(v4 + i);
      acc = fmaf(a.x, b.x, acc);
      acc = fmaf(a.y, b.y, acc);
      acc = fmaf(a.z, b.z, acc);
      acc = fmaf(a.w, b.w, acc);
    }
  } else {
    for (int i = lane; i < n; i += 32) acc = fmaf(__ldg(w + i), __ldg(v + i), acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return acc;
}

// activation[r, h] = silu(gate_e[h] . x) * (up_e[h] . x) for route r's expert e
// (gate rows [0, H), up rows [H, 2H) of gate_up[e]); an expert id outside
// [0, E) contributes zeros.  Warp per (route, feature row).
__global__ void __launch_bounds__(256) moe_selected_up_kernel(
    const float* __restrict__ x, const int64_t* __restrict__ idx,
    const float* __restrict__ gate_up, float* __restrict__ activation, int D, int H, int E) {
  const int r = blockIdx.y;
  const int h = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (h >= H) return;
  const int64_t e = __ldg(idx + r);
  float act = 0.0f;
  if (e >= 0 && e < E) {
    const float* base = gate_up + static_cast<size_t>(e) * 2 * H * D;
    const float g = warp_dot(base + static_cast<size_t>(h) * D, x, D, lane);
    const float u = warp_dot(base + static_cast<size_t>(H + h) * D, x, D, lane);
    act = g / (1.0f + expf(-g)) * u;
  }
  if (lane == 0) activation[static_cast<size_t>(r) * H + h] = act;
}

// route_output[r, d] = prob[r] * (down_e[d] . activation[r]) and
// out[d] = sum over routes in route order.  Warp per output row.
__global__ void __launch_bounds__(256) moe_selected_down_kernel(
    const int64_t* __restrict__ idx, const float* __restrict__ prob,
    const float* __restrict__ down, const float* __restrict__ activation,
    float* __restrict__ route_output, float* __restrict__ out, int D, int H, int E, int k) {
  const int d = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (d >= D) return;
  float sum = 0.0f;
  for (int r = 0; r < k; ++r) {
    const int64_t e = __ldg(idx + r);
    float v = 0.0f;
    if (e >= 0 && e < E)
      v = __ldg(prob + r) * warp_dot(down + (static_cast<size_t>(e) * D + d) * H,
                                     activation + static_cast<size_t>(r) * H, H, lane);
    if (lane == 0) route_output[static_cast<size_t>(r) * D + d] = v;
    sum += v;
  }
  if (lane == 0) out[d] = sum;
}

}  // namespace
}  // namespace llmyb

using namespace llmyb;

LLMYB_API int32_t llmyb_mhc_sinkhorn4(const float* input, float* output, int32_t matrices,
                                      int32_t iterations, void* stream) {
  if (input == nullptr || output == nullptr || matrices <= 0 || iterations < 0)
    return LLMYB_EINVAL;
  if (((reinterpret_cast<uintptr_t>(input) | reinterpret_cast<uintptr_t>(output)) & 15u) != 0)
    return LLMYB_EINVAL;
  const int threads = 256;
  const int64_t blocks = (static_cast<int64_t>(matrices) + threads - 1) / threads;
  sinkhorn4_kernel<<<static_cast<unsigned>(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const float4*>(input), reinterpret_cast<float4*>(output), matrices,
      iterations);
  count_launch();
  return launch_status();
}

LLMYB_API int32_t llmyb_moe_selected_fp32(const float* x, const int64_t* idx, const float* prob,
                                          const float* gate_up, const float* down,
                                          float* activation, float* route_output, float* out,
                                          int32_t D, int32_t H, int32_t E, int32_t k,
                                          void* stream) {
  if (x == nullptr || idx == nullptr || prob == nullptr || gate_up == nullptr ||
      down == nullptr || activation == nullptr || route_output == nullptr || out == nullptr ||
      D <= 0 || H <= 0 || E <= 0 || k <= 0 || k > 65535)
    return LLMYB_EINVAL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  moe_selected_up_kernel<<<dim3((H + 7) / 8, k), 256, 0, s>>>(x, idx, gate_up, activation, D, H,
                                                              E);
  count_launch();
  moe_selected_down_kernel<<<(D + 7) / 8, 256, 0, s>>>(idx, prob, down, activation, route_output,
                                                       out, D, H, E, k);
  count_launch();
  return launch_status();
}
