// Residual stream helpers: token embedding into the fp32 residual stream and
// the fused "residual add + RMSNorm" that sits between every pair of
// sub-layers of PhysicalBlock.
//
// Reference: model/layers/norms.py:13-16 (RMSNorm: variance of the fp32
// value, x * rsqrt(var + eps) * weight), model/model.py:119-126 (with mHC
// off: read = mean over the single stream, write = streams + update) and
// :442-444 (embedding + stream_seed).  Under bf16 autocast the residual
// stream stays fp32 while sub-layer outputs are bf16; the same split is
// used here: streams fp32, normalised activations bf16 (fp32 on request).
#include <algorithm>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"

namespace llmyb {
namespace {

// streams[n] = float(table[ids[n]]) + seed      (one CTA per token)
__global__ void embed_kernel(const int64_t* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                             const float* __restrict__ seed, int D, int64_t vocab,
                             float* __restrict__ streams, int32_t* status) {
  const int64_t n = blockIdx.x;
  int64_t id = ids[n];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) report_status(status, LLMYB_EINVAL);
    id = 0;
  }
  const __nv_bfloat16* row = table + id * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x)
    streams[n * D + d] = bf2f(row[d]) + (seed ? seed[d] : 0.f);
}

// streams += delta (optional); y = streams * rsqrt(mean(streams^2) + eps) * w
// (normalize = 0: y = streams, the plain residual value)
// With route_pos the delta of row n is the sum of the k routed expert rows
// delta[route_pos[n*k + s]] (the MoE combine fused into the residual add).
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(
    float* __restrict__ streams, const __nv_bfloat16* __restrict__ delta,
    const int* __restrict__ route_pos, int k, int D, const float* __restrict__ weight, float eps,
    int normalize, __nv_bfloat16* __restrict__ out_bf16, float* __restrict__ out_f32) {
  __shared__ float red[8];
  const int64_t n = blockIdx.x;
  float* x = streams + n * D;
  float ss = 0.f;
  for (int d = threadIdx.x; d < D; d += 256) {
    float v = x[d];
    if (delta != nullptr) {
      if (route_pos != nullptr) {
        for (int s = 0; s < k; ++s)
          v += bf2f(delta[static_cast<int64_t>(route_pos[n * k + s]) * D + d]);
      } else {
        v += bf2f(delta[n * D + d]);
      }
      x[d] = v;
    }
    ss += v * v;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float r = normalize ? rsqrtf(tot / static_cast<float>(D) + eps) : 1.f;
  for (int d = threadIdx.x; d < D; d += 256) {
    const float y = normalize ? x[d] * r * (weight ? weight[d] : 1.f) : x[d];
    if (out_bf16) out_bf16[n * D + d] = f2bf(y);
    if (out_f32) out_f32[n * D + d] = y;
  }
}

// add_rmsnorm_kernel for D % 8 == 0 with 16-byte rows: thread i owns the
// 8-element vectors i, i+256, ... (at most VMAX of them, kept in registers
// between the sum of squares and the scaled write); the routed delta rows of
// a vector are loaded together.  The per-element sum order (stream value,
// then the k routed rows in slot order) is that of add_rmsnorm_kernel.
// kRouter: out_f32 receives the router's input RMSNorm(y) * weight2 instead of
// y (context_router.py:62, local = norm(hidden) on the FFN-normalised row),
// with the second sum of squares formed exactly as a separate add_rmsnorm
// pass over y would (same per-thread order, same block reduction).
template <int VMAX, bool kRouter = false>
__global__ void __launch_bounds__(256) add_rmsnorm_vec_kernel(
    float* __restrict__ streams, const __nv_bfloat16* __restrict__ delta,
    const int* __restrict__ route_pos, int k, int D, const float* __restrict__ weight, float eps,
    int normalize, __nv_bfloat16* __restrict__ out_bf16, float* __restrict__ out_f32,
    const float* __restrict__ weight2 = nullptr) {
  __shared__ float red[8];
  __shared__ float red2[8];
  const int64_t n = blockIdx.x;
  const int nv = D >> 3;
  float4* x4 = reinterpret_cast<float4*>(streams + n * D);
  float v[VMAX][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < VMAX; ++j) {
    const int c = threadIdx.x + j * 256;
    if (c >= nv) continue;
    const float4 a = x4[2 * c], b = x4[2 * c + 1];
    v[j][0] = a.x; v[j][1] = a.y; v[j][2] = a.z; v[j][3] = a.w;
    v[j][4] = b.x; v[j][5] = b.y; v[j][6] = b.z; v[j][7] = b.w;
    if (delta != nullptr) {
      if (route_pos != nullptr) {
#pragma unroll 4
        for (int s = 0; s < k; ++s) {
          const int64_t pos = __ldg(route_pos + n * k + s);
          const uint4 u = __ldg(reinterpret_cast<const uint4*>(delta + pos * D) + c);
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = unpack_bf16x2(w[q]);
            v[j][2 * q] += f.x;
            v[j][2 * q + 1] += f.y;
          }
        }
      } else {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(delta + n * D) + c);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(w[q]);
          v[j][2 * q] += f.x;
          v[j][2 * q + 1] += f.y;
        }
      }
      x4[2 * c] = make_float4(v[j][0], v[j][1], v[j][2], v[j][3]);
      x4[2 * c + 1] = make_float4(v[j][4], v[j][5], v[j][6], v[j][7]);
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) ss += v[j][q] * v[j][q];
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float r = normalize ? rsqrtf(tot / static_cast<float>(D) + eps) : 1.f;
#pragma unroll
  for (int j = 0; j < VMAX; ++j) {
    const int c = threadIdx.x + j * 256;
    if (c >= nv) continue;
    float y[8];
    if (normalize) {
      float w8[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
      if (weight != nullptr) {
        const float4 wa = __ldg(reinterpret_cast<const float4*>(weight) + 2 * c);
        const float4 wb = __ldg(reinterpret_cast<const float4*>(weight) + 2 * c + 1);
        w8[0] = wa.x; w8[1] = wa.y; w8[2] = wa.z; w8[3] = wa.w;
        w8[4] = wb.x; w8[5] = wb.y; w8[6] = wb.z; w8[7] = wb.w;
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) y[q] = v[j][q] * r * w8[q];
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) y[q] = v[j][q];
    }
    if (out_bf16 != nullptr) {
      uint4 o;
      o.x = pack_bf16x2(y[0], y[1]);
      o.y = pack_bf16x2(y[2], y[3]);
      o.z = pack_bf16x2(y[4], y[5]);
      o.w = pack_bf16x2(y[6], y[7]);
      reinterpret_cast<uint4*>(out_bf16 + n * D)[c] = o;
    }
    if constexpr (kRouter) {
#pragma unroll
      for (int q = 0; q < 8; ++q) v[j][q] = y[q];
    } else if (out_f32 != nullptr) {
      float4* o4 = reinterpret_cast<float4*>(out_f32 + n * D);
      o4[2 * c] = make_float4(y[0], y[1], y[2], y[3]);
      o4[2 * c + 1] = make_float4(y[4], y[5], y[6], y[7]);
    }
  }
  if constexpr (kRouter) {
    float ss2 = 0.f;
#pragma unroll
    for (int j = 0; j < VMAX; ++j) {
      if (threadIdx.x + j * 256 >= nv) continue;
#pragma unroll
      for (int q = 0; q < 8; ++q) ss2 += v[j][q] * v[j][q];
    }
    ss2 = warp_sum(ss2);
    if ((threadIdx.x & 31) == 0) red2[threadIdx.x >> 5] = ss2;
    __syncthreads();
    float tot2 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot2 += red2[i];
    const float r2 = rsqrtf(tot2 / static_cast<float>(D) + eps);
#pragma unroll
    for (int j = 0; j < VMAX; ++j) {
      const int c = threadIdx.x + j * 256;
      if (c >= nv) continue;
      const float4 wa = __ldg(reinterpret_cast<const float4*>(weight2) + 2 * c);
      const float4 wb = __ldg(reinterpret_cast<const float4*>(weight2) + 2 * c + 1);
      float4* o4 = reinterpret_cast<float4*>(out_f32 + n * D);
      o4[2 * c] = make_float4(v[j][0] * r2 * wa.x, v[j][1] * r2 * wa.y, v[j][2] * r2 * wa.z,
                              v[j][3] * r2 * wa.w);
      o4[2 * c + 1] = make_float4(v[j][4] * r2 * wb.x, v[j][5] * r2 * wb.y, v[j][6] * r2 * wb.z,
                                  v[j][7] * r2 * wb.w);
    }
  }
}

// Launch the vectorised kernel when D and every pointer allow 16-byte rows.
int32_t launch_add_rmsnorm(float* streams, const __nv_bfloat16* delta, const int* route_pos, int k,
                           int64_t n, int D, const float* weight, float eps, int normalize,
                           __nv_bfloat16* out_bf16, float* out_f32, cudaStream_t s) {
  const uintptr_t align = reinterpret_cast<uintptr_t>(streams) |
                          reinterpret_cast<uintptr_t>(delta) |
                          reinterpret_cast<uintptr_t>(weight) |
                          reinterpret_cast<uintptr_t>(out_bf16) |
                          reinterpret_cast<uintptr_t>(out_f32);
  const unsigned grid = static_cast<unsigned>(n);
  if (D % 8 == 0 && (align & 15u) == 0 && D <= 8 * 256 * 4) {
    if (D <= 8 * 256)
      add_rmsnorm_vec_kernel<1><<<grid, 256, 0, s>>>(streams, delta, route_pos, k, D, weight, eps,
                                                      normalize, out_bf16, out_f32);
    else if (D <= 8 * 256 * 2)
      add_rmsnorm_vec_kernel<2><<<grid, 256, 0, s>>>(streams, delta, route_pos, k, D, weight, eps,
                                                      normalize, out_bf16, out_f32);
    else
      add_rmsnorm_vec_kernel<4><<<grid, 256, 0, s>>>(streams, delta, route_pos, k, D, weight, eps,
                                                      normalize, out_bf16, out_f32);
  } else {
    add_rmsnorm_kernel<<<grid, 256, 0, s>>>(streams, delta, route_pos, k, D, weight, eps,
                                            normalize, out_bf16, out_f32);
  }
  count_launch();
  return launch_status();
}

// RMSNorm of a bf16 input (used on the collapsed stream before the LM head)
__global__ void __launch_bounds__(256) rmsnorm_bf16_kernel(const __nv_bfloat16* __restrict__ x, int D,
                                                           const float* __restrict__ weight,
                                                           float eps,
                                                           __nv_bfloat16* __restrict__ out) {
  __shared__ float red[8];
  const int64_t n = blockIdx.x;
  float ss = 0.f;
  for (int d = threadIdx.x; d < D; d += 256) {
    const float v = bf2f(x[n * D + d]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float r = rsqrtf(tot / static_cast<float>(D) + eps);
  for (int d = threadIdx.x; d < D; d += 256)
    out[n * D + d] = f2bf(bf2f(x[n * D + d]) * r * (weight ? weight[d] : 1.f));
}

}  // namespace
}  // namespace llmyb

namespace llmyb {
int64_t& launch_counter() {
  static int64_t n = 0;
  return n;
}

int32_t smem_limit_at_least(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, int> set;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int32_t>(e);
  std::lock_guard<std::mutex> lock(mu);
  int& have = set[{dev, kernel}];
  if (bytes <= have) return LLMYB_OK;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return static_cast<int32_t>(e);
  have = bytes;
  return LLMYB_OK;
}
// Zeroes n regions, regions[2r] = device address, regions[2r+1] = bytes:
// blockIdx.y picks the region; 16-byte stores over its aligned body, byte
// stores over the unaligned head and tail.
__global__ void zero_regions_kernel(const int64_t* __restrict__ regions) {
  const int r = blockIdx.y;
  uint8_t* p = reinterpret_cast<uint8_t*>(static_cast<uintptr_t>(regions[2 * r]));
  const int64_t bytes = regions[2 * r + 1];
  const int64_t head =
      min(bytes, static_cast<int64_t>((16u - (reinterpret_cast<uintptr_t>(p) & 15u)) & 15u));
  const int64_t body = (bytes - head) / 16;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (tid < head) p[tid] = 0;
  uint4* b4 = reinterpret_cast<uint4*>(p + head);
  for (int64_t i = tid; i < body; i += nthreads) b4[i] = make_uint4(0, 0, 0, 0);
  const int64_t tail0 = head + body * 16;
  if (tid < bytes - tail0) p[tail0 + tid] = 0;
}

}  // namespace llmyb

using namespace llmyb;

// Number of kernel launches this library has issued since it was loaded.
LLMYB_API int64_t llmyb_launch_count(void) { return launch_counter(); }

LLMYB_API int32_t llmyb_zero_regions(const int64_t* regions, int32_t n_regions, int64_t max_bytes,
                                     void* stream) {
  if (n_regions < 0 || max_bytes < 0 || (n_regions > 0 && !regions)) return LLMYB_EINVAL;
  if (n_regions > 65535) return LLMYB_EUNSUPPORTED;
  if (n_regions == 0 || max_bytes == 0) return LLMYB_OK;
  const int64_t blocks = std::min<int64_t>(ceil_div(max_bytes, 16 * 256), 64);
  zero_regions_kernel<<<dim3(static_cast<unsigned>(std::max<int64_t>(blocks, 1)),
                             static_cast<unsigned>(n_regions)),
                        256, 0, static_cast<cudaStream_t>(stream)>>>(regions);
  count_launch();
  return launch_status();
}

LLMYB_API int32_t llmyb_embed(const int64_t* ids, int64_t n_tokens, const void* table,
                              int64_t vocab, int32_t d_model, const float* stream_seed,
                              float* streams, int32_t* dev_status, void* stream) {
  if (!ids || !table || !streams || n_tokens < 0 || d_model <= 0 || vocab <= 0) return LLMYB_EINVAL;
  if (n_tokens == 0) return LLMYB_OK;
  embed_kernel<<<static_cast<unsigned>(n_tokens), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      ids, static_cast<const __nv_bfloat16*>(table), stream_seed, d_model, vocab, streams,
      dev_status);
  count_launch();
  return launch_status();
}

LLMYB_API int32_t llmyb_add_rmsnorm(float* streams, const void* delta, int64_t n_tokens,
                                    int32_t d_model, const float* weight, float eps,
                                    int32_t normalize, void* out_bf16, float* out_f32,
                                    void* stream) {
  if (!streams || n_tokens < 0 || d_model <= 0) return LLMYB_EINVAL;
  if (n_tokens == 0) return LLMYB_OK;
  return launch_add_rmsnorm(streams, static_cast<const __nv_bfloat16*>(delta), nullptr, 0,
                            n_tokens, d_model, weight, eps, normalize,
                            static_cast<__nv_bfloat16*>(out_bf16), out_f32,
                            static_cast<cudaStream_t>(stream));
}

// streams += sum_s y_rows[route_pos[n*k + s]] (bf16 expert rows, fp32 sum),
// then RMSNorm as llmyb_add_rmsnorm.
LLMYB_API int32_t llmyb_add_rmsnorm_routed(float* streams, const void* y_rows,
                                           const int32_t* route_pos, int32_t top_k,
                                           int64_t n_tokens, int32_t d_model, const float* weight,
                                           float eps, int32_t normalize, void* out_bf16,
                                           float* out_f32, void* stream) {
  if (!streams || !y_rows || !route_pos || top_k <= 0 || n_tokens < 0 || d_model <= 0)
    return LLMYB_EINVAL;
  if (n_tokens == 0) return LLMYB_OK;
  return launch_add_rmsnorm(streams, static_cast<const __nv_bfloat16*>(y_rows), route_pos, top_k,
                            n_tokens, d_model, weight, eps, normalize,
                            static_cast<__nv_bfloat16*>(out_bf16), out_f32,
                            static_cast<cudaStream_t>(stream));
}

// streams += delta; m = RMSNorm(streams) * ffn_weight (bf16 into out_bf16);
// router_in = RMSNorm(m) * router_weight (fp32), in one pass over the row.
LLMYB_API int32_t llmyb_add_rmsnorm_router(float* streams, const void* delta, int64_t n_tokens,
                                           int32_t d_model, const float* ffn_weight,
                                           const float* router_weight, float eps,
                                           void* out_bf16, float* router_in, void* stream) {
  if (!streams || !ffn_weight || !router_weight || !router_in || n_tokens < 0 || d_model <= 0)
    return LLMYB_EINVAL;
  if (n_tokens == 0) return LLMYB_OK;
  const uintptr_t align = reinterpret_cast<uintptr_t>(streams) |
                          reinterpret_cast<uintptr_t>(delta) |
                          reinterpret_cast<uintptr_t>(ffn_weight) |
                          reinterpret_cast<uintptr_t>(router_weight) |
                          reinterpret_cast<uintptr_t>(out_bf16) |
                          reinterpret_cast<uintptr_t>(router_in);
  if (d_model % 8 != 0 || (align & 15u) != 0 || d_model > 8 * 256 * 4) return LLMYB_EUNSUPPORTED;
  const unsigned grid = static_cast<unsigned>(n_tokens);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto* dl = static_cast<const __nv_bfloat16*>(delta);
  auto* ob = static_cast<__nv_bfloat16*>(out_bf16);
  if (d_model <= 8 * 256)
    add_rmsnorm_vec_kernel<1, true><<<grid, 256, 0, s>>>(streams, dl, nullptr, 0, d_model,
                                                         ffn_weight, eps, 1, ob, router_in,
                                                         router_weight);
  else if (d_model <= 8 * 256 * 2)
    add_rmsnorm_vec_kernel<2, true><<<grid, 256, 0, s>>>(streams, dl, nullptr, 0, d_model,
                                                         ffn_weight, eps, 1, ob, router_in,
                                                         router_weight);
  else
    add_rmsnorm_vec_kernel<4, true><<<grid, 256, 0, s>>>(streams, dl, nullptr, 0, d_model,
                                                         ffn_weight, eps, 1, ob, router_in,
                                                         router_weight);
  count_launch();
  return launch_status();
}

LLMYB_API int32_t llmyb_rmsnorm_bf16(const void* x, int64_t n_tokens, int32_t d_model,
                                     const float* weight, float eps, void* out, void* stream) {
  if (!x || !out || n_tokens < 0 || d_model <= 0) return LLMYB_EINVAL;
  if (n_tokens == 0) return LLMYB_OK;
  rmsnorm_bf16_kernel<<<static_cast<unsigned>(n_tokens), 256, 0,
                        static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), d_model, weight, eps, static_cast<__nv_bfloat16*>(out));
  count_launch();
  return launch_status();
}
