// Local-context path of the context-aware router (model/layers/context_router.py:59-74,
// :89-133; model/layers/mla_memory.py:23-48): the router input of token t is
//   local_t + g * context_out(local_context_out(mean of the latents of tokens
//   max(0, t-W+1) .. t)),   latent = LayerNorm(down(local))   (eps 1e-5).
// The two output projections and the router are folded into one [E, L] matrix
// by the caller, so these kernels only produce the latents' window means
// ("box"); the caller's GEMMs add them to the logits.
//
// Decode keeps the latents of the last W positions per row in a ring
// [B, W, L] fp32 (position p at slot p % W), which prefill fills with its last
// W tokens.
#include <cstdint>

#include "common.cuh"

namespace llmyb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float block_sum256(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) t += red[i];
  return t;
}

// LayerNorm of one L-wide row held as (up to) four values per thread.
__device__ __forceinline__ void layer_norm_row(float (&v)[4], int L, const float* __restrict__ w,
                                               const float* __restrict__ b, float* red) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) s += v[i];  // zero beyond L
  const float mean = block_sum256(s, red) / static_cast<float>(L);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int l = threadIdx.x + i * kThreads;
    if (l < L) q += (v[i] - mean) * (v[i] - mean);
  }
  const float rstd = rsqrtf(block_sum256(q, red) / static_cast<float>(L) + 1e-5f);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int l = threadIdx.x + i * kThreads;
    if (l < L) v[i] = (v[i] - mean) * rstd * __ldg(w + l) + __ldg(b + l);
  }
}

// lat [N, L] (down(local) in, LayerNorm'd in place); CTA per row.
__global__ void __launch_bounds__(kThreads) latent_norm_kernel(float* __restrict__ lat, int L,
                                                               const float* __restrict__ w,
                                                               const float* __restrict__ b) {
  __shared__ float red[kThreads / 32];
  float* row = lat + static_cast<int64_t>(blockIdx.x) * L;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int l = threadIdx.x + i * kThreads;
    v[i] = l < L ? row[l] : 0.f;
  }
  layer_norm_row(v, L, w, b, red);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int l = threadIdx.x + i * kThreads;
    if (l < L) row[l] = v[i];
  }
}

// box[b, t, l] = mean of lat[b, max(0, t-W+1) .. t, l] by a running window sum
// (thread per (row, channel), coalesced over channels); the last W latents of
// each row go to the ring.
__global__ void __launch_bounds__(kThreads) box_mean_kernel(const float* __restrict__ lat,
                                                            int64_t rows, int T, int L, int W,
                                                            float* __restrict__ box,
                                                            float* __restrict__ ring) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x;
  if (i >= rows * L) return;
  const int64_t r = i / L;
  const int l = static_cast<int>(i - r * L);
  const float* x = lat + r * T * L + l;
  float* y = box + r * T * L + l;
  float acc = 0.f;
  for (int t = 0; t < T; ++t) {
    const float v = x[static_cast<int64_t>(t) * L];
    acc += v;
    if (t >= W) acc -= x[static_cast<int64_t>(t - W) * L];
    y[static_cast<int64_t>(t) * L] = acc / static_cast<float>(t + 1 < W ? t + 1 : W);
    if (ring != nullptr && t >= T - W) ring[(r * W + t % W) * L + l] = v;
  }
}

// One decode step per row: LayerNorm the new latent, store it at slot pos % W,
// box = mean of the latents of positions max(0, pos-W+1) .. pos.
__global__ void __launch_bounds__(kThreads) ctx_step_kernel(float* __restrict__ lat, int L, int W,
                                                            const float* __restrict__ w,
                                                            const float* __restrict__ b,
                                                            float* __restrict__ ring,
                                                            const int* __restrict__ positions,
                                                            float* __restrict__ box) {
  __shared__ float red[kThreads / 32];
  const int64_t r = blockIdx.x;
  const int pos = __ldg(positions + r);
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int l = threadIdx.x + i * kThreads;
    v[i] = l < L ? lat[r * L + l] : 0.f;
  }
  layer_norm_row(v, L, w, b, red);
  float* rr = ring + r * W * L;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int l = threadIdx.x + i * kThreads;
    if (l < L) rr[(pos % W) * L + l] = v[i];
  }
  __syncthreads();
  const int count = pos + 1 < W ? pos + 1 : W;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int l = threadIdx.x + i * kThreads;
    if (l >= L) continue;
    float acc = 0.f;
    for (int c = count - 1; c >= 0; --c) acc += rr[((pos - c) % W) * L + l];  // oldest first
    box[r * L + l] = acc / static_cast<float>(count);
  }
}

}  // namespace
}  // namespace llmyb

using namespace llmyb;

LLMYB_API int32_t llmyb_router_ctx_prefill(float* lat, int32_t batch, int32_t seq, int32_t latent,
                                           int32_t window, const float* ln_w, const float* ln_b,
                                           float* box, float* ring, void* stream) {
  if (batch < 0 || seq < 0 || latent <= 0 || latent > 4 * kThreads || window < 1)
    return LLMYB_EINVAL;
  if (batch == 0 || seq == 0) return LLMYB_OK;
  if (!lat || !ln_w || !ln_b || !box) return LLMYB_EINVAL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t n = static_cast<int64_t>(batch) * seq;
  latent_norm_kernel<<<static_cast<unsigned>(n), kThreads, 0, s>>>(lat, latent, ln_w, ln_b);
  count_launch();
  const int64_t work = static_cast<int64_t>(batch) * latent;
  box_mean_kernel<<<static_cast<unsigned>((work + kThreads - 1) / kThreads), kThreads, 0, s>>>(
      lat, batch, seq, latent, window, box, ring);
  count_launch();
  return launch_status();
}

LLMYB_API int32_t llmyb_router_ctx_step(float* lat, int32_t batch, int32_t latent, int32_t window,
                                        const float* ln_w, const float* ln_b, float* ring,
                                        const int32_t* positions, float* box, void* stream) {
  if (batch < 0 || latent <= 0 || latent > 4 * kThreads || window < 1) return LLMYB_EINVAL;
  if (batch == 0) return LLMYB_OK;
  if (!lat || !ln_w || !ln_b || !ring || !positions || !box) return LLMYB_EINVAL;
  ctx_step_kernel<<<batch, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      lat, latent, window, ln_w, ln_b, ring, positions, box);
  count_launch();
  return launch_status();
}
