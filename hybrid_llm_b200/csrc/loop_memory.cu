// Loop memory between recurrent loops (model/loop_memory.py LoopMemoryHook,
// called at model/model.py:636 and :661-667 in prefill, :877 and :884-891 in
// a decode step).
//
// Before every loop after the first, each token attends over latent
// summaries ("endpoints") of its own hidden state at the end of the earlier
// loops, and the gated result is added to every residual stream:
//
//   endpoint_j = LayerNorm_L(W_down mean_s(streams after loop j))     (encode)
//   q          = W_q LayerNorm_D(mean_s(streams))                     (inject)
//   k_j, v_j   = W_k endpoint_j, W_v endpoint_j
//   o_h        = sum_j softmax_j(q_h . k_jh / sqrt(hd)) v_jh          (per head)
//   streams[s] += sigmoid(gating_logit) * W_o o                       (every s)
//
// The projections are plain fp32 GEMMs of the caller; these kernels are the
// per-token pieces between them:
//   loop_mem_norm_kernel    mean over the S streams, optionally LayerNorm
//   loop_mem_attend_kernel  softmax over the J endpoints per (token, head)
//   loop_mem_add_kernel     streams[t, s, :] += gate * delta[t, :]
#include "common.cuh"

namespace llmyb {
namespace {

constexpr int kNormThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red may still be read by a previous reduction
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) t += red[i];
  return t;
}

// One CTA per token: y = mean_s x[t, s, :] (width W), then LayerNorm with
// (w, b, eps) when w is non-null.  Two-pass mean / variance in fp32, as
// nn.LayerNorm computes them.
__global__ void __launch_bounds__(kNormThreads)
loop_mem_norm_kernel(const float* __restrict__ x, int64_t ld, int S, int W,
                     const float* __restrict__ w, const float* __restrict__ b, float eps,
                     float* __restrict__ y, int64_t y_ld) {
  extern __shared__ float row[];  // [W]
  __shared__ float red[kNormThreads / 32];
  const int64_t t = blockIdx.x;
  const float* xt = x + t * ld;
  const float inv_s = 1.0f / static_cast<float>(S);
  float sum = 0.f;
  for (int i = threadIdx.x; i < W; i += kNormThreads) {
    float v = 0.f;
    for (int s = 0; s < S; ++s) v += xt[static_cast<int64_t>(s) * W + i];
    v = S == 1 ? v : v * inv_s;
    row[i] = v;
    sum += v;
  }
  float* yt = y + t * y_ld;
  if (w == nullptr) {
    for (int i = threadIdx.x; i < W; i += kNormThreads) yt[i] = row[i];
    return;
  }
  const float mu = block_sum(sum, red) / static_cast<float>(W);
  float sq = 0.f;
  for (int i = threadIdx.x; i < W; i += kNormThreads) {
    const float d = row[i] - mu;
    sq += d * d;
  }
  const float var = block_sum(sq, red) / static_cast<float>(W);
  const float r = rsqrtf(var + eps);
  for (int i = threadIdx.x; i < W; i += kNormThreads)
    yt[i] = (row[i] - mu) * r * w[i] + (b ? b[i] : 0.f);
}

// One warp per (token, head).  q [N, H*hd]; kv [J, N, 2*H*hd] (k of the head
// at h*hd, v at H*hd + h*hd); out [N, H*hd].  Scores and softmax in fp32 over
// the J <= 16 endpoints, held in registers.
constexpr int kMaxMem = 16;

__global__ void loop_mem_attend_kernel(const float* __restrict__ q, const float* __restrict__ kv,
                                       int N, int J, int H, int hd, float scale,
                                       float* __restrict__ out) {
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= static_cast<int64_t>(N) * H) return;
  const int64_t t = gw / H;
  const int h = static_cast<int>(gw - t * H);
  const int width = H * hd;
  const float* qt = q + t * width + h * hd;
  float s[kMaxMem];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < kMaxMem; ++j) {
    if (j < J) {
      const float* kt = kv + (static_cast<int64_t>(j) * N + t) * 2 * width + h * hd;
      float acc = 0.f;
      for (int i = lane; i < hd; i += 32) acc += qt[i] * kt[i];
      s[j] = warp_sum(acc) * scale;
      m = fmaxf(m, s[j]);
    }
  }
  float den = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxMem; ++j) {
    if (j < J) {
      s[j] = expf(s[j] - m);
      den += s[j];
    }
  }
  const float inv = 1.0f / den;
  float* ot = out + t * width + h * hd;
  for (int i = lane; i < hd; i += 32) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxMem; ++j) {
      if (j < J) acc += s[j] * kv[(static_cast<int64_t>(j) * N + t) * 2 * width + width + h * hd + i];
    }
    ot[i] = acc * inv;
  }
}

// streams [N, S*D] += gate * delta [N, D] broadcast over the S streams,
// float4 vectors (D % 4 == 0).
__global__ void loop_mem_add_kernel(float* __restrict__ streams, int64_t N, int S, int D,
                                    const float* __restrict__ delta, float gate) {
  const int dv = D / 4;
  const int64_t total = N * S * dv;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / (static_cast<int64_t>(S) * dv);
    const int c = static_cast<int>(i % dv);
    float4 a = reinterpret_cast<float4*>(streams)[i];
    const float4 d = reinterpret_cast<const float4*>(delta)[t * dv + c];
    a.x += gate * d.x;
    a.y += gate * d.y;
    a.z += gate * d.z;
    a.w += gate * d.w;
    reinterpret_cast<float4*>(streams)[i] = a;
  }
}

int grid_for(int64_t work, int threads) {
  const int64_t blocks = ceil_div(work, threads);
  return static_cast<int>(blocks < 8 * 148 ? (blocks > 0 ? blocks : 1) : 8 * 148);
}

}  // namespace
}  // namespace llmyb

using namespace llmyb;

// y[t] = mean over the S streams of x[t] (x rows of S*width floats at stride
// ld), then LayerNorm(ln_w, ln_b, eps) when ln_w is non-null (ln_b nullable).
LLMYB_API int32_t llmyb_loop_mem_norm(const float* x, int64_t ld, int32_t n_tokens,
                                      int32_t n_streams, int32_t width, const float* ln_w,
                                      const float* ln_b, float eps, float* y, int64_t y_ld,
                                      void* stream) {
  if (n_tokens < 0 || n_streams <= 0 || width <= 0 || ld < static_cast<int64_t>(n_streams) * width ||
      y_ld < width)
    return LLMYB_EINVAL;
  if (n_tokens == 0) return LLMYB_OK;
  if (!x || !y) return LLMYB_EINVAL;
  const int bytes = width * 4;
  if (bytes > 96 * 1024) return LLMYB_EUNSUPPORTED;
  if (bytes > 48 * 1024) {
    int32_t st = ensure_smem(loop_mem_norm_kernel, bytes);
    if (st) return st;
  }
  loop_mem_norm_kernel<<<n_tokens, kNormThreads, bytes, static_cast<cudaStream_t>(stream)>>>(
      x, ld, n_streams, width, ln_w, ln_b, eps, y, y_ld);
  count_launch();
  return launch_status();
}

// out [N, H*hd] = per (token, head) softmax over the n_mem endpoints of
// q . k / sqrt(hd), times v; kv [n_mem, N, 2*H*hd] (k rows then v rows of
// each endpoint's projection).  n_mem <= 16.
LLMYB_API int32_t llmyb_loop_mem_attend(const float* q, const float* kv, int32_t n_tokens,
                                        int32_t n_mem, int32_t heads, int32_t head_dim,
                                        float* out, void* stream) {
  if (n_tokens < 0 || n_mem <= 0 || heads <= 0 || head_dim <= 0) return LLMYB_EINVAL;
  if (n_mem > kMaxMem) return LLMYB_EUNSUPPORTED;
  if (n_tokens == 0) return LLMYB_OK;
  if (!q || !kv || !out) return LLMYB_EINVAL;
  const int64_t warps = static_cast<int64_t>(n_tokens) * heads;
  loop_mem_attend_kernel<<<static_cast<int>(ceil_div(warps * 32, 256)), 256, 0,
                           static_cast<cudaStream_t>(stream)>>>(
      q, kv, n_tokens, n_mem, heads, head_dim, 1.0f / sqrtf(static_cast<float>(head_dim)), out);
  count_launch();
  return launch_status();
}

// streams [N, S*D] fp32 += gate * delta [N, D] fp32 on every stream.
LLMYB_API int32_t llmyb_loop_mem_add(float* streams, int32_t n_tokens, int32_t n_streams,
                                     int32_t d_model, const float* delta, float gate,
                                     void* stream) {
  if (n_tokens < 0 || n_streams <= 0 || d_model <= 0) return LLMYB_EINVAL;
  if (n_tokens == 0) return LLMYB_OK;
  if (!streams || !delta) return LLMYB_EINVAL;
  if (d_model % 4 != 0 || (reinterpret_cast<uintptr_t>(streams) & 15u) ||
      (reinterpret_cast<uintptr_t>(delta) & 15u))
    return LLMYB_EUNSUPPORTED;
  const int64_t work = static_cast<int64_t>(n_tokens) * n_streams * (d_model / 4);
  loop_mem_add_kernel<<<grid_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      streams, n_tokens, n_streams, d_model, delta, gate);
  count_launch();
  return launch_status();
}
