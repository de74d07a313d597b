// Multi-stream hyper-connections (model/layers/mhc.py:52-229) around each
// sub-layer of a block: S live residual streams per token, fp32 [N, S*D]
// (stream s of token n at n*S*D + s*D).  Per sub-layer:
//
//   read  (mhc.py:135-156, :193-206): the input-dependent maps from
//         flat = RMSNorm_{S*D}(streams) (mapping_norm, eps = fp32 epsilon)
//         and logits = theta flat (2S + S*S values):
//           pre  = sigmoid(alpha_pre * logits[0:S] + pre_bias)
//           post = 2 sigmoid(alpha_post * logits[S:2S] + post_bias)
//           res  = Sinkhorn(alpha_res * logits[2S:].view(S,S) + residual_bias)
//         then hidden = LayerNorm(sum_s pre[s] streams[s]) (stream_norm,
//         eps 1e-5) and the block's RMSNorm of hidden (mixer_norm / ffn_norm)
//         as the sub-layer input.
//   write (mhc.py:208-229): streams[i] += g * scale[i] *
//         (sum_j res[i,j] streams[j] + post[i] * update), g = sigmoid(gating).
//
// theta is applied by the caller as one fp32 GEMM over the raw streams with the
// mapping-norm weight folded into its columns (theta * w); this kernel scales
// those products by the token's RMS factor.  The maps of a read are kept
// ([N, 2S+S*S]: pre | post | res row-major) for the write that follows the
// sub-layer.
#include <cfloat>
#include <cstdint>

#include "common.cuh"

namespace llmyb {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxChunks = 4;  // float4 chunks per thread and stream: D <= 4096

template <int S>
__host__ __device__ constexpr int n_maps() {
  return 2 * S + S * S;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();  // red may still be read by a previous reduction
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) t += red[i];
  return t;
}

// update[d..d+3] of token n: the bf16 delta row, or the fp32 sum of the k
// routed expert rows delta[route_pos[n*k + s]] in slot order.
__device__ __forceinline__ float4 load_update(const __nv_bfloat16* __restrict__ delta,
                                              const int* __restrict__ route_pos, int k,
                                              int64_t n, int D, int d) {
  float4 u = make_float4(0.f, 0.f, 0.f, 0.f);
  if (delta == nullptr) return u;
  const int rows = route_pos != nullptr ? k : 1;
  for (int s = 0; s < rows; ++s) {
    const int64_t row = route_pos != nullptr ? __ldg(route_pos + n * k + s) : n;
    const uint2 raw = __ldg(reinterpret_cast<const uint2*>(delta + row * D + d));
    const float2 a = unpack_bf16x2(raw.x), b = unpack_bf16x2(raw.y);
    u.x += a.x;
    u.y += a.y;
    u.z += b.x;
    u.w += b.y;
  }
  return u;
}

template <int S>
__global__ void __launch_bounds__(kThreads) mhc_write_kernel(
    float* __restrict__ streams, const __nv_bfloat16* __restrict__ delta,
    const int* __restrict__ route_pos, int k, int D, const float* __restrict__ maps,
    const float* __restrict__ scale, const float* __restrict__ scalars) {
  constexpr int M = n_maps<S>();
  __shared__ float mp[M];
  const int64_t n = blockIdx.x;
  if (threadIdx.x < M) mp[threadIdx.x] = __ldg(maps + n * M + threadIdx.x);
  __syncthreads();
  const float g = __ldg(scalars + 3);
  float* x = streams + n * S * D;
  for (int d = threadIdx.x * 4; d < D; d += kThreads * 4) {
    const float4 u = load_update(delta, route_pos, k, n, D, d);
    float4 st[S];
#pragma unroll
    for (int i = 0; i < S; ++i) st[i] = *reinterpret_cast<const float4*>(x + i * D + d);
#pragma unroll
    for (int i = 0; i < S; ++i) {
      float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < S; ++j) {
        const float c = mp[2 * S + i * S + j];
        r.x = fmaf(c, st[j].x, r.x);
        r.y = fmaf(c, st[j].y, r.y);
        r.z = fmaf(c, st[j].z, r.z);
        r.w = fmaf(c, st[j].w, r.w);
      }
      const float p = mp[S + i];
      const float4 sc = __ldg(reinterpret_cast<const float4*>(scale + i * D + d));
      float4 o;
      o.x = st[i].x + g * ((r.x + p * u.x) * sc.x);
      o.y = st[i].y + g * ((r.y + p * u.y) * sc.y);
      o.z = st[i].z + g * ((r.z + p * u.z) * sc.z);
      o.w = st[i].w + g * ((r.w + p * u.w) * sc.w);
      *reinterpret_cast<float4*>(x + i * D + d) = o;
    }
  }
}

// log-sum-exp over a group of W consecutive lanes (W | 32), lane stride 1
template <int W>
__device__ __forceinline__ float group_lse_rows(float v) {
  float m = v;
#pragma unroll
  for (int o = 1; o < W; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float e = expf(v - m);
#pragma unroll
  for (int o = 1; o < W; o <<= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
  return m + logf(e);
}

// log-sum-exp over the W lanes lane % W == const within a W*W group
template <int W>
__device__ __forceinline__ float group_lse_cols(float v) {
  float m = v;
#pragma unroll
  for (int o = W; o < W * W; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float e = expf(v - m);
#pragma unroll
  for (int o = W; o < W * W; o <<= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
  return m + logf(e);
}

// C = float4 chunks per thread and stream (D <= 1024 C): the streams of the
// token stay in registers across the reductions.  raw logits of token n, map
// o at raw[n * raw_tok + o * raw_map] (either GEMM orientation).
template <int S, int C>
__global__ void __launch_bounds__(kThreads) mhc_read_kernel(
    const float* __restrict__ streams, const float* __restrict__ raw, int64_t raw_tok,
    int64_t raw_map, const float* __restrict__ bias, const float* __restrict__ scalars,
    const float* __restrict__ ln_w, const float* __restrict__ ln_b,
    const float* __restrict__ norm_w, float rms_eps, int iters, int D,
    float* __restrict__ maps, __nv_bfloat16* __restrict__ out_bf16, float* __restrict__ out_f32) {
  constexpr int M = n_maps<S>();
  __shared__ float red[kThreads / 32];
  __shared__ float pre_s[S];
  const int64_t n = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31;
  const float* x = streams + n * S * D;

  float4 st[S][C];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int d = (tid + c * kThreads) * 4;
#pragma unroll
    for (int s = 0; s < S; ++s) {
      st[s][c] = d < D ? *reinterpret_cast<const float4*>(x + s * D + d)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
      ss += st[s][c].x * st[s][c].x + st[s][c].y * st[s][c].y + st[s][c].z * st[s][c].z +
            st[s][c].w * st[s][c].w;
    }
  }
  const float r = rsqrtf(block_sum(ss, red) / static_cast<float>(S * D) + FLT_EPSILON);

  if (tid < 32) {
    const float* lg = raw + n * raw_tok;
    // pre / post: lanes [0, 2S)
    if (lane < 2 * S) {
      const bool is_pre = lane < S;
      const float z = __ldg(scalars + (is_pre ? 0 : 1)) * (r * __ldg(lg + lane * raw_map)) +
                      __ldg(bias + lane);
      const float v = is_pre ? sigmoidf_(z) : 2.0f * sigmoidf_(z);
      maps[n * M + lane] = v;
      if (is_pre) pre_s[lane] = v;
    }
    // residual map: lane q < S*S holds entry (q / S, q % S); Sinkhorn in the
    // log domain, rows then columns per iteration (mhc.py:12-17)
    float a = 0.f;
    if (lane < S * S)
      a = __ldg(scalars + 2) * (r * __ldg(lg + (2 * S + lane) * raw_map)) +
          __ldg(bias + 2 * S + lane);
    for (int it = 0; it < iters; ++it) {
      a -= group_lse_rows<S>(a);
      a -= group_lse_cols<S>(a);
    }
    if (lane < S * S) maps[n * M + 2 * S + lane] = expf(a);
  }
  __syncthreads();

  // hidden = LayerNorm(sum_s pre[s] streams[s])
  float pre[S];
#pragma unroll
  for (int s = 0; s < S; ++s) pre[s] = pre_s[s];
  float4 v[C];
  float sum = 0.f;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int s = 0; s < S; ++s) {
      acc.x = fmaf(pre[s], st[s][c].x, acc.x);
      acc.y = fmaf(pre[s], st[s][c].y, acc.y);
      acc.z = fmaf(pre[s], st[s][c].z, acc.z);
      acc.w = fmaf(pre[s], st[s][c].w, acc.w);
    }
    v[c] = acc;
    sum += acc.x + acc.y + acc.z + acc.w;  // zero beyond D
  }
  const float mean = block_sum(sum, red) / static_cast<float>(D);
  float var = 0.f;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    if ((tid + c * kThreads) * 4 < D) {
      const float a0 = v[c].x - mean, a1 = v[c].y - mean, a2 = v[c].z - mean, a3 = v[c].w - mean;
      var += a0 * a0 + a1 * a1 + a2 * a2 + a3 * a3;
    }
  }
  const float rstd = rsqrtf(block_sum(var, red) / static_cast<float>(D) + 1e-5f);
  float hs = 0.f;
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int d = (tid + c * kThreads) * 4;
    if (d < D) {
      const float4 w = __ldg(reinterpret_cast<const float4*>(ln_w + d));
      const float4 b = __ldg(reinterpret_cast<const float4*>(ln_b + d));
      v[c].x = (v[c].x - mean) * rstd * w.x + b.x;
      v[c].y = (v[c].y - mean) * rstd * w.y + b.y;
      v[c].z = (v[c].z - mean) * rstd * w.z + b.z;
      v[c].w = (v[c].w - mean) * rstd * w.w + b.w;
      hs += v[c].x * v[c].x + v[c].y * v[c].y + v[c].z * v[c].z + v[c].w * v[c].w;
    }
  }
  // the block's RMSNorm of the read value
  const float rn = rsqrtf(block_sum(hs, red) / static_cast<float>(D) + rms_eps);
#pragma unroll
  for (int c = 0; c < C; ++c) {
    const int d = (tid + c * kThreads) * 4;
    if (d < D) {
      float4 w = make_float4(1.f, 1.f, 1.f, 1.f);
      if (norm_w != nullptr) w = __ldg(reinterpret_cast<const float4*>(norm_w + d));
      const float4 y = make_float4(v[c].x * rn * w.x, v[c].y * rn * w.y, v[c].z * rn * w.z,
                                   v[c].w * rn * w.w);
      if (out_f32 != nullptr) *reinterpret_cast<float4*>(out_f32 + n * D + d) = y;
      if (out_bf16 != nullptr)
        *reinterpret_cast<uint2*>(out_bf16 + n * D + d) =
            make_uint2(pack_bf16x2(y.x, y.y), pack_bf16x2(y.z, y.w));
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace llmyb

using namespace llmyb;

LLMYB_API int32_t llmyb_mhc_write(float* streams, int32_t n_tokens, int32_t n_streams,
                                  int32_t d_model, const void* delta, const int32_t* route_pos,
                                  int32_t top_k, const float* maps, const float* stream_scale,
                                  const float* scalars, void* stream) {
  if (n_tokens < 0 || d_model <= 0 || (route_pos != nullptr && top_k <= 0)) return LLMYB_EINVAL;
  if (n_tokens == 0) return LLMYB_OK;
  if (!streams || !maps || !stream_scale || !scalars) return LLMYB_EINVAL;
  if (d_model % 4 != 0 || !aligned16(streams) || !aligned16(stream_scale) ||
      (delta != nullptr && (reinterpret_cast<uintptr_t>(delta) & 7u) != 0))
    return LLMYB_EINVAL;
  const auto* dl = static_cast<const __nv_bfloat16*>(delta);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (n_streams) {
    case 1:
      mhc_write_kernel<1><<<n_tokens, kThreads, 0, s>>>(streams, dl, route_pos, top_k, d_model,
                                                        maps, stream_scale, scalars);
      break;
    case 2:
      mhc_write_kernel<2><<<n_tokens, kThreads, 0, s>>>(streams, dl, route_pos, top_k, d_model,
                                                        maps, stream_scale, scalars);
      break;
    case 4:
      mhc_write_kernel<4><<<n_tokens, kThreads, 0, s>>>(streams, dl, route_pos, top_k, d_model,
                                                        maps, stream_scale, scalars);
      break;
    default:
      return LLMYB_EUNSUPPORTED;
  }
  count_launch();
  return launch_status();
}

namespace {
template <int S>
void launch_read(int32_t n, int32_t D, const float* streams, const float* raw, int64_t raw_tok,
                 int64_t raw_map, const float* bias, const float* scalars, const float* ln_w,
                 const float* ln_b, const float* norm_w, float eps, int32_t iters, float* maps,
                 __nv_bfloat16* ob, float* of, cudaStream_t s) {
  const int c = (D + kThreads * 4 - 1) / (kThreads * 4);
#define LLMYB_MHC_READ(C_)                                                                   \
  mhc_read_kernel<S, C_><<<n, kThreads, 0, s>>>(streams, raw, raw_tok, raw_map, bias, scalars, \
                                                ln_w, ln_b, norm_w, eps, iters, D, maps, ob, of)
  if (c <= 1)
    LLMYB_MHC_READ(1);
  else if (c <= 2)
    LLMYB_MHC_READ(2);
  else
    LLMYB_MHC_READ(4);
#undef LLMYB_MHC_READ
}
}  // namespace

LLMYB_API int32_t llmyb_mhc_read(const float* streams, int32_t n_tokens, int32_t n_streams,
                                 int32_t d_model, const float* raw, int64_t raw_tok,
                                 int64_t raw_map, const float* bias,
                                 const float* scalars, const float* ln_w, const float* ln_b,
                                 const float* norm_w, float rms_eps, int32_t iterations,
                                 float* maps, void* out_bf16, float* out_f32, void* stream) {
  if (n_tokens < 0 || d_model <= 0 || iterations < 0) return LLMYB_EINVAL;
  if (n_tokens == 0) return LLMYB_OK;
  if (!streams || !raw || !bias || !scalars || !ln_w || !ln_b || !maps) return LLMYB_EINVAL;
  if (d_model % 4 != 0 || d_model > kThreads * 4 * kMaxChunks) return LLMYB_EUNSUPPORTED;
  if (!aligned16(streams) || !aligned16(ln_w) || !aligned16(ln_b) ||
      (norm_w != nullptr && !aligned16(norm_w)) || (out_f32 != nullptr && !aligned16(out_f32)) ||
      (out_bf16 != nullptr && (reinterpret_cast<uintptr_t>(out_bf16) & 7u) != 0))
    return LLMYB_EINVAL;
  auto* ob = static_cast<__nv_bfloat16*>(out_bf16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (n_streams) {
    case 1:
      launch_read<1>(n_tokens, d_model, streams, raw, raw_tok, raw_map, bias, scalars, ln_w, ln_b,
                     norm_w, rms_eps, iterations, maps, ob, out_f32, s);
      break;
    case 2:
      launch_read<2>(n_tokens, d_model, streams, raw, raw_tok, raw_map, bias, scalars, ln_w, ln_b,
                     norm_w, rms_eps, iterations, maps, ob, out_f32, s);
      break;
    case 4:
      launch_read<4>(n_tokens, d_model, streams, raw, raw_tok, raw_map, bias, scalars, ln_w, ln_b,
                     norm_w, rms_eps, iterations, maps, ob, out_f32, s);
      break;
    default:
      return LLMYB_EUNSUPPORTED;
  }
  count_launch();
  return launch_status();
}
