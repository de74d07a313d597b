// Fused decode-step kernels for small batches (up to 8 tokens).
//
// A batch-1 decode step of the looped hybrid stack is a chain of a few
// hundred dependent launches of a few microseconds each: the time goes to
// launch gaps and global-memory round trips, not to bytes.  Per block these
// two kernels replace four or five launches of the unfused path:
//
//   [A] llmyb_decode_norm_gemv   residual add (+ the routed MoE combine of the
//                                previous block) and RMSNorm, recomputed by
//                                every CTA for its own use, then the block's
//                                input projection GEMV (one warp per row)
//   [B] mixer                    gdn_step / csa_local_decode
//   [C] llmyb_decode_out_router  output projection GEMV (+ the GDN conv gate
//                                for its columns) by all CTAs; the last CTA to
//                                finish adds the result to the residual
//                                stream and runs the router and the plan
//   [D],[E] routed experts       moe_decode up / down
//
// Reference: PhysicalBlock.forward_step (model/model.py:214-241), the GDN
// conv gate (model/layers/gated_deltanet.py:257-268), CSA's output path
// (model/layers/csa.py:132) and ContextAwareRouter (context_router.py:62-74).
// The norms reproduce llmyb_add_rmsnorm's vector kernel and the router phase
// runs the routines of router.cu, so both give the values of the unfused path
// for the same inputs; the projections are warp-per-row GEMVs (fp32 sums of
// bf16 products, bf16 outputs like the cuBLAS GEMMs they replace).
#include <cooperative_groups.h>

#include "common.cuh"
#include "router_device.cuh"

#include <algorithm>

namespace cg = cooperative_groups;

namespace llmyb {
namespace {

using namespace rdev;

constexpr int kMaxTokens = 8;

// One weight row (bf16, K = 256*KCH at most, K % 8 == 0) into registers:
// lane holds 16-byte chunks lane, lane+32, ...  Issued at kernel entry, so
// the weight round trip overlaps the preparation of the input rows.
template <int KCH>
__device__ __forceinline__ void warp_load_row(const __nv_bfloat16* __restrict__ wrow, int K,
                                              int lane, uint4 (&w)[KCH]) {
  const int nch = K >> 3;
#pragma unroll
  for (int i = 0; i < KCH; ++i) {
    const int c = lane + 32 * i;
    if (c < nch) w[i] = __ldg(reinterpret_cast<const uint4*>(wrow) + c);
  }
}

// Dot products of the loaded row with the B bf16 rows of s_x [B][K] (shared
// memory), summed over the warp: every lane returns the B sums.
template <int BM, int KCH>
__device__ __forceinline__ void warp_row_dot(const uint4 (&w)[KCH], int K, int B,
                                             const __nv_bfloat16* s_x, int lane, float (&acc)[BM]) {
  const int nch = K >> 3;
#pragma unroll
  for (int b = 0; b < BM; ++b) acc[b] = 0.f;
#pragma unroll
  for (int i = 0; i < KCH; ++i) {
    const int c = lane + 32 * i;
    if (c >= nch) continue;
    const uint32_t ww[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
    for (int b = 0; b < BM; ++b) {
      if (b >= B) break;
      const uint4 x4 = reinterpret_cast<const uint4*>(s_x + b * K)[c];
      const uint32_t xx[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 wf = unpack_bf16x2(ww[e]);
        const float2 xf = unpack_bf16x2(xx[e]);
        acc[b] += wf.x * xf.x + wf.y * xf.y;
      }
    }
  }
#pragma unroll
  for (int b = 0; b < BM; ++b) acc[b] = warp_sum(acc[b]);
}

// Residual add + RMSNorm of token row b into s_x (bf16), by a CTA of 256
// threads with 8-element vectors (D <= 2048): the arithmetic of
// add_rmsnorm_vec_kernel<1> (norm.cu).  CTA 0 also stores the updated
// residual row and the normalised row.
__device__ __forceinline__ void cta_add_norm_row(
    const float* __restrict__ streams_in, const __nv_bfloat16* __restrict__ delta,
    const int* __restrict__ route_pos, int k, int b, int D, const float* __restrict__ weight,
    float eps, __nv_bfloat16* s_x, float* s_red, float* __restrict__ streams_out,
    __nv_bfloat16* __restrict__ normed_out, bool writer) {
  const int nv = D >> 3;
  const int c = threadIdx.x;
  float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float ss = 0.f;
  if (c < nv) {
    const float4* x4 = reinterpret_cast<const float4*>(streams_in + static_cast<int64_t>(b) * D);
    const float4 a = x4[2 * c], bb = x4[2 * c + 1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = bb.x; v[5] = bb.y; v[6] = bb.z; v[7] = bb.w;
    if (delta != nullptr) {
      if (route_pos != nullptr) {
        for (int s = 0; s < k; ++s) {
          const int64_t pos = __ldg(route_pos + static_cast<int64_t>(b) * k + s);
          const uint4 u = __ldg(reinterpret_cast<const uint4*>(delta + pos * D) + c);
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = unpack_bf16x2(w[q]);
            v[2 * q] += f.x;
            v[2 * q + 1] += f.y;
          }
        }
      } else {
        const uint4 u =
            __ldg(reinterpret_cast<const uint4*>(delta + static_cast<int64_t>(b) * D) + c);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = unpack_bf16x2(w[q]);
          v[2 * q] += f.x;
          v[2 * q + 1] += f.y;
        }
      }
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) ss += v[q] * v[q];
  }
  ss = warp_sum(ss);
  __syncthreads();  // earlier readers of s_red are done
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += s_red[i];
  const float r = rsqrtf(tot / static_cast<float>(D) + eps);
  if (c < nv) {
    const float4 wa = __ldg(reinterpret_cast<const float4*>(weight) + 2 * c);
    const float4 wb = __ldg(reinterpret_cast<const float4*>(weight) + 2 * c + 1);
    const float w8[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
    float y[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) y[q] = v[q] * r * w8[q];
    uint4 o;
    o.x = pack_bf16x2(y[0], y[1]);
    o.y = pack_bf16x2(y[2], y[3]);
    o.z = pack_bf16x2(y[4], y[5]);
    o.w = pack_bf16x2(y[6], y[7]);
    reinterpret_cast<uint4*>(s_x + b * D)[c] = o;
    if (writer) {
      float4* so = reinterpret_cast<float4*>(streams_out + static_cast<int64_t>(b) * D);
      so[2 * c] = make_float4(v[0], v[1], v[2], v[3]);
      so[2 * c + 1] = make_float4(v[4], v[5], v[6], v[7]);
      if (normed_out != nullptr)
        reinterpret_cast<uint4*>(normed_out + static_cast<int64_t>(b) * D)[c] = o;
    }
  }
}

// [A] out[b, n] = W[n, :] . RMSNorm(streams_in[b] + delta[b]) for the CTA's
// 8 rows (one per warp).
template <int BM, int KCH>
__global__ void __launch_bounds__(256) decode_norm_gemv_kernel(
    const float* __restrict__ streams_in, const __nv_bfloat16* __restrict__ delta,
    const int* __restrict__ route_pos, int k, int B, int D, const float* __restrict__ norm_w,
    float eps, const __nv_bfloat16* __restrict__ W, int N, __nv_bfloat16* __restrict__ out,
    int64_t out_ld, float* __restrict__ streams_out, __nv_bfloat16* __restrict__ normed_out) {
  extern __shared__ __align__(16) uint8_t smem_a[];
  __shared__ float s_red[8];
  __nv_bfloat16* s_x = reinterpret_cast<__nv_bfloat16*>(smem_a);  // [B][D]
  const int lane = threadIdx.x & 31;
  const int n = blockIdx.x * 8 + (threadIdx.x >> 5);
  uint4 w[KCH];
  if (n < N) warp_load_row<KCH>(W + static_cast<int64_t>(n) * D, D, lane, w);
  pdl_wait();  // the residual stream and the routed rows come from earlier kernels
  pdl_trigger();
  const bool writer = blockIdx.x == 0;
  for (int b = 0; b < B; ++b)
    cta_add_norm_row(streams_in, delta, route_pos, k, b, D, norm_w, eps, s_x, s_red, streams_out,
                     normed_out, writer);
  __syncthreads();
  if (n >= N) return;  // whole warps
  float acc[BM];
  warp_row_dot<BM, KCH>(w, D, B, s_x, lane, acc);
  if (lane == 0)
#pragma unroll
    for (int b = 0; b < BM; ++b)
      if (b < B) out[b * out_ld + n] = f2bf(acc[b]);
}

// [C] mixed[b, d] = W[d, :] . in[b] (bf16), with the GDN conv gate applied
// per column when conv_w is given, and streams += mixed, by the CTA owning
// column d.  The router input r = RMSNorm_rn(RMSNorm_ffn(x)) is a per-token
// scaling of x (x = the updated residual row):
//   inv1 = rsqrt(sum(x^2)/D + eps), inv2 = rsqrt(inv1^2 sum((x ffn_w)^2)/D + eps),
//   logits[e] = inv1 inv2 sum_d w_fold[e, d] x[d],   w_fold = W_r * ffn_w * rn_w,
// so every CTA adds its columns' share of the two sums of squares and of the E
// logits to `partials` [grid][B][2+E]; the last CTA to finish sums them in CTA
// order, forms m_bf = x inv1 ffn_w and runs top-k and the plan (one warp).
template <int BM, int KCH>
__global__ void __launch_bounds__(256) decode_out_router_kernel(
    const __nv_bfloat16* __restrict__ in, int64_t in_ld, int K, const __nv_bfloat16* __restrict__ W,
    int B, int D, const float* __restrict__ conv_w, const __nv_bfloat16* __restrict__ normed,
    __nv_bfloat16* history, float* __restrict__ partials, int* counter,
    float* __restrict__ streams, const float* __restrict__ ffn_w,
    const float* __restrict__ w_fold, float eps, int E, int top_k, int tile_m,
    __nv_bfloat16* __restrict__ m_bf, int64_t* __restrict__ topk_idx,
    float* __restrict__ topk_prob, int* __restrict__ counts, int* __restrict__ offsets,
    int* __restrict__ tile_offsets, int* __restrict__ perm_token, float* __restrict__ perm_prob,
    int* __restrict__ route_pos) {
  extern __shared__ __align__(16) uint8_t smem_c[];
  __shared__ float s_x[kMaxTokens][8];
  __shared__ int s_idx[kMaxTokens * kMaxTopK];
  __shared__ float s_prob[kMaxTokens * kMaxTopK];
  __shared__ int s_cnt[kMaxExperts];
  __shared__ float s_scale[kMaxTokens][2];
  __shared__ int s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int n = blockIdx.x * 8 + warp;
  const int NV = 2 + E;
  uint4 w[KCH];
  if (n < D) warp_load_row<KCH>(W + static_cast<int64_t>(n) * K, K, lane, w);
  pdl_wait();  // the projection input comes from the mixer kernel
  pdl_trigger();
  // ---- output projection rows of this CTA
  __nv_bfloat16* s_in = reinterpret_cast<__nv_bfloat16*>(smem_c);  // [B][K]
  for (int i = threadIdx.x; i < B * (K >> 3); i += 256) {
    const int b = i / (K >> 3), c = i - b * (K >> 3);
    reinterpret_cast<uint4*>(s_in + b * K)[c] =
        __ldg(reinterpret_cast<const uint4*>(in + b * in_ld) + c);
  }
  if (threadIdx.x < kMaxTokens * 8) s_x[threadIdx.x >> 3][threadIdx.x & 7] = 0.f;
  __syncthreads();
  if (n < D) {
    float acc[BM];
    warp_row_dot<BM, KCH>(w, K, B, s_in, lane, acc);
    if (lane < B) {
      float y = 0.f;
#pragma unroll
      for (int b = 0; b < BM; ++b)
        if (b == lane) y = acc[b];
      const int b = lane;
      float yv = bf2f(f2bf(y));  // the projection output is bf16
      if (conv_w != nullptr) {
        // conv gate of the decode step (gdn_conv_gate_kernel with T == 1)
        __nv_bfloat16* hb = history + static_cast<int64_t>(b) * 3 * D + n;
        const __nv_bfloat16 xb = normed[static_cast<int64_t>(b) * D + n];
        const __nv_bfloat16 h0 = hb[0], h1 = hb[D], h2 = hb[2 * D];
        float cacc = 0.f;
        cacc += conv_w[n * 4 + 0] * bf2f(h0);
        cacc += conv_w[n * 4 + 1] * bf2f(h1);
        cacc += conv_w[n * 4 + 2] * bf2f(h2);
        cacc += conv_w[n * 4 + 3] * bf2f(xb);
        yv = yv * sigmoidf_(cacc);
        hb[0] = h1;
        hb[D] = h2;
        hb[2 * D] = xb;
      }
      // residual add with the bf16 sub-layer output (as llmyb_add_rmsnorm)
      float* sp = streams + static_cast<int64_t>(b) * D + n;
      const float x = *sp + bf2f(f2bf(yv));
      *sp = x;
      s_x[b][warp] = x;
    }
  }
  __syncthreads();
  // ---- this CTA's share of the sums of squares and of the logits
  for (int t = threadIdx.x; t < B * NV; t += 256) {
    const int b = t / NV, j = t - b * NV;
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int d = blockIdx.x * 8 + c;
      if (d >= D) break;
      const float x = s_x[b][c];
      if (j == 0) {
        acc += x * x;
      } else if (j == 1) {
        const float xf = x * __ldg(ffn_w + d);
        acc += xf * xf;
      } else {
        acc += __ldg(w_fold + static_cast<int64_t>(j - 2) * D + d) * x;
      }
    }
    partials[(static_cast<int64_t>(blockIdx.x) * B + b) * NV + j] = acc;
  }
  // ---- the last CTA to finish combines the shares and routes
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(counter, 1) == static_cast<int>(gridDim.x) - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float* s_tot = reinterpret_cast<float*>(smem_c);  // [B][NV]
  // one warp per value: lanes take every 32nd CTA, then a fixed xor tree
  for (int t = warp; t < B * NV; t += 8) {
    float acc = 0.f;
    for (int g = lane; g < static_cast<int>(gridDim.x); g += 32)
      acc += __ldcg(partials + static_cast<int64_t>(g) * B * NV + t);
    acc = warp_sum(acc);
    if (lane == 0) s_tot[t] = acc;
  }
  __syncthreads();
  if (threadIdx.x < B) {
    const int b = threadIdx.x;
    const float inv1 = rsqrtf(s_tot[b * NV] / static_cast<float>(D) + eps);
    const float inv2 = rsqrtf(inv1 * inv1 * s_tot[b * NV + 1] / static_cast<float>(D) + eps);
    s_scale[b][0] = inv1;
    s_scale[b][1] = inv1 * inv2;
  }
  __syncthreads();
  float* s_logits = s_tot + B * NV;  // [B][E]
  for (int t = threadIdx.x; t < B * E; t += 256) {
    const int b = t / E, e = t - b * E;
    s_logits[t] = s_scale[b][1] * s_tot[b * NV + 2 + e];
  }
  // m = x * inv1 * ffn_w (bf16), 4 columns per thread step
  for (int i = threadIdx.x; i < B * (D >> 2); i += 256) {
    const int b = i / (D >> 2), c = i - b * (D >> 2);
    const float4 x = __ldcg(reinterpret_cast<const float4*>(streams + static_cast<int64_t>(b) * D) + c);
    const float4 f = __ldg(reinterpret_cast<const float4*>(ffn_w) + c);
    const float inv1 = s_scale[b][0];
    reinterpret_cast<uint2*>(m_bf + static_cast<int64_t>(b) * D)[c] =
        make_uint2(pack_bf16x2(x.x * inv1 * f.x, x.y * inv1 * f.y),
                   pack_bf16x2(x.z * inv1 * f.z, x.w * inv1 * f.w));
  }
  __syncthreads();
  if (warp == 0)
    warp_topk_plan(s_logits, B, E, top_k, tile_m, s_idx, s_prob, s_cnt, topk_idx, topk_prob,
                   counts, offsets, tile_offsets, perm_token, perm_prob, route_pos, lane);
  if (threadIdx.x == 0) *counter = 0;  // ready for the next launch
}

// [C] as one cluster of 8 CTAs x 16 warps (residual widths D = 128 * RPW):
// the same per-column work, but every warp holds RPW weight rows in
// registers (loaded before the dependency wait, together with this CTA's
// slice of the folded router weights, the FFN norm weights, the conv taps
// and the residual rows), the CTAs' shares of the sums are combined through
// distributed shared memory in rank order (no global partials, fences or
// atomics), and every CTA writes m_bf for its own columns; CTA 0 routes.
constexpr int kOrCtas = 8, kOrWarps = 16;

template <int BM, int KCH, int RPW>
__global__ void __cluster_dims__(kOrCtas, 1, 1) __launch_bounds__(kOrWarps * 32, 1)
    decode_out_router_cluster_kernel(
        const __nv_bfloat16* __restrict__ in, int64_t in_ld, int K,
        const __nv_bfloat16* __restrict__ W, int B, int D, const float* __restrict__ conv_w,
        const __nv_bfloat16* __restrict__ normed, __nv_bfloat16* history,
        float* __restrict__ streams, const float* __restrict__ ffn_w,
        const float* __restrict__ w_fold, float eps, int E, int top_k, int tile_m,
        __nv_bfloat16* __restrict__ m_bf, int64_t* __restrict__ topk_idx,
        float* __restrict__ topk_prob, int* __restrict__ counts, int* __restrict__ offsets,
        int* __restrict__ tile_offsets, int* __restrict__ perm_token,
        float* __restrict__ perm_prob, int* __restrict__ route_pos) {
  constexpr int kCols = kOrWarps * RPW;  // residual columns of this CTA
  constexpr int kThreads = kOrWarps * 32;
  constexpr int kMaxNV = 2 + 64;         // B * E <= 64 on this path
  // dynamic: s_in [B][K] bf16 | s_wf [E][kCols] fp32
  extern __shared__ __align__(16) uint8_t smem_c[];
  __shared__ float s_x[kMaxTokens][kCols];      // updated residual (this CTA's columns)
  __shared__ float s_res[kMaxTokens][kCols];    // residual before the update
  __shared__ float s_tap[kMaxTokens][4][kCols]; // conv taps: history 0..2, normed
  __shared__ float s_conv[kCols][4];
  __shared__ float s_ffn[kCols];
  __shared__ float s_part[kMaxTokens * kMaxNV];  // this CTA's shares, read by the peers
  __shared__ float s_tot[kMaxTokens * kMaxNV];
  __shared__ float s_logits[64];
  __shared__ float s_scale[kMaxTokens][2];
  __shared__ int s_idx[kMaxTokens * kMaxTopK];
  __shared__ float s_prob[kMaxTokens * kMaxTopK];
  __shared__ int s_cnt[kMaxExperts];
  cg::cluster_group cluster = cg::this_cluster();
  const int cta = static_cast<int>(cluster.block_rank());
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c0 = cta * kCols;
  const int NV = 2 + E;
  __nv_bfloat16* s_in = reinterpret_cast<__nv_bfloat16*>(smem_c);
  float* s_wf = reinterpret_cast<float*>(smem_c + ((B * K * 2 + 15) & ~15));

  // ---- before the dependency wait: weights, and buffers written two or more
  // launches earlier (the residual and the normalised input by [A], history)
  uint4 w[RPW][KCH];
#pragma unroll
  for (int r = 0; r < RPW; ++r)
    warp_load_row<KCH>(W + static_cast<int64_t>(c0 + warp * RPW + r) * K, K, lane, w[r]);
  for (int i = threadIdx.x; i < E * kCols; i += kThreads) {
    const int e = i / kCols, c = i - e * kCols;
    s_wf[i] = __ldg(w_fold + static_cast<int64_t>(e) * D + c0 + c);
  }
  for (int c = threadIdx.x; c < kCols; c += kThreads) {
    s_ffn[c] = __ldg(ffn_w + c0 + c);
    if (conv_w != nullptr)
#pragma unroll
      for (int j = 0; j < 4; ++j) s_conv[c][j] = __ldg(conv_w + (c0 + c) * 4 + j);
  }
  for (int i = threadIdx.x; i < B * kCols; i += kThreads) {
    const int b = i / kCols, c = i - b * kCols;
    const int64_t o = static_cast<int64_t>(b) * D + c0 + c;
    s_res[b][c] = streams[o];
    if (conv_w != nullptr) {
      const __nv_bfloat16* hb = history + static_cast<int64_t>(b) * 3 * D + c0 + c;
      s_tap[b][0][c] = bf2f(hb[0]);
      s_tap[b][1][c] = bf2f(hb[D]);
      s_tap[b][2][c] = bf2f(hb[2 * D]);
      s_tap[b][3][c] = bf2f(normed[o]);
    }
  }
  pdl_wait();  // the projection input comes from the mixer kernel
  pdl_trigger();
  for (int i = threadIdx.x; i < B * (K >> 3); i += kThreads) {
    const int b = i / (K >> 3), c = i - b * (K >> 3);
    reinterpret_cast<uint4*>(s_in + b * K)[c] =
        __ldg(reinterpret_cast<const uint4*>(in + b * in_ld) + c);
  }
  __syncthreads();
  // ---- output projection rows (+ conv gate) and the residual update
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int c = warp * RPW + r, n = c0 + c;
    float acc[BM];
    warp_row_dot<BM, KCH>(w[r], K, B, s_in, lane, acc);
    if (lane < B) {
      float y = 0.f;
#pragma unroll
      for (int b = 0; b < BM; ++b)
        if (b == lane) y = acc[b];
      const int b = lane;
      float yv = bf2f(f2bf(y));  // the projection output is bf16
      if (conv_w != nullptr) {
        float cacc = 0.f;
        cacc += s_conv[c][0] * s_tap[b][0][c];
        cacc += s_conv[c][1] * s_tap[b][1][c];
        cacc += s_conv[c][2] * s_tap[b][2][c];
        cacc += s_conv[c][3] * s_tap[b][3][c];
        yv = yv * sigmoidf_(cacc);
        __nv_bfloat16* hb = history + static_cast<int64_t>(b) * 3 * D + n;
        hb[0] = f2bf(s_tap[b][1][c]);
        hb[D] = f2bf(s_tap[b][2][c]);
        hb[2 * D] = f2bf(s_tap[b][3][c]);
      }
      const float x = s_res[b][c] + bf2f(f2bf(yv));
      streams[static_cast<int64_t>(b) * D + n] = x;
      s_x[b][c] = x;
    }
  }
  __syncthreads();
  // ---- this CTA's shares: one warp per (token, value), lanes over columns
  for (int t = warp; t < B * NV; t += kOrWarps) {
    const int b = t / NV, j = t - b * NV;
    float acc = 0.f;
    for (int c = lane; c < kCols; c += 32) {
      const float x = s_x[b][c];
      if (j == 0) {
        acc += x * x;
      } else if (j == 1) {
        const float xf = x * s_ffn[c];
        acc += xf * xf;
      } else {
        acc += s_wf[(j - 2) * kCols + c] * x;
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) s_part[t] = acc;
  }
  cluster.sync();
  // ---- every CTA sums the shares in rank order (the same totals everywhere)
  for (int t = threadIdx.x; t < B * NV; t += kThreads) {
    float acc = 0.f;
    for (int q = 0; q < kOrCtas; ++q) acc += cluster.map_shared_rank(s_part, q)[t];
    s_tot[t] = acc;
  }
  __syncthreads();
  if (threadIdx.x < B) {
    const int b = threadIdx.x;
    const float inv1 = rsqrtf(s_tot[b * NV] / static_cast<float>(D) + eps);
    const float inv2 = rsqrtf(inv1 * inv1 * s_tot[b * NV + 1] / static_cast<float>(D) + eps);
    s_scale[b][0] = inv1;
    s_scale[b][1] = inv1 * inv2;
  }
  __syncthreads();
  // m = x * inv1 * ffn_w (bf16) for this CTA's columns, two per thread
  for (int i = threadIdx.x; i < B * (kCols >> 1); i += kThreads) {
    const int b = i / (kCols >> 1), c = 2 * (i - b * (kCols >> 1));
    const float inv1 = s_scale[b][0];
    *reinterpret_cast<uint32_t*>(m_bf + static_cast<int64_t>(b) * D + c0 + c) =
        pack_bf16x2(s_x[b][c] * inv1 * s_ffn[c], s_x[b][c + 1] * inv1 * s_ffn[c + 1]);
  }
  if (cta == 0) {
    for (int t = threadIdx.x; t < B * E; t += kThreads) {
      const int b = t / E, e = t - b * E;
      s_logits[t] = s_scale[b][1] * s_tot[b * NV + 2 + e];
    }
    __syncthreads();
    if (warp == 0)
      warp_topk_plan(s_logits, B, E, top_k, tile_m, s_idx, s_prob, s_cnt, topk_idx, topk_prob,
                     counts, offsets, tile_offsets, perm_token, perm_prob, route_pos, lane);
  }
  cluster.sync();  // keep this CTA's shares alive until every peer has read them
}

int kch_for(int K) {
  if (K <= 0 || K % 8 != 0) return 0;
  if (K <= 768) return 3;
  if (K <= 1024) return 4;
  if (K <= 2048) return 8;
  return 0;
}

int bm_for(int B) { return B <= 1 ? 1 : (B <= 4 ? 4 : 8); }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }


}  // namespace
}  // namespace llmyb

using namespace llmyb;

LLMYB_API int32_t llmyb_decode_norm_gemv(const float* streams_in, const void* delta,
                                         const int32_t* route_pos, int32_t top_k,
                                         int32_t n_tokens, int32_t d_model, const float* norm_w,
                                         float eps, const void* w, int32_t n_out, void* out,
                                         int64_t out_ld, float* streams_out, void* normed_out,
                                         void* stream) {
  if (!streams_in || !norm_w || !w || !out || !streams_out || n_tokens < 0 || d_model <= 0 ||
      n_out <= 0 || out_ld < n_out || (route_pos && (!delta || top_k <= 0)))
    return LLMYB_EINVAL;
  if (n_tokens == 0) return LLMYB_OK;
  const int kch = kch_for(d_model);
  if (n_tokens > kMaxTokens || kch == 0 || streams_in == streams_out || !aligned16(streams_in) ||
      !aligned16(delta) || !aligned16(norm_w) || !aligned16(w) || !aligned16(streams_out) ||
      !aligned16(normed_out))
    return LLMYB_EUNSUPPORTED;
  const int bytes = n_tokens * d_model * 2;
  const int grid = static_cast<int>(ceil_div(n_out, 8));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const auto* dl = static_cast<const __nv_bfloat16*>(delta);
  const auto* wb = static_cast<const __nv_bfloat16*>(w);
  auto* ob = static_cast<__nv_bfloat16*>(out);
  auto* nb = static_cast<__nv_bfloat16*>(normed_out);
  const int bm = bm_for(n_tokens);
  int32_t st = LLMYB_OK;
#define LLMYB_NG(BMV, KCHV)                                                                     \
  do {                                                                                          \
    st = ensure_smem(decode_norm_gemv_kernel<BMV, KCHV>, bytes);                                \
    if (st) return st;                                                                          \
    st = launch_pdl(decode_norm_gemv_kernel<BMV, KCHV>, dim3(grid), dim3(256), bytes, s,         \
                    streams_in, dl, route_pos, top_k, n_tokens, d_model, norm_w, eps, wb, n_out, \
                    ob, out_ld, streams_out, nb);                                                \
    if (st) return st;                                                                          \
  } while (0)
  if (bm == 1) {
    if (kch == 3) LLMYB_NG(1, 3); else if (kch == 4) LLMYB_NG(1, 4); else LLMYB_NG(1, 8);
  } else if (bm == 4) {
    if (kch == 3) LLMYB_NG(4, 3); else if (kch == 4) LLMYB_NG(4, 4); else LLMYB_NG(4, 8);
  } else {
    if (kch == 3) LLMYB_NG(8, 3); else if (kch == 4) LLMYB_NG(8, 4); else LLMYB_NG(8, 8);
  }
#undef LLMYB_NG
  count_launch();
  return launch_status();
}

LLMYB_API int32_t llmyb_decode_out_router(
    const void* in, int64_t in_ld, int32_t k_in, const void* w, int32_t n_tokens,
    int32_t d_model, const float* conv_w, const void* normed, void* history, float* partials,
    int32_t* counter, float* streams, const float* ffn_norm, const float* w_router_folded,
    float eps, int32_t n_experts, int32_t top_k, int32_t tile_m, void* m_bf, int64_t* topk_idx,
    float* topk_prob, int32_t* expert_counts, int32_t* expert_offsets, int32_t* tile_offsets,
    int32_t* perm_token, float* perm_prob, int32_t* route_pos, void* stream) {
  if (!in || !w || !partials || !counter || !streams || !ffn_norm || !w_router_folded || !m_bf ||
      !topk_idx || !topk_prob || !expert_counts || !expert_offsets || !tile_offsets ||
      !perm_token || !perm_prob || !route_pos || n_tokens <= 0 || d_model <= 0 || k_in <= 0 ||
      in_ld < k_in || n_experts <= 0 || top_k <= 0 || top_k > n_experts || tile_m <= 0 ||
      (conv_w && (!normed || !history)))
    return LLMYB_EINVAL;
  const int kch = kch_for(k_in);
  if (n_tokens > kMaxTokens || kch == 0 || d_model % 8 != 0 || d_model > 2048 ||
      top_k > kMaxTopK || n_experts > kMaxExperts || n_tokens * top_k > 64 || in_ld % 8 != 0 ||
      !aligned16(in) || !aligned16(w) || !aligned16(streams) || !aligned16(ffn_norm) ||
      (reinterpret_cast<uintptr_t>(m_bf) & 7u))
    return LLMYB_EUNSUPPORTED;
  const int nv = 2 + n_experts;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int bm = bm_for(n_tokens);
  // one-cluster form: D = 768 (6 rows per warp, K <= 1024) or D = 1024 (8 rows per
  // warp, K <= 768: the weight rows stay in registers), B * E <= 64
  const int rpw_c = d_model % (kOrCtas * kOrWarps) == 0 ? d_model / (kOrCtas * kOrWarps) : 0;
  if (((rpw_c == 6 && kch <= 4) || (rpw_c == 8 && kch == 3)) &&
      n_tokens * n_experts <= 64) {
    const int rpw = d_model / (kOrCtas * kOrWarps);
    const int cbytes = ((n_tokens * k_in * 2 + 15) & ~15) + n_experts * (kOrWarps * rpw) * 4;
    int32_t st = LLMYB_OK;
#define LLMYB_ORC(BMV, KCHV, RPWV)                                                              \
  do {                                                                                          \
    st = ensure_smem(decode_out_router_cluster_kernel<BMV, KCHV, RPWV>, cbytes);                \
    if (st) return st;                                                                          \
    st = launch_pdl(decode_out_router_cluster_kernel<BMV, KCHV, RPWV>, dim3(kOrCtas),            \
        dim3(kOrWarps * 32), cbytes, s, static_cast<const __nv_bfloat16*>(in), in_ld, k_in,     \
        static_cast<const __nv_bfloat16*>(w), n_tokens, d_model, conv_w,                        \
        static_cast<const __nv_bfloat16*>(normed), static_cast<__nv_bfloat16*>(history),        \
        streams, ffn_norm, w_router_folded, eps, n_experts, top_k, tile_m,                      \
        static_cast<__nv_bfloat16*>(m_bf), topk_idx, topk_prob, expert_counts, expert_offsets,  \
        tile_offsets, perm_token, perm_prob, route_pos);                                        \
    if (st) return st;                                                                          \
  } while (0)
#define LLMYB_ORC_R(BMV)                                                                        \
  do {                                                                                          \
    if (rpw == 8) LLMYB_ORC(BMV, 3, 8);                                                         \
    else if (kch == 3) LLMYB_ORC(BMV, 3, 6);                                                    \
    else LLMYB_ORC(BMV, 4, 6);                                                                  \
  } while (0)
    if (bm == 1) LLMYB_ORC_R(1); else if (bm == 4) LLMYB_ORC_R(4); else LLMYB_ORC_R(8);
#undef LLMYB_ORC_R
#undef LLMYB_ORC
    count_launch();
    return launch_status();
  }
  const int bytes =
      std::max(n_tokens * k_in * 2, (n_tokens * nv + n_tokens * n_experts) * 4);
  const int grid = static_cast<int>(ceil_div(d_model, 8));
  int32_t st = LLMYB_OK;
#define LLMYB_OR(BMV, KCHV)                                                                     \
  do {                                                                                          \
    st = ensure_smem(decode_out_router_kernel<BMV, KCHV>, bytes);                               \
    if (st) return st;                                                                          \
    st = launch_pdl(decode_out_router_kernel<BMV, KCHV>, dim3(grid), dim3(256), bytes, s,        \
        static_cast<const __nv_bfloat16*>(in), in_ld, k_in,                                     \
        static_cast<const __nv_bfloat16*>(w), n_tokens, d_model, conv_w,                        \
        static_cast<const __nv_bfloat16*>(normed), static_cast<__nv_bfloat16*>(history),        \
        partials, counter, streams, ffn_norm, w_router_folded, eps, n_experts, top_k, tile_m,   \
        static_cast<__nv_bfloat16*>(m_bf), topk_idx, topk_prob, expert_counts, expert_offsets,  \
        tile_offsets, perm_token, perm_prob, route_pos);                                        \
    if (st) return st;                                                                          \
  } while (0)
  if (bm == 1) {
    if (kch == 3) LLMYB_OR(1, 3); else if (kch == 4) LLMYB_OR(1, 4); else LLMYB_OR(1, 8);
  } else if (bm == 4) {
    if (kch == 3) LLMYB_OR(4, 3); else if (kch == 4) LLMYB_OR(4, 4); else LLMYB_OR(4, 8);
  } else {
    if (kch == 3) LLMYB_OR(8, 3); else if (kch == 4) LLMYB_OR(8, 4); else LLMYB_OR(8, 8);
  }
#undef LLMYB_OR
  count_launch();
  return launch_status();
}
