// Device routines of the router shared by router.cu (route, route_fused,
// route_decode) and decode_fused.cu (the decode output-projection kernel
// that ends in the router): top-k + softmax over a logit row, the stable
// dispatch plan, the CTA-wide router input (residual add + two RMSNorms) and
// the warp-per-pair logit.  Every caller runs the same code, so the same
// inputs give bit-identical routes everywhere.
//
// Reference: model/layers/context_router.py:62-74, model/layers/moe.py:42-60.
#pragma once

#include "common.cuh"

namespace llmyb {
namespace rdev {

constexpr int kMaxTopK = 32;       // one lane per selected slot
constexpr int kMaxPerLane = 8;     // experts per lane -> E <= 256
constexpr int kMaxExperts = 32 * kMaxPerLane;

// Warp-cooperative top-k over one row of E logits.  Returns, in lane s < k,
// the index and value of the s-th selected expert.  P: expert slots per lane
// (E <= 32 P); fewer slots only skip slots that hold no expert.
template <int P = kMaxPerLane>
__device__ __forceinline__ void warp_topk_row(const float* __restrict__ row,
                                              const float* __restrict__ bias, int E, int k,
                                              int lane, int& out_idx, float& out_val) {
  float v[P];
#pragma unroll
  for (int j = 0; j < P; ++j) {
    const int e = j * 32 + lane;
    float x = -INFINITY;
    if (e < E) {
      x = row[e];
      if (bias != nullptr) x += bias[e];
    }
    v[j] = x;
  }
  unsigned taken = 0u;  // bit j: slot j of this lane already selected
  out_idx = -1;
  out_val = -INFINITY;
  for (int s = 0; s < k; ++s) {
    // local best: value desc, index asc (index grows with j for a lane)
    float best = -INFINITY;
    int best_e = 0x7fffffff;  // sentinel: no candidate in this lane
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const int e = j * 32 + lane;
      // e grows with j, so the first candidate wins ties inside a lane
      if (e < E && !((taken >> j) & 1u) && (best_e == 0x7fffffff || v[j] > best)) {
        best = v[j];
        best_e = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, best_e, o);
      if (ov > best || (ov == best && oe < best_e)) {
        best = ov;
        best_e = oe;
      }
    }
    if (lane == s) {
      out_idx = best_e;
      out_val = best;
    }
    if ((best_e & 31) == lane) taken |= 1u << (best_e >> 5);
  }
}

// softmax over the k selected values held in lanes 0..k-1 (value order:
// lane 0 holds the maximum).  fp32, exp via expf.
__device__ __forceinline__ float warp_topk_softmax(float val, int k, int lane) {
  const float mx = __shfl_sync(0xffffffffu, val, 0);
  const float ex = lane < k ? expf(val - mx) : 0.0f;
  const float sum = warp_sum(ex);
  return ex / sum;
}

// Block-wide exclusive scan of one int per thread (blockDim.x a multiple of 32).
__device__ __forceinline__ int block_exclusive_scan(int v, int* s_warp, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) s_warp[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nwarps ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    s_warp[lane] = w;
  }
  __syncthreads();
  total = s_warp[nwarps - 1];
  const int excl = x - v + (warp > 0 ? s_warp[warp - 1] : 0);
  __syncthreads();
  return excl;
}

// Stable scatter of the R = N*k routes of a plan by one warp.  Route r =
// t*k + s goes to expert s_idx[r]; s_base[e] holds the next free position of
// expert e (the expert offsets on entry) and is advanced.  Chunks of 32
// consecutive routes are placed at once: equal experts inside a chunk are
// ranked by lane order (__match_any_sync), so positions follow (token, slot)
// order within every expert.
__device__ __forceinline__ void warp_stable_scatter(const int* s_idx, const float* s_prob, int R,
                                                    int k, int* s_base, int* __restrict__ perm_token,
                                                    float* __restrict__ perm_prob,
                                                    int* __restrict__ route_pos,
                                                    int64_t* __restrict__ sort_order, int lane) {
  for (int r0 = 0; r0 < R; r0 += 32) {
    const int r = r0 + lane;
    const bool active = r < R;
    const int e = active ? s_idx[r] : -1 - lane;  // inactive lanes match nobody
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    const int pos = active ? s_base[e] + rank : 0;
    __syncwarp();
    if (active && rank == __popc(peers) - 1) s_base[e] = pos + 1;
    __syncwarp();
    if (active) {
      perm_token[pos] = r / k;
      perm_prob[pos] = s_prob[r];
      route_pos[r] = pos;
      if (sort_order != nullptr) sort_order[pos] = r;
    }
  }
}

__device__ __forceinline__ void cta_plan_tail(int N, int E, int k, int tile_m, const int* s_idx,
                                              const float* s_prob, int* s_cnt, int* s_warp,
                                              int* __restrict__ counts, int* __restrict__ offsets,
                                              int* __restrict__ tile_offsets,
                                              int* __restrict__ perm_token,
                                              float* __restrict__ perm_prob,
                                              int* __restrict__ route_pos,
                                              int64_t* __restrict__ sort_order);

// Top-k, softmax, counts, offsets, tile offsets and the stable permutation
// of N tokens whose logits [N, E] are `logits` (global or shared memory);
// called by all threads of one CTA (blockDim a multiple of 32, >= E).
__device__ __forceinline__ void cta_topk_plan(const float* logits, const float* __restrict__ bias,
                                              int N, int E, int k, int tile_m, int* s_idx,
                                              float* s_prob, int* s_cnt, int* s_warp,
                                              int64_t* __restrict__ topk_idx,
                                              float* __restrict__ topk_prob,
                                              int* __restrict__ counts, int* __restrict__ offsets,
                                              int* __restrict__ tile_offsets,
                                              int* __restrict__ perm_token,
                                              float* __restrict__ perm_prob,
                                              int* __restrict__ route_pos,
                                              int64_t* __restrict__ sort_order) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  for (int t = warp; t < N; t += nwarps) {
    int idx;
    float val;
    warp_topk_row(logits + static_cast<int64_t>(t) * E, bias, E, k, lane, idx, val);
    const float p = warp_topk_softmax(val, k, lane);
    if (lane < k) {
      s_idx[t * k + lane] = idx;
      s_prob[t * k + lane] = p;
      topk_idx[static_cast<int64_t>(t) * k + lane] = idx;
      topk_prob[static_cast<int64_t>(t) * k + lane] = p;
      atomicAdd(&s_cnt[idx], 1);
    }
  }
  __syncthreads();
  cta_plan_tail(N, E, k, tile_m, s_idx, s_prob, s_cnt, s_warp, counts, offsets, tile_offsets,
                perm_token, perm_prob, route_pos, sort_order);
}

// Counts -> offsets, tile offsets and the stable permutation (one CTA;
// s_cnt[e] holds the route count of expert e on entry).
__device__ __forceinline__ void cta_plan_tail(int N, int E, int k, int tile_m, const int* s_idx,
                                              const float* s_prob, int* s_cnt, int* s_warp,
                                              int* __restrict__ counts, int* __restrict__ offsets,
                                              int* __restrict__ tile_offsets,
                                              int* __restrict__ perm_token,
                                              float* __restrict__ perm_prob,
                                              int* __restrict__ route_pos,
                                              int64_t* __restrict__ sort_order) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = threadIdx.x < E ? s_cnt[threadIdx.x] : 0;
  int total = 0;
  const int off = block_exclusive_scan(c, s_warp, total);
  const int tiles = threadIdx.x < E ? static_cast<int>(ceil_div(c, tile_m)) : 0;
  int total_tiles = 0;
  const int toff = block_exclusive_scan(tiles, s_warp, total_tiles);
  if (threadIdx.x < E) {
    counts[threadIdx.x] = c;
    offsets[threadIdx.x] = off;
    tile_offsets[threadIdx.x] = toff;
    s_cnt[threadIdx.x] = off;
  }
  if (threadIdx.x == 0) {
    offsets[E] = total;
    tile_offsets[E] = total_tiles;
  }
  __syncthreads();
  if (warp == 0)
    warp_stable_scatter(s_idx, s_prob, N * k, k, s_cnt, perm_token, perm_prob, route_pos,
                        sort_order, lane);
}

// Top-k, softmax and the whole plan of N tokens by one warp, for decode
// batches with few routes: the CTA-wide scans of cta_topk_plan and their
// barriers cost more than the work there.  Same results as cta_topk_plan.
// s_idx / s_prob hold N*k entries, s_base E entries (shared memory).
__device__ __forceinline__ void warp_topk_plan(const float* logits, int N, int E, int k,
                                               int tile_m, int* s_idx, float* s_prob, int* s_base,
                                               int64_t* __restrict__ topk_idx,
                                               float* __restrict__ topk_prob,
                                               int* __restrict__ counts, int* __restrict__ offsets,
                                               int* __restrict__ tile_offsets,
                                               int* __restrict__ perm_token,
                                               float* __restrict__ perm_prob,
                                               int* __restrict__ route_pos, int lane) {
  for (int t = 0; t < N; ++t) {
    int idx;
    float val;
    warp_topk_row(logits + static_cast<int64_t>(t) * E, nullptr, E, k, lane, idx, val);
    const float p = warp_topk_softmax(val, k, lane);
    if (lane < k) {
      s_idx[t * k + lane] = idx;
      s_prob[t * k + lane] = p;
      topk_idx[static_cast<int64_t>(t) * k + lane] = idx;
      topk_prob[static_cast<int64_t>(t) * k + lane] = p;
    }
  }
  __syncwarp();
  const int R = N * k;
  int run = 0, trun = 0;
  for (int e0 = 0; e0 < E; e0 += 32) {
    const int e = e0 + lane;
    int c = 0;
    if (e < E)
      for (int r = 0; r < R; ++r) c += s_idx[r] == e ? 1 : 0;
    const int tl = e < E ? static_cast<int>(ceil_div(c, tile_m)) : 0;
    int x = c, y = tl;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int xx = __shfl_up_sync(0xffffffffu, x, o);
      const int yy = __shfl_up_sync(0xffffffffu, y, o);
      if (lane >= o) {
        x += xx;
        y += yy;
      }
    }
    if (e < E) {
      counts[e] = c;
      offsets[e] = run + x - c;
      tile_offsets[e] = trun + y - tl;
      s_base[e] = run + x - c;
    }
    run += __shfl_sync(0xffffffffu, x, 31);
    trun += __shfl_sync(0xffffffffu, y, 31);
  }
  if (lane == 0) {
    offsets[E] = run;
    tile_offsets[E] = trun;
  }
  __syncwarp();
  warp_stable_scatter(s_idx, s_prob, R, k, s_base, perm_token, perm_prob, route_pos, nullptr,
                      lane);
}

// Sum over the 256 threads of a CTA in a fixed order (s_red: 8 floats).
__device__ __forceinline__ float block_sum_256(float v, float* s_red) {
  v = warp_sum(v);
  __syncthreads();  // previous readers of s_red are done
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = v;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += s_red[i];
  return tot;
}

// Router input of one token by a CTA of 256 threads, float4 vectors (VMAX
// per thread: D <= 1024 * VMAX, D % 4 == 0):
//   streams[n] += delta[n] (nullable)
//   m = streams[n] * rsqrt(mean(streams[n]^2) + eps) * ffn_w   -> m_bf (bf16)
//   r = m * rsqrt(mean(m^2) + eps) * rn_w                      -> r_out (fp32)
// (PhysicalBlock ffn_norm, then ContextAwareRouter.norm on the fp32 value,
// context_router.py:62).  Every caller gets identical values.  COHERENT:
// delta was written earlier in the same kernel by other CTAs, so it is read
// through L2 (ld.global.cg) rather than the non-coherent read-only path.
template <int VMAX, bool COHERENT = false>
__device__ __forceinline__ void cta_router_input(float* __restrict__ streams,
                                                 const __nv_bfloat16* __restrict__ delta, int n,
                                                 int D, const float* __restrict__ ffn_w,
                                                 const float* __restrict__ rn_w, float eps,
                                                 __nv_bfloat16* __restrict__ m_bf, float* r_out,
                                                 float* s_red) {
  const int nv = D >> 2;
  float4* x4 = reinterpret_cast<float4*>(streams + static_cast<int64_t>(n) * D);
  const uint2* d2 = delta != nullptr
                        ? reinterpret_cast<const uint2*>(delta + static_cast<int64_t>(n) * D)
                        : nullptr;
  uint2* m2 = reinterpret_cast<uint2*>(m_bf + static_cast<int64_t>(n) * D);
  float4 v[VMAX];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < VMAX; ++j) {
    const int c = threadIdx.x + 256 * j;
    if (c >= nv) continue;
    float4 a = x4[c];
    if (d2 != nullptr) {
      const uint2 u = COHERENT ? __ldcg(d2 + c) : __ldg(d2 + c);
      const float2 lo = unpack_bf16x2(u.x), hi = unpack_bf16x2(u.y);
      a.x += lo.x;
      a.y += lo.y;
      a.z += hi.x;
      a.w += hi.y;
      x4[c] = a;
    }
    v[j] = a;
    ss += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w;
  }
  const float inv = rsqrtf(block_sum_256(ss, s_red) / static_cast<float>(D) + eps);
  float ss2 = 0.f;
#pragma unroll
  for (int j = 0; j < VMAX; ++j) {
    const int c = threadIdx.x + 256 * j;
    if (c >= nv) continue;
    const float4 w = __ldg(reinterpret_cast<const float4*>(ffn_w) + c);
    float4 m = v[j];
    m.x = m.x * inv * w.x;
    m.y = m.y * inv * w.y;
    m.z = m.z * inv * w.z;
    m.w = m.w * inv * w.w;
    m2[c] = make_uint2(pack_bf16x2(m.x, m.y), pack_bf16x2(m.z, m.w));
    v[j] = m;
    ss2 += m.x * m.x + m.y * m.y + m.z * m.z + m.w * m.w;
  }
  const float inv2 = rsqrtf(block_sum_256(ss2, s_red) / static_cast<float>(D) + eps);
#pragma unroll
  for (int j = 0; j < VMAX; ++j) {
    const int c = threadIdx.x + 256 * j;
    if (c >= nv) continue;
    const float4 w = __ldg(reinterpret_cast<const float4*>(rn_w) + c);
    const float4 m = v[j];
    reinterpret_cast<float4*>(r_out)[c] =
        make_float4(m.x * inv2 * w.x, m.y * inv2 * w.y, m.z * inv2 * w.z, m.w * inv2 * w.w);
  }
}

// Logit dot(r, Wr[e]) by one warp: lane-strided float4 products, then the
// xor tree of warp_sum (fp32, the same order for every caller).
__device__ __forceinline__ float warp_logit(const float* __restrict__ Wr, int e, const float* r,
                                            int D, int lane) {
  const float4* w = reinterpret_cast<const float4*>(Wr + static_cast<int64_t>(e) * D);
  const float4* x = reinterpret_cast<const float4*>(r);
  float acc = 0.f;
#pragma unroll 8
  for (int c = lane; c < (D >> 2); c += 32) {
    const float4 a = __ldg(w + c);
    const float4 b = x[c];
    acc += a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
  }
  return warp_sum(acc);
}

}  // namespace rdev
}  // namespace llmyb
