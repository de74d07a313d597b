// Top-k router and MoE dispatch plan.
//
// Reference semantics (StillPillWill/Hybrid_LLM):
//   * top-k + softmax over the selected logits:
//       model/layers/context_router.py:72-74
//       (top_values, top_indices = topk(route_logits.float(), k); softmax(top_values))
//   * dispatch permutation: model/layers/moe.py:42-60 (flat route r = t*k + s,
//     sort by expert, bincount, offsets = cumsum - counts).
//
// Ordering contract (bit-exact): top-k is ordered by (value desc, index asc);
// the permutation is the STABLE sort of the flat route expert ids, i.e. routes
// ordered by (expert, token, slot).  This equals
// torch.sort(flat_experts, stable=True) and, because each token's k experts
// are distinct, every permutation the reference's unstable sort may return
// produces the same per-token sums.
//
// Work split: one warp per token for top-k (HBM-bound: N*E*4 bytes read);
// the plan is a three-pass counting sort over 256-token chunks (histogram,
// one-CTA scan, in-order scatter), with a single-CTA fused path for decode
// batches (N <= 256) so that a decode step costs one launch.
#include "common.cuh"
#include "router_device.cuh"

#include <algorithm>
#include <climits>
#include <cmath>
#include <mutex>

namespace llmyb {
namespace {

constexpr int kChunk = 256;        // tokens per chunk in the multi-CTA plan
using namespace rdev;



template <int P>
__global__ void __launch_bounds__(256) router_topk_kernel(
    const float* __restrict__ logits, const float* __restrict__ bias, int N, int E, int k,
    int64_t* __restrict__ topk_idx, float* __restrict__ topk_prob) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);  // one token per warp
  if (t >= N) return;
  int idx;
  float val;
  warp_topk_row<P>(logits + static_cast<int64_t>(t) * E, bias, E, k, lane, idx, val);
  const float p = warp_topk_softmax(val, k, lane);
  if (lane < k) {
    topk_idx[static_cast<int64_t>(t) * k + lane] = idx;
    topk_prob[static_cast<int64_t>(t) * k + lane] = p;
  }
}

// Prefill router from the FFN-normalised rows m [N, D] fp32, eight tokens per
// 512-thread CTA: warp w < 8 normalises token w into shared memory,
// r = m * rsqrt(mean(m^2) + eps) * router_norm (ContextAwareRouter's RMSNorm,
// context_router.py:62-63), while every warp already holds the row of its
// first expert (w, then w + 16, ...); after the barrier each warp forms the
// fp32 logits W_r r (F.linear, :65) of all eight tokens from its expert rows
// (lane-strided float4 products, a fixed xor tree per token); finally warp
// w < 8 runs the top-k + softmax of router_topk_kernel on token w's logits.
// VPL: float4 chunks per lane (D <= 128 VPL).
template <int VPL>
__global__ void __launch_bounds__(512) router_norm_topk_kernel(
    const float* __restrict__ m, int N, int D, const float* __restrict__ rn_w, float eps,
    const float* __restrict__ Wr, const float* __restrict__ bias, int E, int k,
    float* __restrict__ logits_out, int64_t* __restrict__ topk_idx, float* __restrict__ topk_prob) {
  constexpr int kTok = 8, kWarps = 16;
  extern __shared__ float4 s_r4[];             // [8][D / 4] normalised rows
  __shared__ float s_logit[kTok][kMaxExperts];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * kTok;
  const int nc = D >> 2;
  float4 wrow[VPL];  // the first expert row of this warp, loaded before the barrier
  if (warp < E) {
    const float4* wr = reinterpret_cast<const float4*>(Wr + static_cast<int64_t>(warp) * D);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = lane + 32 * i;
      wrow[i] = c < nc ? __ldg(wr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  if (warp < kTok) {
    const int t = t0 + warp;
    float4 r[VPL];
    float ss = 0.f;
    const float4* mr = reinterpret_cast<const float4*>(m + static_cast<int64_t>(min(t, N - 1)) * D);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = lane + 32 * i;
      r[i] = (c < nc && t < N) ? __ldg(mr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      ss += r[i].x * r[i].x + r[i].y * r[i].y + r[i].z * r[i].z + r[i].w * r[i].w;
    }
    const float inv = rsqrtf(warp_sum(ss) / static_cast<float>(D) + eps);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = lane + 32 * i;
      if (c < nc) {
        const float4 w = __ldg(reinterpret_cast<const float4*>(rn_w) + c);
        s_r4[warp * nc + c] = make_float4(r[i].x * inv * w.x, r[i].y * inv * w.y,
                                          r[i].z * inv * w.z, r[i].w * inv * w.w);
      }
    }
  }
  __syncthreads();
  for (int e = warp; e < E; e += kWarps) {
    if (e != warp) {
      const float4* wr = reinterpret_cast<const float4*>(Wr + static_cast<int64_t>(e) * D);
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const int c = lane + 32 * i;
        wrow[i] = c < nc ? __ldg(wr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float acc[kTok] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int c = lane + 32 * i;
      if (c < nc) {
        const float4 a = wrow[i];
#pragma unroll
        for (int tt = 0; tt < kTok; ++tt) {
          const float4 b = s_r4[tt * nc + c];
          acc[tt] += a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
        }
      }
    }
#pragma unroll
    for (int tt = 0; tt < kTok; ++tt) {
      const float v = warp_sum(acc[tt]);
      if (lane == 0) {
        s_logit[tt][e] = v;
        if (logits_out != nullptr && t0 + tt < N) logits_out[static_cast<int64_t>(t0 + tt) * E + e] = v;
      }
    }
  }
  __syncthreads();
  const int t = t0 + warp;
  if (warp >= kTok || t >= N) return;  // whole warps leave together
  int idx;
  float val;
  warp_topk_row(s_logit[warp], bias, E, k, lane, idx, val);
  const float p = warp_topk_softmax(val, k, lane);
  if (lane < k) {
    topk_idx[static_cast<int64_t>(t) * k + lane] = idx;
    topk_prob[static_cast<int64_t>(t) * k + lane] = p;
  }
}

// Histogram only (top-k supplied by the caller, e.g. the reference router).
__global__ void __launch_bounds__(256) plan_hist_kernel(const int64_t* __restrict__ topk_idx, int N,
                                                        int E, int k, int* __restrict__ hist,
                                                        int* __restrict__ bad) {
  extern __shared__ int s_hist_dyn[];
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_hist_dyn[e] = 0;
  __syncthreads();
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kChunk * k;
  const int64_t r1 = min(static_cast<int64_t>(N) * k, r0 + static_cast<int64_t>(kChunk) * k);
  for (int64_t r = r0 + threadIdx.x; r < r1; r += blockDim.x) {
    const int64_t e = topk_idx[r];
    if (e < 0 || e >= E) {
      report_status(bad, LLMYB_EINVAL);
      continue;
    }
    atomicAdd(&s_hist_dyn[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e * gridDim.x + blockIdx.x] = s_hist_dyn[e];
}


// One CTA of 1024 threads.  hist is [E][nchunks]; on exit it holds the global
// base position of every (expert, chunk) pair.  Also writes counts, offsets
// (E+1) and tile_offsets (E+1, tiles of tile_m rows per expert).
__global__ void __launch_bounds__(1024) plan_scan_kernel(int* __restrict__ hist, int nchunks, int E,
                                                         int tile_m, int* __restrict__ counts,
                                                         int* __restrict__ offsets,
                                                         int* __restrict__ tile_offsets) {
  __shared__ int s_warp[32];
  __shared__ int s_count[1024];
  // groups of chunks per expert handled by one thread
  int G = 1;
  while (G * 2 * E <= 1024 && G * 2 <= nchunks) G *= 2;
  const int per = static_cast<int>(ceil_div(nchunks, G));
  // pass 1: per-(e,g) partial sums and in-group exclusive prefixes
  __shared__ int s_part[1024];
  for (int item = threadIdx.x; item < E * G; item += blockDim.x) {
    const int e = item / G, g = item % G;
    const int c0 = g * per, c1 = min(nchunks, c0 + per);
    int run = 0;
    int* h = hist + static_cast<int64_t>(e) * nchunks;
    for (int c = c0; c < c1; ++c) {
      const int x = h[c];
      h[c] = run;
      run += x;
    }
    s_part[item] = run;
  }
  __syncthreads();
  // per-expert totals and group bases
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int g = 0; g < G; ++g) {
      const int x = s_part[e * G + g];
      s_part[e * G + g] = run;
      run += x;
    }
    s_count[e] = run;
  }
  __syncthreads();
  // exclusive scan over experts (E <= 1024)
  const int c = threadIdx.x < E ? s_count[threadIdx.x] : 0;
  int total = 0;
  const int off = block_exclusive_scan(c, s_warp, total);
  const int tiles = threadIdx.x < E ? static_cast<int>(ceil_div(c, tile_m)) : 0;
  int total_tiles = 0;
  const int toff = block_exclusive_scan(tiles, s_warp, total_tiles);
  if (threadIdx.x < E) {
    counts[threadIdx.x] = c;
    offsets[threadIdx.x] = off;
    tile_offsets[threadIdx.x] = toff;
    s_count[threadIdx.x] = off;  // reuse as expert base
  }
  if (threadIdx.x == 0) {
    offsets[E] = total;
    tile_offsets[E] = total_tiles;
  }
  __syncthreads();
  for (int item = threadIdx.x; item < E * G; item += blockDim.x) {
    const int e = item / G, g = item % G;
    const int c0 = g * per, c1 = min(nchunks, c0 + per);
    const int base = s_count[e] + s_part[item];
    int* h = hist + static_cast<int64_t>(e) * nchunks;
    for (int cc = c0; cc < c1; ++cc) h[cc] += base;
  }
}

// In-order scatter.  CTA = one 256-token chunk = 8 warps x 32 tokens; lane s
// walks slot s of the warp's tokens in token order, so equal experts get
// increasing positions in (token, slot) order.
__global__ void __launch_bounds__(256) plan_scatter_kernel(
    const int64_t* __restrict__ topk_idx, const float* __restrict__ topk_prob, int N, int E, int k,
    const int* __restrict__ hist_base, int* __restrict__ perm_token, float* __restrict__ perm_prob,
    int* __restrict__ route_pos, int64_t* __restrict__ sort_order) {
  extern __shared__ int s_cnt[];  // [8][E]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nchunks = gridDim.x;
  int* my = s_cnt + warp * E;
  for (int e = lane; e < E; e += 32) my[e] = 0;
  __syncwarp();
  const int t0 = blockIdx.x * kChunk + warp * 32;
  const int tn = max(0, min(32, N - t0));
  // lane s holds slot s of the warp's 32 tokens (loads issued together)
  int ev[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    int64_t e = -1;
    if (j < tn && lane < k) e = topk_idx[static_cast<int64_t>(t0 + j) * k + lane];
    ev[j] = (e >= 0 && e < E) ? static_cast<int>(e) : -1;  // -1: absent or flagged
  }
  // phase 1: per-warp counts (a token's experts are distinct: no lane collision)
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (ev[j] >= 0) my[ev[j]] += 1;
    __syncwarp();
  }
  __syncthreads();
  // phase 2: turn counts into starting positions
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = hist_base[e * nchunks + blockIdx.x];
    for (int w = 0; w < 8; ++w) {
      const int x = s_cnt[w * E + e];
      s_cnt[w * E + e] = run;
      run += x;
    }
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (ev[j] >= 0) {
      const int t = t0 + j;
      const int64_t r = static_cast<int64_t>(t) * k + lane;
      const int pos = my[ev[j]];
      my[ev[j]] = pos + 1;
      perm_token[pos] = t;
      perm_prob[pos] = topk_prob[r];
      route_pos[r] = pos;
      if (sort_order != nullptr) sort_order[pos] = r;
    }
    __syncwarp();
  }
}





// Fused single-CTA route for small batches (decode): top-k, softmax, counts,
// offsets, tile offsets and the in-order permutation in one launch.
__global__ void __launch_bounds__(1024) route_small_kernel(
    const float* __restrict__ logits, const float* __restrict__ bias, int N, int E, int k,
    int tile_m, int64_t* __restrict__ topk_idx, float* __restrict__ topk_prob,
    int* __restrict__ counts, int* __restrict__ offsets, int* __restrict__ tile_offsets,
    int* __restrict__ perm_token, float* __restrict__ perm_prob, int* __restrict__ route_pos,
    int64_t* __restrict__ sort_order) {
  __shared__ int s_idx[256 * kMaxTopK / 4];  // N*k <= 2048
  __shared__ float s_prob[256 * kMaxTopK / 4];
  __shared__ int s_cnt[kMaxExperts];
  __shared__ int s_warp[32];
  cta_topk_plan(logits, bias, N, E, k, tile_m, s_idx, s_prob, s_cnt, s_warp, topk_idx, topk_prob,
                counts, offsets, tile_offsets, perm_token, perm_prob, route_pos, sort_order);
}

// Dispatch plan of N*k <= 2048 routes whose top-k (from router_topk_kernel)
// is already in topk_idx / topk_prob: one CTA of 1024 threads.
// The stable permutation of R routes by every warp of the CTA (E <= 64):
// warp w takes routes [w L, (w + 1) L) in 32-route chunks; it counts them per
// expert, a per-expert prefix over the warps turns the counts into the
// segments' first positions (from s_base = the experts' offsets), and each
// warp then places its segment in order: the same permutation as
// warp_stable_scatter, without one warp walking all R routes.
constexpr int kSegExperts = 64;
__device__ __forceinline__ void cta_stable_scatter(const int* s_idx, const float* s_prob, int R,
                                                   int k, int E, const int* s_base,
                                                   int (*s_seg)[kSegExperts],
                                                   int* __restrict__ perm_token,
                                                   float* __restrict__ perm_prob,
                                                   int* __restrict__ route_pos,
                                                   int64_t* __restrict__ sort_order) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int L = static_cast<int>(ceil_div(ceil_div(R, 32), nw)) * 32;
  const int r_lo = min(R, warp * L), r_hi = min(R, r_lo + L);
  for (int e = lane; e < E; e += 32) s_seg[warp][e] = 0;
  __syncwarp();
  for (int r0 = r_lo; r0 < r_hi; r0 += 32) {
    const int r = r0 + lane;
    const bool active = r < r_hi;
    const int e = active ? s_idx[r] : -1 - lane;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (active && lane == 31 - __clz(peers)) s_seg[warp][e] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = s_base[e];
    for (int w = 0; w < nw; ++w) {
      const int c = s_seg[w][e];
      s_seg[w][e] = run;
      run += c;
    }
  }
  __syncthreads();
  for (int r0 = r_lo; r0 < r_hi; r0 += 32) {
    const int r = r0 + lane;
    const bool active = r < r_hi;
    const int e = active ? s_idx[r] : -1 - lane;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    const int pos = active ? s_seg[warp][e] + rank : 0;
    __syncwarp();
    if (active && rank == __popc(peers) - 1) s_seg[warp][e] = pos + 1;
    __syncwarp();
    if (active) {
      perm_token[pos] = r / k;
      perm_prob[pos] = s_prob[r];
      route_pos[r] = pos;
      if (sort_order != nullptr) sort_order[pos] = r;
    }
  }
}

__global__ void __launch_bounds__(1024) plan_small_kernel(
    const int64_t* __restrict__ topk_idx, const float* __restrict__ topk_prob, int N, int E,
    int k, int tile_m, int* __restrict__ counts, int* __restrict__ offsets,
    int* __restrict__ tile_offsets, int* __restrict__ perm_token, float* __restrict__ perm_prob,
    int* __restrict__ route_pos, int64_t* __restrict__ sort_order) {
  __shared__ int s_idx[256 * kMaxTopK / 4];
  __shared__ float s_prob[256 * kMaxTopK / 4];
  __shared__ int s_cnt[kMaxExperts];
  __shared__ int s_warp[32];
  __shared__ int s_seg[32][kSegExperts];
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
  __syncthreads();
  for (int r = threadIdx.x; r < N * k; r += blockDim.x) {
    const int e = static_cast<int>(topk_idx[r]);
    s_idx[r] = e;
    s_prob[r] = topk_prob[r];
    atomicAdd(&s_cnt[e], 1);
  }
  __syncthreads();
  if (E > kSegExperts || N * k <= 64) {
    cta_plan_tail(N, E, k, tile_m, s_idx, s_prob, s_cnt, s_warp, counts, offsets, tile_offsets,
                  perm_token, perm_prob, route_pos, sort_order);
    return;
  }
  // counts, offsets and tile offsets as cta_plan_tail forms them; the
  // permutation by all warps
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
  cta_stable_scatter(s_idx, s_prob, N * k, k, E, s_cnt, s_seg, perm_token, perm_prob, route_pos,
                     sort_order);
}




// Decode-step router in one CTA (small N*E): router input of each token,
// logits (one warp per (token, expert) pair), then top-k and plan.
template <int VMAX>
__global__ void __launch_bounds__(256) router_fused_kernel(
    float* __restrict__ streams, const __nv_bfloat16* __restrict__ delta, int N, int D,
    const float* __restrict__ ffn_w, const float* __restrict__ rn_w, const float* __restrict__ Wr,
    float eps, int E, int k, int tile_m, __nv_bfloat16* __restrict__ m_bf,
    int64_t* __restrict__ topk_idx, float* __restrict__ topk_prob, int* __restrict__ counts,
    int* __restrict__ offsets, int* __restrict__ tile_offsets, int* __restrict__ perm_token,
    float* __restrict__ perm_prob, int* __restrict__ route_pos) {
  extern __shared__ float s_dyn[];
  __shared__ int s_idx[256 * kMaxTopK / 4];
  __shared__ float s_prob[256 * kMaxTopK / 4];
  __shared__ int s_cnt[kMaxExperts];
  __shared__ int s_warp[32];
  __shared__ float s_red[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float* s_r = s_dyn;               // [N][D] router inputs
  float* s_logits = s_dyn + N * D;  // [N][E]
  for (int n = 0; n < N; ++n)
    cta_router_input<VMAX>(streams, delta, n, D, ffn_w, rn_w, eps, m_bf, s_r + n * D, s_red);
  __syncthreads();
  for (int p = warp; p < N * E; p += 8) {
    const int t = p / E, e = p - t * E;
    const float l = warp_logit(Wr, e, s_r + t * D, D, lane);
    if (lane == 0) s_logits[p] = l;
  }
  __syncthreads();
  cta_topk_plan(s_logits, nullptr, N, E, k, tile_m, s_idx, s_prob, s_cnt, s_warp, topk_idx,
                topk_prob, counts, offsets, tile_offsets, perm_token, perm_prob, route_pos,
                nullptr);
}

// Multi-CTA decode router, step 1: router input of one token per CTA.
template <int VMAX>
__global__ void __launch_bounds__(256) router_input_kernel(
    float* __restrict__ streams, const __nv_bfloat16* __restrict__ delta, int D,
    const float* __restrict__ ffn_w, const float* __restrict__ rn_w, float eps,
    __nv_bfloat16* __restrict__ m_bf, float* __restrict__ r) {
  __shared__ float s_red[8];
  cta_router_input<VMAX>(streams, delta, blockIdx.x, D, ffn_w, rn_w, eps, m_bf,
                         r + static_cast<int64_t>(blockIdx.x) * D, s_red);
}

// Multi-CTA decode router, step 2: one warp per (token, expert) logit.
__global__ void __launch_bounds__(256) router_pair_logits_kernel(const float* __restrict__ r,
                                                                 const float* __restrict__ Wr,
                                                                 int N, int D, int E,
                                                                 float* __restrict__ logits) {
  const int lane = threadIdx.x & 31;
  const int p = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (p >= N * E) return;  // whole warps leave together
  const int t = p / E, e = p - t * E;
  const float l = warp_logit(Wr, e, r + static_cast<int64_t>(t) * D, D, lane);
  if (lane == 0) logits[p] = l;
}

}  // namespace
}  // namespace llmyb

namespace llmyb {
namespace {

// float4 vectors per thread of the router-input routine (0: D unsupported)
int router_vmax(int D) {
  if (D <= 0 || D % 4 != 0) return 0;
  if (D <= 1024) return 1;
  if (D <= 2048) return 2;
  if (D <= 4096) return 4;
  if (D <= 8192) return 8;
  return 0;
}

bool router_aligned(const void* streams, const void* delta, const void* ffn_norm,
                    const void* router_norm, const void* w_router, const void* m_bf) {
  return ((reinterpret_cast<uintptr_t>(streams) | reinterpret_cast<uintptr_t>(ffn_norm) |
           reinterpret_cast<uintptr_t>(router_norm) | reinterpret_cast<uintptr_t>(w_router)) &
          15u) == 0 &&
         ((reinterpret_cast<uintptr_t>(delta) | reinterpret_cast<uintptr_t>(m_bf)) & 7u) == 0;
}

// router_topk_kernel with the fewest expert slots per lane that hold E
void launch_router_topk(const float* logits, const float* bias, int N, int E, int k,
                        int64_t* topk_idx, float* topk_prob, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>(ceil_div(N, 8)));
  if (E <= 32)
    router_topk_kernel<1><<<grid, 256, 0, s>>>(logits, bias, N, E, k, topk_idx, topk_prob);
  else if (E <= 64)
    router_topk_kernel<2><<<grid, 256, 0, s>>>(logits, bias, N, E, k, topk_idx, topk_prob);
  else if (E <= 128)
    router_topk_kernel<4><<<grid, 256, 0, s>>>(logits, bias, N, E, k, topk_idx, topk_prob);
  else
    router_topk_kernel<kMaxPerLane><<<grid, 256, 0, s>>>(logits, bias, N, E, k, topk_idx,
                                                         topk_prob);
  count_launch();
}

int32_t check_route_args(int N, int E, int k, int tile_m) {
  if (N < 0 || E <= 0 || k <= 0 || k > E || tile_m <= 0) return LLMYB_EINVAL;
  if (k > kMaxTopK || E > kMaxExperts) return LLMYB_EUNSUPPORTED;
  return LLMYB_OK;
}

}  // namespace
}  // namespace llmyb

using namespace llmyb;

LLMYB_API int32_t llmyb_router_topk(const float* logits, const float* bias, int32_t n_tokens,
                                    int32_t n_experts, int32_t top_k, int64_t* topk_idx,
                                    float* topk_prob, void* stream) {
  int32_t st = check_route_args(n_tokens, n_experts, top_k, 1);
  if (st) return st;
  if (n_tokens == 0) return LLMYB_OK;
  if (!logits || !topk_idx || !topk_prob) return LLMYB_EINVAL;
  launch_router_topk(logits, bias, n_tokens, n_experts, top_k, topk_idx, topk_prob, static_cast<cudaStream_t>(stream));
  return launch_status();
}

LLMYB_API int64_t llmyb_moe_plan_scratch_bytes(int32_t n_tokens, int32_t n_experts) {
  if (n_tokens < 0 || n_experts <= 0) return -1;
  const int64_t nchunks = ceil_div(n_tokens, kChunk);
  return (nchunks * n_experts + 1) * static_cast<int64_t>(sizeof(int));
}

namespace {
int32_t plan_tail(const int64_t* topk_idx, const float* topk_prob, int N, int E, int k, int tile_m,
                  int* counts, int* offsets, int* tile_offsets, int* perm_token, float* perm_prob,
                  int* route_pos, int64_t* sort_order, int* hist, cudaStream_t s) {
  const int nchunks = static_cast<int>(ceil_div(N, kChunk));
  plan_scan_kernel<<<1, 1024, 0, s>>>(hist, nchunks, E, tile_m, counts, offsets, tile_offsets);
  count_launch();
  plan_scatter_kernel<<<nchunks, 256, 8 * E * sizeof(int), s>>>(
      topk_idx, topk_prob, N, E, k, hist, perm_token, perm_prob, route_pos, sort_order);
  count_launch();
  return launch_status();
}

int32_t empty_plan(int E, int* counts, int* offsets, int* tile_offsets, cudaStream_t s) {
  cudaError_t e1 = cudaMemsetAsync(counts, 0, sizeof(int) * E, s);
  cudaError_t e2 = cudaMemsetAsync(offsets, 0, sizeof(int) * (E + 1), s);
  cudaError_t e3 = cudaMemsetAsync(tile_offsets, 0, sizeof(int) * (E + 1), s);
  if (e1 != cudaSuccess) return e1;
  if (e2 != cudaSuccess) return e2;
  return e3;
}
}  // namespace

// Dispatch plan for top-k routes computed elsewhere (e.g. the reference's
// torch.topk router): model/layers/moe.py:42-60.
LLMYB_API int32_t llmyb_moe_plan(const int64_t* topk_idx, const float* topk_prob, int32_t n_tokens,
                                 int32_t n_experts, int32_t top_k, int32_t tile_m,
                                 int32_t* expert_counts, int32_t* expert_offsets,
                                 int32_t* tile_offsets, int32_t* perm_token, float* perm_prob,
                                 int32_t* route_pos, int64_t* sort_order, void* scratch,
                                 int32_t* dev_status, void* stream) {
  int32_t st = check_route_args(n_tokens, n_experts, top_k, tile_m);
  if (st) return st;
  if (!expert_counts || !expert_offsets || !tile_offsets || !dev_status) return LLMYB_EINVAL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_tokens == 0) return empty_plan(n_experts, expert_counts, expert_offsets, tile_offsets, s);
  if (!topk_idx || !topk_prob || !perm_token || !perm_prob || !route_pos || !scratch)
    return LLMYB_EINVAL;
  const int nchunks = static_cast<int>(ceil_div(n_tokens, kChunk));
  int* hist = static_cast<int*>(scratch);
  plan_hist_kernel<<<nchunks, 256, n_experts * sizeof(int), s>>>(topk_idx, n_tokens, n_experts,
                                                                 top_k, hist, dev_status);
  count_launch();
  return plan_tail(topk_idx, topk_prob, n_tokens, n_experts, top_k, tile_m, expert_counts,
                   expert_offsets, tile_offsets, perm_token, perm_prob, route_pos, sort_order,
                   hist, s);
}

namespace llmyb {
namespace {
int32_t route_impl(const float* logits, const float* bias, int32_t n_tokens, int32_t n_experts,
                   int32_t top_k, int32_t tile_m, int64_t* topk_idx, float* topk_prob,
                   int32_t* expert_counts, int32_t* expert_offsets, int32_t* tile_offsets,
                   int32_t* perm_token, float* perm_prob, int32_t* route_pos, int64_t* sort_order,
                   void* scratch, cudaStream_t s) {
  int32_t st = check_route_args(n_tokens, n_experts, top_k, tile_m);
  if (st) return st;
  if (!expert_counts || !expert_offsets || !tile_offsets) return LLMYB_EINVAL;
  if (n_tokens == 0) return empty_plan(n_experts, expert_counts, expert_offsets, tile_offsets, s);
  if (!logits || !topk_idx || !topk_prob || !perm_token || !perm_prob || !route_pos)
    return LLMYB_EINVAL;
  if (n_tokens <= 32 && n_tokens * top_k <= 256 * kMaxTopK / 4) {
    route_small_kernel<<<1, 1024, 0, s>>>(logits, bias, n_tokens, n_experts, top_k, tile_m,
                                          topk_idx, topk_prob, expert_counts, expert_offsets,
                                          tile_offsets, perm_token, perm_prob, route_pos,
                                          sort_order);
    count_launch();
    return launch_status();
  }
  if (n_tokens * top_k <= 256 * kMaxTopK / 4) {
    // top-k spread over CTAs (one token per warp), then the plan in one CTA
    launch_router_topk(logits, bias, n_tokens, n_experts, top_k, topk_idx, topk_prob, s);
    plan_small_kernel<<<1, 1024, 0, s>>>(topk_idx, topk_prob, n_tokens, n_experts, top_k, tile_m,
                                         expert_counts, expert_offsets, tile_offsets, perm_token,
                                         perm_prob, route_pos, sort_order);
    count_launch();
    return launch_status();
  }
  if (!scratch) return LLMYB_EINVAL;
  const int nchunks = static_cast<int>(ceil_div(n_tokens, kChunk));
  int* hist = static_cast<int*>(scratch);
  launch_router_topk(logits, bias, n_tokens, n_experts, top_k, topk_idx, topk_prob, s);
  plan_hist_kernel<<<nchunks, 256, n_experts * sizeof(int), s>>>(topk_idx, n_tokens, n_experts,
                                                                 top_k, hist, nullptr);
  count_launch();
  return plan_tail(topk_idx, topk_prob, n_tokens, n_experts, top_k, tile_m, expert_counts,
                   expert_offsets, tile_offsets, perm_token, perm_prob, route_pos, sort_order,
                   hist, s);
}
}  // namespace
}  // namespace llmyb

// Router top-k + softmax + dispatch plan from fp32 logits (plus an optional
// per-expert bias added before selection).
LLMYB_API int32_t llmyb_route(const float* logits, const float* bias, int32_t n_tokens,
                              int32_t n_experts, int32_t top_k, int32_t tile_m, int64_t* topk_idx,
                              float* topk_prob, int32_t* expert_counts, int32_t* expert_offsets,
                              int32_t* tile_offsets, int32_t* perm_token, float* perm_prob,
                              int32_t* route_pos, int64_t* sort_order, void* scratch,
                              void* stream) {
  return route_impl(logits, bias, n_tokens, n_experts, top_k, tile_m, topk_idx, topk_prob,
                    expert_counts, expert_offsets, tile_offsets, perm_token, perm_prob, route_pos,
                    sort_order, scratch, static_cast<cudaStream_t>(stream));
}

// Router from the FFN-normalised rows (router RMSNorm + fp32 logits + top-k
// in one warp-per-token kernel), then the dispatch plan: one CTA for up to
// 2048 routes, else the chunked multi-CTA plan.
LLMYB_API int32_t llmyb_route_norm(const float* m, int32_t n_tokens, int32_t d_model,
                                   const float* router_norm, const float* w_router, float eps,
                                   const float* bias, int32_t n_experts, int32_t top_k,
                                   int32_t tile_m, float* logits_out, int64_t* topk_idx,
                                   float* topk_prob, int32_t* expert_counts,
                                   int32_t* expert_offsets, int32_t* tile_offsets,
                                   int32_t* perm_token, float* perm_prob, int32_t* route_pos,
                                   int64_t* sort_order, void* scratch, void* stream) {
  int32_t st = check_route_args(n_tokens, n_experts, top_k, tile_m);
  if (st) return st;
  if (!expert_counts || !expert_offsets || !tile_offsets) return LLMYB_EINVAL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_tokens == 0) return empty_plan(n_experts, expert_counts, expert_offsets, tile_offsets, s);
  if (!m || !router_norm || !w_router || !topk_idx || !topk_prob || !perm_token || !perm_prob ||
      !route_pos)
    return LLMYB_EINVAL;
  if (d_model <= 0 || d_model % 4 != 0 || d_model > 1024 ||
      ((reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(router_norm) |
        reinterpret_cast<uintptr_t>(w_router)) & 15u))
    return LLMYB_EUNSUPPORTED;
  const int vpl = static_cast<int>(ceil_div(d_model / 4, 32));
  const int grid = static_cast<int>(ceil_div(n_tokens, 8));
  const int smem = 8 * d_model * static_cast<int>(sizeof(float));  // <= 32 KB
  auto go = [&](auto kern) {
    kern<<<grid, 512, smem, s>>>(m, n_tokens, d_model, router_norm, eps, w_router, bias,
                                 n_experts, top_k, logits_out, topk_idx, topk_prob);
  };
  if (vpl <= 2) go(router_norm_topk_kernel<2>);
  else if (vpl <= 4) go(router_norm_topk_kernel<4>);
  else go(router_norm_topk_kernel<8>);
  count_launch();
  if (n_tokens * top_k <= 256 * kMaxTopK / 4) {
    plan_small_kernel<<<1, 1024, 0, s>>>(topk_idx, topk_prob, n_tokens, n_experts, top_k, tile_m,
                                         expert_counts, expert_offsets, tile_offsets, perm_token,
                                         perm_prob, route_pos, sort_order);
    count_launch();
    return launch_status();
  }
  if (!scratch) return LLMYB_EINVAL;
  const int nchunks = static_cast<int>(ceil_div(n_tokens, kChunk));
  int* hist = static_cast<int*>(scratch);
  plan_hist_kernel<<<nchunks, 256, n_experts * sizeof(int), s>>>(topk_idx, n_tokens, n_experts,
                                                                 top_k, hist, nullptr);
  count_launch();
  return plan_tail(topk_idx, topk_prob, n_tokens, n_experts, top_k, tile_m, expert_counts,
                   expert_offsets, tile_offsets, perm_token, perm_prob, route_pos, sort_order,
                   hist, s);
}

// Decode-step router fused with the residual add and the two RMSNorms that
// precede it (see router_fused_kernel).  streams [N, D] fp32 in/out; delta
// [N, D] bf16 (nullable); ffn_norm / router_norm [D] fp32; w_router [E, D]
// fp32; writes m_bf [N, D] bf16 (the expert input) and the dispatch plan.
// Limited to N*E <= 256 (token, expert) pairs and N*k <= 2048 (a single CTA).
LLMYB_API int32_t llmyb_route_fused(float* streams, const void* delta, int32_t n_tokens,
                                    int32_t d_model, const float* ffn_norm,
                                    const float* router_norm, const float* w_router, float eps,
                                    int32_t n_experts, int32_t top_k, int32_t tile_m, void* m_bf,
                                    int64_t* topk_idx, float* topk_prob, int32_t* expert_counts,
                                    int32_t* expert_offsets, int32_t* tile_offsets,
                                    int32_t* perm_token, float* perm_prob, int32_t* route_pos,
                                    void* stream) {
  int32_t st = check_route_args(n_tokens, n_experts, top_k, tile_m);
  if (st) return st;
  if (!streams || !ffn_norm || !router_norm || !w_router || !m_bf || !topk_idx || !topk_prob ||
      !expert_counts || !expert_offsets || !tile_offsets || !perm_token || !perm_prob || !route_pos)
    return LLMYB_EINVAL;
  if (n_tokens == 0) {
    return empty_plan(n_experts, expert_counts, expert_offsets, tile_offsets,
                      static_cast<cudaStream_t>(stream));
  }
  const int vmax = router_vmax(d_model);
  if (n_tokens > 256 || n_tokens * top_k > 256 * kMaxTopK / 4 || n_tokens * n_experts > 256 ||
      vmax == 0 || !router_aligned(streams, delta, ffn_norm, router_norm, w_router, m_bf))
    return LLMYB_EUNSUPPORTED;
  const int bytes = (n_tokens * d_model + n_tokens * n_experts) * static_cast<int>(sizeof(float));
  if (bytes > 190 * 1024) return LLMYB_EUNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto launch = [&](auto kernel, int) -> int32_t {
    {  // static + dynamic shared memory may pass 48 KB
      int32_t st = ensure_smem(kernel, bytes);
      if (st) return st;
    }
    kernel<<<1, 256, bytes, s>>>(streams, static_cast<const __nv_bfloat16*>(delta), n_tokens,
                                 d_model, ffn_norm, router_norm, w_router, eps, n_experts, top_k,
                                 tile_m, static_cast<__nv_bfloat16*>(m_bf), topk_idx, topk_prob,
                                 expert_counts, expert_offsets, tile_offsets, perm_token,
                                 perm_prob, route_pos);
    return LLMYB_OK;
  };
  switch (vmax) {
    case 1: st = launch(router_fused_kernel<1>, 0); break;
    case 2: st = launch(router_fused_kernel<2>, 1); break;
    case 4: st = launch(router_fused_kernel<4>, 2); break;
    default: st = launch(router_fused_kernel<8>, 3); break;
  }
  if (st) return st;
  count_launch();
  return launch_status();
}

// ----------------------------------------------------------------------------
// Shared experts (model/layers/moe.py:185-198 prefill, :221-234 decode step):
// every token goes through each of the S shared experts and their sum, scaled
// by 1/sqrt(S), is added to the routed output.  They become plan experts
// E..E+S-1 that every token is routed to with probability 1/sqrt(S), placed
// after the routed rows in plan order (expert E+s holds tokens 0..N-1 at rows
// N*k + s*N + t).  The expert kernels then run routed and shared experts in
// one call (weights stacked routed first, then shared), scaling each row by
// its probability, and the combine over a token's k + S rows gives
// routed + sum_s SwiGLU_s(x) / sqrt(S).
namespace llmyb {
namespace {
__global__ void plan_append_shared_kernel(
    int N, int E, int k, int S, int tile_m, float p, const int64_t* __restrict__ idx,
    const float* __restrict__ prob, const int* __restrict__ counts,
    const int* __restrict__ offsets, const int* __restrict__ tiles,
    const int* __restrict__ perm_token, const float* __restrict__ perm_prob,
    const int* __restrict__ route_pos, int64_t* __restrict__ idx2, float* __restrict__ prob2,
    int* __restrict__ counts2, int* __restrict__ offsets2, int* __restrict__ tiles2,
    int* __restrict__ perm_token2, float* __restrict__ perm_prob2,
    int* __restrict__ route_pos2) {
  const int64_t n_routes = static_cast<int64_t>(N) * k;
  const int64_t total = static_cast<int64_t>(N) * (k + S);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += stride) {
    // plan rows: the routed rows unchanged, then S groups of N token rows
    if (i < n_routes) {
      perm_token2[i] = perm_token[i];
      perm_prob2[i] = perm_prob[i];
    } else {
      perm_token2[i] = static_cast<int>((i - n_routes) % N);
      perm_prob2[i] = p;
    }
    // per-token slots: [t, 0..k) routed, [t, k..k+S) shared
    const int64_t t = i / (k + S);
    const int s = static_cast<int>(i - t * (k + S));
    if (s < k) {
      idx2[i] = idx[t * k + s];
      prob2[i] = prob[t * k + s];
      route_pos2[i] = route_pos[t * k + s];
    } else {
      idx2[i] = E + (s - k);
      prob2[i] = p;
      route_pos2[i] = static_cast<int>(n_routes + static_cast<int64_t>(s - k) * N + t);
    }
  }
  if (blockIdx.x == 0) {
    const int tiles_per = (N + tile_m - 1) / tile_m;
    for (int e = threadIdx.x; e <= E + S; e += blockDim.x) {
      if (e < E + S) counts2[e] = e < E ? counts[e] : N;
      offsets2[e] = e <= E ? offsets[e] : static_cast<int>(n_routes + static_cast<int64_t>(e - E) * N);
      tiles2[e] = e <= E ? tiles[e] : tiles[E] + (e - E) * tiles_per;
    }
  }
}
}  // namespace
}  // namespace llmyb

LLMYB_API int32_t llmyb_plan_append_shared(
    int32_t n_tokens, int32_t n_experts, int32_t top_k, int32_t n_shared, int32_t tile_m,
    const int64_t* topk_idx, const float* topk_prob, const int32_t* expert_counts,
    const int32_t* expert_offsets, const int32_t* tile_offsets, const int32_t* perm_token,
    const float* perm_prob, const int32_t* route_pos, int64_t* out_topk_idx,
    float* out_topk_prob, int32_t* out_counts, int32_t* out_offsets, int32_t* out_tile_offsets,
    int32_t* out_perm_token, float* out_perm_prob, int32_t* out_route_pos, void* stream) {
  if (n_tokens < 0 || n_experts <= 0 || top_k <= 0 || n_shared <= 0 || tile_m <= 0)
    return LLMYB_EINVAL;
  if (static_cast<int64_t>(n_tokens) * (top_k + n_shared) > INT32_MAX) return LLMYB_EUNSUPPORTED;
  if (!expert_counts || !expert_offsets || !tile_offsets || !out_counts || !out_offsets ||
      !out_tile_offsets)
    return LLMYB_EINVAL;
  if (n_tokens > 0 && (!topk_idx || !topk_prob || !perm_token || !perm_prob || !route_pos ||
                       !out_topk_idx || !out_topk_prob || !out_perm_token || !out_perm_prob ||
                       !out_route_pos))
    return LLMYB_EINVAL;
  const int64_t total = static_cast<int64_t>(n_tokens) * (top_k + n_shared);
  const int grid = static_cast<int>(std::min<int64_t>(std::max<int64_t>(ceil_div(total, 256), 1),
                                                      4 * 148));
  plan_append_shared_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      n_tokens, n_experts, top_k, n_shared, tile_m,
      static_cast<float>(1.0 / std::sqrt(static_cast<double>(n_shared))),
      topk_idx, topk_prob, expert_counts, expert_offsets, tile_offsets, perm_token, perm_prob,
      route_pos, out_topk_idx, out_topk_prob, out_counts, out_offsets, out_tile_offsets,
      out_perm_token, out_perm_prob, out_route_pos);
  count_launch();
  return launch_status();
}

// ----------------------------------------------------------------------------
// Allocation-free routing.
//
// Some callers cannot call cudaMalloc at all: code that runs while the
// device heap is owned by another allocator, inference servers that reserve
// all memory up front and hand out only input/output buffers, and hosts that
// must not grow memory after start-up.  llmyb_route needs a caller-provided
// scratch buffer (llmyb_moe_plan_scratch_bytes) for its per-chunk expert
// histogram; llmyb_route_noalloc keeps that histogram in a fixed array that
// lives in this library's own device memory instead, so such callers pass
// only inputs and outputs.
//
// The array holds kNoAllocScratchInts ints (256 KiB) and is held on every
// device that loads the library until the process exits.  A call needs
// ceil(n_tokens / 256) * n_experts + 1 ints of it; larger calls are rejected
// with LLMYB_EUNSUPPORTED.  Every call shares the one array per device, so
// two calls that overlap on the GPU (for example on two streams) race and
// must be serialised by the caller.  The histogram is fully rewritten by each
// call before it is read, so nothing carries over from the previous call.
constexpr int kNoAllocScratchInts = 1 << 16;
static __device__ __align__(256) int g_route_scratch[kNoAllocScratchInts];

namespace {
std::mutex g_route_scratch_mu;
constexpr int kMaxDevices = 64;
void* g_route_scratch_addr[kMaxDevices] = {};

// Device address of g_route_scratch on the current device.  In host code the
// array's name only stands in for the symbol, so the address is looked up once
// per device (on the first call made with that device current).
int32_t route_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int32_t>(e);
  if (dev < 0 || dev >= kMaxDevices) return LLMYB_EUNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_route_scratch_mu);
  if (g_route_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_route_scratch);
    if (e != cudaSuccess) return static_cast<int32_t>(e);
    g_route_scratch_addr[dev] = p;
  }
  *out = g_route_scratch_addr[dev];
  return LLMYB_OK;
}
}  // namespace

LLMYB_API int64_t llmyb_route_noalloc_max_scratch_ints(void) { return kNoAllocScratchInts; }

// llmyb_route without the scratch argument (see the block comment above).
// The first call on a device looks up the array's device address; make that
// first call before capturing any CUDA graph that contains this entry point.
LLMYB_API int32_t llmyb_route_noalloc(const float* logits, const float* bias, int32_t n_tokens,
                                      int32_t n_experts, int32_t top_k, int32_t tile_m,
                                      int64_t* topk_idx, float* topk_prob,
                                      int32_t* expert_counts, int32_t* expert_offsets,
                                      int32_t* tile_offsets, int32_t* perm_token,
                                      float* perm_prob, int32_t* route_pos, int64_t* sort_order,
                                      void* stream) {
  int32_t st = check_route_args(n_tokens, n_experts, top_k, tile_m);
  if (st) return st;
  const int64_t need = ceil_div(n_tokens, kChunk) * n_experts + 1;
  if (need > kNoAllocScratchInts) return LLMYB_EUNSUPPORTED;
  void* scratch = nullptr;
  st = route_scratch_address(&scratch);
  if (st) return st;
  return route_impl(logits, bias, n_tokens, n_experts, top_k, tile_m, topk_idx, topk_prob,
                    expert_counts, expert_offsets, tile_offsets, perm_token, perm_prob, route_pos,
                    sort_order, scratch, static_cast<cudaStream_t>(stream));
}

// llmyb_route_fused for any decode batch N <= 256 (N*k <= 2048) in three
// launches: the router input of each token (one CTA per token), the logits
// (one warp per (token, expert) pair), then top-k, softmax and the dispatch
// plan in one CTA.  scratch [N*(D+E)] fp32 holds the router inputs and the
// logits.  The same routines as llmyb_route_fused, so the same results.
LLMYB_API int32_t llmyb_route_decode(float* streams, const void* delta, int32_t n_tokens,
                                     int32_t d_model, const float* ffn_norm,
                                     const float* router_norm, const float* w_router, float eps,
                                     int32_t n_experts, int32_t top_k, int32_t tile_m, void* m_bf,
                                     float* logits_scratch, int64_t* topk_idx, float* topk_prob,
                                     int32_t* expert_counts, int32_t* expert_offsets,
                                     int32_t* tile_offsets, int32_t* perm_token,
                                     float* perm_prob, int32_t* route_pos, void* stream) {
  int32_t st = check_route_args(n_tokens, n_experts, top_k, tile_m);
  if (st) return st;
  if (!streams || !ffn_norm || !router_norm || !w_router || !m_bf || !logits_scratch ||
      !topk_idx || !topk_prob || !expert_counts || !expert_offsets || !tile_offsets ||
      !perm_token || !perm_prob || !route_pos)
    return LLMYB_EINVAL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_tokens == 0) return empty_plan(n_experts, expert_counts, expert_offsets, tile_offsets, s);
  const int vmax = router_vmax(d_model);
  if (n_tokens > 256 || n_tokens * top_k > 256 * kMaxTopK / 4 || vmax == 0 ||
      !router_aligned(streams, delta, ffn_norm, router_norm, w_router, m_bf) ||
      (reinterpret_cast<uintptr_t>(logits_scratch) & 15u))
    return LLMYB_EUNSUPPORTED;
  float* r = logits_scratch;
  float* logits = logits_scratch + static_cast<int64_t>(n_tokens) * d_model;
  const auto* dl = static_cast<const __nv_bfloat16*>(delta);
  auto* mb = static_cast<__nv_bfloat16*>(m_bf);
  switch (vmax) {
    case 1: router_input_kernel<1><<<n_tokens, 256, 0, s>>>(streams, dl, d_model, ffn_norm,
                                                            router_norm, eps, mb, r); break;
    case 2: router_input_kernel<2><<<n_tokens, 256, 0, s>>>(streams, dl, d_model, ffn_norm,
                                                            router_norm, eps, mb, r); break;
    case 4: router_input_kernel<4><<<n_tokens, 256, 0, s>>>(streams, dl, d_model, ffn_norm,
                                                            router_norm, eps, mb, r); break;
    default: router_input_kernel<8><<<n_tokens, 256, 0, s>>>(streams, dl, d_model, ffn_norm,
                                                             router_norm, eps, mb, r); break;
  }
  count_launch();
  router_pair_logits_kernel<<<static_cast<int>(ceil_div(n_tokens * n_experts, 8)), 256, 0, s>>>(
      r, w_router, n_tokens, d_model, n_experts, logits);
  count_launch();
  launch_router_topk(logits, nullptr, n_tokens, n_experts, top_k, topk_idx, topk_prob, s);
  plan_small_kernel<<<1, 1024, 0, s>>>(topk_idx, topk_prob, n_tokens, n_experts, top_k, tile_m,
                                       expert_counts, expert_offsets, tile_offsets, perm_token,
                                       perm_prob, route_pos, nullptr);
  count_launch();
  return launch_status();
}
