// Expert-parallel dispatch and combine around the routed SwiGLU experts.
//
// The reference runs every expert on one device (model/layers/moe.py:29-82,
// _moe_dispatch_fused); expert parallelism deploys the same math over W
// ranks.  Rank q owns experts [q*El, (q+1)*El); token rows stay on their rank
// (data-parallel mixers) and each MoE call exchanges the routed rows:
//
//   local plan (llmyb_route):  routes sorted by expert, so the rows bound for
//                              rank q are one contiguous range of the plan
//   pack       (this file)  :  dispatch segment q <- that range + header
//   exchange   (caller)     :  all-to-all of equal segments (NCCL or peer
//                              stores); no host-side sizes, graph capturable
//   recv plan  (this file)  :  expert-ordered plan over the received rows,
//                              read from the headers, no sort needed
//   experts    (moe_decode) :  y = p * expert(x), written straight into the
//                              return segment of the row's source rank
//   exchange   (caller)     :  all-to-all of the return segments
//   combine    (norm.cu)    :  llmyb_add_rmsnorm_routed with the remapped
//                              route positions from pack
//
// Buffer layout, bf16 rows of D elements, one segment per peer:
//   dispatch segment (H + C rows):
//     rows [0, H)     header: int32 counts[El] (rows per local expert of the
//                     receiving rank, in expert order), then fp32 probs[C]
//     rows [H, H + C) routed token rows in plan order (expert-sorted)
//   return segment (C rows): expert outputs in the dispatch row order.
// C = the sender's maximum routes (tokens x top_k), H = ceil(4 (El + C) / 2D).
// Rows past a segment's count are never read; they are not initialised.
#include "common.cuh"

#include <algorithm>

namespace llmyb {
namespace {

constexpr int kMaxPlanCells = 4096;  // W * El held in shared memory by the recv plan

__device__ __forceinline__ int expert_of_pos(const int* __restrict__ offsets, int E, int pos) {
  int lo = 0, hi = E - 1;  // last e with offsets[e] <= pos
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(offsets + mid) <= pos) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__global__ void ep_pack_kernel(const __nv_bfloat16* __restrict__ x, int D,
                               const int* __restrict__ offsets, const int* __restrict__ perm_token,
                               const float* __restrict__ perm_prob,
                               const int* __restrict__ route_pos, int n_routes, int E, int El,
                               int W, int C, int H, __nv_bfloat16* __restrict__ send,
                               int* __restrict__ ret_route_pos) {
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t seg_rows = static_cast<int64_t>(H) + C;
  const int vec = D / 8;
  // token rows: slot (q, i) <- x[perm_token[offsets[q*El] + i]]
  const int64_t row_work = static_cast<int64_t>(W) * C * vec;
  for (int64_t w = tid; w < row_work; w += stride) {
    const int64_t slot = w / vec;
    const int c = static_cast<int>(w - slot * vec);
    const int q = static_cast<int>(slot / C), i = static_cast<int>(slot - static_cast<int64_t>(q) * C);
    const int b = __ldg(offsets + q * El);
    if (i >= __ldg(offsets + (q + 1) * El) - b) continue;
    const int tok = __ldg(perm_token + b + i);
    reinterpret_cast<uint4*>(send + (q * seg_rows + H + i) * D)[c] =
        __ldg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(tok) * D) + c);
  }
  // header counts and probabilities
  for (int64_t w = tid; w < static_cast<int64_t>(W) * (El + C); w += stride) {
    const int q = static_cast<int>(w / (El + C)), j = static_cast<int>(w - static_cast<int64_t>(q) * (El + C));
    int* hdr = reinterpret_cast<int*>(send + q * seg_rows * D);
    if (j < El) {
      hdr[j] = __ldg(offsets + q * El + j + 1) - __ldg(offsets + q * El + j);
    } else {
      const int i = j - El;
      const int b = __ldg(offsets + q * El);
      if (i < __ldg(offsets + (q + 1) * El) - b)
        reinterpret_cast<float*>(hdr)[El + i] = __ldg(perm_prob + b + i);
    }
  }
  // where each route's expert output comes back: return row q*C + i
  for (int64_t w = tid; w < n_routes; w += stride) {
    const int pos = __ldg(route_pos + w);
    const int q = expert_of_pos(offsets, E, pos) / El;
    ret_route_pos[w] = q * C + (pos - __ldg(offsets + q * El));
  }
}

// Local plan over the received rows.  Rows of local expert e are ordered by
// source rank, then by their order in the source's segment (which is the
// source's plan order), so the layout is deterministic.
__global__ void __launch_bounds__(256) ep_recv_plan_kernel(
    const __nv_bfloat16* __restrict__ recv, int D, int W, int C, int H, int El, int tile_m,
    int* __restrict__ offsets_l, int* __restrict__ tile_offsets_l, int* __restrict__ perm_token_l,
    float* __restrict__ perm_prob_l, int* __restrict__ out_row) {
  __shared__ int s_base[kMaxPlanCells];   // [W][El] first row of expert e in p's segment
  __shared__ int s_src[kMaxPlanCells];    // [W][El] rows of expert e from ranks < p
  __shared__ int s_off[257];              // local expert offsets (El <= 256)
  __shared__ int s_tot[64];               // rows received from each rank (W <= 64)
  const int64_t seg_rows = static_cast<int64_t>(H) + C;
  for (int cell = threadIdx.x; cell < W * El; cell += blockDim.x) {
    const int p = cell / El, e = cell - p * El;
    s_base[cell] = __ldg(reinterpret_cast<const int*>(recv + p * seg_rows * D) + e);
  }
  __syncthreads();
  // per-rank exclusive scan over experts (counts -> first row), one thread per rank
  if (threadIdx.x < W) {
    const int p = threadIdx.x;
    int run = 0;
    for (int e = 0; e < El; ++e) {
      const int c = s_base[p * El + e];
      s_base[p * El + e] = run;
      run += c;
    }
    s_tot[p] = run;
  }
  __syncthreads();
  // per-expert scan over ranks, one thread per expert; then expert offsets
  if (threadIdx.x < El) {
    const int e = threadIdx.x;
    int run = 0;
    for (int p = 0; p < W; ++p) {
      const int next = (e + 1 < El ? s_base[p * El + e + 1] : s_tot[p]);
      const int c = next - s_base[p * El + e];
      s_src[p * El + e] = run;
      run += c;
    }
    s_off[e + 1] = run;  // total rows of expert e, scanned below
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    s_off[0] = 0;
    for (int e = 0; e < El; ++e) s_off[e + 1] += s_off[e];
  }
  __syncthreads();
  if (blockIdx.x == 0) {
    for (int e = threadIdx.x; e <= El; e += blockDim.x) offsets_l[e] = s_off[e];
    if (tile_offsets_l != nullptr && threadIdx.x == 0) {
      int t = 0;
      tile_offsets_l[0] = 0;
      for (int e = 0; e < El; ++e) {
        t += (s_off[e + 1] - s_off[e] + tile_m - 1) / tile_m;
        tile_offsets_l[e + 1] = t;
      }
    }
  }
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t slot = tid; slot < static_cast<int64_t>(W) * C; slot += stride) {
    const int p = static_cast<int>(slot / C), i = static_cast<int>(slot - static_cast<int64_t>(p) * C);
    if (i >= s_tot[p]) continue;
    int lo = 0, hi = El - 1;  // last e with base[p][e] <= i
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_base[p * El + mid] <= i) lo = mid; else hi = mid - 1;
    }
    const int pos = s_off[lo] + s_src[p * El + lo] + (i - s_base[p * El + lo]);
    const float* probs = reinterpret_cast<const float*>(recv + p * seg_rows * D) + El;
    perm_token_l[pos] = static_cast<int>(p * seg_rows + H + i);
    perm_prob_l[pos] = __ldg(probs + i);
    out_row[pos] = static_cast<int>(slot);
  }
}

}  // namespace
}  // namespace llmyb

using namespace llmyb;

// Header rows H of a dispatch segment (see the layout above).
LLMYB_API int32_t llmyb_ep_header_rows(int32_t experts_per_rank, int32_t capacity,
                                       int32_t d_model) {
  if (experts_per_rank <= 0 || capacity <= 0 || d_model <= 0) return -1;
  const int64_t bytes = 4ll * (experts_per_rank + capacity);
  return static_cast<int32_t>(ceil_div(bytes, 2ll * d_model));
}

// Fill the W dispatch segments from the local plan (offsets [E+1],
// perm_token / perm_prob [n_routes], route_pos [n_routes]) and write
// ret_route_pos [n_routes]: the row of the return buffer [W*C, D] that will
// hold each route's expert output, for llmyb_add_rmsnorm_routed.
LLMYB_API int32_t llmyb_ep_dispatch_pack(const void* x, int32_t d_model, const int32_t* offsets,
                                         const int32_t* perm_token, const float* perm_prob,
                                         const int32_t* route_pos, int32_t n_routes,
                                         int32_t n_experts, int32_t world, int32_t capacity,
                                         void* send, int32_t* ret_route_pos, void* stream) {
  if (!offsets || !send) return LLMYB_EINVAL;
  if (n_routes > 0 && (!x || !perm_token || !perm_prob || !route_pos || !ret_route_pos))
    return LLMYB_EINVAL;
  if (d_model <= 0 || n_routes < 0 || n_experts <= 0 || world <= 0 || capacity < n_routes ||
      n_experts % world != 0)
    return LLMYB_EINVAL;
  if (d_model % 8 != 0 || ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(send)) & 15u))
    return LLMYB_EUNSUPPORTED;
  const int El = n_experts / world;
  const int H = llmyb_ep_header_rows(El, capacity, d_model);
  const int64_t work = std::max<int64_t>(static_cast<int64_t>(world) * capacity * (d_model / 8),
                                         static_cast<int64_t>(world) * (El + capacity));
  const int grid = static_cast<int>(std::min<int64_t>(std::max<int64_t>(ceil_div(work, 256), 1), 1184));
  ep_pack_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), d_model, offsets, perm_token, perm_prob, route_pos,
      n_routes, n_experts, El, world, capacity, H, static_cast<__nv_bfloat16*>(send),
      ret_route_pos);
  count_launch();
  return launch_status();
}

// Expert-ordered plan over the received dispatch segments: offsets_l [El+1],
// tile_offsets_l [El+1] (tile_m-row tiles per expert, nullable),
// perm_token_l / perm_prob_l / out_row [W*C] (first offsets_l[El] entries
// valid).  perm_token_l indexes recv viewed as [W*(H+C), D]; out_row is the
// row of the return buffer [W*C, D] for each plan position.
LLMYB_API int32_t llmyb_ep_recv_plan(const void* recv, int32_t d_model, int32_t world,
                                     int32_t capacity, int32_t experts_per_rank, int32_t tile_m,
                                     int32_t* offsets_l, int32_t* tile_offsets_l,
                                     int32_t* perm_token_l, float* perm_prob_l, int32_t* out_row,
                                     void* stream) {
  if (!recv || !offsets_l || !perm_token_l || !perm_prob_l || !out_row) return LLMYB_EINVAL;
  if (d_model <= 0 || world <= 0 || capacity <= 0 || experts_per_rank <= 0 || tile_m <= 0)
    return LLMYB_EINVAL;
  if (world > 64 || experts_per_rank > 256 || world * experts_per_rank > kMaxPlanCells)
    return LLMYB_EUNSUPPORTED;
  const int H = llmyb_ep_header_rows(experts_per_rank, capacity, d_model);
  if (static_cast<int64_t>(world) * (H + capacity) > INT32_MAX) return LLMYB_EUNSUPPORTED;
  const int64_t slots = static_cast<int64_t>(world) * capacity;
  const int grid = static_cast<int>(std::min<int64_t>(std::max<int64_t>(ceil_div(slots, 256), 1), 296));
  ep_recv_plan_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(recv), d_model, world, capacity, H, experts_per_rank,
      tile_m, offsets_l, tile_offsets_l, perm_token_l, perm_prob_l, out_row);
  count_launch();
  return launch_status();
}
