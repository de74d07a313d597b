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
#include <cstring>

namespace llmyb {
namespace {

constexpr int kMaxPlanCells = 4096;  // W * El held in shared memory by the recv plan
constexpr int kMaxPeers = 8;         // ranks of a peer-memory exchange (one node)

// Peer-memory exchange (one process per GPU, buffers mapped with CUDA IPC).
// For each rank q: where this rank's segment lives in q's receive buffer, and
// where this rank's flag lives in q's flag array.
struct PeerTable {
  __nv_bfloat16* seg[kMaxPeers];
  int* flag[kMaxPeers];
};

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Publish the end of a peer-memory send: every CTA has written its rows; the
// last CTA to finish (system-scope ticket) stores `epoch` into each peer's
// flag with release semantics.  sync = [epoch, dispatch ticket, return ticket].
// bump: this send starts a new exchange round (dispatch), so the epoch grows.
__device__ __forceinline__ void publish_send(const PeerTable& peers, int W, int* sync, int ticket,
                                             bool bump) {
  __shared__ int s_epoch;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool last = atomicAdd_system(sync + ticket, 1) == static_cast<int>(gridDim.x) - 1;
    s_epoch = 0;
    if (last) {
      s_epoch = bump ? sync[0] + 1 : sync[0];
      if (bump) sync[0] = s_epoch;
      sync[ticket] = 0;
    }
  }
  __syncthreads();
  if (s_epoch != 0 && threadIdx.x < W) {
    __threadfence_system();
    st_release_sys(peers.flag[threadIdx.x], s_epoch);
  }
}

// Wait until flags[0..W) all hold the current epoch (sync[0]), by thread 0;
// gives up after limit_ns and records LLMYB_ETIMEOUT.  Returns to all
// threads of the CTA.
__device__ __forceinline__ bool wait_flags(const int* flags, int W, const int* sync,
                                           int32_t* dev_status,
                                           uint64_t limit_ns = kWaitLimitNs) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const int e = *reinterpret_cast<const volatile int*>(sync);
    const uint64_t t0 = globaltimer_ns();
    int ok = 1;
    for (int src = 0; src < W && ok; ++src) {
      uint32_t spins = 0;
      while (ld_acquire_sys(flags + src) != e) {
        if (((++spins) & 63u) == 0u && globaltimer_ns() - t0 > limit_ns) {
          report_status(dev_status, LLMYB_ETIMEOUT);
          ok = 0;
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

__device__ __forceinline__ int expert_of_pos(const int* __restrict__ offsets, int E, int pos) {
  int lo = 0, hi = E - 1;  // last e with offsets[e] <= pos
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(offsets + mid) <= pos) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// P2P: segment q is written straight into rank q's receive buffer
// (peers.seg[q]) and the send is published through the peers' flags.
template <bool P2P>
__global__ void ep_pack_kernel(const __nv_bfloat16* __restrict__ x, int D,
                               const int* __restrict__ offsets, const int* __restrict__ perm_token,
                               const float* __restrict__ perm_prob,
                               const int* __restrict__ route_pos, int n_routes, int E, int El,
                               int W, int C, int H, __nv_bfloat16* __restrict__ send,
                               int* __restrict__ ret_route_pos, PeerTable peers, int* sync) {
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t seg_rows = static_cast<int64_t>(H) + C;
  const int vec = D / 8;
  auto seg = [&](int q) { return P2P ? peers.seg[q] : send + q * seg_rows * D; };
  // token rows: slot (q, i) <- x[perm_token[offsets[q*El] + i]]
  const int64_t row_work = static_cast<int64_t>(W) * C * vec;
  for (int64_t w = tid; w < row_work; w += stride) {
    const int64_t slot = w / vec;
    const int c = static_cast<int>(w - slot * vec);
    const int q = static_cast<int>(slot / C), i = static_cast<int>(slot - static_cast<int64_t>(q) * C);
    const int b = __ldg(offsets + q * El);
    if (i >= __ldg(offsets + (q + 1) * El) - b) continue;
    const int tok = __ldg(perm_token + b + i);
    reinterpret_cast<uint4*>(seg(q) + (H + i) * static_cast<int64_t>(D))[c] =
        __ldg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(tok) * D) + c);
  }
  // header counts and probabilities
  for (int64_t w = tid; w < static_cast<int64_t>(W) * (El + C); w += stride) {
    const int q = static_cast<int>(w / (El + C)), j = static_cast<int>(w - static_cast<int64_t>(q) * (El + C));
    int* hdr = reinterpret_cast<int*>(seg(q));
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
  if (P2P) publish_send(peers, W, sync, 1, true);
}

// Local plan over the received rows.  Rows of local expert e are ordered by
// source rank, then by their order in the source's segment (which is the
// source's plan order), so the layout is deterministic.
__global__ void __launch_bounds__(256) ep_recv_plan_kernel(
    const __nv_bfloat16* __restrict__ recv, int D, int W, int C, int H, int El, int tile_m,
    int* __restrict__ offsets_l, int* __restrict__ tile_offsets_l, int* __restrict__ perm_token_l,
    float* __restrict__ perm_prob_l, int* __restrict__ out_row, const int* wait_flags_p,
    const int* sync, int32_t* dev_status) {
  __shared__ int s_base[kMaxPlanCells];   // [W][El] first row of expert e in p's segment
  __shared__ int s_src[kMaxPlanCells];    // [W][El] rows of expert e from ranks < p
  __shared__ int s_off[257];              // local expert offsets (El <= 256)
  __shared__ int s_tot[64];               // rows received from each rank (W <= 64)
  const int64_t seg_rows = static_cast<int64_t>(H) + C;
  if (wait_flags_p != nullptr) wait_flags(wait_flags_p, W, sync, dev_status);
  // counts written by peers in this kernel's lifetime: coherent loads
  for (int cell = threadIdx.x; cell < W * El; cell += blockDim.x) {
    const int p = cell / El, e = cell - p * El;
    s_base[cell] = __ldcg(reinterpret_cast<const int*>(recv + p * seg_rows * D) + e);
  }
  __syncthreads();
  // per-rank exclusive scan over experts (counts -> first row), one thread per
  // rank; a header whose counts are negative or exceed the capacity (only
  // possible after a failed exchange) is treated as empty
  if (threadIdx.x < W) {
    const int p = threadIdx.x;
    int run = 0;
    bool bad = false;
    for (int e = 0; e < El; ++e) {
      const int c = s_base[p * El + e];
      bad |= c < 0 || c > C - run;
      s_base[p * El + e] = run;
      run += bad ? 0 : c;
    }
    if (bad) {
      report_status(dev_status, LLMYB_EINVAL);
      for (int e = 0; e < El; ++e) s_base[p * El + e] = 0;
      run = 0;
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
    perm_prob_l[pos] = __ldcg(probs + i);
    out_row[pos] = static_cast<int>(slot);
  }
}

// Return push (peer-memory exchange): the expert outputs of the rows received
// from rank q (ret_send rows [q*C, q*C + n_q), n_q from q's dispatch header)
// are stored into rank q's return buffer (peers.seg[q]), then published.
__global__ void ep_return_kernel(const __nv_bfloat16* __restrict__ ret_send,
                                 const __nv_bfloat16* __restrict__ recv, int D, int W, int C,
                                 int H, int El, PeerTable peers, int* sync) {
  __shared__ int s_n[kMaxPeers];
  const int64_t seg_rows = static_cast<int64_t>(H) + C;
  if (threadIdx.x < W) {
    const int* hdr = reinterpret_cast<const int*>(recv + threadIdx.x * seg_rows * D);
    int run = 0;
    bool bad = false;
    for (int e = 0; e < El; ++e) {
      const int c = __ldcg(hdr + e);
      bad |= c < 0 || c > C - run;
      run += bad ? 0 : c;
    }
    s_n[threadIdx.x] = bad ? 0 : run;
  }
  __syncthreads();
  const int vec = D / 8;
  const int64_t work = static_cast<int64_t>(W) * C * vec;
  for (int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; w < work;
       w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t slot = w / vec;
    const int c = static_cast<int>(w - slot * vec);
    const int q = static_cast<int>(slot / C), i = static_cast<int>(slot - static_cast<int64_t>(q) * C);
    if (i >= s_n[q]) continue;
    reinterpret_cast<uint4*>(peers.seg[q] + static_cast<int64_t>(i) * D)[c] =
        __ldg(reinterpret_cast<const uint4*>(ret_send + slot * D) + c);
  }
  publish_send(peers, W, sync, 2, false);
}

// Wait for the W return flags of the current exchange round (one CTA).
__global__ void ep_wait_kernel(const int* flags, int W, const int* sync, int32_t* dev_status,
                               uint64_t limit_ns) {
  wait_flags(flags, W, sync, dev_status, limit_ns);
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
  ep_pack_kernel<false><<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), d_model, offsets, perm_token, perm_prob, route_pos,
      n_routes, n_experts, El, world, capacity, H, static_cast<__nv_bfloat16*>(send),
      ret_route_pos, PeerTable{}, nullptr);
  count_launch();
  return launch_status();
}

// Expert-ordered plan over the received dispatch segments: offsets_l [El+1],
// tile_offsets_l [El+1] (tile_m-row tiles per expert, nullable),
// perm_token_l / perm_prob_l / out_row [W*C] (first offsets_l[El] entries
// valid).  perm_token_l indexes recv viewed as [W*(H+C), D]; out_row is the
// row of the return buffer [W*C, D] for each plan position.  With wait_flags
// (peer-memory exchange) the kernel first waits, bounded, for the W dispatch
// flags of the current round (sync[0]).
LLMYB_API int32_t llmyb_ep_recv_plan(const void* recv, int32_t d_model, int32_t world,
                                     int32_t capacity, int32_t experts_per_rank, int32_t tile_m,
                                     int32_t* offsets_l, int32_t* tile_offsets_l,
                                     int32_t* perm_token_l, float* perm_prob_l, int32_t* out_row,
                                     const int32_t* wait_flags, const int32_t* sync,
                                     int32_t* dev_status, void* stream) {
  if (wait_flags && (!sync || !dev_status)) return LLMYB_EINVAL;
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
      tile_m, offsets_l, tile_offsets_l, perm_token_l, perm_prob_l, out_row, wait_flags, sync,
      dev_status);
  count_launch();
  return launch_status();
}

// ------------------------------------------------------------------------
// Peer-memory exchange: a buffer per rank that the other ranks map with CUDA
// IPC (one process per GPU on one node; plain loads and stores over NVLink,
// no TMA and no multicast).

// Allocate `bytes` of zeroed device memory that peers can map; handle (64
// bytes, cudaIpcMemHandle_t) is written for the other processes.
LLMYB_API int32_t llmyb_ep_shared_alloc(int64_t bytes, void** dev_ptr, void* handle) {
  if (bytes <= 0 || !dev_ptr || !handle) return LLMYB_EINVAL;
  cudaError_t e = cudaMalloc(dev_ptr, static_cast<size_t>(bytes));
  if (e != cudaSuccess) return e;
  e = cudaMemset(*dev_ptr, 0, static_cast<size_t>(bytes));
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), *dev_ptr);
  if (e != cudaSuccess) {
    cudaFree(*dev_ptr);
    *dev_ptr = nullptr;
  }
  return e;
}

// Map a peer's buffer into this process.
LLMYB_API int32_t llmyb_ep_shared_open(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return LLMYB_EINVAL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

LLMYB_API int32_t llmyb_ep_shared_close(void* dev_ptr) {
  return dev_ptr ? cudaIpcCloseMemHandle(dev_ptr) : LLMYB_EINVAL;
}

LLMYB_API int32_t llmyb_ep_shared_free(void* dev_ptr) {
  return dev_ptr ? cudaFree(dev_ptr) : LLMYB_EINVAL;
}

static int32_t peer_table(int32_t world, void* const* segs, int32_t* const* flags, PeerTable* t) {
  if (world <= 0 || world > kMaxPeers || !segs || !flags) return LLMYB_EINVAL;
  *t = PeerTable{};
  for (int q = 0; q < world; ++q) {
    if (!segs[q] || !flags[q] || (reinterpret_cast<uintptr_t>(segs[q]) & 15u)) return LLMYB_EINVAL;
    t->seg[q] = static_cast<__nv_bfloat16*>(segs[q]);
    t->flag[q] = flags[q];
  }
  return LLMYB_OK;
}

// llmyb_ep_dispatch_pack writing segment q into rank q's receive buffer:
// peer_segs[q] = address of this rank's segment there, peer_flags[q] = this
// rank's dispatch flag in rank q's flag array (host arrays of W pointers).
// The last CTA starts a new round (sync[0] += 1) and stores it into every
// peer's flag.  sync: int32[3] of this rank, zero-initialised.
LLMYB_API int32_t llmyb_ep_dispatch_p2p(const void* x, int32_t d_model, const int32_t* offsets,
                                        const int32_t* perm_token, const float* perm_prob,
                                        const int32_t* route_pos, int32_t n_routes,
                                        int32_t n_experts, int32_t world, int32_t capacity,
                                        void* const* peer_segs, int32_t* const* peer_flags,
                                        int32_t* sync, int32_t* ret_route_pos, void* stream) {
  PeerTable t;
  int32_t st = peer_table(world, peer_segs, peer_flags, &t);
  if (st) return st;
  if (!offsets || !sync) return LLMYB_EINVAL;
  if (n_routes > 0 && (!x || !perm_token || !perm_prob || !route_pos || !ret_route_pos))
    return LLMYB_EINVAL;
  if (d_model <= 0 || n_routes < 0 || n_experts <= 0 || capacity < n_routes ||
      n_experts % world != 0)
    return LLMYB_EINVAL;
  if (d_model % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15u)) return LLMYB_EUNSUPPORTED;
  const int El = n_experts / world;
  const int H = llmyb_ep_header_rows(El, capacity, d_model);
  const int64_t work = std::max<int64_t>(static_cast<int64_t>(world) * capacity * (d_model / 8),
                                         static_cast<int64_t>(world) * (El + capacity));
  const int grid = static_cast<int>(std::min<int64_t>(std::max<int64_t>(ceil_div(work, 256), 1), 1184));
  ep_pack_kernel<true><<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), d_model, offsets, perm_token, perm_prob, route_pos,
      n_routes, n_experts, El, world, capacity, H, nullptr, ret_route_pos, t, sync);
  count_launch();
  return launch_status();
}

// Return push: rows [q*C, q*C + n_q) of ret_send [W*C, D] (n_q from the
// dispatch header rank q sent, in recv) go to peer_segs[q] (this rank's
// return segment in rank q's buffer); the last CTA stores the current round
// into peer_flags[q].
LLMYB_API int32_t llmyb_ep_return_p2p(const void* ret_send, const void* recv, int32_t d_model,
                                      int32_t world, int32_t capacity, int32_t experts_per_rank,
                                      void* const* peer_segs, int32_t* const* peer_flags,
                                      int32_t* sync, void* stream) {
  PeerTable t;
  int32_t st = peer_table(world, peer_segs, peer_flags, &t);
  if (st) return st;
  if (!ret_send || !recv || !sync || d_model <= 0 || capacity <= 0 || experts_per_rank <= 0)
    return LLMYB_EINVAL;
  if (d_model % 8 != 0 || (reinterpret_cast<uintptr_t>(ret_send) & 15u)) return LLMYB_EUNSUPPORTED;
  const int H = llmyb_ep_header_rows(experts_per_rank, capacity, d_model);
  const int64_t work = static_cast<int64_t>(world) * capacity * (d_model / 8);
  const int grid = static_cast<int>(std::min<int64_t>(std::max<int64_t>(ceil_div(work, 256), 1), 592));
  ep_return_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(ret_send), static_cast<const __nv_bfloat16*>(recv),
      d_model, world, capacity, H, experts_per_rank, t, sync);
  count_launch();
  return launch_status();
}

// Wait (bounded, one CTA) until flags[0..W) hold the current round sync[0];
// dev_status gets LLMYB_ETIMEOUT once limit_ns have passed (0: one second;
// at most one second).
LLMYB_API int32_t llmyb_ep_wait(const int32_t* flags, int32_t world, const int32_t* sync,
                                int32_t* dev_status, int64_t limit_ns, void* stream) {
  if (!flags || !sync || !dev_status || world <= 0 || world > 64 || limit_ns < 0)
    return LLMYB_EINVAL;
  const uint64_t limit = (limit_ns == 0 || static_cast<uint64_t>(limit_ns) > kWaitLimitNs)
                             ? kWaitLimitNs : static_cast<uint64_t>(limit_ns);
  ep_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flags, world, sync, dev_status,
                                                                   limit);
  count_launch();
  return launch_status();
}
