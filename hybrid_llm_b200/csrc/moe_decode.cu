// Routed SwiGLU experts for small token counts (decode): weight streaming.
//
// Same math as moe_gemm.cu (reference model/layers/moe.py:68-81), for the
// regime where each expert sees a handful of rows (batch-1 decode: one row
// for each of the top-k experts; batch-64 decode: ~N*k/E rows).  There the
// cost is reading the routed experts' weights once, so the kernels stream
// every weight row exactly once with 16-byte loads and keep the few token
// rows in shared memory:
//   up  : CTA = (expert, 8 features); warp = one feature; the gate and up
//         rows of that feature are held in registers while the expert's rows
//         (16 at a time, bf16 in shared memory) are dotted against them:
//         h[pos, f] = silu(x.w_gate_f) * (x.w_up_f)
//   down: CTA = (expert, 8 output columns); warp = one column of W2:
//         y[pos, d] = p[pos] * (h[pos, :] . w2_d)
//   combine (moe_gemm.cu): out[t] = sum_s y[route_pos[t, s]]
// Experts without routed rows exit immediately, so an inactive expert costs
// no weight traffic.  Grid size scales with E x features and needs no
// device-to-host read of the routing result.
#include "common.cuh"

#include <algorithm>

namespace llmyb {
namespace {

constexpr int kTok = 16;        // token rows staged per pass

// Expert of grid slot `slot`.  Compacted grids (compact != 0) give each
// routed expert a run of CTAs: slot a is the a-th expert with rows, found from
// the plan offsets on the device (-1: fewer experts have rows than slots);
// otherwise slot e is expert e.  Called by all threads; returns to all.
__device__ __forceinline__ int slot_expert(const int* __restrict__ expert_offsets, int E, int slot,
                                           int compact) {
  if (!compact) return slot;
  __shared__ int s_e;
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int found = -1, seen = 0;
    for (int e0 = 0; e0 < E && found < 0; e0 += 32) {
      const int e = e0 + lane;
      const bool act = e < E && __ldg(expert_offsets + e + 1) > __ldg(expert_offsets + e);
      const unsigned m = __ballot_sync(0xffffffffu, act);
      const int need = slot - seen;  // index among this chunk's active experts
      if (need < __popc(m)) {
        unsigned mm = m;
        for (int i = 0; i < need; ++i) mm &= mm - 1;  // drop the lowest `need` bits
        found = e0 + __ffs(mm) - 1;
      }
      seen += __popc(m);
    }
    if (lane == 0) s_e = found;
  }
  __syncthreads();
  return s_e;
}
constexpr int kWarps = 8;       // features (up) or columns (down) per CTA
constexpr int kMaxChunk = 8;    // 16-byte chunks per lane and row: D, F <= 2048

__global__ void __launch_bounds__(256) moe_decode_up_kernel(
    const __nv_bfloat16* __restrict__ x, const int* __restrict__ perm_token,
    const int* __restrict__ expert_offsets, const __nv_bfloat16* __restrict__ w13, int D, int F,
    int E, int compact, __nv_bfloat16* __restrict__ h_perm) {
  extern __shared__ __nv_bfloat16 s_x[];  // [kTok][D]
  pdl_wait();  // the plan and the expert input come from the router
  pdl_trigger();
  const int fblocks = F / kWarps;
  const int e = slot_expert(expert_offsets, E, blockIdx.x / fblocks, compact);
  if (e < 0) return;
  const int r0 = __ldg(expert_offsets + e), r1 = __ldg(expert_offsets + e + 1);
  if (r1 <= r0) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int f = (blockIdx.x % fblocks) * kWarps + warp;
  const int nch = D / 8;
  // interleaved stack: feature f of tile j = f/128 -> gate row 256j + f%128, up row +128
  const int64_t grow = static_cast<int64_t>(e) * 2 * F + (f / 128) * 256 + (f % 128);
  const uint4* wg = reinterpret_cast<const uint4*>(w13 + grow * D);
  const uint4* wu = reinterpret_cast<const uint4*>(w13 + (grow + 128) * D);
  uint4 g4[kMaxChunk], u4[kMaxChunk];
#pragma unroll
  for (int i = 0; i < kMaxChunk; ++i) {
    const int c = lane + 32 * i;
    if (c < nch) {
      g4[i] = __ldg(wg + c);
      u4[i] = __ldg(wu + c);
    }
  }
  for (int base = r0; base < r1; base += kTok) {
    const int nt = min(kTok, r1 - base);
    __syncthreads();
    for (int i = threadIdx.x; i < nt * nch; i += blockDim.x) {
      const int t = i / nch, c = i - t * nch;
      const int tok = __ldg(perm_token + base + t);
      reinterpret_cast<uint4*>(s_x + t * D)[c] =
          __ldg(reinterpret_cast<const uint4*>(x + static_cast<int64_t>(tok) * D) + c);
    }
    __syncthreads();
    for (int t = 0; t < nt; ++t) {
      float ga = 0.f, ua = 0.f;
      const uint4* xr = reinterpret_cast<const uint4*>(s_x + t * D);
#pragma unroll
      for (int i = 0; i < kMaxChunk; ++i) {
        const int c = lane + 32 * i;
        if (c < nch) {
          const uint4 xv = xr[c];
          const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
          const uint32_t gw[4] = {g4[i].x, g4[i].y, g4[i].z, g4[i].w};
          const uint32_t uw[4] = {u4[i].x, u4[i].y, u4[i].z, u4[i].w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 xf = unpack_bf16x2(xw[k]);
            const float2 gf = unpack_bf16x2(gw[k]);
            const float2 uf = unpack_bf16x2(uw[k]);
            ga += xf.x * gf.x + xf.y * gf.y;
            ua += xf.x * uf.x + xf.y * uf.y;
          }
        }
      }
      ga = warp_sum(ga);
      ua = warp_sum(ua);
      if (lane == 0) h_perm[static_cast<int64_t>(base + t) * F + f] = f2bf(silu_mul(ga, ua));
    }
  }
}

__global__ void __launch_bounds__(256) moe_decode_down_kernel(
    const __nv_bfloat16* __restrict__ h_perm, const float* __restrict__ perm_prob,
    const int* __restrict__ expert_offsets, const __nv_bfloat16* __restrict__ w2, int D, int F,
    int E, int compact, const int* __restrict__ out_row, __nv_bfloat16* __restrict__ y_perm) {
  extern __shared__ __nv_bfloat16 s_h[];  // [kTok][F]
  // The plan (expert_offsets, perm_prob, out_row) was written two or more
  // launches earlier (the up kernel runs in between), so the expert and its
  // weight rows are fetched before waiting for h.
  const int dblocks = D / kWarps;
  const int e = slot_expert(expert_offsets, E, blockIdx.x / dblocks, compact);
  if (e < 0) return;
  const int r0 = __ldg(expert_offsets + e), r1 = __ldg(expert_offsets + e + 1);
  if (r1 <= r0) return;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int d = (blockIdx.x % dblocks) * kWarps + warp;
  const int nch = F / 8;
  const uint4* wr = reinterpret_cast<const uint4*>(w2 + (static_cast<int64_t>(e) * D + d) * F);
  uint4 w4[kMaxChunk];
#pragma unroll
  for (int i = 0; i < kMaxChunk; ++i) {
    const int c = lane + 32 * i;
    if (c < nch) w4[i] = __ldg(wr + c);
  }
  pdl_wait();  // h comes from the up kernel
  pdl_trigger();
  for (int base = r0; base < r1; base += kTok) {
    const int nt = min(kTok, r1 - base);
    __syncthreads();
    for (int i = threadIdx.x; i < nt * nch; i += blockDim.x) {
      const int t = i / nch, c = i - t * nch;
      reinterpret_cast<uint4*>(s_h + t * F)[c] =
          __ldg(reinterpret_cast<const uint4*>(h_perm + static_cast<int64_t>(base + t) * F) + c);
    }
    __syncthreads();
    for (int t = 0; t < nt; ++t) {
      float acc = 0.f;
      const uint4* hr = reinterpret_cast<const uint4*>(s_h + t * F);
#pragma unroll
      for (int i = 0; i < kMaxChunk; ++i) {
        const int c = lane + 32 * i;
        if (c < nch) {
          const uint4 hv = hr[c];
          const uint32_t hw[4] = {hv.x, hv.y, hv.z, hv.w};
          const uint32_t ww[4] = {w4[i].x, w4[i].y, w4[i].z, w4[i].w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 hf = unpack_bf16x2(hw[k]);
            const float2 wf = unpack_bf16x2(ww[k]);
            acc += hf.x * wf.x + hf.y * wf.y;
          }
        }
      }
      acc = warp_sum(acc);
      if (lane == 0) {
        const int pos = base + t;
        const int64_t orow = out_row != nullptr ? __ldg(out_row + pos) : pos;
        y_perm[orow * D + d] = f2bf(acc * __ldg(perm_prob + pos));
      }
    }
  }
}

// out[t] = sum_s y_perm[route_pos[t*k + s]]   (deterministic fp32 sum)
__global__ void moe_decode_combine_kernel(const __nv_bfloat16* __restrict__ y_perm,
                                          const int* __restrict__ route_pos, int N, int k, int D,
                                          __nv_bfloat16* __restrict__ out) {
  const int vec = D / 8;
  const int64_t total = static_cast<int64_t>(N) * vec;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / vec;
    const int c = static_cast<int>(i - t * vec);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int s = 0; s < k; ++s) {
      const int pos = __ldg(route_pos + t * k + s);
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(y_perm + static_cast<int64_t>(pos) * D) + c);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(w[j]);
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(out + t * D)[c] = o;
  }
}

}  // namespace
}  // namespace llmyb

using namespace llmyb;

LLMYB_API int64_t llmyb_moe_decode_scratch_bytes(int32_t n_tokens, int32_t top_k, int32_t d_model,
                                                 int32_t ffn) {
  if (n_tokens < 0 || top_k <= 0 || d_model <= 0 || ffn <= 0) return -1;
  const int64_t rows = static_cast<int64_t>(n_tokens) * top_k;
  auto al = [](int64_t b) { return (b + 255) / 256 * 256; };
  return al(rows * ffn * 2) + al(rows * d_model * 2);
}

namespace llmyb {
namespace {
int32_t launch_experts(const void* x, int32_t n_tokens, int32_t d_model, int32_t top_k,
                       const int32_t* perm_token, const float* perm_prob,
                       const int32_t* expert_offsets, int32_t n_experts, const void* w13,
                       const void* w2, int32_t ffn, __nv_bfloat16* h, __nv_bfloat16* y,
                       const int32_t* out_row, cudaStream_t s) {
  const int up_smem = kTok * d_model * 2, down_smem = kTok * ffn * 2;
  if (up_smem > 48 * 1024) {
    int32_t st = ensure_smem(moe_decode_up_kernel, up_smem);
    if (st) return st;
  }
  if (down_smem > 48 * 1024) {
    int32_t st = ensure_smem(moe_decode_down_kernel, down_smem);
    if (st) return st;
  }
  // at most n_rows experts have rows: a grid over those slots only, each
  // finding its expert on the device, when that is smaller than all E
  const int64_t rows = static_cast<int64_t>(n_tokens) * top_k;
  const int slots = static_cast<int>(std::min<int64_t>(n_experts, rows));
  const int compact = slots < n_experts ? 1 : 0;
  cudaError_t e = launch_pdl(moe_decode_up_kernel, dim3(slots * (ffn / kWarps)), dim3(256),
                             up_smem, s, static_cast<const __nv_bfloat16*>(x), perm_token,
                             expert_offsets, static_cast<const __nv_bfloat16*>(w13), d_model, ffn,
                             n_experts, compact, h);
  if (e != cudaSuccess) return e;
  count_launch();
  e = launch_pdl(moe_decode_down_kernel, dim3(slots * (d_model / kWarps)), dim3(256), down_smem, s,
                 static_cast<const __nv_bfloat16*>(h), perm_prob, expert_offsets,
                 static_cast<const __nv_bfloat16*>(w2), d_model, ffn, n_experts, compact, out_row,
                 y);
  if (e != cudaSuccess) return e;
  count_launch();
  return launch_status();
}

int32_t check_decode_args(const void* x, int32_t n_tokens, int32_t d_model, int32_t top_k,
                          int32_t n_experts, int32_t ffn, const void* w13, const void* w2,
                          const void* a, const void* b) {
  if (n_tokens < 0 || d_model <= 0 || top_k <= 0 || n_experts <= 0 || ffn <= 0) return LLMYB_EINVAL;
  if (!x || !w13 || !w2 || !a || !b) return LLMYB_EINVAL;
  if (d_model % 128 != 0 || ffn % 128 != 0 || d_model > 8 * 32 * kMaxChunk ||
      ffn > 8 * 32 * kMaxChunk)
    return LLMYB_EUNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w13) |
       reinterpret_cast<uintptr_t>(w2) | reinterpret_cast<uintptr_t>(a) |
       reinterpret_cast<uintptr_t>(b)) & 15u)
    return LLMYB_EUNSUPPORTED;
  return LLMYB_OK;
}
}  // namespace
}  // namespace llmyb

// Weight-streaming variant of llmyb_moe_grouped_swiglu for small token counts
// (same inputs, same plan, w13 from llmyb_moe_pack_w13).  D, F multiples of
// 128 and at most 2048.
LLMYB_API int32_t llmyb_moe_decode_swiglu(const void* x, int32_t n_tokens, int32_t d_model,
                                          int32_t top_k, const int32_t* perm_token,
                                          const float* perm_prob, const int32_t* route_pos,
                                          const int32_t* expert_offsets, int32_t n_experts,
                                          const void* w13, const void* w2, int32_t ffn,
                                          void* scratch, void* out, void* stream) {
  int32_t st = check_decode_args(x, n_tokens, d_model, top_k, n_experts, ffn, w13, w2, scratch,
                                 out);
  if (st) return st;
  if (n_tokens == 0) return LLMYB_OK;
  if (!perm_token || !perm_prob || !route_pos || !expert_offsets) return LLMYB_EINVAL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t rows = static_cast<int64_t>(n_tokens) * top_k;
  auto al = [](int64_t b) { return (b + 255) / 256 * 256; };
  auto* h = static_cast<__nv_bfloat16*>(scratch);
  auto* y = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(scratch) + al(rows * ffn * 2));
  st = launch_experts(x, n_tokens, d_model, top_k, perm_token, perm_prob, expert_offsets,
                      n_experts, w13, w2, ffn, h, y, nullptr, s);
  if (st) return st;
  const int64_t work = static_cast<int64_t>(n_tokens) * (d_model / 8);
  moe_decode_combine_kernel<<<static_cast<int>(std::min<int64_t>(ceil_div(work, 256), 1184)), 256,
                              0, s>>>(y, route_pos, n_tokens, top_k, d_model,
                                      static_cast<__nv_bfloat16*>(out));
  count_launch();
  return launch_status();
}

// The two expert kernels of llmyb_moe_decode_swiglu without the combine:
// y_rows [N*k, D] receives p * expert(x) for every route in plan order, to be
// summed per token by llmyb_add_rmsnorm_routed.  h_scratch holds [N*k, F].
LLMYB_API int32_t llmyb_moe_decode_experts(const void* x, int32_t n_tokens, int32_t d_model,
                                           int32_t top_k, const int32_t* perm_token,
                                           const float* perm_prob, const int32_t* expert_offsets,
                                           int32_t n_experts, const void* w13, const void* w2,
                                           int32_t ffn, void* h_scratch, void* y_rows,
                                           void* stream) {
  int32_t st = check_decode_args(x, n_tokens, d_model, top_k, n_experts, ffn, w13, w2, h_scratch,
                                 y_rows);
  if (st) return st;
  if (n_tokens == 0) return LLMYB_OK;
  if (!perm_token || !perm_prob || !expert_offsets) return LLMYB_EINVAL;
  return launch_experts(x, n_tokens, d_model, top_k, perm_token, perm_prob, expert_offsets,
                        n_experts, w13, w2, ffn, static_cast<__nv_bfloat16*>(h_scratch),
                        static_cast<__nv_bfloat16*>(y_rows), nullptr,
                        static_cast<cudaStream_t>(stream));
}

// llmyb_moe_decode_experts with the output row of every plan position given
// by out_row [n_rows] (y_out[out_row[pos]] = p * expert(x)[pos]).  Used by the
// expert-parallel path to write expert outputs straight into the return
// segments (ep.cu).  h_scratch holds [n_rows, F]; n_rows bounds the plan.
LLMYB_API int32_t llmyb_moe_decode_experts_to(const void* x, int32_t n_rows, int32_t d_model,
                                              const int32_t* perm_token, const float* perm_prob,
                                              const int32_t* expert_offsets, int32_t n_experts,
                                              const void* w13, const void* w2, int32_t ffn,
                                              void* h_scratch, void* y_out,
                                              const int32_t* out_row, void* stream) {
  int32_t st = check_decode_args(x, n_rows, d_model, 1, n_experts, ffn, w13, w2, h_scratch, y_out);
  if (st) return st;
  if (n_rows == 0) return LLMYB_OK;
  if (!perm_token || !perm_prob || !expert_offsets || !out_row) return LLMYB_EINVAL;
  return launch_experts(x, n_rows, d_model, 1, perm_token, perm_prob, expert_offsets, n_experts,
                        w13, w2, ffn, static_cast<__nv_bfloat16*>(h_scratch),
                        static_cast<__nv_bfloat16*>(y_out), out_row,
                        static_cast<cudaStream_t>(stream));
}
