// CSA remote compressed branch (model/layers/csa.py:77-131 prefill, :208-256
// decode step) over the causal temporal compressor
// (model/layers/compressed_attention.py:85-206), without segment ids.
//
// The compressor summarises every complete `ratio`-token block of the CSA
// input x by its mean m; the summary's key is W_k m ([H*Dh]) and its value
// W_v m ([D]), visible from the block's last position on.  A query token
// attends, per head, to its top-k visible summaries (scores q_h . k_h /
// sqrt(Dh), ties to the lower index), softmax over the selected scores; the
// heads' weighted value sums are averaged and remote_out of that joins the
// local branch before `out`.
//
// Prefill (three steps around two GEMMs of the caller):
//   csa_block_mean_kernel   block means [B, n, D] bf16 and the pending partial
//                           block's sum / count (carried into decode)
//   (GEMM)                  [keys | values] = means [W_k; W_v]^T
//   csa_remote_rows_kernel  per token, the head-averaged top-k softmax
//                           weights as one dense row P[b, t, 0:n] (bf16)
//   (GEMM)                  remote = P V, one batched [T, n] x [n, D] product
//                           instead of H*k gathered value rows per token
// Decode (three launches per layer and step):
//   csa_emit_kernel         rows whose pending block completes with this token:
//                           [key | value] = W_c mean, stored at the row's next
//                           summary slot (a CTA with no emitting row exits)
//   csa_select_kernel       per (row, head): scores over the row's summaries,
//                           top-k, softmax -> (index, weight) pairs
//   csa_gather_kernel       per row: remote = mean over heads of the weighted
//                           value rows; then the pending sum / count and the
//                           summary count advance
// Only emitted summaries are stored: the reference appends an invisible entry
// (position -1) for every non-completing decode token, which no later query
// can see, so the attention result is the same.
#include <algorithm>
#include <climits>

#include "common.cuh"

namespace llmyb {
namespace {

constexpr int kMaxTopK = 32;       // one lane per selected summary
constexpr int kMaxHeads = 32;      // one warp per head in a prefill row CTA

__device__ __forceinline__ float bf16_dot8(uint4 a, const float* q) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&a);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    s += f.x * q[2 * i] + f.y * q[2 * i + 1];
  }
  return s;
}

// Warp-level top-k + softmax over scores s[0..nv) (shared memory, destroyed:
// taken entries become -inf).  Lane i < kk (kk = min(k, nv)) returns the i-th
// selected index and its softmax weight; other lanes return (-1, 0).  Order:
// score descending, index ascending on ties (torch.topk leaves ties open).
__device__ __forceinline__ void warp_topk_softmax(float* s, int nv, int k, int& sel_j,
                                                  float& sel_w) {
  const int lane = threadIdx.x & 31;
  const int kk = min(k, nv);
  sel_j = -1;
  float sel_s = -INFINITY;
  for (int r = 0; r < kk; ++r) {
    float bv = -INFINITY;
    int bj = INT_MAX;
    for (int j = lane; j < nv; j += 32) {
      const float v = s[j];
      if (v > bv || (v == bv && j < bj)) { bv = v; bj = j; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oj = __shfl_xor_sync(0xffffffffu, bj, o);
      if (ov > bv || (ov == bv && oj < bj)) { bv = ov; bj = oj; }
    }
    if (lane == r) { sel_j = bj; sel_s = bv; }
    __syncwarp();
    if (lane == 0 && bj != INT_MAX) s[bj] = -INFINITY;
    __syncwarp();
  }
  const float top = __shfl_sync(0xffffffffu, sel_s, 0);
  float w = lane < kk ? expf(sel_s - top) : 0.f;
  const float den = warp_sum(w);
  sel_w = lane < kk ? w / den : 0.f;
}

// ------------------------------------------------------------------ prefill
// grid (n + 1, B): CTA i < n averages tokens [i*r, (i+1)*r) of row b into
// means[b, i]; CTA n sums the pending tokens [n*r, T) into pend_sum[b] and
// sets pend_cnt[b].  x rows at stride ldx (bf16), D % 8 == 0.
__global__ void csa_block_mean_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int T,
                                      int D, int r, int n, __nv_bfloat16* __restrict__ means,
                                      float* __restrict__ pend_sum, int* __restrict__ pend_cnt) {
  const int b = blockIdx.y, i = blockIdx.x;
  const int t0 = i * r, t1 = i < n ? t0 + r : T;
  const __nv_bfloat16* xb = x + static_cast<int64_t>(b) * T * ldx;
  const float inv = 1.0f / static_cast<float>(r);
  for (int c = threadIdx.x; c < D / 8; c += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int t = t0; t < t1; ++t) {
      const uint4 u = *reinterpret_cast<const uint4*>(xb + t * ldx + c * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        acc[2 * e] += f.x;
        acc[2 * e + 1] += f.y;
      }
    }
    if (i < n) {
      uint4 o;
      uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int e = 0; e < 4; ++e) op[e] = pack_bf16x2(acc[2 * e] * inv, acc[2 * e + 1] * inv);
      *reinterpret_cast<uint4*>(means + (static_cast<int64_t>(b) * n + i) * D + c * 8) = o;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) pend_sum[static_cast<int64_t>(b) * D + c * 8 + e] = acc[e];
    }
  }
  if (i == n && threadIdx.x == 0) pend_cnt[b] = T - n * r;
}

// One CTA per (token, row): blockDim = 32 * H, warp h = head h.  q rows
// [B*T, >= H*Dh] at stride ldq; keys [B*n] rows of H*Dh at stride ldk.
// Writes P[b, t, 0:n] (bf16, row stride ldp) = mean over heads of the
// top-k softmax weights over the nv = min(n, (t+1)/r) visible summaries.
// Dynamic shared memory: q [H*Dh] fp32 | P row [n] fp32 | scores [H][n] fp32.
__global__ void csa_remote_rows_kernel(const __nv_bfloat16* __restrict__ q, int64_t ldq,
                                       const __nv_bfloat16* __restrict__ keys, int64_t ldk,
                                       int T, int H, int Dh, int n, int r, int top_k, float scale,
                                       __nv_bfloat16* __restrict__ P, int64_t ldp) {
  extern __shared__ float sm[];
  const int t = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hd = H * Dh;
  float* qs = sm;
  float* prow = qs + hd;
  float* sc = prow + n + warp * n;
  const __nv_bfloat16* qt = q + (static_cast<int64_t>(b) * T + t) * ldq;
  for (int i = threadIdx.x; i < hd; i += blockDim.x) qs[i] = bf2f(qt[i]) * scale;
  for (int i = threadIdx.x; i < n; i += blockDim.x) prow[i] = 0.f;
  __syncthreads();
  const int nv = min(n, (t + 1) / r);
  const float* qh = qs + warp * Dh;
  const __nv_bfloat16* kb = keys + static_cast<int64_t>(b) * n * ldk + warp * Dh;
  for (int j = lane; j < nv; j += 32) {
    const __nv_bfloat16* kr = kb + static_cast<int64_t>(j) * ldk;
    float s = 0.f;
    for (int d = 0; d < Dh; d += 8) s += bf16_dot8(*reinterpret_cast<const uint4*>(kr + d), qh + d);
    sc[j] = s;
  }
  __syncwarp();
  int sj;
  float sw;
  warp_topk_softmax(sc, nv, top_k, sj, sw);
  if (sj >= 0) atomicAdd(prow + sj, sw / static_cast<float>(H));
  __syncthreads();
  __nv_bfloat16* pr = P + (static_cast<int64_t>(b) * T + t) * ldp;
  for (int i = threadIdx.x; i < n; i += blockDim.x) pr[i] = f2bf(prow[i]);
}

// ------------------------------------------------------------------- decode
// Emission of completed blocks.  A row emits when pend_cnt[b] + 1 == r; its
// summary's [key | value] = W_c ((pend_sum[b] + x[b]) / r) goes to slot
// count[b] of mem_k [B, cap, HD] / mem_v [B, cap, D].  Grid over output rows
// of W_c [HD + D, D] (a warp per output row, 8 rows per CTA).  The rows'
// means are staged in shared memory `group` rows at a time; groups without
// an emitting row are skipped, so a step where no block completes reads no
// weights.
__global__ void csa_emit_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                const float* __restrict__ pend_sum,
                                const int* __restrict__ pend_cnt, const int* __restrict__ count,
                                int B, int D, int HD, int r, int cap, int group,
                                const __nv_bfloat16* __restrict__ wc,
                                __nv_bfloat16* __restrict__ mem_k,
                                __nv_bfloat16* __restrict__ mem_v, int32_t* dev_status) {
  extern __shared__ float means[];  // [group][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + warp;
  const bool active = row < HD + D;
  const __nv_bfloat16* w = wc + static_cast<int64_t>(active ? row : 0) * D;
  const float inv = 1.0f / static_cast<float>(r);
  for (int b0 = 0; b0 < B; b0 += group) {
    const int nb = min(group, B - b0);
    bool any = false;  // the same value in every thread: the branches stay uniform
    for (int b = b0; b < b0 + nb; ++b) any |= pend_cnt[b] + 1 == r;
    if (!any) continue;
    __syncthreads();  // the previous group's means are no longer read
    for (int i = threadIdx.x; i < nb * D; i += blockDim.x) {
      const int bb = i / D, d = i - bb * D;
      const int64_t b = b0 + bb;
      means[i] = (pend_sum[b * D + d] + bf2f(x[b * ldx + d])) * inv;
    }
    __syncthreads();
    if (!active) continue;
    for (int bb = 0; bb < nb; ++bb) {
      const int b = b0 + bb;
      if (pend_cnt[b] + 1 != r) continue;
      const float* m = means + bb * D;
      float s = 0.f;
      for (int d = lane * 8; d < D; d += 256)
        s += bf16_dot8(*reinterpret_cast<const uint4*>(w + d), m + d);
      s = warp_sum(s);
      if (lane == 0) {
        const int slot = count[b];
        if (slot >= cap) {
          report_status(dev_status, LLMYB_EUNSUPPORTED);
        } else if (row < HD) {
          mem_k[(static_cast<int64_t>(b) * cap + slot) * HD + row] = f2bf(s);
        } else {
          mem_v[(static_cast<int64_t>(b) * cap + slot) * D + (row - HD)] = f2bf(s);
        }
      }
    }
  }
}

// Per (row b, head h) CTA of 128 threads: scores of q_h against the row's
// summaries (the stored ones plus the one emitted by this token), top-k,
// softmax; writes sel_j / sel_w [B, H, top_k] (unused slots: j = 0, w = 0).
// Shared: scores [cnt] fp32.
__global__ void csa_select_kernel(const __nv_bfloat16* __restrict__ q, int64_t ldq,
                                  const __nv_bfloat16* __restrict__ mem_k,
                                  const int* __restrict__ pend_cnt, const int* __restrict__ count,
                                  int H, int Dh, int r, int cap, int top_k, float scale,
                                  int* __restrict__ sel_j, float* __restrict__ sel_w) {
  extern __shared__ float sc[];
  __shared__ float qs[1024];
  const int b = blockIdx.y, h = blockIdx.x;
  const int HD = H * Dh;
  const int cnt = min(cap, count[b] + ((pend_cnt[b] + 1 == r) ? 1 : 0));
  for (int i = threadIdx.x; i < Dh; i += blockDim.x)
    qs[i] = bf2f(q[static_cast<int64_t>(b) * ldq + h * Dh + i]) * scale;
  __syncthreads();
  const __nv_bfloat16* kb = mem_k + static_cast<int64_t>(b) * cap * HD + h * Dh;
  for (int j = threadIdx.x; j < cnt; j += blockDim.x) {
    const __nv_bfloat16* kr = kb + static_cast<int64_t>(j) * HD;
    float s = 0.f;
    for (int d = 0; d < Dh; d += 8) s += bf16_dot8(*reinterpret_cast<const uint4*>(kr + d), qs + d);
    sc[j] = s;
  }
  __syncthreads();
  if (threadIdx.x >= 32) return;
  int sj;
  float sw;
  warp_topk_softmax(sc, cnt, top_k, sj, sw);
  const int lane = threadIdx.x;
  if (lane < top_k) {
    const int64_t o = (static_cast<int64_t>(b) * H + h) * top_k + lane;
    sel_j[o] = sj >= 0 ? sj : 0;
    sel_w[o] = sw;
  }
}

// Per row b: remote[b] = (1/H) sum over heads and selected summaries of
// w * mem_v[b, j] (bf16 out at row stride ldo); then the compressor state
// advances: an emitting row resets its pending block and counts one more
// summary, any other row adds x[b] to its pending sum.
__global__ void csa_gather_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx,
                                  const __nv_bfloat16* __restrict__ mem_v,
                                  const int* __restrict__ sel_j, const float* __restrict__ sel_w,
                                  int H, int top_k, int D, int r, int cap,
                                  float* __restrict__ pend_sum, int* __restrict__ pend_cnt,
                                  int* __restrict__ count, __nv_bfloat16* __restrict__ out,
                                  int64_t ldo) {
  extern __shared__ float pw[];  // [H*top_k] weights
  int* pj = reinterpret_cast<int*>(pw + H * top_k);
  const int b = blockIdx.x;
  const int np = H * top_k;
  for (int i = threadIdx.x; i < np; i += blockDim.x) {
    pw[i] = sel_w[static_cast<int64_t>(b) * np + i] / static_cast<float>(H);
    pj[i] = sel_j[static_cast<int64_t>(b) * np + i];
  }
  __syncthreads();
  const __nv_bfloat16* vb = mem_v + static_cast<int64_t>(b) * cap * D;
  for (int c = threadIdx.x; c < D / 8; c += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int i = 0; i < np; ++i) {
      const float w = pw[i];
      if (w == 0.f) continue;
      const uint4 u = *reinterpret_cast<const uint4*>(vb + static_cast<int64_t>(pj[i]) * D + c * 8);
      const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h2[e]);
        acc[2 * e] += w * f.x;
        acc[2 * e + 1] += w * f.y;
      }
    }
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) op[e] = pack_bf16x2(acc[2 * e], acc[2 * e + 1]);
    *reinterpret_cast<uint4*>(out + static_cast<int64_t>(b) * ldo + c * 8) = o;
  }
  // advance the compressor (every CTA thread has read pend_cnt above through
  // the emit decision only here, after the barrier)
  __syncthreads();
  const bool emit = pend_cnt[b] + 1 == r;
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float* ps = pend_sum + static_cast<int64_t>(b) * D + d;
    *ps = emit ? 0.f : *ps + bf2f(x[static_cast<int64_t>(b) * ldx + d]);
  }
  if (threadIdx.x == 0) {
    pend_cnt[b] = emit ? 0 : pend_cnt[b] + 1;
    if (emit) count[b] = min(cap, count[b] + 1);
  }
}

}  // namespace
}  // namespace llmyb

using namespace llmyb;

LLMYB_API int32_t llmyb_csa_block_means(const void* x, int64_t ldx, int32_t batch, int32_t seq,
                                        int32_t d_model, int32_t ratio, void* means,
                                        float* pend_sum, int32_t* pend_cnt, void* stream) {
  if (batch <= 0 || seq < 0 || d_model <= 0 || ratio <= 0 || ldx < d_model) return LLMYB_EINVAL;
  if (!x || !pend_sum || !pend_cnt) return LLMYB_EINVAL;
  const int n = seq / ratio;
  if (n > 0 && !means) return LLMYB_EINVAL;
  if (d_model % 8 != 0 || ldx % 8 != 0 || (reinterpret_cast<uintptr_t>(x) & 15u) ||
      (reinterpret_cast<uintptr_t>(means) & 15u))
    return LLMYB_EUNSUPPORTED;
  csa_block_mean_kernel<<<dim3(n + 1, batch), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, seq, d_model, ratio, n,
      static_cast<__nv_bfloat16*>(means), pend_sum, pend_cnt);
  count_launch();
  return launch_status();
}

LLMYB_API int32_t llmyb_csa_remote_rows(const void* q, int64_t ldq, const void* keys, int64_t ldk,
                                        int32_t batch, int32_t seq, int32_t heads,
                                        int32_t head_dim, int32_t n_summaries, int32_t ratio,
                                        int32_t top_k, void* P, int64_t ldp, void* stream) {
  if (batch <= 0 || seq < 0 || heads <= 0 || head_dim <= 0 || n_summaries < 0 || ratio <= 0 ||
      top_k <= 0 || ldp < n_summaries)
    return LLMYB_EINVAL;
  if (seq == 0 || n_summaries == 0) return LLMYB_OK;
  if (!q || !keys || !P) return LLMYB_EINVAL;
  const int hd = heads * head_dim;
  if (heads > kMaxHeads || top_k > kMaxTopK || head_dim % 8 != 0 || ldk % 8 != 0 ||
      ldk < hd || ldq < hd || (reinterpret_cast<uintptr_t>(keys) & 15u))
    return LLMYB_EUNSUPPORTED;
  const int64_t bytes = (static_cast<int64_t>(hd) + n_summaries + static_cast<int64_t>(heads) *
                         n_summaries) * 4;
  if (bytes > 220 * 1024) return LLMYB_EUNSUPPORTED;
  {
    int32_t st = ensure_smem(csa_remote_rows_kernel, static_cast<int>(bytes));
    if (st) return st;
  }
  csa_remote_rows_kernel<<<dim3(seq, batch), 32 * heads, bytes,
                           static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(q), ldq, static_cast<const __nv_bfloat16*>(keys), ldk,
      seq, heads, head_dim, n_summaries, ratio, top_k,
      1.0f / sqrtf(static_cast<float>(head_dim)), static_cast<__nv_bfloat16*>(P), ldp);
  count_launch();
  return launch_status();
}

LLMYB_API int32_t llmyb_csa_remote_step(const void* x, int64_t ldx, const void* q, int64_t ldq,
                                        int32_t batch, int32_t heads, int32_t head_dim,
                                        int32_t d_model, int32_t ratio, int32_t top_k,
                                        int32_t capacity, const void* w_comp, void* mem_k,
                                        void* mem_v, int32_t* mem_count, float* pend_sum,
                                        int32_t* pend_cnt, int32_t* sel_j, float* sel_w,
                                        void* out, int64_t ldo, int32_t* dev_status,
                                        void* stream) {
  if (batch <= 0 || heads <= 0 || head_dim <= 0 || d_model <= 0 || ratio <= 0 || top_k <= 0 ||
      capacity <= 0 || ldx < d_model || ldq < heads * head_dim || ldo < d_model)
    return LLMYB_EINVAL;
  if (!x || !q || !w_comp || !mem_k || !mem_v || !mem_count || !pend_sum || !pend_cnt ||
      !sel_j || !sel_w || !out)
    return LLMYB_EINVAL;
  const int hd = heads * head_dim;
  if (top_k > kMaxTopK || head_dim % 8 != 0 || head_dim > 1024 || d_model % 8 != 0 ||
      ldq % 8 != 0 || ldo % 8 != 0 ||
      (reinterpret_cast<uintptr_t>(q) & 15u) || (reinterpret_cast<uintptr_t>(out) & 15u) ||
      (reinterpret_cast<uintptr_t>(w_comp) & 15u) || (reinterpret_cast<uintptr_t>(mem_k) & 15u) ||
      (reinterpret_cast<uintptr_t>(mem_v) & 15u))
    return LLMYB_EUNSUPPORTED;
  const int group = std::max(1, std::min<int>(batch, (96 * 1024) / (d_model * 4)));
  const int64_t emit_bytes = static_cast<int64_t>(group) * d_model * 4;
  const int64_t sel_bytes = static_cast<int64_t>(capacity) * 4;
  const int64_t gat_bytes = static_cast<int64_t>(heads) * top_k * 8;
  if (emit_bytes > 200 * 1024 || sel_bytes > 200 * 1024 || gat_bytes > 200 * 1024)
    return LLMYB_EUNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t st = ensure_smem(csa_emit_kernel, static_cast<int>(emit_bytes));
  if (!st) st = ensure_smem(csa_select_kernel, static_cast<int>(sel_bytes));
  if (!st) st = ensure_smem(csa_gather_kernel, static_cast<int>(gat_bytes));
  if (st) return st;
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const int rows = hd + d_model;
  csa_emit_kernel<<<static_cast<int>(ceil_div(rows, 8)), 256, emit_bytes, s>>>(
      xb, ldx, pend_sum, pend_cnt, mem_count, batch, d_model, hd, ratio, capacity, group,
      static_cast<const __nv_bfloat16*>(w_comp), static_cast<__nv_bfloat16*>(mem_k),
      static_cast<__nv_bfloat16*>(mem_v), dev_status);
  csa_select_kernel<<<dim3(heads, batch), 128, sel_bytes, s>>>(
      static_cast<const __nv_bfloat16*>(q), ldq, static_cast<const __nv_bfloat16*>(mem_k),
      pend_cnt, mem_count, heads, head_dim, ratio, capacity, top_k,
      1.0f / sqrtf(static_cast<float>(head_dim)), sel_j, sel_w);
  csa_gather_kernel<<<batch, 256, gat_bytes, s>>>(
      xb, ldx, static_cast<const __nv_bfloat16*>(mem_v), sel_j, sel_w, heads, top_k, d_model,
      ratio, capacity, pend_sum, pend_cnt, mem_count, static_cast<__nv_bfloat16*>(out), ldo);
  count_launch(3);
  return launch_status();
}
