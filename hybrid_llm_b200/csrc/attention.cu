// Banded (sliding-window) causal attention: prefill and decode.
//
// Reference semantics:
//   * per-head banded attention (per-head V, or one V broadcast to all heads):
//     fused_banded_local_attention / _banded_attn_fwd_kernel
//     (sample_standalone.py:70-85, :253-322); key j is visible from query t
//     iff j <= t and t - j < window.
//   * CSA local branch (model/layers/csa.py:42-75, decode :172-206): per-head
//     softmax over the window, probabilities AVERAGED over heads, applied to
//     one shared value stream of width D:
//         out[t] = sum_j (1/H sum_h P_h[t, j]) V[j].
//
// Prefill kernels (bf16 mma.sync, fp32 accumulate, 64-query x 64-key tiles,
// K/V double-buffered with cp.async; key tiles outside the band are never
// visited, only the two band-edge tiles are masked):
//   banded_attn_kernel<D, STATS>  per-head flash attention (online softmax);
//                                 STATS = true writes only the row max and
//                                 sum-of-exp per head (first CSA pass).
//   csa_pv_kernel<DH, BM, DC>     second CSA pass: for each key tile the
//                                 head-averaged probabilities
//                                 Pbar = sum_h exp2(s_h - m_h) / (H l_h)
//                                 are formed in registers and multiplied with
//                                 a DC-wide slice of the shared V.
// Decode kernel (memory-bound on the K/V window):
//   csa_decode_kernel             one 8-CTA cluster per row; every CTA scores
//                                 one eighth of the window, the per-head
//                                 max/sum and the partial outputs are
//                                 combined through distributed shared memory.
//                                 The current token's K/V are read from the
//                                 projection and written into the ring cache.
#include <cooperative_groups.h>

#include "common.cuh"
#include "mma.cuh"
#include "sm100.cuh"

#include <algorithm>

namespace cg = cooperative_groups;

namespace llmyb {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int BMQ = 64, BNK = 64;

// key block range [kb0, kb1] visited by the query tile starting at m0
__device__ __forceinline__ void band_blocks(int m0, int T, int W, int& kb0, int& kb1) {
  const int lo = max(0, m0 - W + 1);
  const int hi = min(T - 1, m0 + BMQ - 1);
  kb0 = lo / BNK;
  kb1 = hi / BNK;
}

// Copy a [64 x width] bf16 tile (rows r0.. of a token-major tensor with the
// given row stride) into shared memory with leading dimension ld.
template <int WIDTH>
__device__ __forceinline__ void load_tile_async(__nv_bfloat16* dst, int ld,
                                                const __nv_bfloat16* src, int64_t stride, int r0,
                                                int rmax, int tid, int nthreads) {
  constexpr int VPR = WIDTH / 8;  // 16-byte vectors per row
  for (int i = tid; i < 64 * VPR; i += nthreads) {
    const int r = i / VPR, c = (i - r * VPR) * 8;
    const int row = r0 + r;
    const bool ok = row < rmax && row >= 0;
    const __nv_bfloat16* s = src + static_cast<int64_t>(ok ? row : 0) * stride + c;
    mma::cp_async16(dst + r * ld + c, s, ok);
  }
}

// --------------------------------------------------------------- per head
template <int D, bool STATS>
struct BandSmem {
  static constexpr int LD = D + 8;
  __nv_bfloat16 Q[BMQ * LD];
  __nv_bfloat16 K[2][BNK * LD];
  __nv_bfloat16 V[STATS ? 1 : 2][STATS ? 8 : BNK * LD];
};

template <int D, bool STATS>
__global__ void __launch_bounds__(128) banded_attn_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t sq, const __nv_bfloat16* __restrict__ k,
    int64_t sk, const __nv_bfloat16* __restrict__ v, int64_t sv, int v_heads, int B, int T, int H,
    int W, float scale_log2, __nv_bfloat16* __restrict__ out, int64_t so, float* __restrict__ m_out,
    float* __restrict__ l_out) {
  using SM = BandSmem<D, STATS>;
  extern __shared__ uint8_t smem_raw[];
  SM& sm = *reinterpret_cast<SM*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nqb = static_cast<int>(ceil_div(T, BMQ));
  const int qb = blockIdx.x % nqb;
  const int h = (blockIdx.x / nqb) % H;
  const int b = blockIdx.x / (nqb * H);
  const int m0 = qb * BMQ;
  int kb0, kb1;
  band_blocks(m0, T, W, kb0, kb1);
  const int64_t rowb = static_cast<int64_t>(b) * T;
  const __nv_bfloat16* qh = q + rowb * sq + h * D;
  const __nv_bfloat16* kh = k + rowb * sk + h * D;
  const __nv_bfloat16* vh = v + rowb * sv + (v_heads == 1 ? 0 : h * D);

  load_tile_async<D>(sm.Q, SM::LD, qh, sq, m0, T, tid, 128);
  load_tile_async<D>(sm.K[0], SM::LD, kh, sk, kb0 * BNK, T, tid, 128);
  if (!STATS) load_tile_async<D>(sm.V[0], SM::LD, vh, sv, kb0 * BNK, T, tid, 128);
  mma::cp_async_commit();

  const int r_lo = lane >> 2, cq = (lane & 3) * 2;
  const int t_r0 = m0 + warp * 16 + r_lo;  // query rows of this thread: t_r0, t_r0 + 8
  float o[STATS ? 1 : D / 8][4];
  if (!STATS) {
#pragma unroll
    for (int nb = 0; nb < (STATS ? 1 : D / 8); ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[nb][e] = 0.f;
  }
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  uint32_t qf[D / 16][4];

  for (int kb = kb0; kb <= kb1; ++kb) {
    const int st = (kb - kb0) & 1;
    if (kb < kb1) {
      load_tile_async<D>(sm.K[st ^ 1], SM::LD, kh, sk, (kb + 1) * BNK, T, tid, 128);
      if (!STATS) load_tile_async<D>(sm.V[STATS ? 0 : (st ^ 1)], SM::LD, vh, sv, (kb + 1) * BNK,
                                     T, tid, 128);
      mma::cp_async_commit();
      mma::cp_async_wait<1>();
    } else {
      mma::cp_async_wait<0>();
    }
    __syncthreads();
    if (kb == kb0) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) mma::load_a(qf[kk], sm.Q, SM::LD, warp * 16, kk * 16);
    }
    // S = Q K^T (16 x 64 per warp)
    float s[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[nb][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int nb = 0; nb < 8; nb += 2) {
        uint32_t bb[4];
        mma::load_b_nk(bb, sm.K[st], SM::LD, nb * 8, kk * 16);
        mma::mma_bf16(s[nb], qf[kk], bb[0], bb[1]);
        mma::mma_bf16(s[nb + 1], qf[kk], bb[2], bb[3]);
      }
    }
    // scale, mask (only the band-edge tiles), online softmax in base 2
    const int j0 = kb * BNK;
    const bool edge = (j0 + BNK - 1 > m0) || (j0 < m0 + BMQ - W) || (j0 + BNK > T);
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nb = 0; nb < 8; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[nb][e] * scale_log2;
        if (edge) {
          const int t = t_r0 + (e >> 1) * 8;
          const int j = j0 + nb * 8 + cq + (e & 1);
          if (j > t || t - j >= W || j >= T) x = -INFINITY;
        }
        s[nb][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    float corr[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
      const float mnew = fmaxf(mrow[i], mx[i]);
      const float mref = mnew == -INFINITY ? 0.f : mnew;
      corr[i] = exp2f(mrow[i] - mref);
      mrow[i] = mnew;
      mx[i] = mref;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nb = 0; nb < 8; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = exp2f(s[nb][e] - mx[e >> 1]);
        s[nb][e] = p;
        rs[e >> 1] += p;
      }
#pragma unroll
    for (int i = 0; i < 2; ++i) lrow[i] = lrow[i] * corr[i] + rs[i];
    if (!STATS) {
#pragma unroll
      for (int nb = 0; nb < (STATS ? 1 : D / 8); ++nb) {
        o[nb][0] *= corr[0];
        o[nb][1] *= corr[0];
        o[nb][2] *= corr[1];
        o[nb][3] *= corr[1];
      }
      // O += P V
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t a[4];
        a[0] = pack_bf16x2(s[2 * ks][0], s[2 * ks][1]);
        a[1] = pack_bf16x2(s[2 * ks][2], s[2 * ks][3]);
        a[2] = pack_bf16x2(s[2 * ks + 1][0], s[2 * ks + 1][1]);
        a[3] = pack_bf16x2(s[2 * ks + 1][2], s[2 * ks + 1][3]);
#pragma unroll
        for (int nb = 0; nb < (STATS ? 2 : D / 8); nb += 2) {
          uint32_t bb[4];
          mma::load_b_kn(bb, sm.V[STATS ? 0 : st], SM::LD, ks * 16, nb * 8);
          mma::mma_bf16(o[nb], a, bb[0], bb[1]);
          mma::mma_bf16(o[nb + 1], a, bb[2], bb[3]);
        }
      }
    }
    __syncthreads();
  }
  // finalize
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    lrow[i] += __shfl_xor_sync(0xffffffffu, lrow[i], 1);
    lrow[i] += __shfl_xor_sync(0xffffffffu, lrow[i], 2);
  }
  if (STATS) {
    if ((lane & 3) == 0) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int t = t_r0 + i * 8;
        if (t < T) {
          m_out[(rowb + t) * H + h] = mrow[i];
          l_out[(rowb + t) * H + h] = lrow[i];
        }
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int t = t_r0 + i * 8;
      if (t >= T) continue;
      const float inv = 1.f / lrow[i];
      __nv_bfloat16* dst = out + (rowb + t) * so + h * D;
#pragma unroll
      for (int nb = 0; nb < (STATS ? 1 : D / 8); ++nb)
        *reinterpret_cast<uint32_t*>(dst + nb * 8 + cq) =
            pack_bf16x2(o[nb][2 * i] * inv, o[nb][2 * i + 1] * inv);
    }
  }
}

// ------------------------------------------------------- CSA second pass
template <int DH, int BM, int DC>
struct CsaSmem {
  static constexpr int LK = DH + 8, LV = DC + 8;
  __nv_bfloat16 K[2][BNK * LK];
  __nv_bfloat16 V[2][BNK * LV];
  // followed by Q [BM][H*DH + 8] and stats [BM][H] (m, 1/(H l)) in dynamic memory
};

template <int DH, int BM, int DC>
__global__ void __launch_bounds__(BM * 2) csa_pv_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t sq, const __nv_bfloat16* __restrict__ k,
    int64_t sk, const __nv_bfloat16* __restrict__ v, int64_t sv, int B, int T, int H, int D, int W,
    float scale_log2, const float* __restrict__ m_in, const float* __restrict__ l_in,
    __nv_bfloat16* __restrict__ out, int64_t so) {
  using SM = CsaSmem<DH, BM, DC>;
  constexpr int NT = BM * 2;  // threads (BM/16 warps)
  extern __shared__ uint8_t smem_raw[];
  SM& sm = *reinterpret_cast<SM*>(smem_raw);
  const int LQ = H * DH + 8;
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem_raw + sizeof(SM));
  float* sM = reinterpret_cast<float*>(sQ + BM * LQ);  // [BM][H]
  float* sL = sM + BM * H;                             // [BM][H], holds 1/(H l)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nqb = static_cast<int>(ceil_div(T, BM));
  const int ndc = D / DC;
  const int dc = blockIdx.x % ndc;
  const int qb = (blockIdx.x / ndc) % nqb;
  const int b = blockIdx.x / (ndc * nqb);
  const int m0 = qb * BM;
  const int lo = max(0, m0 - W + 1), hi = min(T - 1, m0 + BM - 1);
  const int kb0 = lo / BNK, kb1 = hi / BNK;
  const int64_t rowb = static_cast<int64_t>(b) * T;

  // Q tile for all heads and the per-row stats
  {
    const int vpr = (H * DH) / 8;
    for (int i = tid; i < BM * vpr; i += NT) {
      const int r = i / vpr, c = (i - r * vpr) * 8;
      const int row = m0 + r;
      const bool ok = row < T;
      mma::cp_async16(sQ + r * LQ + c, q + (rowb + (ok ? row : 0)) * sq + c, ok);
    }
    for (int i = tid; i < BM * H; i += NT) {
      const int r = i / H, hh = i - r * H;
      const int row = m0 + r;
      float mm = 0.f, il = 0.f;
      if (row < T) {
        mm = m_in[(rowb + row) * H + hh];
        il = 1.f / (static_cast<float>(H) * l_in[(rowb + row) * H + hh]);
      }
      sM[i] = mm;
      sL[i] = il;
    }
  }
  const int steps = (kb1 - kb0 + 1) * H;
  // step i = (kb, h): K tile of head h; the V tile is loaded with h == 0
  auto issue = [&](int i) {
    const int kb = kb0 + i / H, hh = i % H, st = i & 1;
    load_tile_async<DH>(sm.K[st], SM::LK, k + rowb * sk + hh * DH, sk, kb * BNK, T, tid, NT);
    if (hh == 0)
      load_tile_async<DC>(sm.V[(i / H) & 1], SM::LV, v + rowb * sv + dc * DC, sv, kb * BNK, T,
                          tid, NT);
  };
  issue(0);
  mma::cp_async_commit();

  const int r_lo = lane >> 2, cq = (lane & 3) * 2;
  const int t_r0 = m0 + warp * 16 + r_lo;
  float o[DC / 8][4];
#pragma unroll
  for (int nb = 0; nb < DC / 8; ++nb)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[nb][e] = 0.f;
  float pbar[8][4];

  for (int i = 0; i < steps; ++i) {
    const int kb = kb0 + i / H, hh = i % H, st = i & 1;
    if (i + 1 < steps) {
      issue(i + 1);
      mma::cp_async_commit();
      mma::cp_async_wait<1>();
    } else {
      mma::cp_async_wait<0>();
    }
    __syncthreads();
    if (hh == 0) {
#pragma unroll
      for (int nb = 0; nb < 8; ++nb)
#pragma unroll
        for (int e = 0; e < 4; ++e) pbar[nb][e] = 0.f;
    }
    float s[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[nb][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < DH / 16; ++kk) {
      uint32_t a[4];
      mma::load_a(a, sQ, LQ, warp * 16, hh * DH + kk * 16);
#pragma unroll
      for (int nb = 0; nb < 8; nb += 2) {
        uint32_t bb[4];
        mma::load_b_nk(bb, sm.K[st], SM::LK, nb * 8, kk * 16);
        mma::mma_bf16(s[nb], a, bb[0], bb[1]);
        mma::mma_bf16(s[nb + 1], a, bb[2], bb[3]);
      }
    }
    const int j0 = kb * BNK;
    const float mm0 = sM[(warp * 16 + r_lo) * H + hh], mm1 = sM[(warp * 16 + r_lo + 8) * H + hh];
    const float il0 = sL[(warp * 16 + r_lo) * H + hh], il1 = sL[(warp * 16 + r_lo + 8) * H + hh];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int t = t_r0 + (e >> 1) * 8;
        const int j = j0 + nb * 8 + cq + (e & 1);
        const bool ok = j <= t && t - j < W && t < T;
        const float p = ok ? exp2f(s[nb][e] * scale_log2 - ((e >> 1) ? mm1 : mm0)) *
                                 ((e >> 1) ? il1 : il0)
                           : 0.f;
        pbar[nb][e] += p;
      }
    if (hh == H - 1) {
      const int vst = (i / H) & 1;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t a[4];
        a[0] = pack_bf16x2(pbar[2 * ks][0], pbar[2 * ks][1]);
        a[1] = pack_bf16x2(pbar[2 * ks][2], pbar[2 * ks][3]);
        a[2] = pack_bf16x2(pbar[2 * ks + 1][0], pbar[2 * ks + 1][1]);
        a[3] = pack_bf16x2(pbar[2 * ks + 1][2], pbar[2 * ks + 1][3]);
#pragma unroll
        for (int nb = 0; nb < DC / 8; nb += 2) {
          uint32_t bb[4];
          mma::load_b_kn(bb, sm.V[vst], SM::LV, ks * 16, nb * 8);
          mma::mma_bf16(o[nb], a, bb[0], bb[1]);
          mma::mma_bf16(o[nb + 1], a, bb[2], bb[3]);
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int t = t_r0 + i * 8;
    if (t >= T) continue;
    __nv_bfloat16* dst = out + (rowb + t) * so + dc * DC;
#pragma unroll
    for (int nb = 0; nb < DC / 8; ++nb)
      *reinterpret_cast<uint32_t*>(dst + nb * 8 + cq) = pack_bf16x2(o[nb][2 * i], o[nb][2 * i + 1]);
  }
}

// ------------------------------------------------------------- decode
constexpr int kClusterCtas = 8;
constexpr int kMaxChunks = 8;  // 16-byte chunks of a K row per lane: H*DH <= 2048

// Scores and partial outputs are computed from 16-byte row loads with many
// loads in flight per warp (the kernel is bound by the K/V window bytes).
// Dynamic shared memory: q [H*DH] | scores [H][kpc] | m, l, M, L [H] |
// p [kpc] | partial out [groups][D].
// Per-head sums of one key's scores.  Lane L holds in v[i] its partial
// q.k over 16-byte chunk L + 32 i; chunk i of a group of SEG lanes (one head
// of DH = 8 SEG elements) belongs to head (L / SEG) + (32 / SEG) i.  A
// reduce-scatter over the SEG lanes (each level keeps half of the values and
// adds the partner's other half) leaves every lane one head's full sum with
// log2(KP) + ... = log2(SEG) levels and KP - 1 + (levels beyond log2 KP)
// shuffles instead of KP log2(SEG).  ifin: the chunk index the lane ends with.
template <int SEG, int KP>
__device__ __forceinline__ float head_reduce(float (&v)[KP], int lane, int& ifin) {
  ifin = 0;
  int n = KP;
#pragma unroll
  for (int m = SEG / 2; m >= 1; m >>= 1) {
    if (n > 1) {
      const bool up = (lane & m) != 0;
      const int half = n / 2;
#pragma unroll
      for (int t = 0; t < KP / 2; ++t) {
        if (t < half) {
          const float send = up ? v[t] : v[t + half];
          const float keep = up ? v[t + half] : v[t];
          v[t] = keep + __shfl_xor_sync(0xffffffffu, send, m);
        }
      }
      if (up) ifin += half;
      n = half;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], m);
    }
  }
  return v[0];
}

constexpr int pow2_ceil(int x) { return x <= 1 ? 1 : 2 * pow2_ceil((x + 1) / 2); }

// Four CTAs per SM (64 registers): a batch of 64 rows is 64 clusters of 8,
// which must all be resident at once to run in a single wave.
// STAGED (small batches): the CTA's K and V ring rows are brought into
// shared memory by two bulk copies issued at entry, so the score and value
// loops read shared memory instead of waiting on one global round trip per
// key; the arithmetic is that of the unstaged kernel.
// NT threads per CTA (512 for the staged variant: more warps to hide the
// latency of a batch-1 step); KCH 16-byte K chunks per lane (H*DH <= 256*KCH);
// SEG = DH / 8 lanes per head.
template <bool STAGED, int NT, int KCH, int SEG>
__global__ void __cluster_dims__(kClusterCtas, 1, 1) __launch_bounds__(NT, STAGED ? 1 : 4)
    csa_decode_kernel(const __nv_bfloat16* __restrict__ q, int64_t sq,
                      const __nv_bfloat16* __restrict__ knew, int64_t skn,
                      const __nv_bfloat16* __restrict__ vnew, int64_t svn,
                      __nv_bfloat16* __restrict__ kcache, __nv_bfloat16* __restrict__ vcache,
                      const int* __restrict__ positions, int H, int DH, int D, int Wc,
                      float scale_log2, __nv_bfloat16* __restrict__ out, int64_t so,
                      int32_t* dev_status) {
  extern __shared__ float dsm[];
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = static_cast<int>(cluster.block_rank());
  // q stays bf16 (its input precision): lane c reads q chunk c as 16 bytes,
  // consecutive lanes consecutive chunks, so the reads are conflict-free
  const int b = blockIdx.x / kClusterCtas;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kpc = (Wc + kClusterCtas - 1) / kClusterCtas;  // keys per CTA
  const int HD = H * DH;
  const int nch = HD / 8;            // 16-byte chunks per K row
  const int seg = DH / 8;            // lanes per head within one pass (8 or 16)
  const int vch = D / 8;             // 16-byte chunks per V row
  const int groups = max(1, NT / vch);
  constexpr int NW = NT / 32;
  __nv_bfloat16* s_q = reinterpret_cast<__nv_bfloat16*>(dsm);
  float* s_sc = dsm + HD / 2;
  float* s_m = s_sc + H * kpc;
  float* s_l = s_m + H;
  float* s_M = s_l + H;
  float* s_L = s_M + H;
  float* s_p = s_L + H;
  float* s_o = s_p + kpc;            // [groups][D]
  // STAGED only: K rows [kpc][HD], V rows [kpc][D] (bf16), two mbarriers
  __nv_bfloat16* s_k = reinterpret_cast<__nv_bfloat16*>(
      dsm + ((HD / 2 + H * kpc + 4 * H + kpc + groups * D + 3) & ~3));  // 16-byte aligned
  __nv_bfloat16* s_v = s_k + static_cast<int64_t>(kpc) * HD;
  uint64_t* s_bar = reinterpret_cast<uint64_t*>(s_v + static_cast<int64_t>(kpc) * D);

  const int pos = positions[b];
  const int n_valid = min(pos + 1, Wc);
  const int cur_slot = pos % Wc;
  const int j_begin = crank * kpc;
  const int j_end = min(Wc, j_begin + kpc);
  const int nk = max(0, min(j_end, n_valid) - j_begin);  // valid keys of this CTA
  const int64_t cache_row = static_cast<int64_t>(b) * Wc;
  // rows j of K / V are read at kb + j*HD / vb + j*D (global ring, or the
  // staged copy of this CTA's keys)
  const __nv_bfloat16* kb = kcache + cache_row * HD;
  const __nv_bfloat16* vb = vcache + cache_row * D;
  bool staged_ok = true;
  if (STAGED) {
    if (tid == 0) {
      sm100::mbar_init(&s_bar[0], 1);
      sm100::mbar_init(&s_bar[1], 1);
      sm100::fence_mbar_init();
      if (nk > 0) {
        const uint32_t kbytes = static_cast<uint32_t>(nk) * HD * 2;
        const uint32_t vbytes = static_cast<uint32_t>(nk) * D * 2;
        sm100::mbar_arrive_expect_tx(&s_bar[0], kbytes);
        sm100::bulk_load(s_k, kcache + (cache_row + j_begin) * HD, kbytes, &s_bar[0]);
        sm100::mbar_arrive_expect_tx(&s_bar[1], vbytes);
        sm100::bulk_load(s_v, vcache + (cache_row + j_begin) * D, vbytes, &s_bar[1]);
      }
    }
    kb = s_k - static_cast<int64_t>(j_begin) * HD;
    vb = s_v - static_cast<int64_t>(j_begin) * D;
  }

  // the ring rows and positions were written two or more launches ago; the
  // query and the new key / value come from the projection kernel
  pdl_wait();
  pdl_trigger();
  for (int c = tid; c < nch; c += NT)
    reinterpret_cast<uint4*>(s_q)[c] = reinterpret_cast<const uint4*>(q + b * sq)[c];
  __syncthreads();
  if (STAGED && nk > 0) staged_ok = sm100::mbar_wait(&s_bar[0], 0, dev_status, nullptr);
  // ---- scores: one key per warp iteration, the whole K row in flight.  Each
  // CTA starts at a different key of its range: all CTAs begin together and
  // their ranges start 1 MB apart, so in-order streams would hit the same
  // DRAM channels at the same time.
  const int rot = nk > 0 ? static_cast<int>((static_cast<unsigned>(b) * 131u +
                                             static_cast<unsigned>(crank) * 37u) %
                                            static_cast<unsigned>(nk))
                         : 0;
  for (int it = warp; it < nk; it += NW) {
    const int jl = it + rot < nk ? it + rot : it + rot - nk;
    const int j = j_begin + jl;
    const __nv_bfloat16* kr = (j == cur_slot) ? knew + b * skn : kb + static_cast<int64_t>(j) * HD;
    uint4 kv[KCH];
#pragma unroll
    for (int i = 0; i < KCH; ++i) {
      const int c = lane + 32 * i;
      if (c < nch) kv[i] = reinterpret_cast<const uint4*>(kr)[c];
    }
    constexpr int KP = pow2_ceil(KCH);
    float pv[KP];
#pragma unroll
    for (int i = 0; i < KP; ++i) {
      const int c = lane + 32 * i;
      pv[i] = 0.f;
      if (i < KCH && c < nch) {
        const uint32_t w[4] = {kv[i].x, kv[i].y, kv[i].z, kv[i].w};
        const uint4 q4 = reinterpret_cast<const uint4*>(s_q)[c];
        const uint32_t qw[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16x2(w[e]);
          const float2 qf = unpack_bf16x2(qw[e]);
          pv[i] += qf.x * f.x + qf.y * f.y;
        }
      }
    }
    int ifin;
    const float score = head_reduce<SEG, KP>(pv, lane, ifin);
    constexpr int dup = KP < SEG ? SEG / KP - 1 : 0;  // lanes holding the same head
    if ((lane & dup) == 0 && (lane & ~(SEG - 1)) + 32 * ifin < nch)
      s_sc[((lane + 32 * ifin) / SEG) * kpc + jl] = score * scale_log2;
    if (j == cur_slot) {  // append the current token to the ring
      for (int c = lane; c < nch; c += 32)
        reinterpret_cast<uint4*>(kcache + (cache_row + j) * HD)[c] =
            reinterpret_cast<const uint4*>(knew + b * skn)[c];
      for (int c = lane; c < vch; c += 32)
        reinterpret_cast<uint4*>(vcache + (cache_row + j) * D)[c] =
            reinterpret_cast<const uint4*>(vnew + b * svn)[c];
    }
  }
  __syncthreads();
  for (int hh = warp; hh < H; hh += NW) {
    float mx = -INFINITY;
    for (int j = lane; j < nk; j += 32) mx = fmaxf(mx, s_sc[hh * kpc + j]);
    mx = warp_max(mx);
    float sum = 0.f;
    if (mx != -INFINITY)
      for (int j = lane; j < nk; j += 32) sum += exp2f(s_sc[hh * kpc + j] - mx);
    sum = warp_sum(sum);
    if (lane == 0) {
      s_m[hh] = mx;
      s_l[hh] = sum;
    }
  }
  cluster.sync();
  // ---- cluster-wide per-head max / sum
  for (int hh = warp; hh < H; hh += NW) {
    float mloc = -INFINITY, lloc = 0.f;
    if (lane < kClusterCtas) {
      mloc = *cluster.map_shared_rank(&s_m[hh], lane);
      lloc = *cluster.map_shared_rank(&s_l[hh], lane);
    }
    const float M = warp_max(mloc);
    const float L = warp_sum(mloc == -INFINITY ? 0.f : lloc * exp2f(mloc - M));
    if (lane == 0) {
      s_M[hh] = M;
      s_L[hh] = L;
    }
  }
  __syncthreads();
  // ---- head-averaged probabilities of this CTA's keys
  for (int j = tid; j < nk; j += NT) {
    float p = 0.f;
    for (int hh = 0; hh < H; ++hh) p += exp2f(s_sc[hh * kpc + j] - s_M[hh]) / s_L[hh];
    s_p[j] = p / static_cast<float>(H);
  }
  __syncthreads();
  // ---- partial output: thread = (key group, 16-byte column chunk)
  if (STAGED && nk > 0 && staged_ok) staged_ok = sm100::mbar_wait(&s_bar[1], 0, dev_status, nullptr);
  {
    const int g = tid / vch, c = tid - g * vch;
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (g < groups) {
      int j = g;
      // eight keys' chunks in flight per thread, then their products in key order
      for (; j + 7 * groups < nk; j += 8 * groups) {
        uint4 v8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int jj = j_begin + j + u * groups;
          const __nv_bfloat16* vr =
              (jj == cur_slot) ? vnew + b * svn : vb + static_cast<int64_t>(jj) * D;
          v8[u] = reinterpret_cast<const uint4*>(vr)[c];
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float p = s_p[j + u * groups];
          const uint32_t w[4] = {v8[u].x, v8[u].y, v8[u].z, v8[u].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = unpack_bf16x2(w[e]);
            acc[2 * e] += p * f.x;
            acc[2 * e + 1] += p * f.y;
          }
        }
      }
      for (; j < nk; j += groups) {
        const int jj = j_begin + j;
        const __nv_bfloat16* vr =
            (jj == cur_slot) ? vnew + b * svn : vb + static_cast<int64_t>(jj) * D;
        const uint4 v4 = reinterpret_cast<const uint4*>(vr)[c];
        const float p = s_p[j];
        const uint32_t w[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16x2(w[e]);
          acc[2 * e] += p * f.x;
          acc[2 * e + 1] += p * f.y;
        }
      }
      for (int e = 0; e < 8; ++e) s_o[g * D + c * 8 + e] = acc[e];
    }
  }
  __syncthreads();
  if (groups > 1) {
    for (int d = tid; d < D; d += NT) {
      float acc = s_o[d];
      for (int g = 1; g < groups; ++g) acc += s_o[g * D + d];
      s_o[d] = acc;
    }
  }
  cluster.sync();
  // ---- reduce this CTA's column slice over the cluster
  const int cols = D / kClusterCtas;
  for (int d = crank * cols + tid; d < (crank + 1) * cols; d += NT) {
    float acc = 0.f;
    for (int r = 0; r < kClusterCtas; ++r) acc += *cluster.map_shared_rank(&s_o[d], r);
    out[b * so + d] = f2bf(acc);
  }
  if (STAGED && nk > 0) {  // no bulk copy may still be writing when the CTA exits
    sm100::mbar_wait(&s_bar[0], 0, dev_status, nullptr);
    sm100::mbar_wait(&s_bar[1], 0, dev_status, nullptr);
  }
  cluster.sync();  // keep shared memory alive until every peer finished reading
}

template <int D, bool STATS>
int32_t launch_band(const __nv_bfloat16* q, int64_t sq, const __nv_bfloat16* k, int64_t sk,
                    const __nv_bfloat16* v, int64_t sv, int v_heads, int B, int T, int H, int W,
                    float scale, __nv_bfloat16* out, int64_t so, float* m_out, float* l_out,
                    cudaStream_t s) {
  constexpr int bytes = sizeof(BandSmem<D, STATS>);
  {
    int32_t st = ensure_smem(banded_attn_kernel<D, STATS>, bytes);
    if (st) return st;
  }
  const int grid = B * H * static_cast<int>(ceil_div(T, BMQ));
  banded_attn_kernel<D, STATS><<<grid, 128, bytes, s>>>(q, sq, k, sk, v, sv, v_heads, B, T, H, W,
                                                        scale * kLog2e, out, so, m_out, l_out);
  count_launch();
  return launch_status();
}

bool aligned16(const void* p, int64_t stride) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && stride % 8 == 0;
}

// One token's row of width w: src -> dst, 16-byte vectors when both sides
// allow (VEC), else bf16 elements.
template <bool VEC>
__device__ __forceinline__ void copy_row(const __nv_bfloat16* __restrict__ src,
                                         __nv_bfloat16* __restrict__ dst, int w) {
  if constexpr (VEC) {
    for (int i = threadIdx.x; i < w / 8; i += blockDim.x)
      reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
  } else {
    for (int i = threadIdx.x; i < w; i += blockDim.x) dst[i] = src[i];
  }
}

// The decode ring after a prompt: token p of the last min(T, W) lands in slot
// p % W of kcache [B, W, kw] and vcache [B, W, vw] (blockIdx.x: the token's
// index among them, blockIdx.y: the batch row).
template <bool VEC>
__global__ void csa_ring_write_kernel(const __nv_bfloat16* __restrict__ k, int64_t sk,
                                      const __nv_bfloat16* __restrict__ v, int64_t sv, int T,
                                      int kw, int vw, __nv_bfloat16* __restrict__ kcache,
                                      __nv_bfloat16* __restrict__ vcache, int W) {
  const int b = blockIdx.y;
  const int p = max(0, T - W) + static_cast<int>(blockIdx.x);
  const int64_t row = static_cast<int64_t>(b) * T + p;
  const int64_t slot = static_cast<int64_t>(b) * W + p % W;
  copy_row<VEC>(k + row * sk, kcache + slot * kw, kw);
  copy_row<VEC>(v + row * sv, vcache + slot * vw, vw);
}

}  // namespace
}  // namespace llmyb

namespace llmyb {
// csa_tc.cu: the tcgen05 prefill (statistics, head-averaged probabilities, PV)
void csa_tc_geometry(int T, int W, int* nqt, int* nb);
bool csa_tc_supported(int head_dim, int d_model, int64_t q_stride, int64_t k_stride,
                      int64_t v_stride, int64_t out_stride);
int32_t csa_prefill_tc(const void* q, int64_t sq, const void* k, int64_t sk, const void* v,
                       int64_t sv, int B, int T, int H, int DH, int D, int W, float scale,
                       void* out, int64_t so, void* scratch, int32_t* dev_status,
                       cudaStream_t s);
}  // namespace llmyb

using namespace llmyb;

LLMYB_API int64_t llmyb_csa_prefill_scratch_bytes(int32_t batch, int32_t seq, int32_t heads,
                                                  int32_t window) {
  if (batch < 0 || seq < 0 || heads <= 0 || window <= 0) return -1;
  const int64_t stats = static_cast<int64_t>(batch) * seq * heads * 2 * sizeof(float);
  if (seq == 0) return stats;
  int nqt = 0, nb = 0;
  csa_tc_geometry(seq, std::max(1, std::min<int>(window, seq)), &nqt, &nb);
  return (stats + 255) / 256 * 256 + static_cast<int64_t>(batch) * nqt * nb * 128 * 128 * 2;
}

// CSA local branch, prefill: q,k [B*T, H*DH] (strides), v [B*T, D] shared
// value stream (stride sv); out [B*T, D].  scratch holds the per-head row
// statistics and the head-averaged probability tiles
// (llmyb_csa_prefill_scratch_bytes).  Head dim 64 / 128 with D % 128 == 0 runs
// on tcgen05 (csa_tc.cu); other shapes on the mma.sync kernels below.
LLMYB_API int32_t llmyb_csa_local_prefill(const void* q, int64_t q_stride, const void* k,
                                          int64_t k_stride, const void* v, int64_t v_stride,
                                          int32_t batch, int32_t seq, int32_t heads,
                                          int32_t head_dim, int32_t d_model, int32_t window,
                                          void* out, int64_t out_stride, void* scratch,
                                          int32_t* dev_status, void* stream) {
  if (!q || !k || !v || !out || !scratch || batch < 0 || seq < 0 || heads <= 0 || window <= 0)
    return LLMYB_EINVAL;
  if (batch == 0 || seq == 0) return LLMYB_OK;
  if (!aligned16(q, q_stride) || !aligned16(k, k_stride) || !aligned16(v, v_stride) ||
      !aligned16(out, out_stride) || d_model % 64 != 0)
    return LLMYB_EUNSUPPORTED;
  // csa.py:42: the window never exceeds the sequence
  const int w = std::max(1, std::min<int>(window, seq));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (csa_tc_supported(head_dim, d_model, q_stride, k_stride, v_stride, out_stride) &&
      (reinterpret_cast<uintptr_t>(scratch) & 15u) == 0)
    return csa_prefill_tc(q, q_stride, k, k_stride, v, v_stride, batch, seq, heads, head_dim,
                          d_model, w, 1.0f / sqrtf(static_cast<float>(head_dim)), out, out_stride,
                          scratch, dev_status, s);
  auto Q = static_cast<const __nv_bfloat16*>(q);
  auto K = static_cast<const __nv_bfloat16*>(k);
  auto V = static_cast<const __nv_bfloat16*>(v);
  auto O = static_cast<__nv_bfloat16*>(out);
  float* m = static_cast<float*>(scratch);
  float* l = m + static_cast<int64_t>(batch) * seq * heads;
  const float scale = 1.0f / sqrtf(static_cast<float>(head_dim));
  int32_t st;
  if (head_dim == 64)
    st = launch_band<64, true>(Q, q_stride, K, k_stride, V, v_stride, 1, batch, seq, heads, w,
                               scale, nullptr, 0, m, l, s);
  else if (head_dim == 128)
    st = launch_band<128, true>(Q, q_stride, K, k_stride, V, v_stride, 1, batch, seq, heads, w,
                                scale, nullptr, 0, m, l, s);
  else
    return LLMYB_EUNSUPPORTED;
  if (st) return st;
  const int hd = heads * head_dim;
  constexpr int DC = 64;
  auto run = [&](auto kern, int BM, int base_bytes, int dh) -> int32_t {
    const int bytes = base_bytes + BM * (hd + 8) * 2 + BM * heads * 2 * 4;
    if (bytes > 227 * 1024) return LLMYB_EUNSUPPORTED;
    int32_t e = ensure_smem(kern, bytes);
    if (e) return e;
    const int grid = batch * static_cast<int>(ceil_div(seq, BM)) * (d_model / DC);
    kern<<<grid, BM * 2, bytes, s>>>(Q, q_stride, K, k_stride, V, v_stride, batch, seq, heads,
                                     d_model, w, scale * kLog2e, m, l, O, out_stride);
    count_launch();
    (void)dh;
    return launch_status();
  };
  if (head_dim == 64) {
    if (hd <= 1024) return run(csa_pv_kernel<64, 64, DC>, 64, sizeof(CsaSmem<64, 64, DC>), 64);
    return run(csa_pv_kernel<64, 32, DC>, 32, sizeof(CsaSmem<64, 32, DC>), 64);
  }
  if (hd <= 1024) return run(csa_pv_kernel<128, 64, DC>, 64, sizeof(CsaSmem<128, 64, DC>), 128);
  return run(csa_pv_kernel<128, 32, DC>, 32, sizeof(CsaSmem<128, 32, DC>), 128);
}

// CSA local branch, decode: one new token per row.  q/knew [B, H*DH],
// vnew [B, D] (row strides); the ring caches kcache [B, Wc, H*DH] and
// vcache [B, Wc, D] hold token p at slot p % Wc; positions[b] is the new
// token's position (its K/V are written to slot positions[b] % Wc).  The
// window is the last min(positions[b] + 1, Wc) tokens (csa.py:185-187).
// Ring caches after a prompt (csa.py:208-258 cache layout): kcache [B, W, kw],
// vcache [B, W, vw] get token p of the last min(T, W) tokens of k [B*T, kw]
// (token stride k_stride) and v [B*T, vw] at slot p % W; other slots keep
// their contents.
LLMYB_API int32_t llmyb_csa_ring_write(const void* k, int64_t k_stride, const void* v,
                                       int64_t v_stride, int32_t batch, int32_t seq,
                                       int32_t k_width, int32_t v_width, void* kcache,
                                       void* vcache, int32_t window, void* stream) {
  if (!k || !v || !kcache || !vcache || batch < 0 || seq < 0 || k_width <= 0 || v_width <= 0 ||
      window <= 0 || k_stride < k_width || v_stride < v_width)
    return LLMYB_EINVAL;
  if (batch == 0 || seq == 0) return LLMYB_OK;
  if (batch > 65535) return LLMYB_EUNSUPPORTED;
  const int n = std::min(seq, window);
  const bool vec = aligned16(k, k_stride) && aligned16(v, v_stride) && aligned16(kcache, k_width) &&
                   aligned16(vcache, v_width) && k_width % 8 == 0 && v_width % 8 == 0;
  const auto* kp = static_cast<const __nv_bfloat16*>(k);
  const auto* vp = static_cast<const __nv_bfloat16*>(v);
  auto* kc = static_cast<__nv_bfloat16*>(kcache);
  auto* vc = static_cast<__nv_bfloat16*>(vcache);
  const dim3 grid(static_cast<unsigned>(n), static_cast<unsigned>(batch));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (vec)
    csa_ring_write_kernel<true><<<grid, 128, 0, s>>>(kp, k_stride, vp, v_stride, seq, k_width,
                                                     v_width, kc, vc, window);
  else
    csa_ring_write_kernel<false><<<grid, 128, 0, s>>>(kp, k_stride, vp, v_stride, seq, k_width,
                                                      v_width, kc, vc, window);
  count_launch();
  return launch_status();
}

LLMYB_API int32_t llmyb_csa_local_decode(const void* q, int64_t q_stride, const void* knew,
                                         int64_t knew_stride, const void* vnew,
                                         int64_t vnew_stride, void* kcache, void* vcache,
                                         const int32_t* positions, int32_t batch, int32_t heads,
                                         int32_t head_dim, int32_t d_model, int32_t window,
                                         void* out, int64_t out_stride, int32_t* dev_status,
                                         void* stream) {
  if (!q || !knew || !vnew || !kcache || !vcache || !positions || !out || batch < 0 ||
      heads <= 0 || head_dim <= 0 || window <= 0)
    return LLMYB_EINVAL;
  if (batch == 0) return LLMYB_OK;
  const int hd = heads * head_dim;
  if (d_model % (8 * kClusterCtas) != 0 || head_dim % 8 != 0 || hd > 8 * 32 * kMaxChunks ||
      d_model > 8 * 256 || !(head_dim == 64 || head_dim == 128))
    return LLMYB_EUNSUPPORTED;
  if (((reinterpret_cast<uintptr_t>(knew) | reinterpret_cast<uintptr_t>(vnew) |
        reinterpret_cast<uintptr_t>(kcache) | reinterpret_cast<uintptr_t>(vcache)) & 15u) ||
      knew_stride % 8 != 0 || vnew_stride % 8 != 0)
    return LLMYB_EUNSUPPORTED;
  const int kpc = (window + kClusterCtas - 1) / kClusterCtas;
  auto base_floats = [&](int nt) {
    const int groups = std::max(1, nt / (d_model / 8));
    return (hd / 2 + heads * kpc + 4 * heads + kpc + groups * d_model + 3) & ~3;
  };
  const int64_t staged_bytes = static_cast<int64_t>(base_floats(512)) * 4 +
                               static_cast<int64_t>(kpc) * (hd + d_model) * 2 + 16;
  // small batches: one cluster per row is far from filling the GPU, so each
  // CTA stages its keys in shared memory (one CTA of 512 threads per SM)
  const bool staged = batch <= 32 && staged_bytes <= 220 * 1024;
  const int bytes = staged ? static_cast<int>(staged_bytes) : base_floats(256) * 4;
  const int kch = hd <= 768 ? 3 : (hd <= 1024 ? 4 : 8);
  const bool seg16 = head_dim == 128;
  if (bytes > 227 * 1024) return LLMYB_EUNSUPPORTED;
  auto launch = [&](auto kernel, int nt) -> int32_t {
    {
      int32_t st = ensure_smem(kernel, bytes);
      if (st) return st;
    }
    return static_cast<int32_t>(launch_pdl(
        kernel, dim3(batch * kClusterCtas), dim3(nt), bytes, static_cast<cudaStream_t>(stream),
        static_cast<const __nv_bfloat16*>(q), q_stride, static_cast<const __nv_bfloat16*>(knew),
        knew_stride, static_cast<const __nv_bfloat16*>(vnew), vnew_stride,
        static_cast<__nv_bfloat16*>(kcache), static_cast<__nv_bfloat16*>(vcache), positions,
        heads, head_dim, d_model, window, kLog2e / sqrtf(static_cast<float>(head_dim)),
        static_cast<__nv_bfloat16*>(out), out_stride, dev_status));
  };
  int32_t st;
#define LLMYB_CSA(ST, NTV, SEGV)                                                         \
  (kch == 3 ? launch(csa_decode_kernel<ST, NTV, 3, SEGV>, NTV)                          \
   : kch == 4 ? launch(csa_decode_kernel<ST, NTV, 4, SEGV>, NTV)                        \
              : launch(csa_decode_kernel<ST, NTV, 8, SEGV>, NTV))
  if (staged)
    st = seg16 ? LLMYB_CSA(true, 512, 16) : LLMYB_CSA(true, 512, 8);
  else
    st = seg16 ? LLMYB_CSA(false, 256, 16) : LLMYB_CSA(false, 256, 8);
#undef LLMYB_CSA
  if (st) return st;
  count_launch();
  return launch_status();
}
