// CSA local branch, prefill, on 5th-generation tensor cores.
//
// Reference: model/layers/csa.py:42-75: per head h, P_h = softmax over the
// window of scale q_h.k_h (key j visible from query t iff j <= t and
// t - j < W); the probabilities are AVERAGED over heads and applied to one
// shared value stream of width D:
//     out[t] = sum_j Pbar[t, j] V[j],   Pbar = (1/H) sum_h P_h.
//
// Three kernels, each a persistent loop over work units with TMA loads,
// tcgen05.mma into TMEM and bounded mbarrier waits:
//   csa_stats_tc  (b, h, 128-query tile): S = Q_h K_h^T per 128-key block of
//                 the band; per query row the base-2 max m_h and sum l_h of
//                 exp2(c s - m_h), c = scale * log2(e).
//   csa_pbar_tc   (b, query tile, key block): for every head S_h of the
//                 block, Pbar = sum_h exp2(c s - m_h) / (H l_h), masked to the
//                 band; written as a bf16 [128 x 128] tile.  Eight softmax
//                 warps, two per TMEM lane quarter, each summing 64 columns.
//                 With few units (short prompts) a cluster of G CTAs shares
//                 a unit: each sums H/G heads into an fp32 partial tile in its
//                 shared memory, and after a bounded cluster-wide handoff
//                 (remote mbarrier arrivals) each CTA adds one slice of the G
//                 partials through distributed shared memory, in rank order.
//   csa_pv_tc     (b, query tile, NSW-column slice of D): O = sum over the
//                 band's key blocks of Pbar_blk V_blk, V read in its natural
//                 [key][d] layout as an MN-major B operand; two TMEM
//                 accumulators so one unit's epilogue overlaps the next
//                 unit's products.
// Every score tile is computed twice (statistics, then probabilities),
// independently of D; the PV product runs once per output column.
#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.h"

#include <algorithm>

namespace llmyb {
namespace {

constexpr int kR = 128;               // queries per tile = keys per block
constexpr int kBoxB = 128 * 64 * 2;   // one TMA box: 128 rows x 64 bf16
constexpr int kTileP = kR * kR * 2;   // one Pbar tile (bf16)

struct Geo {
  int B, T, H, W, nqt, nb;
  __device__ __forceinline__ int kb0(int qt) const { return max(0, qt * kR - W + 1) / kR; }
  __device__ __forceinline__ int nblk(int qt) const { return qt - kb0(qt) + 1; }
};

// band-edge test: every key of block kb is visible from every query of tile qt
__device__ __forceinline__ bool interior(int qt, int kb, int W) {
  return kb * kR + kR - 1 <= qt * kR && qt * kR + kR - 1 - kb * kR < W;
}

// ------------------------------------------------------------------ stats
template <int DH>
struct StatsLayout {
  static constexpr int kTile = kR * DH * 2;
  static constexpr int kQ = 0;              // 2 Q buffers
  static constexpr int kK = 2 * kTile;      // 2 K stages
  static constexpr int kBar = 4 * kTile;
  static constexpr int kSmem = kBar + 256 + 1024;
};

template <int DH>
__global__ void __launch_bounds__(192, 1) csa_stats_tc_kernel(
    const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
    Geo g, float c, float* __restrict__ m_out, float* __restrict__ l_out, int32_t* dev_status) {
  using L = StatsLayout<DH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 2;
  uint64_t* k_full = bars + 4;
  uint64_t* k_empty = bars + 6;
  uint64_t* s_full = bars + 8;
  uint64_t* s_empty = bars + 10;
  uint64_t* mma_done = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = g.B * g.H * g.nqt;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&q_full[i], 1);
      sm100::mbar_init(&q_empty[i], 1);
      sm100::mbar_init(&k_full[i], 1);
      sm100::mbar_init(&k_empty[i], 1);
      sm100::mbar_init(&s_full[i], 1);
      sm100::mbar_init(&s_empty[i], 4);
    }
    sm100::mbar_init(mma_done, 1);
    *abort_flag = 0;
    sm100::fence_mbar_init();
    sm100::tma_prefetch_desc(&map_q);
    sm100::tma_prefetch_desc(&map_k);
  }
  if (warp == 1) sm100::tmem_alloc(tmem_slot, 256);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA
    uint32_t nq = 0, nk = 0;
    bool ok = true;
    int gb = 0, ul = 0;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++ul) {
      const int qt = u % g.nqt, h = (u / g.nqt) % g.H, b = u / (g.nqt * g.H);
      const int qb = ul & 1;
      if (!sm100::mbar_wait_warp(&q_empty[qb], ((ul >> 1) & 1) ^ 1u, dev_status, abort_flag)) {
        ok = false;
        break;
      }
      if (lane == 0) {
        sm100::mbar_arrive_expect_tx(&q_full[qb], L::kTile);
#pragma unroll
        for (int cc = 0; cc < DH / 64; ++cc)
          sm100::tma_load_3d(&map_q, &q_full[qb], smem + L::kQ + qb * L::kTile + cc * kBoxB,
                             h * DH + cc * 64, qt * kR, b);
      }
      ++nq;
      const int kb0 = g.kb0(qt), nblk = g.nblk(qt);
      for (int i = 0; i < nblk; ++i, ++gb) {
        const int s = gb & 1;
        if (!sm100::mbar_wait_warp(&k_empty[s], ((gb >> 1) & 1) ^ 1u, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          sm100::mbar_arrive_expect_tx(&k_full[s], L::kTile);
#pragma unroll
          for (int cc = 0; cc < DH / 64; ++cc)
            sm100::tma_load_3d(&map_k, &k_full[s], smem + L::kK + s * L::kTile + cc * kBoxB,
                               h * DH + cc * 64, (kb0 + i) * kR, b);
        }
        ++nk;
      }
    }
    for (uint32_t i = 1; i <= 2; ++i) {
      if (nq >= i) sm100::mbar_wait_warp(&q_full[(nq - i) & 1], ((nq - i) >> 1) & 1, dev_status, nullptr);
      if (nk >= i) sm100::mbar_wait_warp(&k_full[(nk - i) & 1], ((nk - i) >> 1) & 1, dev_status, nullptr);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    constexpr uint32_t idesc = sm100::make_idesc_bf16_f32(kR, kR);
    const uint32_t sq = sm100::smem_u32(smem + L::kQ), sk = sm100::smem_u32(smem + L::kK);
    bool ok = true;
    int gb = 0, ul = 0;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++ul) {
      const int qt = u % g.nqt;
      const int qb = ul & 1, nblk = g.nblk(qt);
      for (int i = 0; i < nblk; ++i, ++gb) {
        const int s = gb & 1;
        const uint32_t ph = (gb >> 1) & 1;
        if ((i == 0 && !sm100::mbar_wait_warp(&q_full[qb], (ul >> 1) & 1, dev_status, abort_flag)) ||
            !sm100::mbar_wait_warp(&k_full[s], ph, dev_status, abort_flag) ||
            !sm100::mbar_wait_warp(&s_empty[s], ph ^ 1u, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        if (lane == 0) {
          const uint32_t qa = sq + qb * L::kTile, ka = sk + s * L::kTile;
#pragma unroll
          for (int kk = 0; kk < DH / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kBoxB + (kk & 3) * 32;
            sm100::umma_bf16_ss(tmem_base + s * 128, sm100::make_sw128_kmajor_desc(qa + off),
                                sm100::make_sw128_kmajor_desc(ka + off), idesc, kk > 0 ? 1u : 0u);
          }
          sm100::umma_commit(&s_full[s]);
          sm100::umma_commit(&k_empty[s]);
          if (i == nblk - 1) sm100::umma_commit(&q_empty[qb]);
        }
        __syncwarp();
      }
    }
    if (lane == 0) sm100::umma_commit(mma_done);
    __syncwarp();
    sm100::mbar_wait_warp(mma_done, 0, dev_status, nullptr);
  } else {
    // ------------------------------------------------- row statistics
    const int qw = warp & 3, row = qw * 32 + lane;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(qw * 32) << 16);
    int gb = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const int qt = u % g.nqt, h = (u / g.nqt) % g.H, b = u / (g.nqt * g.H);
      const int t = qt * kR + row, kb0 = g.kb0(qt), nblk = g.nblk(qt);
      float m = -INFINITY, l = 0.f;
      for (int i = 0; i < nblk; ++i, ++gb) {
        const int sb = gb & 1;
        if (!sm100::mbar_wait_warp(&s_full[sb], (gb >> 1) & 1, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        uint32_t sr[4][32];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) sm100::tmem_ld_32x32b_x32(t_lane + sb * 128 + 32 * cc, sr[cc]);
        sm100::tmem_ld_wait();
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) sm100::tmem_regs_ready(sr[cc]);
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&s_empty[sb]);
        const int kb = kb0 + i;
        if (!interior(qt, kb, g.W)) {
          const int lo = t - g.W + 1 - kb * kR, hi = t - kb * kR;
#pragma unroll
          for (int cc = 0; cc < 4; ++cc)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (32 * cc + e < lo || 32 * cc + e > hi) sr[cc][e] = __float_as_uint(-INFINITY);
        }
        float mx[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) mx[a] = -INFINITY;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
#pragma unroll
          for (int e = 0; e < 32; ++e) mx[e & 7] = fmaxf(mx[e & 7], __uint_as_float(sr[cc][e]));
        const float bm = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * c;
        if (bm == -INFINITY) continue;  // no visible key in this block for this row
        const float nm = fmaxf(m, bm);
        if (m != -INFINITY) l *= fast_exp2(m - nm);
        m = nm;
        float rs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int cc = 0; cc < 4; ++cc)
#pragma unroll
          for (int e = 0; e < 32; ++e)
            rs[e & 7] += fast_exp2(fmaf(__uint_as_float(sr[cc][e]), c, -m));
        l += ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
      }
      if (!ok) break;
      if (t < g.T) {
        const int64_t o = (static_cast<int64_t>(b) * g.T + t) * g.H + h;
        m_out[o] = m;
        l_out[o] = l;
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, 256);
  }
}

// ------------------------------------------------------------------- Pbar
template <int DH>
struct PbarLayout {
  static constexpr int kTile = kR * DH * 2;
  static constexpr int kStages = DH == 64 ? 4 : 2;
  static constexpr int kStage = 2 * kTile;  // Q_h | K_h
  static constexpr int kPartLd = kR + 4;    // partial-tile row stride (fp32): float4 rows conflict-free
  static constexpr int kPart = kStages * kStage;  // this CTA's sum over its heads [128][kPartLd]
  static constexpr int kBar = kPart + kR * kPartLd * 4;
  static constexpr int kSmem = kBar + 256 + 1024;
};

template <int DH>
__global__ void __launch_bounds__(320, 1) csa_pbar_tc_kernel(
    const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
    Geo g, float c, const float* __restrict__ m_in, const float* __restrict__ l_in,
    __nv_bfloat16* __restrict__ pbar, int32_t* dev_status) {
  using L = PbarLayout<DH>;
  constexpr int ST = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* full = bars;             // [ST]
  uint64_t* empty = bars + ST;       // [ST]
  uint64_t* s_full = bars + 2 * ST;  // [2]
  uint64_t* s_empty = s_full + 2;    // [2]
  uint64_t* mma_done = s_empty + 2;
  uint64_t* cl_ready = mma_done + 1;  // every CTA of the cluster wrote its partial
  uint64_t* cl_done = cl_ready + 1;   // every CTA of the cluster read the partials
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(cl_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* part = reinterpret_cast<float*>(smem + L::kPart);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = g.B * g.nqt * g.nb;
  const int H = g.H;
  // a cluster of G CTAs shares each unit, CTA `rank` taking heads
  // [rank H/G, (rank+1) H/G) (G divides H)
  const int G = static_cast<int>(sm100::cluster_nctarank());
  const int rank = static_cast<int>(sm100::cluster_ctarank());
  const int cid = blockIdx.x / G, ncl = gridDim.x / G;
  const int hs = H / G, h0 = rank * hs;

  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      sm100::mbar_init(&full[i], 1);
      sm100::mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&s_full[i], 1);
      sm100::mbar_init(&s_empty[i], 8);
    }
    sm100::mbar_init(mma_done, 1);
    sm100::mbar_init(cl_ready, 8 * G);
    sm100::mbar_init(cl_done, 8 * G);
    *abort_flag = 0;
    sm100::fence_mbar_init();
    sm100::tma_prefetch_desc(&map_q);
    sm100::tma_prefetch_desc(&map_k);
  }
  if (warp == 1) sm100::tmem_alloc(tmem_slot, 256);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::cluster_sync();  // peers' barriers are initialised before anyone arrives on them
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA
    uint32_t issued[ST];
#pragma unroll
    for (int i = 0; i < ST; ++i) issued[i] = 0;
    bool ok = true;
    int n = 0;  // stage loads issued
    for (int u = cid; u < units && ok; u += ncl) {
      const int i = u % g.nb, qt = (u / g.nb) % g.nqt, b = u / (g.nb * g.nqt);
      if (i >= g.nblk(qt)) continue;
      const int kb = g.kb0(qt) + i;
      for (int h = h0; h < h0 + hs; ++h, ++n) {
        const int s = n % ST;
        if (!sm100::mbar_wait_warp(&empty[s], ((n / ST) & 1) ^ 1u, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* st = smem + s * L::kStage;
          sm100::mbar_arrive_expect_tx(&full[s], L::kStage);
#pragma unroll
          for (int cc = 0; cc < DH / 64; ++cc) {
            sm100::tma_load_3d(&map_q, &full[s], st + cc * kBoxB, h * DH + cc * 64, qt * kR, b);
            sm100::tma_load_3d(&map_k, &full[s], st + L::kTile + cc * kBoxB, h * DH + cc * 64,
                               kb * kR, b);
          }
        }
        issued[s]++;
      }
    }
    for (int s = 0; s < ST; ++s)
      if (issued[s] > 0) sm100::mbar_wait_warp(&full[s], (issued[s] - 1u) & 1u, dev_status, nullptr);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    constexpr uint32_t idesc = sm100::make_idesc_bf16_f32(kR, kR);
    const uint32_t s0 = sm100::smem_u32(smem);
    bool ok = true;
    int n = 0;
    for (int u = cid; u < units && ok; u += ncl) {
      const int i = u % g.nb, qt = (u / g.nb) % g.nqt;
      if (i >= g.nblk(qt)) continue;
      for (int h = h0; h < h0 + hs; ++h, ++n) {
        const int s = n % ST, sb = n & 1;
        if (!sm100::mbar_wait_warp(&full[s], (n / ST) & 1, dev_status, abort_flag) ||
            !sm100::mbar_wait_warp(&s_empty[sb], ((n >> 1) & 1) ^ 1u, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        if (lane == 0) {
          const uint32_t qa = s0 + s * L::kStage, ka = qa + L::kTile;
#pragma unroll
          for (int kk = 0; kk < DH / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kBoxB + (kk & 3) * 32;
            sm100::umma_bf16_ss(tmem_base + sb * 128, sm100::make_sw128_kmajor_desc(qa + off),
                                sm100::make_sw128_kmajor_desc(ka + off), idesc, kk > 0 ? 1u : 0u);
          }
          sm100::umma_commit(&s_full[sb]);
          sm100::umma_commit(&empty[s]);
        }
        __syncwarp();
      }
    }
    if (lane == 0) sm100::umma_commit(mma_done);
    __syncwarp();
    sm100::mbar_wait_warp(mma_done, 0, dev_status, nullptr);
  } else if (warp >= 2) {
    // ------------------------------------------- head-averaged probabilities
    const int qw = warp & 3, half = (warp - 2) >> 2;
    const int row = qw * 32 + lane;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(qw * 32) << 16) + half * 64;
    const float invh = 1.0f / static_cast<float>(H);
    int n = 0;
    int uc = 0;  // units this cluster has finished (phase of cl_ready / cl_done)
    bool ok = true;
    for (int u = cid; u < units && ok; u += ncl) {
      const int i = u % g.nb, qt = (u / g.nb) % g.nqt, b = u / (g.nb * g.nqt);
      if (i >= g.nblk(qt)) continue;
      const int kb = g.kb0(qt) + i, t = qt * kR + row;
      const bool edge = !interior(qt, kb, g.W);
      const int lo = t - g.W + 1 - kb * kR - half * 64, hi = t - kb * kR - half * 64;
      const int64_t so = (static_cast<int64_t>(b) * g.T + min(t, g.T - 1)) * H;
      float acc[64];
#pragma unroll
      for (int e = 0; e < 64; ++e) acc[e] = 0.f;
      for (int h = h0; h < h0 + hs; ++h, ++n) {
        const int sb = n & 1;
        // this row's statistics for head h (a row past T contributes zero)
        const float mh = t < g.T ? __ldg(m_in + so + h) : 0.f;
        const float ih = t < g.T ? invh / __ldg(l_in + so + h) : 0.f;
        if (!sm100::mbar_wait_warp(&s_full[sb], (n >> 1) & 1, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        uint32_t sr[2][32];
        sm100::tmem_ld_32x32b_x32(t_lane + sb * 128, sr[0]);
        sm100::tmem_ld_32x32b_x32(t_lane + sb * 128 + 32, sr[1]);
        sm100::tmem_ld_wait();
        sm100::tmem_regs_ready(sr[0]);
        sm100::tmem_regs_ready(sr[1]);
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&s_empty[sb]);
        if (edge) {
#pragma unroll
          for (int e = 0; e < 64; ++e) {
            const float p = fast_exp2(fmaf(__uint_as_float(sr[e >> 5][e & 31]), c, -mh)) * ih;
            acc[e] += (e < lo || e > hi) ? 0.f : p;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 64; ++e)
            acc[e] += fast_exp2(fmaf(__uint_as_float(sr[e >> 5][e & 31]), c, -mh)) * ih;
        }
      }
      if (!ok) break;
      // this CTA's sum over its heads into its partial tile (once every peer
      // has read the previous unit's), then each CTA sums one slice of the
      // tile over the cluster, in rank order, and writes it as bf16
      if (uc > 0 && !sm100::mbar_wait_warp(cl_done, (uc - 1) & 1, dev_status, abort_flag)) break;
      float* prow = part + row * L::kPartLd + half * 64;
#pragma unroll
      for (int v = 0; v < 16; ++v)
        reinterpret_cast<float4*>(prow)[v] =
            make_float4(acc[4 * v], acc[4 * v + 1], acc[4 * v + 2], acc[4 * v + 3]);
      sm100::fence_acq_rel_cluster();
      __syncwarp();
      if (lane < G) sm100::mbar_arrive_cluster(sm100::mapa_shared(sm100::smem_u32(cl_ready), lane));
      if (!sm100::mbar_wait_warp(cl_ready, uc & 1, dev_status, abort_flag)) break;
      sm100::fence_acq_rel_cluster();
      __nv_bfloat16* tile = pbar + ((static_cast<int64_t>(b) * g.nqt + qt) * g.nb + i) * (kR * kR);
      constexpr int kChunks = kR * kR / 8;  // 8-column pieces of the tile
      const int per = (kChunks + G - 1) / G;
      const int c_end = min(kChunks, (rank + 1) * per);
      for (int ch = rank * per + (threadIdx.x - 64); ch < c_end; ch += 256) {
        const int r = ch >> 4, col = (ch & 15) * 8;
        const uint32_t la = sm100::smem_u32(part + r * L::kPartLd + col);
        float sum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int q = 0; q < G; ++q) {
          const uint32_t ra = sm100::mapa_shared(la, static_cast<uint32_t>(q));
          const float4 x0 = sm100::ld_dsmem_f4(ra), x1 = sm100::ld_dsmem_f4(ra + 16);
          sum[0] += x0.x; sum[1] += x0.y; sum[2] += x0.z; sum[3] += x0.w;
          sum[4] += x1.x; sum[5] += x1.y; sum[6] += x1.z; sum[7] += x1.w;
        }
        uint4 w;
        w.x = pack_bf16x2(sum[0], sum[1]);
        w.y = pack_bf16x2(sum[2], sum[3]);
        w.z = pack_bf16x2(sum[4], sum[5]);
        w.w = pack_bf16x2(sum[6], sum[7]);
        *reinterpret_cast<uint4*>(tile + r * kR + col) = w;
      }
      __syncwarp();
      if (lane < G) sm100::mbar_arrive_cluster(sm100::mapa_shared(sm100::smem_u32(cl_done), lane));
      ++uc;
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::cluster_sync();  // no CTA leaves while a peer may still read its partial tile
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, 256);
  }
}

// --------------------------------------------------------------------- PV
template <int NSW>
struct PvLayout {
  static constexpr int kV = kR * NSW * 2;       // V block slice [128 keys][NSW]
  static constexpr int kStage = kTileP + kV;    // Pbar tile | V slice
  static constexpr int kBar = 2 * kStage;
  static constexpr int kSmem = kBar + 256 + 1024;
};

template <int NSW>
__global__ void __launch_bounds__(192, 1) csa_pv_tc_kernel(
    const __grid_constant__ CUtensorMap map_p, const __grid_constant__ CUtensorMap map_v,
    Geo g, int D, __nv_bfloat16* __restrict__ out, int64_t so, int32_t* dev_status) {
  using L = PvLayout<NSW>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* full = bars;        // [2]
  uint64_t* empty = bars + 2;   // [2]
  uint64_t* o_full = bars + 4;  // [2]
  uint64_t* o_empty = bars + 6; // [2]
  uint64_t* mma_done = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nns = D / NSW;
  const int units = g.B * g.nqt * nns;
  constexpr uint32_t kCols = 2 * NSW;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&full[i], 1);
      sm100::mbar_init(&empty[i], 1);
      sm100::mbar_init(&o_full[i], 1);
      sm100::mbar_init(&o_empty[i], 4);
    }
    sm100::mbar_init(mma_done, 1);
    *abort_flag = 0;
    sm100::fence_mbar_init();
    sm100::tma_prefetch_desc(&map_p);
    sm100::tma_prefetch_desc(&map_v);
  }
  if (warp == 1) sm100::tmem_alloc(tmem_slot, kCols);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA
    uint32_t issued[2] = {0, 0};
    bool ok = true;
    int n = 0;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const int ns = u % nns, qt = (u / nns) % g.nqt, b = u / (nns * g.nqt);
      const int kb0 = g.kb0(qt), nblk = g.nblk(qt);
      for (int i = 0; i < nblk; ++i, ++n) {
        const int s = n & 1;
        if (!sm100::mbar_wait_warp(&empty[s], ((n >> 1) & 1) ^ 1u, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* st = smem + s * L::kStage;
          sm100::mbar_arrive_expect_tx(&full[s], L::kStage);
          const int prow = ((b * g.nqt + qt) * g.nb + i) * kR;
          sm100::tma_load_2d(&map_p, &full[s], st, 0, prow);
          sm100::tma_load_2d(&map_p, &full[s], st + kBoxB, 64, prow);
#pragma unroll
          for (int cc = 0; cc < NSW / 64; ++cc)
            sm100::tma_load_3d(&map_v, &full[s], st + kTileP + cc * kBoxB, ns * NSW + cc * 64,
                               (kb0 + i) * kR, b);
        }
        issued[s]++;
      }
    }
    for (int s = 0; s < 2; ++s)
      if (issued[s] > 0) sm100::mbar_wait_warp(&full[s], (issued[s] - 1u) & 1u, dev_status, nullptr);
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA
    constexpr uint32_t idesc = sm100::make_idesc_bf16_f32(kR, NSW) | sm100::kIdescBMajorMN;
    const uint32_t s0 = sm100::smem_u32(smem);
    bool ok = true;
    int n = 0, ul = 0;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++ul) {
      const int qt = (u / nns) % g.nqt;
      const int ob = ul & 1, nblk = g.nblk(qt);
      if (!sm100::mbar_wait_warp(&o_empty[ob], ((ul >> 1) & 1) ^ 1u, dev_status, abort_flag)) break;
      sm100::tc_fence_after();
      for (int i = 0; i < nblk; ++i, ++n) {
        const int s = n & 1;
        if (!sm100::mbar_wait_warp(&full[s], (n >> 1) & 1, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        if (lane == 0) {
          const uint32_t pa = s0 + s * L::kStage, va = pa + kTileP;
#pragma unroll
          for (int kk = 0; kk < kR / 16; ++kk) {
            const uint64_t ad = sm100::make_sw128_kmajor_desc(pa + (kk >> 2) * kBoxB + (kk & 3) * 32);
            const uint64_t bd = sm100::make_sw128_desc(va + kk * 2048, kBoxB, 1024);
            sm100::umma_bf16_ss(tmem_base + ob * NSW, ad, bd, idesc, (i | kk) != 0 ? 1u : 0u);
          }
          sm100::umma_commit(&empty[s]);
          if (i == nblk - 1) sm100::umma_commit(&o_full[ob]);
        }
        __syncwarp();
      }
    }
    if (lane == 0) sm100::umma_commit(mma_done);
    __syncwarp();
    sm100::mbar_wait_warp(mma_done, 0, dev_status, nullptr);
  } else if (warp >= 2) {
    // ------------------------------------------------------- epilogue
    const int qw = warp & 3, row = qw * 32 + lane;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(qw * 32) << 16);
    int ul = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++ul) {
      const int ns = u % nns, qt = (u / nns) % g.nqt, b = u / (nns * g.nqt);
      const int ob = ul & 1, t = qt * kR + row;
      if (!sm100::mbar_wait_warp(&o_full[ob], (ul >> 1) & 1, dev_status, abort_flag)) break;
      sm100::tc_fence_after();
      __nv_bfloat16* dst = out + (static_cast<int64_t>(b) * g.T + t) * so + ns * NSW;
#pragma unroll 1
      for (int cc = 0; cc < NSW / 32; ++cc) {
        uint32_t o[32];
        sm100::tmem_ld_32x32b_x32(t_lane + ob * NSW + 32 * cc, o);
        sm100::tmem_ld_wait();
        sm100::tmem_regs_ready(o);
        if (t < g.T) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(o[8 * v + 0]), __uint_as_float(o[8 * v + 1]));
            w.y = pack_bf16x2(__uint_as_float(o[8 * v + 2]), __uint_as_float(o[8 * v + 3]));
            w.z = pack_bf16x2(__uint_as_float(o[8 * v + 4]), __uint_as_float(o[8 * v + 5]));
            w.w = pack_bf16x2(__uint_as_float(o[8 * v + 6]), __uint_as_float(o[8 * v + 7]));
            reinterpret_cast<uint4*>(dst + 32 * cc)[v] = w;
          }
        }
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&o_empty[ob]);
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, kCols);
  }
}

template <int DH>
int32_t launch_csa_tc(const void* q, int64_t sq, const void* k, int64_t sk, const void* v,
                      int64_t sv, const Geo& g, int D, float c, void* out, int64_t so,
                      float* m, float* l, __nv_bfloat16* pbar, int32_t* dev_status,
                      cudaStream_t s) {
  int32_t st = ensure_smem(csa_stats_tc_kernel<DH>, StatsLayout<DH>::kSmem);
  if (!st) st = ensure_smem(csa_pbar_tc_kernel<DH>, PbarLayout<DH>::kSmem);
  if (!st) st = ensure_smem(csa_pv_tc_kernel<256>, PvLayout<256>::kSmem);
  if (!st) st = ensure_smem(csa_pv_tc_kernel<128>, PvLayout<128>::kSmem);
  if (st) return st;
  const uint64_t HD = static_cast<uint64_t>(g.H) * DH;
  CUtensorMap mq, mk, mv, mp;
  const uint64_t prow = static_cast<uint64_t>(g.B) * g.nqt * g.nb * kR;
  if (!make_bf16_3d_map(&mq, q, g.B, g.T, HD, sq, kR) ||
      !make_bf16_3d_map(&mk, k, g.B, g.T, HD, sk, kR) ||
      !make_bf16_3d_map(&mv, v, g.B, g.T, D, sv, kR) ||
      !make_bf16_2d_map(&mp, pbar, prow, kR, kR, kR, 64))
    return LLMYB_EUNSUPPORTED;
  const int sms = num_sms();
  auto grid = [&](int64_t units) { return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(units, sms))); };
  csa_stats_tc_kernel<DH><<<grid(static_cast<int64_t>(g.B) * g.H * g.nqt), 192,
                            StatsLayout<DH>::kSmem, s>>>(mq, mk, g, c, m, l, dev_status);
  count_launch();
  {
    // few units (short prompts): a cluster of G CTAs per unit splits its heads
    const int64_t units = static_cast<int64_t>(g.B) * g.nqt * g.nb;
    int G = 1;
    for (int d = 8; d >= 2; --d)
      if (g.H % d == 0 && units * d <= sms) {
        G = d;
        break;
      }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(
        G * std::max<int64_t>(1, std::min<int64_t>(units, sms / G))));
    cfg.blockDim = dim3(320);
    cfg.dynamicSmemBytes = PbarLayout<DH>::kSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(G);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e =
        cudaLaunchKernelEx(&cfg, csa_pbar_tc_kernel<DH>, mq, mk, g, c, static_cast<const float*>(m),
                           static_cast<const float*>(l), pbar, dev_status);
    if (e != cudaSuccess) return static_cast<int32_t>(e);
    count_launch();
  }
  auto* o = static_cast<__nv_bfloat16*>(out);
  if (D % 256 == 0)
    csa_pv_tc_kernel<256><<<grid(static_cast<int64_t>(g.B) * g.nqt * (D / 256)), 192,
                            PvLayout<256>::kSmem, s>>>(mp, mv, g, D, o, so, dev_status);
  else
    csa_pv_tc_kernel<128><<<grid(static_cast<int64_t>(g.B) * g.nqt * (D / 128)), 192,
                            PvLayout<128>::kSmem, s>>>(mp, mv, g, D, o, so, dev_status);
  count_launch();
  return launch_status();
}

}  // namespace

// Tile geometry of the tcgen05 CSA prefill: query tiles, key blocks per tile.
void csa_tc_geometry(int T, int W, int* nqt, int* nb) {
  *nqt = (T + kR - 1) / kR;
  *nb = std::min(*nqt, (W - 1 + kR - 1) / kR + 1);
}

bool csa_tc_supported(int head_dim, int d_model, int64_t q_stride, int64_t k_stride,
                      int64_t v_stride, int64_t out_stride) {
  return (head_dim == 64 || head_dim == 128) && d_model % 128 == 0 && q_stride % 8 == 0 &&
         k_stride % 8 == 0 && v_stride % 8 == 0 && out_stride % 8 == 0;
}

// scratch: m, l [B, T, H] fp32, then (256-byte aligned) Pbar tiles.
int32_t csa_prefill_tc(const void* q, int64_t sq, const void* k, int64_t sk, const void* v,
                       int64_t sv, int B, int T, int H, int DH, int D, int W, float scale,
                       void* out, int64_t so, void* scratch, int32_t* dev_status,
                       cudaStream_t s) {
  Geo g{B, T, H, W, 0, 0};
  csa_tc_geometry(T, W, &g.nqt, &g.nb);
  float* m = static_cast<float*>(scratch);
  float* l = m + static_cast<int64_t>(B) * T * H;
  const int64_t stat_bytes = (2 * static_cast<int64_t>(B) * T * H * 4 + 255) / 256 * 256;
  auto* pbar = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(scratch) + stat_bytes);
  const float c = scale * 1.4426950408889634f;
  if (DH == 64) return launch_csa_tc<64>(q, sq, k, sk, v, sv, g, D, c, out, so, m, l, pbar, dev_status, s);
  return launch_csa_tc<128>(q, sq, k, sk, v, sv, g, D, c, out, so, m, l, pbar, dev_status, s);
}

}  // namespace llmyb
