// Per-head banded (sliding-window) causal attention on 5th-generation tensor
// cores: tcgen05.mma with TMEM accumulators, Q/K/V staged by TMA.
//
// Reference: fused_banded_local_attention / _banded_attn_fwd_kernel
// (sample_standalone.py:70-85, :253-322): key j is visible from query t iff
// j <= t and t - j < window; out = softmax(scale q.k over the visible keys) V,
// V per head or one V broadcast to every head.
//
// Persistent kernel, one CTA per SM; a work unit is (batch row, head,
// 128-query tile) and visits, in order, the 128-key blocks that intersect the
// band (key blocks outside it are never loaded).
//   warp 0     TMA: the unit's Q tile (two buffers, so the next unit's Q
//              arrives during the current one), K and V blocks in two-stage
//              rings with separate barriers (S = Q K^T starts before V lands).
//   warp 1     MMA issue (one thread): S_g = Q K_g^T into one of two TMEM
//              score buffers, then O += P_{g-1} V_{g-1}: the products are
//              issued one block apart, so the softmax of block g overlaps the
//              PV product of block g-1 and the score product of block g+1.
//   warps 2-9  softmax, two warps per TMEM lane quarter (query rows = TMEM
//              lanes): each owns 64 of the block's 128 key columns and half of
//              O's columns.  Scores from TMEM, the band mask on the edge
//              blocks, base-2 online softmax with a lazily raised running max
//              shared by the pair (each exchanges its partial block max,
//              rounded up to bf16, through shared memory and a 64-thread named
//              barrier; O is rescaled in TMEM only when a block max exceeds the
//              running max by more than 2^8, so P <= 256 and rescales are
//              rare), P as bf16 into shared memory in the 128-byte-swizzled
//              K-major layout of an MMA A operand; at the end of the unit the
//              pair adds its two row sums and writes O / l to global memory.
// The PV product reads V in its natural [key][dh] layout as an MN-major B
// operand.  TMEM: O in columns [0, D), score buffers at [128, 256), [256, 384).
// Every wait is bounded (1 s): a timeout records LLMYB_ETIMEOUT in the status
// word and all roles unwind; no TMA or MMA is left in flight at exit.
#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.h"

namespace llmyb {
namespace {

constexpr int kRows = 128;         // queries per tile = keys per block
constexpr int kBox = 128 * 64 * 2;  // one TMA box: 128 rows x 64 bf16 (16 KB)
constexpr int kPBytes = kRows * kRows * 2;
constexpr uint32_t kTmemCols = 512;

template <int D>
struct BandTcLayout {
  static constexpr int kTile = kRows * D * 2;  // one Q, K or V tile
  static constexpr int kQ = 0;                 // 2 Q buffers
  static constexpr int kK = 2 * kTile;         // 2 K stages
  static constexpr int kV = 4 * kTile;         // 2 V stages
  static constexpr int kP = 6 * kTile;         // P (one buffer)
  static constexpr int kBar = kP + kPBytes;
  static constexpr int kX = kBar + 256;        // softmax pair exchange: 1 KB
  static constexpr int kSmem = kX + 1024 + 1024;  // + alignment slack
};

struct BandUnit {
  int b, h, qt, kb0, nblk;
};

__device__ __forceinline__ BandUnit band_unit(int u, int nqt, int H, int W) {
  BandUnit x;
  x.qt = u % nqt;
  const int bh = u / nqt;
  x.h = bh % H;
  x.b = bh / H;
  x.kb0 = max(0, x.qt * kRows - W + 1) / kRows;
  x.nblk = x.qt - x.kb0 + 1;
  return x;
}

template <int D>
__global__ void __launch_bounds__(320, 1) band_tc_kernel(
    const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
    const __grid_constant__ CUtensorMap map_v, int v_heads, int B, int T, int H, int W,
    float scale_log2, __nv_bfloat16* __restrict__ out, int64_t so, int32_t* dev_status) {
  using L = BandTcLayout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars;        // [2]
  uint64_t* q_empty = bars + 2;   // [2]
  uint64_t* k_full = bars + 4;    // [2]
  uint64_t* k_empty = bars + 6;   // [2]
  uint64_t* v_full = bars + 8;    // [2]
  uint64_t* v_empty = bars + 10;  // [2]
  uint64_t* s_full = bars + 12;   // [2]
  uint64_t* s_empty = bars + 14;  // [2]
  uint64_t* p_full = bars + 16;
  uint64_t* pv_done = bars + 17;
  uint64_t* o_empty = bars + 18;
  uint64_t* mma_done = bars + 19;
  uint64_t* pair_bar = bars + 20;  // [4]: the two softmax warps of a TMEM lane quarter
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqt = (T + kRows - 1) / kRows;
  const int units = B * H * nqt;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&q_full[i], 1);
      sm100::mbar_init(&q_empty[i], 1);
      sm100::mbar_init(&k_full[i], 1);
      sm100::mbar_init(&k_empty[i], 1);
      sm100::mbar_init(&v_full[i], 1);
      sm100::mbar_init(&v_empty[i], 1);
      sm100::mbar_init(&s_full[i], 1);
      sm100::mbar_init(&s_empty[i], 8);  // one arrival per softmax warp
    }
    sm100::mbar_init(p_full, 8);
    sm100::mbar_init(pv_done, 1);
    sm100::mbar_init(o_empty, 8);
    sm100::mbar_init(mma_done, 1);
    for (int i = 0; i < 4; ++i) sm100::mbar_init(&pair_bar[i], 2);
    *abort_flag = 0;
    sm100::fence_mbar_init();
    sm100::tma_prefetch_desc(&map_q);
    sm100::tma_prefetch_desc(&map_k);
    sm100::tma_prefetch_desc(&map_v);
  }
  if (warp == 1) sm100::tmem_alloc(tmem_slot, kTmemCols);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------- TMA
    // loads issued so far (load n uses buffer n & 1, phase (n >> 1) & 1)
    uint32_t nq = 0, nk = 0, nv = 0;
    bool ok = true;
    int g = 0, ul = 0;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++ul) {
      const BandUnit x = band_unit(u, nqt, H, W);
      const int qb = ul & 1;
      if (!sm100::mbar_wait_warp(&q_empty[qb], ((ul >> 1) & 1) ^ 1u, dev_status, abort_flag)) {
        ok = false;
        break;
      }
      if (lane == 0) {
        sm100::mbar_arrive_expect_tx(&q_full[qb], L::kTile);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          sm100::tma_load_3d(&map_q, &q_full[qb], smem + L::kQ + qb * L::kTile + c * kBox,
                             x.h * D + c * 64, x.qt * kRows, x.b);
      }
      ++nq;
      const int vcol = (v_heads == 1 ? 0 : x.h) * D;
      for (int i = 0; i < x.nblk; ++i, ++g) {
        const int s = g & 1;
        const uint32_t ph = (g >> 1) & 1;
        const int row = (x.kb0 + i) * kRows;
        if (!sm100::mbar_wait_warp(&k_empty[s], ph ^ 1u, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          sm100::mbar_arrive_expect_tx(&k_full[s], L::kTile);
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            sm100::tma_load_3d(&map_k, &k_full[s], smem + L::kK + s * L::kTile + c * kBox,
                               x.h * D + c * 64, row, x.b);
        }
        ++nk;
        if (!sm100::mbar_wait_warp(&v_empty[s], ph ^ 1u, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          sm100::mbar_arrive_expect_tx(&v_full[s], L::kTile);
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            sm100::tma_load_3d(&map_v, &v_full[s], smem + L::kV + s * L::kTile + c * kBox,
                               vcol + c * 64, row, x.b);
        }
        ++nv;
      }
    }
    // no TMA write into shared memory may still be in flight at exit
    // (a stage is only reloaded after its previous load was consumed, so at
    // most the last load of each buffer can still be pending)
    for (uint32_t i = 1; i <= 2; ++i) {
      if (nq >= i) sm100::mbar_wait_warp(&q_full[(nq - i) & 1], ((nq - i) >> 1) & 1, dev_status, nullptr);
      if (nk >= i) sm100::mbar_wait_warp(&k_full[(nk - i) & 1], ((nk - i) >> 1) & 1, dev_status, nullptr);
      if (nv >= i) sm100::mbar_wait_warp(&v_full[(nv - i) & 1], ((nv - i) >> 1) & 1, dev_status, nullptr);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = sm100::make_idesc_bf16_f32(kRows, kRows);
    constexpr uint32_t idesc_o = sm100::make_idesc_bf16_f32(kRows, D) | sm100::kIdescBMajorMN;
    const uint32_t t_o = tmem_base, t_s = tmem_base + 128;
    const uint32_t sq_addr = sm100::smem_u32(smem + L::kQ);
    const uint32_t sk_addr = sm100::smem_u32(smem + L::kK);
    const uint32_t sv_addr = sm100::smem_u32(smem + L::kV);
    const uint32_t sp_addr = sm100::smem_u32(smem + L::kP);

    // O += P V for block gg (first: the unit's first block, which overwrites O)
    auto issue_pv = [&](int gg, bool first, int uu) -> bool {
      const int s = gg & 1;
      if (!sm100::mbar_wait_warp(&v_full[s], (gg >> 1) & 1, dev_status, abort_flag)) return false;
      if (!sm100::mbar_wait_warp(p_full, gg & 1, dev_status, abort_flag)) return false;
      if (first && !sm100::mbar_wait_warp(o_empty, (uu & 1) ^ 1u, dev_status, abort_flag))
        return false;
      sm100::tc_fence_after();
      if (lane == 0) {
        const uint32_t va = sv_addr + s * L::kTile;
#pragma unroll
        for (int kk = 0; kk < kRows / 16; ++kk) {
          const uint64_t ad =
              sm100::make_sw128_kmajor_desc(sp_addr + (kk >> 2) * kBox + (kk & 3) * 32);
          const uint64_t bd = sm100::make_sw128_desc(va + kk * 2048, kBox, 1024);
          sm100::umma_bf16_ss(t_o, ad, bd, idesc_o, (first && kk == 0) ? 0u : 1u);
        }
        sm100::umma_commit(pv_done);
        sm100::umma_commit(&v_empty[s]);
      }
      __syncwarp();
      return true;
    };

    bool ok = true;
    int g = 0, ul = 0;
    int pend_g = -1, pend_u = 0;
    bool pend_first = false;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++ul) {
      const BandUnit x = band_unit(u, nqt, H, W);
      const int qb = ul & 1;
      for (int i = 0; i < x.nblk; ++i, ++g) {
        const int s = g & 1;
        const uint32_t ph = (g >> 1) & 1;
        if (i == 0 &&
            !sm100::mbar_wait_warp(&q_full[qb], (ul >> 1) & 1, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        if (!sm100::mbar_wait_warp(&k_full[s], ph, dev_status, abort_flag) ||
            !sm100::mbar_wait_warp(&s_empty[s], ph ^ 1u, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        if (lane == 0) {
          const uint32_t qa = sq_addr + qb * L::kTile, ka = sk_addr + s * L::kTile;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * kBox + (kk & 3) * 32;
            sm100::umma_bf16_ss(t_s + s * 128, sm100::make_sw128_kmajor_desc(qa + off),
                                sm100::make_sw128_kmajor_desc(ka + off), idesc_s,
                                kk > 0 ? 1u : 0u);
          }
          sm100::umma_commit(&s_full[s]);
          sm100::umma_commit(&k_empty[s]);
          if (i == x.nblk - 1) sm100::umma_commit(&q_empty[qb]);
        }
        __syncwarp();
        if (pend_g >= 0 && !issue_pv(pend_g, pend_first, pend_u)) {
          ok = false;
          break;
        }
        pend_g = g;
        pend_first = i == 0;
        pend_u = ul;
      }
    }
    if (ok && pend_g >= 0) issue_pv(pend_g, pend_first, pend_u);
    // every MMA issued by lane 0 completes before TMEM / shared memory go away
    if (lane == 0) sm100::umma_commit(mma_done);
    __syncwarp();
    sm100::mbar_wait_warp(mma_done, 0, dev_status, nullptr);
  } else {
    // --------------------------------------------------------- softmax
    const int qw = warp & 3;            // TMEM lane quarter of this warp
    const int half = (warp - 2) >> 2;   // key columns [64 half, +64), O columns [D/2 half, +D/2)
    const int row = qw * 32 + lane;
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(qw * 32) << 16);
    // the pair (warps qw + 2 and qw + 6) meets on pair_bar[qw]: both warps
    // arrive once per meeting and wait (bounded) for the meeting's phase
    uint32_t meets = 0;
    auto pair_meet = [&]() -> bool {
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(&pair_bar[qw]);
      const bool r = sm100::mbar_wait_warp(&pair_bar[qw], meets & 1u, dev_status, abort_flag);
      __syncwarp();  // every lane's later reads follow lane 0's acquire
      ++meets;
      return r;
    };
    // exchange: [parity][half][row] bf16 block maxima; at a unit's end the
    // pair's two fp32 row sums.  The four pairs meet only within themselves,
    // so the sums must land in bytes that hold this pair's own rows of the
    // maxima (slot s = parity * 2 + half covers bytes [256 s + 64 qw, +64) for
    // pair qw): sum k = half * 32 + lane goes to float 64 (k / 16) + 16 qw +
    // k % 16.  A layout that spilled into another pair's rows would overwrite
    // maxima that pair is still exchanging.
    uint16_t* xmax = reinterpret_cast<uint16_t*>(smem + L::kX);
    float* xsum = reinterpret_cast<float*>(smem + L::kX);
    auto xsum_at = [&](int h) -> int {
      const int k = h * 32 + lane;
      return 64 * (k >> 4) + 16 * qw + (k & 15);
    };
    uint8_t* prow = smem + L::kP + row * 128;
    const int pswz = row & 7;
    int g = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const BandUnit x = band_unit(u, nqt, H, W);
      const int q0 = x.qt * kRows, t = q0 + row;
      float m = -INFINITY, l = 0.f;
      for (int i = 0; i < x.nblk; ++i, ++g) {
        const int sb = g & 1;
        if (!sm100::mbar_wait_warp(&s_full[sb], (g >> 1) & 1, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        uint32_t sr[2][32];
#pragma unroll
        for (int c = 0; c < 2; ++c)
          sm100::tmem_ld_32x32b_x32(t_lane + 128 + sb * 128 + half * 64 + 32 * c, sr[c]);
        sm100::tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 2; ++c) sm100::tmem_regs_ready(sr[c]);
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&s_empty[sb]);

        const int j0 = (x.kb0 + i) * kRows + half * 64;
        if ((x.kb0 + i) * kRows + kRows - 1 > q0 || q0 + kRows - 1 - (x.kb0 + i) * kRows >= W) {
          // band edge: key column c of this half is visible iff lo <= c <= hi
          const int lo = t - W + 1 - j0, hi = t - j0;
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (32 * c + e < lo || 32 * c + e > hi) sr[c][e] = __float_as_uint(-INFINITY);
        }
        // partial row max of the raw scores (the scale is positive)
        float mx[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) mx[a] = -INFINITY;
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) mx[e & 7] = fmaxf(mx[e & 7], __uint_as_float(sr[c][e]));
        const float pm = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) *
                         scale_log2;
        // both warps of the pair form the block max from the same two bf16
        // values (rounded up, so m stays an upper bound of the row's scores)
        const __nv_bfloat16 pmb = __float2bfloat16_ru(pm);
        xmax[((g & 1) * 2 + half) * 128 + row] = *reinterpret_cast<const uint16_t*>(&pmb);
        if (!pair_meet()) {
          ok = false;
          break;
        }
        const uint16_t o0 = xmax[((g & 1) * 2) * 128 + row], o1 = xmax[((g & 1) * 2 + 1) * 128 + row];
        const float bm = fmaxf(__uint_as_float(static_cast<uint32_t>(o0) << 16),
                               __uint_as_float(static_cast<uint32_t>(o1) << 16));
        const bool need = bm > m + 8.f;
        float alpha = 1.f;
        if (need) {
          alpha = fast_exp2(m - bm);
          l *= alpha;
          m = bm;
        }
        const float nbase = m == -INFINITY ? 0.f : -m;
        float rs[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float p = fast_exp2(fmaf(__uint_as_float(sr[c][e]), scale_log2, nbase));
            rs[e & 7] += p;
            sr[c][e] = __float_as_uint(p);
          }
        l += ((rs[0] + rs[1]) + (rs[2] + rs[3])) + ((rs[4] + rs[5]) + (rs[6] + rs[7]));
        // the single P buffer is free once the PV product of block g-1 is done
        if (!sm100::mbar_wait_warp(pv_done, (g & 1) ^ 1u, dev_status, abort_flag)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int kc = 0; kc < 8; ++kc) {
          const int c = kc >> 2, e = (kc & 3) * 8;
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(sr[c][e + 0]), __uint_as_float(sr[c][e + 1]));
          w.y = pack_bf16x2(__uint_as_float(sr[c][e + 2]), __uint_as_float(sr[c][e + 3]));
          w.z = pack_bf16x2(__uint_as_float(sr[c][e + 4]), __uint_as_float(sr[c][e + 5]));
          w.w = pack_bf16x2(__uint_as_float(sr[c][e + 6]), __uint_as_float(sr[c][e + 7]));
          *reinterpret_cast<uint4*>(prow + half * kBox + ((kc ^ pswz) << 4)) = w;
        }
        sm100::fence_proxy_async_smem();
        if (__any_sync(0xffffffffu, need && i > 0)) {
          // O holds the products of blocks < i (block g-1 is complete); this
          // warp rescales its half of O's columns
          sm100::tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c) {
            uint32_t o[32];
            const uint32_t col = static_cast<uint32_t>(half * (D / 2) + 32 * c);
            sm100::tmem_ld_32x32b_x32(t_lane + col, o);
            sm100::tmem_ld_wait();
            sm100::tmem_regs_ready(o);
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            sm100::tmem_st_32x32b_x32(t_lane + col, o);
          }
          sm100::tmem_st_wait();
        }
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(p_full);
      }
      if (!ok) break;
      // ---------------------------------------------------- epilogue
      // the pair's two partial row sums, in the exchange area once both warps
      // have read this unit's last block maxima
      if (!pair_meet()) break;
      xsum[xsum_at(half)] = l;
      if (!pair_meet()) break;
      const float inv = 1.f / (xsum[xsum_at(0)] + xsum[xsum_at(1)]);
      if (!pair_meet()) break;  // read before the next unit's first exchange overwrites
      if (!sm100::mbar_wait_warp(pv_done, (g - 1) & 1, dev_status, abort_flag)) break;
      sm100::tc_fence_after();
      __nv_bfloat16* dst = out + (static_cast<int64_t>(x.b) * T + t) * so + x.h * D;
#pragma unroll 1
      for (int c = 0; c < D / 64; ++c) {
        uint32_t o[32];
        const int col = half * (D / 2) + 32 * c;
        sm100::tmem_ld_32x32b_x32(t_lane + col, o);
        sm100::tmem_ld_wait();
        sm100::tmem_regs_ready(o);
        if (t < T) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
            reinterpret_cast<uint4*>(dst + col)[v] = w;
          }
        }
      }
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(o_empty);
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <int D>
int32_t launch_band_tc(const void* q, int64_t sq, const void* k, int64_t sk, const void* v,
                       int64_t sv, int v_heads, int B, int T, int H, int W, float scale,
                       void* out, int64_t so, int32_t* dev_status, cudaStream_t stream) {
  using L = BandTcLayout<D>;
  {
    int32_t st = ensure_smem(band_tc_kernel<D>, L::kSmem);
    if (st) return st;
  }
  CUtensorMap mq, mk, mv;
  if (!make_bf16_3d_map(&mq, q, B, T, static_cast<uint64_t>(H) * D, sq, kRows) ||
      !make_bf16_3d_map(&mk, k, B, T, static_cast<uint64_t>(H) * D, sk, kRows) ||
      !make_bf16_3d_map(&mv, v, B, T, static_cast<uint64_t>(v_heads) * D, sv, kRows))
    return LLMYB_EUNSUPPORTED;
  const int64_t units = static_cast<int64_t>(B) * H * ((T + kRows - 1) / kRows);
  const int grid = static_cast<int>(std::min<int64_t>(units, num_sms()));
  constexpr float kLog2e = 1.4426950408889634f;
  band_tc_kernel<D><<<grid, 320, L::kSmem, stream>>>(mq, mk, mv, v_heads, B, T, H, W,
                                                     scale * kLog2e,
                                                     static_cast<__nv_bfloat16*>(out), so,
                                                     dev_status);
  count_launch();
  return launch_status();
}

bool aligned16(const void* p, int64_t stride) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0 && stride % 8 == 0;
}

}  // namespace
}  // namespace llmyb

using namespace llmyb;

// Per-head banded attention: q,k [B*T, H*D] (token stride sq/sk), v with
// v_heads in {1, H} heads of width D, out [B*T, H*D] (stride so).
LLMYB_API int32_t llmyb_banded_attention(const void* q, int64_t q_stride, const void* k,
                                         int64_t k_stride, const void* v, int64_t v_stride,
                                         int32_t v_heads, int32_t batch, int32_t seq,
                                         int32_t heads, int32_t head_dim, int32_t window,
                                         float scale, void* out, int64_t out_stride,
                                         int32_t* dev_status, void* stream) {
  if (!q || !k || !v || !out || batch < 0 || seq < 0 || heads <= 0 || window <= 0 ||
      !(scale > 0.f))
    return LLMYB_EINVAL;
  if (v_heads != 1 && v_heads != heads) return LLMYB_EINVAL;
  if (batch == 0 || seq == 0) return LLMYB_OK;
  if (!aligned16(q, q_stride) || !aligned16(k, k_stride) || !aligned16(v, v_stride) ||
      !aligned16(out, out_stride))
    return LLMYB_EUNSUPPORTED;
  if (q_stride < static_cast<int64_t>(heads) * head_dim ||
      k_stride < static_cast<int64_t>(heads) * head_dim ||
      v_stride < static_cast<int64_t>(v_heads) * head_dim ||
      out_stride < static_cast<int64_t>(heads) * head_dim)
    return LLMYB_EINVAL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (head_dim) {
    case 64:
      return launch_band_tc<64>(q, q_stride, k, k_stride, v, v_stride, v_heads, batch, seq, heads,
                                window, scale, out, out_stride, dev_status, s);
    case 128:
      return launch_band_tc<128>(q, q_stride, k, k_stride, v, v_stride, v_heads, batch, seq,
                                 heads, window, scale, out, out_stride, dev_status, s);
    default:
      return LLMYB_EUNSUPPORTED;
  }
}
