// Grouped SwiGLU expert FFN on 5th-generation tensor cores (tcgen05 + TMEM,
// operands staged by TMA).
//
// Reference: model/layers/moe.py:29-82 (_moe_dispatch_fused) and
// runpod/kernels/triton_swiglu_moe.py:160-218.  The reference scatters routed
// rows into a capacity-padded [E, cap, D] buffer after a host sync on
// counts.max(), runs two cuBLAS bmm calls with a separate SwiGLU pass, then
// gathers and index_adds.  Here the routed rows are kept expert-contiguous
// (no padding, no host sync) and a persistent kernel walks the
// (expert, 128-row tile, N tile) schedule produced by the router plan:
//
//   gather : x_perm[pos]  = x[perm_token[pos]]                    (HBM copy)
//   GEMM1  : h_perm[pos]  = silu(x_perm W_gate^T) * (x_perm W_up^T)  (epilogue)
//   GEMM2  : y_perm[pos]  = perm_prob[pos] * (h_perm W_down^T)       (epilogue)
//   combine: out[t]       = sum_s y_perm[route_pos[t, s]]          (fp32 sum)
//
// GEMM kernel structure (one CTA per SM, 256 threads):
//   warp 0     TMA producer: A tile 128x64 and B tile 256x64 per stage,
//              4-stage ring of 48 KB stages, 128-byte swizzle.
//   warp 1     MMA issuer: 4 x tcgen05.mma (128x256x16, bf16 -> fp32) per
//              stage into a TMEM accumulator; two accumulators of 256 columns
//              so the epilogue of tile i overlaps the main loop of tile i+1.
//   warp 2     TMEM allocation owner.
//   warps 4-7  epilogue: tcgen05.ld 32 lanes x 32 columns (one chunk ahead of
//              the math), fused SwiGLU or probability scale, bf16 stores.
// For GEMM1 the weight rows are pre-interleaved (llmyb_moe_pack_w13) so that
// every 256-wide N tile holds 128 gate rows followed by the matching 128 up
// rows, which keeps silu(gate) * up inside one accumulator.
#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.h"

#include <algorithm>

namespace llmyb {
namespace {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_STAGE_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_STAGE_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int TMEM_COLS = 512;              // 2 accumulators x 256 fp32 columns
constexpr int EPI_SCRATCH = 4 * 32 * 64;  // per epilogue warp: 32 rows x 64 bytes, transposing
constexpr int GEMM_SMEM = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/ + EPI_SCRATCH;

enum Epilogue { kSwiGLU = 0, kScale = 1 };

struct TileInfo {
  int expert, row0, rows_valid, n_tile;
};

// tile index -> (expert, first row, valid rows, n tile).  Experts without
// rows own no tiles; tile_offsets is non-decreasing with E+1 entries.
__device__ __forceinline__ TileInfo map_tile(int tile, int n_tiles, const int* tile_offsets,
                                             const int* expert_offsets, int E) {
  TileInfo ti;
  const int m_global = tile / n_tiles;
  ti.n_tile = tile - m_global * n_tiles;
  int lo = 0, hi = E - 1;  // last e with tile_offsets[e] <= m_global
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(tile_offsets + mid) <= m_global) lo = mid; else hi = mid - 1;
  }
  ti.expert = lo;
  const int m_local = m_global - __ldg(tile_offsets + lo);
  const int e_begin = __ldg(expert_offsets + lo), e_end = __ldg(expert_offsets + lo + 1);
  ti.row0 = e_begin + m_local * BM;
  ti.rows_valid = min(BM, e_end - ti.row0);
  return ti;
}

__device__ __forceinline__ float swiglu_fast(uint32_t g_bits, uint32_t u_bits) {
  const float g = __uint_as_float(g_bits), u = __uint_as_float(u_bits);
  return __fdividef(g * u, 1.0f + __expf(-g));
}

// Epilogue of one warp: its 32 accumulator rows (TMEM lanes) x 256 fp32
// columns starting at t_row, written as bf16 into this lane's output row dst.
//   kSwiGLU: columns [0,128) hold gate, [128,256) up -> 128 outputs
//            silu(g) * u = g u / (1 + e^-g) with the fast exp / divide
//            intrinsics (relative error ~1e-6, far below bf16 rounding).
//   kScale : 256 outputs, each times the row's route probability.
// The TMEM loads of chunk i+1 are in flight while chunk i is converted and
// stored (double-buffered registers).
// One 32-column bf16 chunk of the warp's 32 rows (pk: this lane's row, 64 B)
// to global memory through shared memory: lane L stages its row, then each
// store instruction writes 8 whole 64-byte row pieces (4 lanes per row) rather
// than 32 scattered 16-byte pieces.  Parts are XOR-swizzled so that both the
// staging writes and the reads are free of bank conflicts.
__device__ __forceinline__ void store_chunk_rows(const uint4 (&pk)[4], bool valid,
                                                 __nv_bfloat16* dst, uint4* scratch, int lane) {
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 4; ++j) scratch[lane * 4 + (j ^ ((lane >> 1) & 3))] = pk[j];
  __syncwarp();
  const uint64_t my_dst = reinterpret_cast<uint64_t>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = i * 8 + (lane >> 2), j = lane & 3;
    const uint64_t rd = __shfl_sync(0xffffffffu, my_dst, r);
    const int rv = __shfl_sync(0xffffffffu, valid ? 1 : 0, r);
    const uint4 v = scratch[r * 4 + (j ^ ((r >> 1) & 3))];
    if (rv) reinterpret_cast<uint4*>(rd)[j] = v;
  }
}

// NCH 32-column chunks of the warp's 32 rows starting at output column c0
// (kSwiGLU: gate columns c0.., up columns 128 + c0..; kScale: columns c0..).
template <int EPI, int NCH>
__device__ __forceinline__ void epilogue_part(uint32_t t_row, int c0, bool valid, float scale,
                                              __nv_bfloat16* dst, uint4* scratch, int lane) {
  static_assert(BN == 256, "epilogue assumes 256 accumulator columns");
  if constexpr (EPI == kSwiGLU) {
    uint32_t g[2][32], u[2][32];
    sm100::tmem_ld_32x32b_x32(t_row + c0, g[0]);
    sm100::tmem_ld_32x32b_x32(t_row + BN / 2 + c0, u[0]);
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const int b = i & 1;
      sm100::tmem_ld_wait();
      sm100::tmem_regs_ready(g[b]);
      sm100::tmem_regs_ready(u[b]);
      if (i + 1 < NCH) {
        sm100::tmem_ld_32x32b_x32(t_row + c0 + 32 * (i + 1), g[b ^ 1]);
        sm100::tmem_ld_32x32b_x32(t_row + BN / 2 + c0 + 32 * (i + 1), u[b ^ 1]);
      }
      uint4 pk[4];
      uint32_t* pw = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
      for (int j = 0; j < 16; ++j)
        pw[j] = pack_bf16x2(swiglu_fast(g[b][2 * j], u[b][2 * j]),
                            swiglu_fast(g[b][2 * j + 1], u[b][2 * j + 1]));
      store_chunk_rows(pk, valid, dst + c0 + 32 * i, scratch, lane);
    }
  } else {
    uint32_t a[2][32];
    sm100::tmem_ld_32x32b_x32(t_row + c0, a[0]);
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const int b = i & 1;
      sm100::tmem_ld_wait();
      sm100::tmem_regs_ready(a[b]);
      if (i + 1 < NCH) sm100::tmem_ld_32x32b_x32(t_row + c0 + 32 * (i + 1), a[b ^ 1]);
      uint4 pk[4];
      uint32_t* pw = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
      for (int j = 0; j < 16; ++j)
        pw[j] = pack_bf16x2(__uint_as_float(a[b][2 * j]) * scale,
                            __uint_as_float(a[b][2 * j + 1]) * scale);
      store_chunk_rows(pk, valid, dst + c0 + 32 * i, scratch, lane);
    }
  }
}

// All 256 accumulator columns of the warp's rows (one warp per lane quarter).
template <int EPI>
__device__ __forceinline__ void epilogue_rows(uint32_t t_row, bool valid, float scale,
                                              __nv_bfloat16* dst, uint4* scratch, int lane) {
  epilogue_part<EPI, EPI == kSwiGLU ? BN / 2 / 32 : BN / 32>(t_row, 0, valid, scale, dst, scratch,
                                                            lane);
}

template <int EPI>
__global__ void __launch_bounds__(256, 1) moe_gemm_kernel(
    const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
    const int* __restrict__ expert_offsets, const int* __restrict__ tile_offsets, int E, int K,
    int n_weight_rows, __nv_bfloat16* __restrict__ out, int out_ld,
    const float* __restrict__ row_scale, const int* __restrict__ out_row, int32_t* dev_status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* mma_done = tmem_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = n_weight_rows / BN;
  const int total_tiles = __ldg(tile_offsets + E) * n_tiles;
  const int kblocks = K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      sm100::mbar_init(&tmem_full[a], 1);
      sm100::mbar_init(&tmem_empty[a], 128);
    }
    sm100::mbar_init(mma_done, 1);
    *abort_flag = 0;
    sm100::fence_mbar_init();
    sm100::tma_prefetch_desc(&map_a);
    sm100::tma_prefetch_desc(&map_b);
  }
  if (warp == 2) sm100::tmem_alloc(tmem_slot, TMEM_COLS);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    // The whole warp walks the schedule; lane 0 issues, waits are warp-uniform.
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued[STAGES] = {0, 0, 0, 0};
    bool ok = true;
    for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
      const TileInfo ti = map_tile(tile, n_tiles, tile_offsets, expert_offsets, E);
      const int brow = ti.expert * n_weight_rows + ti.n_tile * BN;
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!sm100::mbar_wait_warp(&empty[stage], phase ^ 1u, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* sa = smem + stage * STAGE_BYTES;
          uint8_t* sb = sa + A_STAGE_BYTES;
          sm100::mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          sm100::tma_load_2d(&map_a, &full[stage], sa, kb * BK, ti.row0);
          sm100::tma_load_2d(&map_b, &full[stage], sb, kb * BK, brow);
        }
        issued[stage]++;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // make sure no TMA write into shared memory is still in flight
    for (int s = 0; s < STAGES; ++s)
      if (issued[s] > 0) sm100::mbar_wait_warp(&full[s], (issued[s] - 1u) & 1u, dev_status, nullptr);
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    constexpr uint32_t idesc = sm100::make_idesc_bf16_f32(BM, BN);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
      if (!sm100::mbar_wait_warp(&tmem_empty[acc], acc_phase ^ 1u, dev_status, abort_flag)) break;
      sm100::tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!sm100::mbar_wait_warp(&full[stage], phase, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        if (lane == 0) {
          const uint32_t sa = sm100::smem_u32(smem + stage * STAGE_BYTES);
          const uint64_t adesc = sm100::make_sw128_kmajor_desc(sa);
          const uint64_t bdesc = sm100::make_sw128_kmajor_desc(sa + A_STAGE_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // advance 16 bf16 (32 bytes) along K inside the swizzle atom
            sm100::umma_bf16_ss(d_tmem, adesc + 2u * kk, bdesc + 2u * kk, idesc,
                                (kb | kk) != 0 ? 1u : 0u);
          }
          sm100::umma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      if (lane == 0) sm100::umma_commit(&tmem_full[acc]);
      __syncwarp();
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // wait for every MMA issued by lane 0 before TMEM/shared memory go away
    if (lane == 0) sm100::umma_commit(mma_done);
    __syncwarp();
    sm100::mbar_wait_warp(mma_done, 0, dev_status, nullptr);
  } else if (warp >= 4) {
    // --------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    uint4* epi_scratch = reinterpret_cast<uint4*>(smem + STAGES * STAGE_BYTES + 256) + q * 128;
    const int r = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      const TileInfo ti = map_tile(tile, n_tiles, tile_offsets, expert_offsets, E);
      if (!sm100::mbar_wait_warp(&tmem_full[acc], acc_phase, dev_status, abort_flag)) break;
      sm100::tc_fence_after();
      const uint32_t t_row = tmem_base + static_cast<uint32_t>(acc * BN) +
                             (static_cast<uint32_t>(q * 32) << 16);
      const bool valid = r < ti.rows_valid;
      const int64_t row = static_cast<int64_t>(ti.row0) + r;
      const float scale = (EPI == kScale && valid) ? __ldg(row_scale + row) : 0.0f;
      const int64_t orow = (out_row != nullptr && valid) ? __ldg(out_row + row) : row;
      __nv_bfloat16* dst = out + orow * out_ld + ti.n_tile * (EPI == kSwiGLU ? BN / 2 : BN);
      epilogue_rows<EPI>(t_row, valid, scale, dst, epi_scratch, lane);
      sm100::tc_fence_before();
      sm100::mbar_arrive(&tmem_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------------
// CTA-pair variant: a cluster of two CTAs computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2.  Each CTA stages 128 A rows and 128 B rows per
// 64-wide K block (32 KB, 6 stages), so the per-SM operand traffic per FLOP is
// half that of the single-CTA 128 x 256 tile.  The even CTA issues the MMAs;
// its commits arrive on the barriers of both CTAs (multicast commit); the odd
// CTA's TMA completions are counted on the even CTA's "full" barrier and its
// epilogue warps arrive remotely on the even CTA's "tmem empty" barrier.
// Loads are plain (no multicast): every operand is read from local HBM.
// Eight epilogue warps (warps 4-11 of 384 threads): two per TMEM lane
// quarter, each draining half of the accumulator's columns, so a tile's
// epilogue (TMEM loads, conversion, staged stores) runs on two warps per SM
// sub-partition and finishes inside the next tile's main loop.
constexpr int PBM = 128, PBN = 256, PBK = 64, PST = 6;
constexpr int P_THREADS = 384, P_EPI_WARPS = 8;
constexpr int P_A_BYTES = PBM * PBK * 2;         // 16 KB
constexpr int P_B_BYTES = (PBN / 2) * PBK * 2;   // 16 KB
constexpr int P_STAGE = P_A_BYTES + P_B_BYTES;   // 32 KB
constexpr int P_EPI_SCRATCH = P_EPI_WARPS * 32 * 64;
constexpr int P_SMEM = PST * P_STAGE + 1024 + 256 + P_EPI_SCRATCH;

__device__ __forceinline__ TileInfo map_tile_pair(int tile, int n_tiles, const int* tile_offsets,
                                                  const int* expert_offsets, int E) {
  TileInfo ti;
  const int m_global = tile / n_tiles;
  ti.n_tile = tile - m_global * n_tiles;
  int lo = 0, hi = E - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(tile_offsets + mid) <= m_global) lo = mid; else hi = mid - 1;
  }
  ti.expert = lo;
  const int m_local = m_global - __ldg(tile_offsets + lo);
  const int e_begin = __ldg(expert_offsets + lo), e_end = __ldg(expert_offsets + lo + 1);
  ti.row0 = e_begin + m_local * 2 * PBM;
  ti.rows_valid = min(2 * PBM, e_end - ti.row0);
  return ti;
}

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(P_THREADS, 1) moe_gemm_pair_kernel(
    const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
    const int* __restrict__ expert_offsets, const int* __restrict__ tile_offsets, int E, int K,
    int n_weight_rows, __nv_bfloat16* __restrict__ out, int out_ld,
    const float* __restrict__ row_scale, const int* __restrict__ out_row, int32_t* dev_status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + PST * P_STAGE);
  uint64_t* empty = full + PST;
  uint64_t* tmem_full = empty + PST;
  uint64_t* tmem_empty = tmem_full + 2;
  uint64_t* mma_done = tmem_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = sm100::cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int n_tiles = n_weight_rows / PBN;
  const int total_tiles = __ldg(tile_offsets + E) * n_tiles;
  const int kblocks = K / PBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PST; ++s) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      sm100::mbar_init(&tmem_full[a], 1);
      sm100::mbar_init(&tmem_empty[a], 2 * P_EPI_WARPS);  // epilogue warps of both CTAs
    }
    sm100::mbar_init(mma_done, 1);
    *abort_flag = 0;
    sm100::fence_mbar_init();
    sm100::tma_prefetch_desc(&map_a);
    sm100::tma_prefetch_desc(&map_b);
  }
  if (warp == 2) sm100::tmem_alloc_pair(tmem_slot, TMEM_COLS);
  sm100::tc_fence_before();
  sm100::cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    int stage = 0;
    uint32_t phase = 0;
    uint32_t issued[PST] = {0, 0, 0, 0, 0, 0};
    bool ok = true;
    for (int tile = cluster; tile < total_tiles && ok; tile += nclusters) {
      const TileInfo ti = map_tile_pair(tile, n_tiles, tile_offsets, expert_offsets, E);
      const int arow = ti.row0 + static_cast<int>(rank) * PBM;
      const int brow = ti.expert * n_weight_rows + ti.n_tile * PBN + static_cast<int>(rank) * (PBN / 2);
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!sm100::mbar_wait_warp(&empty[stage], phase ^ 1u, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* sa = smem + stage * P_STAGE;
          uint8_t* sb = sa + P_A_BYTES;
          const uint32_t full_leader = sm100::mapa_shared(sm100::smem_u32(&full[stage]), 0);
          if (leader) sm100::mbar_arrive_expect_tx(&full[stage], 2 * P_STAGE);
          sm100::tma_load_2d_pair(&map_a, full_leader, sa, kb * PBK, arow);
          sm100::tma_load_2d_pair(&map_b, full_leader, sb, kb * PBK, brow);
        }
        issued[stage]++;
        if (++stage == PST) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // every stage this CTA filled has been consumed by the pair's MMAs once the
    // matching "empty" phase completes
    for (int s = 0; s < PST; ++s)
      if (issued[s] > 0) sm100::mbar_wait_warp(&empty[s], (issued[s] - 1u) & 1u, dev_status, nullptr);
  } else if (warp == 1 && leader) {
    // ------------------------------------------------------- MMA issuer
    constexpr uint32_t idesc = sm100::make_idesc_bf16_f32(2 * PBM, PBN);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int tile = cluster; tile < total_tiles && ok; tile += nclusters) {
      if (!sm100::mbar_wait_warp(&tmem_empty[acc], acc_phase ^ 1u, dev_status, abort_flag)) break;
      sm100::tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * PBN);
      for (int kb = 0; kb < kblocks; ++kb) {
        if (!sm100::mbar_wait_warp(&full[stage], phase, dev_status, abort_flag)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        if (lane == 0) {
          const uint32_t sa = sm100::smem_u32(smem + stage * P_STAGE);
          const uint64_t adesc = sm100::make_sw128_kmajor_desc(sa);
          const uint64_t bdesc = sm100::make_sw128_kmajor_desc(sa + P_A_BYTES);
#pragma unroll
          for (int kk = 0; kk < PBK / 16; ++kk)
            sm100::umma_bf16_ss_pair(d_tmem, adesc + 2u * kk, bdesc + 2u * kk, idesc,
                                     (kb | kk) != 0 ? 1u : 0u);
          sm100::umma_commit_pair(&empty[stage], 0x3);
        }
        __syncwarp();
        if (++stage == PST) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      if (lane == 0) sm100::umma_commit_pair(&tmem_full[acc], 0x3);
      __syncwarp();
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) sm100::umma_commit_pair(mma_done, 0x1);
    __syncwarp();
    sm100::mbar_wait_warp(mma_done, 0, dev_status, nullptr);
  } else if (warp >= 4) {
    // --------------------------------------------------------- epilogue
    const int q = warp & 3;                   // TMEM lane quarter this warp may access
    const int half = (warp - 4) >> 2;         // which half of the columns it drains
    const int r = q * 32 + lane;
    uint4* epi_scratch = reinterpret_cast<uint4*>(smem + PST * P_STAGE + 256) + (warp - 4) * 128;
    const uint32_t empty_leader0 = sm100::mapa_shared(sm100::smem_u32(&tmem_empty[0]), 0);
    const uint32_t empty_leader1 = sm100::mapa_shared(sm100::smem_u32(&tmem_empty[1]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = cluster; tile < total_tiles; tile += nclusters) {
      const TileInfo ti = map_tile_pair(tile, n_tiles, tile_offsets, expert_offsets, E);
      if (!sm100::mbar_wait_warp(&tmem_full[acc], acc_phase, dev_status, abort_flag)) break;
      sm100::tc_fence_after();
      const uint32_t t_row = tmem_base + static_cast<uint32_t>(acc * PBN) +
                             (static_cast<uint32_t>(q * 32) << 16);
      const int my_rows = ti.rows_valid - static_cast<int>(rank) * PBM;
      const bool valid = r < my_rows;
      const int64_t row = static_cast<int64_t>(ti.row0) + static_cast<int>(rank) * PBM + r;
      const float scale = (EPI == kScale && valid) ? __ldg(row_scale + row) : 0.0f;
      const int64_t orow = (out_row != nullptr && valid) ? __ldg(out_row + row) : row;
      __nv_bfloat16* dst = out + orow * out_ld + ti.n_tile * (EPI == kSwiGLU ? PBN / 2 : PBN);
      if constexpr (EPI == kSwiGLU)
        epilogue_part<EPI, PBN / 4 / 32>(t_row, half * (PBN / 4), valid, scale, dst, epi_scratch,
                                         lane);
      else
        epilogue_part<EPI, PBN / 2 / 32>(t_row, half * (PBN / 2), valid, scale, dst, epi_scratch,
                                         lane);
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive_cluster(acc == 0 ? empty_leader0 : empty_leader1);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 2) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// x_perm[pos, :] = x[perm_token[pos], :]   (16-byte vectors), pos < rows and,
// when valid_rows is given, pos < *valid_rows (a count held on the device)
__global__ void gather_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                   const int* __restrict__ perm_token, int64_t rows, int D,
                                   __nv_bfloat16* __restrict__ x_perm,
                                   const int* __restrict__ valid_rows) {
  // one warp per row: the row's source index is loaded once, and each lane
  // has up to eight 16-byte copies in flight (no per-vector division)
  constexpr int kUnroll = 8;
  const int vec = D / 8;
  if (valid_rows != nullptr) rows = min(rows, static_cast<int64_t>(__ldg(valid_rows)));
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t pos = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
       pos < rows; pos += warps) {
    const int t = __ldg(perm_token + pos);
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t) * D);
    uint4* dst = reinterpret_cast<uint4*>(x_perm + pos * D);
    for (int c0 = 0; c0 < vec; c0 += 32 * kUnroll) {
      uint4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < vec) v[u] = __ldg(src + c);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int c = c0 + u * 32 + lane;
        if (c < vec) dst[c] = v[u];
      }
    }
  }
}

// out[t, :] = sum_s y_perm[route_pos[t*k + s], :], fp32 accumulation.
__global__ void combine_rows_kernel(const __nv_bfloat16* __restrict__ y_perm,
                                    const int* __restrict__ route_pos, int64_t N, int k, int D,
                                    __nv_bfloat16* __restrict__ out) {
  const int vec = D / 8;
  const int64_t total = N * vec;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = i / vec;
    const int c = static_cast<int>(i - t * vec);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    // up to eight slots at a time: their positions, then their row pieces, are
    // loaded together (one dependent round each instead of one per slot);
    // the sum stays in slot order
    for (int s0 = 0; s0 < k; s0 += 8) {
      int pos[8];
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (s0 + u < k) pos[u] = __ldg(route_pos + t * k + s0 + u);
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (s0 + u < k)
          v[u] = __ldg(reinterpret_cast<const uint4*>(y_perm + static_cast<int64_t>(pos[u]) * D) + c);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        if (s0 + u >= k) break;
        const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = unpack_bf16x2(w[j]);
          acc[2 * j] += f.x;
          acc[2 * j + 1] += f.y;
        }
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

// w13[e, 256*j + r] = r < 128 ? w_gate[e, 128*j + r] : w_up[e, 128*j + r - 128]
__global__ void pack_w13_kernel(const __nv_bfloat16* __restrict__ w_gate,
                                const __nv_bfloat16* __restrict__ w_up, int E, int F, int D,
                                __nv_bfloat16* __restrict__ w13) {
  const int vec = D / 8;
  const int64_t total = static_cast<int64_t>(E) * 2 * F * vec;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / vec;  // row of w13 (0 .. E*2F)
    const int c = static_cast<int>(i - row * vec);
    const int e = static_cast<int>(row / (2 * F));
    const int rr = static_cast<int>(row - static_cast<int64_t>(e) * 2 * F);
    const int j = rr / BN, r = rr % BN;
    const __nv_bfloat16* src = r < BN / 2 ? w_gate : w_up;
    const int64_t srow = static_cast<int64_t>(e) * F + j * (BN / 2) + (r % (BN / 2));
    reinterpret_cast<uint4*>(w13 + row * D)[c] =
        __ldg(reinterpret_cast<const uint4*>(src + srow * D) + c);
  }
}

int grid_for(int64_t work, int threads) {
  const int64_t blocks = ceil_div(work, threads);
  return static_cast<int>(blocks < 8 * 148 ? (blocks > 0 ? blocks : 1) : 8 * 148);
}

int32_t ensure_gemm_attrs() {
  int32_t st = ensure_smem(moe_gemm_kernel<kSwiGLU>, GEMM_SMEM);
  if (!st) st = ensure_smem(moe_gemm_kernel<kScale>, GEMM_SMEM);
  if (!st) st = ensure_smem(moe_gemm_pair_kernel<kSwiGLU>, P_SMEM);
  if (!st) st = ensure_smem(moe_gemm_pair_kernel<kScale>, P_SMEM);
  return st;
}

// gather -> GEMM1 (SwiGLU) -> GEMM2 (probability scale) for a plan of `rows`
// positions; GEMM2 writes y[out_row ? out_row[pos] : pos].  valid_count: the
// gather stops at expert_offsets[E] (read on the device) instead of `rows`.
int32_t run_grouped(const __nv_bfloat16* x, int32_t d_model, int64_t rows,
                    const int32_t* perm_token, const float* perm_prob,
                    const int32_t* expert_offsets, const int32_t* tile_offsets, int32_t tile_m,
                    int32_t n_experts, const __nv_bfloat16* w13, const __nv_bfloat16* w2,
                    int32_t ffn, __nv_bfloat16* x_perm, __nv_bfloat16* h_perm, __nv_bfloat16* y,
                    const int32_t* out_row, bool valid_count, int32_t* dev_status,
                    cudaStream_t s) {
  int32_t st = ensure_gemm_attrs();
  if (st) return st;
  gather_rows_kernel<<<grid_for(rows * 32, 256), 256, 0, s>>>(
      x, perm_token, rows, d_model, x_perm, valid_count ? expert_offsets + n_experts : nullptr);
  count_launch();

  const bool pair = tile_m == 2 * PBM;
  const uint32_t b_box = pair ? PBN / 2 : BN;
  CUtensorMap ma1, mb1, ma2, mb2;
  if (!make_bf16_2d_map(&ma1, x_perm, rows, d_model, d_model, BM, BK) ||
      !make_bf16_2d_map(&mb1, w13, static_cast<uint64_t>(n_experts) * 2 * ffn, d_model, d_model,
                        b_box, BK) ||
      !make_bf16_2d_map(&ma2, h_perm, rows, ffn, ffn, BM, BK) ||
      !make_bf16_2d_map(&mb2, w2, static_cast<uint64_t>(n_experts) * d_model, ffn, ffn, b_box,
                        BK))
    return LLMYB_EUNSUPPORTED;

  // upper bound of the m-tile count without reading device memory
  const int64_t m_tiles_max = ceil_div(rows, tile_m) + n_experts;
  const int sms = num_sms();
  if (pair) {
    const int clusters = sms / 2;
    const int grid1 = 2 * static_cast<int>(std::min<int64_t>(clusters, m_tiles_max * (2 * ffn / PBN)));
    const int grid2 = 2 * static_cast<int>(std::min<int64_t>(clusters, m_tiles_max * (d_model / PBN)));
    moe_gemm_pair_kernel<kSwiGLU><<<grid1, P_THREADS, P_SMEM, s>>>(
        ma1, mb1, expert_offsets, tile_offsets, n_experts, d_model, 2 * ffn, h_perm, ffn, nullptr,
        nullptr, dev_status);
    count_launch();
    moe_gemm_pair_kernel<kScale><<<grid2, P_THREADS, P_SMEM, s>>>(
        ma2, mb2, expert_offsets, tile_offsets, n_experts, ffn, d_model, y, d_model, perm_prob,
        out_row, dev_status);
    count_launch();
  } else {
    const int grid1 = static_cast<int>(std::min<int64_t>(sms, m_tiles_max * (2 * ffn / BN)));
    const int grid2 = static_cast<int>(std::min<int64_t>(sms, m_tiles_max * (d_model / BN)));
    moe_gemm_kernel<kSwiGLU><<<grid1, 256, GEMM_SMEM, s>>>(ma1, mb1, expert_offsets,
                                                            tile_offsets, n_experts, d_model,
                                                            2 * ffn, h_perm, ffn, nullptr, nullptr,
                                                            dev_status);
    count_launch();
    moe_gemm_kernel<kScale><<<grid2, 256, GEMM_SMEM, s>>>(ma2, mb2, expert_offsets, tile_offsets,
                                                           n_experts, ffn, d_model, y, d_model,
                                                           perm_prob, out_row, dev_status);
    count_launch();
  }
  return launch_status();
}

}  // namespace
}  // namespace llmyb

using namespace llmyb;

LLMYB_API int32_t llmyb_moe_pack_w13(const __nv_bfloat16* w_gate, const __nv_bfloat16* w_up,
                                     int32_t n_experts, int32_t ffn, int32_t d_model,
                                     __nv_bfloat16* w13, void* stream) {
  if (!w_gate || !w_up || !w13 || n_experts <= 0 || ffn <= 0 || d_model <= 0) return LLMYB_EINVAL;
  if (ffn % (BN / 2) != 0 || d_model % BK != 0) return LLMYB_EUNSUPPORTED;
  const int64_t work = static_cast<int64_t>(n_experts) * 2 * ffn * (d_model / 8);
  pack_w13_kernel<<<grid_for(work, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      w_gate, w_up, n_experts, ffn, d_model, w13);
  count_launch();
  return launch_status();
}

// Bytes of caller-provided scratch for llmyb_moe_grouped_swiglu:
// x_perm [N*k, D] + h_perm [N*k, F] + y_perm [N*k, D], bf16, 256-byte aligned.
LLMYB_API int64_t llmyb_moe_grouped_scratch_bytes(int32_t n_tokens, int32_t top_k,
                                                  int32_t d_model, int32_t ffn) {
  if (n_tokens < 0 || top_k <= 0 || d_model <= 0 || ffn <= 0) return -1;
  const int64_t rows = static_cast<int64_t>(n_tokens) * top_k;
  auto al = [](int64_t b) { return (b + 255) / 256 * 256; };
  return al(rows * d_model * 2) + al(rows * ffn * 2) + al(rows * d_model * 2);
}

// Routed SwiGLU experts for a dispatch plan produced by llmyb_route /
// llmyb_moe_plan.  w13 is the [E, 2F, D] interleaved gate/up stack from
// llmyb_moe_pack_w13 and w2 the [E, D, F] down stack (moe.py:119-125 layout).
LLMYB_API int32_t llmyb_moe_grouped_swiglu(
    const __nv_bfloat16* x, int32_t n_tokens, int32_t d_model, int32_t top_k,
    const int32_t* perm_token, const float* perm_prob, const int32_t* route_pos,
    const int32_t* expert_offsets, const int32_t* tile_offsets, int32_t tile_m,
    int32_t n_experts, const __nv_bfloat16* w13, const __nv_bfloat16* w2, int32_t ffn,
    void* scratch, __nv_bfloat16* out, int32_t* dev_status, void* stream) {
  if (n_tokens < 0 || d_model <= 0 || top_k <= 0 || n_experts <= 0 || ffn <= 0)
    return LLMYB_EINVAL;
  if (n_tokens == 0) return LLMYB_OK;
  if (!x || !perm_token || !perm_prob || !route_pos || !expert_offsets || !tile_offsets || !w13 ||
      !w2 || !scratch || !out || !dev_status)
    return LLMYB_EINVAL;
  if (d_model % BN != 0 || ffn % (BN / 2) != 0 || ffn % BK != 0 || d_model % BK != 0)
    return LLMYB_EUNSUPPORTED;
  if (tile_m != BM && tile_m != 2 * PBM) return LLMYB_EINVAL;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out) |
       reinterpret_cast<uintptr_t>(scratch)) & 15u)
    return LLMYB_EINVAL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t st = ensure_gemm_attrs();
  if (st) return st;

  const int64_t rows = static_cast<int64_t>(n_tokens) * top_k;
  auto al = [](int64_t b) { return (b + 255) / 256 * 256; };
  uint8_t* sp = static_cast<uint8_t*>(scratch);
  __nv_bfloat16* x_perm = reinterpret_cast<__nv_bfloat16*>(sp);
  __nv_bfloat16* h_perm = reinterpret_cast<__nv_bfloat16*>(sp + al(rows * d_model * 2));
  __nv_bfloat16* y_perm =
      reinterpret_cast<__nv_bfloat16*>(sp + al(rows * d_model * 2) + al(rows * ffn * 2));
  st = run_grouped(x, d_model, rows, perm_token, perm_prob, expert_offsets, tile_offsets, tile_m,
                   n_experts, w13, w2, ffn, x_perm, h_perm, y_perm, nullptr, false, dev_status, s);
  if (st) return st;
  combine_rows_kernel<<<grid_for(static_cast<int64_t>(n_tokens) * (d_model / 8), 256), 256, 0,
                        s>>>(y_perm, route_pos, n_tokens, top_k, d_model, out);
  count_launch();
  return launch_status();
}

// Routed expert outputs per plan position on the tcgen05 grouped GEMMs, without
// the combine: y_out[out_row ? out_row[pos] : pos] = perm_prob[pos] *
// expert(x[perm_token[pos]]) for pos < expert_offsets[E] (read on the device;
// n_rows bounds it and sizes the scratch of llmyb_moe_grouped_scratch_bytes(
// n_rows, 1, D, F)).  tile_offsets counts tile_m-row tiles per expert.
LLMYB_API int32_t llmyb_moe_grouped_experts_to(
    const __nv_bfloat16* x, int32_t d_model, int32_t n_rows, const int32_t* perm_token,
    const float* perm_prob, const int32_t* expert_offsets, const int32_t* tile_offsets,
    int32_t tile_m, int32_t n_experts, const __nv_bfloat16* w13, const __nv_bfloat16* w2,
    int32_t ffn, void* scratch, __nv_bfloat16* y_out, const int32_t* out_row,
    int32_t* dev_status, void* stream) {
  if (n_rows < 0 || d_model <= 0 || n_experts <= 0 || ffn <= 0) return LLMYB_EINVAL;
  if (n_rows == 0) return LLMYB_OK;
  if (!x || !perm_token || !perm_prob || !expert_offsets || !tile_offsets || !w13 || !w2 ||
      !scratch || !y_out || !dev_status)
    return LLMYB_EINVAL;
  if (d_model % BN != 0 || ffn % (BN / 2) != 0 || ffn % BK != 0 || d_model % BK != 0)
    return LLMYB_EUNSUPPORTED;
  if (tile_m != BM && tile_m != 2 * PBM) return LLMYB_EINVAL;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y_out) |
       reinterpret_cast<uintptr_t>(scratch)) & 15u)
    return LLMYB_EINVAL;
  const int64_t rows = n_rows;
  auto al = [](int64_t b) { return (b + 255) / 256 * 256; };
  uint8_t* sp = static_cast<uint8_t*>(scratch);
  __nv_bfloat16* x_perm = reinterpret_cast<__nv_bfloat16*>(sp);
  __nv_bfloat16* h_perm = reinterpret_cast<__nv_bfloat16*>(sp + al(rows * d_model * 2));
  return run_grouped(x, d_model, rows, perm_token, perm_prob, expert_offsets, tile_offsets, tile_m,
                     n_experts, w13, w2, ffn, x_perm, h_perm, y_out, out_row, true, dev_status,
                     static_cast<cudaStream_t>(stream));
}
