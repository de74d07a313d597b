// Gated DeltaNet recurrence: decode step and chunked prefill scan.
//
// Reference: model/layers/gated_deltanet.py:140-149 (step), :128-132 (q/k
// L2 norm, sigmoid beta/gate, per-head decay = sigmoid(decay_logit)), the
// Triton serial scan/step (sample_standalone.py:435-531) and the native
// gdn_step kernel (llmy_cuda/src/kernels/gdn.cu:22-87).
//
//   S_t = a_t S_{t-1} + k_t w_t^T,   w_t = beta_t (v_t - S_{t-1}^T k_t)
//   o_t = (S_t^T q_t) * gate_t                       (S_t: the updated state)
//   S is zeroed before token t when reset_t is set.
//
// Decode (llmyb_gdn_step): one CTA per (row, head, 32 value columns); four
// warps split the key dimension, lane = value column; the fp32 state streams
// through registers once (read + write = 8*K*V bytes per head).  HBM-bound.
//
// Prefill (llmyb_gdn_chunk_prep + llmyb_gdn_chunk_scan), chunk C = 64:
// inside a chunk with Gamma_t = prod_{j<=t} a_j (segment-masked at resets)
//   S_t = Gamma_t S_0 + sum_{i<=t} (Gamma_t/Gamma_i) k_i w_i^T
//   (I + A) W = diag(beta) V - diag(beta Gamma_{t-1}) K S_0,
//       A[t,i] = beta_t (Gamma_{t-1}/Gamma_i) k_t.k_i  (i < t)
//   O   = diag(Gamma) Q S_0 + (M o Q K^T) W,   M[t,i] = Gamma_t/Gamma_i (i <= t)
//   S_C = Gamma_C S_0 + K^T diag(Gamma_C/Gamma_i) W
// The prep kernel (fully parallel over chunks) forms T = (I + A)^-1 by blocked
// forward substitution and writes U = T diag(beta) V, Kw = T diag(beta
// Gamma_{t-1}) K and Aqk = M o QK^T; the scan kernel (one CTA per row, head
// and value slice) walks the chunks: W = U - Kw S, O = qs*QS + Aqk W,
// S <- sd*S + K^T diag(ks) W, with the fp32 state kept in mma accumulators
// and fed to the tensor cores as a bf16 hi/lo pair.
#include "common.cuh"
#include "mma.cuh"
#include "sm100.cuh"
#include "tma_host.h"

#include <algorithm>

namespace llmyb {
namespace {

constexpr int kC = 64;  // chunk length
constexpr float kLog2e = 1.4426950408889634f;

// ------------------------------------------------------------- activation
// In place on the fused projection [N, width] = [q | k | v | gate | beta]:
// q, k <- x * rsqrt(max(sum x^2, 1e-12)) per head; gate <- sigmoid(gate);
// beta <- sigmoid(beta + bias).  One warp per (token, head).
__global__ void gdn_activate_kernel(__nv_bfloat16* __restrict__ proj, int64_t N, int width, int H,
                                    int KD, int VD, const float* __restrict__ beta_bias) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  if (wid >= N * H) return;
  const int64_t tok = wid / H;
  const int h = static_cast<int>(wid - tok * H);
  __nv_bfloat16* row = proj + tok * width;
  for (int part = 0; part < 2; ++part) {
    __nv_bfloat16* x = row + part * H * KD + h * KD;
    float ss = 0.f;
    for (int i = lane; i < KD; i += 32) {
      const float v = bf2f(x[i]);
      ss += v * v;
    }
    ss = warp_sum(ss);
    const float sc = rsqrtf(fmaxf(ss, 1e-12f));
    for (int i = lane; i < KD; i += 32) x[i] = f2bf(bf2f(x[i]) * sc);
  }
  __nv_bfloat16* g = row + 2 * H * KD + H * VD + h * VD;
  for (int i = lane; i < VD; i += 32) g[i] = f2bf(sigmoidf_(bf2f(g[i])));
  if (lane == 0) {
    __nv_bfloat16* b = row + 2 * H * KD + 2 * H * VD + h;
    *b = f2bf(sigmoidf_(bf2f(*b) + (beta_bias ? beta_bias[h] : 0.f)));
  }
}

// The same activation on 16-byte pieces (8 bf16) for rows whose width is a
// multiple of 8 elements (the model pads its fused projection to that).
// Threads [0, n_norm) take one piece of a q or k head each, KD / 8
// consecutive lanes per head, and form the head's sum of squares with xor
// shuffles inside that lane group; threads [n_norm, n_norm + n_gate) take one
// piece of a gate head, and the first piece of each head also its beta.  Each
// element is read once and written once (the per-head warp kernel above reads
// q and k twice, two bytes per lane).
__global__ void gdn_activate_vec_kernel(__nv_bfloat16* __restrict__ proj, uint32_t n_norm,
                                        uint32_t n_gate, int width, int H, int KD, int VD,
                                        const float* __restrict__ beta_bias) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n_norm) {
    const uint32_t kp = static_cast<uint32_t>(KD) >> 3;  // pieces per head: 2..32, power of 2
    const uint32_t per_tok = 2u * static_cast<uint32_t>(H) * kp;
    const uint32_t tok = i / per_tok;
    uint4* p = reinterpret_cast<uint4*>(proj + static_cast<int64_t>(tok) * width +
                                        static_cast<int64_t>(i - tok * per_tok) * 8);
    uint4 u = *p;
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float v[8];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(w[j]);
      v[2 * j] = f.x;
      v[2 * j + 1] = f.y;
      ss += f.x * f.x + f.y * f.y;
    }
    // n_norm is a multiple of kp and groups start at multiples of kp, so a
    // group never straddles a warp or the end of the q/k range
    const int lane = threadIdx.x & 31;
    const uint32_t gmask = (kp >= 32 ? 0xffffffffu : ((1u << kp) - 1u)) << (lane & ~(kp - 1u));
    for (uint32_t o = kp >> 1; o > 0; o >>= 1) ss += __shfl_xor_sync(gmask, ss, o);
    const float sc = rsqrtf(fmaxf(ss, 1e-12f));
    u.x = pack_bf16x2(v[0] * sc, v[1] * sc);
    u.y = pack_bf16x2(v[2] * sc, v[3] * sc);
    u.z = pack_bf16x2(v[4] * sc, v[5] * sc);
    u.w = pack_bf16x2(v[6] * sc, v[7] * sc);
    *p = u;
  } else if (i - n_norm < n_gate) {
    const uint32_t j = i - n_norm;
    const uint32_t per_tok = static_cast<uint32_t>(H * VD) >> 3;
    const uint32_t tok = j / per_tok;
    const uint32_t off = (j - tok * per_tok) * 8;  // element offset inside the gate block
    __nv_bfloat16* row = proj + static_cast<int64_t>(tok) * width;
    uint4* p = reinterpret_cast<uint4*>(row + 2 * H * KD + H * VD + off);
    uint4 u = *p;
    uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = unpack_bf16x2(w[k]);
      w[k] = pack_bf16x2(sigmoidf_(f.x), sigmoidf_(f.y));
    }
    *p = make_uint4(w[0], w[1], w[2], w[3]);
    if (off % VD == 0) {
      const int h = static_cast<int>(off / VD);
      __nv_bfloat16* b = row + 2 * H * KD + 2 * H * VD + h;
      *b = f2bf(sigmoidf_(bf2f(*b) + (beta_bias ? beta_bias[h] : 0.f)));
    }
  }
}

// --------------------------------------------------------------- decode
struct GdnIO {
  const __nv_bfloat16 *q, *k, *v, *gate, *beta;  // token-major with strides below
  int64_t sq, sk, sv, sg, sb;                    // elements between consecutive tokens
  const float* decay_logit;                      // [H] (alpha = sigmoid), or null
  const float* log_alpha;                        // [B*T, H] per-token log decay, or null
  const uint8_t* reset;                          // [B*T] or null
  const float* beta_bias;                        // raw inputs: beta = sigmoid(beta + bias)
  int raw;  // 1: q/k/gate/beta are raw projections (activated in the kernel)
};

__device__ __forceinline__ float alpha_of(const GdnIO& io, int64_t tok, int h, int H) {
  if (io.log_alpha != nullptr) return expf(io.log_alpha[tok * H + h]);
  return sigmoidf_(io.decay_logit[h]);
}

template <int KD>
__global__ void __launch_bounds__(128) gdn_step_kernel(GdnIO io, int H, int VD,
                                                       float* __restrict__ state,
                                                       __nv_bfloat16* __restrict__ out,
                                                       int64_t so) {
  constexpr int RPW = KD / 4;  // state rows per warp
  __shared__ float s_q[KD], s_k[KD];
  __shared__ float s_red[4][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nvc = VD / 32;
  const int b = blockIdx.x / (H * nvc);
  const int h = (blockIdx.x / nvc) % H;
  const int v0 = (blockIdx.x % nvc) * 32;
  const int64_t tok = b;  // one token per row
  // the state was last written by this kernel one token earlier: it streams in
  // while the projection kernel still runs
  float* S = state + ((static_cast<int64_t>(b) * H + h) * KD) * VD + v0 + lane;
  float s[RPW];
#pragma unroll
  for (int r = 0; r < RPW; ++r) s[r] = S[static_cast<int64_t>(warp * RPW + r) * VD];
  pdl_wait();  // q/k/v/gate/beta come from the projection kernel
  pdl_trigger();
  for (int i = threadIdx.x; i < KD; i += 128) {
    s_q[i] = bf2f(io.q[tok * io.sq + h * KD + i]);
    s_k[i] = bf2f(io.k[tok * io.sk + h * KD + i]);
  }
  __syncthreads();
  if (io.raw) {
    // q, k <- x * rsqrt(max(sum x^2, 1e-12)) per head (gated_deltanet.py:128-129)
    float sq = 0.f, sk = 0.f;
    for (int i = threadIdx.x; i < KD; i += 128) {
      sq += s_q[i] * s_q[i];
      sk += s_k[i] * s_k[i];
    }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    if (lane == 0) {
      s_red[0][warp] = sq;
      s_red[1][warp] = sk;
    }
    __syncthreads();
    const float nq = rsqrtf(fmaxf(s_red[0][0] + s_red[0][1] + s_red[0][2] + s_red[0][3], 1e-12f));
    const float nk = rsqrtf(fmaxf(s_red[1][0] + s_red[1][1] + s_red[1][2] + s_red[1][3], 1e-12f));
    __syncthreads();
    for (int i = threadIdx.x; i < KD; i += 128) {
      s_q[i] *= nq;
      s_k[i] *= nk;
    }
    __syncthreads();
  }
  const bool rst = io.reset != nullptr && io.reset[tok] != 0;
  const float a = alpha_of(io, tok, h, H);
  float beta = bf2f(io.beta[tok * io.sb + h]);
  if (io.raw) beta = sigmoidf_(beta + (io.beta_bias ? io.beta_bias[h] : 0.f));
  float pred = 0.f;
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int kr = warp * RPW + r;
    if (rst) s[r] = 0.f;
    pred += s_k[kr] * s[r];
  }
  s_red[warp][lane] = pred;
  __syncthreads();
  pred = s_red[0][lane] + s_red[1][lane] + s_red[2][lane] + s_red[3][lane];
  const float delta = bf2f(io.v[tok * io.sv + h * VD + v0 + lane]) - pred;
  float o = 0.f;
#pragma unroll
  for (int r = 0; r < RPW; ++r) {
    const int kr = warp * RPW + r;
    const float ns = a * s[r] + beta * s_k[kr] * delta;
    S[static_cast<int64_t>(kr) * VD] = ns;
    o += s_q[kr] * ns;
  }
  __syncthreads();
  s_red[warp][lane] = o;
  __syncthreads();
  if (warp == 0) {
    o = s_red[0][lane] + s_red[1][lane] + s_red[2][lane] + s_red[3][lane];
    // reference order: out.to(hidden dtype) * gate (gated_deltanet.py:149)
    float gt = bf2f(io.gate[tok * io.sg + h * VD + v0 + lane]);
    if (io.raw) gt = sigmoidf_(gt);
    out[tok * so + h * VD + v0 + lane] = f2bf(bf2f(f2bf(o)) * gt);
  }
}

// ----------------------------------------------------------- chunk prep
struct PrepOut {
  __nv_bfloat16* U;   // [B*T, H, VD]
  __nv_bfloat16* Kw;  // [B*T, H, KD]
  __nv_bfloat16* Qs;  // [B*T, H, KD] qscale * q (tcgen05 scan only; else null)
  __nv_bfloat16* Aqk; // [B, H, nC, C, C]
  float* qscale;      // [B, H, T]
  float* kscale;      // [B, H, T]
  float* sdecay;      // [B, H, nC]
};

constexpr int cmax(int a, int b) { return a > b ? a : b; }
constexpr int round16(int x) { return (x + 15) / 16 * 16; }

// Shared memory of the prep kernel, with the phases' buffers aliased so that
// four CTAs fit on an SM:
//   ka  : K (for KK^T / QK^T), then A (the (I + A) factor), then K again
//         (reloaded from L2 for Kw = T2 K)
//   qrv : Q (for KK^T / QK^T), then R (blocked inverse), then V (U = T1 V)
//   Tm  : T = (I + A)^-1, then the staged U / Kw output tiles
// Row strides (in 4-byte words) by access: A is read as tf32 A fragments
// (row g, column t: stride = 4 mod 32 is conflict-free); R and T are written
// as 8-byte fragment pairs and read as B fragments (row t, column g) or as
// 8-byte pairs of the U / Kw A fragments (stride = 8 mod 32).
template <int KD, int VD>
struct PrepSmem {
  static constexpr int LK = KD + 8, LV = VD + 8, LA = kC + 4, LR = kC + 8, LF = kC + 8;
  static constexpr int KA = round16(cmax(kC * LK * 2, kC * LA * 4));
  static constexpr int QRV = round16(cmax(cmax(kC * LK * 2, kC * LR * 4), kC * LV * 2));
  static constexpr int TS = round16(cmax(kC * LF * 4, kC * cmax(KD, VD) * 2));
  alignas(16) uint8_t ka[KA];
  alignas(16) uint8_t qrv[QRV];
  alignas(16) float Tm[TS / 4];
  // per token: inclusive / exclusive cumulative log2-decay, beta, segment, and
  // the T2 column scale beta * Gamma_{t-1} (0 past a reset)
  float g[kC], gprev[kC], beta[kC], s2[kC];
  int seg[kC];
  float wsum[2];
  int wseg[2];
};

// Output tile [64][W] bf16 staged in shared memory with the 16-byte pieces
// of row t XOR-swizzled by t (conflict-free fragment writes and row reads).
template <int W>
__device__ __forceinline__ void stage_pair(uint8_t* tile, int t, int col, uint32_t v) {
  constexpr int kCh = W / 8;
  const int ch = (col >> 3) ^ (t & (kCh - 1));
  *reinterpret_cast<uint32_t*>(tile + t * (W * 2) + ch * 16 + (col & 7) * 2) = v;
}

// rows t < n of the staged tile to dst + t * ld (16-byte stores)
template <int W>
__device__ __forceinline__ void store_staged(const uint8_t* tile, __nv_bfloat16* dst, int64_t ld,
                                             int n, int tid) {
  constexpr int kCh = W / 8;
  for (int i = tid; i < n * kCh; i += 128) {
    const int t = i / kCh, ch = i - t * kCh;
    const uint4 v = *reinterpret_cast<const uint4*>(tile + t * (W * 2) + ((ch ^ (t & (kCh - 1))) * 16));
    *reinterpret_cast<uint4*>(dst + t * ld + ch * 8) = v;
  }
}

template <int KD, int VD>
__global__ void __launch_bounds__(128) gdn_chunk_prep_kernel(GdnIO io, int B, int T, int H,
                                                             PrepOut po) {
  using SM = PrepSmem<KD, VD>;
  extern __shared__ uint8_t smem_raw[];
  SM& sm = *reinterpret_cast<SM*>(smem_raw);
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(sm.qrv);
  float* sR = reinterpret_cast<float*>(sm.qrv);
  __nv_bfloat16* sV = reinterpret_cast<__nv_bfloat16*>(sm.qrv);
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(sm.ka);
  float* sA = reinterpret_cast<float*>(sm.ka);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nC = static_cast<int>(ceil_div(T, kC));
  const int c = blockIdx.x % nC;
  const int h = (blockIdx.x / nC) % H;
  const int b = blockIdx.x / (nC * H);
  const int t0 = c * kC;
  const int n = min(kC, T - t0);
  const int64_t tok0 = static_cast<int64_t>(b) * T + t0;
  const int64_t bh = static_cast<int64_t>(b) * H + h;

  // ---- K, Q (zero rows beyond n) and the per-token scalars
  for (int i = tid; i < kC * (KD / 8); i += 128) {
    const int r = i / (KD / 8), cc = (i % (KD / 8)) * 8;
    const bool ok = r < n;
    const int64_t tok = tok0 + (ok ? r : 0);
    mma::cp_async16(&sK[r * SM::LK + cc], io.k + tok * io.sk + h * KD + cc, ok);
    mma::cp_async16(&sQ[r * SM::LK + cc], io.q + tok * io.sq + h * KD + cc, ok);
  }
  mma::cp_async_commit();
  // V into registers now (it lands in shared memory after the triangular
  // solve, whose space it reuses), so its latency overlaps the whole solve
  constexpr int kVPer = kC * (VD / 8) / 128;
  uint4 vreg[kVPer];
#pragma unroll
  for (int u = 0; u < kVPer; ++u) {
    const int i = tid + 128 * u;
    const int r = i / (VD / 8), cc = (i % (VD / 8)) * 8;
    vreg[u] = r < n ? __ldg(reinterpret_cast<const uint4*>(io.v + (tok0 + r) * io.sv + h * VD + cc))
                    : make_uint4(0, 0, 0, 0);
  }
  // per-token scalars, one thread per token; cumulative sums by warp scans
  // (decays in log2 units, so every Gamma ratio below is one exp2)
  float la = 0.f, la_own = 0.f, bt = 0.f;
  int rs = 0;
  if (tid < kC) {
    const int t = tid;
    if (t < n) {
      const int64_t tok = tok0 + t;
      la = (io.log_alpha != nullptr ? io.log_alpha[tok * H + h]
                                    : logf(sigmoidf_(io.decay_logit[h]))) * kLog2e;
      bt = bf2f(io.beta[tok * io.sb + h]);
      rs = (io.reset != nullptr && io.reset[tok] != 0) ? 1 : 0;
    }
    la_own = la;
    float gs = la;
    int ss = rs;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float gu = __shfl_up_sync(0xffffffffu, gs, o);
      const int su = __shfl_up_sync(0xffffffffu, ss, o);
      if (lane >= o) {
        gs += gu;
        ss += su;
      }
    }
    if (lane == 31) {
      sm.wsum[warp] = gs;
      sm.wseg[warp] = ss;
    }
    la = gs;  // inclusive within the warp
    rs = ss;
  }
  __syncthreads();
  if (tid < kC) {
    const int t = tid;
    const float g = la + (warp == 1 ? sm.wsum[0] : 0.f);
    const int seg = rs + (warp == 1 ? sm.wseg[0] : 0);
    sm.g[t] = g;
    sm.gprev[t] = g - la_own;
    sm.beta[t] = bt;
    sm.seg[t] = seg;
    sm.s2[t] = seg == 0 ? bt * fast_exp2(g - la_own) : 0.f;
  }
  mma::cp_async_wait<0>();
  __syncthreads();
  if (po.Qs != nullptr) {
    // Qs = diag(qscale) Q (0 before the chunk's first reset), for the tcgen05
    // scan's single output accumulator
    for (int i = tid; i < n * (KD / 8); i += 128) {
      const int r = i / (KD / 8), cc = (i % (KD / 8)) * 8;
      const float sc = sm.seg[r] == 0 ? fast_exp2(sm.g[r]) : 0.f;
      const uint4 v = *reinterpret_cast<const uint4*>(&sQ[r * SM::LK + cc]);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(w[j]);
        ow[j] = pack_bf16x2(f.x * sc, f.y * sc);
      }
      *reinterpret_cast<uint4*>(po.Qs + ((tok0 + r) * H + h) * KD + cc) = o;
    }
  }

  // ---- KK^T and QK^T for rows 16*warp .. +15 (all 64 columns)
  float kk[8][4], qk[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) kk[j][e] = qk[j][e] = 0.f;
#pragma unroll
  for (int ks = 0; ks < KD; ks += 16) {
    uint32_t ak[4], aq[4];
    mma::load_a(ak, sK, SM::LK, warp * 16, ks);
    mma::load_a(aq, sQ, SM::LK, warp * 16, ks);
#pragma unroll
    for (int nb = 0; nb < 8; nb += 2) {
      uint32_t bb[4];
      mma::load_b_nk(bb, sK, SM::LK, nb * 8, ks);
      mma::mma_bf16(kk[nb], ak, bb[0], bb[1]);
      mma::mma_bf16(kk[nb + 1], ak, bb[2], bb[3]);
      mma::mma_bf16(qk[nb], aq, bb[0], bb[1]);
      mma::mma_bf16(qk[nb + 1], aq, bb[2], bb[3]);
    }
  }
  __syncthreads();  // Q and K are dead from here on (their spaces become R and A)
  // ---- masks and scales; A to shared memory (fp32), Aqk to global (bf16)
  __nv_bfloat16* aqk_out = po.Aqk + (bh * nC + c) * kC * kC;
  {
    const int r0 = warp * 16 + (lane >> 2);
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int t = r0 + half * 8;
        const int i = nb * 8 + (lane & 3) * 2;
        float av[2], mv[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int ii = i + u;
          const bool same = sm.seg[t] == sm.seg[ii];
          av[u] = (ii < t && same)
                      ? sm.beta[t] * fast_exp2(sm.gprev[t] - sm.g[ii]) * kk[nb][half * 2 + u]
                      : 0.f;
          mv[u] = (ii <= t && same && t < n)
                      ? fast_exp2(sm.g[t] - sm.g[ii]) * qk[nb][half * 2 + u]
                      : 0.f;
        }
        *reinterpret_cast<float2*>(&sA[t * SM::LA + i]) = make_float2(av[0], av[1]);
        *reinterpret_cast<uint32_t*>(aqk_out + t * kC + i) = pack_bf16x2(mv[0], mv[1]);
      }
    }
  }
  __syncthreads();

  // ---- T = (I + A)^-1, blocked: 16x16 diagonal blocks by forward
  // substitution (one thread per column), then off-diagonal blocks
  // T_ij = -T_ii * sum_{k=j}^{i-1} A_ik T_kj, block row by block row.
  if (tid < 64) {
    // column j of diagonal block blk in registers (zero above the diagonal)
    const int blk = tid >> 4, j = tid & 15, base = blk * 16;
    float col[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      float acc = (t == j) ? 1.f : 0.f;
#pragma unroll
      for (int i = 0; i < t; ++i) acc -= sA[(base + t) * SM::LA + base + i] * col[i];
      col[t] = acc;
    }
#pragma unroll
    for (int t = 0; t < 16; ++t) sm.Tm[(base + t) * SM::LF + base + j] = col[t];
  } else {
    // meanwhile warps 2-3 zero the six blocks above the diagonal (16-byte stores)
    for (int i = tid - 64; i < 6 * 16 * 4; i += 64) {
      const int blk = i >> 6, row = (i >> 2) & 15, piece = i & 3;
      const int br = blk < 3 ? 0 : (blk < 5 ? 1 : 2);
      const int bc = blk < 3 ? blk + 1 : (blk < 5 ? blk - 1 : 3);
      *reinterpret_cast<float4*>(&sm.Tm[(br * 16 + row) * SM::LF + bc * 16 + piece * 4]) =
          make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  __syncthreads();
  // off-diagonal blocks, block row by block row, on the tensor cores in tf32
  // (10-bit mantissas, finer than the bf16 rounding T gets afterwards):
  // R = A[bi, <bi] T[<bi, <bi], then T[bi, <bi] = -T[bi, bi] R; warp w takes
  // the 8-column output tiles w, w+4, ...
  {
    const int g = lane >> 2, tq = lane & 3;
    for (int bi = 1; bi < 4; ++bi) {
      const int r0 = bi * 16;
      for (int nt = warp; nt < 2 * bi; nt += 4) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int ks = 0; ks < 2 * bi; ++ks) {  // T is zero above its diagonal blocks
          const uint32_t a[4] = {
              mma::to_tf32(sA[(r0 + g) * SM::LA + 8 * ks + tq]),
              mma::to_tf32(sA[(r0 + g + 8) * SM::LA + 8 * ks + tq]),
              mma::to_tf32(sA[(r0 + g) * SM::LA + 8 * ks + tq + 4]),
              mma::to_tf32(sA[(r0 + g + 8) * SM::LA + 8 * ks + tq + 4])};
          const uint32_t bb[2] = {mma::to_tf32(sm.Tm[(8 * ks + tq) * SM::LF + 8 * nt + g]),
                                  mma::to_tf32(sm.Tm[(8 * ks + tq + 4) * SM::LF + 8 * nt + g])};
          mma::mma_tf32(acc, a, bb);
        }
        *reinterpret_cast<float2*>(&sR[(r0 + g) * SM::LR + 8 * nt + 2 * tq]) =
            make_float2(acc[0], acc[1]);
        *reinterpret_cast<float2*>(&sR[(r0 + g + 8) * SM::LR + 8 * nt + 2 * tq]) =
            make_float2(acc[2], acc[3]);
      }
      __syncthreads();
      for (int nt = warp; nt < 2 * bi; nt += 4) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          const uint32_t a[4] = {
              mma::to_tf32(sm.Tm[(r0 + g) * SM::LF + r0 + 8 * ks + tq]),
              mma::to_tf32(sm.Tm[(r0 + g + 8) * SM::LF + r0 + 8 * ks + tq]),
              mma::to_tf32(sm.Tm[(r0 + g) * SM::LF + r0 + 8 * ks + tq + 4]),
              mma::to_tf32(sm.Tm[(r0 + g + 8) * SM::LF + r0 + 8 * ks + tq + 4])};
          const uint32_t bb[2] = {mma::to_tf32(sR[(r0 + 8 * ks + tq) * SM::LR + 8 * nt + g]),
                                  mma::to_tf32(sR[(r0 + 8 * ks + tq + 4) * SM::LR + 8 * nt + g])};
          mma::mma_tf32(acc, a, bb);
        }
        *reinterpret_cast<float2*>(&sm.Tm[(r0 + g) * SM::LF + 8 * nt + 2 * tq]) =
            make_float2(-acc[0], -acc[1]);
        *reinterpret_cast<float2*>(&sm.Tm[(r0 + g + 8) * SM::LF + 8 * nt + 2 * tq]) =
            make_float2(-acc[2], -acc[3]);
      }
      __syncthreads();
    }
  }

  // ---- K back into the A space (A is dead) for Kw; V into the R space (R is dead)
  for (int i = tid; i < kC * (KD / 8); i += 128) {
    const int r = i / (KD / 8), cc = (i % (KD / 8)) * 8;
    const bool ok = r < n;
    const int64_t tok = tok0 + (ok ? r : 0);
    mma::cp_async16(&sK[r * SM::LK + cc], io.k + tok * io.sk + h * KD + cc, ok);
  }
  mma::cp_async_commit();
#pragma unroll
  for (int u = 0; u < kVPer; ++u) {
    const int i = tid + 128 * u;
    const int r = i / (VD / 8), cc = (i % (VD / 8)) * 8;
    *reinterpret_cast<uint4*>(&sV[r * SM::LV + cc]) = vreg[u];
  }
  if (tid < kC) {
    const int t = tid;
    const int last = n - 1;
    if (t < n) {
      po.qscale[bh * T + t0 + t] = sm.seg[t] == 0 ? fast_exp2(sm.g[t]) : 0.f;
      po.kscale[bh * T + t0 + t] =
          sm.seg[t] == sm.seg[last] ? fast_exp2(sm.g[last] - sm.g[t]) : 0.f;
    }
    if (t == 0) po.sdecay[bh * nC + c] = sm.seg[last] == 0 ? fast_exp2(sm.g[last]) : 0.f;
  }
  mma::cp_async_wait<0>();
  __syncthreads();

  // ---- U = T1 V  (64 x VD), Kw = T2 K (64 x KD) with T1 = T diag(beta) and
  // T2 = T diag(s2) rounded to bf16 straight into the A fragments; rows
  // 16*warp.., staged in the T space once every warp holds its fragments, and
  // written as whole 16-byte row pieces
  {
    uint8_t* s_out = reinterpret_cast<uint8_t*>(sm.Tm);
    uint32_t a1[4][4], a2[4][4];
    {
      const int g = lane >> 2, tq = lane & 3;
      const float* t0 = sm.Tm + (warp * 16 + g) * SM::LF;
      const float* t8 = t0 + 8 * SM::LF;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int c0 = ks * 16 + 2 * tq;
        const float2 x[4] = {*reinterpret_cast<const float2*>(t0 + c0),
                             *reinterpret_cast<const float2*>(t8 + c0),
                             *reinterpret_cast<const float2*>(t0 + c0 + 8),
                             *reinterpret_cast<const float2*>(t8 + c0 + 8)};
        const float2 b0 = *reinterpret_cast<const float2*>(&sm.beta[c0]);
        const float2 b8 = *reinterpret_cast<const float2*>(&sm.beta[c0 + 8]);
        const float2 s0 = *reinterpret_cast<const float2*>(&sm.s2[c0]);
        const float2 s8 = *reinterpret_cast<const float2*>(&sm.s2[c0 + 8]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 bs = e < 2 ? b0 : b8, ss = e < 2 ? s0 : s8;
          a1[ks][e] = pack_bf16x2(x[e].x * bs.x, x[e].y * bs.y);
          a2[ks][e] = pack_bf16x2(x[e].x * ss.x, x[e].y * ss.y);
        }
      }
    }
    __syncthreads();  // T is dead: its space stages the outputs
    const int r = warp * 16 + (lane >> 2);
#pragma unroll
    for (int nb = 0; nb < VD / 8; nb += 2) {
      float acc0[4] = {0, 0, 0, 0}, acc1[4] = {0, 0, 0, 0};
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t bb[4];
        mma::load_b_kn(bb, sV, SM::LV, ks * 16, nb * 8);
        mma::mma_bf16(acc0, a1[ks], bb[0], bb[1]);
        mma::mma_bf16(acc1, a1[ks], bb[2], bb[3]);
      }
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int t = r + half * 8;
        const int col = nb * 8 + (lane & 3) * 2;
        stage_pair<VD>(s_out, t, col, pack_bf16x2(acc0[half * 2], acc0[half * 2 + 1]));
        stage_pair<VD>(s_out, t, col + 8, pack_bf16x2(acc1[half * 2], acc1[half * 2 + 1]));
      }
    }
    __syncthreads();
    store_staged<VD>(s_out, po.U + (tok0 * H + h) * VD, static_cast<int64_t>(H) * VD, n, tid);
    __syncthreads();
#pragma unroll
    for (int nb = 0; nb < KD / 8; nb += 2) {
      float acc0[4] = {0, 0, 0, 0}, acc1[4] = {0, 0, 0, 0};
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t bb[4];
        mma::load_b_kn(bb, sK, SM::LK, ks * 16, nb * 8);
        mma::mma_bf16(acc0, a2[ks], bb[0], bb[1]);
        mma::mma_bf16(acc1, a2[ks], bb[2], bb[3]);
      }
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int t = r + half * 8;
        const int col = nb * 8 + (lane & 3) * 2;
        stage_pair<KD>(s_out, t, col, pack_bf16x2(acc0[half * 2], acc0[half * 2 + 1]));
        stage_pair<KD>(s_out, t, col + 8, pack_bf16x2(acc1[half * 2], acc1[half * 2 + 1]));
      }
    }
    __syncthreads();
    store_staged<KD>(s_out, po.Kw + (tok0 * H + h) * KD, static_cast<int64_t>(H) * KD, n, tid);
  }
}

// ----------------------------------------------------------- chunk scan
// Per (row, head, NG*VC-wide value slice): NG groups of four warps, each
// group owning VC value columns, share the chunk operands (Kw, Q, K, Aqk),
// which are loaded once per CTA.  The chunk operands (Kw, Q, K, Aqk,
// U and gate slices, per-token scales) are double-buffered with cp.async so
// that chunk c+1 streams in while chunk c runs its four small matmuls.
template <int KD, int VC>
struct ScanSmem {
  static constexpr int LK = KD + 8, LVC = VC + 8, LT = kC + 8;
  struct Stage {
    __nv_bfloat16 Kw[kC * LK];
    __nv_bfloat16 Q[kC * LK];
    __nv_bfloat16 K[kC * LK];
    __nv_bfloat16 Aqk[kC * LT];
    __nv_bfloat16 U[kC * LVC];
    float qs[kC], ks[kC];
    float sd, pad[3];
  };
  Stage st[2];
  __nv_bfloat16 Sh[KD * LVC], Sl[KD * LVC];   // state hi/lo
  __nv_bfloat16 Wh[kC * LVC], Wl[kC * LVC];   // W hi/lo
  __nv_bfloat16 Xh[kC * LVC], Xl[kC * LVC];   // diag(kscale) W hi/lo
};

__device__ __forceinline__ void split_store(__nv_bfloat16* hi, __nv_bfloat16* lo, int idx, float x0,
                                            float x1) {
  const __nv_bfloat162 hh = __floats2bfloat162_rn(x0, x1);
  const float2 hf = __bfloat1622float2(hh);
  *reinterpret_cast<__nv_bfloat162*>(hi + idx) = hh;
  *reinterpret_cast<__nv_bfloat162*>(lo + idx) = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
}

template <int KD, int VD, int VC, int NT>
__device__ __forceinline__ void scan_issue_chunk(typename ScanSmem<KD, VC>::Stage& sg,
                                                 const GdnIO& io, const PrepOut& po, int b, int h,
                                                 int H, int T, int nC, int c, int v0, int tid) {
  using SM = ScanSmem<KD, VC>;
  const int t0 = c * kC;
  const int n = min(kC, T - t0);
  const int64_t tok0 = static_cast<int64_t>(b) * T + t0;
  const int64_t bh = static_cast<int64_t>(b) * H + h;
  for (int i = tid; i < kC * (KD / 8); i += NT) {
    const int r = i / (KD / 8), cc = (i % (KD / 8)) * 8;
    const bool ok = r < n;
    const int64_t tok = tok0 + (ok ? r : 0);
    mma::cp_async16(&sg.Kw[r * SM::LK + cc], po.Kw + (tok * H + h) * KD + cc, ok);
    mma::cp_async16(&sg.Q[r * SM::LK + cc], io.q + tok * io.sq + h * KD + cc, ok);
    mma::cp_async16(&sg.K[r * SM::LK + cc], io.k + tok * io.sk + h * KD + cc, ok);
  }
  const __nv_bfloat16* aq = po.Aqk + (bh * nC + c) * kC * kC;
  for (int i = tid; i < kC * (kC / 8); i += NT) {
    const int r = i / (kC / 8), cc = (i % (kC / 8)) * 8;
    mma::cp_async16(&sg.Aqk[r * SM::LT + cc], aq + r * kC + cc, true);
  }
  for (int i = tid; i < kC * (VC / 8); i += NT) {
    const int r = i / (VC / 8), cc = (i % (VC / 8)) * 8;
    const bool ok = r < n;
    const int64_t tok = tok0 + (ok ? r : 0);
    mma::cp_async16(&sg.U[r * SM::LVC + cc], po.U + (tok * H + h) * VD + v0 + cc, ok);
  }
  if (tid < kC) {
    sg.qs[tid] = tid < n ? po.qscale[bh * T + t0 + tid] : 0.f;
    sg.ks[tid] = tid < n ? po.kscale[bh * T + t0 + tid] : 0.f;
  }
  if (tid == 0) sg.sd = po.sdecay[bh * nC + c];
}

template <int KD, int VD, int VC, int NG>
__global__ void __launch_bounds__(128 * NG) gdn_chunk_scan_kernel(GdnIO io, int B, int T, int H,
                                                                  PrepOut po,
                                                                  float* __restrict__ state,
                                                                  __nv_bfloat16* __restrict__ out,
                                                                  int64_t so) {
  constexpr int VS = NG * VC;       // value columns of the CTA
  constexpr int NT = 128 * NG;
  using SM = ScanSmem<KD, VS>;
  constexpr int NB = VC / 8;        // n-blocks of a group's value slice
  constexpr int MT = KD / 64;       // 16-row state tiles per warp (KD/4 rows per warp)
  extern __shared__ uint8_t smem_raw[];
  SM& sm = *reinterpret_cast<SM*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31;
  const int warp = (tid >> 5) & 3;  // warp within its group
  const int cb = (tid >> 7) * VC;   // the group's first column within the CTA slice
  const int nvs = VD / VS;
  const int vs = blockIdx.x % nvs;
  const int h = (blockIdx.x / nvs) % H;
  const int b = blockIdx.x / (nvs * H);
  const int v0 = vs * VS;
  const int nC = static_cast<int>(ceil_div(T, kC));
  const int r_lo = lane >> 2, cq = (lane & 3) * 2;

  scan_issue_chunk<KD, VD, VS, NT>(sm.st[0], io, po, b, h, H, T, nC, 0, v0, tid);
  mma::cp_async_commit();

  // ---- state rows [warp*KD/4, +KD/4) x VC columns in accumulator layout
  float* Sg = state + (static_cast<int64_t>(b) * H + h) * KD * VD + v0 + cb;
  float sacc[MT][NB][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kr = warp * (KD / 4) + mt * 16 + r_lo + (e >> 1) * 8;
        const int vc = nb * 8 + cq + (e & 1);
        sacc[mt][nb][e] = Sg[static_cast<int64_t>(kr) * VD + vc];
      }

  for (int c = 0; c < nC; ++c) {
    typename SM::Stage& sg = sm.st[c & 1];
    const int t0 = c * kC;
    const int n = min(kC, T - t0);
    const int64_t tok0 = static_cast<int64_t>(b) * T + t0;
    if (c + 1 < nC) {
      scan_issue_chunk<KD, VD, VS, NT>(sm.st[(c + 1) & 1], io, po, b, h, H, T, nC, c + 1, v0, tid);
      mma::cp_async_commit();
    }
    // this thread's gate values of the chunk (used by the output phase)
    uint32_t gv[NB][2];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int t = warp * 16 + r_lo + half * 8;
        gv[nb][half] = t < n ? __ldg(reinterpret_cast<const unsigned int*>(
                                   io.gate + (tok0 + t) * io.sg + h * VD + v0 + cb + nb * 8 + cq))
                             : 0u;
      }
    // ---- publish S (hi/lo) for this chunk's products
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int kr = warp * (KD / 4) + mt * 16 + r_lo + half * 8;
          split_store(sm.Sh, sm.Sl, kr * SM::LVC + cb + nb * 8 + cq, sacc[mt][nb][half * 2],
                      sacc[mt][nb][half * 2 + 1]);
        }
    if (c + 1 < nC) mma::cp_async_wait<1>(); else mma::cp_async_wait<0>();
    __syncthreads();

    // ---- W = U - Kw S and QS for rows 16*warp..
    float w[NB][4], qsacc[NB][4];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) w[nb][e] = qsacc[nb][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KD; kk += 16) {
      uint32_t akw[4], aqq[4];
      mma::load_a(akw, sg.Kw, SM::LK, warp * 16, kk);
      mma::load_a(aqq, sg.Q, SM::LK, warp * 16, kk);
#pragma unroll
      for (int nb = 0; nb < NB; nb += 2) {
        uint32_t bh[4], bl[4];
        mma::load_b_kn(bh, sm.Sh, SM::LVC, kk, cb + nb * 8);
        mma::load_b_kn(bl, sm.Sl, SM::LVC, kk, cb + nb * 8);
        mma::mma_bf16(w[nb], akw, bh[0], bh[1]);
        mma::mma_bf16(w[nb + 1], akw, bh[2], bh[3]);
        mma::mma_bf16(w[nb], akw, bl[0], bl[1]);
        mma::mma_bf16(w[nb + 1], akw, bl[2], bl[3]);
        mma::mma_bf16(qsacc[nb], aqq, bh[0], bh[1]);
        mma::mma_bf16(qsacc[nb + 1], aqq, bh[2], bh[3]);
        mma::mma_bf16(qsacc[nb], aqq, bl[0], bl[1]);
        mma::mma_bf16(qsacc[nb + 1], aqq, bl[2], bl[3]);
      }
    }
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int t = warp * 16 + r_lo + half * 8;
        const int col = cb + nb * 8 + cq;
        const float2 u = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sg.U[t * SM::LVC + col]));
        const float w0 = u.x - w[nb][half * 2];
        const float w1 = u.y - w[nb][half * 2 + 1];
        w[nb][half * 2] = w0;
        w[nb][half * 2 + 1] = w1;
        split_store(sm.Wh, sm.Wl, t * SM::LVC + col, w0, w1);
        split_store(sm.Xh, sm.Xl, t * SM::LVC + col, w0 * sg.ks[t], w1 * sg.ks[t]);
      }
    __syncthreads();

    // ---- O = qs * QS + Aqk W ; out = O * gate
    float o[NB][4];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[nb][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kC; kk += 16) {
      uint32_t aa[4];
      mma::load_a(aa, sg.Aqk, SM::LT, warp * 16, kk);
#pragma unroll
      for (int nb = 0; nb < NB; nb += 2) {
        uint32_t bh[4], bl[4];
        mma::load_b_kn(bh, sm.Wh, SM::LVC, kk, cb + nb * 8);
        mma::load_b_kn(bl, sm.Wl, SM::LVC, kk, cb + nb * 8);
        mma::mma_bf16(o[nb], aa, bh[0], bh[1]);
        mma::mma_bf16(o[nb + 1], aa, bh[2], bh[3]);
        mma::mma_bf16(o[nb], aa, bl[0], bl[1]);
        mma::mma_bf16(o[nb + 1], aa, bl[2], bl[3]);
      }
    }
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int t = warp * 16 + r_lo + half * 8;
        if (t < n) {
          const int col = cb + nb * 8 + cq;
          const float o0 = sg.qs[t] * qsacc[nb][half * 2] + o[nb][half * 2];
          const float o1 = sg.qs[t] * qsacc[nb][half * 2 + 1] + o[nb][half * 2 + 1];
          const float2 gt = unpack_bf16x2(gv[nb][half]);
          // reference order: out.to(hidden dtype) * gate
          *reinterpret_cast<uint32_t*>(out + (tok0 + t) * so + h * VD + v0 + col) =
              pack_bf16x2(bf2f(f2bf(o0)) * gt.x, bf2f(f2bf(o1)) * gt.y);
        }
      }

    // ---- S <- sd * S + K^T diag(ks) W   (rows warp*KD/4 ..)
    const float sd = sg.sd;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int e = 0; e < 4; ++e) sacc[mt][nb][e] *= sd;
#pragma unroll
    for (int kk = 0; kk < kC; kk += 16) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        uint32_t ak[4];
        mma::load_a_t(ak, sg.K, SM::LK, warp * (KD / 4) + mt * 16, kk);
#pragma unroll
        for (int nb = 0; nb < NB; nb += 2) {
          uint32_t bh[4], bl[4];
          mma::load_b_kn(bh, sm.Xh, SM::LVC, kk, cb + nb * 8);
          mma::load_b_kn(bl, sm.Xl, SM::LVC, kk, cb + nb * 8);
          mma::mma_bf16(sacc[mt][nb], ak, bh[0], bh[1]);
          mma::mma_bf16(sacc[mt][nb + 1], ak, bh[2], bh[3]);
          mma::mma_bf16(sacc[mt][nb], ak, bl[0], bl[1]);
          mma::mma_bf16(sacc[mt][nb + 1], ak, bl[2], bl[3]);
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kr = warp * (KD / 4) + mt * 16 + r_lo + (e >> 1) * 8;
        const int vc = nb * 8 + cq + (e & 1);
        Sg[static_cast<int64_t>(kr) * VD + vc] = sacc[mt][nb][e];
      }
}

// ------------------------------------------------------------ conv gate
// Decode/prefill epilogue of the GDN mixer (gated_deltanet.py:254-276):
//   y[t] = out_proj(o)[t] * sigmoid(sum_j w[:, j] * x[t - 3 + j])
// x = block input (normed hidden) [B, T, D]; history [B, 3, D] holds the
// previous three inputs (decode) or is null (prefill: zero left padding).
// Taps that cross a reset (same-segment rule of :56-78) are dropped.  With
// `residual` non-null the result is added into it (streams += mixed).
// When `history` is given and `roll_history` is set, the history is advanced
// by the last T inputs (model/model.py:283-289).
__global__ void gdn_conv_gate_kernel(const __nv_bfloat16* __restrict__ x,
                                     const __nv_bfloat16* __restrict__ y_proj,
                                     const float* __restrict__ conv_w, __nv_bfloat16* history,
                                     const uint8_t* __restrict__ reset, int B, int T, int D,
                                     __nv_bfloat16* __restrict__ out,
                                     __nv_bfloat16* __restrict__ residual, int roll1) {
  const int64_t total = static_cast<int64_t>(B) * T * D;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int d = static_cast<int>(i % D);
    const int64_t bt = i / D;
    const int t = static_cast<int>(bt % T);
    const int b = static_cast<int>(bt / T);
    float acc = 0.f;
    // Prefill (no history): taps from before the latest reset at or before t
    // are dropped (same-segment rule).  With a history (the decode path,
    // gated_deltanet.py:257-268) there is no in-sequence masking: the history
    // is zeroed when the row's first token carries a reset.
    int seg_start = 0;
    if (reset != nullptr && history == nullptr) {
      for (int j = 0; j <= min(t, 3); ++j)
        if (reset[static_cast<int64_t>(b) * T + (t - j)]) {
          seg_start = t - j;
          break;
        }
    }
    const bool hist_ok =
        history != nullptr && !(reset != nullptr && reset[static_cast<int64_t>(b) * T] != 0);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int tt = t - 3 + j;
      float xv = 0.f;
      if (tt >= 0) {
        if (tt >= seg_start) xv = bf2f(x[(static_cast<int64_t>(b) * T + tt) * D + d]);
      } else if (hist_ok) {
        xv = bf2f(history[(static_cast<int64_t>(b) * 3 + (3 + tt)) * D + d]);
      }
      acc += conv_w[d * 4 + j] * xv;
    }
    const float yv = bf2f(y_proj[i]) * sigmoidf_(acc);
    if (roll1) {
      // T == 1: this thread owns channel d of row b, so it can shift in place
      __nv_bfloat16* hb = history + static_cast<int64_t>(b) * 3 * D + d;
      const __nv_bfloat16 h1 = hb[D], h2 = hb[2 * D];
      hb[0] = h1;
      hb[D] = h2;
      hb[2 * D] = x[i];
    }
    if (residual != nullptr) {
      residual[i] = f2bf(bf2f(residual[i]) + bf2f(f2bf(yv)));
    } else {
      out[i] = f2bf(yv);
    }
  }
}

// The prompt form of the conv gate (no history, so taps before the row's
// first token are zero) on 16-byte pieces: a thread owns 8 channels of one
// row over a run of `run` tokens and slides the 4-tap window along it in
// registers, so each input row is read once per run (plus three warm-up rows)
// instead of once per tap, and the 8 x 4 filter taps are loaded once.  A reset
// at token t clears the three older taps before x[t] enters the window, which
// keeps exactly the taps at or after the latest reset in [t - 3, t] (the
// same-segment rule of the kernel above).  Consecutive threads take
// consecutive channel pieces of the same run, so a warp reads 512 contiguous
// bytes per token.  Result into out, or added into residual.
__global__ void __launch_bounds__(256) gdn_conv_gate_run_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ y_proj,
    const float* __restrict__ conv_w, const uint8_t* __restrict__ reset, int B, int T, int D,
    int run, __nv_bfloat16* __restrict__ dst, int add) {
  const uint32_t nc = static_cast<uint32_t>(D) >> 3;
  const uint32_t runs = (static_cast<uint32_t>(T) + run - 1) / run;
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= static_cast<uint32_t>(B) * runs * nc) return;
  const uint32_t c = i % nc, rr = i / nc;
  const int r = static_cast<int>(rr % runs), b = static_cast<int>(rr / runs);
  float w[8][4];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float4 f = __ldg(reinterpret_cast<const float4*>(conv_w) + c * 8 + k);
    w[k][0] = f.x;
    w[k][1] = f.y;
    w[k][2] = f.z;
    w[k][3] = f.w;
  }
  const int64_t row0 = static_cast<int64_t>(b) * T;
  // the window holds the inputs as they are stored (bf16 pairs): x[t-3],
  // x[t-2], x[t-1] of the next token t
  uint32_t win[3][4];
#pragma unroll
  for (int j = 0; j < 3; ++j)
#pragma unroll
    for (int k = 0; k < 4; ++k) win[j][k] = 0u;
  const int t0 = r * run, t1 = min(T, t0 + run);
  for (int t = max(0, t0 - 3); t < t1; ++t) {
    if (reset != nullptr && reset[row0 + t]) {
#pragma unroll
      for (int j = 0; j < 3; ++j)
#pragma unroll
        for (int k = 0; k < 4; ++k) win[j][k] = 0u;
    }
    const int64_t off = (row0 + t) * D + static_cast<int64_t>(c) * 8;
    const uint4 xu = __ldg(reinterpret_cast<const uint4*>(x + off));
    const uint32_t xw[4] = {xu.x, xu.y, xu.z, xu.w};
    if (t >= t0) {
      const uint4 yu = __ldg(reinterpret_cast<const uint4*>(y_proj + off));
      const uint32_t yw[4] = {yu.x, yu.y, yu.z, yu.w};
      uint4 ru = make_uint4(0u, 0u, 0u, 0u);
      if (add) ru = *reinterpret_cast<const uint4*>(dst + off);
      const uint32_t rw[4] = {ru.x, ru.y, ru.z, ru.w};
      uint32_t ow[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 a0 = unpack_bf16x2(win[0][k]), a1 = unpack_bf16x2(win[1][k]);
        const float2 a2 = unpack_bf16x2(win[2][k]), a3 = unpack_bf16x2(xw[k]);
        float acc0 = 0.f, acc1 = 0.f;
        acc0 += w[2 * k][0] * a0.x;
        acc0 += w[2 * k][1] * a1.x;
        acc0 += w[2 * k][2] * a2.x;
        acc0 += w[2 * k][3] * a3.x;
        acc1 += w[2 * k + 1][0] * a0.y;
        acc1 += w[2 * k + 1][1] * a1.y;
        acc1 += w[2 * k + 1][2] * a2.y;
        acc1 += w[2 * k + 1][3] * a3.y;
        const float2 yf = unpack_bf16x2(yw[k]);
        const float o0 = yf.x * sigmoidf_(acc0), o1 = yf.y * sigmoidf_(acc1);
        if (add) {
          const float2 rf = unpack_bf16x2(rw[k]);
          const float2 of = unpack_bf16x2(pack_bf16x2(o0, o1));
          ow[k] = pack_bf16x2(rf.x + of.x, rf.y + of.y);
        } else {
          ow[k] = pack_bf16x2(o0, o1);
        }
      }
      *reinterpret_cast<uint4*>(dst + off) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      win[0][k] = win[1][k];
      win[1][k] = win[2][k];
      win[2][k] = xw[k];
    }
  }
}

// history[b] <- the last three block inputs of row b (older slots shift in
// from the previous history when T < 3).  One CTA per row; all reads land in
// shared memory before any write.
__global__ void gdn_conv_roll_kernel(const __nv_bfloat16* __restrict__ x,
                                     __nv_bfloat16* __restrict__ history, int T, int D) {
  extern __shared__ __nv_bfloat16 s_roll[];  // [3, D]
  const int b = blockIdx.x;
  for (int i = threadIdx.x; i < 3 * D; i += blockDim.x) {
    const int j = i / D, d = i - j * D;
    const int src = T - 3 + j;
    s_roll[i] = src >= 0 ? x[(static_cast<int64_t>(b) * T + src) * D + d]
                         : history[(static_cast<int64_t>(b) * 3 + (3 + src)) * D + d];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 3 * D; i += blockDim.x)
    history[static_cast<int64_t>(b) * 3 * D + i] = s_roll[i];
}

// history[b] = the last three inputs x[b, T-3 .. T-1] of a prompt, zero where
// T - 3 + j < 0 (the decode conv history a prefill leaves; 16-byte vectors
// when D % 8 == 0 and both tensors are 16-byte aligned).
template <bool VEC>
__global__ void gdn_history_set_kernel(const __nv_bfloat16* __restrict__ x,
                                       __nv_bfloat16* __restrict__ history, int T, int D) {
  const int b = blockIdx.x;
  __nv_bfloat16* h = history + static_cast<int64_t>(b) * 3 * D;
  if constexpr (VEC) {
    const int dv = D / 8;
    for (int i = threadIdx.x; i < 3 * dv; i += blockDim.x) {
      const int j = i / dv, c = i - j * dv;
      const int src = T - 3 + j;
      reinterpret_cast<uint4*>(h)[i] =
          src >= 0 ? __ldg(reinterpret_cast<const uint4*>(x + (static_cast<int64_t>(b) * T + src) * D) + c)
                   : make_uint4(0, 0, 0, 0);
    }
  } else {
    for (int i = threadIdx.x; i < 3 * D; i += blockDim.x) {
      const int j = i / D, d = i - j * D;
      const int src = T - 3 + j;
      h[i] = src >= 0 ? x[(static_cast<int64_t>(b) * T + src) * D + d] : __float2bfloat16_rn(0.f);
    }
  }
}

// ------------------------------------------------- chunk scan on tcgen05
// K = 128 (or K = 64 padded to 128: the key-dimension boxes past K read as
// zeros, so the state rows K..127 stay zero and only rows < K are loaded and
// stored), value slices of 64 columns; one CTA per (row, head, slice).
//   warp 0     TMA: per chunk [Kw; Qs] (Qs = diag(qscale) q, from the prep
//              kernel), K, [0; Aqk] and the U slice, two stages
//   warp 1     MMA (one thread), per chunk:
//                D1  = [Kw; Qs] S            (rows 0-63: Kw S, rows 64-127: Qs S)
//                D1 += [0; Aqk] W            (rows 64-127 become O)
//                D2  = K^T diag(ks) W        (the state update)
//              S, W and X = diag(ks) W are bf16 hi + lo pairs stored as the
//              two 64-column blocks of one N = 128 operand, so each product is
//              one MMA per K step with the hi and lo results side by side in
//              TMEM (summed by the state warps): about 16 mantissa bits.
//   warps 2-9  state warps, two per TMEM lane quarter, each owning 32 of the
//              64 columns of its lane's row (= key row of S, and token row of
//              D1): the fp32 state slice S[key][..] lives in their registers
//              for the whole sequence.  After D1: W = U - Kw S and X = ks W
//              (token rows) into shared memory as MMA operands; after D1/D2:
//              S <- sd S + D2, S hi/lo into shared memory, and O (D1 rows
//              64-127) times the gate to global memory.
// Operands written by threads use the 128-byte-swizzled MN-major layout of
// an MMA B operand (row = K index, 64 N-columns per row).  TMEM: D1 columns
// [0, 128) (hi | lo), D2 [128, 256).  Every wait is bounded (1 s) and unwinds
// on timeout.
namespace scan_tc {
constexpr int kVS = 64;                                     // value columns per CTA
constexpr int kA1 = 0;                                      // [Kw; Qs]: 2 x (128 rows x 64) bf16
constexpr int kA2 = 32768;                                  // K [64 tok][128 keys]: 2 x 8 KB
constexpr int kA3 = 49152;                                  // [0; Aqk]: 128 rows x 64
constexpr int kU = 65536;                                   // U [64 tok][64 cols]
constexpr int kStage = 73728;
constexpr uint32_t kTx = 2 * 8192 + 2 * 8192 + 2 * 8192 + 8192 + 8192;
constexpr int kS = 2 * kStage;                              // S hi | S lo  [128][64] bf16
constexpr int kW = kS + 32768;                              // W hi | W lo | X hi | X lo  [64][64]
constexpr int kBar = kW + 32768;
constexpr int kSmem = kBar + 256 + 1024;
constexpr uint32_t kTmemCols = 256;

// one half row (32 elements, columns 32 half ..), scale * v (fp32 bit
// patterns), as bf16 hi and lo parts into two swizzled operand tiles
__device__ __forceinline__ void store_row_hilo(uint8_t* hi, uint8_t* lo, int row, int half,
                                               const uint32_t (&v)[32], float scale) {
#pragma unroll
  for (int jj = 0; jj < 4; ++jj) {
    const int j = 4 * half + jj;
    uint4 h, l;
    uint32_t* hw = reinterpret_cast<uint32_t*>(&h);
    uint32_t* lw = reinterpret_cast<uint32_t*>(&l);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int c0 = 8 * jj + 2 * e;
      const float a = __uint_as_float(v[c0]) * scale;
      const float b = __uint_as_float(v[c0 + 1]) * scale;
      const __nv_bfloat162 hh = __floats2bfloat162_rn(a, b);
      const float2 hf = __bfloat1622float2(hh);
      hw[e] = *reinterpret_cast<const uint32_t*>(&hh);
      lw[e] = pack_bf16x2(a - hf.x, b - hf.y);
    }
    const int off = row * 128 + ((j ^ (row & 7)) << 4);
    *reinterpret_cast<uint4*>(hi + off) = h;
    *reinterpret_cast<uint4*>(lo + off) = l;
  }
}
}  // namespace scan_tc

__global__ void __launch_bounds__(320, 1) gdn_scan_tc_kernel(
    const __grid_constant__ CUtensorMap map_kw, const __grid_constant__ CUtensorMap map_qs,
    const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_aqk,
    const __grid_constant__ CUtensorMap map_u, const float* __restrict__ kscale,
    const float* __restrict__ sdecay, const __nv_bfloat16* __restrict__ gate, int64_t sg,
    int B, int T, int H, int KD, int VD, float* __restrict__ state,
    __nv_bfloat16* __restrict__ out, int64_t so, int32_t* dev_status) {
  using namespace scan_tc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kBar);
  uint64_t* st_full = bars;       // [2]
  uint64_t* st_empty = bars + 2;  // [2]
  uint64_t* s_ready = bars + 4;
  uint64_t* d1_full = bars + 5;
  uint64_t* w_ready = bars + 6;
  uint64_t* d23_full = bars + 7;
  uint64_t* mma_done = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvs = VD / kVS;
  const int vs = blockIdx.x % nvs;
  const int h = (blockIdx.x / nvs) % H;
  const int b = blockIdx.x / (nvs * H);
  const int v0 = vs * kVS;
  const int nC = (T + kC - 1) / kC;
  const int64_t bh = static_cast<int64_t>(b) * H + h;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      sm100::mbar_init(&st_full[i], 1);
      sm100::mbar_init(&st_empty[i], 5);  // MMA commit + the four warps that read U
    }
    sm100::mbar_init(s_ready, 8);
    sm100::mbar_init(d1_full, 1);
    sm100::mbar_init(w_ready, 4);
    sm100::mbar_init(d23_full, 1);
    sm100::mbar_init(mma_done, 1);
    *abort_flag = 0;
    sm100::fence_mbar_init();
    sm100::tma_prefetch_desc(&map_kw);
    sm100::tma_prefetch_desc(&map_qs);
    sm100::tma_prefetch_desc(&map_k);
    sm100::tma_prefetch_desc(&map_aqk);
    sm100::tma_prefetch_desc(&map_u);
  }
  // the zero rows of [0; Aqk] (TMA writes only rows 64-127); with K = 64 also
  // the second 64-key block of K, which is never loaded (so the rows K..127
  // of D2 stay zero) -- only the first key block of Kw, Qs and K is fetched
  // and D1 runs over the K / 16 key steps that carry data
  const int kblk = KD / 64;
  for (int i = threadIdx.x; i < 2 * 8192 / 16; i += blockDim.x) {
    const int st = i / 512, o = (i % 512) * 16;
    *reinterpret_cast<uint4*>(smem + st * kStage + kA3 + o) = make_uint4(0, 0, 0, 0);
    if (kblk == 1)
      *reinterpret_cast<uint4*>(smem + st * kStage + kA2 + 8192 + o) = make_uint4(0, 0, 0, 0);
  }
  sm100::fence_proxy_async_smem();
  if (warp == 1) sm100::tmem_alloc(tmem_slot, kTmemCols);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------- TMA
    uint32_t issued = 0;
    for (int c = 0; c < nC; ++c) {
      const int s = c & 1;
      if (!sm100::mbar_wait_warp(&st_empty[s], ((c >> 1) & 1) ^ 1u, dev_status, abort_flag)) break;
      if (lane == 0) {
        uint8_t* st = smem + s * kStage;
        const int t0 = c * kC;
        sm100::mbar_arrive_expect_tx(&st_full[s], kTx - (2 - kblk) * 3 * 8192);
        for (int x = 0; x < kblk; ++x) {
          sm100::tma_load_4d(&map_kw, &st_full[s], st + kA1 + x * 16384, x * 64, h, t0, b);
          sm100::tma_load_4d(&map_qs, &st_full[s], st + kA1 + x * 16384 + 8192, x * 64, h, t0, b);
          sm100::tma_load_4d(&map_k, &st_full[s], st + kA2 + x * 8192, x * 64, h, t0, b);
        }
        sm100::tma_load_2d(&map_aqk, &st_full[s], st + kA3 + 8192, 0,
                           static_cast<int32_t>((bh * nC + c) * kC));
        sm100::tma_load_4d(&map_u, &st_full[s], st + kU, v0, h, t0, b);
      }
      ++issued;
    }
    for (uint32_t i = 1; i <= 2; ++i)
      if (issued >= i)
        sm100::mbar_wait_warp(&st_full[(issued - i) & 1], ((issued - i) >> 1) & 1, dev_status,
                              nullptr);
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    // N = 128: the hi and lo 64-column blocks of S / W / X in one operand
    constexpr uint32_t idesc = sm100::make_idesc_bf16_f32(128, 2 * kVS) | sm100::kIdescBMajorMN;
    constexpr uint32_t idesc_t = idesc | (1u << 15);  // A (K^T) MN-major too
    const uint32_t t_d1 = tmem_base, t_d2 = tmem_base + 128;
    const uint32_t s_hi = sm100::smem_u32(smem + kS), s_lo = s_hi + 16384;
    const uint32_t w_hi = sm100::smem_u32(smem + kW), w_lo = w_hi + 8192;
    const uint32_t x_hi = w_hi + 16384, x_lo = w_hi + 24576;
    for (int c = 0; c < nC; ++c) {
      const int s = c & 1;
      const uint32_t st = sm100::smem_u32(smem + s * kStage);
      if (!sm100::mbar_wait_warp(&st_full[s], (c >> 1) & 1, dev_status, abort_flag) ||
          !sm100::mbar_wait_warp(s_ready, c & 1, dev_status, abort_flag))
        break;
      sm100::tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < 4 * kblk; ++kk) {
          const uint64_t ad =
              sm100::make_sw128_kmajor_desc(st + kA1 + (kk >> 2) * 16384 + (kk & 3) * 32);
          const uint64_t bd = sm100::make_sw128_desc(s_hi + kk * 2048, s_lo - s_hi, 1024);
          sm100::umma_bf16_ss(t_d1, ad, bd, idesc, kk != 0 ? 1u : 0u);
        }
        sm100::umma_commit(d1_full);
      }
      __syncwarp();
      if (!sm100::mbar_wait_warp(w_ready, c & 1, dev_status, abort_flag)) break;
      sm100::tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          // D1 rows 64-127 += Aqk W (rows 0-63 of [0; Aqk] are zero)
          const uint64_t a3 = sm100::make_sw128_kmajor_desc(st + kA3 + kk * 32);
          sm100::umma_bf16_ss(t_d1, a3, sm100::make_sw128_desc(w_hi + kk * 2048, w_lo - w_hi, 1024),
                              idesc, 1u);
          // D2 = K^T X: A = K [token][key] read MN-major (64-key blocks 8 KB apart)
          const uint64_t a2 = sm100::make_sw128_desc(st + kA2 + kk * 2048, 8192, 1024);
          sm100::umma_bf16_ss(t_d2, a2, sm100::make_sw128_desc(x_hi + kk * 2048, x_lo - x_hi, 1024),
                              idesc_t, kk != 0 ? 1u : 0u);
        }
        sm100::umma_commit(d23_full);
        sm100::umma_commit(&st_empty[s]);
      }
      __syncwarp();
    }
    if (lane == 0) sm100::umma_commit(mma_done);
    __syncwarp();
    sm100::mbar_wait_warp(mma_done, 0, dev_status, nullptr);
  } else {
    // ------------------------------------------------------ state warps
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;  // columns [32 half, 32 half + 32)
    const int row = q * 32 + lane;     // TMEM lane: key row of S / D2, row of D1
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + 32 * half;
    uint8_t* s_hi = smem + kS;
    uint8_t* s_lo = s_hi + 16384;
    uint8_t* w_hi = smem + kW;
    uint8_t* w_lo = w_hi + 8192;
    uint8_t* x_hi = w_hi + 16384;
    uint8_t* x_lo = w_hi + 24576;
    const bool key_row = row < KD;  // rows KD..127 of a padded K = 64 state stay zero
    float* Sg = state + (bh * KD + (key_row ? row : 0)) * VD + v0 + 32 * half;
    uint32_t S[32];  // fp32 bit patterns of S[row][v0 + 32 half ..]
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint4 v = key_row ? reinterpret_cast<const uint4*>(Sg)[j] : make_uint4(0, 0, 0, 0);
      S[4 * j] = v.x;
      S[4 * j + 1] = v.y;
      S[4 * j + 2] = v.z;
      S[4 * j + 3] = v.w;
    }
    store_row_hilo(s_hi, s_lo, row, half, S, 1.f);
    sm100::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) sm100::mbar_arrive(s_ready);
    bool ok = true;
    // the chunk's decay scalars, fetched one chunk ahead (off the serial chain)
    float ks_cur = row < 64 && row < T ? __ldg(kscale + bh * T + row) : 0.f;
    float sd_cur = __ldg(sdecay + bh * nC);
    for (int c = 0; c < nC && ok; ++c) {
      const int s = c & 1;
      const int t0 = c * kC;
      const int n = min(kC, T - t0);
      float ks_next = 0.f, sd_next = 0.f;
      if (c + 1 < nC) {
        if (row < 64 && t0 + kC + row < T) ks_next = __ldg(kscale + bh * T + t0 + kC + row);
        sd_next = __ldg(sdecay + bh * nC + c + 1);
      }
      // ---- W = U - Kw S and X = ks W (token rows: lane quarters 0-1)
      // (U of this stage is complete once its "full" phase is)
      if (row < 64 && !sm100::mbar_wait_warp(&st_full[s], (c >> 1) & 1, dev_status, abort_flag))
        break;
      if (!sm100::mbar_wait_warp(d1_full, c & 1, dev_status, abort_flag)) break;
      sm100::tc_fence_after();
      if (row < 64) {
        uint32_t p[32], plo[32];
        sm100::tmem_ld_32x32b_x32(t_lane, p);
        sm100::tmem_ld_32x32b_x32(t_lane + 64, plo);
        const int t = row;
        const uint8_t* urow = smem + s * kStage + kU + t * 128;
        uint4 u4[4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
          u4[jj] = *reinterpret_cast<const uint4*>(urow + (((4 * half + jj) ^ (t & 7)) << 4));
        sm100::tmem_ld_wait();
        sm100::tmem_regs_ready(p);
        sm100::tmem_regs_ready(plo);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          p[j] = __float_as_uint(__uint_as_float(p[j]) + __uint_as_float(plo[j]));
        // W = U - Kw S in place of the loaded product
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const uint32_t uw[4] = {u4[jj].x, u4[jj].y, u4[jj].z, u4[jj].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 uf = unpack_bf16x2(uw[e]);
            const int col = 8 * jj + 2 * e;
            p[col] = __float_as_uint(uf.x - __uint_as_float(p[col]));
            p[col + 1] = __float_as_uint(uf.y - __uint_as_float(p[col + 1]));
          }
        }
        store_row_hilo(w_hi, w_lo, t, half, p, 1.f);
        store_row_hilo(x_hi, x_lo, t, half, p, ks_cur);  // X = diag(ks) W
        sm100::fence_proxy_async_smem();
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          sm100::mbar_arrive(w_ready);
          sm100::mbar_arrive(&st_empty[s]);  // U read
        }
      }
      // ---- S <- sd S + D2; O = D1 rows 64-127 (read before D1 is released)
      if (!sm100::mbar_wait_warp(d23_full, c & 1, dev_status, abort_flag)) break;
      sm100::tc_fence_after();
      uint32_t o[32];
      {
        uint32_t d2[32], d2lo[32];
        sm100::tmem_ld_32x32b_x32(t_lane + 128, d2);
        sm100::tmem_ld_32x32b_x32(t_lane + 192, d2lo);
        sm100::tmem_ld_wait();
        sm100::tmem_regs_ready(d2);
        sm100::tmem_regs_ready(d2lo);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          S[j] = __float_as_uint(sd_cur * __uint_as_float(S[j]) +
                                 (__uint_as_float(d2[j]) + __uint_as_float(d2lo[j])));
      }
      if (row >= 64) {
        uint32_t olo[32];
        sm100::tmem_ld_32x32b_x32(t_lane, o);
        sm100::tmem_ld_32x32b_x32(t_lane + 64, olo);
        sm100::tmem_ld_wait();
        sm100::tmem_regs_ready(o);
        sm100::tmem_regs_ready(olo);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          o[j] = __float_as_uint(__uint_as_float(o[j]) + __uint_as_float(olo[j]));
      }
      if (c + 1 < nC) store_row_hilo(s_hi, s_lo, row, half, S, 1.f);
      sm100::fence_proxy_async_smem();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(s_ready);
      if (row >= 64) {
        const int t = row - 64;
        if (t < n) {
          const int64_t orow = b * static_cast<int64_t>(T) + t0 + t;
          uint4* dst = reinterpret_cast<uint4*>(out + orow * so + h * VD + v0 + 32 * half);
          const uint4* gr =
              reinterpret_cast<const uint4*>(gate + orow * sg + h * VD + v0 + 32 * half);
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const uint4 g4 = __ldg(gr + jj);
            const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w};
            uint4 r4;
            uint32_t* rw = reinterpret_cast<uint32_t*>(&r4);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int col = 8 * jj + 2 * e;
              const float2 g2 = unpack_bf16x2(gw[e]);
              // reference order: out.to(hidden dtype) * gate
              const float o0 = bf2f(f2bf(__uint_as_float(o[col])));
              const float o1 = bf2f(f2bf(__uint_as_float(o[col + 1])));
              rw[e] = pack_bf16x2(o0 * g2.x, o1 * g2.y);
            }
            dst[jj] = r4;
          }
        }
      }
      ks_cur = ks_next;
      sd_cur = sd_next;
    }
    if (key_row)
#pragma unroll
      for (int j = 0; j < 8; ++j)
        reinterpret_cast<uint4*>(Sg)[j] = make_uint4(S[4 * j], S[4 * j + 1], S[4 * j + 2],
                                                     S[4 * j + 3]);
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ------------------------------------------------- value-lane tcgen05 scan
// One CTA per (row, head) for value width 128: the chunk step in transposed
// form, with the value columns as the MMA's M dimension (TMEM lanes).  Every
// operand the threads produce (S^T, W^T, X^T as bf16 hi/lo pairs) is then an
// A operand written straight into tensor memory with tcgen05.st, and shared
// memory holds only the TMA-loaded chunk operands.  Per chunk:
//   D1   = S^T [Kw; Qs]^T  (one N = 128 product: columns 0-63 Kw, 64-127 Qs)
//   D1[:, 0:64] -= U^T     (as U^T (-I): an exact bf16 product)
//                          -> W = -D1[:, 0:64]^T and X = diag(ks) W
//   D2   = X^T K           (K [token][key] read MN-major) -> S <- sd S + D2^T
//   D1[:, 64:128] += W^T Aqk^T  -> O = D1[:, 64:128]^T times the gate
// A hi part and a lo part are two MMAs accumulating into one fp32 tile.
// Warps: 0 TMA (stages of [Kw; Qs], K, Aqk, U), 1 MMA, 2-17 lane warps: lane
// quarter q = warp & 3 (value columns 32q .. 32q+31) and part r = (warp-2)/4
// (tokens 16r .. 16r+15 of W and O, keys r*KD/4 .. of S).  The gate is copied
// by each lane warp (cp.async) into its own shared tile one chunk ahead and
// read transposed; the gated output replaces it there and leaves as 16-byte
// row pieces.  TMEM (512 columns): D1 [0,128) (W part, O part) D2 [128,128+KD)
// S hi|lo [256,256+KD) W hi|lo [384,448) X hi|lo [448,512).
namespace scan_vl {
constexpr int kVD = 128;
constexpr int kLaneWarps = 16;
constexpr int kThreads = 32 * (2 + kLaneWarps);
template <int KD>
struct Geo {
  static constexpr int kNS = KD == 128 ? 2 : 3;     // stages
  static constexpr int kKQ = 0;                     // KD/64 x [Kw 64 rows; Qs 64 rows], 16 KB each
  static constexpr int kK = KD / 64 * 16384;        // KD/64 x K [64 tokens][64 keys], 8 KB each
  static constexpr int kA = kK + KD / 64 * 8192;    // Aqk [64][64]
  static constexpr int kU = kA + 8192;              // 2 x U [64 tokens][64 columns]
  static constexpr int kStage = kU + 16384;
  static constexpr uint32_t kTx = KD / 64 * (16384 + 8192) + 8192 + 16384;
  static constexpr int kNegI = kNS * kStage;        // -I [64][64], the B operand that adds -U
  static constexpr int kGate = kNegI + 8192;        // 16 warps x [16 tokens][32 columns]
  static constexpr int kBar = kGate + kLaneWarps * 1024;
  static constexpr int kSmem = kBar + 256 + 1024;
};
constexpr uint32_t kD1W = 0, kDO = 64, kD2 = 128, kSA = 256, kWA = 384, kXA = 448;

// bf16 hi part of (a, b) and the bf16 rounding of what it leaves
__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 hh = __floats2bfloat162_rn(a, b);
  const float2 hf = __bfloat1622float2(hh);
  hi = *reinterpret_cast<const uint32_t*>(&hh);
  lo = pack_bf16x2(a - hf.x, b - hf.y);
}
}  // namespace scan_vl

template <int KD>
__global__ void __launch_bounds__(scan_vl::kThreads, 1) gdn_scan_vl_kernel(
    const __grid_constant__ CUtensorMap map_kw, const __grid_constant__ CUtensorMap map_qs,
    const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_aqk,
    const __grid_constant__ CUtensorMap map_u, const float* __restrict__ kscale,
    const float* __restrict__ sdecay, const __nv_bfloat16* __restrict__ gate, int64_t sg, int B,
    int T, int H, float* __restrict__ state, __nv_bfloat16* __restrict__ out, int64_t so,
    int32_t* dev_status) {
  using namespace scan_vl;
  using G = Geo<KD>;
  constexpr int VD = kVD, NS = G::kNS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::kBar);
  uint64_t* st_full = bars;         // [NS]
  uint64_t* st_empty = bars + NS;   // [NS]
  uint64_t* s_ready = bars + 2 * NS;
  uint64_t* d1w_full = s_ready + 1;
  uint64_t* w_ready = s_ready + 2;
  uint64_t* d2_full = s_ready + 3;
  uint64_t* o_full = s_ready + 4;
  uint64_t* o_free = s_ready + 5;
  uint64_t* mma_done = s_ready + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_ready + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x % H;
  const int b = blockIdx.x / H;
  const int nC = (T + kC - 1) / kC;
  const int64_t bh = static_cast<int64_t>(b) * H + h;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      sm100::mbar_init(&st_full[i], 1);
      sm100::mbar_init(&st_empty[i], 1);
    }
    sm100::mbar_init(s_ready, kLaneWarps);
    sm100::mbar_init(d1w_full, 1);
    sm100::mbar_init(w_ready, kLaneWarps);
    sm100::mbar_init(d2_full, 1);
    sm100::mbar_init(o_full, 1);
    sm100::mbar_init(o_free, kLaneWarps);
    sm100::mbar_init(mma_done, 1);
    *abort_flag = 0;
    sm100::fence_mbar_init();
    sm100::tma_prefetch_desc(&map_kw);
    sm100::tma_prefetch_desc(&map_qs);
    sm100::tma_prefetch_desc(&map_k);
    sm100::tma_prefetch_desc(&map_aqk);
    sm100::tma_prefetch_desc(&map_u);
  }
  // -I as a 128-byte-swizzled K-major [64][64] bf16 tile (row r: 16-byte piece
  // (c/8) ^ (r%8) holds columns c .. c+7)
  for (int i = threadIdx.x; i < 8192 / 16; i += blockDim.x) {
    const int r = i >> 3, piece = i & 7;
    uint4 z = make_uint4(0, 0, 0, 0);
    if ((piece ^ (r & 7)) == (r >> 3)) {
      uint32_t* zw = reinterpret_cast<uint32_t*>(&z);
      zw[(r & 7) >> 1] = (r & 1) ? 0xBF800000u : 0x0000BF80u;
    }
    *reinterpret_cast<uint4*>(smem + G::kNegI + i * 16) = z;
  }
  sm100::fence_proxy_async_smem();
  if (warp == 1) sm100::tmem_alloc(tmem_slot, 512);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------- TMA
    uint32_t issued = 0;
    for (int c = 0; c < nC; ++c) {
      const int s = c % NS;
      if (!sm100::mbar_wait_warp(&st_empty[s], ((c / NS) & 1) ^ 1u, dev_status, abort_flag))
        break;
      if (lane == 0) {
        uint8_t* st = smem + s * G::kStage;
        const int t0 = c * kC;
        sm100::mbar_arrive_expect_tx(&st_full[s], G::kTx);
#pragma unroll
        for (int x = 0; x < KD / 64; ++x) {
          sm100::tma_load_4d(&map_kw, &st_full[s], st + G::kKQ + x * 16384, x * 64, h, t0, b);
          sm100::tma_load_4d(&map_qs, &st_full[s], st + G::kKQ + x * 16384 + 8192, x * 64, h, t0,
                             b);
          sm100::tma_load_4d(&map_k, &st_full[s], st + G::kK + x * 8192, x * 64, h, t0, b);
        }
        sm100::tma_load_2d(&map_aqk, &st_full[s], st + G::kA, 0,
                           static_cast<int32_t>((bh * nC + c) * kC));
        sm100::tma_load_4d(&map_u, &st_full[s], st + G::kU, 0, h, t0, b);
        sm100::tma_load_4d(&map_u, &st_full[s], st + G::kU + 8192, 64, h, t0, b);
      }
      ++issued;
    }
    // no copy may still be in flight when the CTA exits
    for (uint32_t i = 1; i <= static_cast<uint32_t>(NS); ++i)
      if (issued >= i) {
        const uint32_t c = issued - i;
        sm100::mbar_wait_warp(&st_full[c % NS], (c / NS) & 1, dev_status, nullptr);
      }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA
    constexpr uint32_t id64 = sm100::make_idesc_bf16_f32(128, 64);
    constexpr uint32_t id64_amn = id64 | (1u << 15);  // A (U) MN-major
    constexpr uint32_t idd2 = sm100::make_idesc_bf16_f32(128, KD) | sm100::kIdescBMajorMN;
    const uint32_t tD1W = tmem_base + kD1W, tDO = tmem_base + kDO, tD2 = tmem_base + kD2;
    const uint32_t tSh = tmem_base + kSA, tSl = tSh + KD / 2;
    const uint32_t tWh = tmem_base + kWA, tWl = tWh + 32;
    const uint32_t tXh = tmem_base + kXA, tXl = tXh + 32;
    const uint32_t negi = sm100::smem_u32(smem + G::kNegI);
    constexpr uint32_t id128 = sm100::make_idesc_bf16_f32(128, 128);
    for (int c = 0; c < nC; ++c) {
      const int s = c % NS;
      const uint32_t st = sm100::smem_u32(smem + s * G::kStage);
      // D1 is free once the lane warps have read the previous chunk's O
      if (!sm100::mbar_wait_warp(&st_full[s], (c / NS) & 1, dev_status, abort_flag) ||
          !sm100::mbar_wait_warp(s_ready, c & 1, dev_status, abort_flag) ||
          (c > 0 && !sm100::mbar_wait_warp(o_free, (c - 1) & 1, dev_status, abort_flag)))
        break;
      sm100::tc_fence_after();
      if (lane == 0) {
        // D1 = S^T [Kw; Qs]^T (K steps of 16 keys: 8 packed columns of S), then
        // columns 0-63 -= U^T
#pragma unroll
        for (int kk = 0; kk < KD / 16; ++kk) {
          const uint64_t bkq =
              sm100::make_sw128_kmajor_desc(st + G::kKQ + (kk >> 2) * 16384 + (kk & 3) * 32);
          sm100::umma_bf16_ts(tD1W, tSh + kk * 8, bkq, id128, kk != 0 ? 1u : 0u);
          sm100::umma_bf16_ts(tD1W, tSl + kk * 8, bkq, id128, 1u);
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          sm100::umma_bf16_ss(tD1W, sm100::make_sw128_desc(st + G::kU + kk * 2048, 8192, 1024),
                              sm100::make_sw128_kmajor_desc(negi + kk * 32), id64_amn, 1u);
        sm100::umma_commit(d1w_full);
      }
      __syncwarp();
      if (!sm100::mbar_wait_warp(w_ready, c & 1, dev_status, abort_flag)) break;
      sm100::tc_fence_after();
      if (lane == 0) {
        // D2 = X^T K: K steps of 16 tokens; B = K read MN-major (64-key blocks 8 KB apart)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t bk = sm100::make_sw128_desc(st + G::kK + kk * 2048, 8192, 1024);
          sm100::umma_bf16_ts(tD2, tXh + kk * 8, bk, idd2, kk != 0 ? 1u : 0u);
          sm100::umma_bf16_ts(tD2, tXl + kk * 8, bk, idd2, 1u);
        }
        sm100::umma_commit(d2_full);
        // O part += W^T Aqk^T
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ba = sm100::make_sw128_kmajor_desc(st + G::kA + kk * 32);
          sm100::umma_bf16_ts(tDO, tWh + kk * 8, ba, id64, 1u);
          sm100::umma_bf16_ts(tDO, tWl + kk * 8, ba, id64, 1u);
        }
        sm100::umma_commit(o_full);
        sm100::umma_commit(&st_empty[s]);
      }
      __syncwarp();
    }
    if (lane == 0) sm100::umma_commit(mma_done);
    __syncwarp();
    sm100::mbar_wait_warp(mma_done, 0, dev_status, nullptr);
  } else {
    // ------------------------------------------------------- lane warps
    constexpr int KH = KD / 4;  // keys of S held per thread
    const int q = warp & 3;
    const int r = (warp - 2) >> 2;
    const int v = 32 * q + lane;
    const int key0 = KH * r;
    const uint32_t tl = tmem_base + (static_cast<uint32_t>(32 * q) << 16);
    uint8_t* gtile = smem + G::kGate + (warp - 2) * 1024;  // gate, then the output [16][32]
    const int pr = lane >> 2, pc = lane & 3;                 // 16-byte piece: token pr + 8u
    float S[KH];
    float* Sg = state + (bh * KD + key0) * VD + v;
#pragma unroll
    for (int i = 0; i < KH; ++i) S[i] = Sg[static_cast<int64_t>(i) * VD];

    auto store_s = [&]() {
#pragma unroll
      for (int part = 0; part < KH / 16; ++part) {
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          split_pair(S[16 * part + 2 * j], S[16 * part + 2 * j + 1], hi[j], lo[j]);
        sm100::tmem_st_32x32b_x8(tl + kSA + KH / 2 * r + 8 * part, hi);
        sm100::tmem_st_32x32b_x8(tl + kSA + KD / 2 + KH / 2 * r + 8 * part, lo);
      }
    };
    store_s();
    sm100::tmem_st_wait();
    sm100::tc_fence_before();
    __syncwarp();
    if (lane == 0) sm100::mbar_arrive(s_ready);

    // the lane's two 16-byte pieces of a chunk's gate tile, copied by
    // cp.async one chunk ahead (zero past T)
    auto load_gate = [&](int c) {
      const int tw = c * kC + 16 * r;
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int t = tw + pr + 8 * u;
        const bool ok = c < nC && t < T;
        const int64_t row = static_cast<int64_t>(b) * T + (ok ? t : 0);
        mma::cp_async16(gtile + (pr + 8 * u) * 64 + pc * 16,
                        gate + row * sg + h * VD + 32 * q + 8 * pc, ok);
      }
      mma::cp_async_commit();
    };
    load_gate(0);
    // kscale of the warp's 16 tokens (lane j < 16: token 16r + j) and the
    // chunk decay, one chunk ahead
    auto ks_at = [&](int c) {
      const int t = c * kC + 16 * r + (lane & 15);
      return (c < nC && t < T) ? __ldg(kscale + bh * T + t) : 0.f;
    };
    float ks_pre = ks_at(0), sd_pre = __ldg(sdecay + bh * nC);
    for (int c = 0; c < nC; ++c) {
      const int t0 = c * kC;
      const int n = min(kC, T - t0);
      const float ks_c = ks_pre, sd_c = sd_pre;
      ks_pre = ks_at(c + 1);
      sd_pre = c + 1 < nC ? __ldg(sdecay + bh * nC + c + 1) : 0.f;

      // ---- W = -D1W and X = ks W for tokens 16r .. 16r+15
      if (!sm100::mbar_wait_warp(d1w_full, c & 1, dev_status, abort_flag)) break;
      sm100::tc_fence_after();
      {
        uint32_t p[16];
        sm100::tmem_ld_32x32b_x16(tl + kD1W + 16 * r, p);
        sm100::tmem_ld_wait();
        sm100::tmem_regs_ready(p);
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          split_pair(-__uint_as_float(p[2 * j]), -__uint_as_float(p[2 * j + 1]), hi[j], lo[j]);
        sm100::tmem_st_32x32b_x8(tl + kWA + 8 * r, hi);
        sm100::tmem_st_32x32b_x8(tl + kWA + 32 + 8 * r, lo);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float k0 = __shfl_sync(0xffffffffu, ks_c, 2 * j);
          const float k1 = __shfl_sync(0xffffffffu, ks_c, 2 * j + 1);
          split_pair(-k0 * __uint_as_float(p[2 * j]), -k1 * __uint_as_float(p[2 * j + 1]), hi[j],
                     lo[j]);
        }
        sm100::tmem_st_32x32b_x8(tl + kXA + 8 * r, hi);
        sm100::tmem_st_32x32b_x8(tl + kXA + 32 + 8 * r, lo);
      }
      sm100::tmem_st_wait();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(w_ready);

      // ---- S <- sd S + D2 for keys key0 .. key0+KH-1
      if (!sm100::mbar_wait_warp(d2_full, c & 1, dev_status, abort_flag)) break;
      sm100::tc_fence_after();
#pragma unroll
      for (int part = 0; part < KH / 16; ++part) {
        uint32_t d[16];
        sm100::tmem_ld_32x32b_x16(tl + kD2 + key0 + 16 * part, d);
        sm100::tmem_ld_wait();
        sm100::tmem_regs_ready(d);
#pragma unroll
        for (int j = 0; j < 16; ++j)
          S[16 * part + j] = sd_c * S[16 * part + j] + __uint_as_float(d[j]);
      }
      if (c + 1 < nC) store_s();
      sm100::tmem_st_wait();
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(s_ready);

      // ---- O = DO^T for tokens 16r .. 16r+15, times the gate; the product
      // replaces the gate in its tile and leaves as 16-byte row pieces
      if (!sm100::mbar_wait_warp(o_full, c & 1, dev_status, abort_flag)) break;
      sm100::tc_fence_after();
      uint32_t o[16];
      sm100::tmem_ld_32x32b_x16(tl + kDO + 16 * r, o);
      sm100::tmem_ld_wait();
      sm100::tmem_regs_ready(o);
      sm100::tc_fence_before();
      __syncwarp();
      if (lane == 0) sm100::mbar_arrive(o_free);
      mma::cp_async_wait<0>();  // this chunk's gate
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        __nv_bfloat16* g0 = reinterpret_cast<__nv_bfloat16*>(gtile + (2 * j) * 64 + lane * 2);
        __nv_bfloat16* g1 = g0 + 32;
        // reference order: out.to(hidden dtype) * gate, one rounding each
        const __nv_bfloat162 ob =
            __floats2bfloat162_rn(__uint_as_float(o[2 * j]), __uint_as_float(o[2 * j + 1]));
        const __nv_bfloat162 pg = __hmul2(ob, __halves2bfloat162(*g0, *g1));
        *g0 = __low2bfloat16(pg);
        *g1 = __high2bfloat16(pg);
      }
      __syncwarp();
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int t = 16 * r + pr + 8 * u;
        if (t < n) {
          const int64_t row = static_cast<int64_t>(b) * T + t0 + t;
          *reinterpret_cast<uint4*>(out + row * so + h * VD + 32 * q + 8 * pc) =
              *reinterpret_cast<const uint4*>(gtile + (pr + 8 * u) * 64 + pc * 16);
        }
      }
      __syncwarp();
      load_gate(c + 1);
    }
    mma::cp_async_wait<0>();  // nothing in flight into shared memory at exit
#pragma unroll
    for (int i = 0; i < KH; ++i) Sg[static_cast<int64_t>(i) * VD] = S[i];
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem_base, 512);
  }
}

int32_t check_io(const GdnIO& io, int KD, int VD) {
  if (!io.q || !io.k || !io.v || !io.gate || !io.beta) return LLMYB_EINVAL;
  if (!io.decay_logit && !io.log_alpha) return LLMYB_EINVAL;
  if (!((KD == 64 || KD == 128) && (VD == 64 || VD == 128))) return LLMYB_EUNSUPPORTED;
  return LLMYB_OK;
}

GdnIO make_io(const void* q, int64_t sq, const void* k, int64_t sk, const void* v, int64_t sv,
              const void* gate, int64_t sg, const void* beta, int64_t sb,
              const float* decay_logit, const float* log_alpha, const uint8_t* reset) {
  GdnIO io;
  io.q = static_cast<const __nv_bfloat16*>(q);
  io.k = static_cast<const __nv_bfloat16*>(k);
  io.v = static_cast<const __nv_bfloat16*>(v);
  io.gate = static_cast<const __nv_bfloat16*>(gate);
  io.beta = static_cast<const __nv_bfloat16*>(beta);
  io.sq = sq; io.sk = sk; io.sv = sv; io.sg = sg; io.sb = sb;
  io.decay_logit = decay_logit;
  io.log_alpha = log_alpha;
  io.reset = reset;
  io.beta_bias = nullptr;
  io.raw = 0;
  return io;
}

struct ScratchLayout {
  int64_t u, kw, aqk, qs, ks, sd, qsq, total;
};

ScratchLayout scratch_layout(int B, int T, int H, int KD, int VD) {
  auto al = [](int64_t x) { return (x + 255) / 256 * 256; };
  const int64_t nC = ceil_div(T, kC);
  const int64_t bt = static_cast<int64_t>(B) * T;
  ScratchLayout s;
  s.u = 0;
  s.kw = s.u + al(bt * H * VD * 2);
  s.aqk = s.kw + al(bt * H * KD * 2);
  s.qs = s.aqk + al(static_cast<int64_t>(B) * H * nC * kC * kC * 2);
  s.ks = s.qs + al(bt * H * 4);
  s.sd = s.ks + al(bt * H * 4);
  s.qsq = s.sd + al(static_cast<int64_t>(B) * H * nC * 4);
  // the scaled q of the tcgen05 scan
  s.total = s.qsq + ((KD == 64 || KD == 128) && VD % 64 == 0 ? al(bt * H * KD * 2) : 0);
  return s;
}

// the tcgen05 scan's operand and alignment requirements (else the mma.sync scan)
bool scan_tc_ok(const GdnIO& io, int KD, int VD, const void* state, const void* out,
                int64_t so) {
  const auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return (KD == 64 || KD == 128) && VD % scan_tc::kVS == 0 && io.sg % 8 == 0 && so % 8 == 0 &&
         io.sk % 8 == 0 &&
         a16(io.gate) && a16(out) && a16(state) && a16(io.k);
}

template <int KD, int VD>
int32_t launch_prefill(const GdnIO& io, int B, int T, int H, void* scratch, float* state,
                       __nv_bfloat16* out, int64_t so, int32_t* dev_status, cudaStream_t s) {
  const ScratchLayout L = scratch_layout(B, T, H, KD, VD);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  PrepOut po;
  po.U = reinterpret_cast<__nv_bfloat16*>(base + L.u);
  po.Kw = reinterpret_cast<__nv_bfloat16*>(base + L.kw);
  po.Aqk = reinterpret_cast<__nv_bfloat16*>(base + L.aqk);
  po.qscale = reinterpret_cast<float*>(base + L.qs);
  po.kscale = reinterpret_cast<float*>(base + L.ks);
  po.sdecay = reinterpret_cast<float*>(base + L.sd);
  const bool tc = scan_tc_ok(io, KD, VD, state, out, so) && L.total > L.qsq;
  po.Qs = tc ? reinterpret_cast<__nv_bfloat16*>(base + L.qsq) : nullptr;
  const int nC = static_cast<int>(ceil_div(T, kC));
  constexpr int kPrepSmem = sizeof(PrepSmem<KD, VD>);
  constexpr int VC = 32, NG = 2;  // two 32-column groups per CTA
  constexpr int kScanSmem = sizeof(ScanSmem<KD, VC * NG>);
  {
    int32_t st = ensure_smem(gdn_chunk_prep_kernel<KD, VD>, kPrepSmem);
    if (st) return st;
    st = ensure_smem(gdn_chunk_scan_kernel<KD, VD, VC, NG>, kScanSmem);
    if (st) return st;
  }
  gdn_chunk_prep_kernel<KD, VD><<<B * H * nC, 128, kPrepSmem, s>>>(io, B, T, H, po);
  count_launch();
  if (tc) {
    {
      int32_t st = ensure_smem(gdn_scan_tc_kernel, scan_tc::kSmem);
      if (st) return st;
    }
    CUtensorMap mkw, mqs, mk, maqk, mu;
    if (!make_bf16_4d_map(&mkw, po.Kw, B, T, H, KD, kC) ||
        !make_bf16_4d_map(&mqs, po.Qs, B, T, H, KD, kC) ||
        !make_bf16_4d_map_ld(&mk, io.k, B, T, H, KD, io.sk, kC) ||
        !make_bf16_2d_map(&maqk, po.Aqk, static_cast<uint64_t>(B) * H * nC * kC, kC, kC, kC, kC) ||
        !make_bf16_4d_map(&mu, po.U, B, T, H, VD, kC))
      return LLMYB_EUNSUPPORTED;
    // the value-lane kernel (one CTA per row and head) once the 64-column
    // kernel (two CTAs per row and head) would need more than one wave
    if (VD == scan_vl::kVD && 2 * B * H > num_sms()) {
      constexpr int kVlSmem = scan_vl::Geo<KD>::kSmem;
      int32_t st = ensure_smem(gdn_scan_vl_kernel<KD>, kVlSmem);
      if (st) return st;
      gdn_scan_vl_kernel<KD><<<B * H, scan_vl::kThreads, kVlSmem, s>>>(
          mkw, mqs, mk, maqk, mu, po.kscale, po.sdecay, io.gate, io.sg, B, T, H, state, out, so,
          dev_status);
    } else {
      gdn_scan_tc_kernel<<<B * H * (VD / scan_tc::kVS), 320, scan_tc::kSmem, s>>>(
          mkw, mqs, mk, maqk, mu, po.kscale, po.sdecay, io.gate, io.sg, B, T, H, KD, VD, state,
          out, so, dev_status);
    }
    count_launch();
    return launch_status();
  }
  gdn_chunk_scan_kernel<KD, VD, VC, NG><<<B * H * (VD / (VC * NG)), 128 * NG, kScanSmem, s>>>(
      io, B, T, H, po, state, out, so);
  count_launch();
  return launch_status();
}

}  // namespace
}  // namespace llmyb

using namespace llmyb;

LLMYB_API int32_t llmyb_gdn_activate(void* proj, int64_t n_tokens, int32_t width, int32_t heads,
                                     int32_t key_dim, int32_t value_dim, const float* beta_bias,
                                     void* stream) {
  if (!proj || n_tokens < 0 || heads <= 0 || key_dim <= 0 || value_dim <= 0) return LLMYB_EINVAL;
  if (width < 2 * heads * (key_dim + value_dim) + heads) return LLMYB_EINVAL;
  if (n_tokens == 0) return LLMYB_OK;
  const int kp = key_dim / 8;
  const int64_t n_norm = n_tokens * 2 * heads * static_cast<int64_t>(kp);
  const int64_t n_gate = n_tokens * heads * static_cast<int64_t>(value_dim) / 8;
  if (width % 8 == 0 && key_dim % 8 == 0 && value_dim % 8 == 0 && kp <= 32 &&
      (kp & (kp - 1)) == 0 && (reinterpret_cast<uintptr_t>(proj) & 15u) == 0 &&
      n_norm + n_gate < (int64_t{1} << 31)) {
    gdn_activate_vec_kernel<<<static_cast<int>(ceil_div(n_norm + n_gate, 256)), 256, 0,
                              static_cast<cudaStream_t>(stream)>>>(
        static_cast<__nv_bfloat16*>(proj), static_cast<uint32_t>(n_norm),
        static_cast<uint32_t>(n_gate), width, heads, key_dim, value_dim, beta_bias);
    count_launch();
    return launch_status();
  }
  const int64_t warps = n_tokens * heads;
  gdn_activate_kernel<<<static_cast<int>(ceil_div(warps * 32, 256)), 256, 0,
                        static_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(proj), n_tokens, width, heads, key_dim, value_dim, beta_bias);
  count_launch();
  return launch_status();
}

// One decode token per row: state [B,H,K,V] fp32 updated in place.  With
// raw_inputs the q/k/gate/beta operands are the raw projections and the
// kernel applies the activations of llmyb_gdn_activate itself.
LLMYB_API int32_t llmyb_gdn_step(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                                 const void* v, int64_t v_stride, const void* gate,
                                 int64_t gate_stride, const void* beta, int64_t beta_stride,
                                 const float* decay_logit, const float* log_alpha,
                                 const uint8_t* reset, int32_t batch, int32_t heads,
                                 int32_t key_dim, int32_t value_dim, float* state, void* out,
                                 int64_t out_stride, int32_t raw_inputs, const float* beta_bias,
                                 void* stream) {
  GdnIO io = make_io(q, q_stride, k, k_stride, v, v_stride, gate, gate_stride, beta,
                     beta_stride, decay_logit, log_alpha, reset);
  io.raw = raw_inputs ? 1 : 0;
  io.beta_bias = beta_bias;
  int32_t st = check_io(io, key_dim, value_dim);
  if (st) return st;
  if (!state || !out || batch < 0 || heads <= 0) return LLMYB_EINVAL;
  if (batch == 0) return LLMYB_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = batch * heads * (value_dim / 32);
  auto* o = static_cast<__nv_bfloat16*>(out);
  if (key_dim == 64)
    st = launch_pdl(gdn_step_kernel<64>, dim3(grid), dim3(128), 0, s, io, heads, value_dim, state,
                    o, out_stride);
  else
    st = launch_pdl(gdn_step_kernel<128>, dim3(grid), dim3(128), 0, s, io, heads, value_dim, state,
                    o, out_stride);
  if (st) return st;
  count_launch();
  return launch_status();
}

LLMYB_API int64_t llmyb_gdn_prefill_scratch_bytes(int32_t batch, int32_t seq, int32_t heads,
                                                  int32_t key_dim, int32_t value_dim) {
  if (batch < 0 || seq < 0 || heads <= 0 || key_dim <= 0 || value_dim <= 0) return -1;
  return scratch_layout(batch, seq, heads, key_dim, value_dim).total;
}

// Chunked scan over [B, T] tokens (token index b*T + t): state [B,H,K,V] fp32
// is read as the initial state and overwritten with the final state.
LLMYB_API int32_t llmyb_gdn_prefill(const void* q, int64_t q_stride, const void* k,
                                    int64_t k_stride, const void* v, int64_t v_stride,
                                    const void* gate, int64_t gate_stride, const void* beta,
                                    int64_t beta_stride, const float* decay_logit,
                                    const float* log_alpha, const uint8_t* reset, int32_t batch,
                                    int32_t seq, int32_t heads, int32_t key_dim,
                                    int32_t value_dim, float* state, void* out,
                                    int64_t out_stride, void* scratch, int32_t* dev_status,
                                    void* stream) {
  const GdnIO io = make_io(q, q_stride, k, k_stride, v, v_stride, gate, gate_stride, beta,
                           beta_stride, decay_logit, log_alpha, reset);
  int32_t st = check_io(io, key_dim, value_dim);
  if (st) return st;
  if (!state || !out || !scratch || batch < 0 || seq < 0 || heads <= 0) return LLMYB_EINVAL;
  if (batch == 0 || seq == 0) return LLMYB_OK;
  if ((q_stride | k_stride | v_stride) % 8 != 0) return LLMYB_EUNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
       reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(scratch)) & 15u)
    return LLMYB_EUNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* o = static_cast<__nv_bfloat16*>(out);
  if (key_dim == 64 && value_dim == 64)
    return launch_prefill<64, 64>(io, batch, seq, heads, scratch, state, o, out_stride, dev_status, s);
  if (key_dim == 128 && value_dim == 128)
    return launch_prefill<128, 128>(io, batch, seq, heads, scratch, state, o, out_stride, dev_status, s);
  if (key_dim == 64 && value_dim == 128)
    return launch_prefill<64, 128>(io, batch, seq, heads, scratch, state, o, out_stride, dev_status, s);
  return launch_prefill<128, 64>(io, batch, seq, heads, scratch, state, o, out_stride, dev_status, s);
}

// history [B, 3, D] = the last three rows of x [B, T, D] per batch row, zero
// rows where the prompt is shorter (model/model.py:180-182).
LLMYB_API int32_t llmyb_gdn_history_set(const void* x, void* history, int32_t batch, int32_t seq,
                                        int32_t d_model, void* stream) {
  if (!x || !history || batch < 0 || seq < 0 || d_model <= 0) return LLMYB_EINVAL;
  if (batch == 0) return LLMYB_OK;
  const bool vec = d_model % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(history) & 15u) == 0;
  const auto* xp = static_cast<const __nv_bfloat16*>(x);
  auto* hp = static_cast<__nv_bfloat16*>(history);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (vec)
    gdn_history_set_kernel<true><<<batch, 128, 0, s>>>(xp, hp, seq, d_model);
  else
    gdn_history_set_kernel<false><<<batch, 128, 0, s>>>(xp, hp, seq, d_model);
  count_launch();
  return launch_status();
}

// Conv gate + (optional) residual add + (optional) history roll; see
// gdn_conv_gate_kernel.  x, y_proj, out, residual: [B*T, D] bf16; conv_w
// [D, 4] fp32; history [B, 3, D] bf16 or null.
LLMYB_API int32_t llmyb_gdn_conv_gate(const void* x, const void* y_proj, const float* conv_w,
                                      void* history, const uint8_t* reset, int32_t batch,
                                      int32_t seq, int32_t d_model, void* out, void* residual,
                                      int32_t roll_history, void* stream) {
  if (!x || !y_proj || !conv_w || batch < 0 || seq < 0 || d_model <= 0) return LLMYB_EINVAL;
  if (!out && !residual) return LLMYB_EINVAL;
  if (roll_history && !history) return LLMYB_EINVAL;
  if (batch == 0 || seq == 0) return LLMYB_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t total = static_cast<int64_t>(batch) * seq * d_model;
  void* dst = residual ? residual : out;
  if (!history && d_model % 8 == 0 &&
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y_proj) |
        reinterpret_cast<uintptr_t>(conv_w) | reinterpret_cast<uintptr_t>(dst)) & 15u) == 0 &&
      total / 8 < (int64_t{1} << 30)) {
    // runs long enough to amortise the three warm-up rows, short enough to
    // leave a few thousand threads per SM
    const int64_t pieces = total / 8;
    int run = 1;
    while (run < 16 && pieces / (2 * run) >= static_cast<int64_t>(num_sms()) * 2048) run *= 2;
    const int64_t threads = static_cast<int64_t>(batch) * ceil_div(seq, run) * (d_model / 8);
    gdn_conv_gate_run_kernel<<<static_cast<int>(ceil_div(threads, 256)), 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(y_proj), conv_w,
        reset, batch, seq, d_model, run, static_cast<__nv_bfloat16*>(dst), residual ? 1 : 0);
    count_launch();
    return launch_status();
  }
  const int grid = static_cast<int>(std::min<int64_t>(ceil_div(total, 256), 148 * 16));
  gdn_conv_gate_kernel<<<grid, 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(y_proj), conv_w,
      static_cast<__nv_bfloat16*>(history), reset, batch, seq, d_model,
      static_cast<__nv_bfloat16*>(out), static_cast<__nv_bfloat16*>(residual),
      (roll_history && seq == 1) ? 1 : 0);
  count_launch();
  if (roll_history && seq != 1) {
    gdn_conv_roll_kernel<<<batch, 256, 3 * d_model * sizeof(__nv_bfloat16), s>>>(
        static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(history), seq, d_model);
    count_launch();
  }
  return launch_status();
}
