// Batch-1 decode step of the looped hybrid stack as one persistent,
// cooperative launch (reference: LoopedHybridMoEForCausalLM.decode_step,
// model/model.py:787-915, with the loop output carried as in
// sample_standalone.py; PhysicalBlock.forward_step :266-376; the head
// :913-915).
//
// A batch-1 step is ~0.4 GB of weight and cache reads spread over 24 block
// applications, each a chain of small dependent products.  As separate
// kernels it is bound by the ~5 us each dependent launch costs.  Here one
// 512-thread CTA per SM walks the whole step; the phases of a block are
// separated by grid barriers (one atomic per CTA, a bounded spin), and every
// phase loads its own weight rows into registers BEFORE it waits on the
// barrier, so the weight stream overlaps the barrier and the previous phase.
//
// Per block (x = residual row, fp32; y = the previous block's routed rows):
//   A   x += sum_s y[s]; normed = RMSNorm(x) mixer_norm; proj = W_in normed
//   CSA M1  key-chunk CTAs: scores of the new query against the window's keys
//           (warp per key, per-head dots by lane groups), per-chunk head max /
//           exp-sum; the CTA holding the new slot writes its key and value
//       M2  column CTAs: head-averaged probabilities p_j = mean_h softmax_h,
//           out[cols] = sum_j p_j v'_j where the ring holds v' = W_o W_v x, so
//           out IS the block output (csa.py:132 out(local_out(.)) folded into
//           the values); x[cols] += bf16(out); router partial sums
//   GDN M   (head, 32-column) CTAs: the delta-rule step (gated_deltanet.py
//           :140-149) with in-kernel activation, state in registers
//       C   warp per output column: W_out row . o, conv gate (history roll),
//           x[col] += bf16(.), router partial sums
//   E1  every CTA reduces the partial sums (fixed order), normalises, takes
//       the top-k + softmax (value desc, index asc) and m = RMSNorm(x) ffn_norm;
//       warp per expert feature: h = silu(g . m) * (u . m)
//   E2  warp per (route, column): y[s, col] = p_s * (w2 row . h[s])
// Head: x += sum_s y[s]; collapse GEMV; RMSNorm; LM head GEMV (fp32 logits of
// the bf16 products, as torch's bf16 GEMM followed by .float()).
//
// Cross-CTA data goes through global memory with L2-only loads/stores
// (ld.cg / st.cg) so no SM reads a stale L1 line after a barrier.
#include "common.cuh"
#include "../../include/llmyb.h"

namespace llmyb {
namespace {

constexpr int kPT = 512;                // threads per CTA
constexpr int kPW = kPT / 32;           // warps per CTA
constexpr int kMaxD = 1024;
constexpr int kDC = kMaxD / 256;        // 16-byte chunks per lane of a row of <= 1024
constexpr int kMaxF = 2048;
constexpr int kFC = kMaxF / 256;
constexpr int kMaxE = 64, kMaxK = 8;
constexpr int kMaxW = 1024, kMaxHeads = 16;
constexpr int kVecBytes = kMaxK * kMaxF * 2;  // largest shared bf16 vector (h of all routes)

using bf16 = __nv_bfloat16;

__device__ __forceinline__ uint4 ldcg16(const void* p) {
  return __ldcg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void stcg16(void* p, uint4 v) {
  __stcg(reinterpret_cast<uint4*>(p), v);
}
__device__ __forceinline__ float ldcg_bf(const bf16* p) {
  const unsigned short u = __ldcg(reinterpret_cast<const unsigned short*>(p));
  return __uint_as_float(static_cast<uint32_t>(u) << 16);
}
__device__ __forceinline__ void stcg_bf(bf16* p, float v) {
  const bf16 b = f2bf(v);
  __stcg(reinterpret_cast<unsigned short*>(p), *reinterpret_cast<const unsigned short*>(&b));
}
// 16-byte asynchronous copy global -> shared (L2 only): a prefetch issued
// before a barrier wait that holds no registers while it is in flight
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// wait until at most N of this thread's most recent commit groups are pending
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Row of n8 16-byte chunks into registers: lane holds chunks lane + 32 i.
template <int NC>
__device__ __forceinline__ void load_row(const bf16* __restrict__ row, int n8, int lane,
                                         uint4 (&w)[NC]) {
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = lane + 32 * i;
    if (c < n8) w[i] = __ldg(reinterpret_cast<const uint4*>(row) + c);
  }
}

__device__ __forceinline__ float dot8(uint4 a, uint4 b) {
  const uint32_t aa[4] = {a.x, a.y, a.z, a.w};
  const uint32_t bb[4] = {b.x, b.y, b.z, b.w};
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 x = unpack_bf16x2(aa[e]);
    const float2 y = unpack_bf16x2(bb[e]);
    s += x.x * y.x + x.y * y.y;
  }
  return s;
}

// Warp dot of a register row with a bf16 vector in shared memory.
template <int NC>
__device__ __forceinline__ float row_dot(const uint4 (&w)[NC], const bf16* s_vec, int n8,
                                         int lane) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = lane + 32 * i;
    if (c < n8) s += dot8(w[i], reinterpret_cast<const uint4*>(s_vec)[c]);
  }
  return warp_sum(s);
}

// A row of n8 16-byte chunks copied into shared memory by the warp (lane c,
// c + 32, ...), and its dot with a bf16 vector in shared memory.
__device__ __forceinline__ void warp_copy_row(bf16* srow, const bf16* grow, int n8, int lane) {
  for (int c = lane; c < n8; c += 32) cp_async16(srow + c * 8, grow + c * 8);
}
__device__ __forceinline__ float srow_dot(const bf16* srow, const bf16* s_vec, int n8, int lane) {
  float s = 0.f;
  for (int c = lane; c < n8; c += 32)
    s += dot8(reinterpret_cast<const uint4*>(srow)[c], reinterpret_cast<const uint4*>(s_vec)[c]);
  return warp_sum(s);
}

__device__ __forceinline__ float block_sum(float v, float* s_red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kPW; ++i) t += s_red[i];
  return t;
}

// Grid barrier: arrive (after the CTA's writes) and wait (before reading
// other CTAs' writes) are separate so that loads independent of the previous
// phase can be issued in between.  The wait is bounded: after one second it
// records LLMYB_ETIMEOUT, raises the abort flag and every CTA returns.
struct GridBar {
  uint32_t* bar;
  int32_t* status;
  uint32_t target;
  uint64_t* trace;  // per traced CTA: [wait end | arrive][512]
  int n_arrive, n_wait;
  __device__ __forceinline__ void stamp(int kind, int i) {
    if (trace != nullptr && i < 512)
      trace[kind * 512 + i] = globaltimer_ns();
  }
  // points inside a phase (thread 0 of a traced CTA; debugging only)
  __device__ __forceinline__ void point(int block_app, int k) {
    if (trace != nullptr && threadIdx.x == 0) trace[2048 + (block_app * 8 + k)] = globaltimer_ns();
  }
  // The CTA barrier orders every thread's writes before thread 0's release
  // reduction; waiters acquire the counter (the pattern of a release /
  // acquire grid barrier: no full fence on either side).
  __device__ __forceinline__ void arrive() {
    __syncthreads();
    if (threadIdx.x == 0) {
      stamp(1, n_arrive);
      asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(bar), "r"(1u) : "memory");
    }
    ++n_arrive;
    target += gridDim.x;
  }
  // false: the step was abandoned (a barrier timed out somewhere)
  __device__ __forceinline__ bool wait() {
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
      const uint64_t t0 = globaltimer_ns();
      uint32_t spins = 0;
      int ok = 1;
      for (;;) {
        const uint32_t v = ld_acquire_gpu(bar);
        if (v >= target && v < 0x80000000u) break;
        if (v >= 0x80000000u) { ok = 0; break; }  // aborted by another CTA
        if (((++spins) & 255u) == 0u && globaltimer_ns() - t0 > kWaitLimitNs) {
          report_status(status, LLMYB_ETIMEOUT);
          atomicOr(bar, 0x80000000u);
          ok = 0;
          break;
        }
      }
      stamp(0, n_wait);
      s_ok = ok;
    }
    ++n_wait;
    __syncthreads();
    return s_ok != 0;
  }
};

struct Smem {
  float red[kPW];
  float xrow[kMaxD];                 // residual row (fp32)
  float q[kMaxD];                    // scaled query (CSA) / q, k (GDN)
  float kk[128];
  float sc[kMaxHeads][kPW];          // scores of the CTA's keys
  float hM[kMaxHeads], hInvL[kMaxHeads];
  float part[kPW][2 + kMaxE];        // per-warp router partial sums
  float vred[kPW][8];
  float gred[4][32];
  float logit[kMaxE];
  float prob[kMaxK];
  int idx[kMaxK];
  float scal[4];
  float ptmp[128 * (2 + kMaxE)];     // router partial sums of all producing CTAs
  uint4 vring[kMaxW];                // CSA: this CTA's 8 columns of every cached value;
                                     // GDN: the unit's state slice [64][32] fp32
  bf16 wbuf[kPW][2 * kMaxD];         // per warp: input-projection / expert-down / collapse rows
  bf16 kbuf[kPW][kMaxD];             // per warp: CSA key row / GDN output-projection row
};

// DC / FC: 16-byte chunks per lane of a D-long / F-long weight row (D <= 256 DC,
// F <= 256 FC), so the register arrays are sized for the model.
template <int DC, int FC>
__global__ void __launch_bounds__(kPT, 1) decode_persistent_kernel(const llmyb_pdecode p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  bf16* s_vec = reinterpret_cast<bf16*>(smem_raw);                     // [kVecBytes / 2]
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw + kVecBytes);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cta = blockIdx.x, G = gridDim.x;
  const int gw = cta * kPW + warp, NW = G * kPW;
  const int D = p.d_model, n8 = D >> 3;
  const int E = p.n_experts, K = p.top_k, F = p.ffn, NV = 2 + E;
  const float eps = p.eps;
  uint64_t* trace = nullptr;
  if (p.trace != nullptr && (blockIdx.x == 0 || blockIdx.x == gridDim.x - 1))
    trace = p.trace + (blockIdx.x == 0 ? 0 : 1024);
  GridBar gb{p.bar, p.status, 0, trace, 0, 0};
  // inputs that index memory are clamped into range (an out-of-range token
  // or position is recorded as LLMYB_EINVAL and computes garbage, not a fault)
  const int pos_in = __ldcg(p.positions);
  const int64_t tok_in = __ldcg(p.token);
  const int pos = max(pos_in, 0);
  const int64_t tok = tok_in < 0 ? 0 : (tok_in >= p.vocab ? p.vocab - 1 : tok_in);
  if ((pos != pos_in || tok != tok_in) && blockIdx.x == 0 && threadIdx.x == 0)
    report_status(p.status, LLMYB_EINVAL);
  const bf16* embed = static_cast<const bf16*>(p.embed);
  bf16* proj = static_cast<bf16*>(p.proj);
  bf16* normed_g = static_cast<bf16*>(p.normed);
  bf16* mix = static_cast<bf16*>(p.mix);
  bf16* hbuf = static_cast<bf16*>(p.hbuf);
  bf16* ybuf = static_cast<bf16*>(p.ybuf);
  // CSA geometry
  const int Hc = p.csa_heads, Dh = p.csa_head_dim, HDc = Hc * Dh, W = p.window;
  const int nk = min(pos + 1, W);          // keys in the window (this token included)
  const int slot = pos % W;                // ring slot of this token
  const int nk1 = (nk + kPW - 1) / kPW;    // key-chunk CTAs (one key per warp)
  const int ncs = n8;                      // column CTAs (8 columns each)
  const float qscale = 1.4426950408889634f / sqrtf(static_cast<float>(Dh));
  // GDN geometry
  const int Hg = p.gdn_heads, Kg = p.gdn_dim, HKg = Hg * Kg;
  const int gunits = Hg * (Kg / 32);       // (head, 32-column slice) CTAs
  int xs = 0;                              // residual buffer the next block reads
  bool have_y = false;                     // routed rows of the previous block pending
  bool first = true;

  for (int li = 0; li < p.n_loops; ++li) {
    for (int j = 0; j < p.n_blocks; ++j) {
      const llmyb_pblock& B = p.blocks[j];
      const llmyb_player& L = p.layers[li * p.n_blocks + j];
      const bf16* w_in = static_cast<const bf16*>(B.w_in);
      float* xsrc = p.x + xs * D;
      float* xdst = p.x + (xs ^ 1) * D;
      // ================================================================ A
      {
        // asynchronous copies into shared memory before the wait, in three
        // commit groups: this phase's rows; the next phase's rows (CSA key row,
        // GDN output-projection row); the CSA value chunks / the GDN state slice
        const int r0 = gw, r1 = gw + NW;
        bf16* wb = sm.wbuf[warp];
        if (r0 < B.rows) warp_copy_row(wb, w_in + static_cast<int64_t>(r0) * D, n8, lane);
        if (r1 < B.rows) warp_copy_row(wb + kMaxD, w_in + static_cast<int64_t>(r1) * D, n8, lane);
        cp_async_commit();
        if (B.kind == 0) {
          const int key = cta * kPW + warp;
          if (cta < nk1 && key < nk && key != slot)
            warp_copy_row(sm.kbuf[warp], static_cast<const bf16*>(L.ring_k) + static_cast<int64_t>(key) * HDc,
                          HDc >> 3, lane);
          cp_async_commit();
          if (cta < ncs)
            for (int jj = tid; jj < nk; jj += kPT)
              if (jj != slot)
                cp_async16(&sm.vring[jj], static_cast<const bf16*>(L.ring_v) +
                                              static_cast<int64_t>(jj) * D + cta * 8);
          cp_async_commit();
        } else {
          const int HVg = Hg * Kg;
          if (gw < D)
            warp_copy_row(sm.kbuf[warp], static_cast<const bf16*>(B.w_out) + static_cast<int64_t>(gw) * HVg,
                          HVg >> 3, lane);
          cp_async_commit();
          if (cta < gunits) {  // state rows 0..63, columns v0..v0+31 of the unit (8 chunks a row)
            const int uh = cta / (Kg / 32), uv0 = (cta % (Kg / 32)) * 32;
            const float* S0 = L.gdn_state + (static_cast<int64_t>(uh) * Kg) * Kg + uv0;
            for (int i = tid; i < Kg * 8; i += kPT)
              cp_async16(reinterpret_cast<float*>(sm.vring) + (i >> 3) * 32 + (i & 7) * 4,
                         S0 + static_cast<int64_t>(i >> 3) * Kg + (i & 7) * 4);
          }
          cp_async_commit();
        }
        float4 nwa = make_float4(0.f, 0.f, 0.f, 0.f), nwb = nwa;
        if (tid < n8) {
          nwa = __ldg(reinterpret_cast<const float4*>(B.mixer_norm) + 2 * tid);
          nwb = __ldg(reinterpret_cast<const float4*>(B.mixer_norm) + 2 * tid + 1);
        }
        if (!first && !gb.wait()) return;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        float ss = 0.f;
        if (tid < n8) {
          if (first) {
            const uint4 e = __ldg(reinterpret_cast<const uint4*>(embed + tok * D) + tid);
            const uint32_t ew[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float2 f = unpack_bf16x2(ew[q]);
              v[2 * q] = f.x + __ldg(p.stream_seed + tid * 8 + 2 * q);
              v[2 * q + 1] = f.y + __ldg(p.stream_seed + tid * 8 + 2 * q + 1);
            }
          } else {
            const float4 a = __ldcg(reinterpret_cast<const float4*>(xsrc) + 2 * tid);
            const float4 b = __ldcg(reinterpret_cast<const float4*>(xsrc) + 2 * tid + 1);
            v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
            v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            if (have_y)
              for (int s = 0; s < K; ++s) {
                const uint4 u = ldcg16(ybuf + static_cast<int64_t>(s) * D + tid * 8);
                const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const float2 f = unpack_bf16x2(uw[q]);
                  v[2 * q] += f.x;
                  v[2 * q + 1] += f.y;
                }
              }
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) ss += v[q] * v[q];
        }
        const float r = rsqrtf(block_sum(ss, sm.red) / static_cast<float>(D) + eps);
        if (tid < n8) {
          const float w8[8] = {nwa.x, nwa.y, nwa.z, nwa.w, nwb.x, nwb.y, nwb.z, nwb.w};
          uint4 o;
          o.x = pack_bf16x2(v[0] * r * w8[0], v[1] * r * w8[1]);
          o.y = pack_bf16x2(v[2] * r * w8[2], v[3] * r * w8[3]);
          o.z = pack_bf16x2(v[4] * r * w8[4], v[5] * r * w8[5]);
          o.w = pack_bf16x2(v[6] * r * w8[6], v[7] * r * w8[7]);
          reinterpret_cast<uint4*>(s_vec)[tid] = o;
          if (cta == 0) {
            __stcg(reinterpret_cast<float4*>(xdst) + 2 * tid, make_float4(v[0], v[1], v[2], v[3]));
            __stcg(reinterpret_cast<float4*>(xdst) + 2 * tid + 1,
                   make_float4(v[4], v[5], v[6], v[7]));
            stcg16(normed_g + tid * 8, o);
          }
        }
        cp_async_wait_group<2>();  // this phase's rows (later groups may still fly)
        __syncthreads();
        if (r0 < B.rows) {
          const float acc = srow_dot(wb, s_vec, n8, lane);
          if (lane == 0) stcg_bf(proj + r0, acc);
        }
        if (r1 < B.rows) {
          const float acc = srow_dot(wb + kMaxD, s_vec, n8, lane);
          if (lane == 0) stcg_bf(proj + r1, acc);
        }
        gb.arrive();
        xs ^= 1;
        have_y = false;
        first = false;
      }
      int n_part = 0;
      if (B.kind == 0) {
        // ============================================================ CSA M1
        bf16* ring_k = static_cast<bf16*>(L.ring_k);
        bf16* ring_v = static_cast<bf16*>(L.ring_v);
        const int key = cta * kPW + warp;
        const bool mine = cta < nk1 && key < nk;
        const int hdc8 = HDc >> 3;
        uint4* krow = reinterpret_cast<uint4*>(sm.kbuf[warp]);  // copied during phase A
        if (!gb.wait()) return;
        if (cta < nk1) {
          for (int i = tid; i < HDc; i += kPT) sm.q[i] = ldcg_bf(proj + i) * qscale;
          cp_async_wait_group<1>();
          __syncthreads();
          if (mine) {
            if (key == slot) {
              // the new token's key from the projection, into the ring (its
              // value goes into the ring column by column in M2)
              for (int c = lane; c < hdc8; c += 32) {
                const uint4 kv = ldcg16(proj + HDc + c * 8);
                krow[c] = kv;
                stcg16(ring_k + static_cast<int64_t>(slot) * HDc + c * 8, kv);
              }
              __syncwarp();
            }
            // per-head dots: chunk c covers dims [8c, 8c + 8) of head 8c / Dh;
            // the Dh / 8 lanes of a head reduce by xor shuffles
#pragma unroll
            for (int i = 0; i < DC; ++i) {
              const int c = lane + 32 * i;
              float s = 0.f;
              if (c < hdc8) {
                const uint4 k4 = krow[c];
                const uint32_t kw[4] = {k4.x, k4.y, k4.z, k4.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 f = unpack_bf16x2(kw[e]);
                  s += f.x * sm.q[c * 8 + 2 * e] + f.y * sm.q[c * 8 + 2 * e + 1];
                }
              }
              s += __shfl_xor_sync(0xffffffffu, s, 4);
              s += __shfl_xor_sync(0xffffffffu, s, 2);
              s += __shfl_xor_sync(0xffffffffu, s, 1);
              if ((lane & 7) == 0 && c < hdc8) sm.sc[(c * 8) / Dh][warp] = s;
            }
          }
          __syncthreads();
          const int nkl = min(kPW, nk - cta * kPW);
          if (warp < Hc) {
            const float s = lane < nkl ? sm.sc[warp][lane] : -INFINITY;
            const float m = warp_max(s);
            const float l = warp_sum(lane < nkl ? exp2f(s - m) : 0.f);
            if (lane < nkl) __stcg(p.scores + warp * W + cta * kPW + lane, s);
            if (lane == 0) {
              // [head][key chunk][max, sum]: a head's chunks are contiguous for M2
              __stcg(reinterpret_cast<float2*>(p.stats) + warp * G + cta, make_float2(m, l));
            }
          }
        }
        gb.arrive();
        // ============================================================ CSA M2
        // thread t = (key group g = t / 8, column c = t % 8) of this CTA's 8
        // columns; group g takes keys g, g + 64, ... (at most kKpg of them)
        const int col0 = cta * 8;
        constexpr int kKpg = kMaxW / 64;
        const int grp = tid >> 3, cc = tid & 7;
        float fcol = 0.f, ffc = 0.f;
        if (cta < ncs) {
          // (the cached values' chunks of these columns were copied into
          // sm.vring during phase A)
          // router row t / 8 at column t % 8; threads t < 8: the FFN norm weight
          if (tid < 8 * E) fcol = __ldg(B.router_fold + static_cast<int64_t>(tid >> 3) * D + col0 + (tid & 7));
          if (tid < 8) ffc = __ldg(B.ffn_norm + col0 + tid);
        }
        if (!gb.wait()) return;
        if (cta < ncs) {
          gb.point(li * p.n_blocks + j, 0);
          // loads that depend on the previous phase, issued together
          float sm0 = -INFINITY, sl0 = 0.f, sm1 = -INFINITY, sl1 = 0.f;
          if (warp < Hc) {
            if (lane < nk1) {
              const float2 st0 = __ldcg(reinterpret_cast<const float2*>(p.stats) + warp * G + lane);
              sm0 = st0.x;
              sl0 = st0.y;
            }
            if (lane + 32 < nk1) {
              const float2 st1 =
                  __ldcg(reinterpret_cast<const float2*>(p.stats) + warp * G + lane + 32);
              sm1 = st1.x;
              sl1 = st1.y;
            }
          }
          const float xold = tid < 8 ? __ldcg(xdst + col0 + tid) : 0.f;
          if (tid == 0 && slot < nk) {
            // the new token's value chunk of these columns, from the projection,
            // also stored into the ring for the following steps
            const uint4 vnew = ldcg16(proj + 2 * HDc + col0);
            sm.vring[slot] = vnew;
            stcg16(ring_v + static_cast<int64_t>(slot) * D + col0, vnew);
          }
          // this thread's key's scores, in the same round of loads
          float sck[kMaxHeads];
#pragma unroll
          for (int h = 0; h < kMaxHeads; ++h)
            sck[h] = (h < Hc && tid < nk) ? __ldcg(p.scores + h * W + tid) : 0.f;
          if (warp < Hc) {
            const float m = warp_max(fmaxf(sm0, sm1));
            float l = 0.f;
            if (lane < nk1) l += sl0 * exp2f(sm0 - m);
            if (lane + 32 < nk1) l += sl1 * exp2f(sm1 - m);
            l = warp_sum(l);
            if (lane == 0) {
              sm.hM[warp] = m;
              sm.hInvL[warp] = 1.0f / (l * static_cast<float>(Hc));
            }
          }
          __syncthreads();
          gb.point(li * p.n_blocks + j, 1);
          // head-averaged probability of every key, once
          float* pbar = sm.ptmp;  // [nk]
          cp_async_wait_group<0>();
          if (tid < nk) {
            float pb = 0.f;
#pragma unroll
            for (int h = 0; h < kMaxHeads; ++h)
              if (h < Hc) pb += exp2f(sck[h] - sm.hM[h]) * sm.hInvL[h];
            pbar[tid] = pb;
          }
          for (int jj = tid + kPT; jj < nk; jj += kPT) {  // windows past 512 keys
            float pb = 0.f;
            for (int h = 0; h < Hc; ++h)
              pb += exp2f(__ldcg(p.scores + h * W + jj) - sm.hM[h]) * sm.hInvL[h];
            pbar[jj] = pb;
          }
          __syncthreads();
          float acc = 0.f;
          const bf16* vr = reinterpret_cast<const bf16*>(sm.vring);
#pragma unroll
          for (int i = 0; i < kKpg; ++i) {
            const int jj = grp + 64 * i;
            if (jj < nk) acc += pbar[jj] * bf2f(vr[jj * 8 + cc]);
          }
          // the 4 key groups of a warp share the column: lanes c, c+8, c+16, c+24
          acc += __shfl_xor_sync(0xffffffffu, acc, 8);
          acc += __shfl_xor_sync(0xffffffffu, acc, 16);
          if (lane < 8) sm.vred[warp][lane] = acc;
          __syncthreads();
          if (tid < 8) {
            float o = 0.f;
            for (int w = 0; w < kPW; ++w) o += sm.vred[w][tid];
            const float x = xold + bf2f(f2bf(o));  // the block output is bf16
            __stcg(xdst + col0 + tid, x);
            sm.xrow[tid] = x;
          }
          __syncthreads();
          gb.point(li * p.n_blocks + j, 2);
          // router partial sums over the 8 columns: groups of 8 lanes (one value
          // per group) reduced by xor shuffles
          if (warp < (8 * E + 31) / 32) {
            const float x = sm.xrow[tid & 7];
            float a = tid < 8 * E ? fcol * x : 0.f;
            a += __shfl_xor_sync(0xffffffffu, a, 4);
            a += __shfl_xor_sync(0xffffffffu, a, 2);
            a += __shfl_xor_sync(0xffffffffu, a, 1);
            if ((tid & 7) == 0 && tid < 8 * E) __stcg(p.partials + (2 + (tid >> 3)) * G + cta, a);
          }
          if (warp == 0) {
            const float x = tid < 8 ? sm.xrow[tid] : 0.f;
            float a = x * x, b = (x * ffc) * (x * ffc);
            a += __shfl_xor_sync(0xffffffffu, a, 4);
            a += __shfl_xor_sync(0xffffffffu, a, 2);
            a += __shfl_xor_sync(0xffffffffu, a, 1);
            b += __shfl_xor_sync(0xffffffffu, b, 4);
            b += __shfl_xor_sync(0xffffffffu, b, 2);
            b += __shfl_xor_sync(0xffffffffu, b, 1);
            if (lane == 0) {
              __stcg(p.partials + cta, a);
              __stcg(p.partials + G + cta, b);
            }
          }
        }
        n_part = ncs;
        gb.arrive();
      } else {
        // ============================================================ GDN M
        const int HVg = Hg * Kg;
        float* state = L.gdn_state;
        const int unit_h = cta / (Kg / 32), v0 = (cta % (Kg / 32)) * 32;
        constexpr int RPW = 16;  // 4 warps x 16 state rows = key dim 64
        float sreg[RPW];
        float* S = state + (static_cast<int64_t>(unit_h) * Kg) * Kg + v0 + lane;
        const float a_dec = cta < gunits ? sigmoidf_(__ldg(B.decay_logit + unit_h)) : 0.f;
        const float b_bias = cta < gunits ? __ldg(B.beta_bias + unit_h) : 0.f;
        if (!gb.wait()) return;
        if (cta < gunits) {  // CTA-uniform: the barriers below are reached by all threads
          // q, k, v, gate and beta of the unit in one round of loads
          float vin = 0.f, gin = 0.f, bin = 0.f;
          if (warp < 4) {
            vin = ldcg_bf(proj + 2 * HKg + unit_h * Kg + v0 + lane);
            gin = ldcg_bf(proj + 2 * HKg + HVg + unit_h * Kg + v0 + lane);
            bin = ldcg_bf(proj + 2 * HKg + 2 * HVg + unit_h);
          }
          if (tid < Kg) {
            sm.q[tid] = ldcg_bf(proj + unit_h * Kg + tid);
            sm.kk[tid] = ldcg_bf(proj + HKg + unit_h * Kg + tid);
          }
          cp_async_wait_group<0>();  // the state slice (copied during phase A)
          __syncthreads();
          if (warp < 4) {
            const float* gs = reinterpret_cast<const float*>(sm.vring);
#pragma unroll
            for (int r = 0; r < RPW; ++r) sreg[r] = gs[(warp * RPW + r) * 32 + lane];
          }
          if (warp == 0) {
            // q, k <- x * rsqrt(max(sum x^2, 1e-12)) (gated_deltanet.py:128-129)
            float sq = 0.f, sk = 0.f;
            for (int i = lane; i < Kg; i += 32) {
              sq += sm.q[i] * sm.q[i];
              sk += sm.kk[i] * sm.kk[i];
            }
            sq = warp_sum(sq);
            sk = warp_sum(sk);
            if (lane == 0) {
              sm.scal[0] = rsqrtf(fmaxf(sq, 1e-12f));
              sm.scal[1] = rsqrtf(fmaxf(sk, 1e-12f));
            }
          }
          __syncthreads();
          if (tid < Kg) {
            sm.q[tid] *= sm.scal[0];
            sm.kk[tid] *= sm.scal[1];
          }
          __syncthreads();
          const float a = a_dec;
          const float beta = sigmoidf_(bin + b_bias);
          if (warp < 4) {
            float pred = 0.f;
#pragma unroll
            for (int r = 0; r < RPW; ++r) pred += sm.kk[warp * RPW + r] * sreg[r];
            sm.gred[warp][lane] = pred;
          }
          __syncthreads();
          float opart = 0.f;
          if (warp < 4) {
            const float pr = sm.gred[0][lane] + sm.gred[1][lane] + sm.gred[2][lane] +
                             sm.gred[3][lane];
            const float delta = vin - pr;
#pragma unroll
            for (int r = 0; r < RPW; ++r) {
              const int kr = warp * RPW + r;
              const float ns = a * sreg[r] + beta * sm.kk[kr] * delta;
              __stcg(S + static_cast<int64_t>(kr) * Kg, ns);
              opart += sm.q[kr] * ns;
            }
          }
          __syncthreads();
          if (warp < 4) sm.gred[warp][lane] = opart;
          __syncthreads();
          if (warp == 0) {
            const float o = sm.gred[0][lane] + sm.gred[1][lane] + sm.gred[2][lane] +
                            sm.gred[3][lane];
            // reference order: out.to(hidden dtype) * gate (gated_deltanet.py:149)
            const float gt = sigmoidf_(gin);
            stcg_bf(mix + unit_h * Kg + v0 + lane, bf2f(f2bf(o)) * gt);
          }
        }
        gb.arrive();
        // ============================================================ GDN C
        {
          const bf16* w_out = static_cast<const bf16*>(B.w_out);
          bf16* hist = static_cast<bf16*>(L.conv_hist);
          const int n = gw;  // output column of this warp (D <= warps of the grid)
          const int hv8 = HVg >> 3;
          float c4[4] = {0.f, 0.f, 0.f, 0.f}, h3[3] = {0.f, 0.f, 0.f}, fw = 0.f;
          // router weights of this column for the values v = lane + 32 u (v >= 2);
          // the residual and normalised input of the column (written by phase A)
          float fv[3] = {0.f, 0.f, 0.f};
          float xpre = 0.f, npre = 0.f;
          if (n < D) {
#pragma unroll
            for (int q = 0; q < 4; ++q) c4[q] = __ldg(B.conv + n * 4 + q);
#pragma unroll
            for (int q = 0; q < 3; ++q) h3[q] = ldcg_bf(hist + static_cast<int64_t>(q) * D + n);
            fw = __ldg(B.ffn_norm + n);
            xpre = __ldcg(xdst + n);
            npre = ldcg_bf(normed_g + n);
#pragma unroll
            for (int u = 0; u < 3; ++u) {
              const int v = lane + 32 * u;
              if (v >= 2 && v < NV)
                fv[u] = __ldg(B.router_fold + static_cast<int64_t>(v - 2) * D + n);
            }
          }
          if (!gb.wait()) return;
          for (int c = tid; c < hv8; c += kPT)
            reinterpret_cast<uint4*>(s_vec)[c] = ldcg16(mix + c * 8);
          cp_async_wait_group<0>();  // this warp's output-projection row (phase A)
          __syncthreads();
          float x = 0.f;
          if (n < D) {
            const float y = bf2f(f2bf(srow_dot(sm.kbuf[warp], s_vec, hv8, lane)));
            const float xb = npre;
            // conv gate of the decode step over [history, this input]
            const float cacc = c4[0] * h3[0] + c4[1] * h3[1] + c4[2] * h3[2] + c4[3] * xb;
            const float yv = y * sigmoidf_(cacc);
            if (lane == 0) {
              stcg_bf(hist + n, h3[1]);
              stcg_bf(hist + D + n, h3[2]);
              stcg_bf(hist + 2 * D + n, xb);
              x = xpre + bf2f(f2bf(yv));
              __stcg(xdst + n, x);
            }
            x = __shfl_sync(0xffffffffu, x, 0);
          }
#pragma unroll
          for (int u = 0; u < 3; ++u) {
            const int v = lane + 32 * u;
            if (v >= NV) break;
            float a = 0.f;
            if (n < D) a = v == 0 ? x * x : (v == 1 ? (x * fw) * (x * fw) : fv[u] * x);
            sm.part[warp][v] = a;
          }
          __syncthreads();
          n_part = (D + kPW - 1) / kPW;
          if (cta < n_part && tid < NV) {
            float a = 0.f;
            for (int w = 0; w < kPW; ++w) a += sm.part[w][tid];
            __stcg(p.partials + tid * G + cta, a);
          }
          gb.arrive();
        }
      }
      // ================================================================ E1
      {
        float4 fwa = make_float4(0.f, 0.f, 0.f, 0.f), fwb = fwa;
        if (tid < n8) {
          fwa = __ldg(reinterpret_cast<const float4*>(B.ffn_norm) + 2 * tid);
          fwb = __ldg(reinterpret_cast<const float4*>(B.ffn_norm) + 2 * tid + 1);
        }
        if (!gb.wait()) return;
        // the router partial sums of all producing CTAs ([value][slot], slot =
        // producing CTA) and the residual row in one round of loads: warp w sums
        // values w, w + 16, ... over the slots lane, lane + 32, ... (each load
        // one contiguous line), then a fixed xor tree (the same order in every
        // CTA, so all of them route identically)
        float4 xa = make_float4(0.f, 0.f, 0.f, 0.f), xb4 = xa;
        if (tid < n8) {
          xa = __ldcg(reinterpret_cast<const float4*>(xdst) + 2 * tid);
          xb4 = __ldcg(reinterpret_cast<const float4*>(xdst) + 2 * tid + 1);
        }
        for (int v = warp; v < NV; v += kPW) {  // warp-uniform
          const float* pv = p.partials + v * G;
          float t4[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {  // n_part <= 128 slots
            const int s_ = lane + 32 * u;
            t4[u] = s_ < n_part ? __ldcg(pv + s_) : 0.f;
          }
          const float a = warp_sum((t4[0] + t4[1]) + (t4[2] + t4[3]));
          if (lane == 0) {
            if (v < 2) sm.scal[v] = a; else sm.logit[v - 2] = a;
          }
        }
        __syncthreads();
        gb.point(li * p.n_blocks + j, 4);
        const float inv1 = rsqrtf(sm.scal[0] / static_cast<float>(D) + eps);
        const float inv2 = rsqrtf(inv1 * inv1 * sm.scal[1] / static_cast<float>(D) + eps);
        // warp 0 takes the top-k (value desc, index asc; softmax of the k values)
        // while the others form the experts' input; one CTA barrier hands it on
        if (warp == 0) {
          float v0 = lane < E ? sm.logit[lane] * inv1 * inv2 : -INFINITY;
          float v1 = lane + 32 < E ? sm.logit[lane + 32] * inv1 * inv2 : -INFINITY;
          float top = 0.f, mine = 0.f;
          int mine_i = 0;
          for (int r = 0; r < K; ++r) {
            float bv = v0;
            int bi = lane;
            if (v1 > bv) { bv = v1; bi = lane + 32; }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
              const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
              const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
              if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
            if (r == 0) top = bv;
            if (lane == r) { mine = bv; mine_i = bi; }
            if (bi == lane) v0 = -INFINITY;
            if (bi == lane + 32) v1 = -INFINITY;
          }
          const float ex = lane < K ? expf(mine - top) : 0.f;
          const float den = warp_sum(ex);
          if (lane < K) {
            const int my_e = min(max(mine_i, 0), E - 1);  // a NaN row must not pick a missing expert
            const float my_p = ex / den;
            sm.idx[lane] = my_e;
            sm.prob[lane] = my_p;
            if (cta == 0) {
              p.route_idx[(li * p.n_blocks + j) * K + lane] = my_e;
              p.route_prob[(li * p.n_blocks + j) * K + lane] = my_p;
            }
          }
        }
        // the experts' input m = RMSNorm(x) * ffn_norm (bf16)
        if (tid < n8) {
          const float4 a = xa, b = xb4;
          const float4 wa4 = fwa, wb4 = fwb;
          uint4 o;
          o.x = pack_bf16x2(a.x * inv1 * wa4.x, a.y * inv1 * wa4.y);
          o.y = pack_bf16x2(a.z * inv1 * wa4.z, a.w * inv1 * wa4.w);
          o.z = pack_bf16x2(b.x * inv1 * wb4.x, b.y * inv1 * wb4.y);
          o.w = pack_bf16x2(b.z * inv1 * wb4.z, b.w * inv1 * wb4.w);
          reinterpret_cast<uint4*>(s_vec)[tid] = o;
        }
        __syncthreads();
        gb.point(li * p.n_blocks + j, 5);
        const bf16* w13 = static_cast<const bf16*>(B.w13);
        uint4 wg[DC], wu[DC];
        // features round-robin over the CTAs (warp w of CTA c: w * G + c, ...), so
        // every SM streams about the same number of expert rows
        for (int g = warp * G + cta; g < K * F; g += NW) {
          const int s = g / F, f = g - s * F;
          const int64_t grow = static_cast<int64_t>(sm.idx[s]) * 2 * F + (f / 128) * 256 + (f % 128);
          load_row<DC>(w13 + grow * D, n8, lane, wg);
          load_row<DC>(w13 + (grow + 128) * D, n8, lane, wu);
          const float ga = row_dot<DC>(wg, s_vec, n8, lane);
          const float ua = row_dot<DC>(wu, s_vec, n8, lane);
          if (lane == 0) stcg_bf(hbuf + static_cast<int64_t>(s) * F + f, silu_mul(ga, ua));
        }
        gb.point(li * p.n_blocks + j, 6);
        gb.arrive();
      }
      // ================================================================ E2
      {
        const bf16* w2 = static_cast<const bf16*>(B.w2);
        const int f8 = F >> 3;
        uint4 wd[FC];
        const int r0 = warp * G + cta;  // rows round-robin over the CTAs
        bf16* wb = sm.wbuf[warp];
        if (r0 < K * D) {
          const int s = r0 / D, n = r0 - s * D;
          warp_copy_row(wb, w2 + (static_cast<int64_t>(sm.idx[s]) * D + n) * F, f8, lane);
        }
        cp_async_commit();
        if (!gb.wait()) return;
        for (int c = tid; c < K * f8; c += kPT)
          reinterpret_cast<uint4*>(s_vec)[c] = ldcg16(hbuf + c * 8);
        cp_async_wait_group<0>();
        __syncthreads();
        for (int r = r0; r < K * D; r += NW) {
          const int s = r / D, n = r - s * D;
          float acc;
          if (r == r0) {
            acc = srow_dot(wb, s_vec + s * F, f8, lane);
          } else {
            load_row<FC>(w2 + (static_cast<int64_t>(sm.idx[s]) * D + n) * F, f8, lane, wd);
            acc = row_dot<FC>(wd, s_vec + s * F, f8, lane);
          }
          if (lane == 0) stcg_bf(ybuf + static_cast<int64_t>(s) * D + n, acc * sm.prob[s]);
        }
        gb.arrive();
        have_y = true;
      }
    }
  }
  // ================================================================== head
  if (p.skip_head) {
    cp_async_wait_group<0>();
    if (cta == 0 && tid == 0) *p.positions = pos + 1;  // every CTA read it before a barrier
    return;
  }
  {
    const float* xcur = p.x + xs * D;
    const bf16* collapse = static_cast<const bf16*>(p.collapse);
    bf16* collapsed = static_cast<bf16*>(p.collapsed);
    if (gw < D) warp_copy_row(sm.wbuf[warp], collapse + static_cast<int64_t>(gw) * D, n8, lane);
    cp_async_commit();
    if (!gb.wait()) return;
    if (tid < n8) {
      const float4 a = __ldcg(reinterpret_cast<const float4*>(xcur) + 2 * tid);
      const float4 b = __ldcg(reinterpret_cast<const float4*>(xcur) + 2 * tid + 1);
      float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      if (have_y)
        for (int s = 0; s < K; ++s) {
          const uint4 u = ldcg16(ybuf + static_cast<int64_t>(s) * D + tid * 8);
          const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = unpack_bf16x2(uw[q]);
            v[2 * q] += f.x;
            v[2 * q + 1] += f.y;
          }
        }
      uint4 o;
      o.x = pack_bf16x2(v[0], v[1]);
      o.y = pack_bf16x2(v[2], v[3]);
      o.z = pack_bf16x2(v[4], v[5]);
      o.w = pack_bf16x2(v[6], v[7]);
      reinterpret_cast<uint4*>(s_vec)[tid] = o;
    }
    cp_async_wait_group<0>();
    __syncthreads();
    if (gw < D) {
      const float acc = srow_dot(sm.wbuf[warp], s_vec, n8, lane);
      if (lane == 0) stcg_bf(collapsed + gw, acc);
    }
    gb.arrive();
    // final RMSNorm and the tied LM head
    uint4 we[2][DC];
    int v = gw;
    if (v < p.vocab) load_row<DC>(embed + static_cast<int64_t>(v) * D, n8, lane, we[0]);
    if (!gb.wait()) return;
    float c8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float ss = 0.f;
    if (tid < n8) {
      const uint4 u = ldcg16(collapsed + tid * 8);
      const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = unpack_bf16x2(uw[q]);
        c8[2 * q] = f.x;
        c8[2 * q + 1] = f.y;
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) ss += c8[q] * c8[q];
    }
    const float r = rsqrtf(block_sum(ss, sm.red) / static_cast<float>(D) + eps);
    if (tid < n8) {
      uint4 o;
      uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        op[q] = pack_bf16x2(c8[2 * q] * r * __ldg(p.final_norm + tid * 8 + 2 * q),
                            c8[2 * q + 1] * r * __ldg(p.final_norm + tid * 8 + 2 * q + 1));
      reinterpret_cast<uint4*>(s_vec)[tid] = o;
    }
    __syncthreads();
    // greedy sampling state of this warp: first maximal logit, and the running
    // max / exp-sum of its logits (online log-sum-exp)
    float best = -INFINITY, run_m = -INFINITY, run_s = 0.f;
    int best_i = 0;
    auto track = [&](float l, int vi) {
      if (l > best) { best = l; best_i = vi; }  // rows come in increasing order
      if (l > run_m) {
        run_s = (run_m == -INFINITY ? 0.f : run_s * expf(run_m - l)) + 1.f;
        run_m = l;
      } else {
        run_s += expf(l - run_m);
      }
    };
    // two rows in flight: the next row streams in while this one is reduced
    for (; v < p.vocab; v += 2 * NW) {
      const int v1 = v + NW, v2 = v + 2 * NW;
      if (v1 < p.vocab) load_row<DC>(embed + static_cast<int64_t>(v1) * D, n8, lane, we[1]);
      const float a0 = bf2f(f2bf(row_dot<DC>(we[0], s_vec, n8, lane)));
      if (lane == 0) __stcg(p.logits + v, a0);
      track(a0, v);
      if (v2 < p.vocab) load_row<DC>(embed + static_cast<int64_t>(v2) * D, n8, lane, we[0]);
      if (v1 < p.vocab) {
        const float a1 = bf2f(f2bf(row_dot<DC>(we[1], s_vec, n8, lane)));
        if (lane == 0) __stcg(p.logits + v1, a1);
        track(a1, v1);
      }
    }
    if (p.out_token != nullptr) {
      // CTA: combine the warps in order; then the last CTA to finish combines
      // the CTAs in order (the same result however the CTAs are scheduled)
      if (lane == 0) {
        sm.part[warp][0] = best;
        sm.part[warp][1] = __int_as_float(best_i);
        sm.part[warp][2] = run_m;
        sm.part[warp][3] = run_s;
      }
      __syncthreads();
      __shared__ int s_last;
      if (tid == 0) {
        float b = -INFINITY, m = -INFINITY, s = 0.f;
        int bi = 0;
        for (int w = 0; w < kPW; ++w) {
          const float wb = sm.part[w][0], wm = sm.part[w][2], ws = sm.part[w][3];
          const int wi = __float_as_int(sm.part[w][1]);
          if (wb > b || (wb == b && wi < bi)) { b = wb; bi = wi; }
          const float nm = fmaxf(m, wm);
          s = (m == -INFINITY ? 0.f : s * expf(m - nm)) + (wm == -INFINITY ? 0.f : ws * expf(wm - nm));
          m = nm;
        }
        __stcg(p.head_part + cta * 4, b);
        __stcg(p.head_part + cta * 4 + 1, __int_as_float(bi));
        __stcg(p.head_part + cta * 4 + 2, m);
        __stcg(p.head_part + cta * 4 + 3, s);
        __threadfence();
        s_last = atomicAdd(p.bar + 1, 1u) == static_cast<uint32_t>(G) - 1;
      }
      __syncthreads();
      if (s_last && warp == 0) {
        __threadfence();
        float b = -INFINITY, m = -INFINITY, s = 0.f;
        int bi = 0;
        for (int c = lane; c < G; c += 32) {  // lane-ordered, then a fixed xor tree
          const float cb = __ldcg(p.head_part + c * 4), cm = __ldcg(p.head_part + c * 4 + 2);
          const float cs = __ldcg(p.head_part + c * 4 + 3);
          const int ci = __float_as_int(__ldcg(p.head_part + c * 4 + 1));
          if (cb > b || (cb == b && ci < bi)) { b = cb; bi = ci; }
          const float nm = fmaxf(m, cm);
          s = (m == -INFINITY ? 0.f : s * expf(m - nm)) + (cm == -INFINITY ? 0.f : cs * expf(cm - nm));
          m = nm;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ob = __shfl_xor_sync(0xffffffffu, b, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          const float om = __shfl_xor_sync(0xffffffffu, m, o);
          const float os = __shfl_xor_sync(0xffffffffu, s, o);
          if (ob > b || (ob == b && oi < bi)) { b = ob; bi = oi; }
          const float nm = fmaxf(m, om);
          s = (m == -INFINITY ? 0.f : s * expf(m - nm)) + (om == -INFINITY ? 0.f : os * expf(om - nm));
          m = nm;
        }
        if (lane == 0) {
          *p.out_token = bi;
          if (p.out_logprob != nullptr) *p.out_logprob = b - (m + logf(s));  // raw log-softmax
          if (p.seen != nullptr) atomicOr(p.seen + (bi >> 5), 1 << (bi & 31));
        }
      }
    }
    if (cta == 0 && tid == 0) *p.positions = pos + 1;  // every CTA read it before a barrier
  }
}

constexpr int kSmemBytes = kVecBytes + static_cast<int>(sizeof(Smem));

}  // namespace
}  // namespace llmyb

using namespace llmyb;

namespace {
using PKernel = void (*)(const llmyb_pdecode);
PKernel persistent_kernel_for(int D, int F) {
  const int dc = (D + 255) / 256, fc = (F + 255) / 256;
  if (dc <= 3) return fc <= 4 ? decode_persistent_kernel<3, 4> : decode_persistent_kernel<3, 8>;
  return fc <= 4 ? decode_persistent_kernel<4, 4> : decode_persistent_kernel<4, 8>;
}
}  // namespace

LLMYB_API int32_t llmyb_decode_persistent_grid(void) {
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return -static_cast<int32_t>(e);
  PKernel k = decode_persistent_kernel<4, 8>;  // the largest variant bounds them all
  int32_t st = ensure_smem(k, kSmemBytes);
  if (st) return -st;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kPT, kSmemBytes);
  if (e != cudaSuccess) return -static_cast<int32_t>(e);
  if (per_sm < 1) return -LLMYB_EUNSUPPORTED;
  return sms;
}

LLMYB_API int32_t llmyb_decode_persistent(const llmyb_pdecode* p, void* stream) {
  if (!p || !p->blocks || !p->layers || !p->embed || !p->stream_seed || !p->collapse ||
      !p->final_norm || !p->token || !p->positions || !p->x || !p->proj || !p->normed ||
      !p->mix || !p->partials || !p->hbuf || !p->ybuf || !p->collapsed || !p->route_idx ||
      !p->route_prob || !p->logits || !p->bar || !p->status)
    return LLMYB_EINVAL;
  const int D = p->d_model;
  if (D <= 0 || D % 8 != 0 || D > kMaxD || p->n_blocks <= 0 || p->n_loops <= 0 ||
      p->vocab <= 0 || p->n_experts <= 0 || p->n_experts > kMaxE || p->top_k <= 0 ||
      p->top_k > kMaxK || p->top_k > p->n_experts || p->ffn <= 0 || p->ffn % 128 != 0 ||
      p->ffn > kMaxF || p->grid <= 0)
    return LLMYB_EUNSUPPORTED;
  const int64_t nw = static_cast<int64_t>(p->grid) * kPW;
  if (D > nw || 2 + p->n_experts > kPT / 2) return LLMYB_EUNSUPPORTED;
  if (p->csa_heads > 0) {
    if (!p->scores || !p->stats || p->csa_head_dim != 64 || p->csa_heads > kMaxHeads ||
        p->csa_heads * p->csa_head_dim > kMaxD || p->window <= 0 || p->window > kMaxW ||
        (p->window + kPW - 1) / kPW > p->grid || D / 8 > p->grid)
      return LLMYB_EUNSUPPORTED;
  }
  if (p->gdn_heads > 0 &&
      (p->gdn_dim != 64 || p->gdn_heads * p->gdn_dim > kMaxD ||
       p->gdn_heads * (p->gdn_dim / 32) > p->grid))
    return LLMYB_EUNSUPPORTED;
  PKernel kern = persistent_kernel_for(D, p->ffn);
  int32_t st = ensure_smem(kern, kSmemBytes);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p->out_token != nullptr && !p->head_part) return LLMYB_EINVAL;
  cudaError_t e = cudaMemsetAsync(p->bar, 0, 2 * sizeof(uint32_t), s);
  if (e != cudaSuccess) return static_cast<int32_t>(e);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p->grid));
  cfg.blockDim = dim3(kPT);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, *p);
  count_launch();
  if (e != cudaSuccess) return static_cast<int32_t>(e);
  return launch_status();
}
