// Next-token sampling on device: repetition penalty, greedy, temperature,
// top-k, top-p (nucleus) and the draw, one 1024-thread CTA per row.
//
// Reference: sample_standalone.py:5383-5423 (_sample_next_token) and
// :5596-5636 (sample()); the native sampler llmy_cuda/src/kernels/sample.cu
// (single-block iterated argmax, top-k <= 64, CDF on the host) and
// llmy_sample (llmy_cuda/src/llmy.cpp:132-202).
//
//   penalty  : l > 0 ? l / rep : l * rep for every id set in the row's
//              `seen` bitmask (set(generated)); blocked ids -> -inf
//   greedy   : temp <= 1e-4 -> first maximal index
//   top-k    : exact k-th largest by a 4-pass 8-bit radix select on the
//              order-preserving integer image of the fp32 value; candidates
//              sorted by (value desc, index asc) with a bitonic sort
//   top-p    : remove candidate i when the exclusive cumulative probability
//              exceeds top_p (the first is always kept), renormalise
//   draw     : inverse CDF at the caller's uniform u, in the order the
//              reference hands to multinomial (sorted candidates; plain
//              vocabulary order when neither top-k nor top-p applies)
// Also returns the raw log-softmax of the chosen token (the reference's
// model_logprob) and sets the token's bit in `seen`.
#include "common.cuh"

namespace llmyb {
namespace {

constexpr int kThreads = 1024;
constexpr int kMaxCand = 1024;       // top-k limit
constexpr int kBuf = 2 * kMaxCand;   // candidates incl. boundary ties

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

struct SampleArgs {
  const float* logits;
  int64_t ld;
  int V;
  uint32_t* seen;  // [B, ceil(V/32)] or null
  int64_t seen_ld;
  float rep;
  const int32_t* blocked;
  int n_blocked;
  float temp;
  int top_k;
  float top_p;
  const float* uniforms;
  int64_t* out_tok;
  float* out_logprob;
  int update_seen;
  int32_t* status;
  int cache_keys;  // 1: the top-k order keys of the row are kept in shared memory
};

__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = lane < (blockDim.x >> 5) ? red[lane] : 0.f;
  r = warp_sum(r);
  return r;
}

// inclusive prefix sum over blockDim.x values (one per thread)
__device__ float block_inclusive_scan(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) red[warp] = x;
  __syncthreads();
  if (warp == 0) {
    float w = red[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    red[lane] = w;
  }
  __syncthreads();
  return x + (warp > 0 ? red[warp - 1] : 0.f);
}

__global__ void __launch_bounds__(kThreads) sample_kernel(SampleArgs a) {
  __shared__ uint32_t s_keys[kBuf];
  __shared__ int s_idx[kBuf];
  __shared__ int s_hist[256];
  __shared__ float s_red[32];
  __shared__ float s_redm[32];
  __shared__ int s_redi[32];
  __shared__ int s_count, s_tok;
  __shared__ uint32_t s_prefix;
  __shared__ int s_need;
  extern __shared__ uint32_t s_block[];  // blocked-id bitmask [ceil(V/32)], then the key cache [V]

  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int V = a.V;
  const float* lg = a.logits + row * a.ld;
  const uint32_t* seen = a.seen ? a.seen + row * a.seen_ld : nullptr;
  const int nwords = (V + 31) / 32;
  if (a.n_blocked > 0) {
    for (int i = tid; i < nwords; i += kThreads) s_block[i] = 0u;
    __syncthreads();
    for (int i = tid; i < a.n_blocked; i += kThreads) {
      const int id = a.blocked[i];
      if (id >= 0 && id < V) atomicOr(&s_block[id >> 5], 1u << (id & 31));
    }
    __syncthreads();
  }
  // the penalised / blocked value of element i whose raw logit is x
  auto adjusted_x = [&](float x, int i) -> float {
    if (a.n_blocked > 0 && ((s_block[i >> 5] >> (i & 31)) & 1u)) return -INFINITY;
    if (seen != nullptr && a.rep != 1.0f && ((seen[i >> 5] >> (i & 31)) & 1u))
      x = x > 0.f ? x / a.rep : x * a.rep;
    return x;
  };
  auto adjusted = [&](int i) -> float { return adjusted_x(lg[i], i); };
  // A thread walks its elements i = tid, tid + kThreads, ... in batches of
  // kBatch whose logits are all loaded before any is used, so the loads of a
  // batch are in flight together; the arithmetic keeps the element order.
  constexpr int kBatch = 8;

  // ---- pass 1: raw log-sum-exp, adjusted argmax (value desc, index asc)
  float rm = -INFINITY, rs = 0.f, bm = -INFINITY;
  int bi = 0x7fffffff;
  for (int i0 = tid; i0 < V; i0 += kBatch * kThreads) {
    float xs[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = i0 + u * kThreads;
      xs[u] = i < V ? lg[i] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int i = i0 + u * kThreads;
      if (i >= V) break;
      const float x = xs[u];
      if (x > rm) {
        rs = rs * expf(rm - x) + 1.f;
        rm = x;
      } else {
        rs += expf(x - rm);
      }
      const float w = adjusted_x(x, i);
      if (bi == 0x7fffffff || w > bm) {  // i grows per thread: first maximal index wins
        bm = w;
        bi = i;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, rm, o);
    const float os = __shfl_xor_sync(0xffffffffu, rs, o);
    const float nm = fmaxf(rm, om);
    rs = (rm == -INFINITY ? 0.f : rs * expf(rm - nm)) + (om == -INFINITY ? 0.f : os * expf(om - nm));
    rm = nm;
    const float ob = __shfl_xor_sync(0xffffffffu, bm, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > bm || (ob == bm && oi < bi)) {
      bm = ob;
      bi = oi;
    }
  }
  if (lane == 0) {
    s_red[warp] = rs;
    s_redm[warp] = rm;
    s_redi[warp] = bi;
    s_keys[warp] = __float_as_uint(bm);
  }
  __syncthreads();
  if (warp == 0) {
    rm = s_redm[lane];
    rs = s_red[lane];
    bm = __uint_as_float(s_keys[lane]);
    bi = s_redi[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, rm, o);
      const float os = __shfl_xor_sync(0xffffffffu, rs, o);
      const float nm = fmaxf(rm, om);
      rs = (rm == -INFINITY ? 0.f : rs * expf(rm - nm)) +
           (om == -INFINITY ? 0.f : os * expf(om - nm));
      rm = nm;
      const float ob = __shfl_xor_sync(0xffffffffu, bm, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > bm || (ob == bm && oi < bi)) {
        bm = ob;
        bi = oi;
      }
    }
    if (lane == 0) {
      s_redm[0] = rm + logf(rs);  // raw log-sum-exp
      s_redi[0] = bi;
      s_red[0] = bm;              // adjusted max
    }
  }
  __syncthreads();
  const float raw_lse = s_redm[0];
  const int argmax = s_redi[0];
  const float wmax = s_red[0];
  __syncthreads();

  int tok = argmax;
  const bool greedy = a.temp <= 1e-4f;
  const bool nucleus = a.top_p > 0.f && a.top_p < 1.f;
  const float u = a.uniforms ? a.uniforms[row] : 0.5f;
  if (!greedy && a.top_k <= 0 && !nucleus) {
    // ---- plain softmax over the vocabulary, inverse CDF in index order
    const float M = wmax / a.temp;
    const int chunk = (V + kThreads - 1) / kThreads;
    const int i0 = tid * chunk, i1 = min(V, i0 + chunk);
    float csum = 0.f;
    for (int i = i0; i < i1; ++i) csum += expf(adjusted(i) / a.temp - M);
    const float incl = block_inclusive_scan(csum, s_red);
    const float Z = s_red[31];
    const float target = u * Z;
    if (tid == 0) s_tok = -1;
    __syncthreads();
    const float excl = incl - csum;
    if (target >= excl && target < incl) {
      float c = excl;
      int pick = -1;
      for (int i = i0; i < i1; ++i) {
        c += expf(adjusted(i) / a.temp - M);
        if (target < c) {
          pick = i;
          break;
        }
      }
      if (pick < 0) pick = i1 - 1;
      s_tok = pick;
    }
    __syncthreads();
    tok = s_tok >= 0 ? s_tok : argmax;  // rounding past the end: the top token
  } else if (!greedy) {
    // ---- candidate set: the K largest adjusted/temp values
    const int K = a.top_k > 0 ? min(a.top_k, V) : min(V, kMaxCand);
    if (K > kMaxCand) {
      if (tid == 0) report_status(a.status, LLMYB_EUNSUPPORTED);
      tok = argmax;
    } else {
      if (tid == 0) {
        s_prefix = 0u;
        s_need = K;
      }
      // order keys of one batch of a thread's elements (see kBatch): formed
      // in the first pass into the row's key cache when the launch gave one,
      // read back by the later passes and the candidate collection (the same
      // bits as forming them again)
      uint32_t* s_kc = s_block + (a.n_blocked > 0 ? nwords : 0);
      auto batch_keys = [&](int i0, bool first, uint32_t (&kk)[kBatch]) {
        if (a.cache_keys && !first) {
#pragma unroll
          for (int u = 0; u < kBatch; ++u) {
            const int i = i0 + u * kThreads;
            kk[u] = i < V ? s_kc[i] : 0u;
          }
          return;
        }
        float xs[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int i = i0 + u * kThreads;
          xs[u] = i < V ? lg[i] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int i = i0 + u * kThreads;
          kk[u] = 0u;
          if (i < V) {
            kk[u] = order_key(adjusted_x(xs[u], i) / a.temp);
            if (a.cache_keys) s_kc[i] = kk[u];
          }
        }
      };
      uint32_t mask = 0u;
      for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += kThreads) s_hist[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix;
        for (int i0 = tid; i0 < V; i0 += kBatch * kThreads) {
          uint32_t kk[kBatch];
          batch_keys(i0, shift == 24, kk);
#pragma unroll
          for (int u = 0; u < kBatch; ++u)
            if (i0 + u * kThreads < V && (kk[u] & mask) == prefix)
              atomicAdd(&s_hist[(kk[u] >> shift) & 255u], 1);
        }
        __syncthreads();
        if (tid == 0) {
          int need = s_need, bucket = 255;
          for (; bucket > 0; --bucket) {
            if (s_hist[bucket] >= need) break;
            need -= s_hist[bucket];
          }
          s_need = need;
          s_prefix = prefix | (static_cast<uint32_t>(bucket) << shift);
        }
        mask |= 255u << shift;
        __syncthreads();
      }
      const uint32_t tau = s_prefix;  // key of the K-th largest value
      if (tid == 0) s_count = 0;
      __syncthreads();
      for (int i0 = tid; i0 < V; i0 += kBatch * kThreads) {
        uint32_t kk[kBatch];
        batch_keys(i0, false, kk);
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          const int i = i0 + u * kThreads;
          if (i < V && kk[u] >= tau) {
            const int slot = atomicAdd(&s_count, 1);
            if (slot < kBuf) {
              s_keys[slot] = kk[u];
              s_idx[slot] = i;
            }
          }
        }
      }
      __syncthreads();
      const int n = min(s_count, kBuf);
      // pad and bitonic-sort by (key desc, index asc)
      int P = 1;
      while (P < n) P <<= 1;
      for (int i = n + tid; i < P; i += kThreads) {
        s_keys[i] = 0u;
        s_idx[i] = 0x7fffffff;
      }
      __syncthreads();
      for (int size = 2; size <= P; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          for (int i = tid; i < P; i += kThreads) {
            const int j = i ^ stride;
            if (j > i) {
              const bool up = (i & size) == 0;  // "up" blocks sort descending
              const uint32_t ki = s_keys[i], kj = s_keys[j];
              const int ii = s_idx[i], ij = s_idx[j];
              const bool i_first = ki > kj || (ki == kj && ii < ij);
              if (up != i_first) {
                s_keys[i] = kj;
                s_keys[j] = ki;
                s_idx[i] = ij;
                s_idx[j] = ii;
              }
            }
          }
          __syncthreads();
        }
      }
      // ---- probabilities over the first K candidates (thread i <-> rank i)
      const bool mine = tid < K;
      const int cid = mine ? s_idx[tid] : 0;
      const float v = mine ? adjusted(cid) / a.temp : -INFINITY;
      const float vmax = wmax / a.temp;
      float e = mine ? expf(v - vmax) : 0.f;
      float Zref;
      if (a.top_k > 0) {
        Zref = block_sum(e, s_red);
      } else {
        // top-p alone: the reference normalises over the whole vocabulary
        float part = 0.f;
        for (int i = tid; i < V; i += kThreads) part += expf(adjusted(i) / a.temp - vmax);
        Zref = block_sum(part, s_red);
      }
      bool keep = mine;
      if (nucleus) {
        const float incl = block_inclusive_scan(e, s_red);
        const float excl = (incl - e) / Zref;
        keep = mine && (tid == 0 || !(excl > a.top_p));
        if (a.top_k <= 0 && tid == K - 1 && keep && K < V) report_status(a.status, LLMYB_EUNSUPPORTED);
      }
      const float ek = keep ? e : 0.f;
      const float cum = block_inclusive_scan(ek, s_red);
      const float Zk = s_red[31];
      if (tid == 0) {
        s_tok = -1;
        s_count = 0;
      }
      __syncthreads();
      const float target = u * Zk;
      if (keep && target < cum && target >= cum - ek) s_tok = cid;
      if (keep) atomicMax(&s_count, tid);  // highest kept rank
      __syncthreads();
      // u at the very top of the CDF (rounding): the last kept candidate
      if (tid == 0 && s_tok < 0) s_tok = s_idx[s_count];
      __syncthreads();
      tok = s_tok;
    }
  }
  if (tid == 0) {
    a.out_tok[row] = tok;
    if (a.out_logprob) a.out_logprob[row] = lg[tok] - raw_lse;
    if (a.update_seen && a.seen) atomicOr(a.seen + row * a.seen_ld + (tok >> 5), 1u << (tok & 31));
  }
}

}  // namespace
}  // namespace llmyb

using namespace llmyb;

// logits [B, V] fp32 (row stride ld); seen [B, ceil(V/32)] uint32 bitmask of
// previously generated ids (row stride seen_ld) or null; blocked ids or
// null; uniforms [B] in [0,1); outputs token ids [B] int64 and the raw
// log-probability of each token [B] (nullable).  With update_seen the chosen
// token is added to `seen`.
LLMYB_API int32_t llmyb_sample(const float* logits, int64_t ld, int32_t batch, int32_t vocab,
                               uint32_t* seen, int64_t seen_ld, float repetition_penalty,
                               const int32_t* blocked, int32_t n_blocked, float temperature,
                               int32_t top_k, float top_p, const float* uniforms,
                               int64_t* out_tokens, float* out_logprob, int32_t update_seen,
                               int32_t* dev_status, void* stream) {
  if (!logits || !out_tokens || batch < 0 || vocab <= 0 || n_blocked < 0) return LLMYB_EINVAL;
  if (n_blocked > 0 && !blocked) return LLMYB_EINVAL;
  if (temperature > 1e-4f && !uniforms) return LLMYB_EINVAL;
  if (top_k > kMaxCand) return LLMYB_EUNSUPPORTED;
  if (batch == 0) return LLMYB_OK;
  SampleArgs a;
  a.logits = logits;
  a.ld = ld;
  a.V = vocab;
  a.seen = seen;
  a.seen_ld = seen_ld;
  a.rep = repetition_penalty;
  a.blocked = blocked;
  a.n_blocked = n_blocked;
  a.temp = temperature;
  a.top_k = top_k;
  a.top_p = top_p;
  a.uniforms = uniforms;
  a.out_tok = out_tokens;
  a.out_logprob = out_logprob;
  a.update_seen = update_seen;
  a.status = dev_status;
  int dyn = n_blocked > 0 ? ((vocab + 31) / 32) * 4 : 0;
  // the key cache for the top-k passes when the row fits next to the static
  // buffers (vocabularies up to ~49K ids)
  constexpr int kDynLimit = 227 * 1024 - 20 * 1024;
  const bool topk_path = temperature > 1e-4f && (top_k > 0 || (top_p > 0.f && top_p < 1.f));
  a.cache_keys = topk_path && dyn + static_cast<int64_t>(vocab) * 4 <= kDynLimit ? 1 : 0;
  if (a.cache_keys) dyn += vocab * 4;
  if (dyn > 48 * 1024) {
    int32_t st = ensure_smem(sample_kernel, dyn);
    if (st) return st;
  }
  sample_kernel<<<batch, kThreads, dyn, static_cast<cudaStream_t>(stream)>>>(a);
  count_launch();
  return launch_status();
}
