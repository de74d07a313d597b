// The reference engine's host-side sampler (llmy_cuda/include/llmy.h:62-68,
// llmy_cuda/src/llmy.cpp:132-202): one row of host logits, single-precision
// arithmetic, a caller-owned xorshift64 state.  Its rules differ from the
// Python sampler that llmyb_sample follows (sampling.cu), so it has its own
// entry point:
//   - repetition penalty applied once per entry of `recent` (a repeated id is
//     penalised again; ids outside the vocabulary are skipped);
//   - top_k <= 0 or > vocab means the whole vocabulary, capped at 256;
//   - temperature <= 0 (or NaN) is greedy over the top-k order;
//   - top-p keeps the shortest prefix whose cumulative probability reaches
//     top_p (inclusive), for 0 < top_p < 1;
//   - u = (state >> 11) / 2^53 after one xorshift64 (13, 7, 17) step, drawn
//     against the running single-precision cumulative sum.
// Equal logits are ordered by index (the reference's partial sort leaves their
// order open).  Host code only: the engine API hands it host logits.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <numeric>
#include <vector>

#include "common.cuh"

namespace {

uint64_t xorshift64(uint64_t s) {
  s ^= s << 13;
  s ^= s >> 7;
  s ^= s << 17;
  return s;
}

}  // namespace

LLMYB_API int32_t llmyb_engine_sample(const float* logits, int32_t vocab, float temperature,
                                      int32_t top_k, float top_p, float repetition_penalty,
                                      const int32_t* recent, int32_t n_recent,
                                      uint64_t* rng_state) {
  if (vocab <= 0) return 0;
  if (logits == nullptr || rng_state == nullptr || (n_recent > 0 && recent == nullptr)) return -1;
  const int32_t k = std::min<int32_t>(top_k <= 0 || top_k > vocab ? vocab : top_k, 256);

  std::vector<float> w(logits, logits + vocab);
  if (repetition_penalty != 1.0f) {
    for (int32_t i = 0; i < n_recent; ++i) {
      const int32_t id = recent[i];
      if (id < 0 || id >= vocab) continue;
      w[id] = w[id] > 0.0f ? w[id] / repetition_penalty : w[id] * repetition_penalty;
    }
  }

  std::vector<int32_t> order(vocab);
  std::iota(order.begin(), order.end(), 0);
  std::partial_sort(order.begin(), order.begin() + k, order.end(), [&](int32_t a, int32_t b) {
    return w[a] > w[b] || (w[a] == w[b] && a < b);
  });
  if (!(temperature > 0.0f)) return order[0];

  std::vector<float> p(k);
  const float top = w[order[0]];
  float total = 0.0f;
  for (int32_t i = 0; i < k; ++i) {
    p[i] = std::exp((w[order[i]] - top) / temperature);
    total += p[i];
  }
  for (int32_t i = 0; i < k; ++i) p[i] /= total;

  int32_t keep = k;
  if (top_p > 0.0f && top_p < 1.0f) {
    float cum = 0.0f;
    for (int32_t i = 0; i < k; ++i) {
      cum += p[i];
      if (cum >= top_p) {
        keep = i + 1;
        break;
      }
    }
  }
  float kept = 0.0f;
  for (int32_t i = 0; i < keep; ++i) kept += p[i];
  for (int32_t i = 0; i < keep; ++i) p[i] /= kept;

  const uint64_t s = xorshift64(*rng_state);
  *rng_state = s;
  const double u = static_cast<double>(s >> 11) / static_cast<double>(1ull << 53);
  float cum = 0.0f;
  for (int32_t i = 0; i < keep; ++i) {
    cum += p[i];
    if (u < cum) return order[i];
  }
  return order[keep - 1];
}
