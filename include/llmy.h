/* The reference engine's C API, served natively by libllmyb.so.
 *
 * Same entry points, argument meanings and opaque handles as the reference
 * engine's header (llmy_cuda/include/llmy.h:27-88, implemented there in
 * llmy_cuda/src/llmy.cpp and model.cpp:1955-1972), so a C or ctypes caller of
 * the reference switches by loading hybrid_llm_b200/lib/libllmyb.so instead
 * of libllmy.so.  No Python runs behind these calls: the `.llmy` checkpoint is
 * mapped and uploaded by C++ code, and every token is one cooperative launch
 * of the persistent decode step (llmyb_decode_persistent in llmyb.h).
 *
 * Served models: what the persistent step serves (one plain residual stream
 * with mhc.enabled=0; recurrent_layout of csa_moe / gdn_moe blocks without
 * stem or tail blocks; CSA local attention with index_head_dim 64 and the
 * remote branch off; GDN with key = value head dim 64 and conv_kernel 4;
 * routed experts without shared experts or the router's context; no loop
 * memory, no adaptive halting).  llmy_load prints "[llmy_load] <reason>" to
 * stderr and returns NULL for anything else; the Python engine
 * (hybrid_llm_b200.engine) serves the full feature set with the same calls.
 *
 * The engine runs on the CUDA device current when llmy_load is called, on
 * the legacy default stream, and each forward returns after its logits are
 * written (as the reference's does).  A device-side failure of a step
 * (LLMYB_ETIMEOUT from a grid barrier, a launch error) is printed as
 * "[llmy_decode] ..." / "[llmy_prefill] ..." to stderr. */
#ifndef LLMY_H
#define LLMY_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct llmy_model llmy_model;
typedef struct llmy_state llmy_state;

/* Model lifecycle (llmy.h:31-32). */
llmy_model* llmy_load(const char* path);
void llmy_free(llmy_model* m);

/* Introspection (llmy.h:35-41).  llmy_max_loops is the loop count (adaptive
 * halting is not served); llmy_mhc_streams is 1.  llmy_set_num_loops /
 * llmy_set_fixed_loops set the default loop count of prefill and decode and
 * decode's upper bound (n < 1 is ignored); a state holds as many loops as the
 * model's count when the state was created. */
int32_t llmy_vocab_size(const llmy_model* m);
int32_t llmy_d_model(const llmy_model* m);
int32_t llmy_num_loops(const llmy_model* m);
int32_t llmy_max_loops(const llmy_model* m);
int32_t llmy_mhc_streams(const llmy_model* m);
void llmy_set_num_loops(llmy_model* m, int32_t n);
void llmy_set_fixed_loops(llmy_model* m, int32_t n);

/* State lifecycle (llmy.h:44-46): batch 1; reset zeroes every recurrent
 * state tensor and the position. */
llmy_state* llmy_state_new(llmy_model* m);
void llmy_state_free(llmy_state* s);
void llmy_state_reset(llmy_state* s);

/* Forward passes (llmy.h:51-59).  logits_out: vocab_size floats on the host
 * or the device (NULL skips the copy).  Prefill runs tokens[0:n_tokens] one
 * step each at positions 0..n_tokens-1 and writes the last token's logits;
 * decode runs `token` at absolute `position` with num_loops loops (<= 0: the
 * model default; larger values are capped at it). */
void llmy_prefill(llmy_model* m, llmy_state* s, const int32_t* tokens, int32_t n_tokens,
                  float* logits_out);
void llmy_decode(llmy_model* m, llmy_state* s, int32_t token, int32_t position,
                 int32_t num_loops, float* logits_out);

/* Host sampler (llmy.h:64-68): llmyb_engine_sample. */
int32_t llmy_sample(const float* logits, int32_t vocab_size, float temperature, int32_t top_k,
                    float top_p, float repetition_penalty, const int32_t* recent_tokens,
                    int32_t n_recent, uint64_t* rng_state);

/* Diagnostics (llmy.h:71-72). */
int32_t llmy_last_executed_loops(const llmy_state* s);
void llmy_sync(void);

/* Extension (not in the reference API): the experts the last step routed
 * to, for routing-aware parity checks.  Copies the last llmy_decode's (or
 * the last prompt token's) choices, [loops][blocks][top_k] in loop-major
 * order, into idx (and prob, nullable; host or device pointers) and returns
 * their count, or a negative status (-1 for a null state / idx or a
 * capacity below the count). */
int32_t llmyb_engine_routes(const llmy_state* s, int32_t* idx, float* prob, int32_t capacity);

/* Device operators (llmy.h:76-88): llmyb_mhc_sinkhorn4 and
 * llmyb_moe_selected_fp32. */
int32_t llmy_mhc_sinkhorn4(const float* input, float* output, int32_t matrices,
                           int32_t iterations, void* stream);
int32_t llmy_moe_selected_fp32(const float* x, const int64_t* idx, const float* prob,
                               const float* gate_up, const float* down, float* activation,
                               float* route_output, float* out, int32_t D, int32_t H, int32_t E,
                               int32_t k, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LLMY_H */
