/* llmyb — C ABI of the B200-native (sm_100a) LLMY looped hybrid block kernels.
 *
 * Conventions (after the reference engine's ABI, llmy_cuda/include/llmy.h:74-88
 * and llmy_cuda/include/kernels.h:8-11):
 *   - extern "C", plain C types, contiguous row-major DEVICE pointers;
 *   - `stream` is the caller's cudaStream_t (NULL = legacy default stream);
 *   - calls are asynchronous and never allocate or free: all outputs and
 *     scratch are caller-owned (scratch sizes come from the *_scratch_bytes
 *     queries);
 *   - every entry returns int32: 0 on success, a cudaError_t value on a CUDA
 *     failure (cudaErrorInvalidValue == 1 for bad arguments), LLMYB_EUNSUPPORTED
 *     for shapes a kernel does not implement (the reference returns silently
 *     in that case, llmy_cuda/src/kernels/router.cu:127-129);
 *   - `dev_status` (where present) is a caller-owned device int32, initially 0,
 *     that a kernel sets to LLMYB_ETIMEOUT if a bounded device-side wait gives
 *     up, or LLMYB_EINVAL if it meets an out-of-range index.
 * bf16 tensors are passed as `void*` holding __nv_bfloat16 data.
 */
#ifndef LLMYB_H
#define LLMYB_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LLMYB_OK 0
#define LLMYB_EINVAL 1
#define LLMYB_EUNSUPPORTED 1001
#define LLMYB_ETIMEOUT 1002

/* ------------------------------------------------------------------ router
 * Replaces the top-k/softmax of ContextAwareRouter.forward / forward_step
 * (model/layers/context_router.py:73-74, :132-133) and the native
 * router_topk kernel (llmy_cuda/src/kernels/router.cu:14-132, host
 * llmy::router_topk).  logits [N,E] fp32, optional bias [E] fp32 added before
 * selection; outputs idx [N,k] int64 (value desc, index asc) and prob [N,k]
 * fp32 = softmax of the k selected values.  E <= 256, k <= 32. */
int32_t llmyb_router_topk(const float* logits, const float* bias, int32_t n_tokens,
                          int32_t n_experts, int32_t top_k, int64_t* topk_idx, float* topk_prob,
                          void* stream);

/* Scratch bytes needed by llmyb_moe_plan / llmyb_route. */
int64_t llmyb_moe_plan_scratch_bytes(int32_t n_tokens, int32_t n_experts);

/* Dispatch plan of _moe_dispatch_fused (model/layers/moe.py:42-60) for routes
 * [N,k]: counts [E], offsets [E+1] (expert row ranges in permuted order),
 * tile_offsets [E+1] (prefix of ceil(count/tile_m)), perm_token [N*k],
 * perm_prob [N*k], route_pos [N*k] (permuted row of route t*k+s) and optional
 * sort_order [N*k] int64 (= torch.sort(flat_experts, stable=True) indices). */
int32_t llmyb_moe_plan(const int64_t* topk_idx, const float* topk_prob, int32_t n_tokens,
                       int32_t n_experts, int32_t top_k, int32_t tile_m, int32_t* expert_counts,
                       int32_t* expert_offsets, int32_t* tile_offsets, int32_t* perm_token,
                       float* perm_prob, int32_t* route_pos, int64_t* sort_order, void* scratch,
                       int32_t* dev_status, void* stream);

/* llmyb_router_topk followed by llmyb_moe_plan, fused into one launch for
 * N <= 256 (decode). */
int32_t llmyb_route(const float* logits, const float* bias, int32_t n_tokens, int32_t n_experts,
                    int32_t top_k, int32_t tile_m, int64_t* topk_idx, float* topk_prob,
                    int32_t* expert_counts, int32_t* expert_offsets, int32_t* tile_offsets,
                    int32_t* perm_token, float* perm_prob, int32_t* route_pos,
                    int64_t* sort_order, void* scratch, void* stream);

/* --------------------------------------------------------------- MoE FFN
 * Replaces _moe_dispatch_fused's expert math (model/layers/moe.py:68-81),
 * triton_moe_dispatch (runpod/kernels/triton_swiglu_moe.py:160-266) and the
 * native llmy_moe_selected_fp32 (llmy_cuda/include/llmy.h:83-88). */

/* Interleave w_gate/w_up [E,F,D] bf16 into w13 [E,2F,D]: every 256 rows hold
 * 128 gate rows then the matching 128 up rows.  F % 128 == 0, D % 64 == 0. */
int32_t llmyb_moe_pack_w13(const void* w_gate, const void* w_up, int32_t n_experts, int32_t ffn,
                           int32_t d_model, void* w13, void* stream);

/* Scratch bytes needed by llmyb_moe_grouped_swiglu. */
int64_t llmyb_moe_grouped_scratch_bytes(int32_t n_tokens, int32_t top_k, int32_t d_model,
                                        int32_t ffn);

/* out[t] = sum_s p[t,s] * W2[e] (silu(Wg[e] x_t) * (Wu[e] x_t)), bf16 in/out,
 * fp32 accumulation, tcgen05 grouped GEMM over the plan's expert groups.
 * x [N,D], w13 from llmyb_moe_pack_w13, w2 [E,D,F]; D % 256 == 0,
 * F % 128 == 0. */
int32_t llmyb_moe_grouped_swiglu(const void* x, int32_t n_tokens, int32_t d_model, int32_t top_k,
                                 const int32_t* perm_token, const float* perm_prob,
                                 const int32_t* route_pos, const int32_t* expert_offsets,
                                 const int32_t* tile_offsets, int32_t n_experts, const void* w13,
                                 const void* w2, int32_t ffn, void* scratch, void* out,
                                 int32_t* dev_status, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LLMYB_H */
