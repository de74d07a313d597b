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

/* The prefill router of ContextAwareRouter without the local context
 * (model/layers/context_router.py:62-65) from the FFN-normalised rows
 * m [N, D] fp32: r = RMSNorm(m) * router_norm, logits = w_router [E, D] . r
 * (fp32; written to logits_out [N, E] when it is not null), then top-k +
 * softmax (+ bias before selection, nullable) and the dispatch plan of
 * llmyb_moe_plan.  D % 4 == 0, D <= 1024, 16-byte aligned m / norm / router;
 * scratch (llmyb_moe_plan_scratch_bytes) is only read when N*k > 2048. */
int32_t llmyb_route_norm(const float* m, int32_t n_tokens, int32_t d_model,
                         const float* router_norm, const float* w_router, float eps,
                         const float* bias, int32_t n_experts, int32_t top_k, int32_t tile_m,
                         float* logits_out, int64_t* topk_idx, float* topk_prob,
                         int32_t* expert_counts, int32_t* expert_offsets, int32_t* tile_offsets,
                         int32_t* perm_token, float* perm_prob, int32_t* route_pos,
                         int64_t* sort_order, void* scratch, void* stream);

/* llmyb_route for callers that cannot allocate device memory (a host that
 * hands the library only its input/output buffers, a server whose memory is
 * reserved up front, code running while another allocator owns the heap).
 * No counterpart in the reference.  Same arguments and results as
 * llmyb_route without `scratch`: the expert histogram lives in a fixed
 * 256 KiB array inside the library (held on every device that loads the
 * library until exit).  Calls needing more than
 * llmyb_route_noalloc_max_scratch_ints() ints (ceil(N/256)*E + 1) return
 * LLMYB_EUNSUPPORTED.  All calls on a device share the array, so calls that
 * overlap on the GPU race; each call rewrites it fully before reading it.
 * The first call on a device looks up the array's address: make it before
 * capturing a CUDA graph that uses this entry point. */
int32_t llmyb_route_noalloc(const float* logits, const float* bias, int32_t n_tokens,
                            int32_t n_experts, int32_t top_k, int32_t tile_m, int64_t* topk_idx,
                            float* topk_prob, int32_t* expert_counts, int32_t* expert_offsets,
                            int32_t* tile_offsets, int32_t* perm_token, float* perm_prob,
                            int32_t* route_pos, int64_t* sort_order, void* stream);

/* Capacity of llmyb_route_noalloc's fixed scratch array, in ints. */
int64_t llmyb_route_noalloc_max_scratch_ints(void);

/* Decode-step router fused with what precedes it in PhysicalBlock.forward_step
 * (model/model.py:214-241): streams [N,D] fp32 += delta [N,D] bf16
 * (nullable); m = RMSNorm(streams) * ffn_norm -> m_bf [N,D] bf16 (expert
 * input); logits = w_router [E,D] . (RMSNorm(m) * router_norm) in fp32;
 * then top-k/softmax and the plan as llmyb_route.  One CTA: N*E <= 256,
 * N*k <= 2048, D % 4 == 0. */
int32_t llmyb_route_fused(float* streams, const void* delta, int32_t n_tokens, int32_t d_model,
                          const float* ffn_norm, const float* router_norm, const float* w_router,
                          float eps, int32_t n_experts, int32_t top_k, int32_t tile_m, void* m_bf,
                          int64_t* topk_idx, float* topk_prob, int32_t* expert_counts,
                          int32_t* expert_offsets, int32_t* tile_offsets, int32_t* perm_token,
                          float* perm_prob, int32_t* route_pos, void* stream);

/* llmyb_route_fused for decode batches of any size up to N = 256 (N*k <=
 * 2048, E <= 256, D % 4 == 0, D <= 8192) in three launches: the router input
 * of each token (one CTA per token), the logits (one warp per (token,
 * expert) pair), then top-k, softmax and the plan in one CTA.
 * logits_scratch holds N*(D+E) fp32 (router inputs, then logits).  Results
 * are bit-identical to llmyb_route_fused wherever both apply. */
int32_t llmyb_route_decode(float* streams, const void* delta, int32_t n_tokens, int32_t d_model,
                           const float* ffn_norm, const float* router_norm,
                           const float* w_router, float eps, int32_t n_experts, int32_t top_k,
                           int32_t tile_m, void* m_bf, float* logits_scratch, int64_t* topk_idx,
                           float* topk_prob, int32_t* expert_counts, int32_t* expert_offsets,
                           int32_t* tile_offsets, int32_t* perm_token, float* perm_prob,
                           int32_t* route_pos, void* stream);

/* Shared experts (model/layers/moe.py:185-198 prefill, :221-234 decode, where
 * SparseMoE adds sum_s SwiGLU_s(x) / sqrt(S) to the routed output) as plan
 * experts E..E+S-1: a plan over E routed experts (any llmyb_route* output)
 * is written extended into the out_* buffers ([N, k+S] slots, E+S counts,
 * E+S+1 offsets, N*(k+S) rows).  Every token gets a slot per shared expert
 * with probability 1/sqrt(S); the shared rows follow the routed ones in plan
 * order (row N*k + s*N + t).  The expert entry points then run routed and
 * shared experts in one call over weights stacked routed first, then shared,
 * and the routed combine sums k+S rows per token.  One launch, no host sync. */
int32_t llmyb_plan_append_shared(int32_t n_tokens, int32_t n_experts, int32_t top_k,
                                 int32_t n_shared, int32_t tile_m, const int64_t* topk_idx,
                                 const float* topk_prob, const int32_t* expert_counts,
                                 const int32_t* expert_offsets, const int32_t* tile_offsets,
                                 const int32_t* perm_token, const float* perm_prob,
                                 const int32_t* route_pos, int64_t* out_topk_idx,
                                 float* out_topk_prob, int32_t* out_counts, int32_t* out_offsets,
                                 int32_t* out_tile_offsets, int32_t* out_perm_token,
                                 float* out_perm_prob, int32_t* out_route_pos, void* stream);

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
 * F % 128 == 0.  tile_m is the plan's tile size: 256 selects the CTA-pair
 * kernel (tcgen05.mma.cta_group::2, 256x256 tiles), 128 the single-CTA one. */
int32_t llmyb_moe_grouped_swiglu(const void* x, int32_t n_tokens, int32_t d_model, int32_t top_k,
                                 const int32_t* perm_token, const float* perm_prob,
                                 const int32_t* route_pos, const int32_t* expert_offsets,
                                 const int32_t* tile_offsets, int32_t tile_m, int32_t n_experts,
                                 const void* w13, const void* w2, int32_t ffn, void* scratch,
                                 void* out, int32_t* dev_status, void* stream);

/* The gather and the two grouped GEMMs of llmyb_moe_grouped_swiglu without its
 * combine, over an explicit plan: y_out[out_row ? out_row[pos] : pos] =
 * perm_prob[pos] * expert(x[perm_token[pos]]) for pos < expert_offsets[E]
 * (read on the device; n_rows >= that count bounds the plan).  tile_offsets
 * counts tile_m-row tiles per expert (tile_m 128 or 256).  scratch: at least
 * llmyb_moe_grouped_scratch_bytes(n_rows, 1, D, F) bytes.  The tensor-core
 * path for decode batches with several rows per expert (its outputs feed
 * llmyb_add_rmsnorm_routed or the expert-parallel return segments).  No
 * counterpart in the reference (moe.py:29-82 always combines). */
int32_t llmyb_moe_grouped_experts_to(const void* x, int32_t d_model, int32_t n_rows,
                                     const int32_t* perm_token, const float* perm_prob,
                                     const int32_t* expert_offsets, const int32_t* tile_offsets,
                                     int32_t tile_m, int32_t n_experts, const void* w13,
                                     const void* w2, int32_t ffn, void* scratch, void* y_out,
                                     const int32_t* out_row, int32_t* dev_status, void* stream);

/* Scratch bytes needed by llmyb_moe_decode_swiglu. */
int64_t llmyb_moe_decode_scratch_bytes(int32_t n_tokens, int32_t top_k, int32_t d_model,
                                       int32_t ffn);

/* Same contract as llmyb_moe_grouped_swiglu for small token counts (decode):
 * streams every routed expert's weights once (CUDA-core dot products, token
 * rows staged in shared memory); experts with no routed rows read nothing.
 * D, F multiples of 128, at most 2048. */
int32_t llmyb_moe_decode_swiglu(const void* x, int32_t n_tokens, int32_t d_model, int32_t top_k,
                                const int32_t* perm_token, const float* perm_prob,
                                const int32_t* route_pos, const int32_t* expert_offsets,
                                int32_t n_experts, const void* w13, const void* w2, int32_t ffn,
                                void* scratch, void* out, void* stream);

/* The two expert kernels of llmyb_moe_decode_swiglu without its combine:
 * y_rows [N*k, D] bf16 gets p * expert(x) for each route in plan order
 * (summed per token by llmyb_add_rmsnorm_routed); h_scratch holds [N*k, F]
 * bf16. */
int32_t llmyb_moe_decode_experts(const void* x, int32_t n_tokens, int32_t d_model, int32_t top_k,
                                 const int32_t* perm_token, const float* perm_prob,
                                 const int32_t* expert_offsets, int32_t n_experts,
                                 const void* w13, const void* w2, int32_t ffn, void* h_scratch,
                                 void* y_rows, void* stream);

/* llmyb_moe_decode_experts over an explicit plan of n_rows positions (top_k 1)
 * whose outputs go to y_out[out_row[pos]] instead of y_out[pos]: the
 * expert-parallel path writes each expert output straight into the return
 * segment of the rank that sent the row.  h_scratch holds [n_rows, F] bf16.
 * No counterpart in the reference (its experts all run on one device). */
int32_t llmyb_moe_decode_experts_to(const void* x, int32_t n_rows, int32_t d_model,
                                    const int32_t* perm_token, const float* perm_prob,
                                    const int32_t* expert_offsets, int32_t n_experts,
                                    const void* w13, const void* w2, int32_t ffn, void* h_scratch,
                                    void* y_out, const int32_t* out_row, void* stream);

/* -------------------------------------------------- expert parallelism
 * No counterpart in the reference: it runs model/layers/moe.py:29-82 with all
 * experts on one device.  These deploy the same routed SwiGLU over W ranks,
 * rank q owning experts [q*El, (q+1)*El) (El = E / W).  Per MoE call:
 *   llmyb_ep_dispatch_pack  -> all-to-all of W equal dispatch segments
 *   llmyb_ep_recv_plan      -> llmyb_moe_decode_experts_to (into return segments)
 *   all-to-all of W equal return segments -> llmyb_add_rmsnorm_routed with
 *   ret_route_pos (the combine).
 * A dispatch segment is H + C bf16 rows of D elements: header rows [0, H)
 * hold int32 counts[El] then fp32 probs[C]; rows [H, H+C) the routed token
 * rows in plan (expert) order.  A return segment is C rows.  C (capacity) is
 * at least the sender's route count N*k. */
int32_t llmyb_ep_header_rows(int32_t experts_per_rank, int32_t capacity, int32_t d_model);

/* Pack the W dispatch segments into send [W, H+C, D] from the local plan of
 * llmyb_route (offsets [E+1], perm_token, perm_prob, route_pos [n_routes]);
 * ret_route_pos [n_routes] gets the row of the return buffer [W*C, D] that
 * will hold each route's expert output. */
int32_t llmyb_ep_dispatch_pack(const void* x, int32_t d_model, const int32_t* offsets,
                               const int32_t* perm_token, const float* perm_prob,
                               const int32_t* route_pos, int32_t n_routes, int32_t n_experts,
                               int32_t world, int32_t capacity, void* send,
                               int32_t* ret_route_pos, void* stream);

/* Expert-ordered plan over the received segments recv [W, H+C, D]:
 * offsets_l [El+1]; tile_offsets_l [El+1] (prefix of ceil(rows / tile_m)
 * per expert, for llmyb_moe_grouped_experts_to; nullable); perm_token_l (row
 * of recv viewed as [W*(H+C), D]), perm_prob_l and out_row (row of the
 * return buffer [W*C, D]) [W*C], the first offsets_l[El] entries valid.
 * Rows of one expert are ordered by source rank, then by the source's plan
 * order.  W <= 64, El <= 256, W*El <= 4096. */
int32_t llmyb_ep_recv_plan(const void* recv, int32_t d_model, int32_t world, int32_t capacity,
                           int32_t experts_per_rank, int32_t tile_m, int32_t* offsets_l,
                           int32_t* tile_offsets_l, int32_t* perm_token_l, float* perm_prob_l,
                           int32_t* out_row, const int32_t* wait_flags, const int32_t* sync,
                           int32_t* dev_status, void* stream);

/* Peer-memory exchange (one process per GPU on one node, W <= 8): each rank
 * allocates one buffer the others map with CUDA IPC - its receive segments,
 * its return segments and two flag arrays of W int32 (dispatch, return).
 * Sends are plain stores over NVLink; the last CTA of a send stores the
 * exchange round into every peer's flag (release, system scope); receivers
 * wait on their own flags (acquire, bounded by one second: LLMYB_ETIMEOUT).
 * sync = int32[3] per rank (round, two CTA tickets), zero-initialised.
 * With wait_flags, llmyb_ep_recv_plan first waits for the dispatch flags; a
 * header whose counts exceed the capacity is treated as empty
 * (LLMYB_EINVAL in dev_status). */
int32_t llmyb_ep_shared_alloc(int64_t bytes, void** dev_ptr, void* handle);
int32_t llmyb_ep_shared_open(const void* handle, void** dev_ptr);
int32_t llmyb_ep_shared_close(void* dev_ptr);
int32_t llmyb_ep_shared_free(void* dev_ptr);

/* llmyb_ep_dispatch_pack into the peers' receive buffers: peer_segs[q] is
 * this rank's segment in rank q's buffer, peer_flags[q] this rank's dispatch
 * flag there (host arrays of W device pointers).  Starts a new round. */
int32_t llmyb_ep_dispatch_p2p(const void* x, int32_t d_model, const int32_t* offsets,
                              const int32_t* perm_token, const float* perm_prob,
                              const int32_t* route_pos, int32_t n_routes, int32_t n_experts,
                              int32_t world, int32_t capacity, void* const* peer_segs,
                              int32_t* const* peer_flags, int32_t* sync, int32_t* ret_route_pos,
                              void* stream);

/* Return push: the expert outputs of the rows rank q sent (ret_send rows
 * [q*C, q*C + n_q), n_q from q's header in recv) into peer_segs[q], then the
 * round into peer_flags[q] (this rank's return flag there). */
int32_t llmyb_ep_return_p2p(const void* ret_send, const void* recv, int32_t d_model,
                            int32_t world, int32_t capacity, int32_t experts_per_rank,
                            void* const* peer_segs, int32_t* const* peer_flags, int32_t* sync,
                            void* stream);

/* Bounded wait (one CTA) until flags[0..W) hold the current round.  After
 * limit_ns (0: one second; capped at one second) it records LLMYB_ETIMEOUT in
 * dev_status and returns: a peer that never publishes shows up as an error
 * the host reads, not as a hung kernel. */
int32_t llmyb_ep_wait(const int32_t* flags, int32_t world, const int32_t* sync,
                      int32_t* dev_status, int64_t limit_ns, void* stream);

/* ------------------------------------------------------ gated delta rule
 * Replaces GatedDeltaNet's recurrence (model/layers/gated_deltanet.py:140-149
 * and the seams _triton_gdn_scan/_triton_gdn_step at :179-235), the Triton
 * kernels (sample_standalone.py:435-531) and the native gdn_step /
 * gdn_conv_gate kernels (llmy_cuda/src/kernels/gdn.cu:22-145).
 * Token-major bf16 inputs are given as (pointer, stride): element (token, h, i)
 * lives at ptr[token*stride + h*dim + i], so q/k/v/gate/beta may be views into
 * one fused projection.  alpha = sigmoid(decay_logit[h]) (reference), or
 * exp(log_alpha[token, h]) when log_alpha is non-null.  K, V in {64, 128}. */

/* In place on proj [N, width] = [q (H*K) | k (H*K) | v (H*V) | gate (H*V) | beta (H)]:
 * q,k L2-normalised per head, gate = sigmoid(gate), beta = sigmoid(beta + bias). */
int32_t llmyb_gdn_activate(void* proj, int64_t n_tokens, int32_t width, int32_t heads,
                           int32_t key_dim, int32_t value_dim, const float* beta_bias,
                           void* stream);

/* One token per row (decode): state [B,H,K,V] fp32 updated in place;
 * out (row stride out_stride) = ((S^T q) rounded to bf16) * gate.  With
 * raw_inputs != 0 q/k/gate/beta are the raw projections and the kernel
 * applies the activations of llmyb_gdn_activate (beta_bias [H] fp32). */
int32_t llmyb_gdn_step(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                       const void* v, int64_t v_stride, const void* gate, int64_t gate_stride,
                       const void* beta, int64_t beta_stride, const float* decay_logit,
                       const float* log_alpha, const uint8_t* reset, int32_t batch,
                       int32_t heads, int32_t key_dim, int32_t value_dim, float* state,
                       void* out, int64_t out_stride, int32_t raw_inputs,
                       const float* beta_bias, void* stream);

/* Scratch bytes needed by llmyb_gdn_prefill. */
int64_t llmyb_gdn_prefill_scratch_bytes(int32_t batch, int32_t seq, int32_t heads,
                                        int32_t key_dim, int32_t value_dim);

/* Chunked (C = 64) scan over [B, T] tokens with resets: state [B,H,K,V] fp32
 * holds the initial state on entry and the final state on exit.  For K = 128
 * (16-byte aligned gate/out/state/k rows) the scan runs on tcgen05 with the
 * state in registers of its state warps; dev_status (nullable) receives
 * LLMYB_ETIMEOUT if one of its pipeline waits expires. */
int32_t llmyb_gdn_prefill(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                          const void* v, int64_t v_stride, const void* gate, int64_t gate_stride,
                          const void* beta, int64_t beta_stride, const float* decay_logit,
                          const float* log_alpha, const uint8_t* reset, int32_t batch,
                          int32_t seq, int32_t heads, int32_t key_dim, int32_t value_dim,
                          float* state, void* out, int64_t out_stride, void* scratch,
                          int32_t* dev_status, void* stream);

/* GDN epilogue (gated_deltanet.py:254-276): y = y_proj * sigmoid(conv4(x)),
 * depthwise causal conv over the block input x [B,T,D] with weight [D,4]
 * fp32; history [B,3,D] (decode) or null (prefill, zero left padding).  The
 * result goes to `out`, or is added into `residual` when that is non-null;
 * roll_history advances the history by the last inputs
 * (model/model.py:283-289). */
int32_t llmyb_gdn_conv_gate(const void* x, const void* y_proj, const float* conv_w,
                            void* history, const uint8_t* reset, int32_t batch, int32_t seq,
                            int32_t d_model, void* out, void* residual, int32_t roll_history,
                            void* stream);

/* The decode conv history a prompt leaves (model/model.py:180-182): history
 * [B,3,D] = the last three rows of x [B,T,D] per batch row, zero rows where
 * T < 3.  Replaces the reference's slice assignment of the history buffer. */
int32_t llmyb_gdn_history_set(const void* x, void* history, int32_t batch, int32_t seq,
                              int32_t d_model, void* stream);

/* ------------------------------------------------------ banded attention
 * Replaces fused_banded_local_attention / triton_banded_local_attention
 * (sample_standalone.py:70-85, :253-409), the CSA local branch
 * (model/layers/csa.py:39-75, decode :172-206) and the native
 * banded_attn_kernel / local_attn_decode_kernel
 * (llmy_cuda/src/kernels/attn.cu:17-229).  Key j is visible from query t iff
 * j <= t and t - j < window.  Token-major bf16 tensors with token strides. */

/* Per-head attention: q,k [B*T, H*D], v with v_heads in {1, H} heads of
 * width D, out [B*T, H*D]; D in {64, 128}; scale (> 0) multiplies q.k.  tcgen05
 * kernel (128-query tiles, TMA-staged K/V, only in-band key blocks);
 * dev_status (nullable) receives LLMYB_ETIMEOUT if a pipeline wait expires. */
int32_t llmyb_banded_attention(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                               const void* v, int64_t v_stride, int32_t v_heads, int32_t batch,
                               int32_t seq, int32_t heads, int32_t head_dim, int32_t window,
                               float scale, void* out, int64_t out_stride, int32_t* dev_status,
                               void* stream);

/* Scratch bytes needed by llmyb_csa_local_prefill: the per-head row max /
 * sum [B, T, H] fp32, then B * ceil(T/128) * nb head-averaged probability
 * tiles of 128 x 128 bf16, nb = min(ceil(T/128), ceil((W-1)/128) + 1) with
 * W = min(window, T). */
int64_t llmyb_csa_prefill_scratch_bytes(int32_t batch, int32_t seq, int32_t heads,
                                        int32_t window);

/* CSA local branch, prefill: head-averaged probabilities times the shared
 * value stream v [B*T, D]; out [B*T, D].  Window = min(window, T) as
 * csa.py:42 does.  Head dim in {64, 128}, D % 64 == 0; with D % 128 == 0 the
 * score and PV products run on tcgen05 (the probability tiles go through
 * scratch); dev_status (nullable) gets LLMYB_ETIMEOUT if one of their
 * bounded waits runs out. */
int32_t llmyb_csa_local_prefill(const void* q, int64_t q_stride, const void* k, int64_t k_stride,
                                const void* v, int64_t v_stride, int32_t batch, int32_t seq,
                                int32_t heads, int32_t head_dim, int32_t d_model, int32_t window,
                                void* out, int64_t out_stride, void* scratch,
                                int32_t* dev_status, void* stream);

/* CSA local branch, decode: q/knew [B, H*DH], vnew [B, D]; ring caches
 * kcache [B, window, H*DH], vcache [B, window, D] hold token p at slot
 * p % window; positions[b] is the new token's position.  Writes the new K/V
 * into the ring and attends over the last min(positions[b]+1, window)
 * tokens.  dev_status (nullable) gets LLMYB_ETIMEOUT if a staged copy of
 * the ring rows (small batches) does not arrive within a second. */
int32_t llmyb_csa_local_decode(const void* q, int64_t q_stride, const void* knew,
                               int64_t knew_stride, const void* vnew, int64_t vnew_stride,
                               void* kcache, void* vcache, const int32_t* positions,
                               int32_t batch, int32_t heads, int32_t head_dim, int32_t d_model,
                               int32_t window, void* out, int64_t out_stride,
                               int32_t* dev_status, void* stream);

/* The ring caches a prompt leaves for decode (the cache layout of
 * csa.py:208-258): kcache [B, window, k_width] and vcache [B, window, v_width]
 * receive token p of the last min(seq, window) tokens of k [B*seq, k_width]
 * and v [B*seq, v_width] (token strides k_stride, v_stride) at slot
 * p % window; the other slots keep their contents.  Replaces the
 * reference's indexed assignment of the cache rows. */
int32_t llmyb_csa_ring_write(const void* k, int64_t k_stride, const void* v, int64_t v_stride,
                             int32_t batch, int32_t seq, int32_t k_width, int32_t v_width,
                             void* kcache, void* vcache, int32_t window, void* stream);

/* ------------------------------------------------------------- diagnostics
 * Number of kernel launches this library has issued since it was loaded
 * (host-side count; a captured CUDA graph replays the launches counted while
 * it was captured).  No counterpart in the reference. */
int64_t llmyb_launch_count(void);

/* Zero n_regions device regions in one launch: regions is a device array of
 * n_regions (address, bytes) int64 pairs, max_bytes the largest size (it
 * sizes the grid).  Used to clear a whole recurrent state (every GDN state,
 * conv history, ring cache and position counter) as a fresh conversation
 * (recurrent_state.py:218-244 clears row by row); no reference counterpart. */
int32_t llmyb_zero_regions(const int64_t* regions, int32_t n_regions, int64_t max_bytes,
                           void* stream);

/* --------------------------------------------------------- residual stream
 * PhysicalBlock's residual glue with mHC disabled (model/model.py:119-126,
 * :442-444) and RMSNorm (model/layers/norms.py:13-16).  The residual stream
 * is fp32 (as under the reference's bf16 autocast); sub-layer outputs bf16. */

/* streams[n] = float(table[ids[n]]) + stream_seed (nullable); out-of-range
 * ids set dev_status to LLMYB_EINVAL and read row 0. */
int32_t llmyb_embed(const int64_t* ids, int64_t n_tokens, const void* table, int64_t vocab,
                    int32_t d_model, const float* stream_seed, float* streams,
                    int32_t* dev_status, void* stream);

/* streams (fp32) += delta (bf16, nullable), then
 * y = streams * rsqrt(mean(streams^2) + eps) * weight (normalize != 0) or
 * y = streams (normalize == 0), written to out_bf16 and/or out_f32. */
int32_t llmyb_add_rmsnorm(float* streams, const void* delta, int64_t n_tokens, int32_t d_model,
                          const float* weight, float eps, int32_t normalize, void* out_bf16,
                          float* out_f32, void* stream);

/* llmyb_add_rmsnorm whose delta for row n is the sum of the k routed expert
 * rows y_rows[route_pos[n*k + s]] (the MoE combine fused into the residual
 * add; y_rows from llmyb_moe_decode_experts). */
int32_t llmyb_add_rmsnorm_routed(float* streams, const void* y_rows, const int32_t* route_pos,
                                 int32_t top_k, int64_t n_tokens, int32_t d_model,
                                 const float* weight, float eps, int32_t normalize,
                                 void* out_bf16, float* out_f32, void* stream);

/* The FFN norm and the router's input norm of a prompt's MoE sub-layer in one
 * pass (SparseMoE input m = norms.py:13-16 RMSNorm of the residual;
 * ContextAwareRouter local = RMSNorm(m), context_router.py:62):
 * streams (fp32) += delta (bf16, nullable); m = RMSNorm(streams) * ffn_weight
 * into out_bf16 (bf16, nullable); router_in = RMSNorm(m) * router_weight (fp32),
 * bit-identical to llmyb_add_rmsnorm with out_f32 followed by llmyb_add_rmsnorm
 * of that fp32 row.  D % 8 == 0, D <= 8192, 16-byte aligned rows, else
 * LLMYB_EUNSUPPORTED. */
int32_t llmyb_add_rmsnorm_router(float* streams, const void* delta, int64_t n_tokens,
                                 int32_t d_model, const float* ffn_weight,
                                 const float* router_weight, float eps, void* out_bf16,
                                 float* router_in, void* stream);

/* ------------------------------------------------ fused small-batch decode
 * Two kernels that shorten the launch chain of a decode step at 1..8 tokens
 * (PhysicalBlock.forward_step, model/model.py:214-241).  No counterpart in
 * the reference, whose decode step runs the layers' eager forward_step.
 *
 * llmyb_decode_norm_gemv: x = streams_in + delta (delta: bf16 rows, or with
 * route_pos the sum of the k routed rows delta[route_pos[n*k+s]]; nullable);
 * out[n, :] = w [n_out, D] . (RMSNorm(x) * norm_w) in bf16 (row stride
 * out_ld).  streams_out (a different buffer than streams_in) gets x and
 * normed_out (nullable) the normalised rows.  n_tokens <= 8, D <= 2048,
 * D % 8 == 0; 16-byte aligned pointers. */
int32_t llmyb_decode_norm_gemv(const float* streams_in, const void* delta,
                               const int32_t* route_pos, int32_t top_k, int32_t n_tokens,
                               int32_t d_model, const float* norm_w, float eps, const void* w,
                               int32_t n_out, void* out, int64_t out_ld, float* streams_out,
                               void* normed_out, void* stream);

/* llmyb_decode_out_router: mixed = w [D, k_in] . in [N, k_in] (bf16; with
 * conv_w the GDN decode conv gate of llmyb_gdn_conv_gate is applied per
 * column, normed = the block input, history rolled); streams += mixed; then
 * the work of llmyb_route_fused: m_bf = RMSNorm_ffn(streams), logits of
 * RMSNorm_router(m), top-k and the plan.  The two RMSNorms are per-token
 * scales, so the router weights arrive folded: w_router_folded = W_r *
 * ffn_norm * router_norm (fp32 [E, D], per layer); every CTA adds its
 * columns' share of the sums of squares and logits to partials
 * (ceil(D/8) * N * (2+E) fp32 scratch) and the last CTA to finish combines
 * them in a fixed order.  counter: int32 zero word the kernel leaves at zero.
 * N <= 8, N*k <= 64, D <= 2048, k_in <= 2048. */
int32_t llmyb_decode_out_router(const void* in, int64_t in_ld, int32_t k_in, const void* w,
                                int32_t n_tokens, int32_t d_model, const float* conv_w,
                                const void* normed, void* history, float* partials,
                                int32_t* counter, float* streams, const float* ffn_norm,
                                const float* w_router_folded, float eps, int32_t n_experts,
                                int32_t top_k, int32_t tile_m, void* m_bf, int64_t* topk_idx,
                                float* topk_prob, int32_t* expert_counts, int32_t* expert_offsets,
                                int32_t* tile_offsets, int32_t* perm_token, float* perm_prob,
                                int32_t* route_pos, void* stream);

/* RMSNorm of a bf16 tensor [N, D] (final_norm before the tied LM head). */
int32_t llmyb_rmsnorm_bf16(const void* x, int64_t n_tokens, int32_t d_model, const float* weight,
                           float eps, void* out, void* stream);

/* ---------------------------------------------------------------- sampling
 * Replaces _sample_next_token / the sampling block of sample()
 * (sample_standalone.py:5383-5423, :5596-5636) and the native sampler
 * (llmy_cuda/src/kernels/sample.cu:116-234).  logits [B,V] fp32 (row stride ld);
 * seen [B, ceil(V/32)] bitmask of generated ids (repetition penalty) or null;
 * blocked ids forced to -inf or null; temperature <= 1e-4 is greedy; top_k 0
 * disables top-k (else <= 1024); 0 < top_p < 1 enables nucleus filtering;
 * uniforms [B] in [0,1) drive an inverse-CDF draw.  Writes token ids [B]
 * int64 and raw log-softmax of each token [B] (nullable); update_seen adds
 * the token to `seen`.  dev_status gets LLMYB_EUNSUPPORTED when a top-p-only
 * nucleus would extend beyond the 1024 best tokens. */
int32_t llmyb_sample(const float* logits, int64_t ld, int32_t batch, int32_t vocab,
                     uint32_t* seen, int64_t seen_ld, float repetition_penalty,
                     const int32_t* blocked, int32_t n_blocked, float temperature, int32_t top_k,
                     float top_p, const float* uniforms, int64_t* out_tokens, float* out_logprob,
                     int32_t update_seen, int32_t* dev_status, void* stream);

/* Host function (no device work).  Replaces llmy_sample
 * (llmy_cuda/include/llmy.h:62-68, llmy_cuda/src/llmy.cpp:132-202), the
 * engine's CPU sampler for one row of HOST logits [vocab] fp32: repetition
 * penalty once per entry of recent[n_recent] (ids outside the vocabulary
 * skipped), top_k <= 0 or > vocab = whole vocabulary, capped at 256;
 * temperature <= 0 is greedy; 0 < top_p < 1 keeps the shortest prefix whose
 * cumulative probability reaches top_p; one xorshift64 step of *rng_state gives
 * u = (state >> 11) / 2^53.  Returns the token id (0 when vocab <= 0, -1 for a
 * null logits / rng_state, or a null recent with n_recent > 0).  Equal logits
 * are ordered by index. */
int32_t llmyb_engine_sample(const float* logits, int32_t vocab, float temperature, int32_t top_k,
                            float top_p, float repetition_penalty, const int32_t* recent,
                            int32_t n_recent, uint64_t* rng_state);

/* Replaces llmy_mhc_sinkhorn4 (llmy_cuda/include/llmy.h:74-78; the operation
 * of model/layers/mhc.py:12-17): output[m] = exp(A) after `iterations` rounds
 * of A -= logsumexp over each row, then over each column, for fp32 [matrices,
 * 4, 4] device arrays (16-byte aligned).  LLMYB_EINVAL for null pointers,
 * matrices <= 0 or iterations < 0. */
int32_t llmyb_mhc_sinkhorn4(const float* input, float* output, int32_t matrices,
                            int32_t iterations, void* stream);

/* Replaces llmy_moe_selected_fp32 (llmy_cuda/include/llmy.h:80-88): one
 * token x [D] through its k routed experts idx [k] (int64; ids outside [0, E)
 * contribute zero) with weights prob [k], fp32: activation [k, H] =
 * silu(gate_e x) * (up_e x) with gate_up [E, 2H, D] (gate rows, then up rows),
 * route_output [k, D] = prob * down_e activation with down [E, D, H], and
 * out [D] = the sum of the k route outputs in route order.  Device pointers. */
int32_t llmyb_moe_selected_fp32(const float* x, const int64_t* idx, const float* prob,
                                const float* gate_up, const float* down, float* activation,
                                float* route_output, float* out, int32_t D, int32_t H, int32_t E,
                                int32_t k, void* stream);

/* ------------------------------------------------ hyper-connections (mHC)
 * Replace MultiStreamHyperConnection.read / write (model/layers/mhc.py:135-156,
 * :193-229) around each block sub-layer, for S = n_streams in {1, 2, 4} live
 * fp32 residual streams per token, laid out [N, S*D].  maps [N, 2S+S*S] fp32
 * hold pre | post | res (row-major) of a read for the write that follows it.
 *
 * llmyb_mhc_read: raw = the logits streams @ (theta * mapping_norm.weight)^T
 * (the caller's GEMM), map o of token n at raw[n * raw_tok + o * raw_map]
 * (either orientation); bias = pre_bias | post_bias | residual_bias;
 * scalars = alpha_pre, alpha_post, alpha_residual, sigmoid(gating_logit).
 * Computes the maps (mapping RMSNorm with the fp32 epsilon, sigmoids, Sinkhorn
 * with `iterations` rounds), hidden = LayerNorm(sum_s pre[s] streams[s]) with
 * ln_w / ln_b (eps 1e-5), then RMSNorm(hidden) * norm_w (norm_w nullable = 1)
 * into out_bf16 [N, D] and/or out_f32 [N, D].  D % 4 == 0, D <= 4096.
 *
 * llmyb_mhc_write: streams[i] += g * stream_scale[i] * (sum_j res[i,j]
 * streams[j] + post[i] * update), update = delta [N, D] bf16, or with
 * route_pos the fp32 sum of the top_k routed rows delta[route_pos[n*k + s]]
 * (the MoE combine), or zero for a null delta. */
int32_t llmyb_mhc_read(const float* streams, int32_t n_tokens, int32_t n_streams, int32_t d_model,
                       const float* raw, int64_t raw_tok, int64_t raw_map, const float* bias,
                       const float* scalars,
                       const float* ln_w, const float* ln_b, const float* norm_w, float rms_eps,
                       int32_t iterations, float* maps, void* out_bf16, float* out_f32,
                       void* stream);
int32_t llmyb_mhc_write(float* streams, int32_t n_tokens, int32_t n_streams, int32_t d_model,
                        const void* delta, const int32_t* route_pos, int32_t top_k,
                        const float* maps, const float* stream_scale, const float* scalars,
                        void* stream);

/* ------------------------------------------------- router local context
 * The ContextAwareRouter's local-context path (model/layers/context_router.py:59-74,
 * :89-133; mla_memory.py:23-48) without HCA latents: latents = LayerNorm(down(local))
 * (eps 1e-5) and their causal mean over the last `window` tokens ("box"),
 * which the caller's GEMMs turn into router logits.  fp32 throughout.
 *
 * llmyb_router_ctx_prefill: lat [batch*seq, latent] = down(local) in, the
 * LayerNorm'd latents out (in place); box [batch*seq, latent]; ring
 * [batch, window, latent] (nullable) receives the last `window` latents of each
 * row (position p at slot p % window).  latent <= 1024.
 *
 * llmyb_router_ctx_step: one decode token per row at positions[b]: lat
 * [batch, latent] in (LayerNorm'd in place), stored at ring slot
 * positions[b] % window; box [batch, latent] = mean of the latents of
 * positions max(0, p-window+1) .. p. */
int32_t llmyb_router_ctx_prefill(float* lat, int32_t batch, int32_t seq, int32_t latent,
                                 int32_t window, const float* ln_w, const float* ln_b, float* box,
                                 float* ring, void* stream);
int32_t llmyb_router_ctx_step(float* lat, int32_t batch, int32_t latent, int32_t window,
                              const float* ln_w, const float* ln_b, float* ring,
                              const int32_t* positions, float* box, void* stream);

/* ------------------------------------------------------------- loop memory
 * The loop memory between recurrent loops (model/loop_memory.py:36-66,
 * LatentAttention mla_memory.py:66-86; called at model/model.py:636, :661-667
 * and :877, :884-891).  Before every loop after the first, each token attends
 * over LayerNorm'd latent summaries of its own streams at the end of the
 * earlier loops; the gated result is added to every stream.  The fp32
 * projections (down, q, k|v, o) are the caller's GEMMs; these are the
 * per-token steps between them. */

/* y[t] = mean over the S streams of x[t] (rows of S*width floats at stride
 * ld; S = 1 copies), then LayerNorm(ln_w, ln_b, eps) if ln_w is non-null
 * (ln_b nullable).  width <= 24576. */
int32_t llmyb_loop_mem_norm(const float* x, int64_t ld, int32_t n_tokens, int32_t n_streams,
                            int32_t width, const float* ln_w, const float* ln_b, float eps,
                            float* y, int64_t y_ld, void* stream);

/* out [N, H*hd] = per (token, head) softmax_j(q . k_j / sqrt(hd)) v_j over the
 * n_mem <= 16 endpoints; kv [n_mem, N, 2*H*hd] holds each endpoint's k
 * projection then its v projection (LatentAttention with causal=False). */
int32_t llmyb_loop_mem_attend(const float* q, const float* kv, int32_t n_tokens, int32_t n_mem,
                              int32_t heads, int32_t head_dim, float* out, void* stream);

/* streams [N, S*D] fp32 += gate * delta [N, D] fp32 on every stream
 * (D % 4 == 0, 16-byte aligned pointers). */
int32_t llmyb_loop_mem_add(float* streams, int32_t n_tokens, int32_t n_streams, int32_t d_model,
                           const float* delta, float gate, void* stream);

/* ------------------------------------------------------ CSA remote branch
 * The CSA remote compressed branch (model/layers/csa.py:77-131 prefill,
 * :208-256 decode) over the causal temporal compressor
 * (model/layers/compressed_attention.py:85-206), without segment ids: every
 * complete `ratio`-token block of the CSA input is summarised by its mean m
 * (key W_k m [H*Dh], value W_v m [D]), visible from the block's last
 * position; each query attends per head to its top_k (<= 32) visible
 * summaries (softmax over the selected scores, ties to the lower index) and
 * the heads' results are averaged.  Bf16 inputs/outputs, fp32 arithmetic. */

/* Prefill compressor: means [B, n, D] (n = seq / ratio) of the complete
 * blocks of x [B, seq, D] (rows at stride ldx), and the pending partial
 * block's sum pend_sum [B, D] fp32 / count pend_cnt [B] for decode. */
int32_t llmyb_csa_block_means(const void* x, int64_t ldx, int32_t batch, int32_t seq,
                              int32_t d_model, int32_t ratio, void* means, float* pend_sum,
                              int32_t* pend_cnt, void* stream);

/* Prefill attention weights: P[b, t, 0:n] (bf16, row stride ldp) = the mean
 * over heads of each head's top-k softmax weights over the summaries visible
 * to token t (the first min(n, (t+1)/ratio)); q [B*seq] rows at stride ldq,
 * keys [B*n] rows of H*Dh at stride ldk.  remote = P V is then one batched
 * GEMM of the caller. */
int32_t llmyb_csa_remote_rows(const void* q, int64_t ldq, const void* keys, int64_t ldk,
                              int32_t batch, int32_t seq, int32_t heads, int32_t head_dim,
                              int32_t n_summaries, int32_t ratio, int32_t top_k, void* P,
                              int64_t ldp, void* stream);

/* Decode step (three launches): the token x [B, D] joins each row's pending
 * block; a completing block's summary [key | value] = w_comp [H*Dh + D, D] .
 * mean goes to slot mem_count[b] of mem_k [B, capacity, H*Dh] / mem_v
 * [B, capacity, D]; then out [B, D] (row stride ldo) = the remote attention
 * of q over the row's summaries, and the compressor state (pend_sum fp32
 * [B, D], pend_cnt, mem_count) advances.  sel_j / sel_w [B, H, top_k] are
 * scratch.  A row past `capacity` summaries records LLMYB_EUNSUPPORTED in
 * dev_status (nullable) and keeps its oldest summaries. */
int32_t llmyb_csa_remote_step(const void* x, int64_t ldx, const void* q, int64_t ldq,
                              int32_t batch, int32_t heads, int32_t head_dim, int32_t d_model,
                              int32_t ratio, int32_t top_k, int32_t capacity, const void* w_comp,
                              void* mem_k, void* mem_v, int32_t* mem_count, float* pend_sum,
                              int32_t* pend_cnt, int32_t* sel_j, float* sel_w, void* out,
                              int64_t ldo, int32_t* dev_status, void* stream);

/* ------------------------------------------------- persistent decode step
 * The whole batch-1 decode step of the looped stack (model/model.py:787-915
 * with PhysicalBlock.forward_step :266-376, as in sample_standalone.py's
 * decode, and the head :913-915) as ONE cooperative launch: one 512-thread
 * CTA per SM walks every block of every loop in phases separated by bounded
 * grid barriers (input projection; CSA attention or the GDN step; the GDN
 * output projection; router + expert gate/up; expert down), then the collapse,
 * final norm and LM head.  Each phase loads its weight rows before waiting on
 * the barrier.  The CSA output projection is folded into the cached values:
 * ring_v holds W_o W_v x (W_o = out . local_out), and w_in's value rows are
 * W_o W_v, so the attention output is the block's output.  Served: one plain
 * residual stream, CSA without the remote branch (head_dim 64), GDN with key =
 * value dim 64, routed experts only, D <= 1024 (D % 8 == 0), F <= 2048
 * (F % 128 == 0), E <= 64, top_k <= 8, window <= 1024, CSA heads <= 16.
 * Before every launch the caller zeroes *bar (4 bytes).  A barrier that does
 * not complete within one second records LLMYB_ETIMEOUT in *status and every
 * CTA returns. */
typedef struct {
  int32_t kind;                 /* 0: CSA (local branch), 1: GDN */
  int32_t rows;                 /* rows of w_in */
  const float* mixer_norm;      /* [D] */
  const float* ffn_norm;        /* [D] */
  const float* router_fold;     /* [E, D] = router * ffn_norm * router_norm */
  const void* w_in;             /* CSA [2*H*Dh + D, D]: q | k | W_o W_v;  GDN [P, D] */
  const float* beta_bias;       /* GDN [H] */
  const float* decay_logit;     /* GDN [H] */
  const void* w_out;            /* GDN [D, H*V] */
  const float* conv;            /* GDN [D, 4] */
  const void* w13;              /* [E, 2F, D] interleaved gate/up */
  const void* w2;               /* [E, D, F] */
} llmyb_pblock;

typedef struct {
  void* ring_k;                 /* CSA [W, H*Dh] bf16 */
  void* ring_v;                 /* CSA [W, D] bf16, folded values W_o W_v x */
  float* gdn_state;             /* GDN [H, 64, 64] fp32 */
  void* conv_hist;              /* GDN [3, D] bf16 */
} llmyb_player;

typedef struct {
  int32_t d_model, n_blocks, n_loops, vocab;
  int32_t csa_heads, csa_head_dim, window;
  int32_t gdn_heads, gdn_dim;
  int32_t n_experts, top_k, ffn;
  float eps;
  int32_t grid;                 /* CTAs (one per SM); sizes stats / partials */
  const llmyb_pblock* blocks;   /* device array [n_blocks] */
  const llmyb_player* layers;   /* device array [n_loops * n_blocks] */
  const void* embed;            /* [vocab, D] bf16 (tied LM head) */
  const float* stream_seed;     /* [D] */
  const void* collapse;         /* [D, D] bf16 */
  const float* final_norm;      /* [D] */
  const int64_t* token;         /* [1] */
  int32_t* positions;           /* [1], incremented by the step */
  float* x;                     /* scratch [2, D] */
  void* proj;                   /* scratch [max rows] bf16 */
  void* normed;                 /* scratch [D] bf16 */
  float* scores;                /* scratch [csa_heads, window] */
  float* stats;                 /* scratch [csa_heads, grid, 2] (8-byte aligned) */
  void* mix;                    /* scratch [max(D, gdn_heads*gdn_dim)] bf16 */
  float* partials;               /* scratch [2 + E, grid] */
  void* hbuf;                   /* scratch [top_k, F] bf16 */
  void* ybuf;                   /* scratch [top_k, D] bf16 */
  void* collapsed;              /* scratch [D] bf16 */
  int32_t* route_idx;           /* out [n_loops * n_blocks, top_k] */
  float* route_prob;            /* out [n_loops * n_blocks, top_k] */
  float* logits;                /* out [vocab] fp32 (bf16-rounded LM head output) */
  uint32_t* bar;                /* [2]: grid barrier counter and the greedy step's arrival
                                   count, both zeroed before each launch */
  int32_t* status;              /* device status word */
  uint64_t* trace;              /* nullable: [2, 2, 512] %globaltimer stamps of CTA 0 and the
                                   last CTA, at every barrier wait's end and arrive (and
                                   [2048, ...] points inside phases) */
  /* Greedy sampling fused into the LM head (nullable out_token: logits only).
   * The first maximal logit's index (sample_standalone.py:5383-5423 with
   * temperature <= 1e-4 and no repetition penalty) goes to out_token, its
   * raw log-softmax to out_logprob (nullable), its bit into seen (nullable
   * [ceil(vocab/32)] bitmask); head_part is scratch [grid, 4]. */
  int64_t* out_token;
  float* out_logprob;
  int32_t* seen;
  float* head_part;
  /* Non-zero: a prompt token whose logits nobody reads: the step ends after
   * the last expert phase (no collapse, final norm, LM head or sampling). */
  int32_t skip_head;
} llmyb_pdecode;

/* CTAs per grid that llmyb_decode_persistent will use on the current device
 * (one per SM, if a 512-thread CTA with its shared memory fits), or a
 * negative status. */
int32_t llmyb_decode_persistent_grid(void);

/* One decode step; `p` is a host struct (copied into the launch). */
int32_t llmyb_decode_persistent(const llmyb_pdecode* p, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LLMYB_H */
