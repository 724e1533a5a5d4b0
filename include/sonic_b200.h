/*
 * sonic_b200.h -- C ABI of libsonic_b200.so, the B200 (sm_100a) FP8 MoE-layer forward engine.
 *
 * Conventions (every entry point):
 *   - Pointers are device pointers owned by the caller; nothing is allocated inside except where
 *     an entry point documents it.  Scratch space is an explicit `workspace` argument.
 *   - Work is enqueued on `stream` (a cudaStream_t passed as void*); calls are asynchronous,
 *     perform no host synchronisation and can be captured in a CUDA graph.
 *   - Return 0 on success or a negative errno-style code: SM_EINVAL (bad shape, alignment or
 *     pointer), SM_ENOTSUP (a configuration this engine does not implement), SM_EIO (CUDA
 *     launch error).  sm_last_error() returns a message for the calling thread's last failure.
 *   - Kernels with bounded waits report a timeout through the int32 `err` word (0 = ok); the
 *     host reads it whenever it synchronises.  SM_ERR_TIMEOUT_* values identify the wait.
 *   - bf16 tensors are passed as `const void*` / `void*` (IEEE bfloat16, row-major).
 *
 * FP8 format (this engine's quantiser; the reference has none): e4m3 values, one UE8M0 scale
 * byte (2^(b-127)) per 1x128 activation group or 128x128 weight block, scale = 2^ceil(log2(amax/448)).
 * Scale bytes are stored in 512-byte "SF atoms" of 128 rows x 4 K-blocks, byte
 * 16*(r%32) + 4*((r%128)/32) + (kb%4) for row r and K block kb (activations: atom [r/128][kb/4];
 * weights: atom [expert][n/128][kb/4], every row of a 128-row block holding the block's scale).
 */
#ifndef SONIC_B200_H
#define SONIC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SM_OK 0
#define SM_EIO (-5)
#define SM_EINVAL (-22)
#define SM_ENOTSUP (-95)

#define SM_DTYPE_BF16 0
#define SM_DTYPE_F16 1
#define SM_DTYPE_F32 2

#define SM_ERR_TIMEOUT_PRODUCER 101
#define SM_ERR_TIMEOUT_MMA 102
#define SM_ERR_TIMEOUT_EPILOGUE 103
#define SM_ERR_BAD_EXPERT 201
#define SM_ERR_BAD_RETURN_ROW 202 /* home-down EP: an up-projection row with no valid home row */
#define SM_ERR_BAD_COUNT 203      /* EP with device-side counts: a count outside the exchange buffers */

/* Message describing the calling thread's most recent non-zero return. */
const char* sm_last_error(void);

/* Library version string. */
const char* sm_version(void);

/*
 * Router top-k.  Replaces the custom op `sonicmoe::_softmax_topk_fwd`
 * (reference sonicmoe/functional/forward.py:107-141) and its CuTe kernel
 * (sonicmoe/functional/topk.py:143-260).
 *   logits [T, E] (dtype SM_DTYPE_*), scores [T, K] float32, indices [T, K] int32, both in
 *   descending score order; equal scores go to the lower expert index.
 *   softmax_over_topk = 1: softmax over the k selected logits; = 0: top-k of the full-row softmax,
 *   renormalised to sum to 1 when norm_topk_probs = 1 (only valid with softmax_over_topk = 0).
 *   1 <= K <= min(E, 32), 1 <= E <= 4096.
 */
int sm_router_topk(const void* logits, int dtype, int T, int E, int K, int softmax_over_topk, int norm_topk_probs,
                   float* scores, int32_t* indices, void* stream);

/* Bytes of workspace sm_route_metadata / sm_general_route_metadata need. */
size_t sm_route_metadata_workspace(int T, int TK, int E);

/*
 * Token-choice routing metadata.  Replaces `triton_kernels::TC_topk_router_metadata`
 * (reference sonicmoe/functional/triton_kernels/__init__.py:68-146, bitmatrix.py:18-147).
 *   topk_indices [T, K] int32 ->
 *   expert_frequency [E], expert_frequency_offset [E+1] (exclusive cumsum, [E] = T*K),
 *   s_scatter_idx [T*K] (expert-sorted position -> flat entry t*K+k; stable in entry order),
 *   s_reverse_scatter_idx [T*K] (its inverse), x_gather_idx [T*K] (= s_scatter_idx / K).
 *   err: int32 word set to SM_ERR_BAD_EXPERT if an index is outside [0, E).
 */
int sm_route_metadata(const int32_t* topk_indices, int T, int K, int E, int32_t* expert_frequency,
                      int32_t* expert_frequency_offset, int32_t* x_gather_idx, int32_t* s_scatter_idx,
                      int32_t* s_reverse_scatter_idx, void* workspace, size_t workspace_bytes, int32_t* err,
                      void* stream);

/*
 * General-routing metadata.  Replaces `triton_kernels::general_routing_router_metadata`
 * (reference sonicmoe/functional/triton_kernels/__init__.py:270-353).
 *   sorted_token_idx [TK] (ascending), expert_idx [TK] -> the five arrays above (x_gather_idx =
 *   sorted_token_idx[s_scatter_idx]) and num_activated_expert_per_token_offset [T+1].
 */
int sm_general_route_metadata(const int32_t* sorted_token_idx, const int32_t* expert_idx, int T, int TK, int E,
                              int32_t* expert_frequency, int32_t* expert_frequency_offset, int32_t* x_gather_idx,
                              int32_t* s_scatter_idx, int32_t* s_reverse_scatter_idx,
                              int32_t* num_activated_expert_per_token_offset, void* workspace,
                              size_t workspace_bytes, int32_t* err, void* stream);

/*
 * sm_route_metadata without a workspace argument.  No counterpart in the reference: it exists
 * for callers that cannot allocate device memory when they route -- a host that records the step
 * into a CUDA graph (cudaMalloc is not allowed during stream capture) or a runtime that reserved
 * all device memory up front and has no allocator to hand out scratch.  The scratch (per-tile
 * counts and the padded layout) lives in a 1 MiB static device array that each GPU loading the
 * library keeps until the process exits; shapes needing more (E * ceil(T/128) + T*K/128 + 2E
 * int32 entries, roughly) return SM_EINVAL.  Same outputs as sm_route_metadata.  The first call
 * on a device looks up the array's address and should come before any stream capture.  The
 * address is kept per device with the id of the CUDA context it was taken in; after a device
 * reset (a new primary context) the next call looks it up again, so that call too belongs before
 * any capture.  All calls share the array: calls that overlap on the GPU race, so the caller
 * serialises them.  Allocates nothing (no cudaMalloc / cudaFree).
 */
int sm_route_metadata_noalloc(const int32_t* topk_indices, int T, int K, int E, int32_t* expert_frequency,
                              int32_t* expert_frequency_offset, int32_t* x_gather_idx, int32_t* s_scatter_idx,
                              int32_t* s_reverse_scatter_idx, int32_t* err, void* stream);

/*
 * 1x128 activation quantiser in token order (no reference counterpart; the reference has no FP8
 * path -- this is the spec entry point the pack kernel shares).
 *   x [R, C] bf16 (C % 128 == 0) -> q [R, C] e4m3, sf atoms [ceil(R/128)][ceil(C/512)][512].
 */
int sm_quant_1x128(const void* x, int R, int C, uint8_t* q, uint8_t* sf_atoms, void* stream);

/* Bytes of the weight SF atoms for a [E, N, K] weight. */
size_t sm_weight_sf_bytes(int E, int N, int K);

/*
 * 128x128 weight quantiser (weight preparation, done once per weight version).  Consumes the
 * reference's expert weights `c_fc.weight` [E, 2I, H] / `c_proj.weight` [E, H, I]
 * (reference sonicmoe/moe.py:189-203, layout contract functional/__init__.py:560-566).
 *   w [E, N, K] bf16 (N, K % 128 == 0) -> wq [E, N, K] e4m3 + sf atoms.
 *   concat_glu = 1: w is a concatenated SwiGLU weight [gate; up] (N = 2I); the output rows are
 *   re-blocked to [gate_0..127, up_0..127, gate_128..255, ...] so that one 256-row GEMM tile holds
 *   matching gate and up blocks.  The 128x128 scale blocks are those of the input layout.
 */
int sm_weight_prep(const void* w, int E, int N, int K, int concat_glu, uint8_t* wq, uint8_t* sf_atoms,
                   void* stream);

/* Bytes of workspace sm_moe_forward needs. */
size_t sm_moe_workspace_bytes(int T, int H, int I, int E, int K);

/*
 * Whole FP8 MoE-layer forward (inference).  Replaces the forward of
 * `moe_TC_softmax_topk_layer` after the router GEMM (reference sonicmoe/functional/__init__.py:482-557:
 * router top-k, routing metadata, _UpProjection, _DownProjection with the expert aggregation).
 *   x [T, H] bf16, router_logits [T, E] bf16 (x @ router_w^T, computed by the caller),
 *   w1q/w1_sf from sm_weight_prep of c_fc.weight (interleaved, or concat_layout = 1),
 *   w2q/w2_sf from sm_weight_prep of c_proj.weight ->
 *   out [T, H] bf16, expert_frequency [E] int32; topk_scores [T, K] float32 and
 *   topk_indices [T, K] int32 are written when non-NULL.
 *   H % 256 == 0, I % 128 == 0, 1 <= K <= min(E, 32), E <= 4096.
 *   err: int32 word (may be NULL); set non-zero if a kernel gave up on a bounded wait.
 */
int sm_moe_forward(const void* x, const void* router_logits, int T, int H, int I, int E, int K,
                   int softmax_over_topk, int norm_topk_probs, int concat_layout, const uint8_t* w1q,
                   const uint8_t* w1_sf, const uint8_t* w2q, const uint8_t* w2_sf, void* out,
                   int32_t* expert_frequency, float* topk_scores, int32_t* topk_indices, void* workspace,
                   size_t workspace_bytes, int32_t* err, void* stream);

/*
 * Fused router, opt-in.  Replaces the router GEMM `F.linear(x, router_w)` of
 * moe_TC_softmax_topk_layer (reference sonicmoe/functional/__init__.py:501) together with the
 * top-k of sm_router_topk: one tcgen05 kernel per 128-token tile computes
 * router_logits = x @ router_weight^T (bf16 operands, fp32 accumulation, rounded to bf16) and
 * ranks those rows exactly as sm_router_topk ranks given logits.  The accumulation order is the
 * tensor core's, not cuBLAS's, so a logit can differ from F.linear's in its last bf16 bit (and a
 * near-tie then route differently); the reference has no such path.
 *   x [T, H] bf16, router_weight [E, H] bf16 -> router_logits [T, E] bf16, scores / indices
 *   [T, K] as for sm_router_topk.  E % 32 == 0 with 32 <= E <= 256, H % 64 == 0 (else
 *   SM_ENOTSUP).  workspace: sm_router_fused_workspace(T, E) bytes (per-tile expert counts).
 */
size_t sm_router_fused_workspace(int T, int E);
int sm_router_fused(const void* x, const void* router_weight, int T, int H, int E, int K, int softmax_over_topk,
                    int norm_topk_probs, void* router_logits, float* scores, int32_t* indices, void* workspace,
                    size_t workspace_bytes, int32_t* err, void* stream);

/*
 * sm_moe_forward with the fused router in place of the caller's router GEMM (same workspace
 * size, sm_moe_workspace_bytes): router_weight [E, H] bf16 in, router_logits [T, E] bf16 out.
 * Same limits as sm_router_fused.  Replaces moe_TC_softmax_topk_layer's forward including its
 * F.linear (reference sonicmoe/functional/__init__.py:482-557).
 */
int sm_moe_forward_fused_router(const void* x, const void* router_weight, int T, int H, int I, int E, int K,
                                int softmax_over_topk, int norm_topk_probs, int concat_layout, const uint8_t* w1q,
                                const uint8_t* w1_sf, const uint8_t* w2q, const uint8_t* w2_sf, void* out,
                                void* router_logits, int32_t* expert_frequency, float* topk_scores,
                                int32_t* topk_indices, void* workspace, size_t workspace_bytes, int32_t* err,
                                void* stream);

/* Bytes of workspace sm_moe_general_forward needs for T tokens and TK routed (token, expert) entries. */
size_t sm_moe_general_workspace_bytes(int T, int TK, int H, int I, int E);

/*
 * FP8 MoE-layer forward from explicit routing lists.  Replaces the forward of
 * `moe_general_routing_inputs` (reference sonicmoe/functional/__init__.py:571-652: general routing
 * metadata, _UpProjection / _DownProjection with variable experts per token, varlen-K
 * aggregation of reduction_over_k_gather.py:77-83).
 *   x [T, H] bf16; router_scores [TK] float32, token_indices [TK] int32 sorted ascending,
 *   expert_indices [TK] int32 (entry f routes token token_indices[f] to expert expert_indices[f]
 *   with weight router_scores[f]); w1/w2 as for sm_moe_forward ->
 *   out [T, H] bf16 (tokens without entries get zeros), expert_frequency [E] int32.
 */
int sm_moe_general_forward(const void* x, int T, int H, int I, int E, int TK, const float* router_scores,
                           const int32_t* token_indices, const int32_t* expert_indices, int concat_layout,
                           const uint8_t* w1q, const uint8_t* w1_sf, const uint8_t* w2q, const uint8_t* w2_sf,
                           void* out, int32_t* expert_frequency, void* workspace, size_t workspace_bytes,
                           int32_t* err, void* stream);

/*
 * Stage-level entry points of the forward (same pipeline as sm_moe_forward, exposed so each
 * stage can be checked on its own).  The padded expert layout: expert e owns rows
 * [off_pad[e], off_pad[e] + expert_frequency[e]) of a buffer with max_blocks*128 rows, where
 * max_blocks = sm_max_padded_blocks(T*K, E); blk_expert[b] is the expert of 128-row block b and
 * n_blocks[0] the number of blocks in use.
 */
int sm_max_padded_blocks(long long TK, int E);

/* sm_route_metadata plus the padded layout: off_pad [E+1], blk_expert [max_blocks], n_blocks [1]. */
int sm_route_plan(const int32_t* topk_indices, int T, int K, int E, int32_t* expert_frequency,
                  int32_t* expert_frequency_offset, int32_t* x_gather_idx, int32_t* s_scatter_idx,
                  int32_t* s_reverse_scatter_idx, int32_t* off_pad, int32_t* blk_expert, int32_t* n_blocks,
                  void* workspace, size_t workspace_bytes, int32_t* err, void* stream);

/* sm_route_plan for explicit routing lists (moe_general_routing_inputs): the general metadata of
 * sm_general_route_metadata plus this build's padded layout (off_pad [E+1], blk_expert, n_blocks).
 * Workspace: sm_route_metadata_workspace(T, TK, E). */
int sm_general_route_plan(const int32_t* sorted_token_idx, const int32_t* expert_idx, int T, int TK, int E,
                          int32_t* expert_frequency, int32_t* expert_frequency_offset, int32_t* x_gather_idx,
                          int32_t* s_scatter_idx, int32_t* s_reverse_scatter_idx,
                          int32_t* num_activated_expert_per_token_offset, int32_t* off_pad, int32_t* blk_expert,
                          int32_t* n_blocks, void* workspace, size_t workspace_bytes, int32_t* err, void* stream);
/* sm_quant_pack for explicit routing lists: token t's row goes to the padded rows of its entries
 * [tok_off[t], tok_off[t+1]) (expert_idx per entry). */
int sm_quant_pack_general(const void* x, int T, int H, const int32_t* expert_idx,
                          const int32_t* num_activated_expert_per_token_offset, const int32_t* s_reverse_scatter_idx,
                          const int32_t* expert_frequency_offset, const int32_t* off_pad, uint8_t* xq, uint8_t* xsf,
                          void* stream);

/* Quantise x [T, H] and write each token's row to its K padded positions:
 * xq [max_blocks*128, H] e4m3, xsf atoms [max_blocks][ceil(H/512)][512]. */
int sm_quant_pack(const void* x, int T, int H, const int32_t* topk_indices, int K,
                  const int32_t* s_reverse_scatter_idx, const int32_t* expert_frequency_offset,
                  const int32_t* off_pad, uint8_t* xq, uint8_t* xsf, void* stream);

/* Up projection + SwiGLU + 1x128 requantisation (reference _UpProjection.forward,
 * sonicmoe/functional/__init__.py:227-301): aq [max_blocks*128, I] e4m3 + asf atoms. */
int sm_moe_up(const uint8_t* xq, const uint8_t* xsf, const uint8_t* w1q, const uint8_t* w1_sf, int H, int I, int E,
              int concat_layout, int max_blocks, const int32_t* blk_expert, const int32_t* n_blocks,
              const int32_t* off_pad, const int32_t* expert_frequency, uint8_t* aq, uint8_t* asf, int32_t* err,
              void* stream);

/* sm_moe_up for the training forward: also stores the pre-activation h = x W1^T that the
 * reference keeps for its backward (sonicmoe/functional/__init__.py:253-258 allocates it, :266-268
 * passes preact_out=h, store_preact=True).  preact [T*K, 2I] bf16, row = the entry's expert-sorted
 * position (off[e] + rank within the expert, i.e. the row order of s_scatter_idx), columns in the
 * caller's w1 order (interleaved gate/up, or [gate | up] with concat_layout = 1).  The values are
 * the fp32 tensor-core sums of the e4m3 operands rounded to bf16. */
int sm_moe_up_preact(const uint8_t* xq, const uint8_t* xsf, const uint8_t* w1q, const uint8_t* w1_sf, int H, int I,
                     int E, int concat_layout, int max_blocks, const int32_t* blk_expert, const int32_t* n_blocks,
                     const int32_t* off_pad, const int32_t* expert_frequency_offset, const int32_t* expert_frequency,
                     uint8_t* aq, uint8_t* asf, void* preact, int32_t* err, void* stream);

/* Down projection with the top-k weighted combine fused (reference _DownProjection.forward and
 * _router_forward, sonicmoe/functional/__init__.py:365-420, forward.py:64-85).  Adds
 * score * y into out [T, H] bf16, which the caller zero-fills first (topk_scores = NULL: unit
 * weights, the backward's dX).  Tiles are visited one output-column slice at a time so that the
 * slice being reduced into stays resident in L2. */
int sm_moe_down_combine(const uint8_t* aq, const uint8_t* asf, const uint8_t* w2q, const uint8_t* w2_sf, int H,
                        int I, int E, int T, int max_blocks, const int32_t* blk_expert, const int32_t* n_blocks,
                        const int32_t* off_pad, const int32_t* expert_frequency_offset,
                        const int32_t* expert_frequency, const int32_t* s_scatter_idx, const int32_t* x_gather_idx,
                        const float* topk_scores, void* out, int32_t* err, void* stream);

/*
 * Backward of the layer (reference sonicmoe/functional/backward.py and the autograd functions
 * _UpProjection.backward / _DownProjection.backward, functional/__init__.py:303-362, 422-479), in
 * FP8 with the forward's 1x128 / 128x128 UE8M0 scaling.  For dO [T, H] the stages are:
 *   1. sm_quant_pack of dO (exactly as x in the forward) -> dO rows in the padded layout;
 *   2. sm_moe_dact: dA' = dO W2 per entry (B = W2^T, sm_weight_prep_t of the prepared c_proj.weight), then
 *      from the stored pre-activation h (sm_moe_up_preact): dS [T*K] (accumulated: zero it first),
 *      a' = s * a and dH = SwiGLU backward of s * dA' -- dH as e4m3 + atoms for stage 3 and as bf16,
 *      a' as bf16, both in padded rows (gemm_dact of functional/backward.py:211-278);
 *   3. sm_moe_down_combine with topk_scores = NULL (unit weights) and B = W1^T (sm_weight_prep_t of
 *      the prepared c_fc.weight, interleaved layout): dX [T, H] = sum over the token's entries of dH W1
 *      (the reference's gemm + token_broadcast_backward, :173-206 and :281-305);
 *   4. sm_tq_pack of dO (gathered) / x (gathered) / a' / dH (padded) -> transposed e4m3 operands
 *      with one scale per 128 rows, then sm_moe_wgrad: dW2[e] = dO_e^T a'_e [H, I] and
 *      dW1[e] = dH_e^T x_e [2I, H] (the reference's varlen-K gemms, :339-348, :465-473);
 *   5. sm_router_bwd: dlogits [T, E] fp32 from dS (backward.py:308-430).
 * Both w1 layouts (interleaved, or concatenated with concat_layout = 1 in stage 2).
 */
/* W^T for a backward GEMM from the forward's prepared weight (sm_weight_prep; for a concatenated
 * w1 the K order of the result is the prepared weight's re-blocked row order):
 * wq [E, N, K] e4m3 + atoms -> wq_t [E, K, N] e4m3, the same values and 128x128 block scales read
 * transposed, atoms_t [E][K/128][ceil(N/512)][512] (sm_weight_sf_bytes(E, K, N) bytes). */
int sm_weight_prep_t(const uint8_t* wq, const uint8_t* sf_atoms, int E, int N, int K, uint8_t* wq_t,
                     uint8_t* sf_atoms_t, void* stream);
/* sm_weight_prep and sm_weight_prep_t in one pass over the bf16 weight (a training step's new
 * weight version): wq / sf_atoms exactly as sm_weight_prep, wq_t / sf_atoms_t exactly as
 * sm_weight_prep_t of them. */
int sm_weight_prep_with_t(const void* w, int E, int N, int K, int concat_glu, uint8_t* wq, uint8_t* sf_atoms,
                          uint8_t* wq_t, uint8_t* sf_atoms_t, void* stream);
/* Stage 2 above.  doq/dosf: dO packed like sm_quant_pack's xq/xsf; w2t: [E, I, H]; preact [T*K, 2I]
 * bf16 (expert-sorted rows, the caller's w1 column order); dh_q [max_blocks*128, 2I] + dh_sf atoms,
 * dh_bf16 [max_blocks*128, 2I], a_prime [max_blocks*128, I] (padded rows); dscores [T*K] fp32, flat
 * entries, accumulated.  concat_layout = 1: h and dh_bf16 in [gate | up] order and dh_q in the
 * re-blocked order of the prepared concatenated w1 (gate block j, up block j, ...), matching
 * sm_weight_prep_t of that weight.  dH's e4m3 copy quantises the bf16 dH.  dh_q = dh_sf = NULL:
 * no e4m3 copy (sm_tq_pack_dual makes it from dh_bf16 together with the dW1 operand).
 * I % 256 == 0. */
int sm_moe_dact(const uint8_t* doq, const uint8_t* dosf, const uint8_t* w2t_q, const uint8_t* w2t_sf, int H, int I,
                int E, int max_blocks, const int32_t* blk_expert, const int32_t* n_blocks, const int32_t* off_pad,
                const int32_t* expert_frequency_offset, const int32_t* expert_frequency, const int32_t* s_scatter_idx,
                const float* topk_scores, const void* preact, int concat_layout, uint8_t* dh_q, uint8_t* dh_sf,
                void* dh_bf16, void* a_prime, float* dscores, int32_t* err, void* stream);
/* Transposed, column-quantised operand of a weight-gradient GEMM: out [C, max_blocks*128] e4m3,
 * out[c][p] = q(src[row(p)][c]) with one UE8M0 scale per (c, 128-row block), atoms
 * [C/128][ceil(max_blocks/4)][512]; row(p) = the token of padded row p (src_padded = 0: src is
 * [T, C] token rows, gathered by x_gather_idx) or p itself (src_padded = 1: src [max_blocks*128, C]);
 * padding rows are zero.  C % 128 == 0. */
int sm_tq_pack(const void* src, int C, int src_padded, int max_blocks, const int32_t* blk_expert,
               const int32_t* n_blocks, const int32_t* off_pad, const int32_t* expert_frequency_offset,
               const int32_t* expert_frequency, const int32_t* x_gather_idx, uint8_t* out_q, uint8_t* out_sf,
               void* stream);
/* sm_tq_pack of a padded source (dH [max_blocks*128, C] bf16) that also writes the row-quantised
 * copy from the same read: row_q [max_blocks*128, C] e4m3 with one UE8M0 scale per 128 columns of a
 * row, atoms row_sf [max_blocks][ceil(C/512)][512] -- the dX GEMM's A operand, exactly what
 * sm_moe_dact writes as dh_q / dh_sf.  concat_I = I (C = 2I, src in [gate | up] order): row_q
 * column blocks in the prepared concatenated w1's re-blocked order (gate block j -> 2j, up block
 * j -> 2j + 1); 0: the source order. */
int sm_tq_pack_dual(const void* src, int C, int max_blocks, const int32_t* blk_expert, const int32_t* n_blocks,
                    const int32_t* off_pad, const int32_t* expert_frequency, uint8_t* out_q, uint8_t* out_sf,
                    uint8_t* row_q, uint8_t* row_sf, int concat_I, void* stream);
/* Weight gradient: out_w[e] [M, N] bf16 = A[:, rows_e] B[:, rows_e]^T over expert e's padded rows
 * (off_pad), A [M, max_blocks*128] and B [N, max_blocks*128] from sm_tq_pack.  Experts without rows
 * get zeros.  M % 128 == 0, N % 256 == 0. */
int sm_moe_wgrad(const uint8_t* a_q, const uint8_t* a_sf, const uint8_t* b_q, const uint8_t* b_sf, int M, int N,
                 int E, int max_blocks, const int32_t* off_pad, void* out_w, int32_t* err, void* stream);
/* Router backward: dlogits [T, E] fp32 from dscores [T, K] (fp32), the forward's bf16 logits,
 * scores and indices; same modes as sm_router_topk. */
int sm_router_bwd(const void* router_logits, const float* topk_scores, const int32_t* topk_indices,
                  const float* dscores, int T, int E, int K, int softmax_over_topk, int norm_topk_probs,
                  float* dlogits, void* stream);

/* Number of output-column slices (1, 2 or 4) sm_moe_down_combine visits for T output rows of
 * width H: the largest split whose bf16 slab T x (H / slices) exceeds no 80 MB share of L2.
 * Introspection only (no counterpart in the reference): lets callers and tests know which tile
 * order a shape runs. */
int sm_moe_down_slices(int T, int H);

/*
 * Expert parallelism (no counterpart in the reference, which is single-GPU: its blog lists EP as
 * future work).  E experts are sharded over W ranks, El = E / W contiguous experts per rank.  The
 * host exchanges the buffers these stages produce with NCCL all-to-alls:
 *   1. sm_ep_dispatch_prepare: route this rank's T tokens (router top-k as sm_router_topk) and
 *      write one dispatch record per (token, destination rank), rank-major in token order, plus
 *      send_counts [W] (records per destination) and ret_row [T*K] (the record index of entry k
 *      of token t if it is the first entry of its rank for the token, else -1).
 *   2. all-to-all of send_counts, then of the records (record size sm_ep_record_bytes(H, K):
 *      e4m3 row, H/128 scale bytes, then at the next 16-byte boundary K int32 local expert ids
 *      (-1 = not on this rank), K float32 scores and K int32 home rows -- the entry's row in the
 *      padded layout of the sending rank's own routing plan, or -1; see sm_ep_dispatch_records).
 *   3. sm_ep_expert_forward on the R received records: local routing metadata, packing, the two
 *      FP8 GEMMs; out_rows [R, H] bf16 row j = sum over the record's local experts of
 *      score * expert output (the per-(token, rank) partial sum).
 *   4. all-to-all of out_rows back (reversed splits) into ret [sum(send_counts), H].
 *   5. sm_ep_combine: out [T, H] = sum of each token's returned rows (fp32 accumulation).
 */
int sm_ep_record_bytes(int H, int K);
size_t sm_ep_dispatch_workspace_bytes(int T, int E, int K, int W);
int sm_ep_dispatch_prepare(const void* x, const void* router_logits, int T, int H, int E, int K, int W, int rank,
                           int softmax_over_topk, int norm_topk_probs, uint8_t* records, int32_t* ret_row,
                           int32_t* send_counts, float* topk_scores, int32_t* topk_indices, void* workspace,
                           size_t workspace_bytes, int32_t* err, void* stream);
size_t sm_ep_expert_workspace_bytes(int R, int H, int I, int El, int K);
int sm_ep_expert_forward(const uint8_t* records, int R, int H, int I, int El, int K, const uint8_t* w1q,
                         const uint8_t* w1_sf, const uint8_t* w2q, const uint8_t* w2_sf, int concat_layout,
                         void* out_rows, int32_t* expert_frequency, void* workspace, size_t workspace_bytes,
                         int32_t* err, void* stream);
int sm_ep_combine(const void* ret_rows, const int32_t* ret_row, int T, int K, int H, void* out, void* stream);

/*
 * Peer-memory variants (GPUs of one node, buffers mapped with sm_ipc_open): the exchanges become
 * loads over NVLink inside the stage kernels instead of separate all-to-alls.
 *   sm_ep_expert_forward_p2p reads the records of source rank s directly from s's send buffer
 *   peer_send_bases[s], starting at record seg_off[s] (the offset of this rank's segment there),
 *   recv_counts[s] records; the received records are numbered in source order.
 *   sm_ep_combine_p2p reads each token's partial rows from the output rows of the destination
 *   ranks: this rank's send record p of destination d (send_counts gives the segments) is row
 *   recv_start[d] + (p - segment start) of peer_out_bases[d].
 * All arrays here are host arrays of W <= 16 entries (passed to the kernels by value).  The caller
 * orders the stages with barriers (a rank's send buffer is complete before peers read it, its
 * output rows before peers combine, and nobody rewrites a buffer a peer may still read).
 */
int sm_ep_expert_forward_p2p(const void* const* peer_send_bases, const int32_t* seg_off, const int32_t* recv_counts,
                             int W, int H, int I, int El, int K, const uint8_t* w1q, const uint8_t* w1_sf,
                             const uint8_t* w2q, const uint8_t* w2_sf, int concat_layout, void* out_rows,
                             int32_t* expert_frequency, void* workspace, size_t workspace_bytes, int32_t* err,
                             void* stream);
int sm_ep_combine_p2p(const void* const* peer_out_bases, const int32_t* send_counts, const int32_t* recv_start,
                      int W, const int32_t* ret_row, int T, int K, int H, void* out, void* stream);

/*
 * Home-down variant: the owner of an expert runs only the up projection and returns each entry's
 * e4m3 intermediate row (I bytes + I/128 scale bytes, instead of an H x bf16 partial row) to the
 * token's own rank, which runs the down projection with the fused top-k combine over its own
 * routing plan (sm_route_plan of its topk_indices over all E experts) and a replica of every
 * expert's w2 -- no combine pass, 2.4-8x fewer NVLink bytes back.
 *   sm_ep_dispatch_records: the records of sm_ep_dispatch_prepare from an already computed top-k
 *     (topk_scores / topk_indices [T, K]); with the home plan's s_rev [T*K], off [E+1] and
 *     off_pad [E+1] each record also carries its entries' home rows (all three null: -1).
 *   sm_ep_expert_up_p2p: as sm_ep_expert_forward_p2p up to the up projection, whose epilogue
 *     stores every row straight into rank s's intermediate home_q_bases[s] [home_rows, I] and scale
 *     atoms home_sf_bases[s] ([home_rows/128][ceil(I/512)][512]) for records received from s
 *     (peer stores; a row outside home_rows writes SM_ERR_BAD_RETURN_ROW into err and is dropped).
 *     The caller puts a cross-rank barrier between every rank's up stage and any home's down
 *     projection (sm_moe_down_combine on its own intermediate), and between that down projection
 *     and the next up stage that writes the buffer.
 */
int sm_ep_dispatch_records(const void* x, int T, int H, int E, int K, int W, const float* topk_scores,
                           const int32_t* topk_indices, const int32_t* home_s_rev, const int32_t* home_off,
                           const int32_t* home_off_pad, uint8_t* records, int32_t* ret_row, int32_t* send_counts,
                           void* workspace, size_t workspace_bytes, int32_t* err, void* stream);
int sm_ep_expert_up_p2p(const void* const* peer_send_bases, const int32_t* seg_off, const int32_t* recv_counts,
                        int W, int H, int I, int El, int K, const uint8_t* w1q, const uint8_t* w1_sf,
                        int concat_layout, void* const* home_q_bases, void* const* home_sf_bases,
                        long long home_rows, int32_t* expert_frequency, void* workspace, size_t workspace_bytes,
                        int32_t* err, void* stream);
/*
 *   sm_ep_expert_up_home: sm_ep_expert_up_p2p with the counts left in device memory -- counts is the
 *     all-gathered matrix counts[s * count_stride + d] (records of source s for destination d, this
 *     rank d = me), read by the kernels, so the host never waits for the exchange and the call can
 *     be captured in a CUDA graph.  Every grid is sized for recv_cap records (the most this rank can
 *     receive; workspace from sm_ep_expert_workspace_bytes(recv_cap, ...)); a source's send region
 *     holds send_cap records.  A count outside those bounds writes SM_ERR_BAD_COUNT into err and
 *     nothing is read.
 */
int sm_ep_expert_up_home(const void* const* peer_send_bases, const int32_t* counts, int count_stride, int me, int W,
                         int send_cap, int recv_cap, int H, int I, int El, int K, const uint8_t* w1q,
                         const uint8_t* w1_sf, int concat_layout, void* const* home_q_bases,
                         void* const* home_sf_bases, long long home_rows, int32_t* expert_frequency,
                         void* workspace, size_t workspace_bytes, int32_t* err, void* stream);

/*
 * Device buffers shared between the processes of one node through CUDA IPC (no counterpart in the
 * reference).  sm_ipc_alloc allocates (cudaMalloc -- an explicit allocation, unlike every compute
 * entry point) and returns the 64-byte IPC handle; a peer process maps it with sm_ipc_open and
 * unmaps with sm_ipc_close; the owner frees with sm_ipc_free.
 */
int sm_ipc_alloc(size_t bytes, void** ptr, void* handle);
int sm_ipc_open(const void* handle, void** ptr);
int sm_ipc_close(void* ptr);
int sm_ipc_free(void* ptr);

/* Stream-ordered copy of `bytes` between two device addresses, either of which may be a peer's
 * buffer mapped with sm_ipc_open.  Carried out by the copy engines over NVLink, so it occupies no
 * SMs and overlaps kernels running on other streams; the expert-parallel "copy" transport moves
 * each rank's record segments and returned partial rows with one such copy per peer segment.
 * No counterpart in the reference. */
int sm_copy_d2d_async(void* dst, const void* src, size_t bytes, void* stream);

/* Leave n SMs of each device out of the persistent GEMM grids (process-wide setting, default 0), so
 * that communication kernels launched alongside (the expert-parallel all-to-alls) find free SMs.
 * No counterpart in the reference. */
int sm_set_gemm_sm_reserve(int n);

/* Self-test of the bounded waits (no counterpart in the reference): launches one kernel that waits
 * on a barrier nothing arrives on; the wait gives up after the library's bound (2 s), writes 105
 * into *err (if it held 0) and the kernel returns, leaving the context usable -- the same path by
 * which a lost arrival inside a GEMM becomes an error status instead of a hung GPU. */
int sm_selftest_bounded_wait(int32_t* err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SONIC_B200_H */
