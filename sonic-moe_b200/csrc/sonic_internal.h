// Internal constants and kernel launchers shared by the .cu files of libsonic_b200.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace smb {

constexpr int kTileTokens = 128;  // tokens per routing tile (router histogram / scatter)
constexpr int kBlockM = 128;      // rows of one block of the padded layout (one CTA's GEMM rows)
constexpr int kPadRows = 128;     // experts are padded to multiples of this
constexpr int kBlocksPerPad = kPadRows / kBlockM;
constexpr int kBlockK = 128;      // K extent of one pipeline stage (= one scale-factor group)
constexpr int kSfAtomBytes = 512; // 128 rows x 4 K-blocks of UE8M0 scale factors
constexpr int kMaxEpRanks = 16;   // ranks of one expert-parallel group (peer pointers passed by value)
constexpr int kHomeShift = 27;    // return destination = (home rank << kHomeShift) | row on that rank

enum Dtype : int { kDtypeBF16 = 0, kDtypeF16 = 1, kDtypeF32 = 2 };

// Records the calling thread's message for sm_last_error() and returns `code`.
int set_last_error(int code, const char* fmt, ...);

inline int ceil_div(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }

// Blocks of 128 rows that an expert with f rows occupies in the padded layout (always even).
__host__ __device__ inline int padded_blocks_of(int f) { return kBlocksPerPad * ((f + kPadRows - 1) / kPadRows); }

// Upper bound on the number of 128-row blocks of the padded expert layout: each non-empty expert
// adds fewer than kBlocksPerPad blocks of padding.
inline int max_padded_blocks(long long TK, int E) {
  const long long nonempty = TK < E ? TK : E;
  return static_cast<int>((TK + kBlockM - 1) / kBlockM + kBlocksPerPad * nonempty);
}

cudaError_t launch_router_topk(const void* logits, int dtype, int T, int E, int K, int sot, int renorm,
                               float* scores, int32_t* idx, int32_t* tile_counts, cudaStream_t st);
// Fused router (E % 32 == 0, 32 <= E <= 256, H % 64 == 0): logits = x @ w^T (bf16 [T, E], fp32
// accumulation on tcgen05) and the top-k of each row, plus the per-tile expert histogram.
cudaError_t launch_router_fused(const void* x, const void* w, int T, int H, int E, int K, int sot, int renorm,
                                void* logits, float* scores, int32_t* idx, int32_t* tile_counts, int* err,
                                cudaStream_t st);
// 2-D row-major tensor map: `outer` rows of `inner` elements of `esize` bytes, box box_inner x
// box_outer, 128-byte swizzle when swizzle128 (the host encoder of csrc/gemm.cu).
bool encode_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, uint64_t inner,
                    uint64_t outer, uint32_t box_inner, uint32_t box_outer, bool swizzle128);
cudaError_t launch_route_hist(const int32_t* experts, int TK, int entries_per_tile, int E, int n_tiles,
                              int32_t* tile_counts, int* err, cudaStream_t st);
// Same, but negative expert ids are holes (no entry) instead of errors.
cudaError_t launch_route_hist_holes(const int32_t* experts, int TK, int entries_per_tile, int E, int n_tiles,
                                    int32_t* tile_counts, int* err, cudaStream_t st);
cudaError_t launch_route_scan(int32_t* tile_counts, int n_tiles, int E, int TK, int32_t* freq, int32_t* off,
                              int32_t* off_pad, int32_t* blk_expert, int32_t* n_blocks, cudaStream_t st);
cudaError_t launch_route_scatter(const int32_t* experts, const int32_t* token_of_entry, int TK, int K,
                                 int entries_per_tile, int E, int n_tiles, const int32_t* tile_base,
                                 const int32_t* off, int32_t* s_scatter, int32_t* s_rev, int32_t* x_gather,
                                 cudaStream_t st);
cudaError_t launch_token_offset(const int32_t* sorted_tokens, int T, int TK, int32_t* offset, cudaStream_t st);

// zero_out (optional): a bf16 [T, H] output whose rows the kernel zero-fills, one per token (the
// layer output the down projection reduces into; 16-byte aligned, H % 8 == 0).
cudaError_t launch_quant_pack(const void* x, int T, int H, const int32_t* experts, int K, const int32_t* tok_off,
                              const int32_t* s_rev, const int32_t* off, const int32_t* off_pad, uint8_t* xq,
                              uint8_t* xsf, cudaStream_t st, void* zero_out = nullptr);
// wqt / wsft (both or neither): also the transposed e4m3 weight [E, Kd, N] and its scale atoms
cudaError_t launch_weight_prep(const void* w, int E, int N, int Kd, int concat_glu, uint8_t* wq, uint8_t* wsf,
                               cudaStream_t st, uint8_t* wqt = nullptr, uint8_t* wsft = nullptr);
// backward (csrc/backward.cu)
cudaError_t launch_weight_t(const uint8_t* wq, const uint8_t* wsf, int E, int N, int Kd, uint8_t* wqt, uint8_t* wsft,
                            cudaStream_t st);
// rowq / rowsf (padded sources only): also the row-quantised copy, column blocks re-blocked when
// row_concat_i = I > 0 (a concatenated [gate | up] source)
cudaError_t launch_tq_pack(const void* src, int C, int src_padded, const int32_t* blk_expert, const int32_t* off_pad,
                           const int32_t* off, const int32_t* freq, const int32_t* x_gather, const int32_t* n_blocks,
                           int max_blocks, uint8_t* outq, uint8_t* outsf, cudaStream_t st, uint8_t* rowq = nullptr,
                           uint8_t* rowsf = nullptr, int row_concat_i = 0);
cudaError_t launch_router_bwd(const void* logits, const float* scores, const int32_t* idx, const float* ds, int T,
                              int E, int K, int sot, int renorm, float* dlogits, cudaStream_t st);

struct GemmArgs {
  // A: padded expert-major activations [rows, Kd] e4m3 + SF atoms [rows/128][ceil(Kd/512)][512]
  const uint8_t* a;
  const uint8_t* a_sf;
  long long a_rows;
  // B: expert weights [E, N, Kd] e4m3 + SF atoms [E][N/128][ceil(Kd/512)][512]
  const uint8_t* b;
  const uint8_t* b_sf;
  int E, N, Kd;
  // padded layout
  const int32_t* blk_expert;
  const int32_t* n_blocks;
  const int32_t* off_pad;
  const int32_t* off;
  const int32_t* freq;
  // up-projection outputs: intermediate [rows, N/2] e4m3 + SF atoms
  uint8_t* out_q;
  uint8_t* out_sf;
  int concat;  // 1: B rows are 128-row blocks [gate_j; up_j] (concatenated w1 after weight prep)
  // down-projection epilogue: o[token] += score * y (bf16 atomics)
  const int32_t* s_scatter;
  const int32_t* x_gather;
  const float* scores;
  void* out_bf16;
  // up projection, expert parallel with the down projection at the tokens' home ranks: instead of
  // out_q / out_sf, padded row p goes to row (ret_dst[p] & (2^kHomeShift - 1)) of the intermediate
  // home_q[h] [home_rows, N/2] and its scale atoms home_sf[h] on rank h = ret_dst[p] >> kHomeShift
  // (peer memory; plain stores).  Null ret_dst: the local output of the single-GPU layer.
  const int32_t* ret_dst;
  uint8_t* home_q[kMaxEpRanks];
  uint8_t* home_sf[kMaxEpRanks];
  long long home_rows;
  int n_homes;
  // up projection, training forward: the pre-activation h = x W1^T (bf16, [TK, N] in expert-sorted
  // entry order: row off[e] + (p - off_pad[e]) for padded row p, columns in the caller's w1 order);
  // null: not stored
  __nv_bfloat16* preact;
  // activation-gradient GEMM (A = dO rows packed like the forward's x, B = W2 transposed [E, I, H],
  // N = I): h_in [T*K, 2I] the forward's pre-activation (expert-sorted rows); outputs out_q / out_sf
  // = dH e4m3 + atoms (padded rows, K = 2I), dh_bf16 [rows, 2I] and a_prime [rows, I] (padded
  // rows), ds [T*K] fp32 accumulated by flat entry (zeroed by the caller)
  const __nv_bfloat16* h_in;
  __nv_bfloat16* dh_bf16;
  __nv_bfloat16* a_prime;
  float* ds;
  // weight-gradient GEMM: A [a_rows, Kd] and B [N, Kd] e4m3 with K = padded entry rows (1x128 scale
  // groups along K), expert e owning K rows [off_pad[e], off_pad[e+1]); out_w [E, a_rows, N] bf16
  __nv_bfloat16* out_w;
  int* err;
  int num_sms;
  int tokens;    // T (rows of the token-major output), for the down projection's slice choice
  int n_slices;  // set by the launcher
};

// SMs the persistent GEMMs may occupy: all of the current device's, minus the number reserved with
// sm_set_gemm_sm_reserve (left free for communication kernels that run at the same time).
int gemm_grid_sms();

// Column slices (1, 2 or 4) the down projection splits its output columns into for `tokens` output
// rows of width N; all tiles of one slice run before the next slice.
int down_slices(long long tokens, int N);

cudaError_t launch_moe_up(const GemmArgs& g, cudaStream_t st);
cudaError_t launch_moe_down(const GemmArgs& g, cudaStream_t st);
cudaError_t launch_moe_dact(const GemmArgs& g, cudaStream_t st);
cudaError_t launch_moe_wgrad(const GemmArgs& g, cudaStream_t st);

}  // namespace smb
