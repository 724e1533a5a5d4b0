// extern "C" entry points of libsonic_b200.so (declared in include/sonic_b200.h).
// Argument validation, workspace carving and the stage sequence of the layer forward.
#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/sonic_b200.h"
#include "sonic_internal.h"

using namespace smb;

namespace {
thread_local std::string g_last_error;
}  // namespace

int smb::set_last_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

namespace {

template <typename... A>
int fail(int code, const char* fmt, A... args) {
  return set_last_error(code, fmt, args...);
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SM_OK;
  return fail(SM_EIO, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int num_sms() { return gemm_grid_sms(); }

// Bump allocator over a caller-provided workspace (256-byte aligned pieces).
struct Carve {
  uint8_t* base;
  size_t cap;
  size_t used = 0;
  bool ok = true;
  template <typename T>
  T* take(size_t count) {
    used = (used + 255) & ~static_cast<size_t>(255);
    T* p = reinterpret_cast<T*>(base ? base + used : nullptr);
    used += count * sizeof(T);
    if (base && used > cap) ok = false;
    return p;
  }
};

int route_tiles_tc(int T) { return ceil_div(T, kTileTokens); }
int route_tiles_general(int TK) { return ceil_div(TK, 1024); }

struct RouteWs {
  int32_t* tile_counts;
  int32_t* off_pad;
  int32_t* blk_expert;
  int32_t* n_blocks;
};

RouteWs carve_route(Carve& c, int T, long long TK, int E) {
  RouteWs w;
  const int n_tiles = route_tiles_tc(T) > route_tiles_general(static_cast<int>(TK)) ? route_tiles_tc(T)
                                                                                     : route_tiles_general(static_cast<int>(TK));
  w.tile_counts = c.take<int32_t>(static_cast<size_t>(E) * (n_tiles > 0 ? n_tiles : 1));
  w.off_pad = c.take<int32_t>(E + 1);
  w.blk_expert = c.take<int32_t>(max_padded_blocks(TK, E) + 1);
  w.n_blocks = c.take<int32_t>(1);
  return w;
}

struct FwdWs {
  RouteWs route;
  float* scores;
  int32_t* idx;
  int32_t* off;
  int32_t* s_scatter;
  int32_t* s_rev;
  int32_t* x_gather;
  uint8_t* xq;
  uint8_t* xsf;
  uint8_t* aq;
  uint8_t* asf;
  int32_t* err;
};

FwdWs carve_fwd(Carve& c, int T, int H, int I, int E, int K) {
  FwdWs w;
  const long long TK = static_cast<long long>(T) * K;
  const int mb = max_padded_blocks(TK, E);
  w.route = carve_route(c, T, TK, E);
  w.scores = c.take<float>(TK);
  w.idx = c.take<int32_t>(TK);
  w.off = c.take<int32_t>(E + 1);
  w.s_scatter = c.take<int32_t>(TK);
  w.s_rev = c.take<int32_t>(TK);
  w.x_gather = c.take<int32_t>(TK);
  w.xq = c.take<uint8_t>(static_cast<size_t>(mb) * kBlockM * H);
  w.xsf = c.take<uint8_t>(static_cast<size_t>(mb) * ceil_div(H, 512) * kSfAtomBytes);
  w.aq = c.take<uint8_t>(static_cast<size_t>(mb) * kBlockM * I);
  w.asf = c.take<uint8_t>(static_cast<size_t>(mb) * ceil_div(I, 512) * kSfAtomBytes);
  w.err = c.take<int32_t>(1);
  return w;
}

struct GenWs {
  RouteWs route;
  int32_t* off;
  int32_t* s_scatter;
  int32_t* s_rev;
  int32_t* x_gather;
  int32_t* tok_off;
  uint8_t* xq;
  uint8_t* xsf;
  uint8_t* aq;
  uint8_t* asf;
  int32_t* err;
};

GenWs carve_general(Carve& c, int T, long long TK, int H, int I, int E) {
  GenWs w;
  const int mb = max_padded_blocks(TK, E);
  w.route = carve_route(c, 0, TK, E);
  w.off = c.take<int32_t>(E + 1);
  w.s_scatter = c.take<int32_t>(TK);
  w.s_rev = c.take<int32_t>(TK);
  w.x_gather = c.take<int32_t>(TK);
  w.tok_off = c.take<int32_t>(static_cast<size_t>(T) + 1);
  w.xq = c.take<uint8_t>(static_cast<size_t>(mb) * kBlockM * H);
  w.xsf = c.take<uint8_t>(static_cast<size_t>(mb) * ceil_div(H, 512) * kSfAtomBytes);
  w.aq = c.take<uint8_t>(static_cast<size_t>(mb) * kBlockM * I);
  w.asf = c.take<uint8_t>(static_cast<size_t>(mb) * ceil_div(I, 512) * kSfAtomBytes);
  w.err = c.take<int32_t>(1);
  return w;
}

int check_router_args(int T, int E, int K, int sot, int norm) {
  if (T < 0) return fail(SM_EINVAL, "T must be >= 0 (got %d)", T);
  if (E < 1 || E > 4096) return fail(SM_EINVAL, "E must be in [1, 4096] (got %d)", E);
  if (K < 1 || K > E || K > 32) return fail(SM_EINVAL, "K must be in [1, min(E, 32)] (got K=%d, E=%d)", K, E);
  if (norm && sot)
    return fail(SM_EINVAL, "norm_topk_probs only works with softmax-then-topk (softmax_over_topk = 0)");
  return SM_OK;
}

}  // namespace

extern "C" {

const char* sm_last_error(void) { return g_last_error.c_str(); }

const char* sm_version(void) { return "sonic_b200 0.1.0 (sm_100a)"; }

int sm_router_topk(const void* logits, int dtype, int T, int E, int K, int softmax_over_topk, int norm_topk_probs,
                   float* scores, int32_t* indices, void* stream) {
  int rc = check_router_args(T, E, K, softmax_over_topk, norm_topk_probs);
  if (rc) return rc;
  if (dtype < 0 || dtype > 2) return fail(SM_EINVAL, "unknown logits dtype %d", dtype);
  if (T > 0 && (!logits || !scores || !indices)) return fail(SM_EINVAL, "null pointer");
  return cuda_status(launch_router_topk(logits, dtype, T, E, K, softmax_over_topk, norm_topk_probs, scores, indices,
                                        nullptr, static_cast<cudaStream_t>(stream)),
                     "router_topk");
}

size_t sm_route_metadata_workspace(int T, int TK, int E) {
  Carve c{nullptr, 0};
  carve_route(c, T, TK, E);
  return c.used + 256;
}

static int route_common(const int32_t* experts, const int32_t* token_of_entry, int T, long long TK, int K, int E,
                        int entries_per_tile, int n_tiles, int32_t* freq, int32_t* off, int32_t* x_gather,
                        int32_t* s_scatter, int32_t* s_rev, void* workspace, size_t ws_bytes, int32_t* err,
                        cudaStream_t st, int32_t* off_pad_out = nullptr, int32_t* blk_expert_out = nullptr,
                        int32_t* n_blocks_out = nullptr) {
  Carve c{static_cast<uint8_t*>(workspace), ws_bytes};
  RouteWs w = carve_route(c, T, TK, E);
  if (!c.ok) return fail(SM_EINVAL, "workspace too small (%zu < %zu)", ws_bytes, c.used);
  if (off_pad_out) w.off_pad = off_pad_out;
  if (blk_expert_out) w.blk_expert = blk_expert_out;
  if (n_blocks_out) w.n_blocks = n_blocks_out;
  cudaError_t e = launch_route_hist(experts, static_cast<int>(TK), entries_per_tile, E, n_tiles, w.tile_counts, err, st);
  if (e == cudaSuccess)
    e = launch_route_scan(w.tile_counts, n_tiles, E, static_cast<int>(TK), freq, off, w.off_pad, w.blk_expert,
                          w.n_blocks, st);
  if (e == cudaSuccess)
    e = launch_route_scatter(experts, token_of_entry, static_cast<int>(TK), K, entries_per_tile, E, n_tiles,
                             w.tile_counts, off, s_scatter, s_rev, x_gather, st);
  return cuda_status(e, "route_metadata");
}

int sm_route_metadata(const int32_t* topk_indices, int T, int K, int E, int32_t* expert_frequency,
                      int32_t* expert_frequency_offset, int32_t* x_gather_idx, int32_t* s_scatter_idx,
                      int32_t* s_reverse_scatter_idx, void* workspace, size_t workspace_bytes, int32_t* err,
                      void* stream) {
  if (T < 0 || K < 1 || E < 1 || E > 16384) return fail(SM_EINVAL, "bad shape T=%d K=%d E=%d (E <= 16384)", T, K, E);
  if (!expert_frequency || !expert_frequency_offset || !err) return fail(SM_EINVAL, "null pointer");
  const long long TK = static_cast<long long>(T) * K;
  if (TK > (1ll << 31) - 1) return fail(SM_EINVAL, "T*K exceeds int32");
  return route_common(topk_indices, nullptr, T, TK, K, E, kTileTokens * K, route_tiles_tc(T), expert_frequency,
                      expert_frequency_offset, x_gather_idx, s_scatter_idx, s_reverse_scatter_idx, workspace,
                      workspace_bytes, err, static_cast<cudaStream_t>(stream));
}

int sm_general_route_metadata(const int32_t* sorted_token_idx, const int32_t* expert_idx, int T, int TK, int E,
                              int32_t* expert_frequency, int32_t* expert_frequency_offset, int32_t* x_gather_idx,
                              int32_t* s_scatter_idx, int32_t* s_reverse_scatter_idx,
                              int32_t* num_activated_expert_per_token_offset, void* workspace,
                              size_t workspace_bytes, int32_t* err, void* stream) {
  if (T < 0 || TK < 0 || E < 1 || E > 16384) return fail(SM_EINVAL, "bad shape T=%d TK=%d E=%d (E <= 16384)", T, TK, E);
  if (!expert_frequency || !expert_frequency_offset || !num_activated_expert_per_token_offset || !err)
    return fail(SM_EINVAL, "null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = route_common(expert_idx, sorted_token_idx, T, TK, 1, E, 1024, route_tiles_general(TK), expert_frequency,
                        expert_frequency_offset, x_gather_idx, s_scatter_idx, s_reverse_scatter_idx, workspace,
                        workspace_bytes, err, st);
  if (rc) return rc;
  return cuda_status(launch_token_offset(sorted_token_idx, T, TK, num_activated_expert_per_token_offset, st),
                     "token_offset");
}

int sm_quant_1x128(const void* x, int R, int C, uint8_t* q, uint8_t* sf_atoms, void* stream) {
  if (R < 0 || C <= 0 || C % 128) return fail(SM_EINVAL, "need R >= 0 and C %% 128 == 0 (R=%d C=%d)", R, C);
  if (R > 0 && (!x || !q || !sf_atoms)) return fail(SM_EINVAL, "null pointer");
  if (!aligned16(x) || !aligned16(q) || !aligned16(sf_atoms)) return fail(SM_EINVAL, "pointers must be 16-byte aligned");
  return cuda_status(launch_quant_pack(x, R, C, nullptr, 1, nullptr, nullptr, nullptr, nullptr, q, sf_atoms,
                                       static_cast<cudaStream_t>(stream)),
                     "quant_1x128");
}

size_t sm_weight_sf_bytes(int E, int N, int K) {
  return static_cast<size_t>(E) * (N / 128) * ceil_div(K / 128, 4) * kSfAtomBytes;
}

int sm_weight_prep(const void* w, int E, int N, int K, int concat_glu, uint8_t* wq, uint8_t* sf_atoms, void* stream) {
  if (E < 1 || N <= 0 || K <= 0 || N % 128 || K % 128)
    return fail(SM_EINVAL, "need E >= 1 and N, K multiples of 128 (E=%d N=%d K=%d)", E, N, K);
  if (concat_glu && N % 256) return fail(SM_EINVAL, "concatenated GLU weight needs N = 2I with I %% 128 == 0");
  if (!w || !wq || !sf_atoms) return fail(SM_EINVAL, "null pointer");
  if (!aligned16(w) || !aligned16(wq)) return fail(SM_EINVAL, "pointers must be 16-byte aligned");
  return cuda_status(launch_weight_prep(w, E, N, K, concat_glu, wq, sf_atoms, static_cast<cudaStream_t>(stream)),
                     "weight_prep");
}

int sm_max_padded_blocks(long long TK, int E) { return max_padded_blocks(TK, E); }

size_t sm_moe_workspace_bytes(int T, int H, int I, int E, int K) {
  Carve c{nullptr, 0};
  carve_fwd(c, T, H, I, E, K);
  return c.used + 256;
}

static int check_layer_args(int T, int H, int I, int E, int K) {
  if (T < 0) return fail(SM_EINVAL, "T must be >= 0");
  if (H <= 0 || H % 256) return fail(SM_ENOTSUP, "hidden size must be a positive multiple of 256 (got %d)", H);
  if (I <= 0 || I % 128) return fail(SM_ENOTSUP, "intermediate size must be a positive multiple of 128 (got %d)", I);
  if (E < 1 || E > 4096) return fail(SM_EINVAL, "E must be in [1, 4096] (got %d)", E);
  if (K < 1 || K > E || K > 32) return fail(SM_EINVAL, "K must be in [1, min(E, 32)]");
  if (static_cast<long long>(T) * K > (1ll << 31) - 1) return fail(SM_EINVAL, "T*K exceeds int32");
  return SM_OK;
}

static GemmArgs up_args(const uint8_t* xq, const uint8_t* xsf, const uint8_t* w1q, const uint8_t* w1_sf, int H,
                        int I, int E, int concat, int max_blocks, const int32_t* blk_expert, const int32_t* n_blocks,
                        const int32_t* off_pad, const int32_t* freq, uint8_t* aq, uint8_t* asf, int32_t* err) {
  GemmArgs g{};
  g.a = xq;
  g.a_sf = xsf;
  g.a_rows = static_cast<long long>(max_blocks) * kBlockM;
  g.b = w1q;
  g.b_sf = w1_sf;
  g.E = E;
  g.N = 2 * I;
  g.Kd = H;
  g.blk_expert = blk_expert;
  g.n_blocks = n_blocks;
  g.off_pad = off_pad;
  g.freq = freq;
  g.out_q = aq;
  g.out_sf = asf;
  g.concat = concat;
  g.err = err;
  g.num_sms = num_sms();
  return g;
}

static GemmArgs down_args(const uint8_t* aq, const uint8_t* asf, const uint8_t* w2q, const uint8_t* w2_sf, int H,
                          int I, int E, int T, int max_blocks, const int32_t* blk_expert, const int32_t* n_blocks,
                          const int32_t* off_pad, const int32_t* off, const int32_t* freq, const int32_t* s_scatter,
                          const int32_t* x_gather, const float* scores, void* out, int32_t* err) {
  GemmArgs g{};
  g.a = aq;
  g.a_sf = asf;
  g.a_rows = static_cast<long long>(max_blocks) * kBlockM;
  g.b = w2q;
  g.b_sf = w2_sf;
  g.E = E;
  g.N = H;
  g.Kd = I;
  g.blk_expert = blk_expert;
  g.n_blocks = n_blocks;
  g.off_pad = off_pad;
  g.off = off;
  g.freq = freq;
  g.s_scatter = s_scatter;
  g.x_gather = x_gather;
  g.scores = scores;
  g.out_bf16 = out;
  g.err = err;
  g.num_sms = num_sms();
  g.tokens = T;
  return g;
}

int sm_route_plan(const int32_t* topk_indices, int T, int K, int E, int32_t* expert_frequency,
                  int32_t* expert_frequency_offset, int32_t* x_gather_idx, int32_t* s_scatter_idx,
                  int32_t* s_reverse_scatter_idx, int32_t* off_pad, int32_t* blk_expert, int32_t* n_blocks,
                  void* workspace, size_t workspace_bytes, int32_t* err, void* stream) {
  if (T < 0 || K < 1 || E < 1 || E > 16384) return fail(SM_EINVAL, "bad shape T=%d K=%d E=%d (E <= 16384)", T, K, E);
  if (!expert_frequency || !expert_frequency_offset || !off_pad || !blk_expert || !n_blocks || !err)
    return fail(SM_EINVAL, "null pointer");
  const long long TK = static_cast<long long>(T) * K;
  if (TK > (1ll << 31) - 1) return fail(SM_EINVAL, "T*K exceeds int32");
  return route_common(topk_indices, nullptr, T, TK, K, E, kTileTokens * K, route_tiles_tc(T), expert_frequency,
                      expert_frequency_offset, x_gather_idx, s_scatter_idx, s_reverse_scatter_idx, workspace,
                      workspace_bytes, err, static_cast<cudaStream_t>(stream), off_pad, blk_expert, n_blocks);
}

int sm_general_route_plan(const int32_t* sorted_token_idx, const int32_t* expert_idx, int T, int TK, int E,
                          int32_t* expert_frequency, int32_t* expert_frequency_offset, int32_t* x_gather_idx,
                          int32_t* s_scatter_idx, int32_t* s_reverse_scatter_idx,
                          int32_t* num_activated_expert_per_token_offset, int32_t* off_pad, int32_t* blk_expert,
                          int32_t* n_blocks, void* workspace, size_t workspace_bytes, int32_t* err, void* stream) {
  if (T < 0 || TK < 0 || E < 1 || E > 16384) return fail(SM_EINVAL, "bad shape T=%d TK=%d E=%d (E <= 16384)", T, TK, E);
  if (!expert_frequency || !expert_frequency_offset || !num_activated_expert_per_token_offset || !off_pad ||
      !blk_expert || !n_blocks || !err)
    return fail(SM_EINVAL, "null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = route_common(expert_idx, sorted_token_idx, T, TK, 1, E, 1024, route_tiles_general(TK), expert_frequency,
                        expert_frequency_offset, x_gather_idx, s_scatter_idx, s_reverse_scatter_idx, workspace,
                        workspace_bytes, err, st, off_pad, blk_expert, n_blocks);
  if (rc) return rc;
  return cuda_status(launch_token_offset(sorted_token_idx, T, TK, num_activated_expert_per_token_offset, st),
                     "token_offset");
}

int sm_quant_pack_general(const void* x, int T, int H, const int32_t* expert_idx,
                          const int32_t* num_activated_expert_per_token_offset, const int32_t* s_reverse_scatter_idx,
                          const int32_t* expert_frequency_offset, const int32_t* off_pad, uint8_t* xq, uint8_t* xsf,
                          void* stream) {
  if (T < 0 || H <= 0 || H % 128) return fail(SM_EINVAL, "bad shape T=%d H=%d", T, H);
  if (!aligned16(x) || !aligned16(xq) || !aligned16(xsf)) return fail(SM_EINVAL, "pointers must be 16-byte aligned");
  return cuda_status(launch_quant_pack(x, T, H, expert_idx, 0, num_activated_expert_per_token_offset,
                                       s_reverse_scatter_idx, expert_frequency_offset, off_pad, xq, xsf,
                                       static_cast<cudaStream_t>(stream)),
                     "quant_pack_general");
}

int sm_quant_pack(const void* x, int T, int H, const int32_t* topk_indices, int K, const int32_t* s_reverse_scatter_idx,
                  const int32_t* expert_frequency_offset, const int32_t* off_pad, uint8_t* xq, uint8_t* xsf,
                  void* stream) {
  if (T < 0 || H <= 0 || H % 128 || K < 1 || K > 32) return fail(SM_EINVAL, "bad shape T=%d H=%d K=%d", T, H, K);
  if (!aligned16(x) || !aligned16(xq) || !aligned16(xsf)) return fail(SM_EINVAL, "pointers must be 16-byte aligned");
  return cuda_status(launch_quant_pack(x, T, H, topk_indices, K, nullptr, s_reverse_scatter_idx, expert_frequency_offset,
                                       off_pad, xq, xsf, static_cast<cudaStream_t>(stream)),
                     "quant_pack");
}

int sm_moe_up(const uint8_t* xq, const uint8_t* xsf, const uint8_t* w1q, const uint8_t* w1_sf, int H, int I, int E,
              int concat_layout, int max_blocks, const int32_t* blk_expert, const int32_t* n_blocks,
              const int32_t* off_pad, const int32_t* expert_frequency, uint8_t* aq, uint8_t* asf, int32_t* err,
              void* stream) {
  if (H <= 0 || H % 128 || I <= 0 || I % 128 || E < 1 || max_blocks < 0)
    return fail(SM_EINVAL, "bad shape H=%d I=%d E=%d", H, I, E);
  if (!err) return fail(SM_EINVAL, "err word required");
  GemmArgs g = up_args(xq, xsf, w1q, w1_sf, H, I, E, concat_layout, max_blocks, blk_expert, n_blocks, off_pad,
                       expert_frequency, aq, asf, err);
  return cuda_status(launch_moe_up(g, static_cast<cudaStream_t>(stream)), "moe_up");
}

int sm_moe_up_preact(const uint8_t* xq, const uint8_t* xsf, const uint8_t* w1q, const uint8_t* w1_sf, int H, int I,
                     int E, int concat_layout, int max_blocks, const int32_t* blk_expert, const int32_t* n_blocks,
                     const int32_t* off_pad, const int32_t* expert_frequency_offset, const int32_t* expert_frequency,
                     uint8_t* aq, uint8_t* asf, void* preact, int32_t* err, void* stream) {
  if (H <= 0 || H % 128 || I <= 0 || I % 128 || E < 1 || max_blocks < 0)
    return fail(SM_EINVAL, "bad shape H=%d I=%d E=%d", H, I, E);
  if (!err || !preact || !expert_frequency_offset) return fail(SM_EINVAL, "null pointer");
  if (!aligned16(preact)) return fail(SM_EINVAL, "pointers must be 16-byte aligned");
  GemmArgs g = up_args(xq, xsf, w1q, w1_sf, H, I, E, concat_layout, max_blocks, blk_expert, n_blocks, off_pad,
                       expert_frequency, aq, asf, err);
  g.off = expert_frequency_offset;
  g.preact = static_cast<__nv_bfloat16*>(preact);
  return cuda_status(launch_moe_up(g, static_cast<cudaStream_t>(stream)), "moe_up_preact");
}

int sm_moe_down_combine(const uint8_t* aq, const uint8_t* asf, const uint8_t* w2q, const uint8_t* w2_sf, int H, int I,
                        int E, int T, int max_blocks, const int32_t* blk_expert, const int32_t* n_blocks,
                        const int32_t* off_pad, const int32_t* expert_frequency_offset,
                        const int32_t* expert_frequency, const int32_t* s_scatter_idx, const int32_t* x_gather_idx,
                        const float* topk_scores, void* out, int32_t* err, void* stream) {
  if (H <= 0 || H % 256 || I <= 0 || I % 128 || E < 1 || T < 0 || max_blocks < 0)
    return fail(SM_ENOTSUP, "bad shape H=%d I=%d E=%d T=%d (H %% 256 == 0, I %% 128 == 0)", H, I, E, T);
  if (!err) return fail(SM_EINVAL, "err word required");
  GemmArgs g = down_args(aq, asf, w2q, w2_sf, H, I, E, T, max_blocks, blk_expert, n_blocks, off_pad,
                         expert_frequency_offset, expert_frequency, s_scatter_idx, x_gather_idx, topk_scores, out, err);
  return cuda_status(launch_moe_down(g, static_cast<cudaStream_t>(stream)), "moe_down_combine");
}

// ---------------------------------------------------------------------------------------------
// backward
int sm_weight_prep_t(const uint8_t* wq, const uint8_t* sf_atoms, int E, int N, int K, uint8_t* wq_t,
                     uint8_t* sf_atoms_t, void* stream) {
  if (E < 1 || N <= 0 || K <= 0 || N % 128 || K % 128)
    return fail(SM_EINVAL, "need E >= 1 and N, K multiples of 128 (E=%d N=%d K=%d)", E, N, K);
  if (!wq || !sf_atoms || !wq_t || !sf_atoms_t) return fail(SM_EINVAL, "null pointer");
  if (!aligned16(wq) || !aligned16(wq_t)) return fail(SM_EINVAL, "pointers must be 16-byte aligned");
  return cuda_status(launch_weight_t(wq, sf_atoms, E, N, K, wq_t, sf_atoms_t, static_cast<cudaStream_t>(stream)),
                     "weight_prep_t");
}

int sm_weight_prep_with_t(const void* w, int E, int N, int K, int concat_glu, uint8_t* wq, uint8_t* sf_atoms,
                          uint8_t* wq_t, uint8_t* sf_atoms_t, void* stream) {
  if (E < 1 || N <= 0 || K <= 0 || N % 128 || K % 128)
    return fail(SM_EINVAL, "need E >= 1 and N, K multiples of 128 (E=%d N=%d K=%d)", E, N, K);
  if (concat_glu && N % 256) return fail(SM_EINVAL, "concatenated GLU weight needs N = 2I with I %% 128 == 0");
  if (!w || !wq || !sf_atoms || !wq_t || !sf_atoms_t) return fail(SM_EINVAL, "null pointer");
  if (!aligned16(w) || !aligned16(wq) || !aligned16(wq_t)) return fail(SM_EINVAL, "pointers must be 16-byte aligned");
  return cuda_status(launch_weight_prep(w, E, N, K, concat_glu, wq, sf_atoms, static_cast<cudaStream_t>(stream),
                                        wq_t, sf_atoms_t),
                     "weight_prep_with_t");
}

int sm_moe_dact(const uint8_t* doq, const uint8_t* dosf, const uint8_t* w2t_q, const uint8_t* w2t_sf, int H, int I,
                int E, int max_blocks, const int32_t* blk_expert, const int32_t* n_blocks, const int32_t* off_pad,
                const int32_t* expert_frequency_offset, const int32_t* expert_frequency, const int32_t* s_scatter_idx,
                const float* topk_scores, const void* preact, int concat_layout, uint8_t* dh_q, uint8_t* dh_sf,
                void* dh_bf16, void* a_prime, float* dscores, int32_t* err, void* stream) {
  if (H <= 0 || H % 128 || I <= 0 || I % 256 || E < 1 || max_blocks < 0)
    return fail(SM_ENOTSUP, "bad shape H=%d I=%d E=%d (H %% 128 == 0, I %% 256 == 0)", H, I, E);
  if (!err || !preact || !dh_bf16 || !a_prime || !dscores || !topk_scores || !s_scatter_idx ||
      !expert_frequency_offset || (dh_q == nullptr) != (dh_sf == nullptr))
    return fail(SM_EINVAL, "null pointer (dh_q and dh_sf are both set or both NULL)");
  if (!aligned16(preact) || !aligned16(dh_q) || !aligned16(dh_bf16) || !aligned16(a_prime))
    return fail(SM_EINVAL, "pointers must be 16-byte aligned");
  GemmArgs g = up_args(doq, dosf, w2t_q, w2t_sf, H, I / 2, E, concat_layout ? 1 : 0, max_blocks, blk_expert,
                       n_blocks, off_pad, expert_frequency, dh_q, dh_sf, err);
  g.N = I;  // output columns of this GEMM: the intermediate
  g.off = expert_frequency_offset;
  g.s_scatter = s_scatter_idx;
  g.scores = topk_scores;
  g.h_in = static_cast<const __nv_bfloat16*>(preact);
  g.dh_bf16 = static_cast<__nv_bfloat16*>(dh_bf16);
  g.a_prime = static_cast<__nv_bfloat16*>(a_prime);
  g.ds = dscores;
  return cuda_status(launch_moe_dact(g, static_cast<cudaStream_t>(stream)), "moe_dact");
}

int sm_tq_pack(const void* src, int C, int src_padded, int max_blocks, const int32_t* blk_expert,
               const int32_t* n_blocks, const int32_t* off_pad, const int32_t* expert_frequency_offset,
               const int32_t* expert_frequency, const int32_t* x_gather_idx, uint8_t* out_q, uint8_t* out_sf,
               void* stream) {
  if (C <= 0 || C % 128 || max_blocks < 0) return fail(SM_EINVAL, "need C %% 128 == 0 (C=%d)", C);
  if (!src || !blk_expert || !n_blocks || !off_pad || !expert_frequency || !out_q || !out_sf ||
      (!src_padded && (!x_gather_idx || !expert_frequency_offset)))
    return fail(SM_EINVAL, "null pointer");
  if (!aligned16(src) || !aligned16(out_q)) return fail(SM_EINVAL, "pointers must be 16-byte aligned");
  return cuda_status(launch_tq_pack(src, C, src_padded, blk_expert, off_pad, expert_frequency_offset, expert_frequency,
                                    x_gather_idx, n_blocks, max_blocks, out_q, out_sf,
                                    static_cast<cudaStream_t>(stream)),
                     "tq_pack");
}

int sm_tq_pack_dual(const void* src, int C, int max_blocks, const int32_t* blk_expert, const int32_t* n_blocks,
                    const int32_t* off_pad, const int32_t* expert_frequency, uint8_t* out_q, uint8_t* out_sf,
                    uint8_t* row_q, uint8_t* row_sf, int concat_I, void* stream) {
  if (C <= 0 || C % 128 || max_blocks < 0) return fail(SM_EINVAL, "need C %% 128 == 0 (C=%d)", C);
  if (concat_I < 0 || (concat_I > 0 && (2 * concat_I != C || concat_I % 128)))
    return fail(SM_EINVAL, "concat_I must be 0 or C / 2 with I %% 128 == 0 (C=%d, I=%d)", C, concat_I);
  if (!src || !blk_expert || !n_blocks || !off_pad || !expert_frequency || !out_q || !out_sf || !row_q || !row_sf)
    return fail(SM_EINVAL, "null pointer");
  if (!aligned16(src) || !aligned16(out_q) || !aligned16(row_q)) return fail(SM_EINVAL, "pointers must be 16-byte aligned");
  return cuda_status(launch_tq_pack(src, C, 1, blk_expert, off_pad, nullptr, expert_frequency, nullptr, n_blocks,
                                    max_blocks, out_q, out_sf, static_cast<cudaStream_t>(stream), row_q, row_sf,
                                    concat_I),
                     "tq_pack_dual");
}

int sm_moe_wgrad(const uint8_t* a_q, const uint8_t* a_sf, const uint8_t* b_q, const uint8_t* b_sf, int M, int N,
                 int E, int max_blocks, const int32_t* off_pad, void* out_w, int32_t* err, void* stream) {
  if (M <= 0 || M % 128 || N <= 0 || N % 256 || E < 1 || max_blocks < 0)
    return fail(SM_ENOTSUP, "bad shape M=%d N=%d E=%d (M %% 128 == 0, N %% 256 == 0)", M, N, E);
  if (!a_q || !a_sf || !b_q || !b_sf || !off_pad || !out_w || !err) return fail(SM_EINVAL, "null pointer");
  if (!aligned16(out_w) || !aligned16(a_q) || !aligned16(b_q)) return fail(SM_EINVAL, "pointers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // experts without rows get no tile: their gradient is the zeros written here
  cudaError_t e = cudaMemsetAsync(out_w, 0, static_cast<size_t>(E) * M * N * 2, st);
  if (e != cudaSuccess || max_blocks == 0) return cuda_status(e, "moe_wgrad");
  GemmArgs g{};
  g.a = a_q;
  g.a_sf = a_sf;
  g.a_rows = M;
  g.b = b_q;
  g.b_sf = b_sf;
  g.E = E;
  g.N = N;
  g.Kd = max_blocks * kBlockM;
  g.off_pad = off_pad;
  g.out_w = static_cast<__nv_bfloat16*>(out_w);
  g.err = err;
  g.num_sms = num_sms();
  return cuda_status(launch_moe_wgrad(g, st), "moe_wgrad");
}

int sm_router_bwd(const void* router_logits, const float* topk_scores, const int32_t* topk_indices,
                  const float* dscores, int T, int E, int K, int softmax_over_topk, int norm_topk_probs,
                  float* dlogits, void* stream) {
  int rc = check_router_args(T, E, K, softmax_over_topk, norm_topk_probs);
  if (rc) return rc;
  if (T > 0 && (!router_logits || !topk_scores || !topk_indices || !dscores || !dlogits))
    return fail(SM_EINVAL, "null pointer");
  return cuda_status(launch_router_bwd(router_logits, topk_scores, topk_indices, dscores, T, E, K, softmax_over_topk,
                                       norm_topk_probs, dlogits, static_cast<cudaStream_t>(stream)),
                     "router_bwd");
}

int sm_moe_down_slices(int T, int H) {
  if (T < 0 || H <= 0 || H % 256) return fail(SM_EINVAL, "need T >= 0 and H %% 256 == 0 (T=%d H=%d)", T, H);
  return down_slices(T, H);
}

}  // extern "C"

static int check_fused_router_args(int H, int E) {
  if (E % 32 != 0 || E < 32 || E > 256)
    return fail(SM_ENOTSUP, "the fused router needs E %% 32 == 0 and 32 <= E <= 256 (got E=%d)", E);
  if (H <= 0 || H % 64) return fail(SM_ENOTSUP, "the fused router needs H %% 64 == 0 (got H=%d)", H);
  return SM_OK;
}

// The layer forward; the router stage either ranks the given bf16 logits (router_weight null) or
// computes them from x and router_weight with the fused router, writing them to router_logits.
static int moe_forward_impl(const void* x, const void* router_logits, const void* router_weight, void* logits_out,
                            int T, int H, int I, int E, int K, int softmax_over_topk, int norm_topk_probs,
                            int concat_layout, const uint8_t* w1q, const uint8_t* w1_sf, const uint8_t* w2q,
                            const uint8_t* w2_sf, void* out, int32_t* expert_frequency, float* topk_scores,
                            int32_t* topk_indices, void* workspace, size_t workspace_bytes, int32_t* err,
                            void* stream) {
  int rc = check_layer_args(T, H, I, E, K);
  if (rc) return rc;
  rc = check_router_args(T, E, K, softmax_over_topk, norm_topk_probs);
  if (rc) return rc;
  if (router_weight) {
    rc = check_fused_router_args(H, E);
    if (rc) return rc;
  }
  if (!expert_frequency) return fail(SM_EINVAL, "null pointer");
  if (T == 0) {  // nothing routed: zero expert counts, empty output
    return cuda_status(cudaMemsetAsync(expert_frequency, 0, sizeof(int32_t) * E, static_cast<cudaStream_t>(stream)),
                       "moe_forward");
  }
  if (!x || !router_logits || !w1q || !w1_sf || !w2q || !w2_sf || !out) return fail(SM_EINVAL, "null pointer");
  if (router_weight && !aligned16(router_weight)) return fail(SM_EINVAL, "pointers must be 16-byte aligned");
  if (!aligned16(x) || !aligned16(out) || !aligned16(w1q) || !aligned16(w2q) || !aligned16(w1_sf) ||
      !aligned16(w2_sf) || !aligned16(workspace))
    return fail(SM_EINVAL, "pointers must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carve c{static_cast<uint8_t*>(workspace), workspace_bytes};
  FwdWs w = carve_fwd(c, T, H, I, E, K);
  if (!c.ok) return fail(SM_EINVAL, "workspace too small (%zu < %zu)", workspace_bytes, c.used);
  int32_t* errw = err ? err : w.err;
  float* scores = topk_scores ? topk_scores : w.scores;
  int32_t* idx = topk_indices ? topk_indices : w.idx;
  const long long TK = static_cast<long long>(T) * K;
  const int n_tiles = route_tiles_tc(T);
  const int mb = max_padded_blocks(TK, E);

  cudaError_t e = cudaSuccess;
  if (!err) e = cudaMemsetAsync(w.err, 0, sizeof(int32_t), st);
  if (e == cudaSuccess && router_weight)
    e = launch_router_fused(x, router_weight, T, H, E, K, softmax_over_topk, norm_topk_probs, logits_out, scores, idx,
                            w.route.tile_counts, errw, st);
  else if (e == cudaSuccess)
    e = launch_router_topk(router_logits, kDtypeBF16, T, E, K, softmax_over_topk, norm_topk_probs, scores, idx,
                           w.route.tile_counts, st);
  if (e == cudaSuccess)
    e = launch_route_scan(w.route.tile_counts, n_tiles, E, static_cast<int>(TK), expert_frequency, w.off,
                          w.route.off_pad, w.route.blk_expert, w.route.n_blocks, st);
  if (e == cudaSuccess)
    e = launch_route_scatter(idx, nullptr, static_cast<int>(TK), K, kTileTokens * K, E, n_tiles, w.route.tile_counts,
                             w.off, w.s_scatter, w.s_rev, w.x_gather, st);
  // the pack kernel also zero-fills the output rows the down projection reduces into
  if (e == cudaSuccess)
    e = launch_quant_pack(x, T, H, idx, K, nullptr, w.s_rev, w.off, w.route.off_pad, w.xq, w.xsf, st, out);
  if (e == cudaSuccess) {
    GemmArgs g = up_args(w.xq, w.xsf, w1q, w1_sf, H, I, E, concat_layout, mb, w.route.blk_expert, w.route.n_blocks,
                         w.route.off_pad, expert_frequency, w.aq, w.asf, errw);
    e = launch_moe_up(g, st);
  }
  if (e == cudaSuccess) {
    GemmArgs g = down_args(w.aq, w.asf, w2q, w2_sf, H, I, E, T, mb, w.route.blk_expert, w.route.n_blocks,
                           w.route.off_pad, w.off, expert_frequency, w.s_scatter, w.x_gather, scores, out, errw);
    e = launch_moe_down(g, st);
  }
  return cuda_status(e, "moe_forward");
}

extern "C" {

int sm_moe_forward(const void* x, const void* router_logits, int T, int H, int I, int E, int K,
                   int softmax_over_topk, int norm_topk_probs, int concat_layout, const uint8_t* w1q,
                   const uint8_t* w1_sf, const uint8_t* w2q, const uint8_t* w2_sf, void* out,
                   int32_t* expert_frequency, float* topk_scores, int32_t* topk_indices, void* workspace,
                   size_t workspace_bytes, int32_t* err, void* stream) {
  return moe_forward_impl(x, router_logits, nullptr, nullptr, T, H, I, E, K, softmax_over_topk, norm_topk_probs,
                          concat_layout, w1q, w1_sf, w2q, w2_sf, out, expert_frequency, topk_scores, topk_indices,
                          workspace, workspace_bytes, err, stream);
}

int sm_moe_forward_fused_router(const void* x, const void* router_weight, int T, int H, int I, int E, int K,
                                int softmax_over_topk, int norm_topk_probs, int concat_layout, const uint8_t* w1q,
                                const uint8_t* w1_sf, const uint8_t* w2q, const uint8_t* w2_sf, void* out,
                                void* router_logits, int32_t* expert_frequency, float* topk_scores,
                                int32_t* topk_indices, void* workspace, size_t workspace_bytes, int32_t* err,
                                void* stream) {
  if (T > 0 && (!router_weight || !router_logits)) return fail(SM_EINVAL, "null pointer");
  if (T > 0 && !aligned16(router_logits)) return fail(SM_EINVAL, "pointers must be 16-byte aligned");
  return moe_forward_impl(x, router_logits, router_weight, router_logits, T, H, I, E, K, softmax_over_topk,
                          norm_topk_probs, concat_layout, w1q, w1_sf, w2q, w2_sf, out, expert_frequency, topk_scores,
                          topk_indices, workspace, workspace_bytes, err, stream);
}

int sm_router_fused(const void* x, const void* router_weight, int T, int H, int E, int K, int softmax_over_topk,
                    int norm_topk_probs, void* router_logits, float* scores, int32_t* indices, void* workspace,
                    size_t workspace_bytes, int32_t* err, void* stream) {
  int rc = check_router_args(T, E, K, softmax_over_topk, norm_topk_probs);
  if (rc) return rc;
  rc = check_fused_router_args(H, E);
  if (rc) return rc;
  if (T == 0) return SM_OK;
  if (!x || !router_weight || !router_logits || !scores || !indices || !err || !workspace)
    return fail(SM_EINVAL, "null pointer");
  if (!aligned16(x) || !aligned16(router_weight) || !aligned16(router_logits))
    return fail(SM_EINVAL, "pointers must be 16-byte aligned");
  const size_t need = static_cast<size_t>(E) * route_tiles_tc(T) * sizeof(int32_t);
  if (workspace_bytes < need) return fail(SM_EINVAL, "workspace too small (%zu < %zu)", workspace_bytes, need);
  return cuda_status(launch_router_fused(x, router_weight, T, H, E, K, softmax_over_topk, norm_topk_probs,
                                         router_logits, scores, indices, static_cast<int32_t*>(workspace), err,
                                         static_cast<cudaStream_t>(stream)),
                     "router_fused");
}

size_t sm_router_fused_workspace(int T, int E) {
  return static_cast<size_t>(E > 0 ? E : 1) * (route_tiles_tc(T > 0 ? T : 1)) * sizeof(int32_t);
}

size_t sm_moe_general_workspace_bytes(int T, int TK, int H, int I, int E) {
  Carve c{nullptr, 0};
  carve_general(c, T, TK, H, I, E);
  return c.used + 256;
}

int sm_moe_general_forward(const void* x, int T, int H, int I, int E, int TK, const float* router_scores,
                           const int32_t* token_indices, const int32_t* expert_indices, int concat_layout,
                           const uint8_t* w1q, const uint8_t* w1_sf, const uint8_t* w2q, const uint8_t* w2_sf,
                           void* out, int32_t* expert_frequency, void* workspace, size_t workspace_bytes,
                           int32_t* err, void* stream) {
  int rc = check_layer_args(T, H, I, E, 1);
  if (rc) return rc;
  if (TK < 0) return fail(SM_EINVAL, "TK must be >= 0");
  if (!expert_frequency) return fail(SM_EINVAL, "null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (T == 0 || TK == 0) {
    cudaError_t e0 = cudaMemsetAsync(expert_frequency, 0, sizeof(int32_t) * E, st);
    if (e0 == cudaSuccess && T > 0) e0 = cudaMemsetAsync(out, 0, static_cast<size_t>(T) * H * 2, st);
    return cuda_status(e0, "moe_general_forward");
  }
  if (!x || !router_scores || !token_indices || !expert_indices || !w1q || !w1_sf || !w2q || !w2_sf || !out)
    return fail(SM_EINVAL, "null pointer");
  if (!aligned16(x) || !aligned16(out) || !aligned16(w1q) || !aligned16(w2q) || !aligned16(w1_sf) ||
      !aligned16(w2_sf) || !aligned16(workspace))
    return fail(SM_EINVAL, "pointers must be 16-byte aligned");
  Carve c{static_cast<uint8_t*>(workspace), workspace_bytes};
  GenWs w = carve_general(c, T, TK, H, I, E);
  if (!c.ok) return fail(SM_EINVAL, "workspace too small (%zu < %zu)", workspace_bytes, c.used);
  int32_t* errw = err ? err : w.err;
  const int n_tiles = route_tiles_general(TK);
  const int mb = max_padded_blocks(TK, E);
  cudaError_t e = cudaSuccess;
  if (!err) e = cudaMemsetAsync(w.err, 0, sizeof(int32_t), st);
  if (e == cudaSuccess) e = launch_route_hist(expert_indices, TK, 1024, E, n_tiles, w.route.tile_counts, errw, st);
  if (e == cudaSuccess)
    e = launch_route_scan(w.route.tile_counts, n_tiles, E, TK, expert_frequency, w.off, w.route.off_pad,
                          w.route.blk_expert, w.route.n_blocks, st);
  if (e == cudaSuccess)
    e = launch_route_scatter(expert_indices, token_indices, TK, 1, 1024, E, n_tiles, w.route.tile_counts, w.off,
                             w.s_scatter, w.s_rev, w.x_gather, st);
  if (e == cudaSuccess) e = launch_token_offset(token_indices, T, TK, w.tok_off, st);
  if (e == cudaSuccess)
    e = launch_quant_pack(x, T, H, expert_indices, 0, w.tok_off, w.s_rev, w.off, w.route.off_pad, w.xq, w.xsf, st,
                          out);
  if (e == cudaSuccess) {
    GemmArgs g = up_args(w.xq, w.xsf, w1q, w1_sf, H, I, E, concat_layout, mb, w.route.blk_expert, w.route.n_blocks,
                         w.route.off_pad, expert_frequency, w.aq, w.asf, errw);
    e = launch_moe_up(g, st);
  }
  if (e == cudaSuccess) {
    GemmArgs g = down_args(w.aq, w.asf, w2q, w2_sf, H, I, E, T, mb, w.route.blk_expert, w.route.n_blocks,
                           w.route.off_pad, w.off, expert_frequency, w.s_scatter, w.x_gather, router_scores, out,
                           errw);
    e = launch_moe_down(g, st);
  }
  return cuda_status(e, "moe_general_forward");
}

}  // extern "C"
