// Expert-parallel stages of the layer forward (experts sharded over W ranks, El = E / W per rank;
// rank d owns global experts [d*El, (d+1)*El)).  The exchanges themselves are NCCL all-to-alls
// issued by the host; these kernels build and consume the exchanged buffers.
//
// A dispatch record carries one token to one destination rank (a token routed to several experts
// of the same rank travels once):
//   [ H bytes e4m3 row | H/128 UE8M0 scale bytes | pad to 16 | K int32 local expert ids |
//     K float32 scores | K int32 home rows | pad to 16 ]
// Expert slots not on the destination rank hold -1 / 0 / -1.  A home row is the entry's row in the
// padded expert-major layout of the token's own rank (set by sm_ep_dispatch_records from that
// rank's routing plan, else -1): the expert-parallel variant that runs the down projection at home
// returns the entry's intermediate row there.  The metadata starts on a 16-byte boundary
// (meta_offset) so its 4-byte fields are aligned whatever H is.
//
// ep_dest_kernel       -- per (token, k): destination rank if k is the first entry of that rank for
//                         the token, else -1 (duplicates ride along in the same record)
// ep_send_pack_kernel  -- quantise each token once (1x128, same spec as the local path) and write
//                         its records at their dispatch positions (rank-major, token order)
// ep_recv_unpack_kernel-- local expert ids / scores of the received records as [R, K] arrays
// ep_pack_fp8_kernel   -- copy received e4m3 rows + scales into the padded expert-major layout
//                         (and, for the home-down variant, each row's return destination)
// ep_combine_kernel    -- owner side: o[t] = sum of the returned partial rows of token t (fp32)
#include <cstring>

#include "../../include/sonic_b200.h"
#include "common.cuh"
#include "sonic_internal.h"

namespace smb {

__host__ __device__ constexpr int ep_meta_offset(int H) { return (H + H / kBlockK + 15) / 16 * 16; }

constexpr int kMaxRanks = kMaxEpRanks;

// The segment table of a RecordSource when it is resolved on the device from the all-gathered
// count matrix (ep_resolve_counts_kernel): start[W] is the number of records received.
struct RecordIndex {
  int start[kMaxRanks + 1];
  int seg_off[kMaxRanks];
};

// Where received record j lives: in the send buffer of source rank s (possibly another GPU's memory,
// reached by peer loads) at record index seg_off[s] + (j - start[s]), for start[s] <= j < start[s+1].
// A contiguous local buffer is the case W = 1, seg_off = 0.  With dev != nullptr the table is read
// from device memory instead of the by-value arrays, and the kernels' record count is an upper bound.
struct RecordSource {
  const uint8_t* base[kMaxRanks];
  int seg_off[kMaxRanks];
  int start[kMaxRanks + 1];
  int W;
  int rb;
  const RecordIndex* dev;
};

__device__ __forceinline__ int rs_start(const RecordSource& rs, int s) { return rs.dev ? rs.dev->start[s] : rs.start[s]; }

// records actually received: R itself for a host-resolved table, else the device table's total (<= R)
__device__ __forceinline__ int rs_count(const RecordSource& rs, int R) { return rs.dev ? rs.dev->start[rs.W] : R; }

__device__ __forceinline__ int record_src(const RecordSource& rs, int j) {
  int s = 0;
  while (s + 1 < rs.W && j >= rs_start(rs, s + 1)) ++s;
  return s;
}

__device__ __forceinline__ const uint8_t* record_ptr(const RecordSource& rs, int j) {
  const int s = record_src(rs, j);
  const int seg = rs.dev ? rs.dev->seg_off[s] : rs.seg_off[s];
  return rs.base[s] + static_cast<size_t>(seg + (j - rs_start(rs, s))) * rs.rb;
}

// One thread: this rank's segment table from counts[s * stride + d] (records of source s for
// destination d; device memory, written by the count all-gather).  A count outside the buffers
// (negative, a segment past send_cap records of its source, more than r_cap records in all) sets
// SM_ERR_BAD_COUNT and leaves an empty table, so no record is read.
__global__ void ep_resolve_counts_kernel(const int32_t* __restrict__ counts, int stride, int W, int me, int send_cap,
                                         int r_cap, RecordIndex* __restrict__ out, int32_t* __restrict__ err) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  long long R = 0;
  bool bad = false;
  for (int s = 0; s < W; ++s) {
    long long seg = 0;
    for (int d = 0; d < me; ++d) {
      const int c = counts[static_cast<size_t>(s) * stride + d];
      bad = bad || c < 0;
      seg += c;
    }
    const int n = counts[static_cast<size_t>(s) * stride + me];
    bad = bad || n < 0 || seg + n > send_cap;
    out->start[s] = static_cast<int>(bad ? 0 : R);
    out->seg_off[s] = static_cast<int>(bad ? 0 : seg);
    R += n;
  }
  bad = bad || R > r_cap;
  if (bad) {
    for (int s = 0; s <= W; ++s) out->start[s] = 0;
    for (int s = 0; s < W; ++s) out->seg_off[s] = 0;
    atomicCAS(err, 0, kErrBadCount);
  } else {
    out->start[W] = static_cast<int>(R);
  }
}

// Where the partial row for this rank's send record p lives: p falls in the segment of destination
// rank d (send_off[d] <= p < send_off[d+1]); rank d computed it as row recv_start[d] + (p - send_off[d])
// of its output rows at base[d].
struct RowSource {
  const __nv_bfloat16* base[kMaxRanks];
  int send_off[kMaxRanks + 1];
  int recv_start[kMaxRanks];
  int W;
};

__device__ __forceinline__ const __nv_bfloat16* partial_row_ptr(const RowSource& rs, int p, int H) {
  int d = 0;
  while (d + 1 < rs.W && p >= rs.send_off[d + 1]) ++d;
  return rs.base[d] + static_cast<size_t>(rs.recv_start[d] + (p - rs.send_off[d])) * H;
}

// 16-byte load cached in L2 only (peer memory written by another GPU's kernel).
__device__ __forceinline__ uint4 ld_cg16(const void* p) { return __ldcg(reinterpret_cast<const uint4*>(p)); }

__device__ __forceinline__ void bf16x8_to_f32_ep(const uint4& raw, float* v) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__global__ void ep_dest_kernel(const int32_t* __restrict__ idx, int T, int K, int El, int32_t* __restrict__ dest) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  for (int k = 0; k < K; ++k) {
    const int d = idx[t * K + k] / El;
    bool first = true;
    for (int j = 0; j < k; ++j) first = first && (idx[t * K + j] / El != d);
    dest[t * K + k] = first ? d : -1;
  }
}

// One warp per token (same lane layout as quant_pack_kernel).
__global__ void __launch_bounds__(256)
    ep_send_pack_kernel(const __nv_bfloat16* __restrict__ x, int T, int H, const int32_t* __restrict__ idx,
                        const float* __restrict__ scores, int K, int El, const int32_t* __restrict__ dest,
                        const int32_t* __restrict__ pos, int record_bytes, uint8_t* __restrict__ records,
                        int32_t* __restrict__ ret_row, const int32_t* __restrict__ home_s_rev,
                        const int32_t* __restrict__ home_off, const int32_t* __restrict__ home_off_pad) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  // destination record of each of the token's (up to 32) entries; lane k holds entry k
  int my_pos = -1, my_rank = -1;
  if (lane < K) {
    const int f = t * K + lane;
    my_rank = dest[f];
    my_pos = my_rank >= 0 ? pos[f] : -1;
    ret_row[f] = my_pos;
  }
  const __nv_bfloat16* src = x + static_cast<size_t>(t) * H;
  for (int h0 = 0; h0 < H; h0 += 256) {
    const int h = h0 + 8 * lane;
    float v[8];
    uint4 raw = (h < H) ? *reinterpret_cast<const uint4*>(src + h) : make_uint4(0, 0, 0, 0);
    bf16x8_to_f32_ep(raw, v);
    float am = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(v[i]));
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const int e8 = scale_exp_of_amax(am);
    const float inv = exp2_neg(e8);
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 4; i += 2) {
      lo |= static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(v[i], inv), __fmul_rn(v[i + 1], inv))) << (8 * i);
      hi |= static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(v[4 + i], inv), __fmul_rn(v[5 + i], inv))) << (8 * i);
    }
    for (int k = 0; k < K; ++k) {
      const int p = __shfl_sync(0xffffffffu, my_pos, k);
      if (p < 0) continue;
      uint8_t* rec = records + static_cast<size_t>(p) * record_bytes;
      if (h < H) *reinterpret_cast<uint2*>(rec + h) = make_uint2(lo, hi);
      if ((lane & 15) == 0 && h < H) rec[H + h / kBlockK] = static_cast<uint8_t>(e8 + 127);
    }
  }
  // metadata: the token's experts on each destination rank
  for (int k = 0; k < K; ++k) {
    const int p = __shfl_sync(0xffffffffu, my_pos, k);
    const int d = __shfl_sync(0xffffffffu, my_rank, k);
    if (p < 0) continue;
    uint8_t* rec = records + static_cast<size_t>(p) * record_bytes + ep_meta_offset(H);
    if (lane < K) {
      const int f = t * K + lane;
      const int e = idx[f];
      const bool mine = (e / El) == d;
      reinterpret_cast<int32_t*>(rec)[lane] = mine ? e - d * El : -1;
      reinterpret_cast<float*>(rec + 4 * K)[lane] = mine ? scores[f] : 0.0f;
      // the entry's row in the padded layout of this (home) rank's own routing plan
      reinterpret_cast<int32_t*>(rec + 8 * K)[lane] =
          (mine && home_s_rev) ? home_s_rev[f] - home_off[e] + home_off_pad[e] : -1;
    }
  }
}

__global__ void ep_recv_unpack_kernel(const RecordSource rs, int R, int H, int K, int32_t* __restrict__ idx_local,
                                      float* __restrict__ scores) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= R * K) return;
  if (i >= rs_count(rs, R) * K) {  // past the received records: holes for the metadata passes
    idx_local[i] = -1;
    scores[i] = 0.0f;
    return;
  }
  const int j = i / K, k = i - (i / K) * K;
  const uint8_t* meta = record_ptr(rs, j) + ep_meta_offset(H);
  idx_local[i] = __ldcg(reinterpret_cast<const int32_t*>(meta) + k);
  scores[i] = __ldcg(reinterpret_cast<const float*>(meta + 4 * K) + k);
}

// One warp per received record: its e4m3 row and scale bytes go to the padded row of each of its
// local entries (entries with expert -1 are skipped).  The record may sit in another GPU's send
// buffer; the row is read once (up to 8 x 16 B per lane in flight) and written to every entry.
constexpr int kPackChunks = 8;  // 16-byte loads per lane per pass (H <= 4096 in one pass)

__global__ void __launch_bounds__(256)
    ep_pack_fp8_kernel(const RecordSource rs, int R, int H, int K, int El, const int32_t* __restrict__ idx_local,
                       const int32_t* __restrict__ s_rev, const int32_t* __restrict__ off,
                       const int32_t* __restrict__ off_pad, uint8_t* __restrict__ xq, uint8_t* __restrict__ xsf,
                       int32_t* __restrict__ ret_dst) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = blockIdx.x * 8 + warp;
  if (j >= rs_count(rs, R)) return;
  int my_dst = -1;
  if (lane < K) {
    const int f = j * K + lane;
    const int e = idx_local[f];
    if (e >= 0 && e < El) my_dst = s_rev[f] - off[e] + off_pad[e];
  }
  const uint8_t* rec = record_ptr(rs, j);
  if (ret_dst != nullptr && my_dst >= 0) {
    // where the up projection returns this entry's intermediate row: source rank | its home row
    const int hr = __ldcg(reinterpret_cast<const int32_t*>(rec + ep_meta_offset(H) + 8 * K) + lane);
    ret_dst[my_dst] = (hr >= 0 && hr < (1 << kHomeShift)) ? (record_src(rs, j) << kHomeShift) | hr : -1;
  }
  const int G = H / kBlockK;
  const int KG = (G + 3) / 4;
  const uint8_t sfb = (lane < G) ? __ldcg(rec + H + lane) : 0;
  for (int h0 = 0; h0 < H; h0 += 512 * kPackChunks) {
    uint4 v[kPackChunks];
#pragma unroll
    for (int c = 0; c < kPackChunks; ++c) {
      const int h = h0 + 512 * c + 16 * lane;
      v[c] = (h < H) ? ld_cg16(rec + h) : make_uint4(0, 0, 0, 0);
    }
    for (int k = 0; k < K; ++k) {
      const int p = __shfl_sync(0xffffffffu, my_dst, k);
      if (p < 0) continue;
      uint8_t* dst = xq + static_cast<size_t>(p) * H;
#pragma unroll
      for (int c = 0; c < kPackChunks; ++c) {
        const int h = h0 + 512 * c + 16 * lane;
        if (h < H) *reinterpret_cast<uint4*>(dst + h) = v[c];
      }
    }
  }
  for (int k = 0; k < K; ++k) {
    const int p = __shfl_sync(0xffffffffu, my_dst, k);
    if (p < 0) continue;
    for (int g = lane; g < G; g += 32) {
      const uint8_t b = (g < 32) ? sfb : __ldcg(rec + H + g);  // g == lane below 32
      const size_t o = (static_cast<size_t>(p / kBlockM) * KG + g / 4) * kSfAtomBytes + 16 * (p % 32) +
                       4 * ((p % kBlockM) / 32) + (g % 4);
      xsf[o] = b;
    }
  }
}

// One CTA per token: o[t] = sum over the token's partial rows (fp32), rounded once to bf16.  The
// rows may sit in other GPUs' output buffers (peer loads); all of a token's rows for one 8-column
// slice are loaded before they are summed.
__global__ void __launch_bounds__(256)
    ep_combine_kernel(const RowSource rs, const int32_t* __restrict__ ret_row, int T, int K, int H,
                      __nv_bfloat16* __restrict__ out) {
  const int t = blockIdx.x;
  __shared__ const __nv_bfloat16* rows[32];
  __shared__ int nrows;
  if (threadIdx.x == 0) {
    int n = 0;
    for (int k = 0; k < K; ++k) {
      const int p = ret_row[t * K + k];
      if (p >= 0) rows[n++] = partial_row_ptr(rs, p, H);
    }
    nrows = n;
  }
  __syncthreads();
  const int n = nrows;
  for (int h = 8 * threadIdx.x; h < H; h += 8 * blockDim.x) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i0 = 0; i0 < n; i0 += 8) {
      uint4 raw[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) raw[i] = (i0 + i < n) ? ld_cg16(rows[i0 + i] + h) : make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float v[8];
        bf16x8_to_f32_ep(raw[i], v);
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[q] += v[q];
      }
    }
    uint4 w;
    w.x = (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(acc[1]))) << 16) |
          __bfloat16_as_ushort(__float2bfloat16_rn(acc[0]));
    w.y = (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(acc[3]))) << 16) |
          __bfloat16_as_ushort(__float2bfloat16_rn(acc[2]));
    w.z = (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(acc[5]))) << 16) |
          __bfloat16_as_ushort(__float2bfloat16_rn(acc[4]));
    w.w = (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(acc[7]))) << 16) |
          __bfloat16_as_ushort(__float2bfloat16_rn(acc[6]));
    *reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * H + h) = w;
  }
}

}  // namespace smb

using namespace smb;

namespace {

size_t a256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

int ep_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return SM_OK;
  return set_last_error(SM_EIO, "%s: %s", what, cudaGetErrorString(e));
}

}  // namespace

extern "C" {

int sm_ep_record_bytes(int H, int K) { return (ep_meta_offset(H) + 12 * K + 15) / 16 * 16; }

size_t sm_ep_dispatch_workspace_bytes(int T, int E, int K, int W) {
  const long long TK = static_cast<long long>(T) * K;
  return a256(TK * 4) * 5 + a256(static_cast<size_t>(W) * (ceil_div(T, kTileTokens) + 1) * 4) +
         a256(static_cast<size_t>(W + 1) * 4) * 2 + a256((static_cast<size_t>(max_padded_blocks(TK, W)) + 2) * 4) +
         a256(4) + 4096;
}

// Records of this rank's routed tokens: destination of each entry, rank-major dispatch order (the
// token-choice metadata over "experts" = destination ranks, duplicate (token, rank) entries as
// holes), then one warp per token quantises it and writes its records.
static int ep_dispatch_records(const void* x, int T, int H, int E, int K, int W, const float* topk_scores,
                               const int32_t* topk_indices, const int32_t* home_s_rev, const int32_t* home_off,
                               const int32_t* home_off_pad, uint8_t* records, int32_t* ret_row, int32_t* send_counts,
                               void* workspace, size_t workspace_bytes, int32_t* err, cudaStream_t st) {
  const int El = E / W;
  const long long TK = static_cast<long long>(T) * K;
  const int n_tiles = ceil_div(T, kTileTokens);
  uint8_t* p = static_cast<uint8_t*>(workspace);
  size_t used = 0;
  auto take = [&](size_t bytes) {
    uint8_t* q = p + used;
    used += a256(bytes);
    return q;
  };
  int32_t* dest = reinterpret_cast<int32_t*>(take(TK * 4));
  int32_t* pos = reinterpret_cast<int32_t*>(take(TK * 4));
  int32_t* s_scatter = reinterpret_cast<int32_t*>(take(TK * 4));
  int32_t* x_gather = reinterpret_cast<int32_t*>(take(TK * 4));
  take(TK * 4);
  int32_t* tile_counts = reinterpret_cast<int32_t*>(take(static_cast<size_t>(W) * (n_tiles + 1) * 4));
  int32_t* off = reinterpret_cast<int32_t*>(take(static_cast<size_t>(W + 1) * 4));
  int32_t* off_pad = reinterpret_cast<int32_t*>(take(static_cast<size_t>(W + 1) * 4));
  int32_t* blk = reinterpret_cast<int32_t*>(take((static_cast<size_t>(max_padded_blocks(TK, W)) + 2) * 4));
  int32_t* nblk = reinterpret_cast<int32_t*>(take(4));
  if (used > workspace_bytes) return set_last_error(SM_EINVAL, "ep dispatch: workspace too small");
  ep_dest_kernel<<<(T + 255) / 256, 256, 0, st>>>(topk_indices, T, K, El, dest);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess)
    e = launch_route_hist_holes(dest, static_cast<int>(TK), kTileTokens * K, W, n_tiles, tile_counts, err, st);
  if (e == cudaSuccess)
    e = launch_route_scan(tile_counts, n_tiles, W, static_cast<int>(TK), send_counts, off, off_pad, blk, nblk, st);
  if (e == cudaSuccess)
    e = launch_route_scatter(dest, nullptr, static_cast<int>(TK), K, kTileTokens * K, W, n_tiles, tile_counts, off,
                             s_scatter, pos, x_gather, st);
  if (e == cudaSuccess) {
    ep_send_pack_kernel<<<(T + 7) / 8, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), T, H, topk_indices,
                                                     topk_scores, K, El, dest, pos, sm_ep_record_bytes(H, K), records,
                                                     ret_row, home_s_rev, home_off, home_off_pad);
    e = cudaGetLastError();
  }
  return ep_status(e, "ep dispatch");
}

static int check_dispatch_args(int T, int H, int E, int K, int W) {
  if (T < 0 || H <= 0 || H % 256 || E < 1 || W < 1 || W > kMaxRanks || E % W || K < 1 || K > 32 || K > E)
    return set_last_error(SM_EINVAL, "ep dispatch: bad shape T=%d H=%d E=%d K=%d W=%d", T, H, E, K, W);
  return SM_OK;
}

int sm_ep_dispatch_prepare(const void* x, const void* router_logits, int T, int H, int E, int K, int W, int rank,
                           int softmax_over_topk, int norm_topk_probs, uint8_t* records, int32_t* ret_row,
                           int32_t* send_counts, float* topk_scores, int32_t* topk_indices, void* workspace,
                           size_t workspace_bytes, int32_t* err, void* stream) {
  (void)rank;
  if (int rc = check_dispatch_args(T, H, E, K, W)) return rc;
  if (!send_counts || !err || (T > 0 && (!x || !router_logits || !records || !ret_row || !topk_scores ||
                                         !topk_indices)))
    return set_last_error(SM_EINVAL, "ep dispatch: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (T == 0) return ep_status(cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * W, st), "ep dispatch");
  cudaError_t e = launch_router_topk(router_logits, kDtypeBF16, T, E, K, softmax_over_topk, norm_topk_probs,
                                     topk_scores, topk_indices, nullptr, st);
  if (e != cudaSuccess) return ep_status(e, "ep dispatch");
  return ep_dispatch_records(x, T, H, E, K, W, topk_scores, topk_indices, nullptr, nullptr, nullptr, records, ret_row,
                             send_counts, workspace, workspace_bytes, err, st);
}

int sm_ep_dispatch_records(const void* x, int T, int H, int E, int K, int W, const float* topk_scores,
                           const int32_t* topk_indices, const int32_t* home_s_rev, const int32_t* home_off,
                           const int32_t* home_off_pad, uint8_t* records, int32_t* ret_row, int32_t* send_counts,
                           void* workspace, size_t workspace_bytes, int32_t* err, void* stream) {
  if (int rc = check_dispatch_args(T, H, E, K, W)) return rc;
  if (!send_counts || !err || (T > 0 && (!x || !records || !ret_row || !topk_scores || !topk_indices)))
    return set_last_error(SM_EINVAL, "ep dispatch: null pointer");
  if ((home_s_rev == nullptr) != (home_off == nullptr) || (home_off == nullptr) != (home_off_pad == nullptr))
    return set_last_error(SM_EINVAL, "ep dispatch: the home plan needs s_rev, off and off_pad together");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (T == 0) return ep_status(cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * W, st), "ep dispatch");
  return ep_dispatch_records(x, T, H, E, K, W, topk_scores, topk_indices, home_s_rev, home_off, home_off_pad, records,
                             ret_row, send_counts, workspace, workspace_bytes, err, st);
}

size_t sm_ep_expert_workspace_bytes(int R, int H, int I, int El, int K) {
  const long long TK = static_cast<long long>(R) * K;
  const size_t mb = max_padded_blocks(TK, El);
  return a256(TK * 4) * 5 + a256(static_cast<size_t>(El) * (ceil_div(R, kTileTokens) + 1) * 4) +
         a256(static_cast<size_t>(El + 1) * 4) * 2 + a256((mb + 2) * 4) + a256(4) +
         a256(mb * kBlockM * static_cast<size_t>(H)) + a256(mb * ceil_div(H, 512) * kSfAtomBytes) +
         a256(mb * kBlockM * static_cast<size_t>(I)) + a256(mb * ceil_div(I, 512) * kSfAtomBytes) +
         a256(mb * kBlockM * sizeof(int32_t)) + 4096;
}

// Where the home-down variant's up projection sends its rows: rank h's intermediate rows / scale
// atoms (peer pointers) and the row capacity every home buffer has.
struct HomeReturn {
  uint8_t* q[kMaxRanks];
  uint8_t* sf[kMaxRanks];
  long long rows;
  int W;
};

// The count matrix (device memory) an expert stage resolves its segment table from on the device:
// counts[s * stride + d] records of source s for destination d; this rank is d = me; a source's
// send region holds send_cap records.
struct DeviceCounts {
  const int32_t* counts;
  int stride;
  int me;
  int send_cap;
};

// The expert stage: local routing metadata over the received records, the pack into the padded
// layout, the up projection, then either the down projection with the per-record combine into
// out_rows, or (home != nullptr) nothing more -- the up projection has returned every row to its
// token's home rank.  With dc, R is the capacity: every grid is sized for R records and the table
// resolved on the device says how many arrived (no host round trip).
static int ep_expert_forward(const RecordSource& src, int R, int H, int I, int El, int K, const uint8_t* w1q,
                             const uint8_t* w1_sf, const uint8_t* w2q, const uint8_t* w2_sf, int concat_layout,
                             void* out_rows, int32_t* expert_frequency, void* workspace, size_t workspace_bytes,
                             int32_t* err, void* stream, const HomeReturn* home = nullptr,
                             const DeviceCounts* dc = nullptr) {
  if (R < 0 || H <= 0 || H % 256 || I <= 0 || I % 128 || El < 1 || K < 1 || K > 32)
    return set_last_error(SM_EINVAL, "ep expert: bad shape R=%d H=%d I=%d El=%d K=%d", R, H, I, El, K);
  if (!expert_frequency || !err) return set_last_error(SM_EINVAL, "ep expert: null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (R == 0) return ep_status(cudaMemsetAsync(expert_frequency, 0, sizeof(int32_t) * El, st), "ep expert");
  const long long TK = static_cast<long long>(R) * K;
  const int n_tiles = ceil_div(R, kTileTokens);
  const int mb = max_padded_blocks(TK, El);
  uint8_t* p = static_cast<uint8_t*>(workspace);
  size_t used = 0;
  auto take = [&](size_t bytes) {
    uint8_t* q = p + used;
    used += a256(bytes);
    return q;
  };
  int32_t* idx = reinterpret_cast<int32_t*>(take(TK * 4));
  float* scores = reinterpret_cast<float*>(take(TK * 4));
  int32_t* s_scatter = reinterpret_cast<int32_t*>(take(TK * 4));
  int32_t* s_rev = reinterpret_cast<int32_t*>(take(TK * 4));
  int32_t* x_gather = reinterpret_cast<int32_t*>(take(TK * 4));
  int32_t* tile_counts = reinterpret_cast<int32_t*>(take(static_cast<size_t>(El) * (n_tiles + 1) * 4));
  int32_t* off = reinterpret_cast<int32_t*>(take(static_cast<size_t>(El + 1) * 4));
  int32_t* off_pad = reinterpret_cast<int32_t*>(take(static_cast<size_t>(El + 1) * 4));
  int32_t* blk = reinterpret_cast<int32_t*>(take((static_cast<size_t>(mb) + 2) * 4));
  int32_t* nblk = reinterpret_cast<int32_t*>(take(4));
  uint8_t* xq = take(static_cast<size_t>(mb) * kBlockM * H);
  uint8_t* xsf = take(static_cast<size_t>(mb) * ceil_div(H, 512) * kSfAtomBytes);
  uint8_t* aq = take(static_cast<size_t>(mb) * kBlockM * I);
  uint8_t* asf = take(static_cast<size_t>(mb) * ceil_div(I, 512) * kSfAtomBytes);
  int32_t* ret_dst = reinterpret_cast<int32_t*>(take(static_cast<size_t>(mb) * kBlockM * sizeof(int32_t)));
  RecordIndex* table = dc ? reinterpret_cast<RecordIndex*>(take(sizeof(RecordIndex))) : nullptr;
  if (used > workspace_bytes) return set_last_error(SM_EINVAL, "ep expert: workspace too small");
  RecordSource rs = src;
  if (dc) {
    ep_resolve_counts_kernel<<<1, 32, 0, st>>>(dc->counts, dc->stride, src.W, dc->me, dc->send_cap, R, table, err);
    rs.dev = table;
  }
  ep_recv_unpack_kernel<<<static_cast<int>((TK + 255) / 256), 256, 0, st>>>(rs, R, H, K, idx, scores);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess && home)
    e = cudaMemsetAsync(ret_dst, 0xFF, static_cast<size_t>(mb) * kBlockM * sizeof(int32_t), st);
  if (e == cudaSuccess)
    e = launch_route_hist_holes(idx, static_cast<int>(TK), kTileTokens * K, El, n_tiles, tile_counts, err, st);
  if (e == cudaSuccess)
    e = launch_route_scan(tile_counts, n_tiles, El, static_cast<int>(TK), expert_frequency, off, off_pad, blk, nblk,
                          st);
  if (e == cudaSuccess)
    e = launch_route_scatter(idx, nullptr, static_cast<int>(TK), K, kTileTokens * K, El, n_tiles, tile_counts, off,
                             s_scatter, s_rev, x_gather, st);
  if (e == cudaSuccess) {
    ep_pack_fp8_kernel<<<(R + 7) / 8, 256, 0, st>>>(rs, R, H, K, El, idx, s_rev, off, off_pad, xq, xsf,
                                                    home ? ret_dst : nullptr);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess && !home) e = cudaMemsetAsync(out_rows, 0, static_cast<size_t>(R) * H * 2, st);
  if (e == cudaSuccess) {
    GemmArgs g{};
    g.a = xq;
    g.a_sf = xsf;
    g.a_rows = static_cast<long long>(mb) * kBlockM;
    g.b = w1q;
    g.b_sf = w1_sf;
    g.E = El;
    g.N = 2 * I;
    g.Kd = H;
    g.blk_expert = blk;
    g.n_blocks = nblk;
    g.off_pad = off_pad;
    g.freq = expert_frequency;
    g.out_q = aq;
    g.out_sf = asf;
    g.concat = concat_layout;
    g.err = err;
    g.num_sms = gemm_grid_sms();
    g.tokens = R;
    if (home) {
      g.out_q = nullptr;
      g.out_sf = nullptr;
      g.ret_dst = ret_dst;
      for (int h = 0; h < home->W; ++h) {
        g.home_q[h] = home->q[h];
        g.home_sf[h] = home->sf[h];
      }
      g.home_rows = home->rows;
      g.n_homes = home->W;
    }
    e = launch_moe_up(g, st);
    if (e == cudaSuccess && !home) {
      GemmArgs d = g;
      d.a = aq;
      d.a_sf = asf;
      d.b = w2q;
      d.b_sf = w2_sf;
      d.N = H;
      d.Kd = I;
      d.off = off;
      d.s_scatter = s_scatter;
      d.x_gather = x_gather;
      d.scores = scores;
      d.out_bf16 = out_rows;
      d.out_q = nullptr;
      d.out_sf = nullptr;
      e = launch_moe_down(d, st);
    }
  }
  return ep_status(e, "ep expert forward");
}

int sm_ep_expert_forward(const uint8_t* records, int R, int H, int I, int El, int K, const uint8_t* w1q,
                         const uint8_t* w1_sf, const uint8_t* w2q, const uint8_t* w2_sf, int concat_layout,
                         void* out_rows, int32_t* expert_frequency, void* workspace, size_t workspace_bytes,
                         int32_t* err, void* stream) {
  RecordSource src{};
  src.base[0] = records;
  src.seg_off[0] = 0;
  src.start[0] = 0;
  src.start[1] = R;
  src.W = 1;
  src.rb = sm_ep_record_bytes(H, K);
  return ep_expert_forward(src, R, H, I, El, K, w1q, w1_sf, w2q, w2_sf, concat_layout, out_rows, expert_frequency,
                           workspace, workspace_bytes, err, stream);
}

int sm_ep_expert_forward_p2p(const void* const* peer_send_bases, const int32_t* seg_off, const int32_t* recv_counts,
                             int W, int H, int I, int El, int K, const uint8_t* w1q, const uint8_t* w1_sf,
                             const uint8_t* w2q, const uint8_t* w2_sf, int concat_layout, void* out_rows,
                             int32_t* expert_frequency, void* workspace, size_t workspace_bytes, int32_t* err,
                             void* stream) {
  if (W < 1 || W > kMaxRanks || !peer_send_bases || !seg_off || !recv_counts)
    return set_last_error(SM_EINVAL, "ep expert p2p: W must be in [1, %d] with W peer bases", kMaxRanks);
  RecordSource src{};
  int R = 0;
  for (int s = 0; s < W; ++s) {
    if (recv_counts[s] < 0 || seg_off[s] < 0) return set_last_error(SM_EINVAL, "ep expert p2p: negative count");
    src.base[s] = static_cast<const uint8_t*>(peer_send_bases[s]);
    src.seg_off[s] = seg_off[s];
    src.start[s] = R;
    R += recv_counts[s];
  }
  src.start[W] = R;
  src.W = W;
  src.rb = sm_ep_record_bytes(H, K);
  return ep_expert_forward(src, R, H, I, El, K, w1q, w1_sf, w2q, w2_sf, concat_layout, out_rows, expert_frequency,
                           workspace, workspace_bytes, err, stream);
}

int sm_ep_expert_up_p2p(const void* const* peer_send_bases, const int32_t* seg_off, const int32_t* recv_counts,
                        int W, int H, int I, int El, int K, const uint8_t* w1q, const uint8_t* w1_sf,
                        int concat_layout, void* const* home_q_bases, void* const* home_sf_bases,
                        long long home_rows, int32_t* expert_frequency, void* workspace, size_t workspace_bytes,
                        int32_t* err, void* stream) {
  if (W < 1 || W > kMaxRanks || !peer_send_bases || !seg_off || !recv_counts || !home_q_bases || !home_sf_bases)
    return set_last_error(SM_EINVAL, "ep expert up p2p: W must be in [1, %d] with W peer and home bases", kMaxRanks);
  if (home_rows < 0 || home_rows > (1ll << kHomeShift))
    return set_last_error(SM_EINVAL, "ep expert up p2p: home_rows %lld outside [0, 2^%d]", home_rows, kHomeShift);
  RecordSource src{};
  HomeReturn home{};
  int R = 0;
  for (int s = 0; s < W; ++s) {
    if (recv_counts[s] < 0 || seg_off[s] < 0) return set_last_error(SM_EINVAL, "ep expert up p2p: negative count");
    if (!home_q_bases[s] || !home_sf_bases[s] || reinterpret_cast<uintptr_t>(home_q_bases[s]) % 16)
      return set_last_error(SM_EINVAL, "ep expert up p2p: home buffers must be non-null and 16-byte aligned");
    src.base[s] = static_cast<const uint8_t*>(peer_send_bases[s]);
    src.seg_off[s] = seg_off[s];
    src.start[s] = R;
    R += recv_counts[s];
    home.q[s] = static_cast<uint8_t*>(home_q_bases[s]);
    home.sf[s] = static_cast<uint8_t*>(home_sf_bases[s]);
  }
  src.start[W] = R;
  src.W = W;
  src.rb = sm_ep_record_bytes(H, K);
  home.rows = home_rows;
  home.W = W;
  return ep_expert_forward(src, R, H, I, El, K, w1q, w1_sf, nullptr, nullptr, concat_layout, nullptr,
                           expert_frequency, workspace, workspace_bytes, err, stream, &home);
}

int sm_ep_expert_up_home(const void* const* peer_send_bases, const int32_t* counts, int count_stride, int me, int W,
                         int send_cap, int recv_cap, int H, int I, int El, int K, const uint8_t* w1q,
                         const uint8_t* w1_sf, int concat_layout, void* const* home_q_bases,
                         void* const* home_sf_bases, long long home_rows, int32_t* expert_frequency,
                         void* workspace, size_t workspace_bytes, int32_t* err, void* stream) {
  if (W < 1 || W > kMaxRanks || me < 0 || me >= W || !peer_send_bases || !counts || !home_q_bases ||
      !home_sf_bases || !err)
    return set_last_error(SM_EINVAL, "ep expert up home: W must be in [1, %d], 0 <= me < W, pointers non-null",
                          kMaxRanks);
  if (count_stride < W || send_cap < 0 || recv_cap < 1 || static_cast<long long>(recv_cap) * K > (1ll << 30))
    return set_last_error(SM_EINVAL, "ep expert up home: bad capacities (stride %d, send %d, recv %d)", count_stride,
                          send_cap, recv_cap);
  if (home_rows < 0 || home_rows > (1ll << kHomeShift))
    return set_last_error(SM_EINVAL, "ep expert up home: home_rows %lld outside [0, 2^%d]", home_rows, kHomeShift);
  RecordSource src{};
  HomeReturn home{};
  for (int s = 0; s < W; ++s) {
    if (!home_q_bases[s] || !home_sf_bases[s] || reinterpret_cast<uintptr_t>(home_q_bases[s]) % 16)
      return set_last_error(SM_EINVAL, "ep expert up home: home buffers must be non-null and 16-byte aligned");
    src.base[s] = static_cast<const uint8_t*>(peer_send_bases[s]);
    home.q[s] = static_cast<uint8_t*>(home_q_bases[s]);
    home.sf[s] = static_cast<uint8_t*>(home_sf_bases[s]);
  }
  src.W = W;
  src.rb = sm_ep_record_bytes(H, K);
  home.rows = home_rows;
  home.W = W;
  const DeviceCounts dc{counts, count_stride, me, send_cap};
  return ep_expert_forward(src, recv_cap, H, I, El, K, w1q, w1_sf, nullptr, nullptr, concat_layout, nullptr,
                           expert_frequency, workspace, workspace_bytes, err, stream, &home, &dc);
}

static int ep_combine(const RowSource& rs, const int32_t* ret_row, int T, int K, int H, void* out, void* stream) {
  if (T < 0 || K < 1 || K > 32 || H <= 0 || H % 8) return set_last_error(SM_EINVAL, "ep combine: bad shape");
  if (T == 0) return SM_OK;
  ep_combine_kernel<<<T, 256, 0, static_cast<cudaStream_t>(stream)>>>(rs, ret_row, T, K, H,
                                                                      static_cast<__nv_bfloat16*>(out));
  return ep_status(cudaGetLastError(), "ep combine");
}

int sm_ep_combine(const void* ret_rows, const int32_t* ret_row, int T, int K, int H, void* out, void* stream) {
  RowSource rs{};
  rs.base[0] = static_cast<const __nv_bfloat16*>(ret_rows);
  rs.send_off[0] = 0;
  rs.send_off[1] = 1 << 30;
  rs.recv_start[0] = 0;
  rs.W = 1;
  return ep_combine(rs, ret_row, T, K, H, out, stream);
}

int sm_ep_combine_p2p(const void* const* peer_out_bases, const int32_t* send_counts, const int32_t* recv_start,
                      int W, const int32_t* ret_row, int T, int K, int H, void* out, void* stream) {
  if (W < 1 || W > kMaxRanks || !peer_out_bases || !send_counts || !recv_start)
    return set_last_error(SM_EINVAL, "ep combine p2p: W must be in [1, %d] with W peer bases", kMaxRanks);
  RowSource rs{};
  int acc = 0;
  for (int d = 0; d < W; ++d) {
    rs.base[d] = static_cast<const __nv_bfloat16*>(peer_out_bases[d]);
    rs.send_off[d] = acc;
    rs.recv_start[d] = recv_start[d];
    acc += send_counts[d];
  }
  rs.send_off[W] = acc;
  rs.W = W;
  return ep_combine(rs, ret_row, T, K, H, out, stream);
}

// ---- CUDA IPC buffers shared between the ranks of one node (peer loads over NVLink) ----------
int sm_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return set_last_error(SM_EINVAL, "ipc alloc: bad arguments");
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return ep_status(e, "ipc alloc");
  e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return ep_status(e, "ipc handle");
  }
  return SM_OK;
}

int sm_ipc_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return set_last_error(SM_EINVAL, "ipc open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return ep_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "ipc open");
}

int sm_ipc_close(void* ptr) { return ep_status(cudaIpcCloseMemHandle(ptr), "ipc close"); }

int sm_ipc_free(void* ptr) { return ep_status(cudaFree(ptr), "ipc free"); }

int sm_copy_d2d_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return SM_OK;
  if (!dst || !src) return set_last_error(SM_EINVAL, "copy: null pointer");
  return ep_status(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)),
                   "copy d2d");
}

}  // extern "C"
