// Backward of the FP8 MoE layer: the non-GEMM kernels.  The GEMMs are moe_gemm_kernel's
// activation-gradient and weight-gradient kinds (csrc/gemm.cu) and its down kind with unit weights.
//
// weight_t_kernel      -- the forward's prepared e4m3 weight [E, N, K] transposed to [E, K, N] with
//                         its 128x128 block scales moved along (the same blocks, read the other way),
//                         so that a backward GEMM takes W^T as its K-major B operand.
// tq_pack_kernel       -- the weight gradients' operands: rows of the padded expert layout (gathered
//                         token rows, or rows of a padded array) transposed to [C, rows] and
//                         quantised with one UE8M0 scale per 128 consecutive rows (the K groups of a
//                         weight-gradient GEMM whose K is the expert's rows); padding rows are zero.
// router_bwd_kernel    -- gradient of the router logits from the scores' gradient
//                         (functional/backward.py:308-430: softmax over the top-k, or top-k of the
//                         softmax with optional renormalisation).
#include "common.cuh"
#include "sonic_internal.h"

namespace smb {

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }

// One CTA of 256 threads per 128x128 block of the prepared weight: blockIdx = (k block, n block,
// expert).  The e4m3 bytes are transposed through a shared-memory tile (tt_chunk layout; loaded 8
// lanes per 128-byte row, stored 8 lanes per output row), and the block's scale byte moves from
// atom (n block, k block) of wq to atom (k block, n block) of wq_t -- the same 128x128 block, so the
// values are those of the forward's weight, read transposed.
__global__ void __launch_bounds__(256)
    weight_t_kernel(const uint8_t* __restrict__ wq, const uint8_t* __restrict__ wsf, int N, int Kd,
                    uint8_t* __restrict__ wqt, uint8_t* __restrict__ wsft) {
  __shared__ __align__(16) uint8_t tile[kBlockM * kTtStride];
  const int kb = blockIdx.x, nb = blockIdx.y, e = blockIdx.z;
  const int tid = threadIdx.x;
  const uint8_t* src = wq + (static_cast<size_t>(e) * N + static_cast<size_t>(nb) * kBlockM) * Kd + kb * kBlockK;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int k = i * 256 + tid;
    const int r = k >> 3, ch = k & 7;
    *reinterpret_cast<uint4*>(tile + tt_chunk(r, ch)) =
        *reinterpret_cast<const uint4*>(src + static_cast<size_t>(r) * Kd + 16 * ch);
  }
  __syncthreads();
  store_tile_transposed_128(
      tile, wqt + (static_cast<size_t>(e) * Kd + static_cast<size_t>(kb) * kBlockK) * N + static_cast<size_t>(nb) * kBlockM,
      static_cast<size_t>(N), tid);
  if (tid < 128) {
    // the block's scale: byte (kb % 4) of any row slot of atom (e, nb, kb / 4) of wq
    const int KG = (Kd / kBlockK + 3) / 4;
    const uint8_t sc = wsf[((static_cast<size_t>(e) * (N / kBlockM) + nb) * KG + kb / 4) * kSfAtomBytes + (kb % 4)];
    const int KGn = (N / kBlockK + 3) / 4;
    const size_t atom = ((static_cast<size_t>(e) * (Kd / kBlockM) + kb) * KGn + nb / 4) * kSfAtomBytes;
    wsft[atom + 16 * (tid >> 2) + 4 * (tid & 3) + (nb % 4)] = sc;
  }
}

// One CTA of 256 threads per (block mb of the padded layout, 128-column block cb of the source).
// Padded row p of block mb (expert e = blk_expert[mb], rel = p - off_pad[e]) is valid when
// rel < freq[e]; its source row is x_gather[off[e] + rel] (token rows, gathered) or p itself
// (src_padded).  out [C, rows_pad] e4m3: out[c][p] = q(src[row(p)][c]); atoms [C/128][KG][512] with
// KG = ceil(rows_pad / 512), one scale per (c, 128-row block).
//
// Access pattern (the kernel is bound by L1 / shared-memory wavefronts, not DRAM, unless every warp
// instruction touches few cache lines): the tile is loaded 16 lanes per source row (two 256-byte row
// slices per warp instruction); warp w then owns the 16 columns of column pairs 8w .. 8w + 7 over
// all 128 rows -- lane l reads pair 8w + l / 4 in the 32 rows of quarter l % 4 -- so a column's
// maximum is a 4-lane shuffle and each output store instruction fills 8 cache lines with 4 lanes
// each.  The tile's 32-bit words are XOR-swizzled by quarter (word ^ 8 q) so that the four quarters
// of one column pair fall into different banks.
constexpr int kTqStride = kBlockK / 2 + 4;  // tile row: 64 words of bf16 pairs + 4 words of padding

__device__ __forceinline__ int tq_word(int row, int w) { return row * kTqStride + (w ^ ((row >> 5) << 3)); }

__global__ void __launch_bounds__(256)
    tq_pack_kernel(const __nv_bfloat16* __restrict__ src, int C, int src_padded, const int32_t* __restrict__ blk_expert,
                   const int32_t* __restrict__ off_pad, const int32_t* __restrict__ off,
                   const int32_t* __restrict__ freq, const int32_t* __restrict__ x_gather,
                   const int32_t* __restrict__ n_blocks, long long rows_pad, uint8_t* __restrict__ outq,
                   uint8_t* __restrict__ outsf, uint8_t* __restrict__ rowq, uint8_t* __restrict__ rowsf,
                   int row_concat_i) {
  __shared__ __align__(16) uint32_t tile[kBlockM * kTqStride];
  __shared__ int s_row[kBlockM];  // source row of each padded row, -1 = padding
  const int mb = blockIdx.x, cb = blockIdx.y;
  if (mb >= *n_blocks) return;  // blocks past the layout are never read
  const int tid = threadIdx.x;
  if (tid < kBlockM) {
    const int e = blk_expert[mb];
    const int p = mb * kBlockM + tid;
    const int rel = p - off_pad[e];
    s_row[tid] = rel < freq[e] ? (src_padded ? p : x_gather[off[e] + rel]) : -1;
  }
  __syncthreads();
  // load: chunk k = 16-byte piece k % 16 of row k / 16 (8 chunks per thread)
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int k = i * 256 + tid;
    const int r = k >> 4, c16 = k & 15;
    const int sr = s_row[r];
    const uint4 v = sr >= 0 ? *reinterpret_cast<const uint4*>(src + static_cast<size_t>(sr) * C + cb * kBlockK + 8 * c16)
                            : make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(&tile[tq_word(r, 4 * c16)]) = v;
  }
  __syncthreads();
  const int warp = tid >> 5, lane = tid & 31;
  if (rowq != nullptr) {
    // The same tile quantised along its rows (padded sources: the dX GEMM's dH operand): each row's
    // 128 values of this column block are one 1x128 group.  16 lanes per row, 8 values each (a warp
    // reads two rows per pass and stores two 128-byte lines); column block cb lands at column block
    // cbd of the row-quantised operand -- itself, or for a concatenated [gate | up] source the
    // re-blocked order of the prepared w1 (gate block j -> 2 j, up block j -> 2 j + 1).
    const int hl = lane & 15;
    const int nI = row_concat_i / kBlockK;
    const int cbd = row_concat_i > 0 ? (cb < nI ? 2 * cb : 2 * (cb - nI) + 1) : cb;
    const int KG2 = (C / kBlockK + 3) / 4;
#pragma unroll 1
    for (int pass = 0; pass < 8; ++pass) {
      const int row = 16 * pass + 2 * warp + (lane >> 4);
      const uint4 w4 = *reinterpret_cast<const uint4*>(&tile[tq_word(row, 4 * hl)]);
      const uint32_t wd[4] = {w4.x, w4.y, w4.z, w4.w};
      float am = 0.0f;
#pragma unroll
      for (int k = 0; k < 4; ++k)
        am = fmaxf(am, fmaxf(fabsf(__uint_as_float(wd[k] << 16)), fabsf(__uint_as_float(wd[k] & 0xFFFF0000u))));
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
      const int er = scale_exp_of_amax(am);
      const float ir = exp2_neg(er);
      uint32_t b[2];
#pragma unroll
      for (int k = 0; k < 2; ++k)
        b[k] = static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(__uint_as_float(wd[2 * k] << 16), ir),
                                                __fmul_rn(__uint_as_float(wd[2 * k] & 0xFFFF0000u), ir))) |
               (static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(__uint_as_float(wd[2 * k + 1] << 16), ir),
                                                 __fmul_rn(__uint_as_float(wd[2 * k + 1] & 0xFFFF0000u), ir)))
                << 16);
      const long long p = static_cast<long long>(mb) * kBlockM + row;
      *reinterpret_cast<uint2*>(rowq + p * C + static_cast<long long>(cbd) * kBlockK + 8 * hl) = make_uint2(b[0], b[1]);
      if (hl == 0)
        rowsf[(static_cast<long long>(mb) * KG2 + cbd / 4) * kSfAtomBytes + 16 * (row % 32) + 4 * (row / 32) +
              (cbd % 4)] = static_cast<uint8_t>(er + 127);
    }
  }
  const int q = lane & 3;                   // row quarter: rows 32 q .. 32 q + 31
  const int cp = 8 * warp + (lane >> 2);    // column pair: columns 2 cp, 2 cp + 1
  float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const uint32_t w = tile[tq_word(32 * q + j, cp)];
    a0 = fmaxf(a0, fabsf(__uint_as_float(w << 16)));
    a1 = fmaxf(a1, fabsf(__uint_as_float(w & 0xFFFF0000u)));
  }
#pragma unroll
  for (int o = 1; o <= 2; o <<= 1) {
    a0 = fmaxf(a0, __shfl_xor_sync(0xffffffffu, a0, o));
    a1 = fmaxf(a1, __shfl_xor_sync(0xffffffffu, a1, o));
  }
  const int e0 = scale_exp_of_amax(a0), e1 = scale_exp_of_amax(a1);
  const float i0 = exp2_neg(e0), i1 = exp2_neg(e1);
  const long long col = static_cast<long long>(cb) * kBlockK + 2 * cp;
  uint8_t* d0 = outq + col * rows_pad + static_cast<long long>(mb) * kBlockM + 32 * q;
  uint8_t* d1 = d0 + rows_pad;
#pragma unroll 1
  for (int i = 0; i < 2; ++i) {
    uint32_t w0[4], w1[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = 16 * i + 4 * k;
      float v0[4], v1[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const uint32_t w = tile[tq_word(32 * q + j + t, cp)];
        v0[t] = __uint_as_float(w << 16);
        v1[t] = __uint_as_float(w & 0xFFFF0000u);
      }
      w0[k] = static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(v0[0], i0), __fmul_rn(v0[1], i0))) |
              (static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(v0[2], i0), __fmul_rn(v0[3], i0))) << 16);
      w1[k] = static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(v1[0], i1), __fmul_rn(v1[1], i1))) |
              (static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(v1[2], i1), __fmul_rn(v1[3], i1))) << 16);
    }
    reinterpret_cast<uint4*>(d0)[i] = make_uint4(w0[0], w0[1], w0[2], w0[3]);
    reinterpret_cast<uint4*>(d1)[i] = make_uint4(w1[0], w1[1], w1[2], w1[3]);
  }
  if (q == 0) {
    const long long KG = (rows_pad / kBlockK + 3) / 4;
    const long long atom = (static_cast<long long>(cb) * KG + mb / 4) * kSfAtomBytes;
    const int c0 = 2 * cp, c1 = 2 * cp + 1;
    outsf[atom + 16 * (c0 % 32) + 4 * (c0 / 32) + (mb % 4)] = static_cast<uint8_t>(e0 + 127);
    outsf[atom + 16 * (c1 % 32) + 4 * (c1 / 32) + (mb % 4)] = static_cast<uint8_t>(e1 + 127);
  }
}

// One warp per token row.  sot: dl[idx_k] = s_k (g_k - sum_j g_j s_j), zero elsewhere.  tos: p =
// softmax(logits) over all E; dp_sel = g (or (g - sum_j g_j s_j) / sum_j p_sel_j when renormalised);
// dl = p (dp - sum_k dp_sel_k p_sel_k) with dp zero outside the selection.
__global__ void router_bwd_kernel(const __nv_bfloat16* __restrict__ logits, const float* __restrict__ scores,
                                  const int32_t* __restrict__ idx, const float* __restrict__ ds, int T, int E, int K,
                                  int softmax_over_topk, int renorm, float* __restrict__ dlogits) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const size_t row = static_cast<size_t>(warp);
  float* out = dlogits + row * E;
  const float g = lane < K ? ds[row * K + lane] : 0.0f;
  const float s = lane < K ? scores[row * K + lane] : 0.0f;
  const int ix = lane < K ? idx[row * K + lane] : 0;
  if (softmax_over_topk) {
    float dot = g * s;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    for (int e = lane; e < E; e += 32) out[e] = 0.0f;
    __syncwarp();
    if (lane < K) out[ix] = s * (g - dot);
    return;
  }
  const __nv_bfloat16* lrow = logits + row * E;
  float mx = -__int_as_float(0x7f800000);
  for (int e = lane; e < E; e += 32) mx = fmaxf(mx, __bfloat162float(lrow[e]));
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.0f;
  for (int e = lane; e < E; e += 32) sum += __expf(__bfloat162float(lrow[e]) - mx);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float p_sel = lane < K ? __expf(__bfloat162float(lrow[ix]) - mx) / sum : 0.0f;
  float dp_sel = g;
  if (renorm) {
    float dot_s = g * s, S = p_sel;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      dot_s += __shfl_xor_sync(0xffffffffu, dot_s, o);
      S += __shfl_xor_sync(0xffffffffu, S, o);
    }
    dp_sel = lane < K ? (g - dot_s) / S : 0.0f;
  }
  float dot = dp_sel * p_sel;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
  for (int e = lane; e < E; e += 32) out[e] = -(__expf(__bfloat162float(lrow[e]) - mx) / sum) * dot;
  __syncwarp();
  if (lane < K) out[ix] = p_sel * (dp_sel - dot);
}

cudaError_t launch_weight_t(const uint8_t* wq, const uint8_t* wsf, int E, int N, int Kd, uint8_t* wqt, uint8_t* wsft,
                            cudaStream_t st) {
  if (E == 0) return cudaSuccess;
  dim3 grid(Kd / kBlockK, N / kBlockM, E);
  weight_t_kernel<<<grid, 256, 0, st>>>(wq, wsf, N, Kd, wqt, wsft);
  return cudaGetLastError();
}

cudaError_t launch_tq_pack(const void* src, int C, int src_padded, const int32_t* blk_expert, const int32_t* off_pad,
                           const int32_t* off, const int32_t* freq, const int32_t* x_gather, const int32_t* n_blocks,
                           int max_blocks, uint8_t* outq, uint8_t* outsf, cudaStream_t st, uint8_t* rowq,
                           uint8_t* rowsf, int row_concat_i) {
  if (max_blocks == 0) return cudaSuccess;
  dim3 grid(max_blocks, C / kBlockK);
  tq_pack_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(src), C, src_padded, blk_expert, off_pad, off,
                                       freq, x_gather, n_blocks, static_cast<long long>(max_blocks) * kBlockM, outq,
                                       outsf, rowq, rowsf, row_concat_i);
  return cudaGetLastError();
}

cudaError_t launch_router_bwd(const void* logits, const float* scores, const int32_t* idx, const float* ds, int T,
                              int E, int K, int sot, int renorm, float* dlogits, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  const int warps = 8;
  router_bwd_kernel<<<(T + warps - 1) / warps, warps * 32, 0, st>>>(static_cast<const __nv_bfloat16*>(logits), scores,
                                                                     idx, ds, T, E, K, sot, renorm, dlogits);
  return cudaGetLastError();
}

}  // namespace smb
