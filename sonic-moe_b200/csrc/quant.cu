// Activation quantiser + scatter-pack, and weight quantiser (e4m3, UE8M0 power-of-two scales).
//
// Spec (identical to oracle/quant.py): per group amax = max|x|; e = ceil(log2(amax / 448)) taken
// exactly from the float32 bits and clamped to [-127, 127]; q = e4m3_rn_satfinite(x * 2^-e);
// scale byte = e + 127.  Groups are 1x128 along K for activations and 128x128 for weights.
//
// Scale-factor atoms: 512 bytes per (128 rows, 4 consecutive 128-wide K blocks); byte
// 16*(r % 32) + 4*((r % 128) / 32) + (kb % 4) belongs to row r, K block kb -- the order in which
// tcgen05.cp 32x128b.warpx4 lays scale factors out in tensor memory for the block-scaled MMA.
#include "common.cuh"
#include "sonic_internal.h"

namespace smb {

constexpr int kQuantWarps = 8;
constexpr int kQuantBatch = 4;  // 256-element chunks loaded before any is processed

__device__ __forceinline__ void bf16x8_to_f32(const uint4& raw, float* v) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// One warp per token.  Lane l covers elements [h0 + 8l, h0 + 8l + 8) of each 256-wide chunk, so
// lanes 0-15 and 16-31 each hold one 128-wide group.  The token's quantised row and scale bytes
// are written to each destination row of the padded expert-major layout that one of its routed
// entries owns (row = s_rev[f] - off[e] + off_pad[e] for entry f, e = experts[f]).  The token's
// entries are f in [t*K, t*K + K) for token-choice routing, or [tok_off[t], tok_off[t+1]) for
// general routing (tok_off != nullptr); with experts == nullptr the destination is row t itself
// (plain token-order quantisation).  Destinations are handled 32 at a time (one per lane).
__global__ void __launch_bounds__(kQuantWarps * 32)
    quant_pack_kernel(const __nv_bfloat16* __restrict__ x, int T, int H, const int32_t* __restrict__ experts, int K,
                      const int32_t* __restrict__ tok_off, const int32_t* __restrict__ s_rev,
                      const int32_t* __restrict__ off, const int32_t* __restrict__ off_pad, uint8_t* __restrict__ xq,
                      uint8_t* __restrict__ xsf, uint4* __restrict__ zero_out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * kQuantWarps + warp;
  if (t >= T) return;
  if (zero_out) {
    // the layer's output row t, zeroed for the down projection's reductions (instead of a memset pass)
    uint4* row = zero_out + static_cast<size_t>(t) * (H / 8);
    for (int i = lane; i < H / 8; i += 32) row[i] = make_uint4(0, 0, 0, 0);
  }
  int f0 = t, ncopy = 1;
  if (experts) {
    f0 = tok_off ? tok_off[t] : t * K;
    ncopy = tok_off ? tok_off[t + 1] - f0 : K;
  }
  const int KG = (H / kBlockK + 3) / 4;
  const __nv_bfloat16* src = x + static_cast<size_t>(t) * H;
  for (int c0 = 0; c0 < ncopy; c0 += 32) {
    const int nc = min(32, ncopy - c0);
    int my_dst = 0;
    if (!experts) {
      my_dst = t;
    } else if (lane < nc) {
      const int f = f0 + c0 + lane;
      const int e = experts[f];
      my_dst = s_rev[f] - off[e] + off_pad[e];
    }
    uint32_t sfword = 0;
    for (int hb = 0; hb < H; hb += 256 * kQuantBatch) {
      uint4 raw[kQuantBatch];
#pragma unroll
      for (int c = 0; c < kQuantBatch; ++c) {
        const int h = hb + 256 * c + 8 * lane;
        raw[c] = (h < H) ? *reinterpret_cast<const uint4*>(src + h) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int c = 0; c < kQuantBatch; ++c) {
        const int h0 = hb + 256 * c;
        if (h0 >= H) break;
        const int h = h0 + 8 * lane;
        float v[8];
        bf16x8_to_f32(raw[c], v);
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
        const uint2 packed = make_uint2(lo, hi);
        for (int k = 0; k < nc; ++k) {
          const int p = __shfl_sync(0xffffffffu, my_dst, k);
          if (h < H) *reinterpret_cast<uint2*>(xq + static_cast<size_t>(p) * H + h) = packed;
        }
        const int gA = h0 / kBlockK;
        const int eA = __shfl_sync(0xffffffffu, e8, 0);
        const int eB = __shfl_sync(0xffffffffu, e8, 16);
        sfword |= static_cast<uint32_t>(eA + 127) << (8 * (gA % 4));
        if (h0 + 128 < H) sfword |= static_cast<uint32_t>(eB + 127) << (8 * ((gA + 1) % 4));
        if ((gA % 4) == 2 || h0 + 256 >= H) {
          const int kg = gA / 4;
          if (lane < nc) {
            const int p = my_dst;
            const size_t o = (static_cast<size_t>(p / kBlockM) * KG + kg) * kSfAtomBytes + 16 * (p % 32) +
                             4 * ((p % kBlockM) / 32);
            *reinterpret_cast<uint32_t*>(xsf + o) = sfword;
          }
          sfword = 0;
        }
      }
    }
  }
}

// One CTA per 128x128 block: blockIdx = (k block, destination n block, expert).  With concat_glu
// the destination row blocks interleave the gate and up halves at 128-row granularity:
// destination block 2j <- gate block j, 2j+1 <- up block j (rows I + 128j ...).  With wqt the same
// e4m3 block is also written transposed ([E, Kd, N], the backward GEMMs' operand) with its scale in
// atom (k block, n block) of wsft, through a shared-memory tile, so the transpose costs no second
// pass over the weight.
__global__ void __launch_bounds__(256)
    weight_prep_kernel(const __nv_bfloat16* __restrict__ w, int E, int N, int Kd, int concat_glu,
                       uint8_t* __restrict__ wq, uint8_t* __restrict__ wsf, uint8_t* __restrict__ wqt,
                       uint8_t* __restrict__ wsft) {
  __shared__ __align__(16) uint8_t tile[kBlockM * kTtStride];  // the transposed copy's staging tile
  __shared__ float s_red[8];
  const int kb = blockIdx.x, nb = blockIdx.y, e = blockIdx.z;
  const int nbs = concat_glu ? ((nb % 2 == 0) ? nb / 2 : (N / 2) / kBlockM + nb / 2) : nb;
  const int tid = threadIdx.x;
  // piece i of this thread: 8 values (16 bytes of bf16) at row (256 i + tid) / 16, columns
  // 8 ((256 i + tid) % 16) -- 16 lanes per 256-byte row slice, so a warp's load touches 4 lines
  const __nv_bfloat16* src = w + (static_cast<size_t>(e) * N + static_cast<size_t>(nbs) * kBlockM) * Kd + kb * kBlockK;
  uint4 raw[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int k = i * 256 + tid;
    raw[i] = *reinterpret_cast<const uint4*>(src + static_cast<size_t>(k >> 4) * Kd + 8 * (k & 15));
  }
  float am = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float v[8];
    bf16x8_to_f32(raw[i], v);
#pragma unroll
    for (int j = 0; j < 8; ++j) am = fmaxf(am, fabsf(v[j]));
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
  if ((tid & 31) == 0) s_red[tid >> 5] = am;
  __syncthreads();
  am = s_red[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) am = fmaxf(am, s_red[i]);
  const int e8 = scale_exp_of_amax(am);
  const float inv = exp2_neg(e8);
  uint8_t* dst = wq + (static_cast<size_t>(e) * N + static_cast<size_t>(nb) * kBlockM) * Kd + kb * kBlockK;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int k = i * 256 + tid;
    const int row = k >> 4, c8 = k & 15;
    float v[8];
    bf16x8_to_f32(raw[i], v);
    const uint2 b = make_uint2(
        static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(v[0], inv), __fmul_rn(v[1], inv))) |
            (static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(v[2], inv), __fmul_rn(v[3], inv))) << 16),
        static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(v[4], inv), __fmul_rn(v[5], inv))) |
            (static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(v[6], inv), __fmul_rn(v[7], inv))) << 16));
    *reinterpret_cast<uint2*>(dst + static_cast<size_t>(row) * Kd + 8 * c8) = b;
    if (wqt != nullptr) *reinterpret_cast<uint2*>(tile + tt_chunk(row, c8 >> 1) + 8 * (c8 & 1)) = b;
  }
  if (tid < 128) {
    const int KG = (Kd / kBlockK + 3) / 4;
    const size_t atom = ((static_cast<size_t>(e) * (N / kBlockM) + nb) * KG + kb / 4) * kSfAtomBytes;
    wsf[atom + 16 * (tid >> 2) + 4 * (tid & 3) + (kb % 4)] = static_cast<uint8_t>(e8 + 127);
  }
  if (wqt != nullptr) {  // uniform over the block
    __syncthreads();
    store_tile_transposed_128(
        tile,
        wqt + (static_cast<size_t>(e) * Kd + static_cast<size_t>(kb) * kBlockK) * N + static_cast<size_t>(nb) * kBlockM,
        static_cast<size_t>(N), tid);
    if (tid < 128) {
      const int KGn = (N / kBlockK + 3) / 4;
      const size_t atom = ((static_cast<size_t>(e) * (Kd / kBlockM) + kb) * KGn + nb / 4) * kSfAtomBytes;
      wsft[atom + 16 * (tid >> 2) + 4 * (tid & 3) + (nb % 4)] = static_cast<uint8_t>(e8 + 127);
    }
  }
}

cudaError_t launch_quant_pack(const void* x, int T, int H, const int32_t* experts, int K, const int32_t* tok_off,
                              const int32_t* s_rev, const int32_t* off, const int32_t* off_pad, uint8_t* xq,
                              uint8_t* xsf, cudaStream_t st, void* zero_out) {
  if (T == 0) return cudaSuccess;
  const int grid = (T + kQuantWarps - 1) / kQuantWarps;
  quant_pack_kernel<<<grid, kQuantWarps * 32, 0, st>>>(static_cast<const __nv_bfloat16*>(x), T, H, experts, K,
                                                       tok_off, s_rev, off, off_pad, xq, xsf,
                                                       static_cast<uint4*>(zero_out));
  return cudaGetLastError();
}

cudaError_t launch_weight_prep(const void* w, int E, int N, int Kd, int concat_glu, uint8_t* wq, uint8_t* wsf,
                               cudaStream_t st, uint8_t* wqt, uint8_t* wsft) {
  if (E == 0) return cudaSuccess;
  dim3 grid(Kd / kBlockK, N / kBlockM, E);
  weight_prep_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(w), E, N, Kd, concat_glu, wq, wsf, wqt,
                                           wsft);
  return cudaGetLastError();
}

}  // namespace smb
