// Router top-k and routing metadata kernels.
//
// router_topk_kernel   -- warp-per-row top-k with the reference's index-in-mantissa tie rule
//                         (sonicmoe/functional/topk.py:143-260) and its two softmax modes, plus a
//                         per-128-token tile histogram of the chosen experts for the metadata.
// route_hist_kernel    -- the same tile histogram for externally supplied expert ids.
// route_scan_kernel    -- per-expert exclusive scans over tiles, expert offsets and this build's
//                         128-row padded expert layout (one CTA).
// route_scatter_kernel -- stable expert-major permutation: s_scatter_idx, s_reverse_scatter_idx,
//                         x_gather_idx (triton_kernels/bitmatrix.py:63-147 computes the same
//                         permutation with a sort; here warp ballots/match give each entry its rank).
// token_offset_kernel  -- num_activated_expert_per_token_offset for general routing
//                         (triton_kernels/__init__.py:239-267: searchsorted over sorted tokens).
#include "common.cuh"
#include "sonic_internal.h"

namespace smb {

// ---------------------------------------------------------------------------------------------
// Float32 exp / log with a fixed operation order (the CPU oracle evaluates the same sequence):
// Cody-Waite reduction x = n ln2 + r and the degree-7 Taylor polynomial of e^r by Horner's rule;
// log via s = m 2^e, m in [sqrt(1/2), sqrt(2)), log m = 2 atanh(f / (2 + f)) to the z^11 term.
// __f*_rn intrinsics keep every step a separately rounded IEEE operation (no FMA contraction).
__device__ __forceinline__ float rt_exp(float x) {
  if (x != x) return x;
  const float nf = rintf(__fmul_rn(x, 1.4426950408889634f));
  if (nf < -126.0f) return 0.0f;
  if (nf > 127.0f) return __int_as_float(0x7f800000);
  const float ln2_hi = 0.693145751953125f;
  const float ln2_lo = static_cast<float>(0.6931471805599453 - 0.693145751953125);
  float r = __fsub_rn(x, __fmul_rn(nf, ln2_hi));
  r = __fsub_rn(r, __fmul_rn(nf, ln2_lo));
  float p = static_cast<float>(1.0 / 5040.0);
  p = __fadd_rn(__fmul_rn(p, r), static_cast<float>(1.0 / 720.0));
  p = __fadd_rn(__fmul_rn(p, r), static_cast<float>(1.0 / 120.0));
  p = __fadd_rn(__fmul_rn(p, r), static_cast<float>(1.0 / 24.0));
  p = __fadd_rn(__fmul_rn(p, r), static_cast<float>(1.0 / 6.0));
  p = __fadd_rn(__fmul_rn(p, r), 0.5f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  p = __fadd_rn(__fmul_rn(p, r), 1.0f);
  const int n = static_cast<int>(nf);
  return __fmul_rn(p, __uint_as_float(static_cast<uint32_t>(n + 127) << 23));
}

__device__ __forceinline__ float rt_log(float s) {
  const uint32_t b = __float_as_uint(s);
  int e = static_cast<int>((b >> 23) & 0xFFu) - 127;
  float m = __uint_as_float((b & 0x7FFFFFu) | 0x3F800000u);
  if (m > 1.4142135623730951f) {
    m = __fmul_rn(m, 0.5f);
    e += 1;
  }
  const float f = __fsub_rn(m, 1.0f);
  const float z = __fdiv_rn(f, __fadd_rn(2.0f, f));
  const float w = __fmul_rn(z, z);
  float p = static_cast<float>(2.0 / 11.0);
  p = __fadd_rn(__fmul_rn(p, w), static_cast<float>(2.0 / 9.0));
  p = __fadd_rn(__fmul_rn(p, w), static_cast<float>(2.0 / 7.0));
  p = __fadd_rn(__fmul_rn(p, w), static_cast<float>(2.0 / 5.0));
  p = __fadd_rn(__fmul_rn(p, w), static_cast<float>(2.0 / 3.0));
  p = __fadd_rn(__fmul_rn(p, w), 2.0f);
  const float logm = __fmul_rn(z, p);
  const float ef = static_cast<float>(e);
  const float ln2_hi = 0.693145751953125f;
  const float ln2_lo = static_cast<float>(0.6931471805599453 - 0.693145751953125);
  const float t = __fadd_rn(logm, __fmul_rn(ef, ln2_lo));
  return __fadd_rn(__fmul_rn(ef, ln2_hi), t);
}

// uint32 key whose unsigned order is the IEEE total order of the float bit pattern, and back.
__device__ __forceinline__ uint32_t order_key(uint32_t bits) {
  return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}
__device__ __forceinline__ uint32_t order_key_inv(uint32_t key) {
  return (key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key;
}

template <typename InT>
__device__ __forceinline__ float load_f32(const InT* p);
template <>
__device__ __forceinline__ float load_f32<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <>
__device__ __forceinline__ float load_f32<__half>(const __half* p) {
  return __half2float(*p);
}
template <>
__device__ __forceinline__ float load_f32<float>(const float* p) {
  return *p;
}


// PL: per-lane register capacity (>= ceil(E/32) rounded to the lane vector); KMAX >= K.
// Warps per 128-token tile: narrow rows (<= 8 values per lane) use 32 warps (4 rows each, the next
// row's logits loaded while the current one is scored); wide rows keep register pressure down
// with 8 warps.
template <int PL>
struct RouterShape {
  static constexpr int kWarps = PL <= 8 ? 32 : 8;
  static constexpr bool kPrefetch = PL <= 8;
};

// Top-k (+ softmax) of the rows [row0, row0 + 128) of a [T, E] logits array, kWarps warps of the
// calling CTA, warp w taking rows w, w + kWarps, ... ; the chosen experts are counted into the
// CTA's shared histogram s_hist (when non-null).  Shared by the top-k kernel over given logits and
// by the fused router, which runs it on the logits tile its GEMM has just written.
template <typename InT, int PL, int KMAX, int kWarps, bool kPrefetch>
__device__ __forceinline__ void route_tile_rows(const InT* __restrict__ logits, int row0, int T, int E, int K,
                                                int vec, int softmax_over_topk, int renorm,
                                                float* __restrict__ scores, int32_t* __restrict__ indices,
                                                int32_t* s_hist) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int log_n = 0;
  while ((1 << log_n) < E) ++log_n;
  const uint32_t mask = (1u << log_n) - 1u;
  const int steps = (E + 32 * vec - 1) / (32 * vec);
  // lane's i-th element is column (i / vec) * 32 * vec + lane * vec + i % vec
  auto col_of = [&](int i) -> int {
    const int j = i / vec;
    const int c = j * 32 * vec + lane * vec + (i - j * vec);
    return (j < steps && c < E) ? c : -1;
  };
  auto load_row = [&](int row, float* dst) {
    const InT* src = logits + static_cast<size_t>(row) * E;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const int c = col_of(i);
      dst[i] = (c >= 0) ? load_f32<InT>(src + c) : 0.0f;
    }
  };
  float vn[PL];
  if (kPrefetch && warp < kTileTokens && row0 + warp < T) load_row(row0 + warp, vn);

  for (int r = warp; r < kTileTokens; r += kWarps) {
    const int row = row0 + r;
    if (row >= T) break;
    float v[PL];
    if (kPrefetch) {
#pragma unroll
      for (int i = 0; i < PL; ++i) v[i] = vn[i];
      const int rn = row + kWarps;
      if (r + kWarps < kTileTokens && rn < T) load_row(rn, vn);
    } else {
      load_row(row, v);
    }
    if (!softmax_over_topk) {
      // log-softmax over the full row (topk.py:143-198): max, then sum of exp(x - max) in lane
      // order followed by an xor butterfly (identical result on every lane), then x - log_norm.
      float mx = -__int_as_float(0x7f800000);
#pragma unroll
      for (int i = 0; i < PL; ++i)
        if (col_of(i) >= 0) mx = fmaxf(mx, v[i]);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float s = 0.0f;
#pragma unroll
      for (int i = 0; i < PL; ++i)
        if (col_of(i) >= 0) s = __fadd_rn(s, rt_exp(__fsub_rn(v[i], mx)));
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
      const float log_norm = __fadd_rn(mx, rt_log(s));
#pragma unroll
      for (int i = 0; i < PL; ++i) v[i] = __fsub_rn(v[i], log_norm);
    }
    // index into the low mantissa bits (topk.py:200-215)
    uint32_t key[PL];
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const int ci = col_of(i);
      if (ci < 0) {
        key[i] = 0u;
      } else {
        const uint32_t c = static_cast<uint32_t>(ci);
        const uint32_t enc = (v[i] >= 0.0f) ? (~c & mask) : (c & mask);
        key[i] = order_key((__float_as_uint(v[i]) & ~mask) | enc);
      }
    }
    // K rounds of warp arg-max over unique keys; lane k keeps the k-th selection
    uint32_t mysel = 0u;
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      if (k < K) {
        uint32_t best = 0u;
#pragma unroll
        for (int i = 0; i < PL; ++i) best = max(best, key[i]);
        const uint32_t wmax = __reduce_max_sync(0xffffffffu, best);
#pragma unroll
        for (int i = 0; i < PL; ++i)
          if (key[i] == wmax) key[i] = 0u;
        if (lane == k) mysel = wmax;
      }
    }
    // decode (topk.py:222-234) and score (topk.py:237-260) on lane k for selection k; the K-term
    // sum is accumulated in selection order on every lane from the lanes' exps (same operations,
    // same order as a sequential loop over k)
    const bool act = lane < K;
    const uint32_t bits = order_key_inv(mysel);
    const uint32_t enc = bits & mask;
    float val = __uint_as_float(bits & ~mask);
    const int idx = static_cast<int>((val >= 0.0f) ? (~enc & mask) : enc);
    float e;
    if (softmax_over_topk) {
      float vmax = act ? val : -__int_as_float(0x7f800000);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
      e = act ? rt_exp(__fsub_rn(val, vmax)) : 0.0f;
    } else {
      e = act ? rt_exp(val) : 0.0f;
    }
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
      if (k < K) s = __fadd_rn(s, __shfl_sync(0xffffffffu, e, k));
    if (softmax_over_topk || renorm) e = __fdiv_rn(e, s);
    if (act) {
      scores[static_cast<size_t>(row) * K + lane] = e;
      indices[static_cast<size_t>(row) * K + lane] = idx;
      if (s_hist) atomicAdd(&s_hist[idx], 1);
    }
  }
}

template <typename InT, int PL, int KMAX>
__global__ void __launch_bounds__(RouterShape<PL>::kWarps * 32)
    router_topk_kernel(const InT* __restrict__ logits, int T, int E, int K, int vec, int softmax_over_topk,
                       int renorm, float* __restrict__ scores, int32_t* __restrict__ indices,
                       int32_t* __restrict__ tile_counts, int n_tiles) {
  extern __shared__ int32_t s_hist[];  // [E] when tile_counts != nullptr
  const int tile = blockIdx.x;
  if (tile_counts) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) s_hist[e] = 0;
    __syncthreads();
  }
  route_tile_rows<InT, PL, KMAX, RouterShape<PL>::kWarps, RouterShape<PL>::kPrefetch>(
      logits, tile * kTileTokens, T, E, K, vec, softmax_over_topk, renorm, scores, indices,
      tile_counts ? s_hist : nullptr);
  if (tile_counts) {
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += blockDim.x) tile_counts[static_cast<size_t>(e) * n_tiles + tile] = s_hist[e];
  }
}

// ---------------------------------------------------------------------------------------------
// Fused router: one CTA per 128-token tile computes the tile's logits x[tile] @ w^T with
// tcgen05.mma.kind::f16 (bf16 operands by TMA with the 128-byte swizzle, 64 hidden columns per
// stage, fp32 accumulator of E columns in tensor memory), rounds them to bf16 into the logits
// output, and then all 16 warps run the same top-k (+ softmax) as router_topk_kernel on those
// rows.  It replaces the separate logits GEMM (torch F.linear in the reference,
// functional/__init__.py:501) plus the top-k launch; the tensor-core accumulation order differs
// from cuBLAS's, so logits may differ in the last bf16 bit and the path is opt-in.
// Roles: warp 0 TMA producer, warp 1 MMA issuer, warp 2 tensor-memory allocation, warps 4-7 read
// the accumulator (warp w: rows 32 (w % 4) .. + 31).
constexpr int kRfThreads = 512;
constexpr int kRfKBlock = 64;  // bf16 values per 128-byte swizzled row: K extent of one stage
// Ring depth: 3 stages when a stage is at most 32 KB (E <= 128), so that two CTAs share an SM and
// one tile's top-k and ring refill overlap the other's MMAs; 4 stages (one CTA per SM) above.
constexpr int kRfMaxStages = 4;
__host__ __device__ constexpr int rf_stages(int E) { return E <= 128 ? 3 : 4; }
constexpr int kRfABytes = kTileTokens * 128;  // 16 KB of x per stage

__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// kind::f16 instruction descriptor: bf16 x bf16 -> f32, both operands K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

template <int PL, int KMAX>
__global__ void __launch_bounds__(kRfThreads, 2)
    router_fused_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                        int T, int H, int E, int K, int vec, int softmax_over_topk, int renorm, uint32_t tmem_cols,
                        __nv_bfloat16* __restrict__ logits, float* __restrict__ scores,
                        int32_t* __restrict__ indices, int32_t* __restrict__ tile_counts, int n_tiles, int* err) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  const int stage_bytes = kRfABytes + E * 128;  // multiple of 4 KB (E % 32 == 0)
  const int kRfStages = rf_stages(E);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRfStages * stage_bytes);
  uint64_t* empty = full + kRfMaxStages;
  uint64_t* tmem_full = empty + kRfStages;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tmem_full + 1);
  int32_t* s_hist = reinterpret_cast<int32_t*>(tmem_holder + 4);  // [E]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int row0 = tile * kTileTokens;
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < kRfStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    fence_mbar_init();
    prefetch_tmap(&tmap_x);
    prefetch_tmap(&tmap_w);
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_hist[e] = 0;
  if (warp == 2) {
    tmem_alloc(tmem_holder, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int KB = H / kRfKBlock;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ TMA producer
      const uint64_t pol_x = policy_evict_first();  // x streams through once
      const uint64_t pol_w = policy_evict_last();   // the router weight is read by every tile
      int kb = 0;
      for (; kb < KB; ++kb) {
        const int s = kb % kRfStages;
        const uint32_t ph = (kb / kRfStages) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, err, kErrTimeoutProducer)) break;
        uint8_t* st = smem + s * stage_bytes;
        mbar_arrive_expect_tx(&full[s], stage_bytes);
        tma_load_2d(st, &tmap_x, &full[s], kb * kRfKBlock, row0, pol_x);
        tma_load_2d(st + kRfABytes, &tmap_w, &full[s], kb * kRfKBlock, 0, pol_w);
      }
      if (kb < KB) {
        // an error elsewhere: let the loads already issued land before shared memory goes away
        for (int j = (kb - kRfStages > 0 ? kb - kRfStages : 0); j < kb; ++j)
          mbar_wait_ns(&full[j % kRfStages], (j / kRfStages) & 1, 50000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      const uint32_t idesc = idesc_bf16(kTileTokens, E);
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % kRfStages;
        const uint32_t ph = (kb / kRfStages) & 1;
        if (!mbar_wait(&full[s], ph, err, kErrTimeoutMma)) break;
        tc_fence_after();
        uint8_t* st = smem + s * stage_bytes;
        const uint64_t ad = sdesc_sw128(smem_u32(st));
        const uint64_t bd = sdesc_sw128(smem_u32(st + kRfABytes));
#pragma unroll
        for (int kk = 0; kk < kRfKBlock / 16; ++kk)  // K = 16 per MMA: +32 bytes = +2 in the address field
          tc_mma_bf16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (kb | kk) != 0 ? 1u : 0u);
        tc_commit(&empty[s]);
      }
      // completes once every MMA issued above has finished (also after an early exit)
      tc_commit(tmem_full);
    }
  } else if (warp >= 4 && warp < 8) {
    // -------------------------------------------------------------------- logits out
    const int q = warp & 3;
    const int row = row0 + q * 32 + lane;
    if (mbar_wait(tmem_full, 0, err, kErrTimeoutEpilogue)) {
      tc_fence_after();
      for (int c = 0; c < E / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + 32 * c, v);
        tmem_ld_wait();
        if (row < T) {
          uint4* dst = reinterpret_cast<uint4*>(logits + static_cast<size_t>(row) * E + 32 * c);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint4 w;
            w.x = pack_bf16x2_rn(__uint_as_float(v[8 * j]), __uint_as_float(v[8 * j + 1]));
            w.y = pack_bf16x2_rn(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3]));
            w.z = pack_bf16x2_rn(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5]));
            w.w = pack_bf16x2_rn(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7]));
            dst[j] = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();  // the tile's logits are written (visible to this CTA) and tensor memory is read
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
  // top-k of the tile's rows over the bf16 logits just written, by all 16 warps
  route_tile_rows<__nv_bfloat16, PL, KMAX, kRfThreads / 32, true>(logits, row0, T, E, K, vec, softmax_over_topk,
                                                                   renorm, scores, indices, s_hist);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) tile_counts[static_cast<size_t>(e) * n_tiles + tile] = s_hist[e];
}

// ---------------------------------------------------------------------------------------------
// Tile histogram of externally supplied expert ids.  Tile t covers flat entries
// [t * entries_per_tile, (t + 1) * entries_per_tile).
// With allow_holes, negative ids mark "no entry" (used by the expert-parallel path) and are skipped
// silently; otherwise they are reported like any id outside [0, E).
__global__ void route_hist_kernel(const int32_t* __restrict__ experts, int TK, int entries_per_tile, int E,
                                  int n_tiles, int allow_holes, int32_t* __restrict__ tile_counts,
                                  int* __restrict__ err) {
  extern __shared__ int32_t s_hist[];
  const int tile = blockIdx.x;
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_hist[e] = 0;
  __syncthreads();
  const int f0 = tile * entries_per_tile;
  const int f1 = min(TK, f0 + entries_per_tile);
  for (int f = f0 + threadIdx.x; f < f1; f += blockDim.x) {
    const int e = experts[f];
    if (e >= 0 && e < E) {
      atomicAdd(&s_hist[e], 1);
    } else if (!(allow_holes && e < 0)) {
      atomicCAS(err, 0, kErrBadExpert);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) tile_counts[static_cast<size_t>(e) * n_tiles + tile] = s_hist[e];
}

// ---------------------------------------------------------------------------------------------
// One CTA of 1024 threads.  tile_counts[e][tile] -> exclusive prefix over tiles (in place);
// freq, off (E+1, off[E] = TK), padded layout (off_pad in rows, blk_expert, n_blocks).
constexpr int kScanThreads = 1024;

__global__ void __launch_bounds__(kScanThreads)
    route_scan_kernel(int32_t* __restrict__ tile_counts, int n_tiles, int E, int TK, int32_t* __restrict__ freq,
                      int32_t* __restrict__ off, int32_t* __restrict__ off_pad, int32_t* __restrict__ blk_expert,
                      int32_t* __restrict__ n_blocks) {
  extern __shared__ int32_t s_freq[];  // [E]
  __shared__ int32_t s_wsum[2][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = kScanThreads / 32;
  // (1) per expert: exclusive scan over tiles, one warp per expert
  for (int e = warp; e < E; e += nwarps) {
    int32_t* row = tile_counts + static_cast<size_t>(e) * n_tiles;
    int running = 0;
    for (int base = 0; base < n_tiles; base += 32) {
      const int t = base + lane;
      const int c = (t < n_tiles) ? row[t] : 0;
      int inc = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
      }
      if (t < n_tiles) row[t] = running + inc - c;
      running += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) {
      s_freq[e] = running;
      freq[e] = running;
    }
  }
  __syncthreads();
  // (2) exclusive scans over experts of freq and of the padded block counts; each thread owns a
  // contiguous chunk of experts
  const int per = (E + kScanThreads - 1) / kScanThreads;
  const int e0 = threadIdx.x * per;
  int a = 0, b = 0;
  for (int e = e0; e < min(E, e0 + per); ++e) {
    a += s_freq[e];
    b += padded_blocks_of(s_freq[e]);
  }
  int ia = a, ib = b;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ya = __shfl_up_sync(0xffffffffu, ia, o);
    const int yb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) {
      ia += ya;
      ib += yb;
    }
  }
  if (lane == 31) {
    s_wsum[0][warp] = ia;
    s_wsum[1][warp] = ib;
  }
  __syncthreads();
  if (warp == 0) {
    int wa = s_wsum[0][lane], wb = s_wsum[1][lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int ya = __shfl_up_sync(0xffffffffu, wa, o);
      const int yb = __shfl_up_sync(0xffffffffu, wb, o);
      if (lane >= o) {
        wa += ya;
        wb += yb;
      }
    }
    s_wsum[0][lane] = wa;  // inclusive over warps
    s_wsum[1][lane] = wb;
  }
  __syncthreads();
  int ra = ia - a + (warp > 0 ? s_wsum[0][warp - 1] : 0);
  int rb = ib - b + (warp > 0 ? s_wsum[1][warp - 1] : 0);
  for (int e = e0; e < min(E, e0 + per); ++e) {
    const int f = s_freq[e];
    const int nb = padded_blocks_of(f);
    off[e] = ra;
    off_pad[e] = rb * kBlockM;
    for (int k = 0; k < nb; ++k) blk_expert[rb + k] = e;
    ra += f;
    rb += nb;
  }
  if (threadIdx.x == kScanThreads - 1) {
    off[E] = TK;
    off_pad[E] = s_wsum[1][31] * kBlockM;
    *n_blocks = s_wsum[1][31];
  }
}

// ---------------------------------------------------------------------------------------------
// One warp per tile: entries of the tile in flat order, 32 at a time; each entry's position is
// off[e] + (entries of e in earlier tiles) + (entries of e earlier in this tile), i.e. the stable
// argsort of the flat expert ids.  token_of_entry == nullptr means token = f / K.
__global__ void __launch_bounds__(32)
    route_scatter_kernel(const int32_t* __restrict__ experts, const int32_t* __restrict__ token_of_entry, int TK,
                         int K, int entries_per_tile, int E, int n_tiles, const int32_t* __restrict__ tile_base,
                         const int32_t* __restrict__ off, int32_t* __restrict__ s_scatter,
                         int32_t* __restrict__ s_rev, int32_t* __restrict__ x_gather) {
  extern __shared__ int32_t s_next[];  // [E]
  const int tile = blockIdx.x;
  const int lane = threadIdx.x;
  for (int e = lane; e < E; e += 32) s_next[e] = off[e] + tile_base[static_cast<size_t>(e) * n_tiles + tile];
  __syncwarp();
  const int f0 = tile * entries_per_tile;
  const int f1 = min(TK, f0 + entries_per_tile);
  const uint32_t lt = (1u << lane) - 1u;
  for (int base = f0; base < f1; base += 32) {
    const int f = base + lane;
    const bool valid = f < f1;
    int e = valid ? experts[f] : -1;
    if (e < 0 || e >= E) e = -1;  // rejected by the histogram pass (error word set there)
    const uint32_t peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & lt);
    const int pos = (e >= 0) ? s_next[e] + rank : 0;
    __syncwarp();
    if (e >= 0 && rank == 0) s_next[e] += __popc(peers);
    __syncwarp();
    if (e >= 0) {
      s_rev[f] = pos;
      s_scatter[pos] = f;
      x_gather[pos] = token_of_entry ? token_of_entry[f] : f / K;
    }
  }
}

// offset[t] = first index i with sorted_tokens[i] >= t, t in [0, T]
__global__ void token_offset_kernel(const int32_t* __restrict__ sorted_tokens, int T, int TK,
                                    int32_t* __restrict__ offset) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t > T) return;
  int lo = 0, hi = TK;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (sorted_tokens[mid] < t)
      lo = mid + 1;
    else
      hi = mid;
  }
  offset[t] = lo;
}

// ---------------------------------------------------------------------------------------------
// host launchers
template <typename InT, int PL, int KMAX>
static cudaError_t launch_router_t(const void* logits, int T, int E, int K, int vec, int sot, int renorm, float* scores,
                                   int32_t* idx, int32_t* tile_counts, cudaStream_t st) {
  const int n_tiles = (T + kTileTokens - 1) / kTileTokens;
  const size_t smem = tile_counts ? static_cast<size_t>(E) * sizeof(int32_t) : 0;
  auto kern = router_topk_kernel<InT, PL, KMAX>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  kern<<<n_tiles, RouterShape<PL>::kWarps * 32, smem, st>>>(static_cast<const InT*>(logits), T, E, K, vec, sot,
                                                             renorm, scores, idx, tile_counts, n_tiles);
  return cudaGetLastError();
}

template <typename InT>
static cudaError_t launch_router_dtype(const void* logits, int T, int E, int K, int sot, int renorm, float* scores,
                                       int32_t* idx, int32_t* tile_counts, cudaStream_t st) {
  int vec = 1;
  for (int v : {8, 4, 2})
    if (E % (32 * v) == 0) {
      vec = v;
      break;
    }
  const int per_lane = ((E + 32 * vec - 1) / (32 * vec)) * vec;
  if (K <= 16) {
    if (per_lane <= 4) return launch_router_t<InT, 4, 16>(logits, T, E, K, vec, sot, renorm, scores, idx, tile_counts, st);
    if (per_lane <= 8) return launch_router_t<InT, 8, 16>(logits, T, E, K, vec, sot, renorm, scores, idx, tile_counts, st);
    if (per_lane <= 32) return launch_router_t<InT, 32, 16>(logits, T, E, K, vec, sot, renorm, scores, idx, tile_counts, st);
    return launch_router_t<InT, 128, 16>(logits, T, E, K, vec, sot, renorm, scores, idx, tile_counts, st);
  }
  if (per_lane <= 8) return launch_router_t<InT, 8, 32>(logits, T, E, K, vec, sot, renorm, scores, idx, tile_counts, st);
  if (per_lane <= 32) return launch_router_t<InT, 32, 32>(logits, T, E, K, vec, sot, renorm, scores, idx, tile_counts, st);
  return launch_router_t<InT, 128, 32>(logits, T, E, K, vec, sot, renorm, scores, idx, tile_counts, st);
}

cudaError_t launch_router_topk(const void* logits, int dtype, int T, int E, int K, int sot, int renorm, float* scores,
                               int32_t* idx, int32_t* tile_counts, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  switch (dtype) {
    case kDtypeBF16:
      return launch_router_dtype<__nv_bfloat16>(logits, T, E, K, sot, renorm, scores, idx, tile_counts, st);
    case kDtypeF16:
      return launch_router_dtype<__half>(logits, T, E, K, sot, renorm, scores, idx, tile_counts, st);
    default:
      return launch_router_dtype<float>(logits, T, E, K, sot, renorm, scores, idx, tile_counts, st);
  }
}

template <int PL, int KMAX>
static cudaError_t launch_router_fused_t(const void* x, const void* w, int T, int H, int E, int K, int vec, int sot,
                                         int renorm, void* logits, float* scores, int32_t* idx,
                                         int32_t* tile_counts, int* err, cudaStream_t st) {
  const int n_tiles = (T + kTileTokens - 1) / kTileTokens;
  CUtensorMap tx, tw;
  if (!encode_tmap_2d(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, static_cast<uint64_t>(H), static_cast<uint64_t>(T),
                      kRfKBlock, kTileTokens, true) ||
      !encode_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, static_cast<uint64_t>(H), static_cast<uint64_t>(E),
                      kRfKBlock, static_cast<uint32_t>(E), true))
    return cudaErrorInvalidValue;
  uint32_t cols = 32;
  while (cols < static_cast<uint32_t>(E)) cols <<= 1;
  const int smem = rf_stages(E) * (kRfABytes + E * 128) + (2 * kRfMaxStages + 1) * 8 + 16 + E * 4 + 1024;
  auto kern = router_fused_kernel<PL, KMAX>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  kern<<<n_tiles, kRfThreads, smem, st>>>(tx, tw, T, H, E, K, vec, sot, renorm, cols,
                                          static_cast<__nv_bfloat16*>(logits), scores, idx, tile_counts, n_tiles, err);
  return cudaGetLastError();
}

cudaError_t launch_router_fused(const void* x, const void* w, int T, int H, int E, int K, int sot, int renorm,
                                void* logits, float* scores, int32_t* idx, int32_t* tile_counts, int* err,
                                cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  if (E % 32 != 0 || E < 32 || E > 256 || H % kRfKBlock != 0 || K < 1 || K > 32) return cudaErrorInvalidValue;
  int vec = 1;
  for (int v : {8, 4, 2})
    if (E % (32 * v) == 0) {
      vec = v;
      break;
    }
  const int per_lane = ((E + 32 * vec - 1) / (32 * vec)) * vec;
  if (K <= 16) {
    if (per_lane <= 4)
      return launch_router_fused_t<4, 16>(x, w, T, H, E, K, vec, sot, renorm, logits, scores, idx, tile_counts, err, st);
    return launch_router_fused_t<8, 16>(x, w, T, H, E, K, vec, sot, renorm, logits, scores, idx, tile_counts, err, st);
  }
  if (per_lane <= 4)
    return launch_router_fused_t<4, 32>(x, w, T, H, E, K, vec, sot, renorm, logits, scores, idx, tile_counts, err, st);
  return launch_router_fused_t<8, 32>(x, w, T, H, E, K, vec, sot, renorm, logits, scores, idx, tile_counts, err, st);
}

static cudaError_t route_hist_impl(const int32_t* experts, int TK, int entries_per_tile, int E, int n_tiles,
                                   int allow_holes, int32_t* tile_counts, int* err, cudaStream_t st) {
  if (n_tiles == 0) return cudaSuccess;
  const size_t smem = static_cast<size_t>(E) * sizeof(int32_t);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(route_hist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  route_hist_kernel<<<n_tiles, 256, smem, st>>>(experts, TK, entries_per_tile, E, n_tiles, allow_holes, tile_counts,
                                                err);
  return cudaGetLastError();
}

cudaError_t launch_route_hist(const int32_t* experts, int TK, int entries_per_tile, int E, int n_tiles,
                              int32_t* tile_counts, int* err, cudaStream_t st) {
  return route_hist_impl(experts, TK, entries_per_tile, E, n_tiles, 0, tile_counts, err, st);
}

cudaError_t launch_route_hist_holes(const int32_t* experts, int TK, int entries_per_tile, int E, int n_tiles,
                                    int32_t* tile_counts, int* err, cudaStream_t st) {
  return route_hist_impl(experts, TK, entries_per_tile, E, n_tiles, 1, tile_counts, err, st);
}

cudaError_t launch_route_scan(int32_t* tile_counts, int n_tiles, int E, int TK, int32_t* freq, int32_t* off,
                              int32_t* off_pad, int32_t* blk_expert, int32_t* n_blocks, cudaStream_t st) {
  const size_t smem = static_cast<size_t>(E) * sizeof(int32_t);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(route_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  route_scan_kernel<<<1, kScanThreads, smem, st>>>(tile_counts, n_tiles, E, TK, freq, off, off_pad, blk_expert,
                                                   n_blocks);
  return cudaGetLastError();
}

cudaError_t launch_route_scatter(const int32_t* experts, const int32_t* token_of_entry, int TK, int K,
                                 int entries_per_tile, int E, int n_tiles, const int32_t* tile_base,
                                 const int32_t* off, int32_t* s_scatter, int32_t* s_rev, int32_t* x_gather,
                                 cudaStream_t st) {
  if (n_tiles == 0) return cudaSuccess;
  const size_t smem = static_cast<size_t>(E) * sizeof(int32_t);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(route_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  route_scatter_kernel<<<n_tiles, 32, smem, st>>>(experts, token_of_entry, TK, K, entries_per_tile, E, n_tiles,
                                                  tile_base, off, s_scatter, s_rev, x_gather);
  return cudaGetLastError();
}

cudaError_t launch_token_offset(const int32_t* sorted_tokens, int T, int TK, int32_t* offset, cudaStream_t st) {
  const int n = T + 1;
  token_offset_kernel<<<(n + 255) / 256, 256, 0, st>>>(sorted_tokens, T, TK, offset);
  return cudaGetLastError();
}

}  // namespace smb
