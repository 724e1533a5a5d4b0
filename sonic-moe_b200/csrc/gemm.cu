// Block-scaled FP8 grouped GEMMs of the MoE layer on tcgen05 (sm_100a).
//
// One persistent kernel, two epilogues:
//   up   : h = A x W1[e]^T over a 128x256 tile (A = packed e4m3 tokens, 1x128 UE8M0 scales;
//          W1 = e4m3 weights, 128x128 UE8M0 scales), then a = silu(gate) * up and the 1x128
//          requantisation of `a` to e4m3 + UE8M0, staged in shared memory and written by one TMA
//          tensor store per tile into the padded expert-major layout the down projection reads.
//          (Reference: functional/__init__.py:260-275, QuACK gemm_act.)
//          Expert parallel with the down projection at the tokens' home ranks: each requantised
//          row goes straight from registers into its home rank's padded layout (peer stores over
//          NVLink, tile by tile under the main loop of the next tile) instead of the local tile.
//   down : y = a x W2[e]^T over a 128x256 tile, then o[token] += score * y as TMA bulk bf16
//          reductions (one 128-byte row chunk per thread) straight into the token-major output,
//          i.e. the top-k weighted combine of functional/forward.py:64-85 fused into the epilogue.
//
// Tiles: 128 rows of one expert (the padded layout never mixes experts in a tile) x 256 output
// columns, K consumed 128 at a time.  Roles per CTA (640 threads, one CTA per SM):
//   warp 0      TMA producer: A and B tiles (128B swizzle) + scale-factor atoms (bulk copies)
//   warp 1      MMA issuer: tcgen05.cp of the scale factors to tensor memory, then 4 x
//               tcgen05.mma.kind::mxf8f6f4.block_scale (M=128, N=256, K=32) per stage
//   warp 2      tensor-memory allocation (512 columns: accumulator 0-255, SFA 256-259, SFB 260-267)
//   warps 4-19  epilogue: warp w reads TMEM lanes 32*(w%4)..+31, columns chunk (w-4)/4, releases
//               the accumulator as soon as it sits in registers, then computes and stores while
//               the next tile's main loop runs.
// Tile schedule: static round robin over (m-block, n-tile), n fastest (the down projection in up to
// 4 column slices); the number of m-blocks is read from device memory, so empty experts cost
// nothing and no host synchronisation is needed.
// Every mbarrier wait is bounded (2 s); on a timeout the kernel records an error code, drains its
// outstanding copies and MMAs with short bounded waits, frees tensor memory and returns.
#include "common.cuh"
#include "sonic_internal.h"

namespace smb {

constexpr int kBN = 256;
constexpr int kEpiWarps = 16;
constexpr int kGemmThreads = (4 + kEpiWarps) * 32;
constexpr int kABytes = kBlockM * kBlockK;  // 16 KB
constexpr int kBBytes = kBN * kBlockK;      // 32 KB
constexpr int kSfaBytes = kSfAtomBytes;
constexpr int kSfbBytes = 2 * kSfAtomBytes;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemAcc = 0, kTmemSfa = 256, kTmemSfb = 260;
constexpr int kNumBars = 2 * 4 + 5;  // full/empty per stage (at most 4 stages) + 5
constexpr int kRowChunkBytes = 128;  // down epilogue: one thread's 64 bf16 of one output row
// Staging slots are 144 bytes apart: a warp's 32 slots then start in 8 different 16-byte bank
// groups, so its 16-byte stores are 4-way (the minimum for 512 bytes) instead of 32-way conflicted.
constexpr int kSlotStride = 144;

// Epilogue kinds of the one persistent kernel:
//   kKindDown  down projection + top-k combine (bulk bf16 reductions into the token rows)
//   kKindUp    up projection + SwiGLU + requantisation
//   kKindDact  backward of the down projection and the activation: dA' = dO W2 per entry, then
//              dS (row dot with a), dH (SwiGLU backward from the stored h, e4m3 + bf16) and
//              a' = score * a (bf16)
//   kKindWgrad weight gradient: tiles (expert, m, n) of D[e] = A[:, rows_e] B[:, rows_e]^T with K
//              = the expert's padded rows, stored as bf16
constexpr int kKindDown = 0, kKindUp = 1, kKindDact = 2, kKindWgrad = 3;

// Shared-memory layout per epilogue kind.  The up projection keeps a 4-stage ring plus a 16 KB
// output tile; the down projection gives one stage up for 72 KB of per-thread staging from which
// its output rows are reduced into global memory by TMA bulk reductions; the backward kinds store
// straight from registers.
template <int kKind>
struct GemmSmem {
  static constexpr bool kUp = kKind == kKindUp;
  // down and weight-gradient epilogues stage rows in per-thread slots: one stage fewer makes room
  static constexpr bool kSlots = kKind == kKindDown || kKind == kKindWgrad;
  static constexpr int kStages = kSlots ? 3 : 4;
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + kStages * kABytes;
  static constexpr int kOffSfa = kOffB + kStages * kBBytes;
  static constexpr int kOffSfb = kOffSfa + kStages * kSfaBytes;
  static constexpr int kOffStage = kOffSfb + kStages * kSfbBytes;
  // up: one 128 x 128-byte e4m3 output tile (128B-swizzled, TMA-stored); down, weight gradient:
  // per-thread slots of one 128-byte row chunk
  static constexpr int kStageBytes = kUp ? kBlockM * 128 : (kSlots ? kEpiWarps * 32 * kSlotStride : 0);
  static constexpr int kOffBar = kOffStage + kStageBytes;
  static constexpr int kOffTmemHolder = kOffBar + kNumBars * 8;
  static constexpr int kOffAmax = (kOffTmemHolder + 4 + 15) / 16 * 16;
  // up: [tile parity][column warp][row] row maxima; activation gradient: [parity][gate/up][column warp][row]
  static constexpr int kAmaxFloats = kUp ? 2 * 4 * kBlockM : (kKind == kKindDact ? 2 * 2 * 4 * kBlockM : 0);
  static constexpr int kBytes = kOffAmax + kAmaxFloats * 4;
  static constexpr int kAlloc = kBytes + 1024;  // slack for 1024-byte alignment of the base
  static_assert(kAlloc <= 232448, "shared memory budget");
  static_assert(kOffStage % (kUp ? 1024 : 128) == 0, "staging alignment (128B-swizzled TMA store for up)");
};

__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&p);
}
// Tile -> (m-block, n-tile).  The n-tiles are split into `n_slices` column slices; all tiles of
// one slice come before the next slice, n fastest inside a slice.  With one slice this is plain
// m-major order.  The down projection uses several slices so that the slice of the bf16 output
// its reductions land in stays resident in L2 while the slice is being computed.
__device__ __forceinline__ void tile_coords(int tile, int n_blocks, int ntn, int n_slices, int& mb, int& nt) {
  const int nts = ntn / n_slices;
  const int per_slice = n_blocks * nts;
  const int slice = tile / per_slice;
  const int r = tile - slice * per_slice;
  mb = r / nts;
  nt = slice * nts + (r - mb * nts);
}

// What one epilogue thread needs to know about its row of a tile: the dependent loads block ->
// expert -> offsets -> scatter index -> score, issued after the accumulator has been released.
struct RowMeta {
  int mb, nt, e;
  int p;      // padded row
  int valid;  // a real (token, expert) entry, not padding
  int tok;    // down: token whose output row receives the reduction; up, expert parallel: ret_dst[p]
  float sc;   // down: its router score
};

template <int kKind>
__device__ __forceinline__ RowMeta load_row_meta(const GemmArgs& g, int tile, int n_blocks, int ntn, int r) {
  constexpr bool kUp = kKind == kKindUp;
  RowMeta m;
  tile_coords(tile, n_blocks, ntn, g.n_slices, m.mb, m.nt);
  m.e = g.blk_expert[m.mb];
  m.p = m.mb * kBlockM + r;
  const int rel = m.p - g.off_pad[m.e];
  m.valid = rel < g.freq[m.e];
  m.tok = 0;
  m.sc = 0.0f;
  if constexpr (kUp) {
    if (g.ret_dst != nullptr) m.tok = m.valid ? g.ret_dst[m.p] : -1;
    if (g.preact != nullptr) m.tok = rel + g.off[m.e];  // expert-sorted entry row of the stored h
  } else if constexpr (kKind == kKindDact) {
    if (m.valid) {
      m.tok = rel + g.off[m.e];              // expert-sorted row of h
      m.sc = g.scores[g.s_scatter[m.tok]];  // router score of the entry
    }
  } else {
    if (m.valid) {
      const int rs = rel + g.off[m.e];
      m.tok = g.x_gather[rs];
      m.sc = g.scores ? g.scores[g.s_scatter[rs]] : 1.0f;
    }
  }
  return m;
}

// Activation-gradient epilogue (backward of functional/backward.py:211-278, `gemm_dact` with
// colvec_scale = s and colvec_reduce): this thread holds dA'[entry, i] = (dO[token] W2[e])[i] for the
// 64 intermediate columns i = 256 nt + 64 cc + j of its row.  With (g, u) the stored pre-activation
// (interleaved columns 2i, 2i+1), sig = 1 / (1 + e^-g), a = g sig u:
//   dS[entry] += sum_j dA'_j a_j            (fp32 atomics: four column warps x I/256 tiles)
//   a'_j = s a_j                            (bf16, padded row; the dW2 operand)
//   dg_j = s dA'_j u sig (1 + g (1 - sig)),  du_j = s dA'_j g sig
// dH is written as bf16 (padded row; the dW1 operand) and, quantised from those bf16 values, as
// e4m3 with one UE8M0 scale for its 128 values -- exactly one 1x128 group of the dX GEMM's K --
// plus the scale byte in the atom.
__device__ __forceinline__ void dact_grad(float dap, float gt, float up, float sc, float& a, float& dg, float& du) {
  const float sig = __fdividef(1.0f, 1.0f + __expf(-gt));
  const float silu = gt * sig;
  a = silu * up;
  const float da = sc * dap;
  dg = da * up * sig * (1.0f + gt * (1.0f - sig));
  du = da * silu;
}

__device__ __forceinline__ void dact_tile(const GemmArgs& g, const uint32_t (&v)[64], const RowMeta& m, int cc) {
  if (!m.valid) return;
  const int I = g.N;
  const int i0 = m.nt * kBN + 64 * cc;
  const uint4* hrow = reinterpret_cast<const uint4*>(g.h_in + static_cast<size_t>(m.tok) * (2 * I) + 2 * i0);
  const float sc = m.sc;
  const size_t p = static_cast<size_t>(m.p);
  uint4* adst = reinterpret_cast<uint4*>(g.a_prime + p * I + i0);
  uint4* hdst = reinterpret_cast<uint4*>(g.dh_bf16 + p * (2 * I) + 2 * i0);
  // Pass 1, eight columns at a time: dS, a', and dH as bf16 pairs (dg, du) with the amax of those
  // bf16 values -- the row's 128 dH values are one 1x128 group.  Pass 2 recomputes dH from h (an L2
  // hit; the registers hold one pass at a time, the accumulator is already released) and
  // quantises its bf16 rounding, so the e4m3 copy is the bf16 dH quantised.
  float ds = 0.0f, am = 0.0f;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 h0 = hrow[2 * c], h1 = hrow[2 * c + 1];
    const uint32_t w[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    uint32_t ap[4], dh[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float dap = __uint_as_float(v[8 * c + k]);
      float a, dg, du;
      dact_grad(dap, __uint_as_float(w[k] << 16), __uint_as_float(w[k] & 0xFFFF0000u), sc, a, dg, du);
      ds = fmaf(dap, a, ds);
      dh[k] = pack_bf16x2(dg, du);
      am = fmaxf(am, fmaxf(fabsf(__uint_as_float(dh[k] << 16)), fabsf(__uint_as_float(dh[k] & 0xFFFF0000u))));
      if (k & 1) ap[k >> 1] = pack_bf16x2(__uint_as_float(ap[k >> 1]), sc * a);
      else ap[k >> 1] = __float_as_uint(sc * a);
    }
    adst[c] = make_uint4(ap[0], ap[1], ap[2], ap[3]);
    hdst[2 * c] = make_uint4(dh[0], dh[1], dh[2], dh[3]);
    hdst[2 * c + 1] = make_uint4(dh[4], dh[5], dh[6], dh[7]);
  }
  atomicAdd(g.ds + g.s_scatter[m.tok], ds);
  if (g.out_q == nullptr) return;  // the e4m3 copy is made from dh_bf16 by the dual operand pack
  const int e8 = scale_exp_of_amax(am);
  const float inv = exp2_neg(e8);
  uint4* qdst = reinterpret_cast<uint4*>(g.out_q + p * (2 * I) + 2 * i0);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 h0 = hrow[2 * c], h1 = hrow[2 * c + 1];
    const uint32_t w[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    uint32_t q[4];
#pragma unroll
    for (int k = 0; k < 8; k += 2) {
      float a0, dg0, du0, a1, dg1, du1;
      dact_grad(__uint_as_float(v[8 * c + k]), __uint_as_float(w[k] << 16), __uint_as_float(w[k] & 0xFFFF0000u), sc,
                a0, dg0, du0);
      dact_grad(__uint_as_float(v[8 * c + k + 1]), __uint_as_float(w[k + 1] << 16),
                __uint_as_float(w[k + 1] & 0xFFFF0000u), sc, a1, dg1, du1);
      const uint32_t d0 = pack_bf16x2(dg0, du0), d1 = pack_bf16x2(dg1, du1);
      q[k >> 1] = static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(__uint_as_float(d0 << 16), inv),
                                                   __fmul_rn(__uint_as_float(d0 & 0xFFFF0000u), inv))) |
                  (static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(__uint_as_float(d1 << 16), inv),
                                                    __fmul_rn(__uint_as_float(d1 & 0xFFFF0000u), inv)))
                   << 16);
    }
    qdst[c] = make_uint4(q[0], q[1], q[2], q[3]);
  }
  // K block (2 i0) / 128 = 4 nt + cc of the dX GEMM; atoms hold 4 consecutive K blocks
  const int KG2 = (2 * I / kBlockK + 3) / 4;
  const int kb2 = 4 * m.nt + cc;
  const int rr = m.p % kBlockM;
  g.out_sf[(static_cast<size_t>(m.mb) * KG2 + kb2 / 4) * kSfAtomBytes + 16 * (rr % 32) + 4 * (rr / 32) + (kb2 % 4)] =
      static_cast<uint8_t>(e8 + 127);
}

// Concatenated w1 ([gate | up] rows): h holds g at column i and u at I + i.  dH goes out as bf16 in
// that order (the dW1 operand, so dW1 keeps the caller's layout) and as e4m3 in the forward
// weight's re-blocked order -- column 256 j + c holds gate 128 j + c for c < 128, up 128 j + c - 128
// -- the K order of W1^T transposed from the prepared (re-blocked) W1.  The thread's 64 gate values
// are half of one 1x128 group and its 64 up values half of the next; the other halves belong to
// column warp cc ^ 1 of the same rows, so the group maxima are exchanged through shared memory
// (every epilogue warp arrives once per tile; rows without an entry contribute zeros).
__device__ __forceinline__ bool dact_tile_concat(const GemmArgs& g, const uint32_t (&v)[64], const RowMeta& m, int cc,
                                                 int lane, int tcount, float* s_amax, uint64_t* amax_bar) {
  const int I = g.N;
  const int i0 = m.nt * kBN + 64 * cc;
  const int r = m.p % kBlockM;
  const bool valid = m.valid != 0;
  const float sc = m.sc;
  const size_t p = static_cast<size_t>(m.p);
  const __nv_bfloat16* hrow = g.h_in + static_cast<size_t>(valid ? m.tok : 0) * (2 * I);
  const uint4* hg = reinterpret_cast<const uint4*>(hrow + i0);
  const uint4* hu = reinterpret_cast<const uint4*>(hrow + I + i0);
  float amg = 0.0f, amu = 0.0f;
  // dH as bf16 pairs; the e4m3 copy quantises these bf16 values, recomputed after the maxima
  // exchange (as in dact_tile)
  if (valid) {
    uint4* adst = reinterpret_cast<uint4*>(g.a_prime + p * I + i0);
    uint4* gdst = reinterpret_cast<uint4*>(g.dh_bf16 + p * (2 * I) + i0);
    uint4* udst = reinterpret_cast<uint4*>(g.dh_bf16 + p * (2 * I) + I + i0);
    float ds = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 g4 = hg[c], u4 = hu[c];
      const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w}, uw[4] = {u4.x, u4.y, u4.z, u4.w};
      uint32_t ap[4], dgp[4], dup[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float d0 = __uint_as_float(v[8 * c + 2 * k]), d1 = __uint_as_float(v[8 * c + 2 * k + 1]);
        float a0, dg0, du0, a1, dg1, du1;
        dact_grad(d0, __uint_as_float(gw[k] << 16), __uint_as_float(uw[k] << 16), sc, a0, dg0, du0);
        dact_grad(d1, __uint_as_float(gw[k] & 0xFFFF0000u), __uint_as_float(uw[k] & 0xFFFF0000u), sc, a1, dg1, du1);
        ds = fmaf(d1, a1, fmaf(d0, a0, ds));
        const uint32_t pg = pack_bf16x2(dg0, dg1), pu = pack_bf16x2(du0, du1);
        dgp[k] = pg;
        dup[k] = pu;
        amg = fmaxf(amg, fmaxf(fabsf(__uint_as_float(pg << 16)), fabsf(__uint_as_float(pg & 0xFFFF0000u))));
        amu = fmaxf(amu, fmaxf(fabsf(__uint_as_float(pu << 16)), fabsf(__uint_as_float(pu & 0xFFFF0000u))));
        ap[k] = pack_bf16x2(sc * a0, sc * a1);
      }
      adst[c] = make_uint4(ap[0], ap[1], ap[2], ap[3]);
      gdst[c] = make_uint4(dgp[0], dgp[1], dgp[2], dgp[3]);
      udst[c] = make_uint4(dup[0], dup[1], dup[2], dup[3]);
    }
    atomicAdd(g.ds + g.s_scatter[m.tok], ds);
  }
  if (g.out_q == nullptr) return true;  // no e4m3 copy here: no maxima to exchange (uniform over the CTA)
  float* buf = s_amax + (tcount & 1) * (2 * 4 * kBlockM);
  buf[cc * kBlockM + r] = amg;
  buf[(4 + cc) * kBlockM + r] = amu;
  __syncwarp();
  if (lane == 0) mbar_arrive(amax_bar);
  if (!mbar_wait(amax_bar, tcount & 1, g.err, kErrTimeoutEpilogue)) return false;
  if (!valid) return true;
  amg = fmaxf(amg, buf[(cc ^ 1) * kBlockM + r]);
  amu = fmaxf(amu, buf[(4 + (cc ^ 1)) * kBlockM + r]);
  const int eg = scale_exp_of_amax(amg), eu = scale_exp_of_amax(amu);
  const float ig = exp2_neg(eg), iu = exp2_neg(eu);
  const int j = i0 / kBlockK, c0 = i0 % kBlockK;
  uint4* gq = reinterpret_cast<uint4*>(g.out_q + p * (2 * I) + 256 * j + c0);
  uint4* uq = reinterpret_cast<uint4*>(g.out_q + p * (2 * I) + 256 * j + 128 + c0);
  auto q2 = [](uint32_t wd, float inv) {
    return cvt_e4m3x2(__fmul_rn(__uint_as_float(wd << 16), inv), __fmul_rn(__uint_as_float(wd & 0xFFFF0000u), inv));
  };
#pragma unroll
  for (int c2 = 0; c2 < 4; ++c2) {
    uint32_t wg[4], wu[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = 2 * c2 + h;
      const uint4 g4 = hg[c], u4 = hu[c];
      const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w}, uw[4] = {u4.x, u4.y, u4.z, u4.w};
      uint32_t dgw[4], duw[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float a0, dg0, du0, a1, dg1, du1;
        dact_grad(__uint_as_float(v[8 * c + 2 * k]), __uint_as_float(gw[k] << 16), __uint_as_float(uw[k] << 16), sc,
                  a0, dg0, du0);
        dact_grad(__uint_as_float(v[8 * c + 2 * k + 1]), __uint_as_float(gw[k] & 0xFFFF0000u),
                  __uint_as_float(uw[k] & 0xFFFF0000u), sc, a1, dg1, du1);
        dgw[k] = pack_bf16x2(dg0, dg1);
        duw[k] = pack_bf16x2(du0, du1);
      }
      wg[2 * h] = static_cast<uint32_t>(q2(dgw[0], ig)) | (static_cast<uint32_t>(q2(dgw[1], ig)) << 16);
      wg[2 * h + 1] = static_cast<uint32_t>(q2(dgw[2], ig)) | (static_cast<uint32_t>(q2(dgw[3], ig)) << 16);
      wu[2 * h] = static_cast<uint32_t>(q2(duw[0], iu)) | (static_cast<uint32_t>(q2(duw[1], iu)) << 16);
      wu[2 * h + 1] = static_cast<uint32_t>(q2(duw[2], iu)) | (static_cast<uint32_t>(q2(duw[3], iu)) << 16);
    }
    gq[c2] = make_uint4(wg[0], wg[1], wg[2], wg[3]);
    uq[c2] = make_uint4(wu[0], wu[1], wu[2], wu[3]);
  }
  if (c0 == 0) {
    // K blocks 2 j (gate) and 2 j + 1 (up) of the dX GEMM; atoms hold 4 consecutive K blocks
    const int KG2 = (2 * I / kBlockK + 3) / 4;
    const size_t base = static_cast<size_t>(m.mb) * KG2 * kSfAtomBytes + 16 * (r % 32) + 4 * (r / 32);
    g.out_sf[base + static_cast<size_t>((2 * j) / 4) * kSfAtomBytes + ((2 * j) % 4)] = static_cast<uint8_t>(eg + 127);
    g.out_sf[base + static_cast<size_t>((2 * j + 1) / 4) * kSfAtomBytes + ((2 * j + 1) % 4)] =
        static_cast<uint8_t>(eu + 127);
  }
  return true;
}

// Epilogue of one accumulator tile: this thread holds row r (0..127) of the tile's 128-row block,
// output columns [64 cc, 64 cc + 64) of its n-tile in v (f32 bits).  Returns false if a bounded
// wait gave up.
//   up   : a = silu(gate) * up over the thread's 32 SwiGLU outputs, the row's amax over the 128
//          outputs of the tile (four threads, exchanged through shared memory), 1x128 requant.
//   down : scale by the entry's router score, stage 128 bytes of bf16 in this thread's slot and
//          bulk-reduce them into the token's output row.
template <int kKind>
__device__ __forceinline__ bool epilogue_tile(const GemmArgs& g, const uint32_t (&v)[64], const RowMeta& m, int r,
                                              int cc, int ew, int lane, int tcount, float* s_amax, uint64_t* amax_bar,
                                              uint64_t* store_bar, uint8_t* sStage, const CUtensorMap* tmap_out,
                                              uint64_t pol_out) {
  constexpr bool kUp = kKind == kKindUp;
  const bool valid = m.valid != 0;
  const int p = m.p, mb = m.mb, nt = m.nt;
  if constexpr (kKind == kKindDact) {
    if (g.concat) return dact_tile_concat(g, v, m, cc, lane, tcount, s_amax, amax_bar);
    dact_tile(g, v, m, cc);
  } else if constexpr (kUp) {
    if (g.preact != nullptr && valid) {
      // training forward: h as bf16 in the caller's w1 column order (interleaved: this thread's 64
      // tile columns are consecutive; concatenated: 32 gate columns and the matching 32 up columns)
      __nv_bfloat16* hrow = g.preact + static_cast<size_t>(m.tok) * g.N;
      auto put32 = [&](__nv_bfloat16* dst, const uint32_t* src) {
#pragma unroll
        for (int j = 0; j < 32; j += 8)
          *reinterpret_cast<uint4*>(dst + j) =
              make_uint4(pack_bf16x2(__uint_as_float(src[j]), __uint_as_float(src[j + 1])),
                         pack_bf16x2(__uint_as_float(src[j + 2]), __uint_as_float(src[j + 3])),
                         pack_bf16x2(__uint_as_float(src[j + 4]), __uint_as_float(src[j + 5])),
                         pack_bf16x2(__uint_as_float(src[j + 6]), __uint_as_float(src[j + 7])));
      };
      if (g.concat) {
        put32(hrow + nt * 128 + 32 * cc, v);
        put32(hrow + g.N / 2 + nt * 128 + 32 * cc, v + 32);
      } else {
        put32(hrow + nt * kBN + 64 * cc, v);
        put32(hrow + nt * kBN + 64 * cc + 32, v + 32);
      }
    }
    float o[32];
    float am = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float gt = __uint_as_float(g.concat ? v[j] : v[2 * j]);
      const float up = __uint_as_float(g.concat ? v[32 + j] : v[2 * j + 1]);
      o[j] = valid ? silu_f(gt) * up : 0.0f;
      am = fmaxf(am, fabsf(o[j]));
    }
    float* amax_buf = s_amax + (tcount & 1) * (4 * kBlockM);
    amax_buf[cc * kBlockM + r] = am;
    // the store issuer first makes sure the previous tile's TMA store has read the staging tile;
    // nobody writes the staging tile before this barrier completes
    if (ew == 0 && lane == 0) bulk_wait_read0();
    __syncwarp();
    if (lane == 0) mbar_arrive(amax_bar);
    if (!mbar_wait(amax_bar, tcount & 1, g.err, kErrTimeoutEpilogue)) return false;
    am = fmaxf(fmaxf(amax_buf[r], amax_buf[kBlockM + r]), fmaxf(amax_buf[2 * kBlockM + r], amax_buf[3 * kBlockM + r]));
    const int e8 = scale_exp_of_amax(am);
    const float inv = exp2_neg(e8);
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      w[i] = static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(o[4 * i], inv), __fmul_rn(o[4 * i + 1], inv))) |
             (static_cast<uint32_t>(cvt_e4m3x2(__fmul_rn(o[4 * i + 2], inv), __fmul_rn(o[4 * i + 3], inv))) << 16);
    }
    const int I2 = g.N / 2;
    if (g.ret_dst != nullptr) {
      // expert parallel: the thread's 32 bytes of the row (and, from the first column warp, the
      // row's scale byte) go straight to the token's home rank -- plain 16-byte peer stores, no
      // staging tile; the home's down projection reads them after a cross-rank barrier
      if (valid) {
        const int dst = m.tok;
        const int home = dst >> kHomeShift;
        const long long ph = dst & ((1 << kHomeShift) - 1);
        if (dst < 0 || home >= g.n_homes || ph >= g.home_rows) {
          atomicCAS(g.err, 0, kErrBadReturnRow);
        } else {
          uint8_t* drow = g.home_q[home] + ph * I2 + nt * 128 + cc * 32;
          *reinterpret_cast<uint4*>(drow) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4*>(drow + 16) = make_uint4(w[4], w[5], w[6], w[7]);
          if (cc == 0) {
            const long long KG2 = (I2 / kBlockK + 3) / 4;
            const int rr = static_cast<int>(ph % kBlockM);
            g.home_sf[home][((ph / kBlockM) * KG2 + nt / 4) * kSfAtomBytes + 16 * (rr % 32) + 4 * (rr / 32) +
                            (nt % 4)] = static_cast<uint8_t>(e8 + 127);
          }
        }
      }
      return true;
    }
    // row r of the staging tile, 16-byte chunks 2cc and 2cc+1 at their 128B-swizzled positions
    uint8_t* srow = sStage + r * 128;
    *reinterpret_cast<uint4*>(srow + (((2 * cc) ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4*>(srow + (((2 * cc + 1) ^ (r & 7)) << 4)) = make_uint4(w[4], w[5], w[6], w[7]);
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(store_bar);
    if (ew == 0 && lane == 0) {
      if (!mbar_wait(store_bar, tcount & 1, g.err, kErrTimeoutEpilogue)) return false;
      tma_store_2d(tmap_out, sStage, nt * kBlockM, mb * kBlockM);
      bulk_commit();
    }
    if (cc == 0) {
      const int KG2 = (I2 / kBlockK + 3) / 4;
      g.out_sf[(static_cast<size_t>(mb) * KG2 + nt / 4) * kSfAtomBytes + 16 * (r % 32) + 4 * (r / 32) + (nt % 4)] =
          static_cast<uint8_t>(e8 + 127);
    }
  } else {
    // The slot is reused only after the previous bulk reduction has finished reading it.
    uint8_t* slot = sStage + (ew * 32 + lane) * kSlotStride;
    bulk_wait_read0();
    if (valid) {
      const float sc = m.sc;
#pragma unroll
      for (int j = 0; j < 64; j += 8) {
        uint4 w;
        w.x = pack_bf16x2(sc * __uint_as_float(v[j]), sc * __uint_as_float(v[j + 1]));
        w.y = pack_bf16x2(sc * __uint_as_float(v[j + 2]), sc * __uint_as_float(v[j + 3]));
        w.z = pack_bf16x2(sc * __uint_as_float(v[j + 4]), sc * __uint_as_float(v[j + 5]));
        w.w = pack_bf16x2(sc * __uint_as_float(v[j + 6]), sc * __uint_as_float(v[j + 7]));
        *reinterpret_cast<uint4*>(slot + 2 * j) = w;
      }
      fence_proxy_async_smem();
      __nv_bfloat16* dst =
          static_cast<__nv_bfloat16*>(g.out_bf16) + static_cast<size_t>(m.tok) * g.N + nt * kBN + cc * 64;
      bulk_reduce_add_bf16(dst, slot, kRowChunkBytes, pol_out);
      bulk_commit();
    }
  }
  return true;
}

// Tile t of the schedule: A row block (m-block of the padded layout, or m-tile of the weight-gradient
// output), n-tile, expert, first K block and number of K blocks.
struct TileInfo {
  int mb, nt, e, kb0, nkb;
};
template <int kKind>
__device__ __forceinline__ TileInfo tile_info(const GemmArgs& g, int tile, int n_blocks, int ntn, int KB) {
  TileInfo ti;
  if constexpr (kKind == kKindWgrad) {
    const int mt_n = g.a_rows / kBlockM;
    const int per_e = mt_n * ntn;
    ti.e = tile / per_e;
    const int rem = tile - ti.e * per_e;
    ti.mb = rem / ntn;
    ti.nt = rem - ti.mb * ntn;
    const int p0 = g.off_pad[ti.e];
    ti.kb0 = p0 / kBlockK;
    ti.nkb = (g.off_pad[ti.e + 1] - p0) / kBlockK;
  } else {
    tile_coords(tile, n_blocks, ntn, g.n_slices, ti.mb, ti.nt);
    ti.e = g.blk_expert[ti.mb];
    ti.kb0 = 0;
    ti.nkb = KB;
  }
  return ti;
}

template <int kKind>
__global__ void __launch_bounds__(kGemmThreads, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                    const __grid_constant__ CUtensorMap tmap_out, const GemmArgs g) {
  constexpr bool kUp = kKind == kKindUp;
  constexpr bool kWgrad = kKind == kKindWgrad;
  using L = GemmSmem<kKind>;
  constexpr int kStages = L::kStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint8_t* sA = smem + L::kOffA;
  uint8_t* sB = smem + L::kOffB;
  uint8_t* sSfa = smem + L::kOffSfa;
  uint8_t* sSfb = smem + L::kOffSfb;
  uint8_t* sStage = smem + L::kOffStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* tmem_full = bars + 2 * kStages;
  uint64_t* tmem_empty = tmem_full + 1;
  uint64_t* drain = tmem_full + 2;
  uint64_t* amax_bar = tmem_full + 3;   // up: every epilogue warp has written its row amax partials
  uint64_t* store_bar = tmem_full + 4;  // up: every epilogue warp has written its part of the output tile
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::kOffTmemHolder);
  float* s_amax = reinterpret_cast<float*>(smem + L::kOffAmax);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tmem_full, 1);
    mbar_init(tmem_empty, kEpiWarps);
    mbar_init(drain, 1);
    mbar_init(amax_bar, kEpiWarps);
    mbar_init(store_bar, kEpiWarps);
    fence_mbar_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
    if (kUp) prefetch_tmap(&tmap_out);
  }
  if (warp == 2) {
    tmem_alloc(tmem_holder, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  const int n_blocks = kWgrad ? 0 : *g.n_blocks;
  const int ntn = g.N / kBN;
  const int total = kWgrad ? g.E * static_cast<int>(g.a_rows / kBlockM) * ntn : n_blocks * ntn;
  const int KB = g.Kd / kBlockK;
  const int KG = (KB + 3) / 4;
  const int nbk = g.N / kBlockM;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ TMA producer
      // up: each A block is read by the 8 n-tiles running side by side, keep it; down: A streams
      // through once per column slice (evict_last measured ~1% faster for up, no gain for down)
      const uint64_t pol_a = kKind == kKindDown ? policy_evict_first() : policy_evict_last();
      const uint64_t pol_b = policy_evict_last();
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const TileInfo ti = tile_info<kKind>(g, tile, n_blocks, ntn, KB);
        if (ti.nkb == 0) continue;  // weight gradient of an expert without rows (output pre-zeroed)
        const int a_row = ti.mb * kBlockM;
        // B rows: expert e's N rows; the weight gradient's B has one set of rows for all experts
        const int b_row = (kWgrad ? 0 : ti.e * g.N) + ti.nt * kBN;
        for (int kb = 0; kb < ti.nkb; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, g.err, kErrTimeoutProducer)) {
            ok = false;
            break;
          }
          const int kg = ti.kb0 + kb;  // K block in the operands
          // scale atoms cover 4 K blocks; a weight-gradient tile may start in the middle of one
          const bool sf = (kg & 3) == 0 || kb == 0;
          mbar_arrive_expect_tx(&full[s], kABytes + kBBytes + (sf ? kSfaBytes + kSfbBytes : 0));
          tma_load_2d(sA + s * kABytes, &tmap_a, &full[s], kg * kBlockK, a_row, pol_a);
          tma_load_2d(sB + s * kBBytes, &tmap_b, &full[s], kg * kBlockK, b_row, pol_b);
          if (sf) {
            bulk_load(sSfa + s * kSfaBytes, g.a_sf + (static_cast<size_t>(ti.mb) * KG + kg / 4) * kSfAtomBytes,
                      kSfAtomBytes, &full[s]);
            const size_t nb0 = static_cast<size_t>(kWgrad ? 0 : ti.e) * nbk + static_cast<size_t>(ti.nt) * 2;
            bulk_load(sSfb + s * kSfbBytes, g.b_sf + (nb0 * KG + kg / 4) * kSfAtomBytes, kSfAtomBytes, &full[s]);
            bulk_load(sSfb + s * kSfbBytes + kSfAtomBytes, g.b_sf + ((nb0 + 1) * KG + kg / 4) * kSfAtomBytes,
                      kSfAtomBytes, &full[s]);
          }
        }
      }
      if (!ok) {
        // an error elsewhere: let the loads already issued land before shared memory goes away
        const int first = it - kStages > 0 ? it - kStages : 0;
        for (int j = first; j < it; ++j) mbar_wait_ns(&full[j % kStages], (j / kStages) & 1, 50000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA issuer
      const uint32_t idesc0 = idesc_mxf8_e4m3(kBlockM, kBN, 0, 0);
      int it = 0, tcount = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total && ok; tile += gridDim.x) {
        const TileInfo ti = tile_info<kKind>(g, tile, n_blocks, ntn, KB);
        if (ti.nkb == 0) continue;
        if (!mbar_wait(tmem_empty, (tcount & 1) ^ 1, g.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        ++tcount;
        tc_fence_after();
        for (int kb = 0; kb < ti.nkb; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!mbar_wait(&full[s], ph, g.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int kg = ti.kb0 + kb;
          const uint32_t id = static_cast<uint32_t>(kg & 3);
          if (id == 0 || kb == 0) {
            tc_cp_sf(tmem + kTmemSfa, sdesc_sf(smem_u32(sSfa + s * kSfaBytes)));
            tc_cp_sf(tmem + kTmemSfb, sdesc_sf(smem_u32(sSfb + s * kSfbBytes)));
            tc_cp_sf(tmem + kTmemSfb + 4, sdesc_sf(smem_u32(sSfb + s * kSfbBytes + kSfAtomBytes)));
          }
          const uint64_t ad = sdesc_sw128(smem_u32(sA + s * kABytes));
          const uint64_t bd = sdesc_sw128(smem_u32(sB + s * kBBytes));
          const uint32_t idesc = idesc0 | (id << 4) | (id << 29);
#pragma unroll
          for (int kk = 0; kk < kBlockK / 32; ++kk) {
            // +32 bytes along K inside the 128-byte swizzle row = +2 in the 16-byte address field
            tc_mma_mxf8(tmem + kTmemAcc, ad + 2 * kk, bd + 2 * kk, idesc, (tmem + kTmemSfa) | (id << 30),
                        (tmem + kTmemSfb) | (id << 30), (kb | kk) != 0 ? 1u : 0u);
          }
          tc_commit(&empty[s]);
        }
        if (!ok) break;
        tc_commit(tmem_full);
      }
      // every MMA issued by this thread has finished once `drain` completes
      tc_commit(drain);
      mbar_wait_ns(drain, 0, 100000000ull);
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------------- epilogue
    const int ew = warp - 4;
    const int q = warp & 3;
    const int cc = ew >> 2;
    const int r = q * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    int tcount = 0;
    const uint64_t pol_out = policy_evict_last();
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
      TileInfo ti{};
      if constexpr (kWgrad) {
        ti = tile_info<kKind>(g, tile, n_blocks, ntn, KB);
        if (ti.nkb == 0) continue;
      }
      RowMeta pre{};
      if constexpr (kKind == kKindDact) {
        // the row's metadata, and its stored pre-activation prefetched into L2, while the tile's
        // main loop runs (the epilogue is bound by the latency of these loads)
        pre = load_row_meta<kKind>(g, tile, n_blocks, ntn, r);
        if (pre.valid) {
          const int i0 = pre.nt * kBN + 64 * cc;
          const __nv_bfloat16* hrow = g.h_in + static_cast<size_t>(pre.tok) * (2 * g.N);
          prefetch_l2(g.concat ? hrow + i0 : hrow + 2 * i0);
          prefetch_l2(g.concat ? hrow + g.N + i0 : hrow + 2 * i0 + 64);
        }
      }
      if (!mbar_wait(tmem_full, tcount & 1, g.err, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      uint32_t v[64];
      if (kUp && g.concat) {
        tmem_ld32(lane_base + kTmemAcc + 32 * cc, v);
        tmem_ld32(lane_base + kTmemAcc + 128 + 32 * cc, v + 32);
      } else {
        tmem_ld32(lane_base + kTmemAcc + 64 * cc, v);
        tmem_ld32(lane_base + kTmemAcc + 64 * cc + 32, v + 32);
      }
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tmem_empty);

      if constexpr (kWgrad) {
        // D[e] rows 128 mt + r, columns 256 nt + 64 cc .. + 63, as bf16: staged in this thread's slot
        // and written by one bulk copy (a warp's direct row stores would touch 32 lines each); the
        // slot is rewritten once the previous tile's copy has read it
        __nv_bfloat16* dst = g.out_w + (static_cast<size_t>(ti.e) * g.a_rows + ti.mb * kBlockM + r) * g.N +
                             ti.nt * kBN + 64 * cc;
        uint8_t* slot = sStage + (ew * 32 + lane) * kSlotStride;
        bulk_wait_read0();
#pragma unroll
        for (int j = 0; j < 64; j += 8)
          *reinterpret_cast<uint4*>(slot + 2 * j) =
              make_uint4(pack_bf16x2(__uint_as_float(v[j]), __uint_as_float(v[j + 1])),
                         pack_bf16x2(__uint_as_float(v[j + 2]), __uint_as_float(v[j + 3])),
                         pack_bf16x2(__uint_as_float(v[j + 4]), __uint_as_float(v[j + 5])),
                         pack_bf16x2(__uint_as_float(v[j + 6]), __uint_as_float(v[j + 7])));
        fence_proxy_async_smem();
        bulk_store(dst, slot, kRowChunkBytes);
        bulk_commit();
        ++tcount;
        continue;
      } else {
        // the accumulator is released: the row's metadata loads overlap the next tile's main loop
        const RowMeta meta = kKind == kKindDact ? pre : load_row_meta<kKind>(g, tile, n_blocks, ntn, r);
        const bool ok_tile = epilogue_tile<kKind>(g, v, meta, r, cc, ew, lane, tcount, s_amax, amax_bar, store_bar,
                                                  sStage, &tmap_out, pol_out);
        ++tcount;
        if (!ok_tile) break;
      }
    }
    // rows stored into other GPUs' memory are performed system-wide before the kernel completes
    if (kUp && g.ret_dst != nullptr) __threadfence_system();
    bulk_wait_all();  // outstanding reductions / output stores have finished with shared memory
  }
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------------------------
// host side: tensor maps and launch
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D e4m3 (byte) tensor [rows, cols] row-major; box = box_rows x 128 bytes with the 128B swizzle.
static bool make_tmap(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBlockK), box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, int esize, const void* base, uint64_t inner,
                    uint64_t outer, uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * static_cast<uint64_t>(esize)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Column slices of the down projection: the largest slice whose bf16 output slab (tokens x slice
// columns) fits an 80 MB share of the L2, so the reductions of one slice land in L2 (swept
// 300/160/80/40/20 MB at config 2: 80 best).  Every slice re-reads all of A, so at most 4 slices:
// measured best both for the 268 MB token output of config 2 (4 slices of 67 MB) and for the ~1 GB
// of partial rows an expert-parallel rank reduces into at 4 GPUs (4 slices beat 16).
int down_slices(long long tokens, int N) {
  constexpr long long kSlabBudget = 80ll << 20;
  const int ntn = N / kBN;
  int slices = 1;
  while (slices < ntn && slices < 4 && tokens * (N / slices) * 2 > kSlabBudget && ntn % (slices * 2) == 0)
    slices *= 2;
  return slices;
}

template <int kKind>
static cudaError_t launch_gemm(const GemmArgs& g, cudaStream_t st) {
  constexpr bool kUp = kKind == kKindUp;
  const long long max_blocks = g.a_rows / kBlockM;
  const long long max_tiles = max_blocks * (g.N / kBN) * (kKind == kKindWgrad ? g.E : 1);
  if (max_tiles == 0) return cudaSuccess;
  CUtensorMap ta, tb;
  if (!make_tmap(&ta, g.a, static_cast<uint64_t>(g.a_rows), static_cast<uint64_t>(g.Kd), kBlockM)) return cudaErrorInvalidValue;
  const uint64_t b_rows = static_cast<uint64_t>(kKind == kKindWgrad ? 1 : g.E) * g.N;
  if (!make_tmap(&tb, g.b, b_rows, static_cast<uint64_t>(g.Kd), kBN)) return cudaErrorInvalidValue;
  CUtensorMap to = ta;  // the down projection and the expert-parallel up projection have no tiled output
  if (kUp && g.ret_dst == nullptr &&
      !make_tmap(&to, g.out_q, static_cast<uint64_t>(g.a_rows), static_cast<uint64_t>(g.N / 2), kBlockM))
    return cudaErrorInvalidValue;
  if (kUp && g.ret_dst != nullptr && (g.n_homes < 1 || g.n_homes > kMaxEpRanks || g.home_rows < 0))
    return cudaErrorInvalidValue;
  auto kern = moe_gemm_kernel<kKind>;
  constexpr int kSmemAlloc = GemmSmem<kKind>::kAlloc;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc);
  if (e != cudaSuccess) return e;
  const int grid = static_cast<int>(max_tiles < g.num_sms ? max_tiles : g.num_sms);
  GemmArgs ga = g;
  ga.n_slices = 1;
  if (kKind == kKindDown) ga.n_slices = down_slices(g.tokens, g.N);
  kern<<<grid, kGemmThreads, kSmemAlloc, st>>>(ta, tb, to, ga);
  return cudaGetLastError();
}

static int g_sm_reserve = 0;

int gemm_grid_sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (n <= 0) n = 148;
  const int r = g_sm_reserve < n ? g_sm_reserve : n - 1;
  return n - (r > 0 ? r : 0);
}

cudaError_t launch_moe_up(const GemmArgs& g, cudaStream_t st) { return launch_gemm<kKindUp>(g, st); }
cudaError_t launch_moe_down(const GemmArgs& g, cudaStream_t st) { return launch_gemm<kKindDown>(g, st); }
cudaError_t launch_moe_dact(const GemmArgs& g, cudaStream_t st) { return launch_gemm<kKindDact>(g, st); }
cudaError_t launch_moe_wgrad(const GemmArgs& g, cudaStream_t st) { return launch_gemm<kKindWgrad>(g, st); }

}  // namespace smb

extern "C" int sm_set_gemm_sm_reserve(int n) {
  smb::g_sm_reserve = n < 0 ? 0 : n;
  return 0;
}
