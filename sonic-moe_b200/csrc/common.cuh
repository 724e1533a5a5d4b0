// Shared device helpers for the sm_100a kernels: mbarriers with bounded waits, TMA and bulk
// copies, tcgen05 (tensor memory, block-scaled MMA, smem->tmem copies, tmem->register loads),
// and the UE8M0 / e4m3 conversions of the quantiser spec.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace smb {

// --------------------------------------------------------------------------------------------
// error word written by kernels (0 = ok).  Codes identify the wait that gave up.
enum DevError : int {
  kErrNone = 0,
  kErrTimeoutProducer = 101,
  kErrTimeoutMma = 102,
  kErrTimeoutEpilogue = 103,
  kErrTimeoutDrain = 104,
  kErrSelfTestWait = 105,  // sm_selftest_bounded_wait: the expected give-up
  kErrBadExpert = 201,
  kErrBadReturnRow = 202,  // an up-projection row whose home rank / row lies outside the home buffers
  kErrBadCount = 203,  // expert parallel: an exchange count read on the device lies outside the buffers
};

// A single wait never legitimately lasts more than a few milliseconds; 2 s means a bug.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

// --------------------------------------------------------------------------------------------
// mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity.  Returns false (and records `where` in the
// global error word) after kWaitTimeoutNs, or as soon as another thread or CTA has recorded an
// error, so that every role of every CTA leaves its loops instead of spinning forever.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int where) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t n = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++n & 31u) == 0) {
      if (*reinterpret_cast<volatile int*>(err) != 0) return false;
      if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
        atomicCAS(err, 0, where);
        return false;
      }
    }
  }
}

// Wait with a short explicit limit (teardown after an error).
__device__ __forceinline__ bool mbar_wait_ns(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
  return true;
}

// --------------------------------------------------------------------------------------------
// TMA (tiled, one destination CTA) and bulk copies, completing on an mbarrier
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}
// Tiled store shared -> global (bulk async-group of the issuing thread; coordinates >= 0).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Bulk (TMA) reduction of `bytes` contiguous bf16 values from shared memory into global memory,
// tracked by the issuing thread's bulk async-group.
__device__ __forceinline__ void bulk_reduce_add_bf16(void* gdst, const void* ssrc, uint32_t bytes, uint64_t policy) {
  asm volatile(
      "cp.reduce.async.bulk.global.shared::cta.bulk_group.L2::cache_hint.add.noftz.bf16 [%0], [%1], %2, %3;" ::"l"(
          gdst),
      "r"(smem_u32(ssrc)), "r"(bytes), "l"(policy)
      : "memory");
}
// Bulk (TMA) copy of `bytes` contiguous bytes from shared to global memory (16-byte aligned, size a
// multiple of 16), tracked by the issuing thread's bulk async-group.
__device__ __forceinline__ void bulk_store(void* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(ssrc)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// every bulk operation committed by this thread has finished reading its shared-memory source
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// every bulk operation committed by this thread has completed
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// make this thread's generic-proxy shared-memory writes visible to the async (TMA) proxy
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// --------------------------------------------------------------------------------------------
// tcgen05: tensor memory, block-scaled MMA, copies
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrive (once) on `bar` when every tcgen05 op issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// D[tmem] (+)= (A[smem] * sfA) x (B[smem] * sfB)^T, e4m3 operands, UE8M0 scale factors in tmem.
__device__ __forceinline__ void tc_mma_mxf8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// 32 rows x 16 bytes from smem into 4 tmem columns of all four 32-lane sub-partitions.
__device__ __forceinline__ void tc_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives lane (base_lane + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Shared-memory matrix descriptor, K-major operand stored by TMA with the 128-byte swizzle:
// rows of 128 bytes, 8-row groups 1024 bytes apart (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;            // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;    // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;            // version
  d |= static_cast<uint64_t>(2) << 61;            // SWIZZLE_128B
  return d;
}
// Descriptor of a 32-row x 16-byte scale-factor atom (no swizzle, 8-row core matrices 128 B apart).
__device__ __forceinline__ uint64_t sdesc_sf(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(128 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  return d;
}
// Instruction descriptor, kind::mxf8f6f4 with block scaling: e4m3 x e4m3 -> f32, K-major A and B,
// UE8M0 scale factors, scale-factor ids select the byte of the 32-bit tmem word.
__host__ __device__ constexpr uint32_t idesc_mxf8_e4m3(int M, int N, uint32_t sfa_id, uint32_t sfb_id) {
  return (sfb_id << 4) | (0u << 7) | (0u << 10) | (static_cast<uint32_t>(N >> 3) << 17) | (1u << 23) |
         (static_cast<uint32_t>(M >> 4) << 24) | (sfa_id << 29);
}

// two floats -> packed bf16x2 (round to nearest even), low half = a
__device__ __forceinline__ uint32_t pack_bf16x2_rn(float a, float b) {
  __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&p);
}

// --------------------------------------------------------------------------------------------
// named barrier among a subset of warps
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// --------------------------------------------------------------------------------------------
// Quantiser spec helpers (match oracle/quant.py bit for bit)

// Exact ceil(log2(s)) for s >= 0 (s == 0 -> -127), clamped to [-127, 127].
__device__ __forceinline__ int ceil_log2_f32(float s) {
  const uint32_t b = __float_as_uint(s);
  const int ex = static_cast<int>((b >> 23) & 0xFFu);
  const uint32_t man = b & 0x7FFFFFu;
  int e;
  if (ex > 0) {
    e = (man == 0) ? ex - 127 : ex - 126;
  } else if (man == 0) {
    e = -127;
  } else {
    e = (32 - __clz(man - 1)) - 149;  // ceil(log2(man)) - 149
  }
  return max(-127, min(127, e));
}
// UE8M0 exponent of the scale of a group with absolute maximum `amax`.
__device__ __forceinline__ int scale_exp_of_amax(float amax) { return ceil_log2_f32(__fdiv_rn(amax, 448.0f)); }
// 2^-e as float (e in [-127, 127]).
__device__ __forceinline__ float exp2_neg(int e) {
  const int ne = -e;  // in [-127, 127]
  if (ne >= -126) return __uint_as_float(static_cast<uint32_t>(ne + 127) << 23);
  return __uint_as_float(1u << 22);  // 2^-127 (subnormal)
}
// Two floats -> two e4m3 bytes (round to nearest even, saturating), packed low byte = a.
__device__ __forceinline__ uint16_t cvt_e4m3x2(float a, float b) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(r) : "f"(a), "f"(b));
  return r;
}

// A 128 x 128 byte tile in shared memory for a transposed store: row n at n * kTtStride bytes, its
// eight 16-byte chunks permuted (chunk k stored at k ^ ((n >> 4) & 7)), so that both the row-wise
// 16-byte writes that fill it and the column-wise word reads of store_tile_transposed_128 are free
// of bank conflicts.  tt_chunk: byte offset of chunk k of row n.
constexpr int kTtStride = 144;
__device__ __forceinline__ int tt_chunk(int n, int k) { return n * kTtStride + ((k ^ ((n >> 4) & 7)) << 4); }

// Transposed store of such a tile: byte (n, c) goes to dst[c * ld + n].  256 threads: warp w, lane l
// writes output rows 4 (4w + l / 8) .. + 3, bytes 16 (l % 8) .. + 15 -- it reads one 32-bit word of
// each of its 16 tile rows and transposes 4 x 4 byte blocks with byte permutes -- so each store
// instruction of a warp fills 4 whole 128-byte output lines.  dst and ld must keep the 16-byte
// stores aligned (ld % 16 == 0).
__device__ __forceinline__ void store_tile_transposed_128(const uint8_t* tile, uint8_t* dst, size_t ld, int tid) {
  const int lane = tid & 31, w = tid >> 5;
  const int c = lane & 7;                 // output bytes 16c .. 16c + 15 = tile rows 16c ..
  const int rq = 4 * w + (lane >> 3);     // output rows 4 rq .. 4 rq + 3 = tile bytes 4 rq ..
  uint32_t r[4][4];                       // [output row b][tile-row quad q]
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t x[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int n = 16 * c + 4 * q + t;
      x[t] = *reinterpret_cast<const uint32_t*>(tile + tt_chunk(n, rq >> 2) + 4 * (rq & 3));
    }
    const uint32_t t0 = __byte_perm(x[0], x[1], 0x5140), t1 = __byte_perm(x[2], x[3], 0x5140);
    const uint32_t t2 = __byte_perm(x[0], x[1], 0x7362), t3 = __byte_perm(x[2], x[3], 0x7362);
    r[0][q] = __byte_perm(t0, t1, 0x5410);
    r[1][q] = __byte_perm(t0, t1, 0x7632);
    r[2][q] = __byte_perm(t2, t3, 0x5410);
    r[3][q] = __byte_perm(t2, t3, 0x7632);
  }
  uint8_t* d = dst + static_cast<size_t>(4 * rq) * ld + 16 * c;
#pragma unroll
  for (int b = 0; b < 4; ++b)
    *reinterpret_cast<uint4*>(d + static_cast<size_t>(b) * ld) = make_uint4(r[b][0], r[b][1], r[b][2], r[b][3]);
}

}  // namespace smb
