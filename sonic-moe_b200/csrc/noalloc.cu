// Routing metadata without a caller-provided workspace (sm_route_metadata_noalloc).
//
// Some callers cannot allocate device memory at the point where they route tokens: a C or
// foreign-language host that records the MoE step into a CUDA graph cannot call cudaMalloc
// while the stream is being captured, and a serving process that reserves all device memory up
// front (or an embedding runtime with no device allocator at all) has nothing to hand out as
// scratch.  For them this entry point keeps the routing scratch -- per-tile expert counts and
// the padded-layout arrays -- in a fixed static device array that every GPU loading the library
// holds until the process exits.
//
// The first call on each device looks up the array's device address (cudaGetSymbolAddress) with
// that device current; make that first call before any stream capture.  Later calls only launch
// kernels.  The address is remembered together with the unique id of the CUDA context it was taken
// in (cuCtxGetId): after cudaDeviceReset, or any destruction and re-creation of the device's
// primary context, the module is loaded again and the array may sit elsewhere, so a call in a
// context with a different id looks the address up again instead of using a stale one (such a
// call, like a first call, belongs before any stream capture).  The array's size is fixed at kNoAllocScratchBytes (1 MiB).  Each call writes every scratch
// entry it later reads, so nothing has to start at zero, but all calls share the one array:
// calls whose kernels overlap on the GPU (different streams, or host threads without stream
// ordering between them) race and must be serialised by the caller.
#include <mutex>

#include "../../include/sonic_b200.h"
#include "common.cuh"
#include "sonic_internal.h"

namespace smb {

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) int32_t g_noalloc_scratch[kNoAllocScratchBytes / sizeof(int32_t)];

namespace {

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

std::mutex g_noalloc_mu;
struct ScratchEntry {
  int32_t* ptr = nullptr;
  unsigned long long ctx_id = 0;  // 0: unknown (then the address is looked up on every call)
};
ScratchEntry g_noalloc[kMaxDevices];

// Unique id of the calling thread's current context (ids are never reused within a process), or
// false when there is no current context or the driver does not provide the query.
bool current_context_id(unsigned long long* id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static bool resolved = false;
  if (!resolved) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
    resolved = true;
  }
  if (!get_current || !get_id) return false;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
  return get_id(ctx, id) == CUDA_SUCCESS && *id != 0;
}

// Device address of the static scratch in the current device's current context.  In host code
// the array's name is only a host-side stand-in, so the address comes from cudaGetSymbolAddress,
// taken with the device current and kept per device for as long as the context stays the same.
cudaError_t scratch_for_current_device(int32_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  ScratchEntry& en = g_noalloc[dev];
  unsigned long long id = 0;
  if (en.ptr && en.ctx_id != 0 && current_context_id(&id) && id == en.ctx_id) {
    *out = en.ptr;
    return cudaSuccess;
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_scratch);  // also creates the context if there is none yet
  if (e != cudaSuccess) return e;
  en.ptr = static_cast<int32_t*>(p);
  en.ctx_id = current_context_id(&id) ? id : 0;
  *out = en.ptr;
  return cudaSuccess;
}

size_t align256(size_t n) { return (n + 255) & ~static_cast<size_t>(255); }

}  // namespace
}  // namespace smb

using namespace smb;

extern "C" int sm_route_metadata_noalloc(const int32_t* topk_indices, int T, int K, int E, int32_t* expert_frequency,
                                         int32_t* expert_frequency_offset, int32_t* x_gather_idx,
                                         int32_t* s_scatter_idx, int32_t* s_reverse_scatter_idx, int32_t* err,
                                         void* stream) {
  if (T < 0 || K < 1 || E < 1 || E > 16384) return set_last_error(SM_EINVAL, "bad shape T=%d K=%d E=%d", T, K, E);
  if (!expert_frequency || !expert_frequency_offset || !err) return set_last_error(SM_EINVAL, "null pointer");
  const long long TK = static_cast<long long>(T) * K;
  if (TK > (1ll << 31) - 1) return set_last_error(SM_EINVAL, "T*K exceeds int32");
  const int n_tiles = ceil_div(T, kTileTokens);
  // scratch carve: tile counts [E][n_tiles], off_pad [E+1], blk_expert [max_blocks+1], n_blocks [1]
  const size_t b_counts = align256(static_cast<size_t>(E) * (n_tiles > 0 ? n_tiles : 1) * sizeof(int32_t));
  const size_t b_offpad = align256(static_cast<size_t>(E + 1) * sizeof(int32_t));
  const size_t b_blk = align256(static_cast<size_t>(max_padded_blocks(TK, E) + 1) * sizeof(int32_t));
  const size_t need = b_counts + b_offpad + b_blk + sizeof(int32_t);
  if (need > kNoAllocScratchBytes)
    return set_last_error(SM_EINVAL,
                           "sm_route_metadata_noalloc: T=%d K=%d E=%d needs %zu bytes of scratch, the static "
                           "area holds %zu; use sm_route_metadata with a workspace",
                           T, K, E, need, kNoAllocScratchBytes);
  int32_t* base = nullptr;
  cudaError_t e = scratch_for_current_device(&base);
  if (e != cudaSuccess) return set_last_error(SM_EIO, "scratch address: %s", cudaGetErrorString(e));
  uint8_t* p = reinterpret_cast<uint8_t*>(base);
  int32_t* tile_counts = reinterpret_cast<int32_t*>(p);
  int32_t* off_pad = reinterpret_cast<int32_t*>(p + b_counts);
  int32_t* blk_expert = reinterpret_cast<int32_t*>(p + b_counts + b_offpad);
  int32_t* n_blocks = reinterpret_cast<int32_t*>(p + b_counts + b_offpad + b_blk);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  e = launch_route_hist(topk_indices, static_cast<int>(TK), kTileTokens * K, E, n_tiles, tile_counts, err, st);
  if (e == cudaSuccess)
    e = launch_route_scan(tile_counts, n_tiles, E, static_cast<int>(TK), expert_frequency, expert_frequency_offset,
                          off_pad, blk_expert, n_blocks, st);
  if (e == cudaSuccess)
    e = launch_route_scatter(topk_indices, nullptr, static_cast<int>(TK), K, kTileTokens * K, E, n_tiles, tile_counts,
                             expert_frequency_offset, s_scatter_idx, s_reverse_scatter_idx, x_gather_idx, st);
  if (e != cudaSuccess) return set_last_error(SM_EIO, "route_metadata_noalloc: %s", cudaGetErrorString(e));
  return SM_OK;
}
