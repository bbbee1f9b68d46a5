// MemoryPool forward for callers that cannot hand the library a workspace.
//
// Some callers own all device memory and cannot allocate or pass a scratch
// buffer for this call: a runtime whose custom-call operands are fixed when
// the program is compiled, or a serving loop that must not enter the CUDA
// allocator on its per-token path.  This entry point runs the same kernels
// as memlayer_pool_forward, all on the caller's stream (without the
// library-stream overlap memlayer_pool_forward uses for large calls), with
// the workspace carved from a fixed array in
// the library's own device memory (MEMLAYER_NOALLOC_SCRATCH_BYTES; every GPU
// that loads the library holds it until the process exits).
//
// Set-up: the first call on each device (with that device current) looks up
// the array's device address with cudaGetSymbolAddress and caches it; make
// that first call before any stream capture.  All calls share the array and
// it keeps the previous call's contents; the forward itself resets what must
// start at zero (its status word and reduction ticket), but two calls whose
// kernels overlap on the GPU (different streams, no ordering) race on it.
#include <mutex>

#include "common.cuh"

namespace ml {
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[MEMLAYER_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set-up once).
int scratch_for_current_device(void** ptr) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MEMLAYER_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return MEMLAYER_ERR_CUDA;
    g_scratch_ptr[dev] = p;
  }
  *ptr = g_scratch_ptr[dev];
  return MEMLAYER_OK;
}

}  // namespace
}  // namespace ml

extern "C" int32_t memlayer_pool_forward_noalloc(const memlayer_config* cfg, const memlayer_pool_args* args,
                                                 void* stream) {
  size_t need = 0;
  int32_t st = memlayer_pool_workspace_size(cfg, &need);
  if (st != MEMLAYER_OK) return st;
  if (need > (size_t)MEMLAYER_NOALLOC_SCRATCH_BYTES) return MEMLAYER_ERR_WORKSPACE;  // too large for the array
  void* ws = nullptr;
  st = ml::scratch_for_current_device(&ws);
  if (st != MEMLAYER_OK) return st;
  // every launch on the caller's stream: no event or stream is created either
  return ml::pool_forward_single_stream(cfg, args, ws, (size_t)MEMLAYER_NOALLOC_SCRATCH_BYTES, stream);
}
