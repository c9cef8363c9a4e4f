// carekv_decode_attention_noalloc: decode attention whose scratch lives in a
// fixed array compiled into this library, for callers that cannot allocate
// device memory when they run a decode step.
//
// Who needs it: code that runs the decode step somewhere a cudaMalloc is not
// allowed or not wanted -- a serving engine that carves all device memory
// out of its own pool up front, a host-language runtime (Go, Java, Rust,
// ...) that binds this C ABI without any access to a CUDA allocator, or a
// latency-critical loop where an allocation's implicit device
// synchronisation is unacceptable.  Such a caller passes its inputs and its
// output buffer and nothing else.
//
// How it works: the scratch (selection readback, slot scores, logits and
// split-K partials) is the file-scope array below, kMaxBytes long.  Every
// GPU that loads this library reserves it for the life of the process.
// Host code cannot use the array's name as a device address (on the host it
// is only a stand-in symbol), so the first call made while a given device is
// current looks up that device's copy with cudaGetSymbolAddress and caches
// the pointer; make that first call before any stream capture.
//
// Limits: a call whose scratch need (carekv_decode_workspace_bytes) exceeds
// kMaxBytes is rejected with CAREKV_ERR_WORKSPACE before anything runs.
// Every call shares the one array and it keeps the previous call's
// contents: nothing in it has to start at zero, because each call writes
// every scratch location before reading it; calls that may overlap on the
// GPU (different streams, or other host threads) race on the array and must
// be serialised by the caller.  The call itself allocates nothing: no
// cudaMalloc / cudaFree and no allocating library routine.
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace carekv {
namespace {

constexpr size_t kMaxBytes = CAREKV_NOALLOC_MAX_BYTES;  // 64 MiB per device

static __device__ __align__(256) unsigned char g_noalloc_scratch[kMaxBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_ptr[kMaxDevices] = {};

// Device address of this device's scratch; set up once per device while it
// is the current device.
int scratch_for_current_device(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return CAREKV_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return CAREKV_ERR_CUDA;
    g_ptr[dev] = p;
  }
  *out = g_ptr[dev];
  return CAREKV_OK;
}

}  // namespace
}  // namespace carekv

extern "C" int carekv_decode_attention_noalloc(const carekv_config_t* cfg, const carekv_cache_t* cache,
                                               int32_t layer, const void* q, void* out, int32_t dtype,
                                               int32_t seq_begin, int32_t seq_count, int32_t max_pages_used,
                                               const carekv_route_params_t* params, const float* sketch_proj,
                                               void* stream) {
  if (cfg == nullptr || max_pages_used < 0) return CAREKV_ERR_INVALID_ARG;
  size_t need = 0;
  const int st = carekv_decode_workspace_bytes(cfg, seq_count, max_pages_used, &need);
  if (st != CAREKV_OK) return st;
  if (need > carekv::kMaxBytes) return CAREKV_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int s2 = carekv::scratch_for_current_device(&scratch);
  if (s2 != CAREKV_OK) return s2;
  return carekv_decode_attention(cfg, cache, layer, q, out, dtype, seq_begin, seq_count, max_pages_used, params,
                                 sketch_proj, scratch, carekv::kMaxBytes, stream);
}
