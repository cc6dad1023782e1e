// The one entry point of this library that allocates no device memory.
//
// Who needs it: code that may not allocate GPU memory while it runs.  A host
// framework that reserves the device for its own memory pool makes any later
// cudaMalloc fail; C or C++ callers embedding this library without a caching
// allocator would pay a device-wide synchronisation for every cudaMalloc /
// cudaFree pair in a step.  Such callers can still produce the NVFP4 input
// of a projection — RMSNorm + adaLN modulate of x, then e2m1 codes, block
// scales and the global scale — in one call: the two-call path
// (h3b_rmsnorm_modulate, then h3b_quant_nvfp4) needs two caller-owned
// device buffers in between, the modulated rows h and the |h| max, which
// this entry point keeps in a fixed array of the library's own device
// memory instead.  The caller still passes x, the tables and the outputs.
//
// The array (16 MiB + 256 bytes) exists once on every GPU that loads the
// library and stays there until the process exits.  All calls on a device
// share it and it keeps the last call's contents; the |h| max is cleared at
// the start of every call.  Two calls that overlap on the GPU (on different
// streams, without ordering between them) race on it.  The array's device
// address is looked up once per device and cached, so the entry point must
// not be used across a cudaDeviceReset of that device (the reset unloads the
// module and the cached address would dangle).
#include <cstdint>
#include <mutex>

#include "h3b.h"
#include "h3b_common.cuh"
#include "h3b_host.hpp"

namespace {

constexpr size_t kAmaxBytes = 256;        // the |h| max (one float), padded to keep h 256-byte aligned
constexpr size_t kRowsBytes = 16u << 20;  // h: bf16 rows of stride ld, m * ld * 2 <= 16 MiB

static __device__ __align__(256) unsigned char g_noalloc_scratch[kAmaxBytes + kRowsBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the array on the current device.  The name of a
// __device__ array in host code is only a host-side stand-in, so the
// address is looked up once per device (the first call on that device) and
// cached.
int scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return H3B_ERR_LAUNCH;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return H3B_ERR_LAUNCH;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return H3B_OK;
}

}  // namespace

extern "C" int h3b_rmsnorm_modulate_quant_nvfp4_noalloc(const void* x, int64_t m, int64_t hidden, int64_t ld,
                                                        const void* w, const void* shift, const void* scale,
                                                        int64_t tab_ld, const int32_t* row_sel, float eps,
                                                        uint8_t* codes, uint8_t* sf, float* gs_out, int hi_first,
                                                        h3b_stream_t stream) {
  // Every check of both callees runs here first, so a rejected call queues
  // nothing and leaves the shared array as it was.
  if (x == nullptr || w == nullptr || shift == nullptr || scale == nullptr || codes == nullptr || sf == nullptr ||
      gs_out == nullptr)
    return H3B_ERR_ARG;
  if (m <= 0 || hidden <= 0 || (hidden % 64) != 0 || ld < hidden || (ld % 8) != 0) return H3B_ERR_SHAPE;
  // h is held with the row stride of x: reject what does not fit the array
  if (ld > static_cast<int64_t>(kRowsBytes / 2) || m > static_cast<int64_t>(kRowsBytes / 2) / ld)
    return H3B_ERR_SHAPE;
  if (!h3b::aligned16(x) || !h3b::aligned16(w) || !h3b::aligned16(shift) || !h3b::aligned16(scale) ||
      !h3b::aligned16(codes) || (reinterpret_cast<uintptr_t>(sf) & 3u) != 0 || tab_ld < 0 || (tab_ld % 8) != 0)
    return H3B_ERR_ALIGN;
  void* base = nullptr;
  int rc = scratch_address(&base);
  if (rc != H3B_OK) return rc;
  float* amax = static_cast<float*>(base);
  void* h = static_cast<unsigned char*>(base) + kAmaxBytes;
  if (cudaMemsetAsync(amax, 0, sizeof(float), reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess)
    return H3B_ERR_LAUNCH;
  rc = h3b_rmsnorm_modulate(x, h, m, hidden, ld, w, shift, scale, tab_ld, row_sel, eps, amax, stream);
  if (rc != H3B_OK) return rc;
  return h3b_quant_nvfp4(h, m, hidden, ld, amax, codes, sf, gs_out, hi_first, stream);
}
