// Library-wide C-ABI pieces: version, device status aggregation, tensor-map
// encoding through cudaGetDriverEntryPoint, SM-count cache, and the CUDA IPC
// registration of peer buffers for the P2P Ulysses exchange.
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "h3b_common.cuh"
#include "h3b_host.hpp"

namespace h3b {

static std::vector<StatusReader>& readers() {
  static std::vector<StatusReader> r;
  return r;
}

int register_status_reader(StatusReader fn) {
  readers().push_back(fn);
  return 1;
}

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
              uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (fn == nullptr) return H3B_ERR_LAUNCH;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? H3B_OK : H3B_ERR_TMAP;
}

int encode_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t d1,
              uint64_t d2, uint64_t s1_bytes, uint64_t s2_bytes, uint32_t box_inner, uint32_t box_d1,
              uint32_t box_d2, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (fn == nullptr) return H3B_ERR_LAUNCH;
  cuuint64_t dims[3] = {inner, d1, d2};
  cuuint64_t strides[2] = {s1_bytes, s2_bytes};
  cuuint32_t box[3] = {box_inner, box_d1, box_d2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? H3B_OK : H3B_ERR_TMAP;
}

}  // namespace h3b

extern "C" int h3b_version(void) { return 100; }

extern "C" int h3b_device_status(int32_t* out4, int clear) {
  if (out4 == nullptr) return H3B_ERR_ARG;
  if (cudaDeviceSynchronize() != cudaSuccess) return H3B_ERR_DEVICE;
  out4[0] = out4[1] = out4[2] = out4[3] = 0;
  for (auto fn : h3b::readers()) {
    int32_t s[4];
    int rc = fn(s, clear);
    if (rc != H3B_OK) return rc;
    if (out4[0] == 0 && s[0] != 0) {
      for (int i = 0; i < 4; ++i) out4[i] = s[i];
    }
  }
  return H3B_OK;
}

// ---------------------------------------------------------------- CUDA IPC
namespace {

using PFN_addr_range = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

PFN_addr_range addr_range_fn() {
  static PFN_addr_range fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_addr_range>(p);
  });
  return fn;
}

}  // namespace

extern "C" int h3b_ipc_export(const void* dev_ptr, uint8_t* handle64, int64_t* offset) {
  if (dev_ptr == nullptr || handle64 == nullptr || offset == nullptr) return H3B_ERR_ARG;
  auto range = addr_range_fn();
  if (range == nullptr) return H3B_ERR_LAUNCH;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS) return H3B_ERR_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return H3B_ERR_LAUNCH;
  static_assert(sizeof(h) == 64, "CUDA IPC handle size");
  memcpy(handle64, &h, 64);
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return H3B_OK;
}

extern "C" int h3b_ipc_import(const uint8_t* handle64, int64_t offset, void** dev_ptr) {
  if (handle64 == nullptr || dev_ptr == nullptr || offset < 0) return H3B_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, 64);
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return H3B_ERR_LAUNCH;
  *dev_ptr = static_cast<uint8_t*>(base) + offset;
  return H3B_OK;
}

extern "C" int h3b_ipc_close(void* dev_ptr, int64_t offset) {
  if (dev_ptr == nullptr || offset < 0) return H3B_ERR_ARG;
  return cudaIpcCloseMemHandle(static_cast<uint8_t*>(dev_ptr) - offset) == cudaSuccess ? H3B_OK : H3B_ERR_LAUNCH;
}
