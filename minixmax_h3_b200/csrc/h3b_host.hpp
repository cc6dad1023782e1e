// Host-side helpers shared by the C-ABI entry points: TMA descriptor encoding
// through the driver entry point (no link against libcuda), SM counts, launch
// checks and the registry of per-translation-unit device status readers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/h3b.h"

namespace h3b {

// Reads (and optionally clears) one translation unit's device status word.
using StatusReader = int (*)(int32_t* out4, int clear);
int register_status_reader(StatusReader fn);

// Current device's SM count (cached per device ordinal).
int num_sms();

// Encodes a row-major 2D tensor map: `inner` contiguous elements per row,
// `outer` rows `row_stride_bytes` apart; box = box_inner x box_outer.
int encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t outer,
              uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle);

// 3D variant: dims (inner, d1, d2) with byte strides s1, s2 for d1, d2.
int encode_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t inner, uint64_t d1,
              uint64_t d2, uint64_t s1_bytes, uint64_t s2_bytes, uint32_t box_inner, uint32_t box_d1,
              uint32_t box_d2, CUtensorMapSwizzle swizzle);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? H3B_OK : H3B_ERR_LAUNCH;
}

}  // namespace h3b

// Defines the reader for this translation unit's `g_status` and registers it.
#define H3B_REGISTER_STATUS_READER(tag)                                              \
  static int h3b_status_reader_##tag(int32_t* out4, int clear) {                     \
    H3bDeviceStatus s;                                                               \
    if (cudaMemcpyFromSymbol(&s, g_status, sizeof(s)) != cudaSuccess) return H3B_ERR_LAUNCH; \
    out4[0] = s.code;                                                                \
    out4[1] = s.site;                                                                \
    out4[2] = s.info;                                                                \
    out4[3] = s.block;                                                               \
    if (clear) {                                                                     \
      H3bDeviceStatus z = {0, 0, 0, 0};                                              \
      if (cudaMemcpyToSymbol(g_status, &z, sizeof(z)) != cudaSuccess) return H3B_ERR_LAUNCH; \
    }                                                                                \
    return H3B_OK;                                                                   \
  }                                                                                  \
  static int h3b_status_reader_registered_##tag = h3b::register_status_reader(h3b_status_reader_##tag)
