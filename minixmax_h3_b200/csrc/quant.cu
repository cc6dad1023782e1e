// Activation quantisers of the DiT-block hot path (HBM-bound kernels).
//
//  * quant_i8_rows: per-row dynamic INT8 (the semantics of the reference's
//    _dynamic_quant_rows, ops/int8_convrot.py:99-111): one CTA per row, the row
//    held in registers as 16-byte vectors, warp-shuffle absmax, IEEE division
//    and round-half-even so the codes are bit-identical to torch on the CPU.
//  * amax_bf16: grid-stride |x| max with a single atomicMax per CTA.
//  * quant_nvfp4: 64 elements (four 16-element blocks) per thread; writes
//    packed e2m1 codes and the 4 scale bytes of those blocks as one 32-bit word
//    of the 128x4 blocked scale layout (ops/nvfp4.py:46-62).
#include <cuda_fp8.h>

#include "h3b_common.cuh"
#include "h3b_host.hpp"
#include "h3b_rownorm.cuh"

H3B_DECLARE_STATUS();
H3B_REGISTER_STATUS_READER(quant);

namespace {

template <typename T>
H3B_DEV float to_f32(T v);
template <>
H3B_DEV float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
H3B_DEV float to_f32<__half>(__half v) {
  return __half2float(v);
}

template <typename T>
H3B_DEV void unpack8(const uint4& v, float (&f)[8]) {
  const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f32<T>(e[i]);
}

H3B_DEV uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Block-wide max of non-negative floats (THREADS multiple of 32, <= 1024).
template <int THREADS>
H3B_DEV float block_max(float v, float* red) {
  v = warp_max(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float w = lane < THREADS / 32 ? red[lane] : 0.0f;
    w = warp_max(w);
    if (lane == 0) red[32] = w;
  }
  __syncthreads();
  return red[32];
}

// RN(a / b) from y = RN(1/b) by Markstein's correction: q0 = RN(a*y) is within
// one ulp of a/b, the FMA residual a - q0*b is exact, and RN(q0 + r*y) is the
// correctly rounded quotient (Markstein 1990) — three FMA-pipe operations
// instead of a full division per element.  The theorem needs no overflow or
// underflow in the residual; callers take __fdiv_rn outside
// |a| >= 2^-90 and 2^-96 <= b <= 2^96.
H3B_DEV float div_rn_by_rcp(float a, float b, float y) {
  const float q0 = __fmul_rn(a, y);
  const float r = __fmaf_rn(-q0, b, a);
  return __fmaf_rn(r, y, q0);
}

H3B_DEV bool rcp_div_ok(float b) { return b >= 0x1p-96f && b <= 0x1p96f; }

// A divisor in [2^-86, 2^96] lets every element of its row or block take the
// Markstein quotient, with no per-element guard.  An element with
// |a| < 2^-90, whose residual may underflow, has |a / b| < 2^-4, and the
// corrected value stays below 2^-4 + 2^-3: both give a zero code (rint of
// less than 1/2 for INT8, e2m1 of less than 1/4).  The sign of that zero:
// a -0 dividend comes out +0, so e2m1 callers restore it with copysign (a
// no-op for every non-zero dividend, whose quotient keeps its sign).
H3B_DEV bool rcp_div_ok_all(float b) { return b >= 0x1p-86f && b <= 0x1p96f; }

template <typename T, int THREADS, int MAXV>
__global__ void __launch_bounds__(THREADS) quant_i8_rows_kernel(const T* __restrict__ x, int64_t k, int64_t ldx,
                                                                int8_t* __restrict__ q, float* __restrict__ scale) {
  __shared__ float red[33];
  const int64_t row = blockIdx.x;
  const int nvec = static_cast<int>(k >> 3);
  const T* xr = x + row * ldx;
  uint4 v[MAXV];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = threadIdx.x + i * THREADS;
    if (vi < nvec) {
      v[i] = ld_nc_v4(xr + static_cast<int64_t>(vi) * 8);
      float f[8];
      unpack8<T>(v[i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
    }
  }
  amax = block_max<THREADS>(amax, red);
  amax = fmaxf(amax, 1e-12f);
  const float s = __fdiv_rn(amax, 127.0f);
  const bool fast = rcp_div_ok_all(s);  // s >= 1e-12 / 127 > 2^-47
  const float y = __frcp_rn(s);
  int8_t* qr = q + row * k;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = threadIdx.x + i * THREADS;
    if (vi < nvec) {
      float f[8];
      unpack8<T>(v[i], f);
      uint32_t packed[2] = {0u, 0u};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float r = rintf(fast ? div_rn_by_rcp(f[j], s, y) : __fdiv_rn(f[j], s));
        r = fminf(fmaxf(r, -128.0f), 127.0f);
        const uint32_t b = static_cast<uint32_t>(static_cast<int32_t>(r)) & 0xFFu;
        packed[j >> 2] |= b << ((j & 3) * 8);
      }
      *reinterpret_cast<uint2*>(qr + static_cast<int64_t>(vi) * 8) = make_uint2(packed[0], packed[1]);
    }
  }
  if (threadIdx.x == 0) scale[row] = s;
}

// ---------------------------------------------------------------- ConvRot
// Online activation rotation of ops/hadamard.py:35-44 (rotate_activation):
// every 256-column group of a row is multiplied by the regular Hadamard
// matrix H = H4 (x) H4 (x) H4 (x) H4 / 16, H4 = [[1,1,1,-1],[1,1,-1,1],
// [1,-1,1,1],[-1,1,1,1]] (hadamard.py:11-32), then the row is quantised as
// in quant_i8_rows_kernel (int8_convrot.py:139-157 rotates, then calls
// _dynamic_quant_rows).
//
// The product is computed exactly and rounded once: inputs are 16-bit
// floats, coefficients +-1, so every partial sum of a group is exact in fp64
// unless the group's magnitudes span more than 2^37; the result is scaled by
// 1/16 (exact) and converted with one round-to-nearest-even to the input
// type.  (The reference's value comes from a 16-bit GEMM whose fp32
// accumulation order belongs to its backend.)  H is symmetric, so x.H = H.x,
// and H applies H4 along each base-4 digit of the column index in turn.

template <typename T>
H3B_DEV T f64_round(double v);
template <>
H3B_DEV __nv_bfloat16 f64_round<__nv_bfloat16>(double v) {
  unsigned short h;
  asm("cvt.rn.bf16.f64 %0, %1;" : "=h"(h) : "d"(v));
  return __ushort_as_bfloat16(h);
}
template <>
H3B_DEV __half f64_round<__half>(double v) {
  unsigned short h;
  asm("cvt.rn.f16.f64 %0, %1;" : "=h"(h) : "d"(v));
  return __ushort_as_half(h);
}

// H4 along one base-4 digit whose two index bits are lane bits (lo, hi):
// y = (sum of the 4 values) - 2 * (value at both bits flipped).
template <int LO, int HI>
H3B_DEV void h4_lanes(double (&v)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    double s = v[e] + __shfl_xor_sync(0xffffffffu, v[e], LO);
    s += __shfl_xor_sync(0xffffffffu, s, HI);
    const double p = __shfl_xor_sync(0xffffffffu, v[e], LO | HI);
    v[e] = s - 2.0 * p;
  }
}

// x.H (unscaled) for the 256-element group held by one warp: lane l holds
// columns 8l .. 8l+7.  Column index bits 0-2 are the element, 3-7 the lane;
// the digits are bits (0,1), (2,3), (4,5), (6,7).
H3B_DEV void hadamard256_warp(double (&v)[8]) {
#pragma unroll
  for (int b = 0; b < 8; b += 4) {  // digit bits 0,1: within the thread
    const double s = (v[b] + v[b + 1]) + (v[b + 2] + v[b + 3]);
    const double y0 = s - 2.0 * v[b + 3], y1 = s - 2.0 * v[b + 2];
    const double y2 = s - 2.0 * v[b + 1], y3 = s - 2.0 * v[b];
    v[b] = y0;
    v[b + 1] = y1;
    v[b + 2] = y2;
    v[b + 3] = y3;
  }
  {  // digit bits 2,3: element bit 2 and lane bit 0
    double t[4], w[8];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      t[e] = v[e] + v[e + 4];
      t[e] += __shfl_xor_sync(0xffffffffu, t[e], 1);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) w[e] = t[e & 3] - 2.0 * __shfl_xor_sync(0xffffffffu, v[e ^ 4], 1);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = w[e];
  }
  h4_lanes<2, 4>(v);    // digit bits 4,5 = lane bits 1,2
  h4_lanes<8, 16>(v);   // digit bits 6,7 = lane bits 3,4
}

// One CTA (8 warps) per row; warp w rotates groups w, w+8, ... (at most
// MAXG each), keeps the rounded values, then the row is quantised.
template <typename T, int MAXG>
__global__ void __launch_bounds__(256) quant_i8_rows_rot_kernel(const T* __restrict__ x, int64_t k, int64_t ldx,
                                                                 int8_t* __restrict__ q, float* __restrict__ scale,
                                                                 T* __restrict__ x_rot) {
  __shared__ float red[33];
  const int64_t row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = static_cast<int>(k >> 8);
  const T* xr = x + row * ldx;
  float f[MAXG][8];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXG; ++i) {
    const int g = warp + 8 * i;
    if (g < groups) {  // warp-uniform
      const uint4 raw = ld_nc_v4(xr + static_cast<int64_t>(g) * 256 + lane * 8);
      float in[8];
      unpack8<T>(raw, in);
      double v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = static_cast<double>(in[e]);
      hadamard256_warp(v);
      uint32_t packed[4];
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const T a = f64_round<T>(v[e] * 0.0625), b = f64_round<T>(v[e + 1] * 0.0625);
        f[i][e] = static_cast<float>(a);
        f[i][e + 1] = static_cast<float>(b);
        packed[e >> 1] = static_cast<uint32_t>(*reinterpret_cast<const unsigned short*>(&a)) |
                         (static_cast<uint32_t>(*reinterpret_cast<const unsigned short*>(&b)) << 16);
        amax = fmaxf(amax, fmaxf(fabsf(f[i][e]), fabsf(f[i][e + 1])));
      }
      if (x_rot != nullptr)
        *reinterpret_cast<uint4*>(x_rot + row * k + static_cast<int64_t>(g) * 256 + lane * 8) =
            make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
  }
  amax = block_max<256>(amax, red);
  amax = fmaxf(amax, 1e-12f);
  const float s = __fdiv_rn(amax, 127.0f);
  const bool fast = rcp_div_ok_all(s);  // s >= 1e-12 / 127 > 2^-47
  const float y = __frcp_rn(s);
  int8_t* qr = q + row * k;
#pragma unroll
  for (int i = 0; i < MAXG; ++i) {
    const int g = warp + 8 * i;
    if (g < groups) {
      uint32_t packed[2] = {0u, 0u};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float fj = f[i][j];
        float r = rintf(fast ? div_rn_by_rcp(fj, s, y) : __fdiv_rn(fj, s));
        r = fminf(fmaxf(r, -128.0f), 127.0f);
        const uint32_t b = static_cast<uint32_t>(static_cast<int32_t>(r)) & 0xFFu;
        packed[j >> 2] |= b << ((j & 3) * 8);
      }
      *reinterpret_cast<uint2*>(qr + static_cast<int64_t>(g) * 256 + lane * 8) = make_uint2(packed[0], packed[1]);
    }
  }
  if (threadIdx.x == 0) scale[row] = s;
}

template <typename T>
int launch_quant_i8_rot(const void* x, int64_t m, int64_t k, int64_t ldx, int8_t* q, float* scale, void* x_rot,
                        cudaStream_t st) {
  const T* xt = static_cast<const T*>(x);
  T* xr = static_cast<T*>(x_rot);
  const int64_t groups = k / 256;
  const unsigned grid = static_cast<unsigned>(m);
  if (groups <= 16) {
    quant_i8_rows_rot_kernel<T, 2><<<grid, 256, 0, st>>>(xt, k, ldx, q, scale, xr);
  } else if (groups <= 48) {
    quant_i8_rows_rot_kernel<T, 6><<<grid, 256, 0, st>>>(xt, k, ldx, q, scale, xr);
  } else {
    return H3B_ERR_SHAPE;
  }
  return h3b::launch_status();
}

__global__ void __launch_bounds__(256) amax_bf16_kernel(const __nv_bfloat16* __restrict__ x, int64_t nvec,
                                                        float* __restrict__ out) {
  __shared__ float red[33];
  float amax = 0.0f;
  for (int64_t i = blockIdx.x * 256ll + threadIdx.x; i < nvec; i += static_cast<int64_t>(gridDim.x) * 256) {
    const uint4 v = ld_nc_v4(x + i * 8);
    float f[8];
    unpack8<__nv_bfloat16>(v, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(f[j]));
  }
  amax = block_max<256>(amax, red);
  if (threadIdx.x == 0) atomicMax(reinterpret_cast<unsigned int*>(out), __float_as_uint(amax));
}

// Exact decode of an e4m3fn byte (finite, non-negative) to fp32.
H3B_DEV float e4m3_to_f32(uint32_t b) {
  const uint32_t e = (b >> 3) & 15u, mnt = b & 7u;
  if (e == 0) return static_cast<float>(mnt) * 0.001953125f;  // mnt * 2^-9
  return __uint_as_float(((e + 120u) << 23) | (mnt << 20));  // (1 + mnt/8) * 2^(e-7)
}

H3B_DEV float nvfp4_global_scale(float amax) { return amax > 0.0f ? __fdiv_rn(amax, 2688.0f) : 1.0f; }

// Four packed e2m1 bytes of r[0..7] with the hardware's round-half-even,
// saturate-at-6 conversion (the recipe's e2m1_rne_sat; the sign of zero is
// kept).  hi_first: element 2i in the high nibble of byte i.
H3B_DEV uint32_t e2m1x8(const float* r, int hi_first) {
  uint32_t out;
  if (hi_first) {
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b0, %1, %2;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b1, %3, %4;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b2, %5, %6;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b3, %7, %8;\n\t"
        "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
        : "=r"(out)
        : "f"(r[0]), "f"(r[1]), "f"(r[2]), "f"(r[3]), "f"(r[4]), "f"(r[5]), "f"(r[6]), "f"(r[7]));
  } else {
    asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
        "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
        "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
        : "=r"(out)
        : "f"(r[0]), "f"(r[1]), "f"(r[2]), "f"(r[3]), "f"(r[4]), "f"(r[5]), "f"(r[6]), "f"(r[7]));
  }
  return out;
}

// GELU: the input is fc1's bf16 output y and the quantised value is
// u = bf16(gelu(y)) (h3b_quant_nvfp4_gelu); amax_ptr then points at ymax2.
template <bool GELU>
__global__ void __launch_bounds__(256) quant_nvfp4_kernel(const __nv_bfloat16* __restrict__ x, int64_t m,
                                                          int64_t k, int64_t ldx, int64_t rows_padded,
                                                          const float* __restrict__ amax_ptr,
                                                          uint8_t* __restrict__ codes, uint8_t* __restrict__ sf,
                                                          float* __restrict__ gs_out, int hi_first) {
  const int64_t groups = k >> 6;  // 64-element groups per row
  const int64_t item = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  if (item >= rows_padded * groups) return;
  const int64_t row = item / groups;
  const int64_t g = item - row * groups;
  const float gs = nvfp4_global_scale(GELU ? gelu_input_amax(amax_ptr) : *amax_ptr);
  if (item == 0) *gs_out = gs;
  // blocked layout: ((r/128)*ncb + c/4)*512 + (r%32)*16 + ((r%128)/32)*4 + c%4, ncb = groups
  const int64_t sf_off = ((row >> 7) * groups + g) * 512 + (row & 31) * 16 + ((row & 127) >> 5) * 4;
  if (row >= m) {
    *reinterpret_cast<uint32_t*>(sf + sf_off) = 0u;
    return;
  }
  const __nv_bfloat16* xr = x + row * ldx + g * 64;
  const float six_gs = 6.0f * gs;
  const bool six_ok = rcp_div_ok(six_gs);
  const float y6 = __frcp_rn(six_gs);
  uint32_t sf_word = 0u;
  uint32_t out_words[8];
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    float f[16];
    {
      const uint4 v0 = ld_nc_v4(xr + b * 16);
      const uint4 v1 = ld_nc_v4(xr + b * 16 + 8);
      float a0[8], a1[8];
      unpack8<__nv_bfloat16>(v0, a0);
      unpack8<__nv_bfloat16>(v1, a1);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        f[j] = a0[j];
        f[8 + j] = a1[j];
      }
      if constexpr (GELU) {
#pragma unroll
        for (int j = 0; j < 16; ++j) f[j] = bf16r(gelu_erf(f[j]));
      }
    }
    float amax_b = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; j += 2) amax_b = fmax3(amax_b, fabsf(f[j]), fabsf(f[j + 1]));
    const float ratio = (six_ok && amax_b >= 0x1p-90f) ? div_rn_by_rcp(amax_b, six_gs, y6) : __fdiv_rn(amax_b, six_gs);
    const __nv_fp8_storage_t sb = __nv_cvt_float_to_fp8(ratio, __NV_SATFINITE, __NV_E4M3);
    const uint32_t sbits = static_cast<uint32_t>(sb) & 0xFFu;
    sf_word |= sbits << (8 * b);
    const float sval = e4m3_to_f32(sbits);
    const float denom = sval * gs;
    float r[16];
    if (sval > 0.0f) {
      const float y = __frcp_rn(denom);
      if (rcp_div_ok_all(denom)) {
        // div_rn_by_rcp two elements per packed fp32x2 instruction (same bits)
        const float2 y2 = make_float2(y, y), nd2 = make_float2(-denom, -denom);
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          const float2 f2 = make_float2(f[j], f[j + 1]);
          const float2 q0 = mul2(f2, y2);
          const float2 qq = fma2(fma2(q0, nd2, f2), y2, q0);
          r[j] = copysignf(qq.x, f[j]);
          r[j + 1] = copysignf(qq.y, f[j + 1]);
        }
      } else {  // blocks of tiny magnitude (or a huge divisor): per-element guard
        const bool ok = rcp_div_ok(denom);
#pragma unroll
        for (int j = 0; j < 16; ++j)
          r[j] = (ok && fabsf(f[j]) >= 0x1p-90f) ? div_rn_by_rcp(f[j], denom, y) : __fdiv_rn(f[j], denom);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) r[j] = 0.0f;  // an all-zero block: every code is +0
    }
    out_words[2 * b] = e2m1x8(r, hi_first);
    out_words[2 * b + 1] = e2m1x8(r + 8, hi_first);
  }
  uint8_t* cr = codes + row * (k >> 1) + g * 32;
  *reinterpret_cast<uint4*>(cr) = make_uint4(out_words[0], out_words[1], out_words[2], out_words[3]);
  *reinterpret_cast<uint4*>(cr + 16) = make_uint4(out_words[4], out_words[5], out_words[6], out_words[7]);
  *reinterpret_cast<uint32_t*>(sf + sf_off) = sf_word;
}

__global__ void swap_nibbles_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int64_t nvec) {
  for (int64_t i = blockIdx.x * 256ll + threadIdx.x; i < nvec; i += static_cast<int64_t>(gridDim.x) * 256) {
    uint4 v = src[i];
    v.x = ((v.x >> 4) & 0x0F0F0F0Fu) | ((v.x << 4) & 0xF0F0F0F0u);
    v.y = ((v.y >> 4) & 0x0F0F0F0Fu) | ((v.y << 4) & 0xF0F0F0F0u);
    v.z = ((v.z >> 4) & 0x0F0F0F0Fu) | ((v.z << 4) & 0xF0F0F0F0u);
    v.w = ((v.w >> 4) & 0x0F0F0F0Fu) | ((v.w << 4) & 0xF0F0F0F0u);
    dst[i] = v;
  }
}

template <typename T>
int launch_quant_i8(const void* x, int64_t m, int64_t k, int64_t ldx, int8_t* q, float* scale, cudaStream_t st) {
  const T* xt = static_cast<const T*>(x);
  const int64_t nvec = k / 8;
  if (nvec <= 128 * 4) {
    quant_i8_rows_kernel<T, 128, 4><<<static_cast<unsigned>(m), 128, 0, st>>>(xt, k, ldx, q, scale);
  } else if (nvec <= 256 * 6) {
    quant_i8_rows_kernel<T, 256, 6><<<static_cast<unsigned>(m), 256, 0, st>>>(xt, k, ldx, q, scale);
  } else if (nvec <= 512 * 12) {
    quant_i8_rows_kernel<T, 512, 12><<<static_cast<unsigned>(m), 512, 0, st>>>(xt, k, ldx, q, scale);
  } else {
    return H3B_ERR_SHAPE;
  }
  return h3b::launch_status();
}

// RMSNorm + adaLN modulate + INT8 row quantisation (ROT: with the ConvRot
// rotation of every 256-column group in between) — the values of
// rmsnorm_modulate followed by quant_i8_rows / quant_i8_rows_convrot on its
// bf16 output (int8_convrot.py:114-157 on the output of dit.py:433-434),
// without writing that output: the row stays in registers.  In the row
// layout of rmsnorm_modulate_row, warp w's chunk i is exactly ConvRot group
// w + (THREADS / 32) i with element 8 lane + e in lane `lane`, the order
// hadamard256_warp rotates, so ROT needs no data movement.
template <int THREADS, int MAXV, bool ROT>
__global__ void __launch_bounds__(THREADS, THREADS == 128 ? (ROT ? 6 : 8) : 1) rmsnorm_modulate_quant_i8_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t m, int64_t hidden, int64_t ld, const __nv_bfloat16* __restrict__ w,
    const __nv_bfloat16* __restrict__ shift, const __nv_bfloat16* __restrict__ scale, int64_t tab_ld,
    const int32_t* __restrict__ row_sel, float eps, int8_t* __restrict__ q, float* __restrict__ q_scale) {
  __shared__ h3b::RowSlots sum_slots, max_slots;
  __shared__ float red[33];
  const int nvec = static_cast<int>(hidden >> 3);
  int64_t row = blockIdx.x;
  uint4 nxt[MAXV] = {};
  if (row < m) h3b::load_row<THREADS, MAXV>(x + row * ld, nvec, nxt);
  for (int par = 0; row < m; row += gridDim.x, par ^= 1) {
    uint4 v[MAXV];
#pragma unroll
    for (int i = 0; i < MAXV; ++i) v[i] = nxt[i];
    // the next row's loads stay in flight while this one is worked on
    if (row + gridDim.x < m) h3b::load_row<THREADS, MAXV>(x + (row + gridDim.x) * ld, nvec, nxt);
    const int sel = row_sel != nullptr ? row_sel[row] : 0;
    const bool modulate = sel >= 0;
    const __nv_bfloat16* shift_r = shift + static_cast<int64_t>(modulate ? sel : 0) * tab_ld;
    const __nv_bfloat16* scale_r = scale + static_cast<int64_t>(modulate ? sel : 0) * tab_ld;
    // amax: NaN if any element of this thread's share is NaN
    float amax = h3b::rmsnorm_modulate_regs<THREADS, MAXV>(v, nvec, hidden, eps, w, shift_r, scale_r, modulate,
                                                           sum_slots.v[par]);
    // ROT: the rotated row as floats; otherwise h is read from v directly
    float f[ROT ? MAXV : 1][8];
    if constexpr (ROT) {
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int vi = threadIdx.x + i * THREADS;
        if (vi < nvec) {  // warp-uniform (hidden % 256 == 0)
          unpack8<__nv_bfloat16>(v[i], f[i]);
          double d[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) d[e] = static_cast<double>(f[i][e]);
          hadamard256_warp(d);
#pragma unroll
          for (int e = 0; e < 8; ++e) f[i][e] = __bfloat162float(f64_round<__nv_bfloat16>(d[e] * 0.0625));
        }
      }
      amax = 0.0f;
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        if (threadIdx.x + i * THREADS < nvec) {
#pragma unroll
          for (int e = 0; e < 8; ++e) amax = h3b::fmax_nan(amax, fabsf(f[i][e]));
        }
      }
    }
    // The row max, NaN if the row holds a NaN (one barrier).  A finite row
    // whose scale admits the reciprocal quotient everywhere takes the packed
    // path; any other row the per-element path with NaNs skipped in the max.
    auto elem = [&](int i, int j) -> float {
      if constexpr (ROT) {
        return f[i][j];
      } else {
        const uint32_t u = j < 2 ? v[i].x : j < 4 ? v[i].y : j < 6 ? v[i].z : v[i].w;
        return (j & 1) ? bf16hi_to_f32(u) : bf16lo_to_f32(u);
      }
    };
    const float row_max = h3b::block_max_nan_1bar<THREADS>(amax, max_slots.v[par]);
    float s = __fdiv_rn(fmaxf(row_max, 1e-12f), 127.0f);
    int8_t* qr = q + row * hidden;
    if (row_max <= 3.4028234663852886e38f && rcp_div_ok_all(s)) {
      // q = rint(x / s) by Markstein's quotient (packed fp32x2, the same
      // bits as div_rn_by_rcp) and the 1.5 * 2^23 rounding add, which
      // leaves rint(q) in the low byte.  |x / s| <= 127 (1 + 2^-23) here,
      // so the clamp to [-128, 127] never binds.
      const float y = __frcp_rn(s);
      const float2 y2 = make_float2(y, y), ns2 = make_float2(-s, -s);
      const float2 magic2 = make_float2(0x1.8p23f, 0x1.8p23f);
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int vi = threadIdx.x + i * THREADS;
        if (vi < nvec) {
          uint32_t b[8];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f2 = make_float2(elem(i, 2 * e), elem(i, 2 * e + 1));
            const float2 q0 = mul2(f2, y2);
            const float2 qq = fma2(fma2(q0, ns2, f2), y2, q0);
            const float2 t = add2_rn(qq, magic2);
            b[2 * e] = __float_as_uint(t.x);
            b[2 * e + 1] = __float_as_uint(t.y);
          }
          const uint32_t w0 = __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
          const uint32_t w1 = __byte_perm(__byte_perm(b[4], b[5], 0x0040), __byte_perm(b[6], b[7], 0x0040), 0x5410);
          *reinterpret_cast<uint2*>(qr + static_cast<int64_t>(vi) * 8) = make_uint2(w0, w1);
        }
      }
    } else {
      float a = 0.0f;
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        if (threadIdx.x + i * THREADS < nvec) {
#pragma unroll
          for (int e = 0; e < 8; ++e) a = fmaxf(a, fabsf(elem(i, e)));
        }
      }
      a = block_max<THREADS>(a, red);
      s = __fdiv_rn(fmaxf(a, 1e-12f), 127.0f);
      const bool fast = rcp_div_ok_all(s);
      const float y = __frcp_rn(s);
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int vi = threadIdx.x + i * THREADS;
        if (vi < nvec) {
          uint32_t packed[2] = {0u, 0u};
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float fj = elem(i, j);
            float r = rintf(fast ? div_rn_by_rcp(fj, s, y) : __fdiv_rn(fj, s));
            r = fminf(fmaxf(r, -128.0f), 127.0f);
            const uint32_t bj = static_cast<uint32_t>(static_cast<int32_t>(r)) & 0xFFu;
            packed[j >> 2] |= bj << ((j & 3) * 8);
          }
          *reinterpret_cast<uint2*>(qr + static_cast<int64_t>(vi) * 8) = make_uint2(packed[0], packed[1]);
        }
      }
      __syncthreads();  // red[] is read by every thread above before the next row writes it
    }
    if (threadIdx.x == 0) q_scale[row] = s;
  }
}

}  // namespace

extern "C" int h3b_quant_i8_rows(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, int8_t* q,
                                 float* scale, h3b_stream_t stream) {
  if (x == nullptr || q == nullptr || scale == nullptr) return H3B_ERR_ARG;
  if (m < 0 || k <= 0 || (k % 8) != 0 || ldx < k || (ldx % 8) != 0 || m > 0x7fffffff) return H3B_ERR_SHAPE;
  if (!h3b::aligned16(x) || (reinterpret_cast<uintptr_t>(q) & 7u) != 0) return H3B_ERR_ALIGN;
  if (m == 0) return H3B_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (x_dtype == H3B_BF16) return launch_quant_i8<__nv_bfloat16>(x, m, k, ldx, q, scale, st);
  if (x_dtype == H3B_F16) return launch_quant_i8<__half>(x, m, k, ldx, q, scale, st);
  return H3B_ERR_DTYPE;
}

extern "C" int h3b_quant_i8_rows_convrot(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx,
                                         int64_t group_size, int8_t* q, float* scale, void* x_rot,
                                         h3b_stream_t stream) {
  if (x == nullptr || q == nullptr || scale == nullptr) return H3B_ERR_ARG;
  if (group_size != 256) return H3B_ERR_SHAPE;
  if (m < 0 || k <= 0 || (k % 256) != 0 || ldx < k || (ldx % 8) != 0 || m > 0x7fffffff) return H3B_ERR_SHAPE;
  if (!h3b::aligned16(x) || (reinterpret_cast<uintptr_t>(q) & 7u) != 0) return H3B_ERR_ALIGN;
  if (x_rot != nullptr && !h3b::aligned16(x_rot)) return H3B_ERR_ALIGN;
  if (m == 0) return H3B_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (x_dtype == H3B_BF16) return launch_quant_i8_rot<__nv_bfloat16>(x, m, k, ldx, q, scale, x_rot, st);
  if (x_dtype == H3B_F16) return launch_quant_i8_rot<__half>(x, m, k, ldx, q, scale, x_rot, st);
  return H3B_ERR_DTYPE;
}

extern "C" int h3b_amax_bf16(const void* x, int64_t n, float* amax_out, h3b_stream_t stream) {
  if (x == nullptr || amax_out == nullptr) return H3B_ERR_ARG;
  if (n < 0 || (n % 8) != 0) return H3B_ERR_SHAPE;
  if (!h3b::aligned16(x)) return H3B_ERR_ALIGN;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(amax_out, 0, sizeof(float), st) != cudaSuccess) return H3B_ERR_LAUNCH;
  if (n == 0) return H3B_OK;
  const int64_t nvec = n / 8;
  int64_t blocks = (nvec + 255) / 256;
  const int64_t cap = static_cast<int64_t>(h3b::num_sms()) * 8;
  if (blocks > cap) blocks = cap;
  amax_bf16_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x), nvec,
                                                                   amax_out);
  return h3b::launch_status();
}

extern "C" int h3b_quant_nvfp4(const void* x, int64_t m, int64_t k, int64_t ldx, const float* amax, uint8_t* codes,
                               uint8_t* sf, float* gs_out, int hi_first, h3b_stream_t stream) {
  if (x == nullptr || amax == nullptr || codes == nullptr || sf == nullptr || gs_out == nullptr)
    return H3B_ERR_ARG;
  if (m <= 0 || k <= 0 || (k % 64) != 0 || ldx < k || (ldx % 8) != 0) return H3B_ERR_SHAPE;
  if (!h3b::aligned16(x) || !h3b::aligned16(codes) || (reinterpret_cast<uintptr_t>(sf) & 3u) != 0)
    return H3B_ERR_ALIGN;
  const int64_t rows_padded = (m + 127) / 128 * 128;
  const int64_t items = rows_padded * (k / 64);
  const int64_t blocks = (items + 255) / 256;
  if (blocks > 0x7fffffff) return H3B_ERR_SHAPE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  quant_nvfp4_kernel<false><<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(x), m, k, ldx, rows_padded, amax, codes, sf, gs_out, hi_first);
  return h3b::launch_status();
}

extern "C" int h3b_quant_nvfp4_gelu(const void* y, int64_t m, int64_t k, int64_t ldy, const float* ymax2,
                                    uint8_t* codes, uint8_t* sf, float* gs_out, int hi_first, h3b_stream_t stream) {
  if (y == nullptr || ymax2 == nullptr || codes == nullptr || sf == nullptr || gs_out == nullptr)
    return H3B_ERR_ARG;
  if (m <= 0 || k <= 0 || (k % 64) != 0 || ldy < k || (ldy % 8) != 0) return H3B_ERR_SHAPE;
  if (!h3b::aligned16(y) || !h3b::aligned16(codes) || (reinterpret_cast<uintptr_t>(sf) & 3u) != 0)
    return H3B_ERR_ALIGN;
  const int64_t rows_padded = (m + 127) / 128 * 128;
  const int64_t items = rows_padded * (k / 64);
  const int64_t blocks = (items + 255) / 256;
  if (blocks > 0x7fffffff) return H3B_ERR_SHAPE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  quant_nvfp4_kernel<true><<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      static_cast<const __nv_bfloat16*>(y), m, k, ldy, rows_padded, ymax2, codes, sf, gs_out, hi_first);
  return h3b::launch_status();
}

// ymax2[1] = max |bf16(gelu(y))| when bf16(gelu(ymax2[0])) is below the
// bound for negative inputs (every block leaves at once otherwise).  Rows of
// k bf16 values with row stride ldy, 8 values per step.
__global__ void __launch_bounds__(256) gelu_amax_scan_kernel(const __nv_bfloat16* __restrict__ y, int64_t m,
                                                             int64_t k, int64_t ldy, float* __restrict__ ymax2) {
  __shared__ float red[33];
  if (bf16r(gelu_erf(ymax2[0])) >= GELU_BF16_NEG_BOUND) return;  // uniform across the grid
  const int64_t vpr = k >> 3;  // 8-value vectors per row
  const int64_t nvec = m * vpr;
  float amax = 0.0f;
  for (int64_t i = blockIdx.x * 256ll + threadIdx.x; i < nvec; i += static_cast<int64_t>(gridDim.x) * 256) {
    const int64_t row = i / vpr;
    const uint4 v = ld_nc_v4(y + row * ldy + (i - row * vpr) * 8);
    float f[8];
    unpack8<__nv_bfloat16>(v, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fabsf(bf16r(gelu_erf(f[j]))));
  }
  amax = block_max<256>(amax, red);
  if (threadIdx.x == 0) atomicMax(reinterpret_cast<unsigned int*>(ymax2 + 1), __float_as_uint(amax));
}

extern "C" int h3b_gelu_amax_scan(const void* y, int64_t m, int64_t k, int64_t ldy, float* ymax2,
                                  h3b_stream_t stream) {
  if (y == nullptr || ymax2 == nullptr) return H3B_ERR_ARG;
  if (m < 0 || k <= 0 || (k % 8) != 0 || ldy < k || (ldy % 8) != 0) return H3B_ERR_SHAPE;
  if (!h3b::aligned16(y)) return H3B_ERR_ALIGN;
  if (m == 0) return H3B_OK;
  const int64_t nvec = m * (k / 8);
  const int64_t want = (nvec + 255) / 256;
  const int blocks = static_cast<int>(want < 4 * h3b::num_sms() ? want : 4 * h3b::num_sms());
  gelu_amax_scan_kernel<<<blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(y), m, k, ldy, ymax2);
  return h3b::launch_status();
}

extern "C" int h3b_nvfp4_swap_nibbles(const uint8_t* src, uint8_t* dst, int64_t nbytes, h3b_stream_t stream) {
  if (src == nullptr || dst == nullptr) return H3B_ERR_ARG;
  if (nbytes < 0 || (nbytes % 16) != 0) return H3B_ERR_SHAPE;
  if (!h3b::aligned16(src) || !h3b::aligned16(dst)) return H3B_ERR_ALIGN;
  if (nbytes == 0) return H3B_OK;
  const int64_t nvec = nbytes / 16;
  int64_t blocks = (nvec + 255) / 256;
  const int64_t cap = static_cast<int64_t>(h3b::num_sms()) * 8;
  if (blocks > cap) blocks = cap;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  swap_nibbles_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(reinterpret_cast<const uint4*>(src),
                                                                      reinterpret_cast<uint4*>(dst), nvec);
  return h3b::launch_status();
}

extern "C" int h3b_rmsnorm_modulate_quant_i8(const void* x, int64_t m, int64_t hidden, int64_t ld, const void* w,
                                             const void* shift, const void* scale, int64_t tab_ld,
                                             const int32_t* row_sel, float eps, int64_t convrot_group, int8_t* q,
                                             float* q_scale, h3b_stream_t stream) {
  if (x == nullptr || w == nullptr || shift == nullptr || scale == nullptr || q == nullptr || q_scale == nullptr)
    return H3B_ERR_ARG;
  if (m < 0 || hidden <= 0 || (hidden % 8) != 0 || ld < hidden || (ld % 8) != 0 || m > 0x7fffffff)
    return H3B_ERR_SHAPE;
  if (convrot_group != 0 && (convrot_group != 256 || (hidden % 256) != 0)) return H3B_ERR_SHAPE;
  if (!h3b::aligned16(x) || !h3b::aligned16(w) || !h3b::aligned16(shift) || !h3b::aligned16(scale) ||
      (reinterpret_cast<uintptr_t>(q) & 7u) != 0 || tab_ld < 0 || (tab_ld % 8) != 0)
    return H3B_ERR_ALIGN;
  if (m == 0) return H3B_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const auto* wb = static_cast<const __nv_bfloat16*>(w);
  const auto* sh = static_cast<const __nv_bfloat16*>(shift);
  const auto* sc = static_cast<const __nv_bfloat16*>(scale);
  const int64_t nvec = hidden / 8;
  // rows up to 3072 wide: 128-thread CTAs, 8 resident per SM (6 with
  // ConvRot), each with one row in work and the next one loading; the grid
  // is one resident wave
  const bool narrow = nvec <= 128 * 3;
  int64_t blocks = static_cast<int64_t>(h3b::num_sms()) * (narrow ? (convrot_group == 256 ? 6 : 8) : 8);
  if (blocks > m) blocks = m;
  const unsigned g = static_cast<unsigned>(blocks);
  const bool rot = convrot_group == 256;
  if (narrow) {
    if (rot)
      rmsnorm_modulate_quant_i8_kernel<128, 3, true><<<g, 128, 0, st>>>(xb, m, hidden, ld, wb, sh, sc, tab_ld,
                                                                        row_sel, eps, q, q_scale);
    else
      rmsnorm_modulate_quant_i8_kernel<128, 3, false><<<g, 128, 0, st>>>(xb, m, hidden, ld, wb, sh, sc, tab_ld,
                                                                         row_sel, eps, q, q_scale);
  } else if (nvec <= 256 * 8) {
    if (rot)
      rmsnorm_modulate_quant_i8_kernel<256, 8, true><<<g, 256, 0, st>>>(xb, m, hidden, ld, wb, sh, sc, tab_ld,
                                                                        row_sel, eps, q, q_scale);
    else
      rmsnorm_modulate_quant_i8_kernel<256, 8, false><<<g, 256, 0, st>>>(xb, m, hidden, ld, wb, sh, sc, tab_ld,
                                                                         row_sel, eps, q, q_scale);
  } else {
    return H3B_ERR_SHAPE;
  }
  return h3b::launch_status();
}
