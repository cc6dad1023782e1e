// RMSNorm + adaLN modulate of one row, the arithmetic of the reference's
// RMSNorm (modules/linear.py:15-32) followed by _mod_scale_shift
// (model/dit.py:332-336) in its bf16 steps:
//   n = bf16((x * rstd) * w),  rstd = 1 / sqrt(mean(x^2) + eps)   (fp32)
//   h = bf16(bf16(n * bf16(1 + scale)) + shift)   for rows with a table row,
//   h = n                                           for rows outside every segment.
// Shared by the stand-alone kernel and the fused quantising kernels so that
// both produce the same bits (same element-to-thread map, same reduction
// order).  A CTA of THREADS threads holds the row in registers: thread t
// keeps elements 8(t + THREADS i) .. +7 of the row in v[i] (i < MAXV), so
// warp w's chunk i is the 256 consecutive elements starting at
// 256 (w + (THREADS / 32) i).
#pragma once

#include "h3b_common.cuh"

namespace h3b {

// Loads row xr into v (bf16 x) and leaves the modulated bf16 h there;
// returns max |h| over this thread's elements.  red: 33 floats of shared
// memory; the call holds three CTA barriers.
template <int THREADS, int MAXV>
H3B_DEV float rmsnorm_modulate_row(const __nv_bfloat16* __restrict__ xr, int nvec, int64_t hidden, float eps,
                                   const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ shift_r,
                                   const __nv_bfloat16* __restrict__ scale_r, bool modulate, float* red,
                                   uint4 (&v)[MAXV]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = threadIdx.x + i * THREADS;
    if (vi < nvec) {
      v[i] = *reinterpret_cast<const uint4*>(xr + vi * 8);
      const uint32_t u[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float a = bf16lo_to_f32(u[e]), b = bf16hi_to_f32(u[e]);
        ss += a * a + b * b;
      }
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float t = lane < THREADS / 32 ? red[lane] : 0.0f;
    t = warp_sum(t);
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(red[32], static_cast<float>(hidden)) + eps));
  __syncthreads();  // red[] is free again for the caller
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = threadIdx.x + i * THREADS;
    if (vi < nvec) {
      const uint4 wv = *reinterpret_cast<const uint4*>(w + vi * 8);
      const uint4 sh = *reinterpret_cast<const uint4*>(shift_r + vi * 8);
      const uint4 sc = *reinterpret_cast<const uint4*>(scale_r + vi * 8);
      const uint32_t xu[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
      const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
      const uint32_t shu[4] = {sh.x, sh.y, sh.z, sh.w};
      const uint32_t scu[4] = {sc.x, sc.y, sc.z, sc.w};
      uint32_t outw[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        // both bf16 halves of the 32-bit word together: one packed rounding per step
        const float2 nrm = bf16r2(__fmul_rn(__fmul_rn(bf16lo_to_f32(xu[e]), rstd), bf16lo_to_f32(wu[e])),
                                  __fmul_rn(__fmul_rn(bf16hi_to_f32(xu[e]), rstd), bf16hi_to_f32(wu[e])));
        float2 mod = nrm;
        if (modulate) {
          const float2 s1 = bf16r2(1.0f + bf16lo_to_f32(scu[e]), 1.0f + bf16hi_to_f32(scu[e]));
          const float2 t = bf16r2(nrm.x * s1.x, nrm.y * s1.y);
          mod = bf16r2(t.x + bf16lo_to_f32(shu[e]), t.y + bf16hi_to_f32(shu[e]));
        }
        amax = fmax3(amax, fabsf(mod.x), fabsf(mod.y));
        outw[e] = pack_bf16x2(mod.x, mod.y);
      }
      v[i] = make_uint4(outw[0], outw[1], outw[2], outw[3]);
    }
  }
  return amax;
}

}  // namespace h3b
