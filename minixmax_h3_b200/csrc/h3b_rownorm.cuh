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
//
// The kernels keep the next row's loads in flight while they work on the
// current one (load_row into a second register set), and each CTA-wide
// reduction takes one barrier: every thread adds the per-warp partials in
// the same order, from one of two slot sets used by alternate rows (a set
// is written again only two rows later, after a barrier every reader of
// its previous values has passed).
#pragma once

#include "h3b_common.cuh"

namespace h3b {

// Packed bf16x2 arithmetic (sm_90+), each half correctly rounded.  For two
// bf16 operands, bf16(fp32(a) op fp32(b)) is the same value: a product of
// two 8-bit significands is exact in fp32, and a sum is exact in fp32
// unless the exponents differ by more than 16, when the smaller operand is
// below a quarter of the larger one's bf16 ulp and both roundings return
// the larger operand.
H3B_DEV uint32_t bf16x2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
H3B_DEV uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// Max of each half; a NaN in either operand gives NaN.
H3B_DEV uint32_t bf16x2_max_nan(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
H3B_DEV float fmax_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// Two reduction slot sets of 32 floats; row r uses set r & 1.
struct RowSlots {
  float v[2][32];
};

// CTA-wide sum with one barrier; the same value in every thread.
template <int THREADS>
H3B_DEV float block_sum_1bar(float x, float* slots) {
  x = warp_sum(x);
  if ((threadIdx.x & 31) == 0) slots[threadIdx.x >> 5] = x;
  __syncthreads();
  float t = slots[0];
#pragma unroll
  for (int i = 1; i < THREADS / 32; ++i) t += slots[i];
  return t;
}

// CTA-wide max of non-negative values (NaN-propagating) with one barrier.
template <int THREADS>
H3B_DEV float block_max_nan_1bar(float x, float* slots) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmax_nan(x, __shfl_xor_sync(0xffffffffu, x, o));
  if ((threadIdx.x & 31) == 0) slots[threadIdx.x >> 5] = x;
  __syncthreads();
  float t = slots[0];
#pragma unroll
  for (int i = 1; i < THREADS / 32; ++i) t = fmax_nan(t, slots[i]);
  return t;
}

// Issues the loads of row xr into v (bf16 x, 16 bytes per vector).
template <int THREADS, int MAXV>
H3B_DEV void load_row(const __nv_bfloat16* __restrict__ xr, int nvec, uint4 (&v)[MAXV]) {
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = threadIdx.x + i * THREADS;
    if (vi < nvec) v[i] = *reinterpret_cast<const uint4*>(xr + vi * 8);
  }
}

// v holds the row's bf16 x on entry (load_row) and the modulated bf16 h on
// exit; returns max |h| over this thread's elements, NaN if any of them is
// NaN.  slots: this row's reduction set (one CTA barrier).
template <int THREADS, int MAXV>
H3B_DEV float rmsnorm_modulate_regs(uint4 (&v)[MAXV], int nvec, int64_t hidden, float eps,
                                    const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ shift_r,
                                    const __nv_bfloat16* __restrict__ scale_r, bool modulate, float* slots) {
  float2 ss2 = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = threadIdx.x + i * THREADS;
    if (vi < nvec) {
      const uint32_t u[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 x2 = make_float2(bf16lo_to_f32(u[e]), bf16hi_to_f32(u[e]));
        ss2 = fma2(x2, x2, ss2);
      }
    }
  }
  const float ss = block_sum_1bar<THREADS>(ss2.x + ss2.y, slots);
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(ss, static_cast<float>(hidden)) + eps));
  const float2 r2 = make_float2(rstd, rstd);
  constexpr uint32_t ONE2 = 0x3F803F80u;  // bf16x2 (1, 1)
  uint32_t amax2 = 0u;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = threadIdx.x + i * THREADS;
    if (vi < nvec) {
      const uint4 wv = *reinterpret_cast<const uint4*>(w + vi * 8);
      const uint32_t xu[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
      const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
      uint32_t hw[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 x2 = make_float2(bf16lo_to_f32(xu[e]), bf16hi_to_f32(xu[e]));
        const float2 w2 = make_float2(bf16lo_to_f32(wu[e]), bf16hi_to_f32(wu[e]));
        const float2 n2 = mul2(mul2(x2, r2), w2);  // (x * rstd) * w, each product rounded
        hw[e] = pack_bf16x2(n2.x, n2.y);
      }
      if (modulate) {
        const uint4 sh = *reinterpret_cast<const uint4*>(shift_r + vi * 8);
        const uint4 sc = *reinterpret_cast<const uint4*>(scale_r + vi * 8);
        const uint32_t shu[4] = {sh.x, sh.y, sh.z, sh.w};
        const uint32_t scu[4] = {sc.x, sc.y, sc.z, sc.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) hw[e] = bf16x2_add(bf16x2_mul(hw[e], bf16x2_add(scu[e], ONE2)), shu[e]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) amax2 = bf16x2_max_nan(amax2, hw[e] & 0x7FFF7FFFu);
      v[i] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    }
  }
  return fmax_nan(bf16lo_to_f32(amax2), bf16hi_to_f32(amax2));
}

// max |h| over this thread's elements of v (bf16 h), NaNs skipped: the
// maximum the kernels report when rmsnorm_modulate_regs returned NaN.
template <int THREADS, int MAXV>
H3B_DEV float regs_amax(const uint4 (&v)[MAXV], int nvec) {
  float a = 0.0f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    if (static_cast<int>(threadIdx.x) + i * THREADS < nvec) {
      const uint32_t u[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) a = fmax3(a, fabsf(bf16lo_to_f32(u[e])), fabsf(bf16hi_to_f32(u[e])));
    }
  }
  return a;
}

}  // namespace h3b
