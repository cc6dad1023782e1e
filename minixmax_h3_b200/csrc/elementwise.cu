// Row-wise elementwise kernels of the DiT block (HBM-bound).
//
//  * qk_rmsnorm_rope: q/k RMSNorm + split-half RoPE in one pass over each
//    token's head rows, the rotation table built on the fly from the token's
//    (t, h, w) grid position, once per token (ops/rope.py:7-55,
//    model/dit.py:746-752).  The
//    rotation uses the reference's bf16 arithmetic: bf16 cos/sin table, each
//    product and the sum rounded to bf16.
//  * rmsnorm_modulate: RMSNorm(hidden) then h*(1+scale)+shift with the
//    reference's bf16 rounding after each step (model/dit.py:332-335,
//    modules/linear.py:29-32), optional |h| max for the NVFP4 global scale.
//  * gate_residual: x += y*gate (model/dit.py:338-341).
#include "h3b_common.cuh"
#include "h3b_host.hpp"
#include "h3b_rownorm.cuh"

namespace {

// One warp per token; lane l owns d = 4l..4l+3 of every 128-element head
// row.  The token's rotation (bf16 cos/sin of its 64 angles) is computed once
// and applied to all heads of q and k, four head rows in flight at a time.
// The four rows' sums of squares are reduced together (a reduce-scatter over
// lane bits 4 and 3, then a butterfly over bits 2-0: ten shuffles instead of
// twenty), lanes 8u..8u+7 compute row u's rstd and pass it on, and the bf16
// steps of the rotation run two elements per packed bf16x2 instruction: the
// product of two bf16 values and the sum of two are exact in fp32, so each
// packed result equals the reference's fp32 operation rounded to bf16.
__global__ void __launch_bounds__(256) qk_rmsnorm_rope_kernel(
    __nv_bfloat16* __restrict__ q, __nv_bfloat16* __restrict__ k, int64_t s_len, int heads, int64_t seq_stride,
    int64_t head_stride, const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw, float eps,
    const float* __restrict__ pos, int64_t pos_offset, const float* __restrict__ inv_freq, int n_t, int n_h) {
  constexpr int ROWS = 4;
  const int lane = threadIdx.x & 31;
  const int64_t s = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (s >= s_len) return;  // warp-uniform
  // element j (lane < 16: j = 4*lane.. in the first half; lane >= 16: second half)
  const float* ps = pos + (pos_offset + s) * 3;
  const bool first = lane < 16;
  // bf16x2 cos and sin of the lane's four angles; the first half rotates by
  // c*x[j] + (-s)*x[j+64], the second by s*x[j] + c*x[j+64], so the first
  // half's sin is negated (bf16 rounding is symmetric).
  uint32_t cw[2], sw[2];
#pragma unroll
  for (int e = 0; e < 4; e += 2) {
    float cc[2], ss[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int jj = (lane & 15) * 4 + e + t;  // frequency index 0..63
      const int axis = jj < n_t ? 0 : (jj < n_t + n_h ? 1 : 2);
      const float ang = __fmul_rn(ps[axis], inv_freq[jj]);
      cc[t] = cosf(ang);
      ss[t] = first ? -sinf(ang) : sinf(ang);
    }
    cw[e >> 1] = pack_bf16x2(cc[0], cc[1]);
    sw[e >> 1] = pack_bf16x2(ss[0], ss[1]);
  }
  float2 wq[2], wk[2];
  {
    const uint2 a = *reinterpret_cast<const uint2*>(qw + lane * 4);
    wq[0] = make_float2(bf16lo_to_f32(a.x), bf16hi_to_f32(a.x));
    wq[1] = make_float2(bf16lo_to_f32(a.y), bf16hi_to_f32(a.y));
    if (k != nullptr) {
      const uint2 b = *reinterpret_cast<const uint2*>(kw + lane * 4);
      wk[0] = make_float2(bf16lo_to_f32(b.x), bf16hi_to_f32(b.x));
      wk[1] = make_float2(bf16lo_to_f32(b.y), bf16hi_to_f32(b.y));
    }
  }
  const bool b4 = (lane & 16) != 0, b3 = (lane & 8) != 0;
  const int rows = heads * (k != nullptr ? 2 : 1);  // q heads, then k heads
  for (int r0 = 0; r0 < rows; r0 += ROWS) {
    uint2 raw[ROWS];
    __nv_bfloat16* base[ROWS];
    float ssq[ROWS];
#pragma unroll
    for (int u = 0; u < ROWS; ++u) {
      const int r = r0 + u;
      raw[u] = make_uint2(0u, 0u);
      if (r < rows) {
        const bool is_k = r >= heads;
        const int h = is_k ? r - heads : r;
        base[u] = (is_k ? k : q) + s * seq_stride + static_cast<int64_t>(h) * head_stride;
        raw[u] = *reinterpret_cast<const uint2*>(base[u] + lane * 4);
      }
    }
#pragma unroll
    for (int u = 0; u < ROWS; ++u) {
      const float2 x01 = make_float2(bf16lo_to_f32(raw[u].x), bf16hi_to_f32(raw[u].x));
      const float2 x23 = make_float2(bf16lo_to_f32(raw[u].y), bf16hi_to_f32(raw[u].y));
      const float2 t = fma2(x23, x23, mul2(x01, x01));
      ssq[u] = t.x + t.y;
    }
    // reduce-scatter: after xor 16 a lane holds rows 2*b4, 2*b4+1; after
    // xor 8 row 2*b4+b3; xor 4, 2, 1 complete its sum in lanes 8u..8u+7
    const float s0 = __shfl_xor_sync(0xffffffffu, b4 ? ssq[0] : ssq[2], 16);
    const float s1 = __shfl_xor_sync(0xffffffffu, b4 ? ssq[1] : ssq[3], 16);
    const float k0 = (b4 ? ssq[2] : ssq[0]) + s0;
    const float k1 = (b4 ? ssq[3] : ssq[1]) + s1;
    float tot = (b3 ? k1 : k0) + __shfl_xor_sync(0xffffffffu, b3 ? k0 : k1, 8);
    tot += __shfl_xor_sync(0xffffffffu, tot, 4);
    tot += __shfl_xor_sync(0xffffffffu, tot, 2);
    tot += __shfl_xor_sync(0xffffffffu, tot, 1);
    // mean = tot / 128 (exact scaling), rstd = RN(1 / RN(sqrt(mean + eps)))
    const float my_rstd = __frcp_rn(__fsqrt_rn(__fmul_rn(tot, 0.0078125f) + eps));
#pragma unroll
    for (int u = 0; u < ROWS; ++u) {
      const int r = r0 + u;
      const float rstd = __shfl_sync(0xffffffffu, my_rstd, 8 * u);
      if (r >= rows) break;  // warp-uniform
      const float2* w = r >= heads ? wk : wq;
      const float2 r2 = make_float2(rstd, rstd);
      const float2 x01 = make_float2(bf16lo_to_f32(raw[u].x), bf16hi_to_f32(raw[u].x));
      const float2 x23 = make_float2(bf16lo_to_f32(raw[u].y), bf16hi_to_f32(raw[u].y));
      const float2 n01 = mul2(mul2(x01, r2), w[0]);  // (x * rstd) * w, each product rounded
      const float2 n23 = mul2(mul2(x23, r2), w[1]);
      const uint32_t nb[2] = {pack_bf16x2(n01.x, n01.y), pack_bf16x2(n23.x, n23.y)};
      // partner elements j +- 64 live in lane +- 16, same slots
      uint32_t ow[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const uint32_t pb = __shfl_xor_sync(0xffffffffu, nb[e], 16);
        ow[e] = h3b::bf16x2_add(h3b::bf16x2_mul(cw[e], nb[e]), h3b::bf16x2_mul(sw[e], pb));
      }
      *reinterpret_cast<uint2*>(base[u] + lane * 4) = make_uint2(ow[0], ow[1]);
    }
  }
}

// CTAs of THREADS threads stride over rows; a row is held in registers
// (<= MAXV x 8 bf16 per thread).  The optional |h| max is reduced per CTA and
// published with one atomic.
template <int THREADS, int MAXV>
__global__ void __launch_bounds__(THREADS, THREADS == 128 ? 8 : 1) rmsnorm_modulate_kernel(
    const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ h, int64_t m, int64_t hidden, int64_t ld,
    const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ shift,
    const __nv_bfloat16* __restrict__ scale, int64_t tab_ld, const int32_t* __restrict__ row_sel, float eps,
    float* __restrict__ amax_out) {
  __shared__ h3b::RowSlots slots;
  __shared__ float red[33];
  const int nvec = static_cast<int>(hidden >> 3);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float amax = 0.0f;
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
    float a = h3b::rmsnorm_modulate_regs<THREADS, MAXV>(v, nvec, hidden, eps, w, shift_r, scale_r, modulate,
                                                        slots.v[par]);
    if (a != a) a = h3b::regs_amax<THREADS, MAXV>(v, nvec);  // NaNs are skipped in the reported max
    amax = fmaxf(amax, a);
    __nv_bfloat16* hr = h + row * ld;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = threadIdx.x + i * THREADS;
      if (vi < nvec) *reinterpret_cast<uint4*>(hr + vi * 8) = v[i];
    }
  }
  if (amax_out != nullptr) {
    amax = warp_max(amax);
    if (lane == 0) red[warp] = amax;
    __syncthreads();
    if (warp == 0) {
      float t = lane < THREADS / 32 ? red[lane] : 0.0f;
      t = warp_max(t);
      if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(amax_out), __float_as_uint(t));
    }
  }
}

__global__ void __launch_bounds__(256) gate_residual_kernel(__nv_bfloat16* __restrict__ x,
                                                            const __nv_bfloat16* __restrict__ y, int64_t m,
                                                            int64_t hidden, int64_t ld,
                                                            const __nv_bfloat16* __restrict__ gate, int64_t tab_ld,
                                                            const int32_t* __restrict__ row_sel) {
  const int64_t nvec_row = hidden >> 3;
  const int64_t total = m * nvec_row;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * 256) {
    const int64_t r = i / nvec_row, c = (i - r * nvec_row) * 8;
    const int sel = row_sel != nullptr ? row_sel[r] : 0;
    if (sel < 0) continue;  // token outside every mod segment: x unchanged
    uint4* xp = reinterpret_cast<uint4*>(x + r * ld + c);
    const uint4 xv = *xp;
    const uint4 yv = *reinterpret_cast<const uint4*>(y + r * ld + c);
    const uint4 gv = *reinterpret_cast<const uint4*>(gate + static_cast<int64_t>(sel) * tab_ld + c);
    const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w}, yu[4] = {yv.x, yv.y, yv.z, yv.w},
                   gu[4] = {gv.x, gv.y, gv.z, gv.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      o[e] = pack_bf16x2(__fadd_rn(bf16lo_to_f32(xu[e]), __fmul_rn(bf16lo_to_f32(yu[e]), bf16lo_to_f32(gu[e]))),
                         __fadd_rn(bf16hi_to_f32(xu[e]), __fmul_rn(bf16hi_to_f32(yu[e]), bf16hi_to_f32(gu[e]))));
    }
    *xp = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace

// Merge of two attention results over disjoint key sets through their row
// log-sum-exps, in fp32 (ops/fa_h3.py:141-156):
//   o   <- o - sigmoid(l_b - l_o) * (o - o_b)
//   l_o <- l_o - logsigmoid(l_o - l_b) = max(l_o, l_b) + log1p(exp(-|l_o - l_b|))
// first: o <- o_b, l_o <- l_b.  One warp per (token, head) row of 128; acc is
// fp32 and blk / out bf16, all token-major [s, heads, 128]; lse [heads, s].
// With out given (the last merge) the result goes to out as bf16, with its
// max |value| into amax_out, and acc is not written back.
__global__ void __launch_bounds__(256) merge_lse_kernel(float* __restrict__ acc, float* __restrict__ acc_lse,
                                                        const __nv_bfloat16* __restrict__ blk,
                                                        const float* __restrict__ blk_lse, int64_t s,
                                                        int64_t heads, int first,
                                                        __nv_bfloat16* __restrict__ out,
                                                        float* __restrict__ amax_out) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = s * heads;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  float amax = 0.0f;
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const int64_t t = r / heads;
    const int64_t li = (r - t * heads) * s + t;
    const uint2 bv = *reinterpret_cast<const uint2*>(blk + r * 128 + lane * 4);
    const float b[4] = {bf16lo_to_f32(bv.x), bf16hi_to_f32(bv.x), bf16lo_to_f32(bv.y), bf16hi_to_f32(bv.y)};
    float4* ap = reinterpret_cast<float4*>(acc + r * 128 + lane * 4);
    const float lb = blk_lse[li];
    float o[4];
    float l_new;
    if (first) {
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = b[e];
      l_new = lb;
    } else {
      const float4 av = *ap;
      const float a[4] = {av.x, av.y, av.z, av.w};
      const float lo = acc_lse[li];
      const float d = lo - lb;
      const float w = __fdiv_rn(1.0f, 1.0f + expf(d));  // sigmoid(lb - lo)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = a[e] - w * (a[e] - b[e]);
      l_new = fmaxf(lo, lb) + log1pf(expf(-fabsf(d)));
    }
    if (lane == 0) acc_lse[li] = l_new;
    if (out == nullptr) {
      *ap = make_float4(o[0], o[1], o[2], o[3]);
    } else {
      const uint2 ov = make_uint2(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]));
      *reinterpret_cast<uint2*>(out + r * 128 + lane * 4) = ov;
      amax = fmax3(amax, fmaxf(fabsf(bf16lo_to_f32(ov.x)), fabsf(bf16hi_to_f32(ov.x))),
                   fmaxf(fabsf(bf16lo_to_f32(ov.y)), fabsf(bf16hi_to_f32(ov.y))));
    }
  }
  if (amax_out != nullptr) {
    amax = warp_max(amax);
    if (lane == 0 && amax > 0.0f) atomicMax(reinterpret_cast<unsigned int*>(amax_out), __float_as_uint(amax));
  }
}

extern "C" int h3b_qk_rmsnorm_rope(void* q, void* k, int64_t s, int64_t heads, int64_t seq_stride,
                                   int64_t head_stride, const void* q_weight, const void* k_weight, float eps,
                                   const float* pos, int64_t pos_offset, const float* inv_freq, int n_t, int n_h,
                                   h3b_stream_t stream) {
  if (q == nullptr || q_weight == nullptr || pos == nullptr || inv_freq == nullptr) return H3B_ERR_ARG;
  if (k != nullptr && k_weight == nullptr) return H3B_ERR_ARG;
  if (s < 0 || heads <= 0 || n_t < 0 || n_h < 0 || n_t + n_h > 64 || pos_offset < 0) return H3B_ERR_SHAPE;
  if ((seq_stride % 4) != 0 || (head_stride % 4) != 0) return H3B_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(q) & 7u) || (k != nullptr && (reinterpret_cast<uintptr_t>(k) & 7u)))
    return H3B_ERR_ALIGN;
  if (s == 0) return H3B_OK;
  if (heads > 65535) return H3B_ERR_SHAPE;
  const int64_t blocks = (s + 7) / 8;  // one warp per token
  if (blocks > 0x7fffffff) return H3B_ERR_SHAPE;
  qk_rmsnorm_rope_kernel<<<static_cast<unsigned>(blocks), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(k), s, static_cast<int>(heads), seq_stride,
      head_stride, static_cast<const __nv_bfloat16*>(q_weight), static_cast<const __nv_bfloat16*>(k_weight), eps,
      pos, pos_offset, inv_freq, n_t, n_h);
  return h3b::launch_status();
}

extern "C" int h3b_rmsnorm_modulate(const void* x, void* h, int64_t m, int64_t hidden, int64_t ld, const void* w,
                                    const void* shift, const void* scale, int64_t tab_ld, const int32_t* row_sel,
                                    float eps, float* amax_out, h3b_stream_t stream) {
  if (x == nullptr || h == nullptr || w == nullptr || shift == nullptr || scale == nullptr) return H3B_ERR_ARG;
  if (m < 0 || hidden <= 0 || (hidden % 8) != 0 || ld < hidden || (ld % 8) != 0 || m > 0x7fffffff)
    return H3B_ERR_SHAPE;
  if (!h3b::aligned16(x) || !h3b::aligned16(h) || !h3b::aligned16(w) || !h3b::aligned16(shift) ||
      !h3b::aligned16(scale) || tab_ld < 0 || (tab_ld % 8) != 0)
    return H3B_ERR_ALIGN;
  if (m == 0) return H3B_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  auto* hb = static_cast<__nv_bfloat16*>(h);
  const auto* wb = static_cast<const __nv_bfloat16*>(w);
  const auto* sh = static_cast<const __nv_bfloat16*>(shift);
  const auto* sc = static_cast<const __nv_bfloat16*>(scale);
  const int64_t nvec = hidden / 8;
  // rows up to 3072 wide: 128-thread CTAs, 8 resident per SM, each with one
  // row in work and the next one loading; the grid is one resident wave
  const bool narrow = nvec <= 128 * 3;
  int64_t blocks = static_cast<int64_t>(h3b::num_sms()) * 8;
  if (blocks > m) blocks = m;
  const unsigned g = static_cast<unsigned>(blocks);
  if (narrow)
    rmsnorm_modulate_kernel<128, 3><<<g, 128, 0, st>>>(xb, hb, m, hidden, ld, wb, sh, sc, tab_ld, row_sel, eps,
                                                       amax_out);
  else if (nvec <= 256 * 8)
    rmsnorm_modulate_kernel<256, 8><<<g, 256, 0, st>>>(xb, hb, m, hidden, ld, wb, sh, sc, tab_ld, row_sel, eps,
                                                       amax_out);
  else
    return H3B_ERR_SHAPE;
  return h3b::launch_status();
}

extern "C" int h3b_gate_residual(void* x, const void* y, int64_t m, int64_t hidden, int64_t ld, const void* gate,
                                 int64_t tab_ld, const int32_t* row_sel, h3b_stream_t stream) {
  if (x == nullptr || y == nullptr || gate == nullptr) return H3B_ERR_ARG;
  if (m < 0 || hidden <= 0 || (hidden % 8) != 0 || ld < hidden || (ld % 8) != 0) return H3B_ERR_SHAPE;
  if (tab_ld < 0 || (tab_ld % 8) != 0) return H3B_ERR_ALIGN;
  if (!h3b::aligned16(x) || !h3b::aligned16(y) || !h3b::aligned16(gate)) return H3B_ERR_ALIGN;
  if (m == 0) return H3B_OK;
  int64_t blocks = (m * (hidden / 8) + 255) / 256;
  const int64_t cap = static_cast<int64_t>(h3b::num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  gate_residual_kernel<<<static_cast<unsigned>(blocks), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(y), m, hidden, ld,
      static_cast<const __nv_bfloat16*>(gate), tab_ld, row_sel);
  return h3b::launch_status();
}

extern "C" int h3b_attention_merge_lse(float* acc, float* acc_lse, const void* blk, const float* blk_lse, int64_t s,
                                       int64_t heads, int first, void* out, float* amax_out, h3b_stream_t stream) {
  if (acc == nullptr || acc_lse == nullptr || blk == nullptr || blk_lse == nullptr) return H3B_ERR_ARG;
  if (s < 0 || heads <= 0) return H3B_ERR_SHAPE;
  if (!h3b::aligned16(acc) || !h3b::aligned16(blk) || (out != nullptr && !h3b::aligned16(out))) return H3B_ERR_ALIGN;
  if (s == 0) return H3B_OK;
  int64_t blocks = (s * heads + 7) / 8;
  const int64_t cap = static_cast<int64_t>(h3b::num_sms()) * 16;
  if (blocks > cap) blocks = cap;
  merge_lse_kernel<<<static_cast<unsigned>(blocks), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      acc, acc_lse, static_cast<const __nv_bfloat16*>(blk), blk_lse, s, heads, first,
      static_cast<__nv_bfloat16*>(out), amax_out);
  return h3b::launch_status();
}
