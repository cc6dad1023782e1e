// Non-causal flash attention forward (head_dim 128, bf16) on tcgen05.
//
// Replaces the reference's attention entry points (ops/fa_h3.py:224-304
// h3_attention_bnsd, ops/attention.py:100-131 fusion_attention_bnsd), whose
// host path is softmax(q k^T * scale) v via SDPA.
//
// One CTA = one head x 256 query rows (two 128-row tiles Q0, Q1), looping
// over all 128-row K/V tiles of that head:
//   warps 0-3   softmax for Q0 (thread = query row = TMEM lane)
//   warps 4-7   softmax for Q1
//   warp 8      TMA producer: Q0/Q1 once, K and V through 2-deep rings
//   warp 9      TMEM allocator + single-thread MMA issuer
// TMEM (512 columns): S0 | S1 | O0 | O1, 128 fp32 columns each.  The softmax
// writes P as packed bf16 into the first 64 columns of its S region and the
// P.V product reads it straight from TMEM (tcgen05.mma with the A operand in
// TMEM), so P never touches shared memory.  The row max is rescaled lazily:
// O and the row sum are corrected only when the running max grows by more
// than 8 (log2 domain), which bounds P by 2^8.
// Q/K tiles are K-major and V tiles MN-major, all with the 128-byte swizzle,
// loaded by non-multicast TMA from any (seq, head) strides.  Every wait is
// bounded.
#include "h3b_common.cuh"
#include "h3b_host.hpp"

H3B_DECLARE_STATUS();
H3B_REGISTER_STATUS_READER(attention);

namespace {

constexpr int D = 128;
constexpr int BQ = 128;    // rows per Q tile (one softmax warpgroup)
constexpr int BKV = 128;   // rows per K/V tile
constexpr int KST = 2;     // K ring depth
constexpr int VST = 2;     // V ring depth
constexpr int TILE_BYTES = 128 * D * 2;  // 32 KB: two 16 KB swizzle boxes (d 0-63, 64-127)
constexpr int HALF_BYTES = TILE_BYTES / 2;
constexpr int THREADS = 320;
constexpr float RESCALE_THRESHOLD = 8.0f;

constexpr uint32_t IDESC_S = idesc_bf16_f32(128, BKV, 0, 0);  // Q (K-major) x K^T (K-major)
constexpr uint32_t IDESC_O = idesc_bf16_f32(128, D, 0, 1);    // P (TMEM) x V (MN-major)

struct __align__(8) Bars {
  uint64_t q_full;
  uint64_t k_full[KST];
  uint64_t k_empty[KST];
  uint64_t v_full[VST];
  uint64_t v_empty[VST];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t pv_done[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};

constexpr size_t SMEM_BYTES = 1024 + 2 * TILE_BYTES + KST * TILE_BYTES + VST * TILE_BYTES + sizeof(Bars);

struct AttnArgs {
  __nv_bfloat16* o;
  float* lse;
  float* amax_out;
  int64_t o_seq_stride;
  int64_t o_head_stride;
  int s_q;
  int s_kv;
  float scale_log2;
};

H3B_DEV bool warp_wait(uint64_t* bar, uint32_t parity, int site, volatile int* abort_flag) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, &g_status, site, abort_flag) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

H3B_DEV float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(THREADS, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                           // Q0 | Q1
  uint8_t* sK = sQ + 2 * TILE_BYTES;            // K ring
  uint8_t* sV = sK + KST * TILE_BYTES;          // V ring
  Bars* bars = reinterpret_cast<Bars*>(sV + VST * TILE_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int q0 = blockIdx.x * (2 * BQ);
  const int n_kv = (args.s_kv + BKV - 1) / BKV;
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < KST; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], 128);
      mbar_init(&bars->pv_done[i], 1);
    }
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      mbar_arrive_expect_tx(&bars->q_full, 2 * TILE_BYTES);
      for (int t = 0; t < 2; ++t)
        for (int h = 0; h < 2; ++h)
          tma_load_3d(sQ + t * TILE_BYTES + h * HALF_BYTES, &tm_q, h * 64, q0 + t * BQ, head, &bars->q_full);
      bool ok = true;
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int ks = j % KST;
        if (j >= KST && !mbar_wait(&bars->k_empty[ks], ((j / KST) - 1) & 1, &g_status, 1, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&bars->k_full[ks], TILE_BYTES);
        for (int h = 0; h < 2; ++h)
          tma_load_3d(sK + ks * TILE_BYTES + h * HALF_BYTES, &tm_k, h * 64, j * BKV, head, &bars->k_full[ks]);
        issued_k = j + 1;
        const int vs = j % VST;
        if (j >= VST && !mbar_wait(&bars->v_empty[vs], ((j / VST) - 1) & 1, &g_status, 2, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&bars->v_full[vs], TILE_BYTES);
        for (int h = 0; h < 2; ++h)
          tma_load_3d(sV + vs * TILE_BYTES + h * HALF_BYTES, &tm_v, h * 64, j * BKV, head, &bars->v_full[vs]);
        issued_v = j + 1;
      }
      if (!ok || *abort_flag) {
        // Drain the copies still in flight (bounded) before the CTA exits.
        mbar_wait(&bars->q_full, 0, &g_status, 10, nullptr);
        for (int j = issued_k - KST > 0 ? issued_k - KST : 0; j < issued_k; ++j)
          mbar_wait(&bars->k_full[j % KST], (j / KST) & 1, &g_status, 11, nullptr);
        for (int j = issued_v - VST > 0 ? issued_v - VST : 0; j < issued_v; ++j)
          mbar_wait(&bars->v_full[j % VST], (j / VST) & 1, &g_status, 12, nullptr);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(&bars->q_full, 0, &g_status, 3, abort_flag);
      tc_fence_after();
      const uint32_t q_addr[2] = {smem_u32(sQ), smem_u32(sQ + TILE_BYTES)};
      for (int j = 0; j < n_kv && ok; ++j) {
        const int ks = j % KST;
        if (!mbar_wait(&bars->k_full[ks], (j / KST) & 1, &g_status, 4, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + ks * TILE_BYTES);
        for (int i = 0; i < 2 && ok; ++i) {
          // S_i aliases P_i of the previous tile: wait until P_i.V has run.
          if (j > 0 && !mbar_wait(&bars->pv_done[i], (j - 1) & 1, &g_status, 5, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t s_tmem = tmem + i * 128;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * HALF_BYTES;
            const uint64_t ad = sdesc_kmajor_sw128(q_addr[i] + off) + (kk & 3) * 2;
            const uint64_t bd = sdesc_kmajor_sw128(k_addr + off) + (kk & 3) * 2;
            mma_f16_ss(s_tmem, ad, bd, IDESC_S, kk > 0);
          }
          tc_commit(&bars->s_full[i]);
        }
        if (!ok) break;
        tc_commit(&bars->k_empty[ks]);
        const int vs = j % VST;
        if (!mbar_wait(&bars->v_full[vs], (j / VST) & 1, &g_status, 6, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t v_addr = smem_u32(sV + vs * TILE_BYTES);
        for (int i = 0; i < 2 && ok; ++i) {
          if (!mbar_wait(&bars->p_full[i], j & 1, &g_status, 7, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t p_tmem = tmem + i * 128;
          const uint32_t o_tmem = tmem + 256 + i * 128;
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk) {
            const uint64_t bd = sdesc_mnmajor_sw128(v_addr + kk * 2048, HALF_BYTES, 1024);
            mma_f16_ts(o_tmem, p_tmem + kk * 8, bd, IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&bars->pv_done[i]);
        }
        if (!ok) break;
        tc_commit(&bars->v_empty[vs]);
      }
      tc_commit(&bars->drain);
      mbar_wait(&bars->drain, 0, &g_status, 8, nullptr);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int wg = warp >> 2;                  // Q tile 0 / 1
    const int quad = warp & 3;
    const int row = quad * 32 + lane;          // row within the Q tile
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t s_tmem = tmem + wg * 128 + lane_off;
    const uint32_t o_tmem = tmem + 256 + wg * 128 + lane_off;
    float m_run = -INFINITY;  // running max, log2 domain (already scaled)
    float l_run = 0.0f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (!warp_wait(&bars->s_full[wg], j & 1, 20, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(s_tmem + c * 32, r);
        tc_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) s[c * 32 + e] = __uint_as_float(r[e]);
      }
      const int valid = args.s_kv - j * BKV;  // columns >= valid are padding
      if (valid < BKV) {
#pragma unroll
        for (int e = 0; e < 128; ++e)
          if (e >= valid) s[e] = -INFINITY;
      }
      float mx = s[0];
#pragma unroll
      for (int e = 1; e < 128; ++e) mx = fmaxf(mx, s[e]);
      const float m_tile = mx * args.scale_log2;
      float m_use = m_run;
      bool rescale = false;
      if (m_tile > m_run + RESCALE_THRESHOLD) {
        m_use = m_tile;
        rescale = true;
      }
      const float neg_m = -m_use;
      float sum = 0.0f;
      uint32_t p[64];
#pragma unroll
      for (int e = 0; e < 64; ++e) {
        const float a = fast_exp2(fmaf(s[2 * e], args.scale_log2, neg_m));
        const float b = fast_exp2(fmaf(s[2 * e + 1], args.scale_log2, neg_m));
        sum += a + b;
        p[e] = pack_bf16x2(a, b);
      }
      // The correction runs warp-uniformly: tcgen05.ld/st are .sync.aligned
      // and warp_wait shuffles over the full warp, so a per-row branch here
      // would deadlock the warp.  Rows that need no rescale use factor 1.
      if (__any_sync(0xffffffffu, rescale)) {
        const float factor = rescale ? fast_exp2(m_run - m_use) : 1.0f;  // 0 on the first tile
        l_run = l_run * factor;
        if (j > 0) {
          // O_i holds P.V of tiles < j: wait for the last one, then scale it.
          if (!warp_wait(&bars->pv_done[wg], (j - 1) & 1, 21, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t r[32];
            tmem_ld32(o_tmem + c * 32, r);
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * factor);
            tmem_st32(o_tmem + c * 32, r);
          }
        }
        if (rescale) m_run = m_use;
      }
      l_run += sum;
      {
        uint32_t lo[32], hi[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          lo[e] = p[e];
          hi[e] = p[32 + e];
        }
        tmem_st32(s_tmem, lo);
        tmem_st32(s_tmem + 32, hi);
      }
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_full[wg]);
    }
    // ---- epilogue: O / l -> bf16 rows
    if (ok && warp_wait(&bars->pv_done[wg], (n_kv - 1) & 1, 22, abort_flag)) {
      tc_fence_after();
      const int q_row = q0 + wg * BQ + row;
      const float inv_l = 1.0f / l_run;
      float o_amax = 0.0f;
      __nv_bfloat16* orow = args.o + static_cast<int64_t>(q_row) * args.o_seq_stride +
                            static_cast<int64_t>(head) * args.o_head_stride;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(o_tmem + c * 32, r);
        tc_wait_ld();
        if (q_row < args.s_q) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 v;
            v.x = pack_bf16x2(__uint_as_float(r[e]) * inv_l, __uint_as_float(r[e + 1]) * inv_l);
            v.y = pack_bf16x2(__uint_as_float(r[e + 2]) * inv_l, __uint_as_float(r[e + 3]) * inv_l);
            v.z = pack_bf16x2(__uint_as_float(r[e + 4]) * inv_l, __uint_as_float(r[e + 5]) * inv_l);
            v.w = pack_bf16x2(__uint_as_float(r[e + 6]) * inv_l, __uint_as_float(r[e + 7]) * inv_l);
            *reinterpret_cast<uint4*>(orow + c * 32 + e) = v;
            const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int t = 0; t < 4; ++t)
              o_amax = fmaxf(o_amax, fmaxf(fabsf(bf16lo_to_f32(w4[t])), fabsf(bf16hi_to_f32(w4[t]))));
          }
        }
      }
      if (args.amax_out != nullptr) {
        const float wmax = warp_max(o_amax);
        if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(args.amax_out), __float_as_uint(wmax));
      }
      if (args.lse != nullptr && q_row < args.s_q) {
        args.lse[static_cast<int64_t>(head) * args.s_q + q_row] = (m_run + __log2f(l_run)) * 0.69314718055994531f;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

extern "C" int h3b_attention_fwd(const void* q, const void* k, const void* v, void* o, float* lse, float* amax_out,
                                 int64_t heads,
                                 int64_t s_q, int64_t s_kv, int64_t q_seq_stride, int64_t q_head_stride,
                                 int64_t kv_seq_stride, int64_t kv_head_stride, int64_t o_seq_stride,
                                 int64_t o_head_stride, float scale, h3b_stream_t stream) {
  if (q == nullptr || k == nullptr || v == nullptr || o == nullptr) return H3B_ERR_ARG;
  if (heads <= 0 || s_q <= 0 || s_kv <= 0 || heads > 65535 || s_q > (1ll << 30) || s_kv > (1ll << 30))
    return H3B_ERR_SHAPE;
  if (!(scale > 0.0f)) return H3B_ERR_ARG;
  const int64_t strides[6] = {q_seq_stride, q_head_stride, kv_seq_stride, kv_head_stride, o_seq_stride,
                              o_head_stride};
  for (int64_t st : strides)
    if (st <= 0 || (st % 8) != 0) return H3B_ERR_ALIGN;
  if (!h3b::aligned16(q) || !h3b::aligned16(k) || !h3b::aligned16(v) || !h3b::aligned16(o)) return H3B_ERR_ALIGN;
  CUtensorMap tq, tk, tv;
  int rc = h3b::encode_3d(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, q, D, s_q, heads, q_seq_stride * 2,
                          q_head_stride * 2, 64, BQ, 1, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc == H3B_OK)
    rc = h3b::encode_3d(&tk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, k, D, s_kv, heads, kv_seq_stride * 2,
                        kv_head_stride * 2, 64, BKV, 1, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc == H3B_OK)
    rc = h3b::encode_3d(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, v, D, s_kv, heads, kv_seq_stride * 2,
                        kv_head_stride * 2, 64, BKV, 1, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != H3B_OK) return rc;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(SMEM_BYTES)) != cudaSuccess)
      return H3B_ERR_LAUNCH;
    attr = true;
  }
  AttnArgs a;
  a.o = static_cast<__nv_bfloat16*>(o);
  a.lse = lse;
  a.amax_out = amax_out;
  a.o_seq_stride = o_seq_stride;
  a.o_head_stride = o_head_stride;
  a.s_q = static_cast<int>(s_q);
  a.s_kv = static_cast<int>(s_kv);
  a.scale_log2 = scale * 1.4426950408889634f;
  dim3 grid(static_cast<unsigned>((s_q + 2 * BQ - 1) / (2 * BQ)), static_cast<unsigned>(heads));
  attention_kernel<<<grid, THREADS, SMEM_BYTES, reinterpret_cast<cudaStream_t>(stream)>>>(tq, tk, tv, a);
  return h3b::launch_status();
}
