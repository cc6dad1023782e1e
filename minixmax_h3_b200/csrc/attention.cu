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
//   warp 8      TMA producer: Q0/Q1 once, K through a 2-deep ring, V through
//               a 3-deep ring (one release wait per K/V tile covers both)
//   warp 9      TMEM allocator + MMA issuer (the warp polls together, one
//               elected lane issues)
//   warps 10-11 idle (complete the third warpgroup for setmaxnreg)
// TMEM (512 columns): S0 | S1 | O0 | O1, 128 fp32 columns each.  The softmax
// writes P as packed bf16 into the first 64 columns of the S region it read,
// and P.V reads it straight from TMEM (tcgen05.mma with the A operand in
// TMEM), so P never touches shared memory.
// MMA issue order: S0(0) S1(0) PV0(0), then per K/V tile j >= 1:
//   S0(j)  PV1(j-1)  S1(j)  PV0(j)        (and PV1(n-1) at the end)
// so the tensor pipe always holds the other tile's work while a softmax runs.
// S_i(j) is issued right behind PV_i(j-1), which reads P_i(j-1) from the same
// columns: the tcgen05.mma stream of one thread executes in order, so the
// write cannot overtake the read.  The commit after S_i(j) also covers
// PV_i(j-1), so when a softmax sees S_i(j) ready, O_i is settled.
// The issuing thread sits on each tile's critical path (softmax -> P.V ->
// S -> softmax), so it commits three times per K/V tile: S_0(j+1) ready,
// S_1(j+1) ready, and kv_free(j) right behind S_0(j+1) (it covers every MMA
// issued before), which releases K_j (both S MMAs read it) and V_{j-1} (both
// P.V MMAs read it); S_0(j+1) follows PV_0(j) in straight-line code.  The
// final commit publishes both O tiles.
// After the first K/V tile a softmax exponentiates half 0 against its
// running max while it finds the tile's row max on the ALU alongside; only a
// row whose max outgrew the running max by more than the threshold sends
// its warp back to reload S from TMEM (P has not been written over it yet)
// and rescale first.
// The row max is rescaled lazily: O and the row sum are corrected only when
// the running max grows by more than 8 (log2 domain), which bounds P by 2^8.
// Head->sequence scatter (h3b_attention_fwd_head2seq, the Ulysses exchange
// of ops/ulysses.py:32-41 fused into the epilogue): query row t of local head
// h is written to rank t / s_local's out-projection input [s_local, H, 128]
// at row t % s_local, global head head0 + h, through that rank's buffer
// pointer (this GPU's own or a peer's, mapped by CUDA IPC).
// Q/K tiles are K-major and V tiles MN-major, all with the 128-byte swizzle,
// loaded by non-multicast TMA from any (seq, head) strides.  Every wait is
// bounded, and every parity wait is at most one phase behind its barrier
// (the argument is given at each wait).
#include "h3b_common.cuh"
#include "h3b_host.hpp"

H3B_DECLARE_STATUS();
H3B_REGISTER_STATUS_READER(attention);

namespace {

constexpr int D = 128;
constexpr int BQ = 128;    // rows per Q tile (one softmax warpgroup)
constexpr int BKV = 128;   // rows per K/V tile
constexpr int KST = 2;     // K ring depth
constexpr int VST = 3;     // V ring depth: V_j's slot is free at kv_free(j-2), like K_j's
constexpr int Q_TILE_BYTES = BQ * D * 2;        // 32 KB: two 16 KB boxes (d 0-63, 64-127)
constexpr int Q_HALF_BYTES = Q_TILE_BYTES / 2;
constexpr int KV_TILE_BYTES = BKV * D * 2;      // 32 KB: two 16 KB boxes
constexpr int KV_HALF_BYTES = KV_TILE_BYTES / 2;
constexpr int THREADS = 384;  // 3 warpgroups: softmax Q0, softmax Q1, load/MMA
// Register split (setmaxnreg): launched at 168/thread (384 x 168 = 64512); the
// load/MMA warpgroup drops to 56 and the two softmax warpgroups rise to 224:
// 4*32*56 + 8*32*224 = 64512, exactly the launch allocation.
constexpr int REGS_LOADER = 88;
constexpr int REGS_SOFTMAX = 208;
static_assert(4 * 32 * REGS_LOADER + 8 * 32 * REGS_SOFTMAX <= THREADS * 168, "register split exceeds launch");
constexpr float RESCALE_THRESHOLD = 8.0f;

constexpr uint32_t IDESC_S = idesc_bf16_f32(128, BKV, 0, 0);  // Q (K-major) x K^T (K-major)
constexpr uint32_t IDESC_O = idesc_bf16_f32(128, D, 0, 1);    // P (TMEM) x V (MN-major)

// TMEM column of S_i (P_i in its first 64 columns) and of O_i.
__host__ __device__ constexpr uint32_t s_col(int i) { return static_cast<uint32_t>(i * 128); }
__host__ __device__ constexpr uint32_t o_col(int i) { return static_cast<uint32_t>(256 + i * 128); }

struct __align__(8) Bars {
  uint64_t q_full;
  uint64_t k_full[KST];
  uint64_t v_full[VST];
  uint64_t kv_free[2];     // [j % 2]: K_j and V_{j-1} no longer read (tcgen05.commit behind S_0(j+1))
  uint64_t s_full[2];      // [tile]: S_i(j) ready (tcgen05.commit)
  uint64_t p_half[2][2];   // [tile][half]: P_i(j) columns 64h..64h+63 written (one arrival per softmax warp)
  uint64_t o_done;         // both O tiles final (one phase; tcgen05.commit after the last P.V)
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(KST == 2 && VST == 3, "the producer's single kv_free wait per tile assumes these ring depths");

constexpr size_t SMEM_BYTES = 1024 + 2 * Q_TILE_BYTES + KST * KV_TILE_BYTES + VST * KV_TILE_BYTES + sizeof(Bars);

constexpr int MAX_PEERS = 8;

struct AttnArgs {
  __nv_bfloat16* o;
  __nv_bfloat16* o_peers[MAX_PEERS];  // head->seq scatter destinations (peer_mode)
  int peer_mode;
  int o_wide;  // every destination and both strides 32-byte aligned: 32-byte row stores
  int s_local;
  int head0;
  float* lse;
  float* amax_out;
  int64_t o_seq_stride;
  int64_t o_head_stride;
  int s_q;
  int s_kv;
  float scale_log2;
};

// Every lane polls the barrier (one shared state, so one verdict per poll);
// the vote keeps the warp's view uniform in every case.
template <bool SPIN = false>
H3B_DEV bool warp_wait(uint64_t* bar, uint32_t parity, int site, volatile int* abort_flag) {
  const bool ok = mbar_wait<SPIN>(bar, parity, &g_status, site, abort_flag);
  return __all_sync(0xffffffffu, ok);
}

H3B_DEV float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Row max of one 64-column S tile: 8 independent chains of three-input max
// (MASK: columns >= valid of the last K/V tile are padding).
template <bool MASK>
H3B_DEV float row_max64(const uint32_t* r, int valid) {
  auto v = [&](int e) { return (!MASK || e < valid) ? __uint_as_float(r[e]) : -INFINITY; };
  float mx[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) mx[c] = fmax3(v(c), v(c + 8), v(c + 16));
#pragma unroll
  for (int e = 24; e < 64; e += 16) {
#pragma unroll
    for (int c = 0; c < 8; ++c) mx[c] = fmax3(mx[c], v(e + c), e + 8 + c < 64 ? v(e + 8 + c) : -INFINITY);
  }
  return fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
}

// 2^x on the FMA pipe for a pair of lanes (FA4-style MUFU offload), from
// Cody-Waite range reduction and a polynomial:
//   x = n + f with n = round(x) (via the 1.5*2^23 magic add), f in [-1/2, 1/2]
//   2^f ~= c0 + f(c1 + f(c2 + f c3)), a degree-3 fit of 2^f on [-1/2, 1/2]
//        made for this kernel (relative-error weighted least squares on
//        Chebyshev nodes, refined toward equi-ripple): max relative error
//        7.5e-5, far below the 2^-9 rounding of the bf16 P it feeds
//   2^x = 2^f * 2^n by adding n to the exponent field.
// x is clamped to >= -125 so the exponent add cannot underflow (2^-125 is
// zero for every downstream use); x <= 9 holds by the lazy-rescale bound.
H3B_DEV float2 exp2_poly2(float2 x) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  constexpr float c0 = 0.99992805719f, c1 = 0.69326102734f, c2 = 0.24261114001f, c3 = 0.05517161265f;
  x.x = fmaxf(x.x, -125.0f);
  x.y = fmaxf(x.y, -125.0f);
  const float2 t = add2(x, make_float2(kMagic, kMagic));         // round(x) in the low mantissa bits
  const float2 n = add2(t, make_float2(-kMagic, -kMagic));        // round(x) as a float (exact)
  const float2 f = add2(x, make_float2(-n.x, -n.y));              // f in [-1/2, 1/2]
  float2 p = fma2(make_float2(c3, c3), f, make_float2(c2, c2));
  p = fma2(p, f, make_float2(c1, c1));
  p = fma2(p, f, make_float2(c0, c0));
  // t's bit pattern is 0x4B400000 + n; shifting it left by 23 leaves n << 23.
  const uint32_t bx = __float_as_uint(p.x) + (__float_as_uint(t.x) << 23);
  const uint32_t by = __float_as_uint(p.y) + (__float_as_uint(t.y) << 23);
  return make_float2(__uint_as_float(bx), __uint_as_float(by));
}

// Pairs (out of every 8) whose exponentials go to the FMA pipe instead of
// MUFU.  Measured on B200 at S = 32768..131072: 0 -> 1131 / 1074 TFLOP/s,
// 1 -> 1122 / 1057, 2 -> 1107 / -, 3 -> 1060 / 1020 (24 heads); the
// softmax's FMA and ALU work already fills those pipes, MUFU has room.
constexpr int POLY_PAIRS_PER_8 = 0;

// In-place softmax numerator for 64 columns r[0..63] (fp32 S bits in, packed
// bf16 P out in dst[0..31]): packed fp32x2 FMA, 64 independent exponentials
// (split between MUFU ex2 and the FMA-pipe polynomial), then pack and packed
// sums.  dst may alias r (dst[e] is written after r[2e], r[2e+1] are read,
// and e <= 2e).  Returns the partial row sum.  With MAX, the raw max of all
// 128 columns r[0..127] is found alongside (r[0..63] read before they are
// overwritten, r[64..127] untouched), so the ALU max work runs under the MUFU
// work; it is returned in .y.
template <bool MASK, bool MAX = false>
H3B_DEV float2 exp_pack64(uint32_t* r, uint32_t* dst, int valid, float scale_log2, float neg_m) {
  const float2 sc = make_float2(scale_log2, scale_log2);
  const float2 nm = make_float2(neg_m, neg_m);
  float mx[8];
  if constexpr (MAX) {
#pragma unroll
    for (int c = 0; c < 8; ++c) mx[c] = -INFINITY;
  }
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const float sa = (!MASK || 2 * e < valid) ? __uint_as_float(r[2 * e]) : -INFINITY;
    const float sb = (!MASK || 2 * e + 1 < valid) ? __uint_as_float(r[2 * e + 1]) : -INFINITY;
    if constexpr (MAX) {
      mx[e & 7] = fmax3(mx[e & 7], sa, sb);
      mx[e & 7] = fmax3(mx[e & 7], __uint_as_float(r[64 + 2 * e]), __uint_as_float(r[64 + 2 * e + 1]));
    }
    float2 x = fma2(make_float2(sa, sb), sc, nm);
    if ((e & 7) < POLY_PAIRS_PER_8) {
      x = exp2_poly2(x);
    } else {
      x.x = fast_exp2(x.x);
      x.y = fast_exp2(x.y);
    }
    r[2 * e] = __float_as_uint(x.x);
    r[2 * e + 1] = __float_as_uint(x.y);
  }
  float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const float2 p = make_float2(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]));
    acc[e & 3] = add2(acc[e & 3], p);
    dst[e] = pack_bf16x2(p.x, p.y);
  }
  const float2 t = add2(add2(acc[0], acc[1]), add2(acc[2], acc[3]));
  float m = 0.0f;
  if constexpr (MAX) m = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
  return make_float2(t.x + t.y, m);
}

// 12 warps = 3 per SM sub-partition: launched at 168 registers per thread,
// then rebalanced with setmaxnreg (see REGS_LOADER / REGS_SOFTMAX).
__global__ void __launch_bounds__(THREADS, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                            // Q0 | Q1
  uint8_t* sK = sQ + 2 * Q_TILE_BYTES;           // K ring
  uint8_t* sV = sK + KST * KV_TILE_BYTES;        // V ring
  Bars* bars = reinterpret_cast<Bars*>(sV + VST * KV_TILE_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int head = blockIdx.y;
  const int q0 = blockIdx.x * (2 * BQ);
  const int n_kv = (args.s_kv + BKV - 1) / BKV;
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < KST; ++s) mbar_init(&bars->k_full[s], 1);
    for (int s = 0; s < VST; ++s) mbar_init(&bars->v_full[s], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->kv_free[i], 1);
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_half[i][0], 4);  // one arrival per softmax warp
      mbar_init(&bars->p_half[i][1], 4);
    }
    mbar_init(&bars->o_done, 1);
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

  if (warp >= 8) {
    // ------------------------------------------------------------ load / MMA warpgroup
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REGS_LOADER));
  if (warp == 8) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      mbar_arrive_expect_tx(&bars->q_full, 2 * Q_TILE_BYTES);
      for (int t = 0; t < 2; ++t)
        for (int h = 0; h < 2; ++h)
          tma_load_3d(sQ + t * Q_TILE_BYTES + h * Q_HALF_BYTES, &tm_q, h * 64, q0 + t * BQ, head,
                      &bars->q_full);
      bool ok = true;
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j < n_kv && ok; ++j) {
        // K_j reuses K_{j-2}'s slot and V_j reuses V_{j-3}'s: both were
        // released by kv_free(j-2), phase (j-2)/2 of kv_free[j % 2].  Its next
        // phase, kv_free(j), needs K_j and V_j, so the wait is at most one
        // phase behind.
        if (j >= 2 && !mbar_wait(&bars->kv_free[j & 1], ((j - 2) >> 1) & 1, &g_status, 1, abort_flag)) {
          ok = false;
          break;
        }
        const int ks = j % KST;
        mbar_arrive_expect_tx(&bars->k_full[ks], KV_TILE_BYTES);
        for (int h = 0; h < 2; ++h)
          tma_load_3d(sK + ks * KV_TILE_BYTES + h * KV_HALF_BYTES, &tm_k, h * 64, j * BKV, head,
                      &bars->k_full[ks]);
        issued_k = j + 1;
        const int vs = j % VST;
        mbar_arrive_expect_tx(&bars->v_full[vs], KV_TILE_BYTES);
        for (int h = 0; h < 2; ++h)
          tma_load_3d(sV + vs * KV_TILE_BYTES + h * KV_HALF_BYTES, &tm_v, h * 64, j * BKV, head,
                      &bars->v_full[vs]);
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
    // The whole warp runs the schedule converged: every lane polls each
    // barrier (without a suspend hint: this is the latency-critical hand-off
    // from the softmax back to the tensor pipe) and the verdict is a vote,
    // every lane computes the descriptors, and one elected lane issues each
    // batch of tcgen05.mma and its commit.
    bool ok = warp_wait<true>(&bars->q_full, 0, 3, abort_flag);
    tc_fence_after();
    // k_full[j % 2] completes once per use of the slot; its next phase is
    // K_{j+2}, loaded only after kv_free(j), which this warp commits later
    // (behind S_0(j+1)): one phase behind.  Likewise v_full[j % 3] (next:
    // V_{j+3}, after kv_free(j+1)).  K_{j+1} is waited for in iteration j,
    // after kv_free(j-1) released the slot it is loaded into.
    auto wait_k = [&](int j) -> bool {
      if (!warp_wait<true>(&bars->k_full[j % KST], (j / KST) & 1, 4, abort_flag)) return false;
      tc_fence_after();
      return true;
    };
    auto wait_v = [&](int j) -> bool {
      if (!warp_wait<true>(&bars->v_full[j % VST], (j / VST) & 1, 6, abort_flag)) return false;
      tc_fence_after();
      return true;
    };
    auto commit = [&](uint64_t* bar) {
      if (elect_one()) tc_commit(bar);
      __syncwarp();
    };
    // S_i = Q_i K_j^T (fresh accumulator), then publish it.  K-major Q/K
    // tiles advance 32 bytes (encoded 2) per 16-wide K step inside a
    // 64-column half and a half tile (16 KB) every 4 steps: a descriptor
    // step moves only the start-address field (desc_add_lo).
    auto issue_s = [&](int i, int j) {
      const uint32_t d = tmem + s_col(i);
      const uint64_t qd = sdesc_kmajor_sw128(smem_u32(sQ + i * Q_TILE_BYTES));
      const uint64_t kd = sdesc_kmajor_sw128(smem_u32(sK + (j % KST) * KV_TILE_BYTES));
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t step = static_cast<uint32_t>((kk >> 2) * (Q_HALF_BYTES >> 4) + (kk & 3) * 2);
          mma_f16_ss(d, desc_add_lo(qd, step), desc_add_lo(kd, step), IDESC_S, kk > 0);
        }
        tc_commit(&bars->s_full[i]);
      }
      __syncwarp();
    };
    // O_i (+)= P_i(j) V_j once the softmax has written P_i(j).  Each
    // p_half[i][h] completes once per tile; the softmax cannot arrive for
    // j+1 before S_i(j+1), which is issued after these waits, so each wait
    // is one phase behind.  P is published in two halves (K/V rows 0-63,
    // 64-127) so the first half of P.V runs while the softmax computes the
    // second.  The MN-major V tile advances 2048 bytes per 16 keys.
    auto issue_pv = [&](int i, int j) -> bool {
      const uint32_t p_tmem = tmem + s_col(i);
      const uint32_t o_tmem = tmem + o_col(i);
      const uint64_t vd = sdesc_mnmajor_sw128(smem_u32(sV + (j % VST) * KV_TILE_BYTES), KV_HALF_BYTES, 1024);
      for (int h = 0; h < 2; ++h) {
        if (!warp_wait<true>(&bars->p_half[i][h], j & 1, 7, abort_flag)) return false;
        tc_fence_after();
        if (elect_one()) {
#pragma unroll
          for (int kk = 4 * h; kk < 4 * h + 4; ++kk)
            mma_f16_ts(o_tmem, p_tmem + kk * 8, desc_add_lo(vd, static_cast<uint32_t>(kk * (2048 >> 4))),
                       IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
        }
        __syncwarp();
      }
      return true;
    };
    ok = ok && wait_k(0);
    if (ok) {
      issue_s(0, 0);
      issue_s(1, 0);
    }
    ok = ok && wait_v(0) && (n_kv == 1 || wait_k(1)) && issue_pv(0, 0);
    for (int j = 1; j < n_kv && ok; ++j) {
      issue_s(0, j);                    // behind PV0(j-1) in the pipe
      commit(&bars->kv_free[(j - 1) & 1]);  // K_{j-1} and V_{j-2} no longer read
      if (!issue_pv(1, j - 1)) {        // PV1(j-1)
        ok = false;
        break;
      }
      issue_s(1, j);                    // behind PV1(j-1)
      if (!wait_v(j) || (j + 1 < n_kv && !wait_k(j + 1)) || !issue_pv(0, j)) {
        ok = false;
        break;
      }
    }
    if (ok && issue_pv(1, n_kv - 1)) commit(&bars->o_done);
    commit(&bars->drain);
    warp_wait(&bars->drain, 0, 8, nullptr);
  }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REGS_SOFTMAX));
    const int wg = warp >> 2;                  // Q tile 0 / 1
    const int quad = warp & 3;
    const int row = quad * 32 + lane;          // row within the Q tile
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t o_tmem = tmem + o_col(wg) + lane_off;
    float m_run = -INFINITY;  // running max, log2 domain (already scaled)
    float l_run = 0.0f;
    bool ok = true;
    const uint32_t s_tmem = tmem + s_col(wg) + lane_off;
    for (int j = 0; j < n_kv; ++j) {
      // s_full[wg] completes once per tile; the MMA cannot publish S(j+1)
      // before P(j) is written below, so this wait is one phase behind.
      // (polled without a suspend hint: +0.8 % against a hinted wait)
      if (!warp_wait<true>(&bars->s_full[wg], j & 1, 20, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int valid = args.s_kv - j * BKV;  // columns >= valid are padding
      const bool full = valid >= BKV;  // uniform across the warp (same tile)
      // One TMEM round trip: all 128 columns in flight, one wait.
      uint32_t r[128];
      auto load_s = [&]() {
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32p(s_tmem + c * 32, r + 32 * c);
        tmem_wait_fence<4>(r);
        if (!full) {  // last K/V tile only (warp-uniform): padding columns -> -inf
#pragma unroll
          for (int e = 0; e < 128; ++e)
            if (e >= valid) r[e] = __float_as_uint(-INFINITY);
        }
      };
      load_s();
      // After the first tile, half 0 is exponentiated against the running
      // max straight away and the tile's max is found alongside.  Only if a
      // row's max exceeds the running max by more than the threshold (rare
      // after the first tiles) does the warp reload S from TMEM — P has not
      // been written over it yet — and take the rescaling path.
      float m_use = m_run;
      float sum = 0.0f;
      bool slow = j == 0;
      if (!slow) {
        const float2 sm = exp_pack64<false, true>(r, r, BKV, args.scale_log2, -m_run);
        slow = __any_sync(0xffffffffu, sm.y * args.scale_log2 > m_run + RESCALE_THRESHOLD);
        if (slow) {
          load_s();
        } else {
          sum = sm.x;
        }
      }
      if (slow) {
        const float row_max = fmaxf(row_max64<false>(r, BKV), row_max64<false>(r + 64, BKV));
        const float m_tile = row_max * args.scale_log2;
        bool rescale = false;
        if (m_tile > m_run + RESCALE_THRESHOLD) {
          m_use = m_tile;
          rescale = true;
        }
        // O correction first: O must be rescaled before P_i(j).V starts.  It
        // runs warp-uniformly: tcgen05.ld/st are .sync.aligned and warp_wait
        // shuffles over the full warp, so a per-row branch here would
        // deadlock the warp.  Rows that need no rescale use factor 1.
        if (__any_sync(0xffffffffu, rescale)) {
          const float factor = rescale ? fast_exp2(m_run - m_use) : 1.0f;  // 0 on the first tile
          l_run = l_run * factor;
          if (j > 0) {
            // O_i holds P.V of tiles < j: the commit that published S_i(j)
            // also covered PV_i(j-1), and PV_i(j) waits for P_i(j) below.
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              uint32_t o[32];
              tmem_ld32p(o_tmem + c * 32, o);
              tmem_wait_fence<1>(o);
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * factor);
              tmem_st32(o_tmem + c * 32, o);
            }
          }
          if (rescale) m_run = m_use;
        }
        sum = exp_pack64<false>(r, r, BKV, args.scale_log2, -m_use).x;
      }
      // P = exp2(s*scale - m) as packed bf16, published half by half: half h
      // (K/V rows 64h..64h+63) lands in columns 32h..32h+31 over S columns
      // already consumed.
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (h == 1) sum += exp_pack64<false>(r + 64, r + 32, BKV, args.scale_log2, -m_use).x;
        tmem_st32(s_tmem + 32 * h, *reinterpret_cast<uint32_t(*)[32]>(r + 32 * h));
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_half[wg][h]);
      }
      l_run += sum;
    }
    // ---- epilogue: O / l -> bf16 rows once the last P.V of both tiles is
    // complete (o_done has a single phase).
    if (ok && warp_wait(&bars->o_done, 0, 23, abort_flag)) {
      tc_fence_after();
      const int q_row = q0 + wg * BQ + row;
      const float inv_l = 1.0f / l_run;
      float o_amax = 0.0f;
      __nv_bfloat16* orow;
      if (args.peer_mode) {
        const int dst = q_row < args.s_q ? q_row / args.s_local : 0;
        orow = args.o_peers[dst] + static_cast<int64_t>(q_row - dst * args.s_local) * args.o_seq_stride +
               static_cast<int64_t>(args.head0 + head) * args.o_head_stride;
      } else {
        orow = args.o + static_cast<int64_t>(q_row) * args.o_seq_stride +
               static_cast<int64_t>(head) * args.o_head_stride;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32p(o_tmem + c * 32, r);
        tmem_wait_fence<1>(r);
        if (q_row < args.s_q && args.o_wide) {
#pragma unroll
          for (int e = 0; e < 32; e += 16) {
            uint32_t w[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              w[t] = pack_bf16x2(__uint_as_float(r[e + 2 * t]) * inv_l, __uint_as_float(r[e + 2 * t + 1]) * inv_l);
              o_amax = fmaxf(o_amax, fmaxf(fabsf(bf16lo_to_f32(w[t])), fabsf(bf16hi_to_f32(w[t]))));
            }
            st_global_v8(orow + c * 32 + e, w);
          }
        } else if (q_row < args.s_q) {
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
      if (args.peer_mode) __threadfence_system();  // peer writes visible system-wide
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

namespace {

int launch_attention(const void* q, const void* k, const void* v, AttnArgs a, int64_t heads, int64_t s_q,
                     int64_t s_kv, int64_t q_seq_stride, int64_t q_head_stride, int64_t kv_seq_stride,
                     int64_t kv_head_stride, float scale, cudaStream_t stream) {
  if (q == nullptr || k == nullptr || v == nullptr) return H3B_ERR_ARG;
  if (heads <= 0 || s_q < 0 || s_kv <= 0 || heads > 65535 || s_q > (1ll << 30) || s_kv > (1ll << 30))
    return H3B_ERR_SHAPE;
  if (!(scale > 0.0f)) return H3B_ERR_ARG;
  const int64_t strides[6] = {q_seq_stride, q_head_stride, kv_seq_stride, kv_head_stride, a.o_seq_stride,
                              a.o_head_stride};
  for (int64_t st : strides)
    if (st <= 0 || (st % 8) != 0) return H3B_ERR_ALIGN;
  if (!h3b::aligned16(q) || !h3b::aligned16(k) || !h3b::aligned16(v)) return H3B_ERR_ALIGN;
  if (s_q == 0) return H3B_OK;  // no query rows: nothing to write
  CUtensorMap tq, tk, tv;
  int rc = h3b::encode_3d(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, q, D, s_q, heads, q_seq_stride * 2,
                          q_head_stride * 2, 64, BQ, 1, CU_TENSOR_MAP_SWIZZLE_128B);
  static_assert(BKV % 16 == 0 && BKV <= 256, "K/V tile rows");
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
  a.s_q = static_cast<int>(s_q);
  a.s_kv = static_cast<int>(s_kv);
  a.scale_log2 = scale * 1.4426950408889634f;
  dim3 grid(static_cast<unsigned>((s_q + 2 * BQ - 1) / (2 * BQ)), static_cast<unsigned>(heads));
  attention_kernel<<<grid, THREADS, SMEM_BYTES, stream>>>(tq, tk, tv, a);
  return h3b::launch_status();
}

// 32-byte output stores need every destination base 32-byte aligned and both
// strides (elements) multiples of 16; row offsets within a head are 32-value
// chunks, so every store address is then 32-byte aligned.
int wide_rows_ok(void* const* bufs, int64_t n, int64_t seq_stride, int64_t head_stride) {
  for (int64_t r = 0; r < n; ++r)
    if ((reinterpret_cast<uintptr_t>(bufs[r]) & 31u) != 0) return 0;
  return (seq_stride % 16 == 0 && head_stride % 16 == 0) ? 1 : 0;
}

}  // namespace

extern "C" int h3b_attention_fwd(const void* q, const void* k, const void* v, void* o, float* lse, float* amax_out,
                                 int64_t heads,
                                 int64_t s_q, int64_t s_kv, int64_t q_seq_stride, int64_t q_head_stride,
                                 int64_t kv_seq_stride, int64_t kv_head_stride, int64_t o_seq_stride,
                                 int64_t o_head_stride, float scale, h3b_stream_t stream) {
  if (o == nullptr) return H3B_ERR_ARG;
  if (!h3b::aligned16(o)) return H3B_ERR_ALIGN;
  AttnArgs a{};
  a.o = static_cast<__nv_bfloat16*>(o);
  a.lse = lse;
  a.amax_out = amax_out;
  a.o_seq_stride = o_seq_stride;
  a.o_head_stride = o_head_stride;
  a.o_wide = wide_rows_ok(&o, 1, o_seq_stride, o_head_stride);
  return launch_attention(q, k, v, a, heads, s_q, s_kv, q_seq_stride, q_head_stride, kv_seq_stride, kv_head_stride,
                          scale, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int h3b_attention_fwd_head2seq(const void* q, const void* k, const void* v, void* const* o_bufs,
                                          int64_t world_size, int64_t s_local, int64_t head0, int64_t o_seq_stride,
                                          int64_t o_head_stride, float* amax_out, int64_t heads, int64_t s_q,
                                          int64_t s_kv, int64_t q_seq_stride, int64_t q_head_stride,
                                          int64_t kv_seq_stride, int64_t kv_head_stride, float scale,
                                          h3b_stream_t stream) {
  if (o_bufs == nullptr) return H3B_ERR_ARG;
  if (world_size < 1 || world_size > MAX_PEERS || s_local <= 0 || s_q != world_size * s_local || head0 < 0)
    return H3B_ERR_SHAPE;
  AttnArgs a{};
  for (int64_t r = 0; r < world_size; ++r) {
    if (o_bufs[r] == nullptr) return H3B_ERR_ARG;
    if (!h3b::aligned16(o_bufs[r])) return H3B_ERR_ALIGN;
    a.o_peers[r] = static_cast<__nv_bfloat16*>(o_bufs[r]);
  }
  a.o = a.o_peers[0];
  a.peer_mode = 1;
  a.s_local = static_cast<int>(s_local);
  a.head0 = static_cast<int>(head0);
  a.amax_out = amax_out;
  a.o_seq_stride = o_seq_stride;
  a.o_head_stride = o_head_stride;
  a.o_wide = wide_rows_ok(o_bufs, world_size, o_seq_stride, o_head_stride);
  return launch_attention(q, k, v, a, heads, s_q, s_kv, q_seq_stride, q_head_stride, kv_seq_stride, kv_head_stride,
                          scale, reinterpret_cast<cudaStream_t>(stream));
}
