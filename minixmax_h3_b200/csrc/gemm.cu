// Quantised GEMMs of the DiT-block linears on 5th-generation tensor cores.
//
//   INT8  (W8A8):  kind::i8, int32 accumulators in TMEM, epilogue
//                  y = acc * xs[m] * ws[n] (+ bias[n])  — the semantics of
//                  torch_npu.npu_quant_matmul at ops/int8_convrot.py:86-93.
//   NVFP4 (W4A4):  kind::mxf4nvf4.block_scale.block16, e2m1 operands with one
//                  ue4m3 scale per 16 elements written into TMEM by
//                  scale-writer warps, epilogue y = acc * a_gs * w_gs (+ bias[n]).
//
// Structure (persistent, one CTA per SM; every GEMM with M > 128 works in
// clusters of two CTAs on 256 x BN tiles with cta_group::2 MMAs; M <= 128
// keeps single-CTA 128 x BN tiles):
//   warp 0      TMA producer: this CTA's 128 rows of A, its BN/PAIR rows of B
//               (+ scale factors) into a 4-, 5- or 6-deep smem ring.  In a
//               pair, both CTAs' A/B copies complete on the leader's full
//               barrier, which only the leader arms (for both CTAs' bytes);
//               NVFP4 scale bytes land on each CTA's own sf_ready barrier.
//   warp 1      TMEM allocator; in the leader (the only CTA of a single-CTA
//               launch) the MMA issuer: the warp polls the barriers
//               together, one elected lane issues.  tcgen05.commit (to
//               both CTAs of a pair) releases smem slots and publishes
//               finished accumulators.
//   epilogue    8 warps (2-9; 8-15 in an NVFP4 pair) for this CTA's 128
//               accumulator rows, two per TMEM lane quadrant (a warp reaches
//               only the lanes of quadrant warp % 4) taking alternate
//               32-column chunks: tcgen05.ld 32x32b (one output row per
//               thread), fp32 dequant/bias and GELU / SwiGLU / gate-residual /
//               seq->head scatter, bf16 blocks staged in 64B-swizzled shared
//               memory and written by TMA stores; each warp releases the
//               accumulator to the leader.  (With one warp per quadrant, a
//               GELU or gate-residual epilogue outlasted the MMAs of a
//               K = 3072 tile.)  Each epilogue mode is its own kernel instance.
//   writers     (NVFP4) scale writers (warps 10-17 single-CTA, two per TMEM
//               lane quadrant on alternate slabs; warps 4-7 in a pair, one per
//               quadrant): each loads its slab's scales from shared memory into
//               registers, stores them into its 32 TMEM lanes with tcgen05.st
//               and arrives on the slab's full barrier (the leader's, in a
//               pair), so the MMA thread waits once per slab and issues
//               nothing but MMAs.  (With one single-CTA writer per quadrant,
//               the ones sharing a scheduler with the producer or the MMA
//               thread fell a slab behind and paced the pipe.)
// The issuing lane is the MMA pipe's feeder: a block-scaled MMA
// takes ~55-75 cycles to issue, a commit ~60-75 and a barrier poll ~80, so 4
// NVFP4 MMAs of 128x192x64 per 384-cycle slab leave it no room for the 12
// scale copies (tcgen05.cp, ~45 cycles of issue each) a slab would need.
// Accumulators in TMEM:
//   INT8:        BN = 256, two accumulators (columns 0 and 256), so the MMAs
//                of tile t+1 run while the epilogue drains tile t.
//   NVFP4 1-CTA: BN = 192, two accumulators (0, 192), plus two 48-column
//                scale slots at columns 384 and 432 (slab it uses slot it&1;
//                the writers refill it once the MMAs of slab it-2 have
//                completed, seen through that slab's empty barrier).
//   NVFP4 pair:  BN = 256, one accumulator (0-255), five scale slots at
//                256 + 48s (slab it uses slot it % 5, refilled after the MMAs
//                of slab it-5); the epilogue reads its whole share into
//                registers and releases the accumulator before computing.
//   A slot holds, per K-step j, 4 columns of A scales (the four-quadrant image
//   of the blocked 128x4 atom: lane 32q+b, column 4j+a = scales of row 32a+b)
//   and 8 columns of B scales (column 8j+i = scales of tile rows 32i+b in
//   every quadrant).  In a pair each CTA holds the A scales of its own rows
//   and the B scales of all 256 tile rows.
// Operands are K-major with the 128-byte swizzle.  No load uses cluster
// multicast.  Every wait is bounded; both CTAs of a pair stay resident until
// a final cluster barrier.
#include "h3b_common.cuh"
#include "h3b_host.hpp"

H3B_DECLARE_STATUS();
H3B_REGISTER_STATUS_READER(gemm);

namespace {

constexpr int BM = 128;       // accumulator rows per CTA (TMEM lanes)
constexpr int MAX_STAGES = 6;
constexpr int A_BYTES = BM * 128;  // one 128-byte K slab of A
constexpr int SFA_BYTES = 2048;    // 128 rows x 16 scales (4 blocked chunks)
constexpr int SFB_BYTES = 4096;    // two 128-row blocks x 16 scales
constexpr int EPI_THREADS = 256;  // two epilogue warps per TMEM lane quadrant
constexpr int EPI_WARPS = EPI_THREADS / 32;
constexpr int OUT_STAGE_BYTES = 32 * 64;  // one warp's 32 rows x 32 bf16 staging buffer
constexpr int SF_SLOT_COLS = 48;          // 16 (A: 4 K-steps x 4) + 32 (B: 4 K-steps x 8)

enum Kind { KIND_I8 = 0, KIND_NVF4 = 1 };
enum OutMode { OUT_BF16 = 0, OUT_I32 = 1, OUT_SEQ2HEAD = 2 };
// Epilogue specialisation of a kernel instance: the activation (H3B_EPI_*)
// or the output form.  Each mode is its own instance so a kernel carries
// only the epilogue code it runs (runtime selection among all of them left
// every instance's code large enough to cost ~6 % in instruction fetch).
enum EpiMode { EM_STORE = 0, EM_GELU = 1, EM_GATE_RES = 2, EM_SWIGLU = 3, EM_I32 = 4, EM_SEQ2HEAD = 5 };
template <int EM>
struct EpiOf {
  static constexpr int epilogue = EM <= EM_SWIGLU ? EM : H3B_EPI_STORE;  // H3B_EPI_* values
  static constexpr int out_mode = EM == EM_I32 ? OUT_I32 : (EM == EM_SEQ2HEAD ? OUT_SEQ2HEAD : OUT_BF16);
};

constexpr int MAX_PEERS = 8;
struct PeerMaps {
  CUtensorMap m[MAX_PEERS];  // per destination rank (OUT_SEQ2HEAD)
};

struct GemmArgs {
  const float* xs;     // i8: per-row activation scale [m]
  const float* ws;     // i8: per-column weight scale [n]
  const float* a_gs;   // nvf4: activation global scale (device scalar)
  const float* w_gs;   // nvf4: weight global scale (device scalar)
  const uint8_t* a_sf; // nvf4: blocked scales of A
  const uint8_t* w_sf; // nvf4: blocked scales of B
  const __nv_bfloat16* bias;
  const __nv_bfloat16* resid;
  const __nv_bfloat16* gate;  // [rows, gate_ld] adaLN gate table
  const int32_t* row_sel;     // per output row: gate table row (NULL = 0, < 0 = keep resid)
  float* amax_out;            // optional max |y|
  int64_t gate_ld;
  void* y;
  int64_t ldy;
  int m, n, k;         // k in elements
  int epilogue;
  int out_mode;
  int heads_per_rank;  // OUT_SEQ2HEAD: H / world_size
  int hd;              // OUT_SEQ2HEAD: H * 128 (columns per q|k|v part)
  int no_loads;        // wait self-test: the producer issues nothing (h3b_selftest_wait_timeout)
  int amax_signed;     // amax_out receives max(0, max y) instead of max |y| (H3B_EPI_STORE_POSMAX)
};

// PAIR = 1: one CTA per 128 x BN tile.  PAIR = 2: a cluster of two CTAs per
// 256 x BN tile with cta_group::2 MMAs issued by the leader (rank 0): each
// CTA stages its 128 rows of A and BN/2 rows of B, and holds its 128 rows of
// the accumulator, so each SM moves half as much B through shared memory.
//
// NVFP4 pairs (256 x 256 tiles) exist for shared-memory bandwidth: a 128x192
// FP4 tile at full MMA rate reads ~107 B/clk of operands from shared memory
// while TMA writes as many, against ~128 B/clk per SM; a pair's 128 rows of
// A plus 128 of B per SM need half of that per FLOP, and its 4 MMAs per slab
// take 512 cycles instead of 384, which leaves the issuing lane room.
// Two 256-column accumulators would fill TMEM, so an NVFP4 pair has one: the
// epilogue reads its whole share into registers (184 per thread through
// setmaxnreg) and releases it before computing, and five scale slots let
// the writers run up to five slabs ahead of the MMAs.
template <int KIND, int PAIR, int EM = EM_STORE>
struct Cfg {
  static constexpr bool NVF4_PAIR = KIND == KIND_NVF4 && PAIR == 2;
  static constexpr int BN = (KIND == KIND_I8 || PAIR == 2) ? 256 : 192;  // MMA N
  static constexpr int B_ROWS = BN / PAIR;                 // B rows staged by this CTA
  static constexpr int B_BYTES = B_ROWS * 128;
  static constexpr int STAGES = PAIR == 1 ? 4 : (NVF4_PAIR ? 5 : 6);
  static constexpr int NACC = NVF4_PAIR ? 1 : 2;  // TMEM accumulators (double-buffered unless NVF4_PAIR)
  static constexpr int ACC_STRIDE = BN;        // TMEM columns between the accumulators
  static constexpr int SF_BASE = NACC * BN;    // NVFP4 scale slots follow the accumulators
  static constexpr int SF_SLOTS = NVF4_PAIR ? 5 : 2;  // NVFP4 scale slots in TMEM, one K slab each
  static constexpr int SF_WPQ = NVF4_PAIR ? 1 : 2;    // NVFP4 scale writer warps per TMEM lane quadrant
  static constexpr int OUT_BUFS = 2;                   // epilogue staging buffers per warp (32x32 bf16 each)
  static_assert(EM >= EM_STORE && EM <= EM_SEQ2HEAD, "epilogue mode");
  static constexpr int TMEM_COLS = 512;
  static constexpr int SF_STAGE_BYTES = KIND == KIND_NVF4 ? SFA_BYTES + SFB_BYTES : 0;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SF_STAGE_BYTES;
  // The leader's full barrier counts both CTAs' A and B bytes (and, for
  // NVFP4, one scale writer per quadrant of each CTA); scale bytes land on
  // each CTA's own sf_ready.
  static constexpr int TX_BYTES = PAIR * (A_BYTES + B_BYTES);
  static constexpr int FULL_ARRIVALS = KIND == KIND_NVF4 ? 1 + 4 * PAIR : 1;  // the arm + the writers
  // Warp roles: 0 TMA producer, 1 TMEM allocator + MMA issuer, then the
  // epilogue and (NVFP4) the scale writers.  An NVFP4 pair aligns roles to
  // warpgroups for setmaxnreg: warps 2-3 idle, 4-7 writers, 8-15 epilogue.
  static constexpr int EPI_WARP0 = NVF4_PAIR ? 8 : 2;
  static constexpr int SF_WARP0 = NVF4_PAIR ? 4 : 2 + EPI_WARPS;
  static constexpr int SF_WARPS = KIND == KIND_NVF4 ? 4 * SF_WPQ : 0;
  static constexpr int THREADS = NVF4_PAIR ? 512 : 64 + EPI_THREADS + 32 * SF_WARPS;
  static constexpr int K_PER_STAGE = KIND == KIND_I8 ? 128 : 256;  // elements per 128-byte slab
  static constexpr uint32_t IDESC = KIND == KIND_I8 ? idesc_s8_s32(BM * PAIR, BN) : idesc_nvf4(BM * PAIR, BN);
  static_assert(STAGES <= MAX_STAGES, "barrier arrays");
  static_assert(NACC * ACC_STRIDE <= TMEM_COLS, "accumulators exceed TMEM");
  static_assert(KIND == KIND_I8 || SF_BASE + SF_SLOTS * SF_SLOT_COLS <= TMEM_COLS, "scale slots exceed TMEM");
  // A writer waits for slab it - SF_SLOTS to release its slot on that slab's
  // empty barrier; with SF_SLOTS <= STAGES that barrier cannot have moved on
  // by another phase before this writer's own later arrival.
  static_assert(KIND == KIND_I8 || SF_SLOTS <= STAGES, "scale slot reuse needs a stage per slot");
  static_assert(STAGE_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "SW128 tiles need 1024-byte alignment");
};

// NVFP4 pair register split (setmaxnreg per warpgroup): launched at 128 per
// thread (512 x 128), the control warpgroup (producer, MMA, two idle warps)
// and the scale writers drop to 72, and the two epilogue warpgroups rise to
// 184 so each epilogue thread can hold its 128 accumulator columns.  (With
// the control warpgroup at 56 and the epilogue at 192 the issuer's loop
// spilled: 4-16 % slower on store and gate-residual epilogues.)
constexpr int PAIR_LAUNCH_REGS = 128;
constexpr int REGS_CTL = 72;
constexpr int REGS_SFW = 72;
constexpr int REGS_EPI = 184;
static_assert(4 * REGS_CTL + 4 * REGS_SFW + 8 * REGS_EPI <= 16 * PAIR_LAUNCH_REGS, "register split exceeds launch");

// TMEM column of NVFP4 scale slot `slot` (A scales at +4j, B scales at
// +16+8j for K-step j).
template <int KIND, int PAIR, int EM>
H3B_DEV uint32_t sf_slot_col(int slot) {
  return static_cast<uint32_t>(Cfg<KIND, PAIR, EM>::SF_BASE + slot * SF_SLOT_COLS);
}

struct __align__(8) Barriers {
  uint64_t full[MAX_STAGES];
  uint64_t empty[MAX_STAGES];
  uint64_t sf_ready[MAX_STAGES];  // NVFP4: the scale bytes of stage s landed in shared memory
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
  int consumed;  // k-slabs whose full barrier the MMA thread has observed
};

template <int KIND, int PAIR, int EM = EM_STORE>
constexpr size_t smem_bytes() {
  using C = Cfg<KIND, PAIR, EM>;
  return 1024 /*alignment slack*/ + static_cast<size_t>(C::STAGES) * C::STAGE_BYTES +
         EPI_WARPS * C::OUT_BUFS * OUT_STAGE_BYTES + sizeof(Barriers);
}
static_assert(smem_bytes<KIND_I8, 2>() <= 227 * 1024 && smem_bytes<KIND_NVF4, 1>() <= 227 * 1024 &&
                  smem_bytes<KIND_I8, 1>() <= 227 * 1024 && smem_bytes<KIND_NVF4, 2>() <= 227 * 1024 &&
                  smem_bytes<KIND_NVF4, 2, EM_SEQ2HEAD>() <= 227 * 1024 && smem_bytes<KIND_I8, 2, EM_SEQ2HEAD>() <= 227 * 1024,
              "shared memory budget");

// Every lane polls the barrier (one shared state, so one verdict per poll);
// the vote keeps the warp's view uniform in every case.  (A lane-0 poll
// with the verdict shuffled to the others cost the attention kernel 5 %.)
template <bool SPIN = false, bool CLUSTER = false>
H3B_DEV bool warp_wait(uint64_t* bar, uint32_t parity, int site, volatile int* abort_flag) {
  const bool ok = mbar_wait<SPIN, CLUSTER>(bar, parity, &g_status, site, abort_flag);
  return __all_sync(0xffffffffu, ok);
}

// Byte offset of 16-byte chunk c of row r in a 32-row x 64-byte staging
// buffer in the TMA 64-byte swizzle (address bits 4-5 ^= bits 7-8).  The
// buffer must be 512-byte aligned.
H3B_DEV uint32_t swz64(int r, int c) { return static_cast<uint32_t>(r * 64 + ((c ^ ((r >> 1) & 3)) << 4)); }

template <int KIND, int PAIR, int EM>
__global__ void __launch_bounds__(Cfg<KIND, PAIR, EM>::THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                const __grid_constant__ CUtensorMap tmap_y, const __grid_constant__ PeerMaps peers,
                const GemmArgs args) {
  using C = Cfg<KIND, PAIR, EM>;
  constexpr int BN = C::BN;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sSFA = sB + STAGES * C::B_BYTES;             // used by KIND_NVF4 only
  uint8_t* sSFB = sSFA + STAGES * SFA_BYTES;
  uint8_t* sOut = smem + STAGES * C::STAGE_BYTES;       // 4 warps x 2 staging buffers, 1024-aligned
  Barriers* bars = reinterpret_cast<Barriers*>(sOut + EPI_WARPS * C::OUT_BUFS * OUT_STAGE_BYTES);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR == 2 ? cluster_ctarank() : 0u;  // CTA within the pair; 0 = leader
  const bool leader = rank == 0;
  const int cluster = static_cast<int>(blockIdx.x) / PAIR, n_clusters = static_cast<int>(gridDim.x) / PAIR;
  const int m_tiles = (args.m + BM * PAIR - 1) / (BM * PAIR);
  const int n_tiles = (args.n + BN - 1) / BN;
  const int num_tiles = m_tiles * n_tiles;
  const int nk = args.k / C::K_PER_STAGE;
  volatile int* abort_flag = &bars->abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->full[s], C::FULL_ARRIVALS);
      mbar_init(&bars->empty[s], 1);
      mbar_init(&bars->sf_ready[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->acc_full[b], 1);
      mbar_init(&bars->acc_empty[b], EPI_WARPS * PAIR);  // one arrival per epilogue warp of each CTA
    }
    mbar_init(&bars->drain, 1);
    bars->abort_flag = 0;
    bars->consumed = 0;
    fence_barrier_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
    prefetch_tmap(&tmap_y);
  }
  if (warp == 1) {
    if constexpr (PAIR == 2) {
      tmem_alloc_pair(&bars->tmem_base, C::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&bars->tmem_base, C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (PAIR == 2) {
    cluster_sync();  // both CTAs' barriers initialised before any cross-CTA signal
  } else {
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  // Under NVF4_PAIR each role branch opens with its warpgroup's setmaxnreg
  // (one static instruction per warpgroup, executed by all of its warps).
  if (warp < (C::NVF4_PAIR ? 4 : 2)) {
   if constexpr (C::NVF4_PAIR) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REGS_CTL));
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // (no_loads: nothing is issued, so no copy is ever in flight and the
    // consumers' first waits can only run out)
    if (lane == 0 && !args.no_loads) {
      int it = 0;
      bool ok = true;
      for (int tile = cluster; tile < num_tiles && ok; tile += n_clusters) {
        const int mt = tile / n_tiles, nt = tile % n_tiles;
        const int m0 = (mt * PAIR + static_cast<int>(rank)) * BM;  // this CTA's A rows
        const int n0 = nt * BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          const int round = it / STAGES;
          if (round > 0 && !mbar_wait(&bars->empty[s], (round - 1) & 1, &g_status, 1, abort_flag)) {
            ok = false;
            break;
          }
          if constexpr (PAIR == 2) {
            // Both CTAs' copies complete on the leader's full[s]; only the
            // leader arms it, for the pair's bytes.
            const uint32_t full_l = mapa_shared(smem_u32(&bars->full[s]), 0);
            if (leader) mbar_arrive_expect_tx(&bars->full[s], C::TX_BYTES);
            tma_load_2d_pair(sA + s * A_BYTES, &tmap_a, kb * 128, m0, full_l);
            tma_load_2d_pair(sB + s * C::B_BYTES, &tmap_b, kb * 128, n0 + static_cast<int>(rank) * C::B_ROWS,
                             full_l);
            if constexpr (KIND == KIND_NVF4) {
              // This CTA's scales land in its own shared memory (own
              // sf_ready): the A block of its 128 rows and both 128-row B
              // blocks of the 256-row tile.  A block or a second B block past
              // the last one is replaced by the tile's first (in bounds; the
              // rows or columns it would scale are never stored).
              const int64_t ncb = args.k / 64;
              const int a_blocks = (args.m + BM - 1) / BM;
              const int ab = mt * 2 + static_cast<int>(rank) < a_blocks ? mt * 2 + static_cast<int>(rank) : mt * 2;
              const int nb0 = n0 / 128;
              const int nb1 = (nb0 + 1) * 128 < args.n ? nb0 + 1 : nb0;
              mbar_arrive_expect_tx(&bars->sf_ready[s], C::SF_STAGE_BYTES);
              bulk_load(sSFA + s * SFA_BYTES, args.a_sf + ((static_cast<int64_t>(ab) * ncb) + kb * 4) * 512,
                        SFA_BYTES, &bars->sf_ready[s]);
              bulk_load(sSFB + s * SFB_BYTES, args.w_sf + ((static_cast<int64_t>(nb0) * ncb) + kb * 4) * 512,
                        SFB_BYTES / 2, &bars->sf_ready[s]);
              bulk_load(sSFB + s * SFB_BYTES + SFB_BYTES / 2,
                        args.w_sf + ((static_cast<int64_t>(nb1) * ncb) + kb * 4) * 512, SFB_BYTES / 2,
                        &bars->sf_ready[s]);
            }
            continue;
          }
          mbar_arrive_expect_tx(&bars->full[s], C::TX_BYTES);
          tma_load_2d(sA + s * A_BYTES, &tmap_a, kb * 128, m0, &bars->full[s]);
          tma_load_2d(sB + s * C::B_BYTES, &tmap_b, kb * 128, n0, &bars->full[s]);
          if constexpr (KIND == KIND_NVF4) {
            const int64_t ncb = args.k / 64;  // 64-element scale groups per row
            const uint8_t* sfa = args.a_sf + ((static_cast<int64_t>(mt) * ncb) + kb * 4) * 512;
            // The 128-row scale blocks that cover rows n0 .. n0+191.  Past the
            // last block the first is reloaded (in bounds; those output
            // columns are never stored).
            const int nb0 = n0 / 128;
            const int nb1 = (nb0 + 1) * 128 < args.n ? nb0 + 1 : nb0;
            const uint8_t* sfb0 = args.w_sf + ((static_cast<int64_t>(nb0) * ncb) + kb * 4) * 512;
            const uint8_t* sfb1 = args.w_sf + ((static_cast<int64_t>(nb1) * ncb) + kb * 4) * 512;
            mbar_arrive_expect_tx(&bars->sf_ready[s], C::SF_STAGE_BYTES);
            bulk_load(sSFA + s * SFA_BYTES, sfa, SFA_BYTES, &bars->sf_ready[s]);
            bulk_load(sSFB + s * SFB_BYTES, sfb0, SFB_BYTES / 2, &bars->sf_ready[s]);
            bulk_load(sSFB + s * SFB_BYTES + SFB_BYTES / 2, sfb1, SFB_BYTES / 2, &bars->sf_ready[s]);
          }
        }
      }
      if (!ok || *abort_flag) {
        if (leader) {
          // Drain: wait (bounded) for every slab issued but not yet consumed,
          // so no copy is still writing this CTA's shared memory at exit.
          const int consumed = *reinterpret_cast<volatile int*>(&bars->consumed);
          for (int j = consumed; j < it; ++j) {
            if constexpr (KIND == KIND_NVF4) {
              // full[] also counts the writers' arrivals: wait for the
              // scale bytes, then give the A/B copies a bounded 200 us.
              mbar_wait(&bars->sf_ready[j % STAGES], (j / STAGES) & 1, &g_status, 9, nullptr);
            } else {
              mbar_wait(&bars->full[j % STAGES], (j / STAGES) & 1, &g_status, 9, nullptr);
            }
          }
          if constexpr (KIND == KIND_NVF4) {
            const uint64_t t0 = globaltimer_ns();
            while (globaltimer_ns() - t0 < 200000ull) {
            }
          }
        } else {
          // The peer's copies complete on the leader's barriers, which it
          // cannot wait on: give its copies in flight a bounded 200 us to
          // land (both CTAs stay resident until the final cluster barrier).
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 200000ull) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // (the leader only under PAIR = 2: its MMAs fill both CTAs' TMEM).  The
    // whole warp runs the loop converged: every lane polls the barriers and
    // computes the descriptors, one elected lane issues each slab's MMAs and
    // commit.  Against a lone issuing lane: INT8 +3 %, NVFP4 GELU epilogue
    // +12 %, gate-residual +4 %.
    if (leader) {
      int it = 0;
      int local = 0;
      // stage, its phase and the scale slot of slab `it`, kept as running
      // counters (no division per slab in this latency-critical loop)
      int s = 0, ph = 0, slot = 0;
      bool ok = true;
      for (int tile = cluster; tile < num_tiles && ok; tile += n_clusters, ++local) {
        const int buf = local % C::NACC;
        const int use = local / C::NACC;
        if (use > 0 && !warp_wait<false, PAIR == 2>(&bars->acc_empty[buf], (use - 1) & 1, 2, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * C::ACC_STRIDE;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          if (!warp_wait<true>(&bars->full[s], static_cast<uint32_t>(ph), 3, abort_flag)) {
            ok = false;
            break;
          }
          if (lane == 0) *reinterpret_cast<volatile int*>(&bars->consumed) = it + 1;
          tc_fence_after();
          const uint64_t adesc = sdesc_kmajor_sw128(smem_u32(sA + s * A_BYTES));
          const uint64_t bdesc = sdesc_kmajor_sw128(smem_u32(sB + s * C::B_BYTES));
          if (elect_one()) {
            if constexpr (KIND == KIND_I8) {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                if constexpr (PAIR == 2)
                  mma_i8_ss_pair(d_tmem, adesc + 2 * j, bdesc + 2 * j, C::IDESC, (kb | j) != 0);
                else
                  mma_i8_ss(d_tmem, adesc + 2 * j, bdesc + 2 * j, C::IDESC, (kb | j) != 0);
              }
            } else {
              // full[s] also means: this slab's scales are in TMEM slot it % SF_SLOTS
              const uint32_t sf_col = tmem_base + sf_slot_col<KIND, PAIR, EM>(slot);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                if constexpr (PAIR == 2)
                  mma_nvf4_ss_pair(d_tmem, adesc + 2 * j, bdesc + 2 * j, C::IDESC, sf_col + j * 4,
                                   sf_col + 16 + j * 8, (kb | j) != 0);
                else
                  mma_nvf4_ss(d_tmem, adesc + 2 * j, bdesc + 2 * j, C::IDESC, sf_col + j * 4,
                              sf_col + 16 + j * 8, (kb | j) != 0);
              }
            }
            // stage reusable (in both CTAs) once these MMAs have read it
            if constexpr (PAIR == 2)
              tc_commit_pair_mc(&bars->empty[s], 0x3);
            else
              tc_commit(&bars->empty[s]);
          }
          __syncwarp();
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
          if (++slot == C::SF_SLOTS) slot = 0;
        }
        if (!ok) break;
        if (elect_one()) {
          if constexpr (PAIR == 2)  // accumulator complete in both CTAs
            tc_commit_pair_mc(&bars->acc_full[buf], 0x3);
          else
            tc_commit(&bars->acc_full[buf]);
        }
        __syncwarp();
      }
      // Drain all MMAs this warp issued before TMEM is released.
      if (elect_one()) {
        if constexpr (PAIR == 2)
          tc_commit_pair(&bars->drain);
        else
          tc_commit(&bars->drain);
      }
      __syncwarp();
      warp_wait(&bars->drain, 0, 8, nullptr);
    }
  }
  } else if (KIND == KIND_NVF4 && warp >= C::SF_WARP0 && warp < C::SF_WARP0 + C::SF_WARPS) {
    // ------------------------------------------------------ scale writers
   if constexpr (C::NVF4_PAIR) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REGS_SFW));
    // Pair: one writer per quadrant and CTA, every slab, slot it % 5.  Each
    // CTA's TMEM holds the A scales of its own 128 rows (the layout below)
    // and the B scales of the whole 256-row tile: column 16+8j+i = tile rows
    // 32i+b, i < 8, in every quadrant.  The slab's scales are read from
    // shared memory right before they are stored: five slots of lead leave
    // no need to prefetch.  The follower's writers arrive on the leader's
    // full barrier.
    const int quad = warp & 3;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const int my_tiles = cluster < num_tiles ? (num_tiles - 1 - cluster) / n_clusters + 1 : 0;
    const int total = my_tiles * nk;
    bool ok = true;
    for (int it = 0; it < total && ok; ++it) {
      const int s = it % STAGES;
      if (!warp_wait<true>(&bars->sf_ready[s], (it / STAGES) & 1, 7, abort_flag)) {
        ok = false;
        break;
      }
      uint32_t ra[16], rb[32];
      const uint8_t* sfa = sSFA + s * SFA_BYTES + lane * 16;
      const uint8_t* sfb = sSFB + s * SFB_BYTES + lane * 16;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 a4 = *reinterpret_cast<const uint4*>(sfa + j * 512);
        const uint4 b0 = *reinterpret_cast<const uint4*>(sfb + j * 512);
        const uint4 b1 = *reinterpret_cast<const uint4*>(sfb + SFB_BYTES / 2 + j * 512);
        ra[4 * j] = a4.x, ra[4 * j + 1] = a4.y, ra[4 * j + 2] = a4.z, ra[4 * j + 3] = a4.w;
        rb[8 * j] = b0.x, rb[8 * j + 1] = b0.y, rb[8 * j + 2] = b0.z, rb[8 * j + 3] = b0.w;
        rb[8 * j + 4] = b1.x, rb[8 * j + 5] = b1.y, rb[8 * j + 6] = b1.z, rb[8 * j + 7] = b1.w;
      }
      // slot it % 5 was last read by the MMAs of slab it-5
      if (it >= C::SF_SLOTS && !warp_wait<true>(&bars->empty[(it - C::SF_SLOTS) % STAGES],
                                                ((it - C::SF_SLOTS) / STAGES) & 1, 6, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t t = tmem_base + lane_off + sf_slot_col<KIND, PAIR, EM>(it % C::SF_SLOTS);
      tmem_st16(t, ra);
      tmem_st32(t + 16, rb);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(&bars->full[s]);
        else
          mbar_arrive_remote(mapa_shared(smem_u32(&bars->full[s]), 0));
      }
    }
   } else {
    // Warp q writes TMEM lanes 32q..32q+31 of slot it&1 for slab it:
    //   A part, column 4j+a: word a of row b of blocked chunk j (the four
    //     scales of A row 32a+b for K-step j; quadrant q reads column 4j+q);
    //   B part, column 8j+i (i < 6): the scales of tile row 32i+b for K-step
    //     j, the same in every quadrant.  A 192-row tile starts on a 128-row
    //     scale block (even tiles) or 64 rows into one (odd tiles), so tile
    //     row group i is word (g & 3) of block g >> 2, g = i (+2 if odd).
    // The slab's scales are read from shared memory one slab ahead, while
    // the previous slab's stores are in flight.
    // Two warps per quadrant take alternate slabs (slab parity = slot), so
    // a writer that shares its scheduler with the producer or the MMA thread
    // still has two slab periods for each store.
    const int quad = warp & 3;
    const int parity = (warp - 2 - EPI_THREADS / 32) >> 2;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const int my_tiles = cluster < num_tiles ? (num_tiles - 1 - cluster) / n_clusters + 1 : 0;
    const int total = my_tiles * nk;
    uint4 nx[12];  // slab it's scales: A chunks 0-3, then B (block h, chunk j) at 4 + 2j + h
    auto load = [&](int slab) -> bool {
      const int s = slab % STAGES;
      if (!warp_wait<true>(&bars->sf_ready[s], (slab / STAGES) & 1, 7, abort_flag)) return false;
      const uint8_t* sfa = sSFA + s * SFA_BYTES + lane * 16;
      const uint8_t* sfb = sSFB + s * SFB_BYTES + lane * 16;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        nx[j] = *reinterpret_cast<const uint4*>(sfa + j * 512);
        nx[4 + 2 * j] = *reinterpret_cast<const uint4*>(sfb + j * 512);
        nx[5 + 2 * j] = *reinterpret_cast<const uint4*>(sfb + SFB_BYTES / 2 + j * 512);
      }
      return true;
    };
    bool ok = parity < total ? load(parity) : true;
    for (int it = parity; it < total && ok; it += 2) {
      const int tile = cluster + (it / nk) * n_clusters;
      const bool odd = ((tile % n_tiles) & 1) != 0;
      uint32_t ra[16], rb[32];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ra[4 * j] = nx[j].x, ra[4 * j + 1] = nx[j].y, ra[4 * j + 2] = nx[j].z, ra[4 * j + 3] = nx[j].w;
        const uint32_t w[8] = {nx[4 + 2 * j].x, nx[4 + 2 * j].y, nx[4 + 2 * j].z, nx[4 + 2 * j].w,
                               nx[5 + 2 * j].x, nx[5 + 2 * j].y, nx[5 + 2 * j].z, nx[5 + 2 * j].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) rb[8 * j + i] = odd ? (i < 6 ? w[i + 2] : 0u) : w[i];
      }
      // slot it&1 was last read by the MMAs of slab it-2
      if (it >= 2 && !warp_wait<true>(&bars->empty[(it - 2) % STAGES], ((it - 2) / STAGES) & 1, 6, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t t = tmem_base + lane_off + sf_slot_col<KIND, PAIR, EM>(it & 1);
      tmem_st16(t, ra);
      tmem_st32(t + 16, rb);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->full[it % STAGES]);
      if (it + 2 < total) ok = load(it + 2);
    }
   }
  } else if (warp >= C::EPI_WARP0 && warp < C::EPI_WARP0 + EPI_WARPS) {
    // ------------------------------------------------------------ epilogue
    if constexpr (C::NVF4_PAIR) asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REGS_EPI));
    const int quad = warp & 3;              // TMEM lane quadrant this warp may access
    const int row_in_tile = quad * 32 + lane;
    const int half = (warp - C::EPI_WARP0) / 4;  // the quadrant's two warps take alternate 32-column chunks
    uint8_t* out_stage = sOut + (warp - C::EPI_WARP0) * C::OUT_BUFS * OUT_STAGE_BYTES;
    float y_amax = 0.0f;                    // max |y| over every tile this thread stored
    int local = 0;
    int stage_seq = 0;                      // cycles through this warp's staging buffers
    // acc_empty lives in the leader; the peer's warps arrive remotely.
    auto release_acc = [&](int buf) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (C::NVF4_PAIR) {
          if (leader)
            mbar_arrive(&bars->acc_empty[buf]);
          else
            mbar_arrive_remote(mapa_shared(smem_u32(&bars->acc_empty[buf]), 0));
        } else if constexpr (PAIR == 2) {
          mbar_arrive_cluster(mapa_shared(smem_u32(&bars->acc_empty[buf]), 0));
        } else {
          mbar_arrive(&bars->acc_empty[buf]);
        }
      }
    };
    for (int tile = cluster; tile < num_tiles; tile += n_clusters, ++local) {
      const int buf = local % C::NACC;
      const int use = local / C::NACC;
      if (!warp_wait<true>(&bars->acc_full[buf], use & 1, 4, abort_flag)) break;
      tc_fence_after();
      const int m0 = ((tile / n_tiles) * PAIR + static_cast<int>(rank)) * BM;
      const int n0 = (tile % n_tiles) * BN;
      const int row = m0 + row_in_tile;
      const bool row_ok = row < args.m;
      int gate_row = 0;
      if (EpiOf<EM>::epilogue == H3B_EPI_GATE_RES && args.row_sel != nullptr && row_ok) gate_row = args.row_sel[row];
      const __nv_bfloat16* gate_r = args.gate + static_cast<int64_t>(gate_row < 0 ? 0 : gate_row) * args.gate_ld;
      const float gmul = gate_row < 0 ? 0.0f : 1.0f;  // rows outside every segment keep resid
      // 16-byte gate loads when the table and its row pitch allow them
      const bool gate_vec = ((reinterpret_cast<uintptr_t>(args.gate) | static_cast<uintptr_t>(args.gate_ld * 2)) & 15u) == 0;
      float row_scale = 1.0f;
      if constexpr (KIND == KIND_I8) {
        if (EpiOf<EM>::out_mode != OUT_I32 && row_ok) row_scale = args.xs[row];
      } else {
        row_scale = (*args.a_gs) * (*args.w_gs);
      }
      const uint32_t t_row = tmem_base + buf * C::ACC_STRIDE + (static_cast<uint32_t>(quad * 32) << 16);
      // acc -> fp32 output of column `col` before any activation.  Explicit
      // _rn ops: no FMA contraction, so the INT8 epilogue is bit-reproducible
      // as (acc*xs)*ws + bias in fp32.
      auto dequant = [&](uint32_t raw, int col) -> float {
        float a;
        if constexpr (KIND == KIND_I8) {
          a = __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int32_t>(raw)), row_scale), __ldg(args.ws + col));
        } else {
          a = __fmul_rn(__uint_as_float(raw), row_scale);
        }
        if (args.bias != nullptr) a = __fadd_rn(a, __bfloat162float(args.bias[col]));
        return a;
      };
      // dequant of 32 consecutive columns with packed fp32x2 arithmetic (the
      // same roundings as dequant, half the instructions).
      auto dequant32 = [&](const uint32_t* r, int col0, float (&v)[32]) {
        const float2 rs = make_float2(row_scale, row_scale);
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          float2 a;
          if constexpr (KIND == KIND_I8) {
            a = mul2(make_float2(static_cast<float>(static_cast<int32_t>(r[j])),
                                 static_cast<float>(static_cast<int32_t>(r[j + 1]))), rs);
            a = mul2(a, make_float2(__ldg(args.ws + col0 + j), __ldg(args.ws + col0 + j + 1)));
          } else {
            a = mul2(make_float2(__uint_as_float(r[j]), __uint_as_float(r[j + 1])), rs);
          }
          if (args.bias != nullptr)
            a = add2(a, make_float2(__bfloat162float(args.bias[col0 + j]), __bfloat162float(args.bias[col0 + j + 1])));
          v[j] = a.x;
          v[j + 1] = a.y;
        }
      };
      // Stage a 32x32 bf16 block and TMA-store it at output column ocol.  A
      // staging buffer is reused every OUT_BUFS blocks: first wait until at
      // most OUT_BUFS-1 stores (the other buffers') may still be reading
      // shared memory.
      auto store_block = [&](const float (&v)[32], int ocol) {
        uint8_t* sb = out_stage + (stage_seq % C::OUT_BUFS) * OUT_STAGE_BYTES;
        if (lane == 0) bulk_wait_group_read<C::OUT_BUFS - 1>();
        __syncwarp();
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int j = q4 * 8;
          const uint4 pk = make_uint4(pack_bf16x2(v[j], v[j + 1]), pack_bf16x2(v[j + 2], v[j + 3]),
                                      pack_bf16x2(v[j + 4], v[j + 5]), pack_bf16x2(v[j + 6], v[j + 7]));
          *reinterpret_cast<uint4*>(sb + swz64(lane, q4)) = pk;
          if (args.amax_out != nullptr && row_ok) {
            const uint32_t w4[4] = {pk.x, pk.y, pk.z, pk.w};
            if (args.amax_signed) {  // max of the stored values, floored at 0 by y_amax's start
#pragma unroll
              for (int e = 0; e < 4; ++e) y_amax = fmax3(y_amax, bf16lo_to_f32(w4[e]), bf16hi_to_f32(w4[e]));
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e)
                y_amax = fmaxf(y_amax, fmaxf(fabsf(bf16lo_to_f32(w4[e])), fabsf(bf16hi_to_f32(w4[e]))));
            }
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (EpiOf<EM>::out_mode == OUT_SEQ2HEAD) {
            const int part = ocol / args.hd, rem = ocol - part * args.hd;
            const int head = rem >> 7, d0 = rem & 127;
            const int dst = head / args.heads_per_rank, lh = head - dst * args.heads_per_rank;
            tma_store_2d(&peers.m[dst], sb, (part * args.heads_per_rank + lh) * 128 + d0, m0 + quad * 32);
          } else {
            tma_store_2d(&tmap_y, sb, ocol, m0 + quad * 32);  // rows >= m are clipped by the map
          }
          bulk_commit_group();
        }
        ++stage_seq;
      };
      // Column pair p: gate rows n0+64p .. +31 and up rows n0+64p+32 .. +63
      // of the interleaved weight -> output columns (n0 + 64p)/2 .. +31.
      auto swiglu_pair = [&](const uint32_t* rg, const uint32_t* ru, int p) {
        const int gcol = n0 + p * 64;
        if (gcol >= args.n) return;  // warp-uniform
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float g = bf16r(dequant(rg[j], gcol + j));
          const float u = bf16r(dequant(ru[j], gcol + 32 + j));
          const float sg = bf16r(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))));
          v[j] = __fmul_rn(sg, u);
        }
        store_block(v, gcol / 2);
      };
      // Accumulator chunk c (output columns n0+32c .. +31) from its raw words.
      auto plain_chunk = [&](const uint32_t* r, int c) {
        const int col0 = n0 + c * 32;
        if (col0 >= args.n) return;  // warp-uniform: the whole chunk is past the last column
        if (EpiOf<EM>::out_mode == OUT_I32) {
          if (row_ok) {
            int32_t* out = static_cast<int32_t*>(args.y) + static_cast<int64_t>(row) * args.ldy + col0;
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              *reinterpret_cast<uint4*>(out + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
            }
          }
          return;
        }
        float v[32];
        dequant32(r, col0, v);
        if (EpiOf<EM>::epilogue == H3B_EPI_GELU) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = gelu_erf(bf16r(v[j]));  // gelu of the bf16 linear output
        } else if (EpiOf<EM>::epilogue == H3B_EPI_GATE_RES && row_ok) {
          const __nv_bfloat16* res = args.resid + static_cast<int64_t>(row) * args.ldy + col0;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            const uint4 rv = *reinterpret_cast<const uint4*>(res + j);
            const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
            uint32_t gw[4];
            if (gate_vec) {  // eight gate values in one 16-byte load
              const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gate_r + col0 + j));
              gw[0] = gv.x, gw[1] = gv.y, gw[2] = gv.z, gw[3] = gv.w;
            } else {
#pragma unroll
              for (int e = 0; e < 4; ++e)
                gw[e] = static_cast<uint32_t>(__bfloat16_as_ushort(gate_r[col0 + j + 2 * e])) |
                        (static_cast<uint32_t>(__bfloat16_as_ushort(gate_r[col0 + j + 2 * e + 1])) << 16);
            }
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float g0 = bf16lo_to_f32(gw[e]) * gmul;
              const float g1 = bf16hi_to_f32(gw[e]) * gmul;
              v[j + 2 * e] = __fadd_rn(bf16lo_to_f32(rw[e]), __fmul_rn(v[j + 2 * e], g0));
              v[j + 2 * e + 1] = __fadd_rn(bf16hi_to_f32(rw[e]), __fmul_rn(v[j + 2 * e + 1], g1));
            }
          }
        }
        store_block(v, col0);
      };
      if constexpr (C::NVF4_PAIR) {
        // Single accumulator: read this warp's four chunks (128 columns),
        // release the accumulator to the next tile's MMAs, then compute.
        const bool swi = EpiOf<EM>::epilogue == H3B_EPI_SWIGLU;
        uint32_t racc[4][32];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c = swi ? 2 * half + (i & 1) + 4 * (i >> 1) : half + 2 * i;
          tmem_ld32p(t_row + c * 32, racc[i]);
        }
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 4; ++i) reg_fence32(racc[i]);
        release_acc(buf);
        if (swi) {
          swiglu_pair(racc[0], racc[1], half);
          swiglu_pair(racc[2], racc[3], half + 2);
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) plain_chunk(racc[i], half + 2 * i);
        }
        continue;
      }
      if (EpiOf<EM>::epilogue == H3B_EPI_SWIGLU) {
        for (int p = half; p < BN / 64; p += 2) {
          uint32_t rg[32], ru[32];
          tmem_ld32p(t_row + p * 64, rg);
          tmem_ld32p(t_row + p * 64 + 32, ru);
          tc_wait_ld();
          reg_fence32(rg);
          reg_fence32(ru);
          if (p + 2 >= BN / 64) release_acc(buf);  // this warp's last pair
          swiglu_pair(rg, ru, p);
        }
        continue;
      }
      for (int c = half; c < BN / 32; c += 2) {
        uint32_t r[32];
        tmem_ld32p(t_row + c * 32, r);
        tmem_wait_fence<1>(r);
        if (c + 2 >= BN / 32) release_acc(buf);  // this warp's last chunk
        plain_chunk(r, c);
      }
    }
    if (lane == 0) {
      bulk_wait_group<0>();  // stores complete before the CTA exits
      if (EpiOf<EM>::out_mode == OUT_SEQ2HEAD) __threadfence_system();  // peer writes visible system-wide
    }
    __syncwarp();
    if (args.amax_out != nullptr) {
      y_amax = warp_max(y_amax);
      if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(args.amax_out), __float_as_uint(y_amax));
    }
  }

  tc_fence_before();
  if constexpr (PAIR == 2) {
    cluster_sync();  // neither CTA leaves while its partner may still signal it
  } else {
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR == 2)
      tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

template <int KIND, int PAIR, int EM>
int launch_gemm_t(const void* a, const void* b, int64_t a_row_bytes, int64_t b_row_bytes, const GemmArgs& args,
                  cudaStream_t st, const PeerMaps* peer_maps) {
  using C = Cfg<KIND, PAIR, EM>;
  CUtensorMap ta, tb, ty;
  int rc = h3b::encode_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, a, a_row_bytes, args.m, a_row_bytes, 128, BM,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != H3B_OK) return rc;
  rc = h3b::encode_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, b, b_row_bytes, args.n, b_row_bytes, 128, C::B_ROWS,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != H3B_OK) return rc;
  if (args.out_mode == OUT_BF16) {
    // y viewed as [m rows, n (n/2 for SwiGLU) cols] bf16 with row pitch ldy; 32x32 boxes.
    const int out_cols = args.epilogue == H3B_EPI_SWIGLU ? args.n / 2 : args.n;
    rc = h3b::encode_2d(&ty, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, args.y, out_cols, args.m, args.ldy * 2, 32, 32,
                        CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc != H3B_OK) return rc;
  } else {
    ty = ta;  // the int32 and scatter paths never use this map
  }
  const size_t smem = smem_bytes<KIND, PAIR, EM>();
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(gemm_kernel<KIND, PAIR, EM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return H3B_ERR_LAUNCH;
    if constexpr (C::NVF4_PAIR) {
      // setmaxnreg.inc waits for registers the launch must have provided:
      // refuse to launch a build whose kernel got fewer than the split needs.
      cudaFuncAttributes fa{};
      if (cudaFuncGetAttributes(&fa, gemm_kernel<KIND, PAIR, EM>) != cudaSuccess || fa.numRegs < PAIR_LAUNCH_REGS)
        return H3B_ERR_LAUNCH;
    }
    attr_set = true;
  }
  const int m_tiles = static_cast<int>((args.m + BM * PAIR - 1) / (BM * PAIR));
  const int n_tiles = static_cast<int>((args.n + C::BN - 1) / C::BN);
  const int tiles = m_tiles * n_tiles;
  const int max_units = h3b::num_sms() / PAIR;
  const int units = tiles < max_units ? tiles : max_units;
  static const PeerMaps no_peers = {};
  const PeerMaps& pm = peer_maps ? *peer_maps : no_peers;
  if constexpr (PAIR == 2) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * units));
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, gemm_kernel<KIND, 2, EM>, ta, tb, ty, pm, args) != cudaSuccess)
      return H3B_ERR_LAUNCH;
  } else {
    gemm_kernel<KIND, 1, EM><<<units, C::THREADS, smem, st>>>(ta, tb, ty, pm, args);
  }
  return h3b::launch_status();
}

// CTA pairs for every GEMM with more than one 128-row tile of M; a single
// row tile keeps one CTA per output tile (twice the CTAs for small M).
template <int KIND, int EM>
int launch_gemm_e(const void* a, const void* b, int64_t a_row_bytes, int64_t b_row_bytes, const GemmArgs& args,
                  cudaStream_t st, const PeerMaps* peer_maps) {
  if (args.m > BM && !args.no_loads)
    return launch_gemm_t<KIND, 2, EM>(a, b, a_row_bytes, b_row_bytes, args, st, peer_maps);
  return launch_gemm_t<KIND, 1, EM>(a, b, a_row_bytes, b_row_bytes, args, st, peer_maps);
}

// One kernel instance per epilogue mode (EpiMode): the output form first,
// then the activation.
template <int KIND>
int launch_gemm(const void* a, const void* b, int64_t a_row_bytes, int64_t b_row_bytes, const GemmArgs& args,
                cudaStream_t st, const PeerMaps* peer_maps = nullptr) {
  if (args.out_mode == OUT_SEQ2HEAD)
    return launch_gemm_e<KIND, EM_SEQ2HEAD>(a, b, a_row_bytes, b_row_bytes, args, st, peer_maps);
  if (args.out_mode == OUT_I32) {
    if constexpr (KIND == KIND_I8) return launch_gemm_e<KIND, EM_I32>(a, b, a_row_bytes, b_row_bytes, args, st, peer_maps);
    return H3B_ERR_ARG;
  }
  switch (args.epilogue) {
    case H3B_EPI_STORE:
      return launch_gemm_e<KIND, EM_STORE>(a, b, a_row_bytes, b_row_bytes, args, st, peer_maps);
    case H3B_EPI_GELU:
      return launch_gemm_e<KIND, EM_GELU>(a, b, a_row_bytes, b_row_bytes, args, st, peer_maps);
    case H3B_EPI_GATE_RES:
      return launch_gemm_e<KIND, EM_GATE_RES>(a, b, a_row_bytes, b_row_bytes, args, st, peer_maps);
    case H3B_EPI_SWIGLU:
      return launch_gemm_e<KIND, EM_SWIGLU>(a, b, a_row_bytes, b_row_bytes, args, st, peer_maps);
    case H3B_EPI_STORE_POSMAX: {
      GemmArgs s = args;
      s.epilogue = H3B_EPI_STORE;
      s.amax_signed = 1;
      return launch_gemm_e<KIND, EM_STORE>(a, b, a_row_bytes, b_row_bytes, s, st, peer_maps);
    }
    default:
      return H3B_ERR_ARG;
  }
}

// m == 0 (an empty batch) passes: the plain GEMM entries then return
// H3B_OK without a launch, as an empty F.linear returns an empty result.
int check_common(int64_t m, int64_t n, int64_t k, int64_t kmul) {
  if (m < 0 || n <= 0 || k <= 0) return H3B_ERR_SHAPE;
  if ((k % kmul) != 0 || (n % 32) != 0) return H3B_ERR_SHAPE;
  if (m > (1ll << 30) || n > (1ll << 30) || k > (1ll << 30)) return H3B_ERR_SHAPE;
  return H3B_OK;
}

}  // namespace

extern "C" int h3b_gemm_i8_bf16(const int8_t* q, const float* xs, const int8_t* w, const float* ws,
                                const void* bias, void* y, int64_t ldy, const void* resid, const void* gate,
                                int64_t gate_ld, const int32_t* row_sel, float* amax_out, int epilogue, int64_t m,
                                int64_t n, int64_t k, h3b_stream_t stream) {
  if (q == nullptr || xs == nullptr || w == nullptr || ws == nullptr || y == nullptr) return H3B_ERR_ARG;
  int rc = check_common(m, n, k, 128);
  if (rc != H3B_OK) return rc;
  if (epilogue < H3B_EPI_STORE || epilogue > H3B_EPI_STORE_POSMAX) return H3B_ERR_ARG;
  if (epilogue == H3B_EPI_SWIGLU && (n % 64) != 0) return H3B_ERR_SHAPE;
  if (ldy < (epilogue == H3B_EPI_SWIGLU ? n / 2 : n) || (ldy % 8) != 0) return H3B_ERR_SHAPE;
  if (epilogue == H3B_EPI_GATE_RES && (resid == nullptr || gate == nullptr || gate_ld < 0)) return H3B_ERR_ARG;
  if (!h3b::aligned16(q) || !h3b::aligned16(w) || !h3b::aligned16(y)) return H3B_ERR_ALIGN;
  if (resid != nullptr && !h3b::aligned16(resid)) return H3B_ERR_ALIGN;
  if (m == 0) return H3B_OK;
  GemmArgs a{};
  a.xs = xs;
  a.ws = ws;
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.resid = static_cast<const __nv_bfloat16*>(resid);
  a.gate = static_cast<const __nv_bfloat16*>(gate);
  a.gate_ld = gate_ld;
  a.row_sel = row_sel;
  a.amax_out = amax_out;
  a.y = y;
  a.ldy = ldy;
  a.m = static_cast<int>(m);
  a.n = static_cast<int>(n);
  a.k = static_cast<int>(k);
  a.epilogue = epilogue;
  a.out_mode = OUT_BF16;
  return launch_gemm<KIND_I8>(q, w, k, k, a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int h3b_gemm_i8_acc_i32(const int8_t* q, const int8_t* w, int32_t* acc, int64_t m, int64_t n,
                                   int64_t k, h3b_stream_t stream) {
  if (q == nullptr || w == nullptr || acc == nullptr) return H3B_ERR_ARG;
  int rc = check_common(m, n, k, 128);
  if (rc != H3B_OK) return rc;
  if (!h3b::aligned16(q) || !h3b::aligned16(w) || !h3b::aligned16(acc)) return H3B_ERR_ALIGN;
  if (m == 0) return H3B_OK;
  GemmArgs a{};
  a.y = acc;
  a.ldy = n;
  a.m = static_cast<int>(m);
  a.n = static_cast<int>(n);
  a.k = static_cast<int>(k);
  a.epilogue = H3B_EPI_STORE;
  a.out_mode = OUT_I32;
  return launch_gemm<KIND_I8>(q, w, k, k, a, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int h3b_gemm_nvfp4_bf16(const uint8_t* a_codes, const uint8_t* a_sf, const float* a_gs,
                                   const uint8_t* w_codes, const uint8_t* w_sf, const float* w_gs,
                                   const void* bias, void* y, int64_t ldy, const void* resid, const void* gate,
                                   int64_t gate_ld, const int32_t* row_sel, float* amax_out, int epilogue,
                                   int64_t m, int64_t n, int64_t k, h3b_stream_t stream) {
  if (a_codes == nullptr || a_sf == nullptr || a_gs == nullptr || w_codes == nullptr || w_sf == nullptr ||
      w_gs == nullptr || y == nullptr)
    return H3B_ERR_ARG;
  int rc = check_common(m, n, k, 256);
  if (rc != H3B_OK) return rc;
  if (epilogue < H3B_EPI_STORE || epilogue > H3B_EPI_STORE_POSMAX) return H3B_ERR_ARG;
  if (epilogue == H3B_EPI_SWIGLU && (n % 64) != 0) return H3B_ERR_SHAPE;
  if (ldy < (epilogue == H3B_EPI_SWIGLU ? n / 2 : n) || (ldy % 8) != 0) return H3B_ERR_SHAPE;
  if (epilogue == H3B_EPI_GATE_RES && (resid == nullptr || gate == nullptr || gate_ld < 0)) return H3B_ERR_ARG;
  if (!h3b::aligned16(a_codes) || !h3b::aligned16(w_codes) || !h3b::aligned16(y) || !h3b::aligned16(a_sf) ||
      !h3b::aligned16(w_sf))
    return H3B_ERR_ALIGN;
  if (resid != nullptr && !h3b::aligned16(resid)) return H3B_ERR_ALIGN;
  if (m == 0) return H3B_OK;
  GemmArgs a{};
  a.a_gs = a_gs;
  a.w_gs = w_gs;
  a.a_sf = a_sf;
  a.w_sf = w_sf;
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.resid = static_cast<const __nv_bfloat16*>(resid);
  a.gate = static_cast<const __nv_bfloat16*>(gate);
  a.gate_ld = gate_ld;
  a.row_sel = row_sel;
  a.amax_out = amax_out;
  a.y = y;
  a.ldy = ldy;
  a.m = static_cast<int>(m);
  a.n = static_cast<int>(n);
  a.k = static_cast<int>(k);
  a.epilogue = epilogue;
  a.out_mode = OUT_BF16;
  return launch_gemm<KIND_NVF4>(a_codes, w_codes, k / 2, k / 2, a, reinterpret_cast<cudaStream_t>(stream));
}

namespace {

// Validates the seq->head scatter arguments and encodes one tensor map per
// destination rank: recv_bufs[r] + rank*m rows, m rows of 3*(H/ws)*128 bf16.
int make_seq2head_maps(void* const* recv_bufs, int64_t world_size, int64_t rank, int64_t heads, int64_t m,
                       int64_t n, PeerMaps* maps, GemmArgs* a) {
  if (recv_bufs == nullptr) return H3B_ERR_ARG;
  if (world_size < 1 || world_size > MAX_PEERS || rank < 0 || rank >= world_size) return H3B_ERR_ARG;
  if (heads <= 0 || heads % world_size != 0 || n != 3 * heads * 128) return H3B_ERR_SHAPE;
  const int64_t hl = heads / world_size;
  const int64_t row_elems = 3 * hl * 128;
  for (int64_t r = 0; r < world_size; ++r) {
    if (recv_bufs[r] == nullptr || !h3b::aligned16(recv_bufs[r])) return H3B_ERR_ALIGN;
    const uint8_t* base = static_cast<const uint8_t*>(recv_bufs[r]) + rank * m * row_elems * 2;
    const int rc = h3b::encode_2d(&maps->m[r], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, row_elems, m, row_elems * 2,
                                  32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc != H3B_OK) return rc;
  }
  a->out_mode = OUT_SEQ2HEAD;
  a->heads_per_rank = static_cast<int>(hl);
  a->hd = static_cast<int>(heads * 128);
  a->epilogue = H3B_EPI_STORE;
  a->y = recv_bufs[rank];
  a->ldy = row_elems;
  return H3B_OK;
}

}  // namespace

extern "C" int h3b_gemm_i8_seq2head(const int8_t* q, const float* xs, const int8_t* w, const float* ws,
                                    const void* bias, void* const* recv_bufs, int64_t world_size, int64_t rank,
                                    int64_t heads, int64_t m, int64_t n, int64_t k, h3b_stream_t stream) {
  if (q == nullptr || xs == nullptr || w == nullptr || ws == nullptr) return H3B_ERR_ARG;
  int rc = check_common(m, n, k, 128);
  if (rc != H3B_OK) return rc;
  if (m == 0) return H3B_ERR_SHAPE;  // every rank holds an equal, non-empty sequence shard
  if (!h3b::aligned16(q) || !h3b::aligned16(w)) return H3B_ERR_ALIGN;
  GemmArgs a{};
  PeerMaps maps{};
  rc = make_seq2head_maps(recv_bufs, world_size, rank, heads, m, n, &maps, &a);
  if (rc != H3B_OK) return rc;
  a.xs = xs;
  a.ws = ws;
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.m = static_cast<int>(m);
  a.n = static_cast<int>(n);
  a.k = static_cast<int>(k);
  return launch_gemm<KIND_I8>(q, w, k, k, a, reinterpret_cast<cudaStream_t>(stream), &maps);
}

extern "C" int h3b_gemm_nvfp4_seq2head(const uint8_t* a_codes, const uint8_t* a_sf, const float* a_gs,
                                       const uint8_t* w_codes, const uint8_t* w_sf, const float* w_gs,
                                       const void* bias, void* const* recv_bufs, int64_t world_size, int64_t rank,
                                       int64_t heads, int64_t m, int64_t n, int64_t k, h3b_stream_t stream) {
  if (a_codes == nullptr || a_sf == nullptr || a_gs == nullptr || w_codes == nullptr || w_sf == nullptr ||
      w_gs == nullptr)
    return H3B_ERR_ARG;
  int rc = check_common(m, n, k, 256);
  if (rc != H3B_OK) return rc;
  if (m == 0) return H3B_ERR_SHAPE;  // every rank holds an equal, non-empty sequence shard
  if (!h3b::aligned16(a_codes) || !h3b::aligned16(w_codes) || !h3b::aligned16(a_sf) || !h3b::aligned16(w_sf))
    return H3B_ERR_ALIGN;
  GemmArgs a{};
  PeerMaps maps{};
  rc = make_seq2head_maps(recv_bufs, world_size, rank, heads, m, n, &maps, &a);
  if (rc != H3B_OK) return rc;
  a.a_gs = a_gs;
  a.w_gs = w_gs;
  a.a_sf = a_sf;
  a.w_sf = w_sf;
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.m = static_cast<int>(m);
  a.n = static_cast<int>(n);
  a.k = static_cast<int>(k);
  return launch_gemm<KIND_NVF4>(a_codes, w_codes, k / 2, k / 2, a, reinterpret_cast<cudaStream_t>(stream), &maps);
}

// Self-test of the bounded waits (no reference counterpart).  The NVFP4 GEMM
// kernel is launched on the caller's operands with its producer issuing no
// loads: no TMA or bulk copy is ever started, so the MMA thread's wait for
// the first slab can never complete, nor can the scale writers' and the
// epilogue's waits behind it.  After the 2 s budget the first wait to run out
// records H3B_ERR_DEVICE_TIMEOUT and its site (3, 4 or 7), raises the CTA's
// abort flag, and every other warp leaves its own wait; the kernel frees its
// TMEM and returns.  Nothing is written to y.
extern "C" int h3b_selftest_wait_timeout(const uint8_t* a_codes, const uint8_t* a_sf, const float* a_gs,
                                         const uint8_t* w_codes, const uint8_t* w_sf, const float* w_gs, void* y,
                                         int64_t m, int64_t n, int64_t k, h3b_stream_t stream) {
  if (a_codes == nullptr || a_sf == nullptr || a_gs == nullptr || w_codes == nullptr || w_sf == nullptr ||
      w_gs == nullptr || y == nullptr)
    return H3B_ERR_ARG;
  int rc = check_common(m, n, k, 256);
  if (rc != H3B_OK) return rc;
  if (m == 0 || m > BM || n > 192) return H3B_ERR_SHAPE;  // one output tile, one CTA
  if (!h3b::aligned16(a_codes) || !h3b::aligned16(w_codes) || !h3b::aligned16(y) || !h3b::aligned16(a_sf) ||
      !h3b::aligned16(w_sf))
    return H3B_ERR_ALIGN;
  GemmArgs a{};
  a.a_gs = a_gs;
  a.w_gs = w_gs;
  a.a_sf = a_sf;
  a.w_sf = w_sf;
  a.y = y;
  a.ldy = n;
  a.m = static_cast<int>(m);
  a.n = static_cast<int>(n);
  a.k = static_cast<int>(k);
  a.epilogue = H3B_EPI_STORE;
  a.out_mode = OUT_BF16;
  a.no_loads = 1;
  return launch_gemm<KIND_NVF4>(a_codes, w_codes, k / 2, k / 2, a, reinterpret_cast<cudaStream_t>(stream));
}
