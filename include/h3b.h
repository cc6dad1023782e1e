/*
 * h3b.h — C ABI of the B200 (sm_100a) kernels behind the MiniMax-H3 DiT-block
 * hot path.
 *
 * Conventions
 *  - Plain device pointers, int64 sizes/strides in elements, scalars, and an
 *    explicit cudaStream_t.  No torch types, no exceptions across the ABI.
 *  - Every entry point returns 0 (H3B_OK) or one of the H3B_ERR_* codes below.
 *    Shape, alignment and dtype violations are rejected on the host before any
 *    launch.  Device-side waits are bounded; a wait that times out records
 *    H3B_ERR_DEVICE_TIMEOUT in a device status word read by
 *    h3b_device_status().
 *  - Entry points allocate no device memory and never synchronise the host
 *    (h3b_device_status() excepted); callers own every buffer.
 *  - An empty batch (zero rows / query rows) is a valid no-op returning
 *    H3B_OK for the row-wise kernels, the plain GEMMs and attention, as the
 *    reference's F.linear / SDPA return empty results; the sequence-parallel
 *    variants (*_seq2head, *_head2seq) and h3b_quant_nvfp4 (whose global
 *    scale output would be left unwritten) require rows.
 *  - bf16 = IEEE bfloat16 stored as uint16; e4m3 = OCP float8 e4m3fn; e2m1
 *    codes are 4-bit values packed two per byte.
 *
 * Reference paths (repository BHUHD/minixmax-h3) are given relative to
 * Ref2VA-910C-FastAPI-INT8-CANN9.1.0/runtime/src/h3_npu/.
 */
#ifndef H3B_H_
#define H3B_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* h3b_stream_t; /* == cudaStream_t */

#if defined(__GNUC__)
#define H3B_API __attribute__((visibility("default")))
#else
#define H3B_API
#endif

enum {
  H3B_OK = 0,
  H3B_ERR_SHAPE = 1,          /* unsupported or inconsistent sizes          */
  H3B_ERR_ALIGN = 2,          /* pointer or stride alignment violated        */
  H3B_ERR_DTYPE = 3,          /* unsupported element type code               */
  H3B_ERR_LAUNCH = 4,         /* cudaLaunch / driver entry point failure     */
  H3B_ERR_TMAP = 5,           /* cuTensorMapEncodeTiled rejected a map       */
  H3B_ERR_DEVICE_TIMEOUT = 6, /* a bounded device wait ran out               */
  H3B_ERR_DEVICE = 7,         /* device reported a failure (see status)      */
  H3B_ERR_ARG = 8             /* null pointer or bad scalar argument         */
};

/* Element type codes for activation inputs. */
enum { H3B_BF16 = 0, H3B_F16 = 1 };

/* GEMM epilogue modes (applied in fp32 before the single bf16 rounding). */
enum {
  H3B_EPI_STORE = 0,    /* y = acc*scales (+ bias)                            */
  H3B_EPI_GELU = 1,     /* y = gelu_erf(acc*scales (+ bias))                  */
  H3B_EPI_GATE_RES = 2, /* y[m,n] = resid[m,n] + (acc*scales (+bias)) * gate[n] */
  H3B_EPI_SWIGLU = 3,   /* y[m,j] = silu(g)*u of a row-interleaved fc1, see below */
  H3B_EPI_STORE_POSMAX = 4 /* as H3B_EPI_STORE; amax_out receives max(0, max y)  */
};

/* Library version (major*10000 + minor*100 + patch). */
H3B_API int h3b_version(void);

/*
 * Reads (and with clear != 0 resets) the device status words of every kernel
 * family: out[0] = first error code, out[1] = site, out[2] = info, out[3] =
 * block.  Synchronises the current device.
 */
H3B_API int h3b_device_status(int32_t* out4, int clear);

/* ---------------------------------------------------------------- INT8 W8A8 */

/*
 * Per-row dynamic INT8 quantisation: amax = max|x[r,:]| clamped to 1e-12,
 * scale[r] = amax/127, q = round_half_even(x/scale) clamped to [-128,127].
 * Replaces ops/int8_convrot.py:99-111 (_dynamic_quant_rows, the host fallback
 * of torch_npu.npu_dynamic_quant).  x: [m, k] rows `ldx` elements apart,
 * dtype H3B_BF16 or H3B_F16; q: [m, k] int8 dense; scale: [m] fp32.
 * k % 8 == 0, ldx % 8 == 0, x 16-byte aligned.
 */
H3B_API int h3b_quant_i8_rows(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, int8_t* q,
                      float* scale, h3b_stream_t stream);

/*
 * ConvRot variant of h3b_quant_i8_rows: each 256-column group of a row is
 * first multiplied by the regular Hadamard matrix H4 (x) H4 (x) H4 (x) H4 / 16
 * (H4 = [[1,1,1,-1],[1,1,-1,1],[1,-1,1,1],[-1,1,1,1]]), rounded once to the
 * input dtype, then quantised as above.  Replaces ops/int8_convrot.py:139-157
 * (rotate_activation of ops/hadamard.py:35-44 followed by
 * _dynamic_quant_rows) for QuantLinear weights with meta "convrot".
 * group_size must be 256 (the reference's default convrot_groupsize,
 * modules/linear.py:149-151); k % 256 == 0, k <= 12288.  x_rot, if not NULL,
 * receives the rotated activation [m, k] dense in the input dtype.
 */
H3B_API int h3b_quant_i8_rows_convrot(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx,
                                      int64_t group_size, int8_t* q, float* scale, void* x_rot,
                                      h3b_stream_t stream);

/*
 * W8A8 GEMM on tcgen05 kind::i8 with int32 accumulation in TMEM:
 * y[m,n] = epi(acc[m,n] * xs[m] * ws[n] + bias[n]) as bf16, acc = sum_k
 * q[m,k]*w[n,k].  Replaces ops/int8_convrot.py:75-96 (torch_npu.
 * npu_quant_matmul with pertoken_scale, output_dtype bf16).
 * q: [m,k] int8, w: [n,k] int8 (the module's [N,K] weight, no transpose),
 * xs: [m] fp32, ws: [n] fp32, bias: [n] bf16 or NULL, y: [m,n] bf16 (row
 * stride ldy).
 * H3B_EPI_GATE_RES (the fused _mod_gate of model/dit.py:338-341):
 * y[m,n] = resid[m,n] + v * gate[row_sel[m]*gate_ld + n]; resid is bf16 with
 * row stride ldy and may alias y; row_sel (int32 [m]) may be NULL (row 0);
 * rows with row_sel < 0 keep resid unchanged (tokens outside every segment).
 * H3B_EPI_SWIGLU (the fc1 -> _swiglu step of model/dit.py:120-129, 298-301):
 * the weight rows are interleaved in blocks of 32 (rows 64b..64b+31 = gate
 * outputs 32b.., rows 64b+32..64b+63 = up outputs 32b..); y is [m, n/2] and
 * y[m,j] = bf16(bf16(silu(g)) * u) with g, u the bf16-rounded outputs of the
 * gate and up rows, the rounding chain of the reference's unfused
 * F.silu(gate) * up.  Needs n % 64 == 0.
 * H3B_EPI_GELU: y = bf16(gelu(bf16(v))), the reference's F.gelu of the bf16
 * linear output (model/dit.py:298-301 with the benchmark's GELU MLP).
 * amax_out (optional, caller-zeroed fp32) receives max |y| over the output;
 * under H3B_EPI_STORE_POSMAX it receives max(0, max y) instead (the input of
 * h3b_gelu_amax_scan / h3b_quant_nvfp4_gelu).
 * k % 128 == 0, n % 32 == 0, ldy % 8 == 0.
 */
H3B_API int h3b_gemm_i8_bf16(const int8_t* q, const float* xs, const int8_t* w, const float* ws, const void* bias,
                             void* y, int64_t ldy, const void* resid, const void* gate, int64_t gate_ld,
                             const int32_t* row_sel, float* amax_out, int epilogue, int64_t m, int64_t n,
                             int64_t k, h3b_stream_t stream);

/*
 * Same GEMM, raw int32 accumulators acc[m,n] (row stride n) for bit-exact
 * checks of the tensor-core path against sum_k q*w.
 */
H3B_API int h3b_gemm_i8_acc_i32(const int8_t* q, const int8_t* w, int32_t* acc, int64_t m, int64_t n, int64_t k,
                        h3b_stream_t stream);

/* ------------------------------------------------------------------- NVFP4 */

/*
 * amax_out[0] = max over i of |x[i]| for n bf16 values (x 16-byte aligned,
 * n % 8 == 0).  amax_out is overwritten (not accumulated).  Global-scale pass
 * of the NVFP4 activation quantiser; no reference counterpart (the reference
 * never quantises activations to NVFP4, ops/nvfp4.py:154-173 is W4A16).
 */
H3B_API int h3b_amax_bf16(const void* x, int64_t n, float* amax_out, h3b_stream_t stream);

/*
 * NVFP4 quantiser (e2m1 codes, one e4m3 scale per 16 elements along k, fp32
 * global scale gs = amax/(6*448), gs = 1 when amax == 0):
 *   s_b = e4m3_rn_satfinite(amax_b / (6*gs)),  code = e2m1_rne_sat(x/(s_b*gs)).
 * codes: [m, k/2] bytes; hi_first != 0 stores the even element in the high
 * nibble (the checkpoint order decoded by ops/nvfp4.py:113-121), 0 stores it
 * in the low nibble (tensor-core order).  sf: block scales in the 128x4
 * "blocked" layout decoded by ops/nvfp4.py:46-62 (from_blocked), padded to
 * (ceil(m/128)*128) x (ceil(k/64)*4) bytes; padding bytes are written as 0.
 * gs_out[0] receives gs.  The reference holds no quantiser: this follows the
 * published NVFP4 recipe that its decode (ops/nvfp4.py:86-151) inverts.
 * k % 64 == 0.
 */
H3B_API int h3b_quant_nvfp4(const void* x, int64_t m, int64_t k, int64_t ldx, const float* amax, uint8_t* codes,
                    uint8_t* sf, float* gs_out, int hi_first, h3b_stream_t stream);

/*
 * The MLP's activation fused with fc2's input quantisation (the fc1 ->
 * gelu -> fc2 input of model/dit.py:120-129 / ops/fused_block.py:61-63 with
 * the benchmark's GELU MLP): h3b_quant_nvfp4 of u = bf16(gelu(y)) computed on
 * the fly from fc1's bf16 output y [m, k] (row stride ldy), u never written.
 * The global scale needs max |u| before any code is written; it comes from
 * ymax2 (fp32 [2], device):
 *   ymax2[0] = max(0, max y)  (fc1 with H3B_EPI_STORE_POSMAX, max-reduced
 *              across ranks when sharded),
 *   ymax2[1] = max |u| by h3b_gelu_amax_scan (0 unless needed, see there),
 * max |u| = a when a = bf16(gelu(ymax2[0])) >= 0.169921875 (GELU and bf16
 * rounding are monotone for y >= 0, and |bf16(gelu(y))| <= 0.169921875 for
 * y < 0), else ymax2[1].  Codes, scales and gs as h3b_quant_nvfp4.
 * k % 64 == 0, ldy % 8 == 0, m >= 1.
 */
H3B_API int h3b_quant_nvfp4_gelu(const void* y, int64_t m, int64_t k, int64_t ldy, const float* ymax2,
                                 uint8_t* codes, uint8_t* sf, float* gs_out, int hi_first, h3b_stream_t stream);

/*
 * ymax2[1] = max(ymax2[1], max |bf16(gelu(y))|) over y [m, k] (row stride
 * ldy), computed only when bf16(gelu(ymax2[0])) < 0.169921875 (every block
 * returns at once otherwise).  ymax2[1] must start at 0.  Run after fc1 and
 * before the cross-rank max of ymax2: a rank whose own ymax2[0] is below the
 * bound scans, and if the global one is too, every rank has scanned.
 * k % 8 == 0, ldy % 8 == 0.
 */
H3B_API int h3b_gelu_amax_scan(const void* y, int64_t m, int64_t k, int64_t ldy, float* ymax2, h3b_stream_t stream);

/*
 * Swap the two nibbles of every byte (checkpoint hi-first order <-> tensor-core
 * lo-first order).  One-time weight repack, the NVFP4 analogue of
 * QuantLinear.prepare_cube (modules/linear.py:171-181).  src may equal dst.
 */
H3B_API int h3b_nvfp4_swap_nibbles(const uint8_t* src, uint8_t* dst, int64_t nbytes, h3b_stream_t stream);

/*
 * W4A4 NVFP4 GEMM on tcgen05 kind::mxf4nvf4 (block16, ue4m3 scales in TMEM):
 * y[m,n] = epi(a_gs*w_gs * sum_k A[m,k]*W[n,k] + bias[n]) as bf16, where
 * A = dequant(a_codes, a_sf), W = dequant(w_codes, w_sf), codes in lo-first
 * order, scales in the blocked layout above.  Replaces ops/nvfp4.py:154-173
 * (nvfp4_linear: dequantize_nvfp4 + F.linear) with the activation quantised
 * as well.  a_gs / w_gs: device fp32 scalars.  Other arguments as
 * h3b_gemm_i8_bf16.  k % 256 == 0, n % 32 == 0.
 */
H3B_API int h3b_gemm_nvfp4_bf16(const uint8_t* a_codes, const uint8_t* a_sf, const float* a_gs,
                                const uint8_t* w_codes, const uint8_t* w_sf, const float* w_gs, const void* bias,
                                void* y, int64_t ldy, const void* resid, const void* gate, int64_t gate_ld,
                                const int32_t* row_sel, float* amax_out, int epilogue, int64_t m, int64_t n,
                                int64_t k, h3b_stream_t stream);

/* --------------------------------------------------------------- attention */

/*
 * Non-causal flash attention forward, head_dim 128, bf16 in/out, fp32
 * softmax and accumulation on tcgen05 kind::f16:
 *   o[s,h,:] = softmax_j(scale * q[s,h,:].k[j,h,:]) v[j,h,:]
 * Element (s,h,d) of q lives at q + s*q_seq_stride + h*q_head_stride + d
 * (likewise k, v, o), so both the packed-QKV token-major layout [S,3,H,D]
 * and BNSD [H,S,D] are accepted without copies.  lse (optional, [heads, s_q]
 * fp32, natural log) receives the row log-sum-exp; amax_out (optional,
 * caller-zeroed fp32) receives max |o|.  Replaces
 * ops/fa_h3.py:224-304 (h3_attention_bnsd) and ops/attention.py:100-131
 * (fusion_attention_bnsd), whose host path is F.scaled_dot_product_attention.
 * Strides % 8 == 0, pointers 16-byte aligned.
 */
H3B_API int h3b_attention_fwd(const void* q, const void* k, const void* v, void* o, float* lse, float* amax_out,
                              int64_t heads,
                      int64_t s_q, int64_t s_kv, int64_t q_seq_stride, int64_t q_head_stride,
                      int64_t kv_seq_stride, int64_t kv_head_stride, int64_t o_seq_stride,
                      int64_t o_head_stride, float scale, h3b_stream_t stream);

/*
 * In-place q/k RMSNorm (fp32 math, weight [128] bf16, eps) followed by
 * split-half RoPE over all 128 dims in bf16 arithmetic with a bf16 rotation
 * table, exactly as ops/rope.py:7-55 (rope_rotation_table + rms_rope_apply)
 * computes it.  The table is built on the fly: angle[s,j] = pos[s,axis(j)] *
 * inv_freq[j] for j < 64 (fp32), where j < n_t uses axis 0 (t), j < n_t+n_h
 * axis 1 (h), else axis 2 (w) — the layout of model/dit.py:746-752
 * (rope_freqs).  pos: [s_total,3] fp32 grid positions, row s of q/k uses
 * pos[pos_offset + s].  q/k element (s,h,d) at base + s*seq_stride +
 * h*head_stride + d.  k may be NULL.
 */
H3B_API int h3b_qk_rmsnorm_rope(void* q, void* k, int64_t s, int64_t heads, int64_t seq_stride, int64_t head_stride,
                        const void* q_weight, const void* k_weight, float eps, const float* pos,
                        int64_t pos_offset, const float* inv_freq, int n_t, int n_h, h3b_stream_t stream);

/* ------------------------------------------------------- block elementwise */

/*
 * h[r,:] = rmsnorm(x[r,:]) * w * (1 + scale_r) + shift_r: the fused
 * norm1/norm2 + _mod_scale_shift of model/dit.py:332-335,433-438 and
 * modules/linear.py:15-32, with the reference's bf16 rounding after each
 * step.  shift_r = shift + row_sel[r]*tab_ld (likewise scale): the adaLN
 * chunk tables of AdalnProj (model/dit.py:326-329) addressed in place;
 * row_sel (int32 [m]) may be NULL (row 0); row_sel[r] < 0 leaves h = the
 * plain RMSNorm (tokens outside every mod segment).  x, h: [m, hidden] bf16
 * with row stride ld; w: [hidden] bf16.  amax_out (optional, caller-zeroed)
 * receives max |h| for the NVFP4 global scale.
 */
H3B_API int h3b_rmsnorm_modulate(const void* x, void* h, int64_t m, int64_t hidden, int64_t ld, const void* w,
                                 const void* shift, const void* scale, int64_t tab_ld, const int32_t* row_sel,
                                 float eps, float* amax_out, h3b_stream_t stream);

/*
 * h3b_rmsnorm_modulate followed by the INT8 row quantiser of the QKV / fc1
 * input — h3b_quant_i8_rows (convrot_group 0) or h3b_quant_i8_rows_convrot
 * (convrot_group 256) applied to h — in one pass, without writing h: the
 * norm + _mod_scale_shift of model/dit.py:433-438 feeding
 * int8_convrot_linear (ops/int8_convrot.py:114-157).  q: [m, hidden] int8
 * (row stride hidden, 8-byte aligned), q_scale: [m] fp32.  Same bits as the
 * two-kernel sequence.  hidden % 256 == 0 with ConvRot.
 */
H3B_API int h3b_rmsnorm_modulate_quant_i8(const void* x, int64_t m, int64_t hidden, int64_t ld, const void* w,
                                          const void* shift, const void* scale, int64_t tab_ld,
                                          const int32_t* row_sel, float eps, int64_t convrot_group, int8_t* q,
                                          float* q_scale, h3b_stream_t stream);

/*
 * x[r,:] += y[r,:] * gate_r  (bf16, in place), the _mod_gate of
 * model/dit.py:338-341; gate_r = gate + row_sel[r]*tab_ld, rows with
 * row_sel < 0 unchanged.
 */
H3B_API int h3b_gate_residual(void* x, const void* y, int64_t m, int64_t hidden, int64_t ld, const void* gate,
                              int64_t tab_ld, const int32_t* row_sel, h3b_stream_t stream);

/* ------------------------------------------------- Ulysses P2P exchange */

/*
 * CUDA IPC registration of the exchange buffers (the receive buffers of the
 * P2P Ulysses path; the reference allocates its SP buffers once and reuses
 * them, runtime/dist.py:30,172-203).  h3b_ipc_export writes the 64-byte IPC
 * handle of the allocation holding dev_ptr and dev_ptr's byte offset in it;
 * a peer process passes both to h3b_ipc_import to map the same memory
 * (*dev_ptr = mapped base + offset) and to h3b_ipc_close to unmap it.
 * Setup-time calls, not for the step loop.
 */
H3B_API int h3b_ipc_export(const void* dev_ptr, uint8_t* handle64, int64_t* offset);
H3B_API int h3b_ipc_import(const uint8_t* handle64, int64_t offset, void** dev_ptr);
H3B_API int h3b_ipc_close(void* dev_ptr, int64_t offset);

/*
 * QKV projection fused with the sequence->head all-to-all (ops/ulysses.py:
 * 14-30 applied to the qkv_proj output of model/dit.py:169-190): the GEMM of
 * h3b_gemm_i8_bf16 / h3b_gemm_nvfp4_bf16 with n = 3*heads*128, whose output
 * column (part, head, d) of local row t is stored to rank
 * head / (heads/world_size)'s receive buffer recv_bufs[r] — laid out
 * [world_size*m, 3, heads/world_size, 128] bf16 — at row rank*m + t.
 * recv_bufs: world_size device pointers valid in this process (own buffer
 * and IPC-imported peers').  No activation or residual epilogue.  The
 * caller orders the exchange (all ranks' launches complete) before reading
 * a receive buffer, e.g. with a collective on the same stream.
 */
H3B_API int h3b_gemm_i8_seq2head(const int8_t* q, const float* xs, const int8_t* w, const float* ws,
                                 const void* bias, void* const* recv_bufs, int64_t world_size, int64_t rank,
                                 int64_t heads, int64_t m, int64_t n, int64_t k, h3b_stream_t stream);
H3B_API int h3b_gemm_nvfp4_seq2head(const uint8_t* a_codes, const uint8_t* a_sf, const float* a_gs,
                                    const uint8_t* w_codes, const uint8_t* w_sf, const float* w_gs,
                                    const void* bias, void* const* recv_bufs, int64_t world_size, int64_t rank,
                                    int64_t heads, int64_t m, int64_t n, int64_t k, h3b_stream_t stream);

/*
 * Attention fused with the head->sequence all-to-all (ops/ulysses.py:32-41
 * on the attention output, model/dit.py:248-289): h3b_attention_fwd over
 * this rank's `heads` local heads and all s_q = world_size*s_local tokens,
 * writing query row t of local head h into o_bufs[t / s_local] (rank
 * t/s_local's out-projection input, [s_local, H, 128] with strides
 * o_seq_stride / o_head_stride elements) at row t % s_local, head head0 + h.
 * Same ordering contract as h3b_gemm_*_seq2head.
 */
H3B_API int h3b_attention_fwd_head2seq(const void* q, const void* k, const void* v, void* const* o_bufs,
                                       int64_t world_size, int64_t s_local, int64_t head0, int64_t o_seq_stride,
                                       int64_t o_head_stride, float* amax_out, int64_t heads, int64_t s_q,
                                       int64_t s_kv, int64_t q_seq_stride, int64_t q_head_stride,
                                       int64_t kv_seq_stride, int64_t kv_head_stride, float scale,
                                       h3b_stream_t stream);

/*
 * Self-test of the bounded device waits; no counterpart in the reference,
 * whose distributed waits are host-side timeouts (runtime/dist.py:43,99-116).
 * Launches the NVFP4 GEMM of h3b_gemm_nvfp4_bf16 on the given operands (one
 * output tile: m <= 128, n <= 192) with its producer issuing no loads, so no
 * copy is ever in flight and the MMA thread's wait for the first K slab can
 * never complete, nor can the waits of the other warps behind it.  The
 * waits run out after their budget (2 s); the first records
 * H3B_ERR_DEVICE_TIMEOUT and its site in the device status word (3: the MMA
 * thread's slab wait, 4: an epilogue warp's accumulator wait, 7: a scale
 * writer's wait), and every warp unwinds; the kernel frees its TMEM and
 * returns without writing y.
 * Returns the launch status; read the outcome with h3b_device_status().
 */
H3B_API int h3b_selftest_wait_timeout(const uint8_t* a_codes, const uint8_t* a_sf, const float* a_gs,
                                      const uint8_t* w_codes, const uint8_t* w_sf, const float* w_gs, void* y,
                                      int64_t m, int64_t n, int64_t k, h3b_stream_t stream);

/* Merge of an attention result over one key chunk into a running result
 * over earlier chunks through the rows' log-sum-exps, in fp32 — the ring
 * sequence-parallel step of ops/fa_h3.py:141-156 (_merge_lse), used by
 * ring_attention_lse_bnsd (ops/fa_h3.py:159-218):
 *   acc <- acc - sigmoid(blk_lse - acc_lse) * (acc - blk)
 *   acc_lse <- acc_lse - logsigmoid(acc_lse - blk_lse)
 * acc fp32 and blk bf16 are token-major [s, heads, 128], contiguous; lse
 * arrays [heads, s] fp32 (natural log, as h3b_attention_fwd writes them).
 * first != 0 initialises acc / acc_lse from blk / blk_lse.  With out given
 * (bf16 [s, heads, 128]) the merged rows are written there instead of acc,
 * and max |out| into amax_out (optional, caller-zeroed fp32).
 */
H3B_API int h3b_attention_merge_lse(float* acc, float* acc_lse, const void* blk, const float* blk_lse, int64_t s,
                                    int64_t heads, int first, void* out, float* amax_out, h3b_stream_t stream);

/*
 * Allocation-free variant of the NVFP4 projection input: the results of
 * h3b_rmsnorm_modulate (x -> h, with the |h| max) followed by
 * h3b_quant_nvfp4 (h -> codes, sf, gs_out), with h and the max kept in a
 * fixed array of this library's device memory instead of two caller
 * buffers.  No counterpart in the reference: it is for callers that may not
 * allocate device memory while they run (a framework that owns the GPU's
 * memory pool, or C/C++ code without a caching allocator, for which
 * cudaMalloc/cudaFree would synchronise the device).  The caller passes x,
 * the tables and the outputs, with the meanings of the two entry points
 * above (hidden % 64 == 0).  Limit: m * ld * 2 <= 16 MiB (h is held with the
 * row stride of x); larger calls return H3B_ERR_SHAPE and do nothing.  The
 * array (16 MiB + 256 bytes) is resident on every GPU that loads the
 * library until the process exits; all calls on a device share it, so calls
 * that overlap on the GPU race.  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress) and caches it; make that
 * first call before any stream capture, and do not use the entry point
 * across a cudaDeviceReset.  Every argument is validated before any work is
 * queued: a rejected call leaves the array untouched.
 */
H3B_API int h3b_rmsnorm_modulate_quant_nvfp4_noalloc(const void* x, int64_t m, int64_t hidden, int64_t ld,
                                                     const void* w, const void* shift, const void* scale,
                                                     int64_t tab_ld, const int32_t* row_sel, float eps,
                                                     uint8_t* codes, uint8_t* sf, float* gs_out, int hi_first,
                                                     h3b_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* H3B_H_ */
