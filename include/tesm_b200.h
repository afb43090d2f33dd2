/*
 * tesm_b200.h -- C ABI of the B200 (sm_100a) TESM inference hot path.
 *
 * All entry points are `extern "C"`, take raw device pointers, element counts
 * and byte/element strides, enqueue work on the given CUDA stream and return an
 * int status (0 = ok).  They never allocate, free or synchronise, except where a
 * comment says otherwise.  On error, tesm_b200_last_error() returns a message
 * (thread-local).  Device-side bounded waits that give up set a sticky device
 * status readable with tesm_b200_device_status().
 *
 * Each function names the reference interface (WANGLILIN360/tesm, path:line)
 * whose computation it replaces; the Python bindings of the reference call these
 * through ctypes.
 */
#ifndef TESM_B200_H_
#define TESM_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *tesm_stream_t; /* == cudaStream_t */

/* element types */
enum { TESM_F32 = 0, TESM_BF16 = 1 };

/* status codes */
enum {
  TESM_OK = 0,
  TESM_EINVAL = 1,      /* bad argument, shape, stride or alignment */
  TESM_EDTYPE = 2,      /* unsupported element type */
  TESM_ELAUNCH = 3,     /* CUDA launch / runtime error */
  TESM_ETIMEOUT = 4,    /* a device-side bounded wait gave up */
  TESM_EUNSUPPORTED = 5 /* configuration outside the implemented envelope */
};

/* activation code layouts produced by tesm_b200_quant_act */
enum { TESM_LAYOUT_ROWMAJOR = 0, TESM_LAYOUT_GEMV = 1 };

const char *tesm_b200_last_error(void);
int tesm_b200_version(void);
/* Reads and clears the sticky device status word (TESM_ETIMEOUT after a wait gave up). */
int tesm_b200_device_status(int *status_out);

/* ---------------------------------------------------------------- BitLinear
 * Weight quantisation of BitLinear.quantized_weight (tesm_ssm/modules/tesm.py:211-215)
 * and the INT2 byte format of pack_int2_to_uint8 (tesm_ssm/utils/int2_quantization.py:21-60).
 *
 * tesm_b200_weight_scale: scale = 1/max(mean|W|, eps) in the weight dtype (per tensor,
 * or per row when per_row != 0); deq = fl(1/scale), the magnitude of every non-zero
 * dequantised weight.  scale/deq hold 1 (per tensor) or N floats.
 */
int tesm_b200_weight_scale(const void *w, int dtype, int64_t N, int64_t K, int64_t ldw, int per_row, float eps,
                           float *scale, float *deq, double *work /* N doubles, caller-owned */,
                           tesm_stream_t stream);

/* t = clamp(round(W*scale), -1, 1).  packed (N x ld_packed bytes, ld_packed >= ceil(Kp/4) with
 * Kp = K rounded up to 256) receives the reference byte format (code t+1, four per byte,
 * lowest column in the low bits, padding code 1); tern (nullable, N x ld_tern int8,
 * ld_tern >= Kp) receives t with zero padding.  Bit-exact w.r.t. the reference. */
int tesm_b200_pack_ternary(const void *w, int dtype, int64_t N, int64_t K, int64_t ldw, int per_row,
                           const float *scale, uint8_t *packed, int64_t ld_packed, int8_t *tern, int64_t ld_tern,
                           tesm_stream_t stream);

/* Packed INT2 bytes (the format of pack_int2_to_uint8, int2_quantization.py:21-60) -> the
 * int8 ternary operand of tesm_b200_gemm_i8 (unpack_uint8_to_int2, int2_quantization.py:64-94,
 * without the dequantisation): tern[n, k] = code(n, k) - 1 for k < Kp (Kp a multiple of 16).
 * Loads exported INT2 weights without going back to the latent weights. */
int tesm_b200_unpack_ternary(const uint8_t *packed, int64_t ld_packed, int64_t N, int64_t Kp, int8_t *tern,
                             int64_t ld_tern, tesm_stream_t stream);

/* Per-token int8 activation quantisation of BitLinear.quantized_input (tesm.py:206-209):
 * s = 127 * fl(1/max(max|x|, eps)), c = clamp(round(x*s), -128, 127), bit-exact codes for
 * fp32 and bf16 input.  inv_scale[m] = 1/s.  layout TESM_LAYOUT_GEMV writes the permuted
 * layout consumed by tesm_b200_gemv_int2 and needs rowsum (sum of codes per row);
 * ld_codes >= K rounded up to 256 (zero padded). */
int tesm_b200_quant_act(const void *x, int dtype, int64_t M, int64_t K, int64_t ldx, float eps, int8_t *codes,
                        int64_t ld_codes, int layout, float *inv_scale, int32_t *rowsum, tesm_stream_t stream);

/* Decode-shaped (M <= 64) INT2 x INT8 GEMV on the packed weights (replaces the F.linear rung
 * of BitLinear._project_quantized, tesm.py:275-276):
 *   acc[m,n] = sum_k c[m,k] * t[n,k]  (exact int32),  out[m,n] = acc * inv_scale[m] * w_deq[n|0].
 * codes in TESM_LAYOUT_GEMV.  out dtype TESM_F32 / TESM_BF16 with row stride ldo (elements);
 * acc_out (nullable) receives the raw int32 accumulators (row stride ld_acc). */
int tesm_b200_gemv_int2(const int8_t *codes, int64_t ld_codes, const float *inv_scale, const int32_t *rowsum,
                        const uint8_t *packed, int64_t ld_packed, const float *w_deq, int per_row, int64_t M,
                        int64_t N, int64_t K, void *out, int out_dtype, int64_t ldo, int32_t *acc_out,
                        int64_t ld_acc, tesm_stream_t stream);

/* Prefill-shaped int8 GEMM on the 5th-generation tensor cores (tcgen05.mma kind::i8,
 * TMEM accumulators, TMA-staged operands); same contract as tesm_b200_gemv_int2 but the
 * activation codes are row-major (TESM_LAYOUT_ROWMAJOR, ld_codes multiple of 16) and the
 * weights are the int8 ternary matrix from tesm_b200_pack_ternary (ld_tern multiple of 16).
 * splitk_ws (nullable, caller-owned scratch of ws_bytes, 16-byte aligned): when the output tiles
 * do not fill the SMs (decode batches), K is split across up to 8 CTAs (or CTA pairs) per tile.
 * The first 16 KB of the scratch are 4096 int32 tile counters that must be zero before the first
 * call (e.g. cudaMemset once at allocation); every call leaves them zero again.  The rest holds
 * up to 8 int32 M*N slices: each split stores its partial tile into its slice and counts itself;
 * the split that arrives last adds the others' partials to its own accumulators (exact integers:
 * the result does not depend on the arrival order) and writes the output.  The split count is
 * capped so 16 KB + S*M*N*4 <= ws_bytes.  Calls that share one scratch must not overlap on the
 * GPU. */
/* Dense bf16 GEMM on the tensor cores (tcgen05.mma kind::f16, fp32 accumulators in TMEM, TMA
 * staged operands): out[m, n] = sum_k a[m, k] * b[n, k], written as out_dtype.  The tied lm_head
 * of a bf16 model (mixer_seq_simple.py:250-252, :334: F.linear(hidden, embedding.weight)).
 * Rows of a and b 16-byte aligned (lda, ldb multiples of 8). */
int tesm_b200_gemm_bf16(const void *a, int64_t lda, const void *b, int64_t ldb, int64_t M, int64_t N, int64_t K,
                        void *out, int out_dtype, int64_t ldo, tesm_stream_t stream);

/* tesm_b200_decode_step for one SISO layer (H = 1) with the per-token int8 codes of tanh(ent) and
 * ent - s as outputs instead of the values (tesm.py:1385-1396 then BitLinear.quantized_input
 * tesm.py:206-209 of state_proj / ent_proj): codes (B x ldc, ldc >= 2*Dp, Dp = D rounded up to
 * 128) hold the tanh codes in [0, D) and the change codes in [Dp, Dp + D), zero padded, ready
 * for tesm_b200_gemm_i8_combine; inv1 / inv2 receive 1/s per token.  The values are rounded to
 * act_dtype before quantisation, like the unfused path.
 * With xstate set (B x D fp32: the previous layer's new state), the step also computes the
 * cross-layer query bias itself, as cross_layer_q_proj(xstate) (tesm.py:1302-1305 with BitLinear
 * tesm.py:287-290): per-row int8 codes of the state (eps xq_eps), exact dot products with the
 * int8 ternary rows xq_tern (ent_rank rows, pitch xq_ld >= D rounded up to 16, 16-byte aligned)
 * and (float)acc * (1/s) * xq_deq[0] -- the values the separate quantiser + BitLinear GEMM give;
 * `cross` is then ignored.  xstate = NULL: `cross` (or no bias) as before. */
int tesm_b200_siso_decode_step_codes(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t Dm, int64_t D,
                                     int64_t R, int64_t W, const float *decay_bias, const float *bias,
                                     const float *cross, double *state, float *k_cache, float *v_cache, int *ctl,
                                     float thr, float es, float rope_base, int act_dtype, float eps1, float eps2,
                                     int8_t *codes, int64_t ldc, int64_t Dp, float *inv1, float *inv2,
                                     float *new_state, const float *xstate, const int8_t *xq_tern,
                                     int64_t xq_ld, const float *xq_deq, float xq_eps, tesm_stream_t stream);

/* Tensor-parallel pieces of the row-parallel BitLinear (down_proj / out_proj split along K over
 * ranks; no counterpart in the reference, which runs on one device):
 * tesm_b200_row_absmax: amax[m] = max_k |x[m,k]| of this rank's K-shard (the caller reduces it
 *   with MAX across ranks);
 * tesm_b200_quant_act_amax: tesm_b200_quant_act with the row maxima given (the global ones), so
 *   every rank's codes equal the single-device codes of its columns;
 * tesm_b200_gemm_i8 with out == NULL and acc_out set writes only the int32 partial accumulators
 *   (summed exactly across ranks by the caller);
 * tesm_b200_acc_scale: out[m,n] = acc[m,n] * inv_scale[m] * w_deq[n or 0] (acc is M x N, dense),
 *   the same float operations as the GEMM epilogue, so the result is bit-identical to one device. */
int tesm_b200_row_absmax(const void *x, int dtype, int64_t M, int64_t K, int64_t ldx, float *amax,
                         tesm_stream_t stream);
int tesm_b200_quant_act_amax(const void *x, int dtype, int64_t M, int64_t K, int64_t ldx, float eps,
                             const float *amax, int8_t *codes, int64_t ld_codes, int layout, float *inv_scale,
                             int32_t *rowsum, tesm_stream_t stream);
int tesm_b200_acc_scale(const int32_t *acc, int64_t M, int64_t N, const float *inv_scale, const float *w_deq,
                        int per_row, void *out, int out_dtype, int64_t ldo, tesm_stream_t stream);

/* Tensor-parallel MIMO output combine (no reference counterpart; the single-device operation is
 * tesm_b200_gemm_i8_combine, tesm.py:1255-1261 / tesm_mimo.py:1044-1049): the combine epilogue
 * of the dual-accumulator GEMM applied to int32 accumulators of state_proj (acc1) and ent_proj
 * (acc2) summed over the ranks' head shards: out = local + sigmoid(gate) * acc1 * inv1 * deq1
 * + acc2 * inv2 * deq2 with the GEMM epilogue's float operations (bit-identical to one device);
 * local / gate are columns c_local / c_gate of proj. */
int tesm_b200_combine_acc(const int32_t *acc1, const int32_t *acc2, int64_t ld_acc, int64_t M, int64_t N,
                          const float *inv1, const float *inv2, const float *deq1, const float *deq2, const void *proj,
                          int proj_dtype, int64_t ldp, int64_t c_local, int64_t c_gate, void *out, int out_dtype,
                          int64_t ldo, tesm_stream_t stream);

/* state_proj + ent_proj + output combine in one tcgen05 GEMM (tesm.py:1256-1260): two TMEM
 * accumulators, acc1 over the first Kh columns (codes of tanh(ent) x state_proj ternary weights),
 * acc2 over the next Kh (codes of ent - s x ent_proj weights); the epilogue writes
 *   out = local + sigmoid(gate) * acc1 * inv1 * deq1[0] + acc2 * inv2 * deq2[0]
 * with local / gate read from proj at columns c_local / c_gate.  tern (N, ld_tern) = [W_state | W_ent]
 * ternary rows, each half Kh wide (zero padded), Kh % 128 == 0. */
int tesm_b200_gemm_i8_combine(const int8_t *codes, int64_t ld_codes, int64_t Kh, const float *inv1, const float *inv2,
                              const int8_t *tern, int64_t ld_tern, const float *deq1, const float *deq2,
                              const void *proj, int proj_dtype, int64_t ldp, int64_t c_local, int64_t c_gate,
                              int64_t M, int64_t N, void *out, int out_dtype, int64_t ldo, tesm_stream_t stream);

int tesm_b200_gemm_i8(const int8_t *codes, int64_t ld_codes, const float *inv_scale, const int8_t *tern,
                      int64_t ld_tern, const float *w_deq, int per_row, int64_t M, int64_t N, int64_t K, void *out,
                      int out_dtype, int64_t ldo, int32_t *acc_out, int64_t ld_acc, int32_t *splitk_ws,
                      int64_t ws_bytes, tesm_stream_t stream);

/* ---------------------------------------------------------------- TESM layer (prefill)
 * `proj` is the in_proj output (B*L rows, row stride ldp elements, dtype TESM_F32/BF16) with the
 * reference column split [local Dm | value C | decay C | write C | gate Dm | q Rc | k Rc]
 * (tesm.py:1195-1205; MIMO tesm_mimo.py:940-956 with C = H*D, Rc = H*R, head-major).
 *
 * Selective state scan (replaces TESM_SISO._parallel_state_scan, tesm.py:1091-1164; MIMO
 * _parallel_state_scan_mimo, tesm_mimo.py:281-392): a = sigmoid(decay + decay_bias),
 * u = sigmoid(write)*tanh(value) (MIMO: u_r = (write*x_r)*(value*x_r), x = mimo_x[h,r,:]),
 * h_t = a_t h_{t-1} + u_t.  states: (B, L, RM, C) fp32; final_*: rank-0 state at t = L-1.
 * h0 (nullable, SISO only): prev_state (B, D) fp64.  workspace: caller-owned device
 * memory of at least tesm_b200_scan_workspace() bytes (look-back aggregates and flags). */
int tesm_b200_scan_workspace(int64_t B, int64_t L, int64_t C, int64_t RM, int64_t *bytes);
/* scan_chunk: the module's state_scan_chunk_size (reference default 16).  The reference scans
 * in chunks with h_t = A_t (h_c + sum_s u_s / max(A_s, 1e-12)), A the in-chunk cumulative
 * product of max(a, 1e-12) (tesm.py:1065-1089, :1133-1153); once A falls below 1e-12 inside a
 * chunk this departs from the plain recurrence, and the kernel reproduces it.  0 runs the plain
 * recurrence.  Supported chunk sizes divide 16 (or are >= L). */
int tesm_b200_siso_scan(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L, int64_t Dm, int64_t D,
                        int64_t R, int64_t scan_chunk, const float *decay_bias, const double *h0, float *states,
                        float *final_f32, double *final_f64, void *workspace, int64_t ws_bytes,
                        tesm_stream_t stream);
int tesm_b200_mimo_scan(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L, int64_t Dm, int64_t H,
                        int64_t D, int64_t R, int64_t RM, const float *decay_bias, const float *mimo_x,
                        float *states, float *final_f32, double *final_f64, void *workspace, int64_t ws_bytes,
                        tesm_stream_t stream);

/* Local (sliding-window) ternary entanglement + lerp (replaces _compute_local_entanglement,
 * tesm.py:853-952, and the lerp :1231-1232).  q, k are read from proj with RoPE applied on the
 * fly; cross (nullable, (B*L, R) fp32) is the cross-layer q bias.  Outputs (B*L, D):
 * out_tanh = tanh(ent), out_chg = ent - states, ent = s + es*(avg - s).  W in {4,8,16,32}. */
int tesm_b200_siso_local_ent(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L, int64_t Dm,
                             int64_t D, int64_t R, int64_t W, const float *cross, const float *bias,
                             const float *states, float thr, float es, float rope_base, void *out_tanh,
                             void *out_chg, int out_dtype, tesm_stream_t stream);

/* Local entanglement fused with the per-token int8 quantisation of its two outputs (the inputs of
 * state_proj and ent_proj, tesm.py:1256-1257, quantised as BitLinear.quantized_input with eps1 / eps2
 * after rounding to act_dtype).  codes (B*L, ldc): tanh(ent) codes in [0, D), ent - s codes in
 * [Dp, Dp + D), zeros elsewhere (Dp = D rounded up to 128, ldc >= 2*Dp); inv1 / inv2 = 1/s per row. */
int tesm_b200_siso_local_ent_codes(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L, int64_t Dm,
                                   int64_t D, int64_t R, int64_t W, const float *cross, const float *bias,
                                   const float *states, float thr, float es, float rope_base, int act_dtype,
                                   float eps1, float eps2, int8_t *codes, int64_t ldc, int64_t Dp, float *inv1,
                                   float *inv2, tesm_stream_t stream);

/* Relative-position bias vector of global entanglement (tesm.py:970-982), length 2L-1,
 * entry d + L - 1 for d = i - j. */
int tesm_b200_global_relbias(const float *embed, int64_t dim, float scale, float bias0, int64_t L, float *out,
                             tesm_stream_t stream);

/* Causal global ternary entanglement + lerp (replaces _compute_entanglement's global rung,
 * tesm.py:963-1043); same outputs as tesm_b200_siso_local_ent. */
int tesm_b200_siso_global_ent(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L, int64_t Dm,
                              int64_t D, int64_t R, const float *cross, const float *relb, const float *states,
                              float thr, float es, float rope_base, void *out_tanh, void *out_chg, int out_dtype,
                              tesm_stream_t stream);

/* Tensor-core version of tesm_b200_siso_global_ent (same reference code, same outputs): q.k in
 * three fp16 hi/lo MMAs (fp32 accumulation), ternary weights and states as fp16 MMA operands.
 * Needs ent_rank <= 64 (even) and d_state <= 256 (else status 5).  The caller provides a device
 * workspace of tesm_b200_global_ent_tc_workspace() bytes, 1024-byte aligned. */
int tesm_b200_global_ent_tc_workspace(int64_t B, int64_t L, int64_t D, int64_t R, int64_t *bytes);
int tesm_b200_siso_global_ent_tc(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L, int64_t Dm,
                                 int64_t D, int64_t R, const float *cross, const float *relb, const float *states,
                                 float thr, float es, float rope_base, void *out_tanh, void *out_chg, int out_dtype,
                                 void *workspace, int64_t ws_bytes, tesm_stream_t stream);

/* MIMO global entanglement with the rank merge (replaces _compute_global_entanglement_mimo's torch
 * rung, tesm_mimo.py:590-687, as used per rank at :1007-1017): scores over all heads' flattened
 * q.k / sqrt(H*R) (RoPE per head) + relative bias, ternary, causal; per rank avg_r = (tern/norm) @
 * states_r with NO lerp (the reference's global MIMO path returns the average itself);
 * out_tanh = tanh(sum_r mo_r * avg_r), out_chg = sum_r mo_r * (avg_r - s_r).  acc_e / acc_c: fp32
 * (B*L, H*D) caller workspaces (unused when RM == 1). */
int tesm_b200_mimo_global_ent(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L, int64_t Dm, int64_t H,
                              int64_t D, int64_t R, int64_t RM, const float *relb, const float *mimo_o,
                              const float *states, float thr, float rope_base, float *acc_e, float *acc_c,
                              void *out_tanh, void *out_chg, int out_dtype, tesm_stream_t stream);

/* MIMO local entanglement with the rank merge (replaces _compute_local_entanglement_mimo and the
 * mimo_o merge, tesm_mimo.py:394-588, :996-1017): out_tanh = tanh(sum_r mo_r*ent_r),
 * out_chg = sum_r mo_r*(ent_r - s_r), (B*L, H*D).  quirk != 0 keeps the reference's window
 * truncation for t < W-1.  (W, RM) in {8,16} x {1,2,4}. */
int tesm_b200_mimo_local_ent(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L, int64_t Dm, int64_t H,
                             int64_t D, int64_t R, int64_t RM, int64_t W, const float *bias, const float *mimo_o,
                             const float *states, float thr, float es, float rope_base, int quirk, void *out_tanh,
                             void *out_chg, int out_dtype, tesm_stream_t stream);

/* Output combine y = local + sigmoid(gate) * sp + ep (tesm.py:1256-1260); sp, ep: (M, Dm). */
int tesm_b200_combine(const void *proj, int dtype, int64_t ldp, int64_t M, int64_t Dm, int64_t D, int64_t R,
                      const void *sp, const void *ep, int sdtype, void *y, int ydtype, tesm_stream_t stream);

/* ---------------------------------------------------------------- decode cache
 * Prefill -> cache (tesm.py:1235-1253; MIMO rank 0, tesm_mimo.py:1022-1038): rope(k) and states
 * of the last min(L, W) positions into k_cache (B, W, H, R) / v_cache (B, W, H, D), state (B, H, D)
 * fp64 <- final_f64, ctl = {L, 0, 0}. */
int tesm_b200_cache_fill(const void *proj, int dtype, int64_t ldp, const float *states, int64_t RM, int64_t B,
                         int64_t L, int64_t Dm, int64_t H, int64_t D, int64_t R, int64_t W, float rope_base,
                         const double *final_f64, double *state, float *k_cache, float *v_cache, int *ctl,
                         tesm_stream_t stream);

/* One-token step (replaces TESM_SISO._forward_incremental, tesm.py:1274-1381, and the MIMO one,
 * tesm_mimo.py:753-894; H = 1 for SISO): fp64 state update, ring write at ctl[1], the reference's
 * window order and bias alignment, ternary average and lerp -> out_tanh / out_chg (B, H*D);
 * new_state (nullable) gets the fp32 state; ctl = {seq_pos, cache_idx, 0} is advanced on device. */
int tesm_b200_decode_step(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t Dm, int64_t H, int64_t D,
                          int64_t R, int64_t W, const float *decay_bias, const float *bias, const float *cross,
                          double *state, float *k_cache, float *v_cache, int *ctl, float thr, float es,
                          float rope_base, void *out_tanh, void *out_chg, int out_dtype, float *new_state,
                          tesm_stream_t stream);

/* ---------------------------------------------------------------- model glue
 * Embedding + learned positions (mixer_seq_simple.py:183-184); position offset from pos_dev[0]
 * when non-null (graph replay), else pos_host. */
int tesm_b200_embed(const int64_t *ids, int64_t B, int64_t L, const void *emb, const void *pos_emb, int wdtype,
                    int64_t Dm, const int *pos_dev, int64_t pos_host, void *out, int odtype, tesm_stream_t stream);

/* Block pre-norm fused with the next BitLinear's activation quantisation (block.py:28-45):
 * residual_out = x + residual (fp32; residual nullable), y = RMSNorm(residual_out) * weight,
 * codes/inv_scale/rowsum as tesm_b200_quant_act (codes nullable: norm only); y_out nullable. */
int tesm_b200_add_rmsnorm_quant(const void *x, int xdtype, const float *residual, float *residual_out,
                                const float *weight, float eps, int64_t M, int64_t K, float qeps, int8_t *codes,
                                int64_t ld_codes, int layout, float *inv_scale, int32_t *rowsum, void *y_out,
                                int ydtype, tesm_stream_t stream);

/* FeedForward gate (mixer_seq_simple.py:59-66): out[m, f] = silu(gate) * up, where gu (M, 2F) holds
 * [gate | up] halves (blk = 0) or blocks of blk gate columns each followed by the matching blk up
 * columns (blk = 128: the interleaved layout of tesm_b200_gemm_i8_swiglu's weights). */
int tesm_b200_silu_mul(const void *gu, int dtype, int64_t M, int64_t F, int64_t blk, void *out, int odtype,
                       tesm_stream_t stream);

/* Grouped gate/up BitLinear with the SiLU gate in the GEMM epilogue (replaces
 * FeedForward._grouped_gate_up + F.silu(gate)*up, mixer_seq_simple.py:45-66): tern (2F, ld_tern)
 * holds the gate and up ternary rows interleaved in blocks of 128 ([gate 0..127 | up 0..127 | gate
 * 128..255 | ...]), w_deq (2F) the per-row dequantisation factor in the same order; out (M, F) =
 * silu(acc_g * inv_scale * deq_g) * (acc_u * inv_scale * deq_u).  F % 128 == 0. */
int tesm_b200_gemm_i8_swiglu(const int8_t *codes, int64_t ld_codes, const float *inv_scale, const int8_t *tern,
                             int64_t ld_tern, const float *w_deq, int64_t M, int64_t F, int64_t K, void *out,
                             int out_dtype, int64_t ldo, int32_t *splitk_ws, int64_t ws_bytes, tesm_stream_t stream);

/* Allocation-free SISO scan.  No counterpart in the reference: it exists for callers that
 * cannot allocate device memory (runtimes with a fixed memory plan, embeddings of this
 * library without a device allocator).  Same computation and arguments as
 * tesm_b200_siso_scan minus the workspace: the look-back scratch is a fixed 8 MiB array
 * inside the library, present on every GPU that loads it until the process exits.  Shapes
 * whose scratch (tesm_b200_scan_workspace) exceeds 8 MiB are rejected with TESM_EUNSUPPORTED.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress) and
 * keeps it for the life of the process (it is not looked up again, so a cudaDeviceReset
 * between calls is not supported); make that first call before any stream capture.  Every call shares the one array, so calls
 * that overlap on the GPU (different streams, or several host threads) race; serialise them.
 * Nothing is allocated or freed. */
int tesm_b200_siso_scan_noalloc(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L, int64_t Dm,
                                int64_t D, int64_t R, int64_t scan_chunk, const float *decay_bias,
                                const double *h0, float *states, float *final_f32, double *final_f64,
                                tesm_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* TESM_B200_H_ */
