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
 * weights are the int8 ternary matrix from tesm_b200_pack_ternary (ld_tern multiple of 16). */
int tesm_b200_gemm_i8(const int8_t *codes, int64_t ld_codes, const float *inv_scale, const int8_t *tern,
                      int64_t ld_tern, const float *w_deq, int per_row, int64_t M, int64_t N, int64_t K, void *out,
                      int out_dtype, int64_t ldo, int32_t *acc_out, int64_t ld_acc, tesm_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* TESM_B200_H_ */
