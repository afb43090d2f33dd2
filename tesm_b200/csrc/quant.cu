// Ternary weight quantisation + INT2 packing, and per-token int8 activation quantisation.
//
// Bit-exactness notes (reference: tesm_ssm/modules/tesm.py:206-215,
// tesm_ssm/utils/int2_quantization.py:21-60):
//  * torch evaluates `c / t` for a python scalar c as `t.reciprocal() * c`, i.e. two
//    roundings in the tensor dtype; we use __frcp_rn then __fmul_rn (then bf16 RNE for
//    bf16 tensors).
//  * the product of two bf16 values is exact in fp32, so fp32 multiply followed by bf16
//    RNE reproduces torch's bf16 multiply.
//  * torch.round is round-half-to-even == rintf.
// This file is compiled without fast-math; explicit _rn intrinsics keep it that way.
#include "rowio.cuh"

namespace tesm {

// ---------------------------------------------------------------- weight scale
// One warp per row: fp64 sum of |w| in a fixed order (deterministic).
__global__ void k_row_abs_sum(const void *__restrict__ w, int dtype, int64_t N, int64_t K, int64_t ldw,
                              double *__restrict__ row_sum) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= N) return;
  double s = 0.0;
  const int64_t base = row * ldw;
  for (int64_t k = lane; k < K; k += 32) s += (double)fabsf(load_f(w, dtype, base + k));
  s = warp_sum_d(s);
  if (lane == 0) row_sum[row] = s;
}

__device__ __forceinline__ void scale_from_sum(double sum, double count, int dtype, float eps, float *scale,
                                               float *deq) {
  float m = (float)(sum / count);
  m = round_to(dtype, fmaxf(m, eps));
  float sc = round_to(dtype, __frcp_rn(m));  // 1.0 / t -> reciprocal * 1.0
  *scale = sc;
  *deq = round_to(dtype, __frcp_rn(sc));    // q / scale for q = +-1
}

// Per-tensor: one block sums the per-row partials in a fixed order.
__global__ void k_tensor_scale(const double *__restrict__ row_sum, int64_t N, int64_t K, int dtype, float eps,
                               float *scale, float *deq) {
  __shared__ double red[32];
  double s = 0.0;
  for (int64_t r = threadIdx.x; r < N; r += blockDim.x) s += row_sum[r];
  s = block_reduce(s, red, [](double a, double b) { return a + b; }, 0.0);
  if (threadIdx.x == 0) scale_from_sum(s, (double)N * (double)K, dtype, eps, scale, deq);
}

__global__ void k_row_scale(const double *__restrict__ row_sum, int64_t N, int64_t K, int dtype, float eps,
                            float *scale, float *deq) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r < N) scale_from_sum(row_sum[r], (double)K, dtype, eps, scale + r, deq + r);
}

// ---------------------------------------------------------------- pack
// One thread per 16-column group of a row: 16 ternary codes -> one 32-bit word of the
// reference byte format (4 bytes, lowest column in the low bits) + 16 int8 values.
__global__ void k_pack(const void *__restrict__ w, int dtype, int64_t N, int64_t K, int64_t ldw, int per_row,
                       const float *__restrict__ scale, uint8_t *__restrict__ packed, int64_t ld_packed,
                       int8_t *__restrict__ tern, int64_t ld_tern, int64_t groups_per_row) {
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= N * groups_per_row) return;
  const int64_t row = gid / groups_per_row;
  const int64_t grp = gid - row * groups_per_row;
  const float sc = per_row ? scale[row] : scale[0];
  uint32_t word = 0;
  uint32_t tw[4] = {0, 0, 0, 0};
  const int64_t k0 = grp * 16;
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const int64_t k = k0 + e;
    int t = 0;
    if (k < K) {
      float v = round_to(dtype, __fmul_rn(load_f(w, dtype, row * ldw + k), sc));
      v = rintf(v);
      t = (int)fminf(fmaxf(v, -1.f), 1.f);
    }
    word |= (uint32_t)(t + 1) << (2 * e);
    tw[e >> 2] |= ((uint32_t)(uint8_t)(int8_t)t) << (8 * (e & 3));
  }
  reinterpret_cast<uint32_t *>(packed + row * ld_packed)[grp] = word;
  if (tern) {
    uint4 v = make_uint4(tw[0], tw[1], tw[2], tw[3]);
    reinterpret_cast<uint4 *>(tern + row * ld_tern)[grp] = v;
  }
}

// Packed INT2 bytes -> int8 ternary operand (unpack_uint8_to_int2, int2_quantization.py:64-94:
// code c in bits 2i..2i+1 of byte j is column 4j + i, t = c - 1).  One thread per packed word of
// 4 bytes = 16 columns; padding codes (1) give t = 0.
__global__ void k_unpack(const uint8_t *__restrict__ packed, int64_t ld_packed, int64_t N, int64_t words_per_row,
                         int8_t *__restrict__ tern, int64_t ld_tern) {
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= N * words_per_row) return;
  const int64_t row = gid / words_per_row, wd = gid - row * words_per_row;
  const uint32_t w = reinterpret_cast<const uint32_t *>(packed + row * ld_packed)[wd];
  uint32_t out[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {  // byte q of the word -> columns 4q .. 4q+3
    const uint32_t b = (w >> (8 * q)) & 0xffu;
    uint32_t v = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) v |= (uint32_t)(uint8_t)(int8_t)((int)((b >> (2 * i)) & 3u) - 1) << (8 * i);
    out[q] = v;
  }
  reinterpret_cast<uint4 *>(tern + row * ld_tern)[wd] = make_uint4(out[0], out[1], out[2], out[3]);
}

// ---------------------------------------------------------------- activation quant
// One block per row; each thread owns up to GPT 16-element groups kept in registers
// (16-byte vector loads when the row is aligned).
constexpr int kQuantGPT = 4;

__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;\n" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// bf16 rows with row-major codes.  A group's 16 values stay packed as 8 bf16x2 words.  Row maximum
// of |x| on the bit patterns (non-negative bf16 values order like their 16-bit patterns).  Codes:
// the exact product x * s of two bf16 values rounded once to bf16 (mul.rn.bf16x2) is the fp32
// __fmul_rn followed by act_code's round to bf16; then act_code_bits.  Same codes as act_code.
template <int GPT>
__device__ __forceinline__ void quant_row_bf16(const __nv_bfloat16 *xrow, float eps, int8_t *crow, int64_t groups,
                                               float *inv_scale, const float *amax_in, int64_t row, float *redf) {
  uint32_t w[GPT][8];
  uint32_t m = 0;
#pragma unroll
  for (int j = 0; j < GPT; ++j) {
    const int64_t g = threadIdx.x + (int64_t)j * blockDim.x;
    if (g < groups) {
      const uint4 *p = reinterpret_cast<const uint4 *>(xrow + g * 16);
      const uint4 a = p[0], b = p[1];
      w[j][0] = a.x, w[j][1] = a.y, w[j][2] = a.z, w[j][3] = a.w;
      w[j][4] = b.x, w[j][5] = b.y, w[j][6] = b.z, w[j][7] = b.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) w[j][i] = 0u;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) m = __vmaxu2(m, w[j][i] & 0x7fff7fffu);
  }
  float amax = __uint_as_float(max(m & 0xffffu, m >> 16) << 16);
  amax = block_reduce(amax, redf, [](float a, float b) { return fmaxf(a, b); }, 0.f);
  if (amax_in) amax = amax_in[row];
  const float s = act_scale(amax, eps, TESM_BF16);
  if (threadIdx.x == 0) inv_scale[row] = __frcp_rn(s);
  const uint32_t sb = __float_as_uint(s) >> 16, s2 = sb | (sb << 16);
#pragma unroll
  for (int j = 0; j < GPT; ++j) {
    const int64_t g = threadIdx.x + (int64_t)j * blockDim.x;
    if (g >= groups) continue;
    uint32_t wv[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t p0 = mul_bf16x2(w[j][2 * q], s2), p1 = mul_bf16x2(w[j][2 * q + 1], s2);
      wv[q] = pack_code_bytes(act_code_bits(__uint_as_float(p0 << 16)), act_code_bits(__uint_as_float(p0 & 0xffff0000u)),
                              act_code_bits(__uint_as_float(p1 << 16)), act_code_bits(__uint_as_float(p1 & 0xffff0000u)));
    }
    reinterpret_cast<uint4 *>(crow)[g] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
  }
}

// bf16 rows, 16-byte aligned, row-major codes (the GEMM operand): quant_row_bf16, one block per row
template <int GPT>
__global__ void k_quant_act_bf16(const __nv_bfloat16 *__restrict__ x, int64_t K, int64_t ldx, float eps,
                                 int8_t *__restrict__ codes, int64_t ld_codes, float *__restrict__ inv_scale,
                                 const float *__restrict__ amax_in) {
  __shared__ float redf[32];
  pdl_trigger();
  pdl_wait();
  const int64_t row = blockIdx.x;
  quant_row_bf16<GPT>(x + row * ldx, eps, codes + row * ld_codes, (K + 15) / 16, inv_scale, amax_in, row, redf);
}

template <int GPT>
__global__ void k_quant_act(const void *__restrict__ x, int dtype, int64_t K, int64_t ldx, float eps,
                            int8_t *__restrict__ codes, int64_t ld_codes, int layout, int64_t groups_out,
                            float *__restrict__ inv_scale, int32_t *__restrict__ rowsum, int vec,
                            const float *__restrict__ amax_in) {
  __shared__ float redf[32];
  __shared__ int redi[32];
  // let a programmatically serialized consumer (the GEMV, the GEMM) start its weight prefetch
  // now; it still waits for this whole grid before reading the codes
  pdl_trigger();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const int64_t groups_in = (K + 15) / 16;
  const int esz = dtype == TESM_BF16 ? 2 : 4;
  const void *xrow = reinterpret_cast<const uint8_t *>(x) + row * ldx * esz;
  float v[GPT][16];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < GPT; ++j) {
    const int64_t g = threadIdx.x + (int64_t)j * blockDim.x;
    if (g < groups_in) {
      load16(xrow, dtype, g * 16, K, vec, v[j]);
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) v[j][e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < 16; ++e) amax = fmaxf(amax, fabsf(v[j][e]));
  }
  amax = block_reduce(amax, redf, [](float a, float b) { return fmaxf(a, b); }, 0.f);
  if (amax_in) amax = amax_in[row];  // the row's max |x| over all tensor-parallel shards
  const float s = act_scale(amax, eps, dtype);
  if (threadIdx.x == 0) inv_scale[row] = __frcp_rn(s);
  int csum = 0;
  int8_t *crow = codes + row * ld_codes;
#pragma unroll
  for (int j = 0; j < GPT; ++j) {
    const int64_t g = threadIdx.x + (int64_t)j * blockDim.x;
    if (g >= groups_out) continue;
    int c[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      c[e] = act_code(v[j][e], s, dtype);
      csum += c[e];
    }
    store_codes16(crow, g, layout, c);
  }
  if (rowsum) {
    csum = block_reduce(csum, redi, [](int a, int b) { return a + b; }, 0);
    if (threadIdx.x == 0) rowsum[row] = csum;
  }
}

// Short rows (K <= 1024): one warp per row, 8 rows per block, warp-shuffle reductions (a
// 32-thread block per row of a few hundred elements is bound by block scheduling).
__global__ void k_quant_act_warp(const void *__restrict__ x, int dtype, int64_t M, int64_t K, int64_t ldx, float eps,
                                 int8_t *__restrict__ codes, int64_t ld_codes, int layout, int64_t groups_out,
                                 float *__restrict__ inv_scale, int32_t *__restrict__ rowsum, int vec,
                                 const float *__restrict__ amax_in) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= M) return;
  const int64_t groups_in = (K + 15) / 16;
  const int esz = dtype == TESM_BF16 ? 2 : 4;
  const void *xrow = reinterpret_cast<const uint8_t *>(x) + row * ldx * esz;
  float v[2][16];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int64_t g = lane + 32 * j;
    if (g < groups_in) {
      load16(xrow, dtype, g * 16, K, vec, v[j]);
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) v[j][e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < 16; ++e) amax = fmaxf(amax, fabsf(v[j][e]));
  }
  amax = warp_max(amax);
  if (amax_in) amax = amax_in[row];
  const float s = act_scale(amax, eps, dtype);
  if (lane == 0) inv_scale[row] = __frcp_rn(s);
  int csum = 0;
  int8_t *crow = codes + row * ld_codes;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int64_t g = lane + 32 * j;
    if (g >= groups_out) continue;
    int c[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      c[e] = act_code(v[j][e], s, dtype);
      csum += c[e];
    }
    store_codes16(crow, g, layout, c);
  }
  if (rowsum) {
    csum = warp_sum_i(csum);
    if (lane == 0) rowsum[row] = csum;
  }
}

// max |x| of each row (tensor-parallel shards: reduced across ranks, then quantised with it).
__global__ void k_row_absmax(const void *__restrict__ x, int dtype, int64_t K, int64_t ldx, int vec,
                             float *__restrict__ amax_out) {
  __shared__ float redf[32];
  const int64_t row = blockIdx.x;
  const void *xrow = reinterpret_cast<const uint8_t *>(x) + row * ldx * (dtype == TESM_BF16 ? 2 : 4);
  float amax = 0.f;
  for (int64_t g = threadIdx.x; g < (K + 15) / 16; g += blockDim.x) {
    float v[16];
    load16(xrow, dtype, g * 16, K, vec, v);
#pragma unroll
    for (int e = 0; e < 16; ++e) amax = fmaxf(amax, fabsf(v[e]));
  }
  amax = block_reduce(amax, redf, [](float a, float b) { return fmaxf(a, b); }, 0.f);
  if (threadIdx.x == 0) amax_out[row] = amax;
}

}  // namespace tesm

using namespace tesm;

extern "C" int tesm_b200_weight_scale(const void *w, int dtype, int64_t N, int64_t K, int64_t ldw, int per_row,
                                      float eps, float *scale, float *deq, double *work, tesm_stream_t stream) {
  TESM_REQUIRE(w && scale && deq && work, "weight_scale: null pointer");
  TESM_REQUIRE(N > 0 && K > 0 && ldw >= K, "weight_scale: bad shape");
  if (dtype != TESM_F32 && dtype != TESM_BF16) return fail(TESM_EDTYPE, "weight_scale: dtype must be f32 or bf16");
  cudaStream_t st = (cudaStream_t)stream;
  k_row_abs_sum<<<(unsigned)ceil_div(N, 8), 256, 0, st>>>(w, dtype, N, K, ldw, work);
  if (per_row)
    k_row_scale<<<(unsigned)ceil_div(N, 256), 256, 0, st>>>(work, N, K, dtype, eps, scale, deq);
  else
    k_tensor_scale<<<1, 1024, 0, st>>>(work, N, K, dtype, eps, scale, deq);
  return check_launch("weight_scale");
}

extern "C" int tesm_b200_pack_ternary(const void *w, int dtype, int64_t N, int64_t K, int64_t ldw, int per_row,
                                      const float *scale, uint8_t *packed, int64_t ld_packed, int8_t *tern,
                                      int64_t ld_tern, tesm_stream_t stream) {
  TESM_REQUIRE(w && scale && packed, "pack_ternary: null pointer");
  TESM_REQUIRE(N > 0 && K > 0 && ldw >= K, "pack_ternary: bad shape");
  if (dtype != TESM_F32 && dtype != TESM_BF16) return fail(TESM_EDTYPE, "pack_ternary: dtype must be f32 or bf16");
  const int64_t Kp = round_up(K, 256);
  TESM_REQUIRE(ld_packed >= Kp / 4 && ld_packed % 4 == 0 && ((uintptr_t)packed & 3) == 0,
               "pack_ternary: ld_packed must be >= ceil(K/256)*64 bytes, a multiple of 4, pointer 4-aligned");
  if (tern)
    TESM_REQUIRE(ld_tern >= Kp && ld_tern % 16 == 0 && ((uintptr_t)tern & 15) == 0,
                 "pack_ternary: ld_tern must be >= K rounded up to 256, a multiple of 16, pointer 16-aligned");
  const int64_t gpr = Kp / 16;
  const int64_t total = N * gpr;
  k_pack<<<(unsigned)ceil_div(total, 256), 256, 0, (cudaStream_t)stream>>>(w, dtype, N, K, ldw, per_row, scale,
                                                                            packed, ld_packed, tern, ld_tern, gpr);
  return check_launch("pack_ternary");
}

static int quant_act_impl(const void *x, int dtype, int64_t M, int64_t K, int64_t ldx, float eps,
                          const float *amax, int8_t *codes, int64_t ld_codes, int layout, float *inv_scale,
                          int32_t *rowsum, tesm_stream_t stream) {
  if (M == 0) return TESM_OK;  // empty batch: nothing to do (its buffers may be null)
  TESM_REQUIRE(x && codes && inv_scale, "quant_act: null pointer");
  TESM_REQUIRE(M > 0 && K > 0 && ldx >= K, "quant_act: bad shape");
  if (dtype != TESM_F32 && dtype != TESM_BF16) return fail(TESM_EDTYPE, "quant_act: dtype must be f32 or bf16");
  TESM_REQUIRE(((uintptr_t)codes & 15) == 0 && ld_codes % 16 == 0, "quant_act: codes must be 16-byte aligned rows");
  int64_t groups_out;
  if (layout == TESM_LAYOUT_GEMV) {
    TESM_REQUIRE(rowsum != nullptr, "quant_act: GEMV layout needs rowsum");
    groups_out = round_up(K, 256) / 16;
    TESM_REQUIRE(ld_codes >= groups_out * 16, "quant_act: ld_codes < K rounded up to 256 for GEMV layout");
  } else if (layout == TESM_LAYOUT_ROWMAJOR) {
    groups_out = ceil_div(K, 16);
    TESM_REQUIRE(ld_codes >= groups_out * 16, "quant_act: ld_codes < K rounded up to 16");
  } else {
    return fail(TESM_EINVAL, "quant_act: unknown layout");
  }
  // few rows: short per-row chains; short rows (K < 2048): one group per thread, else most of
  // a 32-thread block would sit idle
  const int gpt = (M < 1024 && groups_out <= 1024) || groups_out < 128 ? 1 : kQuantGPT;
  int64_t threads = round_up(ceil_div(groups_out, gpt), 32);
  if (threads < 32) threads = 32;
  TESM_REQUIRE(threads <= 1024, "quant_act: K too large (max 65536)");
  const int esz = dtype == TESM_BF16 ? 2 : 4;
  const int vec = (K % 16 == 0) && ((uintptr_t)x % 16 == 0) && ((ldx * esz) % 16 == 0);
  if (M >= 1024 && groups_out <= 64)  // many short rows: one warp per row
    return launch_k("quant_act", k_quant_act_warp, dim3((unsigned)ceil_div(M, 8)), dim3(256), 0, (cudaStream_t)stream,
                    x, dtype, M, K, ldx, eps, codes, ld_codes, layout, groups_out, inv_scale, rowsum, vec, amax);
  if (dtype == TESM_BF16 && vec && layout == TESM_LAYOUT_ROWMAJOR)
    return launch_k("quant_act", gpt == 1 ? k_quant_act_bf16<1> : k_quant_act_bf16<kQuantGPT>, dim3((unsigned)M),
                    dim3((unsigned)threads), 0, (cudaStream_t)stream, reinterpret_cast<const __nv_bfloat16 *>(x), K,
                    ldx, eps, codes, ld_codes, inv_scale, amax);
  return launch_k("quant_act", gpt == 1 ? k_quant_act<1> : k_quant_act<kQuantGPT>, dim3((unsigned)M),
                  dim3((unsigned)threads), 0, (cudaStream_t)stream, x, dtype, K, ldx, eps, codes, ld_codes, layout,
                  groups_out, inv_scale, rowsum, vec, amax);
}

extern "C" int tesm_b200_quant_act(const void *x, int dtype, int64_t M, int64_t K, int64_t ldx, float eps,
                                   int8_t *codes, int64_t ld_codes, int layout, float *inv_scale, int32_t *rowsum,
                                   tesm_stream_t stream) {
  return quant_act_impl(x, dtype, M, K, ldx, eps, nullptr, codes, ld_codes, layout, inv_scale, rowsum, stream);
}

extern "C" int tesm_b200_quant_act_amax(const void *x, int dtype, int64_t M, int64_t K, int64_t ldx, float eps,
                                        const float *amax, int8_t *codes, int64_t ld_codes, int layout,
                                        float *inv_scale, int32_t *rowsum, tesm_stream_t stream) {
  TESM_REQUIRE(amax, "quant_act_amax: null amax");
  return quant_act_impl(x, dtype, M, K, ldx, eps, amax, codes, ld_codes, layout, inv_scale, rowsum, stream);
}

extern "C" int tesm_b200_row_absmax(const void *x, int dtype, int64_t M, int64_t K, int64_t ldx, float *amax,
                                    tesm_stream_t stream) {
  if (M == 0) return TESM_OK;  // empty batch: nothing to do (its buffers may be null)
  TESM_REQUIRE(x && amax && M >= 0 && K > 0 && ldx >= K, "row_absmax: bad argument");
  if (dtype != TESM_F32 && dtype != TESM_BF16) return fail(TESM_EDTYPE, "row_absmax: dtype must be f32 or bf16");
  const int esz = dtype == TESM_BF16 ? 2 : 4;
  const int vec = (K % 16 == 0) && ((uintptr_t)x % 16 == 0) && ((ldx * esz) % 16 == 0);
  k_row_absmax<<<(unsigned)M, 128, 0, (cudaStream_t)stream>>>(x, dtype, K, ldx, vec, amax);
  return check_launch("row_absmax");
}

extern "C" int tesm_b200_unpack_ternary(const uint8_t *packed, int64_t ld_packed, int64_t N, int64_t Kp,
                                        int8_t *tern, int64_t ld_tern, tesm_stream_t stream) {
  TESM_REQUIRE(packed && tern && N > 0 && Kp > 0 && Kp % 16 == 0, "unpack_ternary: need Kp a multiple of 16");
  TESM_REQUIRE(ld_packed >= Kp / 4 && ld_packed % 4 == 0 && ((uintptr_t)packed & 3) == 0,
               "unpack_ternary: packed rows must hold Kp / 4 bytes, 4-byte aligned");
  TESM_REQUIRE(ld_tern >= Kp && ld_tern % 16 == 0 && ((uintptr_t)tern & 15) == 0,
               "unpack_ternary: tern rows must hold Kp bytes, 16-byte aligned");
  const int64_t wpr = Kp / 16, total = N * wpr;
  k_unpack<<<(unsigned)ceil_div(total, 256), 256, 0, (cudaStream_t)stream>>>(packed, ld_packed, N, wpr, tern, ld_tern);
  return check_launch("unpack_ternary");
}
