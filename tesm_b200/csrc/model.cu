// Model-level glue kernels: embedding gather, fused residual + RMSNorm + int8 quantisation,
// SiLU-gated product, prefill -> decode-cache fill.
// References: MixerModel.forward (tesm_ssm/models/mixer_seq_simple.py:171-242),
// Block.forward / RMSNorm (tesm_ssm/modules/block.py:14-45), FeedForward.forward
// (mixer_seq_simple.py:59-67), prefill cache write (tesm.py:1235-1253, tesm_mimo.py:1022-1038).
#include "layer_common.cuh"
#include "rowio.cuh"

namespace tesm {

// hidden[m] = E[ids[m]] + P[pos0 + m % L]  (mixer_seq_simple.py:183-184)
__global__ void k_embed(const int64_t *ids, int64_t M, int L, const void *emb, const void *pemb, int wdtype, int Dm,
                        const int *pos_dev, int pos_host, void *out, int odtype) {
  pdl_trigger();
  pdl_wait();
  const int64_t m = blockIdx.x;
  const int pos = (pos_dev ? pos_dev[0] : pos_host) + (int)(m % L);
  const int64_t id = ids[m];
  for (int c = threadIdx.x; c < Dm; c += blockDim.x) {
    const float v = load_f(emb, wdtype, id * Dm + c) + load_f(pemb, wdtype, (int64_t)pos * Dm + c);
    store_f(out, odtype, m * Dm + c, v);
  }
}

// residual_out = x (+ residual); y = residual_out * rsqrt(mean(residual_out^2) + eps) * w;
// then the per-token int8 codes of y (same arithmetic as quant.cu), optionally y itself.
// Rows are held in registers (GPT 16-element groups per thread) with 16-byte vector I/O.
template <int GPT>
__global__ void k_add_rmsnorm_quant(const void *x, int xdtype, const float *residual, float *residual_out,
                                    const float *w, float eps, int K, float qeps, int8_t *codes, int64_t ld_codes,
                                    int layout, int64_t groups_out, float *inv_scale, int32_t *rowsum, void *y_out,
                                    int ydtype, int vec) {
  __shared__ float redf[32];
  __shared__ int redi[32];
  pdl_trigger();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const int64_t groups_in = (K + 15) / 16;
  const int xsz = xdtype == TESM_BF16 ? 2 : 4, ysz = ydtype == TESM_BF16 ? 2 : 4;
  const void *xrow = reinterpret_cast<const uint8_t *>(x) + row * K * xsz;
  float v[GPT][16];
  float ss = 0.f;
  // one group per thread (decode rows): the norm weight is requested with the inputs instead of
  // after the sum-of-squares reduction (one dependent round trip fewer)
  float wpre[16];
  if (GPT == 1 && (int64_t)threadIdx.x < groups_in) load16(w, TESM_F32, (int64_t)threadIdx.x * 16, K, vec, wpre);
#pragma unroll
  for (int j = 0; j < GPT; ++j) {
    const int64_t g = threadIdx.x + (int64_t)j * blockDim.x;
    if (g < groups_in) {
      load16(xrow, xdtype, g * 16, K, vec, v[j]);
      if (residual) {
        float r[16];
        load16(residual + row * K, TESM_F32, g * 16, K, vec, r);
#pragma unroll
        for (int e = 0; e < 16; ++e) v[j][e] += r[e];
      }
      if (residual_out) store16(residual_out + row * K, TESM_F32, g * 16, K, vec, v[j]);
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) v[j][e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < 16; ++e) ss = fmaf(v[j][e], v[j][e], ss);
  }
  ss = block_reduce(ss, redf, [](float a, float b) { return a + b; }, 0.f);
  const float rs = rsqrtf(ss / (float)K + eps);
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < GPT; ++j) {
    const int64_t g = threadIdx.x + (int64_t)j * blockDim.x;
    if (g < groups_in) {
      float wv[16];
      if (GPT == 1) {
#pragma unroll
        for (int e = 0; e < 16; ++e) wv[e] = wpre[e];
      } else {
        load16(w, TESM_F32, g * 16, K, vec, wv);
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) v[j][e] = (v[j][e] * rs) * wv[e];
      if (y_out) store16(reinterpret_cast<uint8_t *>(y_out) + row * K * ysz, ydtype, g * 16, K, vec, v[j]);
    }
#pragma unroll
    for (int e = 0; e < 16; ++e) amax = fmaxf(amax, fabsf(v[j][e]));
  }
  if (!codes) return;
  amax = block_reduce(amax, redf, [](float a, float b) { return fmaxf(a, b); }, 0.f);
  const float s = act_scale(amax, qeps, TESM_F32);
  if (threadIdx.x == 0) inv_scale[row] = __frcp_rn(s);
  int csum = 0;
  int8_t *crow = codes + row * ld_codes;
#pragma unroll
  for (int j = 0; j < GPT; ++j) {
    const int64_t g = threadIdx.x + (int64_t)j * blockDim.x;
    if (g >= groups_out) continue;
    if (layout == TESM_LAYOUT_ROWMAJOR && !rowsum) {  // act_code via act_code_bits (FMA pipe only)
      uint32_t wv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        wv[q] = pack_code_bytes(act_code_bits(__fmul_rn(v[j][4 * q], s)), act_code_bits(__fmul_rn(v[j][4 * q + 1], s)),
                                act_code_bits(__fmul_rn(v[j][4 * q + 2], s)),
                                act_code_bits(__fmul_rn(v[j][4 * q + 3], s)));
      reinterpret_cast<uint4 *>(crow)[g] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
      continue;
    }
    int c[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      c[e] = act_code(v[j][e], s, TESM_F32);
      csum += c[e];
    }
    store_codes16(crow, g, layout, c);
  }
  if (rowsum) {
    csum = block_reduce(csum, redi, [](int a, int b) { return a + b; }, 0);
    if (threadIdx.x == 0) rowsum[row] = csum;
  }
}

// out[m, f] = silu(gate[m, f]) * up[m, f]; gu holds [gate | up] halves (blk == 0) or
// blocks of `blk` gate columns followed by the matching `blk` up columns.
// Thread = 8 consecutive output columns of one row (grid.y strides over rows): 16-byte
// bf16 / 32-byte fp32 vectors when aligned; blk is a multiple of 8, so a group never straddles
// an interleave block.
__global__ void k_silu_mul(const void *gu, int dtype, int64_t M, int F, void *out, int odtype, int blk, int vec) {
  pdl_trigger();
  pdl_wait();
  const int f0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (f0 >= F) return;
  int gcol, ucol;
  if (blk) {
    const int b = f0 / blk, j = f0 - b * blk;
    gcol = b * 2 * blk + j;
    ucol = gcol + blk;
  } else {
    gcol = f0;
    ucol = f0 + F;
  }
  const int gsz = dtype == TESM_BF16 ? 2 : 4, osz = odtype == TESM_BF16 ? 2 : 4;
  for (int64_t m = blockIdx.y; m < M; m += gridDim.y) {
    const uint8_t *row = reinterpret_cast<const uint8_t *>(gu) + m * 2 * (int64_t)F * gsz;
    float g[8], u[8], o[8];
    // columns past F only occur without an interleave (blk == 0, F % 8 != 0, scalar path)
    load8(row, dtype, gcol, blk ? gcol + 8 : F, vec != 0, g);
    load8(row, dtype, ucol, blk ? ucol + 8 : 2 * F, vec != 0, u);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = (g[e] * sigmoidf_(g[e])) * u[e];
    store8(reinterpret_cast<uint8_t *>(out) + m * (int64_t)F * osz, odtype, f0, F, vec != 0, o);
  }
}

// Prefill -> cache (tesm.py:1235-1253): last min(L, W) positions of rope(k) and of the
// (rank-0) states; L >= W fills slots 0..W-1, L < W fills slots W-L..W-1; cache_idx = 0.
__global__ void k_cache_fill(ProjCols pc, const float *states, int RM, int B, int L, int H, int D, int R, int W,
                             const __grid_constant__ RopeTab rt, const double *final_f64, double *state, float *kc, float *vc,
                             int *ctl) {
  const int b = blockIdx.y, n = min(L, W), i = blockIdx.x;
  if (i >= n) return;
  const int t = L - n + i;
  const int slot = L >= W ? i : W - L + t;
  const int64_t row = (int64_t)b * L + t;
  const int C = H * D;
  for (int h = 0; h < H; ++h)
    load_rope_row(kc + (((int64_t)b * W + slot) * H + h) * R, pc, pc.c_k + h * R, row, R, t, rt.v, nullptr,
                  threadIdx.x, blockDim.x);
  for (int c = threadIdx.x; c < C; c += blockDim.x) vc[((int64_t)b * W + slot) * C + c] = states[row * RM * C + c];
  if (i == 0) {
    for (int c = threadIdx.x; c < C; c += blockDim.x) state[(int64_t)b * C + c] = final_f64[(int64_t)b * C + c];
    if (b == 0 && threadIdx.x == 0) {
      ctl[0] = L;
      ctl[1] = 0;
      ctl[2] = 0;
    }
  }
}

}  // namespace tesm

using namespace tesm;

extern "C" int tesm_b200_embed(const int64_t *ids, int64_t B, int64_t L, const void *emb, const void *pos_emb,
                               int wdtype, int64_t Dm, const int *pos_dev, int64_t pos_host, void *out, int odtype,
                               tesm_stream_t stream) {
  TESM_REQUIRE(ids && emb && pos_emb && out && B > 0 && L > 0 && Dm > 0, "embed: bad argument");
  return launch_k("embed", k_embed, dim3((unsigned)(B * L)), dim3(256), 0, (cudaStream_t)stream, ids, B * L, (int)L,
                  emb, pos_emb, wdtype, (int)Dm, pos_dev, (int)pos_host, out, odtype);
}

extern "C" int tesm_b200_add_rmsnorm_quant(const void *x, int xdtype, const float *residual, float *residual_out,
                                           const float *weight, float eps, int64_t M, int64_t K, float qeps,
                                           int8_t *codes, int64_t ld_codes, int layout, float *inv_scale,
                                           int32_t *rowsum, void *y_out, int ydtype, tesm_stream_t stream) {
  if (M == 0) return TESM_OK;  // empty batch: nothing to do (its buffers may be null)
  TESM_REQUIRE(x && weight && M >= 0 && K > 0, "add_rmsnorm_quant: bad argument");
  int64_t groups_out = ceil_div(K, 16);
  if (codes) {
    TESM_REQUIRE(inv_scale && ((uintptr_t)codes & 15) == 0 && ld_codes % 16 == 0, "add_rmsnorm_quant: codes");
    if (layout == TESM_LAYOUT_GEMV) {
      TESM_REQUIRE(rowsum != nullptr, "add_rmsnorm_quant: GEMV layout needs rowsum");
      groups_out = round_up(K, 256) / 16;
    }
    TESM_REQUIRE(ld_codes >= groups_out * 16, "add_rmsnorm_quant: ld_codes too small");
  }
  const int vec = (K % 16 == 0) && ((uintptr_t)x % 16 == 0) && (!residual || (uintptr_t)residual % 16 == 0) &&
                  (!residual_out || (uintptr_t)residual_out % 16 == 0) && ((uintptr_t)weight % 16 == 0) &&
                  (!y_out || (uintptr_t)y_out % 16 == 0);
  // few rows (decode): one 16-element group per thread, so each row's latency chain is short
  static const int gpt_big = [] {
    const char *e = getenv("TESM_ARQ_GPT");  // tuning override: 16-element groups per thread, many rows
    const int v = e ? atoi(e) : 2;  // 2: 56 registers, 0.76 of HBM at 16384 x 4096 (4: 0.70, 1: 0.74)
    return v == 4 ? 4 : v == 1 ? 1 : 2;
  }();
  const int gpt = M < 1024 && groups_out <= 1024 ? 1 : gpt_big;
  int64_t threads = round_up(ceil_div(groups_out, gpt), 32);
  if (threads < 32) threads = 32;
  TESM_REQUIRE(threads <= 1024, "add_rmsnorm_quant: K too large");
  return launch_k("add_rmsnorm_quant",
                  gpt == 1 ? k_add_rmsnorm_quant<1> : gpt == 2 ? k_add_rmsnorm_quant<2> : k_add_rmsnorm_quant<4>,
                  dim3((unsigned)M), dim3((unsigned)threads), 0, (cudaStream_t)stream, x, xdtype, residual,
                  residual_out, weight, eps, (int)K, qeps, codes, ld_codes, layout, groups_out, inv_scale, rowsum,
                  y_out, ydtype, vec);
}

extern "C" int tesm_b200_silu_mul(const void *gu, int dtype, int64_t M, int64_t F, int64_t blk, void *out,
                                  int odtype, tesm_stream_t stream) {
  if (M == 0) return TESM_OK;  // empty batch: nothing to do (its buffers may be null)
  TESM_REQUIRE(blk == 0 || F % blk == 0, "silu_mul: F must be a multiple of the interleave block");
  TESM_REQUIRE(gu && out && M >= 0 && F > 0, "silu_mul: bad argument");
  TESM_REQUIRE(blk == 0 || blk % 8 == 0, "silu_mul: interleave block must be a multiple of 8");
  const int gsz = dtype == TESM_BF16 ? 2 : 4, osz = odtype == TESM_BF16 ? 2 : 4;
  const int vec = (F % 8 == 0) && ((uintptr_t)gu % 16 == 0) && ((uintptr_t)out % 16 == 0) && ((F * gsz) % 16 == 0) &&
                  ((F * osz) % 16 == 0);
  const int64_t groups = ceil_div(F, 8);
  const int threads = groups >= 128 ? 128 : (int)round_up(groups, 32);
  dim3 grid((unsigned)ceil_div(groups, threads), (unsigned)(M < 65535 ? M : 65535));
  return launch_k("silu_mul", k_silu_mul, grid, dim3(threads), 0, (cudaStream_t)stream, gu, dtype, M, (int)F, out,
                  odtype, (int)blk, vec);
}

extern "C" int tesm_b200_cache_fill(const void *proj, int dtype, int64_t ldp, const float *states, int64_t RM,
                                    int64_t B, int64_t L, int64_t Dm, int64_t H, int64_t D, int64_t R, int64_t W,
                                    float rope_base, const double *final_f64, double *state, float *k_cache,
                                    float *v_cache, int *ctl, tesm_stream_t stream) {
  TESM_REQUIRE(proj && states && final_f64 && state && k_cache && v_cache && ctl, "cache_fill: null pointer");
  TESM_REQUIRE(B > 0 && L > 0 && W > 0, "cache_fill: bad shape");
  ProjCols pc = make_cols(proj, dtype, ldp, (int)Dm, (int)(H * D), (int)(H * R));
  dim3 grid((unsigned)(L < W ? L : W), (unsigned)B);
  k_cache_fill<<<grid, 128, 0, (cudaStream_t)stream>>>(pc, states, (int)RM, (int)B, (int)L, (int)H, (int)D, (int)R,
                                                       (int)W, rope_table((int)R, rope_base), final_f64, state, k_cache, v_cache, ctl);
  return check_launch("cache_fill");
}
