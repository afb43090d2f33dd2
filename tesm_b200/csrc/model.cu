// Model-level glue kernels: embedding gather, fused residual + RMSNorm + int8 quantisation,
// SiLU-gated product, prefill -> decode-cache fill.
// References: MixerModel.forward (tesm_ssm/models/mixer_seq_simple.py:171-242),
// Block.forward / RMSNorm (tesm_ssm/modules/block.py:14-45), FeedForward.forward
// (mixer_seq_simple.py:59-67), prefill cache write (tesm.py:1235-1253, tesm_mimo.py:1022-1038).
#include "layer_common.cuh"

namespace tesm {

// hidden[m] = E[ids[m]] + P[pos0 + m % L]  (mixer_seq_simple.py:183-184)
__global__ void k_embed(const int64_t *ids, int64_t M, int L, const void *emb, const void *pemb, int wdtype, int Dm,
                        const int *pos_dev, int pos_host, void *out, int odtype) {
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
template <int GPT>
__global__ void k_add_rmsnorm_quant(const void *x, int xdtype, const float *residual, float *residual_out,
                                    const float *w, float eps, int K, float qeps, int8_t *codes, int64_t ld_codes,
                                    int layout, int64_t groups_out, float *inv_scale, int32_t *rowsum, void *y_out,
                                    int ydtype) {
  __shared__ float redf[32];
  __shared__ int redi[32];
  __shared__ double redd[32];
  const int64_t row = blockIdx.x;
  const int64_t groups_in = (K + 15) / 16;
  float v[GPT][16];
  double ss = 0.0;
#pragma unroll
  for (int j = 0; j < GPT; ++j) {
    const int64_t g = threadIdx.x + (int64_t)j * blockDim.x;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int64_t k = g * 16 + e;
      float r = 0.f;
      if (g < groups_in && k < K) {
        r = load_f(x, xdtype, row * K + k);
        if (residual) r += residual[row * K + k];
        if (residual_out) residual_out[row * K + k] = r;
      }
      v[j][e] = r;
      ss += (double)r * (double)r;
    }
  }
  ss = block_reduce(ss, redd, [](double a, double b) { return a + b; }, 0.0);
  const float rs = rsqrtf((float)(ss / (double)K) + eps);
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < GPT; ++j) {
    const int64_t g = threadIdx.x + (int64_t)j * blockDim.x;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int64_t k = g * 16 + e;
      float y = 0.f;
      if (g < groups_in && k < K) {
        y = (v[j][e] * rs) * w[k];
        if (y_out) store_f(y_out, ydtype, row * K + k, y);
      }
      v[j][e] = y;
      amax = fmaxf(amax, fabsf(y));
    }
  }
  if (!codes) return;
  amax = block_reduce(amax, redf, [](float a, float b) { return fmaxf(a, b); }, 0.f);
  const float mx = fmaxf(amax, qeps);
  const float s = __fmul_rn(__frcp_rn(mx), 127.f);
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
      c[e] = (int)fminf(fmaxf(rintf(__fmul_rn(v[j][e], s)), -128.f), 127.f);
      csum += c[e];
    }
    uint32_t wv[4];
    if (layout == TESM_LAYOUT_GEMV) {
#pragma unroll
      for (int sw = 0; sw < 4; ++sw)
        wv[sw] = (uint32_t)(uint8_t)c[sw] | ((uint32_t)(uint8_t)c[4 + sw] << 8) |
                 ((uint32_t)(uint8_t)c[8 + sw] << 16) | ((uint32_t)(uint8_t)c[12 + sw] << 24);
      const int64_t s256 = g >> 4, tig = (g >> 2) & 3, u = g & 3;
      reinterpret_cast<uint4 *>(crow)[s256 * 16 + u * 4 + tig] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        wv[q] = (uint32_t)(uint8_t)c[4 * q] | ((uint32_t)(uint8_t)c[4 * q + 1] << 8) |
                ((uint32_t)(uint8_t)c[4 * q + 2] << 16) | ((uint32_t)(uint8_t)c[4 * q + 3] << 24);
      reinterpret_cast<uint4 *>(crow)[g] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
  }
  if (rowsum) {
    csum = block_reduce(csum, redi, [](int a, int b) { return a + b; }, 0);
    if (threadIdx.x == 0) rowsum[row] = csum;
  }
}

// out[m, f] = silu(gu[m, f]) * gu[m, F + f]
__global__ void k_silu_mul(const void *gu, int dtype, int64_t M, int F, void *out, int odtype) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= M * F) return;
  const int64_t m = i / F;
  const int f = (int)(i - m * F);
  const float g = load_f(gu, dtype, m * 2 * F + f);
  const float u = load_f(gu, dtype, m * 2 * F + F + f);
  store_f(out, odtype, i, (g * sigmoidf_(g)) * u);
}

// Prefill -> cache (tesm.py:1235-1253): last min(L, W) positions of rope(k) and of the
// (rank-0) states; L >= W fills slots 0..W-1, L < W fills slots W-L..W-1; cache_idx = 0.
__global__ void k_cache_fill(ProjCols pc, const float *states, int RM, int B, int L, int H, int D, int R, int W,
                             float rope_base, const double *final_f64, double *state, float *kc, float *vc,
                             int *ctl) {
  const int b = blockIdx.y, n = min(L, W), i = blockIdx.x;
  if (i >= n) return;
  const int t = L - n + i;
  const int slot = L >= W ? i : W - L + t;
  const int64_t row = (int64_t)b * L + t;
  const int C = H * D;
  for (int h = 0; h < H; ++h)
    load_rope_row(kc + (((int64_t)b * W + slot) * H + h) * R, pc, pc.c_k + h * R, row, R, t, rope_base, nullptr,
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
  k_embed<<<(unsigned)(B * L), 256, 0, (cudaStream_t)stream>>>(ids, B * L, (int)L, emb, pos_emb, wdtype, (int)Dm,
                                                               pos_dev, (int)pos_host, out, odtype);
  return check_launch("embed");
}

extern "C" int tesm_b200_add_rmsnorm_quant(const void *x, int xdtype, const float *residual, float *residual_out,
                                           const float *weight, float eps, int64_t M, int64_t K, float qeps,
                                           int8_t *codes, int64_t ld_codes, int layout, float *inv_scale,
                                           int32_t *rowsum, void *y_out, int ydtype, tesm_stream_t stream) {
  TESM_REQUIRE(x && weight && M >= 0 && K > 0, "add_rmsnorm_quant: bad argument");
  if (M == 0) return TESM_OK;
  int64_t groups_out = ceil_div(K, 16);
  if (codes) {
    TESM_REQUIRE(inv_scale && ((uintptr_t)codes & 15) == 0 && ld_codes % 16 == 0, "add_rmsnorm_quant: codes");
    if (layout == TESM_LAYOUT_GEMV) {
      TESM_REQUIRE(rowsum != nullptr, "add_rmsnorm_quant: GEMV layout needs rowsum");
      groups_out = round_up(K, 256) / 16;
    }
    TESM_REQUIRE(ld_codes >= groups_out * 16, "add_rmsnorm_quant: ld_codes too small");
  }
  int64_t threads = round_up(ceil_div(groups_out, 4), 32);
  if (threads < 32) threads = 32;
  TESM_REQUIRE(threads <= 1024, "add_rmsnorm_quant: K too large");
  k_add_rmsnorm_quant<4><<<(unsigned)M, (unsigned)threads, 0, (cudaStream_t)stream>>>(
      x, xdtype, residual, residual_out, weight, eps, (int)K, qeps, codes, ld_codes, layout, groups_out, inv_scale,
      rowsum, y_out, ydtype);
  return check_launch("add_rmsnorm_quant");
}

extern "C" int tesm_b200_silu_mul(const void *gu, int dtype, int64_t M, int64_t F, void *out, int odtype,
                                  tesm_stream_t stream) {
  TESM_REQUIRE(gu && out && M >= 0 && F > 0, "silu_mul: bad argument");
  if (M == 0) return TESM_OK;
  const int64_t n = M * F;
  k_silu_mul<<<(unsigned)ceil_div(n, 256), 256, 0, (cudaStream_t)stream>>>(gu, dtype, M, (int)F, out, odtype);
  return check_launch("silu_mul");
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
                                                       (int)W, rope_base, final_f64, state, k_cache, v_cache, ctl);
  return check_launch("cache_fill");
}
