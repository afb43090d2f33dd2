// MIMO local entanglement with the rank merge (tesm_mimo.py:996-1017, torch rung :525-588).
//
// Per (b, t, h) the ternary weights depend only on q, k and the per-head bias, so they are
// computed once and shared by all mimo ranks; each rank's states get the signed window
// average, the lerp toward it, and the ranks are merged with mimo_o:
//   ent = sum_r mo[h,r,:] * (s_r + es (avg_r - s_r)),  chg = sum_r mo[h,r,:] * es (avg_r - s_r).
// The reference's window truncation for t < W-1 (only lags o in [W-1-t, t] take part) is
// reproduced when `quirk` is set (the default, for parity).
#include "layer_common.cuh"

namespace tesm {

struct MimoEntParams {
  ProjCols pc;
  const float *bias;    // (H, W)
  const float *mimo_o;  // (H, RM, D)
  const float *states;  // (B, L, RM, H*D)
  int B, L, H, D, R, RM, T, quirk;
  float thr, es, sqrt_r, rope_base;
  void *out_tanh, *out_chg;  // (B*L, H*D)
  int out_dtype;
};

template <int W, int RM>
__global__ void __launch_bounds__(128, 3) k_mimo_local_ent(MimoEntParams p) {
  extern __shared__ float sm[];
  const int R = p.R, T = p.T, RP = R + 1;
  float *qs = sm;
  float *ks = qs + T * RP;
  float *tw = ks + (T + W - 1) * RP;
  float *invf = tw + T * W;
  const int h = blockIdx.y, b = blockIdx.z;
  const int t0 = blockIdx.x * T;
  const int64_t row0 = (int64_t)b * p.L;
  const int nt = min(T, p.L - t0);
  const int C = p.H * p.D;
  const int nwarp = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < R / 2; i += blockDim.x) invf[i] = rope_inv_freq(i, R, p.rope_base);
  __syncthreads();
  for (int r = warp; r < nt; r += nwarp)
    load_rope_row_tab(qs + r * RP, p.pc, p.pc.c_q + h * R, row0 + t0 + r, R, t0 + r, invf, nullptr, lane, 32);
  for (int r = warp; r < nt + W - 1; r += nwarp) {
    const int pos = t0 - (W - 1) + r;
    if (pos < 0) continue;
    load_rope_row_tab(ks + r * RP, p.pc, p.pc.c_k + h * R, row0 + pos, R, pos, invf, nullptr, lane, 32);
  }
  __syncthreads();
  const int quirk = p.quirk;
  window_scores<W>(qs, ks, RP, R, nt, t0, p.bias + h * W, p.sqrt_r, p.thr, tw, [quirk](int gt, int o) {
    return gt - o >= 0 && (!quirk || o >= W - 1 - gt);
  });
  __syncthreads();
  for (int d = threadIdx.x; d < p.D; d += blockDim.x) {
    const int c = h * p.D + d;
    float mo[RM];
#pragma unroll
    for (int r = 0; r < RM; ++r) mo[r] = p.mimo_o[((int64_t)h * RM + r) * p.D + d];
    float win[RM][W];  // before the first shift win[r][o] = states_r[t0 - 1 - o]
#pragma unroll
    for (int r = 0; r < RM; ++r) win[r][W - 1] = 0.f;
#pragma unroll
    for (int o = 1; o < W; ++o) {
      const int j = t0 - o;
#pragma unroll
      for (int r = 0; r < RM; ++r) win[r][o - 1] = j >= 0 ? p.states[((row0 + j) * RM + r) * C + c] : 0.f;
    }
    constexpr int PF = 4;  // timesteps prefetched per batch (x RM loads)
    for (int tb = 0; tb < nt; tb += PF) {
      float sv[PF][RM];
#pragma unroll
      for (int j = 0; j < PF; ++j)
#pragma unroll
        for (int r = 0; r < RM; ++r)
          sv[j][r] = tb + j < nt ? p.states[((row0 + t0 + tb + j) * RM + r) * C + c] : 0.f;
#pragma unroll
      for (int j = 0; j < PF; ++j) {
        if (tb + j < nt) {
          const int t = tb + j;
          const int64_t row = row0 + t0 + t;
          float ent = 0.f, chg = 0.f;
#pragma unroll
          for (int r = 0; r < RM; ++r) {
#pragma unroll
            for (int o = W - 1; o > 0; --o) win[r][o] = win[r][o - 1];
            const float s = sv[j][r];
            win[r][0] = s;
            float avg = 0.f;
#pragma unroll
            for (int o = 0; o < W; ++o) avg = fmaf(tw[t * W + o], win[r][o], avg);
            const float e_r = s + p.es * (avg - s);
            ent = fmaf(mo[r], e_r, ent);
            chg = fmaf(mo[r], e_r - s, chg);
          }
          store_f(p.out_tanh, p.out_dtype, row * C + c, tanhf(ent));
          store_f(p.out_chg, p.out_dtype, row * C + c, chg);
        }
      }
    }
  }
}

template <int W, int RM>
static int launch_mimo_ent(MimoEntParams &p, cudaStream_t st) {
  const size_t smem = sizeof(float) * ((size_t)p.T * (p.R + 1) + (size_t)(p.T + W - 1) * (p.R + 1) + p.T * W +
                                       p.R / 2);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_mimo_local_ent<W, RM>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    cudaFuncSetAttribute(k_mimo_local_ent<W, RM>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    attr = true;
  }
  if (smem > 160 * 1024) return fail(TESM_EUNSUPPORTED, "mimo_local_ent: ent_rank too large");
  dim3 grid((unsigned)ceil_div(p.L, p.T), (unsigned)p.H, (unsigned)p.B);
  const int threads = p.D >= 128 ? 128 : (p.D <= 64 ? 64 : 128);
  k_mimo_local_ent<W, RM><<<grid, threads, smem, st>>>(p);
  return check_launch("mimo_local_ent");
}

}  // namespace tesm

using namespace tesm;

extern "C" int tesm_b200_mimo_local_ent(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L, int64_t Dm,
                                        int64_t H, int64_t D, int64_t R, int64_t RM, int64_t W, const float *bias,
                                        const float *mimo_o, const float *states, float thr, float es,
                                        float rope_base, int quirk, void *out_tanh, void *out_chg, int out_dtype,
                                        tesm_stream_t stream) {
  TESM_REQUIRE(proj && bias && mimo_o && states && out_tanh && out_chg, "mimo_local_ent: null pointer");
  TESM_REQUIRE(B > 0 && L > 0 && H > 0 && D > 0 && R > 0 && R % 2 == 0, "mimo_local_ent: bad shape");
  if (dtype != TESM_F32 && dtype != TESM_BF16) return fail(TESM_EDTYPE, "mimo_local_ent: dtype");
  MimoEntParams p;
  p.pc = make_cols(proj, dtype, ldp, (int)Dm, (int)(H * D), (int)(H * R));
  p.bias = bias;
  p.mimo_o = mimo_o;
  p.states = states;
  p.B = (int)B;
  p.L = (int)L;
  p.H = (int)H;
  p.D = (int)D;
  p.R = (int)R;
  p.RM = (int)RM;
  p.T = 64;
  p.quirk = quirk;
  p.thr = thr;
  p.es = es;
  p.sqrt_r = (float)sqrt((double)R);
  p.rope_base = rope_base;
  p.out_tanh = out_tanh;
  p.out_chg = out_chg;
  p.out_dtype = out_dtype;
  cudaStream_t st = (cudaStream_t)stream;
#define TESM_MIMO_CASE(WW, RR) \
  if (W == WW && RM == RR) return launch_mimo_ent<WW, RR>(p, st);
  TESM_MIMO_CASE(8, 1) TESM_MIMO_CASE(8, 2) TESM_MIMO_CASE(8, 4) TESM_MIMO_CASE(16, 1) TESM_MIMO_CASE(16, 2)
  TESM_MIMO_CASE(16, 4)
#undef TESM_MIMO_CASE
  return fail(TESM_EUNSUPPORTED, "mimo_local_ent: supported (window, mimo_rank) are {8,16} x {1,2,4}");
}
