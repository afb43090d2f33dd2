// MIMO local entanglement with the rank merge (tesm_mimo.py:996-1017, torch rung :525-588).
//
// Per (b, t, h) the ternary weights depend only on q, k and the per-head bias, so they are
// computed once and shared by all mimo ranks; each rank's states get the signed window
// average, the lerp toward it, and the ranks are merged with mimo_o:
//   ent = sum_r mo[h,r,:] * (s_r + es (avg_r - s_r)),  chg = sum_r mo[h,r,:] * es (avg_r - s_r).
// The reference's window truncation for t < W-1 (only lags o in [W-1-t, t] take part) is
// reproduced when `quirk` is set (the default, for parity).  The kernel is the persistent window
// kernel of window.cuh in its MIMO mode (ranks in the tensor-core columns, merge in the epilogue).
#include "window.cuh"

#include <algorithm>

namespace tesm {

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
  if (out_dtype != TESM_F32 && out_dtype != TESM_BF16) return fail(TESM_EDTYPE, "mimo_local_ent: out dtype");
  const ProjCols pc = make_cols(proj, dtype, ldp, (int)Dm, (int)(H * D), (int)(H * R));
  WinEntParams p{};
  p.proj = proj;
  p.ld = ldp;
  p.c_q = pc.c_q;
  p.c_k = pc.c_k;
  p.states = states;
  p.pos_ld = RM * H * D;
  p.rank_ld = H * D;
  p.bias = bias;
  p.mimo_o = mimo_o;
  p.B = (int)B;
  p.L = (int)L;
  p.H = (int)H;
  p.D = (int)D;
  p.R = (int)R;
  p.quirk = quirk;
  p.thr = thr;
  p.es = es;
  p.sqrt_r = (float)sqrt((double)R);
  p.rope_base = rope_base;
  p.out_tanh = out_tanh;
  p.out_chg = out_chg;
  p.out_dtype = out_dtype;
  p.out_ld = H * D;
  cudaStream_t st = (cudaStream_t)stream;
#define TESM_MIMO_CASE(WW, RR)                                                                              \
  if (W == WW && RM == RR)                                                                                  \
    return dtype == TESM_BF16 ? win_launch<WW, RR, 2, kWinMimo>(p, st, "mimo_local_ent")                    \
                              : win_launch<WW, RR, 4, kWinMimo>(p, st, "mimo_local_ent");
  TESM_MIMO_CASE(8, 1) TESM_MIMO_CASE(8, 2) TESM_MIMO_CASE(8, 4) TESM_MIMO_CASE(16, 1) TESM_MIMO_CASE(16, 2)
  TESM_MIMO_CASE(16, 4)
#undef TESM_MIMO_CASE
  return fail(TESM_EUNSUPPORTED, "mimo_local_ent: supported (window, mimo_rank) are {8,16} x {1,2,4}");
}
