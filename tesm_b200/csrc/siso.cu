// SISO layer kernels: selective state scan, local / global ternary entanglement, output
// combine.  Reference: tesm_ssm/modules/tesm.py (TESM_SISO.forward :1175-1272).
//
// Layout: the in_proj output `proj` is (B*L, Nproj) row-major with the reference's
// column split [local Dm | value D | decay D | write D | gate Dm | q R | k R]
// (tesm.py:1195-1205); kernels read their columns in place through offsets.
#include "window.cuh"
#include "rowio.cuh"

#include <algorithm>

namespace tesm {


// ---------------------------------------------------------------- global entanglement
// Causal O(L^2) variant (tesm.py:963-1043): relative bias depends on i - j only and is
// passed as a vector over d = i - j (index d + L - 1).
__global__ void k_global_relbias(const float *embed, int dim, float scale, float bias0, int L, float *out) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= 2 * L - 1) return;
  const float d = (float)(idx - (L - 1));
  float ss = 0.f, cc = 0.f;
  const float pi_f = 3.14159265358979323846f;
  for (int k = 0; k < dim; ++k) {
    const float f = __fdiv_rn(__fmul_rn((float)(k + 1), pi_f), 1000.f);
    float sn, cs;
    sincosf(d * f, &sn, &cs);
    ss += sn * embed[k];
    cc += cs * embed[k];
  }
  out[idx] = (ss + cc) * scale + bias0;
}

struct GlobalEntParams {
  ProjCols pc;
  const float *cross;
  const float *relb;    // (2L - 1)
  const float *states;  // row r, channel c at states[r * s_ld + s_off + c]
  int64_t s_ld;
  int s_off;
  int B, L, D, R;       // D: state channels (H*Dh for MIMO), R: q/k columns (H*Rh for MIMO)
  int rope_heads;       // RoPE applied per head on R / rope_heads columns
  int dslice;           // channels per CTA (blockIdx.z)
  float thr, es, sqrt_r, rope_base;
  RopeTab rt;
  void *out_tanh, *out_chg;
  int out_dtype;
  // MIMO rank accumulation (tesm_mimo.py:1007-1017 with the global rung :669-687, no lerp)
  int mimo, RM, r, Dh;
  const float *mo;
  float *acc_e, *acc_c;
};

// One CTA per (query tile of 32 rows, batch, channel slice); loops over causal key tiles of 32.
__global__ void __launch_bounds__(256) k_siso_global_ent(const __grid_constant__ GlobalEntParams p) {
  extern __shared__ float sm[];
  constexpr int TQ = 32, TK = 32;
  const int R = p.R, RP = R + 1, DS = p.dslice;
  const int d0 = blockIdx.z * DS, DL = min(DS, p.D - d0);
  const int Rh = R / p.rope_heads;
  float *qs = sm;               // TQ x RP
  float *ks = qs + TQ * RP;     // TK x RP
  float *tt = ks + TK * RP;     // TQ x TK ternary
  float *cnt = tt + TQ * TK;    // TQ
  float *vs = cnt + TQ;         // TK x DS
  float *acc = vs + TK * DS;    // TQ x DS
  const int b = blockIdx.y, q0 = blockIdx.x * TQ;
  const int64_t row0 = (int64_t)b * p.L;
  const int nq = min(TQ, p.L - q0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarp = blockDim.x >> 5;
  for (int r = warp; r < nq; r += nwarp) {
    const int64_t row = row0 + q0 + r;
    for (int h = 0; h < p.rope_heads; ++h)
      load_rope_row(qs + r * RP + h * Rh, p.pc, p.pc.c_q + h * Rh, row, Rh, q0 + r, p.rt.v,
                    p.cross ? p.cross + row * R + h * Rh : nullptr, lane, 32);
  }
  for (int i = threadIdx.x; i < TQ * DS; i += blockDim.x) acc[i] = 0.f;
  if (threadIdx.x < TQ) cnt[threadIdx.x] = 0.f;
  for (int k0 = 0; k0 < q0 + nq; k0 += TK) {
    const int nk = min(TK, p.L - k0);
    __syncthreads();
    for (int r = warp; r < nk; r += nwarp)
      for (int h = 0; h < p.rope_heads; ++h)
        load_rope_row(ks + r * RP + h * Rh, p.pc, p.pc.c_k + h * Rh, row0 + k0 + r, Rh, k0 + r, p.rt.v,
                      nullptr, lane, 32);
    for (int i = threadIdx.x; i < nk * DL; i += blockDim.x) {
      const int r = i / DL, d = i - r * DL;
      vs[r * DS + d] = p.states[(row0 + k0 + r) * p.s_ld + p.s_off + d0 + d];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < TQ * TK; i += blockDim.x) {
      const int qi = i / TK, kj = i - qi * TK;
      float tv = 0.f;
      const int gi = q0 + qi, gj = k0 + kj;
      if (qi < nq && kj < nk && gj <= gi) {
        float dot = 0.f;
        for (int c = 0; c < R; ++c) dot = fmaf(qs[qi * RP + c], ks[kj * RP + c], dot);
        const float sc = __fdiv_rn(dot, p.sqrt_r) + p.relb[gi - gj + p.L - 1];
        tv = ternary_of(sc, p.thr);
      }
      tt[i] = tv;
    }
    __syncthreads();
    if (threadIdx.x < TQ) {
      float c = 0.f;
      for (int kj = 0; kj < TK; ++kj) c += fabsf(tt[threadIdx.x * TK + kj]);
      cnt[threadIdx.x] += c;
    }
    for (int i = threadIdx.x; i < TQ * DL; i += blockDim.x) {
      const int qi = i / DL, d = i - qi * DL;
      float a = acc[qi * DS + d];
      for (int kj = 0; kj < nk; ++kj) a = fmaf(tt[qi * TK + kj], vs[kj * DS + d], a);
      acc[qi * DS + d] = a;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nq * DL; i += blockDim.x) {
    const int qi = i / DL, d = i - qi * DL, c = d0 + d;
    const int64_t row = row0 + q0 + qi;
    const float s = p.states[row * p.s_ld + p.s_off + c];
    const float avg = acc[qi * DS + d] / fmaxf(cnt[qi], 1.f);
    if (!p.mimo) {
      const float ent = s + p.es * (avg - s);
      store_f(p.out_tanh, p.out_dtype, row * p.D + c, tanhf(ent));
      store_f(p.out_chg, p.out_dtype, row * p.D + c, ent - s);
    } else {
      const int h = c / p.Dh, dd = c - h * p.Dh;
      const float m = p.mo[((int64_t)h * p.RM + p.r) * p.Dh + dd];
      const int64_t o = row * p.D + c;
      const float e = (p.r ? p.acc_e[o] : 0.f) + m * avg;
      const float cg = (p.r ? p.acc_c[o] : 0.f) + m * (avg - s);
      if (p.r + 1 < p.RM) {
        p.acc_e[o] = e;
        p.acc_c[o] = cg;
      } else {
        store_f(p.out_tanh, p.out_dtype, o, tanhf(e));
        store_f(p.out_chg, p.out_dtype, o, cg);
      }
    }
  }
}

static int launch_global(GlobalEntParams &p, cudaStream_t st) {
  p.dslice = p.D <= 256 ? p.D : 256;
  const size_t smem = sizeof(float) * (32 * (p.R + 1) * 2 + 32 * 32 + 32 + 32 * (size_t)p.dslice * 2);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_siso_global_ent, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    attr = true;
  }
  if (smem > 200 * 1024) return fail(TESM_EUNSUPPORTED, "global_ent: ent_rank too large");
  dim3 grid((unsigned)ceil_div(p.L, 32), (unsigned)p.B, (unsigned)ceil_div(p.D, p.dslice));
  TESM_REQUIRE(p.R / p.rope_heads <= 256, "global_ent: ent_rank per head above 256");
  p.rt = rope_table(p.R / p.rope_heads, p.rope_base);
  k_siso_global_ent<<<grid, 256, smem, st>>>(p);
  return check_launch("global_ent");
}

// ---------------------------------------------------------------- combine
// y = local + sigmoid(gate) * sp + ep   (tesm.py:1256-1260)
// Thread = 8 consecutive columns of one row (grid.y strides over rows).
__global__ void k_combine(ProjCols pc, const void *sp, const void *ep, int sdtype, int64_t M, int Dm, void *y,
                          int ydtype, int vec) {
  pdl_trigger();
  pdl_wait();
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c0 >= Dm) return;
  const int psz = pc.dtype == TESM_BF16 ? 2 : 4, ssz = sdtype == TESM_BF16 ? 2 : 4, ysz = ydtype == TESM_BF16 ? 2 : 4;
  for (int64_t m = blockIdx.y; m < M; m += gridDim.y) {
    const uint8_t *prow = reinterpret_cast<const uint8_t *>(pc.proj) + m * pc.ld * psz;
    float loc[8], gt[8], a[8], b[8], v[8];
    load8(prow, pc.dtype, pc.c_local + c0, pc.c_local + Dm, vec != 0, loc);
    load8(prow, pc.dtype, pc.c_gate + c0, pc.c_gate + Dm, vec != 0, gt);
    load8(reinterpret_cast<const uint8_t *>(sp) + m * Dm * ssz, sdtype, c0, Dm, vec != 0, a);
    load8(reinterpret_cast<const uint8_t *>(ep) + m * Dm * ssz, sdtype, c0, Dm, vec != 0, b);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = loc[e] + sigmoidf_(gt[e]) * a[e] + b[e];
    store8(reinterpret_cast<uint8_t *>(y) + m * Dm * ysz, ydtype, c0, Dm, vec != 0, v);
  }
}

}  // namespace tesm

using namespace tesm;

// Local entanglement (tesm.py:922-952 with the lerp :1231-1232): the persistent window kernel
// of window.cuh, SISO mode (one head of d_state channels, cross-layer q bias).
static int siso_win_params(WinEntParams &p, const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L,
                           int64_t Dm, int64_t D, int64_t R, const float *cross, const float *bias,
                           const float *states, float thr, float es, float rope_base) {
  if (dtype != TESM_F32 && dtype != TESM_BF16) return fail(TESM_EDTYPE, "local_ent: dtype");
  const ProjCols pc = make_cols(proj, dtype, ldp, (int)Dm, (int)D, (int)R);
  p = WinEntParams{};
  p.proj = proj;
  p.ld = ldp;
  p.c_q = pc.c_q;
  p.c_k = pc.c_k;
  p.states = states;
  p.pos_ld = D;
  p.rank_ld = 0;
  p.cross = cross;
  p.bias = bias;
  p.B = (int)B;
  p.L = (int)L;
  p.H = 1;
  p.D = (int)D;
  p.R = (int)R;
  p.thr = thr;
  p.es = es;
  p.sqrt_r = (float)sqrt((double)R);
  p.rope_base = rope_base;
  return TESM_OK;
}

template <int MODE>
static int siso_win_dispatch(WinEntParams &p, int dtype, int64_t W, cudaStream_t st, const char *what) {
#define TESM_SISO_WIN(WW)                                                                       \
  if (W == WW)                                                                                  \
    return dtype == TESM_BF16 ? win_launch<WW, 1, 2, MODE>(p, st, what) : win_launch<WW, 1, 4, MODE>(p, st, what);
  TESM_SISO_WIN(4) TESM_SISO_WIN(8) TESM_SISO_WIN(16) TESM_SISO_WIN(32)
#undef TESM_SISO_WIN
  return fail(TESM_EUNSUPPORTED, std::string(what) + ": entanglement_window must be 4, 8, 16 or 32");
}

extern "C" int tesm_b200_siso_local_ent(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L, int64_t Dm,
                                        int64_t D, int64_t R, int64_t W, const float *cross, const float *bias,
                                        const float *states, float thr, float es, float rope_base, void *out_tanh,
                                        void *out_chg, int out_dtype, tesm_stream_t stream) {
  TESM_REQUIRE(proj && bias && states && out_tanh && out_chg, "local_ent: null pointer");
  TESM_REQUIRE(B > 0 && L > 0 && D > 0 && R > 0 && R % 2 == 0, "local_ent: bad shape");
  if (out_dtype != TESM_F32 && out_dtype != TESM_BF16) return fail(TESM_EDTYPE, "local_ent: out dtype");
  WinEntParams p;
  int rc = siso_win_params(p, proj, dtype, ldp, B, L, Dm, D, R, cross, bias, states, thr, es, rope_base);
  if (rc) return rc;
  p.out_tanh = out_tanh;
  p.out_chg = out_chg;
  p.out_dtype = out_dtype;
  p.out_ld = D;
  return siso_win_dispatch<kWinSiso>(p, dtype, W, (cudaStream_t)stream, "local_ent");
}

extern "C" int tesm_b200_siso_local_ent_codes(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L,
                                              int64_t Dm, int64_t D, int64_t R, int64_t W, const float *cross,
                                              const float *bias, const float *states, float thr, float es,
                                              float rope_base, int act_dtype, float eps1, float eps2, int8_t *codes,
                                              int64_t ldc, int64_t Dp, float *inv1, float *inv2,
                                              tesm_stream_t stream) {
  TESM_REQUIRE(proj && bias && states && codes && inv1 && inv2, "local_ent_codes: null pointer");
  TESM_REQUIRE(B > 0 && L > 0 && D > 0 && R > 0 && R % 2 == 0, "local_ent_codes: bad shape");
  TESM_REQUIRE(Dp >= D && Dp % 128 == 0 && ldc >= 2 * Dp && ldc % 16 == 0 && ((uintptr_t)codes & 15) == 0,
               "local_ent_codes: codes layout (Dp multiple of 128 >= D, ldc >= 2*Dp, 16-byte rows)");
  WinEntParams p;
  int rc = siso_win_params(p, proj, dtype, ldp, B, L, Dm, D, R, cross, bias, states, thr, es, rope_base);
  if (rc) return rc;
  p.act_dtype = act_dtype;
  p.eps1 = eps1;
  p.eps2 = eps2;
  p.codes = codes;
  p.ldc = ldc;
  p.Dp = (int)Dp;
  p.inv1 = inv1;
  p.inv2 = inv2;
  return siso_win_dispatch<kWinSisoCodes>(p, dtype, W, (cudaStream_t)stream, "local_ent_codes");
}

extern "C" int tesm_b200_global_relbias(const float *embed, int64_t dim, float scale, float bias0, int64_t L,
                                        float *out, tesm_stream_t stream) {
  TESM_REQUIRE(embed && out && dim > 0 && L > 0, "global_relbias: bad argument");
  const int64_t n = 2 * L - 1;
  k_global_relbias<<<(unsigned)ceil_div(n, 256), 256, 0, (cudaStream_t)stream>>>(embed, (int)dim, scale, bias0,
                                                                                   (int)L, out);
  return check_launch("global_relbias");
}

extern "C" int tesm_b200_siso_global_ent(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L,
                                         int64_t Dm, int64_t D, int64_t R, const float *cross, const float *relb,
                                         const float *states, float thr, float es, float rope_base, void *out_tanh,
                                         void *out_chg, int out_dtype, tesm_stream_t stream) {
  TESM_REQUIRE(proj && relb && states && out_tanh && out_chg, "global_ent: null pointer");
  TESM_REQUIRE(B > 0 && L > 0 && D > 0 && R > 0 && R % 2 == 0, "global_ent: bad shape");
  GlobalEntParams p;
  p.pc = make_cols(proj, dtype, ldp, (int)Dm, (int)D, (int)R);
  p.cross = cross;
  p.relb = relb;
  p.states = states;
  p.B = (int)B;
  p.L = (int)L;
  p.D = (int)D;
  p.R = (int)R;
  p.thr = thr;
  p.es = es;
  p.sqrt_r = (float)sqrt((double)R);
  p.rope_base = rope_base;
  p.out_tanh = out_tanh;
  p.out_chg = out_chg;
  p.out_dtype = out_dtype;
  p.states = states;
  p.s_ld = D;
  p.s_off = 0;
  p.rope_heads = 1;
  p.mimo = 0;
  return launch_global(p, (cudaStream_t)stream);
}

extern "C" int tesm_b200_mimo_global_ent(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L, int64_t Dm,
                                         int64_t H, int64_t D, int64_t R, int64_t RM, const float *relb,
                                         const float *mimo_o, const float *states, float thr, float rope_base,
                                         float *acc_e, float *acc_c, void *out_tanh, void *out_chg, int out_dtype,
                                         tesm_stream_t stream) {
  TESM_REQUIRE(proj && relb && mimo_o && states && out_tanh && out_chg, "mimo_global_ent: null pointer");
  TESM_REQUIRE(B > 0 && L > 0 && H > 0 && D > 0 && R > 0 && R % 2 == 0 && RM > 0, "mimo_global_ent: bad shape");
  TESM_REQUIRE(RM == 1 || (acc_e && acc_c), "mimo_global_ent: accumulators needed for mimo_rank > 1");
  if (dtype != TESM_F32 && dtype != TESM_BF16) return fail(TESM_EDTYPE, "mimo_global_ent: dtype");
  GlobalEntParams p;
  p.pc = make_cols(proj, dtype, ldp, (int)Dm, (int)(H * D), (int)(H * R));
  p.cross = nullptr;
  p.relb = relb;
  p.states = states;
  p.s_ld = RM * H * D;
  p.B = (int)B;
  p.L = (int)L;
  p.D = (int)(H * D);
  p.R = (int)(H * R);
  p.rope_heads = (int)H;
  p.thr = thr;
  p.es = 0.f;
  p.sqrt_r = (float)sqrt((double)(H * R));
  p.rope_base = rope_base;
  p.out_tanh = out_tanh;
  p.out_chg = out_chg;
  p.out_dtype = out_dtype;
  p.mimo = 1;
  p.RM = (int)RM;
  p.Dh = (int)D;
  p.mo = mimo_o;
  p.acc_e = acc_e;
  p.acc_c = acc_c;
  for (int r = 0; r < RM; ++r) {
    p.r = r;
    p.s_off = (int)(r * H * D);
    int rc = launch_global(p, (cudaStream_t)stream);
    if (rc) return rc;
  }
  return TESM_OK;
}

extern "C" int tesm_b200_combine(const void *proj, int dtype, int64_t ldp, int64_t M, int64_t Dm, int64_t D,
                                 int64_t R, const void *sp, const void *ep, int sdtype, void *y, int ydtype,
                                 tesm_stream_t stream) {
  if (M == 0) return TESM_OK;  // empty batch: nothing to do (its buffers may be null)
  TESM_REQUIRE(proj && sp && ep && y && M >= 0 && Dm > 0, "combine: bad argument");
  ProjCols pc = make_cols(proj, dtype, ldp, (int)Dm, (int)D, (int)R);
  const int64_t n = M * Dm;
  const int psz = dtype == TESM_BF16 ? 2 : 4, ssz = sdtype == TESM_BF16 ? 2 : 4, ysz = ydtype == TESM_BF16 ? 2 : 4;
  const int vec = (Dm % 8 == 0) && ((uintptr_t)proj % 16 == 0) && ((ldp * psz) % 16 == 0) &&
                  ((pc.c_local * psz) % 16 == 0) && ((pc.c_gate * psz) % 16 == 0) && ((uintptr_t)sp % 16 == 0) &&
                  ((uintptr_t)ep % 16 == 0) && ((uintptr_t)y % 16 == 0) && ((Dm * ssz) % 16 == 0) &&
                  ((Dm * ysz) % 16 == 0);
  (void)n;
  const int64_t groups = ceil_div(Dm, 8);
  const int threads = groups >= 128 ? 128 : (int)round_up(groups, 32);
  dim3 grid((unsigned)ceil_div(groups, threads), (unsigned)(M < 65535 ? M : 65535));
  return launch_k("combine", k_combine, grid, dim3(threads), 0, (cudaStream_t)stream, pc, sp, ep, sdtype, M, (int)Dm, y,
                  ydtype, vec);
}
