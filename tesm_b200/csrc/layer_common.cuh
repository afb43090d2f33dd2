// Helpers shared by the layer kernels (scan, entanglement, decode).
#pragma once

#include <cmath>

#include "common.cuh"

namespace tesm {

// Column view of the in_proj output.  SISO split (tesm.py:1195-1205):
//   [local Dm | value D | decay D | write D | gate Dm | q R | k R]
// MIMO split (tesm_mimo.py:940-956) is the same with D -> H*D and R -> H*R, head-major.
struct ProjCols {
  const void *proj;
  int dtype;
  int64_t ld;  // row stride (elements)
  int c_local, c_value, c_decay, c_write, c_gate, c_q, c_k;
};

// Dc = state columns (D or H*D), Rc = q/k columns (R or H*R)
inline ProjCols make_cols(const void *proj, int dtype, int64_t ld, int Dm, int Dc, int Rc) {
  ProjCols pc;
  pc.proj = proj;
  pc.dtype = dtype;
  pc.ld = ld;
  pc.c_local = 0;
  pc.c_value = Dm;
  pc.c_decay = Dm + Dc;
  pc.c_write = Dm + 2 * Dc;
  pc.c_gate = Dm + 3 * Dc;
  pc.c_q = 2 * Dm + 3 * Dc;
  pc.c_k = 2 * Dm + 3 * Dc + Rc;
  return pc;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + expf(-x)); }

__device__ __forceinline__ float ternary_of(float s, float thr) { return s > thr ? 1.f : (s < -thr ? -1.f : 0.f); }

// theta = pos * (1 / base^(2i/R)) in fp32 (tesm.py:783-793; tesm_mimo.py:210-220).  The table
// is built on the host: the power evaluated in double and rounded to fp32 once (the correctly
// rounded fp32 power), then the fp32 reciprocal.  For every even R <= 64 this reproduces the
// reference's torch values bit for bit, which matters because theta = pos * inv_freq magnifies a
// one-ulp difference in inv_freq by the position (a few 1e-4 rad at pos ~ 8000).  Kernels take
// it as a __grid_constant__ parameter (R <= 256).
struct RopeTab {
  float v[128];
};
inline RopeTab rope_table(int R, float base) {
  RopeTab t;
  for (int i = 0; i < 128; ++i) {
    const float ex = (2.f * (float)i) / (float)(R > 0 ? R : 1);
    const float pw = (float)std::pow((double)base, (double)ex);
    t.v[i] = 1.f / pw;
  }
  return t;
}

// One q/k row of R values starting at column `col` -> dst with RoPE at `pos`, plus an
// optional additive row (the cross-layer q bias, applied after RoPE as in tesm.py:1213-1218).
// invf: the RopeTab of R (parameter or shared memory).
__device__ __forceinline__ void load_rope_row(float *dst, const ProjCols &pc, int col, int64_t row, int R, int pos,
                                              const float *invf, const float *add, int tid, int nthr) {
  const int half = R / 2;
  for (int i = tid; i < half; i += nthr) {
    const float x1 = load_f(pc.proj, pc.dtype, row * pc.ld + col + i);
    const float x2 = load_f(pc.proj, pc.dtype, row * pc.ld + col + half + i);
    const float th = (float)pos * invf[i];
    float sn, cs;
    sincosf(th, &sn, &cs);
    float o1 = x1 * cs - x2 * sn, o2 = x1 * sn + x2 * cs;
    if (add) {
      o1 += add[i];
      o2 += add[half + i];
    }
    dst[i] = o1;
    dst[half + i] = o2;
  }
}

__device__ __forceinline__ int ld_acquire(const int *p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(int *p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

}  // namespace tesm
