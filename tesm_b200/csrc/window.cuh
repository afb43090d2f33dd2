// Local-window ternary entanglement: one persistent kernel for the SISO layer (bf16/fp32
// outputs, or int8 codes for the combine GEMM) and the MIMO layer (rank merge).
// Reference: tesm.py:922-952 (torch rung) with ternary_entanglement :672-714 and the lerp
// :1231-1232; MIMO tesm_mimo.py:525-588 (per-rank window sums) and :996-1017 (merge).
//
// Work unit = (sequence b, tile of T = 32 positions, head h); a CTA owns a strided list of
// tiles and walks each tile's heads in turn (SISO: one head).  Per unit:
//   fill     every byte the unit reads -- its q rows, the k rows and state rows of the window
//            (positions t0-(W-1) ..), all mimo ranks -- is requested with 16-byte cp.async
//            copies into shared memory.  Two 256-thread CTAs per SM with one stage each when
//            that fits (one CTA's copies and barriers hide behind the other's arithmetic),
//            else one 512-thread CTA with two stages whose next unit's copies are issued
//            before the current unit is computed.  Positions outside the sequence / tile are
//            zero-filled by the copy itself.
//   table    (cos, sin) of every (position, frequency) of the tile, once per tile (shared by
//            q, k and all heads), theta = fl(pos * inv_freq) as in tesm.py:783-793.
//   rope     q rows (+ cross-layer bias, tesm.py:1213-1218) and k rows, fp32 in shared memory.
//   scores   q_t . k_{t-o} / sqrt(R) + bias[W-1-o] for the W lags o, thresholded to {-1,0,1};
//            a lane owns one lag of one row and the row's |tern| count is a shuffle sum.
//   window   avg[t][n] = sum_o tern[t][o] s[t-o][n] is a banded matrix product: for a block of
//            16 positions, A[16 x K] holds the ternary weights on a diagonal band (exact in
//            TF32) and B[K x 8] the states of K = 16 + W - 1 (rounded to 8) consecutive
//            positions of 8 channels.  It runs on the tensor cores (mma.sync m16n8k8 TF32) with
//            the fp32 states split as hi + lo (two MMAs, error ~2^-21 relative), then is scaled
//            by 1 / max(sum |tern|, 1).
//   epilogue ent = s + es (avg - s); SISO writes tanh(ent) and ent - s (or stages them for the
//            per-token int8 codes), MIMO merges the ranks with mimo_o first.
#pragma once

#include "layer_common.cuh"
#include "rowio.cuh"

#include <algorithm>

namespace tesm {

enum WinMode { kWinSiso = 0, kWinSisoCodes = 1, kWinMimo = 2 };

constexpr int kWinT = 32;         // positions per tile

struct WinEntParams {
  const void *proj;
  int64_t ld;          // proj row stride (elements)
  int64_t c_q, c_k;    // first q / k column; head h at + h * R
  const float *states; // states[(row0 + pos) * pos_ld + k * rank_ld + h * D + ch]
  int64_t pos_ld, rank_ld;
  const float *cross;  // SISO cross-layer q bias (B*L, R) or null
  const float *bias;   // window bias of head h at bias + h * W, read at [W-1-o]
  const float *mimo_o; // MIMO (H, RM, D)
  int B, L, H, D, R, quirk, async16, ntiles_b;
  int stage_out;  // bf16 outputs with 16-byte aligned 8-channel groups: staged 16-byte row stores
  float thr, es, sqrt_r, rope_base;
  RopeTab rt;
  void *out_tanh, *out_chg;  // out[(row0 + t) * out_ld + h * D + ch]
  int out_dtype;
  int64_t out_ld;
  // kWinSisoCodes
  int act_dtype, Dp;
  float eps1, eps2;
  int8_t *codes;
  int64_t ldc;
  float *inv1, *inv2;
};

// Tile geometry shared by host (shared-memory size) and device (carving).
struct WinGeom {
  int W, R, D, RM, ES, mode, nst;  // nst: staging buffers (2: the next unit streams in meanwhile)
  int half, RP, nk, KS, NROWS, SR, SRR, QRS;
};

__host__ __device__ inline int64_t win_r16(int64_t b) { return (b + 15) & ~(int64_t)15; }

__host__ __device__ inline WinGeom win_geom(int W, int R, int D, int RM, int ES, int mode, int nst) {
  WinGeom g;
  g.nst = nst;
  g.W = W;
  g.R = R;
  g.D = D;
  g.RM = RM;
  g.ES = ES;
  g.mode = mode;
  g.half = R / 2;
  g.RP = ((R + 3) / 4) * 4 + 4;
  g.nk = kWinT + W - 1;
  g.KS = (15 + W + 7) / 8;          // k-steps of 8 covering the 16 + W - 1 window rows of a block
  g.NROWS = kWinT - 16 + g.KS * 8;  // state rows staged (>= nk)
  g.SR = ((D + 3) / 4) * 4;         // rank stride in a state row
  int srr = RM * g.SR;
  while (srr % 32 != 8) srr += 4;   // row stride: the 4 rows x 8 channels of a B fragment hit 32 banks
  g.SRR = srr;
  g.QRS = (int)win_r16((int64_t)R * ES);
  return g;
}

struct WinStage {
  float *st;      // NROWS x SRR
  uint8_t *qraw;  // T x QRS
  uint8_t *kraw;  // nk x QRS
};

struct WinSmem {
  WinStage stage[2];
  float2 *cs;      // nk x half
  float *invf;     // half
  float *qs;       // T x RP
  float *ks;       // nk x RP
  float *twr;      // T x W ternary
  float *inv;      // T     1 / max(sum |tern|, 1)
  float *oT, *oC;  // kWinSisoCodes: T x (D + 1) staged outputs
  int *amT, *amC;  // kWinSisoCodes: per-row max |value| (non-negative float bits)
  uint32_t *stg;   // other modes: per warp 16 rows x 20 words (32 bf16 + 16 bytes of padding)
};

// warps of the CTA: one staging buffer (nst = 1) runs 256 threads, two run 512
__host__ __device__ inline int win_warps(const WinGeom &g) { return g.nst == 1 ? 8 : 16; }

__host__ __device__ inline size_t win_smem_bytes(const WinGeom &g) {
  const size_t stage = win_r16((int64_t)g.NROWS * g.SRR * 4) + win_r16((int64_t)kWinT * g.QRS) +
                       win_r16((int64_t)g.nk * g.QRS);
  size_t b = g.nst * stage + win_r16((int64_t)g.nk * g.half * 8) + win_r16((int64_t)g.half * 4) +
             win_r16((int64_t)kWinT * g.RP * 4) + win_r16((int64_t)g.nk * g.RP * 4) +
             win_r16((int64_t)kWinT * g.W * 4) + win_r16((int64_t)kWinT * 4);
  if (g.mode == kWinSisoCodes)
    b += 2 * win_r16((int64_t)kWinT * (g.D + 1) * 4) + 2 * win_r16((int64_t)kWinT * 4);
  else
    b += win_r16((int64_t)win_warps(g) * 16 * 20 * 4);
  return b;
}

__device__ __forceinline__ WinSmem win_carve(uint8_t *p, const WinGeom &g) {
  WinSmem s;
  auto take = [&p](int64_t bytes) {
    uint8_t *r = p;
    p += win_r16(bytes);
    return r;
  };
  for (int i = 0; i < g.nst; ++i) {
    s.stage[i].st = reinterpret_cast<float *>(take((int64_t)g.NROWS * g.SRR * 4));
    s.stage[i].qraw = take((int64_t)kWinT * g.QRS);
    s.stage[i].kraw = take((int64_t)g.nk * g.QRS);
  }
  if (g.nst == 1) s.stage[1] = s.stage[0];
  s.cs = reinterpret_cast<float2 *>(take((int64_t)g.nk * g.half * 8));
  s.invf = reinterpret_cast<float *>(take((int64_t)g.half * 4));
  s.qs = reinterpret_cast<float *>(take((int64_t)kWinT * g.RP * 4));
  s.ks = reinterpret_cast<float *>(take((int64_t)g.nk * g.RP * 4));
  s.twr = reinterpret_cast<float *>(take((int64_t)kWinT * g.W * 4));
  s.inv = reinterpret_cast<float *>(take((int64_t)kWinT * 4));
  s.oT = s.oC = nullptr;
  s.amT = s.amC = nullptr;
  s.stg = nullptr;
  if (g.mode == kWinSisoCodes) {
    s.oT = reinterpret_cast<float *>(take((int64_t)kWinT * (g.D + 1) * 4));
    s.oC = reinterpret_cast<float *>(take((int64_t)kWinT * (g.D + 1) * 4));
    s.amT = reinterpret_cast<int *>(take((int64_t)kWinT * 4));
    s.amC = reinterpret_cast<int *>(take((int64_t)kWinT * 4));
  } else {
    s.stg = reinterpret_cast<uint32_t *>(take((int64_t)win_warps(g) * 16 * 20 * 4));
  }
  return s;
}

// Whether every q/k row and state chunk starts on a 16-byte boundary (then units are staged
// with asynchronous 16-byte copies; otherwise with plain element copies).
inline bool win_async_ok(const WinEntParams &p, int ES, int nthr) {
  return ((uintptr_t)p.proj & 15) == 0 && (p.ld * ES) % 16 == 0 && (p.c_q * ES) % 16 == 0 &&
         (p.c_k * ES) % 16 == 0 && (p.R * ES) % 16 == 0 && ((uintptr_t)p.states & 15) == 0 && p.D % 4 == 0 &&
         p.pos_ld % 4 == 0 && p.rank_ld % 4 == 0 && p.R * ES / 16 <= nthr &&
         (int64_t)p.D / 4 * (p.rank_ld ? (p.pos_ld / p.rank_ld) : 1) <= nthr;
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src, int src_bytes) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }

__device__ __forceinline__ uint32_t f32_to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void mma_tf32(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Per-thread strided walk over a (rows x per_row) index space without per-element division:
// the thread handles (r0 + k * rstep, c0); threads beyond rstep * per_row stay idle.
struct WinMap {
  int r0, c0, rstep;
  bool active;
};
template <int NT>
__device__ __forceinline__ WinMap win_map(int per_row) {
  WinMap m;
  m.rstep = per_row > 0 ? NT / per_row : 0;
  m.r0 = per_row > 0 ? (int)threadIdx.x / per_row : 0;
  m.c0 = (int)threadIdx.x - m.r0 * per_row;
  m.active = per_row > 0 && per_row <= NT && m.r0 < m.rstep;
  return m;
}

// Stage the unit (tile at row0 + t0, nt positions, head h) into `sg`.  Asynchronous path: a
// thread owns one 16-byte column chunk of the q/k rows (mq) and one of the state rows (ms:
// rank k, chunk c) and walks rows with pointer increments.
template <int W, int RM, int ES, int NT>
__device__ __forceinline__ void win_fill(const WinEntParams &p, const WinGeom &g, const WinStage &sg,
                                         const WinMap &mq, const WinMap &ms, int64_t row0, int t0, int nt, int h) {
  const int nkv = nt + W - 1;
  const uint8_t *proj = reinterpret_cast<const uint8_t *>(p.proj);
  const int64_t qcol = p.c_q + (int64_t)h * p.R, kcol = p.c_k + (int64_t)h * p.R;
  const int64_t scol = (int64_t)h * p.D;
  if (p.async16) {
    if (mq.active) {
      const int64_t rstride = (int64_t)mq.rstep * p.ld * ES;
      const uint8_t *src = proj + ((row0 + t0 + mq.r0) * p.ld + qcol) * ES + mq.c0 * 16;
      uint8_t *dst = sg.qraw + (size_t)mq.r0 * g.QRS + mq.c0 * 16;
      for (int r = mq.r0; r < nt; r += mq.rstep, src += rstride, dst += mq.rstep * g.QRS) cp_async16(dst, src, 16);
      int pos = t0 - (W - 1) + mq.r0;
      src = proj + ((row0 + pos) * p.ld + kcol) * ES + mq.c0 * 16;
      dst = sg.kraw + (size_t)mq.r0 * g.QRS + mq.c0 * 16;
      for (int r = mq.r0; r < nkv; r += mq.rstep, pos += mq.rstep, src += rstride, dst += mq.rstep * g.QRS)
        cp_async16(dst, pos < 0 ? proj : src, pos < 0 ? 0 : 16);
    }
    if (ms.active) {
      const int cpr = p.D / 4;  // chunks per rank block
      const int k = ms.c0 / cpr, c = ms.c0 - k * cpr;
      int pos = t0 - (W - 1) + ms.r0;
      const int lim = t0 + nt;
      const float *src = p.states + (row0 + pos) * p.pos_ld + k * p.rank_ld + scol + c * 4;
      float *dst = sg.st + (size_t)ms.r0 * g.SRR + k * g.SR + c * 4;
      const int64_t sstride = (int64_t)ms.rstep * p.pos_ld;
      for (int r = ms.r0; r < g.NROWS; r += ms.rstep, pos += ms.rstep, src += sstride, dst += ms.rstep * g.SRR) {
        const bool ok = pos >= 0 && pos < lim;
        cp_async16(dst, ok ? src : p.states, ok ? 16 : 0);
      }
    }
  } else {
    for (int idx = threadIdx.x; idx < (nt + nkv) * p.R; idx += NT) {
      const int r = idx / p.R, e = idx - r * p.R;
      const bool isq = r < nt;
      const int rr = isq ? r : r - nt;
      const int pos = isq ? t0 + rr : t0 - (W - 1) + rr;
      uint8_t *dst = (isq ? sg.qraw : sg.kraw) + (size_t)rr * g.QRS + e * ES;
      const int64_t off = (row0 + pos) * p.ld + (isq ? qcol : kcol) + e;
      if (ES == 2)
        *reinterpret_cast<uint16_t *>(dst) = pos < 0 ? 0 : reinterpret_cast<const uint16_t *>(proj)[off];
      else
        *reinterpret_cast<float *>(dst) = pos < 0 ? 0.f : reinterpret_cast<const float *>(proj)[off];
    }
    for (int idx = threadIdx.x; idx < g.NROWS * RM * p.D; idx += NT) {
      const int rk = idx / p.D, j = idx - rk * p.D;
      const int r = rk / RM, k = rk - r * RM;
      const int pos = t0 - (W - 1) + r;
      const bool ok = pos >= 0 && pos < t0 + nt;
      sg.st[(size_t)r * g.SRR + k * g.SR + j] = ok ? p.states[(row0 + pos) * p.pos_ld + k * p.rank_ld + scol + j] : 0.f;
    }
  }
}

// tanh from the hardware exponential: 1 - 2 / (1 + e^{2x}) (absolute error ~2e-7; saturates
// to +-1 through the infinities of e^{2x}).
__device__ __forceinline__ float win_tanh(float x) { return 1.f - __fdividef(2.f, 1.f + __expf(2.f * x)); }

template <int ES>
__device__ __forceinline__ float raw_at(const uint8_t *row, int i) {
  if (ES == 2) return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(row)[i]);
  return reinterpret_cast<const float *>(row)[i];
}

__device__ __forceinline__ void win_store2(void *out, int dtype, int64_t o, float x, float y, bool pair, bool has_y) {
  if (pair) {
    if (dtype == TESM_BF16)
      *reinterpret_cast<__nv_bfloat162 *>(reinterpret_cast<__nv_bfloat16 *>(out) + o) = __floats2bfloat162_rn(x, y);
    else
      *reinterpret_cast<float2 *>(reinterpret_cast<float *>(out) + o) = make_float2(x, y);
  } else {
    store_f(out, dtype, o, x);
    if (has_y) store_f(out, dtype, o + 1, y);
  }
}

// NT threads; NST = 2: one CTA per SM streams the next unit in while computing this one;
// NST = 1: two CTAs per SM, each loading its next unit after finishing the current one.
template <int W, int RM, int ES, int MODE, int NT, int NST>
__global__ void __launch_bounds__(NT, NST == 1 ? 2 : 1) k_win_ent(const __grid_constant__ WinEntParams p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const WinGeom g = win_geom(W, p.R, p.D, RM, ES, MODE, NST);
  const WinSmem s = win_carve(smem_raw, g);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tig = lane & 3;
  const int half = g.half, R = p.R, RP = g.RP, D = p.D, H = p.H;
  const int R4 = (R + 3) & ~3;
  const WinMap mq = win_map<NT>(R * ES / 16), ms = win_map<NT>(RM * (D / 4)), mh = win_map<NT>(half);

  for (int i = tid; i < half; i += NT) s.invf[i] = p.rt.v[i];
  if (R4 > R)  // pad columns read by the 4-wide dot products stay zero
    for (int i = tid; i < (kWinT + g.nk) * (R4 - R); i += NT) {
      const int row = i / (R4 - R), j = i - row * (R4 - R);
      (row < kWinT ? s.qs + row * RP : s.ks + (row - kWinT) * RP)[R + j] = 0.f;
    }

  const int ntiles = p.B * p.ntiles_b;
  int tile = blockIdx.x, h = 0;
  auto unit_of = [&](int tl, int64_t &row0, int &t0, int &nt) {
    const int b = tl / p.ntiles_b;
    t0 = (tl - b * p.ntiles_b) * kWinT;
    row0 = (int64_t)b * p.L;
    nt = min(kWinT, p.L - t0);
  };
  if (tile < ntiles) {
    int64_t row0;
    int t0, nt;
    unit_of(tile, row0, t0, nt);
    win_fill<W, RM, ES, NT>(p, g, s.stage[0], mq, ms, row0, t0, nt, 0);
  }
  cp_async_commit();
  __syncthreads();

  const float es = p.es;
  const int tb = (warp & 1) * 16;  // this warp's 16-position block for the window product
  int stage = 0;
  bool new_tile = true;
  while (tile < ntiles) {
    int64_t row0;
    int t0, nt;
    unit_of(tile, row0, t0, nt);
    const int nkv = nt + W - 1;
    // NST = 2: issue the next unit's copies into the other stage (released at the end of the
    // previous unit), then wait for this unit's
    if (NST == 2) {
      int nh = h + 1, ntl = tile;
      if (nh == H) {
        nh = 0;
        ntl += gridDim.x;
      }
      if (ntl < ntiles) {
        int64_t r1;
        int a1, n1;
        unit_of(ntl, r1, a1, n1);
        win_fill<W, RM, ES, NT>(p, g, stage ? s.stage[0] : s.stage[1], mq, ms, r1, a1, n1, nh);
      }
      cp_async_commit();
    }
    if (new_tile && mh.active) {
      for (int r = mh.r0; r < nkv; r += mh.rstep) {
        const int pos = t0 - (W - 1) + r;
        float sn = 0.f, cn = 1.f;
        if (pos >= 0) sincosf((float)pos * s.invf[mh.c0], &sn, &cn);
        s.cs[r * half + mh.c0] = make_float2(cn, sn);
      }
    }
    if (NST == 2)
      cp_async_wait_1();
    else
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    __syncthreads();
    const WinStage sg = stage ? s.stage[1] : s.stage[0];  // static indices keep s in registers
    // RoPE: q rows then k rows (rows before the sequence start hold zeros)
    if (mh.active) {
      for (int r = mh.r0; r < nt + nkv; r += mh.rstep) {
        const bool isq = r < nt;
        const int rr = isq ? r : r - nt;
        const uint8_t *raw = (isq ? sg.qraw : sg.kraw) + (size_t)rr * g.QRS;
        const float2 c = s.cs[(isq ? rr + W - 1 : rr) * half + mh.c0];
        const float x1 = raw_at<ES>(raw, mh.c0), x2 = raw_at<ES>(raw, half + mh.c0);
        float o1 = x1 * c.x - x2 * c.y, o2 = x1 * c.y + x2 * c.x;
        if (isq && MODE != kWinMimo && p.cross) {
          const float *add = p.cross + (row0 + t0 + rr) * R;
          o1 += add[mh.c0];
          o2 += add[half + mh.c0];
        }
        float *dst = isq ? s.qs + rr * RP : s.ks + rr * RP;
        dst[mh.c0] = o1;
        dst[half + mh.c0] = o2;
      }
    }
    __syncthreads();
    if (MODE == kWinSisoCodes && tid < 2 * kWinT) (tid < kWinT ? s.amT : s.amC)[tid & (kWinT - 1)] = 0;
    // scores: lane = (row t, lag group og) with lags og + j * OG, j < LPT, so one q load feeds
    // LPT independent dot products; the row's OG lanes are adjacent (shuffle-summed count)
    {
      constexpr int LPT = (kWinT * W) / NT >= 2 ? (kWinT * W) / NT : 1;  // lags per lane
      constexpr int OG = W / LPT;                                        // lanes per row
      const float *brow = p.bias + (MODE == kWinMimo ? h * W : 0);
      for (int item = tid; item < kWinT * OG; item += NT) {
        const int t = item / OG, og = item - t * OG;  // OG compile-time
        float tv[LPT];
#pragma unroll
        for (int j = 0; j < LPT; ++j) tv[j] = 0.f;
        if (t < nt) {
          const float *qr = s.qs + t * RP, *k0 = s.ks + (t + W - 1 - og) * RP;
          float d[LPT];
#pragma unroll
          for (int j = 0; j < LPT; ++j) d[j] = 0.f;
          for (int c = 0; c < R4; c += 4) {
            const float4 q4 = *reinterpret_cast<const float4 *>(qr + c);
#pragma unroll
            for (int j = 0; j < LPT; ++j) {
              const float4 k4 = *reinterpret_cast<const float4 *>(k0 - j * OG * RP + c);  // lag og + j*OG
              d[j] = fmaf(q4.x, k4.x, d[j]);
              d[j] = fmaf(q4.y, k4.y, d[j]);
              d[j] = fmaf(q4.z, k4.z, d[j]);
              d[j] = fmaf(q4.w, k4.w, d[j]);
            }
          }
          const int gt = t0 + t;
#pragma unroll
          for (int j = 0; j < LPT; ++j) {
            const int o = og + j * OG;
            if (gt - o >= 0 && (MODE != kWinMimo || !p.quirk || o >= W - 1 - gt))
              tv[j] = ternary_of(__fdiv_rn(d[j], p.sqrt_r) + brow[W - 1 - o], p.thr);
          }
        }
        float cnt = 0.f;
#pragma unroll
        for (int j = 0; j < LPT; ++j) {
          s.twr[t * W + og + j * OG] = tv[j];
          cnt += fabsf(tv[j]);
        }
#pragma unroll
        for (int m = OG / 2; m >= 1; m >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, m);
        if (og == 0) s.inv[t] = 1.f / fmaxf(cnt, 1.f);
      }
    }
    __syncthreads();
    // banded window product on the tensor cores + epilogue.  A warp pair owns a contiguous range
    // of 8-channel groups and walks it in batches of 4 groups; with staged bf16 outputs each
    // batch's 16 rows x 32 channels are transposed through the warp's shared block (tanh rows,
    // then change rows) and leave as 16-byte row segments.
    {
      constexpr int KS = (15 + W + 7) / 8;
      const int SRR = g.SRR, SR = g.SR;
      uint32_t a[KS][4];
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int row = gq + ((j & 1) ? 8 : 0), k = ks * 8 + tig + ((j & 2) ? 4 : 0);
          const int o = row + W - 1 - k;
          const float v = (o >= 0 && o < W) ? s.twr[(tb + row) * W + o] : 0.f;
          a[ks][j] = __float_as_uint(v);
        }
      }
      const int ngroups = (D + 7) / 8;
      const float *st = sg.st;
      constexpr int NWP = NT / 64;
      const int gpw = (ngroups + NWP - 1) / NWP;
      const int g_lo = min(ngroups, (warp >> 1) * gpw), g_hi = min(ngroups, g_lo + gpw);
      const bool staged = MODE != kWinSisoCodes && p.stage_out;
      uint32_t *stg = MODE != kWinSisoCodes ? s.stg + warp * 320 : nullptr;
      float rmT[2] = {0.f, 0.f}, rmC[2] = {0.f, 0.f};  // codes: max |value| of rows gq, gq + 8
      for (int cb = g_lo; cb < g_hi; cb += 4) {
        float2 keepC[4][2];  // staged: the batch's change values, transposed after the tanh rows
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          keepC[j][0] = keepC[j][1] = make_float2(0.f, 0.f);
          const int cg = cb + j;
          if (cg >= g_hi) continue;
          float acc[RM][4];
#pragma unroll
          for (int k = 0; k < RM; ++k) acc[k][0] = acc[k][1] = acc[k][2] = acc[k][3] = 0.f;
          const float *bcol = st + (size_t)(tb + tig) * SRR + cg * 8 + gq;
#pragma unroll
          for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
            for (int k = 0; k < RM; ++k) {
              const float x0 = bcol[(size_t)(ks * 8) * SRR + k * SR], x1 = bcol[(size_t)(ks * 8 + 4) * SRR + k * SR];
              const uint32_t h0 = f32_to_tf32(x0), h1 = f32_to_tf32(x1);
              mma_tf32(acc[k], a[ks], h0, h1);
              mma_tf32(acc[k], a[ks], __float_as_uint(x0 - __uint_as_float(h0)),
                       __float_as_uint(x1 - __uint_as_float(h1)));
            }
          }
          // epilogue: the lane holds rows tb+gq, tb+gq+8 x channels ch, ch+1 of every rank
          const int ch = cg * 8 + 2 * tig;
          const bool has_x = ch < D, has_y = ch + 1 < D;
          float2 mo[RM];
          if (MODE == kWinMimo) {
#pragma unroll
            for (int k = 0; k < RM; ++k) {
              const float *m = p.mimo_o + ((int64_t)h * RM + k) * D + ch;
              mo[k] = make_float2(has_x ? m[0] : 0.f, has_y ? m[1] : 0.f);
            }
          }
#pragma unroll
          for (int hr = 0; hr < 2; ++hr) {
            const int t = tb + gq + 8 * hr;
            if (t >= nt || !has_x) continue;
            const float iv = s.inv[t];
            const float *srow = st + (size_t)(t + W - 1) * SRR + ch;
            // the two channels ch, ch+1 in packed fp32 (FFMA2): e = s + es (acc / norm - s)
            const float2 iv2 = make_float2(iv, iv), es2 = make_float2(es, es);
            float2 E = make_float2(0.f, 0.f), Cg = make_float2(0.f, 0.f);
#pragma unroll
            for (int k = 0; k < RM; ++k) {
              float2 sv;
              if (has_y) {
                sv = *reinterpret_cast<const float2 *>(srow + k * SR);  // ch even, SR % 4 == 0
              } else {
                sv = make_float2(srow[k * SR], 0.f);
              }
              const float2 nsv = make_float2(-sv.x, -sv.y);
              const float2 dlt = __ffma2_rn(make_float2(acc[k][2 * hr], acc[k][2 * hr + 1]), iv2, nsv);
              const float2 e = __ffma2_rn(es2, dlt, sv);
              const float2 chg = __fadd2_rn(e, nsv);
              if (MODE == kWinMimo) {
                E = __ffma2_rn(mo[k], e, E);
                Cg = __ffma2_rn(mo[k], chg, Cg);
              } else {
                E = e;
                Cg = chg;
              }
            }
            const float ex = E.x, ey = E.y, cx = Cg.x, cy = Cg.y;
            if (MODE == kWinSisoCodes) {
              float *rt = s.oT + t * (D + 1) + ch, *rc = s.oC + t * (D + 1) + ch;
              const float vt = round_to(p.act_dtype, win_tanh(ex)), vc = round_to(p.act_dtype, cx);
              rt[0] = vt;
              rc[0] = vc;
              rmT[hr] = fmaxf(rmT[hr], fabsf(vt));
              rmC[hr] = fmaxf(rmC[hr], fabsf(vc));
              if (has_y) {
                const float wt = round_to(p.act_dtype, win_tanh(ey)), wc = round_to(p.act_dtype, cy);
                rt[1] = wt;
                rc[1] = wc;
                rmT[hr] = fmaxf(rmT[hr], fabsf(wt));
                rmC[hr] = fmaxf(rmC[hr], fabsf(wc));
              }
            } else if (staged) {
              const __nv_bfloat162 tv = __floats2bfloat162_rn(win_tanh(ex), win_tanh(ey));
              stg[(gq + 8 * hr) * 20 + j * 4 + tig] = *reinterpret_cast<const uint32_t *>(&tv);
              keepC[j][hr] = make_float2(cx, cy);
            } else {
              const int64_t o = (row0 + t0 + t) * p.out_ld + (int64_t)h * D + ch;
              const bool pair = has_y && (o & 1) == 0;
              win_store2(p.out_tanh, p.out_dtype, o, win_tanh(ex), has_y ? win_tanh(ey) : 0.f, pair, has_y);
              win_store2(p.out_chg, p.out_dtype, o, cx, cy, pair, has_y);
            }
          }
        }
        if (MODE != kWinSisoCodes && staged) {
#pragma unroll
          for (int arr = 0; arr < 2; ++arr) {
            if (arr == 1) {
              __syncwarp();  // the tanh rows have been read
#pragma unroll
              for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int hr = 0; hr < 2; ++hr) {
                  const __nv_bfloat162 cv = __floats2bfloat162_rn(keepC[j][hr].x, keepC[j][hr].y);
                  stg[(gq + 8 * hr) * 20 + j * 4 + tig] = *reinterpret_cast<const uint32_t *>(&cv);
                }
            }
            __syncwarp();
#pragma unroll
            for (int ps = 0; ps < 2; ++ps) {
              const int row = ps * 8 + (lane >> 2), chunk = lane & 3, t = tb + row;
              if (t < nt && cb + chunk < g_hi) {
                const uint4 v = *reinterpret_cast<const uint4 *>(stg + row * 20 + chunk * 4);
                const int64_t o = (row0 + t0 + t) * p.out_ld + (int64_t)h * D + (cb + chunk) * 8;
                *reinterpret_cast<uint4 *>(reinterpret_cast<__nv_bfloat16 *>(arr ? p.out_chg : p.out_tanh) + o) = v;
              }
            }
          }
          __syncwarp();  // the block is rewritten by the next batch
        }
      }
      if (MODE == kWinSisoCodes) {
        // row maxima: the row's 4 lanes, then the warps of the CTA (shared atomics on the bits
        // of non-negative floats, which order like their values)
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          float mt = rmT[hr], mc = rmC[hr];
#pragma unroll
          for (int o = 1; o <= 2; o <<= 1) {
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
            mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, o));
          }
          const int t = tb + gq + 8 * hr;
          if (tig == 0 && t < nt && g_lo < g_hi) {
            atomicMax(s.amT + t, __float_as_int(mt));
            atomicMax(s.amC + t, __float_as_int(mc));
          }
        }
      }
    }
    if (MODE == kWinSisoCodes) {
      // per-token int8 codes of both staged outputs (the codes of tesm_b200_quant_act): lane =
      // row (conflict-free on the D + 1 row pitch), 16 channels per item, 16-byte stores
      __syncthreads();
      const int gpr = p.Dp / 16;
      for (int item = tid; item < 2 * kWinT * gpr; item += NT) {
        const int t = item & (kWinT - 1), which = (item / kWinT) & 1, g16 = item / (2 * kWinT);
        if (t >= nt) continue;
        const float amax = __int_as_float(which ? s.amC[t] : s.amT[t]);
        const float sc = act_scale(amax, which ? p.eps2 : p.eps1, p.act_dtype);
        const float *src = (which ? s.oC : s.oT) + t * (D + 1);
        uint32_t wv[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t bts[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int d = g16 * 16 + 4 * q + i;
            bts[i] = d < D ? act_code_bits(round_to(p.act_dtype, __fmul_rn(src[d], sc))) : act_code_bits(0.f);
          }
          wv[q] = pack_code_bytes(bts[0], bts[1], bts[2], bts[3]);
        }
        const int64_t row = row0 + t0 + t;
        *reinterpret_cast<uint4 *>(p.codes + row * p.ldc + (which ? p.Dp : 0) + g16 * 16) =
            make_uint4(wv[0], wv[1], wv[2], wv[3]);
        if (g16 == 0) (which ? p.inv2 : p.inv1)[row] = __frcp_rn(sc);
      }
    }
    __syncthreads();  // this stage, qs/ks, twr and the staged outputs are free again
    stage ^= (NST == 2);
    if (++h == H) {
      h = 0;
      tile += gridDim.x;
      new_tile = true;
    } else {
      new_tile = false;
    }
    if (NST == 1 && tile < ntiles) {
      int64_t r1;
      int a1, n1;
      unit_of(tile, r1, a1, n1);
      win_fill<W, RM, ES, NT>(p, g, s.stage[0], mq, ms, r1, a1, n1, h);
      cp_async_commit();
    }
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");
}

template <int W, int RM, int ES, int MODE, int NT, int NST>
static int win_launch_v(WinEntParams &p, const WinGeom &g, int ctas_per_sm, cudaStream_t st, const char *what) {
  p.async16 = win_async_ok(p, ES, NT);
  if (p.R > 256) return fail(TESM_EUNSUPPORTED, std::string(what) + ": ent_rank above 256");
  p.rt = rope_table(p.R, p.rope_base);
  p.stage_out = MODE != kWinSisoCodes && p.out_dtype == TESM_BF16 && p.D % 8 == 0 && p.out_ld % 8 == 0 &&
                (uintptr_t)p.out_tanh % 16 == 0 && (uintptr_t)p.out_chg % 16 == 0;
  if (MODE == kWinSisoCodes && ((uintptr_t)p.codes % 16 != 0 || p.ldc % 16 != 0 || p.Dp % 16 != 0))
    return fail(TESM_EINVAL, std::string(what) + ": codes rows must be 16-byte aligned");
  const size_t smem = win_smem_bytes(g);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_win_ent<W, RM, ES, MODE, NT, NST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         227 * 1024);
    attr = true;
  }
  const int64_t ntiles = (int64_t)p.B * p.ntiles_b;
  const int grid = (int)std::min<int64_t>(ntiles, (int64_t)sm_count() * ctas_per_sm);
  k_win_ent<W, RM, ES, MODE, NT, NST><<<grid, NT, smem, st>>>(p);
  return check_launch(what);
}

// Host launcher: a persistent grid.  Two CTAs of 256 threads per SM when one staging buffer
// per CTA fits twice in shared memory, else one CTA of 512 threads with two buffers
// (TESM_WIN_VARIANT = 1 / 2 forces one of them).
template <int W, int RM, int ES, int MODE>
static int win_launch(WinEntParams &p, cudaStream_t st, const char *what) {
  p.ntiles_b = (int)ceil_div(p.L, kWinT);
  const WinGeom g1 = win_geom(W, p.R, p.D, RM, ES, MODE, 1), g2 = win_geom(W, p.R, p.D, RM, ES, MODE, 2);
  static int force = -1;
  if (force < 0) {
    const char *e = getenv("TESM_WIN_VARIANT");
    force = e ? atoi(e) : 0;
  }
  const bool two = win_smem_bytes(g1) <= 113 * 1024;
  if ((two && force != 2) || (force == 1 && win_smem_bytes(g1) <= 227 * 1024))
    return win_launch_v<W, RM, ES, MODE, 256, 1>(p, g1, two ? 2 : 1, st, what);
  if (win_smem_bytes(g2) <= 227 * 1024) return win_launch_v<W, RM, ES, MODE, 512, 2>(p, g2, 1, st, what);
  if (win_smem_bytes(g1) <= 227 * 1024) return win_launch_v<W, RM, ES, MODE, 256, 1>(p, g1, 1, st, what);
  return fail(TESM_EUNSUPPORTED, std::string(what) + ": d_state / ent_rank too large for one tile in shared memory");
}

}  // namespace tesm
