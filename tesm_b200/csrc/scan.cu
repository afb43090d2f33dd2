// Selective state scan h_t = a_t * h_{t-1} + u_t for SISO and MIMO layers.
//
//   SISO (tesm.py:1198-1223, scan :1091-1164): a = sigmoid(decay + decay_bias),
//        u = sigmoid(write) * tanh(value); the reference scans in fp64 chunks, here fp32 FMA in
//        time order (relative error ~1e-6, within the 1e-3 fp32 bar).
//        The reference's chunk formula h_t = A_t (h_c + sum_s u_s / max(A_s, 1e-12)), with A the
//        in-chunk cumulative product of max(a, 1e-12) (tesm.py:1085-1088, 1133-1153), differs
//        from the plain recurrence once A drops below 1e-12 inside a chunk (small decays, e.g.
//        a = sigmoid(N(0,1))).  It equals the recurrence h_t = a_t h_{t-1} + u_t min(1, A_t/1e-12),
//        which the SISO kernels run with A restarted at every multiple of the reference's
//        state_scan_chunk_size (`cs`; 0 = the plain recurrence).
//   MIMO (tesm_mimo.py:959-989, scan :375-392): ranks r share a; u_r = (write*x_r)*(value*x_r)
//        with x_r = mimo_x[h, r, :]; the reference scans in fp32 with separate mul/add roundings,
//        reproduced with __fmul_rn/__fadd_rn.
//
// Parallel structure: one thread per channel (all ranks of that channel), chunks of T
// positions; the chunks of a (batch, channel-slice) chain exchange carries by decoupled
// look-back.  Each chunk publishes its aggregate affine map (A, U_r) as soon as its first pass
// is done, then its inclusive states once its carry-in is known; successors fold aggregates
// until they meet an inclusive value.  Chunk order comes from an atomic ticket, so a chunk only
// ever waits on chunks that are already running -- no deadlock regardless of launch order.
// The wait is bounded (~2 s); on timeout the sticky device status is set.
#include "layer_common.cuh"

namespace tesm {

struct ScanParams {
  ProjCols pc;
  const float *decay_bias;  // (C)
  const float *mimo_x;      // (H, RM, D) or null (SISO)
  const double *h0;         // (B, C) or null
  int B, L, C, D, RM;
  int cs;                   // reference scan chunk for the 1e-12 clamp (SISO), 0 = none
  int T, nchunks, nslices;
  float *states;            // (B, L, RM, C)
  float *final_f32;         // (B, C) rank 0
  double *final_f64;        // (B, C) rank 0
  float *aggA;              // (B, nchunks, C)
  float *aggU;              // (B, nchunks, RM, C)
  float *incl;              // (B, nchunks, RM, C)
  int *flags;               // (B, nslices, nchunks)
  int *ticket;
};

template <bool MIMO>
__device__ __forceinline__ float step(float a, float h, float u) {
  return MIMO ? __fadd_rn(__fmul_rn(a, h), u) : fmaf(a, h, u);
}


// Stage the chunk's inputs in shared memory, transformed once: plane 0 = a = sigmoid(decay +
// decay_bias); SISO plane 1 = u = sigmoid(write) * tanh(value); MIMO planes 1, 2 = sigmoid(write),
// tanh(value) (the ranks are formed on the fly).  Rows are read once with 16-byte loads when
// rows and column offsets are aligned.  (sigmoid with __expf: relative error ~1e-7.)
template <bool MIMO, int VPT>
__device__ __forceinline__ void stage_store(const ScanParams &p, int o, int c, const float *dv, const float *wv,
                                            const float *vv, float *s0, float *s1, float *s2) {
  float a[VPT], x[VPT], y[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    a[j] = fast_sigmoid(dv[j] + p.decay_bias[c + j]);
    const float w = fast_sigmoid(wv[j]), v = tanhf(vv[j]);
    x[j] = MIMO ? w : w * v;
    y[j] = v;
  }
  if (VPT == 8 || VPT == 4) {  // 16-byte stores (o is a multiple of VPT)
#pragma unroll
    for (int q = 0; q < VPT; q += 4) {
      *reinterpret_cast<float4 *>(s0 + o + q) = make_float4(a[q], a[q + 1], a[q + 2], a[q + 3]);
      *reinterpret_cast<float4 *>(s1 + o + q) = make_float4(x[q], x[q + 1], x[q + 2], x[q + 3]);
      if (MIMO) *reinterpret_cast<float4 *>(s2 + o + q) = make_float4(y[q], y[q + 1], y[q + 2], y[q + 3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      s0[o + j] = a[j];
      s1[o + j] = x[j];
      if (MIMO) s2[o + j] = y[j];
    }
  }
}

// Stage the chunk's inputs in shared memory, transformed once: plane 0 = a = sigmoid(decay +
// decay_bias); SISO plane 1 = u = sigmoid(write) * tanh(value); MIMO planes 1, 2 = sigmoid(write),
// tanh(value) (the ranks are formed on the fly).  With aligned rows every thread issues all of
// its 16-byte loads (PFI groups at a time) before converting any, and stores 16-byte vectors.
// (sigmoid with __expf: relative error ~1e-7.)
template <bool MIMO>
__device__ __forceinline__ void stage_inputs(const ScanParams &p, int64_t row0, int t0, int nt, int c0, int S,
                                             float *s0, float *s1, float *s2, int vec) {
  const int esz = p.pc.dtype == TESM_BF16 ? 2 : 4;
  const uint8_t *base = reinterpret_cast<const uint8_t *>(p.pc.proj);
  if (vec) {
    const int VPT = 16 / esz;
    const int groups = S / VPT, items = nt * groups;
    constexpr int PFI = 2;
    for (int i0 = threadIdx.x; i0 < items; i0 += PFI * blockDim.x) {
      uint4 d4[PFI], w4[PFI], v4[PFI];
      int tt[PFI], cg[PFI];
      bool ok[PFI];
#pragma unroll
      for (int k = 0; k < PFI; ++k) {
        const int i = i0 + k * blockDim.x;
        tt[k] = i / groups;
        cg[k] = (i - tt[k] * groups) * VPT;
        ok[k] = i < items && c0 + cg[k] < p.C;
        if (ok[k]) {
          const uint8_t *rowp = base + ((row0 + t0 + tt[k]) * p.pc.ld) * esz;
          const int c = c0 + cg[k];
          d4[k] = *reinterpret_cast<const uint4 *>(rowp + (int64_t)(p.pc.c_decay + c) * esz);
          w4[k] = *reinterpret_cast<const uint4 *>(rowp + (int64_t)(p.pc.c_write + c) * esz);
          v4[k] = *reinterpret_cast<const uint4 *>(rowp + (int64_t)(p.pc.c_value + c) * esz);
        }
      }
#pragma unroll
      for (int k = 0; k < PFI; ++k) {
        if (!ok[k]) continue;
        float dv[8], wv[8], vv[8];
        if (esz == 2) {
          const __nv_bfloat16 *dh = reinterpret_cast<const __nv_bfloat16 *>(&d4[k]);
          const __nv_bfloat16 *wh = reinterpret_cast<const __nv_bfloat16 *>(&w4[k]);
          const __nv_bfloat16 *vh = reinterpret_cast<const __nv_bfloat16 *>(&v4[k]);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            dv[j] = __bfloat162float(dh[j]);
            wv[j] = __bfloat162float(wh[j]);
            vv[j] = __bfloat162float(vh[j]);
          }
        } else {
          const float *df = reinterpret_cast<const float *>(&d4[k]);
          const float *wf = reinterpret_cast<const float *>(&w4[k]);
          const float *vf = reinterpret_cast<const float *>(&v4[k]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            dv[j] = df[j];
            wv[j] = wf[j];
            vv[j] = vf[j];
          }
        }
        if (esz == 2)
          stage_store<MIMO, 8>(p, tt[k] * S + cg[k], c0 + cg[k], dv, wv, vv, s0, s1, s2);
        else
          stage_store<MIMO, 4>(p, tt[k] * S + cg[k], c0 + cg[k], dv, wv, vv, s0, s1, s2);
      }
    }
  } else {
    for (int i = threadIdx.x; i < nt * S; i += blockDim.x) {
      const int t = i / S, cg = i - t * S, c = c0 + cg;
      if (c >= p.C) continue;
      const int64_t rb = (row0 + t0 + t) * p.pc.ld;
      float dv[1], wv[1], vv[1];
      dv[0] = load_f(p.pc.proj, p.pc.dtype, rb + p.pc.c_decay + c);
      wv[0] = load_f(p.pc.proj, p.pc.dtype, rb + p.pc.c_write + c);
      vv[0] = load_f(p.pc.proj, p.pc.dtype, rb + p.pc.c_value + c);
      stage_store<MIMO, 1>(p, t * S + cg, c, dv, wv, vv, s0, s1, s2);
    }
  }
}

template <int RM, bool MIMO>
__global__ void __launch_bounds__(256, 4) k_scan(ScanParams p, int vec) {
  extern __shared__ __align__(16) uint8_t sm_scan[];
  __shared__ int s_tile, s_jinc;
  if (threadIdx.x == 0) s_tile = atomicAdd(p.ticket, 1);
  __syncthreads();
  const int tile = s_tile;
  const int per_chunk = p.B * p.nslices;
  const int chunk = tile / per_chunk;
  const int bs = tile - chunk * per_chunk;
  const int b = bs / p.nslices, slice = bs - b * p.nslices;
  const int S = blockDim.x;
  const int c0 = slice * S;
  const int c = c0 + threadIdx.x;
  const bool active = c < p.C;
  const int t0 = chunk * p.T, t1 = min(t0 + p.T, p.L), nt = t1 - t0;
  float *s0 = reinterpret_cast<float *>(sm_scan), *s1 = s0 + p.T * S, *s2 = s1 + p.T * S;
  const int64_t row0 = (int64_t)b * p.L;
  stage_inputs<MIMO>(p, row0, t0, nt, c0, S, s0, s1, s2, vec);
  float mx[RM];
#pragma unroll
  for (int r = 0; r < RM; ++r) mx[r] = 0.f;
  if (active && MIMO) {
    const int h = c / p.D, d = c - h * p.D;
#pragma unroll
    for (int r = 0; r < RM; ++r) mx[r] = p.mimo_x[((int64_t)h * RM + r) * p.D + d];
  }
  __syncthreads();
  // SISO: running product of max(a, 1e-12) since the last reference chunk start (T % cs == 0,
  // so every kernel chunk starts one); the caller resets `cp` to 1 before each pass
  float cp = 1.f;
  auto inputs = [&](int t, float &a, float (&u)[RM]) {
    const int i = t * S + threadIdx.x;
    a = s0[i];
    if (MIMO) {
      const float w = s1[i], v = s2[i];
#pragma unroll
      for (int r = 0; r < RM; ++r) u[r] = __fmul_rn(__fmul_rn(w, mx[r]), __fmul_rn(v, mx[r]));
    } else {
      u[0] = s1[i];
      if (p.cs > 0) {
        if (t % p.cs == 0) cp = 1.f;
        cp *= fmaxf(a, 1e-12f);
        u[0] *= fminf(1.f, cp * 1e12f);
      }
    }
  };

  // pass 1: aggregate affine map of this chunk (A shared by the ranks)
  float A = 1.f, U[RM];
#pragma unroll
  for (int r = 0; r < RM; ++r) U[r] = 0.f;
  if (active) {
    cp = 1.f;
    for (int t = 0; t < nt; ++t) {
      float a, u[RM];
      inputs(t, a, u);
#pragma unroll
      for (int r = 0; r < RM; ++r) U[r] = step<MIMO>(a, U[r], u[r]);
      A *= a;
    }
  }
  int *flag_row = p.flags + ((int64_t)b * p.nslices + slice) * p.nchunks;
  const int64_t cidx = ((int64_t)b * p.nchunks + chunk);
  if (chunk > 0 && chunk + 1 < p.nchunks) {  // the last chunk has no successor
    if (active) {
      p.aggA[cidx * p.C + c] = A;
#pragma unroll
      for (int r = 0; r < RM; ++r) p.aggU[(cidx * RM + r) * p.C + c] = U[r];
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) st_release(flag_row + chunk, 1);
  }
  // look-back for the carry entering this chunk: warp 0 scans 32 predecessor flags per round
  // trip and finds the nearest inclusive chunk j with every chunk in (j, chunk) published;
  // then every thread folds the inclusive state and those aggregates forward.
  float h[RM];
#pragma unroll
  for (int r = 0; r < RM; ++r) h[r] = 0.f;
  if (active && p.h0) h[0] = (float)p.h0[(int64_t)b * p.C + c];
  if (chunk > 0) {
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      int base = chunk - 1, jinc = -1;
      const long long start = clock64();
      while (true) {
        const int j = base - lane;
        const int f = j >= 0 ? ld_acquire(flag_row + j) : 2;
        const unsigned b2 = __ballot_sync(0xffffffffu, f == 2);
        const unsigned b0 = __ballot_sync(0xffffffffu, f == 0);
        const int first2 = b2 ? __ffs(b2) - 1 : 32, first0 = b0 ? __ffs(b0) - 1 : 32;
        if (first2 < 32 && first2 < first0) {
          jinc = base - first2;
          break;
        }
        if (first0 == 32) {  // 32 published aggregates, no inclusive yet: look further back
          base -= 32;
          continue;
        }
        if (clock64() - start > kSpinLimit * 64) {
          if (lane == 0) flag_timeout();
          jinc = -2;
          break;
        }
      }
      if (lane == 0) s_jinc = jinc;
    }
    __syncthreads();
    const int jinc = s_jinc;
    if (active && jinc >= 0) {
      const int64_t ji = (int64_t)b * p.nchunks + jinc;
#pragma unroll
      for (int r = 0; r < RM; ++r) h[r] = p.incl[(ji * RM + r) * p.C + c];
      // fold forward, FB aggregates per batch with all their loads issued first
      constexpr int FB = RM >= 4 ? 2 : (RM == 2 ? 4 : 8);
      for (int j0 = jinc + 1; j0 < chunk; j0 += FB) {
        float gA[FB], gU[FB][RM];
#pragma unroll
        for (int k = 0; k < FB; ++k) {
          const int j = j0 + k;
          const int64_t jj = (int64_t)b * p.nchunks + (j < chunk ? j : jinc);
          gA[k] = j < chunk ? p.aggA[jj * p.C + c] : 1.f;
#pragma unroll
          for (int r = 0; r < RM; ++r) gU[k][r] = j < chunk ? p.aggU[(jj * RM + r) * p.C + c] : 0.f;
        }
#pragma unroll
        for (int k = 0; k < FB; ++k)
#pragma unroll
          for (int r = 0; r < RM; ++r) h[r] = fmaf(gA[k], h[r], gU[k][r]);
      }
    }
  }
  // publish the inclusive states for successors
  if (chunk + 1 < p.nchunks) {
    if (active) {
#pragma unroll
      for (int r = 0; r < RM; ++r) p.incl[(cidx * RM + r) * p.C + c] = fmaf(A, h[r], U[r]);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) st_release(flag_row + chunk, 2);
  }
  // pass 2: states of this chunk from the carry
  if (active) {
    cp = 1.f;
    for (int t = 0; t < nt; ++t) {
      float a, u[RM];
      inputs(t, a, u);
      const int64_t orow = (row0 + t0 + t) * RM;
#pragma unroll
      for (int r = 0; r < RM; ++r) {
        h[r] = step<MIMO>(a, h[r], u[r]);
        p.states[(orow + r) * p.C + c] = h[r];
      }
    }
    if (t1 == p.L) {
      p.final_f32[(int64_t)b * p.C + c] = h[0];
      p.final_f64[(int64_t)b * p.C + c] = (double)h[0];
    }
  }
}

// SISO scan with the chunk held in registers.  A CTA covers SLICE2 = 256 channels x G*TT
// positions: thread (g, cp) owns channels c0 + 2cp, c0 + 2cp + 1 (one bf16x2 load per column per
// position) over positions g*TT .. g*TT+TT-1 of the chunk.  All 3*TT loads of a thread are issued
// before any use, a and u are formed in registers, the G time groups combine their affine maps
// through shared memory, and CTAs chain by the same decoupled look-back as k_scan.
constexpr int SLICE2 = 256;


__device__ __forceinline__ uint32_t ldg_nc_u32(const void *p) {
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.b32 %0, [%1];\n" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;
// carry words: gpu-scope relaxed accesses (L1 bypassed); 0xffffffff marks "not yet written"
__device__ __forceinline__ void st_relaxed_f2(float *p, float x, float y) {
  asm volatile("st.relaxed.gpu.global.v2.f32 [%0], {%1, %2};\n" ::"l"(p), "f"(x), "f"(y) : "memory");
}
__device__ __forceinline__ float2 ld_relaxed_f2(const float *p) {
  float2 v;
  asm volatile("ld.relaxed.gpu.global.v2.f32 {%0, %1}, [%2];\n" : "=f"(v.x), "=f"(v.y) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool ready2(float2 v) {
  return __float_as_uint(v.x) != 0xffffffffu && __float_as_uint(v.y) != 0xffffffffu;
}
// a = sigmoid(d + bias) = 1 / (1 + 2^(-(d + bias) log2 e)); nbias = -bias log2 e.
// Relative error a few ulp (approximate 2^x and 1/x instructions).
__device__ __forceinline__ float decay_gate(float d, float nbias) {
  return rcp_approx(1.f + ex2_approx(fmaf(d, -kLog2e, nbias)));
}
// u = sigmoid(w) tanh(v) = (e^(2v) - 1) / ((1 + e^(-w)) (1 + e^(2v))), one reciprocal; v is
// clamped to +-15 (tanh(15) rounds to 1 in fp32) so e^(2v) stays finite.  Absolute error a few
// 1e-7 (the difference e^(2v) - 1 near v = 0 carries the exponential's rounding).
__device__ __forceinline__ float write_value(float w, float v) {
  v = fminf(fmaxf(v, -15.f), 15.f);
  const float e1 = ex2_approx(w * -kLog2e), e2 = ex2_approx(v * (2.f * kLog2e));
  return (e2 - 1.f) * rcp_approx((1.f + e1) * (1.f + e2));
}

template <int TT, int G>
__global__ void __launch_bounds__(128 * G) k_scan_siso_reg(ScanParams p) {
  __shared__ float4 s_map[G][128];  // per time group: (A0, A1, U0, U1)
  __shared__ float2 s_carry[128];   // carry entering the chunk
  __shared__ int s_tile;
  if (threadIdx.x == 0) s_tile = atomicAdd(p.ticket, 1);
  __syncthreads();
  const int tile = s_tile;
  const int per_chunk = p.B * p.nslices;
  const int chunk = tile / per_chunk;
  const int bs = tile - chunk * per_chunk;
  const int b = bs / p.nslices, slice = bs - b * p.nslices;
  const int g = threadIdx.x >> 7, cp = threadIdx.x & 127;
  const int c = slice * SLICE2 + 2 * cp;
  const bool active = c < p.C;  // C even: both channels or neither
  const int t0 = chunk * (G * TT) + g * TT;
  const int64_t row0 = (int64_t)b * p.L;
  const __nv_bfloat16 *proj = reinterpret_cast<const __nv_bfloat16 *>(p.pc.proj);

  uint32_t rd[TT], rw[TT], rv[TT];
#pragma unroll
  for (int t = 0; t < TT; ++t) {
    if (active && t0 + t < p.L) {
      const __nv_bfloat16 *row = proj + (row0 + t0 + t) * p.pc.ld + c;
      rd[t] = ldg_nc_u32(row + p.pc.c_decay);
      rw[t] = ldg_nc_u32(row + p.pc.c_write);
      rv[t] = ldg_nc_u32(row + p.pc.c_value);
    } else {
      rd[t] = 0x7f807f80u;  // +inf, +inf: a = 1 ...
      rw[t] = 0;
      rv[t] = 0;            // ... and u = 0: an identity step
    }
  }
  float nb0 = 0.f, nb1 = 0.f;
  if (active) {
    nb0 = -kLog2e * p.decay_bias[c];
    nb1 = -kLog2e * p.decay_bias[c + 1];
  }
  float a0[TT], a1[TT], u0[TT], u1[TT];
  float A0 = 1.f, A1 = 1.f, U0 = 0.f, U1 = 0.f;
#pragma unroll
  for (int t = 0; t < TT; ++t) {
    a0[t] = decay_gate(bf16lo(rd[t]), nb0);
    a1[t] = decay_gate(bf16hi(rd[t]), nb1);
    A0 *= a0[t];
    A1 *= a1[t];
  }
  // The reference's chunk clamp u_t * min(1, P_t / 1e-12), P_t the running decay product since
  // the last multiple of cs (TT % cs == 0).  P_t >= A (the thread's whole product: factors <= 1),
  // so when A >= 2e-12 every factor min(1, P_t * 1e12) is exactly 1 and the clamp is skipped.
  const int cs = p.cs;
  const bool clamp = cs > 0 && __any_sync(0xffffffffu, A0 < 2e-12f || A1 < 2e-12f);
  float P0 = 1.f, P1 = 1.f;
#pragma unroll
  for (int t = 0; t < TT; ++t) {
    u0[t] = write_value(bf16lo(rw[t]), bf16lo(rv[t]));
    u1[t] = write_value(bf16hi(rw[t]), bf16hi(rv[t]));
    if (clamp) {
      if (t % cs == 0) P0 = P1 = 1.f;
      P0 *= fmaxf(a0[t], 1e-12f);
      P1 *= fmaxf(a1[t], 1e-12f);
      u0[t] *= fminf(1.f, P0 * 1e12f);
      u1[t] *= fminf(1.f, P1 * 1e12f);
    }
    U0 = fmaf(a0[t], U0, u0[t]);
    U1 = fmaf(a1[t], U1, u1[t]);
  }
  // combine the time groups: exclusive map E of groups 0..g-1, total map of the chunk
  s_map[g][cp] = make_float4(A0, A1, U0, U1);
  __syncthreads();
  float EA0 = 1.f, EA1 = 1.f, EU0 = 0.f, EU1 = 0.f, TA0, TA1, TU0, TU1;
#pragma unroll
  for (int k = 0; k < G; ++k) {
    const float4 m = s_map[k][cp];
    if (k == g) {
      TA0 = EA0, TA1 = EA1, TU0 = EU0, TU1 = EU1;  // save the exclusive map
    }
    EU0 = fmaf(m.x, EU0, m.z);
    EU1 = fmaf(m.y, EU1, m.w);
    EA0 *= m.x;
    EA1 *= m.y;
  }
  // now (EA, EU) is the chunk's total map and (TA, TU) this group's exclusive map.
  // Carry exchange without flags or fences: aggregate and inclusive words start as the
  // all-ones NaN pattern (reset before the launch) and each channel's value is its own
  // readiness signal.  Group 0 publishes, then walks back through its predecessors, K per
  // round trip, folding aggregates until it meets an inclusive state.
  const int64_t cidx = ((int64_t)b * p.nchunks + chunk);
  if (g == 0) {
    if (active && chunk > 0 && chunk + 1 < p.nchunks) {
      st_relaxed_f2(p.aggA + cidx * p.C + c, EA0, EA1);
      st_relaxed_f2(p.aggU + cidx * p.C + c, EU0, EU1);
    }
    float h0 = 0.f, h1 = 0.f;
    if (active && p.h0) {
      h0 = (float)p.h0[(int64_t)b * p.C + c];
      h1 = (float)p.h0[(int64_t)b * p.C + c + 1];
    }
    if (active && chunk > 0) {
      constexpr int K = 4;
      float FA0 = 1.f, FA1 = 1.f, FU0 = 0.f, FU1 = 0.f;  // fold of chunks (j, chunk)
      int j = chunk - 1;
      bool done = false;
      const long long start = clock64();
      while (!done) {
        float2 inc[K], ga[K], gu[K];
#pragma unroll
        for (int k = 0; k < K; ++k) {
          const int64_t jj = (int64_t)b * p.nchunks + max(j - k, 0);
          inc[k] = ld_relaxed_f2(p.incl + jj * p.C + c);
          ga[k] = ld_relaxed_f2(p.aggA + jj * p.C + c);
          gu[k] = ld_relaxed_f2(p.aggU + jj * p.C + c);
        }
        int next = j;
#pragma unroll
        for (int k = 0; k < K; ++k) {
          if (done || next != j - k || j - k < 0) continue;
          if (ready2(inc[k])) {
            h0 = fmaf(FA0, inc[k].x, FU0);
            h1 = fmaf(FA1, inc[k].y, FU1);
            done = true;
          } else if (ready2(ga[k]) && ready2(gu[k])) {
            FU0 = fmaf(FA0, gu[k].x, FU0);
            FU1 = fmaf(FA1, gu[k].y, FU1);
            FA0 *= ga[k].x;
            FA1 *= ga[k].y;
            next = j - k - 1;
          }
        }
        j = next;
        if (!done && clock64() - start > kSpinLimit * 64) {
          flag_timeout();
          break;
        }
      }
    }
    s_carry[cp] = make_float2(h0, h1);
    if (active && chunk + 1 < p.nchunks)
      st_relaxed_f2(p.incl + cidx * p.C + c, fmaf(EA0, h0, EU0), fmaf(EA1, h1, EU1));
  }
  __syncthreads();
  if (!active) return;
  const float2 hin = s_carry[cp];
  float h0 = fmaf(TA0, hin.x, TU0), h1 = fmaf(TA1, hin.y, TU1);
#pragma unroll
  for (int t = 0; t < TT; ++t) {
    if (t0 + t < p.L) {
      h0 = fmaf(a0[t], h0, u0[t]);
      h1 = fmaf(a1[t], h1, u1[t]);
      __stcs(reinterpret_cast<float2 *>(p.states + (row0 + t0 + t) * p.C + c), make_float2(h0, h1));
      if (t0 + t == p.L - 1) {
        p.final_f32[(int64_t)b * p.C + c] = h0;
        p.final_f32[(int64_t)b * p.C + c + 1] = h1;
        p.final_f64[(int64_t)b * p.C + c] = (double)h0;
        p.final_f64[(int64_t)b * p.C + c + 1] = (double)h1;
      }
    }
  }
}

struct ScanLayout {
  int T, slice, nchunks, nslices;
  int64_t off_aggU, off_incl, off_flags, bytes;
};

static ScanLayout scan_layout(int64_t B, int64_t L, int64_t C, int64_t RM) {
  ScanLayout s;
  s.T = RM > 1 ? 16 : 32;  // measured: MIMO (3 staged planes) prefers more, shorter chunks
  static int force = -1;
  if (force < 0) {
    const char *e = getenv("TESM_SCAN_T");  // tuning override: positions per chunk
    force = e ? atoi(e) : 0;
  }
  if (force > 0) s.T = force;
  s.slice = C < 256 ? (int)round_up(C, 32) : 256;
  if (RM == 1) s.slice = 256;  // the register-resident SISO kernel always covers 256 channels per CTA
  s.nchunks = (int)ceil_div(L, s.T);
  s.nslices = (int)ceil_div(C, s.slice);
  const int64_t nA = B * s.nchunks * C;
  s.off_aggU = round_up(nA * 4, 256);
  s.off_incl = s.off_aggU + round_up(nA * RM * 4, 256);
  s.off_flags = s.off_incl + round_up(nA * RM * 4, 256);
  s.bytes = s.off_flags + round_up((B * s.nslices * s.nchunks + 1) * 4, 256);
  return s;
}

template <int RM, bool MIMO>
static int launch_scan(ScanParams &p, cudaStream_t st, int slice) {
  const int64_t grid = (int64_t)p.nchunks * p.B * p.nslices;
  const size_t smem = sizeof(float) * (size_t)(MIMO ? 3 : 2) * p.T * slice;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_scan<RM, MIMO>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
    cudaFuncSetAttribute(k_scan<RM, MIMO>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    attr = true;
  }
  const int esz = p.pc.dtype == TESM_BF16 ? 2 : 4, vpt = 16 / esz;
  const int vec = ((uintptr_t)p.pc.proj % 16 == 0) && ((p.pc.ld * esz) % 16 == 0) && (p.pc.c_decay % vpt == 0) &&
                  (p.pc.c_write % vpt == 0) && (p.pc.c_value % vpt == 0) && (p.C % vpt == 0) && (slice % vpt == 0);
  k_scan<RM, MIMO><<<(unsigned)grid, slice, smem, st>>>(p, vec);
  return check_launch("scan");
}

static int run_scan(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L, int64_t Dm, int64_t H,
                    int64_t D, int64_t R, int64_t RM, const float *decay_bias, const float *mimo_x,
                    const double *h0, float *states, float *final_f32, double *final_f64, void *workspace,
                    int64_t ws_bytes, cudaStream_t st, int64_t scan_chunk = 0) {
  TESM_REQUIRE(proj && decay_bias && states && final_f32 && final_f64 && workspace, "scan: null pointer");
  TESM_REQUIRE(B > 0 && L > 0 && D > 0 && H > 0 && ldp >= 2 * Dm + 3 * H * D + 2 * H * R, "scan: bad shape");
  if (dtype != TESM_F32 && dtype != TESM_BF16) return fail(TESM_EDTYPE, "scan: dtype");
  const int64_t C = H * D;
  ScanLayout s = scan_layout(B, L, C, RM);
  TESM_REQUIRE(ws_bytes >= s.bytes, "scan: workspace too small (query the *_workspace function)");
  ScanParams p;
  p.pc = make_cols(proj, dtype, ldp, (int)Dm, (int)C, (int)(H * R));
  p.decay_bias = decay_bias;
  p.mimo_x = mimo_x;
  p.h0 = h0;
  p.B = (int)B;
  p.L = (int)L;
  p.C = (int)C;
  p.D = (int)D;
  p.RM = (int)RM;
  TESM_REQUIRE(scan_chunk >= 0, "scan: bad state_scan_chunk_size");
  // the reference's chunk is min(state_scan_chunk_size, L) (tesm.py:1094)
  p.cs = mimo_x ? 0 : (int)(scan_chunk < L ? scan_chunk : L);
  p.T = s.T;
  p.nchunks = s.nchunks;
  p.nslices = s.nslices;
  p.states = states;
  p.final_f32 = final_f32;
  p.final_f64 = final_f64;
  uint8_t *ws = (uint8_t *)workspace;
  p.aggA = (float *)ws;
  p.aggU = (float *)(ws + s.off_aggU);
  p.incl = (float *)(ws + s.off_incl);
  p.flags = (int *)(ws + s.off_flags);
  p.ticket = p.flags + B * s.nslices * s.nchunks;
  cudaError_t e = cudaMemsetAsync(p.flags, 0, (B * s.nslices * s.nchunks + 1) * sizeof(int), st);
  if (e != cudaSuccess) return fail(TESM_ELAUNCH, std::string("scan memset: ") + cudaGetErrorString(e));
  if (!mimo_x) {
    // register-resident kernel for bf16 projections with 4-byte aligned channel pairs
    static int reg_mode = -1, reg_tt = 16;
    if (reg_mode < 0) {
      const char *e = getenv("TESM_SCAN_REG");  // tuning override: 0 = shared-memory kernel
      reg_mode = e ? atoi(e) : 1;
      if (const char *t = getenv("TESM_SCAN_TT")) reg_tt = atoi(t);  // positions per thread
    }
    const bool pairs = dtype == TESM_BF16 && (uintptr_t)proj % 4 == 0 && ldp % 2 == 0 && C % 2 == 0 &&
                       p.pc.c_decay % 2 == 0 && p.pc.c_write % 2 == 0 && p.pc.c_value % 2 == 0 &&
                       (uintptr_t)states % 8 == 0;
    if (reg_mode && pairs && (p.cs == 0 || reg_tt % p.cs == 0 || L <= reg_tt)) {
      const int G = s.T / reg_tt;
      e = cudaMemsetAsync(workspace, 0xff, s.off_flags, st);  // carry words to "not yet written"
      if (e != cudaSuccess) return fail(TESM_ELAUNCH, std::string("scan memset: ") + cudaGetErrorString(e));
      const unsigned grid = (unsigned)((int64_t)p.nchunks * p.B * p.nslices);
#define TESM_SCAN_REG_CASE(TT_, G_)                                              \
  if (reg_tt == TT_ && G == G_) {                                                \
    k_scan_siso_reg<TT_, G_><<<grid, 128 * G_, 0, st>>>(p);                      \
    return check_launch("scan");                                                 \
  }
      TESM_SCAN_REG_CASE(16, 2)
      TESM_SCAN_REG_CASE(16, 1)
      TESM_SCAN_REG_CASE(16, 4)
      TESM_SCAN_REG_CASE(8, 2)
      TESM_SCAN_REG_CASE(8, 4)
      TESM_SCAN_REG_CASE(32, 1)
      TESM_SCAN_REG_CASE(32, 2)
#undef TESM_SCAN_REG_CASE
    }
    // every restart of the clamp product must fall inside one thread's chunk of T positions
    if (p.cs > 0 && p.T % p.cs != 0 && L > p.T)
      return fail(TESM_EUNSUPPORTED, "scan: state_scan_chunk_size " + std::to_string(scan_chunk) +
                                         " must divide " + std::to_string(p.T) + " (the kernel's chunk)");
    return launch_scan<1, false>(p, st, s.slice);
  }
  switch (RM) {
    case 1: return launch_scan<1, true>(p, st, s.slice);
    case 2: return launch_scan<2, true>(p, st, s.slice);
    case 4: return launch_scan<4, true>(p, st, s.slice);
    case 8: return launch_scan<8, true>(p, st, s.slice);
    default: return fail(TESM_EUNSUPPORTED, "scan: mimo_rank must be 1, 2, 4 or 8");
  }
}

}  // namespace tesm

using namespace tesm;


extern "C" int tesm_b200_scan_workspace(int64_t B, int64_t L, int64_t C, int64_t RM, int64_t *bytes) {
  TESM_REQUIRE(bytes && B > 0 && L > 0 && C > 0 && RM > 0, "scan_workspace: bad argument");
  *bytes = scan_layout(B, L, C, RM).bytes;
  return TESM_OK;
}

extern "C" int tesm_b200_siso_scan(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L, int64_t Dm,
                                   int64_t D, int64_t R, int64_t scan_chunk, const float *decay_bias,
                                   const double *h0, float *states, float *final_f32, double *final_f64,
                                   void *workspace, int64_t ws_bytes, tesm_stream_t stream) {
  return run_scan(proj, dtype, ldp, B, L, Dm, 1, D, R, 1, decay_bias, nullptr, h0, states, final_f32, final_f64,
                  workspace, ws_bytes, (cudaStream_t)stream, scan_chunk);
}

extern "C" int tesm_b200_mimo_scan(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L, int64_t Dm,
                                   int64_t H, int64_t D, int64_t R, int64_t RM, const float *decay_bias,
                                   const float *mimo_x, float *states, float *final_f32, double *final_f64,
                                   void *workspace, int64_t ws_bytes, tesm_stream_t stream) {
  TESM_REQUIRE(mimo_x != nullptr, "mimo_scan: null mimo_x");
  return run_scan(proj, dtype, ldp, B, L, Dm, H, D, R, RM, decay_bias, mimo_x, nullptr, states, final_f32,
                  final_f64, workspace, ws_bytes, (cudaStream_t)stream);
}
