// Causal global ternary entanglement on the tensor cores (tcgen05.mma kind::f16, TMEM).
//
// Reference: tesm_ssm/modules/tesm.py _compute_entanglement, torch rung :1031-1043 with the
// relative bias of :970-982 and the lerp of :1231-1232.  Per batch b and query position i:
//   sc[i,j]  = (q_i . k_j) / sqrt(R) + relb[i - j]            (j <= i)
//   t[i,j]   = +1 if sc > thr, -1 if sc < -thr, else 0
//   avg_i    = sum_j t[i,j] v_j / max(sum_j |t[i,j]|, 1)      (v = scan states)
//   ent_i    = s_i + es (avg_i - s_i);  outputs tanh(ent_i) and ent_i - s_i
//
// Layout and precision.  A prep pass writes q (RoPE + cross-layer bias) and k (RoPE) as fp16
// hi/lo pairs (x = hi + lo, lo = fp16(x - hi)), R zero-padded to 64, and the states transposed
// to fp16 hi/lo pairs (B, DS, Lp) with DS = D rounded up to 16.  q.k is three MMAs (hi.hi +
// hi.lo + lo.hi, fp32 accumulation): ~22 mantissa bits, so a ternary decision differs from the
// fp32 torch path only for scores within ~1e-6 of the threshold.  t is exact in fp16 and t.v is
// two MMAs (t.v_hi + t.v_lo), so avg carries ~2^-22 relative rounding, like fp32.
//
// Kernel: one CTA per (batch, 128-query tile), heaviest tiles first, blocks of 64 keys.
// (Warp roles below; the score MMAs and the t.v^T MMAs are issued by two separate warps, warps 1
// and 19, so that neither waits behind the other's issue.)  Warp 0
// streams k tiles (hi + lo) and warp 18 v^T tiles (hi + lo, 4x larger) through 2-stage TMA
// rings; warp 1 issues the MMAs; warps 2..17 (four per TMEM lane quarter, 16 key columns each)
// turn scores into ternaries written straight into the shared-memory A operand of the t.v^T MMA,
// then run the epilogue.  Scores are triple-buffered in TMEM (3 x 64 columns next to the 128 x DS
// fp32 accumulator) and ternary tiles double-buffered in shared memory; the MMA warp issues the
// score MMAs of block j+2 before the t.v^T MMAs of block j, so the ternary warps never wait for
// scores and the tensor pipe never waits for more than one ternary pass.  Every wait is bounded.

#include "layer_common.cuh"

#include <cuda_fp16.h>

namespace tesm {
namespace gtc {

using tc::fence_after;
using tc::fence_before;
using tc::mbar_arrive;
using tc::mbar_expect_tx;
using tc::mbar_init;
using tc::mbar_wait;
using tc::smem_desc_sw128;
using tc::smem_u32;
using tc::tma_load_2d;
using tc::tmem_ld32;

constexpr int QT = 128;  // query rows per CTA (TMEM lanes)
constexpr int KB = 64;   // keys per block
constexpr int RP = 64;   // padded ent_rank (one 128-byte swizzle atom of fp16)
constexpr int NSK = 3;   // k ring stages
constexpr int NSV = 2;   // v^T ring stages
constexpr int TW = 16;   // ternary / epilogue warps: 4 per TMEM lane quarter, 16 key columns each
constexpr int NUM_THREADS = 32 * (4 + TW);  // + TMA k / v producers, score-MMA and t.v-MMA issuers

#ifdef TESM_GTC_TRACE
// Development-only timeline of CTA 0 (heaviest tile): clock64 at 8 points for each key block.
__device__ unsigned long long g_gtc_trace[8 * 256];
#define GTC_MARK(pt, j) \
  do {                  \
    if (blockIdx.x == 0 && (j) < 256) g_gtc_trace[(pt) * 256 + (j)] = clock64(); \
  } while (0)
#else
#define GTC_MARK(pt, j) \
  do {                  \
  } while (0)
#endif

struct Params {
  int B, L, D, DS, nqt, nkb_max;
  const float *relb;    // (2L - 1), index i - j + L - 1
  const float *states;  // (B*L, D) fp32
  float thr, es, inv_sqrt_r;  // scores use q.k * fp32(1/sqrt(R)): within an ulp of q.k / sqrt(R)
  void *out_tanh, *out_chg;
  int out_dtype;
};

// kind::f16 instruction descriptor: D f32, A/B f16, both K-major, M=128, N=n.
__host__ __device__ constexpr uint32_t idesc_f16(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(QT >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// A operand from TMEM: [a_tmem] holds the M x 16 fp16 slice (lane = row, 8 columns of packed pairs).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

// TMEM columns: accumulator O, score buffers S0/S1, q hi / lo (A of the score MMAs), ternary
// tiles T0/T1 (A of the t.v^T MMAs); fp16 operands pack two values per 32-bit column.
constexpr uint32_t COL_O = 0, COL_S = 256, COL_QH = 384, COL_QL = 416, COL_T = 448;

__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_global_ent_tc(const __grid_constant__ CUtensorMap tmKh, const __grid_constant__ CUtensorMap tmKl,
                    const __grid_constant__ CUtensorMap tmVh, const __grid_constant__ CUtensorMap tmVl,
                    const __half *__restrict__ qh_g, const __half *__restrict__ ql_g, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  constexpr int K_BYTES = KB * RP * 2;   // 8 KB per hi / lo
  const int V_BYTES = p.DS * KB * 2;     // <= 32 KB per hi / lo
  uint8_t *sK = smem;                         // NSK x [hi | lo]
  uint8_t *sV = sK + NSK * 2 * K_BYTES;       // NSV x [hi | lo]
  uint64_t *bars = reinterpret_cast<uint64_t *>(sV + NSV * 2 * V_BYTES);
  uint64_t *qready = bars, *kfull = bars + 1, *kempty = kfull + NSK, *vfull = kempty + NSK, *vempty = vfull + NSV,
           *sfull = vempty + NSV, *sfree = sfull + 2, *tready = sfree + 2, *tfree = tready + 2, *ofull = tfree + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(ofull + 1);
  float *cnt_s = reinterpret_cast<float *>(bars + 32);  // [4][QT]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = p.nqt - 1 - (int)(blockIdx.x / p.B), b = (int)(blockIdx.x % p.B);
  const int q0 = qt * QT;
  const int nkb = (min(q0 + QT, p.L) + KB - 1) / KB;
  const int64_t rowq = (int64_t)b * p.L;

  if (threadIdx.x == 0) {
    mbar_init(qready, TW);
    for (int i = 0; i < NSK; ++i) {
      mbar_init(&kfull[i], 1);
      mbar_init(&kempty[i], 1);
    }
    for (int i = 0; i < NSV; ++i) {
      mbar_init(&vfull[i], 1);
      mbar_init(&vempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&sfree[i], TW);
      mbar_init(&tready[i], TW);
      mbar_init(&tfree[i], 1);
    }
    mbar_init(ofull, 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // the k ring
      for (int j = 0; j < nkb; ++j) {
        const int s = j % NSK;
        if (!mbar_wait(&kempty[s], ((j / NSK) & 1) ^ 1)) break;
        mbar_expect_tx(&kfull[s], 2 * K_BYTES);
        uint8_t *k = sK + s * 2 * K_BYTES;
        tma_load_2d(k, &tmKh, &kfull[s], 0, (int)(rowq + j * KB));
        tma_load_2d(k + K_BYTES, &tmKl, &kfull[s], 0, (int)(rowq + j * KB));
      }
    }
  } else if (warp == 2 + TW) {
    if (lane == 0) {  // the v^T ring
      for (int j = 0; j < nkb; ++j) {
        const int s = j % NSV;
        if (!mbar_wait(&vempty[s], ((j / NSV) & 1) ^ 1)) break;
        mbar_expect_tx(&vfull[s], 2 * V_BYTES);
        tma_load_2d(sV + s * 2 * V_BYTES, &tmVh, &vfull[s], j * KB, b * p.DS);
        tma_load_2d(sV + s * 2 * V_BYTES + V_BYTES, &tmVl, &vfull[s], j * KB, b * p.DS);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // score MMAs, running ahead of the ternary pass by one buffer
      constexpr uint32_t idS = idesc_f16(KB);
      bool ok = mbar_wait(qready, 0);
      fence_after();
      for (int j = 0; ok && j < nkb; ++j) {
        const int s = j % NSK, bs = j & 1;
        if (!mbar_wait(&kfull[s], (j / NSK) & 1)) break;
        // S[bs] was read (tcgen05.ld) by the ternary pass of block j - 2
        if (j >= 2 && !mbar_wait(&sfree[bs], ((j - 2) >> 1) & 1)) break;
        GTC_MARK(0, j);
        fence_after();
        const uint64_t kh = smem_desc_sw128(sK + s * 2 * K_BYTES), kl = smem_desc_sw128(sK + s * 2 * K_BYTES + K_BYTES);
        const uint32_t dS = tmem + COL_S + bs * KB;
#pragma unroll
        for (int kk = 0; kk < RP / 16; ++kk) {  // 16 fp16 per K step: +8 TMEM columns, +2 descriptor units
          mma_f16_ts(dS, tmem + COL_QH + 8 * kk, kh + 2 * kk, idS, kk > 0);
          mma_f16_ts(dS, tmem + COL_QH + 8 * kk, kl + 2 * kk, idS, 1);
          mma_f16_ts(dS, tmem + COL_QL + 8 * kk, kh + 2 * kk, idS, 1);
        }
        commit(&kempty[s]);
        commit(&sfull[bs]);
        GTC_MARK(7, j);
      }
    }
  } else if (warp == 3 + TW) {
    if (lane == 0) {  // t.v^T MMAs into the accumulator
      const uint32_t idO = idesc_f16(p.DS);
      for (int j = 0; j < nkb; ++j) {
        const int sv = j % NSV, bt = j & 1;
        if (!mbar_wait(&tready[bt], (j >> 1) & 1)) break;
        GTC_MARK(1, j);
        if (!mbar_wait(&vfull[sv], (j / NSV) & 1)) break;
        GTC_MARK(2, j);
        fence_after();
        const uint64_t vh = smem_desc_sw128(sV + sv * 2 * V_BYTES), vl = smem_desc_sw128(sV + sv * 2 * V_BYTES + V_BYTES);
        const uint32_t ta = tmem + COL_T + bt * (KB / 2);
#pragma unroll
        for (int kk = 0; kk < KB / 16; ++kk) {
          mma_f16_ts(tmem + COL_O, ta + 8 * kk, vh + 2 * kk, idO, (j | kk) != 0);
          mma_f16_ts(tmem + COL_O, ta + 8 * kk, vl + 2 * kk, idO, 1);
        }
        commit(&vempty[sv]);
        commit(&tfree[bt]);
      }
      commit(ofull);
    }
  } else {
    // ternary warps 2 .. 2+TW-1 (warps 0, 1, 2+TW, 3+TW are the producers and MMA issuers): a warp reaches only TMEM lanes 32*(warp % 4) .. +31, so its lane
    // quarter is q = warp % 4; part = which 16 of the block's 64 key columns it handles
    const int tw = warp - 2, q = warp & 3, part = tw >> 2;
    const int rl = q * 32 + lane, i = q0 + rl;
    const bool row_ok = i < p.L;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    {  // q hi / lo of this row into TMEM: this part's 16 of the 64 values (8 columns each)
      uint32_t vh[8], vl[8];
      const int64_t qrow = rowq + min(i, p.L - 1);
      const uint4 *gh = reinterpret_cast<const uint4 *>(qh_g + qrow * RP + part * 16);
      const uint4 *gl = reinterpret_cast<const uint4 *>(ql_g + qrow * RP + part * 16);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const uint4 h = gh[u], l = gl[u];
        vh[4 * u] = h.x, vh[4 * u + 1] = h.y, vh[4 * u + 2] = h.z, vh[4 * u + 3] = h.w;
        vl[4 * u] = l.x, vl[4 * u + 1] = l.y, vl[4 * u + 2] = l.z, vl[4 * u + 3] = l.w;
      }
      tmem_st8(lane_base + COL_QH + part * 8, vh);
      tmem_st8(lane_base + COL_QL + part * 8, vl);
      asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(qready);
    }
    // relb[i - key + L - 1] for this lane's row and its 16 keys of a block: 16 consecutive
    // entries (descending), loaded one block ahead; clamped indices are used only where
    // key > i or i >= L, where the score is masked.
    const int top = 2 * p.L - 2;
    auto load_relb = [&](int jj, float (&rb)[16]) {
      const int x0 = i - (jj * KB + part * 16) + p.L - 1;
#pragma unroll
      for (int c = 0; c < 16; ++c) rb[c] = __ldg(&p.relb[min(max(x0 - c, 0), top)]);
    };
    float rb[16], rbn[16];
    load_relb(0, rbn);
    const uint32_t sgn_one = 0x3f800000u;
    float cnt = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      const int bt = j & 1;
      const int key0 = j * KB + part * 16;
#pragma unroll
      for (int c = 0; c < 16; ++c) rb[c] = rbn[c];
      if (j + 1 < nkb) load_relb(j + 1, rbn);
      if (!mbar_wait(&sfull[bt], (j >> 1) & 1)) {
        ok = false;
        break;
      }
      if (tw == 0 && lane == 0) GTC_MARK(3, j);
      fence_after();
      uint32_t r[16];
      tmem_ld16(lane_base + COL_S + bt * KB + part * 16, r);
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfree[bt]);  // the score MMAs may refill this buffer
      // whole warp strictly below the diagonal and inside the sequence: no per-score mask
      const bool dense = key0 + 15 <= q0 + q * 32 && q0 + q * 32 + 31 < p.L;
      uint32_t packed[8];
#pragma unroll
      for (int c = 0; c < 16; c += 2) {
        float tv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float sc = fmaf(__uint_as_float(r[c + e]), p.inv_sqrt_r, rb[c + e]);
          // t = sign(sc) where |sc| > thr, else 0
          float t = fabsf(sc) > p.thr ? __uint_as_float((__float_as_uint(sc) & 0x80000000u) | sgn_one) : 0.f;
          if (!dense && !(row_ok && key0 + c + e <= i)) t = 0.f;
          cnt = fmaf(t, t, cnt);
          tv[e] = t;
        }
        const __half2 h = __floats2half2_rn(tv[0], tv[1]);
        packed[c >> 1] = *reinterpret_cast<const uint32_t *>(&h);
      }
      if (tw == 0 && lane == 0) GTC_MARK(4, j);
      // the t.v^T MMA of block j - 2 has finished reading this buffer
      if (j >= 2 && !mbar_wait(&tfree[bt], ((j - 2) >> 1) & 1)) {
        ok = false;
        break;
      }
      if (tw == 0 && lane == 0) GTC_MARK(5, j);
      fence_after();
      tmem_st8(lane_base + COL_T + bt * (KB / 2) + part * 8, packed);
      asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tready[bt]);
      if (tw == 0 && lane == 0) GTC_MARK(6, j);
    }
    // the row's count is split over its 4 column parts
    cnt_s[part * QT + rl] = cnt;
    asm volatile("bar.sync 1, %0;\n" ::"n"(32 * TW) : "memory");  // the ternary warps
    const float denom = fmaxf(cnt_s[rl] + cnt_s[QT + rl] + cnt_s[2 * QT + rl] + cnt_s[3 * QT + rl], 1.f);
    if (ok && mbar_wait(ofull, 0)) {
      fence_after();
      const int nch = (p.DS + 15) / 16;  // 16-column chunks; TMEM columns past DS are allocated, unused
      const int64_t row = rowq + i;
      for (int ch = part; ch < nch; ch += 4) {
        uint32_t r[16];
        tmem_ld16(lane_base + COL_O + ch * 16, r);
        if (!row_ok) continue;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int d = ch * 16 + c;
          if (d >= p.D) continue;
          const float s = p.states[row * p.D + d];
          const float avg = __uint_as_float(r[c]) / denom;
          const float ent = s + p.es * (avg - s);
          store_f(p.out_tanh, p.out_dtype, row * p.D + d, tanhf(ent));
          store_f(p.out_chg, p.out_dtype, row * p.D + d, ent - s);
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(512));
  }
}

// q (RoPE + cross-layer bias) and k (RoPE) of every row as fp16 hi / lo, zero-padded to RP columns.
__global__ void k_gtc_prep_qk(ProjCols pc, const float *cross, int64_t M, int L, int R, const __grid_constant__ RopeTab rt, __half *qh,
                              __half *ql, __half *kh, __half *kl) {
  __shared__ float sq[8][RP], sk[8][RP];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + w;
  if (row >= M) return;
  const int t = (int)(row % L);
  load_rope_row(sq[w], pc, pc.c_q, row, R, t, rt.v, cross ? cross + row * R : nullptr, lane, 32);
  load_rope_row(sk[w], pc, pc.c_k, row, R, t, rt.v, nullptr, lane, 32);
  __syncwarp();
  for (int c = lane; c < RP; c += 32) {
    const float x = c < R ? sq[w][c] : 0.f, y = c < R ? sk[w][c] : 0.f;
    const __half xh = __float2half_rn(x), yh = __float2half_rn(y);
    qh[row * RP + c] = xh;
    ql[row * RP + c] = __float2half_rn(x - __half2float(xh));
    kh[row * RP + c] = yh;
    kl[row * RP + c] = __float2half_rn(y - __half2float(yh));
  }
}

// states (B*L, D) fp32 -> v^T (B*DS, Lp) as fp16 hi / lo, zero where d >= D or t >= L.
__global__ void k_gtc_prep_v(const float *states, int L, int D, int DS, int Lp, __half *vh, __half *vl) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z, t0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  for (int k = ty; k < 32; k += 8) {
    const int t = t0 + k, d = d0 + tx;
    tile[k][tx] = (t < L && d < D) ? states[((int64_t)b * L + t) * D + d] : 0.f;
  }
  __syncthreads();
  for (int k = ty; k < 32; k += 8) {
    const int d = d0 + k, t = t0 + tx;
    if (d < DS && t < Lp) {
      const float x = tile[tx][k];
      const __half h = __float2half_rn(x);
      vh[((int64_t)b * DS + d) * Lp + t] = h;
      vl[((int64_t)b * DS + d) * Lp + t] = __float2half_rn(x - __half2float(h));
    }
  }
}

static int make_map_f16(CUtensorMap *map, const void *ptr, int64_t inner, int64_t outer, int box_inner,
                        int box_outer) {
  auto fn = tc::encode_fn();
  if (!fn) return fail(TESM_ELAUNCH, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(inner * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TESM_EINVAL, "global_ent_tc: tensor map (" + std::to_string((int)r) + ")");
  return TESM_OK;
}

struct Layout {
  int64_t qk_bytes, vt_bytes, total;
  int DS, Lp;
};

static Layout layout(int64_t B, int64_t L, int64_t D) {
  Layout l;
  l.DS = (int)round_up(D, 16);
  l.Lp = (int)round_up(L, 64);
  l.qk_bytes = round_up(B * L * RP * 2, 1024);
  l.vt_bytes = round_up(B * l.DS * (int64_t)l.Lp * 2, 1024);
  l.total = 4 * l.qk_bytes + 2 * l.vt_bytes;
  return l;
}

}  // namespace gtc
}  // namespace tesm

using namespace tesm;

#ifdef TESM_GTC_TRACE
extern "C" int tesm_b200_gtc_trace_read(unsigned long long *host) {
  return cudaMemcpyFromSymbol(host, gtc::g_gtc_trace, sizeof(gtc::g_gtc_trace)) == cudaSuccess ? 0 : 3;
}
#endif

extern "C" int tesm_b200_global_ent_tc_workspace(int64_t B, int64_t L, int64_t D, int64_t R, int64_t *bytes) {
  TESM_REQUIRE(bytes && B > 0 && L > 0 && D > 0 && R > 0, "global_ent_tc_workspace: bad argument");
  if (R > gtc::RP || D > 256 || R % 2)
    return fail(TESM_EUNSUPPORTED, "global_ent_tc: needs ent_rank <= 64 (even) and d_state <= 256");
  *bytes = gtc::layout(B, L, D).total;
  return TESM_OK;
}

extern "C" int tesm_b200_siso_global_ent_tc(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L,
                                            int64_t Dm, int64_t D, int64_t R, const float *cross, const float *relb,
                                            const float *states, float thr, float es, float rope_base, void *out_tanh,
                                            void *out_chg, int out_dtype, void *workspace, int64_t ws_bytes,
                                            tesm_stream_t stream) {
  TESM_REQUIRE(proj && relb && states && out_tanh && out_chg && workspace, "global_ent_tc: null pointer");
  TESM_REQUIRE(B > 0 && L > 0 && D > 0 && R > 0 && R % 2 == 0, "global_ent_tc: bad shape");
  TESM_REQUIRE(B * L < (1ll << 31), "global_ent_tc: too many rows");
  if (R > gtc::RP || D > 256) return fail(TESM_EUNSUPPORTED, "global_ent_tc: needs ent_rank <= 64 and d_state <= 256");
  if (dtype != TESM_F32 && dtype != TESM_BF16) return fail(TESM_EDTYPE, "global_ent_tc: proj dtype");
  if (out_dtype != TESM_F32 && out_dtype != TESM_BF16) return fail(TESM_EDTYPE, "global_ent_tc: out dtype");
  const gtc::Layout lay = gtc::layout(B, L, D);
  TESM_REQUIRE(ws_bytes >= lay.total && ((uintptr_t)workspace & 1023) == 0,
               "global_ent_tc: workspace too small or not 1024-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t *ws = reinterpret_cast<uint8_t *>(workspace);
  __half *qh = reinterpret_cast<__half *>(ws), *ql = reinterpret_cast<__half *>(ws + lay.qk_bytes),
         *kh = reinterpret_cast<__half *>(ws + 2 * lay.qk_bytes), *kl = reinterpret_cast<__half *>(ws + 3 * lay.qk_bytes),
         *vth = reinterpret_cast<__half *>(ws + 4 * lay.qk_bytes),
         *vtl = reinterpret_cast<__half *>(ws + 4 * lay.qk_bytes + lay.vt_bytes);
  const int64_t M = B * L;
  ProjCols pc = make_cols(proj, dtype, ldp, (int)Dm, (int)D, (int)R);
  gtc::k_gtc_prep_qk<<<(unsigned)ceil_div(M, 8), 256, 0, st>>>(pc, cross, M, (int)L, (int)R, rope_table((int)R, rope_base), qh, ql, kh,
                                                               kl);
  int rc = check_launch("global_ent_tc prep q/k");
  if (rc) return rc;
  dim3 gv((unsigned)ceil_div(lay.Lp, 32), (unsigned)ceil_div(lay.DS, 32), (unsigned)B);
  gtc::k_gtc_prep_v<<<gv, 256, 0, st>>>(states, (int)L, (int)D, lay.DS, lay.Lp, vth, vtl);
  if ((rc = check_launch("global_ent_tc prep v"))) return rc;

  CUtensorMap mkh, mkl, mvh, mvl;
  if ((rc = gtc::make_map_f16(&mkh, kh, gtc::RP, M, gtc::RP, gtc::KB))) return rc;
  if ((rc = gtc::make_map_f16(&mkl, kl, gtc::RP, M, gtc::RP, gtc::KB))) return rc;
  if ((rc = gtc::make_map_f16(&mvh, vth, lay.Lp, B * lay.DS, gtc::KB, lay.DS))) return rc;
  if ((rc = gtc::make_map_f16(&mvl, vtl, lay.Lp, B * lay.DS, gtc::KB, lay.DS))) return rc;

  gtc::Params p;
  p.B = (int)B;
  p.L = (int)L;
  p.D = (int)D;
  p.DS = lay.DS;
  p.nqt = (int)ceil_div(L, gtc::QT);
  p.nkb_max = (int)ceil_div(L, gtc::KB);
  p.relb = relb;
  p.states = states;
  p.thr = thr;
  p.es = es;
  p.inv_sqrt_r = (float)(1.0 / sqrt((double)R));
  p.out_tanh = out_tanh;
  p.out_chg = out_chg;
  p.out_dtype = out_dtype;
  const size_t smem = 1024 + gtc::NSK * 2 * (size_t)gtc::KB * gtc::RP * 2 + gtc::NSV * 2 * (size_t)lay.DS * gtc::KB * 2 +
                      256 + 4 * gtc::QT * sizeof(float);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gtc::k_global_ent_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    attr = true;
  }
  TESM_REQUIRE(smem <= 227 * 1024, "global_ent_tc: shared memory");
  gtc::k_global_ent_tc<<<(unsigned)(B * p.nqt), gtc::NUM_THREADS, smem, st>>>(mkh, mkl, mvh, mvl, qh, ql, p);
  return check_launch("global_ent_tc");
}
