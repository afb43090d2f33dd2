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
// Kernel: one CTA per (batch, 128-query tile), heaviest tiles first.  Warp 0 streams the k and
// v^T tiles of 64 keys through a 2-stage TMA ring, warp 1 issues the MMAs, warps 2..9 (two per
// TMEM lane quarter, one half of the 64 key columns each) turn scores into ternaries written
// straight into the shared-memory A operand of the t.v^T MMA, then run the epilogue.  Scores are
// double-buffered in TMEM (2 x 64 columns) next to the (128 x DS) fp32 accumulator, so the
// score MMA of block j+1 overlaps the ternary pass of block j.  Every wait is bounded.

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
constexpr int NS = 2;    // k / v^T ring stages
constexpr int NUM_THREADS = 64 + 256;

struct Params {
  int B, L, D, DS, nqt, nkb_max;
  const float *relb;    // (2L - 1), index i - j + L - 1
  const float *states;  // (B*L, D) fp32
  float thr, es, sqrt_r;
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

__global__ void __launch_bounds__(NUM_THREADS, 1)
    k_global_ent_tc(const __grid_constant__ CUtensorMap tmQh, const __grid_constant__ CUtensorMap tmQl,
                    const __grid_constant__ CUtensorMap tmKh, const __grid_constant__ CUtensorMap tmKl,
                    const __grid_constant__ CUtensorMap tmVh, const __grid_constant__ CUtensorMap tmVl, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  constexpr int Q_BYTES = QT * RP * 2;   // 16 KB per hi / lo
  constexpr int K_BYTES = KB * RP * 2;   // 8 KB per hi / lo
  constexpr int T_BYTES = QT * KB * 2;   // 16 KB
  const int V_BYTES = p.DS * KB * 2;     // <= 32 KB per hi / lo
  uint8_t *sQ = smem;                         // [hi | lo]
  uint8_t *sK = sQ + 2 * Q_BYTES;             // NS x [hi | lo]
  uint8_t *sT = sK + NS * 2 * K_BYTES;        // 2 x T
  uint8_t *sV = sT + 2 * T_BYTES;             // NS x [hi | lo]
  uint64_t *bars = reinterpret_cast<uint64_t *>(sV + NS * 2 * V_BYTES);
  uint64_t *qfull = bars, *kvfull = bars + 1, *kvempty = kvfull + NS, *sfull = kvempty + NS, *tready = sfull + 2,
           *tfree = tready + 2, *ofull = tfree + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(ofull + 1);
  float *cnt_s = reinterpret_cast<float *>(tmem_slot + 4);  // [2][QT]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = p.nqt - 1 - (int)(blockIdx.x / p.B), b = (int)(blockIdx.x % p.B);
  const int q0 = qt * QT;
  const int nkb = (min(q0 + QT, p.L) + KB - 1) / KB;
  const int64_t rowq = (int64_t)b * p.L;

  if (threadIdx.x == 0) {
    mbar_init(qfull, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&kvfull[i], 1);
      mbar_init(&kvempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&tready[i], 8);
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
  const uint32_t tmem = *tmem_slot;  // S[0] cols 0..63, S[1] 64..127, O 128..128+DS

  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(qfull, 2 * Q_BYTES);
      tma_load_2d(sQ, &tmQh, qfull, 0, (int)(rowq + q0));
      tma_load_2d(sQ + Q_BYTES, &tmQl, qfull, 0, (int)(rowq + q0));
      for (int j = 0; j < nkb; ++j) {
        const int s = j % NS;
        if (!mbar_wait(&kvempty[s], ((j / NS) & 1) ^ 1)) break;
        mbar_expect_tx(&kvfull[s], 2 * K_BYTES + 2 * V_BYTES);
        uint8_t *k = sK + s * 2 * K_BYTES;
        tma_load_2d(k, &tmKh, &kvfull[s], 0, (int)(rowq + j * KB));
        tma_load_2d(k + K_BYTES, &tmKl, &kvfull[s], 0, (int)(rowq + j * KB));
        tma_load_2d(sV + s * 2 * V_BYTES, &tmVh, &kvfull[s], j * KB, b * p.DS);
        tma_load_2d(sV + s * 2 * V_BYTES + V_BYTES, &tmVl, &kvfull[s], j * KB, b * p.DS);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idS = idesc_f16(KB);
      const uint32_t idO = idesc_f16(p.DS);
      bool ok = mbar_wait(qfull, 0);
      fence_after();
      const uint64_t qh = smem_desc_sw128(sQ), ql = smem_desc_sw128(sQ + Q_BYTES);
      for (int j = 0; ok && j <= nkb; ++j) {
        if (j < nkb) {
          const int s = j % NS;
          if (!mbar_wait(&kvfull[s], (j / NS) & 1)) break;
          fence_after();
          const uint64_t kh = smem_desc_sw128(sK + s * 2 * K_BYTES), kl = smem_desc_sw128(sK + s * 2 * K_BYTES + K_BYTES);
          const uint32_t dS = tmem + (j & 1) * KB;
#pragma unroll
          for (int kk = 0; kk < RP / 16; ++kk) {  // 16 fp16 = 32 bytes per K step: +2 in 16-byte units
            mma_f16(dS, qh + 2 * kk, kh + 2 * kk, idS, kk > 0);
            mma_f16(dS, qh + 2 * kk, kl + 2 * kk, idS, 1);
            mma_f16(dS, ql + 2 * kk, kh + 2 * kk, idS, 1);
          }
          commit(&sfull[j & 1]);
        }
        if (j >= 1) {
          const int jp = j - 1, bp = jp & 1, sp = jp % NS;
          if (!mbar_wait(&tready[bp], (jp >> 1) & 1)) break;
          fence_after();
          const uint64_t ta = smem_desc_sw128(sT + bp * T_BYTES), vh = smem_desc_sw128(sV + sp * 2 * V_BYTES),
                         vl = smem_desc_sw128(sV + sp * 2 * V_BYTES + V_BYTES);
#pragma unroll
          for (int kk = 0; kk < KB / 16; ++kk) {
            mma_f16(tmem + 2 * KB, ta + 2 * kk, vh + 2 * kk, idO, (jp | kk) != 0);
            mma_f16(tmem + 2 * KB, ta + 2 * kk, vl + 2 * kk, idO, 1);
          }
          commit(&kvempty[sp]);
          commit(&tfree[bp]);
        }
      }
      commit(ofull);
    }
  } else {
    // ternary warps: TMEM lane quarter q, key columns [half*32, half*32+32) of each block
    const int q = warp & 3, half = (warp - 2) >> 2;
    const int rl = q * 32 + lane, i = q0 + rl;
    const bool row_ok = i < p.L;
    float cnt = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      const int buf = j & 1;
      if (!mbar_wait(&sfull[buf], (j >> 1) & 1)) {
        ok = false;
        break;
      }
      fence_after();
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + buf * KB + half * 32, r);
      if (j >= 2 && !mbar_wait(&tfree[buf], ((j - 2) >> 1) & 1)) {
        ok = false;
        break;
      }
      const int key0 = j * KB + half * 32;
      uint32_t packed[16];
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        float tv[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = key0 + c + e;
          float t = 0.f;
          if (row_ok && key <= i) {
            const float sc = __fdiv_rn(__uint_as_float(r[c + e]), p.sqrt_r) + __ldg(&p.relb[i - key + p.L - 1]);
            t = ternary_of(sc, p.thr);
          }
          cnt += fabsf(t);
          tv[e] = t;
        }
        const __half2 h = __floats2half2_rn(tv[0], tv[1]);
        packed[c >> 1] = *reinterpret_cast<const uint32_t *>(&h);
      }
      // row rl of the 128 x 64 fp16 tile (128-byte rows, 128-byte swizzle): 16-byte chunk u of
      // this half sits at chunk index (half*4 + u) ^ (rl & 7)
      uint8_t *trow = sT + buf * T_BYTES + rl * 128;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        *reinterpret_cast<uint4 *>(trow + (((half * 4 + u) ^ (rl & 7)) << 4)) =
            make_uint4(packed[4 * u], packed[4 * u + 1], packed[4 * u + 2], packed[4 * u + 3]);
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tready[buf]);
    }
    cnt_s[half * QT + rl] = cnt;
    asm volatile("bar.sync 1, 256;\n" ::: "memory");  // the eight ternary warps
    const float denom = fmaxf(cnt_s[rl] + cnt_s[QT + rl], 1.f);
    if (ok && mbar_wait(ofull, 0)) {
      fence_after();
      const int nch = (p.DS + 31) / 32;  // TMEM columns past DS are allocated, their values unused
      const int64_t row = rowq + i;
      for (int ch = half; ch < nch; ch += 2) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + 2 * KB + ch * 32, r);
        if (!row_ok) continue;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int d = ch * 32 + c;
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
__global__ void k_gtc_prep_qk(ProjCols pc, const float *cross, int64_t M, int L, int R, float base, __half *qh,
                              __half *ql, __half *kh, __half *kl) {
  __shared__ float sq[8][RP], sk[8][RP];
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + w;
  if (row >= M) return;
  const int t = (int)(row % L);
  load_rope_row(sq[w], pc, pc.c_q, row, R, t, base, cross ? cross + row * R : nullptr, lane, 32);
  load_rope_row(sk[w], pc, pc.c_k, row, R, t, base, nullptr, lane, 32);
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
  gtc::k_gtc_prep_qk<<<(unsigned)ceil_div(M, 8), 256, 0, st>>>(pc, cross, M, (int)L, (int)R, rope_base, qh, ql, kh,
                                                               kl);
  int rc = check_launch("global_ent_tc prep q/k");
  if (rc) return rc;
  dim3 gv((unsigned)ceil_div(lay.Lp, 32), (unsigned)ceil_div(lay.DS, 32), (unsigned)B);
  gtc::k_gtc_prep_v<<<gv, 256, 0, st>>>(states, (int)L, (int)D, lay.DS, lay.Lp, vth, vtl);
  if ((rc = check_launch("global_ent_tc prep v"))) return rc;

  CUtensorMap mqh, mql, mkh, mkl, mvh, mvl;
  if ((rc = gtc::make_map_f16(&mqh, qh, gtc::RP, M, gtc::RP, gtc::QT))) return rc;
  if ((rc = gtc::make_map_f16(&mql, ql, gtc::RP, M, gtc::RP, gtc::QT))) return rc;
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
  p.sqrt_r = (float)sqrt((double)R);
  p.out_tanh = out_tanh;
  p.out_chg = out_chg;
  p.out_dtype = out_dtype;
  const size_t smem = 1024 + 2 * (size_t)gtc::QT * gtc::RP * 2 + gtc::NS * 2 * (size_t)gtc::KB * gtc::RP * 2 +
                      2 * (size_t)gtc::QT * gtc::KB * 2 + gtc::NS * 2 * (size_t)lay.DS * gtc::KB * 2 + 256 +
                      2 * gtc::QT * sizeof(float);
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gtc::k_global_ent_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    attr = true;
  }
  TESM_REQUIRE(smem <= 227 * 1024, "global_ent_tc: shared memory");
  gtc::k_global_ent_tc<<<(unsigned)(B * p.nqt), gtc::NUM_THREADS, smem, st>>>(mqh, mql, mkh, mkl, mvh, mvl, p);
  return check_launch("global_ent_tc");
}
