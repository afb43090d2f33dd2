// Decode-shaped INT2 x INT8 GEMV (M <= 64 tokens) straight from the packed ternary bytes.
//
// Design (HBM-bound: every packed weight byte is read once):
//  * swap-AB on the warp-level int8 MMA (m16n8k32): the MMA "M" is 16 weight rows, "N" is
//    8 tokens, so a single token still fills 1/8 of each MMA and the weights never touch
//    shared memory.
//  * the 2-bit codes are used unshifted (c = t + 1 in {0,1,2}); the exact integer result is
//    recovered as sum c*x - sum x, with sum x (rowsum) produced by the quantisation kernel.
//    Spreading one 32-bit word of 16 codes into four int8x4 registers costs a shift and a
//    mask per register; the activation codes are stored pre-permuted (TESM_LAYOUT_GEMV) so
//    that the k-order the spread produces matches the B fragment.
//  * one CTA per 16 weight rows over the whole K; its warps split K into contiguous ranges and
//    the int32 partial tiles are summed in shared memory in a fixed order (deterministic, no
//    global scratch, no cluster barriers).
#include "common.cuh"

namespace tesm {

struct GemvParams {
  const int8_t *codes;
  int64_t ld_codes;
  const float *inv_scale;
  const int32_t *rowsum;
  const uint8_t *packed;
  int64_t ld_packed;
  const float *w_deq;
  int per_row;
  int M, N;
  int steps_total;  // K rounded up to 256, divided by 256
  void *out;
  int out_dtype;
  int64_t ldo;
  int32_t *acc_out;
  int64_t ld_acc;
};


__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Row-block GEMV: one CTA per 16 weight rows over the whole K, its WPC warps splitting K into
// contiguous step ranges (a step = 256 columns); partial 16 x TOK tiles are summed in shared
// memory.  No cluster barriers on the critical path: every weight byte of the CTA is requested
// before the activation wait, and the activation fragments are read straight from L2 (every
// CTA reads the same few KB of codes).
template <int NT, int WPC, int PF>
__global__ void __launch_bounds__(WPC * 32, (NT >= 4 ? 1 : NT == 2 ? (WPC == 8 ? 3 : 1) : (WPC == 8 ? 5 : 2))) k_gemv_rows(GemvParams p) {
  constexpr int TOK = NT * 8;
  __shared__ int32_t red[WPC][16][TOK + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int row0 = blockIdx.x * 16;
  pdl_trigger();
  const int rA = min(row0 + g, p.N - 1), rB = min(row0 + g + 8, p.N - 1);
  const int spw = (p.steps_total + WPC - 1) / WPC;  // steps per warp
  const int s_begin = warp * spw, s_end = min(s_begin + spw, p.steps_total);
  const int nsteps = max(s_end - s_begin, 0);
  const uint8_t *wA = p.packed + (int64_t)rA * p.ld_packed + (int64_t)s_begin * 64 + tig * 16;
  const uint8_t *wB = p.packed + (int64_t)rB * p.ld_packed + (int64_t)s_begin * 64 + tig * 16;
  uint4 bufA[PF], bufB[PF];
#pragma unroll
  for (int i = 0; i < PF; ++i)
    if (i < nsteps) {
      bufA[i] = ldg_nc_v4(wA + i * 64);
      bufB[i] = ldg_nc_v4(wB + i * 64);
    }
  // programmatic stream serialization: the weight requests above overlap the tail of the
  // quantisation kernel; wait for its codes before reading them
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  const int8_t *xrow[NT];
  bool xok[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int tok = t * 8 + g;
    xok[t] = tok < p.M;
    xrow[t] = p.codes + (int64_t)(xok[t] ? tok : 0) * p.ld_codes + (int64_t)s_begin * 256 + tig * 16;
  }
  int acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0;
  for (int s0 = 0; s0 < nsteps; s0 += PF) {
#pragma unroll
    for (int i = 0; i < PF; ++i) {
      const int s = s0 + i;
      if (s < nsteps) {
        uint4 xv[NT][4];
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int u = 0; u < 4; ++u)
            xv[t][u] = xok[t] ? *reinterpret_cast<const uint4 *>(xrow[t] + s * 256 + u * 64) : make_uint4(0, 0, 0, 0);
        const uint4 A4 = bufA[i], B4 = bufB[i];
        if (s + PF < nsteps) {
          bufA[i] = ldg_nc_v4(wA + (s + PF) * 64);
          bufB[i] = ldg_nc_v4(wB + (s + PF) * 64);
        }
        const uint32_t wa[4] = {A4.x, A4.y, A4.z, A4.w};
        const uint32_t wb[4] = {B4.x, B4.y, B4.z, B4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint32_t ra[4], rb[4];
#pragma unroll
          for (int sw = 0; sw < 4; ++sw) {
            ra[sw] = (wa[u] >> (2 * sw)) & 0x03030303u;
            rb[sw] = (wb[u] >> (2 * sw)) & 0x03030303u;
          }
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            mma_s8(acc[t], ra[0], rb[0], ra[1], rb[1], xv[t][u].x, xv[t][u].y);
            mma_s8(acc[t], ra[2], rb[2], ra[3], rb[3], xv[t][u].z, xv[t][u].w);
          }
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    red[warp][g][t * 8 + tig * 2] = acc[t][0];
    red[warp][g][t * 8 + tig * 2 + 1] = acc[t][1];
    red[warp][g + 8][t * 8 + tig * 2] = acc[t][2];
    red[warp][g + 8][t * 8 + tig * 2 + 1] = acc[t][3];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 16 * TOK; i += WPC * 32) {
    const int r = i / TOK, tok = i - r * TOK;
    const int n = row0 + r;
    if (tok >= p.M || n >= p.N) continue;
    int32_t sum = 0;
#pragma unroll
    for (int w = 0; w < WPC; ++w) sum += red[w][r][tok];
    const int32_t a = sum - p.rowsum[tok];
    const float wd = p.per_row ? p.w_deq[n] : p.w_deq[0];
    store_f(p.out, p.out_dtype, (int64_t)tok * p.ldo + n, (float)a * p.inv_scale[tok] * wd);
    if (p.acc_out) p.acc_out[(int64_t)tok * p.ld_acc + n] = a;
  }
}

template <int NT, int WPC, int PF>
static int launch_gemv_rows(const GemvParams &p, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ceil_div(p.N, 16), 1, 1);
  cfg.blockDim = dim3(WPC * 32, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see griddepcontrol.wait
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  // the GEMV follows its activation quantiser: launched programmatically it requests every weight
  // byte of its rows while the quantiser runs (TESM_GEMV_PDL=0 turns this off)
  static const int gemv_pdl = [] {
    const char *e = getenv("TESM_GEMV_PDL");
    return e ? atoi(e) : 1;
  }();
  cfg.numAttrs = (gemv_pdl || pdl_enabled()) ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemv_rows<NT, WPC, PF>, p);
  if (e != cudaSuccess) return fail(TESM_ELAUNCH, std::string("gemv_int2 launch: ") + cudaGetErrorString(e));
  return TESM_OK;
}

// Warps per CTA for M <= 16: short K (<= 16 steps of 256) -> 8 warps of <= 2 steps with a
// small register budget, so the whole grid is resident in one wave; longer K -> 16 warps.
static bool gemv_wide(const GemvParams &p) {
  static int wpc_force = -1;
  if (wpc_force < 0) {
    const char *e = getenv("TESM_GEMV_WPC");  // tuning override: 8 or 16
    wpc_force = e ? atoi(e) : 0;
  }
  return wpc_force ? wpc_force == 16 : p.steps_total > 16;
}

}  // namespace tesm

using namespace tesm;

extern "C" int tesm_b200_gemv_int2(const int8_t *codes, int64_t ld_codes, const float *inv_scale,
                                   const int32_t *rowsum, const uint8_t *packed, int64_t ld_packed,
                                   const float *w_deq, int per_row, int64_t M, int64_t N, int64_t K, void *out,
                                   int out_dtype, int64_t ldo, int32_t *acc_out, int64_t ld_acc,
                                   tesm_stream_t stream) {
  if (M == 0) return TESM_OK;  // empty batch: nothing to do (its buffers may be null)
  TESM_REQUIRE(codes && inv_scale && rowsum && packed && w_deq && out, "gemv_int2: null pointer");
  TESM_REQUIRE(M > 0 && M <= 64 && N > 0 && K > 0, "gemv_int2: need 0 <= M <= 64, N > 0, K > 0");
  TESM_REQUIRE(N < (1ll << 31), "gemv_int2: N too large");
  if (out_dtype != TESM_F32 && out_dtype != TESM_BF16) return fail(TESM_EDTYPE, "gemv_int2: out dtype");
  const int64_t Kp = round_up(K, 256);
  TESM_REQUIRE(ld_codes >= Kp && ld_codes % 16 == 0 && ((uintptr_t)codes & 15) == 0,
               "gemv_int2: codes must be GEMV layout with ld_codes >= K rounded up to 256, 16-byte aligned");
  TESM_REQUIRE(ld_packed >= Kp / 4 && ld_packed % 16 == 0 && ((uintptr_t)packed & 15) == 0,
               "gemv_int2: packed rows must hold K rounded up to 256 codes, 16-byte aligned");
  TESM_REQUIRE(ldo >= N, "gemv_int2: ldo < N");
  GemvParams p = {};
  p.codes = codes;
  p.ld_codes = ld_codes;
  p.inv_scale = inv_scale;
  p.rowsum = rowsum;
  p.packed = packed;
  p.ld_packed = ld_packed;
  p.w_deq = w_deq;
  p.per_row = per_row;
  p.M = (int)M;
  p.N = (int)N;
  p.out = out;
  p.out_dtype = out_dtype;
  p.ldo = ldo;
  p.acc_out = acc_out;
  p.ld_acc = ld_acc;
  p.steps_total = (int)(Kp / 256);
  cudaStream_t st = (cudaStream_t)stream;
  const bool wide = gemv_wide(p);
  if (M <= 8) return wide ? launch_gemv_rows<1, 16, 4>(p, st) : launch_gemv_rows<1, 8, 2>(p, st);
  if (M <= 16) return wide ? launch_gemv_rows<2, 16, 4>(p, st) : launch_gemv_rows<2, 8, 4>(p, st);
  if (M <= 32) return launch_gemv_rows<4, 8, 4>(p, st);
  return launch_gemv_rows<8, 8, 4>(p, st);
}
