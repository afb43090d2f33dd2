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
//  * split-K across a thread-block cluster (up to 8 CTAs) with the int32 partials reduced
//    through distributed shared memory: no global scratch, deterministic.
#include "common.cuh"

#include <cooperative_groups.h>

namespace cg = cooperative_groups;

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
  int steps_total;      // K rounded up to 256, divided by 256
  int steps_per_split;  // steps handled by one CTA of the cluster
  int split;            // cluster size along K (1, 2, 4, 8)
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

template <int NT>
__global__ void __launch_bounds__(256) k_gemv_int2(GemvParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int TOK = NT * 8;
  const int split_idx = blockIdx.y;
  const int s_begin = split_idx * p.steps_per_split;
  const int s_end = min(s_begin + p.steps_per_split, p.steps_total);
  const int nsteps = max(s_end - s_begin, 0);
  const int act_stride = nsteps * 256 + 64;  // +64: rows of one 8-lane phase hit different banks

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int row0 = blockIdx.x * 128 + warp * 16;
  const int rA = min(row0 + g, p.N - 1), rB = min(row0 + g + 8, p.N - 1);
  const uint8_t *wA = p.packed + (int64_t)rA * p.ld_packed + tig * 16;
  const uint8_t *wB = p.packed + (int64_t)rB * p.ld_packed + tig * 16;

  // weight prefetch first: it does not depend on the activations
  constexpr int PF = 4;  // prefetch depth in steps (2 x 16 B per step per thread)
  uint4 bufA[PF], bufB[PF];
#pragma unroll
  for (int i = 0; i < PF; ++i) {
    if (i < nsteps) {
      bufA[i] = ldg_nc_v4(wA + (int64_t)(s_begin + i) * 64);
      bufB[i] = ldg_nc_v4(wB + (int64_t)(s_begin + i) * 64);
    }
  }

  // Launched with programmatic stream serialization: the weight prefetch above overlaps the tail
  // of the quantisation kernel that produces the codes; wait for that grid (and its memory)
  // before touching them.  A no-op for an ordinary launch.
  asm volatile("griddepcontrol.wait;\n" ::: "memory");

  // ---- stage this CTA's K-slice of the activation codes in shared memory
  {
    const int chunks = nsteps * 16;  // 16-byte chunks per token row
    for (int i = threadIdx.x; i < TOK * chunks; i += blockDim.x) {
      const int tok = i / chunks, c = i - tok * chunks;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (tok < p.M)
        v = *reinterpret_cast<const uint4 *>(p.codes + (int64_t)tok * p.ld_codes + (int64_t)s_begin * 256 + c * 16);
      *reinterpret_cast<uint4 *>(smem + tok * act_stride + c * 16) = v;
    }
  }
  __syncthreads();

  int acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0;

  for (int s0 = 0; s0 < nsteps; s0 += PF) {
#pragma unroll
    for (int i = 0; i < PF; ++i) {
      const int s = s0 + i;
      if (s < nsteps) {
        const uint4 A4 = bufA[i], B4 = bufB[i];
        if (s + PF < nsteps) {
          bufA[i] = ldg_nc_v4(wA + (int64_t)(s_begin + s + PF) * 64);
          bufB[i] = ldg_nc_v4(wB + (int64_t)(s_begin + s + PF) * 64);
        }
        const uint32_t wa[4] = {A4.x, A4.y, A4.z, A4.w};
        const uint32_t wb[4] = {B4.x, B4.y, B4.z, B4.w};
        const uint8_t *arow = smem + s * 256 + tig * 16;
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
            const uint4 x = *reinterpret_cast<const uint4 *>(arow + (t * 8 + g) * act_stride + u * 64);
            mma_s8(acc[t], ra[0], rb[0], ra[1], rb[1], x.x, x.y);
            mma_s8(acc[t], ra[2], rb[2], ra[3], rb[3], x.z, x.w);
          }
        }
      }
    }
  }

  // ---- partial tile -> shared memory [128 rows][TOK+1] (reuses the activation buffer)
  __syncthreads();
  int32_t *red = reinterpret_cast<int32_t *>(smem);
  constexpr int RS = TOK + 1;
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const int lr = warp * 16 + g;
    red[lr * RS + t * 8 + tig * 2] = acc[t][0];
    red[lr * RS + t * 8 + tig * 2 + 1] = acc[t][1];
    red[(lr + 8) * RS + t * 8 + tig * 2] = acc[t][2];
    red[(lr + 8) * RS + t * 8 + tig * 2 + 1] = acc[t][3];
  }

  int r_begin = 0, r_count = 128;
  cg::cluster_group cluster = cg::this_cluster();
  if (p.split > 1) {
    cluster.sync();
    r_count = 128 / p.split;
    r_begin = (int)cluster.block_rank() * r_count;
  } else {
    __syncthreads();
  }
  const int items = r_count * TOK;
  for (int i = threadIdx.x; i < items; i += blockDim.x) {
    const int tok = i / r_count;
    const int lr = r_begin + (i - tok * r_count);
    int32_t sum = 0;
    if (p.split > 1) {
      for (int q = 0; q < p.split; ++q) {
        const int32_t *rq = cluster.map_shared_rank(red, q);
        sum += rq[lr * RS + tok];
      }
    } else {
      sum = red[lr * RS + tok];
    }
    const int n = blockIdx.x * 128 + lr;
    if (tok < p.M && n < p.N) {
      const int32_t a = sum - p.rowsum[tok];
      const float wd = p.per_row ? p.w_deq[n] : p.w_deq[0];
      const float v = (float)a * p.inv_scale[tok] * wd;
      store_f(p.out, p.out_dtype, (int64_t)tok * p.ldo + n, v);
      if (p.acc_out) p.acc_out[(int64_t)tok * p.ld_acc + n] = a;
    }
  }
  if (p.split > 1) cluster.sync();  // keep shared memory alive until every peer has read it
}

template <int NT>
static int launch_gemv(const GemvParams &p, cudaStream_t st) {
  const int act_stride = p.steps_per_split * 256 + 64;
  size_t smem = (size_t)NT * 8 * act_stride;
  const size_t red = (size_t)128 * (NT * 8 + 1) * 4;
  if (smem < red) smem = red;
  static bool attr_done = false;
  if (!attr_done) {
    cudaFuncSetAttribute(k_gemv_int2<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(k_gemv_int2<NT>, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
    attr_done = true;
  }
  if (smem > 200 * 1024) return fail(TESM_EUNSUPPORTED, "gemv_int2: K slice too large for shared memory");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ceil_div(p.N, 128), (unsigned)p.split, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = (unsigned)p.split;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see griddepcontrol.wait
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemv_int2<NT>, p);
  if (e != cudaSuccess) return fail(TESM_ELAUNCH, std::string("gemv_int2 launch: ") + cudaGetErrorString(e));
  return TESM_OK;
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
  GemvParams p;
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
  p.steps_total = (int)(Kp / 256);
  const int64_t rowblocks = ceil_div(N, 128);
  int split = 1;
  while (split < 8 && rowblocks * split < 2 * sm_count() && split * 2 <= p.steps_total) split *= 2;
  p.split = split;
  p.steps_per_split = (int)ceil_div(p.steps_total, split);
  p.out = out;
  p.out_dtype = out_dtype;
  p.ldo = ldo;
  p.acc_out = acc_out;
  p.ld_acc = ld_acc;
  cudaStream_t st = (cudaStream_t)stream;
  if (M <= 8) return launch_gemv<1>(p, st);
  if (M <= 16) return launch_gemv<2>(p, st);
  if (M <= 32) return launch_gemv<4>(p, st);
  return launch_gemv<8>(p, st);
}
