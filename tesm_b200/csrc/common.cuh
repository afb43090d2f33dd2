// Shared helpers for the tesm_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <cstdlib>
#include <string>

#include "../../include/tesm_b200.h"

namespace tesm {

// ------------------------------------------------------------ host-side errors
void set_error(const std::string &msg);
int fail(int code, const std::string &msg);
int check_launch(const char *what);

#define TESM_REQUIRE(cond, msg)                                   \
  do {                                                            \
    if (!(cond)) return ::tesm::fail(TESM_EINVAL, (msg));         \
  } while (0)

inline int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

inline int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }
inline int64_t ceil_div(int64_t x, int64_t m) { return (x + m - 1) / m; }

// ------------------------------------------------------------ device status
// Sticky word set by device code when a bounded wait gives up (TESM_ETIMEOUT).
// The library is built as one translation unit (tesm_b200.cu includes every .cu).
__device__ int g_device_status = 0;

__device__ __forceinline__ void flag_timeout() { atomicExch(&g_device_status, TESM_ETIMEOUT); }

// ------------------------------------------------------------ element access
__device__ __forceinline__ float load_f(const void *p, int dtype, int64_t i) {
  return dtype == TESM_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[i])
                            : reinterpret_cast<const float *>(p)[i];
}

__device__ __forceinline__ void store_f(void *p, int dtype, int64_t i, float v) {
  if (dtype == TESM_BF16)
    reinterpret_cast<__nv_bfloat16 *>(p)[i] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float *>(p)[i] = v;
}

// Round a float to the nearest bfloat16 value (ties to even) and return it as float.
__device__ __forceinline__ float round_bf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Logistic sigmoid from the hardware exponential and an IEEE-rounded reciprocal: no
// slow-path branches, so a thread can interleave many of them (relative error ~1e-6).
__device__ __forceinline__ float fast_sigmoid(float x) { return __frcp_rn(1.f + __expf(-x)); }

// Round to the arithmetic precision of `dtype` (identity for fp32).
__device__ __forceinline__ float round_to(int dtype, float v) { return dtype == TESM_BF16 ? round_bf16(v) : v; }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide reductions for blockDim.x a multiple of 32 (<= 1024). `red` holds 32 slots.
template <class T, class Op>
__device__ __forceinline__ T block_reduce(T v, T *red, Op op, T init) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[wid] = v;
  __syncthreads();
  T r = lane < nw ? red[lane] : init;
#pragma unroll
  for (int o = 16; o; o >>= 1) r = op(r, __shfl_xor_sync(0xffffffffu, r, o));
  return r;
}

// Bounded spin limit for device waits (~seconds at B200 clocks with backoff).
constexpr long long kSpinLimit = 1ll << 26;

// ------------------------------------------------------------ programmatic dependent launch
// Kernels launched with launch_k may start while the previous kernel in the stream is still
// finishing: each one signals its own dependents early (pdl_trigger) and waits for its
// predecessor's completion and memory (pdl_wait) before it touches any global memory that a
// previous kernel writes or reads -- so the launch latency and the prologue (barrier setup,
// TMEM allocation, constant-weight prefetch) overlap the predecessor's tail.  Every kernel
// launched this way executes pdl_wait, which keeps the ordering transitive along the stream.
// Without the launch attribute both instructions are no-ops.  Off by default (TESM_PDL=1 turns
// it on): measured on the batch-256 decode step it was 2-3% slower than plain stream order.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

inline bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char *e = getenv("TESM_PDL");
    v = e ? atoi(e) : 0;
  }
  return v != 0;
}

template <typename... KArgs, typename... Args>
inline int launch_k(const char *what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                    Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) return fail(TESM_ELAUNCH, std::string(what) + ": " + cudaGetErrorString(e));
  return TESM_OK;
}

}  // namespace tesm
