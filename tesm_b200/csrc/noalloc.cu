// Allocation-free variant of the SISO state scan.
//
// tesm_b200_siso_scan needs a caller-owned device workspace for its chunk-to-chunk carries.
// Some callers cannot provide one: code running where cudaMalloc is not allowed or not
// wanted (a host runtime with its own fixed memory plan, an allocator-less embedding of the
// library, a caller holding no device allocator at all).  This entry point keeps that
// scratch in a fixed array that lives in the library itself, so it allocates nothing.
#include "layer_common.cuh"

#include <mutex>

namespace tesm {

// Fixed scratch for the look-back carries: 8 MiB, resident on every GPU that loads the
// library until the process exits.  A SISO scan needs about B * ceil(L/32) * d_state * 12
// bytes plus flags (tesm_b200_scan_workspace is the exact figure), e.g. batch 8 x 8192
// positions x d_state 256 needs 6.0 MiB.
constexpr int64_t kNoAllocScratchBytes = 8ll << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the array, looked up once per device and kept for the life of the
// process (in host code the array's name is only a host-side stand-in, never a device
// pointer).
static int noalloc_scratch_ptr(void **out) {
  static std::mutex mu;
  static void *ptrs[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(TESM_ELAUNCH, std::string("siso_scan_noalloc: cudaGetDevice: ") +
                                                      cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(TESM_EUNSUPPORTED, "siso_scan_noalloc: device index above 63");
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(TESM_ELAUNCH, std::string("siso_scan_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    ptrs[dev] = p;
  }
  *out = ptrs[dev];
  return TESM_OK;
}

}  // namespace tesm

using namespace tesm;

extern "C" int tesm_b200_siso_scan_noalloc(const void *proj, int dtype, int64_t ldp, int64_t B, int64_t L,
                                           int64_t Dm, int64_t D, int64_t R, int64_t scan_chunk,
                                           const float *decay_bias, const double *h0, float *states,
                                           float *final_f32, double *final_f64, tesm_stream_t stream) {
  TESM_REQUIRE(B > 0 && L > 0 && D > 0, "siso_scan_noalloc: bad shape");
  int64_t need = 0;
  int rc = tesm_b200_scan_workspace(B, L, D, 1, &need);
  if (rc) return rc;
  if (need > kNoAllocScratchBytes)
    return fail(TESM_EUNSUPPORTED, "siso_scan_noalloc: this shape (about batch * ceil(L/32) * d_state * 12 bytes) needs " + std::to_string(need) +
                                       " bytes of scratch, above the fixed " +
                                       std::to_string(kNoAllocScratchBytes) +
                                       " bytes; use tesm_b200_siso_scan with a workspace");
  void *scratch = nullptr;
  rc = noalloc_scratch_ptr(&scratch);
  if (rc) return rc;
  // run_scan clears the flags and the chunk ticket with cudaMemsetAsync before its launch,
  // so the previous call's contents never leak into this one.
  return run_scan(proj, dtype, ldp, B, L, Dm, 1, D, R, 1, decay_bias, nullptr, h0, states, final_f32, final_f64,
                  scratch, kNoAllocScratchBytes, (cudaStream_t)stream, scan_chunk);
}
