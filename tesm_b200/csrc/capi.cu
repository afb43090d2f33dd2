// Library-wide C-ABI plumbing: error strings, version, sticky device status.
#include "common.cuh"

#include <cstdio>

namespace tesm {

static thread_local std::string t_last_error;

void set_error(const std::string &msg) { t_last_error = msg; }

int fail(int code, const std::string &msg) {
  t_last_error = msg;
  return code;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return fail(TESM_ELAUNCH, std::string(what) + ": " + cudaGetErrorString(e));
  }
  return TESM_OK;
}

}  // namespace tesm

extern "C" const char *tesm_b200_last_error(void) { return tesm::t_last_error.c_str(); }

extern "C" int tesm_b200_version(void) { return 1; }

extern "C" int tesm_b200_device_status(int *status_out) {
  int zero = 0, v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, tesm::g_device_status, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(tesm::g_device_status, &zero, sizeof(int));
  if (e != cudaSuccess) return tesm::fail(TESM_ELAUNCH, std::string("device_status: ") + cudaGetErrorString(e));
  if (status_out) *status_out = v;
  return TESM_OK;
}
