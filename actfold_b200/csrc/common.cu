// Library-wide state: version string, per-thread error messages, device info.
#include <mutex>
#include <vector>

#include "common.cuh"

namespace af {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(AF_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return AF_OK;
}

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if ((int)cache.size() <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

}  // namespace af

extern "C" const char* af_version(void) { return "actfold_b200 0.1.0 sm_100a"; }

extern "C" const char* af_last_error_string(void) { return af::g_last_error.c_str(); }
