// af_dense_forward_static: the parent pass with its scratch in a file-scope
// device array, so a caller supplies no workspace and the library allocates
// nothing.
//
// The array lives in this translation unit alone, so under lazy module
// loading its device memory is taken only by processes that call this entry
// point. Its device address is looked up once per device with
// cudaGetSymbolAddress (the device that owns the stream must be current; a
// stream of another device is refused) and cached for the life of the
// process: after cudaDeviceReset the cached address is stale, so a process
// that resets a device must not call this entry point again. The call then
// runs af_dense_forward unchanged on that scratch.
// Every scratch buffer of the dense pass is written in full before it is read
// (normalised rows, attention output, residual rows, SwiGLU rows, positions),
// so no part of the array has to start at zero; the outputs that must start
// at zero (the logit row sums) are cleared by af_dense_forward itself.
//
// One array per device means two calls in flight at once on the same device
// (different streams, or different host threads) race on the scratch.

#include <mutex>
#include <string>

#include "common.cuh"

static __device__ __align__(256) unsigned char g_dense_scratch[AF_DENSE_STATIC_WORKSPACE_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

int scratch_of_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return af::fail(AF_ERR_CUDA, std::string("af_dense_forward_static: cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return af::fail(AF_ERR_ARG, "af_dense_forward_static: device ordinal out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_dense_scratch);
    if (e != cudaSuccess || !p)
      return af::fail(AF_ERR_CUDA, std::string("af_dense_forward_static: cudaGetSymbolAddress: ") +
                                       (e != cudaSuccess ? cudaGetErrorString(e) : "null address"));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return AF_OK;
}

}  // namespace

extern "C" int af_dense_forward_static(const af_model* model, const int64_t* tokens, int64_t T, float tau,
                                       void* layer_in, void* qkv, void* logits, uint8_t* self_stable,
                                       float* logit_row_sums, uint32_t* status, void* stream) {
  AF_REQUIRE(model, "af_dense_forward_static: null model");
  AF_REQUIRE(T > 0, "af_dense_forward_static: T out of range");
  int64_t need = 0;
  int st = af_dense_workspace_bytes(&model->dims, T, &need);
  if (st) return st;
  if (need > (int64_t)AF_DENSE_STATIC_WORKSPACE_BYTES)
    return af::fail(AF_ERR_CAPACITY, "af_dense_forward_static: T=" + std::to_string(T) + " needs " + std::to_string(need) +
                                         " scratch bytes, above the static limit of " +
                                         std::to_string((long long)AF_DENSE_STATIC_WORKSPACE_BYTES));
  if (stream) {
    // The cached address belongs to the current device; a stream of another
    // device would hand the kernels a scratch pointer of the wrong GPU.
    int cur = -1, sdev = -1;
    cudaError_t e = cudaGetDevice(&cur);
    if (e == cudaSuccess) e = cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev);
    if (e != cudaSuccess)
      return af::fail(AF_ERR_CUDA, std::string("af_dense_forward_static: stream device: ") + cudaGetErrorString(e));
    if (sdev != cur)
      return af::fail(AF_ERR_ARG, "af_dense_forward_static: the stream belongs to device " + std::to_string(sdev) +
                                      " but device " + std::to_string(cur) + " is current");
  }
  void* scratch = nullptr;
  if ((st = scratch_of_current_device(&scratch))) return st;
  return af_dense_forward(model, tokens, T, tau, layer_in, qkv, logits, self_stable, logit_row_sums, scratch,
                          (int64_t)AF_DENSE_STATIC_WORKSPACE_BYTES, status, stream);
}
