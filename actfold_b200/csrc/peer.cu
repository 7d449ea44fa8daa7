// CUDA IPC of device buffers between the ranks of one node, for the
// tensor-parallel pass's peer-memory sums (af_fold_set_peer_sum).
#include <cuda.h>

#include <mutex>

#include "common.cuh"

namespace af {
namespace {

typedef CUresult (*PFN_addressRange_t)(CUdeviceptr*, size_t*, CUdeviceptr);

PFN_addressRange_t address_range_fn() {
  static PFN_addressRange_t fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_addressRange_t>(f);
  });
  return fn;
}

}  // namespace
}  // namespace af

using namespace af;

extern "C" int af_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  AF_REQUIRE(ptr && handle && offset, "af_ipc_export: null pointer");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "CUDA IPC handles are 64 bytes");
  PFN_addressRange_t range = address_range_fn();
  if (!range) return fail(AF_ERR_CUDA, "af_ipc_export: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS)
    return fail(AF_ERR_ARG, "af_ipc_export: not a device allocation (cuMemGetAddressRange " + std::to_string((int)r) + ")");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess)
    return fail(AF_ERR_CUDA, std::string("af_ipc_export: cudaIpcGetMemHandle failed (") + cudaGetErrorString(e) +
                                 "; allocations made through cuMemCreate, e.g. expandable segments, cannot be exported)");
  memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return AF_OK;
}

extern "C" int af_ipc_import(const void* handle, int64_t offset, void** ptr, void** base) {
  AF_REQUIRE(handle && ptr && base && offset >= 0, "af_ipc_import: bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* b = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess)
    return fail(AF_ERR_CUDA, std::string("af_ipc_import: cudaIpcOpenMemHandle failed (") + cudaGetErrorString(e) + ")");
  *base = b;
  *ptr = static_cast<char*>(b) + offset;
  return AF_OK;
}

extern "C" int af_ipc_close(void* base) {
  AF_REQUIRE(base, "af_ipc_close: null pointer");
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess)
    return fail(AF_ERR_CUDA, std::string("af_ipc_close: cudaIpcCloseMemHandle failed (") + cudaGetErrorString(e) + ")");
  return AF_OK;
}
