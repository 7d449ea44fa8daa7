// Shared device/host helpers for libactfold_b200 (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string.h>

#include <string>
#include <utility>

#include "../../include/actfold_b200.h"

namespace af {

// ---------------------------------------------------------------------------
// Error reporting: every C entry point returns an af_status and leaves a
// message retrievable with af_last_error_string() on the calling thread.
// ---------------------------------------------------------------------------
void set_error(const std::string& msg);
int fail(int status, const std::string& msg);
int check_launch(const char* what);

#define AF_REQUIRE(cond, msg)                         \
  do {                                                \
    if (!(cond)) return ::af::fail(AF_ERR_ARG, msg);  \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ---------------------------------------------------------------------------
// Element types. DT codes follow af_dtype: 0 = f32, 1 = f16, 2 = bf16.
// ---------------------------------------------------------------------------
template <int DT>
struct Elt;
template <>
struct Elt<AF_DTYPE_F32> {
  static constexpr int kPerVec = 4;  // elements per 16-byte vector
  static constexpr int kBytes = 4;
};
template <>
struct Elt<AF_DTYPE_F16> {
  static constexpr int kPerVec = 8;
  static constexpr int kBytes = 2;
};
template <>
struct Elt<AF_DTYPE_BF16> {
  static constexpr int kPerVec = 8;
  static constexpr int kBytes = 2;
};

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Round a float to the storage type DT and back (round to nearest even).
template <int DT>
__device__ __forceinline__ float rnd(float x) {
  if constexpr (DT == AF_DTYPE_BF16) {
    return __bfloat162float(__float2bfloat16_rn(x));
  } else if constexpr (DT == AF_DTYPE_F16) {
    return __half2float(__float2half_rn(x));
  } else {
    return x;
  }
}

__device__ __forceinline__ uint16_t f2bf_bits(float x) {
  __nv_bfloat16 b = __float2bfloat16_rn(x);
  return *reinterpret_cast<uint16_t*>(&b);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return (uint32_t)f2bf_bits(lo) | ((uint32_t)f2bf_bits(hi) << 16);
}

// Unpack one 16-byte vector into floats.
template <int DT>
__device__ __forceinline__ void unpack(const uint4& v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  if constexpr (DT == AF_DTYPE_BF16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = bf16_lo(w[i]);
      f[2 * i + 1] = bf16_hi(w[i]);
    }
  } else if constexpr (DT == AF_DTYPE_F16) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
      float2 g = __half22float2(h);
      f[2 * i] = g.x;
      f[2 * i + 1] = g.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = __uint_as_float(w[i]);
  }
}

template <int DT>
__device__ __forceinline__ float load_scalar(const char* p, int i) {
  if constexpr (DT == AF_DTYPE_BF16) {
    return __uint_as_float((uint32_t)(*reinterpret_cast<const uint16_t*>(p + 2 * i)) << 16);
  } else if constexpr (DT == AF_DTYPE_F16) {
    return __half2float(*reinterpret_cast<const __half*>(p + 2 * i));
  } else {
    return *reinterpret_cast<const float*>(p + 4 * i);
  }
}

__device__ __forceinline__ uint4 ldg16(const void* p) {
  uint4 r;
  asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Pull the 128-byte line holding `p` into L2 (no register result, no wait).
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

__device__ __forceinline__ void stg16(void* p, const uint4& v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Launch priority applied by launch_ex on this host thread (kNoPriority: the
// stream's own). Set it for a stretch of launches with LaunchPriority.
constexpr int kNoPriority = -1000000;
inline int& launch_priority() {
  static thread_local int prio = kNoPriority;
  return prio;
}
struct LaunchPriority {
  int saved;
  explicit LaunchPriority(int prio) : saved(launch_priority()) { launch_priority() = prio; }
  ~LaunchPriority() { launch_priority() = saved; }
};

// Launch `kernel` on `stream` as clusters of `cluster` CTAs (none when the
// cluster has one CTA), when `pdl` with programmatic dependent launch, and at
// the current launch_priority().
template <typename... KArgs, typename... Args>
inline cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             bool pdl, dim3 cluster, Args&&... args) {
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[3];
  int n = 0;
  if (launch_priority() != kNoPriority) {
    at[n].id = cudaLaunchAttributePriority;
    at[n].val.priority = launch_priority();
    ++n;
  }
  if (cluster.x * cluster.y * cluster.z > 1) {
    at[n].id = cudaLaunchAttributeClusterDimension;
    at[n].val.clusterDim.x = cluster.x;
    at[n].val.clusterDim.y = cluster.y;
    at[n].val.clusterDim.z = cluster.z;
    ++n;
  }
  if (pdl) {
    at[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}


// Programmatic dependent launch. A kernel launched with the programmatic
// stream-serialization attribute may start while its stream predecessor is
// still running. pdl_wait() blocks the calling thread until the predecessor
// grid has completed and its memory operations are visible (it returns at once
// for a normal launch); pdl_trigger() lets this grid's own dependents begin
// launching. Kernels of the folded and dense passes call pdl_trigger() first
// and pdl_wait() before their first access to memory that another kernel of
// the stream writes or reads; only read-only weights may be touched before it.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Thread-block cluster helpers: a full cluster barrier (release/acquire, so
// shared-memory writes before it are visible to peers after it), the address
// of the same shared-memory offset in CTA `rank` of the cluster, and loads
// from such an address.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_map(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ void st_cluster_f4(uint32_t addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

__device__ __forceinline__ void st_cluster_f2(uint32_t addr, float2 v) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1,%2};" ::"r"(addr), "f"(v.x), "f"(v.y) : "memory");
}

__device__ __forceinline__ float2 ld_cluster_f2(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared::cluster.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
  return v;
}


// Number of SMs of the current device (cached per device).
int sm_count();

}  // namespace af
