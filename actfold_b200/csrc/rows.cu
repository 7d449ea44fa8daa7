// Row-granular select / gather kernels (HBM-bound, sm_100a).
//
// A warp owns one (b, t) row and moves it with 128-bit vector loads/stores,
// four vectors in flight per lane. Only the selected source row is read, so
// a merge costs one row read + one row write (the reference Triton kernel
// reads both candidates). Unaligned or odd-sized rows take a byte loop.
#include "common.cuh"

namespace af {

struct RowSel {
  // select-source description
  const char* a;  // source when sel == 1 (parent / cached rows)
  int64_t a_bs, a_ts;
  const char* b;  // source when sel == 0 (child rows), or nullptr for zero fill
  int64_t b_bs, b_ts;
  const uint8_t* mask;
  int64_t m_bs;
  const uint8_t* present;  // per-token presence (gather mode 1), nullable
  int mode;                // 0: sel = mask[b,t]; 1: sel = present[t] && any_b mask[b,t]
  int64_t B, T;
  char* out;
  int64_t o_bs, o_ts;
  int64_t row_bytes;
};

__device__ __forceinline__ bool row_selected(const RowSel& p, int64_t b, int64_t t) {
  if (p.mode == 0) return p.mask[b * p.m_bs + t] != 0;
  if (p.present && !p.present[t]) return false;
  for (int64_t bb = 0; bb < p.B; ++bb)
    if (p.mask[bb * p.m_bs + t]) return true;
  return false;
}

template <bool VEC>
__global__ void __launch_bounds__(256) k_select_rows(const RowSel p) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= p.B * p.T) return;
  const int64_t b = row / p.T, t = row - b * p.T;
  const bool sel = row_selected(p, b, t);
  const char* src = sel ? p.a + b * p.a_bs + t * p.a_ts : (p.b ? p.b + b * p.b_bs + t * p.b_ts : nullptr);
  char* dst = p.out + b * p.o_bs + t * p.o_ts;
  if constexpr (VEC) {
    const int64_t nvec = p.row_bytes >> 4;
    int64_t v = lane;
    if (src) {
      for (; v + 96 < nvec; v += 128) {
        const uint4 x0 = ldg16(src + 16 * v), x1 = ldg16(src + 16 * (v + 32));
        const uint4 x2 = ldg16(src + 16 * (v + 64)), x3 = ldg16(src + 16 * (v + 96));
        stg16(dst + 16 * v, x0);
        stg16(dst + 16 * (v + 32), x1);
        stg16(dst + 16 * (v + 64), x2);
        stg16(dst + 16 * (v + 96), x3);
      }
      for (; v < nvec; v += 32) stg16(dst + 16 * v, ldg16(src + 16 * v));
    } else {
      const uint4 z = make_uint4(0u, 0u, 0u, 0u);
      for (; v < nvec; v += 32) stg16(dst + 16 * v, z);
    }
  } else {
    for (int64_t i = lane; i < p.row_bytes; i += 32) dst[i] = src ? src[i] : (char)0;
  }
}

static int launch_select(const RowSel& p, void* stream, const char* what) {
  if (p.B == 0 || p.T == 0 || p.row_bytes == 0) return AF_OK;
  const int64_t rows = p.B * p.T;
  const int64_t blocks = ceil_div(rows, 8);
  if (blocks > 0x7fffffff) return fail(AF_ERR_ARG, std::string(what) + ": too many rows");
  uintptr_t al = reinterpret_cast<uintptr_t>(p.a) | reinterpret_cast<uintptr_t>(p.b) |
                 reinterpret_cast<uintptr_t>(p.out) | (uintptr_t)p.a_bs | (uintptr_t)p.a_ts | (uintptr_t)p.b_bs |
                 (uintptr_t)p.b_ts | (uintptr_t)p.o_bs | (uintptr_t)p.o_ts | (uintptr_t)p.row_bytes;
  cudaStream_t s = as_stream(stream);
  if ((al & 15u) == 0)
    k_select_rows<true><<<(unsigned)blocks, 256, 0, s>>>(p);
  else
    k_select_rows<false><<<(unsigned)blocks, 256, 0, s>>>(p);
  return check_launch(what);
}

// out[b, j] = idx[j] >= 0 ? src[b, idx[j]] : 0   (one warp per output row)
template <bool VEC>
__global__ void __launch_bounds__(256) k_gather_index(const char* __restrict__ src, int64_t s_bs, int64_t s_ts,
                                                      const int32_t* __restrict__ idx, int64_t n, int64_t B,
                                                      char* __restrict__ out, int64_t o_bs, int64_t o_ts,
                                                      int64_t row_bytes) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= B * n) return;
  const int64_t b = row / n, j = row - b * n;
  const int32_t t = idx[j];
  const char* s = t >= 0 ? src + b * s_bs + (int64_t)t * s_ts : nullptr;
  char* d = out + b * o_bs + j * o_ts;
  if constexpr (VEC) {
    const int64_t nvec = row_bytes >> 4;
    for (int64_t v = lane; v < nvec; v += 32) stg16(d + 16 * v, s ? ldg16(s + 16 * v) : make_uint4(0u, 0u, 0u, 0u));
  } else {
    for (int64_t i = lane; i < row_bytes; i += 32) d[i] = s ? s[i] : (char)0;
  }
}

}  // namespace af

using namespace af;

extern "C" int af_gather_rows_index(const void* src, int64_t src_bstride, int64_t src_tstride, const int32_t* idx,
                                    int64_t n, int64_t batch, void* out, int64_t out_bstride, int64_t out_tstride,
                                    int64_t row_bytes, void* stream) {
  AF_REQUIRE(n >= 0 && batch >= 0 && row_bytes >= 0, "af_gather_rows_index: bad shape");
  if (n == 0 || batch == 0 || row_bytes == 0) return AF_OK;
  AF_REQUIRE(src && idx && out, "af_gather_rows_index: null pointer");
  const int64_t blocks = ceil_div(n * batch, 8);
  if (blocks > 0x7fffffff) return fail(AF_ERR_ARG, "af_gather_rows_index: too many rows");
  const uintptr_t al = reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(out) | (uintptr_t)src_bstride |
                       (uintptr_t)src_tstride | (uintptr_t)out_bstride | (uintptr_t)out_tstride | (uintptr_t)row_bytes;
  cudaStream_t s = as_stream(stream);
  if ((al & 15u) == 0)
    k_gather_index<true><<<(unsigned)blocks, 256, 0, s>>>(static_cast<const char*>(src), src_bstride, src_tstride, idx,
                                                          n, batch, static_cast<char*>(out), out_bstride, out_tstride,
                                                          row_bytes);
  else
    k_gather_index<false><<<(unsigned)blocks, 256, 0, s>>>(static_cast<const char*>(src), src_bstride, src_tstride,
                                                           idx, n, batch, static_cast<char*>(out), out_bstride,
                                                           out_tstride, row_bytes);
  return check_launch("af_gather_rows_index");
}

extern "C" int af_merge_rows(const void* parent, int64_t parent_bstride, int64_t parent_tstride, const void* child,
                             int64_t child_bstride, int64_t child_tstride, const uint8_t* stable,
                             int64_t stable_bstride, void* out, int64_t out_bstride, int64_t out_tstride,
                             int64_t batch, int64_t seq, int64_t row_bytes, void* stream) {
  AF_REQUIRE(batch >= 0 && seq >= 0 && row_bytes >= 0, "af_merge_rows: bad shape");
  if (batch == 0 || seq == 0 || row_bytes == 0) return AF_OK;
  AF_REQUIRE(parent && child && stable && out, "af_merge_rows: null pointer");
  RowSel p{};
  p.a = static_cast<const char*>(parent);
  p.a_bs = parent_bstride;
  p.a_ts = parent_tstride;
  p.b = static_cast<const char*>(child);
  p.b_bs = child_bstride;
  p.b_ts = child_tstride;
  p.mask = stable;
  p.m_bs = stable_bstride;
  p.mode = 0;
  p.B = batch;
  p.T = seq;
  p.out = static_cast<char*>(out);
  p.o_bs = out_bstride;
  p.o_ts = out_tstride;
  p.row_bytes = row_bytes;
  return launch_select(p, stream, "af_merge_rows");
}

extern "C" int af_gather_rows_masked(const void* src, int64_t src_bstride, int64_t src_tstride, const uint8_t* mask,
                                     int64_t mask_bstride, const uint8_t* present, int mode, void* out,
                                     int64_t out_bstride, int64_t out_tstride, int64_t batch, int64_t seq,
                                     int64_t row_bytes, void* stream) {
  AF_REQUIRE(mode == 0 || mode == 1, "af_gather_rows_masked: mode must be 0 or 1");
  AF_REQUIRE(batch >= 0 && seq >= 0 && row_bytes >= 0, "af_gather_rows_masked: bad shape");
  if (batch == 0 || seq == 0 || row_bytes == 0) return AF_OK;
  AF_REQUIRE(src && mask && out, "af_gather_rows_masked: null pointer");
  RowSel p{};
  p.a = static_cast<const char*>(src);
  p.a_bs = src_bstride;
  p.a_ts = src_tstride;
  p.b = nullptr;
  p.mask = mask;
  p.m_bs = mask_bstride;
  p.present = present;
  p.mode = mode;
  p.B = batch;
  p.T = seq;
  p.out = static_cast<char*>(out);
  p.o_bs = out_bstride;
  p.o_ts = out_tstride;
  p.row_bytes = row_bytes;
  return launch_select(p, stream, "af_gather_rows_masked");
}
