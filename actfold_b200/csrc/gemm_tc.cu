// Weight-streaming tcgen05 GEMM: OUT[m, :] = X[m, :] . W^T for a small number
// of packed token rows m and a large weight matrix W [n, k] (nn.Linear layout).
//
// Swap-AB mapping: the 128-row MMA "M" dimension walks the weight rows (output
// features) and the MMA "N" dimension holds the token tile (16..256 tokens),
// so a handful of divergent tokens still fills the tensor core and every
// weight byte is read from HBM once per token tile.
//
// CTA = 6 warps: warp 0 lane 0 issues TMA loads of W and X k-blocks (64 wide,
// 128-byte swizzle) into a multi-stage shared-memory ring; warp 1 owns the
// TMEM accumulator (128 lanes x ntok fp32 columns) and its lane 0 issues
// tcgen05.mma (K = 16 per instruction, 4 per k-block) and tcgen05.commit to
// release ring slots; warps 2-5 drain TMEM (tcgen05.ld) into shared memory and
// run the fused epilogue. When the k-range is split across CTAs (split-K, used
// to put >= 2 CTAs on every SM for the small projections), partial tiles are
// reduced with vector red.global.add into an fp32 accumulator and the last
// arriving CTA (per-tile counter) runs the epilogue and re-zeroes its slice,
// so the workspace is clean again when the kernel ends.
//
// Every mbarrier wait is bounded (about one second); on timeout the CTA sets
// AF_STATUS_TIMEOUT in the status word, stops issuing, waits (bounded) for its
// in-flight TMA loads, frees its TMEM and returns.
#include <mutex>
#include <vector>

#include "gemm_tc.cuh"

namespace af {

constexpr int kBlockK = 64;   // bf16 elements per k-block (one 128-byte swizzle row)
constexpr int kTileN = 128;   // weight rows per CTA (MMA M)
constexpr int kThreads = 192;

struct GemmDev {
  int n, k, m_cap, m_pad, ntok, n_tiles, nkb, kb_per_split, splits, stages;
  const int* m_dev;
  int epi;
  __nv_bfloat16* out;
  int64_t ldo;
  const int* out_rows;
  const __nv_bfloat16* res;
  int64_t ldr;
  const int* res_rows;
  const float* rope_cos;
  const float* rope_sin;
  const int* positions;
  int rope_cols, half_dim;
  float* acc;
  int* counters;
  unsigned* status;
  float* row_sums;
};

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__global__ void __launch_bounds__(kThreads, 1) k_gemm_tc(const __grid_constant__ CUtensorMap tmW,
                                                          const __grid_constant__ CUtensorMap tmX, const GemmDev p) {
  extern __shared__ uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int M = p.m_dev ? *p.m_dev : p.m_cap;
  if (M > p.m_cap) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) atomicOr(p.status, AF_STATUS_CAPACITY);
    M = p.m_cap;
  }
  const int m0 = blockIdx.z * p.ntok;
  if (m0 >= M) return;  // uniform: nothing to compute for this token tile
  const int Mv = min(p.ntok, M - m0);
  const int n0 = blockIdx.x * kTileN;
  const int kb0 = blockIdx.y * p.kb_per_split;
  const int nkb = min(p.kb_per_split, p.nkb - kb0);
  const int S = p.stages;
  const uint32_t w_bytes = kTileN * kBlockK * 2, x_bytes = p.ntok * kBlockK * 2;
  const uint32_t stage_bytes = w_bytes + x_bytes;

  // 1024-byte aligned ring, then barriers and flags.
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bars = base + S * stage_bytes;
  uint64_t* bar_ptr = reinterpret_cast<uint64_t*>(gbase + S * stage_bytes);
  (void)bar_ptr;
  const uint32_t full0 = bars, empty0 = bars + 8 * S, accb = bars + 16 * S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + S * stage_bytes + 16 * S + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + S * stage_bytes + 16 * S + 16);
  volatile int* last_flag = reinterpret_cast<volatile int*>(gbase + S * stage_bytes + 16 * S + 20);
  volatile int* issued_slot = reinterpret_cast<volatile int*>(gbase + S * stage_bytes + 16 * S + 24);

  uint32_t ncols = 32;
  while ((int)ncols < p.ntok) ncols <<= 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(accb, 1);
    *abort_flag = 0;
    *last_flag = 0;
    *issued_slot = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), ncols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    int i = 0;
    for (; i < nkb; ++i) {
      const int s = i % S;
      const uint32_t ph = (i / S) & 1;
      if (!mbar_wait(empty0 + 8 * s, ph ^ 1, abort_flag)) {
        atomicOr(p.status, AF_STATUS_TIMEOUT);
        *abort_flag = 1;
        break;
      }
      const uint32_t st = base + s * stage_bytes;
      mbar_arrive_expect_tx(full0 + 8 * s, stage_bytes);
      const int kx = (kb0 + i) * kBlockK;
      tma_load_2d(st, &tmW, full0 + 8 * s, kx, n0);
      tma_load_2d(st + w_bytes, &tmX, full0 + 8 * s, kx, m0);
    }
    *issued_slot = i;
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = idesc_bf16(kTileN, p.ntok);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % S;
      const uint32_t ph = (i / S) & 1;
      if (!mbar_wait(full0 + 8 * s, ph, abort_flag)) {
        atomicOr(p.status, AF_STATUS_TIMEOUT);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t st = base + s * stage_bytes;
      const uint64_t adesc = sw128_desc(st), bdesc = sw128_desc(st + w_bytes);
#pragma unroll
      for (int kk = 0; kk < kBlockK / 16; ++kk)
        tc_mma_bf16(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (i | kk) != 0 ? 1u : 0u);
      tc_commit(empty0 + 8 * s);
    }
    tc_commit(accb);
  } else if (warp >= 2) {
    // ---------------- epilogue (128 threads) ----------------
    const int q = warp & 3;
    const int r = 32 * q + lane;  // tile row = output feature n0 + r
    const int ld = p.ntok + 1;
    float* tile = reinterpret_cast<float*>(gbase);  // ring memory is idle once the accumulator is final
    const bool ok = mbar_wait(accb, 0, abort_flag);
    if (!ok) {
      atomicOr(p.status, AF_STATUS_TIMEOUT);
      *abort_flag = 1;
    }
    tc_fence_after();
    const int nchunk = (Mv + 15) / 16;
    if (ok && !*abort_flag) {
      float* arow = p.acc + (int64_t)(n0 + r) * p.m_pad + m0;
      for (int c = 0; c < nchunk; ++c) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(16 * c), v);
        if (p.splits > 1) {
#pragma unroll
          for (int j = 0; j < 16; j += 4) red_add_v4(arow + 16 * c + j, v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) tile[r * ld + 16 * c + j] = v[j];
        }
      }
      if (p.splits > 1) {
        __threadfence();
        named_bar_sync(1, 128);
        if (threadIdx.x == 64) {
          const int tile_id = blockIdx.z * p.n_tiles + blockIdx.x;
          const int old = atomicAdd(&p.counters[tile_id], 1);
          *last_flag = (old == p.splits - 1) ? 1 : 0;
          if (old == p.splits - 1) p.counters[tile_id] = 0;
        }
        named_bar_sync(1, 128);
        if (*last_flag) {
          __threadfence();
          for (int c = 0; c < nchunk * 16; c += 4) {
            const float4 a = __ldcg(reinterpret_cast<const float4*>(arow + c));
            __stcg(reinterpret_cast<float4*>(arow + c), make_float4(0.f, 0.f, 0.f, 0.f));
            tile[r * ld + c] = a.x;
            tile[r * ld + c + 1] = a.y;
            tile[r * ld + c + 2] = a.z;
            tile[r * ld + c + 3] = a.w;
          }
        }
      }
      const bool do_epi = (p.splits == 1) || *last_flag;
      named_bar_sync(1, 128);
      if (do_epi) {
        const int n = n0 + r;
        for (int m = 0; m < Mv; ++m) {
          const int gm = m0 + m;
          const int64_t orow = p.out_rows ? p.out_rows[gm] : gm;
          const float a = tile[r * ld + m];
          if (p.epi == EPI_STORE) {
            const __nv_bfloat16 ob = __float2bfloat16_rn(a);
            p.out[orow * p.ldo + n] = ob;
            if (p.row_sums) {
              const float part = warp_sum(__bfloat162float(ob));
              if (lane == 0) atomicAdd(p.row_sums + orow, part);
            }
          } else if (p.epi == EPI_RESIDUAL) {
            const int64_t rrow = p.res_rows ? p.res_rows[gm] : gm;
            const float rv = __bfloat162float(p.res[rrow * p.ldr + n]);
            p.out[orow * p.ldo + n] = __float2bfloat16_rn(__fadd_rn(rv, bf(a)));
          } else if (p.epi == EPI_SWIGLU) {
            if (r < 64) {
              const float g = bf(a), u = bf(tile[(r + 64) * ld + m]);
              const float silu = __fdiv_rn(g, __fadd_rn(1.f, expf(-g)));
              p.out[orow * p.ldo + (n0 >> 1) + r] = __float2bfloat16_rn(__fmul_rn(silu, u));
            }
          } else {  // EPI_ROPE
            const float x = bf(a);
            float y = x;
            if (n < p.rope_cols) {
              const int i = r & (p.half_dim - 1);
              const float other = bf(tile[(r ^ p.half_dim) * ld + m]);
              const int pos = p.positions[gm];
              const float cs = p.rope_cos[(int64_t)pos * p.half_dim + i];
              const float sn = p.rope_sin[(int64_t)pos * p.half_dim + i];
              y = (r & p.half_dim) ? __fadd_rn(__fmul_rn(x, cs), __fmul_rn(other, sn))
                                   : __fsub_rn(__fmul_rn(x, cs), __fmul_rn(other, sn));
            }
            p.out[orow * p.ldo + n] = __float2bfloat16_rn(y);
          }
        }
      }
    }
  }

  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag) {
    // Drain TMA loads that may still be in flight into the ring (bounded).
    const int issued = *issued_slot;
    volatile int no_abort = 0;
    for (int i = max(0, issued - S); i < issued; ++i) mbar_wait(full0 + 8 * (i % S), (i / S) & 1, &no_abort);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
}

// ------------------------------------------------------------------ host side
typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled_t encode_fn() {
  static PFN_encodeTiled_t fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled_t>(f);
  });
  return fn;
}

int make_tmap_bf16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld_elems,
                   uint32_t box_rows) {
  PFN_encodeTiled_t fn = encode_fn();
  if (!fn) return fail(AF_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (ld_elems * 2) % 16 || cols % 64)
    return fail(AF_ERR_ARG, "TMA operand must be 16-byte aligned with a 16-byte row stride and 64-multiple width");
  const cuuint64_t gdim[2] = {cols, rows};
  const cuuint64_t gstride[1] = {ld_elems * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), gdim, gstride, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AF_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return AF_OK;
}

int gemm_ntok(int m_cap) {
  const int mt = (m_cap + 255) / 256;
  int nt = (m_cap + mt - 1) / mt;
  nt = (nt + 15) / 16 * 16;
  return nt < 16 ? 16 : nt;
}

void gemm_workspace(int n, int m_cap, int64_t* acc_elems, int* counter_elems) {
  const int nt = gemm_ntok(m_cap);
  const int mt = (m_cap + nt - 1) / nt;
  *acc_elems = (int64_t)n * mt * nt;
  *counter_elems = (n / kTileN) * mt;
}

static int stages_for(int ntok) {
  const int stage = kTileN * kBlockK * 2 + ntok * kBlockK * 2;
  int s = (100 * 1024) / stage;  // two CTAs per SM when it fits
  if (s < 2) s = 2;
  if (s > 8) s = 8;
  const int staging = kTileN * (ntok + 1) * 4;
  while (s * stage < staging) ++s;
  return s;
}

int gemm_run(const GemmCall& c, cudaStream_t stream) {
  AF_REQUIRE(c.x && c.w && c.out && c.status, "gemm: null pointer");
  AF_REQUIRE(c.n > 0 && c.n % kTileN == 0, "gemm: n must be a positive multiple of 128");
  AF_REQUIRE(c.k > 0 && c.k % kBlockK == 0, "gemm: k must be a positive multiple of 64");
  AF_REQUIRE(c.m_cap > 0, "gemm: m_cap must be positive");
  AF_REQUIRE(c.epi >= EPI_STORE && c.epi <= EPI_ROPE, "gemm: bad epilogue");
  AF_REQUIRE(c.epi != EPI_RESIDUAL || c.res, "gemm: residual epilogue needs res");
  AF_REQUIRE(c.epi != EPI_ROPE || (c.rope_cos && c.rope_sin && c.positions && c.head_dim == 128 && c.rope_cols % 128 == 0),
             "gemm: rope epilogue needs cos/sin/positions and head_dim 128");
  const int ntok = gemm_ntok(c.m_cap);
  const int m_tiles = (c.m_cap + ntok - 1) / ntok;
  const int n_tiles = c.n / kTileN;
  const int nkb = c.k / kBlockK;
  int splits = c.splits;
  const int stages = stages_for(ntok);
  const int stage_bytes = kTileN * kBlockK * 2 + ntok * kBlockK * 2;
  const int smem = stages * stage_bytes + 1024 + 16 * stages + 64;
  const int per_sm = (2 * smem <= 227 * 1024) ? 2 : 1;
  if (splits <= 0) {
    const int target = per_sm * sm_count();
    splits = target / (n_tiles * m_tiles);
    const int max_splits = nkb / 4 > 0 ? nkb / 4 : 1;
    if (splits > max_splits) splits = max_splits;
    if (splits < 1) splits = 1;
  }
  int64_t need_acc;
  int need_cnt;
  gemm_workspace(c.n, c.m_cap, &need_acc, &need_cnt);
  if (splits > 1 && (!c.acc || !c.counters || c.acc_elems < need_acc || c.counter_elems < need_cnt)) splits = 1;
  const int kb_per = (nkb + splits - 1) / splits;
  splits = (nkb + kb_per - 1) / kb_per;

  CUtensorMap tw, tx;
  const CUtensorMap* pw = c.tmap_w;
  const CUtensorMap* px = c.tmap_x;
  if (!pw) {
    int st = make_tmap_bf16(&tw, c.w, c.n, c.k, c.k, kTileN);
    if (st) return st;
    pw = &tw;
  }
  if (!px) {
    int st = make_tmap_bf16(&tx, c.x, c.m_cap, c.k, c.ldx, ntok);
    if (st) return st;
    px = &tx;
  }
  GemmDev d;
  d.n = c.n;
  d.k = c.k;
  d.m_cap = c.m_cap;
  d.m_pad = m_tiles * ntok;
  d.ntok = ntok;
  d.n_tiles = n_tiles;
  d.nkb = nkb;
  d.kb_per_split = kb_per;
  d.splits = splits;
  d.stages = stages;
  d.m_dev = c.m_dev;
  d.epi = c.epi;
  d.out = static_cast<__nv_bfloat16*>(c.out);
  d.ldo = c.ldo;
  d.out_rows = c.out_rows;
  d.res = static_cast<const __nv_bfloat16*>(c.res);
  d.ldr = c.ldr;
  d.res_rows = c.res_rows;
  d.rope_cos = c.rope_cos;
  d.rope_sin = c.rope_sin;
  d.positions = c.positions;
  d.rope_cols = c.rope_cols;
  d.half_dim = c.head_dim / 2;
  d.acc = c.acc;
  d.counters = c.counters;
  d.status = c.status;
  d.row_sums = c.epi == EPI_STORE ? c.row_sums : nullptr;

  static std::once_flag attr_once;
  std::call_once(attr_once, [] {
    cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  dim3 grid(n_tiles, splits, m_tiles);
  k_gemm_tc<<<grid, kThreads, smem, stream>>>(*pw, *px, d);
  return check_launch("gemm_tc");
}

}  // namespace af

using namespace af;

extern "C" int af_linear_workspace(int64_t n, int64_t m_cap, int64_t* acc_floats, int64_t* counters) {
  AF_REQUIRE(n > 0 && m_cap > 0 && acc_floats && counters, "af_linear_workspace: bad argument");
  int64_t a;
  int c;
  gemm_workspace((int)n, (int)m_cap, &a, &c);
  *acc_floats = a;
  *counters = c;
  return AF_OK;
}

extern "C" int af_linear_bf16(const void* x, int64_t ldx, int64_t m_cap, const int32_t* m_dev, const void* w,
                              int64_t n, int64_t k, int epilogue, void* out, int64_t ldo, const int32_t* out_rows,
                              const void* residual, int64_t ldr, const int32_t* res_rows, const float* rope_cos,
                              const float* rope_sin, const int32_t* positions, int64_t rope_cols, float* acc,
                              int64_t acc_floats, int32_t* counters, int64_t n_counters, int splits,
                              uint32_t* status, void* stream) {
  AF_REQUIRE(n <= (1 << 30) && k <= (1 << 30) && m_cap <= (1 << 30), "af_linear_bf16: size too large");
  GemmCall c{};
  c.x = x;
  c.ldx = ldx;
  c.m_cap = (int)m_cap;
  c.m_dev = m_dev;
  c.w = w;
  c.n = (int)n;
  c.k = (int)k;
  c.epi = epilogue;
  c.out = out;
  c.ldo = ldo;
  c.out_rows = out_rows;
  c.res = residual;
  c.ldr = ldr;
  c.res_rows = res_rows;
  c.rope_cos = rope_cos;
  c.rope_sin = rope_sin;
  c.positions = positions;
  c.rope_cols = (int)rope_cols;
  c.head_dim = 128;
  c.acc = acc;
  c.acc_elems = acc_floats;
  c.counters = counters;
  c.counter_elems = (int)n_counters;
  c.splits = splits;
  c.status = status;
  return gemm_run(c, as_stream(stream));
}
