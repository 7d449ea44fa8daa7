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
// release ring slots; warps 2-5 drain TMEM (tcgen05.ld) into shared memory.
//
// Split-K for the narrow projections: the k-range of one output tile is split
// over the CTAs of a thread-block cluster (up to 8, along grid y), so every SM
// streams weights. Each CTA parks its fp32 partial tile in its own shared
// memory; after a cluster barrier, CTA j sums rows {lo_j..hi_j} and
// {64+lo_j..64+hi_j} over all CTAs of the cluster through distributed shared
// memory (ld.shared::cluster) and runs the epilogue for those rows (the row
// pairs r, r+64 keep RoPE and SwiGLU partners in one CTA). No global scratch,
// no atomics, a deterministic summation order.
//
// Every mbarrier wait is bounded (about one second); on timeout the CTA sets
// AF_STATUS_TIMEOUT in the status word, stops issuing, skips its stores, waits
// (bounded) for its in-flight TMA loads, frees its TMEM and returns. Cluster
// barriers are reached by every thread on every path.
#include <algorithm>
#include <mutex>
#include <vector>

#include "gemm_tc.cuh"

namespace af {

constexpr int kBlockK = 64;   // bf16 elements per k-block (one 128-byte swizzle row)
constexpr int kTileN = 128;   // weight rows per CTA (MMA M)
constexpr int kThreads = 192;
constexpr int kMaxSplits = 8; // portable cluster size
constexpr int kMaxPartialSplits = 16;  // launches that leave partials need no cluster
constexpr int kEpiTok = 256;            // tokens staged per epilogue chunk (wide token tiles take two)

struct GemmDev {
  int n, k, m_cap, ntok, n_tiles, m_tiles, nkb, kb_per_split, splits, stages;
  int w_tiled;  // 1: weights stored as contiguous 128 x 64 tiles (3-D descriptor)
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
  unsigned* status;
  float* row_sums;
  int push;      // split-K partials pushed into the owners' shared memory (else pulled over DSMEM)
  int has_side;  // CTA (0, 0, 0) runs `side` (the layer compaction) in its epilogue warps
  CompactArgs side;
  float* partial;  // split-K partials to global memory, reduced by the consumer (no cluster)
  int xbox;        // token rows per TMA box (ntok or ntok / 2)
};

__device__ __forceinline__ float bf(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Staged accumulator: tile[m * kLdt + r] (fp32, token-major) for tile row r
// (feature n0 + r) and token m; the 4-float pad keeps rows 16-byte aligned.
constexpr int kLdt = kTileN + 4;

// Split-K by push: CTA j of an S-way cluster owns tokens [j*Mv/S, (j+1)*Mv/S);
// after the staged tile, its shared memory holds S - 1 receive slots of
// ceil(ntok/S) staged rows, slot k for source k < j and k - 1 for k > j.
__host__ __device__ __forceinline__ int xch_slot_bytes(int ntok, int splits) {
  return ((ntok + splits - 1) / splits) * kLdt * 4;
}
__host__ __device__ __forceinline__ int xch_recv_bytes(int ntok, int splits) {
  return (splits - 1) * xch_slot_bytes(ntok, splits);
}

__device__ __forceinline__ void load8(const float* s, float* v) {
  const float4 x = *reinterpret_cast<const float4*>(s), y = *reinterpret_cast<const float4*>(s + 4);
  v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
  v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
}

__device__ __forceinline__ uint4 pack8(const float* y) {
  uint4 o;
  o.x = pack_bf16x2(y[0], y[1]);
  o.y = pack_bf16x2(y[2], y[3]);
  o.z = pack_bf16x2(y[4], y[5]);
  o.w = pack_bf16x2(y[6], y[7]);
  return o;
}

// Epilogues of 8 consecutive tile rows r0..r0+7 (r0 % 8 == 0) of one token,
// written as one 16-byte vector to output row `orow`. `a` holds the rows' fp32
// sums; `b` those of rows r0 ^ 64 (the RoPE rotation partner, the SwiGLU up
// rows). Every global operand (residual vector, RoPE cos/sin) is loaded by the
// caller ahead of the split-K reduction, so its latency overlaps the reads of
// the peer partial tiles.

// Plain store; returns the sum of the bf16 outputs (logit row sums).
__device__ __forceinline__ float epi_store(const GemmDev& p, int n0, int r0, int64_t orow, const float* a) {
  float y[8];
  float rs = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    y[i] = bf(a[i]);
    rs += y[i];
  }
  stg16(p.out + orow * p.ldo + n0 + r0, pack8(y));
  return rs;
}

// out = bf16(bf16(acc) + residual), residual vector `rv` (8 bf16).
__device__ __forceinline__ void epi_residual(const GemmDev& p, int n0, int r0, int64_t orow, const uint4& rv,
                                             const float* a) {
  float r[8], y[8];
  unpack<AF_DTYPE_BF16>(rv, r);
#pragma unroll
  for (int i = 0; i < 8; ++i) y[i] = __fadd_rn(r[i], bf(a[i]));
  stg16(p.out + orow * p.ldo + n0 + r0, pack8(y));
}

// out[:, (n0 >> 1) + r0 ..] = silu(bf16(gate)) * bf16(up) for gate rows r0 < 64.
__device__ __forceinline__ void epi_swiglu(const GemmDev& p, int n0, int r0, int64_t orow, const float* a,
                                           const float* b) {
  float y[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float g = bf(a[i]), u = bf(b[i]);
    // Fast exp and divide (relative error near 1e-6 here, far below the bf16
    // rounding of the product): the accurate forms made this loop math-bound.
    // For g -> -inf the quotient tends to -0, as silu does.
    const float silu = __fdividef(g, __fadd_rn(1.f, __expf(-g)));
    y[i] = __fmul_rn(silu, u);
  }
  stg16(p.out + orow * p.ldo + (n0 >> 1) + r0, pack8(y));
}

// Rotary embedding of the 8 rows (half-dimension 64, rotation partner r0 ^ 64);
// `cs` / `sn` hold cos / sin of the token's position at i0 = r0 & 63.
__device__ __forceinline__ void epi_rope(const GemmDev& p, int n0, int r0, int64_t orow, const float* a,
                                         const float* b, const float* cs, const float* sn) {
  float y[8];
  const bool second = (r0 & p.half_dim) != 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float x = bf(a[i]), other = bf(b[i]);
    y[i] = second ? __fadd_rn(__fmul_rn(x, cs[i]), __fmul_rn(other, sn[i]))
                  : __fsub_rn(__fmul_rn(x, cs[i]), __fmul_rn(other, sn[i]));
  }
  stg16(p.out + orow * p.ldo + n0 + r0, pack8(y));
}

// Global operands of one (token, chunk pair) unit: rows r0 = 8c and 8c + 64.
struct EpiOperands {
  uint4 ra, rb;         // residual vectors (EPI_RESIDUAL)
  float cs[8], sn[8];   // RoPE cos / sin (EPI_ROPE, rotated columns); shared by both rows
};

__device__ __forceinline__ void epi_operands(const GemmDev& p, int n0, int c, int rrow, int pos, EpiOperands& o) {
  if (p.epi == EPI_RESIDUAL) {
    const __nv_bfloat16* rp = p.res + (int64_t)rrow * p.ldr + n0 + 8 * c;
    o.ra = ldg16(rp);
    o.rb = ldg16(rp + 64);
  } else if (p.epi == EPI_ROPE && n0 < p.rope_cols) {
    const int i0 = (8 * c) & (p.half_dim - 1);
    load8(p.rope_cos + (int64_t)pos * p.half_dim + i0, o.cs);
    load8(p.rope_sin + (int64_t)pos * p.half_dim + i0, o.sn);
  }
}

// Both rows of a unit: r0 = 8c with partner rows `b`, and r0 + 64 with partner `a`.
__device__ __forceinline__ void epi_pair(const GemmDev& p, int n0, int c, int64_t orow, const EpiOperands& o,
                                         const float* a, const float* b) {
  const int r0 = 8 * c;
  if (p.epi == EPI_RESIDUAL) {
    epi_residual(p, n0, r0, orow, o.ra, a);
    epi_residual(p, n0, r0 + 64, orow, o.rb, b);
  } else if (p.epi == EPI_SWIGLU) {
    epi_swiglu(p, n0, r0, orow, a, b);
  } else if (p.epi == EPI_ROPE) {
    if (n0 < p.rope_cols) {
      epi_rope(p, n0, r0, orow, a, b, o.cs, o.sn);
      epi_rope(p, n0, r0 + 64, orow, b, a, o.cs, o.sn);
    } else {
      epi_store(p, n0, r0, orow, a);
      epi_store(p, n0, r0 + 64, orow, b);
    }
  } else {
    epi_store(p, n0, r0, orow, a);
    epi_store(p, n0, r0 + 64, orow, b);
  }
}

// kPair: the two CTAs of a 2-CTA cluster (adjacent weight tiles, same token
// tile and k-range) run one cta_group::2 MMA of M = 256: each streams its own
// 128 weight rows and HALF of the token tile, so a pair moves 3/4 of the
// shared-memory bytes two single CTAs would for the same MMA work (the token
// tile is as large as the weight tile at ~128 tokens). CTA 0 of the pair
// issues the MMAs; every stage's TMA loads, from both CTAs, complete on CTA
// 0's `full` barrier, and CTA 0's MMA commits arrive on both CTAs' `empty` and
// accumulator barriers.
// kWide: 512-token tiles (two 256-token MMAs per stage, epilogue in 256-token
// chunks); the narrow instantiation is the 256-token kernel unchanged.
template <bool kPair, bool kWide>
__global__ void __launch_bounds__(kThreads, 1) k_gemm_tc(const __grid_constant__ CUtensorMap tmW,
                                                          const __grid_constant__ CUtensorMap tmX, const GemmDev p) {
  extern __shared__ uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  // Grid x enumerates (weight tile, token tile) with the token tile fastest:
  // the CTAs that stream the same weight tile for different token tiles are
  // launched next to each other, so they run together and the second reads the
  // tile from L2 instead of HBM. Pairs: x = 2 (weight pair, token tile) + rank.
  const int prank = kPair ? (int)(blockIdx.x & 1) : 0;
  const int xq = kPair ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int mtile = xq % p.m_tiles, wtile = kPair ? 2 * (xq / p.m_tiles) + prank : xq / p.m_tiles;
  const bool leader = prank == 0;
  const int m0 = mtile * p.ntok;
  const int n0 = wtile * kTileN;
  const int kb0 = blockIdx.y * p.kb_per_split;
  const int nkb = min(p.kb_per_split, p.nkb - kb0);
  const int S = p.stages;
  // This CTA's token rows per stage: the whole tile, or its half of it in a pair.
  const int xrows = kPair ? (kWide ? p.ntok / 2 : p.xbox) : p.ntok;
  const uint32_t w_bytes = kTileN * kBlockK * 2, x_bytes = xrows * kBlockK * 2;
  const uint32_t stage_bytes = w_bytes + x_bytes;

  // 1024-byte aligned ring, then barriers and flags.
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bars = base + S * stage_bytes;
  const uint32_t full0 = bars, empty0 = bars + 8 * S, accb = bars + 16 * S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + S * stage_bytes + 16 * S + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + S * stage_bytes + 16 * S + 16);
  volatile int* issued_slot = reinterpret_cast<volatile int*>(gbase + S * stage_bytes + 16 * S + 24);
  const uint32_t recv_bar = bars + 16 * S + 32;  // split-K push: this CTA's receive slots are full
  const uint32_t alloc_bar = bars + 16 * S + 40;  // pair: CTA 1's TMEM is allocated (CTA 0's barrier)
  // Per-token epilogue metadata (output row, residual row, RoPE position).
  int* s_orow = reinterpret_cast<int*>(gbase + S * stage_bytes + 16 * S + 64);
  int* s_rrow = s_orow + p.ntok;
  int* s_pos = s_rrow + p.ntok;
  int* s_scan = s_pos + p.ntok;  // 32 ints: the side task's scan buffer
  const bool side_cta = p.has_side && blockIdx.x == 0 && blockIdx.y == 0;

  // Tiles start at different k-blocks (rotation by tile index) so concurrent CTAs
  // do not all read the same activation lines at the same time (a pair's two
  // CTAs stream the same k-block at every step: rotation by pair index).
  const int rot = (kPair ? wtile >> 1 : wtile) % nkb;
  auto kb_of = [&](int i) {
    int kb = i + rot;
    if (kb >= nkb) kb -= nkb;
    return kb + kb0;
  };
  // Loads complete on `bar`: this CTA's barrier, or in a pair CTA 0's (a cluster address).
  auto load_w = [&](int i, uint32_t dst, uint32_t bar) {
    if constexpr (kPair) {
      if (p.w_tiled)
        tma_load_3d_pair(dst, &tmW, bar, 0, 0, wtile * p.nkb + kb_of(i));
      else
        tma_load_2d_pair(dst, &tmW, bar, kb_of(i) * kBlockK, n0);
    } else {
      if (p.w_tiled)
        tma_load_3d(dst, &tmW, bar, 0, 0, wtile * p.nkb + kb_of(i));
      else
        tma_load_2d(dst, &tmW, bar, kb_of(i) * kBlockK, n0);
    }
  };
  auto load_x = [&](int i, uint32_t dst, uint32_t bar) {
    if constexpr (kPair && kWide) {
      // Box h of CTA r holds tokens m0 + (2h + r) * xbox: the pair's MMA h
      // (one box of each CTA) then covers tokens [2h * xbox, (2h + 2) * xbox).
      for (int h = 0; 2 * h * p.xbox < p.ntok; ++h)
        tma_load_2d_pair(dst + (uint32_t)(h * p.xbox) * (kBlockK * 2), &tmX, bar, kb_of(i) * kBlockK,
                         m0 + (2 * h + prank) * p.xbox);
    } else if constexpr (kPair) {
      tma_load_2d_pair(dst, &tmX, bar, kb_of(i) * kBlockK, m0 + prank * p.xbox);
    } else {
      for (int h = 0; h < p.ntok; h += p.xbox)
        tma_load_2d(dst + (uint32_t)h * (kBlockK * 2), &tmX, bar, kb_of(i) * kBlockK, m0 + h);
    }
  };
  // The barrier this CTA's loads of stage s complete on, and the bytes a
  // stage's phase expects (both CTAs' in a pair; armed by CTA 0 only).
  auto full_of = [&](int s) -> uint32_t {
    const uint32_t b = bars + 8u * (uint32_t)s;
    return kPair ? cluster_map(b, 0) : b;
  };
  const uint32_t w_expect = kPair ? 2 * w_bytes : w_bytes, x_expect = kPair ? 2 * x_bytes : x_bytes;
  // Stages whose weight tile is loaded before the dependency wait.
  const int npre = min(S, nkb);

  uint32_t ncols = 32;
  while ((int)ncols < p.ntok) ncols <<= 1;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(accb, 1);
    if (p.push) mbar_init(recv_bar, 1);
    if (kPair) mbar_init(alloc_bar, 1);
    *abort_flag = 0;
    *issued_slot = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmW);
    tma_prefetch_desc(&tmX);
  }
  // A pair's barriers exist in both CTAs before any load completes on CTA 0's.
  if constexpr (kPair) cluster_sync_all();
  if (threadIdx.x == 0) {
    // Weights never depend on the preceding kernel: the first ring stages are
    // filled with weight tiles, and the next k-blocks pulled into L2, while
    // that kernel may still be running. Each of these stages expects its
    // weight bytes now and is armed (arrive + activation bytes) after the wait,
    // so it cannot complete before its activation tile has landed.
    for (int i = 0; i < npre; ++i) {
      if (leader) mbar_expect_tx(full0 + 8 * i, w_expect);
      load_w(i, base + i * stage_bytes, full_of(i));
    }
    for (int i = npre; i < min(nkb, 2 * S); ++i) {
      if (p.w_tiled)
        tma_prefetch_l2_3d(&tmW, 0, 0, wtile * p.nkb + kb_of(i));
      else
        tma_prefetch_l2_2d(&tmW, kb_of(i) * kBlockK, n0);
    }
  }
  pdl_wait();
  // The activation tiles of the pre-filled stages go out at once: they need
  // no valid count (rows past it are never stored), so the count's round
  // trip overlaps them.
  if (threadIdx.x == 0) {
    for (int i = 0; i < npre; ++i) {
      if (leader) mbar_arrive_expect_tx(full0 + 8 * i, x_expect);  // weight tile already requested
      load_x(i, base + i * stage_bytes + w_bytes, full_of(i));
    }
  }
  int M = p.m_dev ? *p.m_dev : p.m_cap;
  if (M > p.m_cap) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) atomicOr(p.status, AF_STATUS_CAPACITY);
    M = p.m_cap;
  }
  if (m0 >= M) {  // uniform over a cluster (all its CTAs share the token tile)
    // No tokens for this tile (none at all for CTA (0, 0, 0)): the side task
    // still runs, with every thread of the CTA.
    if (side_cta) compact_rows<kThreads>(p.side, s_scan, threadIdx.x, 1);
    // The early loads land before the CTA exits (a pair's on CTA 0's
    // barriers: CTA 1 leaves after CTA 0 has seen them land).
    if (threadIdx.x == 0 && leader) {
      volatile int no_abort = 0;
      for (int i = 0; i < npre; ++i) mbar_wait(full0 + 8 * i, 0, &no_abort);
    }
    if constexpr (kPair) {
      __syncwarp();
      cluster_sync_all();
    }
    return;
  }
  const int Mv = min(p.ntok, M - m0);

  if (warp == 1) {
    if constexpr (kPair) {
      // CTA 0's MMAs write this CTA's TMEM: CTA 1 reports its allocation.
      tmem_alloc_pair(smem_u32(tmem_slot), ncols);
      if (!leader && lane == 0) {
        tc_fence_before();
        mbar_arrive_cluster(cluster_map(alloc_bar, 0));
      }
    } else {
      tmem_alloc(smem_u32(tmem_slot), ncols);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  float* tile = reinterpret_cast<float*>(gbase);  // staging (the ring is idle once the accumulator is final)

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer ----------------
    int i = npre;  // stages 0..npre-1 are fully requested already
    for (; i < nkb; ++i) {
      const int s = i % S;
      const uint32_t ph = (i / S) & 1;
      const uint32_t st = base + s * stage_bytes;
      if (!mbar_wait(empty0 + 8 * s, ph ^ 1, abort_flag)) {
        atomicOr(p.status, AF_STATUS_TIMEOUT);
        *abort_flag = 1;
        break;
      }
      if (leader) mbar_arrive_expect_tx(full0 + 8 * s, w_expect + x_expect);
      load_w(i, st, full_of(s));
      load_x(i, st + w_bytes, full_of(s));
    }
    *issued_slot = i;
  } else if (warp == 1 && lane == 0 && leader) {
    // ---------------- MMA issuer ----------------
    // Wide token tiles run as 256-token MMAs side by side in TMEM.
    const int nsub = kWide ? p.ntok / 256 : 1;
    const uint32_t sub_b = (uint32_t)(kPair ? p.xbox : 256) * (kBlockK * 2);  // B bytes per sub-MMA per CTA
    const uint32_t idesc = idesc_bf16(kPair ? 2 * kTileN : kTileN, kWide ? 256 : p.ntok);
    bool ready = true;
    if constexpr (kPair) {
      ready = mbar_wait(alloc_bar, 0, abort_flag);
      if (!ready) {
        atomicOr(p.status, AF_STATUS_TIMEOUT);
        *abort_flag = 1;
      }
      tc_fence_after();
    }
    for (int i = 0; i < nkb && ready; ++i) {
      const int s = i % S;
      const uint32_t ph = (i / S) & 1;
      if (!mbar_wait(full0 + 8 * s, ph, abort_flag)) {
        atomicOr(p.status, AF_STATUS_TIMEOUT);
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t st = base + s * stage_bytes;
      const uint64_t adesc = sw128_desc(st);
      if constexpr (!kWide) {
        const uint64_t bdesc = sw128_desc(st + w_bytes);
        if constexpr (kPair) {
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk)
            tc_mma_bf16_pair(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (i | kk) != 0 ? 1u : 0u);
          tc_commit_pair_both(empty0 + 8 * s);
        } else {
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk)
            tc_mma_bf16(tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (i | kk) != 0 ? 1u : 0u);
          tc_commit(empty0 + 8 * s);
        }
      } else if constexpr (kPair) {
        for (int h = 0; h < nsub; ++h) {
          const uint64_t bdesc = sw128_desc(st + w_bytes + (uint32_t)h * sub_b);
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk)
            tc_mma_bf16_pair(tmem + (uint32_t)(256 * h), adesc + 2 * kk, bdesc + 2 * kk, idesc,
                             (i | kk) != 0 ? 1u : 0u);
        }
        tc_commit_pair_both(empty0 + 8 * s);
      } else {
        for (int h = 0; h < nsub; ++h) {
          const uint64_t bdesc = sw128_desc(st + w_bytes + (uint32_t)h * sub_b);
#pragma unroll
          for (int kk = 0; kk < kBlockK / 16; ++kk)
            tc_mma_bf16(tmem + (uint32_t)(256 * h), adesc + 2 * kk, bdesc + 2 * kk, idesc, (i | kk) != 0 ? 1u : 0u);
        }
        tc_commit(empty0 + 8 * s);
      }
    }
    if constexpr (kPair) {
      tc_commit_pair_both(accb);
    } else {
      tc_commit(accb);
    }
  } else if (warp >= 2) {
    // ---------------- TMEM -> shared memory (128 threads, one tile row each) ----------------
    const int q = warp & 3;
    const int r = 32 * q + lane;
    // While the ring streams: the side task, per-token metadata into shared
    // memory, and the epilogue's global operands (residual rows, RoPE cos/sin
    // rows) into L2.
    if (side_cta) compact_rows<kThreads - 64>(p.side, s_scan, threadIdx.x - 64, 1);
    for (int m = threadIdx.x - 64; m < Mv; m += kThreads - 64) {
      const int gm = m0 + m;
      s_orow[m] = p.out_rows ? p.out_rows[gm] : gm;
      if (p.epi == EPI_RESIDUAL) {
        const int rrow = p.res_rows ? p.res_rows[gm] : gm;
        s_rrow[m] = rrow;
        const char* rp = reinterpret_cast<const char*>(p.res + (int64_t)rrow * p.ldr + n0);
        prefetch_l2(rp);
        prefetch_l2(rp + 128);
        prefetch_l2(rp + 255);
      } else if (p.epi == EPI_ROPE) {
        const int pos = p.positions[gm];
        s_pos[m] = pos;
        if (n0 < p.rope_cols) {
          const char* cp = reinterpret_cast<const char*>(p.rope_cos + (int64_t)pos * p.half_dim);
          const char* sp = reinterpret_cast<const char*>(p.rope_sin + (int64_t)pos * p.half_dim);
          for (int o = 0; o < p.half_dim * 4; o += 128) {
            prefetch_l2(cp + o);
            prefetch_l2(sp + o);
          }
        }
      }
    }
    if (!mbar_wait(accb, 0, abort_flag)) {
      atomicOr(p.status, AF_STATUS_TIMEOUT);
      *abort_flag = 1;
    }
    tc_fence_after();
    if constexpr (!kWide) {
      if (!*abort_flag) {
        // Thread r holds tile row r (TMEM lane) across the token columns; the
        // token-major staging makes a warp's 32 stores one contiguous line.
        const int nchunk = (Mv + 15) / 16;
        for (int c = 0; c < nchunk; ++c) {
          float v[16];
          tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(16 * c), v);
#pragma unroll
          for (int j = 0; j < 16; ++j) tile[(16 * c + j) * kLdt + r] = v[j];
        }
        if (p.push) fence_proxy_async_smem();  // the staged rows are read by bulk copies (async proxy)
      }
    }
  }
  // Wide tiles: tokens [t0, t0 + kEpiTok) of the accumulator into `tile` (warps 2-5):
  // thread r holds tile row r (TMEM lane) across the token columns; the
  // token-major staging makes a warp's 32 stores one contiguous line.
  auto stage = [&](int t0) {
    const int q = warp & 3;
    const int r = 32 * q + lane;
    const int nchunk = (min(kEpiTok, Mv - t0) + 15) / 16;
    for (int c = 0; c < nchunk; ++c) {
      float v[16];
      tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(t0 + 16 * c), v);
#pragma unroll
      for (int j = 0; j < 16; ++j) tile[(16 * c + j) * kLdt + r] = v[j];
    }
    if (p.push) fence_proxy_async_smem();  // the staged rows are read by bulk copies (async proxy)
  };
  if constexpr (kWide) {
    if (warp >= 2 && !*abort_flag) stage(0);
  }
  __syncthreads();
  const bool ok = !*abort_flag;

  if constexpr (!kWide) {
    if (p.partial) {
      // ---------------- split j's fp32 partial rows to global memory ----------------
      // Row m of this tile: 128 features = 512 contiguous bytes, one warp-wide
      // 16-byte store per lane; the consumer sums the splits.
      if (ok) {
        float* dst = p.partial + ((int64_t)blockIdx.y * p.m_cap + m0) * p.n + n0;
        for (int idx = threadIdx.x; idx < Mv * 32; idx += kThreads) {
          const int m = idx >> 5, c4 = idx & 31;
          *reinterpret_cast<float4*>(dst + (int64_t)m * p.n + 4 * c4) =
              *reinterpret_cast<const float4*>(tile + m * kLdt + 4 * c4);
        }
      }
    } else if (p.splits == 1) {
      if (ok && p.epi == EPI_SWIGLU) {
        // ---------------- SwiGLU: one unit per (token, gate chunk), all threads ----------------
        const int total = Mv * 8;
        for (int u = threadIdx.x; u < total; u += kThreads) {
          const int m = u >> 3, r0 = 8 * (u & 7);
          float a[8], b[8];
          load8(tile + m * kLdt + r0, a);
          load8(tile + m * kLdt + r0 + 64, b);
          epi_swiglu(p, n0, r0, s_orow[m], a, b);
        }
      } else if (ok) {
        // ---------------- units (token m, chunk pair c / c + 8), warp-uniform loop ----------------
        // Lanes 8k..8k+7 of a warp cover the 8 units of one token, so the logit
        // row sums reduce over groups of 8 lanes.
        const int total = Mv * 8;
        for (int base_u = warp * 32; base_u < total; base_u += kThreads) {
          const int u = base_u + lane;
          const bool valid = u < total;
          const int m = u >> 3, c = u & 7;
          float rs = 0.f;
          if (valid) {
            EpiOperands o;
            epi_operands(p, n0, c, p.epi == EPI_RESIDUAL ? s_rrow[m] : 0, p.epi == EPI_ROPE ? s_pos[m] : 0, o);
            float a[8], b[8];
            load8(tile + m * kLdt + 8 * c, a);
            load8(tile + m * kLdt + 8 * c + 64, b);
            if (p.epi == EPI_STORE) {
              rs = epi_store(p, n0, 8 * c, s_orow[m], a);
              rs += epi_store(p, n0, 8 * c + 64, s_orow[m], b);
            } else {
              epi_pair(p, n0, c, s_orow[m], o, a, b);
            }
          }
          if (p.row_sums) {
            rs += __shfl_xor_sync(0xffffffffu, rs, 1);
            rs += __shfl_xor_sync(0xffffffffu, rs, 2);
            rs += __shfl_xor_sync(0xffffffffu, rs, 4);
            if (valid && (lane & 7) == 0) atomicAdd(p.row_sums + s_orow[m], rs);
          }
        }
      }
    } else {
      // ---------------- cluster split-K reduction ----------------
      // CTA j owns tokens [tlo, thi) and sums their units (token m, chunk pair
      // c / c + 8: rows 8c..8c+7 and their partners 64+8c..64+8c+7) over every
      // CTA of the cluster in a fixed source order. The other CTAs' partial rows
      // of those tokens are either pushed into this CTA's receive slots by bulk
      // copies (push) or read from their shared memory (pull); the sums are the
      // same. Per unit the global operands are requested first, then every
      // source's partials (up to 4 in flight), so their latencies overlap.
      const int j = blockIdx.y, Sp = p.splits;
      const int tlo = (j * Mv) / Sp, thi = ((j + 1) * Mv) / Sp;
      const int lo = tlo * 8, hi = thi * 8;
      const uint32_t row_b = kLdt * 4;
      const uint32_t recv_off = (uint32_t)(p.ntok * kLdt * 4);
      const uint32_t slot_b = (uint32_t)xch_slot_bytes(p.ntok, Sp);
      if (p.push && threadIdx.x == 0)
        mbar_arrive_expect_tx(recv_bar, (uint32_t)((Sp - 1) * (thi - tlo)) * row_b);
      __syncwarp();
      cluster_sync_all();  // every partial tile is staged, every receive barrier armed, every ring idle
      bool got = true;
      if (p.push) {
        if (threadIdx.x == 0)
          for (int k = 0; k < Sp; ++k) {
            const int klo = (k * Mv) / Sp, khi = ((k + 1) * Mv) / Sp;
            if (k == j || khi <= klo) continue;
            const uint32_t dst = cluster_map(base + recv_off + (uint32_t)(j < k ? j : j - 1) * slot_b, (uint32_t)k);
            bulk_copy_s2c(dst, base + (uint32_t)klo * row_b, (uint32_t)(khi - klo) * row_b, cluster_map(recv_bar, (uint32_t)k));
          }
        volatile int no_abort = 0;
        got = mbar_wait(recv_bar, 0, &no_abort);
        if (!got && threadIdx.x == 0) atomicOr(p.status, AF_STATUS_TIMEOUT);
      }
      if (ok && got) {
        for (int u = lo + threadIdx.x; u < hi; u += kThreads) {
          const int m = u >> 3, c = u & 7;
          EpiOperands o;
          epi_operands(p, n0, c, p.epi == EPI_RESIDUAL ? s_rrow[m] : 0, p.epi == EPI_ROPE ? s_pos[m] : 0, o);
          const uint32_t oa = base + (uint32_t)((m * kLdt + 8 * c) * 4);
          const uint32_t ob = oa + 64 * 4;
          float sa[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, sb[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          for (int s0 = 0; s0 < Sp; s0 += 4) {
            float4 v[4][4];
  #pragma unroll
            for (int q = 0; q < 4; ++q) {
              if (s0 + q < Sp) {
                const int src = s0 + q;
                if (p.push) {
                  const float* t = src == j ? tile + m * kLdt + 8 * c
                                            : reinterpret_cast<const float*>(gbase + recv_off + (src < j ? src : src - 1) * slot_b +
                                                                             (m - tlo) * row_b) + 8 * c;
                  v[q][0] = *reinterpret_cast<const float4*>(t);
                  v[q][1] = *reinterpret_cast<const float4*>(t + 4);
                  v[q][2] = *reinterpret_cast<const float4*>(t + 64);
                  v[q][3] = *reinterpret_cast<const float4*>(t + 68);
                } else {
                  v[q][0] = ld_cluster_f4(cluster_map(oa, (uint32_t)src));
                  v[q][1] = ld_cluster_f4(cluster_map(oa + 16, (uint32_t)src));
                  v[q][2] = ld_cluster_f4(cluster_map(ob, (uint32_t)src));
                  v[q][3] = ld_cluster_f4(cluster_map(ob + 16, (uint32_t)src));
                }
              }
            }
  #pragma unroll
            for (int q = 0; q < 4; ++q) {
              if (s0 + q < Sp) {
                sa[0] += v[q][0].x; sa[1] += v[q][0].y; sa[2] += v[q][0].z; sa[3] += v[q][0].w;
                sa[4] += v[q][1].x; sa[5] += v[q][1].y; sa[6] += v[q][1].z; sa[7] += v[q][1].w;
                sb[0] += v[q][2].x; sb[1] += v[q][2].y; sb[2] += v[q][2].z; sb[3] += v[q][2].w;
                sb[4] += v[q][3].x; sb[5] += v[q][3].y; sb[6] += v[q][3].z; sb[7] += v[q][3].w;
              }
            }
          }
          epi_pair(p, n0, c, s_orow[m], o, sa, sb);
        }
      }
      __syncwarp();
      // Pull: peers may still read this CTA's partial tile until here. Push:
      // every CTA has received its slots, so this CTA's outgoing copies are done.
      cluster_sync_all();
    }
  } else {
    // A wide tile's launch has one split or leaves partials (no cluster reduction).
    if (p.partial || p.splits == 1) {
     // Wide token tiles are staged and stored kEpiTok tokens at a time (token
     // m of the tile is row m - t0 of the staged chunk).
     for (int t0 = 0;;) {
      const int tn = min(kEpiTok, Mv - t0);
      if (p.partial) {
        // ---------------- split j's fp32 partial rows to global memory ----------------
        // Row m of this tile: 128 features = 512 contiguous bytes, one warp-wide
        // 16-byte store per lane; the consumer sums the splits.
        if (ok) {
          float* dst = p.partial + ((int64_t)blockIdx.y * p.m_cap + m0) * p.n + n0;
          for (int idx = threadIdx.x; idx < tn * 32; idx += kThreads) {
            const int m = t0 + (idx >> 5), c4 = idx & 31;
            *reinterpret_cast<float4*>(dst + (int64_t)m * p.n + 4 * c4) =
                *reinterpret_cast<const float4*>(tile + (m - t0) * kLdt + 4 * c4);
          }
        }
      } else if (ok && p.epi == EPI_SWIGLU) {
        // ---------------- SwiGLU: one unit per (token, gate chunk), all threads ----------------
        const int total = tn * 8;
        for (int u = threadIdx.x; u < total; u += kThreads) {
          const int m = t0 + (u >> 3), r0 = 8 * (u & 7);
          float a[8], b[8];
          load8(tile + (m - t0) * kLdt + r0, a);
          load8(tile + (m - t0) * kLdt + r0 + 64, b);
          epi_swiglu(p, n0, r0, s_orow[m], a, b);
        }
      } else if (ok) {
        // ---------------- units (token m, chunk pair c / c + 8), warp-uniform loop ----------------
        // Lanes 8k..8k+7 of a warp cover the 8 units of one token, so the logit
        // row sums reduce over groups of 8 lanes.
        const int total = tn * 8;
        for (int base_u = warp * 32; base_u < total; base_u += kThreads) {
          const int u = base_u + lane;
          const bool valid = u < total;
          const int m = t0 + (u >> 3), c = u & 7;
          float rs = 0.f;
          if (valid) {
            EpiOperands o;
            epi_operands(p, n0, c, p.epi == EPI_RESIDUAL ? s_rrow[m] : 0, p.epi == EPI_ROPE ? s_pos[m] : 0, o);
            float a[8], b[8];
            load8(tile + (m - t0) * kLdt + 8 * c, a);
            load8(tile + (m - t0) * kLdt + 8 * c + 64, b);
            if (p.epi == EPI_STORE) {
              rs = epi_store(p, n0, 8 * c, s_orow[m], a);
              rs += epi_store(p, n0, 8 * c + 64, s_orow[m], b);
            } else {
              epi_pair(p, n0, c, s_orow[m], o, a, b);
            }
          }
          if (p.row_sums) {
            rs += __shfl_xor_sync(0xffffffffu, rs, 1);
            rs += __shfl_xor_sync(0xffffffffu, rs, 2);
            rs += __shfl_xor_sync(0xffffffffu, rs, 4);
            if (valid && (lane & 7) == 0) atomicAdd(p.row_sums + s_orow[m], rs);
          }
        }
      }
      t0 += kEpiTok;
      if (t0 >= Mv) break;
      __syncthreads();  // every thread is done with the staged chunk
      if (warp >= 2 && ok) stage(t0);
      __syncthreads();
     }
    }
  }

  if (threadIdx.x == 0 && leader && *abort_flag) {
    // Drain TMA loads that may still be in flight into the ring (bounded; a
    // pair's loads all complete on CTA 0's barriers).
    const int issued = *issued_slot;
    volatile int no_abort = 0;
    for (int i = max(0, issued - S); i < issued; ++i) mbar_wait(full0 + 8 * (i % S), (i / S) & 1, &no_abort);
  }
  __syncthreads();
  if constexpr (kPair) {
    // Neither CTA leaves while the other may still signal its barriers or
    // read its shared memory (CTA 0's MMAs; CTA 1's loads onto CTA 0's barriers).
    tc_fence_before();
    cluster_sync_all();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc_pair(tmem, ncols);
    }
  } else {
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem, ncols);
    }
  }
}

// Rows finished from split-K partials: the epilogue of k_gemm_tc (RoPE,
// residual or plain store) applied to the sum of the splits' fp32 partial
// tiles, added in split order 0, 1, ... like the cluster reduction. One
// thread per unit (row m, chunk pair c / c + 8 of a 128-column tile): 32 rows
// of one tile per CTA. The partials and the row's indices are requested
// together with the valid count (m < m_cap keeps every read in bounds).
__global__ void __launch_bounds__(256) k_gemm_finish(const GemmDev p) {
  pdl_trigger();
  pdl_wait();
  const int n0 = blockIdx.x * kTileN;
  const int m = blockIdx.y * 32 + (int)(threadIdx.x >> 3), c = threadIdx.x & 7;
  if (m >= p.m_cap) return;
  const int pos = p.epi == EPI_ROPE ? p.positions[m] : 0;
  const int orow = p.out_rows ? p.out_rows[m] : m;
  const int rrow = p.epi == EPI_RESIDUAL && p.res_rows ? p.res_rows[m] : m;
  const int M = p.m_dev ? min(*p.m_dev, p.m_cap) : p.m_cap;
  const float* src = p.partial + (int64_t)m * p.n + n0 + 8 * c;
  const int64_t split_stride = (int64_t)p.m_cap * p.n;
  float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, b[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int s0 = 0; s0 < p.splits; s0 += 4) {
    float4 v[4][4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (s0 + q < p.splits) {
        const float4* t = reinterpret_cast<const float4*>(src + (s0 + q) * split_stride);
        v[q][0] = t[0];
        v[q][1] = t[1];
        v[q][2] = t[16];
        v[q][3] = t[17];
      }
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (s0 + q < p.splits) {
        a[0] += v[q][0].x; a[1] += v[q][0].y; a[2] += v[q][0].z; a[3] += v[q][0].w;
        a[4] += v[q][1].x; a[5] += v[q][1].y; a[6] += v[q][1].z; a[7] += v[q][1].w;
        b[0] += v[q][2].x; b[1] += v[q][2].y; b[2] += v[q][2].z; b[3] += v[q][2].w;
        b[4] += v[q][3].x; b[5] += v[q][3].y; b[6] += v[q][3].z; b[7] += v[q][3].w;
      }
  }
  if (m >= M) return;
  EpiOperands o;
  epi_operands(p, n0, c, rrow, pos, o);
  epi_pair(p, n0, c, orow, o, a, b);
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

int make_tmap_bf16_tiled(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols) {
  PFN_encodeTiled_t fn = encode_fn();
  if (!fn) return fail(AF_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || rows % 128 || cols % 64)
    return fail(AF_ERR_ARG, "tiled weight must be 16-byte aligned with 128-row / 64-column multiples");
  const cuuint64_t gdim[3] = {64, 128, (rows / 128) * (cols / 64)};
  const cuuint64_t gstride[2] = {128, 128 * 128};  // bytes: tile row, tile
  const cuuint32_t box[3] = {64, 128, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), gdim, gstride, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AF_ERR_CUDA, "cuTensorMapEncodeTiled (tiled) failed (" + std::to_string((int)r) + ")");
  return AF_OK;
}

int make_tmap_bf16_heads(CUtensorMap* map, const void* base, uint64_t rows, uint64_t depth) {
  PFN_encodeTiled_t fn = encode_fn();
  if (!fn) return fail(AF_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (reinterpret_cast<uintptr_t>(base) & 15u) return fail(AF_ERR_ARG, "head-major K/V must be 16-byte aligned");
  const cuuint64_t gdim[3] = {128, rows, depth};
  const cuuint64_t gstride[2] = {256, rows * 256};  // bytes: row, matrix
  const cuuint32_t box[3] = {64, 128, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), gdim, gstride, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AF_ERR_CUDA, "cuTensorMapEncodeTiled (heads) failed (" + std::to_string((int)r) + ")");
  return AF_OK;
}

// Row capacities that are multiples of 512 (>= 1024) take 512-token tiles
// where their (weight tile, token tile) CTAs fill at least two waves of one
// CTA per SM: two 256-token MMAs per stage, staged and stored 256 tokens at a
// time, so every weight and activation byte loaded into shared memory feeds
// twice the MMA work of a 256-token tile (measured on B200 at 1024 rows:
// gate/up -21 %, LM head -15 %; fewer CTAs, e.g. QKV's 192, lose more to the
// partly filled last wave than they gain). ACTFOLD_GEMM_WIDE=0 turns it off.
static bool gemm_wide() {
  static const bool on = [] {
    const char* e = getenv("ACTFOLD_GEMM_WIDE");
    return !(e && e[0] == '0');
  }();
  return on;
}

int gemm_ntok(int m_cap, int n) {
  if (gemm_wide() && m_cap >= 1024 && m_cap % 512 == 0 && (n / kTileN) * (m_cap / 512) >= 2 * sm_count()) return 512;
  const int mt = (m_cap + 255) / 256;
  int nt = (m_cap + mt - 1) / mt;
  nt = (nt + 15) / 16 * 16;
  return nt < 16 ? 16 : nt;
}

int gemm_xbox(int ntok) { return ntok > 256 ? 128 : (ntok % 32 == 0 ? ntok / 2 : ntok); }

// Paired-CTA launches (tuning override ACTFOLD_GEMM_PAIR=0 keeps single CTAs).
static bool pair_off() {
  static const bool off = [] {
    const char* e = getenv("ACTFOLD_GEMM_PAIR");
    return e && e[0] == '0';
  }();
  return off;
}

struct GemmShape {
  int ntok, m_tiles, n_tiles, nkb, splits, kb_per, stages, smem;
  int push;  // split-K partials pushed into the owners' shared memory (bulk copies)
  int pair;  // CTA pairs (cta_group::2): adjacent weight tiles share one M = 256 MMA
};

// Tuning override of the k-splits of launches that leave partials (0: the heuristic).
static int env_partial_splits() {
  static const int v = [] {
    const char* e = getenv("ACTFOLD_PARTIAL_SPLITS");
    return e ? atoi(e) : 0;
  }();
  return v;
}

static GemmShape plan_shape(int n, int k, int m_cap, int want_splits, bool row_sums, bool partial = false) {
  GemmShape g;
  g.ntok = gemm_ntok(m_cap, n);
  g.m_tiles = (m_cap + g.ntok - 1) / g.ntok;
  g.n_tiles = n / kTileN;
  g.nkb = k / kBlockK;
  static const int env_stages = [] {
    const char* e = getenv("ACTFOLD_GEMM_STAGES");  // tuning override of the ring depth
    return e ? atoi(e) : 0;
  }();
  const int tiles = g.n_tiles * g.m_tiles;
  int splits = want_splits;
  if (splits <= 0 && partial && env_partial_splits() > 0) splits = env_partial_splits();
  if (splits <= 0 && partial && g.ntok >= 256) {
    // Tensor-bound token tiles leaving partials: at most one CTA per SM.
    // Every split adds a partial slice that the next row kernel reads, and at
    // 512 rows two splits of the O / down projections beat three and four
    // (measured on B200: d = 64 at 512 tokens 12.08 -> 11.3 ms, 32 children
    // 13.7 -> 13.2 ms; one split 12.7 ms).
    splits = std::max(1, std::min(4, sm_count() / tiles));
  } else if (splits <= 0) {
    // About 4/3 CTAs per SM, at most 4 splits: measured on B200 for the
    // LLaDA/Dream projections, more and shorter split CTAs lose more to their
    // ramp-up and cluster reduction than they gain in parallel streams.
    splits = (4 * sm_count()) / (3 * tiles);
    splits = std::max(1, std::min(splits, 4));
    splits = std::min(splits, std::max(1, g.nkb / 4));
  }
  if (partial) splits = std::min(splits, kMaxPartialSplits);
  if (row_sums) splits = 1;
  if (!partial) splits = std::min(splits, kMaxSplits);
  if (g.ntok > 256 && !partial) splits = 1;  // a wide tile's epilogue has no cluster reduction
  g.kb_per = (g.nkb + splits - 1) / splits;
  g.splits = (g.nkb + g.kb_per - 1) / g.kb_per;
  // CTA pairs need an even number of weight tiles, a token tile that halves
  // into 16-row multiples, and no exchange between split CTAs (their cluster
  // is the pair).
  g.pair = !pair_off() && g.n_tiles % 2 == 0 && g.ntok % 32 == 0 && (g.splits == 1 || partial) ? 1 : 0;
  const int stage = kTileN * kBlockK * 2 + (g.pair ? g.ntok / 2 : g.ntok) * kBlockK * 2;
  // A CTA streams at most (bytes its ring keeps in flight) / (load latency):
  // a launch whose CTAs all fit one per SM and stream long k-ranges (the down
  // projection) gets the deepest ring that fits; otherwise ~100 KB rings let
  // two CTAs share an SM.
  const bool one_per_sm = (tiles * g.splits <= sm_count() && g.kb_per >= 24) || g.ntok > 256;
  int st = (one_per_sm ? 220 * 1024 : 100 * 1024) / stage;
  if (env_stages > 0) st = env_stages;
  st = std::max(2, std::min(16, st));
  const int tile_bytes = std::min(g.ntok, kEpiTok) * kLdt * 4;  // fp32 staging of the accumulator (one chunk)
  while (st * stage < tile_bytes) ++st;
  // Ring + alignment slack + barriers/flags + per-token metadata (3 ints per
  // token) + the side task's 32-int scan buffer.
  auto smem_of = [&](int stages) { return stages * stage + 1024 + 16 * stages + 64 + 12 * g.ntok + 128; };
  while (st > 2 && smem_of(st) > 227 * 1024 && (st - 1) * stage >= tile_bytes) --st;
  // Split-K by push: the owners' receive slots follow the staged tile in the
  // idle ring. Used when they fit, or when a deeper ring costs nothing (one
  // CTA per SM); otherwise the owners pull the partials over DSMEM.
  g.push = 0;
  if (g.splits > 1) {
    const int need = tile_bytes + xch_recv_bytes(g.ntok, g.splits);
    int st2 = st;
    if (tiles * g.splits <= sm_count())
      while (st2 * stage < need && smem_of(st2 + 1) <= 227 * 1024) ++st2;
    if (st2 * stage >= need) {
      g.push = 1;
      st = st2;
    }
  }
  g.stages = st;
  g.smem = smem_of(st);
  return g;
}

int gemm_splits(int n, int k, int m_cap, bool partial) { return plan_shape(n, k, m_cap, 0, false, partial).splits; }

int gemm_run(const GemmCall& c, cudaStream_t stream) {
  AF_REQUIRE(c.x && c.w && c.out && c.status, "gemm: null pointer");
  AF_REQUIRE(c.n > 0 && c.n % kTileN == 0, "gemm: n must be a positive multiple of 128");
  AF_REQUIRE(c.k > 0 && c.k % kBlockK == 0, "gemm: k must be a positive multiple of 64");
  AF_REQUIRE(c.m_cap > 0, "gemm: m_cap must be positive");
  AF_REQUIRE(c.epi >= EPI_STORE && c.epi <= EPI_ROPE, "gemm: bad epilogue");
  AF_REQUIRE(c.ldo % 8 == 0 && (reinterpret_cast<uintptr_t>(c.out) & 15u) == 0,
             "gemm: out must be 16-byte aligned with a row stride that is a multiple of 8");
  AF_REQUIRE(!c.res || (c.ldr % 8 == 0 && (reinterpret_cast<uintptr_t>(c.res) & 15u) == 0),
             "gemm: residual must be 16-byte aligned with a row stride that is a multiple of 8");
  AF_REQUIRE(c.epi != EPI_RESIDUAL || c.res, "gemm: residual epilogue needs res");
  AF_REQUIRE(c.epi != EPI_ROPE || (c.rope_cos && c.rope_sin && c.positions && c.head_dim == 128 && c.rope_cols % 128 == 0),
             "gemm: rope epilogue needs cos/sin/positions and head_dim 128");
  const bool partial = c.partial_out != nullptr;  // the caller asks for partials (also with one split)
  GemmShape g = plan_shape(c.n, c.k, c.m_cap, c.splits, c.row_sums != nullptr, partial);
  AF_REQUIRE(!partial || (reinterpret_cast<uintptr_t>(c.partial_out) & 15u) == 0, "gemm: partial_out must be 16-byte aligned");
  if (partial) g.push = 0;  // no exchange between the splits: no receive slots in shared memory
  AF_REQUIRE(!g.pair || g.splits == 1 || partial, "gemm: CTA pairs cannot exchange split-K partials");
  AF_REQUIRE(g.ntok <= 256 || g.splits == 1 || partial, "gemm: wide token tiles need one split or partials");
  AF_REQUIRE(g.smem <= 227 * 1024, "gemm: shared memory budget exceeded");

  CUtensorMap tw, tx;
  const CUtensorMap* pw = c.tmap_w;
  const CUtensorMap* px = c.tmap_x;
  if (!pw) {
    int st = c.w_tiled ? make_tmap_bf16_tiled(&tw, c.w, c.n, c.k) : make_tmap_bf16(&tw, c.w, c.n, c.k, c.k, kTileN);
    if (st) return st;
    pw = &tw;
  }
  if (!px) {
    int st = make_tmap_bf16(&tx, c.x, c.m_cap, c.k, c.ldx, gemm_xbox(g.ntok));
    if (st) return st;
    px = &tx;
  }
  GemmDev d;
  d.n = c.n;
  d.k = c.k;
  d.m_cap = c.m_cap;
  d.ntok = g.ntok;
  d.n_tiles = g.n_tiles;
  d.m_tiles = g.m_tiles;
  d.nkb = g.nkb;
  d.kb_per_split = g.kb_per;
  d.splits = g.splits;
  d.stages = g.stages;
  d.w_tiled = c.w_tiled ? 1 : 0;
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
  d.status = c.status;
  d.row_sums = c.epi == EPI_STORE ? c.row_sums : nullptr;
  d.push = g.push;
  d.has_side = c.has_side;
  d.side = c.side;
  d.partial = partial ? c.partial_out : nullptr;
  d.xbox = gemm_xbox(g.ntok);

  static std::once_flag attr_once;
  std::call_once(attr_once, [] {
    cudaFuncSetAttribute(k_gemm_tc<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    cudaFuncSetAttribute(k_gemm_tc<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    cudaFuncSetAttribute(k_gemm_tc<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    cudaFuncSetAttribute(k_gemm_tc<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  });
  // Tensor maps built elsewhere (c.tmap_x) use box rows gemm_xbox(ntok).
  const dim3 grid(g.n_tiles * g.m_tiles, g.splits, 1), block(kThreads, 1, 1);
  const dim3 cl_pair(2, 1, 1), cl_one(1, partial ? 1 : g.splits, 1);
  const bool wide = g.ntok > 256;
  cudaError_t e =
      g.pair ? (wide ? launch_ex(k_gemm_tc<true, true>, grid, block, (size_t)g.smem, stream, c.pdl != 0, cl_pair, *pw, *px, d)
                     : launch_ex(k_gemm_tc<true, false>, grid, block, (size_t)g.smem, stream, c.pdl != 0, cl_pair, *pw, *px, d))
             : (wide ? launch_ex(k_gemm_tc<false, true>, grid, block, (size_t)g.smem, stream, c.pdl != 0, cl_one, *pw, *px, d)
                     : launch_ex(k_gemm_tc<false, false>, grid, block, (size_t)g.smem, stream, c.pdl != 0, cl_one, *pw, *px, d));
  if (e != cudaSuccess) return fail(AF_ERR_CUDA, std::string("gemm_tc launch: ") + cudaGetErrorString(e));
  return check_launch("gemm_tc");
}

int gemm_finish_run(const GemmCall& c, int splits, cudaStream_t stream) {
  AF_REQUIRE(c.partial_out && c.out && c.status, "gemm_finish: null pointer");
  AF_REQUIRE(c.n > 0 && c.n % kTileN == 0 && c.m_cap > 0, "gemm_finish: bad shape");
  AF_REQUIRE(splits >= 1 && splits <= kMaxPartialSplits, "gemm_finish: bad split count");
  AF_REQUIRE(c.epi >= EPI_STORE && c.epi <= EPI_ROPE && c.epi != EPI_SWIGLU && !c.row_sums,
             "gemm_finish: store, residual or RoPE epilogue without row sums");
  AF_REQUIRE(c.epi != EPI_RESIDUAL || c.res, "gemm_finish: residual epilogue needs res");
  AF_REQUIRE(c.epi != EPI_ROPE || (c.rope_cos && c.rope_sin && c.positions && c.head_dim == 128 && c.rope_cols % 128 == 0),
             "gemm_finish: rope epilogue needs cos/sin/positions and head_dim 128");
  GemmDev d{};
  d.n = c.n;
  d.k = c.k;
  d.m_cap = c.m_cap;
  d.m_dev = c.m_dev;
  d.splits = splits;
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
  d.status = c.status;
  d.partial = c.partial_out;
  cudaError_t e = launch_ex(k_gemm_finish, dim3(c.n / kTileN, (c.m_cap + 31) / 32, 1), dim3(256, 1, 1), 0, stream,
                            c.pdl != 0, dim3(1, 1, 1), d);
  if (e != cudaSuccess) return fail(AF_ERR_CUDA, std::string("gemm_finish launch: ") + cudaGetErrorString(e));
  return check_launch("gemm_finish");
}

}  // namespace af

using namespace af;

extern "C" int af_linear_bf16(const void* x, int64_t ldx, int64_t m_cap, const int32_t* m_dev, const void* w,
                              int64_t n, int64_t k, int w_layout, int epilogue, void* out, int64_t ldo,
                              const int32_t* out_rows, const void* residual, int64_t ldr, const int32_t* res_rows,
                              const float* rope_cos, const float* rope_sin, const int32_t* positions,
                              int64_t rope_cols, int splits, uint32_t* status, void* stream) {
  AF_REQUIRE(n <= (1 << 30) && k <= (1 << 30) && m_cap <= (1 << 30), "af_linear_bf16: size too large");
  AF_REQUIRE(splits >= 0 && splits <= kMaxSplits, "af_linear_bf16: splits must be in [0, 8]");
  AF_REQUIRE(w_layout == 0 || w_layout == 1, "af_linear_bf16: w_layout must be 0 (row-major) or 1 (tiled)");
  GemmCall c;
  memset(&c, 0, sizeof(c));
  c.w_tiled = w_layout;
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
  c.splits = splits;
  c.status = status;
  return gemm_run(c, as_stream(stream));
}
