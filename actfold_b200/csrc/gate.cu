// Similarity gate with fused stream compaction (sm_100a).
//
// One warp per token row of up to 64 16-byte vectors, one 256-thread CTA per
// longer row (up to 512 vectors: H <= 4096 bf16 or 2048 f32), and for a bf16
// cosine gate against one parent row shared by every child, one CTA per
// position and 8 children. The row is loaded once with 128-bit non-coherent
// loads into registers, then reduced twice from registers (norms, then
// normalized products) with shuffle / block sums in fp32. Larger or unaligned
// rows use a scalar path that re-reads the row.
//
// Numerics follow the reference gate (actfold/core/similarity_gate.py:76-103
// -> ATen cosine_similarity): for reduced-precision inputs every elementwise
// op is evaluated in fp32 and rounded to the input dtype, reductions
// accumulate in fp32 and round once. The per-element quotient bf16(x / n)
// is formed as x * (1/n) and recomputed with a true IEEE division whenever the
// fp32 product lies within 4 ulp of a bf16 rounding midpoint, so the bf16
// result equals bf16(fp32(x / n)) exactly.
#include "gate_row.cuh"
#include "tc_common.cuh"

namespace af {

struct GateParams {
  const char* child;
  const char* parent;
  int64_t c_bs, c_ts, p_bs, p_ts;
  int64_t rows, T;
  int H, nvec;
  GateConsts k;
  uint8_t* mask;
  int64_t m_bs;
  float* sim;
};

template <int DT, int METRIC, int NV>
__global__ void __launch_bounds__(256) k_gate_vec(const GateParams p) {
  pdl_trigger();  // the compaction kernel may launch now; it waits for this grid
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int64_t b = row / p.T, t = row - b * p.T;
  const char* c = p.child + b * p.c_bs + t * p.c_ts;
  const char* q = p.parent + b * p.p_bs + t * p.p_ts;
  GateOut r = gate_row_vec<DT, METRIC, NV>(c, q, p.nvec, p.H, p.k, lane);
  if (lane == 0) {
    p.mask[b * p.m_bs + t] = r.stable;
    if (p.sim) p.sim[row] = r.sim;
  }
}

// Rows of more than 64 16-byte vectors (bf16 H > 512): one CTA of
// kGateRowThreads threads per row, at most two vectors per thread per tensor,
// and block reductions. With a warp per row such rows keep up to 128 values
// per lane in registers and add them in one dependent chain, which caps the
// kernel far below HBM speed (one CTA per SM, latency bound). 256 threads
// (two vectors each at H = 4096) keep enough CTAs resident per SM for the
// broadcast kernel's streaming; the folded pass's in-pass gates use
// 512-thread rows instead (their latency, not their bandwidth, is what
// counts there), so the two may add a row's squares in different orders.
constexpr int kGateRowThreads = 256;

template <int DT, int METRIC, int NV>
__global__ void __launch_bounds__(kGateRowThreads) k_gate_row(const GateParams p) {
  pdl_trigger();  // the compaction kernel may launch now; it waits for this grid
  __shared__ __align__(16) float red[2 * kGateRowThreads / 32];
  const int64_t row = blockIdx.x;
  if (row >= p.rows) return;
  const int64_t b = row / p.T, t = row - b * p.T;
  uint4 cv[NV], pv[NV];
  load_row<NV, kGateRowThreads>(p.child + b * p.c_bs + t * p.c_ts, p.nvec, threadIdx.x, cv);
  load_row<NV, kGateRowThreads>(p.parent + b * p.p_bs + t * p.p_ts, p.nvec, threadIdx.x, pv);
  GateOut r;
  if constexpr (DT == AF_DTYPE_BF16 && METRIC == AF_METRIC_COSINE)
    r = gate_regs_bf16_cos<NV>(cv, pv, p.nvec, p.k, threadIdx.x, CtaRows<kGateRowThreads>{red});
  else
    r = gate_regs<DT, METRIC, NV>(cv, pv, p.nvec, p.H, p.k, threadIdx.x, CtaRows<kGateRowThreads>{red});
  if (threadIdx.x == 0) {
    p.mask[b * p.m_bs + t] = r.stable;
    if (p.sim) p.sim[row] = r.sim;
  }
}

// bf16 cosine gate of children against ONE parent row per position (parent
// batch stride 0, the cached parent broadcast over the children): CTA
// (t, chunk) takes position t for kBcastChildren children. The parent row is
// loaded and normalised once (kept as bf16x2 words). The children's rows
// stream through a ring of kBcastRing shared-memory slots filled by bulk
// copies (one per row, completing on the slot's mbarrier), so up to
// kBcastRing rows per CTA are in flight whatever the register budget.
//
// The per-element chain runs on packed pairs, so the instruction count per
// element roughly halves (the kernel was bound by instruction issue): x^2
// sums and x * (1/n) as fp32x2 FMA / MUL, the two quotients rounded to bf16 by
// one cvt.rn.bf16x2, both products y_c * y_p by one mul.rn.bf16x2, and the
// products added into two fp32 accumulators (even and odd elements) by one
// fp32x2 add. The rounding points are the reference's: a product of two bf16
// values is exact in fp32, so rounding it once to bf16 equals rnd(fp32
// product); x * (1/n) rounds to the same bf16 as x / n (rcp_for_bf16_quot)
// except where x / n is an fp32 subnormal, and such products (and any
// product below 2^-126) are too small to change a similarity sum of normal
// size. Only the order of the fp32 additions differs from the reference's
// (whose order is ATen's), as it does for every other gate kernel here.
constexpr int kBcastChildren = 8;
constexpr int kBcastRing = 3;
// 128 threads per row: with the packed chain the block reductions and the
// per-row steps (square root, reciprocal, ring wait, outputs) are a large
// share of the instructions, and 32 elements per thread halve it against 256
// threads (the kernel is bound by instruction issue).
constexpr int kBcastThreads = 128;

__device__ __forceinline__ void bulk_load_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

template <int NV>
__global__ void __launch_bounds__(kBcastThreads) k_gate_bcast(const GateParams p) {
  pdl_trigger();  // the compaction kernel may launch now; it waits for this grid
  constexpr int G = kBcastThreads;
  extern __shared__ __align__(128) uint4 ring[];  // [kBcastRing][nvec] child rows
  __shared__ __align__(16) float red[2 * G / 32];
  __shared__ __align__(8) uint64_t full[kBcastRing];
  __shared__ volatile int fail;
  const CtaRows<G> rows{red};
  const int tid = threadIdx.x;
  const int64_t t = blockIdx.x;
  const int64_t B = p.rows / p.T;
  const int64_t b0 = (int64_t)blockIdx.y * kBcastChildren;
  const int64_t b1 = min(B, b0 + kBcastChildren);
  if (t >= p.T || b0 >= B) return;
  const int nb = (int)(b1 - b0);
  const uint32_t row_bytes = (uint32_t)p.nvec * 16u;
  auto issue = [&](int k) {  // child b0 + k into slot k % kBcastRing (thread 0)
    const uint32_t bar = smem_u32(&full[k % kBcastRing]);
    mbar_arrive_expect_tx(bar, row_bytes);
    bulk_load_g2s(smem_u32(ring + (k % kBcastRing) * p.nvec), p.child + (b0 + k) * p.c_bs + t * p.c_ts, row_bytes,
                  bar);
  };
  if (tid == 0) {
    for (int s = 0; s < kBcastRing; ++s) mbar_init(smem_u32(&full[s]), 1);
    fail = 0;
    fence_barrier_init();
    for (int k = 0; k < min(kBcastRing, nb); ++k) issue(k);
  }
  uint4 pv[NV];
  load_row<NV, G>(p.parent + t * p.p_ts, p.nvec, tid, pv);
  // Parent: norm and normalised values (bf16x2 words), once.
  uint32_t yp[NV][4];
  {
    float fp[NV][8];
    float sp = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      unpack<AF_DTYPE_BF16>(pv[i], fp[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) sp = fmaf(fp[i][e], fp[i][e], sp);
    }
    sp = rows.sum(sp);  // its barriers also publish the ring's barrier set-up
    float np = rnd<AF_DTYPE_BF16>(__fsqrt_rn(sp));
    np = np < p.k.eps_r ? p.k.eps_r : np;  // clamp_min keeps NaN
    const float rp = __frcp_rn(np);
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
      for (int e = 0; e < 8; e += 2)
        yp[i][e / 2] = bf2_round(f2_pack(quot_bf16(fp[i][e], np, rp), quot_bf16(fp[i][e + 1], np, rp)));
  }
  for (int k = 0; k < nb; ++k) {
    const int slot = k % kBcastRing;
    const bool landed = mbar_wait(smem_u32(&full[slot]), (uint32_t)(k / kBcastRing) & 1u, &fail);
    if (!landed) fail = 1;  // bounded wait ran out: this row's outputs are marked invalid below
    uint64_t xc[NV][4];
    uint64_t sc2 = 0;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = i * G + tid;
      const uint4 v = j < p.nvec ? ring[slot * p.nvec + j] : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        xc[i][e] = bf2_widen(w[e]);
        sc2 = f2_fma(xc[i][e], xc[i][e], sc2);
      }
    }
    // After this sum's barriers every thread has read the slot: refill it.
    float nc = sqrt_to_bf16(rows.sum(f2_lo(sc2) + f2_hi(sc2)));
    if (tid == 0 && k + kBcastRing < nb && !fail) {
      fence_proxy_async_smem();
      issue(k + kBcastRing);
    }
    nc = nc < p.k.eps_r ? p.k.eps_r : nc;  // clamp_min keeps NaN
    const float rc = rcp_for_bf16_quot(nc);
    const uint64_t rc2 = f2_pack(rc, rc);
    uint64_t s2 = 0;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (i * G + tid >= p.nvec) continue;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t yc = bf2_round(f2_mul(xc[i][e], rc2));
        s2 = f2_add(s2, bf2_widen(bf2_mul(yc, yp[i][e])));
      }
    }
    const float sim = rnd<AF_DTYPE_BF16>(rows.sum(f2_lo(s2) + f2_hi(s2)));
    if (tid == 0) {
      const int64_t b = b0 + k;
      p.mask[b * p.m_bs + t] = (!fail && sim > p.k.tau_r) ? 1 : 0;
      if (p.sim) p.sim[b * p.T + t] = fail ? __int_as_float(0x7fc00000) : sim;
    }
  }
}

template <int DT, int METRIC>
__global__ void __launch_bounds__(256) k_gate_scalar(const GateParams p) {
  pdl_trigger();  // the compaction kernel may launch now; it waits for this grid
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= p.rows) return;
  const int64_t b = row / p.T, t = row - b * p.T;
  const char* c = p.child + b * p.c_bs + t * p.c_ts;
  const char* q = p.parent + b * p.p_bs + t * p.p_ts;
  GateOut r = gate_row_scalar<DT, METRIC>(c, q, p.H, p.k, lane);
  if (lane == 0) {
    p.mask[b * p.m_bs + t] = r.stable;
    if (p.sim) p.sim[row] = r.sim;
  }
}

// Order-preserving compaction of one batch row's mask into stable / divergent
// index lists. One CTA per batch row, chunks of blockDim.x tokens.
__global__ void __launch_bounds__(1024) k_compact(const uint8_t* __restrict__ mask, int64_t m_bs, int64_t T,
                                                  int32_t* __restrict__ stable_idx, int32_t* __restrict__ div_idx,
                                                  int64_t idx_bs, int32_t* __restrict__ div_count) {
  __shared__ int warp_tot[32];
  __shared__ int chunk_base[2];
  pdl_wait();  // launched as a programmatic dependent of the gate kernel: its masks are complete past this
  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  int base_d = 0, base_s = 0;
  for (int64_t t0 = 0; t0 < T; t0 += blockDim.x) {
    const int64_t t = t0 + tid;
    const bool valid = t < T;
    const bool st = valid && mask[b * m_bs + t] != 0;
    const bool dv = valid && !st;
    // packed counts: divergent in the low 16 bits, stable in the high 16 bits
    const unsigned bd = __ballot_sync(0xffffffffu, dv), bs = __ballot_sync(0xffffffffu, st);
    const unsigned lt = (1u << lane) - 1u;
    const int pre = __popc(bd & lt) | (__popc(bs & lt) << 16);
    if (lane == 0) warp_tot[warp] = __popc(bd) | (__popc(bs) << 16);
    __syncthreads();
    if (warp == 0) {
      int v = lane < nwarps ? warp_tot[lane] : 0;
      // inclusive scan across warps
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
      }
      int excl = __shfl_up_sync(0xffffffffu, v, 1);
      if (lane == 0) excl = 0;
      if (lane < nwarps) warp_tot[lane] = excl;
      if (lane == 31) {
        chunk_base[0] = v & 0xffff;
        chunk_base[1] = v >> 16;
      }
    }
    __syncthreads();
    const int off = warp_tot[warp] + pre;
    if (dv) div_idx[b * idx_bs + base_d + (off & 0xffff)] = (int32_t)t;
    if (st && stable_idx) stable_idx[b * idx_bs + base_s + (off >> 16)] = (int32_t)t;
    base_d += chunk_base[0];
    base_s += chunk_base[1];
    __syncthreads();
  }
  // -1 padding past each list
  for (int64_t i = base_d + tid; i < T; i += blockDim.x) div_idx[b * idx_bs + i] = -1;
  if (stable_idx)
    for (int64_t i = base_s + tid; i < T; i += blockDim.x) stable_idx[b * idx_bs + i] = -1;
  if (tid == 0) div_count[b] = base_d;
}

template <int DT, int METRIC>
static int launch_gate(const GateParams& p, bool vec, cudaStream_t s) {
  const int threads = 256, rows_per_block = threads / 32;
  const int64_t blocks = ceil_div(p.rows, rows_per_block);
  if (blocks > 0x7fffffff) return fail(AF_ERR_ARG, "af_gate: too many rows");
  if (!vec) {
    k_gate_scalar<DT, METRIC><<<(unsigned)blocks, threads, 0, s>>>(p);
    return check_launch("af_gate(scalar)");
  }
  if constexpr (DT == AF_DTYPE_BF16 && METRIC == AF_METRIC_COSINE) {
    if (p.p_bs == 0 && p.nvec > 64 && p.nvec <= 4 * kBcastThreads) {
      const int64_t B = p.rows / p.T;
      if (p.T > 0x7fffffff) return fail(AF_ERR_ARG, "af_gate: seq too large");
      const dim3 grid((unsigned)p.T, (unsigned)ceil_div(B, (int64_t)kBcastChildren));
      if (grid.y > 65535) return fail(AF_ERR_ARG, "af_gate: batch too large");
      const size_t ring_bytes = (size_t)kBcastRing * p.nvec * 16;  // <= 24 KB: eight CTAs per SM
      if (p.nvec <= kBcastThreads) k_gate_bcast<1><<<grid, kBcastThreads, ring_bytes, s>>>(p);
      else if (p.nvec <= 2 * kBcastThreads) k_gate_bcast<2><<<grid, kBcastThreads, ring_bytes, s>>>(p);
      else k_gate_bcast<4><<<grid, kBcastThreads, ring_bytes, s>>>(p);
      return check_launch("af_gate(broadcast)");
    }
  }
  if (p.nvec > 64 && p.nvec <= 2 * kGateRowThreads) {
    if (p.rows > 0x7fffffff) return fail(AF_ERR_ARG, "af_gate: too many rows");
    if (p.nvec <= kGateRowThreads) k_gate_row<DT, METRIC, 1><<<(unsigned)p.rows, kGateRowThreads, 0, s>>>(p);
    else k_gate_row<DT, METRIC, 2><<<(unsigned)p.rows, kGateRowThreads, 0, s>>>(p);
    return check_launch("af_gate(row)");
  }
  const int nv = (p.nvec + 31) / 32;
  if (nv <= 1) k_gate_vec<DT, METRIC, 1><<<(unsigned)blocks, threads, 0, s>>>(p);
  else if (nv <= 2) k_gate_vec<DT, METRIC, 2><<<(unsigned)blocks, threads, 0, s>>>(p);
  else if (nv <= 4) k_gate_vec<DT, METRIC, 4><<<(unsigned)blocks, threads, 0, s>>>(p);
  else if (nv <= 8) k_gate_vec<DT, METRIC, 8><<<(unsigned)blocks, threads, 0, s>>>(p);
  else k_gate_vec<DT, METRIC, 16><<<(unsigned)blocks, threads, 0, s>>>(p);
  return check_launch("af_gate(vec)");
}

template <int DT>
static int dispatch_metric(int metric, const GateParams& p, bool vec, cudaStream_t s) {
  switch (metric) {
    case AF_METRIC_COSINE: return launch_gate<DT, AF_METRIC_COSINE>(p, vec, s);
    case AF_METRIC_L2: return launch_gate<DT, AF_METRIC_L2>(p, vec, s);
    case AF_METRIC_PEARSON: return launch_gate<DT, AF_METRIC_PEARSON>(p, vec, s);
    default: return fail(AF_ERR_ARG, "af_gate: unsupported metric");
  }
}

int gate_launch(const GateParams& p, int dtype, int metric, bool vec, cudaStream_t s) {
  switch (dtype) {
    case AF_DTYPE_BF16: return dispatch_metric<AF_DTYPE_BF16>(metric, p, vec, s);
    case AF_DTYPE_F16: return dispatch_metric<AF_DTYPE_F16>(metric, p, vec, s);
    case AF_DTYPE_F32: return dispatch_metric<AF_DTYPE_F32>(metric, p, vec, s);
    default: return fail(AF_ERR_ARG, "af_gate: unsupported dtype");
  }
}

}  // namespace af

using namespace af;

extern "C" int af_gate(const void* child, int64_t child_bstride, int64_t child_tstride, const void* parent,
                       int64_t parent_bstride, int64_t parent_tstride, int64_t batch, int64_t seq, int64_t hidden,
                       int dtype, int metric, float tau, float eps, float l2_denom, uint8_t* stable_mask,
                       int64_t mask_bstride, float* sim, int32_t* stable_idx, int32_t* div_idx, int64_t idx_bstride,
                       int32_t* div_count, void* stream) {
  AF_REQUIRE(batch >= 0 && seq >= 0 && hidden > 0, "af_gate: bad shape");
  if (batch == 0 || seq == 0) return AF_OK;
  AF_REQUIRE(child && parent && stable_mask, "af_gate: null pointer");
  AF_REQUIRE(hidden <= (1 << 24), "af_gate: hidden too large");
  AF_REQUIRE(dtype == AF_DTYPE_F32 || dtype == AF_DTYPE_F16 || dtype == AF_DTYPE_BF16, "af_gate: bad dtype");
  AF_REQUIRE(!div_idx || div_count, "af_gate: div_idx needs div_count");
  AF_REQUIRE(!stable_idx || div_idx, "af_gate: stable_idx needs div_idx");
  AF_REQUIRE(!div_idx || seq < (1 << 16) * 1024, "af_gate: seq too large for compaction");
  AF_REQUIRE(!div_idx || idx_bstride >= seq, "af_gate: idx_bstride < seq");
  cudaStream_t s = as_stream(stream);
  const int esize = dtype == AF_DTYPE_F32 ? 4 : 2;
  const int64_t row_bytes = hidden * esize;
  GateParams p;
  p.child = static_cast<const char*>(child);
  p.parent = static_cast<const char*>(parent);
  p.c_bs = child_bstride;
  p.c_ts = child_tstride;
  p.p_bs = parent_bstride;
  p.p_ts = parent_tstride;
  p.rows = batch * seq;
  p.T = seq;
  p.H = (int)hidden;
  p.nvec = (int)(row_bytes / 16);
  p.k = make_gate_consts(dtype, tau, eps, l2_denom);
  p.mask = stable_mask;
  p.m_bs = mask_bstride;
  p.sim = sim;
  const uintptr_t align = reinterpret_cast<uintptr_t>(child) | reinterpret_cast<uintptr_t>(parent) |
                          (uintptr_t)child_bstride | (uintptr_t)child_tstride | (uintptr_t)parent_bstride |
                          (uintptr_t)parent_tstride | (uintptr_t)row_bytes;
  const bool vec = (align % 16) == 0 && p.nvec <= 16 * 32;
  int st = gate_launch(p, dtype, metric, vec, s);
  if (st != AF_OK || !div_idx) return st;
  // Programmatic dependent launch: the compaction's CTAs are set up while the
  // gate's last CTAs run, and wait for the gate grid inside the kernel.
  const cudaError_t e = launch_ex(k_compact, dim3((unsigned)batch), dim3(1024), 0, s, true, dim3(1, 1, 1),
                                  (const uint8_t*)stable_mask, mask_bstride, (int64_t)seq, stable_idx, div_idx,
                                  idx_bstride, div_count);
  if (e != cudaSuccess) return fail(AF_ERR_CUDA, std::string("af_gate: compact launch: ") + cudaGetErrorString(e));
  return check_launch("af_gate(compact)");
}
