// Native batched Branch Folding pass for LLaDA/Dream-architecture blocks (sm_100a).
//
// All C children of one parent are verified together, with no host
// synchronisation inside the pass. A child's layer-l input differs from the
// parent's only on its "fresh" rows: the edited tokens at layer 0, then the
// rows that were divergent at layer l-1 (a stable row takes the parent's
// output, so its next input is bit-identical to the parent's). Per layer:
//
//   candidates  = fresh rows (+ any row the parent itself fails the gate on)
//   k_fold_gate     gate(child row, parent row) + copy + attention RMSNorm   [CTA / candidate]
//   (compaction)    divergent list, fresh-key bitmap, next layer's candidates: a side task of
//                   the QKV GEMM's epilogue warps (compact.cuh)
//   QKV GEMM (+RoPE) on candidates           (tcgen05)
//   attention of divergent rows over parent K/V + fresh K/V
//   O GEMM + residual, RMSNorm, gate/up GEMM + SwiGLU, down GEMM + residual
//                                            (tcgen05) -> next layer's fresh rows
//
// After the last layer only the final fresh rows go through the final norm and
// the LM head; every other logits row is the parent's (copied once per row for
// all children). Stable rows therefore cost nothing but the copy of their
// logits, and the per-layer cost scales with the number of divergent rows.
//
// The dense parent pass (af_dense_forward) runs the same kernels on all T rows
// and fills the parent cache: layer inputs, QKV rows (K/V reused by children),
// logits, logit row sums and the parent's self-gate results.
#include <cstring>
#include <mutex>
#include <vector>

#include "attention.cuh"
#include "compact.cuh"
#include "gate_row.cuh"
#include "gemm_tc.cuh"

namespace af {

// ----------------------------------------------------------------------------
// Block-wide exclusive scan (blockDim.x == 1024).
// ----------------------------------------------------------------------------
__device__ __forceinline__ int block_scan_1024(int v, int* warp_buf, int* total_out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += n;
  }
  if (lane == 31) warp_buf[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = warp_buf[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    warp_buf[lane] = w;  // inclusive per-warp totals
  }
  __syncthreads();
  const int excl = x - v + (warp > 0 ? warp_buf[warp - 1] : 0);
  *total_out = warp_buf[31];
  __syncthreads();
  return excl;
}

// ----------------------------------------------------------------------------
// Candidate builder for layer 0 and for layers where the parent fails its own
// gate on some row (one CTA of 1024 threads).
// ----------------------------------------------------------------------------
struct CandArgs {
  int layer, C, T, m_cap;
  const int64_t* ctok;           // [C*T]  (layer 0)
  const int64_t* ptok;           // [T]    (layer 0)
  const uint8_t* self_stable;    // [T] of this layer, nullable
  int all_rows;                  // 1: every row is a candidate (a layer that does not fold)
  const uint8_t* ss_all;         // layer 0, nullable: [L, T] parent self-gate results of the pass
  int n_layers;
  uint8_t* later;                // layer 0, nullable: later[t] = 1 if some layer >= 1 fails the parent's gate at t
  const int* prev_div_pos;       // layer >= 1: fresh rows = previous layer's divergent rows
  const int* prev_n_div;
  int* slot;                     // [C*T] scratch
  int* cand_child;
  int* cand_pos;
  int* cand_src;
  int* n_cand;
  int* fresh0_pos;               // layer 0: positions (c*T + t) of edited tokens
  int* n_fresh0;
  unsigned* status;
};

__global__ void __launch_bounds__(1024) k_fold_candidates(const CandArgs a) {
  pdl_trigger();
  pdl_wait();
  __shared__ int wbuf[32];
  const int N = a.C * a.T;
  int base = 0, total;
  if (a.layer == 0) {
    // One pass, 8 consecutive positions per thread: the edited (fresh) tokens
    // in order, then the candidates (fresh within capacity, or rows the parent
    // fails its own gate on) in order.
    constexpr int E = 8;
    int base1 = 0;
    for (int i0 = 0; i0 < N; i0 += 1024 * E) {
      const int ib = i0 + threadIdx.x * E;
      uint32_t fm = 0, sm = 0;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int i = ib + e;
        if (i < N) {
          const int t = i % a.T;
          if (a.ctok[i] != a.ptok[t]) fm |= 1u << e;
          if (a.all_rows || (a.self_stable && !a.self_stable[t])) sm |= 1u << e;
        }
      }
      int total1, total2;
      int r1 = base1 + block_scan_1024(__popc(fm), wbuf, &total1);
      int src[E];
      uint32_t cm = 0;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        src[e] = -1;
        if ((fm >> e) & 1u) {
          if (r1 < a.m_cap) {
            a.fresh0_pos[r1] = ib + e;
            src[e] = r1;
          } else {
            atomicOr(a.status, AF_STATUS_CAPACITY);
          }
          ++r1;
        }
        if (src[e] >= 0 || ((sm >> e) & 1u)) cm |= 1u << e;
      }
      int r2 = base + block_scan_1024(__popc(cm), wbuf, &total2);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        if ((cm >> e) & 1u) {
          if (r2 < a.m_cap) {
            a.cand_child[r2] = (ib + e) / a.T;
            a.cand_pos[r2] = (ib + e) % a.T;
            a.cand_src[r2] = src[e];
          } else {
            atomicOr(a.status, AF_STATUS_CAPACITY);
          }
          ++r2;
        }
      }
      base1 += total1;
      base += total2;
    }
    if (threadIdx.x == 0) {
      *a.n_fresh0 = min(base1, a.m_cap);
      *a.n_cand = min(base, a.m_cap);
    }
    if (a.later)
      for (int t = threadIdx.x; t < a.T; t += 1024) {
        uint8_t v = 0;
        for (int l = 1; l < a.n_layers && !v; ++l) v = a.ss_all[(int64_t)l * a.T + t] == 0;
        a.later[t] = v;
      }
    return;
  }
  // Later layers (the parent fails its own gate on some rows, or the layer
  // does not fold): fresh rows are the previous layer's divergent rows.
  for (int i = threadIdx.x; i < N; i += 1024) a.slot[i] = -1;
  __syncthreads();
  const int nd = *a.prev_n_div;
  for (int j = threadIdx.x; j < nd; j += 1024) a.slot[a.prev_div_pos[j]] = j;
  __syncthreads();
  for (int i0 = 0; i0 < N; i0 += 1024) {
    const int i = i0 + threadIdx.x;
    int s = -1, f = 0;
    if (i < N) {
      s = a.slot[i];
      f = (a.all_rows || s >= 0 || (a.self_stable && !a.self_stable[i % a.T])) ? 1 : 0;
    }
    const int rank = base + block_scan_1024(f, wbuf, &total);
    if (f) {
      if (rank < a.m_cap) {
        a.cand_child[rank] = i / a.T;
        a.cand_pos[rank] = i % a.T;
        a.cand_src[rank] = s;
      } else {
        atomicOr(a.status, AF_STATUS_CAPACITY);
      }
    }
    base += total;
  }
  if (threadIdx.x == 0) *a.n_cand = min(base, a.m_cap);
}

// ----------------------------------------------------------------------------
// Row gathers (warp per row) and RMSNorm (CTA per row).
// ----------------------------------------------------------------------------
// out[i] = embed[tokens[rows[i]]]; an id outside [0, vocab) sets AF_STATUS_BOUNDS and yields a zero row.
__global__ void __launch_bounds__(256) k_embed_rows(const __nv_bfloat16* embed, int H, int64_t vocab,
                                                    const int64_t* tokens, const int* rows, const int* n_dev,
                                                    int n_cap, __nv_bfloat16* out, unsigned* status) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int i = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int n = n_dev ? min(*n_dev, n_cap) : n_cap;
  if (i >= n) return;
  const int64_t tok = tokens[rows ? rows[i] : i];
  char* dst = reinterpret_cast<char*>(out + (int64_t)i * H);
  if (tok < 0 || tok >= vocab) {
    if (lane == 0) atomicOr(status, AF_STATUS_BOUNDS);
    for (int v = lane; v < H / 8; v += 32) stg16(dst + 16 * v, make_uint4(0u, 0u, 0u, 0u));
    return;
  }
  const char* src = reinterpret_cast<const char*>(embed + tok * H);
  for (int v = lane; v < H / 8; v += 32) stg16(dst + 16 * v, ldg16(src + 16 * v));
}

// Rows of the per-row kernels below are spread over one CTA of kRowThreads
// threads (H <= 4096 gives each thread one 16-byte vector, H <= 8192 two), so
// a few hundred packed rows still occupy every SM. These kernels sit between
// the projections of every layer, where their latency is on the critical
// path: 512 threads give each thread the fewest elements (measured on B200:
// 256-thread CTAs spent ~4 us of dependent arithmetic per 4096-wide row).
constexpr int kRowThreads = 512;
using RowGroup = CtaRows<kRowThreads>;

template <int NV, class Rows = WarpRows>
__device__ __forceinline__ void rmsnorm_regs(const uint4 (&v)[NV], int nvec, int H, const __nv_bfloat16* w, float eps,
                                             char* out, int tid, const Rows& rows = Rows(), float ss_pre = -1.f) {
  constexpr int G = Rows::kThreads;
  // ss_pre >= 0: the row's sum of squares, already reduced in exactly this
  // order (the cosine gate's candidate norm), so the reduction is skipped.
  float ss = 0.f;
  if (ss_pre >= 0.f) {
    ss = ss_pre;
  } else {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float f[8];
      unpack<AF_DTYPE_BF16>(v[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
    }
    ss = rows.sum(ss);
  }
  const float var = __fdiv_rn(ss, (float)H);
  const float rinv = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(var, eps)));
  const char* wb = reinterpret_cast<const char*>(w);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int j = i * G + tid;
    if (j >= nvec) continue;
    float f[8], g[8];
    unpack<AF_DTYPE_BF16>(v[i], f);
    unpack<AF_DTYPE_BF16>(ldg16(wb + 16 * j), g);
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float y0 = rnd<AF_DTYPE_BF16>(__fmul_rn(rnd<AF_DTYPE_BF16>(__fmul_rn(f[2 * e], rinv)), g[2 * e]));
      const float y1 = rnd<AF_DTYPE_BF16>(__fmul_rn(rnd<AF_DTYPE_BF16>(__fmul_rn(f[2 * e + 1], rinv)), g[2 * e + 1]));
      ow[e] = pack_bf16x2(y0, y1);
    }
    stg16(out + 16 * (int64_t)j, o);
  }
}

// Rows whose split-K GEMM left fp32 partials (GemmCall::partial_out): the
// row's value is the residual GEMM epilogue applied here, bit for bit:
// bf16(res + bf16(p_0 + p_1 + ... + p_{S-1})), the splits summed from 0 up.
struct PartialRows {
  const float* part;               // [S][m_cap][H] fp32, null: rows are read from `in`
  int64_t split_stride;            // m_cap * H
  int nsplit;                      // S (<= 16)
  const __nv_bfloat16* res;        // residual rows [.., H]
  const int* res_rows;             // nullable: residual row of row i
  __nv_bfloat16* store;            // the finished rows are written here (row i)
  // Peer-memory sums (af_fold_set_peer_sum): the S slices are the ranks'
  // sums, stored here by k_sum_push on every rank; they are read once
  // peer_flags[0..S) have reached this rank's launch count of that sum
  // (*peer_ctr / peer_grid). Null: no wait.
  const unsigned* peer_flags;
  const unsigned long long* peer_ctr;
  unsigned peer_grid;
  unsigned* status;
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

constexpr unsigned long long kPeerWaitNs = 5000000000ull;  // bound of one wait on the other ranks' sums

// Thread 0 waits until every rank's sum of this launch is in place, then the
// CTA goes on. A wait that runs out ORs AF_STATUS_TIMEOUT into the status
// word, and later waits of the pass see the bit and do not wait again (the
// rows are then wrong, and the host raises on the status).
__device__ __forceinline__ void peer_rows_wait(const PartialRows& pr) {
  if (!pr.peer_flags) return;
  if (threadIdx.x == 0) {
    const unsigned expect = (unsigned)(__ldcg(pr.peer_ctr) / pr.peer_grid);
    if (!(__ldcg(pr.status) & AF_STATUS_TIMEOUT)) {
      const unsigned long long t0 = global_ns();
      for (int q = 0; q < pr.nsplit; ++q) {
        bool late = false;
        while ((int)(ld_acquire_sys(pr.peer_flags + q) - expect) < 0) {
          if (global_ns() - t0 > kPeerWaitNs) {
            atomicOr(pr.status, AF_STATUS_TIMEOUT);
            late = true;
            break;
          }
          __nanosleep(32);
        }
        if (late) break;
      }
    }
  }
  __syncthreads();
}

template <int NV>
__device__ __forceinline__ void load_row_partials(const PartialRows& pr, int row, int64_t rrow, int nvec, int tid,
                                                  uint4 (&v)[NV], bool store = true) {
  // rrow: the residual row of `row` (pr.res_rows[row], or row), read by the
  // caller together with its other indices. store = false: the caller stores
  // the finished row (store_row) once it knows the row is the right one.
  const char* rp = reinterpret_cast<const char*>(pr.res + rrow * (int64_t)(nvec * 8));
  const float* pp = pr.part + (int64_t)row * (nvec * 8);
  float acc[NV][8];
  uint4 rv[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int j = i * kRowThreads + tid;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[i][e] = 0.f;
    if (j < nvec) rv[i] = ldg16(rp + 16 * (int64_t)j);
  }
  // Splits in order, four at a time in flight (the sum order is split 0, 1, 2, ...).
  for (int s0 = 0; s0 < pr.nsplit; s0 += 4) {
    float4 a[NV][4][2];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = i * kRowThreads + tid;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (j < nvec && s0 + q < pr.nsplit) {
          const float4* src = reinterpret_cast<const float4*>(pp + (s0 + q) * pr.split_stride + 8 * (int64_t)j);
          a[i][q][0] = src[0];
          a[i][q][1] = src[1];
        }
    }
#pragma unroll
    for (int i = 0; i < NV; ++i)
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (s0 + q < pr.nsplit) {
          acc[i][0] += a[i][q][0].x; acc[i][1] += a[i][q][0].y; acc[i][2] += a[i][q][0].z; acc[i][3] += a[i][q][0].w;
          acc[i][4] += a[i][q][1].x; acc[i][5] += a[i][q][1].y; acc[i][6] += a[i][q][1].z; acc[i][7] += a[i][q][1].w;
        }
  }
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int j = i * kRowThreads + tid;
    if (j >= nvec) {
      v[i] = make_uint4(0u, 0u, 0u, 0u);
      continue;
    }
    float r[8];
    unpack<AF_DTYPE_BF16>(rv[i], r);
    uint32_t* ow = reinterpret_cast<uint32_t*>(&v[i]);
#pragma unroll
    for (int e = 0; e < 4; ++e)
      ow[e] = pack_bf16x2(__fadd_rn(r[2 * e], rnd<AF_DTYPE_BF16>(acc[i][2 * e])),
                          __fadd_rn(r[2 * e + 1], rnd<AF_DTYPE_BF16>(acc[i][2 * e + 1])));
    if (store) stg16(reinterpret_cast<char*>(pr.store + (int64_t)row * (nvec * 8)) + 16 * (int64_t)j, v[i]);
  }
}

template <int NV>
__device__ __forceinline__ void store_row(__nv_bfloat16* dst, int nvec, int tid, const uint4 (&v)[NV]) {
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int j = i * kRowThreads + tid;
    if (j < nvec) stg16(reinterpret_cast<char*>(dst) + 16 * (int64_t)j, v[i]);
  }
}

// part[0][i] = part[0][i] + part[1][i] + ... (splits in order), i < n: the
// tensor-parallel pass adds its k-splits locally before the cross-rank sum,
// which then moves one slice instead of one per split.
__global__ void __launch_bounds__(256) k_sum_splits(float* part, int64_t stride, int nsplit, int64_t n4,
                                                    const int* rows_dev, int64_t row_len4) {
  pdl_trigger();
  pdl_wait();
  const int64_t lim = rows_dev ? min(n4, (int64_t)(*rows_dev) * row_len4) : n4;
  float4* p0 = reinterpret_cast<float4*>(part);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < lim; i += (int64_t)gridDim.x * blockDim.x) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < nsplit; ++sp) {
      const float4 v = reinterpret_cast<const float4*>(part + sp * stride)[i];
      a.x += v.x;
      a.y += v.y;
      a.z += v.z;
      a.w += v.w;
    }
    p0[i] = a;
  }
}

// Peer-memory cross-rank sum, producer side: this rank's k-splits added in
// order and stored into its slot of every rank's exchange buffer; when the
// launch's last CTA is done, each rank's flag for this rank is raised to the
// launch count. Every thread fences its stores at system scope before its CTA
// counts itself in, so the flag orders after every CTA's stores.
constexpr int kMaxRanks = 8;
struct PeerPush {
  float* dst[kMaxRanks];       // rank q's slot for this rank's sum
  unsigned* flag[kMaxRanks];   // rank q's flag for this rank's sum
  unsigned long long* ctr;     // this rank's CTA count of this sum (grows by the grid size per launch)
  int world;
};

__global__ void __launch_bounds__(256) k_sum_push(const float* part, int64_t stride, int nsplit, int64_t n4,
                                                  const int* rows_dev, int64_t row_len4, const PeerPush pp) {
  pdl_trigger();
  pdl_wait();
  const int64_t lim = rows_dev ? min(n4, (int64_t)(*rows_dev) * row_len4) : n4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < lim; i += (int64_t)gridDim.x * blockDim.x) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp = 0; sp < nsplit; ++sp) {
      const float4 v = reinterpret_cast<const float4*>(part + sp * stride)[i];
      a.x += v.x;
      a.y += v.y;
      a.z += v.z;
      a.w += v.w;
    }
    for (int q = 0; q < pp.world; ++q) reinterpret_cast<float4*>(pp.dst[q])[i] = a;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long done = atomicAdd(pp.ctr, 1ull) + 1ull;
    if (done % gridDim.x == 0) {
      const unsigned seq = (unsigned)(done / gridDim.x);
      __threadfence_system();
      for (int q = 0; q < pp.world; ++q) st_release_sys(pp.flag[q], seq);
    }
  }
}

// out[i] = rmsnorm(in[i]) * w for i < n (rows strided by H); one CTA per row.
// With pr.part, row i is first finished from its split-K partials (and stored).
template <int NV>
__global__ void __launch_bounds__(kRowThreads) k_rmsnorm_rows(const __nv_bfloat16* in, const __nv_bfloat16* w, int H,
                                                              float eps, const int* n_dev, int n_cap,
                                                              __nv_bfloat16* out, const PartialRows pr) {
  pdl_trigger();
  __shared__ __align__(16) float red[2 * kRowThreads / 32];
  const int i = blockIdx.x;  // < n_cap: the index arrays are read before the count is known
  // The residual row index was written two or more kernels back and is
  // usually in place before the wait: the row loads go out with it at once,
  // and the index read again after the wait decides whether they stand (L2
  // reads: no stale L1 line can answer either read).
  const int rrow_e = pr.part && pr.res_rows ? min(max(__ldcg(pr.res_rows + i), 0), n_cap - 1) : i;
  pdl_wait();
  const int nvec = H / 8;
  uint4 v[NV];
  if (pr.part) peer_rows_wait(pr);
  if (pr.part) load_row_partials<NV>(pr, i, rrow_e, nvec, threadIdx.x, v, false);
  const int rrow = pr.part && pr.res_rows ? __ldcg(pr.res_rows + i) : i;
  const int n = n_dev ? min(*n_dev, n_cap) : n_cap;
  if (i >= n) return;
  if (pr.part) {
    if (rrow != rrow_e) load_row_partials<NV>(pr, i, rrow, nvec, threadIdx.x, v, false);
    store_row<NV>(pr.store + (int64_t)i * H, nvec, threadIdx.x, v);
  } else
    load_row<NV, kRowThreads>(reinterpret_cast<const char*>(in + (int64_t)i * H), nvec, threadIdx.x, v);
  rmsnorm_regs<NV>(v, nvec, H, w, eps, reinterpret_cast<char*>(out + (int64_t)i * H), threadIdx.x, RowGroup{red});
}

// ----------------------------------------------------------------------------
// Gate of candidate rows + packed copy + attention RMSNorm (warp per candidate).
// ----------------------------------------------------------------------------
struct FoldGateArgs {
  const int* n_cand;
  int m_cap, H, T;
  const int* cand_pos;
  const int* cand_src;
  const __nv_bfloat16* x_fresh;   // fresh rows of this layer [m_cap, H]
  const __nv_bfloat16* p_in;      // parent layer input [T, H]
  const __nv_bfloat16* norm_w;
  float eps;
  GateConsts k;
  int force_div;                  // 1: the layer does not fold, every candidate is divergent
  PartialRows fresh_part;         // part non-null: fresh rows are finished here from the previous down GEMM's partials
  uint8_t* stable;
  __nv_bfloat16* xc;              // packed candidate hidden [m_cap, H]
  __nv_bfloat16* a;               // packed normalized rows [m_cap, H]
};

template <int METRIC, int NV>
__global__ void __launch_bounds__(kRowThreads) k_fold_gate(const FoldGateArgs g) {
  pdl_trigger();
  __shared__ __align__(16) float red[2 * kRowThreads / 32];
  const int tid = threadIdx.x;
  const int r = blockIdx.x;  // < m_cap: the candidate arrays are read before the count is known
  const int nvec = g.H / 8;
  const RowGroup rows{red};
  // This layer's candidate list was written two or more kernels back and is
  // usually in place before the wait: the row loads go out with the indices
  // read now, and the indices read again after the wait decide whether they
  // stand (both reads from L2, so no stale L1 line answers the second).
  const int t_e = min(max(__ldcg(g.cand_pos + r), 0), g.T - 1);
  const int src_e = min(max(__ldcg(g.cand_src + r), -1), g.m_cap - 1);
  uint4 hv[NV], pv[NV];
  // The parent's row is constant data: it is requested before the wait.
  load_row<NV, kRowThreads>(reinterpret_cast<const char*>(g.p_in + (int64_t)t_e * g.H), nvec, tid, pv);
  pdl_wait();
  if (g.fresh_part.part) peer_rows_wait(g.fresh_part);
  auto load_fresh = [&](int t, int src) {
    if (src >= 0 && g.fresh_part.part) {
      const int rrow = g.fresh_part.res_rows ? g.fresh_part.res_rows[src] : src;
      load_row_partials<NV>(g.fresh_part, src, rrow, nvec, tid, hv, false);
    } else if (src >= 0) {
      load_row<NV, kRowThreads>(reinterpret_cast<const char*>(g.x_fresh + (int64_t)src * g.H), nvec, tid, hv);
    } else {
#pragma unroll
      for (int i = 0; i < NV; ++i) hv[i] = pv[i];  // no fresh row: the parent's (as loaded for t)
    }
  };
  load_fresh(t_e, src_e);
  const int t = __ldcg(g.cand_pos + r), src = __ldcg(g.cand_src + r);
  const int n = min(*g.n_cand, g.m_cap);
  if (r >= n) return;
  if (t != t_e) load_row<NV, kRowThreads>(reinterpret_cast<const char*>(g.p_in + (int64_t)t * g.H), nvec, tid, pv);
  if (t != t_e || src != src_e) load_fresh(t, src);
  // The finished fresh row (from the previous down GEMM's partials) is kept in x_fresh.
  if (src >= 0 && g.fresh_part.part) store_row<NV>(g.fresh_part.store + (int64_t)src * g.H, nvec, tid, hv);
  GateOut o;
  if constexpr (METRIC == AF_METRIC_COSINE) o = gate_regs_bf16_cos<NV>(hv, pv, nvec, g.k, tid, rows);
  else o = gate_regs<AF_DTYPE_BF16, METRIC, NV>(hv, pv, nvec, g.H, g.k, tid, rows);
  if (tid == 0) g.stable[r] = g.force_div ? 0 : o.stable;
  char* xc = reinterpret_cast<char*>(g.xc + (int64_t)r * g.H);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int j = i * kRowThreads + tid;
    if (j < nvec) stg16(xc + 16 * j, hv[i]);
  }
  rmsnorm_regs<NV>(hv, nvec, g.H, g.norm_w, g.eps, reinterpret_cast<char*>(g.a + (int64_t)r * g.H), tid, rows, o.ss_c);
}

// ----------------------------------------------------------------------------
// Logits of stable rows: copy the parent's row t to every child whose final
// row t is not fresh. CTA = one 16 KB chunk of one position (the parent chunk
// is read once), so the fill's CTAs are short and free their SM slots quickly
// when it runs beside the last layer at a lower launch priority.
// ----------------------------------------------------------------------------
constexpr int kFillChunk = 8192;  // logits per CTA

// Which children take the parent's logits row t:
//   FILL_ALL   every child whose final row t is not fresh (final_bits);
//   FILL_EARLY, right after layer 0, every child whose row t was stable at layer 0 (bits0) at a
//              position that no later layer can make a candidate again (later[t] == 0): such a row
//              keeps the parent's input at every layer, so it is stable at the end;
//   FILL_LATE  after the last layer, the remaining final-stable rows (fresh at layer 0, or at a
//              position a later layer re-examines).
enum FillMode : int { FILL_ALL = 0, FILL_EARLY = 1, FILL_LATE = 2 };

__device__ __forceinline__ bool bit_of(const unsigned* b, int bits_ld, int c, int t) {
  return (b[c * bits_ld + (t >> 5)] >> (t & 31)) & 1u;
}

__global__ void __launch_bounds__(256) k_logits_fill(const __nv_bfloat16* p_logits, int64_t V, int C, int T,
                                                     const unsigned* final_bits, const unsigned* bits0,
                                                     const uint8_t* later, int mode, int bits_ld,
                                                     __nv_bfloat16* logits) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ int kids[];  // children that take the parent row
  __shared__ int nk;
  const int t = blockIdx.y;
  if (threadIdx.x == 0) nk = 0;
  __syncthreads();
  const bool later_t = mode != FILL_ALL && later[t] != 0;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    bool take;
    if (mode == FILL_EARLY) take = !later_t && !bit_of(bits0, bits_ld, c, t);
    else if (mode == FILL_LATE) take = !bit_of(final_bits, bits_ld, c, t) && (later_t || bit_of(bits0, bits_ld, c, t));
    else take = !bit_of(final_bits, bits_ld, c, t);
    if (take) kids[atomicAdd(&nk, 1)] = c;
  }
  __syncthreads();
  const int n = nk;
  if (n == 0) return;
  const int64_t v0 = (int64_t)blockIdx.x * (kFillChunk / 8), v1 = min(V / 8, v0 + kFillChunk / 8);
  const char* src = reinterpret_cast<const char*>(p_logits + (int64_t)t * V);
  for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    const uint4 x = ldg16(src + 16 * v);
    for (int k = 0; k < n; ++k)
      stg16(reinterpret_cast<char*>(logits + ((int64_t)kids[k] * T + t) * V) + 16 * v, x);
  }
}

// score[c] = mean over [T, V] of child c's logits (fp32 sums of the bf16 values).
__global__ void __launch_bounds__(256) k_scores(const float* p_row_sums, const float* fresh_row_sums, int C, int T,
                                                int64_t V, const unsigned* final_bits, int bits_ld, float* scores) {
  pdl_trigger();
  pdl_wait();
  const int c = blockIdx.x;
  float s = 0.f;
  for (int t = threadIdx.x; t < T; t += blockDim.x) {
    const bool fresh = (final_bits[c * bits_ld + (t >> 5)] >> (t & 31)) & 1u;
    s += fresh ? fresh_row_sums[(int64_t)c * T + t] : p_row_sums[t];
  }
  s = warp_sum(s);
  __shared__ float ws[8];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) tot += ws[i];
    scores[c] = tot / ((float)T * (float)V);
  }
}

// Dense layer state of every child: parent rows, then fresh rows scattered over them.
__global__ void __launch_bounds__(256) k_state_parent(const __nv_bfloat16* p_in, int H, int C, int T,
                                                      __nv_bfloat16* out) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= (int64_t)C * T) return;
  const int t = (int)(row % T);
  const char* s = reinterpret_cast<const char*>(p_in + (int64_t)t * H);
  char* d = reinterpret_cast<char*>(out + row * H);
  for (int v = lane; v < H / 8; v += 32) stg16(d + 16 * v, ldg16(s + 16 * v));
}

__global__ void __launch_bounds__(256) k_state_scatter(const __nv_bfloat16* x, int H, const int* pos, const int* n_dev,
                                                       int n_cap, __nv_bfloat16* out) {
  pdl_trigger();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int i = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int n = min(*n_dev, n_cap);
  if (i >= n) return;
  const char* s = reinterpret_cast<const char*>(x + (int64_t)i * H);
  char* d = reinterpret_cast<char*>(out + (int64_t)pos[i] * H);
  for (int v = lane; v < H / 8; v += 32) stg16(d + 16 * v, ldg16(s + 16 * v));
}

__global__ void k_iota(int* p, int n) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = i;
}

__global__ void k_zero_f32(float* p, int64_t n) {
  pdl_trigger();
  pdl_wait();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = 0.f;
}

// Self gate of the parent rows of one layer (does the parent pass its own
// gate?). Same row grouping and arithmetic as k_fold_gate, so a parent row
// that fails here fails there too when a child carries it unchanged.
template <int NV>
__global__ void __launch_bounds__(kRowThreads) k_self_gate(const __nv_bfloat16* x, int H, int T, GateConsts k,
                                                           uint8_t* self_stable) {
  pdl_trigger();
  pdl_wait();
  __shared__ __align__(16) float red[2 * kRowThreads / 32];
  const int t = blockIdx.x;
  if (t >= T) return;
  const int nvec = H / 8;
  uint4 v[NV];
  load_row<NV, kRowThreads>(reinterpret_cast<const char*>(x + (int64_t)t * H), nvec, threadIdx.x, v);
  const GateOut o = gate_regs_bf16_cos<NV>(v, v, nvec, k, threadIdx.x, RowGroup{red});
  if (threadIdx.x == 0) self_stable[t] = o.stable;
}

// ----------------------------------------------------------------------------
// Promotion of a verified child to a parent. The reference stores every
// branch's per-layer activations, children included (_store_activations after
// the merge, actfold/core/folded_transformer.py:190-199), so a child can be
// the parent of the next verification. A child's layer-l input differs from
// its parent's only on its fresh rows of layer l, so promoting it rewrites
// just those rows of a parent cache: the layer input, the QKV row (kept by
// k_keep_rows during the pass) and the self-gate flag.
// ----------------------------------------------------------------------------

// Candidate QKV rows of the current layer, copied to the caller's store
// [L, m_cap, qkv] (one CTA per row) while promotion is enabled.
__global__ void __launch_bounds__(256) k_keep_rows(const __nv_bfloat16* src, int cols, const int* n_dev, int n_cap,
                                                   __nv_bfloat16* dst) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x;
  if (i >= min(*n_dev, n_cap)) return;
  const char* s = reinterpret_cast<const char*>(src + (int64_t)i * cols);
  char* d = reinterpret_cast<char*>(dst + (int64_t)i * cols);
  for (int v = threadIdx.x; v < cols / 8; v += blockDim.x) stg16(d + 16 * (int64_t)v, ldg16(s + 16 * (int64_t)v));
}

struct PromoteArgs {
  int child, T, H, L, m_cap, qkv_cols, q_cols, n_kv_heads;
  const int *cand_child, *cand_pos, *cand_src, *n_cand;  // [(L+1) * m_cap], [L+1]
  const __nv_bfloat16* x_all;                             // [L+1, m_cap, H] fresh rows of each layer
  const __nv_bfloat16* kept_qkv;                          // [L, m_cap, qkv_cols] QKV row of each candidate
  __nv_bfloat16* layer_in;                                // [L+1, T, H]
  __nv_bfloat16* qkv;                                     // [L, T, qkv_cols]
  uint8_t* self_stable;                                   // [L, T]
  __nv_bfloat16* kv_hm;                                   // nullable: [L, 2, n_kv_heads, T, 128]
  GateConsts k;
};

// One CTA per (candidate slot, layer): a fresh row of the promoted child is
// written over the parent's, with its QKV row and its self-gate result (same
// arithmetic as k_self_gate in the parent pass).
template <int NV>
__global__ void __launch_bounds__(kRowThreads) k_promote_rows(const PromoteArgs a) {
  pdl_trigger();
  pdl_wait();
  __shared__ __align__(16) float red[2 * kRowThreads / 32];
  const int j = blockIdx.x, l = blockIdx.y;
  if (j >= min(a.n_cand[l], a.m_cap)) return;
  const int64_t cj = (int64_t)l * a.m_cap + j;
  const int src = a.cand_src[cj];
  if (a.cand_child[cj] != a.child || src < 0) return;
  const int t = a.cand_pos[cj];
  const int nvec = a.H / 8;
  uint4 v[NV];
  load_row<NV, kRowThreads>(reinterpret_cast<const char*>(a.x_all + ((int64_t)l * a.m_cap + src) * a.H), nvec,
                            threadIdx.x, v);
  char* drow = reinterpret_cast<char*>(a.layer_in + ((int64_t)l * a.T + t) * a.H);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int jj = i * kRowThreads + threadIdx.x;
    if (jj < nvec) stg16(drow + 16 * (int64_t)jj, v[i]);
  }
  if (l >= a.L) return;  // the final hidden state has no QKV row or gate
  const char* qs = reinterpret_cast<const char*>(a.kept_qkv + cj * a.qkv_cols);
  char* qd = reinterpret_cast<char*>(a.qkv + ((int64_t)l * a.T + t) * a.qkv_cols);
  for (int jj = threadIdx.x; jj < a.qkv_cols / 8; jj += kRowThreads) stg16(qd + 16 * (int64_t)jj, ldg16(qs + 16 * (int64_t)jj));
  if (a.kv_hm) {
    // The same K and V columns into the head-major copy: 16-byte chunk c of
    // head h of K (kv = 0) or V (kv = 1) is [l][kv][h][t][8c .. 8c + 7].
    const int chunks = 2 * a.n_kv_heads * 16;
    for (int jj = threadIdx.x; jj < chunks; jj += kRowThreads) {
      const int kv = jj / (a.n_kv_heads * 16), h = (jj / 16) % a.n_kv_heads, c = jj % 16;
      const int64_t off = ((((int64_t)l * 2 + kv) * a.n_kv_heads + h) * a.T + t) * 128 + 8 * c;
      stg16(reinterpret_cast<char*>(a.kv_hm + off), ldg16(qs + 2 * (int64_t)a.q_cols + 16 * (int64_t)jj));
    }
  }
  const GateOut o = gate_regs_bf16_cos<NV>(v, v, nvec, a.k, threadIdx.x, RowGroup{red});
  if (threadIdx.x == 0) a.self_stable[(int64_t)l * a.T + t] = o.stable;
}

// Head-major copy of a parent's keys and values: row t of layer l, K or V
// (kv), head h goes to kv_hm[l][kv][h][t][0..127]. One CTA per (8 rows,
// layer); each thread moves 16-byte chunks, reading whole rows in order.
__global__ void __launch_bounds__(256) k_kv_headmajor(const __nv_bfloat16* __restrict__ qkv, int T, int q_cols,
                                                      int qkv_cols, int n_kv_heads, __nv_bfloat16* __restrict__ kv_hm) {
  const int l = blockIdx.y;
  const int chunks = 2 * n_kv_heads * 16;  // per row
  for (int r = 0; r < 8; ++r) {
    const int t = blockIdx.x * 8 + r;
    if (t >= T) return;
    const char* src = reinterpret_cast<const char*>(qkv + ((int64_t)l * T + t) * qkv_cols + q_cols);
    for (int jj = threadIdx.x; jj < chunks; jj += blockDim.x) {
      const int kv = jj / (n_kv_heads * 16), h = (jj / 16) % n_kv_heads, c = jj % 16;
      const int64_t off = ((((int64_t)l * 2 + kv) * n_kv_heads + h) * T + t) * 128 + 8 * c;
      stg16(reinterpret_cast<char*>(kv_hm + off), ldg16(src + 16 * (int64_t)jj));
    }
  }
}

extern "C" int af_parent_kv_headmajor(const af_model_dims* dims, int64_t T, const void* qkv, void* kv_headmajor,
                                      void* stream) {
  AF_REQUIRE(dims && qkv && kv_headmajor, "af_parent_kv_headmajor: null pointer");
  AF_REQUIRE(T > 0 && T <= (1 << 24), "af_parent_kv_headmajor: bad sequence length");
  AF_REQUIRE(dims->head_dim == 128, "af_parent_kv_headmajor: head_dim must be 128");
  AF_REQUIRE(((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(kv_headmajor)) & 15) == 0,
             "af_parent_kv_headmajor: buffers must be 16-byte aligned");
  AF_REQUIRE(dims->n_layers > 0 && dims->n_kv_heads > 0 && dims->n_heads > 0, "af_parent_kv_headmajor: bad dims");
  const int q = (int)(dims->n_heads * 128), qkv_cols = q + 2 * (int)(dims->n_kv_heads * 128);
  cudaStream_t s = as_stream(stream);
  k_kv_headmajor<<<dim3((unsigned)((T + 7) / 8), (unsigned)dims->n_layers), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(qkv), (int)T, q, qkv_cols, (int)dims->n_kv_heads,
      static_cast<__nv_bfloat16*>(kv_headmajor));
  return check_launch("af_parent_kv_headmajor");
}

// Logits rows and logit row sums of the promoted child's last-layer divergent
// rows (its other rows hold the parent's logits already). One CTA per row.
__global__ void __launch_bounds__(256) k_promote_final(int child, int T, int64_t V, const int* div_pos, const int* n_div,
                                                       int m_cap, const __nv_bfloat16* child_logits,
                                                       const float* fresh_row_sums, __nv_bfloat16* p_logits,
                                                       float* p_row_sums) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x;
  if (i >= min(*n_div, m_cap)) return;
  const int pos = div_pos[i];
  if (pos / T != child) return;
  const int t = pos % T;
  const char* s = reinterpret_cast<const char*>(child_logits + (int64_t)pos * V);
  char* d = reinterpret_cast<char*>(p_logits + (int64_t)t * V);
  for (int64_t v = threadIdx.x; v < V / 8; v += blockDim.x) stg16(d + 16 * v, ldg16(s + 16 * v));
  if (threadIdx.x == 0) p_row_sums[t] = fresh_row_sums[pos];
}

// ----------------------------------------------------------------------------
// Host side
// ----------------------------------------------------------------------------
struct Bump {
  char* base;
  int64_t off = 0, cap;
  Bump(void* b, int64_t c) : base(static_cast<char*>(b)), cap(c) {}
  template <class T>
  T* take(int64_t n) {
    off = (off + 255) & ~int64_t(255);
    T* p = reinterpret_cast<T*>(base ? base + off : nullptr);
    off += n * (int64_t)sizeof(T);
    return p;
  }
};

// Kernels of the dense and folded passes are launched with programmatic
// dependent launch (each waits for its predecessor inside the kernel, see
// pdl_wait), so a kernel's launch and prologue overlap the previous kernel's
// tail. ACTFOLD_PDL=0 turns it off.
// ACTFOLD_SPLITK_PARTIALS=0: the O / down GEMMs reduce their k-splits inside
// the launch (thread-block cluster) instead of leaving fp32 partials to the
// next row kernel (comparison runs).
static bool partials_off() {
  static const bool off = [] {
    const char* e = getenv("ACTFOLD_SPLITK_PARTIALS");
    return e && e[0] == '0';
  }();
  return off;
}

// ACTFOLD_EARLY_FILL=0: every parent logits row is copied after the last
// layer instead of from layer 0 on (comparison runs).
static bool early_fill_off() {
  static const bool off = [] {
    const char* e = getenv("ACTFOLD_EARLY_FILL");
    return e && e[0] == '0';
  }();
  return off;
}

static bool pass_pdl() {
  static const bool on = [] {
    const char* e = getenv("ACTFOLD_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

#define AF_LAUNCH(KERNEL, GRID, BLOCK, SMEM, STREAM, ...) \
  launch_ex(KERNEL, dim3(GRID), dim3(BLOCK), (size_t)(SMEM), STREAM, pass_pdl(), dim3(1, 1, 1), __VA_ARGS__)

// Per-row kernels on one CTA of kRowThreads threads per row: H <= 8192.
#define AF_DISPATCH_ROWS(H, KERNEL, ROWS, STREAM, ...)                                   \
  do {                                                                                   \
    if ((H) / 8 <= kRowThreads) AF_LAUNCH(KERNEL<1>, (unsigned)(ROWS), kRowThreads, 0, STREAM, __VA_ARGS__); \
    else AF_LAUNCH(KERNEL<2>, (unsigned)(ROWS), kRowThreads, 0, STREAM, __VA_ARGS__);    \
  } while (0)

static int validate_model(const af_model* m) {
  AF_REQUIRE(m && m->layers && m->embed && m->final_norm && m->lm_head && m->rope_cos && m->rope_sin,
             "model: null pointer");
  const af_model_dims& d = m->dims;
  AF_REQUIRE(d.n_layers > 0 && d.head_dim == 128, "model: head_dim must be 128");
  AF_REQUIRE(d.n_heads > 0 && d.n_kv_heads > 0 && d.n_heads % d.n_kv_heads == 0, "model: bad head counts");
  AF_REQUIRE(d.hidden % 128 == 0 && d.hidden <= 4096, "model: hidden must be a multiple of 128 and <= 4096");
  AF_REQUIRE(d.ffn % 64 == 0 && (2 * d.ffn) % 128 == 0, "model: ffn must be a multiple of 64");
  AF_REQUIRE(d.vocab % 128 == 0, "model: vocab must be a multiple of 128");
  return AF_OK;
}

struct Sizes {
  int H, q, kv, qkv, FF, V, L;
};
static Sizes sizes_of(const af_model_dims& d) {
  Sizes s;
  s.H = d.hidden;
  s.q = d.n_heads * d.head_dim;
  s.kv = d.n_kv_heads * d.head_dim;
  s.qkv = s.q + 2 * s.kv;
  s.FF = d.ffn;
  s.V = d.vocab;
  s.L = d.n_layers;
  return s;
}

// ---------------------------------------------------------------- dense pass
struct DenseWs {
  __nv_bfloat16 *A, *att, *h1, *bn, *f;
  int* pos;
};

static DenseWs carve_dense(Bump& b, const Sizes& s, int T) {
  DenseWs w;
  w.A = b.take<__nv_bfloat16>((int64_t)T * s.H);
  w.att = b.take<__nv_bfloat16>((int64_t)T * s.q);
  w.h1 = b.take<__nv_bfloat16>((int64_t)T * s.H);
  w.bn = b.take<__nv_bfloat16>((int64_t)T * s.H);
  w.f = b.take<__nv_bfloat16>((int64_t)T * s.FF);
  w.pos = b.take<int>(T);
  return w;
}

// Model projections are stored tiled (see af_model in the header).
static GemmCall base_call(unsigned* status) {
  GemmCall c;
  memset(&c, 0, sizeof(c));
  c.status = status;
  c.w_tiled = 1;
  c.head_dim = 128;
  c.pdl = pass_pdl() ? 1 : 0;
  return c;
}

}  // namespace af

using namespace af;

extern "C" int af_dense_workspace_bytes(const af_model_dims* d, int64_t T, int64_t* bytes) {
  AF_REQUIRE(d && bytes && T > 0, "af_dense_workspace_bytes: bad argument");
  Bump b(nullptr, 0);
  carve_dense(b, sizes_of(*d), (int)T);
  *bytes = b.off + 256;
  return AF_OK;
}

extern "C" int af_dense_forward(const af_model* m, const int64_t* tokens, int64_t T, float tau, void* layer_in,
                                void* qkv, void* logits, uint8_t* self_stable, float* logit_row_sums, void* workspace,
                                int64_t workspace_bytes, uint32_t* status, void* stream) {
  int st = validate_model(m);
  if (st) return st;
  AF_REQUIRE(tokens && layer_in && qkv && logits && self_stable && logit_row_sums && workspace && status,
             "af_dense_forward: null pointer");
  AF_REQUIRE(T > 0 && T <= m->max_pos && T <= (1 << 20), "af_dense_forward: T out of range");
  cudaStream_t s = as_stream(stream);
  const Sizes z = sizes_of(m->dims);
  const int Ti = (int)T;
  Bump b(workspace, workspace_bytes);
  DenseWs w = carve_dense(b, z, Ti);
  AF_REQUIRE(b.off <= workspace_bytes, "af_dense_forward: workspace too small");
  __nv_bfloat16* xin = static_cast<__nv_bfloat16*>(layer_in);
  __nv_bfloat16* qkvb = static_cast<__nv_bfloat16*>(qkv);
  unsigned* stw = reinterpret_cast<unsigned*>(status);
  const float eps = m->dims.rms_eps;
  const unsigned rows_blocks = (unsigned)((Ti + 7) / 8);
  const GateConsts gk = make_gate_consts(AF_DTYPE_BF16, tau, 1e-8f, 0.f);

  AF_LAUNCH(k_iota, (Ti + 255) / 256, 256, 0, s, w.pos, Ti);
  AF_LAUNCH(k_embed_rows, rows_blocks, 256, 0, s, static_cast<const __nv_bfloat16*>(m->embed), z.H, z.V, tokens, nullptr,
                                           nullptr, Ti, xin, stw);
  for (int l = 0; l < z.L; ++l) {
    const af_layer_weights& lw = m->layers[l];
    const __nv_bfloat16* x = xin + (int64_t)l * Ti * z.H;
    __nv_bfloat16* xnext = xin + (int64_t)(l + 1) * Ti * z.H;
    __nv_bfloat16* qkv_l = qkvb + (int64_t)l * Ti * z.qkv;
    AF_DISPATCH_ROWS(z.H, k_rmsnorm_rows, Ti, s, x, static_cast<const __nv_bfloat16*>(lw.attn_norm), z.H, eps, nullptr,
                     Ti, w.A, PartialRows{});
    AF_DISPATCH_ROWS(z.H, k_self_gate, Ti, s, x, z.H, Ti, gk, self_stable + (int64_t)l * Ti);
    GemmCall c = base_call(stw);
    c.x = w.A;
    c.ldx = z.H;
    c.m_cap = Ti;
    c.w = lw.w_qkv;
    c.n = z.qkv;
    c.k = z.H;
    c.epi = EPI_ROPE;
    c.out = qkv_l;
    c.ldo = z.qkv;
    c.rope_cos = m->rope_cos;
    c.rope_sin = m->rope_sin;
    c.positions = w.pos;
    c.rope_cols = z.q + z.kv;
    if ((st = gemm_run(c, s))) return st;
    AttnParams ap;
    memset(&ap, 0, sizeof(ap));
    ap.q = qkv_l;
    ap.q_ld = z.qkv;
    ap.n_q_cap = Ti;
    ap.pk = qkv_l + z.q;
    ap.pv = qkv_l + z.q + z.kv;
    ap.kv_ld = z.qkv;
    ap.T = Ti;
    ap.out = w.att;
    ap.out_ld = z.q;
    ap.n_heads = m->dims.n_heads;
    ap.n_kv_heads = m->dims.n_kv_heads;
    ap.scale_log2 = (1.0f / sqrtf((float)m->dims.head_dim)) * 1.4426950408889634f;
    ap.pdl = pass_pdl() ? 1 : 0;
    ap.status = stw;
    if ((st = attention_run(ap, s))) return st;
    c = base_call(stw);
    c.x = w.att;
    c.ldx = z.q;
    c.m_cap = Ti;
    c.w = lw.w_o;
    c.n = z.H;
    c.k = z.q;
    c.epi = EPI_RESIDUAL;
    c.out = w.h1;
    c.ldo = z.H;
    c.res = x;
    c.ldr = z.H;
    if ((st = gemm_run(c, s))) return st;
    AF_DISPATCH_ROWS(z.H, k_rmsnorm_rows, Ti, s, w.h1, static_cast<const __nv_bfloat16*>(lw.ffn_norm), z.H, eps,
                     nullptr, Ti, w.bn, PartialRows{});
    c = base_call(stw);
    c.x = w.bn;
    c.ldx = z.H;
    c.m_cap = Ti;
    c.w = lw.w_gateup;
    c.n = 2 * z.FF;
    c.k = z.H;
    c.epi = EPI_SWIGLU;
    c.out = w.f;
    c.ldo = z.FF;
    if ((st = gemm_run(c, s))) return st;
    c = base_call(stw);
    c.x = w.f;
    c.ldx = z.FF;
    c.m_cap = Ti;
    c.w = lw.w_down;
    c.n = z.H;
    c.k = z.FF;
    c.epi = EPI_RESIDUAL;
    c.out = xnext;
    c.ldo = z.H;
    c.res = w.h1;
    c.ldr = z.H;
    if ((st = gemm_run(c, s))) return st;
  }
  const __nv_bfloat16* xl = xin + (int64_t)z.L * Ti * z.H;
  AF_DISPATCH_ROWS(z.H, k_rmsnorm_rows, Ti, s, xl, static_cast<const __nv_bfloat16*>(m->final_norm), z.H, eps,
                   nullptr, Ti, w.A, PartialRows{});
  AF_LAUNCH(k_zero_f32, (Ti + 255) / 256, 256, 0, s, logit_row_sums, (int64_t)Ti);
  GemmCall c = base_call(stw);
  c.x = w.A;
  c.ldx = z.H;
  c.m_cap = Ti;
  c.w = m->lm_head;
  c.n = z.V;
  c.k = z.H;
  c.epi = EPI_STORE;
  c.out = logits;
  c.ldo = z.V;
  c.row_sums = logit_row_sums;
  if ((st = gemm_run(c, s))) return st;
  return check_launch("af_dense_forward");
}

// ---------------------------------------------------------------- fold plan
namespace af {

struct FoldWs {
  int* slot;
  int *cand_child, *cand_pos, *cand_src, *n_cand;  // [(L+1) * m_cap], [L+1]
  int *div_cand, *div_child, *div_pos, *n_div;     // [L * m_cap], [L]
  int *fresh0_pos, *n_fresh0;
  uint8_t* stable;
  unsigned *bits, *final_bits;
  int* div_count;  // [L, C]
  __nv_bfloat16 *x_all, *xc, *A, *qkv, *att, *h1, *bn, *f;
  float* row_sums;  // [C*T] fresh logit row sums
  unsigned* status;
  int* cand_div;  // [m_cap] divergent rank of each candidate of the current layer, -1 if stable
  int bits_ld;
  // Split-K partials of the O and down GEMMs ([S][m_cap][H] fp32, S = their
  // k-splits), finished by the next row kernel; null when neither splits.
  float* part;
  int split_o, split_down, split_qkv;
  int part_o, part_down, part_qkv;  // 1: that GEMM leaves its partials in `part`
  unsigned* bits0;        // [C, bits_ld] divergent rows of layer 0 (the early logits fill)
  uint8_t* later;         // [T] positions a layer >= 1 re-examines (the parent fails its own gate there)
};

// k-splits of the QKV projection when it leaves partials (tuning override
// ACTFOLD_QKV_SPLITS: 0 for a cluster reduction in its own epilogue, 1 for
// no split; else the partial-launch heuristic).
static int qkv_partial_splits(const Sizes& z, int m_cap) {
  static const int env = [] {
    const char* e = getenv("ACTFOLD_QKV_SPLITS");
    return e ? atoi(e) : -1;
  }();
  if (env >= 0) return std::min(env, 16);
  return gemm_splits(z.qkv, z.H, m_cap, true);
}

static FoldWs carve_fold(Bump& b, const Sizes& z, int C, int T, int m_cap, bool partial_always) {
  FoldWs w;
  const int L = z.L;
  w.bits_ld = (T + 31) / 32;
  w.slot = b.take<int>((int64_t)C * T);
  w.cand_child = b.take<int>((int64_t)(L + 1) * m_cap);
  w.cand_pos = b.take<int>((int64_t)(L + 1) * m_cap);
  w.cand_src = b.take<int>((int64_t)(L + 1) * m_cap);
  w.n_cand = b.take<int>(L + 1);
  w.div_cand = b.take<int>((int64_t)L * m_cap);
  w.div_child = b.take<int>((int64_t)L * m_cap);
  w.div_pos = b.take<int>((int64_t)L * m_cap);
  w.n_div = b.take<int>(L);
  w.fresh0_pos = b.take<int>(m_cap);
  w.n_fresh0 = b.take<int>(1);
  w.stable = b.take<uint8_t>(m_cap);
  w.bits = b.take<unsigned>((int64_t)C * w.bits_ld);
  w.final_bits = b.take<unsigned>((int64_t)C * w.bits_ld);
  w.div_count = b.take<int>((int64_t)L * C);
  w.x_all = b.take<__nv_bfloat16>((int64_t)(L + 1) * m_cap * z.H);
  w.xc = b.take<__nv_bfloat16>((int64_t)m_cap * z.H);
  w.A = b.take<__nv_bfloat16>((int64_t)m_cap * z.H);
  w.qkv = b.take<__nv_bfloat16>((int64_t)m_cap * z.qkv);
  w.att = b.take<__nv_bfloat16>((int64_t)m_cap * z.q);
  w.h1 = b.take<__nv_bfloat16>((int64_t)m_cap * z.H);
  w.bn = b.take<__nv_bfloat16>((int64_t)m_cap * z.H);
  w.f = b.take<__nv_bfloat16>((int64_t)m_cap * z.FF);
  w.row_sums = b.take<float>((int64_t)C * T);
  w.status = b.take<unsigned>(1);
  w.cand_div = b.take<int>(m_cap);
  w.bits0 = b.take<unsigned>((int64_t)C * w.bits_ld);
  w.later = b.take<uint8_t>(T);
  // The O / down projections leave partials where they split k (always for
  // a tensor-parallel shard); their split counts are then those of launches
  // without a cluster.
  const bool split_o = gemm_splits(z.H, z.q, m_cap) > 1, split_d = gemm_splits(z.H, z.FF, m_cap) > 1;
  w.part_o = partial_always || (split_o && !partials_off());
  w.part_down = partial_always || (split_d && !partials_off());
  w.split_o = w.part_o ? gemm_splits(z.H, z.q, m_cap, true) : 1;
  w.split_down = w.part_down ? gemm_splits(z.H, z.FF, m_cap, true) : 1;
  // The QKV projection leaves its k-splits as partials too, finished (summed,
  // rotated, stored) by k_gemm_finish before attention: a cluster reduction
  // in its own epilogue costs more than that launch.
  w.part_qkv = gemm_splits(z.qkv, z.H, m_cap) > 1 && !partials_off() && qkv_partial_splits(z, m_cap) > 1;
  w.split_qkv = w.part_qkv ? qkv_partial_splits(z, m_cap) : 1;
  const int S = std::max(w.split_o, w.split_down);
  const int64_t per_row = std::max((int64_t)S * z.H, w.part_qkv ? (int64_t)w.split_qkv * z.qkv : 0);
  w.part = (w.part_o || w.part_down || w.part_qkv) ? b.take<float>(per_row * m_cap) : nullptr;
  return w;
}

// Kernel classes of a folded pass (per-class CUDA-event timing).
enum FoldKind {
  FK_SETUP = 0, FK_GATE, FK_COMPACT, FK_QKV, FK_ATTN, FK_O, FK_NORM, FK_GATEUP, FK_DOWN, FK_LM, FK_FILL, FK_SCORES,
  FK_FINISH, FK_COUNT
};

// Optional CUDA-event brackets around each launch of a pass, on the pass's stream.
struct KernelTimer {
  bool on = false;
  std::vector<cudaEvent_t> pool;
  size_t used = 0;
  struct Mark {
    int kind;
    cudaEvent_t b, e;
  };
  std::vector<Mark> marks;
  double ms[FK_COUNT] = {};
  int64_t n[FK_COUNT] = {};
  int64_t launches = 0;

  cudaEvent_t next() {
    if (used == pool.size()) {
      cudaEvent_t ev;
      cudaEventCreate(&ev);
      pool.push_back(ev);
    }
    return pool[used++];
  }
  cudaEvent_t begin(cudaStream_t s) {
    if (!on) return nullptr;
    cudaEvent_t b = next();
    cudaEventRecord(b, s);
    return b;
  }
  void end(int kind, cudaStream_t s, cudaEvent_t b) {
    ++launches;
    if (!on || !b) return;
    cudaEvent_t e = next();
    cudaEventRecord(e, s);
    marks.push_back({kind, b, e});
  }
  void collect() {
    if (!marks.empty()) cudaEventSynchronize(marks.back().e);
    for (const Mark& m : marks) {
      float t = 0.f;
      if (cudaEventElapsedTime(&t, m.b, m.e) == cudaSuccess) {
        ms[m.kind] += t;
        n[m.kind] += 1;
      }
    }
    marks.clear();
    used = 0;
  }
  ~KernelTimer() {
    for (cudaEvent_t e : pool) cudaEventDestroy(e);
  }
};

#define AF_TIMED(KIND, ...)                  \
  do {                                       \
    cudaEvent_t _b = p->tk.begin(s);         \
    __VA_ARGS__;                             \
    p->tk.end(KIND, s, _b);                  \
  } while (0)

struct FoldPlan {
  af_model model;
  std::vector<af_layer_weights> layers;
  af_parent_cache parent;
  int C, T, m_cap;
  float tau;
  int metric;
  std::vector<uint8_t> su;
  std::vector<float> taus;       // gate threshold per layer
  std::vector<uint8_t> folds;    // 0: the layer recomputes every row
  const uint8_t* self_stable;    // [L, T] parent self-gate results at the plan's thresholds
  FoldWs w;
  int ntok;
  std::vector<CUtensorMap> tm_qkv, tm_o, tm_gu, tm_down;
  CUtensorMap tm_lm, tx_A, tx_Alm, tx_att, tx_bn, tx_f, tx_qkv;  // tx_Alm: w.A for the LM head
  KernelTimer tk;
  int64_t last_launches = 0;
  // Side stream of the pass: the logits fill of stable rows runs there from the
  // last layer's QKV GEMM (which writes the final divergent bitmap) on, beside
  // the last layer and the LM head, and joins before the scores.
  cudaStream_t side = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  // Caller store [L, m_cap, qkv] for each layer's candidate QKV rows
  // (af_fold_keep_kv); null when promotion is off.
  __nv_bfloat16* kv_keep = nullptr;
  // Bound on any child's candidate rows per layer (af_fold_set_child_cap); 0: none.
  int child_cap = 0;
  // Tensor-parallel shard (af_fold_set_tensor_parallel): cross-rank sums, the
  // full embedding's rows, the whole vocabulary.
  bool partial_always = false;
  af_collective_fn coll = nullptr;
  void* coll_user = nullptr;
  int64_t embed_rows = 0, vocab_total = 0;
  // Peer-memory sums (af_fold_set_peer_sum): this rank, the number of ranks
  // (0: sums through the hook) and each rank's exchange buffer as mapped here.
  int peer_rank = 0, peer_world = 0;
  char* exch[kMaxRanks] = {};
  ~FoldPlan() {
    if (ev_fork) cudaEventDestroy(ev_fork);
    if (ev_join) cudaEventDestroy(ev_join);
    if (side) cudaStreamDestroy(side);
  }
};

static int build_maps(FoldPlan* p) {
  const Sizes z = sizes_of(p->model.dims);
  // Token rows per box of each activation map: those of the token tile of the
  // GEMM that reads it (w.A feeds QKV and the LM head: one map each).
  auto nt = [&](int n) { return gemm_xbox(gemm_ntok(p->m_cap, n)); };
  p->ntok = gemm_ntok(p->m_cap, z.qkv);
  int st;
  p->tm_qkv.resize(z.L);
  p->tm_o.resize(z.L);
  p->tm_gu.resize(z.L);
  p->tm_down.resize(z.L);
  for (int l = 0; l < z.L; ++l) {
    const af_layer_weights& lw = p->layers[l];
    if ((st = make_tmap_bf16_tiled(&p->tm_qkv[l], lw.w_qkv, z.qkv, z.H))) return st;
    if ((st = make_tmap_bf16_tiled(&p->tm_o[l], lw.w_o, z.H, z.q))) return st;
    if ((st = make_tmap_bf16_tiled(&p->tm_gu[l], lw.w_gateup, 2 * z.FF, z.H))) return st;
    if ((st = make_tmap_bf16_tiled(&p->tm_down[l], lw.w_down, z.H, z.FF))) return st;
  }
  if ((st = make_tmap_bf16_tiled(&p->tm_lm, p->model.lm_head, z.V, z.H))) return st;
  if ((st = make_tmap_bf16(&p->tx_A, p->w.A, p->m_cap, z.H, z.H, nt(z.qkv)))) return st;
  if ((st = make_tmap_bf16(&p->tx_Alm, p->w.A, p->m_cap, z.H, z.H, nt(z.V)))) return st;
  if ((st = make_tmap_bf16(&p->tx_att, p->w.att, p->m_cap, z.q, z.q, nt(z.H)))) return st;
  if ((st = make_tmap_bf16(&p->tx_bn, p->w.bn, p->m_cap, z.H, z.H, nt(2 * z.FF)))) return st;
  if ((st = make_tmap_bf16(&p->tx_qkv, p->w.qkv, p->m_cap, z.qkv, z.qkv, 128))) return st;
  if ((st = make_tmap_bf16(&p->tx_f, p->w.f, p->m_cap, z.FF, z.FF, nt(z.H)))) return st;
  return AF_OK;
}

template <int METRIC>
static void launch_fold_gate(const FoldGateArgs& g, int H, int rows, cudaStream_t s) {
  if (H / 8 <= kRowThreads) AF_LAUNCH((k_fold_gate<METRIC, 1>), (unsigned)rows, kRowThreads, 0, s, g);
  else AF_LAUNCH((k_fold_gate<METRIC, 2>), (unsigned)rows, kRowThreads, 0, s, g);
}

// A cross-rank sum of a tensor-parallel pass, handed to the caller's hook on the pass stream.
static int collective(FoldPlan* p, int kind, int layer, void* data, int64_t count, cudaStream_t s) {
  ++p->tk.launches;
  const int rc = p->coll(p->coll_user, kind, layer, data, count, static_cast<void*>(s));
  if (rc) return fail(AF_ERR_COMM, "af_fold_run: the collective hook failed (kind " + std::to_string(kind) + ", layer " +
                                       std::to_string(layer) + ", code " + std::to_string(rc) + ")");
  return AF_OK;
}

// Exchange buffer of the peer-memory sums, per rank: the ranks' sums of the O
// and down projections [2][world][m_cap][H] fp32, then the flags
// [2][kMaxRanks] u32 (flag q of a sum: rank q's launch count of it, raised by
// rank q), then this rank's CTA counters [2] u64.
static int64_t peer_flags_off(const FoldPlan* p, int world) {
  const int64_t recv = 2 * (int64_t)world * p->m_cap * sizes_of(p->model.dims).H * 4;
  return (recv + 255) / 256 * 256;
}
static int64_t peer_bytes(const FoldPlan* p, int world) { return peer_flags_off(p, world) + 256; }
static float* peer_slot(const FoldPlan* p, char* ex, int kind, int q) {
  return reinterpret_cast<float*>(ex) + ((int64_t)kind * p->peer_world + q) * p->m_cap * sizes_of(p->model.dims).H;
}
static unsigned* peer_flag(const FoldPlan* p, char* ex, int kind, int q) {
  return reinterpret_cast<unsigned*>(ex + peer_flags_off(p, p->peer_world)) + kind * kMaxRanks + q;
}
static unsigned long long* peer_ctr(const FoldPlan* p, int kind) {
  return reinterpret_cast<unsigned long long*>(p->exch[p->peer_rank] + peer_flags_off(p, p->peer_world) + 64) + kind;
}
static unsigned peer_grid() { return (unsigned)(2 * sm_count()); }

// Where the rows of an O / down projection are finished from: this rank's
// k-splits (one GPU), the hook's in-place sum (one slice), or the ranks' sums
// in every rank's exchange buffer (peer-memory sums, added in rank order).
static void tp_partials(const FoldPlan* p, int kind, int local_splits, PartialRows& pr) {
  if (!p->coll) {
    pr.nsplit = local_splits;
  } else if (!p->peer_world) {
    pr.nsplit = 1;
  } else {
    char* own = p->exch[p->peer_rank];
    pr.part = peer_slot(p, own, kind, 0);
    pr.nsplit = p->peer_world;
    pr.peer_flags = peer_flag(p, own, kind, 0);
    pr.peer_ctr = peer_ctr(p, kind);
    pr.peer_grid = peer_grid();
    pr.status = p->w.status;
  }
}

// Tensor parallel: this rank's k-splits of an O / down projection added into
// the first slice, then that slice summed over the ranks by the hook; or, with
// peer-memory sums, added and stored into every rank's exchange buffer.
static int cross_rank_sum(FoldPlan* p, int kind, int layer, int nsplit, const int* rows_dev, cudaStream_t s) {
  const Sizes z = sizes_of(p->model.dims);
  const int64_t n = (int64_t)p->m_cap * z.H;
  if (p->peer_world) {
    PeerPush pp;
    memset(&pp, 0, sizeof(pp));
    pp.world = p->peer_world;
    for (int q = 0; q < p->peer_world; ++q) {
      pp.dst[q] = peer_slot(p, p->exch[q], kind, p->peer_rank);
      pp.flag[q] = peer_flag(p, p->exch[q], kind, p->peer_rank);
    }
    pp.ctr = peer_ctr(p, kind);
    AF_TIMED(FK_NORM, AF_LAUNCH(k_sum_push, peer_grid(), 256, 0, s, (const float*)p->w.part, n, nsplit, n / 4,
                                rows_dev, (int64_t)z.H / 4, pp));
    return AF_OK;
  }
  if (nsplit > 1)
    AF_TIMED(FK_NORM, AF_LAUNCH(k_sum_splits, (unsigned)(2 * sm_count()), 256, 0, s, p->w.part, n, nsplit, n / 4,
                                rows_dev, (int64_t)z.H / 4));
  return collective(p, kind, layer, p->w.part, n, s);
}

static int fold_run(FoldPlan* p, const int64_t* ctok, __nv_bfloat16* logits, float* scores, cudaStream_t s) {
  const Sizes z = sizes_of(p->model.dims);
  const FoldWs& w = p->w;
  const int C = p->C, T = p->T, M = p->m_cap, L = z.L;
  const float eps = p->model.dims.rms_eps;
  const unsigned mblocks = (unsigned)((M + 7) / 8);
  const float hn = (float)(std::sqrt((double)z.H) + 1e-8);
  const __nv_bfloat16* p_in = static_cast<const __nv_bfloat16*>(p->parent.layer_in);
  const __nv_bfloat16* p_qkv = static_cast<const __nv_bfloat16*>(p->parent.qkv);
  int st;
  p->tk.launches = 0;

  // Layer-0 candidates: edited tokens (+ rows the parent fails its own gate on).
  CandArgs ca;
  memset(&ca, 0, sizeof(ca));
  ca.layer = 0;
  ca.C = C;
  ca.T = T;
  ca.m_cap = M;
  ca.ctok = ctok;
  ca.ptok = p->parent.tokens;
  ca.self_stable = p->su[0] ? p->self_stable : nullptr;
  ca.all_rows = p->folds[0] ? 0 : 1;
  // Logits rows that are the parent's can be filled from layer 0 on when no
  // later layer recomputes every row (a row stable at layer 0 then keeps the
  // parent's input, and stays stable, unless the parent fails its own gate at
  // that position in a later layer: `later`).
  const bool fork_fill = !p->tk.on;
  bool early = fork_fill && L > 1 && !early_fill_off();
  for (int l = 1; l < L; ++l) early = early && p->folds[l];
  ca.ss_all = p->self_stable;
  ca.n_layers = L;
  ca.later = early ? w.later : nullptr;
  ca.slot = w.slot;
  ca.cand_child = w.cand_child;
  ca.cand_pos = w.cand_pos;
  ca.cand_src = w.cand_src;
  ca.n_cand = w.n_cand;
  ca.fresh0_pos = w.fresh0_pos;
  ca.n_fresh0 = w.n_fresh0;
  ca.status = w.status;
  AF_TIMED(FK_SETUP, AF_LAUNCH(k_fold_candidates, 1, 1024, 0, s, ca));
  AF_TIMED(FK_SETUP, AF_LAUNCH(k_embed_rows, mblocks, 256, 0, s, static_cast<const __nv_bfloat16*>(p->model.embed), z.H,
                               p->embed_rows ? p->embed_rows : (int64_t)z.V,
                                                           ctok, w.fresh0_pos, w.n_fresh0, M, w.x_all, w.status));

  // Logits fill on the side stream (not in the per-class timing mode, which
  // times every launch class on the pass stream).
  const int fill_smem = C * (int)sizeof(int);
  const dim3 fill_grid((unsigned)((z.V + kFillChunk - 1) / kFillChunk), (unsigned)T);
  // The pass's kernels launch at the device's greatest priority, the side
  // stream's fill at the least: the block scheduler then prefers the pass's
  // pending CTAs whenever a slot frees.
  int prio_low = 0, prio_high = 0;
  cudaDeviceGetStreamPriorityRange(&prio_low, &prio_high);
  LaunchPriority high(fork_fill ? prio_high : kNoPriority);
  if (fork_fill && !p->side) {
    if (cudaStreamCreateWithFlags(&p->side, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&p->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&p->ev_join, cudaEventDisableTiming) != cudaSuccess)
      return check_launch("af_fold_run: side stream");
  }

  for (int l = 0; l < L; ++l) {
    const af_layer_weights& lw = p->layers[l];
    int* cc = w.cand_child + (int64_t)l * M;
    int* cp = w.cand_pos + (int64_t)l * M;
    int* cs = w.cand_src + (int64_t)l * M;
    int* nc = w.n_cand + l;
    int* dcand = w.div_cand + (int64_t)l * M;
    int* dchild = w.div_child + (int64_t)l * M;
    int* dpos = w.div_pos + (int64_t)l * M;
    int* nd = w.n_div + l;
    const __nv_bfloat16* pin_l = p_in + (int64_t)l * T * z.H;
    const __nv_bfloat16* pqkv_l = p_qkv + (int64_t)l * T * z.qkv;
    __nv_bfloat16* x_l = w.x_all + (int64_t)l * M * z.H;
    __nv_bfloat16* x_next = w.x_all + (int64_t)(l + 1) * M * z.H;
    const bool last = l == L - 1;
    const bool next_su = !last && (p->su[l + 1] || !p->folds[l + 1]);

    FoldGateArgs g;
    g.n_cand = nc;
    g.m_cap = M;
    g.H = z.H;
    g.T = T;
    g.cand_pos = cp;
    g.cand_src = cs;
    g.x_fresh = x_l;
    g.p_in = pin_l;
    g.norm_w = static_cast<const __nv_bfloat16*>(lw.attn_norm);
    g.eps = eps;
    g.k = make_gate_consts(AF_DTYPE_BF16, p->taus[l], 1e-8f, hn);
    g.force_div = p->folds[l] ? 0 : 1;
    memset(&g.fresh_part, 0, sizeof(g.fresh_part));
    if (l > 0 && w.part_down) {
      // Layer l's fresh rows are the previous down GEMM's outputs, left as
      // split-K partials: finish them here (residual = that layer's h1).
      g.fresh_part.part = w.part;
      g.fresh_part.split_stride = (int64_t)M * z.H;
      g.fresh_part.res = w.h1;
      g.fresh_part.store = x_l;
      tp_partials(p, AF_COLL_DOWN, w.split_down, g.fresh_part);
    }
    g.stable = w.stable;
    g.xc = w.xc;
    g.a = w.A;
    AF_TIMED(FK_GATE, if (p->metric == AF_METRIC_COSINE) launch_fold_gate<AF_METRIC_COSINE>(g, z.H, M, s);
             else if (p->metric == AF_METRIC_L2) launch_fold_gate<AF_METRIC_L2>(g, z.H, M, s);
             else launch_fold_gate<AF_METRIC_PEARSON>(g, z.H, M, s));

    CompactArgs a;
    memset(&a, 0, sizeof(a));
    a.C = C;
    a.T = T;
    a.m_cap = M;
    a.bits_ld = w.bits_ld;
    a.n_cand = nc;
    a.stable = w.stable;
    a.cand_child = cc;
    a.cand_pos = cp;
    a.div_cand = dcand;
    a.div_child = dchild;
    a.div_pos = dpos;
    a.n_div = nd;
    a.cand_div = w.cand_div;
    a.div_count = w.div_count + (int64_t)l * C;
    a.bits = w.bits;
    a.final_bits = last ? w.final_bits : (l == 0 && early ? w.bits0 : nullptr);
    a.zero_f = last ? w.row_sums : nullptr;
    a.zero_n = C * T;
    a.write_next = !next_su;
    a.next_child = w.cand_child + (int64_t)(l + 1) * M;
    a.next_pos = w.cand_pos + (int64_t)(l + 1) * M;
    a.next_src = w.cand_src + (int64_t)(l + 1) * M;
    a.next_n_cand = w.n_cand + l + 1;

    // The QKV GEMM runs the compaction in the epilogue warps of one CTA while
    // its weights stream (all consumers come after it).
    GemmCall c = base_call(w.status);
    c.has_side = 1;
    c.side = a;
    c.x = w.A;
    c.ldx = z.H;
    c.m_cap = M;
    c.m_dev = nc;
    c.w = lw.w_qkv;
    c.n = z.qkv;
    c.k = z.H;
    c.epi = EPI_ROPE;
    c.out = w.qkv;
    c.ldo = z.qkv;
    c.rope_cos = p->model.rope_cos;
    c.rope_sin = p->model.rope_sin;
    c.positions = cp;
    c.rope_cols = z.q + z.kv;
    c.tmap_w = &p->tm_qkv[l];
    c.tmap_x = &p->tx_A;
    if (w.part_qkv) {
      c.partial_out = w.part;
      c.splits = w.split_qkv;
    } else if (qkv_partial_splits(z, M) == 1) {
      c.splits = 1;  // one CTA per weight tile, RoPE in its own epilogue
    }
    AF_TIMED(FK_QKV, if ((st = gemm_run(c, s))) return st);
    if (w.part_qkv) AF_TIMED(FK_FINISH, if ((st = gemm_finish_run(c, w.split_qkv, s))) return st);
    if (fork_fill && ((l == 0 && early) || last)) {
      // After layer 0's compaction (a side task of this GEMM) the rows stable
      // for good are known; after the last layer's, every final-stable row is.
      // Their logits are the parent's: copy them on the side stream, at the
      // least priority, while the pass goes on here (the LM head writes only
      // final-divergent rows, so the copies never meet its stores).
      if (cudaEventRecord(p->ev_fork, s) != cudaSuccess || cudaStreamWaitEvent(p->side, p->ev_fork, 0) != cudaSuccess)
        return check_launch("af_fold_run: fork");
      const int mode = !last ? FILL_EARLY : (early ? FILL_LATE : FILL_ALL);
      cudaError_t e;
      {
        LaunchPriority low(prio_low);
        e = launch_ex(k_logits_fill, fill_grid, dim3(256), (size_t)fill_smem, p->side, false, dim3(1, 1, 1),
                      static_cast<const __nv_bfloat16*>(p->parent.logits), (int64_t)z.V, C, T,
                      (const unsigned*)w.final_bits, (const unsigned*)w.bits0, (const uint8_t*)w.later, mode,
                      w.bits_ld, logits);
      }
      if (e != cudaSuccess) return fail(AF_ERR_CUDA, std::string("af_fold_run: fill launch: ") + cudaGetErrorString(e));
      ++p->tk.launches;
      if (last && cudaEventRecord(p->ev_join, p->side) != cudaSuccess) return check_launch("af_fold_run: join");
    }

    AttnParams ap;
    memset(&ap, 0, sizeof(ap));
    ap.q = w.qkv;
    ap.q_ld = z.qkv;
    ap.qsrc = dcand;
    ap.qchild = dchild;
    ap.n_q_dev = nd;
    ap.n_q_cap = M;
    ap.pk = pqkv_l + z.q;
    ap.pv = pqkv_l + z.q + z.kv;
    ap.kv_hm = p->parent.kv_headmajor ? static_cast<const __nv_bfloat16*>(p->parent.kv_headmajor) + (int64_t)l * 2 * z.kv * T
                                      : nullptr;
    ap.kv_ld = z.qkv;
    ap.T = T;
    ap.fresh_bits = w.bits;
    ap.bits_ld = w.bits_ld;
    ap.fk = w.qkv + z.q;
    ap.fv = w.qkv + z.q + z.kv;
    ap.f_ld = z.qkv;
    ap.fchild = cc;
    ap.n_f_dev = nc;
    ap.n_f_cap = M;
    ap.out = w.att;
    ap.out_ld = z.q;
    ap.n_heads = p->model.dims.n_heads;
    ap.n_kv_heads = p->model.dims.n_kv_heads;
    ap.scale_log2 = (1.0f / sqrtf(128.f)) * 1.4426950408889634f;
    ap.pdl = pass_pdl() ? 1 : 0;
    ap.kv_static = 1;  // the parent's K/V are fixed for the whole pass
    ap.status = w.status;
    // Candidate keys of a query tile's children lie within cand_win candidate
    // blocks of the tile when no child has more than child_cap candidates.
    ap.cand_win = p->child_cap > 0 ? 2 * ((p->child_cap - 1 + 127) / 128) + 1 : 0;
    AttnParams probe = ap;
    probe.cand_tma = 1;
    probe.qsrc = nullptr;
    probe.tmap_c = &p->tx_qkv;
    if (attention_uses_tc(probe)) {
      // Candidate-row mode: every candidate row is a query (the query tile is
      // 128 rows whatever the divergent count), so the queries and the
      // candidate keys are plain TMA boxes of the QKV output; only divergent
      // rows are written, at their packed rank.
      ap.qsrc = nullptr;
      ap.qchild = cc;
      ap.n_q_dev = nc;
      ap.out_rows = w.cand_div;
      ap.cand_tma = 1;
      ap.tmap_c = &p->tx_qkv;
      ap.fk_col = z.q;
      ap.fv_col = z.q + z.kv;
    }
    AF_TIMED(FK_ATTN, if ((st = attention_run(ap, s))) return st);

    c = base_call(w.status);
    c.x = w.att;
    c.ldx = z.q;
    c.m_cap = M;
    c.m_dev = nd;
    c.w = lw.w_o;
    c.n = z.H;
    c.k = z.q;
    c.epi = EPI_RESIDUAL;
    c.out = w.h1;
    c.ldo = z.H;
    c.res = w.xc;
    c.ldr = z.H;
    c.res_rows = dcand;
    c.tmap_w = &p->tm_o[l];
    c.tmap_x = &p->tx_att;
    c.partial_out = w.part_o ? w.part : nullptr;
    AF_TIMED(FK_O, if ((st = gemm_run(c, s))) return st);
    if (p->coll && (st = cross_rank_sum(p, AF_COLL_O, l, w.split_o, nd, s))) return st;

    PartialRows pr_o;
    memset(&pr_o, 0, sizeof(pr_o));
    if (w.part_o) {  // h1 = xc + O, finished from the O GEMM's partials
      pr_o.part = w.part;
      pr_o.split_stride = (int64_t)M * z.H;
      pr_o.res = w.xc;
      pr_o.res_rows = dcand;
      pr_o.store = w.h1;
      tp_partials(p, AF_COLL_O, w.split_o, pr_o);
    }
    AF_TIMED(FK_NORM, AF_DISPATCH_ROWS(z.H, k_rmsnorm_rows, M, s, w.h1, static_cast<const __nv_bfloat16*>(lw.ffn_norm),
                                       z.H, eps, nd, M, w.bn, pr_o));
    c = base_call(w.status);
    c.x = w.bn;
    c.ldx = z.H;
    c.m_cap = M;
    c.m_dev = nd;
    c.w = lw.w_gateup;
    c.n = 2 * z.FF;
    c.k = z.H;
    c.epi = EPI_SWIGLU;
    c.out = w.f;
    c.ldo = z.FF;
    c.tmap_w = &p->tm_gu[l];
    c.tmap_x = &p->tx_bn;
    AF_TIMED(FK_GATEUP, if ((st = gemm_run(c, s))) return st);

    c = base_call(w.status);
    c.x = w.f;
    c.ldx = z.FF;
    c.m_cap = M;
    c.m_dev = nd;
    c.w = lw.w_down;
    c.n = z.H;
    c.k = z.FF;
    c.epi = EPI_RESIDUAL;
    c.out = x_next;
    c.ldo = z.H;
    c.res = w.h1;
    c.ldr = z.H;
    c.tmap_w = &p->tm_down[l];
    c.tmap_x = &p->tx_f;
    c.partial_out = w.part_down ? w.part : nullptr;  // finished by the next gate (or the final norm)
    AF_TIMED(FK_DOWN, if ((st = gemm_run(c, s))) return st);
    if (p->coll && (st = cross_rank_sum(p, AF_COLL_DOWN, l, w.split_down, nd, s))) return st;
    if (p->kv_keep)
      AF_TIMED(FK_SETUP, AF_LAUNCH(k_keep_rows, (unsigned)M, 256, 0, s, (const __nv_bfloat16*)w.qkv, z.qkv,
                                   (const int*)nc, M, p->kv_keep + (int64_t)l * M * z.qkv));

    if (next_su) {
      CandArgs cn;
      memset(&cn, 0, sizeof(cn));
      cn.layer = l + 1;
      cn.C = C;
      cn.T = T;
      cn.m_cap = M;
      cn.self_stable = p->su[l + 1] ? p->self_stable + (int64_t)(l + 1) * T : nullptr;
      cn.all_rows = p->folds[l + 1] ? 0 : 1;
      cn.prev_div_pos = dpos;
      cn.prev_n_div = nd;
      cn.slot = w.slot;
      cn.cand_child = w.cand_child + (int64_t)(l + 1) * M;
      cn.cand_pos = w.cand_pos + (int64_t)(l + 1) * M;
      cn.cand_src = w.cand_src + (int64_t)(l + 1) * M;
      cn.n_cand = w.n_cand + l + 1;
      cn.status = w.status;
      AF_TIMED(FK_SETUP, AF_LAUNCH(k_fold_candidates, 1, 1024, 0, s, cn));
    }
  }

  // Final rows: fresh after the last layer = its divergent rows.
  int* nd_last = w.n_div + (L - 1);
  int* pos_last = w.div_pos + (int64_t)(L - 1) * M;
  const __nv_bfloat16* x_final = w.x_all + (int64_t)L * M * z.H;
  PartialRows pr_f;
  memset(&pr_f, 0, sizeof(pr_f));
  if (w.part_down) {  // the last layer's outputs, finished from its down GEMM's partials
    pr_f.part = w.part;
    pr_f.split_stride = (int64_t)M * z.H;
    pr_f.res = w.h1;
    pr_f.store = const_cast<__nv_bfloat16*>(x_final);
    tp_partials(p, AF_COLL_DOWN, w.split_down, pr_f);
  }
  AF_TIMED(FK_NORM, AF_DISPATCH_ROWS(z.H, k_rmsnorm_rows, M, s, x_final,
                                     static_cast<const __nv_bfloat16*>(p->model.final_norm), z.H, eps, nd_last, M, w.A,
                                     pr_f));
  GemmCall c = base_call(w.status);
  c.x = w.A;
  c.ldx = z.H;
  c.m_cap = M;
  c.m_dev = nd_last;
  c.w = p->model.lm_head;
  c.n = z.V;
  c.k = z.H;
  c.epi = EPI_STORE;
  c.out = logits;
  c.ldo = z.V;
  c.out_rows = pos_last;
  c.row_sums = w.row_sums;
  c.tmap_w = &p->tm_lm;
  c.tmap_x = &p->tx_Alm;
  AF_TIMED(FK_LM, if ((st = gemm_run(c, s))) return st);
  if (p->coll && (st = collective(p, AF_COLL_ROWSUM, L - 1, w.row_sums, (int64_t)C * T, s))) return st;
  if (fork_fill) {
    if (cudaStreamWaitEvent(s, p->ev_join, 0) != cudaSuccess) return check_launch("af_fold_run: join");
  } else {
    AF_TIMED(FK_FILL, AF_LAUNCH(k_logits_fill, fill_grid, 256, fill_smem, s, static_cast<const __nv_bfloat16*>(p->parent.logits),
                                 (int64_t)z.V, C, T, (const unsigned*)w.final_bits, (const unsigned*)nullptr,
                                 (const uint8_t*)nullptr, (int)FILL_ALL, w.bits_ld, logits));
  }
  if (scores)
    AF_TIMED(FK_SCORES, AF_LAUNCH(k_scores, C, 256, 0, s, (const float*)p->parent.logit_row_sums,
                                  (const float*)w.row_sums, C, T, p->vocab_total ? p->vocab_total : (int64_t)z.V,
                                  (const unsigned*)w.final_bits,
                                  w.bits_ld, scores));
  p->last_launches = p->tk.launches;
  return check_launch("af_fold_run");
}

}  // namespace af

extern "C" int af_fold_workspace_bytes(const af_model_dims* d, const af_fold_config* cfg, int64_t* bytes) {
  AF_REQUIRE(d && cfg && bytes, "af_fold_workspace_bytes: null pointer");
  AF_REQUIRE(cfg->n_children > 0 && cfg->seq > 0 && cfg->m_cap > 0, "af_fold_workspace_bytes: bad sizes");
  Bump b(nullptr, 0);
  carve_fold(b, sizes_of(*d), (int)cfg->n_children, (int)cfg->seq, (int)cfg->m_cap, cfg->partial_always != 0);
  *bytes = b.off + 256;
  return AF_OK;
}

extern "C" int af_fold_plan_create(const af_model* m, const af_parent_cache* parent, const af_fold_config* cfg,
                                   void* workspace, int64_t workspace_bytes, void** plan_out) {
  int st = validate_model(m);
  if (st) return st;
  AF_REQUIRE(parent && cfg && workspace && plan_out, "af_fold_plan_create: null pointer");
  AF_REQUIRE(parent->tokens && parent->layer_in && parent->qkv && parent->logits && parent->self_stable &&
                 parent->logit_row_sums,
             "af_fold_plan_create: incomplete parent cache");
  AF_REQUIRE(cfg->seq == parent->seq, "af_fold_plan_create: child length must equal the parent's");
  AF_REQUIRE(cfg->n_children > 0 && cfg->n_children <= 4096, "af_fold_plan_create: n_children out of range");
  AF_REQUIRE(cfg->seq > 0 && cfg->seq <= m->max_pos, "af_fold_plan_create: seq out of range");
  AF_REQUIRE(cfg->m_cap > 0 && cfg->m_cap <= cfg->n_children * cfg->seq, "af_fold_plan_create: bad m_cap");
  AF_REQUIRE(cfg->n_children * cfg->seq <= (1 << 24), "af_fold_plan_create: C * T too large");
  AF_REQUIRE(cfg->metric >= AF_METRIC_COSINE && cfg->metric <= AF_METRIC_PEARSON, "af_fold_plan_create: bad metric");
  AF_REQUIRE(cfg->su_layers, "af_fold_plan_create: su_layers required");
  FoldPlan* p = new FoldPlan();
  p->model = *m;
  p->layers.assign(m->layers, m->layers + m->dims.n_layers);
  p->model.layers = p->layers.data();
  p->parent = *parent;
  p->C = (int)cfg->n_children;
  p->T = (int)cfg->seq;
  p->m_cap = (int)cfg->m_cap;
  p->tau = cfg->tau;
  p->metric = cfg->metric;
  p->su.assign(cfg->su_layers, cfg->su_layers + m->dims.n_layers);
  p->taus.assign(m->dims.n_layers, cfg->tau);
  if (cfg->tau_layers) p->taus.assign(cfg->tau_layers, cfg->tau_layers + m->dims.n_layers);
  p->folds.assign(m->dims.n_layers, 1);
  if (cfg->fold_layers) p->folds.assign(cfg->fold_layers, cfg->fold_layers + m->dims.n_layers);
  p->self_stable = cfg->self_stable ? cfg->self_stable : parent->self_stable;
  for (uint8_t f : p->folds)
    if (!f && p->m_cap < p->C * p->T) {
      delete p;
      return fail(AF_ERR_ARG, "af_fold_plan_create: a layer that does not fold needs m_cap >= n_children * seq");
    }
  Bump b(workspace, workspace_bytes);
  p->w = carve_fold(b, sizes_of(m->dims), p->C, p->T, p->m_cap, cfg->partial_always != 0);
  p->partial_always = cfg->partial_always != 0;
  if (b.off > workspace_bytes) {
    delete p;
    return fail(AF_ERR_ARG, "af_fold_plan_create: workspace too small");
  }
  if ((st = build_maps(p))) {
    delete p;
    return st;
  }
  *plan_out = p;
  return AF_OK;
}

extern "C" int af_fold_run(void* plan, const int64_t* child_tokens, void* logits, float* scores, void* stream) {
  AF_REQUIRE(plan && child_tokens && logits, "af_fold_run: null pointer");
  return fold_run(static_cast<FoldPlan*>(plan), child_tokens, static_cast<__nv_bfloat16*>(logits), scores,
                  as_stream(stream));
}

extern "C" int af_fold_get_outputs(void* plan, af_fold_outputs* out) {
  AF_REQUIRE(plan && out, "af_fold_get_outputs: null pointer");
  FoldPlan* p = static_cast<FoldPlan*>(plan);
  out->n_cand = p->w.n_cand;
  out->n_div = p->w.n_div;
  out->div_pos = p->w.div_pos;
  out->div_count = p->w.div_count;
  out->status = p->w.status;
  out->m_cap = p->m_cap;
  out->n_fresh0 = p->w.n_fresh0;
  out->fresh0_pos = p->w.fresh0_pos;
  return AF_OK;
}

extern "C" int af_fold_materialize(void* plan, int64_t layer, void* out, void* stream) {
  AF_REQUIRE(plan && out, "af_fold_materialize: null pointer");
  FoldPlan* p = static_cast<FoldPlan*>(plan);
  const Sizes z = sizes_of(p->model.dims);
  AF_REQUIRE(layer >= 0 && layer <= z.L, "af_fold_materialize: layer out of range");
  cudaStream_t s = as_stream(stream);
  const int64_t rows = (int64_t)p->C * p->T;
  const __nv_bfloat16* pin = static_cast<const __nv_bfloat16*>(p->parent.layer_in) + layer * p->T * z.H;
  __nv_bfloat16* o = static_cast<__nv_bfloat16*>(out);
  k_state_parent<<<(unsigned)((rows + 7) / 8), 256, 0, s>>>(pin, z.H, p->C, p->T, o);
  const int* pos = layer == 0 ? p->w.fresh0_pos : p->w.div_pos + (layer - 1) * p->m_cap;
  const int* n = layer == 0 ? p->w.n_fresh0 : p->w.n_div + (layer - 1);
  k_state_scatter<<<(unsigned)((p->m_cap + 7) / 8), 256, 0, s>>>(p->w.x_all + layer * p->m_cap * z.H, z.H, pos, n,
                                                                  p->m_cap, o);
  return check_launch("af_fold_materialize");
}

extern "C" int af_fold_set_child_cap(void* plan, int64_t max_candidates_per_child) {
  AF_REQUIRE(plan, "af_fold_set_child_cap: null plan");
  AF_REQUIRE(max_candidates_per_child >= 0 && max_candidates_per_child <= (1 << 24),
             "af_fold_set_child_cap: bound out of range");
  static_cast<FoldPlan*>(plan)->child_cap = (int)max_candidates_per_child;
  return AF_OK;
}

extern "C" int af_fold_set_tensor_parallel(void* plan, int64_t embed_rows, int64_t vocab_total,
                                           af_collective_fn collective, void* user) {
  AF_REQUIRE(plan && collective, "af_fold_set_tensor_parallel: null pointer");
  FoldPlan* p = static_cast<FoldPlan*>(plan);
  AF_REQUIRE(p->partial_always, "af_fold_set_tensor_parallel: the plan must be created with partial_always = 1");
  AF_REQUIRE(embed_rows > 0 && vocab_total >= p->model.dims.vocab, "af_fold_set_tensor_parallel: bad vocabulary sizes");
  p->coll = collective;
  p->coll_user = user;
  p->embed_rows = embed_rows;
  p->vocab_total = vocab_total;
  return AF_OK;
}

extern "C" int af_fold_peer_bytes(void* plan, int32_t world, int64_t* bytes) {
  AF_REQUIRE(plan && bytes, "af_fold_peer_bytes: null pointer");
  AF_REQUIRE(world >= 1 && world <= kMaxRanks, "af_fold_peer_bytes: world must be 1..8");
  *bytes = peer_bytes(static_cast<FoldPlan*>(plan), world);
  return AF_OK;
}

extern "C" int af_fold_set_peer_sum(void* plan, int32_t rank, int32_t world, void* const* exchange) {
  AF_REQUIRE(plan && exchange, "af_fold_set_peer_sum: null pointer");
  FoldPlan* p = static_cast<FoldPlan*>(plan);
  AF_REQUIRE(p->coll, "af_fold_set_peer_sum: call af_fold_set_tensor_parallel first");
  AF_REQUIRE(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world, "af_fold_set_peer_sum: bad rank / world");
  for (int q = 0; q < world; ++q)
    AF_REQUIRE(exchange[q] && !(reinterpret_cast<uintptr_t>(exchange[q]) & 255u),
               "af_fold_set_peer_sum: exchange buffers must be non-null and 256-byte aligned");
  p->peer_rank = rank;
  p->peer_world = world;
  for (int q = 0; q < kMaxRanks; ++q) p->exch[q] = q < world ? static_cast<char*>(exchange[q]) : nullptr;
  return AF_OK;
}

extern "C" int af_fold_keep_kv(void* plan, void* store, int64_t store_bytes) {
  AF_REQUIRE(plan, "af_fold_keep_kv: null plan");
  FoldPlan* p = static_cast<FoldPlan*>(plan);
  if (!store) {
    p->kv_keep = nullptr;
    return AF_OK;
  }
  const Sizes z = sizes_of(p->model.dims);
  AF_REQUIRE(store_bytes >= (int64_t)z.L * p->m_cap * z.qkv * (int64_t)sizeof(__nv_bfloat16),
             "af_fold_keep_kv: store smaller than n_layers * m_cap * (q_dim + 2 kv_dim) bf16");
  AF_REQUIRE((reinterpret_cast<uintptr_t>(store) & 15) == 0, "af_fold_keep_kv: store must be 16-byte aligned");
  p->kv_keep = static_cast<__nv_bfloat16*>(store);
  return AF_OK;
}

extern "C" int af_fold_promote(void* plan, int64_t child, const int64_t* child_tokens, const void* child_logits,
                               const af_parent_cache* dst, void* stream) {
  AF_REQUIRE(plan && child_tokens && child_logits && dst, "af_fold_promote: null pointer");
  FoldPlan* p = static_cast<FoldPlan*>(plan);
  AF_REQUIRE(p->kv_keep, "af_fold_promote: the pass did not keep its QKV rows (call af_fold_keep_kv before af_fold_run)");
  AF_REQUIRE(child >= 0 && child < p->C, "af_fold_promote: child out of range");
  AF_REQUIRE(dst->seq == p->T, "af_fold_promote: destination length differs from the pass's");
  AF_REQUIRE(dst->tokens && dst->layer_in && dst->qkv && dst->logits && dst->self_stable && dst->logit_row_sums,
             "af_fold_promote: incomplete destination cache");
  const Sizes z = sizes_of(p->model.dims);
  const int T = p->T, M = p->m_cap;
  cudaStream_t s = as_stream(stream);
  cudaError_t e = cudaMemcpyAsync(const_cast<int64_t*>(dst->tokens), child_tokens + child * T, (size_t)T * sizeof(int64_t),
                                  cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess) return fail(AF_ERR_CUDA, std::string("af_fold_promote: tokens: ") + cudaGetErrorString(e));
  PromoteArgs a;
  a.child = (int)child;
  a.T = T;
  a.H = z.H;
  a.L = z.L;
  a.m_cap = M;
  a.qkv_cols = z.qkv;
  a.q_cols = z.q;
  a.n_kv_heads = (int)p->model.dims.n_kv_heads;
  a.kv_hm = static_cast<__nv_bfloat16*>(dst->kv_headmajor);
  a.cand_child = p->w.cand_child;
  a.cand_pos = p->w.cand_pos;
  a.cand_src = p->w.cand_src;
  a.n_cand = p->w.n_cand;
  a.x_all = p->w.x_all;
  a.kept_qkv = p->kv_keep;
  a.layer_in = static_cast<__nv_bfloat16*>(const_cast<void*>(dst->layer_in));
  a.qkv = static_cast<__nv_bfloat16*>(const_cast<void*>(dst->qkv));
  a.self_stable = const_cast<uint8_t*>(dst->self_stable);
  a.k = make_gate_consts(AF_DTYPE_BF16, p->tau, 1e-8f, 0.f);
  const dim3 grid((unsigned)M, (unsigned)(z.L + 1));
  if (z.H / 8 <= kRowThreads) k_promote_rows<1><<<grid, kRowThreads, 0, s>>>(a);
  else k_promote_rows<2><<<grid, kRowThreads, 0, s>>>(a);
  k_promote_final<<<(unsigned)M, 256, 0, s>>>((int)child, T, (int64_t)z.V, p->w.div_pos + (int64_t)(z.L - 1) * M,
                                              p->w.n_div + (z.L - 1), M, static_cast<const __nv_bfloat16*>(child_logits),
                                              p->w.row_sums, static_cast<__nv_bfloat16*>(const_cast<void*>(dst->logits)),
                                              const_cast<float*>(dst->logit_row_sums));
  return check_launch("af_fold_promote");
}

extern "C" int af_fold_set_timing(void* plan, int enabled) {
  AF_REQUIRE(plan, "af_fold_set_timing: null plan");
  FoldPlan* p = static_cast<FoldPlan*>(plan);
  p->tk.collect();
  p->tk.on = enabled != 0;
  return AF_OK;
}

extern "C" int af_fold_get_timing(void* plan, double* ms, int64_t* counts, int n_kinds, int64_t* launches_per_run) {
  AF_REQUIRE(plan && ms && counts && launches_per_run, "af_fold_get_timing: null pointer");
  FoldPlan* p = static_cast<FoldPlan*>(plan);
  p->tk.collect();
  for (int k = 0; k < n_kinds && k < FK_COUNT; ++k) {
    ms[k] = p->tk.ms[k];
    counts[k] = p->tk.n[k];
    p->tk.ms[k] = 0.0;
    p->tk.n[k] = 0;
  }
  *launches_per_run = p->last_launches;
  return AF_OK;
}

extern "C" int af_fold_plan_destroy(void* plan) {
  delete static_cast<FoldPlan*>(plan);
  return AF_OK;
}
