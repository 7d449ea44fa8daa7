// tcgen05 attention of packed query rows over the parent's K/V with per-child
// fresh-key overrides (sm_100a). Same semantics as k_attention (attention.cu):
// query row i (child qchild[i]) attends to every parent position t except the
// fresh positions of its child, and to its child's candidate keys.
//
// CTA = 4 warps = 128 query rows of one head (MMA M = 128; thread r owns query
// row r, i.e. TMEM lane r) and at most three 128-key blocks (a key split of a
// thread-block cluster along grid z). All S tiles fit in TMEM at once
// (3 x 128 columns, plus 128 for O = the whole 512-column TMEM), so the
// softmax is exact in two sweeps per row (max, then exp / sum) and O is never
// rescaled:
//   1. Q, K_j, V_j into 128-byte-swizzled shared tiles: a cached parent's
//      K / V blocks by TMA, issued before the programmatic-dependency wait
//      (they do not depend on the preceding kernel), the rest by cp.async;
//   2. S_j = Q K_j^T (tcgen05.mma, bf16 -> fp32 TMEM, K-major operands);
//   3. each thread masks its row, finds the max over its blocks, writes
//      P_j = exp2(S_j - max) in bf16 over K_j's tiles and sums the row;
//   4. O = sum_j P_j V_j (A = P K-major, B = V MN-major: V rows stay [key][dim]);
//   5. one split: O / l is written; several: the (max, sum, O) partials are
//      combined across the cluster through distributed shared memory.
// Every mbarrier wait is bounded; a timeout sets AF_STATUS_TIMEOUT.
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "attention.cuh"
#include "tc_common.cuh"

namespace af {

namespace {

constexpr int kTQ = 128;            // query rows per CTA (MMA M)
constexpr int kThreads = 512;       // 16 warps: 4 per TMEM lane quadrant, one 32-column group each
constexpr int kTK = 128;            // keys per block
constexpr int kMaxBlk = 3;          // key blocks per CTA
constexpr int kTileB = 128 * 64 * 2;  // [128 rows][64 cols] bf16 tile = 16 KB
constexpr int kOpB = 2 * kTileB;      // a 128 x 128 operand: columns 0-63, then 64-127
constexpr int kOffQ = 0;
constexpr int kOffKP = kOffQ + kOpB;              // K_j, overwritten by P_j
constexpr int kOffV = kOffKP + kMaxBlk * kOpB;
constexpr int kOffF = kOffV + kMaxBlk * kOpB;      // child of each candidate key [3][128]
constexpr int kOffBar = kOffF + kMaxBlk * kTK * 4;  // barS, barO, TMEM slot, fail flag, barK, barV, barC, barCV, barX
constexpr int kSmemTc = kOffBar + 72 + 1024;        // + alignment slack

// Byte offset of 16-byte chunk `ch` (0..7) of row `row` in a swizzled tile.
__device__ __forceinline__ uint32_t sw_off(int row, int ch) { return (uint32_t)(row * 128 + ((ch ^ (row & 7)) << 4)); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// 128 rows x 128 bf16 columns from global rows into two swizzled tiles; a
// null row is zero-filled (its copy reads nothing from `dummy`).
template <class RowPtr>
__device__ __forceinline__ void load_op(uint32_t dst, RowPtr row_ptr, const void* dummy, int tid) {
  for (int idx = tid; idx < 128 * 16; idx += kThreads) {
    const int r = idx >> 4, c16 = idx & 15;
    const __nv_bfloat16* src = row_ptr(r);
    cp_async16(dst + (c16 >> 3) * kTileB + sw_off(r, c16 & 7), src ? (const void*)(src + c16 * 8) : dummy,
               src != nullptr);
  }
}

}  // namespace

// Candidate key blocks each query tile scans (see AttnParams::cand_win).
__host__ __device__ __forceinline__ int cand_blocks(const AttnParams& p) {
  const int all = p.fk ? (p.n_f_cap + kTK - 1) / kTK : 0;
  return (p.cand_tma && p.cand_win > 0 && p.cand_win < all) ? p.cand_win : all;
}

__global__ void __launch_bounds__(kThreads, 1) k_attention_tc(const __grid_constant__ CUtensorMap tmK,
                                                              const __grid_constant__ CUtensorMap tmV,
                                                              const __grid_constant__ CUtensorMap tmC,
                                                              const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();
  const int q0 = blockIdx.x * kTQ;
  const int h = blockIdx.y;
  const int ns = gridDim.z, split = blockIdx.z;
  const int kvh = h / (p.n_heads / p.n_kv_heads);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qd = warp & 3, cg = warp >> 2;  // TMEM lane quadrant, 32-column group
  const int r = 32 * qd + lane;             // this thread's query row (TMEM lane)
  const int c0 = 32 * cg;                   // its 32 key (then head-dim) columns
  // Key blocks: the T parent keys, then the candidate keys. The split over the
  // cluster counts candidate blocks by capacity, so every CTA knows its parent
  // blocks (the first n_par of its blocks) before its predecessor finishes.
  const int n_pb = (p.T + kTK - 1) / kTK;
  // Candidate key blocks of this query tile: all of them, or in candidate-row
  // mode with a window, the n_fb blocks from fb0 on (candidates are ordered by
  // child, so the candidates of this tile's children lie around the tile's own
  // block; checked after the dependency wait).
  const int n_fb_all = p.fk ? (p.n_f_cap + kTK - 1) / kTK : 0;
  const int n_fb = cand_blocks(p), nb = n_pb + n_fb;
  const int fb0 = n_fb < n_fb_all ? min(max((int)blockIdx.x - (p.cand_win - 1) / 2, 0), n_fb_all - n_fb) : 0;
  const int b_lo = split * nb / ns, b_hi = (split + 1) * nb / ns;  // balanced, at most kMaxBlk
  const int nbl = b_hi - b_lo;
  const int n_par = max(0, min(b_hi, n_pb) - b_lo);
  const bool kv_tma = p.kv_static != 0 && n_par > 0;

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gb = smem_raw + (base - raw);
  const uint32_t sQ = base + kOffQ, sKP = base + kOffKP, sV = base + kOffV;
  int* sF = reinterpret_cast<int*>(gb + kOffF);
  float* red = reinterpret_cast<float*>(gb + kOffQ);  // [2][4][128] row max / sum partials, after S is done
  const uint32_t barS = base + kOffBar, barO = barS + 8, barK = barS + 32, barV = barS + 40;
  const uint32_t barC = barS + 48;   // candidate-row mode: query tile and candidate key blocks by TMA
  const uint32_t barCV = barS + 56;  // candidate-row mode: candidate value blocks by TMA
  const uint32_t barX = barS + 64;   // key splits: the other splits' partial rows of this CTA's share have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gb + kOffBar + 16);
  volatile int* fail = reinterpret_cast<volatile int*>(gb + kOffBar + 24);

  if (tid == 0) {
    mbar_init(barS, 1);
    mbar_init(barO, 1);
    mbar_init(barK, 1);
    mbar_init(barV, 1);
    mbar_init(barC, 1);
    mbar_init(barCV, 1);
    mbar_init(barX, 1);
    *fail = 0;
    fence_barrier_init();
    if (kv_tma) {
      // Parent K / V blocks: two 64-column boxes of 128 keys each, swizzled
      // like the cp.async tiles; rows past T are zero-filled by the TMA unit.
      const uint32_t bytes = (uint32_t)n_par * kOpB;
      mbar_arrive_expect_tx(barK, bytes);
      mbar_arrive_expect_tx(barV, bytes);
      // Every K block first: S needs only K, V is not read before P.V.
      // Head-major parent K / V: a block of one head's keys is 32 KB of
      // contiguous memory (row-major [T, q + 2 kv] rows would cost one DRAM
      // page per 128-byte key row).
      for (int j = 0; j < n_par; ++j)
        for (int hf = 0; hf < 2; ++hf) {
          if (p.kv_hm) tma_load_3d(sKP + j * kOpB + hf * kTileB, &tmK, barK, 64 * hf, (b_lo + j) * kTK, kvh);
          else tma_load_2d(sKP + j * kOpB + hf * kTileB, &tmK, barK, kvh * 128 + 64 * hf, (b_lo + j) * kTK);
        }
      for (int j = 0; j < n_par; ++j)
        for (int hf = 0; hf < 2; ++hf) {
          if (p.kv_hm) tma_load_3d(sV + j * kOpB + hf * kTileB, &tmV, barV, 64 * hf, (b_lo + j) * kTK, kvh);
          else tma_load_2d(sV + j * kOpB + hf * kTileB, &tmV, barV, kvh * 128 + 64 * hf, (b_lo + j) * kTK);
        }
    }
  }
  pdl_wait();
  const bool c_tma = p.cand_tma != 0;
  if (c_tma && tid == 0) {
    // Candidate-row mode: the query tile (rows q0..q0+127 of the buffer) and
    // this CTA's candidate key blocks, as soon as their producer is done (they
    // do not depend on the valid counts: rows past them are masked below,
    // queries are not written and keys get zero weight).
    uint32_t kbytes = kOpB, vbytes = 0;
    for (int j = 0; j < nbl; ++j)
      if (b_lo + j >= n_pb) {
        kbytes += kOpB;
        vbytes += kOpB;
      }
    mbar_arrive_expect_tx(barC, kbytes);
    mbar_arrive_expect_tx(barCV, vbytes);  // zero bytes: the barrier completes on the arrival alone
    for (int hf = 0; hf < 2; ++hf) tma_load_2d(sQ + hf * kTileB, &tmC, barC, h * 128 + 64 * hf, q0);
    for (int j = 0; j < nbl; ++j) {
      const int b = b_lo + j;
      if (b < n_pb) continue;
      const int y = (fb0 + b - n_pb) * kTK;
      for (int hf = 0; hf < 2; ++hf)
        tma_load_2d(sKP + j * kOpB + hf * kTileB, &tmC, barC, p.fk_col + kvh * 128 + 64 * hf, y);
    }
    for (int j = 0; j < nbl; ++j) {
      const int b = b_lo + j;
      if (b < n_pb) continue;
      const int y = (fb0 + b - n_pb) * kTK;
      for (int hf = 0; hf < 2; ++hf)
        tma_load_2d(sV + j * kOpB + hf * kTileB, &tmC, barCV, p.fv_col + kvh * 128 + 64 * hf, y);
    }
  }
  // Every per-row value read from global memory is requested here, in one
  // round trip with the valid counts: the query row's child and output row,
  // and the child of each candidate key of this CTA's candidate blocks.
  const int qi = q0 + r;
  const int child_ld = (p.qchild && qi < p.n_q_cap) ? p.qchild[qi] : -1;
  const int orow_ld = qi < p.n_q_cap ? (p.out_rows ? p.out_rows[qi] : qi) : -1;
  int fch[kMaxBlk];
#pragma unroll
  for (int j = 0; j < kMaxBlk; ++j) {
    fch[j] = -1;
    const int b = b_lo + j;
    if (j < nbl && b >= n_pb && tid < kTK) {
      const int jj = (fb0 + b - n_pb) * kTK + tid;
      fch[j] = jj < p.n_f_cap ? (p.fchild ? p.fchild[jj] : -1) : -2;
    }
  }
  const int n_q = p.n_q_dev ? min(*p.n_q_dev, p.n_q_cap) : p.n_q_cap;
  const int n_f = p.fk ? (p.n_f_dev ? min(*p.n_f_dev, p.n_f_cap) : p.n_f_cap) : 0;
  if (q0 >= n_q) {  // uniform over a cluster (its CTAs share blockIdx.x)
    // Nothing to compute; TMA writes into this CTA's shared memory land before it exits.
    if (tid == 0) {
      volatile int no_abort = 0;
      if (kv_tma) {
        mbar_wait(barK, 0, &no_abort);
        mbar_wait(barV, 0, &no_abort);
      }
      if (c_tma) {
        mbar_wait(barC, 0, &no_abort);
        mbar_wait(barCV, 0, &no_abort);
      }
    }
    __syncthreads();
    return;
  }
  if (warp == 0) tmem_alloc(smem_u32(tmem_slot), 512);

  // ---- operands (cp.async): whatever is not loaded by TMA ----
  if (!c_tma)
    load_op(sQ, [&](int rr) -> const __nv_bfloat16* {
      const int qi = q0 + rr;
      if (qi >= n_q) return nullptr;
      return p.q + (int64_t)(p.qsrc ? p.qsrc[qi] : qi) * p.q_ld + h * 128;
    }, p.q, tid);
  for (int j = 0; j < nbl; ++j) {
    const int b = b_lo + j;
    const bool parent_blk = b < n_pb;
    if (!parent_blk && tid < kTK) {
      const int jj = (fb0 + b - n_pb) * kTK + tid;
      int f = -1;
#pragma unroll
      for (int jx = 0; jx < kMaxBlk; ++jx)
        if (jx == j) f = fch[jx];
      sF[j * kTK + tid] = jj >= n_f ? -2 : f;
    }
    if ((parent_blk && kv_tma) || (!parent_blk && c_tma)) continue;
    const int r0 = (parent_blk ? b : fb0 + b - n_pb) * kTK;
    const int lim = parent_blk ? p.T : n_f;
    const __nv_bfloat16* kb = parent_blk ? p.pk : p.fk;
    const __nv_bfloat16* vb = parent_blk ? p.pv : p.fv;
    const int64_t ld = parent_blk ? p.kv_ld : p.f_ld;
    load_op(sKP + j * kOpB, [&](int rr) -> const __nv_bfloat16* {
      return r0 + rr < lim ? kb + (int64_t)(r0 + rr) * ld + kvh * 128 : nullptr;
    }, p.q, tid);
    load_op(sV + j * kOpB, [&](int rr) -> const __nv_bfloat16* {
      return r0 + rr < lim ? vb + (int64_t)(r0 + rr) * ld + kvh * 128 : nullptr;
    }, p.q, tid);
  }
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = tmem + ((uint32_t)(32 * qd) << 16);

  // ---- S_j = Q K_j^T ----
  if (tid == 0 && nbl > 0) {
    bool k_ok = true;
    volatile int no_abort = 0;
    if (kv_tma) k_ok = mbar_wait(barK, 0, &no_abort);
    if (c_tma) k_ok = mbar_wait(barC, 0, &no_abort) && k_ok;
    if (!k_ok) *fail = 1;
    tc_fence_after();
    const uint32_t idesc = idesc_bf16(kTQ, kTK);
    for (int j = 0; j < nbl && k_ok; ++j)
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t half = (uint32_t)(kk >> 2) * kTileB;
        tc_mma_bf16(tmem + (uint32_t)(j * kTK), sw128_desc(sQ + half) + 2 * (kk & 3),
                    sw128_desc(sKP + j * kOpB + half) + 2 * (kk & 3), idesc, kk > 0 ? 1u : 0u);
      }
    tc_commit(barS);  // also when nothing was issued, so the waits below end
  }
  if (n_fb < n_fb_all && tid == 0 && p.fchild) {
    // The window holds every candidate of this tile's children iff the
    // candidates just outside it belong to other children (the list is
    // ordered by child); otherwise keys would be missed: flag it.
    const int qa = q0, qb = min(q0 + kTQ, n_q) - 1;
    const int before = fb0 * kTK - 1, after = (fb0 + n_fb) * kTK;
    const bool miss = (before >= 0 && before < n_f && p.fchild[before] == p.fchild[qa]) ||
                      (after < n_f && p.fchild[after] == p.fchild[qb]);
    if (miss && p.status) atomicOr(p.status, AF_STATUS_CAPACITY);
  }

  // ---- masked softmax: row r, key columns c0..c0+31 of every block ----
  // The masks are built while S is computed.
  const bool row_ok = qi < n_q;
  const int child = row_ok ? child_ld : -1;
  uint32_t vm[kMaxBlk];  // valid keys among this thread's 32 columns of each block
  {
#pragma unroll
    for (int j = 0; j < kMaxBlk; ++j) {
      if (j >= nbl) break;
      const int b = b_lo + j;
      uint32_t v = 0;
      if (b < n_pb) {
        const int tw = b * kTK + c0;
        const int nv = min(32, max(0, p.T - tw));
        v = nv >= 32 ? 0xffffffffu : ((1u << nv) - 1u);
        if (p.fresh_bits && child >= 0 && nv > 0) v &= ~p.fresh_bits[(int64_t)child * p.bits_ld + (tw >> 5)];
      } else {
#pragma unroll 8
        for (int k = 0; k < 32; ++k) {
          const int cf = sF[j * kTK + c0 + k];
          if (cf == -1 || (cf >= 0 && cf == child)) v |= 1u << k;
        }
      }
      vm[j] = v;
    }
  }
  if (nbl > 0) {
    volatile int no_abort = 0;
    if (!mbar_wait(barS, 0, &no_abort)) *fail = 1;
  }
  const bool s_bad = __syncthreads_or(*fail);  // also: S is complete, Q's tiles are free for `red`
  tc_fence_after();
  // Output row of query row `tid` for the split combine (Q's tiles are free now).
  int* s_orow = reinterpret_cast<int*>(gb + kOffQ + 8 * kTQ * 4);
  if (ns > 1 && cg == 0) s_orow[r] = row_ok ? orow_ld : -1;
  float m = -INFINITY, l = 0.f;
  const float sc = p.scale_log2;
  if (!s_bad) {
    auto sweep1 = [&](int j, const uint32_t* sv) {
      const uint32_t v = vm[j];
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if ((v >> i) & 1u) m = fmaxf(m, __uint_as_float(sv[i]) * sc);
    };
    uint32_t sa[32], sb[32];
#pragma unroll
    for (int jp = 0; jp < kMaxBlk; jp += 2) {
      if (jp < nbl) {
        tmem_ld32_nowait(lane_base + (uint32_t)(jp * kTK + c0), sa);
        if (jp + 1 < nbl) tmem_ld32_nowait(lane_base + (uint32_t)((jp + 1) * kTK + c0), sb);
        tmem_wait_ld();
        sweep1(jp, sa);
        if (jp + 1 < nbl) sweep1(jp + 1, sb);
      }
    }
  }
  red[cg * kTQ + r] = m;
  __syncthreads();
  m = fmaxf(fmaxf(red[r], red[kTQ + r]), fmaxf(red[2 * kTQ + r], red[3 * kTQ + r]));
  if (!s_bad) {
    auto sweep2 = [&](int j, const uint32_t* sv) {
      const uint32_t v = vm[j];
#pragma unroll
      for (int g = 0; g < 4; ++g) {  // 8-key groups of the thread's 32 keys
        float pv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const bool ok = ((v >> (8 * g + i)) & 1u) && m != -INFINITY;
          // The special-function unit's exp2 (ex2.approx.ftz: relative error near
          // 2^-22, far below the bf16 rounding of P right after); x <= 0 here.
          float e;
          asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(__uint_as_float(sv[8 * g + i]) * sc - m));
          pv[i] = ok ? e : 0.f;
          l += pv[i];
        }
        const int key8 = (c0 >> 3) + g;
        const uint32_t dst = sKP + j * kOpB + (key8 >> 3) * kTileB + sw_off(r, key8 & 7);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(pack2(pv[0], pv[1])),
                     "r"(pack2(pv[2], pv[3])), "r"(pack2(pv[4], pv[5])), "r"(pack2(pv[6], pv[7]))
                     : "memory");
      }
    };
    // Blocks in pairs: both TMEM loads in flight before one wait.
    uint32_t sa[32], sb[32];
#pragma unroll
    for (int jp = 0; jp < kMaxBlk; jp += 2) {
      if (jp < nbl) {
        tmem_ld32_nowait(lane_base + (uint32_t)(jp * kTK + c0), sa);
        if (jp + 1 < nbl) tmem_ld32_nowait(lane_base + (uint32_t)((jp + 1) * kTK + c0), sb);
        tmem_wait_ld();
        sweep2(jp, sa);
        if (jp + 1 < nbl) sweep2(jp + 1, sb);
      }
    }
  }
  red[4 * kTQ + cg * kTQ + r] = l;
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  l = (red[4 * kTQ + r] + red[5 * kTQ + r]) + (red[6 * kTQ + r] + red[7 * kTQ + r]);

  // ---- O = sum_j P_j V_j ----
  const bool have_o = nbl > 0 && !s_bad;
  bool v_ok = true;
  if (tid == 0 && (kv_tma || c_tma)) {  // also on the failure paths: the V loads land before the CTA moves on
    volatile int no_abort = 0;
    if (kv_tma) v_ok = mbar_wait(barV, 0, &no_abort);
    if (c_tma) v_ok = mbar_wait(barCV, 0, &no_abort) && v_ok;
    if (!v_ok) *fail = 1;
    tc_fence_after();
  }
  if (tid == 0 && have_o) {
    const uint32_t idesc = idesc_bf16_bmn(kTQ, 128);
    for (int j = 0; j < nbl && v_ok; ++j)
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint64_t a = sw128_desc(sKP + j * kOpB + (uint32_t)(kk >> 2) * kTileB) + 2 * (kk & 3);
        const uint64_t bdesc = sw128_desc_mn(sV + j * kOpB + (uint32_t)kk * 2048u, kTileB, 1024);
        tc_mma_bf16(tmem + 3 * kTK, a, bdesc, idesc, (j | kk) != 0 ? 1u : 0u);
      }
    tc_commit(barO);
  }
  if (have_o) {
    volatile int no_abort = 0;
    if (!mbar_wait(barO, 0, &no_abort)) *fail = 1;
  }
  const bool bad = __syncthreads_or(*fail);
  if (bad && tid == 0 && p.status) atomicOr(p.status, AF_STATUS_TIMEOUT);
  tc_fence_after();

  // This thread's 32 head-dim columns of row r of O.
  uint32_t o[32];
  if (have_o && !bad) {
    tmem_ld32_nowait(lane_base + (uint32_t)(3 * kTK + c0), o);
    tmem_wait_ld();
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = 0u;
  }
  if (ns == 1) {
    const int orow = row_ok ? orow_ld : -1;
    if (orow >= 0 && !bad) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(p.out + (int64_t)orow * p.out_ld + h * 128 + c0);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 w;
        w.x = pack2(__uint_as_float(o[8 * c]) * inv, __uint_as_float(o[8 * c + 1]) * inv);
        w.y = pack2(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv);
        w.z = pack2(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv);
        w.w = pack2(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv);
        dst[c] = w;
      }
    }
  } else {
    // Each CTA stages its partial rows (O | m | l, fp32, padded rows) in its
    // idle P region, then one thread sends CTA k the rows k owns with a bulk
    // copy into k's idle V region (slot per source split), completing on k's
    // barX. Owners combine from their own shared memory; a last cluster
    // barrier keeps every CTA alive until the copies out of it are done.
    constexpr int kPoLd = 132;  // padded row: 128 values, m, l, 2 spare; conflict-free 16-byte accesses
    constexpr uint32_t kRowB = kPoLd * 4;
    const int rows_per = (kTQ + ns - 1) / ns;
    float* stg = reinterpret_cast<float*>(gb + kOffKP);   // [128][kPoLd] this split's partial rows
    float* rcv = reinterpret_cast<float*>(gb + kOffV);    // [ns - 1][rows_per][kPoLd] the other splits' rows
    const uint32_t stg_s = smem_u32(stg), rcv_s = smem_u32(rcv);
    {
      float* row = stg + r * kPoLd;
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        *reinterpret_cast<float4*>(row + c0 + i) = make_float4(__uint_as_float(o[i]), __uint_as_float(o[i + 1]),
                                                               __uint_as_float(o[i + 2]), __uint_as_float(o[i + 3]));
      if (cg == 0) *reinterpret_cast<float2*>(row + 128) = make_float2(bad ? -INFINITY : m, bad ? 0.f : l);
    }
    const int rlo = split * rows_per, rhi = min(kTQ, rlo + rows_per);
    if (tid == 0) mbar_arrive_expect_tx(barX, (uint32_t)((ns - 1) * (rhi - rlo)) * kRowB);
    fence_proxy_async();  // the staged rows are read by bulk copies (async proxy)
    __syncthreads();
    cluster_sync_all();  // every CTA's P.V is done: the V regions are free to receive
    if (tid == 0) {
      for (int k = 0; k < ns; ++k) {
        const int klo = k * rows_per, khi = min(kTQ, klo + rows_per);
        if (k == split || khi <= klo) continue;
        const uint32_t slot = (uint32_t)(split < k ? split : split - 1);
        bulk_copy_s2c(cluster_map(rcv_s + slot * (uint32_t)rows_per * kRowB, (uint32_t)k), stg_s + (uint32_t)klo * kRowB,
                      (uint32_t)(khi - klo) * kRowB, cluster_map(barX, (uint32_t)k));
      }
    }
    bool got = true;
    {
      volatile int no_abort = 0;
      got = mbar_wait(barX, 0, &no_abort);
    }
    if (!got && tid == 0 && p.status) atomicOr(p.status, AF_STATUS_TIMEOUT);
    for (int idx = tid; idx < (rhi - rlo) * 32 && got; idx += kThreads) {
      const int lr = idx / 32, c4 = idx % 32, rr = rlo + lr;
      const float* src[8];
      float mk[8], lk[8];
      float mx = -INFINITY;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (k < ns) {
          src[k] = k == split ? stg + rr * kPoLd : rcv + ((k < split ? k : k - 1) * rows_per + lr) * kPoLd;
          const float2 v = *reinterpret_cast<const float2*>(src[k] + 128);
          mk[k] = v.x;
          lk[k] = v.y;
          mx = fmaxf(mx, v.x);
        }
      }
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      float lsum = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (k < ns && mk[k] != -INFINITY) {
          const float4 v = *reinterpret_cast<const float4*>(src[k] + 4 * c4);
          const float f = exp2f(mk[k] - mx);
          lsum += f * lk[k];
          acc.x += f * v.x;
          acc.y += f * v.y;
          acc.z += f * v.z;
          acc.w += f * v.w;
        }
      }
      const int orow = s_orow[rr];
      if (orow >= 0 && !bad) {
        const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
        uint2 w;
        w.x = pack2(acc.x * inv, acc.y * inv);
        w.y = pack2(acc.z * inv, acc.w * inv);
        *reinterpret_cast<uint2*>(p.out + (int64_t)orow * p.out_ld + h * 128 + 4 * c4) = w;
      }
    }
    __syncwarp();
    cluster_sync_all();  // every CTA has received its rows: the copies out of this CTA are done
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Key splits for the tcgen05 kernel, or 0 when the shape needs more than
// kMaxBlk blocks per split in an 8-CTA cluster.
int attention_tc_splits(const AttnParams& p) {
  const int nb = (p.T + kTK - 1) / kTK + cand_blocks(p);
  const int need = (nb + kMaxBlk - 1) / kMaxBlk;
  if (need > 8) return 0;
  // The slowest CTA (most key blocks) sets the time; among the split counts
  // that fit one wave, take the fewest that reach the smallest per-CTA block
  // count: more splits at the same maximum only add CTAs to wait on and
  // partials to combine.
  const int ctas = (p.n_q_cap + kTQ - 1) / kTQ * p.n_heads;
  int ns = need;
  while (ns < 8 && ns < nb && (ns + 1) * ctas <= sm_count()) ++ns;
  const int most = (nb + ns - 1) / ns;
  while (ns > need && (nb + ns - 2) / (ns - 1) == most) --ns;
  return ns;
}

// Tensor maps of a cached parent's K or V ([T keys, n_kv_heads * 128] columns
// of a row-major buffer with row stride ld, or head-major [heads][T][128]
// when cols < 0), reused across passes: the parent cache keeps its buffers
// for its lifetime.
int attention_kv_tmap(CUtensorMap* map, const __nv_bfloat16* base, int T, int cols, int64_t ld) {
  struct Entry {
    const void* base;
    int T, cols;
    int64_t ld;
    CUtensorMap map;
  };
  static std::mutex mu;
  static std::vector<Entry> cache;
  std::lock_guard<std::mutex> lock(mu);
  for (const Entry& e : cache)
    if (e.base == base && e.T == T && e.cols == cols && e.ld == ld) {
      *map = e.map;
      return AF_OK;
    }
  Entry e{base, T, cols, ld, {}};
  // cols < 0: head-major layout of -cols heads ([heads][T][128]).
  if (int st = cols < 0 ? make_tmap_bf16_heads(&e.map, base, (uint64_t)T, (uint64_t)(-cols))
                        : make_tmap_bf16(&e.map, base, (uint64_t)T, (uint64_t)cols, (uint64_t)ld, 128))
    return st;
  if (cache.size() >= 512) cache.erase(cache.begin());
  cache.push_back(e);
  *map = e.map;
  return AF_OK;
}

int attention_tc_run(const AttnParams& p, int ns, cudaStream_t s) {
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_attention_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTc);
    attr = true;
  }
  CUtensorMap tk, tv, tc;
  memset(&tk, 0, sizeof(tk));
  memset(&tv, 0, sizeof(tv));
  memset(&tc, 0, sizeof(tc));
  if (p.cand_tma) {
    AF_REQUIRE(p.tmap_c && !p.qsrc && p.fk && p.fv && p.f_ld == p.q_ld && (p.fk_col | p.fv_col) % 8 == 0,
               "attention_tc: candidate-row mode needs a buffer map, contiguous queries and key columns in that buffer");
    tc = *p.tmap_c;
  }
  if (p.kv_static && p.kv_hm) {
    const __nv_bfloat16* vbase = p.kv_hm + (int64_t)p.n_kv_heads * p.T * 128;
    if (int st = attention_kv_tmap(&tk, p.kv_hm, p.T, -p.n_kv_heads, 0)) return st;
    if (int st = attention_kv_tmap(&tv, vbase, p.T, -p.n_kv_heads, 0)) return st;
  } else if (p.kv_static) {
    const int cols = p.n_kv_heads * 128;
    if (int st = attention_kv_tmap(&tk, p.pk, p.T, cols, p.kv_ld)) return st;
    if (int st = attention_kv_tmap(&tv, p.pv, p.T, cols, p.kv_ld)) return st;
  }
  cudaError_t e = launch_ex(k_attention_tc, dim3((p.n_q_cap + kTQ - 1) / kTQ, p.n_heads, ns), dim3(kThreads, 1, 1),
                            (size_t)kSmemTc, s, p.pdl != 0, dim3(1, 1, ns), tk, tv, tc, p);
  if (e != cudaSuccess) return fail(AF_ERR_CUDA, std::string("attention_tc: launch: ") + cudaGetErrorString(e));
  return check_launch("attention_tc");
}

}  // namespace af
