// Flash-style tcgen05 attention (sm_100a): one CTA per (128 query rows, head)
// streams every key block of that head through a two-stage shared-memory ring
// and keeps the softmax online, so no key split and no cross-CTA combine is
// needed. Same semantics as k_attention_tc (attention_tc.cu): query row i
// (child qchild[i]) attends to every parent position t except the fresh
// positions of its child, and to its child's candidate keys.
//
// Warps 0-15 run the softmax (warp w: TMEM lane quadrant w & 3 = 32 query
// rows, column group w >> 2 = 32 of the 128 key columns, then 32 of the 128
// head-dim columns of O); warp 16 issues the TMA loads, warp 17 the MMAs:
//   S_j = Q K_j^T     into TMEM buffer j & 1 (two 128-column buffers),
//   P_j = exp2(S_j * scale - m) in bf16 over K_j's tiles (K_j is consumed),
//   O  += P_j V_j     (TMEM columns 256..383),
// with S_{j+1} computed while the softmax of block j runs. The running row
// maximum m is raised only when a block's maximum exceeds it by more than
// 2^8 (then O and the partial row sums are rescaled); otherwise P stays below
// 256, which bf16 and the fp32 sums hold exactly as well. Every mbarrier wait
// is bounded; a timeout sets AF_STATUS_TIMEOUT.
#include <cstring>

#include "attention.cuh"
#include "tc_common.cuh"

namespace af {

namespace {

constexpr int kFQ = 128;                    // query rows per CTA (MMA M)
constexpr int kFK = 128;                    // keys per block
constexpr int kFSoftWarps = 16;             // 4 lane quadrants x 4 column groups
constexpr int kFThreads = (kFSoftWarps + 2) * 32;
constexpr int kFTileB = 128 * 64 * 2;       // [128 rows][64 cols] bf16 = 16 KB
constexpr int kFOpB = 2 * kFTileB;          // 128 x 128 operand
constexpr int kFOffQ = 0;
constexpr int kFOffK = kFOffQ + kFOpB;      // K stage s (then P), s = 0, 1
constexpr int kFOffV = kFOffK + 2 * kFOpB;  // V stage s
constexpr int kFOffRed = kFOffV + 2 * kFOpB;  // [2][4][128] floats: per-column-group row maxima (by block parity)
constexpr int kFOffBar = kFOffRed + 2 * 4 * kFQ * 4;
// barQ, barK[2], barV[2], barS[2], barP[2], barO[2], barE[2], TMEM slot, fail flag
constexpr int kFSmem = kFOffBar + 128 + 1024;  // + alignment slack
constexpr float kFRescale = 8.f;            // log2 headroom before the running maximum is raised

__device__ __forceinline__ uint32_t swz(int row, int ch) { return (uint32_t)(row * 128 + ((ch ^ (row & 7)) << 4)); }

__device__ __forceinline__ uint32_t pack2f(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// 32 lanes x 32 columns of 32-bit TMEM data from registers (lane = thread).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

}  // namespace

// Key blocks of a CTA: the T parent keys in blocks of 128, then its window of
// candidate blocks (all of them outside candidate-row mode).
struct FaBlocks {
  int n_pb, n_fb, fb0;
  __device__ __forceinline__ int count() const { return n_pb + n_fb; }
};

__device__ __forceinline__ FaBlocks fa_blocks(const AttnParams& p, int qtile) {
  FaBlocks b;
  b.n_pb = (p.T + kFK - 1) / kFK;
  const int all = p.fk ? (p.n_f_cap + kFK - 1) / kFK : 0;
  b.n_fb = (p.cand_tma && p.cand_win > 0 && p.cand_win < all) ? p.cand_win : all;
  b.fb0 = b.n_fb < all ? min(max(qtile - (p.cand_win - 1) / 2, 0), all - b.n_fb) : 0;
  return b;
}

__global__ void __launch_bounds__(kFThreads, 1) k_attention_fa(const __grid_constant__ CUtensorMap tmQ,
                                                               const __grid_constant__ CUtensorMap tmK,
                                                               const __grid_constant__ CUtensorMap tmV,
                                                               const __grid_constant__ CUtensorMap tmC,
                                                               const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  pdl_trigger();
  const int q0 = blockIdx.x * kFQ;
  const int h = blockIdx.y;
  const int kvh = h / (p.n_heads / p.n_kv_heads);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const FaBlocks kb = fa_blocks(p, blockIdx.x);
  const int nb = kb.count();

  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gb = smem_raw + (base - raw);
  const uint32_t sQ = base + kFOffQ, sK = base + kFOffK, sV = base + kFOffV;
  float* red = reinterpret_cast<float*>(gb + kFOffRed);
  const uint32_t bars = base + kFOffBar;
  // barO[i & 1] completes when P_i V_i has: with two barriers a waiter is
  // never more than one phase behind either of them (see the softmax loop).
  const uint32_t barQ = bars, barK = bars + 8, barV = bars + 24, barS = bars + 40, barP = bars + 56, barO = bars + 72,
                 barE = bars + 88;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gb + kFOffBar + 104);
  volatile int* fail = reinterpret_cast<volatile int*>(gb + kFOffBar + 112);
  const bool producer = warp == kFSoftWarps && lane == 0;
  const bool mma = warp == kFSoftWarps + 1 && lane == 0;

  if (tid == 0) {
    mbar_init(barQ, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(barK + 8 * s, 1);
      mbar_init(barV + 8 * s, 1);
      mbar_init(barS + 8 * s, 1);
      mbar_init(barP + 8 * s, kFSoftWarps);
      mbar_init(barE + 8 * s, 1);
      mbar_init(barO + 8 * s, 1);
    }
    *fail = 0;
    fence_barrier_init();
  }
  __syncthreads();

  // Key block j into ring stage j & 1: parent blocks from the parent's K / V
  // (head-major maps when present), candidate blocks from the QKV buffer.
  auto issue_kv = [&](int j) {
    const int st = j & 1;
    const uint32_t dK = sK + st * kFOpB, dV = sV + st * kFOpB;
    mbar_arrive_expect_tx(barK + 8 * st, kFOpB);
    mbar_arrive_expect_tx(barV + 8 * st, kFOpB);
    if (j < kb.n_pb) {
      for (int hf = 0; hf < 2; ++hf) {
        if (p.kv_hm) tma_load_3d(dK + hf * kFTileB, &tmK, barK + 8 * st, 64 * hf, j * kFK, kvh);
        else tma_load_2d(dK + hf * kFTileB, &tmK, barK + 8 * st, kvh * 128 + 64 * hf, j * kFK);
      }
      for (int hf = 0; hf < 2; ++hf) {
        if (p.kv_hm) tma_load_3d(dV + hf * kFTileB, &tmV, barV + 8 * st, 64 * hf, j * kFK, kvh);
        else tma_load_2d(dV + hf * kFTileB, &tmV, barV + 8 * st, kvh * 128 + 64 * hf, j * kFK);
      }
    } else {
      const int y = (kb.fb0 + j - kb.n_pb) * kFK;
      for (int hf = 0; hf < 2; ++hf)
        tma_load_2d(dK + hf * kFTileB, &tmC, barK + 8 * st, p.fk_col + kvh * 128 + 64 * hf, y);
      for (int hf = 0; hf < 2; ++hf)
        tma_load_2d(dV + hf * kFTileB, &tmC, barV + 8 * st, p.fv_col + kvh * 128 + 64 * hf, y);
    }
  };
  // A cached parent's first blocks do not depend on the preceding kernel.
  const int n_early = p.kv_static ? min(min(2, nb), kb.n_pb) : 0;
  if (producer) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    for (int j = 0; j < n_early; ++j) issue_kv(j);
  }
  pdl_wait();
  const int n_q = p.n_q_dev ? min(*p.n_q_dev, p.n_q_cap) : p.n_q_cap;
  if (q0 >= n_q) {
    // Nothing to compute; TMA writes into this CTA's shared memory land before it exits.
    if (producer) {
      volatile int no_abort = 0;
      for (int j = 0; j < n_early; ++j) {
        mbar_wait(barK + 8 * j, 0, &no_abort);
        mbar_wait(barV + 8 * j, 0, &no_abort);
      }
    }
    __syncthreads();
    return;
  }
  if (warp == 0) tmem_alloc(smem_u32(tmem_slot), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (producer) {
    // ---------------- TMA producer ----------------
    mbar_arrive_expect_tx(barQ, kFOpB);
    for (int hf = 0; hf < 2; ++hf) tma_load_2d(sQ + hf * kFTileB, &tmQ, barQ, h * 128 + 64 * hf, q0);
    for (int j = n_early; j < nb; ++j) {
      if (j >= 2 && !mbar_wait(barE + 8 * (j & 1), ((j - 2) >> 1) & 1, fail)) {
        *fail = 1;
        break;
      }
      issue_kv(j);
    }
    if (kb.n_fb > 0 && p.fchild && p.cand_win > 0) {
      // The window holds every candidate of this tile's children iff the
      // candidates just outside it belong to other children (the list is
      // ordered by child); otherwise keys would be missed: flag it.
      const int n_f = p.n_f_dev ? min(*p.n_f_dev, p.n_f_cap) : p.n_f_cap;
      const int qa = q0, qb = min(q0 + kFQ, n_q) - 1;
      const int before = kb.fb0 * kFK - 1, after = (kb.fb0 + kb.n_fb) * kFK;
      const bool miss = (before >= 0 && before < n_f && p.fchild[before] == p.fchild[qa]) ||
                        (after < n_f && p.fchild[after] == p.fchild[qb]);
      if (miss && p.status) atomicOr(p.status, AF_STATUS_CAPACITY);
    }
  } else if (mma) {
    // ---------------- MMA issuer: S_j, then P_{j-1} V_{j-1} ----------------
    const uint32_t idS = idesc_bf16(kFQ, kFK), idO = idesc_bf16_bmn(kFQ, 128);
    bool ok = mbar_wait(barQ, 0, fail);
    for (int j = 0; j <= nb && ok; ++j) {
      if (j < nb) {
        const int sb = j & 1;
        ok = mbar_wait(barK + 8 * sb, (j >> 1) & 1, fail);
        if (ok && j >= 2) ok = mbar_wait(barP + 8 * sb, ((j - 2) >> 1) & 1, fail);  // S buffer sb is read
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t half = (uint32_t)(kk >> 2) * kFTileB;
          tc_mma_bf16(tmem + (uint32_t)(sb * kFK), sw128_desc(sQ + half) + 2 * (kk & 3),
                      sw128_desc(sK + sb * kFOpB + half) + 2 * (kk & 3), idS, kk > 0 ? 1u : 0u);
        }
        tc_commit(barS + 8 * sb);
      }
      if (j >= 1) {
        const int i = j - 1, st = i & 1;
        ok = mbar_wait(barP + 8 * st, (i >> 1) & 1, fail) && mbar_wait(barV + 8 * st, (i >> 1) & 1, fail);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t a = sw128_desc(sK + st * kFOpB + (uint32_t)(kk >> 2) * kFTileB) + 2 * (kk & 3);
          const uint64_t b = sw128_desc_mn(sV + st * kFOpB + (uint32_t)kk * 2048u, kFTileB, 1024);
          tc_mma_bf16(tmem + 2 * kFK, a, b, idO, (i | kk) != 0 ? 1u : 0u);
        }
        tc_commit(barO + 8 * st);
        tc_commit(barE + 8 * st);
      }
    }
    if (!ok) {
      *fail = 1;
      if (p.status) atomicOr(p.status, AF_STATUS_TIMEOUT);
    }
  } else if (warp < kFSoftWarps) {
    // ---------------- online softmax of row r, columns c0..c0+31 ----------------
    const int qd = warp & 3, cg = warp >> 2;
    const int r = 32 * qd + lane, c0 = 32 * cg;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * qd) << 16);
    const int qi = q0 + r;
    const bool row_ok = qi < n_q;
    const int child = (p.qchild && row_ok) ? p.qchild[qi] : -1;
    const int n_f = p.fk ? (p.n_f_dev ? min(*p.n_f_dev, p.n_f_cap) : p.n_f_cap) : 0;
    const float sc = p.scale_log2;
    // Inputs of block j's key mask, requested one block ahead: the fresh-bit
    // word of a parent block, or (lane k) the child of candidate key c0 + k.
    auto mask_input = [&](int j) -> uint32_t {
      if (j >= nb) return 0u;
      if (j < kb.n_pb) {
        const int tw = j * kFK + c0;
        return (p.fresh_bits && child >= 0 && tw < p.T) ? p.fresh_bits[(int64_t)child * p.bits_ld + (tw >> 5)] : 0u;
      }
      const int jj = (kb.fb0 + j - kb.n_pb) * kFK + c0 + lane;
      return (uint32_t)(jj >= n_f ? -2 : (p.fchild ? p.fchild[jj] : -1));
    };
    uint32_t in_next = mask_input(0);
    float m_run = -INFINITY, l_part = 0.f;
    uint32_t s[32];
    for (int j = 0; j < nb; ++j) {
      const int sb = j & 1;
      const uint32_t in = in_next;
      in_next = mask_input(j + 1);
      uint32_t v = 0;
      if (j < kb.n_pb) {
        const int tw = j * kFK + c0;
        const int nv = min(32, max(0, p.T - tw));
        v = (nv >= 32 ? 0xffffffffu : ((1u << nv) - 1u)) & ~in;
      } else {
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const int cf = __shfl_sync(0xffffffffu, (int)in, k);
          if (cf == -1 || (cf >= 0 && cf == child)) v |= 1u << k;
        }
      }
      mbar_wait(barS + 8 * sb, (j >> 1) & 1, fail);
      tc_fence_after();
      tmem_ld32_nowait(lane_base + (uint32_t)(sb * kFK + c0), s);
      tmem_wait_ld();
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if ((v >> i) & 1u) mx = fmaxf(mx, __uint_as_float(s[i]) * sc);
      float* rb = red + sb * 4 * kFQ;
      rb[cg * kFQ + r] = mx;
      named_bar_sync(1 + qd, 128);
      const float m_blk = fmaxf(fmaxf(rb[r], rb[kFQ + r]), fmaxf(rb[2 * kFQ + r], rb[3 * kFQ + r]));
      // P_{j-2} V_{j-2} is observed at every block (long done by now), so
      // each O barrier is at most one phase ahead of any wait on it: P_i V_i
      // needs P_i, which this thread has not produced for i >= j.
      if (j >= 2) mbar_wait(barO + 8 * (j & 1), ((j - 2) >> 1) & 1, fail);
      // Raise the running maximum only when this block exceeds it by more
      // than 2^kFRescale (the first finite block always does).
      const bool raise = m_blk > m_run + kFRescale;
      if (__any_sync(0xffffffffu, raise)) {
        const float m_new = raise ? m_blk : m_run;
        const float alpha = raise ? (m_run == -INFINITY ? 0.f : exp2f(m_run - m_new)) : 1.f;
        l_part *= alpha;
        if (j > 0) {
          // O holds blocks 0..j-1 once P_{j-1} V_{j-1} has completed.
          mbar_wait(barO + 8 * ((j - 1) & 1), ((j - 1) >> 1) & 1, fail);
          tc_fence_after();
          uint32_t o[32];
          tmem_ld32_nowait(lane_base + (uint32_t)(2 * kFK + c0), o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(lane_base + (uint32_t)(2 * kFK + c0), o);
          tmem_wait_st();
        }
        m_run = m_new;
      }
#pragma unroll
      for (int g = 0; g < 4; ++g) {  // 8-key groups of the thread's 32 keys
        float pv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const bool ok = ((v >> (8 * g + i)) & 1u) && m_run != -INFINITY;
          // The special-function unit's exp2 (ex2.approx.ftz: relative error near
          // 2^-22, far below the bf16 rounding of P right after); x <= 8 here.
          float e;
          asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(__uint_as_float(s[8 * g + i]) * sc - m_run));
          pv[i] = ok ? e : 0.f;
          l_part += pv[i];
        }
        const int key8 = (c0 >> 3) + g;
        const uint32_t dst = sK + sb * kFOpB + (key8 >> 3) * kFTileB + swz(r, key8 & 7);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(pack2f(pv[0], pv[1])),
                     "r"(pack2f(pv[2], pv[3])), "r"(pack2f(pv[4], pv[5])), "r"(pack2f(pv[6], pv[7]))
                     : "memory");
      }
      fence_proxy_async_smem();  // P_j is read by the MMA (async proxy)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(barP + 8 * sb);
    }
    // ---- O / l for row r, head-dim columns c0..c0+31 ----
    float* rl = red + (nb & 1) * 4 * kFQ;
    rl[cg * kFQ + r] = l_part;
    named_bar_sync(1 + qd, 128);
    const float l = (rl[r] + rl[kFQ + r]) + (rl[2 * kFQ + r] + rl[3 * kFQ + r]);
    bool got = nb > 0 && mbar_wait(barO + 8 * ((nb - 1) & 1), ((nb - 1) >> 1) & 1, fail);
    tc_fence_after();
    uint32_t o[32];
    tmem_ld32_nowait(lane_base + (uint32_t)(2 * kFK + c0), o);
    tmem_wait_ld();
    const int orow = row_ok ? (p.out_rows ? p.out_rows[qi] : qi) : -1;
    if (orow >= 0 && got && !*fail) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(p.out + (int64_t)orow * p.out_ld + h * 128 + c0);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint4 w;
        w.x = pack2f(__uint_as_float(o[8 * c]) * inv, __uint_as_float(o[8 * c + 1]) * inv);
        w.y = pack2f(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv);
        w.z = pack2f(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv);
        w.w = pack2f(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv);
        dst[c] = w;
      }
    }
    if (!got && lane == 0 && p.status) atomicOr(p.status, AF_STATUS_TIMEOUT);
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (tid == 0 && *fail) {
    // Loads that may still be in flight into this CTA's ring land before it exits (bounded).
    volatile int no_abort = 0;
    for (int j = max(0, nb - 2); j < nb; ++j) {
      mbar_wait(barK + 8 * (j & 1), (j >> 1) & 1, &no_abort);
      mbar_wait(barV + 8 * (j & 1), (j >> 1) & 1, &no_abort);
    }
  }
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Kernel choice: AF_ATTN_AUTO / STREAM / SPLIT (af_set_attention_kernel; the
// environment variable ACTFOLD_ATTN_FA=1 / 0 sets the starting value).
static int g_attn_kind = [] {
  const char* e = std::getenv("ACTFOLD_ATTN_FA");
  return e ? (e[0] == '0' ? AF_ATTN_SPLIT : AF_ATTN_STREAM) : AF_ATTN_AUTO;
}();

bool attention_fa_ok(const AttnParams& p) {
  if (g_attn_kind == AF_ATTN_SPLIT) return false;
  // Queries are contiguous rows (no gather), and candidate keys, if any, come
  // as TMA boxes of the QKV buffer.
  if (p.qsrc || p.n_q_cap <= 0 || p.T <= 0 || (p.fk && !(p.cand_tma && p.tmap_c))) return false;
  // A CTA walks its key blocks one after another (~2.3 us each on B200, the
  // K / V reload, S, the softmax and P.V of a block in a chain), so this
  // kernel pays off when its (query tile, head) CTAs fill the GPU (the dense
  // parent pass) or when the key-split kernel cannot take the sequence; few
  // query tiles over a short sequence (the folded pass) run faster as key
  // splits in parallel CTAs.
  if (g_attn_kind == AF_ATTN_STREAM) return true;
  const int ctas = (p.n_q_cap + kFQ - 1) / kFQ * p.n_heads;
  return ctas >= sm_count() || attention_tc_splits(p) == 0;
}

int attention_fa_run(const AttnParams& p, cudaStream_t s) {
  AF_REQUIRE(attention_fa_ok(p), "attention_fa: unsupported parameters");
  AF_REQUIRE(!p.fk || (p.fchild && p.f_ld == p.q_ld && (p.fk_col | p.fv_col) % 8 == 0),
             "attention_fa: candidate keys need their children and columns of the query buffer");
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_attention_fa, cudaFuncAttributeMaxDynamicSharedMemorySize, kFSmem);
    attr = true;
  }
  CUtensorMap tq, tk, tv, tc;
  memset(&tk, 0, sizeof(tk));
  memset(&tv, 0, sizeof(tv));
  memset(&tc, 0, sizeof(tc));
  if (p.cand_tma) {
    tq = *p.tmap_c;
    tc = *p.tmap_c;
  } else if (int st = make_tmap_bf16(&tq, p.q, (uint64_t)p.n_q_cap, (uint64_t)p.q_ld, (uint64_t)p.q_ld, 128)) {
    return st;
  }
  if (p.kv_hm) {
    const __nv_bfloat16* vbase = p.kv_hm + (int64_t)p.n_kv_heads * p.T * 128;
    if (int st = attention_kv_tmap(&tk, p.kv_hm, p.T, -p.n_kv_heads, 0)) return st;
    if (int st = attention_kv_tmap(&tv, vbase, p.T, -p.n_kv_heads, 0)) return st;
  } else if (p.kv_static) {
    if (int st = attention_kv_tmap(&tk, p.pk, p.T, p.n_kv_heads * 128, p.kv_ld)) return st;
    if (int st = attention_kv_tmap(&tv, p.pv, p.T, p.n_kv_heads * 128, p.kv_ld)) return st;
  } else {
    // K / V of this pass (written just before): maps are built per call.
    if (int st = make_tmap_bf16(&tk, p.pk, (uint64_t)p.T, (uint64_t)p.n_kv_heads * 128, (uint64_t)p.kv_ld, 128)) return st;
    if (int st = make_tmap_bf16(&tv, p.pv, (uint64_t)p.T, (uint64_t)p.n_kv_heads * 128, (uint64_t)p.kv_ld, 128)) return st;
  }
  cudaError_t e = launch_ex(k_attention_fa, dim3((p.n_q_cap + kFQ - 1) / kFQ, p.n_heads, 1), dim3(kFThreads, 1, 1),
                            (size_t)kFSmem, s, p.pdl != 0, dim3(1, 1, 1), tq, tk, tv, tc, p);
  if (e != cudaSuccess) return fail(AF_ERR_CUDA, std::string("attention_fa: launch: ") + cudaGetErrorString(e));
  return check_launch("attention_fa");
}

}  // namespace af

extern "C" int af_set_attention_kernel(int kind) {
  AF_REQUIRE(kind == AF_ATTN_AUTO || kind == AF_ATTN_STREAM || kind == AF_ATTN_SPLIT,
             "af_set_attention_kernel: kind must be AF_ATTN_AUTO, AF_ATTN_STREAM or AF_ATTN_SPLIT");
  af::g_attn_kind = kind;
  return AF_OK;
}
