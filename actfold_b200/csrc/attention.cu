// Non-causal attention of packed query rows over a parent K/V cache with
// per-child overrides (sm_100a; bf16 tensor-core mma, fp32 softmax).
//
// Query row i belongs to child qchild[i]. Its keys are every position t of the
// sequence: the parent's cached K/V row t, except where t is "fresh" for that
// child (its layer input differs from the parent's), in which case the key is
// the child's recomputed K/V row, found among the layer's candidate rows
// (fchild[j] == qchild[i]). Both segments go through one online softmax:
// parent blocks with fresh positions masked out, then the candidate blocks
// masked to the query's own child. With no fresh data this is plain
// non-causal attention (the parent pass).
//
// CTA = 4 warps, 64 query rows of one head; each warp owns 16 rows. K/V blocks
// of 64 keys are double-buffered in XOR-swizzled shared memory with cp.async;
// S = Q K^T and O += P V use mma.m16n8k16 (bf16 in, fp32 accumulate).
//
// Key split: when few query rows give few CTAs (the folded pass packs only the
// divergent rows), the key blocks of one (query block, head) are divided over
// the S CTAs of a thread-block cluster (grid z). Each CTA leaves its softmax
// partials (row max m, row sum l, unnormalised O) in its own shared memory;
// after a cluster barrier CTA z combines rows [z*64/S, (z+1)*64/S) from all S
// partials through distributed shared memory and writes them, and a second
// barrier keeps every CTA's partials alive until its peers have read them.
#include <cstdlib>

#include "attention.cuh"

namespace af {

constexpr int kHD = 128, kQB = 64, kKB = 64;
constexpr int kSmemKV = 16384 + 2 * 32768;      // Q tile + two K/V stages
constexpr int kSmem = kSmemKV + 2 * kKB * 4;    // + candidate-key children per stage

__device__ __forceinline__ uint32_t swz(int row, int chunk) {  // byte offset in a [64][128] bf16 tile
  return (uint32_t)(row * 256 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__global__ void __launch_bounds__(128) k_attention(const AttnParams p) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(128) uint8_t sm[];
  const int n_q = p.n_q_dev ? min(*p.n_q_dev, p.n_q_cap) : p.n_q_cap;
  const int q0 = blockIdx.x * kQB;
  if (q0 >= n_q) return;
  const int h = blockIdx.y;
  const int ns = gridDim.z, split = blockIdx.z;  // key splits = cluster size along z
  const int kvh = h / (p.n_heads / p.n_kv_heads);
  const int n_f = p.fk ? (p.n_f_dev ? min(*p.n_f_dev, p.n_f_cap) : p.n_f_cap) : 0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t4 = lane & 3;

  const uint32_t sQ = static_cast<uint32_t>(__cvta_generic_to_shared(sm));
  const uint32_t sK[2] = {sQ + 16384, sQ + 16384 + 32768};
  const uint32_t sV[2] = {sQ + 16384 + 16384, sQ + 16384 + 32768 + 16384};
  int* sF = reinterpret_cast<int*>(sm + kSmemKV);  // [2][kKB] child of each candidate key of a block

  // ---- Q tile (64 rows x 128) ----
  for (int idx = tid; idx < kQB * 16; idx += 128) {
    const int r = idx >> 4, c = idx & 15;
    const int qi = q0 + r;
    const bool ok = qi < n_q;
    const int src = ok ? (p.qsrc ? p.qsrc[qi] : qi) : 0;
    cp_async16(sQ + swz(r, c), p.q + (int64_t)src * p.q_ld + h * kHD + c * 8, ok);
  }
  cp_commit();

  const int n_pb = (p.T + kKB - 1) / kKB;
  const int n_fb = (n_f + kKB - 1) / kKB;
  const int n_blocks = n_pb + n_fb;
  const int b_lo = split * n_blocks / ns, b_hi = (split + 1) * n_blocks / ns;  // balanced, possibly empty

  auto load_block = [&](int b, int buf) {
    for (int idx = tid; idx < kKB * 16; idx += 128) {
      const int r = idx >> 4, c = idx & 15;
      const __nv_bfloat16 *ks, *vs;
      bool ok;
      if (b < n_pb) {
        const int t = b * kKB + r;
        ok = t < p.T;
        const int64_t off = (int64_t)(ok ? t : 0) * p.kv_ld + kvh * kHD + c * 8;
        ks = p.pk + off;
        vs = p.pv + off;
      } else {
        const int j = (b - n_pb) * kKB + r;
        ok = j < n_f;
        const int64_t off = (int64_t)(ok ? j : 0) * p.f_ld + kvh * kHD + c * 8;
        ks = p.fk + off;
        vs = p.fv + off;
      }
      cp_async16(sK[buf] + swz(r, c), ks, ok);
      cp_async16(sV[buf] + swz(r, c), vs, ok);
    }
    cp_commit();
    if (b >= n_pb && tid < kKB) {
      const int j = (b - n_pb) * kKB + tid;
      sF[buf * kKB + tid] = j >= n_f ? -2 : (p.fchild ? p.fchild[j] : -1);
    }
  };

  if (b_lo < b_hi) load_block(b_lo, 0);

  // Per-thread rows: r0 = 16*warp + g, r1 = r0 + 8 (within the CTA's 64).
  const int row0 = q0 + 16 * warp + g, row1 = row0 + 8;
  const int child0 = (p.qchild && row0 < n_q) ? p.qchild[row0] : -1;
  const int child1 = (p.qchild && row1 < n_q) ? p.qchild[row1] : -1;

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  uint32_t qa[8][4];

  for (int b = b_lo; b < b_hi; ++b) {
    const int buf = (b - b_lo) & 1;
    if (b + 1 < b_hi) {
      load_block(b + 1, buf ^ 1);
      cp_wait_1();
    } else {
      cp_wait_0();
    }
    __syncthreads();
    if (b == b_lo) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int r = 16 * warp + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = 2 * kk + (lane >> 4);
        ldsm_x4(sQ + swz(r, c), qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3]);
      }
    }
    // ---- S = Q K^T (16 x 64 per warp) ----
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {  // pairs of n8 tiles
        uint32_t b0, b1, b2, b3;
        const int r = 16 * jp + (lane & 7) + ((lane >> 4) << 3);
        const int c = 2 * kk + ((lane >> 3) & 1);
        ldsm_x4(sK[buf] + swz(r, c), b0, b1, b2, b3);
        mma16816(s[2 * jp], qa[kk], b0, b1);
        mma16816(s[2 * jp + 1], qa[kk], b2, b3);
      }
    }
    // ---- mask + online softmax ----
    // Valid keys of this block as 64-bit masks for the thread's two rows:
    // parent keys minus the row's fresh positions, or the candidate keys of
    // the row's own child (-1 in sF: no child filter; -2: past n_f).
    const bool parent_blk = b < n_pb;
    uint64_t v0, v1;
    if (parent_blk) {
      const int t0 = b * kKB;
      const int nvalid = min(kKB, p.T - t0);
      const uint64_t range = nvalid >= 64 ? ~0ull : ((1ull << nvalid) - 1ull);
      uint64_t f0 = 0, f1 = 0;
      if (p.fresh_bits) {
        const int w = t0 >> 5;
        if (child0 >= 0) {
          const uint32_t* fb = p.fresh_bits + (int64_t)child0 * p.bits_ld;
          f0 = (uint64_t)fb[w] | ((w + 1 < p.bits_ld) ? (uint64_t)fb[w + 1] << 32 : 0ull);
        }
        if (child1 >= 0) {
          const uint32_t* fb = p.fresh_bits + (int64_t)child1 * p.bits_ld;
          f1 = (uint64_t)fb[w] | ((w + 1 < p.bits_ld) ? (uint64_t)fb[w + 1] << 32 : 0ull);
        }
      }
      v0 = range & ~f0;
      v1 = range & ~f1;
    } else {
      v0 = v1 = 0;
      const int* fc = sF + buf * kKB;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int key = 8 * j + 2 * t4 + e;
          const int cf = fc[key];
          if (cf == -1 || (cf >= 0 && cf == child0)) v0 |= 1ull << key;
          if (cf == -1 || (cf >= 0 && cf == child1)) v1 |= 1ull << key;
        }
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = 8 * j + 2 * t4 + (e & 1);
        const bool valid = (((e < 2) ? v0 : v1) >> key) & 1ull;
        const float v = valid ? s[j][e] * p.scale_log2 : -INFINITY;
        s[j][e] = v;
        if (e < 2) mx0 = fmaxf(mx0, v);
        else mx1 = fmaxf(mx1, v);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float base0 = mn0 == -INFINITY ? 0.f : mn0, base1 = mn1 == -INFINITY ? 0.f : mn1;
    const float sc0 = exp2f(m0 - base0), sc1 = exp2f(m1 - base1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s[j][0] = exp2f(s[j][0] - base0);
      s[j][1] = exp2f(s[j][1] - base0);
      s[j][2] = exp2f(s[j][2] - base1);
      s[j][3] = exp2f(s[j][3] - base1);
      ps0 += s[j][0] + s[j][1];
      ps1 += s[j][2] + s[j][3];
    }
    l0 = l0 * sc0 + ps0;
    l1 = l1 * sc1 + ps1;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= sc0;
      o[j][1] *= sc0;
      o[j][2] *= sc1;
      o[j][3] *= sc1;
    }
    // ---- O += P V ----
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      a[0] = pack2(s[2 * kk][0], s[2 * kk][1]);
      a[1] = pack2(s[2 * kk][2], s[2 * kk][3]);
      a[2] = pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      a[3] = pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int jp = 0; jp < 8; ++jp) {  // pairs of n8 dim tiles
        uint32_t b0, b1, b2, b3;
        const int r = 16 * kk + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = 2 * jp + (lane >> 4);
        ldsm_x4_t(sV[buf] + swz(r, c), b0, b1, b2, b3);
        mma16816(o[2 * jp], a, b0, b1);
        mma16816(o[2 * jp + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }
  // ---- finalize ----
  cp_wait_0();  // a split without key blocks still has its Q copy in flight
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  if (ns == 1) {
    const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int d = h * kHD + 8 * j + 2 * t4;
      if (row0 < n_q)
        *reinterpret_cast<uint32_t*>(p.out + (int64_t)row0 * p.out_ld + d) = pack2(o[j][0] * inv0, o[j][1] * inv0);
      if (row1 < n_q)
        *reinterpret_cast<uint32_t*>(p.out + (int64_t)row1 * p.out_ld + d) = pack2(o[j][2] * inv1, o[j][3] * inv1);
    }
    return;
  }
  // Partials into this CTA's shared memory (the K/V buffers are free after the
  // loop's final barrier): O [64][128] f32 at sK[0], (m, l) [64] at sK[0] + 32 KB.
  __syncthreads();
  float* po = reinterpret_cast<float*>(sm + 16384);
  float2* pml = reinterpret_cast<float2*>(sm + 16384 + 32768);
  const int r0 = 16 * warp + g, r1 = r0 + 8;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int d = 8 * j + 2 * t4;
    *reinterpret_cast<float2*>(po + r0 * kHD + d) = make_float2(o[j][0], o[j][1]);
    *reinterpret_cast<float2*>(po + r1 * kHD + d) = make_float2(o[j][2], o[j][3]);
  }
  if (t4 == 0) {
    pml[r0] = make_float2(m0, l0);
    pml[r1] = make_float2(m1, l1);
  }
  cluster_sync_all();
  const int rows_per = kQB / ns;
  const uint32_t po_s = static_cast<uint32_t>(__cvta_generic_to_shared(po));
  const uint32_t pml_s = static_cast<uint32_t>(__cvta_generic_to_shared(pml));
  for (int idx = tid; idx < rows_per * (kHD / 4); idx += 128) {
    const int r = split * rows_per + idx / (kHD / 4);
    const int c4 = idx % (kHD / 4);
    float mk[8], lk[8];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k < ns) {
        const float2 v = ld_cluster_f2(cluster_map(pml_s + 8u * r, (uint32_t)k));
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
        const float f = exp2f(mk[k] - mx);
        lsum += f * lk[k];
        const float4 v = ld_cluster_f4(cluster_map(po_s + 4u * (r * kHD + 4 * c4), (uint32_t)k));
        acc.x += f * v.x;
        acc.y += f * v.y;
        acc.z += f * v.z;
        acc.w += f * v.w;
      }
    }
    const int row = q0 + r;
    if (row < n_q) {
      const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
      uint2 w;
      w.x = pack2(acc.x * inv, acc.y * inv);
      w.y = pack2(acc.z * inv, acc.w * inv);
      *reinterpret_cast<uint2*>(p.out + (int64_t)row * p.out_ld + h * kHD + 4 * c4) = w;
    }
  }
  cluster_sync_all();  // peers may read this CTA's partials until here
}

// Key splits per (query block, head): the largest of 1, 2, 4, 8 (the portable
// cluster size) that keeps every CTA resident in one wave (two CTAs per SM,
// bound by registers and shared memory) and leaves each split at least two
// key blocks. ACTFOLD_ATTN_SPLITS (1, 2, 4 or 8) overrides the choice.
static int attention_splits(const AttnParams& p) {
  const char* env = std::getenv("ACTFOLD_ATTN_SPLITS");
  if (env) {
    const int v = std::atoi(env);
    if (v == 1 || v == 2 || v == 4 || v == 8) return v;
  }
  const int ctas = (p.n_q_cap + kQB - 1) / kQB * p.n_heads;
  const int n_blocks = (p.T + kKB - 1) / kKB + (p.fk ? (p.n_f_cap + kKB - 1) / kKB : 0);
  const int resident = 2 * sm_count();
  int ns = 1;
  while (ns < 8 && 2 * ns * ctas <= resident && n_blocks / (2 * ns) >= 2) ns *= 2;
  return ns;
}

bool attention_uses_tc(const AttnParams& p) {
  const char* impl = std::getenv("ACTFOLD_ATTN_IMPL");
  return !(impl && impl[0] == 'm') && (attention_fa_ok(p) || attention_tc_splits(p) > 0);
}

int attention_run(const AttnParams& p, cudaStream_t s) {
  AF_REQUIRE(p.q && p.pk && p.pv && p.out, "attention: null pointer");
  AF_REQUIRE(p.n_heads > 0 && p.n_kv_heads > 0 && p.n_heads % p.n_kv_heads == 0, "attention: bad head counts");
  AF_REQUIRE(p.T > 0 && p.n_q_cap >= 0, "attention: bad sizes");
  AF_REQUIRE(!p.fk || (p.fv && p.n_f_cap >= 0), "attention: fresh keys need values");
  AF_REQUIRE(((p.q_ld | p.kv_ld | p.out_ld | p.f_ld) & 7) == 0, "attention: row strides must be multiples of 8");
  if (p.n_q_cap == 0) return AF_OK;
  // The tcgen05 kernel covers up to 24 key blocks of 128 (an 8-CTA cluster of
  // 3 blocks each); ACTFOLD_ATTN_IMPL=mma selects this mma.sync kernel instead.
  const char* impl = std::getenv("ACTFOLD_ATTN_IMPL");
  if (!(impl && impl[0] == 'm')) {
    if (attention_fa_ok(p)) return attention_fa_run(p, s);
    const int ns_tc = attention_tc_splits(p);
    if (ns_tc > 0) return attention_tc_run(p, ns_tc, s);
  }
  AF_REQUIRE(!p.cand_tma && !p.out_rows, "attention: candidate-row mode and output row maps need the tcgen05 kernel");
  const int smem = kSmem;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    cudaFuncSetAttribute(k_attention, cudaFuncAttributeNonPortableClusterSizeAllowed, 0);
    attr = true;
  }
  const int ns = attention_splits(p);
  cudaError_t e = launch_ex(k_attention, dim3((p.n_q_cap + kQB - 1) / kQB, p.n_heads, ns), dim3(128, 1, 1),
                            (size_t)smem, s, p.pdl != 0, dim3(1, 1, ns), p);
  if (e != cudaSuccess) return fail(AF_ERR_CUDA, std::string("attention: launch: ") + cudaGetErrorString(e));
  return check_launch("attention");
}


}  // namespace af

using namespace af;

extern "C" int af_attention_bf16(const void* q, int64_t q_ld, const int32_t* qsrc, const int32_t* qchild,
                                 const int32_t* n_q_dev, int64_t n_q_cap, const void* pk, const void* pv,
                                 int64_t kv_ld, int64_t T, const uint32_t* fresh_bits, int64_t bits_ld,
                                 const void* fk, const void* fv, int64_t f_ld, const int32_t* fchild,
                                 const int32_t* n_f_dev, int64_t n_f_cap, void* out, int64_t out_ld, int n_heads,
                                 int n_kv_heads, int head_dim, float scale, uint32_t* status, void* stream) {
  AF_REQUIRE(head_dim == kHD, "af_attention_bf16: head_dim must be 128");
  AF_REQUIRE(T <= (1 << 24) && n_q_cap <= (1 << 24) && n_f_cap <= (1 << 24), "af_attention_bf16: size too large");
  AttnParams p;
  memset(&p, 0, sizeof(p));
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_ld = q_ld;
  p.qsrc = qsrc;
  p.qchild = qchild;
  p.n_q_dev = n_q_dev;
  p.n_q_cap = (int)n_q_cap;
  p.pk = static_cast<const __nv_bfloat16*>(pk);
  p.pv = static_cast<const __nv_bfloat16*>(pv);
  p.kv_ld = kv_ld;
  p.T = (int)T;
  p.fresh_bits = fresh_bits;
  p.bits_ld = (int)bits_ld;
  p.fk = static_cast<const __nv_bfloat16*>(fk);
  p.fv = static_cast<const __nv_bfloat16*>(fv);
  p.f_ld = f_ld;
  p.fchild = fchild;
  p.n_f_dev = n_f_dev;
  p.n_f_cap = (int)n_f_cap;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_ld = out_ld;
  p.n_heads = n_heads;
  p.n_kv_heads = n_kv_heads;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.status = reinterpret_cast<unsigned*>(status);
  // A plain stream-ordered launch (no programmatic dependency): every earlier
  // kernel of the stream has finished when it starts, so the parent K/V may be
  // loaded at kernel entry.
  p.kv_static = 1;
  return attention_run(p, as_stream(stream));
}
