// Per-layer compaction of the folded pass (sm_100a), run by a group of NT
// threads that synchronise on their own named barrier: the divergent-row list
// of the layer, the per-child fresh-key bitmap, divergent counts per child and
// the next layer's candidate list.
//
// It is run as a side task by the epilogue warps of one CTA of the layer's QKV
// GEMM, while that CTA's weight ring streams (no kernel of its own): every
// consumer (attention, the FFN GEMMs, the next layer's gate) comes after the
// QKV GEMM, and the stable flags it reads come from the gate kernel before it.
//
// Follows actfold/core/folded_transformer.py:148 (stable_mask = self.gate(...))
// and :196 (merge_stable_divergent): the divergent rows of a layer are the
// candidates that fail the similarity gate, kept in candidate order; they are
// recomputed and become the fresh rows of the next layer.
#pragma once

#include "common.cuh"

namespace af {

// Barrier over the NT threads (whole warps) of a group; id 0 is __syncthreads.
template <int NT>
__device__ __forceinline__ void group_sync(int bar_id) {
  asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "n"(NT) : "memory");
}

// Exclusive scan over the NT threads of a group (tid = rank in the group,
// a multiple of 32 threads, at most 1024); the group's total in *total_out.
template <int NT>
__device__ __forceinline__ int group_scan(int v, int* warp_buf, int* total_out, int tid, int bar_id) {
  constexpr int kWarps = NT / 32;
  const int lane = tid & 31, warp = tid >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += n;
  }
  if (lane == 31) warp_buf[warp] = x;
  group_sync<NT>(bar_id);
  if (warp == 0) {
    int w = lane < kWarps ? warp_buf[lane] : 0;
#pragma unroll
    for (int o = 1; o < kWarps; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    if (lane < kWarps) warp_buf[lane] = w;  // inclusive per-warp totals
  }
  group_sync<NT>(bar_id);
  const int excl = x - v + (warp > 0 ? warp_buf[warp - 1] : 0);
  *total_out = warp_buf[kWarps - 1];
  group_sync<NT>(bar_id);
  return excl;
}

struct CompactArgs {
  int C, T, m_cap, bits_ld;
  const int* n_cand;
  const uint8_t* stable;
  const int* cand_child;
  const int* cand_pos;
  int* div_cand;
  int* div_child;
  int* div_pos;
  int* n_div;
  int* cand_div;        // nullable: [m_cap] divergent rank of each candidate, -1 if stable
  int* div_count;       // [C] divergent rows per child
  unsigned* bits;       // [C, bits_ld] candidates of this layer (fresh keys)
  unsigned* final_bits; // nullable: divergent rows of this layer (last layer only)
  float* zero_f;        // nullable: buffer zeroed here (logit row sums, last layer)
  int zero_n;
  int write_next;
  int* next_child;
  int* next_pos;
  int* next_src;
  int* next_n_cand;
};

// Ordered compaction: divergent row k of the layer is the k-th candidate whose
// gate decision is "unstable". `wbuf` holds 32 ints of shared memory.
template <int NT>
__device__ __forceinline__ void compact_rows(const CompactArgs& a, int* wbuf, int tid, int bar_id) {
  const int nb = a.C * a.bits_ld;
  for (int i = tid; i < nb; i += NT) {
    a.bits[i] = 0u;
    if (a.final_bits) a.final_bits[i] = 0u;
  }
  for (int i = tid; i < a.C; i += NT) a.div_count[i] = 0;
  if (a.zero_f)
    for (int i = tid; i < a.zero_n; i += NT) a.zero_f[i] = 0.f;
  __threadfence_block();
  group_sync<NT>(bar_id);
  const int n = min(*a.n_cand, a.m_cap);
  int base = 0, total;
  for (int r0 = 0; r0 < n || r0 == 0; r0 += NT) {
    const int r = r0 + tid;
    int c = 0, t = 0, d = 0;
    if (r < n) {
      c = a.cand_child[r];
      t = a.cand_pos[r];
      atomicOr(&a.bits[c * a.bits_ld + (t >> 5)], 1u << (t & 31));
      d = a.stable[r] ? 0 : 1;
    }
    const int rank = base + group_scan<NT>(d, wbuf, &total, tid, bar_id);
    if (a.cand_div && r < n) a.cand_div[r] = d ? rank : -1;
    if (d) {
      a.div_cand[rank] = r;
      a.div_child[rank] = c;
      a.div_pos[rank] = c * a.T + t;
      atomicAdd(&a.div_count[c], 1);
      if (a.final_bits) atomicOr(&a.final_bits[c * a.bits_ld + (t >> 5)], 1u << (t & 31));
      if (a.write_next) {
        a.next_child[rank] = c;
        a.next_pos[rank] = t;
        a.next_src[rank] = rank;
      }
    }
    base += total;
    if (r0 + NT >= n) break;
  }
  if (tid == 0) {
    *a.n_div = base;
    if (a.write_next) *a.next_n_cand = base;
  }
}

}  // namespace af
