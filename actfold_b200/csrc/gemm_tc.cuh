// Weight-streaming tcgen05 GEMM for packed token rows (sm_100a).
#pragma once

#include "compact.cuh"
#include "tc_common.cuh"

namespace af {

enum GemmEpilogue : int {
  EPI_STORE = 0,     // out[m, n] = bf16(acc)
  EPI_RESIDUAL = 1,  // out[m, n] = bf16(res[m, n] + bf16(acc))
  EPI_SWIGLU = 2,    // 128-row tile = 64 gate rows + 64 up rows: out[m, f] = bf16(silu(bf16 g) * bf16 u)
  EPI_ROPE = 3,      // QKV: rotate-half RoPE on columns [0, rope_cols), plain store after
};

struct GemmCall {
  const void* x;       // activations [m_cap, k] bf16 (row stride ldx elements)
  int64_t ldx;
  int m_cap;           // activation row capacity
  const int* m_dev;    // device-side valid row count (nullable: m_cap)
  const void* w;       // weights [n, k] bf16, row-major
  int n, k;
  int epi;
  void* out;           // bf16 output
  int64_t ldo;         // output row stride (elements)
  const int* out_rows; // nullable: output row of packed row m
  const void* res;     // residual (EPI_RESIDUAL)
  int64_t ldr;
  const int* res_rows; // nullable
  const float* rope_cos;  // [positions, head_dim/2]
  const float* rope_sin;
  const int* positions;   // position of packed row m
  int rope_cols;          // columns [0, rope_cols) are rotated (multiple of head_dim)
  int head_dim;           // 128
  int splits;          // k-range split over a thread-block cluster (<= 8); 0 = choose automatically
  unsigned* status;    // device status word (AF_STATUS_* bits)
  float* row_sums;     // EPI_STORE only, nullable: row_sums[out row] += sum of the row's bf16 outputs
  // Pre-built descriptors (optional; built per call when null).
  const CUtensorMap* tmap_w;
  const CUtensorMap* tmap_x;
  int w_tiled;         // 1: w is stored tiled [n/128][k/64][128][64] (contiguous 16 KB tiles)
  int pdl;             // 1: programmatic dependent launch (the kernel waits for its predecessor)
  // Optional side task: the layer compaction, run by CTA (0, 0, 0)'s epilogue
  // warps while its weight ring streams (the folded pass's QKV GEMM).
  int has_side;
  CompactArgs side;
  // GEMM without a reduction or epilogue (nullable): split j of the k-range
  // writes its fp32 partial rows to partial_out[j][m][0..n) (m < m_cap); the
  // next row kernel sums the splits in order 0, 1, ... and applies the
  // epilogue (gemm_splits tells it how many; one split is allowed).
  float* partial_out;
};

// k-splits a launch of this shape uses (1: no split); `partial`: one that leaves partials.
int gemm_splits(int n, int k, int m_cap, bool partial = false);

// Token-tile width the kernel uses for a given row capacity and output width n.
int gemm_ntok(int m_cap, int n);
// Token rows per TMA box of the activation operand: tensor maps passed in
// GemmCall::tmap_x must be built with this box height for gemm_ntok(m_cap, n).
int gemm_xbox(int ntok);
// Launch (stream-ordered, no synchronisation).
int gemm_run(const GemmCall& c, cudaStream_t stream);
// The epilogue of a launch that left `splits` partials (c.partial_out):
// sums them in split order and applies c's store / residual / RoPE epilogue.
int gemm_finish_run(const GemmCall& c, int splits, cudaStream_t stream);

}  // namespace af
