// Packed-query attention over parent K/V with fresh-key overrides (see attention.cu).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace af {

struct AttnParams {
  const __nv_bfloat16* q;  // query rows: q + qsrc[i] * q_ld + h * 128
  int64_t q_ld;
  const int* qsrc;         // nullable: i
  const int* qchild;       // nullable: no masking
  const int* n_q_dev;      // nullable: n_q_cap
  int n_q_cap;
  const __nv_bfloat16* pk;  // parent keys  [T, kv_ld] (head kvh at kvh * 128)
  const __nv_bfloat16* pv;  // parent values
  int64_t kv_ld;
  int T;
  const uint32_t* fresh_bits;  // [children][bits_ld] bitmap of fresh positions, nullable
  int bits_ld;
  const __nv_bfloat16* fk;  // candidate keys  fk + j * f_ld + kvh * 128
  const __nv_bfloat16* fv;
  int64_t f_ld;
  const int* fchild;
  const int* n_f_dev;
  int n_f_cap;
  __nv_bfloat16* out;  // out + i * out_ld + h * 128
  int64_t out_ld;
  int n_heads, n_kv_heads;
  float scale_log2;  // softmax scale * log2(e)
  int pdl;           // 1: programmatic dependent launch (the kernel waits for its predecessor)
  const __nv_bfloat16* kv_hm;  // nullable: parent K / V head-major [2][n_kv_heads][T][128] (this layer), used with kv_static
  int kv_static;     // 1: pk / pv are not written by the preceding kernels (a cached parent), so the
                     //    tcgen05 kernel loads them by TMA before it waits for its predecessor
  // Output row of query row i (nullable: i); rows mapped to -1 are not written.
  const int* out_rows;
  // Candidate-row mode of the tcgen05 kernel: query rows are q + i * q_ld
  // (qsrc null), and the query tile and the candidate key blocks (fk / fv,
  // in the same buffer at columns fk_col / fv_col) are loaded by TMA through
  // `tmap_c`, a map over that buffer ([n_q_cap rows, q_ld columns], box 64 x 128).
  int cand_tma;
  const CUtensorMap* tmap_c;
  int fk_col, fv_col;
  // Candidate-row mode only: > 0 limits each query tile i to cand_win
  // candidate key blocks centred on block i. Exact when no child has more
  // than 128 * (cand_win - 1) / 2 + 1 candidates; a tile whose children have
  // candidates outside its window ORs AF_STATUS_CAPACITY into status.
  int cand_win;
  unsigned* status;  // nullable: AF_STATUS_TIMEOUT is ORed in when a bounded wait runs out
};

int attention_run(const AttnParams& p, cudaStream_t s);
// tcgen05 kernel (attention_tc.cu): key splits for `p` (0: shape not supported) and launch.
int attention_tc_splits(const AttnParams& p);
int attention_tc_run(const AttnParams& p, int splits, cudaStream_t s);
// Whether attention_run takes a tcgen05 kernel for `p`.
bool attention_uses_tc(const AttnParams& p);
// Flash-style tcgen05 kernel (attention_fa.cu): one CTA per query tile and
// head over every key block, for contiguous query rows (candidate keys, if
// any, in candidate-row mode).
bool attention_fa_ok(const AttnParams& p);
int attention_fa_run(const AttnParams& p, cudaStream_t s);
// Cached tensor map of a parent's K or V: [T keys, cols] of a row-major
// buffer with row stride ld, or head-major [-cols heads][T][128] when cols < 0.
int attention_kv_tmap(CUtensorMap* map, const __nv_bfloat16* base, int T, int cols, int64_t ld);

}  // namespace af
