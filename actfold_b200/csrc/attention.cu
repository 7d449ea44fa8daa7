// Non-causal attention of packed query rows over a parent K/V cache with
// per-child overrides: the dispatcher over the two tcgen05 kernels and the
// af_attention_bf16 entry point.
//
// Query row i belongs to child qchild[i]. Its keys are every position t of the
// sequence: the parent's cached K/V row t, except where t is "fresh" for that
// child (its layer input differs from the parent's), in which case the key is
// the child's recomputed K/V row, found among the layer's candidate rows
// (fchild[j] == qchild[i]). With no fresh data this is plain non-causal
// attention (the parent pass).
//
// attention_tc.cu: key splits over a thread-block cluster, up to 24 key
// blocks of 128 (8 CTAs x 3 blocks), any query gather. attention_fa.cu: one
// CTA per (query tile, head) streaming every key block, any length, for
// contiguous queries whose candidate keys (if any) are TMA boxes of the query
// buffer. Shapes neither kernel takes are refused before any launch.
#include <cstdlib>

#include "attention.cuh"

namespace af {

constexpr int kHD = 128;

bool attention_uses_tc(const AttnParams& p) { return attention_fa_ok(p) || attention_tc_splits(p) > 0; }

int attention_run(const AttnParams& p, cudaStream_t s) {
  AF_REQUIRE(p.q && p.pk && p.pv && p.out, "attention: null pointer");
  AF_REQUIRE(p.n_heads > 0 && p.n_kv_heads > 0 && p.n_heads % p.n_kv_heads == 0, "attention: bad head counts");
  AF_REQUIRE(p.T > 0 && p.n_q_cap >= 0, "attention: bad sizes");
  AF_REQUIRE(!p.fk || (p.fv && p.n_f_cap >= 0), "attention: fresh keys need values");
  AF_REQUIRE(((p.q_ld | p.kv_ld | p.out_ld | p.f_ld) & 7) == 0, "attention: row strides must be multiples of 8");
  if (p.n_q_cap == 0) return AF_OK;
  if (attention_fa_ok(p)) return attention_fa_run(p, s);
  const int ns_tc = attention_tc_splits(p);
  if (ns_tc > 0) return attention_tc_run(p, ns_tc, s);
  return fail(AF_ERR_ARG,
              "attention: more than 24 key blocks of 128 need contiguous query rows (no qsrc gather) and, with "
              "candidate keys, candidate-row mode (keys as TMA boxes of the query buffer)");
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
