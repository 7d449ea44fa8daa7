/*
 * libactfold_b200 -- C ABI of the B200 (sm_100a) Branch Folding verification path.
 *
 * Conventions
 *   - Every function returns an af_status; on failure af_last_error_string()
 *     returns a message for the calling thread.
 *   - All device pointers are caller-owned; no entry point allocates device
 *     memory. Work that needs scratch takes it as an argument and reports its
 *     size through a *_workspace_size() query.
 *   - `stream` is a cudaStream_t (CUstream) handle; every launch is ordered on
 *     it and no entry point synchronizes the device.
 *   - Strides are in BYTES unless stated otherwise; the innermost (hidden)
 *     dimension is contiguous.
 *
 * The reference (ShaneLiu04/ActFold) is pure Python/PyTorch; the functions
 * below replace the tensor work of the Python calls cited beside each one.
 * Paths are relative to the reference checkout.
 */
#ifndef ACTFOLD_B200_H_
#define ACTFOLD_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  AF_OK = 0,
  AF_ERR_ARG = 1,      /* bad argument (ValueError on the Python side)        */
  AF_ERR_CAPACITY = 2, /* a size exceeds a buffer capacity                    */
  AF_ERR_DEVICE = 3,   /* a device-side check failed (status word set)       */
  AF_ERR_TIMEOUT = 4,  /* a bounded device wait ran out                       */
  AF_ERR_CUDA = 5,     /* a CUDA runtime call failed                          */
  AF_ERR_COMM = 6      /* a cross-rank collective (caller hook) failed        */
} af_status;

typedef enum { AF_DTYPE_F32 = 0, AF_DTYPE_F16 = 1, AF_DTYPE_BF16 = 2 } af_dtype;

typedef enum { AF_METRIC_COSINE = 0, AF_METRIC_L2 = 1, AF_METRIC_PEARSON = 2 } af_metric;

/* Library version string, e.g. "actfold_b200 0.1.0 sm_100a". */
const char* af_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* af_last_error_string(void);

/*
 * af_gate -- per-token similarity gate with fused stream compaction.
 *
 * Replaces SimilarityGate.forward / _compute_similarity
 * (actfold/core/similarity_gate.py:43-103) and the host-side statistics of
 * GLOBAL_STABILITY_PROFILER.record (actfold/profiler/stability_profiler.py:106-158).
 *
 * For every row (b, t) of child[B, T, H] and parent[B, T, H] computes the
 * similarity with the reference's rounding chain in `dtype` and writes
 *   stable_mask[b * mask_bstride + t] = sim > round_dtype(tau)   (1 byte, 0/1)
 *   sim[b * T + t]                      (optional, f32 value of the rounded sim)
 * and, when div_idx is non-NULL, order-preserving index lists per batch row:
 *   stable_idx[b * idx_bstride + i]  (optional) i-th stable token, -1 padded
 *   div_idx[b * idx_bstride + i]     i-th divergent token, -1 padded
 *   div_count[b]                     number of divergent tokens
 * parent_bstride may be 0 to broadcast one parent row block over the batch.
 * l2_denom = sqrt(H) + eps evaluated in double (the "l2" metric only).
 */
int af_gate(const void* child, int64_t child_bstride, int64_t child_tstride,
            const void* parent, int64_t parent_bstride, int64_t parent_tstride,
            int64_t batch, int64_t seq, int64_t hidden, int dtype, int metric,
            float tau, float eps, float l2_denom,
            uint8_t* stable_mask, int64_t mask_bstride, float* sim,
            int32_t* stable_idx, int32_t* div_idx, int64_t idx_bstride,
            int32_t* div_count, void* stream);

/*
 * af_merge_rows -- out[b, t, :] = stable[b, t] ? parent[b, t, :] : child[b, t, :].
 *
 * Replaces merge_stable_divergent and the Triton _merge_kernel
 * (actfold/core/fused_ops.py:95-135, 206-253). Rows are `row_bytes` long
 * (any element type); only the selected source row is read.
 */
int af_merge_rows(const void* parent, int64_t parent_bstride, int64_t parent_tstride,
                  const void* child, int64_t child_bstride, int64_t child_tstride,
                  const uint8_t* stable, int64_t stable_bstride,
                  void* out, int64_t out_bstride, int64_t out_tstride,
                  int64_t batch, int64_t seq, int64_t row_bytes, void* stream);

/*
 * af_gather_rows_masked -- zero-filled reconstruction of cached rows.
 *
 * Replaces gather_cached_activations (actfold/core/fused_ops.py:54-87, 256-324)
 * for one activation tensor. src holds the cached [Bs, T, row] block
 * (src_bstride 0 broadcasts a stored batch of 1). present[t] (nullable = all
 * present) marks cached tokens.
 *   mode 0 (all tokens present): out[b,t] = mask[b,t] ? src[b,t] : 0
 *   mode 1 (some token missing): out[b,t] = present[t] && any_b' mask[b',t] ? src[b,t] : 0
 */
int af_gather_rows_masked(const void* src, int64_t src_bstride, int64_t src_tstride,
                          const uint8_t* mask, int64_t mask_bstride, const uint8_t* present,
                          int mode, void* out, int64_t out_bstride, int64_t out_tstride,
                          int64_t batch, int64_t seq, int64_t row_bytes, void* stream);

/*
 * af_gather_rows_index -- out[b, j, :] = idx[j] >= 0 ? src[b, idx[j], :] : 0.
 *
 * Replaces the token-subset gather of ChunkedActivationCache.get
 * (actfold/core/chunked_cache.py:182-225: dense[:, valid_indices]) and packs
 * rows by index list. src_bstride 0 broadcasts one stored batch row.
 */
int af_gather_rows_index(const void* src, int64_t src_bstride, int64_t src_tstride,
                         const int32_t* idx, int64_t n, int64_t batch,
                         void* out, int64_t out_bstride, int64_t out_tstride,
                         int64_t row_bytes, void* stream);

/* Epilogues of af_linear_bf16. */
typedef enum {
  AF_EPI_STORE = 0,    /* out[m, n] = bf16(acc)                                        */
  AF_EPI_RESIDUAL = 1, /* out[m, n] = bf16(res[m, n] + bf16(acc))                      */
  AF_EPI_SWIGLU = 2,   /* weight rows interleaved per 128: 64 gate rows then 64 up rows;
                          out[m, f] = bf16(silu(bf16 g) * bf16 u), out width n / 2      */
  AF_EPI_ROPE = 3      /* rotate-half RoPE (head_dim 128) on columns [0, rope_cols)    */
} af_epilogue;

/*
 * af_linear_bf16 -- out[row(m)] = epilogue(x[m, :] . w^T) for packed token rows.
 *
 * Replaces the projections inside the wrapped layer that
 * FoldedTransformerLayer._recompute_all runs on every row
 * (actfold/core/folded_transformer.py:224-258): here only the packed divergent
 * rows are computed, with tcgen05 tensor cores (bf16 x bf16 -> fp32 in TMEM).
 *   x [m_cap, k] bf16, row stride ldx (elements); valid rows = *m_dev (device
 *   int, nullable -> m_cap); w [n, k] bf16 (n % 128 == 0, k % 64 == 0),
 *   w_layout 0 = row-major, 1 = tiled [n/128][k/64][128][64] (each 128 x 64
 *   tile one contiguous 16 KB block; streams from HBM in whole blocks);
 *   out rows: out_rows[m] (nullable -> m), row stride ldo; residual rows:
 *   res_rows[m] (nullable -> m); rope tables cos/sin [P, 64] fp32 indexed by
 *   positions[m]. splits (0..8, 0 = automatic) divides the k-range over a
 *   thread-block cluster whose partial tiles are summed in distributed shared
 *   memory (no workspace); status receives AF_STATUS bits (1 timeout,
 *   2 capacity).
 */
int af_linear_bf16(const void* x, int64_t ldx, int64_t m_cap, const int32_t* m_dev,
                   const void* w, int64_t n, int64_t k, int w_layout, int epilogue,
                   void* out, int64_t ldo, const int32_t* out_rows,
                   const void* residual, int64_t ldr, const int32_t* res_rows,
                   const float* rope_cos, const float* rope_sin, const int32_t* positions,
                   int64_t rope_cols, int splits, uint32_t* status, void* stream);

/*
 * af_attention_bf16 -- non-causal attention of packed query rows over the
 * parent's cached K/V, with per-child fresh-key overrides.
 *
 * Replaces the self-attention the wrapped layer recomputes over the FULL child
 * context (actfold/core/folded_transformer.py:188-195): only divergent query
 * rows are computed, and keys whose child input equals the parent's come from
 * the parent cache. Query i (child qchild[i]) reads q + qsrc[i] * q_ld; its
 * keys are parent rows t of pk/pv except where bit t of
 * fresh_bits[qchild[i] * bits_ld] is set, plus candidate rows j of fk/fv with
 * fchild[j] == qchild[i]. Valid query / candidate counts are read from
 * n_q_dev / n_f_dev (nullable -> caps). head_dim must be 128; GQA when
 * n_kv_heads < n_heads. Runs on tcgen05 tensor cores: key splits combined in
 * a thread-block cluster (up to 24 blocks of 128 keys), or one CTA per query
 * tile and head streaming every key block with an online softmax (contiguous
 * queries: qsrc null, no candidate keys; chosen when those CTAs fill the GPU,
 * or when the sequence is too long for key splits). Gathered queries or
 * candidate keys over more than 24 key blocks are refused with AF_ERR_ARG
 * before any launch. status (nullable) receives AF_STATUS_TIMEOUT if a
 * bounded wait ran out.
 */
int af_attention_bf16(const void* q, int64_t q_ld, const int32_t* qsrc, const int32_t* qchild,
                      const int32_t* n_q_dev, int64_t n_q_cap, const void* pk, const void* pv,
                      int64_t kv_ld, int64_t T, const uint32_t* fresh_bits, int64_t bits_ld,
                      const void* fk, const void* fv, int64_t f_ld, const int32_t* fchild,
                      const int32_t* n_f_dev, int64_t n_f_cap, void* out, int64_t out_ld,
                      int n_heads, int n_kv_heads, int head_dim, float scale, uint32_t* status,
                      void* stream);

/* Attention kernel choice for later calls (process-wide; no counterpart in
 * the reference): AF_ATTN_AUTO picks per shape as above, AF_ATTN_STREAM
 * takes the streaming (one CTA per query tile and head) kernel wherever it
 * applies, AF_ATTN_SPLIT never takes it. Returns AF_ERR_ARG for other values. */
enum { AF_ATTN_AUTO = 0, AF_ATTN_STREAM = 1, AF_ATTN_SPLIT = 2 };
int af_set_attention_kernel(int kind);

/* ------------------------------------------------------------------------
 * Native folded verification of LLaDA / Dream-architecture models.
 *
 * Replaces, for a model whose blocks are pre-norm RMSNorm -> QKV (+RoPE) ->
 * non-causal attention -> O + residual -> RMSNorm -> SwiGLU FFN + residual,
 * the whole per-layer loop of FoldedModel.forward / FoldedTransformerLayer
 * (actfold/core/model_wrapper.py:137-208, actfold/core/folded_transformer.py:60-203)
 * for a batch of children sharing one parent: gates, index compaction,
 * recompute of divergent rows only, merge of parent rows, logits.
 * ---------------------------------------------------------------------- */
typedef struct {
  int32_t n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab;
  float rms_eps;
} af_model_dims;

/* Projection weights are bf16 matrices [n, k] stored TILED, i.e. as
 * [n/128][k/64][128][64] (af_linear_bf16 w_layout 1); norms are plain [hidden]. */
typedef struct {
  const void* attn_norm; /* [hidden] bf16 */
  const void* w_qkv;     /* [q_dim + 2 kv_dim, hidden]: Wq rows, Wk rows, Wv rows (tiled) */
  const void* w_o;       /* [hidden, q_dim] (tiled) */
  const void* ffn_norm;  /* [hidden] */
  const void* w_gateup;  /* [2 ffn, hidden]: per 128 rows, 64 gate rows then the 64 matching up rows (tiled) */
  const void* w_down;    /* [hidden, ffn] (tiled) */
} af_layer_weights;

typedef struct {
  af_model_dims dims;
  const af_layer_weights* layers; /* host array of n_layers entries (copied by plans) */
  const void* embed;              /* [vocab, hidden] bf16 */
  const void* final_norm;         /* [hidden] */
  const void* lm_head;            /* [vocab, hidden] (tiled) */
  const float* rope_cos;          /* [max_pos, head_dim / 2] fp32 */
  const float* rope_sin;
  int64_t max_pos;
} af_model;

/* Parent activation cache (the dense equivalent of ActivationCache entries of the parent branch). */
typedef struct {
  int64_t seq;                  /* T */
  const int64_t* tokens;        /* [T] */
  const void* layer_in;         /* [n_layers + 1, T, hidden] bf16: layer inputs; [n_layers] = final hidden */
  const void* qkv;              /* [n_layers, T, q_dim + 2 kv_dim] bf16 (K at column q_dim, V after it) */
  const void* logits;           /* [T, vocab] bf16 */
  const uint8_t* self_stable;   /* [n_layers, T] gate(parent row, parent row) */
  const float* logit_row_sums;  /* [T] fp32 sums of each logits row */
  /* Nullable: [n_layers, 2, n_kv_heads, T, head_dim] bf16, the K (0) and V (1)
   * columns of qkv stored head-major (af_parent_kv_headmajor), so one head's
   * block of keys is one contiguous run of memory. The folded pass reads the
   * parent's keys and values from here when it is set, and promotions keep it
   * in step with qkv. */
  void* kv_headmajor;
} af_parent_cache;

/* Builds af_parent_cache.kv_headmajor from qkv ([n_layers, T, q_dim + 2 kv_dim]);
 * stream-ordered. No counterpart in the reference (a layout of the cache). */
int af_parent_kv_headmajor(const af_model_dims* dims, int64_t T, const void* qkv, void* kv_headmajor, void* stream);

/* Workspace of af_dense_forward for T tokens. */
int af_dense_workspace_bytes(const af_model_dims* dims, int64_t T, int64_t* bytes);

/*
 * af_dense_forward -- the parent pass (FoldedTransformerLayer with
 * parent_branch_id None -> _recompute_all + _store_activations,
 * actfold/core/folded_transformer.py:100-104): runs every layer on all T rows
 * and writes the parent cache arrays.
 */
int af_dense_forward(const af_model* model, const int64_t* tokens, int64_t T, float tau,
                     void* layer_in, void* qkv, void* logits, uint8_t* self_stable,
                     float* logit_row_sums, void* workspace, int64_t workspace_bytes,
                     uint32_t* status, void* stream);

/* Size of the file-scope device scratch array behind af_dense_forward_static. */
#define AF_DENSE_STATIC_WORKSPACE_BYTES (32ll << 20)

/*
 * af_dense_forward_static -- af_dense_forward with its scratch in a
 * file-scope __device__ array of AF_DENSE_STATIC_WORKSPACE_BYTES (32 MiB) per
 * device instead of a caller workspace. It has no counterpart in the
 * reference: it exists so a caller that must not allocate (no
 * cudaMalloc/cudaFree, no allocating library routine) can run the parent pass.
 *   - The outputs are bit-identical to af_dense_forward on the same inputs.
 *   - T is rejected with AF_ERR_CAPACITY when af_dense_workspace_bytes(dims, T)
 *     exceeds the array (LLaDA-8B dims: 585 tokens at most).
 *   - The first call on a device looks up the array's address with
 *     cudaGetSymbolAddress, with that device current, and caches it; make that
 *     first call before any stream capture. The device owning `stream` must be
 *     current on every call (a stream of another device: AF_ERR_ARG). The
 *     cached address does not survive cudaDeviceReset; do not call this entry
 *     point again in a process after resetting the device.
 *   - No part of the scratch has to start at zero.
 *   - There is one array per device: calls that overlap on the same device
 *     (another stream or host thread before the previous call's kernels have
 *     finished) race on it.
 */
int af_dense_forward_static(const af_model* model, const int64_t* tokens, int64_t T, float tau,
                            void* layer_in, void* qkv, void* logits, uint8_t* self_stable,
                            float* logit_row_sums, uint32_t* status, void* stream);

typedef struct {
  int64_t n_children;          /* C */
  int64_t seq;                 /* T (equal to the parent's) */
  int64_t m_cap;               /* capacity for candidate / divergent rows per layer (all children) */
  float tau;                   /* SimilarityGate tau (compared in bf16) */
  int32_t metric;              /* af_metric */
  const uint8_t* su_layers;    /* host [n_layers]: 1 where some parent row fails its own gate
                                  (at this layer's threshold) or where the layer does not fold */
  /* Per-layer schedule, all nullable (null: the plain pass above). It replaces
   * FoldingScheduler.get_tau / should_fold inside FoldedTransformerLayer.forward
   * (actfold/core/folded_transformer.py:107-119, folding_scheduler.py:48-115):
   *   tau_layers  host [n_layers]: the gate threshold of each layer;
   *   fold_layers host [n_layers]: 0 where the layer does not fold -- every row
   *               of every child is recomputed, as _recompute_all does there
   *               (needs m_cap = n_children * seq and a per-child bound of seq);
   *   self_stable device [n_layers, seq]: the parent's own gate results at these
   *               thresholds (null: the parent cache's, taken at its own tau). */
  const float* tau_layers;
  const uint8_t* fold_layers;
  const uint8_t* self_stable;
  /* 1: the O and down projections always leave fp32 partials [S][m_cap][hidden]
   * for the next row kernel (needed by tensor-parallel shards, whose partials
   * are summed across ranks in between); 0: only when they split k. */
  int32_t partial_always;
} af_fold_config;

typedef struct {
  const int32_t* n_cand;       /* [n_layers + 1] candidate rows per layer (device) */
  const int32_t* n_div;        /* [n_layers] divergent rows per layer */
  const int32_t* div_pos;      /* [n_layers, m_cap] divergent rows as child * T + t, in that order */
  const int32_t* div_count;    /* [n_layers, C] divergent rows per child */
  const uint32_t* status;      /* device status word (AF_STATUS bits) */
  int64_t m_cap;
  const int32_t* n_fresh0;     /* edited rows at layer 0 */
  const int32_t* fresh0_pos;   /* [m_cap] */
} af_fold_outputs;

int af_fold_workspace_bytes(const af_model_dims* dims, const af_fold_config* cfg, int64_t* bytes);
int af_fold_plan_create(const af_model* model, const af_parent_cache* parent, const af_fold_config* cfg,
                        void* workspace, int64_t workspace_bytes, void** plan);
/* One verification pass of child_tokens [C, T]; writes logits [C, T, vocab] bf16 and
 * (nullable) scores [C] = mean of each child's logits. No host synchronisation. */
int af_fold_run(void* plan, const int64_t* child_tokens, void* logits, float* scores, void* stream);
int af_fold_get_outputs(void* plan, af_fold_outputs* out);
/* Dense input of layer `layer` (0..n_layers) for every child: out [C, T, hidden] bf16. */
int af_fold_materialize(void* plan, int64_t layer, void* out, void* stream);
int af_fold_plan_destroy(void* plan);
/*
 * Bound on the candidate rows of any one child per layer, for the next runs
 * (0, the default: no bound). A child's candidates at layer l are its edited
 * tokens that are still divergent plus the rows its parent fails its own gate
 * on, so max edited tokens per child + such parent rows is a bound. With it,
 * attention lets each tile of 128 packed query rows scan only the candidate
 * keys near its own rows (the candidate list is ordered by child) instead of
 * every candidate of every child, which makes attention linear rather than
 * quadratic in the number of children. A run in which some child exceeds the
 * bound sets AF_STATUS_CAPACITY in the status word. Host-side setting: make it
 * before capturing a run into a graph. Has no counterpart in the reference
 * (the reference recomputes each child separately).
 */
int af_fold_set_child_cap(void* plan, int64_t max_candidates_per_child);

/*
 * Tensor-parallel folded pass (no counterpart in the reference, which runs a
 * child on one device). Every rank holds a shard of each layer -- a slice of
 * the attention heads (Wq / Wk / Wv rows, Wo columns), a slice of the FFN
 * (gate / up rows, down columns) and a slice of the LM-head vocabulary -- plus
 * the full embedding table and its own slice of the parent cache, and runs the
 * same pass. Three sums cross the ranks, through `collective`, which must
 * add the `count` fp32 values at `data` over every rank, in place and
 * stream-ordered on `stream` (e.g. an NCCL all-reduce), and return 0:
 *   AF_COLL_O     after layer `layer`'s O projection: its split-K partials;
 *   AF_COLL_DOWN  after its down projection: its split-K partials;
 *   AF_COLL_ROWSUM after the LM head: the fresh logits' row sums [C * T].
 * Needs a plan created with partial_always = 1. embed_rows: rows of the
 * (full) embedding table; vocab_total: the whole vocabulary (the scores are
 * means over it). Host-side setting: make it before capturing a run.
 */
#define AF_COLL_O 0
#define AF_COLL_DOWN 1
#define AF_COLL_ROWSUM 2
typedef int (*af_collective_fn)(void* user, int32_t kind, int32_t layer, void* data, int64_t count, void* stream);
int af_fold_set_tensor_parallel(void* plan, int64_t embed_rows, int64_t vocab_total, af_collective_fn collective,
                                void* user);

/*
 * Peer-memory sums for a tensor-parallel plan (ranks on one node, GPUs with
 * peer access over NVLink). With it the AF_COLL_O and AF_COLL_DOWN sums no
 * longer go through the hook: after each of those projections one kernel adds
 * this rank's k-splits and stores the fp32 sum into a slot of EVERY rank's
 * exchange buffer (its own through local stores, the others' through peer
 * stores), then raises a flag in each; the kernel that consumes the sum waits
 * (bounded, AF_STATUS_TIMEOUT after about 5 s) until every rank's flag for that
 * launch is up and adds the slots in rank order, so every rank finishes the
 * same rows bit for bit. The hook still carries AF_COLL_ROWSUM.
 *
 * af_fold_peer_bytes: bytes of one rank's exchange buffer for `world` ranks.
 * af_fold_set_peer_sum: exchange[q] (q < world <= 8) is rank q's exchange
 *   buffer as this process addresses it (exchange[rank] its own), 256-byte
 *   aligned; every buffer must be zero-filled, and the fill complete on every
 *   rank, before any rank runs the plan. Needs af_fold_set_tensor_parallel
 *   first. Host-side setting: make it before capturing a run.
 * af_ipc_export / af_ipc_import / af_ipc_close: CUDA IPC of a device address
 *   inside any cudaMalloc allocation (a caching allocator's block included):
 *   export writes the 64-byte handle of the enclosing allocation and the
 *   address's offset in it; import maps a handle exported by another process
 *   of this node (peer access enabled on first use) and returns the mapped
 *   address of the same byte (`ptr`) and the mapping's base, which close
 *   unmaps.
 */
int af_fold_peer_bytes(void* plan, int32_t world, int64_t* bytes);
int af_fold_set_peer_sum(void* plan, int32_t rank, int32_t world, void* const* exchange);
int af_ipc_export(const void* ptr, void* handle, int64_t* offset);
int af_ipc_import(const void* handle, int64_t offset, void** ptr, void** base);
int af_ipc_close(void* base);

/*
 * Promotion of a verified child to a parent. Replaces the child branch's own
 * ActivationCache entries, which the reference writes after every merge
 * (_store_activations, actfold/core/folded_transformer.py:190-199 and
 * :260-274) so that a later call may name the child as parent_branch_id.
 *
 * af_fold_keep_kv: while `store` is set, every af_fold_run also copies each
 * layer's candidate QKV rows into it (one extra launch per layer). `store`
 * holds n_layers * m_cap * (q_dim + 2 kv_dim) bf16, 16-byte aligned; NULL
 * turns the copy off. Set it before capturing a pass into a graph.
 *
 * af_fold_promote: writes child `child` of the last run into `dst`, whose
 * arrays must hold a copy of the plan's parent cache or be the plan's parent
 * cache itself (in place). Only the child's fresh rows are written: tokens,
 * layer inputs, QKV rows, self-gate flags (at the plan's tau), and the logits
 * rows and logit row sums of its last-layer divergent rows, taken from the
 * run's `child_tokens` [C, T] and `child_logits` [C, T, vocab]. Stream-ordered
 * after the run; valid until the plan runs again. After an in-place promotion
 * the caller re-derives su_layers from self_stable and makes a new plan if it
 * changed.
 */
int af_fold_keep_kv(void* plan, void* store, int64_t store_bytes);
int af_fold_promote(void* plan, int64_t child, const int64_t* child_tokens, const void* child_logits,
                    const af_parent_cache* dst, void* stream);

/*
 * Per-kernel-class CUDA-event timing of af_fold_run, recorded on the pass's
 * stream when enabled. Classes: 0 candidates/embedding, 1 gate, 2 compaction,
 * 3 QKV GEMM, 4 attention, 5 O GEMM, 6 RMSNorm, 7 gate/up GEMM, 8 down GEMM,
 * 9 LM-head GEMM, 10 parent-logit fill, 11 scores, 12 QKV rows finished from
 * the QKV GEMM's split partials. af_fold_get_timing
 * synchronizes on the last event, returns the accumulated milliseconds and
 * launch counts per class (then resets them) and the number of kernel
 * launches of the last run. No counterpart in the reference (measurement).
 */
int af_fold_set_timing(void* plan, int enabled);
int af_fold_get_timing(void* plan, double* ms, int64_t* counts, int n_kinds, int64_t* launches_per_run);

#ifdef __cplusplus
}
#endif

#endif /* ACTFOLD_B200_H_ */
