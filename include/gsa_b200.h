/*
 * gsa_b200.h -- C ABI of the B200 (sm_100a) implementation of the Gated Sparse Attention
 * forward path.
 *
 * Every entry point takes raw device pointers, sizes, a dtype code and a cudaStream_t, runs
 * stream-ordered, allocates nothing, and returns an int status (GSA_OK or a GSA_ERR_* code).
 * No exception crosses the ABI.  Scratch memory is passed in by the caller; its size comes
 * from gsa_workspace_size().  Activations are row-major; a "row" is one (batch, token) pair.
 *
 * Reference interfaces replaced (alfredcs/Gated-Sparse-Attention, paths inside that project):
 *   GatedSparseAttention.forward          gsa/attention/gated_sparse_attention.py:139-232
 *   ValueGate.forward (G2)                gsa/attention/value_gate.py:77-113
 *   RotaryEmbedding / apply_rotary_pos_emb gsa/attention/rope.py:117-185
 *   GatedLightningIndexer.forward         gsa/attention/gated_indexer.py:88-155
 *   AdaptiveTopKSelector                  gsa/attention/adaptive_topk.py:68-193
 *   _sparse_attention / _gather_along_seq gsa/attention/gated_sparse_attention.py:234-323
 *   OutputGate.forward (G1)               gsa/attention/output_gate.py:86-126
 */
#ifndef GSA_B200_H_
#define GSA_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without pulling in the CUDA headers. */
typedef struct CUstream_st* gsa_stream_t;

enum {
  GSA_OK = 0,
  GSA_ERR_BAD_ARG = 1,         /* a size, stride, pointer or alignment the kernels cannot take */
  GSA_ERR_UNSUPPORTED = 2,     /* a dtype / head size / activation with no kernel */
  GSA_ERR_WORKSPACE = 3,       /* workspace smaller than gsa_workspace_size() */
  GSA_ERR_TIMEOUT = 4,         /* a bounded device-side wait gave up (read via gsa_get_device_error) */
  GSA_ERR_LAUNCH = 5,          /* kernel launch failed */
  GSA_ERR_INDEX = 6,           /* a device-side index check failed (read via gsa_get_device_error) */
  GSA_ERR_CUDA = 7             /* another CUDA runtime error */
};

enum { GSA_DTYPE_F32 = 0, GSA_DTYPE_BF16 = 1 };
enum { GSA_ACT_SIGMOID = 0, GSA_ACT_TANH = 1, GSA_ACT_SILU = 2, GSA_ACT_RELU = 3 };

/* Shape of one GSA layer (GSAConfig fields, gsa/config.py:24-74). */
typedef struct {
  int32_t d_model;
  int32_t n_heads;
  int32_t n_kv_heads;
  int32_t d_head;
  int32_t n_idx_heads;  /* n_indexer_heads */
  int32_t d_idx;        /* d_indexer */
  int32_t gate_act;     /* GSA_ACT_SIGMOID | TANH | SILU */
  int32_t idx_act;      /* GSA_ACT_SIGMOID | RELU */
} gsa_dims;

/* Column offsets (in elements) of each projection inside one row of the fused projection
 * output ``proj`` = x . [W_q | W_k | W_v | W_g2 | W_g1 | W_qI | W_kI | W_w]^T (+ biases).
 * -1 marks a segment that is absent (gate disabled). */
typedef struct {
  int64_t q, k, v, g2, g1, qi, ki, wi;
} gsa_proj_layout;

/* Adaptive-k parameters (AdaptiveTopKSelector.__init__, adaptive_topk.py:29-57). */
typedef struct {
  int32_t k_base, k_min, k_max;
  int32_t use_adaptive;
  float temperature;
} gsa_topk_params;

/* Last error code recorded by a kernel on the current device (0 if none); clears it. */
int gsa_get_device_error(int* code_out, gsa_stream_t stream);

/* Library version string. */
const char* gsa_version(void);

/*
 * Projection epilogue: RoPE on q and k (rope.py:151-185), G2 v <- v * act(g2)
 * (value_gate.py:95-113), the G1 gate act(g1) (output_gate.py:101-117), the indexer head
 * weights w = sigmoid(wI) (gated_indexer.py:121) and the per-row score centre
 * shift = 0.5 * sum_j w_j.  ``proj`` rows already hold x.W^T + bias for every segment.
 * Replaces gated_sparse_attention.py:175-186 after the GEMM, and the G1 logits of :226-227.
 *   proj          [T, proj_ld]            dtype
 *   positions     [T] int64
 *   cos_tab/sin_tab [tab_rows, d_head]    tab_dtype (the module's RoPE buffers)
 *   q_out [T, H, D]; k_out, v_out: token t's [Hk, D] row at t * kv_ld (kv_ld = 2*Hk*D and
 *   v_out = k_out + Hk*D gives the interleaved KV layout gsa_sparse_sdpa reads fastest);
 *   g1_out [T, H, D] (NULL if no G1), w_out [T, H_I] fp32, shift_out [T] fp32
 */
int gsa_proj_epilogue(const gsa_dims* dims, const gsa_proj_layout* layout, int dtype, int64_t T,
                      const void* proj, int64_t proj_ld, const int64_t* positions,
                      const void* cos_tab, const void* sin_tab, int tab_dtype, int64_t tab_rows,
                      void* q_out, void* k_out, void* v_out, int64_t kv_ld, void* g1_out,
                      float* w_out, float* shift_out, gsa_stream_t stream);

/*
 * The layer's projections and their epilogue in one tensor-core GEMM (bf16): replaces the GEMM
 * proj = x . Wcat^T + b followed by gsa_proj_epilogue (gated_sparse_attention.py:175-186,
 * value_gate.py:95-113, output_gate.py:101-117, gated_indexer.py:114-121, rope.py:151-185), with
 * the epilogue applied to the accumulator tile in registers so that no projection tensor exists.
 *   x     [T, d_model] bf16, rows of stride x_ld
 *   wp    [gsa_proj_fused_rows(dims), d_model] bf16: the projection weights with rows in this order
 *         (D = d_head): q (H*D), k (Hk*D), then for each KV head h: v_h (D) followed by g2_h (D),
 *         g1 (H*D), q^I (H_I*d_I), k^I (d_I), w (H_I), zero rows up to the returned count
 *   bias  [gsa_proj_fused_rows(dims)] fp32 in the same order (0 for the bias-free projections)
 *   positions [T] int64 or NULL (row t = b*L + i at position pos0 + i)
 *   outputs as gsa_proj_epilogue_cache (L rows per sequence; K/V/k^I at the batch strides) plus
 *   qi_out [T, qi_ld] bf16 (the indexer queries) and ki_out (the indexer keys, required).
 * Supported: d_head 64 or 128 with H*D, Hk*D multiples of 256, d_I and H_I*d_I multiples of 16,
 * H_I <= 16, d_model a multiple of 64, both gates present (per-head G1), bf16 cos / sin tables,
 * 16-byte aligned rows and strides; otherwise GSA_ERR_UNSUPPORTED (use the GEMM +
 * gsa_proj_epilogue pair).  Outputs are bit-identical to that pair's.
 */
int64_t gsa_proj_fused_rows(const gsa_dims* dims);
int gsa_proj_fused(const gsa_dims* dims, int dtype, int64_t T, int64_t L, const void* x, int64_t x_ld,
                   const void* wp, const float* bias, const int64_t* positions, int64_t pos0,
                   const void* cos_tab, const void* sin_tab, int tab_dtype, int64_t tab_rows,
                   void* q_out, void* k_out, void* v_out, int64_t kv_ld, int64_t kv_bstride,
                   void* g1_out, void* qi_out, int64_t qi_ld, void* ki_out, int64_t ki_ld,
                   int64_t ki_bstride, float* w_out, float* shift_out, gsa_stream_t stream);

/*
 * gsa_proj_epilogue writing K, V and the indexer keys k^I straight into a KV cache that holds
 * room for more tokens than it has (the append-in-place cache of GatedSparseAttention).  The
 * T = B * L rows of ``proj`` are L new tokens of each of B sequences; token t of sequence b goes to
 *   k_out, v_out at b * kv_bstride + t * kv_ld    (kv_bstride >= L * kv_ld; pass the cache
 *                                                  pointers already offset to the first new slot)
 *   ki_out       at b * ki_bstride + t * ki_ld    (d_I elements copied from proj's k^I columns;
 *                                                  NULL: not written)
 * q_out, g1_out, w_out and shift_out are dense [T, ...] as in gsa_proj_epilogue.  Replaces the
 * torch.cat of gated_sparse_attention.py:188-192 (the reference has no k^I cache).
 */
int gsa_proj_epilogue_cache(const gsa_dims* dims, const gsa_proj_layout* layout, int dtype,
                            int64_t B, int64_t L, const void* proj, int64_t proj_ld,
                            const int64_t* positions, const void* cos_tab, const void* sin_tab,
                            int tab_dtype, int64_t tab_rows, void* q_out, void* k_out, void* v_out,
                            int64_t kv_ld, int64_t kv_bstride, void* ki_out, int64_t ki_ld,
                            int64_t ki_bstride, void* g1_out, float* w_out, float* shift_out,
                            gsa_stream_t stream);

/*
 * Gated indexer scores, I[t,s] = sum_j w[t,j] * act(scale * <qI[t,j], kI[s]> + bias[j])
 * (gated_indexer.py:106-145), for query rows t in [0, Lq) of each batch against keys
 * s in [0, Lkv).  With ``causal`` set, key s is masked for query row t when
 * s > q_pos0 + t (gated_indexer.py:148-153 with a query offset); masked entries are written
 * as -inf only if ``write_masked`` is set.
 *   qI  [B, Lq, H_I*d_I] rows of stride qi_ld (elements), batch stride qi_bstride
 *   kI  [B, Lkv, d_I]    rows of stride ki_ld, batch stride ki_bstride
 *   w   [B*Lq, H_I] fp32 ; bias [H_I] fp32
 *   scores [B*Lq, scores_ld] fp32
 *   row_stats [B*Lq, 3] fp64 accumulated (+=) : sum(x - shift), sum((x - shift)^2), count
 *     over unmasked entries; NULL to skip.  shift [B*Lq] fp32 or NULL (0).
 */
int gsa_indexer_scores(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv,
                       int64_t q_pos0, int causal, int write_masked, const void* qI,
                       int64_t qi_ld, int64_t qi_bstride, const void* kI, int64_t ki_ld,
                       int64_t ki_bstride, const float* w, const float* bias, float scale,
                       const float* shift, float* scores, int64_t scores_ld, double* row_stats,
                       gsa_stream_t stream);

/*
 * Row statistics of a materialised score matrix (adaptive_topk.py:84-88): per row
 * sum(x), sum(x^2) and the count of finite entries, accumulated into row_stats[R, 3] (fp64,
 * caller zeroes).  scores [R, scores_ld] fp32, first ``n_cols`` columns.
 */
int gsa_row_stats(int64_t R, int64_t n_cols, const float* scores, int64_t scores_ld,
                  double* row_stats, gsa_stream_t stream);

/*
 * Per-row statistics for the entropy and learned adaptive-k methods (adaptive_topk.py:84-127), of a
 * score matrix whose values are of dtype ``dtype`` (stored as fp32; -inf = masked):
 *   out [R, 5] fp32 = {valid count, mean, unbiased std, max of the masked scores (masked entries
 *   count as 0 over all n_cols columns), softmax entropy -sum p log(p + 1e-10) over the valid
 *   entries}, every value but the count rounded to ``dtype`` as the reference's torch ops round it.
 */
int gsa_row_summary(int64_t R, int64_t n_cols, const float* scores, int64_t scores_ld, int dtype,
                    float* out, gsa_stream_t stream);

/*
 * Top-k candidates: for every row r, the k_eff largest finite scores among the first n_r
 * columns, ties broken lower column first, written in ascending column order
 * (the candidate set of adaptive_topk.py:174-177).  n_r = n_cols, or, with ``causal``,
 * min(n_cols, q_pos0 + (r % Lq) + 1).  cand_count[r] = min(k_eff, finite entries).
 *   scores [R, scores_ld] fp32 ; cand_idx [R, k_eff] int32 ; cand_score [R, k_eff] fp32
 *   row_center [R] fp32 or NULL: when given, every finite score of row r must lie in
 *     [0, 2 row_center[r]] (true of sigmoid indexer scores with row_center = the
 *     gsa_proj_epilogue shift); the selection then takes two passes over the row instead of
 *     four.  Requires 16-byte aligned rows (scores_ld % 4 == 0).
 *   row_stats [R, 3] fp64 or NULL (needs row_center): the row statistics gsa_indexer_scores
 *     produced for these rows with shift = row_center; the selection then usually takes one
 *     pass (a threshold at the row's estimated (1 - 1.5 k_eff / n) quantile).  The result is
 *     the same with or without it.
 */
int gsa_topk_candidates(int64_t R, int64_t Lq, int64_t n_cols, int64_t q_pos0, int causal,
                        const float* scores, int64_t scores_ld, const float* row_center,
                        const double* row_stats, int32_t k_eff, int32_t* cand_idx,
                        float* cand_score, int32_t* cand_count, gsa_stream_t stream);

/*
 * Per-row variance over all N_r = n_cols entries with masked entries counted as 0, unbiased
 * (adaptive_topk.py:84-93), rounded to the activation dtype; plus the layer-wide sum of the
 * rounded variances and the row count, var_total[2] (fp64, overwritten).  row_stats as
 * produced by gsa_indexer_scores / gsa_row_stats, shift as passed there (NULL = 0).
 */
int gsa_row_variance(int64_t R, int64_t n_cols, int dtype, const double* row_stats,
                     const float* shift, float* var_out, double* var_total, gsa_stream_t stream);

/*
 * Adaptive k (adaptive_topk.py:96-136 and :161-172): k[r] from var[r], the layer mean
 * var_total[0] / var_total[1] and the valid count, in the activation dtype's arithmetic;
 * with use_adaptive == 0, k[r] = min(k_base, n_cols).  valid count = row_stats[r,2].
 */
int gsa_adaptive_k(int64_t R, int64_t n_cols, int dtype, const gsa_topk_params* p,
                   const float* var, const double* var_total, const double* row_stats,
                   int32_t* k_out, gsa_stream_t stream);

/*
 * Final selection: the top k[r] of each row's candidates (ties lower column first), in
 * ascending column order, into sel_idx[R, sel_ld]; sel_count[r] = min(k[r], cand_count[r],
 * sel_ld).  The candidates are cand_idx / cand_score [R, k_eff] with cand_count[r] <= k_eff.
 * Reproduces the mask p < k_t of adaptive_topk.py:181-189.  If sel_mask [R, k_eff] (uint8)
 * is given, sel_mask[r, p] = 1 iff candidate p of row r is selected (the reference's
 * (indices, mask) pair with indices = the candidates).
 */
int gsa_select_finalize(int64_t R, int32_t k_eff, const int32_t* cand_idx,
                        const float* cand_score, const int32_t* cand_count, const int32_t* k,
                        int32_t* sel_idx, int64_t sel_ld, int32_t* sel_count,
                        uint8_t* sel_mask, gsa_stream_t stream);

/*
 * Elementwise gate out = x * act(logits) over n elements, each op rounded to the dtype as
 * torch evaluates it (value_gate.py:98-113, output_gate.py:111-126).  gate_out (nullable)
 * receives act(logits) (the modules' last_gate_scores).
 */
int gsa_apply_gate(int dtype, int act, int64_t n, const void* x, const void* logits, void* out,
                   void* gate_out, gsa_stream_t stream);

/*
 * GQA sparse SDPA with the G1 epilogue (gated_sparse_attention.py:234-290 and
 * output_gate.py:124-126): for every row r = (b, t), softmax(scale * q K_sel^T) V_sel per
 * head over the sel_count[r] keys sel_idx[r, :] shared by all heads, times gate[r] if given.
 *   q [B, Lq, H, D] ; gate like q ; out [B, Lq, H, D] in dtype
 *   k, v: key s of batch b is the [Hk, D] row at (b * Lkv + s) * kv_ld (16-byte aligned).
 *     The interleaved layout (kv_ld = 2*Hk*D, v = k + Hk*D) moves each selected key as one
 *     contiguous copy.  sel indices are key positions inside the batch's sequence.
 */
int gsa_sparse_sdpa(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv,
                    const void* q, const void* k, const void* v, int64_t kv_ld,
                    const int32_t* sel_idx, int64_t sel_ld, const int32_t* sel_count,
                    const void* gate, void* out, float scale, gsa_stream_t stream);

/*
 * gsa_sparse_sdpa over a KV cache with room beyond its Lkv tokens: key s of batch b is the
 * [Hk, D] row at b * kv_bstride + s * kv_ld (kv_bstride >= Lkv * kv_ld, a multiple of 8
 * elements).  With fewer rows B*Lq than the GPU holds CTAs (decode), a workspace of
 * gsa_sdpa_workspace_size bytes (16-byte aligned; NULL or smaller: not used) lets each row's
 * selected keys be split over several CTAs, whose partial softmax results a second kernel
 * merges.  gsa_sparse_sdpa is this call with kv_bstride = Lkv * kv_ld and no workspace.
 */
int64_t gsa_sdpa_workspace_size(const gsa_dims* dims, int64_t B, int64_t Lq);
int gsa_sparse_sdpa_strided(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv,
                            const void* q, const void* k, const void* v, int64_t kv_ld,
                            int64_t kv_bstride, const int32_t* sel_idx, int64_t sel_ld,
                            const int32_t* sel_count, const void* gate, void* out, float scale,
                            void* workspace, int64_t workspace_bytes, gsa_stream_t stream);

/*
 * gsa_sparse_sdpa_strided (no workspace) that also writes lse_out [B*Lq, H] fp32: the
 * natural-log sum-exp of scale * q.k over each row's selected keys per head (-inf for a row
 * without keys), which gsa_sparse_sdpa_backward needs.
 */
int gsa_sparse_sdpa_lse(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv,
                        const void* q, const void* k, const void* v, int64_t kv_ld,
                        int64_t kv_bstride, const int32_t* sel_idx, int64_t sel_ld,
                        const int32_t* sel_count, const void* gate, void* out, float* lse_out,
                        float scale, gsa_stream_t stream);

/*
 * Backward of the sparse SDPA without the gate (gated_sparse_attention.py:256-290 under
 * autograd; the selected indices carry no gradient, adaptive_topk.py:177).  With p = exp(scale
 * q.k - lse) over row r's selected keys and D = dO.O per head:
 *   dq [B*Lq, H, D] fp32 (written):  scale * sum_s p (dO.v_s - D) k_s
 *   dk, dv fp32 accumulators (added to; the caller zeroes them), key s of batch b at
 *     b * dkv_bstride + s * dkv_ld: dk_s += scale p (dO.v_s - D) q, dv_s += p dO (over the
 *     rows and the group's heads that selected s; atomics, so the last bits vary run to run)
 *   q, o, d_o [B*Lq, H, D] dtype; k, v, sel as in gsa_sparse_sdpa_strided; lse from
 *   gsa_sparse_sdpa_lse.  D in {64, 128}.
 */
int gsa_sparse_sdpa_backward(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv,
                             const void* q, const void* k, const void* v, int64_t kv_ld,
                             int64_t kv_bstride, const int32_t* sel_idx, int64_t sel_ld,
                             const int32_t* sel_count, const void* o, const void* d_o,
                             const float* lse, float* dq, float* dk, float* dv, int64_t dkv_ld,
                             int64_t dkv_bstride, float scale, gsa_stream_t stream);

/*
 * Attention probabilities of the sparse SDPA, the analysis output of output_attentions
 * (gated_sparse_attention.py:268-285): probs[r, h, j] = exp(scale * q[r, h] . k[idx[r, j]] - lse[r, h])
 * for every candidate j that mask[r, j] keeps (mask NULL: all k_eff), 0 for the others.  lse is what
 * gsa_sparse_sdpa_lse wrote for the same kept keys, so a row's probabilities of one head sum to 1.
 *   q [B*Lq, H, D] dtype; k as in gsa_sparse_sdpa_strided; idx, mask [B*Lq, idx_ld] (int32, uint8);
 *   probs [B*Lq, H, k_eff] dtype.  B*Lq <= 65535: an output of small shapes.
 */
int gsa_sparse_sdpa_probs(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv,
                          const void* q, const void* k, int64_t kv_ld, int64_t kv_bstride,
                          const int32_t* idx, const uint8_t* mask, int64_t idx_ld, int64_t k_eff,
                          const float* lse, float scale, void* probs, gsa_stream_t stream);

/*
 * Diagnostic of the failure path (no counterpart in the reference, whose only failure handling is
 * a try/except around its Triton calls): one CTA waits, with the bounded mbarrier wait of the
 * pipelined kernels, on a barrier nothing arrives on; after wait_limit polls it records
 * GSA_ERR_TIMEOUT in the device error word and returns.  Read the code with gsa_get_device_error.
 */
int gsa_selftest_bounded_wait(uint32_t wait_limit, gsa_stream_t stream);

/*
 * Decoder-layer elementwise ops around the attention (gsa/models/gsa_llama.py), each evaluated
 * as torch evaluates it for the dtype.  Rows of d (n) elements with row strides *_ld.
 *   gsa_add_rmsnorm: h = x + a (a nullable: no add; h_out then NULL) and
 *     y = (h * rsqrt(mean(h^2) + eps)).type_as(h) * weight        (RMSNorm, gsa_llama.py:18-30,
 *     after the residual adds of GSADecoderLayer.forward, :100-110); y_out or h_out may be NULL.
 *   gsa_silu_mul: z = silu(gu[:, :n]) * gu[:, n:2n]               (GSAMlp, gsa_llama.py:45-46)
 */
int gsa_add_rmsnorm(int dtype, int64_t T, int64_t d, const void* x, int64_t x_ld, const void* a,
                    int64_t a_ld, const void* weight, float eps, void* h_out, int64_t h_ld,
                    void* y_out, int64_t y_ld, gsa_stream_t stream);
int gsa_silu_mul(int dtype, int64_t T, int64_t n, const void* gu, int64_t gu_ld, void* z,
                 int64_t z_ld, gsa_stream_t stream);

/*
 * Workspace for gsa_indexer_select: bytes needed for a query chunk of ``chunk_rows`` rows
 * against n_cols keys.
 */
int64_t gsa_workspace_size(int64_t chunk_rows, int64_t n_cols);

/*
 * Indexer + top-k candidates over all query rows, chunk by chunk, so that at most
 * chunk_rows x Lkv scores exist at any time (in ``workspace``).  Row statistics for the
 * adaptive k are accumulated into row_stats (caller zeroes).  Same tensors as
 * gsa_indexer_scores and gsa_topk_candidates; causal prefill when ``causal``.
 */
int gsa_indexer_select(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv,
                       int64_t q_pos0, int causal, const void* qI, int64_t qi_ld,
                       int64_t qi_bstride, const void* kI, int64_t ki_ld, int64_t ki_bstride,
                       const float* w, const float* bias, float scale, const float* shift,
                       int32_t k_eff, int32_t* cand_idx, float* cand_score,
                       int32_t* cand_count, double* row_stats, int64_t chunk_rows,
                       void* workspace, int64_t workspace_bytes, gsa_stream_t stream);

/*
 * Indexer + threshold survivors, chunk by chunk (the layer's selection path for the sigmoid
 * indexer; gated_indexer.py:106-155 with the candidate stage of adaptive_topk.py:138-177).
 * Like gsa_indexer_select, but each row's candidates are its survivors: every score at or
 * above the row's estimated (1 - 1.25 k_eff / n_r) quantile (from the row statistics the
 * indexer accumulates), in ascending column order, up to ``cap`` per row.  Rows of n_r <= cap
 * keep every score; a row whose survivors are fewer than min(k_eff, n_r) or more than cap is
 * selected exactly (its k_eff best).  The candidates of every row therefore contain its k_eff
 * best scores, and gsa_select_finalize (with k_eff := cap) takes the final k_t from them.
 *   cand_idx / cand_score [B*Lq, cap]; cand_count [B*Lq]; row_stats [B*Lq, 3] (caller zeroes)
 *   shift (the row centre of gsa_proj_epilogue) is required; 2 cap >= 3 k_eff + 2048 (room
 *   above the threshold's aim).
 *   workspace: gsa_survivors_workspace_size(chunk_rows, Lkv) bytes, 256-byte aligned.
 * The score pass streams each chunk once at HBM rate, instead of a per-row selection.
 */
int64_t gsa_survivors_workspace_size(int64_t chunk_rows, int64_t n_cols);
int gsa_indexer_survivors(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv,
                          int64_t q_pos0, int causal, const void* qI, int64_t qi_ld,
                          int64_t qi_bstride, const void* kI, int64_t ki_ld, int64_t ki_bstride,
                          const float* w, const float* bias, float scale, const float* shift,
                          int32_t k_eff, int32_t cap, int32_t* cand_idx, float* cand_score,
                          int32_t* cand_count, double* row_stats, int64_t chunk_rows,
                          void* workspace, int64_t workspace_bytes, gsa_stream_t stream);

/*
 * gsa_indexer_survivors without the score matrix: same arguments, same outputs, bit for bit
 * (candidates, their order and count, row_stats).  Each chunk runs the tensor-core indexer
 * three times:
 *   1. the row statistics over every 16th key tile only, from which each row's threshold is
 *      its normal quantile of 1.4 k_eff / n_r (1/16 of the indexer's work);
 *   2. the full pass: the row statistics, and every score at or above the row's threshold
 *      written to the row's segment of that key range (4096 keys), in ascending column order;
 *      the segments are then joined into cand_idx / cand_score;
 *   3. a row whose survivors are fewer than min(k_eff, n_r), more than cap, or more than its
 *      segment's room has its 32-row query block's scores computed into the workspace and is
 *      selected exactly (its k_eff best), as gsa_indexer_survivors does.
 * Since every row's candidates hold all of its scores at or above a threshold below its k_eff-th
 * best, they hold its k_eff best, as in gsa_indexer_survivors; step 3 runs no block when no row
 * fails.  Supported: bf16, n_idx_heads 8, d_idx 64, sigmoid, 16-byte aligned qI / kI rows;
 * otherwise GSA_ERR_UNSUPPORTED (use gsa_indexer_survivors).
 *   workspace: gsa_survivors_fused_workspace_size(chunk_rows, Lkv, k_eff, cap) bytes.
 * ("Gated lightning indexer" scores and the candidate stage: gated_indexer.py:106-155,
 * adaptive_topk.py:138-177.)
 */
int64_t gsa_survivors_fused_workspace_size(int64_t chunk_rows, int64_t n_cols, int32_t k_eff,
                                           int32_t cap);
int gsa_indexer_survivors_fused(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq,
                                int64_t Lkv, int64_t q_pos0, int causal, const void* qI,
                                int64_t qi_ld, int64_t qi_bstride, const void* kI, int64_t ki_ld,
                                int64_t ki_bstride, const float* w, const float* bias,
                                float scale, const float* shift, int32_t k_eff, int32_t cap,
                                int32_t* cand_idx, float* cand_score, int32_t* cand_count,
                                double* row_stats, int64_t chunk_rows, void* workspace,
                                int64_t workspace_bytes, gsa_stream_t stream);

/*
 * gsa_indexer_select without a workspace argument: it allocates no device memory.  No
 * counterpart in the reference (whose indexer materialises the score matrix with torch).
 *
 * For callers that cannot provide or allocate scratch at call time: serving runtimes that
 * reserve all device memory for their own pools up front, and host code with no device
 * allocator of its own.  The chunk scores live in a buffer of GSA_STATIC_SCRATCH_BYTES that
 * the library holds per device, so a chunk is GSA_STATIC_SCRATCH_BYTES / (4 * round4(Lkv))
 * query rows and Lkv may be at most 16,777,216; a longer key length returns
 * GSA_ERR_WORKSPACE.  row_stats (if given) is zeroed by the call itself, on ``stream``.
 *
 * Each call looks up the buffer's device address in the calling thread's current context (the
 * address belongs to the context, so it is never cached across calls); the first call in a
 * context also loads the library's device code there: make it before any stream capture.
 * Arguments are checked before anything is written.  All calls on a device
 * share the buffer: calls that overlap in time on one device (two streams or two host threads)
 * race on it, so the caller serialises them.
 */
#define GSA_STATIC_SCRATCH_BYTES (64LL << 20)
int gsa_indexer_select_static(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq,
                              int64_t Lkv, int64_t q_pos0, int causal, const void* qI,
                              int64_t qi_ld, int64_t qi_bstride, const void* kI, int64_t ki_ld,
                              int64_t ki_bstride, const float* w, const float* bias, float scale,
                              const float* shift, int32_t k_eff, int32_t* cand_idx,
                              float* cand_score, int32_t* cand_count, double* row_stats,
                              gsa_stream_t stream);

/*
 * The attention of one decode step between its two GEMMs, in one call: B sequences of L new
 * tokens each, whose K/V and k^I caches hold ``past`` tokens in stores with room for the new ones
 * (GatedSparseAttention.forward, gated_sparse_attention.py:175-230, after the fused projection
 * GEMM and before o_proj; the reference concatenates the caches at :188-192 and has no k^I cache):
 *   gsa_proj_epilogue_cache (K, V, k^I of the new tokens into slots past .. past+L-1)
 *   -> gsa_indexer_survivors (gsa_indexer_select where the survivor pass does not apply) over
 *      the past+L keys, offset-causal -> gsa_row_variance -> gsa_adaptive_k (variance mean over
 *      the B*L rows of the call) -> gsa_select_finalize -> gsa_sparse_sdpa_strided.
 *   proj       [B*L, proj_ld] dtype: x . Wcat^T + b (the layout of gsa_proj_layout)
 *   positions  [B*L] int64, or NULL: token t of a sequence at position past + t
 *   kv_store   [B, cap, 2, Hk, D] dtype (K and V interleaved), batch stride kv_bstride elements
 *   ki_store   [B, cap, d_I] dtype, batch stride ki_bstride elements
 *   idx_bias   [H_I] fp32 (GatedLightningIndexer.bias); idx_scale = 1/sqrt(d_I); attn_scale = 1/sqrt(D)
 *   attn_out   [B*L, H*D] dtype: the gated attention output (o_proj's input)
 *   k_out      [B*L] int32 or NULL: each row's k_t
 *   phase      GSA_DECODE_ALL: the whole step.  When the batch's sequences are spread over several
 *              GPUs (the adaptive k's variance mean spans all of them, adaptive_topk.py:93-96):
 *              GSA_DECODE_SCORE runs up to the row variances and leaves (sum of variances, row
 *              count) in var_total [2] fp64; the caller all-reduces it; GSA_DECODE_ATTEND with the
 *              same arguments and workspace finishes the step from var_total.
 *   var_total  [2] fp64, required for the two phases (NULL with GSA_DECODE_ALL)
 *   workspace  gsa_decode_workspace_size(dims, tp, dtype, B, L, n_keys) bytes with n_keys >= past + L
 *              (size it once for the cache capacity), 256-byte aligned.
 */
enum { GSA_DECODE_ALL = 0, GSA_DECODE_SCORE = 1, GSA_DECODE_ATTEND = 2 };
int64_t gsa_decode_workspace_size(const gsa_dims* dims, const gsa_topk_params* tp, int dtype,
                                  int64_t B, int64_t L, int64_t n_keys);
int gsa_decode_attend(const gsa_dims* dims, const gsa_proj_layout* layout, const gsa_topk_params* tp,
                      int dtype, int64_t B, int64_t L, int64_t past, const void* proj, int64_t proj_ld,
                      const int64_t* positions, const void* cos_tab, const void* sin_tab, int tab_dtype,
                      int64_t tab_rows, void* kv_store, int64_t kv_bstride, void* ki_store,
                      int64_t ki_bstride, const float* idx_bias, float idx_scale, float attn_scale,
                      void* attn_out, int32_t* k_out, double* var_total, int phase, void* workspace,
                      int64_t workspace_bytes, gsa_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GSA_B200_H_ */
