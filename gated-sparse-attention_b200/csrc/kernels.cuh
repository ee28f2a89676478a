// Argument blocks and launchers of the GSA kernels, shared by the kernel translation units
// and the C-ABI layer (abi.cu).
#pragma once

#include "common.cuh"

namespace gsa {

// Layer shape the kernels can take (shared by every entry point's argument check).
inline bool dims_ok(const gsa_dims* d) {
  return d && d->d_model > 0 && d->n_heads > 0 && d->n_kv_heads > 0 && d->n_heads % d->n_kv_heads == 0 &&
         d->d_head > 0 && d->d_head % 2 == 0 && d->n_idx_heads > 0 && d->d_idx > 0;
}

struct EpiArgs {
  gsa_dims d;
  gsa_proj_layout lay;
  int dtype;
  int64_t T;
  const void* proj;
  int64_t proj_ld;
  const int64_t* positions;
  const void* cos_tab;
  const void* sin_tab;
  int tab_dtype;
  int64_t tab_rows;
  void* q_out;
  void* k_out;
  void* v_out;
  int64_t kv_ld;      // elements between consecutive tokens of k_out and of v_out
  void* g1_out;
  float* w_out;
  float* shift_out;
  int* err;
  // cache layout (gsa_proj_epilogue_cache): token t = b * L + i of k_out/v_out at
  // b * kv_bstride + i * kv_ld, its k^I at b * ki_bstride + i * ki_ld; L = 0: t * kv_ld, no k^I
  int64_t L;
  int64_t kv_bstride;
  void* ki_out;
  int64_t ki_ld, ki_bstride;
  int64_t pos0;       // positions == NULL: token t = b * L + i sits at position pos0 + i
  double* zero_stats; // [T, 3] set to zero (the indexer's row statistics of a decode step), or NULL
};

// RoPE position of the epilogue's token t.
__device__ __forceinline__ int64_t epi_position(const EpiArgs& a, int64_t t) {
  return a.positions ? a.positions[t] : a.pos0 + (a.L ? t % a.L : t);
}

// Offset of token t's K (or V) row in an epilogue's k_out / v_out.
__host__ __device__ __forceinline__ int64_t epi_kv_off(const EpiArgs& a, int64_t t) {
  return a.L ? (t / a.L) * a.kv_bstride + (t % a.L) * a.kv_ld : t * a.kv_ld;
}

struct IdxArgs {
  int dtype;
  int64_t Lq, Lkv, q_pos0;
  int causal, write_masked;
  int HI, dI, act;
  const void* qI;
  int64_t qi_ld, qi_bstride;
  const void* kI;
  int64_t ki_ld, ki_bstride;
  const float* w;
  const float* bias;
  float scale;
  const float* shift;
  float* scores;
  int64_t scores_ld;
  double* row_stats;
  // Deterministic row statistics (tensor-core path): per-(row, key range) partials [Lq, ranges, 3],
  // summed into row_stats in range order after the launch.  NULL: fp64 atomics (summation order
  // varies run to run in the last bits).
  double* stat_part = nullptr;
};
int64_t indexer_tc_stat_ranges(int64_t Lkv);  // key ranges per row of the tensor-core indexer

// Rows of the fused survivor pass (the tensor-core indexer writes each row's survivors itself, in
// segments, one per key range of kRangeKeys keys).  Host and device compute the same layout.
struct SurvivorShape {
  static constexpr int64_t kRangeKeys = 4096;  // keys of one range (= one indexer work item)
  int32_t K;    // keys the final selection may need per row (k_eff)
  int32_t cap;  // candidate row length
  int32_t K14;  // survivors the threshold aims at per row: ceil(1.4 K)
  __host__ __device__ static int64_t ranges(int64_t n) { return (n + kRangeKeys - 1) / kRangeKeys; }
  // Room of one (row, range) for a row of n keys: the whole range where the row keeps every key
  // (n <= cap); else four times the range's share of K14, plus 128, in multiples of 32.
  __host__ __device__ int64_t seg_cap(int64_t n) const {
    if (n <= cap) return kRangeKeys;
    int64_t c = (4 * kRangeKeys * (int64_t)K14 + n - 1) / n;
    c = (c + 31) / 32 * 32 + 128;
    return c < kRangeKeys ? c : kRangeKeys;
  }
};

// Launch modes of the tensor-core indexer (bf16, d_I 64): every score to the scratch; the row
// statistics of every 16th key tile only (the survivor thresholds' estimate); the statistics and
// each row's survivors written to its per-range segments (H_I = 8).
constexpr int kTcScores = 0, kTcSample = 1, kTcEmit = 2;
struct TcSurvivorArgs {
  const int32_t* blk_mask = nullptr;   // kTcScores: query blocks to compute (NULL: all)
  const double* samp_stats = nullptr;  // kTcEmit: [Lq, 3] sampled statistics of (score - shift)
  int32_t* seg_idx = nullptr;          // kTcEmit: row r, range j at r * seg_stride + j * sv.seg_cap(n_r)
  float* seg_score = nullptr;
  int32_t* seg_cnt = nullptr;          // kTcEmit: [Lq, indexer_tc_stat_ranges(Lkv)]
  int64_t seg_stride = 0;
  SurvivorShape sv{};
};
int launch_indexer_tc_mode(const IdxArgs& a, int mode, const TcSurvivorArgs& x, int* err, cudaStream_t stream);
constexpr int kTcQueryBlock8 = 32;     // query rows of one tensor-core indexer block at H_I = 8

struct SdpaArgs {
  int64_t B, Lq, Lkv;
  int Hk;
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t kv_ld;      // elements between consecutive key rows of k and of v
  int interleaved;    // v == k + Hk*D and kv_ld == 2*Hk*D: one 4 KiB copy per key
  const int32_t* sel_idx;
  int64_t sel_ld;
  const int32_t* sel_count;
  const __nv_bfloat16* gate;
  __nv_bfloat16* out;
  float scale_log2;
  int nstages;
  int nprod;          // producer warps
  int* err;
  int64_t kv_bstride; // elements between batches of k and of v (>= Lkv * kv_ld)
  // key splits per row (few rows: each row's selected keys are cut into `splits` ranges taken by
  // different CTAs; partial outputs o [R*splits, H, D] fp32 and their log2-sum-exp [R*splits, H]
  // in `part`, merged by a second kernel).  1: no split.
  int splits;
  float* part;
  int64_t part_floats; // capacity of part
  int prefetch;        // stages ahead whose keys the producers prefetch into L2 (0: none)
  float* lse_out;      // [R, H] natural-log sum-exp of the scaled scores (unsplit launches), or NULL
};

struct SdpaF32Args {
  int64_t B, Lq, Lkv;
  int H, Hk, D;
  const float* q;
  const float* k;
  const float* v;
  int64_t kv_ld;
  const int32_t* sel_idx;
  int64_t sel_ld;
  const int32_t* sel_count;
  const float* gate;
  float* out;
  float scale;
  int* err;
  int64_t kv_bstride;
  float* lse_out;      // [R, H] natural-log sum-exp of the scaled scores, or NULL
};

// Backward of the sparse SDPA (without the gate): per row r and head h, with p = exp(scale q.k_s
// - lse) over the row's selected keys s, D = dO.O:
//   dq_h = scale sum_s p_s (dO.v_s - D) k_s;  dk_s += scale p_s (dO.v_s - D) q_h;  dv_s += p_s dO_h
struct SdpaBwdArgs {
  int64_t B, Lq, Lkv;
  int H, Hk, D;
  int dtype;
  const void* q;       // [R, H, D]
  const void* k;       // key s of batch b at b * kv_bstride + s * kv_ld (elements)
  const void* v;
  int64_t kv_ld, kv_bstride;
  const int32_t* sel_idx;
  int64_t sel_ld;
  const int32_t* sel_count;
  const void* o;       // [R, H, D] the forward output (ungated)
  const void* d_o;     // [R, H, D]
  const float* lse;    // [R, H]
  float* dq;           // [R, H, D] fp32
  float* dk;           // fp32 accumulators, key s of batch b at b * dkv_bstride + s * dkv_ld
  float* dv;
  int64_t dkv_ld, dkv_bstride;
  float scale;
  int* err;
};
int launch_sdpa_backward(const SdpaBwdArgs& a, cudaStream_t stream);

// Attention probabilities of kept candidates (analysis output): out [R, H, k_eff].
struct SdpaProbsArgs {
  int64_t B, Lq, Lkv;
  int H, Hk, D;
  const void* q;        // [R, H, D]
  const void* k;        // key s of batch b at b * kv_bstride + s * kv_ld (elements)
  int64_t kv_ld, kv_bstride;
  const int32_t* idx;   // [R, idx_ld] candidate key positions
  const uint8_t* mask;  // [R, idx_ld] 1 = kept, or NULL (all k_eff kept)
  int64_t idx_ld;
  int64_t k_eff;
  const float* lse;     // [R, H]
  float scale;
  void* out;            // [R, H, k_eff]
  int* err;
};
int launch_sdpa_probs(const SdpaProbsArgs& a, int dtype, cudaStream_t stream);

// Fused projection GEMM + epilogue (bf16): see proj_gemm.cu for the weight row order.
struct ProjGemmArgs {
  gsa_dims d;
  int64_t T;
  int64_t L;                  // rows per sequence (K/V/k^I batch strides apply per sequence)
  const void* x;              // [T, d_model]
  int64_t x_ld;
  const void* w;              // [proj_gemm_columns(d), d_model]
  const float* bias;          // [proj_gemm_columns(d)]
  const int64_t* positions;   // [T] or NULL
  int64_t pos0;
  const void* cos_tab;
  const void* sin_tab;
  int tab_dtype;
  int64_t tab_rows;
  void* q_out;
  void* k_out;
  void* v_out;
  int64_t kv_ld, kv_bstride;
  void* g1_out;
  void* qi_out;
  int64_t qi_ld;
  void* ki_out;
  int64_t ki_ld, ki_bstride;
  float* w_out;
  float* shift_out;
  int* err;
};
bool proj_gemm_eligible(const ProjGemmArgs& a);
int64_t proj_gemm_columns(const gsa_dims& d);
int launch_proj_gemm(const ProjGemmArgs& a, int num_sms, cudaStream_t stream);
int launch_wait_selftest(uint32_t limit, int* err, cudaStream_t stream);
int launch_variance_adaptive_k(int64_t R, int64_t n_cols, int dtype, const gsa_topk_params& p,
                               const double* stats, const float* shift, float* var_out, double* total,
                               int32_t* k_out, cudaStream_t stream);
int launch_add_rmsnorm(int dtype, int64_t T, int64_t d, const void* x, int64_t x_ld, const void* a, int64_t a_ld,
                       const void* w, float eps, void* h_out, int64_t h_ld, void* y_out, int64_t y_ld,
                       cudaStream_t stream);
int launch_silu_mul(int dtype, int64_t T, int64_t n, const void* gu, int64_t gu_ld, void* z, int64_t z_ld,
                    cudaStream_t stream);

int launch_proj_epilogue(const EpiArgs& a, cudaStream_t stream);
int launch_apply_gate(int dtype, int act, int64_t n, const void* x, const void* logits, void* out, void* gate_out,
                      cudaStream_t stream);
int launch_indexer_simt(const IdxArgs& a, int64_t B, cudaStream_t stream);
bool indexer_tc_eligible(const IdxArgs& a);
int launch_indexer_tc(const IdxArgs& a, int* err, cudaStream_t stream);
bool indexer_decode_eligible(const IdxArgs& a, int64_t B);
int launch_indexer_decode(const IdxArgs& a, int64_t B, int num_sms, cudaStream_t stream);
int launch_topk_candidates(int64_t R, int64_t Lq, int64_t n_cols, int64_t q_pos0, int causal, const float* scores,
                           int64_t ld, const float* row_center, const double* row_stats, int32_t k_eff,
                           int32_t* cand_idx, float* cand_score, int32_t* cand_count, cudaStream_t stream);
int launch_threshold_candidates(int64_t R, int64_t Lq, int64_t n_cols, int64_t q_pos0, int causal,
                                const float* scores, int64_t ld, const float* center, const double* stats,
                                int32_t K, int32_t cap, int32_t* cand_idx, float* cand_score, int32_t* cand_count,
                                int32_t* fail_list, int32_t* fail_count, int32_t* seg_count, int num_sms, int* err,
                                cudaStream_t stream);
int launch_seg_concat(int64_t R, int64_t Lq, int64_t n_cols, int64_t q_pos0, int causal, const SurvivorShape& sv,
                      const int32_t* seg_idx, const float* seg_score, const int32_t* seg_cnt, int64_t seg_stride,
                      int64_t n_ranges, int32_t* cand_idx, float* cand_score, int32_t* cand_count,
                      int32_t* fail_list, int32_t* fail_count, int32_t* blk_flag, int32_t blk_rows,
                      cudaStream_t stream);
int launch_survivor_fallback(int64_t R, int64_t Lq, int64_t n_cols, int64_t q_pos0, int causal,
                             const float* scores, int64_t ld, const float* center, const double* stats, int32_t K,
                             int32_t cap, int32_t* cand_idx, float* cand_score, int32_t* cand_count,
                             int32_t* fail_list, int32_t* fail_count, int num_sms, int* err, cudaStream_t stream);
int launch_select_finalize_warp(int64_t R, int32_t cand_ld, const int32_t* cand_idx, const float* cand_score,
                                const int32_t* cand_count, const int32_t* k, int32_t* sel_idx, int64_t sel_ld,
                                int32_t* sel_count, int num_sms, cudaStream_t stream);
int launch_select_finalize(int64_t R, int32_t k_eff, const int32_t* cand_idx, const float* cand_score,
                           const int32_t* cand_count, const int32_t* k, int32_t* sel_idx, int64_t sel_ld,
                           int32_t* sel_count, uint8_t* sel_mask, cudaStream_t stream);
int launch_row_summary(int64_t R, int64_t n_cols, const float* scores, int64_t ld, int dtype, float* out,
                       cudaStream_t stream);
int launch_row_stats(int64_t R, int64_t n_cols, const float* scores, int64_t ld, double* stats,
                     cudaStream_t stream);
int launch_row_variance(int64_t R, int64_t n_cols, int dtype, const double* stats, const float* shift,
                        float* var_out, double* total, cudaStream_t stream);
int launch_adaptive_k(int64_t R, int64_t n_cols, int dtype, const gsa_topk_params& p, const float* var,
                      const double* var_total, const double* stats, int32_t* k_out, cudaStream_t stream);
int launch_sdpa_bf16(SdpaArgs a, int D, int nrep, int num_sms, cudaStream_t stream);
int launch_sdpa_f32(const SdpaF32Args& a, cudaStream_t stream);

}  // namespace gsa
