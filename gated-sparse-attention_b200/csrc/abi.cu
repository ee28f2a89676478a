// extern "C" entry points of libgsa_b200.so: argument validation, launch configuration and
// the chunked indexer + top-k loop.  Declarations and reference citations: include/gsa_b200.h.
#include <mutex>

#include "kernels.cuh"

namespace gsa {

__device__ int g_device_error;

// ---------------------------------------------------------------------------------------------
// Per-call device state: the address of the error word in the current context, and the SM count.
// The address is looked up on every call: it belongs to the CUDA context (a cudaDeviceReset, or a
// driver-API caller's own context on the same device, loads the module at another address), and
// once the module is loaded in a context the lookup is a table search.  The SM count is a
// property of the device and is cached per ordinal.
// ---------------------------------------------------------------------------------------------
struct DeviceInfo {
  int* err = nullptr;
  int num_sms = 0;
};
static std::mutex g_mu;
static int g_num_sms[64];

static int device_info(DeviceInfo* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return GSA_ERR_CUDA;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess || p == nullptr) {
    cudaGetLastError();
    return GSA_ERR_CUDA;
  }
  out->err = static_cast<int*>(p);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_num_sms[dev] == 0) {
      int sms = 0;
      if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
        return GSA_ERR_CUDA;
      g_num_sms[dev] = sms;
    }
    out->num_sms = g_num_sms[dev];
  }
  return GSA_OK;
}

static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Query chunks of at most ``rows`` rows for the indexer passes.  Lq <= rows: whole sequences,
// nb of them from sequence b0 (n = Lq rows each), so that short rows (decode) of many sequences
// share one launch; otherwise rows [t0, t0 + n) of the single sequence b0 (nb = 1).
struct ChunkIter {
  int64_t B, Lq, rows;
  int64_t b0 = 0, nb = 0, t0 = 0, n = 0;
  bool started = false;
  ChunkIter(int64_t B_, int64_t Lq_, int64_t rows_) : B(B_), Lq(Lq_), rows(rows_) {}
  bool next() {
    if (Lq <= rows) {
      if (started) b0 += nb;
      started = true;
      if (b0 >= B) return false;
      nb = std::min(rows / Lq, B - b0);
      t0 = 0;
      n = Lq;
      return true;
    }
    if (started) {
      t0 += n;
      if (t0 >= Lq) {
        t0 = 0;
        ++b0;
      }
    }
    started = true;
    if (b0 >= B) return false;
    nb = 1;
    n = std::min(rows, Lq - t0);
    return true;
  }
};

}  // namespace gsa

using namespace gsa;

extern "C" {

const char* gsa_version(void) { return "gsa_b200 0.1.0 (sm_100a)"; }

int gsa_get_device_error(int* code_out, gsa_stream_t stream) {
  DeviceInfo dinfo, *di = &dinfo;
  int st = device_info(di);
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int h = 0;
  if (cudaMemcpyAsync(&h, di->err, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) return GSA_ERR_CUDA;
  if (cudaStreamSynchronize(s) != cudaSuccess) return GSA_ERR_CUDA;
  if (cudaMemsetAsync(di->err, 0, sizeof(int), s) != cudaSuccess) return GSA_ERR_CUDA;
  if (code_out) *code_out = h;
  return GSA_OK;
}

int gsa_proj_epilogue(const gsa_dims* dims, const gsa_proj_layout* layout, int dtype, int64_t T,
                      const void* proj, int64_t proj_ld, const int64_t* positions, const void* cos_tab,
                      const void* sin_tab, int tab_dtype, int64_t tab_rows, void* q_out, void* k_out,
                      void* v_out, int64_t kv_ld, void* g1_out, float* w_out, float* shift_out,
                      gsa_stream_t stream) {
  if (!dims_ok(dims) || !layout || T < 0 || (dtype != GSA_DTYPE_F32 && dtype != GSA_DTYPE_BF16) ||
      (tab_dtype != GSA_DTYPE_F32 && tab_dtype != GSA_DTYPE_BF16))
    return GSA_ERR_BAD_ARG;
  if (T == 0) return GSA_OK;
  if (!proj || !positions || !cos_tab || !sin_tab || !q_out || !k_out || !v_out || !w_out || !shift_out ||
      tab_rows <= 0 || layout->q < 0 || layout->k < 0 || layout->v < 0 || layout->wi < 0)
    return GSA_ERR_BAD_ARG;
  if (dims->gate_act < GSA_ACT_SIGMOID || dims->gate_act > GSA_ACT_SILU) return GSA_ERR_UNSUPPORTED;
  if (kv_ld < (int64_t)dims->n_kv_heads * dims->d_head) return GSA_ERR_BAD_ARG;
  DeviceInfo dinfo, *di = &dinfo;
  int st = device_info(di);
  if (st) return st;
  EpiArgs a{*dims, *layout, dtype, T, proj, proj_ld, positions, cos_tab, sin_tab, tab_dtype, tab_rows,
            q_out, k_out, v_out, kv_ld, g1_out, w_out, shift_out, di->err};
  return launch_proj_epilogue(a, reinterpret_cast<cudaStream_t>(stream));
}

int gsa_proj_epilogue_cache(const gsa_dims* dims, const gsa_proj_layout* layout, int dtype, int64_t B, int64_t L,
                            const void* proj, int64_t proj_ld, const int64_t* positions, const void* cos_tab,
                            const void* sin_tab, int tab_dtype, int64_t tab_rows, void* q_out, void* k_out,
                            void* v_out, int64_t kv_ld, int64_t kv_bstride, void* ki_out, int64_t ki_ld,
                            int64_t ki_bstride, void* g1_out, float* w_out, float* shift_out, gsa_stream_t stream) {
  if (!dims_ok(dims) || !layout || B < 0 || L < 0 || (dtype != GSA_DTYPE_F32 && dtype != GSA_DTYPE_BF16) ||
      (tab_dtype != GSA_DTYPE_F32 && tab_dtype != GSA_DTYPE_BF16))
    return GSA_ERR_BAD_ARG;
  if (B * L == 0) return GSA_OK;
  if (!proj || !positions || !cos_tab || !sin_tab || !q_out || !k_out || !v_out || !w_out || !shift_out ||
      tab_rows <= 0 || layout->q < 0 || layout->k < 0 || layout->v < 0 || layout->wi < 0)
    return GSA_ERR_BAD_ARG;
  if (dims->gate_act < GSA_ACT_SIGMOID || dims->gate_act > GSA_ACT_SILU) return GSA_ERR_UNSUPPORTED;
  if (kv_ld < (int64_t)dims->n_kv_heads * dims->d_head || kv_bstride < L * kv_ld) return GSA_ERR_BAD_ARG;
  if (ki_out && (layout->ki < 0 || ki_ld < dims->d_idx || ki_bstride < L * ki_ld)) return GSA_ERR_BAD_ARG;
  DeviceInfo dinfo, *di = &dinfo;
  int st = device_info(di);
  if (st) return st;
  EpiArgs a{*dims, *layout, dtype, B * L, proj, proj_ld, positions, cos_tab, sin_tab, tab_dtype, tab_rows,
            q_out, k_out, v_out, kv_ld, g1_out, w_out, shift_out, di->err, L, kv_bstride, ki_out, ki_ld,
            ki_bstride};
  return launch_proj_epilogue(a, reinterpret_cast<cudaStream_t>(stream));
}

int64_t gsa_proj_fused_rows(const gsa_dims* dims) {
  if (!dims_ok(dims)) return 0;
  return proj_gemm_columns(*dims);
}

int gsa_proj_fused(const gsa_dims* dims, int dtype, int64_t T, int64_t L, const void* x, int64_t x_ld,
                   const void* wp, const float* bias, const int64_t* positions, int64_t pos0, const void* cos_tab,
                   const void* sin_tab, int tab_dtype, int64_t tab_rows, void* q_out, void* k_out, void* v_out,
                   int64_t kv_ld, int64_t kv_bstride, void* g1_out, void* qi_out, int64_t qi_ld, void* ki_out,
                   int64_t ki_ld, int64_t ki_bstride, float* w_out, float* shift_out, gsa_stream_t stream) {
  if (!dims_ok(dims) || T < 0 || L < 0 || (tab_dtype != GSA_DTYPE_F32 && tab_dtype != GSA_DTYPE_BF16))
    return GSA_ERR_BAD_ARG;
  if (dtype != GSA_DTYPE_BF16) return GSA_ERR_UNSUPPORTED;
  if (T == 0) return GSA_OK;
  if (!x || !wp || !bias || !cos_tab || !sin_tab || !q_out || !k_out || !v_out || !g1_out || !qi_out || !ki_out ||
      !w_out || !shift_out || tab_rows <= 0 || x_ld < dims->d_model)
    return GSA_ERR_BAD_ARG;
  const int64_t seq = L > 0 ? L : T;
  if (T % seq != 0 || kv_ld < (int64_t)dims->n_kv_heads * dims->d_head || qi_ld < (int64_t)dims->n_idx_heads * dims->d_idx ||
      ki_ld < dims->d_idx || (T > seq && (kv_bstride < seq * kv_ld || ki_bstride < seq * ki_ld)))
    return GSA_ERR_BAD_ARG;
  DeviceInfo dinfo, *di = &dinfo;
  int st = device_info(di);
  if (st) return st;
  ProjGemmArgs a{*dims, T, seq, x, x_ld, wp, bias, positions, pos0, cos_tab, sin_tab, tab_dtype, tab_rows,
                 q_out, k_out, v_out, kv_ld, kv_bstride, g1_out, qi_out, qi_ld, ki_out, ki_ld, ki_bstride,
                 w_out, shift_out, di->err};
  if (!proj_gemm_eligible(a)) return GSA_ERR_UNSUPPORTED;
  return launch_proj_gemm(a, di->num_sms, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"

// gsa_indexer_scores with, optionally, room for the tensor-core path's per-key-range statistic
// partials ([Lq, indexer_tc_stat_ranges(Lkv), 3] doubles, reused per batch row), which makes the row
// statistics the same bits on every run.
static int indexer_scores_impl(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv, int64_t q_pos0,
                               int causal, int write_masked, const void* qI, int64_t qi_ld, int64_t qi_bstride,
                               const void* kI, int64_t ki_ld, int64_t ki_bstride, const float* w,
                               const float* bias, float scale, const float* shift, float* scores,
                               int64_t scores_ld, double* row_stats, double* stat_part, gsa_stream_t stream) {
  if (!dims_ok(dims) || B < 0 || Lq < 0 || Lkv < 0 || (dtype != GSA_DTYPE_F32 && dtype != GSA_DTYPE_BF16))
    return GSA_ERR_BAD_ARG;
  if (B == 0 || Lq == 0 || Lkv == 0) return GSA_OK;
  if (!qI || !kI || !w || !bias || !scores || scores_ld < Lkv) return GSA_ERR_BAD_ARG;
  if (dims->idx_act != GSA_ACT_SIGMOID && dims->idx_act != GSA_ACT_RELU) return GSA_ERR_UNSUPPORTED;
  IdxArgs a{dtype, Lq, Lkv, q_pos0, causal, write_masked, dims->n_idx_heads, dims->d_idx, dims->idx_act,
            qI, qi_ld, qi_bstride, kI, ki_ld, ki_bstride, w, bias, scale, shift, scores, scores_ld, row_stats};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (indexer_decode_eligible(a, B)) {
    // a few tokens per sequence (decode): every sequence in one launch, streaming k^I once
    DeviceInfo dinfo, *di = &dinfo;
    int st = device_info(di);
    if (st) return st;
    return launch_indexer_decode(a, B, di->num_sms, s);
  }
  if (indexer_tc_eligible(a)) {
    // tensor-core kernel: bf16, d_I = 64, H_I in {4, 8}, sigmoid; one launch per batch row
    DeviceInfo dinfo, *di = &dinfo;
    int st = device_info(di);
    if (st) return st;
    const int64_t HI = dims->n_idx_heads;
    for (int64_t b = 0; b < B; ++b) {
      IdxArgs ab = a;
      ab.qI = static_cast<const __nv_bfloat16*>(qI) + b * qi_bstride;
      ab.kI = static_cast<const __nv_bfloat16*>(kI) + b * ki_bstride;
      ab.w = w + b * Lq * HI;
      ab.shift = shift ? shift + b * Lq : nullptr;
      ab.scores = scores + b * Lq * scores_ld;
      ab.row_stats = row_stats ? row_stats + b * Lq * 3 : nullptr;
      ab.stat_part = stat_part;
      st = launch_indexer_tc(ab, di->err, s);
      if (st) return st;
    }
    return GSA_OK;
  }
  return launch_indexer_simt(a, B, s);
}

extern "C" {

int gsa_indexer_scores(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv, int64_t q_pos0,
                       int causal, int write_masked, const void* qI, int64_t qi_ld, int64_t qi_bstride,
                       const void* kI, int64_t ki_ld, int64_t ki_bstride, const float* w, const float* bias,
                       float scale, const float* shift, float* scores, int64_t scores_ld, double* row_stats,
                       gsa_stream_t stream) {
  return indexer_scores_impl(dims, dtype, B, Lq, Lkv, q_pos0, causal, write_masked, qI, qi_ld, qi_bstride, kI,
                             ki_ld, ki_bstride, w, bias, scale, shift, scores, scores_ld, row_stats, nullptr,
                             stream);
}

int gsa_row_stats(int64_t R, int64_t n_cols, const float* scores, int64_t scores_ld, double* row_stats,
                  gsa_stream_t stream) {
  if (R < 0 || n_cols < 0 || scores_ld < n_cols) return GSA_ERR_BAD_ARG;
  if (R == 0) return GSA_OK;
  if (!scores || !row_stats) return GSA_ERR_BAD_ARG;
  return launch_row_stats(R, n_cols, scores, scores_ld, row_stats, reinterpret_cast<cudaStream_t>(stream));
}

int gsa_row_summary(int64_t R, int64_t n_cols, const float* scores, int64_t scores_ld, int dtype, float* out,
                    gsa_stream_t stream) {
  if (R < 0 || n_cols < 1 || scores_ld < n_cols || R > 0x7fffffffLL) return GSA_ERR_BAD_ARG;
  if (dtype != GSA_DTYPE_F32 && dtype != GSA_DTYPE_BF16) return GSA_ERR_BAD_ARG;
  if (R == 0) return GSA_OK;
  if (!scores || !out) return GSA_ERR_BAD_ARG;
  return launch_row_summary(R, n_cols, scores, scores_ld, dtype, out, reinterpret_cast<cudaStream_t>(stream));
}

int gsa_topk_candidates(int64_t R, int64_t Lq, int64_t n_cols, int64_t q_pos0, int causal, const float* scores,
                        int64_t scores_ld, const float* row_center, const double* row_stats, int32_t k_eff,
                        int32_t* cand_idx, float* cand_score, int32_t* cand_count, gsa_stream_t stream) {
  if (R < 0 || Lq <= 0 || n_cols < 0 || k_eff < 1 || scores_ld < n_cols || n_cols > 0x7fffffffLL)
    return GSA_ERR_BAD_ARG;
  if (R == 0) return GSA_OK;
  if (!scores || !cand_idx || !cand_score || !cand_count) return GSA_ERR_BAD_ARG;
  return launch_topk_candidates(R, Lq, n_cols, q_pos0, causal, scores, scores_ld, row_center, row_stats, k_eff,
                                cand_idx, cand_score, cand_count, reinterpret_cast<cudaStream_t>(stream));
}

int gsa_row_variance(int64_t R, int64_t n_cols, int dtype, const double* row_stats, const float* shift,
                     float* var_out, double* var_total, gsa_stream_t stream) {
  if (R < 0 || n_cols < 0 || (dtype != GSA_DTYPE_F32 && dtype != GSA_DTYPE_BF16)) return GSA_ERR_BAD_ARG;
  if (!var_total) return GSA_ERR_BAD_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (R == 0) {
    return cudaMemsetAsync(var_total, 0, 2 * sizeof(double), s) == cudaSuccess ? GSA_OK : GSA_ERR_CUDA;
  }
  if (!row_stats || !var_out) return GSA_ERR_BAD_ARG;
  return launch_row_variance(R, n_cols, dtype, row_stats, shift, var_out, var_total, s);
}

int gsa_adaptive_k(int64_t R, int64_t n_cols, int dtype, const gsa_topk_params* p, const float* var,
                   const double* var_total, const double* row_stats, int32_t* k_out, gsa_stream_t stream) {
  if (R < 0 || n_cols < 0 || !p || (dtype != GSA_DTYPE_F32 && dtype != GSA_DTYPE_BF16)) return GSA_ERR_BAD_ARG;
  if (R == 0) return GSA_OK;
  if (!k_out || (p->use_adaptive && (!var || !var_total || !row_stats))) return GSA_ERR_BAD_ARG;
  return launch_adaptive_k(R, n_cols, dtype, *p, var, var_total, row_stats, k_out,
                           reinterpret_cast<cudaStream_t>(stream));
}

int gsa_select_finalize(int64_t R, int32_t k_eff, const int32_t* cand_idx, const float* cand_score,
                        const int32_t* cand_count, const int32_t* k, int32_t* sel_idx, int64_t sel_ld,
                        int32_t* sel_count, uint8_t* sel_mask, gsa_stream_t stream) {
  if (R < 0 || k_eff < 1 || sel_ld < 1) return GSA_ERR_BAD_ARG;
  if (R == 0) return GSA_OK;
  if (!cand_idx || !cand_score || !cand_count || !k || !sel_idx || !sel_count) return GSA_ERR_BAD_ARG;
  if (!sel_mask) {
    // one warp per row when the rows fill the GPU; few rows (decode) take a CTA each, since a
    // row's passes over its candidates are latency-bound on one warp (the selection mask needs
    // the per-row CTA kernel as well)
    DeviceInfo dinfo, *di = &dinfo;
    int st = device_info(di);
    if (st) return st;
    if (R >= 2LL * di->num_sms)
      return launch_select_finalize_warp(R, k_eff, cand_idx, cand_score, cand_count, k, sel_idx, sel_ld, sel_count,
                                         di->num_sms, reinterpret_cast<cudaStream_t>(stream));
  }
  return launch_select_finalize(R, k_eff, cand_idx, cand_score, cand_count, k, sel_idx, sel_ld, sel_count,
                                sel_mask, reinterpret_cast<cudaStream_t>(stream));
}

int gsa_apply_gate(int dtype, int act, int64_t n, const void* x, const void* logits, void* out, void* gate_out,
                   gsa_stream_t stream) {
  if (n < 0 || (dtype != GSA_DTYPE_F32 && dtype != GSA_DTYPE_BF16)) return GSA_ERR_BAD_ARG;
  if (act < GSA_ACT_SIGMOID || act > GSA_ACT_SILU) return GSA_ERR_UNSUPPORTED;
  if (n == 0) return GSA_OK;
  if (!x || !logits || !out) return GSA_ERR_BAD_ARG;
  return launch_apply_gate(dtype, act, n, x, logits, out, gate_out, reinterpret_cast<cudaStream_t>(stream));
}

int gsa_sparse_sdpa(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv, const void* q,
                    const void* k, const void* v, int64_t kv_ld, const int32_t* sel_idx, int64_t sel_ld,
                    const int32_t* sel_count, const void* gate, void* out, float scale, gsa_stream_t stream) {
  return gsa_sparse_sdpa_strided(dims, dtype, B, Lq, Lkv, q, k, v, kv_ld, Lkv * kv_ld, sel_idx, sel_ld, sel_count,
                                 gate, out, scale, nullptr, 0, stream);
}

int64_t gsa_sdpa_workspace_size(const gsa_dims* dims, int64_t B, int64_t Lq) {
  if (!dims_ok(dims) || B <= 0 || Lq <= 0) return 0;
  DeviceInfo dinfo, *di = &dinfo;
  if (device_info(di)) return 0;
  // room for the most key ranges the launch may choose (one per resident CTA, at most 8 per
  // row; at most two resident CTAs per SM)
  const int64_t R = B * Lq, slots = 2LL * di->num_sms;
  if (R >= slots) return 0;
  const int64_t splits = std::min<int64_t>(slots / R, 8);
  if (splits < 2) return 0;
  return R * splits * (int64_t)dims->n_heads * (dims->d_head + 1) * (int64_t)sizeof(float);
}

}  // extern "C"

static int sdpa_impl(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv, const void* q, const void* k,
                     const void* v, int64_t kv_ld, int64_t kv_bstride, const int32_t* sel_idx, int64_t sel_ld,
                     const int32_t* sel_count, const void* gate, void* out, float scale, void* workspace,
                     int64_t workspace_bytes, float* lse_out, gsa_stream_t stream) {
  if (!dims_ok(dims) || B < 0 || Lq < 0 || Lkv < 0 || sel_ld < 0) return GSA_ERR_BAD_ARG;
  if (B * Lq == 0) return GSA_OK;
  if (!q || !k || !v || !sel_idx || !sel_count || !out) return GSA_ERR_BAD_ARG;
  const int64_t row_elems = (int64_t)dims->n_kv_heads * dims->d_head;
  if (kv_ld < row_elems || kv_bstride < Lkv * kv_ld) return GSA_ERR_BAD_ARG;
  DeviceInfo dinfo, *di = &dinfo;
  int st = device_info(di);
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype == GSA_DTYPE_BF16) {
    if (!aligned(k, 16) || !aligned(v, 16) || !aligned(q, 4) || (kv_ld * 2) % 16 != 0 || (kv_bstride * 2) % 16 != 0)
      return GSA_ERR_BAD_ARG;
    const bool inter = kv_ld == 2 * row_elems &&
                       static_cast<const __nv_bfloat16*>(v) == static_cast<const __nv_bfloat16*>(k) + row_elems;
    SdpaArgs a{B, Lq, Lkv, dims->n_kv_heads,
               static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
               static_cast<const __nv_bfloat16*>(v), kv_ld, inter ? 1 : 0, sel_idx, sel_ld, sel_count,
               static_cast<const __nv_bfloat16*>(gate), static_cast<__nv_bfloat16*>(out),
               scale * 1.4426950408889634f, 0, 2, di->err, kv_bstride, 1,
               (workspace && aligned(workspace, 16)) ? static_cast<float*>(workspace) : nullptr,
               workspace ? workspace_bytes / (int64_t)sizeof(float) : 0, 0, lse_out};
    return launch_sdpa_bf16(a, dims->d_head, dims->n_heads / dims->n_kv_heads, di->num_sms, s);
  }
  if (dtype == GSA_DTYPE_F32) {
    SdpaF32Args a{B, Lq, Lkv, dims->n_heads, dims->n_kv_heads, dims->d_head,
                  static_cast<const float*>(q), static_cast<const float*>(k), static_cast<const float*>(v),
                  kv_ld, sel_idx, sel_ld, sel_count, static_cast<const float*>(gate), static_cast<float*>(out),
                  scale, di->err, kv_bstride, lse_out};
    return launch_sdpa_f32(a, s);
  }
  return GSA_ERR_BAD_ARG;
}

extern "C" {

int gsa_sparse_sdpa_strided(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv, const void* q,
                            const void* k, const void* v, int64_t kv_ld, int64_t kv_bstride, const int32_t* sel_idx,
                            int64_t sel_ld, const int32_t* sel_count, const void* gate, void* out, float scale,
                            void* workspace, int64_t workspace_bytes, gsa_stream_t stream) {
  return sdpa_impl(dims, dtype, B, Lq, Lkv, q, k, v, kv_ld, kv_bstride, sel_idx, sel_ld, sel_count, gate, out, scale,
                   workspace, workspace_bytes, nullptr, stream);
}

int gsa_sparse_sdpa_lse(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv, const void* q,
                        const void* k, const void* v, int64_t kv_ld, int64_t kv_bstride, const int32_t* sel_idx,
                        int64_t sel_ld, const int32_t* sel_count, const void* gate, void* out, float* lse_out,
                        float scale, gsa_stream_t stream) {
  if (!lse_out) return GSA_ERR_BAD_ARG;
  return sdpa_impl(dims, dtype, B, Lq, Lkv, q, k, v, kv_ld, kv_bstride, sel_idx, sel_ld, sel_count, gate, out, scale,
                   nullptr, 0, lse_out, stream);
}

int gsa_sparse_sdpa_backward(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv, const void* q,
                             const void* k, const void* v, int64_t kv_ld, int64_t kv_bstride, const int32_t* sel_idx,
                             int64_t sel_ld, const int32_t* sel_count, const void* o, const void* d_o,
                             const float* lse, float* dq, float* dk, float* dv, int64_t dkv_ld, int64_t dkv_bstride,
                             float scale, gsa_stream_t stream) {
  if (!dims_ok(dims) || B < 0 || Lq < 0 || Lkv < 0 || sel_ld < 0 || (dtype != GSA_DTYPE_F32 && dtype != GSA_DTYPE_BF16))
    return GSA_ERR_BAD_ARG;
  if (B * Lq == 0) return GSA_OK;
  if (!q || !k || !v || !sel_idx || !sel_count || !o || !d_o || !lse || !dq || !dk || !dv) return GSA_ERR_BAD_ARG;
  const int64_t row_elems = (int64_t)dims->n_kv_heads * dims->d_head;
  if (kv_ld < row_elems || kv_bstride < Lkv * kv_ld || dkv_ld < row_elems || dkv_bstride < Lkv * dkv_ld)
    return GSA_ERR_BAD_ARG;
  const size_t esz = dtype == GSA_DTYPE_BF16 ? 2 : 4;
  // vector loads of a lane's D/32 consecutive elements, vector atomics into dk / dv
  if (!aligned(q, 16) || !aligned(k, 8) || !aligned(v, 8) || !aligned(o, 8) || !aligned(d_o, 8) || !aligned(dk, 16) ||
      !aligned(dv, 16) || !aligned(dq, 16) || (kv_ld * esz) % 8 || (kv_bstride * esz) % 8 || dkv_ld % 4 ||
      dkv_bstride % 4)
    return GSA_ERR_BAD_ARG;
  DeviceInfo dinfo, *di = &dinfo;
  int st = device_info(di);
  if (st) return st;
  SdpaBwdArgs a{B, Lq, Lkv, dims->n_heads, dims->n_kv_heads, dims->d_head, dtype, q, k, v, kv_ld, kv_bstride,
                sel_idx, sel_ld, sel_count, o, d_o, lse, dq, dk, dv, dkv_ld, dkv_bstride, scale, di->err};
  return launch_sdpa_backward(a, reinterpret_cast<cudaStream_t>(stream));
}

int gsa_sparse_sdpa_probs(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv, const void* q,
                          const void* k, int64_t kv_ld, int64_t kv_bstride, const int32_t* idx, const uint8_t* mask,
                          int64_t idx_ld, int64_t k_eff, const float* lse, float scale, void* probs,
                          gsa_stream_t stream) {
  if (!dims_ok(dims) || B < 0 || Lq < 0 || Lkv < 0 || k_eff < 0 || idx_ld < k_eff ||
      (dtype != GSA_DTYPE_F32 && dtype != GSA_DTYPE_BF16))
    return GSA_ERR_BAD_ARG;
  if (B * Lq == 0 || k_eff == 0) return GSA_OK;
  if (!q || !k || !idx || !lse || !probs || B * Lq > 65535) return GSA_ERR_BAD_ARG;
  const int64_t row_elems = (int64_t)dims->n_kv_heads * dims->d_head;
  if (kv_ld < row_elems || kv_bstride < Lkv * kv_ld) return GSA_ERR_BAD_ARG;
  DeviceInfo dinfo, *di = &dinfo;
  int st = device_info(di);
  if (st) return st;
  SdpaProbsArgs a{B, Lq, Lkv, dims->n_heads, dims->n_kv_heads, dims->d_head, q, k, kv_ld, kv_bstride,
                  idx, mask, idx_ld, k_eff, lse, scale, probs, di->err};
  return launch_sdpa_probs(a, dtype, reinterpret_cast<cudaStream_t>(stream));
}

int gsa_selftest_bounded_wait(uint32_t wait_limit, gsa_stream_t stream) {
  if (wait_limit == 0) return GSA_ERR_BAD_ARG;
  DeviceInfo dinfo, *di = &dinfo;
  int st = device_info(di);
  if (st) return st;
  return launch_wait_selftest(wait_limit, di->err, reinterpret_cast<cudaStream_t>(stream));
}

int gsa_add_rmsnorm(int dtype, int64_t T, int64_t d, const void* x, int64_t x_ld, const void* a, int64_t a_ld,
                    const void* weight, float eps, void* h_out, int64_t h_ld, void* y_out, int64_t y_ld,
                    gsa_stream_t stream) {
  if (T < 0 || d < 1 || (dtype != GSA_DTYPE_F32 && dtype != GSA_DTYPE_BF16)) return GSA_ERR_BAD_ARG;
  if (T == 0) return GSA_OK;
  if (!x || x_ld < d || (a && a_ld < d) || (h_out && (!a || h_ld < d)) || (y_out && (!weight || y_ld < d)) ||
      (!h_out && !y_out))
    return GSA_ERR_BAD_ARG;
  return launch_add_rmsnorm(dtype, T, d, x, x_ld, a, a_ld, weight, eps, h_out, h_ld, y_out, y_ld,
                            reinterpret_cast<cudaStream_t>(stream));
}

int gsa_silu_mul(int dtype, int64_t T, int64_t n, const void* gu, int64_t gu_ld, void* z, int64_t z_ld,
                 gsa_stream_t stream) {
  if (T < 0 || n < 0 || (dtype != GSA_DTYPE_F32 && dtype != GSA_DTYPE_BF16)) return GSA_ERR_BAD_ARG;
  if (T * n == 0) return GSA_OK;
  if (!gu || !z || gu_ld < 2 * n || z_ld < n) return GSA_ERR_BAD_ARG;
  return launch_silu_mul(dtype, T, n, gu, gu_ld, z, z_ld, reinterpret_cast<cudaStream_t>(stream));
}

int64_t gsa_workspace_size(int64_t chunk_rows, int64_t n_cols) {
  if (chunk_rows <= 0 || n_cols <= 0) return 0;
  const int64_t ld = (n_cols + 3) / 4 * 4;
  return chunk_rows * ld * (int64_t)sizeof(float);
}

int gsa_indexer_select(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv, int64_t q_pos0,
                       int causal, const void* qI, int64_t qi_ld, int64_t qi_bstride, const void* kI,
                       int64_t ki_ld, int64_t ki_bstride, const float* w, const float* bias, float scale,
                       const float* shift, int32_t k_eff, int32_t* cand_idx, float* cand_score,
                       int32_t* cand_count, double* row_stats, int64_t chunk_rows, void* workspace,
                       int64_t workspace_bytes, gsa_stream_t stream) {
  if (!dims_ok(dims) || B < 0 || Lq < 0 || Lkv < 0 || chunk_rows <= 0 || k_eff < 1) return GSA_ERR_BAD_ARG;
  if (B * Lq == 0 || Lkv == 0) return GSA_OK;
  if (workspace_bytes < gsa_workspace_size(chunk_rows, Lkv) || !workspace) return GSA_ERR_WORKSPACE;
  if (!aligned(workspace, 16)) return GSA_ERR_BAD_ARG;
  const int64_t ld = (Lkv + 3) / 4 * 4;
  float* scratch = static_cast<float*>(workspace);
  const size_t esz = dtype == GSA_DTYPE_BF16 ? 2 : 4;
  const int HI = dims->n_idx_heads;
  for (ChunkIter c(B, Lq, chunk_rows); c.next();) {
    const int64_t r0 = c.b0 * Lq + c.t0, n = c.nb * c.n;
    const void* q_ptr = static_cast<const char*>(qI) + (c.b0 * qi_bstride + c.t0 * qi_ld) * (int64_t)esz;
    const void* k_ptr = static_cast<const char*>(kI) + (c.b0 * ki_bstride) * (int64_t)esz;
    int st = gsa_indexer_scores(dims, dtype, c.nb, c.n, Lkv, q_pos0 + c.t0, causal, 0, q_ptr, qi_ld, qi_bstride,
                                k_ptr, ki_ld, ki_bstride, w + r0 * HI, bias, scale, shift ? shift + r0 : nullptr,
                                scratch, ld, row_stats ? row_stats + r0 * 3 : nullptr, stream);
    if (st) return st;
    // sigmoid scores of row r lie in [0, sum_j w_rj] = [0, 2 shift_r]: the bounded-range selection
    const float* center = (shift && dims->idx_act == GSA_ACT_SIGMOID) ? shift + r0 : nullptr;
    st = gsa_topk_candidates(n, c.n, Lkv, q_pos0 + c.t0, causal, scratch, ld, center,
                             (center && row_stats) ? row_stats + r0 * 3 : nullptr, k_eff,
                             cand_idx + r0 * k_eff, cand_score + r0 * k_eff, cand_count + r0, stream);
    if (st) return st;
  }
  return GSA_OK;
}

static int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

int64_t gsa_survivors_workspace_size(int64_t chunk_rows, int64_t n_cols) {
  if (chunk_rows <= 0 || n_cols <= 0) return 0;
  // score scratch, failed-row list, its count, per-row segment counts (few-row compaction), the
  // indexer's per-key-range statistic partials
  return align256(gsa_workspace_size(chunk_rows, n_cols)) + align256(chunk_rows * 4) + 256 +
         align256(chunk_rows * 16 * 4) + align256(chunk_rows * indexer_tc_stat_ranges(n_cols) * 3 * 8);
}

int gsa_indexer_survivors(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv, int64_t q_pos0,
                          int causal, const void* qI, int64_t qi_ld, int64_t qi_bstride, const void* kI,
                          int64_t ki_ld, int64_t ki_bstride, const float* w, const float* bias, float scale,
                          const float* shift, int32_t k_eff, int32_t cap, int32_t* cand_idx, float* cand_score,
                          int32_t* cand_count, double* row_stats, int64_t chunk_rows, void* workspace,
                          int64_t workspace_bytes, gsa_stream_t stream) {
  if (!dims_ok(dims) || B < 0 || Lq < 0 || Lkv < 0 || chunk_rows <= 0 || k_eff < 1 || cap < k_eff)
    return GSA_ERR_BAD_ARG;
  if (B * Lq == 0 || Lkv == 0) return GSA_OK;
  if (!shift || !row_stats || !cand_idx || !cand_score || !cand_count || !w || !bias || !qI || !kI)
    return GSA_ERR_BAD_ARG;
  // sigmoid scores (the threshold statistics are relative to the row centre) and room above
  // the 1.5 k_eff survivors the threshold aims at
  if (dims->idx_act != GSA_ACT_SIGMOID || 2 * (int64_t)cap < 3 * (int64_t)k_eff + 2048) return GSA_ERR_UNSUPPORTED;
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < gsa_survivors_workspace_size(chunk_rows, Lkv))
    return GSA_ERR_WORKSPACE;
  DeviceInfo dinfo, *di = &dinfo;
  int st = device_info(di);
  if (st) return st;
  const int64_t ld = (Lkv + 3) / 4 * 4;
  uint8_t* wsb = static_cast<uint8_t*>(workspace);
  float* scratch = reinterpret_cast<float*>(wsb);
  int32_t* fail_list = reinterpret_cast<int32_t*>(wsb + align256(gsa_workspace_size(chunk_rows, Lkv)));
  int32_t* fail_count = fail_list + align256(chunk_rows * 4) / 4;
  int32_t* seg_count = fail_count + 256 / 4;
  double* stat_part = reinterpret_cast<double*>(reinterpret_cast<uint8_t*>(seg_count) + align256(chunk_rows * 16 * 4));
  const size_t esz = dtype == GSA_DTYPE_BF16 ? 2 : 4;
  const int HI = dims->n_idx_heads;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (ChunkIter c(B, Lq, chunk_rows); c.next();) {
    const int64_t r0 = c.b0 * Lq + c.t0, n = c.nb * c.n;
    const void* q_ptr = static_cast<const char*>(qI) + (c.b0 * qi_bstride + c.t0 * qi_ld) * (int64_t)esz;
    const void* k_ptr = static_cast<const char*>(kI) + (c.b0 * ki_bstride) * (int64_t)esz;
    st = indexer_scores_impl(dims, dtype, c.nb, c.n, Lkv, q_pos0 + c.t0, causal, 0, q_ptr, qi_ld, qi_bstride, k_ptr,
                             ki_ld, ki_bstride, w + r0 * HI, bias, scale, shift + r0, scratch, ld,
                             row_stats + r0 * 3, stat_part, stream);
    if (st) return st;
    st = launch_threshold_candidates(n, c.n, Lkv, q_pos0 + c.t0, causal, scratch, ld, shift + r0, row_stats + r0 * 3,
                                     k_eff, cap, cand_idx + r0 * cap, cand_score + r0 * cap, cand_count + r0,
                                     fail_list, fail_count, seg_count, di->num_sms, di->err, s);
    if (st) return st;
  }
  return GSA_OK;
}

// ---- the fused survivor pass ----
static gsa::SurvivorShape survivor_shape(int32_t k_eff, int32_t cap) {
  gsa::SurvivorShape sv;
  sv.K = k_eff;
  sv.cap = cap;
  sv.K14 = (int32_t)((14LL * k_eff + 9) / 10);
  return sv;
}

// Entries of a row's segment area for rows of n_lo..n_hi keys: the most any of them needs.
static int64_t survivor_stride(const gsa::SurvivorShape& sv, int64_t n_lo, int64_t n_hi) {
  using gsa::SurvivorShape;
  int64_t best = 0;
  if (n_lo < 1) n_lo = 1;
  for (int64_t b = SurvivorShape::ranges(n_lo); b <= SurvivorShape::ranges(n_hi); ++b) {
    // seg_cap falls with n inside a block of equal range counts: its first n holds the block's most
    const int64_t n = std::max<int64_t>(n_lo, (b - 1) * SurvivorShape::kRangeKeys + 1);
    if (n > n_hi) break;
    best = std::max<int64_t>(best, b * sv.seg_cap(n));
  }
  return best;
}

int64_t gsa_survivors_fused_workspace_size(int64_t chunk_rows, int64_t n_cols, int32_t k_eff, int32_t cap) {
  if (chunk_rows <= 0 || n_cols <= 0 || k_eff < 1 || cap < k_eff) return 0;
  const gsa::SurvivorShape sv = survivor_shape(k_eff, cap);
  const int64_t stride = survivor_stride(sv, 1, n_cols);
  // the materialised pass's workspace (its scratch takes the recomputed blocks), the sampled
  // statistics, the segment counts, the segments' columns and scores, the failed-block flags
  return gsa_survivors_workspace_size(chunk_rows, n_cols) + align256(chunk_rows * 3 * 8) +
         align256(chunk_rows * indexer_tc_stat_ranges(n_cols) * 4) + 2 * align256(chunk_rows * stride * 4) +
         align256(chunk_rows * 4 + 4);
}

int gsa_indexer_survivors_fused(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv, int64_t q_pos0,
                                int causal, const void* qI, int64_t qi_ld, int64_t qi_bstride, const void* kI,
                                int64_t ki_ld, int64_t ki_bstride, const float* w, const float* bias, float scale,
                                const float* shift, int32_t k_eff, int32_t cap, int32_t* cand_idx,
                                float* cand_score, int32_t* cand_count, double* row_stats, int64_t chunk_rows,
                                void* workspace, int64_t workspace_bytes, gsa_stream_t stream) {
  if (!dims_ok(dims) || B < 0 || Lq < 0 || Lkv < 0 || chunk_rows <= 0 || k_eff < 1 || cap < k_eff)
    return GSA_ERR_BAD_ARG;
  if (B * Lq == 0 || Lkv == 0) return GSA_OK;
  if (!shift || !row_stats || !cand_idx || !cand_score || !cand_count || !w || !bias || !qI || !kI)
    return GSA_ERR_BAD_ARG;
  if (dims->idx_act != GSA_ACT_SIGMOID || 2 * (int64_t)cap < 3 * (int64_t)k_eff + 2048 || dims->n_idx_heads != 8)
    return GSA_ERR_UNSUPPORTED;
  if (!workspace || !aligned(workspace, 256) ||
      workspace_bytes < gsa_survivors_fused_workspace_size(chunk_rows, Lkv, k_eff, cap))
    return GSA_ERR_WORKSPACE;
  {
    IdxArgs probe{dtype, Lq, Lkv, q_pos0, causal, 0, dims->n_idx_heads, dims->d_idx, dims->idx_act,
                  qI, qi_ld, qi_bstride, kI, ki_ld, ki_bstride, w, bias, scale, shift, nullptr, 0, row_stats};
    if (!indexer_tc_eligible(probe)) return GSA_ERR_UNSUPPORTED;
  }
  DeviceInfo dinfo, *di = &dinfo;
  int st = device_info(di);
  if (st) return st;
  const gsa::SurvivorShape sv = survivor_shape(k_eff, cap);
  const int64_t stride = survivor_stride(sv, 1, Lkv);
  const int64_t n_ranges = indexer_tc_stat_ranges(Lkv);
  const int64_t ld = (Lkv + 3) / 4 * 4;
  uint8_t* wsb = static_cast<uint8_t*>(workspace);
  float* scratch = reinterpret_cast<float*>(wsb);
  int32_t* fail_list = reinterpret_cast<int32_t*>(wsb + align256(gsa_workspace_size(chunk_rows, Lkv)));
  int32_t* fail_count = fail_list + align256(chunk_rows * 4) / 4;
  int32_t* seg_count = fail_count + 256 / 4;
  double* stat_part = reinterpret_cast<double*>(reinterpret_cast<uint8_t*>(seg_count) + align256(chunk_rows * 16 * 4));
  uint8_t* tail = wsb + gsa_survivors_workspace_size(chunk_rows, Lkv);
  double* samp = reinterpret_cast<double*>(tail);
  tail += align256(chunk_rows * 3 * 8);
  int32_t* seg_cnt = reinterpret_cast<int32_t*>(tail);
  tail += align256(chunk_rows * n_ranges * 4);
  int32_t* seg_idx = reinterpret_cast<int32_t*>(tail);
  tail += align256(chunk_rows * stride * 4);
  float* seg_score = reinterpret_cast<float*>(tail);
  tail += align256(chunk_rows * stride * 4);
  int32_t* blk_flag = reinterpret_cast<int32_t*>(tail);
  const int HI = dims->n_idx_heads;
  const int32_t blk_rows = gsa::kTcQueryBlock8;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (ChunkIter c(B, Lq, chunk_rows); c.next();) {
    const int64_t r0 = c.b0 * Lq + c.t0, n = c.nb * c.n;
    const int64_t blks = (c.n + blk_rows - 1) / blk_rows;
    if (cudaMemsetAsync(samp, 0, (size_t)n * 3 * sizeof(double), s) != cudaSuccess ||
        cudaMemsetAsync(blk_flag, 0, (size_t)(c.nb * blks + 1) * sizeof(int32_t), s) != cudaSuccess ||
        cudaMemsetAsync(fail_count, 0, sizeof(int32_t), s) != cudaSuccess)
      return GSA_ERR_CUDA;
    for (int pass = 0; pass < 3; ++pass) {
      // 0: sampled statistics; 1: statistics + survivors; 2: scores of the failed rows' blocks
      for (int64_t b = 0; b < c.nb; ++b) {
        const int64_t rb = r0 + b * c.n;  // first row of this sequence's slice, over all rows
        const int64_t lb = b * c.n;       // the same, within the chunk
        const void* q_ptr = static_cast<const __nv_bfloat16*>(qI) + (c.b0 + b) * qi_bstride + c.t0 * qi_ld;
        const void* k_ptr = static_cast<const __nv_bfloat16*>(kI) + (c.b0 + b) * ki_bstride;
        IdxArgs a{dtype, c.n, Lkv, q_pos0 + c.t0, causal, 0, HI, dims->d_idx, dims->idx_act, q_ptr, qi_ld, qi_bstride,
                  k_ptr, ki_ld, ki_bstride, w + rb * HI, bias, scale, shift + rb, nullptr, ld, nullptr};
        gsa::TcSurvivorArgs x;
        int mode;
        if (pass == 0) {
          mode = gsa::kTcSample;
          a.row_stats = samp + lb * 3;
        } else if (pass == 1) {
          mode = gsa::kTcEmit;
          a.row_stats = row_stats + rb * 3;
          a.stat_part = stat_part;
          x.samp_stats = samp + lb * 3;
          x.seg_idx = seg_idx + lb * stride;
          x.seg_score = seg_score + lb * stride;
          x.seg_cnt = seg_cnt + lb * n_ranges;
          x.seg_stride = stride;
          x.sv = sv;
        } else {
          mode = gsa::kTcScores;
          a.scores = scratch + lb * ld;
          x.blk_mask = blk_flag + b * blks;
        }
        st = launch_indexer_tc_mode(a, mode, x, di->err, s);
        if (st) return st;
      }
      if (pass == 1) {
        st = launch_seg_concat(n, c.n, Lkv, q_pos0 + c.t0, causal, sv, seg_idx, seg_score, seg_cnt, stride, n_ranges,
                               cand_idx + r0 * cap, cand_score + r0 * cap, cand_count + r0, fail_list, fail_count,
                               blk_flag, blk_rows, s);
        if (st) return st;
      }
    }
    st = launch_survivor_fallback(n, c.n, Lkv, q_pos0 + c.t0, causal, scratch, ld, shift + r0, row_stats + r0 * 3,
                                  k_eff, cap, cand_idx + r0 * cap, cand_score + r0 * cap, cand_count + r0, fail_list,
                                  fail_count, di->num_sms, di->err, s);
    if (st) return st;
  }
  return GSA_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// One decode step between the two GEMMs
// ---------------------------------------------------------------------------------------------
namespace gsa {

constexpr int32_t kSurvivorCap = 8192;  // candidate row of the threshold-survivor pass

// Byte offsets of the scratch tensors of gsa_decode_attend inside its workspace.
struct DecodeLayout {
  int64_t q, g1, w, shift, stats, var, total, kt, cidx, cscore, ccount, idx_ws, idx_ws_bytes, sel, scount,
      sdpa_ws, sdpa_ws_bytes, bytes;
  int32_t k_eff, cand_ld;
  bool survivors;
};

static DecodeLayout decode_layout(const gsa_dims* d, const gsa_topk_params* tp, int dtype, int64_t B, int64_t L,
                                  int64_t n_keys) {
  DecodeLayout o;
  const int64_t R = B * L, H = d->n_heads, D = d->d_head, HI = d->n_idx_heads;
  const int64_t esz = dtype == GSA_DTYPE_BF16 ? 2 : 4;
  int64_t k_eff = std::min<int64_t>(tp->use_adaptive ? tp->k_max : tp->k_base, n_keys);
  if (k_eff < 1) k_eff = 1;
  o.k_eff = (int32_t)k_eff;
  o.survivors = d->idx_act == GSA_ACT_SIGMOID && 2LL * kSurvivorCap >= 3 * k_eff + 2048;
  o.cand_ld = o.survivors ? kSurvivorCap : o.k_eff;
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    const int64_t p = off;
    off += align256(bytes);
    return p;
  };
  o.q = take(R * H * D * esz);
  o.g1 = take(R * H * D * esz);
  o.w = take(R * HI * 4);
  o.shift = take(R * 4);
  o.stats = take(R * 3 * 8);
  o.var = take(R * 4);
  o.total = take(16);
  o.kt = take(R * 4);
  o.cidx = take(R * o.cand_ld * 4);
  o.cscore = take(R * o.cand_ld * 4);
  o.ccount = take(R * 4);
  o.idx_ws_bytes = o.survivors ? gsa_survivors_workspace_size(R, n_keys) : gsa_workspace_size(R, n_keys);
  o.idx_ws = take(o.idx_ws_bytes);
  o.sel = take(R * k_eff * 4);
  o.scount = take(R * 4);
  o.sdpa_ws_bytes = dtype == GSA_DTYPE_BF16 ? gsa_sdpa_workspace_size(d, B, L) : 0;
  o.sdpa_ws = take(o.sdpa_ws_bytes);
  o.bytes = off;
  return o;
}

}  // namespace gsa

extern "C" {

int64_t gsa_decode_workspace_size(const gsa_dims* dims, const gsa_topk_params* tp, int dtype, int64_t B, int64_t L,
                                  int64_t n_keys) {
  if (!dims_ok(dims) || !tp || B <= 0 || L <= 0 || n_keys < L || (dtype != GSA_DTYPE_F32 && dtype != GSA_DTYPE_BF16))
    return 0;
  return decode_layout(dims, tp, dtype, B, L, n_keys).bytes;
}

int gsa_decode_attend(const gsa_dims* dims, const gsa_proj_layout* layout, const gsa_topk_params* tp, int dtype,
                      int64_t B, int64_t L, int64_t past, const void* proj, int64_t proj_ld,
                      const int64_t* positions, const void* cos_tab, const void* sin_tab, int tab_dtype,
                      int64_t tab_rows, void* kv_store, int64_t kv_bstride, void* ki_store, int64_t ki_bstride,
                      const float* idx_bias, float idx_scale, float attn_scale, void* attn_out, int32_t* k_out,
                      double* var_total, int phase, void* workspace, int64_t workspace_bytes, gsa_stream_t stream) {
  if (!dims_ok(dims) || !layout || !tp || B < 0 || L < 0 || past < 0 ||
      (dtype != GSA_DTYPE_F32 && dtype != GSA_DTYPE_BF16) || (tab_dtype != GSA_DTYPE_F32 && tab_dtype != GSA_DTYPE_BF16))
    return GSA_ERR_BAD_ARG;
  if (phase < GSA_DECODE_ALL || phase > GSA_DECODE_ATTEND || (phase != GSA_DECODE_ALL && !var_total))
    return GSA_ERR_BAD_ARG;
  if (B * L == 0) return GSA_OK;
  if (!proj || !cos_tab || !sin_tab || !kv_store || !ki_store || !idx_bias || !attn_out || tab_rows <= 0 ||
      layout->q < 0 || layout->k < 0 || layout->v < 0 || layout->qi < 0 || layout->ki < 0 || layout->wi < 0)
    return GSA_ERR_BAD_ARG;
  if (dims->gate_act < GSA_ACT_SIGMOID || dims->gate_act > GSA_ACT_SILU) return GSA_ERR_UNSUPPORTED;
  const int64_t R = B * L, n = past + L;
  const int64_t row = (int64_t)dims->n_kv_heads * dims->d_head, kv_ld = 2 * row, dI = dims->d_idx;
  if (kv_bstride < n * kv_ld || ki_bstride < n * dI) return GSA_ERR_BAD_ARG;
  const DecodeLayout o = decode_layout(dims, tp, dtype, B, L, n);
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < o.bytes) return GSA_ERR_WORKSPACE;
  DeviceInfo dinfo, *di = &dinfo;
  int st = device_info(di);
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const size_t esz = dtype == GSA_DTYPE_BF16 ? 2 : 4;
  uint8_t* kvb = static_cast<uint8_t*>(kv_store);
  uint8_t* kib = static_cast<uint8_t*>(ki_store);
  void* q = ws + o.q;
  void* g1 = layout->g1 >= 0 ? ws + o.g1 : nullptr;
  float* w = reinterpret_cast<float*>(ws + o.w);
  float* shift = reinterpret_cast<float*>(ws + o.shift);
  double* stats = reinterpret_cast<double*>(ws + o.stats);
  float* var = reinterpret_cast<float*>(ws + o.var);
  double* total = var_total ? var_total : reinterpret_cast<double*>(ws + o.total);
  int32_t* kt = reinterpret_cast<int32_t*>(ws + o.kt);
  int32_t* cidx = reinterpret_cast<int32_t*>(ws + o.cidx);
  float* cscore = reinterpret_cast<float*>(ws + o.cscore);
  int32_t* ccount = reinterpret_cast<int32_t*>(ws + o.ccount);
  int32_t* sel = reinterpret_cast<int32_t*>(ws + o.sel);
  int32_t* scount = reinterpret_cast<int32_t*>(ws + o.scount);

  if (phase == GSA_DECODE_ATTEND) goto attend;
  {
  // 1. RoPE / gates / head weights; K, V and k^I of the new tokens into slots past .. past+L-1
  // (it also clears the indexer's row statistics)
  EpiArgs ea{*dims, *layout, dtype, R, proj, proj_ld, positions, cos_tab, sin_tab, tab_dtype, tab_rows,
             q, kvb + past * kv_ld * esz, kvb + (past * kv_ld + row) * esz, kv_ld, g1, w, shift, di->err, L,
             kv_bstride, kib + past * dI * esz, dI, ki_bstride, past, stats};
  if ((st = launch_proj_epilogue(ea, s))) return st;
  // 2. indexer over every cached key + the candidates of each row
  const void* qI = static_cast<const uint8_t*>(proj) + layout->qi * esz;
  if (o.survivors)
    st = gsa_indexer_survivors(dims, dtype, B, L, n, past, 1, qI, proj_ld, L * proj_ld, ki_store, dI, ki_bstride, w,
                               idx_bias, idx_scale, shift, o.k_eff, o.cand_ld, cidx, cscore, ccount, stats, R,
                               ws + o.idx_ws, o.idx_ws_bytes, stream);
  else
    st = gsa_indexer_select(dims, dtype, B, L, n, past, 1, qI, proj_ld, L * proj_ld, ki_store, dI, ki_bstride, w,
                            idx_bias, idx_scale, shift, o.k_eff, cidx, cscore, ccount, stats, R, ws + o.idx_ws,
                            o.idx_ws_bytes, stream);
  if (st) return st;
  // 3. per-row variances and their sum (all-reduced between the phases when the sequences of
  // the batch are spread over several GPUs); one call with the adaptive k for few rows
  if (phase == GSA_DECODE_ALL && tp->use_adaptive && R <= 1024) {
    if ((st = launch_variance_adaptive_k(R, n, dtype, *tp, stats, shift, var, total, kt, s))) return st;
    goto select;
  }
  if (tp->use_adaptive) {
    if ((st = gsa_row_variance(R, n, dtype, stats, shift, var, total, stream))) return st;
  } else if (var_total && cudaMemsetAsync(var_total, 0, 2 * sizeof(double), s) != cudaSuccess) {
    return GSA_ERR_CUDA;
  }
  if (phase == GSA_DECODE_SCORE) return GSA_OK;
  }
attend:
  // 4. adaptive k (variance mean over every row of the batch), final selection
  if ((st = gsa_adaptive_k(R, n, dtype, tp, var, total, stats, kt, stream))) return st;
select:
  if ((st = gsa_select_finalize(R, o.cand_ld, cidx, cscore, ccount, kt, sel, o.k_eff, scount, nullptr, stream)))
    return st;
  // 5. sparse SDPA with the G1 gate
  if ((st = gsa_sparse_sdpa_strided(dims, dtype, B, L, n, q, kv_store, kvb + row * esz, kv_ld, kv_bstride, sel,
                                    o.k_eff, scount, g1, attn_out, attn_scale, ws + o.sdpa_ws, o.sdpa_ws_bytes,
                                    stream)))
    return st;
  if (k_out && cudaMemcpyAsync(k_out, kt, R * sizeof(int32_t), cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return GSA_ERR_CUDA;
  return GSA_OK;
}

}  // extern "C"
