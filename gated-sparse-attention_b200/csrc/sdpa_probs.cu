// Attention probabilities of the sparse SDPA for analysis callers (output_attentions,
// gated_sparse_attention.py:268-285): p[r, h, j] = exp(scale * q[r, h] . k[idx[r, j]] - lse[r, h])
// for the candidates j a row keeps (mask), 0 elsewhere, with lse the row's natural-log sum-exp
// that gsa_sparse_sdpa_lse writes.  The SDPA kernel never forms p in memory; this pass re-reads
// each kept key once per row (small shapes only: the output is [R, H, k_eff]).
#include "kernels.cuh"

namespace gsa {
namespace {

constexpr int kProbsWarps = 8;

// One warp per (row, candidate): lanes split the head dimension; the H dot products of a key
// against the row's heads are reduced with shuffles.
template <typename T>
__global__ void __launch_bounds__(kProbsWarps * 32) sdpa_probs_kernel(SdpaProbsArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = blockIdx.y;
  const int64_t b = r / a.Lq;
  const T* q = static_cast<const T*>(a.q) + r * (int64_t)a.H * a.D;
  const T* kb = static_cast<const T*>(a.k) + b * a.kv_bstride;
  const int32_t* idx = a.idx + r * a.idx_ld;
  const uint8_t* mask = a.mask ? a.mask + r * a.idx_ld : nullptr;
  T* out = static_cast<T*>(a.out) + r * (int64_t)a.H * a.k_eff;
  const int nrep = a.H / a.Hk;
  for (int64_t j = (int64_t)blockIdx.x * kProbsWarps + warp; j < a.k_eff; j += (int64_t)gridDim.x * kProbsWarps) {
    const int32_t s = idx[j];
    bool keep = mask ? mask[j] != 0 : true;
    if (keep && (s < 0 || s >= a.Lkv)) {
      set_error(a.err, GSA_ERR_INDEX);
      keep = false;
    }
    for (int h = 0; h < a.H; ++h) {
      float p = 0.f;
      if (keep) {
        const T* kr = kb + (int64_t)s * a.kv_ld + (int64_t)(h / nrep) * a.D;
        const T* qh = q + (int64_t)h * a.D;
        float dot = 0.f;
        for (int d = lane; d < a.D; d += 32) dot = fmaf(to_float(qh[d]), to_float(kr[d]), dot);
        dot = warp_sum(dot);
        p = expf(dot * a.scale - a.lse[r * a.H + h]);
      }
      if (lane == 0) out[(int64_t)h * a.k_eff + j] = from_float<T>(p);
    }
  }
}

}  // namespace

int launch_sdpa_probs(const SdpaProbsArgs& a, int dtype, cudaStream_t stream) {
  const int64_t R = a.B * a.Lq;
  if (R > 65535) return GSA_ERR_BAD_ARG;
  const unsigned gx = (unsigned)std::min<int64_t>((a.k_eff + kProbsWarps - 1) / kProbsWarps, 1024);
  const dim3 grid(gx, (unsigned)R);
  if (dtype == GSA_DTYPE_BF16)
    sdpa_probs_kernel<__nv_bfloat16><<<grid, kProbsWarps * 32, 0, stream>>>(a);
  else
    sdpa_probs_kernel<float><<<grid, kProbsWarps * 32, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

}  // namespace gsa
