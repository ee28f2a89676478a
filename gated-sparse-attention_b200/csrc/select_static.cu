// gsa_indexer_select_static: the chunked indexer + top-k candidates with its score scratch in a
// fixed buffer that the library owns, so that the call allocates no device memory.
//
// Who needs it: callers that cannot hand the library a workspace and must not have it allocate
// one mid-step -- serving runtimes that reserve all HBM for their own pools up front, and host
// code (a C or Go caller of the ABI) that has no device allocator at hand.  The price is a
// bounded scratch: GSA_STATIC_SCRATCH_BYTES (64 MiB) per device, which caps one chunk at
// 64 MiB / (4 * round4(Lkv)) query rows and the key length at 16,777,216.
//
// The buffer is a file-scope __device__ array.  In host code its name only stands for the
// symbol; the kernels get the device address that cudaGetSymbolAddress returns in the calling
// thread's current context.  That address belongs to the context (a cudaDeviceReset, or a
// driver-API caller's own context on the same device, places the module elsewhere), so it is
// looked up on every call; once the module is loaded in a context the lookup is a table search.
// The first call in a context loads the module: make it before any stream capture.  Because every
// call on a device shares the one buffer, calls that overlap in time on the same device (two
// streams, two host threads) race on it: callers serialise them.
#include "kernels.cuh"

namespace gsa {

static_assert(GSA_STATIC_SCRATCH_BYTES % 256 == 0, "scratch size is a whole number of 256-byte blocks");

static __device__ __align__(256) float g_select_scratch[GSA_STATIC_SCRATCH_BYTES / sizeof(float)];

namespace {

// Device address of the scratch in the current context.
int static_scratch(float** out) {
  void* p = nullptr;
  const cudaError_t rc = cudaGetSymbolAddress(&p, g_select_scratch);
  if (rc != cudaSuccess || p == nullptr) {
    cudaGetLastError();  // clear the (non-sticky) error so the caller's next CUDA call is clean
    return GSA_ERR_CUDA;
  }
  *out = static_cast<float*>(p);
  return GSA_OK;
}

}  // namespace
}  // namespace gsa

using namespace gsa;

extern "C" int gsa_indexer_select_static(const gsa_dims* dims, int dtype, int64_t B, int64_t Lq, int64_t Lkv,
                                         int64_t q_pos0, int causal, const void* qI, int64_t qi_ld,
                                         int64_t qi_bstride, const void* kI, int64_t ki_ld, int64_t ki_bstride,
                                         const float* w, const float* bias, float scale, const float* shift,
                                         int32_t k_eff, int32_t* cand_idx, float* cand_score, int32_t* cand_count,
                                         double* row_stats, gsa_stream_t stream) {
  // every check gsa_indexer_select and its stages make, before this call writes anything
  if (!dims_ok(dims) || B < 0 || Lq < 0 || Lkv < 0 || k_eff < 1 ||
      (dtype != GSA_DTYPE_F32 && dtype != GSA_DTYPE_BF16))
    return GSA_ERR_BAD_ARG;
  if (B * Lq == 0 || Lkv == 0) return GSA_OK;
  if (!qI || !kI || !w || !bias || !cand_idx || !cand_score || !cand_count || Lkv > 0x7fffffffLL)
    return GSA_ERR_BAD_ARG;
  if (dims->idx_act != GSA_ACT_SIGMOID && dims->idx_act != GSA_ACT_RELU) return GSA_ERR_UNSUPPORTED;
  // one row of scores must fit; a chunk is as many rows as fit
  const int64_t row_bytes = gsa_workspace_size(1, Lkv);
  if (row_bytes <= 0 || row_bytes > (int64_t)GSA_STATIC_SCRATCH_BYTES) return GSA_ERR_WORKSPACE;
  int64_t chunk_rows = (int64_t)GSA_STATIC_SCRATCH_BYTES / row_bytes;
  if (chunk_rows > Lq) chunk_rows = Lq;
  float* scratch = nullptr;
  int st = static_scratch(&scratch);
  if (st) return st;
  // the row statistics are accumulated with atomics: they must start at zero
  if (row_stats &&
      cudaMemsetAsync(row_stats, 0, (size_t)(B * Lq) * 3 * sizeof(double),
                      reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess)
    return GSA_ERR_CUDA;
  return gsa_indexer_select(dims, dtype, B, Lq, Lkv, q_pos0, causal, qI, qi_ld, qi_bstride, kI, ki_ld, ki_bstride,
                            w, bias, scale, shift, k_eff, cand_idx, cand_score, cand_count, row_stats, chunk_rows,
                            scratch, (int64_t)GSA_STATIC_SCRATCH_BYTES, stream);
}
