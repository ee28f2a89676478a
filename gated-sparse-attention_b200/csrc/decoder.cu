// Decoder-layer elementwise kernels around the attention (gsa/models/gsa_llama.py):
//
//   RMSNorm          y = (x * rsqrt(mean(x^2) + eps)).type_as(x) * w          (gsa_llama.py:18-30)
//   residual + RMSNorm   h = residual + a;  y = RMSNorm(h)  (the two adds of GSADecoderLayer,
//                    gsa_llama.py:100-110, each followed by the next norm)
//   SwiGLU gate      z = silu(g) * u                                          (gsa_llama.py:45-46)
//
// Every op is evaluated as torch evaluates it for the tensor's dtype: the norm in fp32 from the
// (upcast) input, rounded to the dtype before the weight product; the add, silu and product each
// rounded to the dtype.  One CTA per row; bf16 rows move in 16-byte vectors.
#include "kernels.cuh"

namespace gsa {

namespace dec_layer {

constexpr int kThreads = 256;

__device__ __forceinline__ float ld_el(const void* p, int64_t i, int dtype) {
  return dtype == GSA_DTYPE_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i])
                                 : static_cast<const float*>(p)[i];
}
__device__ __forceinline__ void st_el(void* p, int64_t i, float v, int dtype) {
  if (dtype == GSA_DTYPE_BF16)
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else
    static_cast<float*>(p)[i] = v;
}
__device__ __forceinline__ float round_to(float v, int dtype) {
  return dtype == GSA_DTYPE_BF16 ? __bfloat162float(__float2bfloat16_rn(v)) : v;
}

// Block sum of one float per thread (kThreads threads).
__device__ __forceinline__ float block_sum(float v, float* ws) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) ws[wid] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) t += ws[w];
  return t;
}

// h = residual + a (if residual), y = RMSNorm(h or x) * w.  Rows of d elements, row strides ld.
__global__ void __launch_bounds__(kThreads) add_rmsnorm_kernel(int dtype, int64_t d, const void* x, int64_t x_ld,
                                                               const void* a, int64_t a_ld, const void* w,
                                                               float eps, void* h_out, int64_t h_ld, void* y_out,
                                                               int64_t y_ld) {
  __shared__ float ws[kThreads / 32];
  const int64_t r = blockIdx.x;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < d; i += kThreads) {
    float v = ld_el(x, r * x_ld + i, dtype);
    if (a) {
      v = round_to(v + ld_el(a, r * a_ld + i, dtype), dtype);
      if (h_out) st_el(h_out, r * h_ld + i, v, dtype);
    }
    ss = fmaf(v, v, ss);
  }
  const float mean = block_sum(ss, ws) / (float)d;
  const float inv = 1.0f / sqrtf(mean + eps);
  if (!y_out) return;
  for (int64_t i = threadIdx.x; i < d; i += kThreads) {
    float v = ld_el(x, r * x_ld + i, dtype);
    if (a) v = round_to(v + ld_el(a, r * a_ld + i, dtype), dtype);
    const float n = round_to(v * inv, dtype);
    st_el(y_out, r * y_ld + i, n * ld_el(w, i, dtype), dtype);
  }
}

// z = silu(g) * u with g, u the two halves of a row of gu (gu[r, 0:n] and gu[r, n:2n]).
__global__ void silu_mul_kernel(int dtype, int64_t T, int64_t n, const void* gu, int64_t gu_ld, void* z,
                                int64_t z_ld) {
  const int64_t total = T * n;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / n, i = e % n;
    const float g = ld_el(gu, r * gu_ld + i, dtype);
    const float u = ld_el(gu, r * gu_ld + n + i, dtype);
    const float s = round_to(g / (1.0f + expf(-g)), dtype);  // F.silu, rounded to the dtype
    st_el(z, r * z_ld + i, s * u, dtype);
  }
}

}  // namespace dec_layer

int launch_add_rmsnorm(int dtype, int64_t T, int64_t d, const void* x, int64_t x_ld, const void* a, int64_t a_ld,
                       const void* w, float eps, void* h_out, int64_t h_ld, void* y_out, int64_t y_ld,
                       cudaStream_t stream) {
  if (T == 0) return GSA_OK;
  if (T > 0x7fffffffLL) return GSA_ERR_BAD_ARG;
  dec_layer::add_rmsnorm_kernel<<<(unsigned)T, dec_layer::kThreads, 0, stream>>>(dtype, d, x, x_ld, a, a_ld, w, eps,
                                                                                 h_out, h_ld, y_out, y_ld);
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

int launch_silu_mul(int dtype, int64_t T, int64_t n, const void* gu, int64_t gu_ld, void* z, int64_t z_ld,
                    cudaStream_t stream) {
  if (T * n == 0) return GSA_OK;
  int64_t blocks = (T * n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  dec_layer::silu_mul_kernel<<<(unsigned)blocks, 256, 0, stream>>>(dtype, T, n, gu, gu_ld, z, z_ld);
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

}  // namespace gsa
