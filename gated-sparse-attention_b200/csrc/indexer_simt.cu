// Gated lightning indexer on the CUDA cores, fp32 arithmetic throughout.
//
//   I[t,s] = sum_j w[t,j] * act(scale * <qI[t,j,:], kI[s,:]> + bias[j])   (gated_indexer.py:114-145)
//
// This is the precise kernel: the layer's fp32 configuration runs on it (its scores must match
// the reference within 1e-3 relative), and it is the kernel the tensor-core indexer is
// checked against.  Each op after the dot product is evaluated in the reference's order
// (scale, + bias, activation, * w, sum over heads in head order) without FMA contraction.
//
// Tile: 32 query rows x 64 keys per 256-thread CTA; each thread owns 2 rows x 4 keys.
// Row statistics for the adaptive k (sum of x - shift, of (x - shift)^2, and the count of
// unmasked entries) are reduced across the 16 threads of a row and added in fp64.
#include "kernels.cuh"

namespace gsa {



constexpr int kTQ = 32, kTK = 64, kMaxDI = 128;

__global__ void __launch_bounds__(256) indexer_simt_kernel(IdxArgs a) {
  extern __shared__ float idx_smem[];
  const int pitch = a.dI + 1;
  float* q_s = idx_smem;                 // [kTQ][pitch]
  float* k_s = idx_smem + kTQ * pitch;   // [kTK][pitch]
  const int b = blockIdx.z;
  const int64_t t0 = (int64_t)blockIdx.y * kTQ;
  const int64_t s0 = (int64_t)blockIdx.x * kTK;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int dI = a.dI;

  // rows of this batch handled by the CTA start at score row (b * Lq + t0)
  const int64_t row_base = (int64_t)b * a.Lq;
  const int64_t last_t = min(t0 + kTQ, a.Lq) - 1;
  const bool tile_masked = a.causal && (s0 > a.q_pos0 + last_t);
  if (tile_masked) {
    if (a.write_masked) {
      for (int i = tid; i < kTQ * kTK; i += 256) {
        int r = i / kTK, c = i % kTK;
        if (t0 + r < a.Lq && s0 + c < a.Lkv)
          a.scores[(row_base + t0 + r) * a.scores_ld + s0 + c] = -INFINITY;
      }
    }
    return;
  }

  // key tile (shared by every head)
  for (int i = tid; i < kTK * dI; i += 256) {
    int r = i / dI, c = i % dI;
    int64_t s = s0 + r;
    float v = 0.f;
    if (s < a.Lkv) v = load_elem(a.kI, (int64_t)b * a.ki_bstride + s * a.ki_ld + c, a.dtype);
    k_s[r * pitch + c] = v;
  }

  float acc_score[2][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc_score[i][j] = 0.f;

  for (int h = 0; h < a.HI; ++h) {
    __syncthreads();  // previous head done with q_s (and k_s written on the first pass)
    for (int i = tid; i < kTQ * dI; i += 256) {
      int r = i / dI, c = i % dI;
      int64_t t = t0 + r;
      float v = 0.f;
      if (t < a.Lq) v = load_elem(a.qI, (int64_t)b * a.qi_bstride + t * a.qi_ld + (int64_t)h * dI + c, a.dtype);
      q_s[r * pitch + c] = v;
    }
    __syncthreads();
    float dot[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) dot[i][j] = 0.f;
    for (int c = 0; c < dI; ++c) {
      float q0 = q_s[(ty * 2) * pitch + c], q1 = q_s[(ty * 2 + 1) * pitch + c];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float kv = k_s[(tx * 4 + j) * pitch + c];
        dot[0][j] = fmaf(q0, kv, dot[0][j]);
        dot[1][j] = fmaf(q1, kv, dot[1][j]);
      }
    }
    const float bj = a.bias[h];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      int64_t t = t0 + ty * 2 + i;
      float wj = t < a.Lq ? a.w[(row_base + t) * a.HI + h] : 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float z = fadd(fmul(dot[i][j], a.scale), bj);
        float g = a.act == GSA_ACT_RELU ? fmaxf(z, 0.f) : sigmoid_precise(z);
        acc_score[i][j] = fadd(acc_score[i][j], fmul(g, wj));
      }
    }
  }

  // store + row statistics
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    int64_t t = t0 + ty * 2 + i;
    bool row_ok = t < a.Lq;
    float sh = (row_ok && a.shift) ? a.shift[row_base + t] : 0.f;
    float s1 = 0.f, s2 = 0.f, cnt = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int64_t s = s0 + tx * 4 + j;
      bool in = row_ok && s < a.Lkv;
      bool masked = a.causal && (s > a.q_pos0 + t);
      if (in && !masked) {
        float y = acc_score[i][j] - sh;
        s1 += y;
        s2 = fmaf(y, y, s2);
        cnt += 1.f;
      }
      if (in && (!masked || a.write_masked))
        a.scores[(row_base + t) * a.scores_ld + s] = masked ? -INFINITY : acc_score[i][j];
    }
    if (a.row_stats) {
      double d1 = s1, d2 = s2, dc = cnt;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) {
        d1 += __shfl_xor_sync(0xffffffffu, d1, o);
        d2 += __shfl_xor_sync(0xffffffffu, d2, o);
        dc += __shfl_xor_sync(0xffffffffu, dc, o);
      }
      if (tx == 0 && row_ok && dc > 0.0) {
        double* st = a.row_stats + (row_base + t) * 3;
        atomicAdd(st + 0, d1);
        atomicAdd(st + 1, d2);
        atomicAdd(st + 2, dc);
      }
    }
  }
}

int launch_indexer_simt(const IdxArgs& a, int64_t B, cudaStream_t stream) {
  if (a.Lq == 0 || a.Lkv == 0 || B == 0) return GSA_OK;
  if (a.dI > kMaxDI) return GSA_ERR_UNSUPPORTED;
  dim3 grid((unsigned)((a.Lkv + kTK - 1) / kTK), (unsigned)((a.Lq + kTQ - 1) / kTQ), (unsigned)B);
  if (grid.y > 65535u || grid.z > 65535u) return GSA_ERR_BAD_ARG;
  const size_t smem = (size_t)(kTQ + kTK) * (a.dI + 1) * sizeof(float);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(indexer_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return GSA_ERR_LAUNCH;
  indexer_simt_kernel<<<grid, 256, smem, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

}  // namespace gsa
