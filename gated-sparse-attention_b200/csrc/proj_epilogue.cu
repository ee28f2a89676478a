// Projection epilogue: turns one row of the fused projection GEMM output into the tensors the
// rest of the layer reads.  Elementwise and HBM-bound; one CTA per token row.
//
//   q, k  <- rotate-half RoPE at the row's position        (rope.py:151-185)
//   v     <- v * act(g2)                                   (value_gate.py:95-113)
//   g1    <- act(g1 logits)                                (output_gate.py:101-117)
//   w     <- sigmoid(wI logits), shift <- 0.5 * sum_j w_j  (gated_indexer.py:121)
//
// Every op is evaluated as torch evaluates it: in fp32, rounded to the activation dtype after
// each op, with no FMA contraction, so that a bf16 layer matches the reference's bf16 ops.
#include "kernels.cuh"

namespace gsa {



// rotate-half on one head: out[i] = x[i]*cos[i] + rot[i]*sin[i], rot = cat(-x2, x1)
__device__ __forceinline__ void rope_head(const EpiArgs& a, int64_t src_row, int64_t col0,
                                          const void* cos_row, const void* sin_row,
                                          void* dst, int64_t dst0, int D) {
  const int half = D / 2;
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float x = load_elem(a.proj, src_row + col0 + i, a.dtype);
    float partner = load_elem(a.proj, src_row + col0 + (i < half ? i + half : i - half), a.dtype);
    float rot = i < half ? -partner : partner;
    float c = load_elem(cos_row, i, a.tab_dtype);
    float s = load_elem(sin_row, i, a.tab_dtype);
    // torch: (x * cos) + (rot * sin), each product and the sum rounded to the dtype
    float t1 = rnd(fmul(x, c), a.dtype);
    float t2 = rnd(fmul(rot, s), a.dtype);
    store_elem(dst, dst0 + i, fadd(t1, t2), a.dtype);
  }
}

__global__ void proj_epilogue_kernel(EpiArgs a) {
  const int64_t t = blockIdx.x;
  if (t >= a.T) return;
  const int H = a.d.n_heads, Hk = a.d.n_kv_heads, D = a.d.d_head, HI = a.d.n_idx_heads;
  const int64_t row = t * a.proj_ld;
  int64_t pos = a.positions[t];
  if (pos < 0 || pos >= a.tab_rows) {
    set_error(a.err, GSA_ERR_INDEX);
    pos = pos < 0 ? 0 : a.tab_rows - 1;
  }
  const int64_t tab_off = pos * D;
  const void* cos_row = a.tab_dtype == GSA_DTYPE_BF16
                            ? (const void*)(reinterpret_cast<const __nv_bfloat16*>(a.cos_tab) + tab_off)
                            : (const void*)(reinterpret_cast<const float*>(a.cos_tab) + tab_off);
  const void* sin_row = a.tab_dtype == GSA_DTYPE_BF16
                            ? (const void*)(reinterpret_cast<const __nv_bfloat16*>(a.sin_tab) + tab_off)
                            : (const void*)(reinterpret_cast<const float*>(a.sin_tab) + tab_off);

  for (int h = 0; h < H; ++h)
    rope_head(a, row, a.lay.q + (int64_t)h * D, cos_row, sin_row, a.q_out, (t * H + h) * D, D);
  for (int h = 0; h < Hk; ++h)
    rope_head(a, row, a.lay.k + (int64_t)h * D, cos_row, sin_row, a.k_out, t * a.kv_ld + (int64_t)h * D, D);

  // G2 on v, applied before RoPE and never rotated (gated_sparse_attention.py:180-186)
  for (int i = threadIdx.x; i < Hk * D; i += blockDim.x) {
    float v = load_elem(a.proj, row + a.lay.v + i, a.dtype);
    if (a.lay.g2 >= 0) {
      float g = gate_act(load_elem(a.proj, row + a.lay.g2 + i, a.dtype), a.d.gate_act, a.dtype);
      v = fmul(v, g);
    }
    store_elem(a.v_out, t * a.kv_ld + i, v, a.dtype);
  }
  if (a.lay.g1 >= 0 && a.g1_out) {
    for (int i = threadIdx.x; i < H * D; i += blockDim.x) {
      float g = gate_act(load_elem(a.proj, row + a.lay.g1 + i, a.dtype), a.d.gate_act, a.dtype);
      store_elem(a.g1_out, t * H * D + i, g, a.dtype);
    }
  }
  if (threadIdx.x == 0) {
    float sum = 0.f;
    for (int j = 0; j < HI; ++j) {
      float w = rnd(sigmoid_precise(load_elem(a.proj, row + a.lay.wi + j, a.dtype)), a.dtype);
      a.w_out[t * HI + j] = w;
      sum += w;
    }
    a.shift_out[t] = 0.5f * sum;
  }
}

int launch_proj_epilogue(const EpiArgs& a, cudaStream_t stream) {
  if (a.T == 0) return GSA_OK;
  proj_epilogue_kernel<<<(unsigned)a.T, 128, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

// Standalone gate (ValueGate / OutputGate modules): out = x * act(logits).
__global__ void apply_gate_kernel(int dtype, int act, int64_t n, const void* x, const void* logits, void* out,
                                  void* gate_out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float g = gate_act(load_elem(logits, i, dtype), act, dtype);
    if (gate_out) store_elem(gate_out, i, g, dtype);
    store_elem(out, i, fmul(load_elem(x, i, dtype), g), dtype);
  }
}

int launch_apply_gate(int dtype, int act, int64_t n, const void* x, const void* logits, void* out, void* gate_out,
                      cudaStream_t stream) {
  int64_t blocks = (n + 255) / 256;
  if (blocks > 65536) blocks = 65536;
  apply_gate_kernel<<<(unsigned)blocks, 256, 0, stream>>>(dtype, act, n, x, logits, out, gate_out);
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

}  // namespace gsa
