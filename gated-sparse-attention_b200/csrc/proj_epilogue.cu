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
  chain_wait();
  chain_release();
  const int64_t t = blockIdx.x;
  if (t >= a.T) return;
  const int H = a.d.n_heads, Hk = a.d.n_kv_heads, D = a.d.d_head, HI = a.d.n_idx_heads;
  const int64_t row = t * a.proj_ld;
  int64_t pos = epi_position(a, t);
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
  const int64_t kv_off = epi_kv_off(a, t);
  for (int h = 0; h < Hk; ++h)
    rope_head(a, row, a.lay.k + (int64_t)h * D, cos_row, sin_row, a.k_out, kv_off + (int64_t)h * D, D);

  // G2 on v, applied before RoPE and never rotated (gated_sparse_attention.py:180-186)
  for (int i = threadIdx.x; i < Hk * D; i += blockDim.x) {
    float v = load_elem(a.proj, row + a.lay.v + i, a.dtype);
    if (a.lay.g2 >= 0) {
      float g = gate_act(load_elem(a.proj, row + a.lay.g2 + i, a.dtype), a.d.gate_act, a.dtype);
      v = fmul(v, g);
    }
    store_elem(a.v_out, kv_off + i, v, a.dtype);
  }
  if (a.ki_out) {
    const int64_t ki_off = (t / a.L) * a.ki_bstride + (t % a.L) * a.ki_ld;
    for (int i = threadIdx.x; i < a.d.d_idx; i += blockDim.x)
      store_elem(a.ki_out, ki_off + i, load_elem(a.proj, row + a.lay.ki + i, a.dtype), a.dtype);
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
  if (a.zero_stats && threadIdx.x < 3) a.zero_stats[t * 3 + threadIdx.x] = 0.0;
}

// ---------------------------------------------------------------------------------------------
// bf16 fast path: the same ops and roundings, 8 elements per thread with 16-byte accesses.  A
// RoPE task takes elements i..i+7 of a head's first half together with their rotate-half
// partners i+D/2..i+D/2+7, so every loaded element is used once.
// ---------------------------------------------------------------------------------------------
struct Vec8 {
  float f[8];
};

__device__ __forceinline__ Vec8 ld8_bf16(const __nv_bfloat16* p) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  Vec8 v;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v.f[2 * k] = __uint_as_float(w[k] << 16);
    v.f[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
  }
  return v;
}

__device__ __forceinline__ Vec8 ld8_tab(const __nv_bfloat16* p) { return ld8_bf16(p); }
__device__ __forceinline__ Vec8 ld8_tab(const float* p) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  Vec8 v;
  v.f[0] = a.x; v.f[1] = a.y; v.f[2] = a.z; v.f[3] = a.w;
  v.f[4] = b.x; v.f[5] = b.y; v.f[6] = b.z; v.f[7] = b.w;
  return v;
}

// store rounds each value to bf16 (round to nearest even), as store_elem does
__device__ __forceinline__ void st8_bf16(__nv_bfloat16* p, const Vec8& v) {
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(v.f[2 * k], v.f[2 * k + 1]);
    w[k] = *reinterpret_cast<const uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

template <typename TabT>
__global__ void __launch_bounds__(256) proj_epilogue_bf16_kernel(EpiArgs a) {
  chain_wait();
  chain_release();
  const int64_t t = blockIdx.x;
  if (t >= a.T) return;
  constexpr int dt = GSA_DTYPE_BF16;
  const int H = a.d.n_heads, Hk = a.d.n_kv_heads, D = a.d.d_head, HI = a.d.n_idx_heads;
  const int half = D / 2, vh = half / 8;
  const __nv_bfloat16* prow = reinterpret_cast<const __nv_bfloat16*>(a.proj) + t * a.proj_ld;
  int64_t pos = epi_position(a, t);
  if (pos < 0 || pos >= a.tab_rows) {
    set_error(a.err, GSA_ERR_INDEX);
    pos = pos < 0 ? 0 : a.tab_rows - 1;
  }
  const TabT* cr = reinterpret_cast<const TabT*>(a.cos_tab) + pos * D;
  const TabT* sr = reinterpret_cast<const TabT*>(a.sin_tab) + pos * D;
  __nv_bfloat16* qo = reinterpret_cast<__nv_bfloat16*>(a.q_out);
  __nv_bfloat16* ko = reinterpret_cast<__nv_bfloat16*>(a.k_out);
  __nv_bfloat16* vo = reinterpret_cast<__nv_bfloat16*>(a.v_out);
  __nv_bfloat16* go = reinterpret_cast<__nv_bfloat16*>(a.g1_out);
  const int nq = H * vh, nk = Hk * vh, nv = Hk * D / 8;
  const int ng = (a.lay.g1 >= 0 && a.g1_out) ? H * D / 8 : 0;
  const int nki = a.ki_out ? a.d.d_idx / 8 : 0;
  const int ntask = nq + nk + nv + ng + nki;
  const int64_t kv_off = epi_kv_off(a, t);
  // gridDim.y CTAs share a token's tasks (few tokens: decode)
  for (int task = blockIdx.y * blockDim.x + threadIdx.x; task < ntask; task += gridDim.y * blockDim.x) {
    if (task < nq + nk) {
      const bool isq = task < nq;
      const int tt = isq ? task : task - nq;
      const int h = tt / vh, i = (tt % vh) * 8;
      const __nv_bfloat16* src = prow + (isq ? a.lay.q : a.lay.k) + (int64_t)h * D;
      const Vec8 x1 = ld8_bf16(src + i), x2 = ld8_bf16(src + i + half);
      const Vec8 c1 = ld8_tab(cr + i), c2 = ld8_tab(cr + i + half);
      const Vec8 s1 = ld8_tab(sr + i), s2 = ld8_tab(sr + i + half);
      Vec8 o1, o2;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        // (x * cos) + (rotate_half(x) * sin), rotate_half = cat(-x2, x1); each op rounded
        o1.f[e] = fadd(rnd(fmul(x1.f[e], c1.f[e]), dt), rnd(fmul(-x2.f[e], s1.f[e]), dt));
        o2.f[e] = fadd(rnd(fmul(x2.f[e], c2.f[e]), dt), rnd(fmul(x1.f[e], s2.f[e]), dt));
      }
      __nv_bfloat16* dst = isq ? qo + (t * H + h) * D : ko + kv_off + (int64_t)h * D;
      st8_bf16(dst + i, o1);
      st8_bf16(dst + i + half, o2);
    } else if (task < nq + nk + nv) {
      const int i = (task - nq - nk) * 8;
      Vec8 v = ld8_bf16(prow + a.lay.v + i);
      if (a.lay.g2 >= 0) {
        const Vec8 g = ld8_bf16(prow + a.lay.g2 + i);
#pragma unroll
        for (int e = 0; e < 8; ++e) v.f[e] = fmul(v.f[e], gate_act(g.f[e], a.d.gate_act, dt));
      }
      st8_bf16(vo + kv_off + i, v);
    } else if (task >= nq + nk + nv + ng) {
      // k^I into the cache: a plain 16-byte copy (already bf16)
      const int i = (task - nq - nk - nv - ng) * 8;
      __nv_bfloat16* kio = reinterpret_cast<__nv_bfloat16*>(a.ki_out) + (t / a.L) * a.ki_bstride +
                           (t % a.L) * a.ki_ld;
      *reinterpret_cast<uint4*>(kio + i) = *reinterpret_cast<const uint4*>(prow + a.lay.ki + i);
    } else {
      const int i = (task - nq - nk - nv) * 8;
      Vec8 g = ld8_bf16(prow + a.lay.g1 + i);
#pragma unroll
      for (int e = 0; e < 8; ++e) g.f[e] = gate_act(g.f[e], a.d.gate_act, dt);
      st8_bf16(go + t * (int64_t)H * D + i, g);
    }
  }
  if (threadIdx.x == 0 && blockIdx.y == 0) {
    float sum = 0.f;
    for (int j = 0; j < HI; ++j) {
      float w = rnd(sigmoid_precise(__bfloat162float(prow[a.lay.wi + j])), dt);
      a.w_out[t * HI + j] = w;
      sum += w;
    }
    a.shift_out[t] = 0.5f * sum;
  }
  if (a.zero_stats && blockIdx.y == 0 && threadIdx.x < 3) a.zero_stats[t * 3 + threadIdx.x] = 0.0;
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) % 16) == 0; }

// The vector path needs every row segment it touches to start on a 16-byte boundary.
static bool epilogue_vec_ok(const EpiArgs& a) {
  const int D = a.d.d_head;
  auto el = [](int64_t x) { return (x * 2) % 16 == 0; };
  bool ok = a.dtype == GSA_DTYPE_BF16 && D % 16 == 0 && al16(a.proj) && el(a.proj_ld) && el(a.lay.q) &&
            el(a.lay.k) && el(a.lay.v) && (a.lay.g2 < 0 || el(a.lay.g2)) && al16(a.q_out) && al16(a.k_out) &&
            al16(a.v_out) && el(a.kv_ld);
  if (a.lay.g1 >= 0 && a.g1_out) ok = ok && el(a.lay.g1) && al16(a.g1_out);
  if (a.L) ok = ok && el(a.kv_bstride);
  if (a.ki_out) ok = ok && a.d.d_idx % 8 == 0 && el(a.lay.ki) && al16(a.ki_out) && el(a.ki_ld) && el(a.ki_bstride);
  const size_t tab_el = a.tab_dtype == GSA_DTYPE_BF16 ? 2 : 4;
  ok = ok && al16(a.cos_tab) && al16(a.sin_tab) && ((int64_t)D * tab_el) % 16 == 0;
  return ok;
}

int launch_proj_epilogue(const EpiArgs& a, cudaStream_t stream) {
  if (a.T == 0) return GSA_OK;
  if (a.T > 0x7fffffffLL) return GSA_ERR_BAD_ARG;
  if (epilogue_vec_ok(a)) {
    // few tokens (decode): four CTAs per token, so that the copy latency is spread over more SMs
    const dim3 grid((unsigned)a.T, a.T < 512 ? 4u : 1u);
    const cudaError_t e = a.tab_dtype == GSA_DTYPE_BF16
                              ? launch_chained(proj_epilogue_bf16_kernel<__nv_bfloat16>, grid, dim3(256), 0, stream, a)
                              : launch_chained(proj_epilogue_bf16_kernel<float>, grid, dim3(256), 0, stream, a);
    if (e != cudaSuccess) return GSA_ERR_LAUNCH;
  } else if (launch_chained(proj_epilogue_kernel, dim3((unsigned)a.T), dim3(128), 0, stream, a) != cudaSuccess) {
    return GSA_ERR_LAUNCH;
  }
  return GSA_OK;
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
