// Backward of the sparse GQA SDPA (gated_sparse_attention.py:256-290, differentiated as torch
// autograd differentiates _gather_along_seq, the masked softmax and the two einsums).  The index
// sets carry no gradient (they come from torch.topk, adaptive_topk.py:177), so neither does the
// indexer.  For row r, head h of KV group g, selected keys s, p_s = exp(scale q.k_s - lse) (the
// forward's log-sum-exp), D = dO.O:
//
//   dq_h  = scale sum_s p_s (dO.v_s - D) k_s
//   dk_s += scale p_s (dO.v_s - D) q_h          (summed over the group's heads)
//   dv_s += p_s dO_h
//
// One CTA per row, one warp per KV group; a lane owns D/32 consecutive dimensions of every head
// of its group (q, dO and the dq accumulator in registers).  dk and dv are fp32 accumulators
// shared by every row that selected the key: vector atomics (red.v4/v2.f32), so their summation
// order -- and the last bits of dk, dv -- vary from run to run.  Keys are taken two at a time so
// that their loads overlap.
#include "kernels.cuh"

namespace gsa {

namespace bwd {

template <typename T, int N>
struct Ld;
template <>
struct Ld<float, 4> {
  static __device__ __forceinline__ void run(const void* p, float (&x)[4]) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
  }
};
template <>
struct Ld<float, 2> {
  static __device__ __forceinline__ void run(const void* p, float (&x)[2]) {
    const float2 v = *reinterpret_cast<const float2*>(p);
    x[0] = v.x; x[1] = v.y;
  }
};
template <>
struct Ld<__nv_bfloat16, 4> {
  static __device__ __forceinline__ void run(const void* p, float (&x)[4]) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    x[0] = __uint_as_float(u.x << 16); x[1] = __uint_as_float(u.x & 0xffff0000u);
    x[2] = __uint_as_float(u.y << 16); x[3] = __uint_as_float(u.y & 0xffff0000u);
  }
};
template <>
struct Ld<__nv_bfloat16, 2> {
  static __device__ __forceinline__ void run(const void* p, float (&x)[2]) {
    const uint32_t u = *reinterpret_cast<const uint32_t*>(p);
    x[0] = __uint_as_float(u << 16); x[1] = __uint_as_float(u & 0xffff0000u);
  }
};

__device__ __forceinline__ void red_add(float* p, const float (&x)[4]) {
  atomicAdd(reinterpret_cast<float4*>(p), make_float4(x[0], x[1], x[2], x[3]));
}
__device__ __forceinline__ void red_add(float* p, const float (&x)[2]) {
  atomicAdd(reinterpret_cast<float2*>(p), make_float2(x[0], x[1]));
}

template <typename T, int NREP, int DPL>
__global__ void __launch_bounds__(512) sdpa_bwd_kernel(SdpaBwdArgs a) {
  constexpr int U = 2;  // keys in flight per warp
  const int64_t row = blockIdx.x;
  const int g = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (g >= a.Hk) return;
  const int64_t b = row / a.Lq;
  const int H = a.H, D = a.D;
  int cnt = a.sel_count[row];
  if (cnt < 0) cnt = 0;
  if (cnt > a.sel_ld) cnt = (int)a.sel_ld;
  const int d0 = lane * DPL;
  const T* qr = reinterpret_cast<const T*>(a.q) + (row * H + (int64_t)g * NREP) * D + d0;
  const T* orow = reinterpret_cast<const T*>(a.o) + (row * H + (int64_t)g * NREP) * D + d0;
  const T* dorow = reinterpret_cast<const T*>(a.d_o) + (row * H + (int64_t)g * NREP) * D + d0;
  float q[NREP][DPL], dO[NREP][DPL], dq[NREP][DPL], lse[NREP], Dh[NREP];
#pragma unroll
  for (int h = 0; h < NREP; ++h) {
    float ov[DPL];
    Ld<T, DPL>::run(qr + h * D, q[h]);
    Ld<T, DPL>::run(dorow + h * D, dO[h]);
    Ld<T, DPL>::run(orow + h * D, ov);
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      t = fmaf(dO[h][i], ov[i], t);
      dq[h][i] = 0.f;
    }
    Dh[h] = warp_sum(t);
    lse[h] = a.lse[row * H + g * NREP + h];
  }
  const int32_t* idx = a.sel_idx + row * a.sel_ld;
  const T* kb = reinterpret_cast<const T*>(a.k) + b * a.kv_bstride + (int64_t)g * D + d0;
  const T* vb = reinterpret_cast<const T*>(a.v) + b * a.kv_bstride + (int64_t)g * D + d0;
  float* dkb = a.dk + b * a.dkv_bstride + (int64_t)g * D + d0;
  float* dvb = a.dv + b * a.dkv_bstride + (int64_t)g * D + d0;
  for (int j0 = 0; j0 < cnt; j0 += U) {
    float kx[U][DPL], vx[U][DPL];
    int64_t sk[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      sk[u] = -1;
      if (j0 + u < cnt) {
        const int64_t s = idx[j0 + u];
        if (s >= 0 && s < a.Lkv) {
          sk[u] = s;
        } else if (lane == 0) {
          set_error(a.err, GSA_ERR_INDEX);
        }
      }
      if (sk[u] >= 0) {
        Ld<T, DPL>::run(kb + sk[u] * a.kv_ld, kx[u]);
        Ld<T, DPL>::run(vb + sk[u] * a.kv_ld, vx[u]);
      } else {
#pragma unroll
        for (int i = 0; i < DPL; ++i) kx[u][i] = vx[u][i] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (sk[u] < 0) continue;  // uniform across the warp
      float qk[NREP], pv[NREP];
#pragma unroll
      for (int h = 0; h < NREP; ++h) {
        float x = 0.f, y = 0.f;
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          x = fmaf(q[h][i], kx[u][i], x);
          y = fmaf(dO[h][i], vx[u][i], y);
        }
        qk[h] = x;
        pv[h] = y;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int h = 0; h < NREP; ++h) {
          qk[h] += __shfl_xor_sync(0xffffffffu, qk[h], o);
          pv[h] += __shfl_xor_sync(0xffffffffu, pv[h], o);
        }
      }
      float dk[DPL], dv[DPL];
#pragma unroll
      for (int i = 0; i < DPL; ++i) dk[i] = dv[i] = 0.f;
#pragma unroll
      for (int h = 0; h < NREP; ++h) {
        const float p = lse[h] > -INFINITY ? expf(qk[h] * a.scale - lse[h]) : 0.f;
        const float ds = p * (pv[h] - Dh[h]) * a.scale;
#pragma unroll
        for (int i = 0; i < DPL; ++i) {
          dq[h][i] = fmaf(ds, kx[u][i], dq[h][i]);
          dk[i] = fmaf(ds, q[h][i], dk[i]);
          dv[i] = fmaf(p, dO[h][i], dv[i]);
        }
      }
      red_add(dkb + sk[u] * a.dkv_ld, dk);
      red_add(dvb + sk[u] * a.dkv_ld, dv);
    }
  }
  float* dqr = a.dq + (row * H + (int64_t)g * NREP) * D + d0;
#pragma unroll
  for (int h = 0; h < NREP; ++h) {
#pragma unroll
    for (int i = 0; i < DPL; ++i) dqr[h * D + i] = dq[h][i];
  }
}

template <typename T, int DPL>
static int launch_nrep(const SdpaBwdArgs& a, int64_t R, cudaStream_t s) {
  const int threads = a.Hk * 32;
  switch (a.H / a.Hk) {
    case 1: sdpa_bwd_kernel<T, 1, DPL><<<(unsigned)R, threads, 0, s>>>(a); break;
    case 2: sdpa_bwd_kernel<T, 2, DPL><<<(unsigned)R, threads, 0, s>>>(a); break;
    case 4: sdpa_bwd_kernel<T, 4, DPL><<<(unsigned)R, threads, 0, s>>>(a); break;
    case 8: sdpa_bwd_kernel<T, 8, DPL><<<(unsigned)R, threads, 0, s>>>(a); break;
    default: return GSA_ERR_UNSUPPORTED;
  }
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

}  // namespace bwd

int launch_sdpa_backward(const SdpaBwdArgs& a, cudaStream_t stream) {
  const int64_t R = a.B * a.Lq;
  if (R == 0) return GSA_OK;
  if (R > 0x7fffffffLL || a.Hk < 1 || a.Hk > 16 || a.H % a.Hk) return GSA_ERR_UNSUPPORTED;
  if (a.dtype == GSA_DTYPE_BF16) {
    if (a.D == 128) return bwd::launch_nrep<__nv_bfloat16, 4>(a, R, stream);
    if (a.D == 64) return bwd::launch_nrep<__nv_bfloat16, 2>(a, R, stream);
  } else {
    if (a.D == 128) return bwd::launch_nrep<float, 4>(a, R, stream);
    if (a.D == 64) return bwd::launch_nrep<float, 2>(a, R, stream);
  }
  return GSA_ERR_UNSUPPORTED;
}

}  // namespace gsa
