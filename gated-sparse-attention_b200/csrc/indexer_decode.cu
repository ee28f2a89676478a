// Gated indexer for a few query tokens per sequence against a long key sequence (decode: one
// new token of each of B sequences scored against every cached key), all sequences in one launch.
//
//   I[t,s] = sum_j w[t,j] * sigmoid(scale * <qI[t,j,:], kI[s,:]> + b[j])      (gated_indexer.py:114-145)
//
// With one token per sequence the contraction is a matrix-vector product per sequence (H_I = 8
// heads against each 64-wide key), so the kernel streams k^I once at HBM rate: 128 bytes per key,
// against 2 * 8 * 64 flops.  Those flops run on mma.sync m16n8k16 (16 keys x 8 (token, head)
// columns x 16 of d_I per instruction) straight from registers: each lane loads two 16-byte
// chunks of two key rows, which is exactly one A fragment per k-step once the d_I order is
// permuted the same way for the query fragment (a dot product does not depend on the order of
// its terms).  The 5th-generation tcgen05 path would need a 128-key x 8-column tile per MMA and
// a TMEM round trip for a kernel whose bound is the k^I read, not the tensor pipe.
//
// Epilogue: the arithmetic of the tensor-core prefill indexer (indexer_tc.cu): z = fma(acc,
// scale/2, b_j/2), tanh.approx, the heads' (w_j/2) tanh terms added to c_t = sum_j w_j/2.  A lane
// holds two heads of two keys; the head sum finishes with two xor-shuffles across its quad (the
// prefill kernel sums the heads in another order, so a score may differ from it in the last bit).
// Per 16 keys a warp issues 4 loads, 4 mma, 8 tanh and a dozen other instructions per lane,
// which keeps the kernel on the HBM bound.
//
// Grid: x = ranges of 8 warps x keys_per_warp keys (sized for about two waves), y = sequence.
// Row statistics (sum, sum of squares of the centred score, unmasked count) are reduced per CTA
// and added with one fp64 atomic per value.
#include "kernels.cuh"

namespace gsa {

namespace dec {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kGroup = 16;                        // keys per mma row block
constexpr int kDI = 64;

__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint4 ld_stream(const __nv_bfloat16* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void split8(const uint4& lo, const uint4& hi, uint32_t (&r)[8]) {
  r[0] = lo.x; r[1] = lo.y; r[2] = lo.z; r[3] = lo.w;
  r[4] = hi.x; r[5] = hi.y; r[6] = hi.z; r[7] = hi.w;
}

// HI heads per token; TPM = 8 / HI tokens share one mma's 8 columns; NT column blocks per key
// group cover up to NT * TPM tokens of a sequence.  U key groups are loaded before first use.
// Each warp scores keys_per_warp consecutive keys (a multiple of 16 * U).
template <int HI, int NT, int U>
__global__ void __launch_bounds__(kThreads, 2) indexer_decode_kernel(IdxArgs a, int keys_per_warp) {
  chain_wait();
  chain_release();
  constexpr int TPM = 8 / HI;
  constexpr int MAXT = NT * TPM;
  const int64_t b = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int Lq = (int)a.Lq;
  const int64_t key_limit = a.causal ? min(a.Lkv, a.q_pos0 + a.Lq) : a.Lkv;
  const int64_t k_cta0 = (int64_t)blockIdx.x * kWarps * keys_per_warp;
  const int64_t k_cta1 = min(k_cta0 + (int64_t)kWarps * keys_per_warp, key_limit);

  __shared__ float w_s[MAXT][HI];    // w / 2
  __shared__ float2 cd_s[MAXT];      // (c_t, c_t - shift_t), c_t = sum_j w_tj / 2
  __shared__ float red_s[kWarps][MAXT][2];

  const int64_t row0 = b * a.Lq;     // score / weight row of this sequence's first token
  for (int i = threadIdx.x; i < MAXT * HI; i += kThreads) {
    const int t = i / HI, j = i % HI;
    w_s[t][j] = t < Lq ? 0.5f * a.w[(row0 + t) * HI + j] : 0.f;
  }
  __syncthreads();
  if (threadIdx.x < MAXT) {
    const int t = threadIdx.x;
    float c = 0.f;
#pragma unroll
    for (int j = 0; j < HI; ++j) c += w_s[t][j];
    cd_s[t] = make_float2(c, (a.shift && t < Lq) ? c - a.shift[row0 + t] : c);
  }

  // query fragments: column n = g is (token tg * TPM + g / HI, head g % HI); this lane supplies
  // d_I chunks q and q + 4 of it (the same chunks it loads of every key row)
  const __nv_bfloat16* qI = reinterpret_cast<const __nv_bfloat16*>(a.qI) + b * a.qi_bstride;
  uint32_t qb[NT][8];
#pragma unroll
  for (int tg = 0; tg < NT; ++tg) {
    const int t = tg * TPM + g / HI, j = g % HI;
    if (t < Lq) {
      const __nv_bfloat16* qp = qI + (int64_t)t * a.qi_ld + j * kDI;
      split8(ld_stream(qp + 8 * q), ld_stream(qp + 32 + 8 * q), qb[tg]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) qb[tg][i] = 0u;
    }
  }
  __syncthreads();

  // this lane's accumulator columns 2q, 2q+1: token tok of the column block, heads j0, j0 + 1.
  // After the quad reduction the lane finishes key g + 8 * (q & 1) of token tok (H_I = 8: lanes
  // q = 0, 1 only; the four lanes of a quad hold one token's eight heads).
  const int tok = (2 * q) / HI, j0 = (2 * q) % HI;
  const bool finisher = HI == 8 ? q < 2 : true;
  const float hs = 0.5f * a.scale;
  const float hb0 = 0.5f * a.bias[j0], hb1 = 0.5f * a.bias[j0 + 1];
  const int64_t kw0 = k_cta0 + (int64_t)warp * keys_per_warp;
  const int nw = (int)max((int64_t)0, min((int64_t)keys_per_warp, k_cta1 - kw0));
  float w0[NT], w1[NT], s1[NT], s2[NT];
  float2 cdt[NT];
  int lim[NT];       // keys [0, lim) of this warp are unmasked for the lane's token
  float* srow[NT];
#pragma unroll
  for (int tg = 0; tg < NT; ++tg) {
    const int t = tg * TPM + tok;
    w0[tg] = w_s[t][j0];
    w1[tg] = w_s[t][j0 + 1];
    cdt[tg] = cd_s[t];
    s1[tg] = s2[tg] = 0.f;
    int64_t l = a.causal ? min((int64_t)nw, a.q_pos0 + t + 1 - kw0) : (int64_t)nw;
    lim[tg] = (finisher && t < Lq) ? (int)max((int64_t)0, l) : 0;
    srow[tg] = a.scores + (row0 + min(t, Lq - 1)) * a.scores_ld + kw0;
  }

  const __nv_bfloat16* kbase = reinterpret_cast<const __nv_bfloat16*>(a.kI) + b * a.ki_bstride + kw0 * a.ki_ld +
                               8 * q;
  const int ld = (int)a.ki_ld;
  for (int kb = 0; kb < nw; kb += U * kGroup) {
    uint4 ka[U][4];  // rows g and g + 8: d_I chunks q and q + 4
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int r0 = kb + u * kGroup + g, r1 = r0 + 8;
      const uint4 z = make_uint4(0u, 0u, 0u, 0u);
      const __nv_bfloat16* p0 = kbase + r0 * ld;
      const __nv_bfloat16* p1 = kbase + r1 * ld;
      ka[u][0] = r0 < nw ? ld_stream(p0) : z;
      ka[u][1] = r0 < nw ? ld_stream(p0 + 32) : z;
      ka[u][2] = r1 < nw ? ld_stream(p1) : z;
      ka[u][3] = r1 < nw ? ld_stream(p1 + 32) : z;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      uint32_t ra[8], rb[8];
      split8(ka[u][0], ka[u][1], ra);
      split8(ka[u][2], ka[u][3], rb);
      const int key = kb + u * kGroup + g + 8 * (q & 1);
#pragma unroll
      for (int tg = 0; tg < NT; ++tg) {
        if (tg * TPM >= Lq) break;
        float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_bf16(c, ra[2 * kk], rb[2 * kk], ra[2 * kk + 1], rb[2 * kk + 1], qb[tg][2 * kk], qb[tg][2 * kk + 1]);
        // sum_j (w_j / 2) tanh((scale acc_j + b_j) / 2) over this lane's two heads, keys g and g + 8
        float y0 = fmaf(w0[tg], tanh_fast(fmaf(c[0], hs, hb0)), w1[tg] * tanh_fast(fmaf(c[1], hs, hb1)));
        float y1 = fmaf(w0[tg], tanh_fast(fmaf(c[2], hs, hb0)), w1[tg] * tanh_fast(fmaf(c[3], hs, hb1)));
        // over the quad lanes of the same token: H_I = 8 all four, H_I = 4 pairs
        y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
        y1 += __shfl_xor_sync(0xffffffffu, y1, 1);
        if (HI == 8) {
          y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
          y1 += __shfl_xor_sync(0xffffffffu, y1, 2);
        }
        const float y = (q & 1) ? y1 : y0;
        if (key < lim[tg]) {
          srow[tg][key] = cdt[tg].x + y;
          const float yy = cdt[tg].y + y;
          s1[tg] += yy;
          s2[tg] = fmaf(yy, yy, s2[tg]);
        }
      }
    }
  }

  if (!a.row_stats) return;
  // per token: H_I = 8 lanes 0, 1 of every quad hold partial sums; H_I = 4 lanes of equal q >> 1
#pragma unroll
  for (int tg = 0; tg < NT; ++tg) {
    float x = s1[tg], y = s2[tg];
#pragma unroll
    for (int o = 16; o >= 4; o >>= 1) {
      x += __shfl_xor_sync(0xffffffffu, x, o);
      y += __shfl_xor_sync(0xffffffffu, y, o);
    }
    x += __shfl_xor_sync(0xffffffffu, x, 1);
    y += __shfl_xor_sync(0xffffffffu, y, 1);
    if (HI == 8) {
      x += __shfl_xor_sync(0xffffffffu, x, 2);
      y += __shfl_xor_sync(0xffffffffu, y, 2);
    }
    if (lane < 4 && (lane & 1) == 0 && lane / 2 < TPM) {
      red_s[warp][tg * TPM + lane / 2][0] = x;
      red_s[warp][tg * TPM + lane / 2][1] = y;
    }
  }
  __syncthreads();
  if (threadIdx.x < Lq && threadIdx.x < MAXT) {
    const int t = threadIdx.x;
    float x = 0.f, y = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      x += red_s[w][t][0];
      y += red_s[w][t][1];
    }
    double* st = a.row_stats + (row0 + t) * 3;
    atomicAdd(st + 0, (double)x);
    atomicAdd(st + 1, (double)y);
    const int64_t hi_k = a.causal ? min(k_cta1, a.q_pos0 + t + 1) : k_cta1;
    atomicAdd(st + 2, (double)(hi_k > k_cta0 ? hi_k - k_cta0 : 0));
  }
}

template <int HI, int NT, int U>
static int launch(const IdxArgs& a, int64_t B, int64_t key_limit, int num_sms, cudaStream_t s) {
  // keys per warp: enough CTAs for about two waves of two resident CTAs per SM, in steps of
  // 16 * U keys, at most 2048 (one warp's 32-bit key offsets stay small)
  constexpr int step = kGroup * U;
  const int64_t target_ctas = 4LL * num_sms;
  int64_t kpw = (key_limit * B + target_ctas * kWarps - 1) / (target_ctas * kWarps);
  kpw = (kpw + step - 1) / step * step;
  kpw = std::max<int64_t>(step, std::min<int64_t>(kpw, 2048));
  if ((kpw + kGroup) * a.ki_ld > 0x7fffffffLL) return GSA_ERR_BAD_ARG;
  const int64_t ranges = (key_limit + kWarps * kpw - 1) / (kWarps * kpw);
  if (ranges > 0x7fffffffLL) return GSA_ERR_BAD_ARG;
  dim3 grid((unsigned)ranges, (unsigned)B);
  return launch_chained(indexer_decode_kernel<HI, NT, U>, grid, dim3(kThreads), 0, s, a, (int)kpw) == cudaSuccess
             ? GSA_OK
             : GSA_ERR_LAUNCH;
}

}  // namespace dec

bool indexer_decode_eligible(const IdxArgs& a, int64_t B) {
  const bool hi_ok = a.HI == 8 || a.HI == 4;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) % 16) == 0; };
  auto el = [](int64_t x) { return x % 8 == 0; };
  return a.dtype == GSA_DTYPE_BF16 && a.dI == dec::kDI && hi_ok && a.act == GSA_ACT_SIGMOID && !a.write_masked &&
         a.Lq >= 1 && a.Lq <= 4 * (8 / a.HI) && B >= 1 && B <= 65535 && al(a.qI) && al(a.kI) && el(a.qi_ld) &&
         el(a.ki_ld) && el(a.qi_bstride) && el(a.ki_bstride) && a.Lkv <= ((int64_t)1 << 40);
}

// B sequences of Lq tokens each: rows b * Lq + t of w, shift, scores and row_stats.
int launch_indexer_decode(const IdxArgs& a, int64_t B, int num_sms, cudaStream_t s) {
  using namespace dec;
  const int64_t key_limit = a.causal ? std::min<int64_t>(a.Lkv, a.q_pos0 + a.Lq) : a.Lkv;
  if (key_limit <= 0 || B <= 0) return GSA_OK;
  const int tpm = 8 / a.HI;
  const bool one = a.Lq <= tpm;
  if (a.HI == 8)
    return one ? launch<8, 1, 4>(a, B, key_limit, num_sms, s) : launch<8, 4, 1>(a, B, key_limit, num_sms, s);
  return one ? launch<4, 1, 4>(a, B, key_limit, num_sms, s) : launch<4, 4, 1>(a, B, key_limit, num_sms, s);
}

}  // namespace gsa
