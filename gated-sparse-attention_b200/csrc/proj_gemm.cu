// Fused projection GEMM on the 5th-generation tensor cores: every projection of the layer and its
// epilogue in one persistent kernel (gated_sparse_attention.py:175-186, value_gate.py:95-113,
// output_gate.py:101-117, gated_indexer.py:114-121, rope.py:151-185).
//
//   acc[t, n] = x[t, :] . Wp[n, :]                    (tcgen05.mma, fp32 in TMEM)
//   p[t, n]   = bf16(acc + bias[n])                   (the bf16 projection output torch would store)
//   then, on p in registers, per 256-column tile of Wp (its "kind" by position):
//     Q   2 heads of q     -> rotate-half RoPE at the row's position          -> q_out
//     K   2 heads of k     -> RoPE                                           -> K rows of the KV layout
//     VG  v_h | g2_h       -> v * act(g2)  (G2 before RoPE, never rotated)    -> V rows of the KV layout
//     G1  2 heads of g1    -> act(g1)      (the output gate the SDPA epilogue multiplies in)
//     IDX q^I | k^I | w    -> q^I, k^I copied; w = sigmoid(.), shift = 0.5 * sum_j w_j
// with every op rounded to bf16 as torch evaluates it (the same ops and order as the unfused
// epilogue kernel), so no [T, Ncat] projection tensor is written and re-read.
//
// Wp is the layer's projection weights with rows in that tile order (D = 128):
//   [q (H*D)] [k (Hk*D)] [v_0 g2_0 v_1 g2_1 ... (2*Hk*D)] [g1 (H*D)] [q^I (H_I*d_I)] [k^I (d_I)] [w (H_I)] [0 pad]
// padded to a multiple of 256 rows; bias likewise (fp32; 0 where a projection has none).
//
// Roles (320 threads, one CTA per SM, persistent over (row block, column tile) work items):
// warp 0 = TMA producer (x tile 128 x 64 and Wp tile 256 x 64 per stage, 128-byte swizzle),
// warp 1 = TMEM allocator + MMA issuer (one lane; M = 128, N = 256, K = 16 per instruction),
// warps 2-9 = epilogue, two per TMEM lane quarter (each takes half of the tile's columns): a thread
// owns one token row of the tile.
// The 512 TMEM columns hold two accumulators, so a tile's epilogue overlaps the next tile's MMAs.
// Every wait is bounded; on a timeout the kernel records GSA_ERR_TIMEOUT and returns.
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace gsa {
namespace pg {

using namespace tc;

constexpr int kBM = 128;   // token rows per tile (TMEM lanes)
constexpr int kBN = 256;   // output columns per tile (fp32 TMEM columns per accumulator)
constexpr int kBK = 64;    // K per stage: one 128-byte swizzle atom of bf16
constexpr int kStages = 4;
#ifndef PG_EPI_WARPS
#define PG_EPI_WARPS 16
#endif
constexpr int kEpiWarps = PG_EPI_WARPS;  // kSplit per TMEM lane quarter, each taking 1/kSplit of the columns
constexpr int kSplit = kEpiWarps / 4;
constexpr int kCols = kBN / kSplit;      // columns of a tile per epilogue warp
constexpr int kPairs = kBN / 2 / kSplit; // RoPE pairs (or v / g2 pairs) of a tile per epilogue warp
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kATile = kBM * kBK * 2;  // 16 KiB
constexpr int kBTile = kBN * kBK * 2;  // 32 KiB
constexpr int kSmem = 1024 + kStages * (kATile + kBTile) + 256;

enum Kind { kQ = 0, kK = 1, kVG = 2, kG1 = 3, kIdx = 4 };

struct Params {
  int64_t T;
  int n_kblk;                 // d_model / 64
  int m_tiles, n_tiles;
  int t_q, t_k, t_vg, t_g1, t_idx;  // first column tile of each kind (IDX tiles up to n_tiles)
  int H, Hk, D, HI, dI;
  int gate_act;
  const float* bias;          // [n_tiles * 256]
  const int64_t* positions;   // [T] or NULL: row t at pos0 + t % L
  int64_t pos0, L;
  const void* cos_tab;
  const void* sin_tab;
  int tab_dtype;
  int64_t tab_rows;
  __nv_bfloat16* q_out;       // [T, H, D]
  __nv_bfloat16* k_out;       // token t's [Hk, D] K row at (t / L) * kv_bstride + (t % L) * kv_ld
  __nv_bfloat16* v_out;
  int64_t kv_ld, kv_bstride;
  __nv_bfloat16* g1_out;      // [T, H, D]
  __nv_bfloat16* qi_out;      // [T, qi_ld]
  int64_t qi_ld;
  __nv_bfloat16* ki_out;      // token t's k^I at (t / L) * ki_bstride + (t % L) * ki_ld
  int64_t ki_ld, ki_bstride;
  float* w_out;               // [T, H_I]
  float* shift_out;           // [T]
  int* err;
};

// Eight fp32 accumulator columns of this thread's row as the bf16-rounded projection values
// p = bf16(acc + bias) (bias NULL: none).
__device__ __forceinline__ void acc8(const uint32_t* r, const float* bias, float (&x)[8]) {
  float b[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (bias) {  // 32-byte aligned: two vector loads
    const float4 b0 = reinterpret_cast<const float4*>(bias)[0], b1 = reinterpret_cast<const float4*>(bias)[1];
    b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
    b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float v = __uint_as_float(r[i]);
    if (bias) v = fadd(v, b[i]);
    x[i] = __bfloat162float(__float2bfloat16_rn(v));
  }
}

// Eight values rounded to bf16 into one 16-byte store.
__device__ __forceinline__ void store8(__nv_bfloat16* dst, const float (&v)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
    w[k] = *reinterpret_cast<const uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
}

// Eight RoPE table entries (16-byte aligned) as fp32.
__device__ __forceinline__ void tab8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[2 * k] = __uint_as_float(w[k] << 16);
    v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
  }
}
__device__ __forceinline__ void tab8(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// RoPE of 32 element pairs (i, i + D/2) of one head, i = i0 .. i0+31: TMEM columns c1 (first half)
// and c2 (second half) of this thread's row; rotate-half with the row's cos / sin.
template <typename TabT>
__device__ __forceinline__ void rope32(uint32_t taddr, int c1, int c2, int i0, int half, const TabT* cr,
                                       const TabT* sr, __nv_bfloat16* dst, bool ok) {
  constexpr int dt = GSA_DTYPE_BF16;
  uint32_t r1[32], r2[32];
  tmem_ld32(taddr + c1, r1);
  tmem_ld32(taddr + c2, r2);
  tmem_wait_ld(r1);
  tmem_wait_ld(r2);
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    float x1[8], x2[8], cs1[8], sn1[8], cs2[8], sn2[8], o1[8], o2[8];
    acc8(r1 + 8 * g, nullptr, x1);
    acc8(r2 + 8 * g, nullptr, x2);
    tab8(cr + i0 + 8 * g, cs1);
    tab8(sr + i0 + 8 * g, sn1);
    tab8(cr + half + i0 + 8 * g, cs2);
    tab8(sr + half + i0 + 8 * g, sn2);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      // (x * cos) + (rotate_half(x) * sin), rotate_half = cat(-x2, x1); each op rounded
      o1[e] = fadd(rnd(fmul(x1[e], cs1[e]), dt), rnd(fmul(-x2[e], sn1[e]), dt));
      o2[e] = fadd(rnd(fmul(x2[e], cs2[e]), dt), rnd(fmul(x1[e], sn2[e]), dt));
    }
    if (ok) {
      store8(dst + i0 + 8 * g, o1);
      store8(dst + half + i0 + 8 * g, o2);
    }
  }
}

#ifndef PG_GROUP_M
#define PG_GROUP_M 4
#endif
// Work item -> (row block m, column tile n).  Items run in groups of kGroupM row blocks: inside a
// group the column tile advances every kGroupM items, so the CTAs in flight share a few Wp tiles and
// a few x row blocks, and Wp stays resident in L2 from one group to the next.
constexpr int kGroupM = PG_GROUP_M;
__device__ __forceinline__ void tile_of(const Params& p, int64_t item, int& m, int& n) {
  const int64_t per_group = (int64_t)kGroupM * p.n_tiles;
  const int64_t g = item / per_group, r = item % per_group;
  const int64_t m0 = g * kGroupM;
  const int64_t rows = min((int64_t)kGroupM, (int64_t)p.m_tiles - m0);  // the last group may be short
  n = (int)(r / rows);
  m = (int)(m0 + r % rows);
}

template <typename TabT>
__global__ void __launch_bounds__(kThreads, 1)
    proj_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint8_t* sA = base;
  uint8_t* sB = base + kStages * kATile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + kStages * kBTile);
  uint64_t* a_full = bars;
  uint64_t* a_empty = bars + kStages;
  uint64_t* t_full = bars + 2 * kStages;
  uint64_t* t_empty = t_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(t_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n_items = (int64_t)p.m_tiles * p.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&t_full[b], 1);
      mbar_init(&t_empty[b], kEpiWarps);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------ TMA producer ------------------------------------
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int64_t item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
        int m, n;
        tile_of(p, item, m, n);
        for (int kb = 0; kb < p.n_kblk; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&a_empty[s], ((it / kStages) & 1u) ^ 1u, p.err)) { ok = false; break; }
          mbar_arrive_expect_tx(&a_full[s], kATile + kBTile);
          tma_load_2d(sA + s * kATile, &tmA, kb * kBK, m * kBM, &a_full[s]);
          tma_load_2d(sB + s * kBTile, &tmB, kb * kBK, n * kBN, &a_full[s]);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------- MMA issuer -------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(kBM, kBN);
      uint32_t it = 0, tc = 0;
      bool ok = true;
      for (int64_t item = blockIdx.x; ok && item < n_items; item += gridDim.x, ++tc) {
        const int buf = tc & 1;
        if (!mbar_wait(&t_empty[buf], ((tc >> 1) & 1u) ^ 1u, p.err)) { ok = false; break; }
        fence_after();
        for (int kb = 0; kb < p.n_kblk; ++kb, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(&a_full[s], (it / kStages) & 1u, p.err)) { ok = false; break; }
          fence_after();
          const uint64_t ad = sw128_desc(smem_u32(sA + s * kATile));
          const uint64_t bd = sw128_desc(smem_u32(sB + s * kBTile));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma(tmem + buf * kBN, ad + 2 * k, bd + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(&a_empty[s]);
        }
        if (!ok) break;
        umma_commit(&t_full[buf]);
      }
      // every MMA must have completed before TMEM is released
      if (tc > 0) mbar_wait(&t_full[(tc - 1) & 1], ((tc - 1) >> 1) & 1u, p.err);
    }
  } else {
    // -------------------------------------- epilogue --------------------------------------
    constexpr int dt = GSA_DTYPE_BF16;
    const int quarter = warp & 3;           // TMEM lane quarter this warp may access
    const int sp = (warp - 2) / 4;          // which 1/kSplit of the tile's columns
    uint32_t tc = 0;
    for (int64_t item = blockIdx.x; item < n_items; item += gridDim.x, ++tc) {
      const int buf = tc & 1;
      if (!mbar_wait(&t_full[buf], (tc >> 1) & 1u, p.err)) break;
      fence_after();
      int m, n;
      tile_of(p, item, m, n);
      const int64_t t = (int64_t)m * kBM + quarter * 32 + lane;
      const bool ok = t < p.T;
      const int64_t tr = ok ? t : p.T - 1;  // rows past T read a valid position, store nothing
      const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + buf * kBN;
      const float* bias = p.bias + (int64_t)n * kBN;
      const int64_t b_of_t = tr / p.L, i_of_t = tr % p.L;
      const int kind = n < p.t_k ? kQ : n < p.t_vg ? kK : n < p.t_g1 ? kVG : n < p.t_idx ? kG1 : kIdx;
      const int D = p.D, half = D / 2;
      if (kind == kQ || kind == kK) {
        int64_t pos = p.positions ? p.positions[tr] : p.pos0 + i_of_t;
        if (pos < 0 || pos >= p.tab_rows) {
          set_error(p.err, GSA_ERR_INDEX);
          pos = pos < 0 ? 0 : p.tab_rows - 1;
        }
        const TabT* cr = reinterpret_cast<const TabT*>(p.cos_tab) + pos * D;
        const TabT* sr = reinterpret_cast<const TabT*>(p.sin_tab) + pos * D;
        // this warp's RoPE pairs (i, i + D/2) of the tile's heads, 32 at a time
        for (int slot = sp * kPairs; slot < (sp + 1) * kPairs; slot += 32) {
          const int hh = slot / half, i0 = slot % half, c0 = hh * D;
          const int h = (n - (kind == kQ ? p.t_q : p.t_k)) * (kBN / D) + hh;
          __nv_bfloat16* dst = kind == kQ ? p.q_out + (tr * p.H + h) * (int64_t)D
                                          : p.k_out + b_of_t * p.kv_bstride + i_of_t * p.kv_ld + (int64_t)h * D;
          rope32<TabT>(taddr, c0 + i0, c0 + half + i0, i0, half, cr, sr, dst, ok);
        }
      } else if (kind == kVG) {
        // [v_h | g2_h] column blocks of D per KV head: this warp's v dims, 32 at a time
        for (int slot = sp * kPairs; slot < (sp + 1) * kPairs; slot += 32) {
          const int pair = slot / D, i0 = slot % D;
          const int h = (n - p.t_vg) * (kBN / (2 * D)) + pair;
          __nv_bfloat16* dst = p.v_out + b_of_t * p.kv_bstride + i_of_t * p.kv_ld + (int64_t)h * D;
          const int cv = pair * 2 * D + i0, cg = cv + D;
          uint32_t rv[32], rg[32];
          tmem_ld32(taddr + cv, rv);
          tmem_ld32(taddr + cg, rg);
          tmem_wait_ld(rv);
          tmem_wait_ld(rg);
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            float v[8], gl[8];
            acc8(rv + 8 * g, nullptr, v);  // v has no bias
            acc8(rg + 8 * g, bias + cg + 8 * g, gl);
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = fmul(v[e], gate_act(gl[e], p.gate_act, dt));
            if (ok) store8(dst + i0 + 8 * g, v);
          }
        }
      } else if (kind == kG1) {
        __nv_bfloat16* dst = p.g1_out + tr * (int64_t)p.H * D + (int64_t)(n - p.t_g1) * kBN;
        for (int c0 = sp * kCols; c0 < (sp + 1) * kCols; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(taddr + c0, r);
          tmem_wait_ld(r);
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            float x[8];
            acc8(r + 8 * g, bias + c0 + 8 * g, x);
#pragma unroll
            for (int e = 0; e < 8; ++e) x[e] = gate_act(x[e], p.gate_act, dt);
            if (ok) store8(dst + c0 + 8 * g, x);
          }
        }
      } else {
        // q^I | k^I | w | padding; every 32-column chunk lies inside one segment
        const int nqi = p.HI * p.dI;
        const int col0 = (n - p.t_idx) * kBN;
        for (int c0 = sp * kCols; c0 < (sp + 1) * kCols; c0 += 32) {
          const int col = col0 + c0;
          if (col >= nqi + p.dI + p.HI) break;
          uint32_t r[32];
          tmem_ld32(taddr + c0, r);
          tmem_wait_ld(r);
          if (col < nqi + p.dI) {
            __nv_bfloat16* dst = col < nqi ? p.qi_out + tr * p.qi_ld + col
                                           : p.ki_out + b_of_t * p.ki_bstride + i_of_t * p.ki_ld + (col - nqi);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              float x[8];
              acc8(r + 8 * g, nullptr, x);  // q^I, k^I have no bias
              if (ok) store8(dst + 8 * g, x);
            }
          } else if (ok) {
            float sum = 0.f;
            for (int j = 0; j < p.HI; ++j) {
              const float xb = __bfloat162float(__float2bfloat16_rn(fadd(__uint_as_float(r[j]), bias[c0 + j])));
              const float w = rnd(sigmoid_precise(xb), dt);
              p.w_out[tr * p.HI + j] = w;
              sum += w;
            }
            p.shift_out[tr] = 0.5f * sum;
          }
        }
      }
      // every TMEM load of this accumulator is done: hand it back to the MMA warp
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&t_empty[buf]);
    }
  }

  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

}  // namespace pg

bool proj_gemm_eligible(const ProjGemmArgs& a) {
  const int D = a.d.d_head, H = a.d.n_heads, Hk = a.d.n_kv_heads, HI = a.d.n_idx_heads, dI = a.d.d_idx;
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) % 16) == 0; };
  auto el16 = [](int64_t x) { return (x * 2) % 16 == 0; };
  return (D == 64 || D == 128) && (H * D) % pg::kBN == 0 && (2 * Hk * D) % pg::kBN == 0 && (Hk * D) % pg::kBN == 0 &&
         dI % 32 == 0 && (HI * dI) % 32 == 0 && HI <= 32 && a.d.d_model % pg::kBK == 0 &&
         a.d.gate_act >= GSA_ACT_SIGMOID && a.d.gate_act <= GSA_ACT_SILU && al16(a.x) && el16(a.x_ld) && al16(a.w) &&
         al16(a.q_out) && al16(a.k_out) && al16(a.v_out) && al16(a.g1_out) && al16(a.qi_out) && al16(a.ki_out) &&
         el16(a.kv_ld) && el16(a.kv_bstride) && el16(a.qi_ld) && el16(a.ki_ld) && el16(a.ki_bstride) &&
         a.T <= 0x7fffffffLL && tc::encode_fn() != nullptr;
}

int64_t proj_gemm_columns(const gsa_dims& d) {
  const int64_t n = (int64_t)d.n_heads * d.d_head * 2 + 3LL * d.n_kv_heads * d.d_head +
                    (int64_t)d.n_idx_heads * d.d_idx + d.d_idx + d.n_idx_heads;
  return (n + pg::kBN - 1) / pg::kBN * pg::kBN;
}

int launch_proj_gemm(const ProjGemmArgs& a, int num_sms, cudaStream_t stream) {
  using namespace pg;
  if (a.T == 0) return GSA_OK;
  const int D = a.d.d_head, H = a.d.n_heads, Hk = a.d.n_kv_heads;
  const int64_t Ncols = proj_gemm_columns(a.d);
  auto enc = tc::encode_fn();
  CUtensorMap tmA, tmB;
  {
    cuuint64_t dims[2] = {(cuuint64_t)a.d.d_model, (cuuint64_t)a.T};
    cuuint64_t strides[1] = {(cuuint64_t)a.x_ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBM};
    cuuint32_t es[2] = {1, 1};
    if (enc(&tmA, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a.x), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return GSA_ERR_BAD_ARG;
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)a.d.d_model, (cuuint64_t)Ncols};
    cuuint64_t strides[1] = {(cuuint64_t)a.d.d_model * 2};
    cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBN};
    cuuint32_t es[2] = {1, 1};
    if (enc(&tmB, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a.w), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return GSA_ERR_BAD_ARG;
  }
  Params p;
  p.T = a.T;
  p.n_kblk = a.d.d_model / kBK;
  p.m_tiles = (int)((a.T + kBM - 1) / kBM);
  p.n_tiles = (int)(Ncols / kBN);
  p.t_q = 0;
  p.t_k = (H * D) / kBN;
  p.t_vg = p.t_k + (Hk * D) / kBN;
  p.t_g1 = p.t_vg + (2 * Hk * D) / kBN;
  p.t_idx = p.t_g1 + (H * D) / kBN;
  p.H = H;
  p.Hk = Hk;
  p.D = D;
  p.HI = a.d.n_idx_heads;
  p.dI = a.d.d_idx;
  p.gate_act = a.d.gate_act;
  p.bias = a.bias;
  p.positions = a.positions;
  p.pos0 = a.pos0;
  p.L = a.L > 0 ? a.L : a.T;
  p.cos_tab = a.cos_tab;
  p.sin_tab = a.sin_tab;
  p.tab_dtype = a.tab_dtype;
  p.tab_rows = a.tab_rows;
  p.q_out = static_cast<__nv_bfloat16*>(a.q_out);
  p.k_out = static_cast<__nv_bfloat16*>(a.k_out);
  p.v_out = static_cast<__nv_bfloat16*>(a.v_out);
  p.kv_ld = a.kv_ld;
  p.kv_bstride = a.L > 0 ? a.kv_bstride : 0;
  p.g1_out = static_cast<__nv_bfloat16*>(a.g1_out);
  p.qi_out = static_cast<__nv_bfloat16*>(a.qi_out);
  p.qi_ld = a.qi_ld;
  p.ki_out = static_cast<__nv_bfloat16*>(a.ki_out);
  p.ki_ld = a.ki_ld;
  p.ki_bstride = a.L > 0 ? a.ki_bstride : 0;
  p.w_out = a.w_out;
  p.shift_out = a.shift_out;
  p.err = a.err;
  const int64_t items = (int64_t)p.m_tiles * p.n_tiles;
  const unsigned grid = (unsigned)std::min<int64_t>(items, num_sms);
  if (a.tab_dtype == GSA_DTYPE_BF16) {
    if (cudaFuncSetAttribute(proj_gemm_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) !=
        cudaSuccess)
      return GSA_ERR_LAUNCH;
    proj_gemm_kernel<__nv_bfloat16><<<grid, kThreads, kSmem, stream>>>(tmA, tmB, p);
  } else {
    if (cudaFuncSetAttribute(proj_gemm_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) !=
        cudaSuccess)
      return GSA_ERR_LAUNCH;
    proj_gemm_kernel<float><<<grid, kThreads, kSmem, stream>>>(tmA, tmB, p);
  }
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

}  // namespace gsa
