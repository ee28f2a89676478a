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
// Roles (576 threads, one CTA per SM, persistent over (row block, column tile) work items):
// warp 0 = TMA producer (x tile 128 x 64 and Wp tile 256 x 64 per stage, 128-byte swizzle),
// warp 1 = TMEM allocator + MMA issuer (one lane; M = 128, N = 256, K = 16 per instruction),
// warps 2-17 = epilogue, four per TMEM lane quarter (each takes a quarter of the tile's columns): a
// thread owns one token row of the tile.  Outputs leave through shared memory and TMA stores.
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
constexpr int kEpiWarps = 16;            // kSplit per TMEM lane quarter, each taking 1/kSplit of the columns
constexpr int kSplit = kEpiWarps / 4;
constexpr int kCols = kBN / kSplit;      // columns of a tile per epilogue warp
constexpr int kPairs = kBN / 2 / kSplit; // v / g2 column pairs of a tile per epilogue warp
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kATile = kBM * kBK * 2;    // 16 KiB
constexpr int kBTile = kBN * kBK * 2;    // 32 KiB
// Output staging: per epilogue warp two 1 KiB buffers, each a 32-row x 16-column bf16 chunk that a
// TMA store writes out (32-byte swizzle), so the epilogue's global writes leave the SM as bulk copies
// instead of one 16-byte store per row per instruction.
constexpr int kStgBytes = 1024;
constexpr int kStaging = kEpiWarps * 2 * kStgBytes;
constexpr int kSmem = 1024 + kStages * (kATile + kBTile) + kStaging + 256;
static_assert(kSmem <= 232448, "shared memory per CTA");

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
  const __nv_bfloat16* cos_tab;  // [tab_rows, D] bf16: the module's RoPE buffers
  const __nv_bfloat16* sin_tab;
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
  // token rows per batch entry of the K / V and k^I tensor maps (T and 1 batch when contiguous)
  int64_t kv_rows, kv_batches, ki_rows, ki_batches;
};

// Tensor maps of the outputs written by TMA stores (box: 16 columns x 32 rows).
struct OutMaps {
  CUtensorMap q;   // [T, H*D]
  CUtensorMap k;   // [batches, rows, Hk*D] (strides kv_bstride, kv_ld)
  CUtensorMap v;
  CUtensorMap g1;  // [T, H*D]
  CUtensorMap qi;  // [T, H_I*d_I] (row stride qi_ld)
  CUtensorMap ki;  // [batches, rows, d_I]
};

// ---- bf16 arithmetic on packed pairs ----
// torch evaluates a bf16 product or sum in fp32 and rounds the result to bf16.  The fp32 product of
// two bf16 values is exact, and an fp32 sum rounded again to bf16 is the correctly rounded bf16 sum
// (24 >= 2 * 8 + 2 significand bits: the double rounding is innocuous), so both equal the correctly
// rounded bf16x2 instructions below, two elements per instruction.
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t badd2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bneg2(uint32_t a) { return a ^ 0x80008000u; }
// two fp32 values rounded to a bf16 pair (lo in the low half)
__device__ __forceinline__ uint32_t bpack(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ float blo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bhi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// 16 accumulator columns (+ bias, NULL: none) as 8 bf16 pairs: the projection values torch stores.
__device__ __forceinline__ void acc16(const uint32_t (&r)[16], const float* bias, uint32_t (&x)[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float lo = __uint_as_float(r[2 * k]), hi = __uint_as_float(r[2 * k + 1]);
    if (bias) {
      const float2 b = reinterpret_cast<const float2*>(bias)[k];
      lo = fadd(lo, b.x);
      hi = fadd(hi, b.y);
    }
    x[k] = bpack(lo, hi);
  }
}

__device__ __forceinline__ void store16(__nv_bfloat16* dst, const uint32_t (&v)[8]) {
  reinterpret_cast<uint4*>(dst)[0] = make_uint4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<uint4*>(dst)[1] = make_uint4(v[4], v[5], v[6], v[7]);
}

__device__ __forceinline__ void load16(const __nv_bfloat16* src, uint32_t (&v)[8]) {
  const uint4 a = reinterpret_cast<const uint4*>(src)[0], b = reinterpret_cast<const uint4*>(src)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int c0, int c1, const void* src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(c0),
               "r"(c1), "r"(smem_u32(src))
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, int c0, int c1, int c2, const void* src) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(map),
               "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(src))
               : "memory");
}

// One warp's output chunk on its way out: rows [t0, t0 + 32) x 16 columns, lane = row.  The chunk is
// written to the warp's next staging buffer in the 32-byte swizzle (16-byte half c of row r at
// r * 32 + (c ^ (r / 4 % 2)) * 16: the eight rows of a shared-memory phase hit distinct banks), then
// lane 0 issues the TMA store.  A buffer is rewritten only after the store issued from it before has
// read it (at most one store group in flight per warp).
struct Stager {
  uint8_t* buf;  // the warp's two buffers
  int next;
  __device__ __forceinline__ uint8_t* put(const uint32_t (&v)[8], int lane) {
    uint8_t* b = buf + next * kStgBytes;
    next ^= 1;
    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
    __syncwarp();
    const int sw = (lane >> 2) & 1;
    *reinterpret_cast<uint4*>(b + lane * 32 + (sw << 4)) = make_uint4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<uint4*>(b + lane * 32 + ((sw ^ 1) << 4)) = make_uint4(v[4], v[5], v[6], v[7]);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    return b;
  }
  __device__ __forceinline__ void store2d(const CUtensorMap* map, int col, int64_t row, const uint32_t (&v)[8],
                                          int lane) {
    uint8_t* b = put(v, lane);
    if (lane == 0) {
      tma_store_2d(map, col, (int)row, b);
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
  }
  __device__ __forceinline__ void store3d(const CUtensorMap* map, int col, int64_t row, int64_t batch,
                                          const uint32_t (&v)[8], int lane) {
    uint8_t* b = put(v, lane);
    if (lane == 0) {
      tma_store_3d(map, col, (int)row, (int)batch, b);
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
  }
};

// The gate activation of 8 bf16 pairs, rounded to bf16, as torch evaluates it.
__device__ __forceinline__ void gate16(uint32_t (&x)[8], int act) {
  constexpr int dt = GSA_DTYPE_BF16;
#pragma unroll
  for (int k = 0; k < 8; ++k) x[k] = bpack(gate_act(blo(x[k]), act, dt), gate_act(bhi(x[k]), act, dt));
}

// RoPE of 16 element pairs (i, i + D/2), i = i0 .. i0+15, of one head: TMEM columns c1 (first half)
// and c2 (second half) of this thread's row, rotate-half with the row's bf16 cos / sin entries
// (cs1 / sn1 at i, cs2 / sn2 at i + D/2):
//   out_i = x_i cos_i - x_{i+D/2} sin_i,   out_{i+D/2} = x_{i+D/2} cos_{i+D/2} + x_i sin_{i+D/2}
// ((x * cos) + (rotate_half(x) * sin), each op rounded to bf16).
__device__ __forceinline__ void rope16(uint32_t taddr, int c1, int c2, const uint32_t (&cs1)[8],
                                       const uint32_t (&sn1)[8], const uint32_t (&cs2)[8], const uint32_t (&sn2)[8],
                                       uint32_t (&x1)[8], uint32_t (&x2)[8]) {
  uint32_t r1[16], r2[16];
  tmem_ld16(taddr + c1, r1);
  tmem_ld16(taddr + c2, r2);
  tmem_wait_ld(r1, r2);
  acc16(r1, nullptr, x1);
  acc16(r2, nullptr, x2);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t a = badd2(bmul2(x1[k], cs1[k]), bmul2(bneg2(x2[k]), sn1[k]));
    const uint32_t b = badd2(bmul2(x2[k], cs2[k]), bmul2(x1[k], sn2[k]));
    x1[k] = a;
    x2[k] = b;
  }
}

// Work item -> (row block m, column tile n).  Items run in groups of kGroupM row blocks: inside a
// group the column tile advances every kGroupM items, so the ~148 CTAs in flight work on about six
// Wp tiles (12 MiB) and the group's 24 x row blocks (24 MiB), both L2-resident while the group sweeps
// the columns; Wp is read from HBM once per group.  Measured at 131072 tokens: 4 row blocks per
// group 9.4 ms, 16: 8.8 ms, 24-32: 8.6-8.7 ms, 64: 9.4 ms (x no longer stays in L2).
constexpr int kGroupM = 24;
__device__ __forceinline__ void tile_of(const Params& p, int64_t item, int& m, int& n) {
  const int64_t per_group = (int64_t)kGroupM * p.n_tiles;
  const int64_t g = item / per_group, r = item % per_group;
  const int64_t m0 = g * kGroupM;
  const int64_t rows = min((int64_t)kGroupM, (int64_t)p.m_tiles - m0);  // the last group may be short
  n = (int)(r / rows);
  m = (int)(m0 + r % rows);
}

__global__ void __launch_bounds__(kThreads, 1)
    proj_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ OutMaps om, Params p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint8_t* sA = base;
  uint8_t* sB = base + kStages * kATile;
  uint8_t* sStg = sB + kStages * kBTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStg + kStaging);
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
    const int quarter = warp & 3;           // TMEM lane quarter this warp may access
    const int sp = (warp - 2) / 4;          // which 1/kSplit of the tile's columns
    Stager stg{sStg + (warp - 2) * 2 * kStgBytes, 0};
    uint32_t tc = 0;
    for (int64_t item = blockIdx.x; item < n_items; item += gridDim.x, ++tc) {
      const int buf = tc & 1;
      if (!mbar_wait(&t_full[buf], (tc >> 1) & 1u, p.err)) break;
      fence_after();
      int m, n;
      tile_of(p, item, m, n);
      const int64_t t0 = (int64_t)m * kBM + quarter * 32;  // this warp's first row
      if (t0 < p.T) {
        const int64_t t = t0 + lane;
        const bool ok = t < p.T;
        const int64_t tr = ok ? t : p.T - 1;  // rows past T read a valid position; TMA clips their stores
        const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + buf * kBN;
        const float* bias = p.bias + (int64_t)n * kBN;
        const int kind = n < p.t_k ? kQ : n < p.t_vg ? kK : n < p.t_g1 ? kVG : n < p.t_idx ? kG1 : kIdx;
        const int D = p.D, half = D / 2;
        // where the warp's 32 rows sit in the K / V (k^I) maps; a group that runs from one sequence into
        // the next (L % 32 != 0, batches not contiguous) is stored row by row instead
        const int64_t kv_i = t0 % p.kv_rows, kv_b = t0 / p.kv_rows;
        const bool kv_bulk = kv_i + 32 <= p.kv_rows || kv_b == p.kv_batches - 1;
        const int64_t ki_i = t0 % p.ki_rows, ki_b = t0 / p.ki_rows;
        const bool ki_bulk = ki_i + 32 <= p.ki_rows || ki_b == p.ki_batches - 1;
        const int64_t b_of_t = tr / p.L, i_of_t = tr % p.L;
        if (kind == kQ || kind == kK) {
          int64_t pos = p.positions ? p.positions[tr] : p.pos0 + i_of_t;
          if (pos < 0 || pos >= p.tab_rows) {
            set_error(p.err, GSA_ERR_INDEX);
            pos = pos < 0 ? 0 : p.tab_rows - 1;
          }
          const __nv_bfloat16* cr = p.cos_tab + pos * D;
          const __nv_bfloat16* sr = p.sin_tab + pos * D;
          // This warp's RoPE pairs: pairs (i, i + D/2), i in [i0, i0 + 16), of every (kSplit / nc)-th head
          // of the tile, so that the warp reads its table entries once for all of its heads.
          const int nc = half / 16;  // 16-pair chunks per head
          const int i0 = (sp % nc) * 16;
          uint32_t cs1[8], sn1[8], cs2[8], sn2[8];
          load16(cr + i0, cs1);
          load16(sr + i0, sn1);
          load16(cr + half + i0, cs2);
          load16(sr + half + i0, sn2);
          for (int hh = sp / nc; hh < kBN / D; hh += kSplit / nc) {
            const int c0 = hh * D;
            const int h = (n - (kind == kQ ? p.t_q : p.t_k)) * (kBN / D) + hh;
            uint32_t x1[8], x2[8];
            rope16(taddr, c0 + i0, c0 + half + i0, cs1, sn1, cs2, sn2, x1, x2);
            if (kind == kQ) {
              stg.store2d(&om.q, h * D + i0, t0, x1, lane);
              stg.store2d(&om.q, h * D + half + i0, t0, x2, lane);
            } else if (kv_bulk) {
              stg.store3d(&om.k, h * D + i0, kv_i, kv_b, x1, lane);
              stg.store3d(&om.k, h * D + half + i0, kv_i, kv_b, x2, lane);
            } else if (ok) {
              __nv_bfloat16* dst = p.k_out + b_of_t * p.kv_bstride + i_of_t * p.kv_ld + (int64_t)h * D;
              store16(dst + i0, x1);
              store16(dst + half + i0, x2);
            }
          }
        } else if (kind == kVG) {
          // [v_h | g2_h] column blocks of D per KV head: v * act(g2), this warp's v dims 16 at a time
          for (int slot = sp * kPairs; slot < (sp + 1) * kPairs; slot += 16) {
            const int pair = slot / D, i0 = slot % D;
            const int h = (n - p.t_vg) * (kBN / (2 * D)) + pair;
            const int cv = pair * 2 * D + i0, cg = cv + D;
            uint32_t rv[16], rg[16];
            tmem_ld16(taddr + cv, rv);
            tmem_ld16(taddr + cg, rg);
            tmem_wait_ld(rv, rg);
            uint32_t v[8], g[8];
            acc16(rv, nullptr, v);  // v has no bias
            acc16(rg, bias + cg, g);
            gate16(g, p.gate_act);
#pragma unroll
            for (int k = 0; k < 8; ++k) v[k] = bmul2(v[k], g[k]);
            if (kv_bulk) {
              stg.store3d(&om.v, h * D + i0, kv_i, kv_b, v, lane);
            } else if (ok) {
              store16(p.v_out + b_of_t * p.kv_bstride + i_of_t * p.kv_ld + (int64_t)h * D + i0, v);
            }
          }
        } else if (kind == kG1) {
          const int cbase = (n - p.t_g1) * kBN;
          for (int c0 = sp * kCols; c0 < (sp + 1) * kCols; c0 += 16) {
            uint32_t r[16];
            tmem_ld16(taddr + c0, r);
            tmem_wait_ld(r);
            uint32_t g[8];
            acc16(r, bias + c0, g);
            gate16(g, p.gate_act);
            stg.store2d(&om.g1, cbase + c0, t0, g, lane);
          }
        } else {
          // q^I | k^I | w | padding; every 16-column chunk lies inside one segment
          const int nqi = p.HI * p.dI;
          const int col0 = (n - p.t_idx) * kBN;
          for (int c0 = sp * kCols; c0 < (sp + 1) * kCols; c0 += 16) {
            const int col = col0 + c0;
            if (col >= nqi + p.dI + p.HI) break;
            uint32_t r[16];
            tmem_ld16(taddr + c0, r);
            tmem_wait_ld(r);
            if (col < nqi + p.dI) {
              uint32_t x[8];
              acc16(r, nullptr, x);  // q^I, k^I have no bias
              if (col < nqi) {
                stg.store2d(&om.qi, col, t0, x, lane);
              } else if (ki_bulk) {
                stg.store3d(&om.ki, col - nqi, ki_i, ki_b, x, lane);
              } else if (ok) {
                store16(p.ki_out + b_of_t * p.ki_bstride + i_of_t * p.ki_ld + (col - nqi), x);
              }
            } else if (ok) {
              constexpr int dt = GSA_DTYPE_BF16;
              float sum = 0.f;
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                if (j < p.HI) {
                  const float xb = __bfloat162float(__float2bfloat16_rn(fadd(__uint_as_float(r[j]), bias[c0 + j])));
                  const float w = rnd(sigmoid_precise(xb), dt);
                  p.w_out[tr * p.HI + j] = w;
                  sum += w;
                }
              }
              p.shift_out[tr] = 0.5f * sum;
            }
          }
        }
      }
      // every TMEM load of this accumulator is done: hand it back to the MMA warp
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&t_empty[buf]);
    }
    // the staging buffers must stay valid until the last stores have completed
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
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
  static_assert(pg::kSplit % 4 == 0, "the RoPE split needs kSplit a multiple of D / 32 for D <= 128");
  return (D == 64 || D == 128) && (H * D) % pg::kBN == 0 && (2 * Hk * D) % pg::kBN == 0 && (Hk * D) % pg::kBN == 0 &&
         dI % 16 == 0 && (HI * dI) % 16 == 0 && HI <= 16 && a.d.d_model % pg::kBK == 0 &&
         a.tab_dtype == GSA_DTYPE_BF16 && a.tab_rows > 0 &&
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
  p.cos_tab = static_cast<const __nv_bfloat16*>(a.cos_tab);
  p.sin_tab = static_cast<const __nv_bfloat16*>(a.sin_tab);
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
  // the row geometry of the K / V and k^I outputs: one run of T rows when the sequences are contiguous
  const int64_t B = a.T / p.L;
  const bool kv_contig = B == 1 || p.kv_bstride == p.L * p.kv_ld;
  const bool ki_contig = B == 1 || p.ki_bstride == p.L * p.ki_ld;
  p.kv_rows = kv_contig ? a.T : p.L;
  p.kv_batches = kv_contig ? 1 : B;
  p.ki_rows = ki_contig ? a.T : p.L;
  p.ki_batches = ki_contig ? 1 : B;
  OutMaps om;
  auto map2d = [&](CUtensorMap* m, void* base, int64_t cols, int64_t rows, int64_t ld) {
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {16, 32};
    cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  };
  auto map3d = [&](CUtensorMap* m, void* base, int64_t cols, int64_t rows, int64_t batches, int64_t ld,
                   int64_t bstride) {
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batches};
    // a single batch entry still needs a valid stride: any multiple of 16 bytes covering the rows
    cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)(batches > 1 ? bstride : rows * ld) * 2};
    cuuint32_t box[3] = {16, 32, 1};
    cuuint32_t es[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  };
  if (!map2d(&om.q, a.q_out, (int64_t)H * D, a.T, (int64_t)H * D) ||
      !map3d(&om.k, a.k_out, (int64_t)Hk * D, p.kv_rows, p.kv_batches, a.kv_ld, p.kv_bstride) ||
      !map3d(&om.v, a.v_out, (int64_t)Hk * D, p.kv_rows, p.kv_batches, a.kv_ld, p.kv_bstride) ||
      !map2d(&om.g1, a.g1_out, (int64_t)H * D, a.T, (int64_t)H * D) ||
      !map2d(&om.qi, a.qi_out, (int64_t)a.d.n_idx_heads * a.d.d_idx, a.T, a.qi_ld) ||
      !map3d(&om.ki, a.ki_out, a.d.d_idx, p.ki_rows, p.ki_batches, a.ki_ld, p.ki_bstride))
    return GSA_ERR_BAD_ARG;
  if (cudaFuncSetAttribute(proj_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
    return GSA_ERR_LAUNCH;
  const int64_t items = (int64_t)p.m_tiles * p.n_tiles;
  const unsigned grid = (unsigned)std::min<int64_t>(items, num_sms);
  proj_gemm_kernel<<<grid, kThreads, kSmem, stream>>>(tmA, tmB, om, p);
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

}  // namespace gsa
