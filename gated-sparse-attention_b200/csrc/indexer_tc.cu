// Gated lightning indexer on the 5th-generation tensor cores (tcgen05 + TMEM, TMA-fed).
//
//   I[t,s] = sum_j w[t,j] * sigmoid(scale * <qI[t,j,:], kI[s,:]> + b[j])      (gated_indexer.py:114-145)
//
// The one dense contraction of the layer.  Its shape: every query row has H_I heads of d_I = 64
// and all heads share one key vector kI[s] (gated_indexer.py:66-67, 126).  So the MMA is
//
//   D[s, (t,j)] = kI[s, :] . qI[t, j, :]       M = 128 keys, N = 256 (token, head) pairs, K = 64
//
// A = a 128-key tile of kI (16 KiB, TMA, ring of stages), B = the (TOK x H_I) x 64 query block
// of the CTA (32 KiB, loaded once; TOK = 256 / H_I tokens), D in TMEM (256 fp32 columns,
// double-buffered in the 512-column TMEM).  TMEM lane = key, column = token * H_I + head, so an
// epilogue thread owns one key and finds the H_I heads of a token in adjacent columns: the head
// reduction needs no data exchange, and for a fixed token the 32 lanes of a warp hold 32
// consecutive keys, so score stores are coalesced 128-byte rows.
//
// Epilogue (the bound: H_I sigmoids per (t, s) pair, on the MUFU pipe):
//   sigmoid(z) = 0.5 + 0.5 tanh(z / 2)  =>  I[t,s] = c_t + sum_j (w_tj / 2) tanh((scale*acc + b_j) / 2)
// with c_t = sum_j w_tj / 2, i.e. one FFMA, one tanh.approx and one FFMA per (t, s, j).  The
// tanh form's error (< 1e-3 relative on the score) is inside the bf16 parity bar (2e-2); the
// fp32 layer runs on the precise CUDA-core kernel instead.  The epilogue is latency-bound
// (MUFU and TMEM-load latencies), so it runs 16 warps: four per TMEM lane quarter.
//
// Roles (576 threads): warp 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer (one lane),
// warps 2..17 = epilogue (four warps per TMEM lane quarter, each taking a quarter of the tokens).
// Work item (CTA) = one query block x a range of up to kTilesPerCta key tiles; causal tiles
// beyond the block's last query are never visited.  Every wait is bounded.
//
// Three instantiations share this pipeline (Mode): kScores stores every score (and the row
// statistics when asked for); kSample visits every kSampleStride-th key tile and keeps only the
// statistics (the survivor thresholds' estimate); kEmit keeps the statistics and writes the scores
// at or above each row's threshold to the row's segment of the work item's key range, in key
// order, the four lane-quarter warps of a token group exchanging their per-tile counts through
// shared memory.  kEmit serves gsa_indexer_survivors_fused and has a loop of its own, so that the
// other two modes carry none of its code.
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace gsa {

namespace tc {

constexpr int kKeys = 128;          // M: keys per tile (TMEM lanes)
constexpr int kN = 256;             // N: (token, head) pairs per tile
constexpr int kDI = 64;             // K: indexer dim (one 128-byte swizzle atom)
constexpr int kStages = 6;          // kI tile ring
constexpr int kTilesPerCta = 32;    // key tiles per work item
constexpr int kThreads = 576;
constexpr int kEpiWarps = 16;
constexpr int kATileBytes = kKeys * kDI * 2;  // 16 KiB
constexpr int kBTileBytes = kN * kDI * 2;     // 32 KiB
// shared memory: swizzle alignment, B tile, A ring, w / 2, (c, c - shift), barriers, the statistic
// quarters, and (survivor emission) each token's threshold and segment capacity and the per-tile
// survivor counts of the four lane quarters, double-buffered
constexpr int kSmemBytes = 1024 + kBTileBytes + kStages * kATileBytes + kN * 4 + 2 * 64 * 4 + 256 + 4 * 64 * 8 +
                           2 * 64 * 4 + 2 * 4 * 64 * 4;

// What a launch computes.  kScores: every score to the scratch (and the row statistics when asked
// for); kSample: the row statistics only, over every kSampleStride-th key tile (the survivor
// thresholds' estimate); kEmit: the row statistics, and the scores at or above the row's
// threshold written to the row's segment of this key range, in ascending key order.
enum Mode { kScores = 0, kSample = 1, kEmit = 2 };
constexpr int kSampleStride = 16;

struct Params {
  int n_rows;
  int64_t Lkv;
  int64_t q_pos0;
  int causal;
  float half_scale;
  const float* bias;
  const float* w;
  const float* shift;
  float* scores;
  int64_t ld;
  double* row_stats;
  double* stat_part;   // [n_rows, n_ranges, 3] per-key-range partials, or NULL (fp64 atomics)
  int64_t n_ranges;
  int* err;
  const int32_t* blk_mask;    // kScores: query blocks to compute (the others exit at once), or NULL
  const double* samp_stats;   // kEmit: [n_rows, 3] sampled statistics of (score - shift)
  int32_t* seg_idx;           // kEmit: row r, range j at r * seg_stride + j * seg_cap(n_r)
  float* seg_score;
  int32_t* seg_cnt;           // kEmit: [n_rows, n_ranges] survivors of each (row, range), all counted
  int64_t seg_stride;
  SurvivorShape sv;
};

__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One (token, key) of the epilogue: y = sum_j (w_j / 2) tanh((scale * acc_j + b_j) / 2), two heads
// per f32x2 FMA; the score c + y is stored and (y + c - shift) enters the row statistics.  FULL:
// the tile is unmasked for every token, so no per-token check.
template <int HI, bool FULL, int MODE>
__device__ __forceinline__ void epi_token(const uint32_t* r, uint64_t hs2, const uint64_t* hb2, const float* w_t,
                                          float2 cd, bool ok, float* dst, float& s1, float& s2, float& sc) {
  float th[HI];
#pragma unroll
  for (int j = 0; j < HI / 2; ++j) {
    const uint64_t z2 = ffma2(pack2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1])), hs2, hb2[j]);
    float z0, z1;
    unpack2(z2, z0, z1);
    th[2 * j] = tanh_fast(z0);
    th[2 * j + 1] = tanh_fast(z1);
  }
  const float4* w4 = reinterpret_cast<const float4*>(w_t);
  uint64_t y2 = pack2(0.f, 0.f);
#pragma unroll
  for (int j4 = 0; j4 < HI / 4; ++j4) {
    const float4 w = w4[j4];
    y2 = ffma2(pack2(w.x, w.y), pack2(th[4 * j4 + 0], th[4 * j4 + 1]), y2);
    y2 = ffma2(pack2(w.z, w.w), pack2(th[4 * j4 + 2], th[4 * j4 + 3]), y2);
  }
  float ya, yb;
  unpack2(y2, ya, yb);
  const float y = ya + yb;
  if (FULL || ok) {
    if constexpr (MODE == kScores) *dst = cd.x + y;
    if constexpr (MODE == kEmit) sc = cd.x + y;
    const float yy = cd.y + y;
    s1 += yy;
    s2 = fmaf(yy, yy, s2);
  } else if constexpr (MODE == kEmit) {
    sc = -INFINITY;
  }
}

template <int HI, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
    indexer_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmQ, Params p) {
  constexpr int TOK = kN / HI;        // tokens per query block
  constexpr int TOK_Q = TOK / 4;      // tokens per epilogue warp
  constexpr int TOK_PER_LD = 32 / HI; // tokens per 32-column TMEM load
  static_assert(MODE != kEmit || TOK_Q == 8, "survivor emission: 4 lane quarters x 8 tokens fill one warp");
  constexpr int ts = MODE == kSample ? kSampleStride : 1;  // key tiles per visited tile
  extern __shared__ uint8_t smem_raw[];

  // ---- work item ----
  const int blk = blockIdx.y;
  if (MODE == kScores && p.blk_mask && p.blk_mask[blk] == 0) return;
  const int tok0 = blk * TOK;
  const int ntok = min(TOK, p.n_rows - tok0);
  if (ntok <= 0) return;
  const int64_t pos_last = p.q_pos0 + tok0 + ntok - 1;
  const int64_t key_limit = p.causal ? min(p.Lkv, pos_last + 1) : p.Lkv;
  const int tiles_total = (int)((key_limit + (int64_t)kKeys * ts - 1) / ((int64_t)kKeys * ts));
  const int t_begin = blockIdx.x * kTilesPerCta;
  const int t_end = min(tiles_total, t_begin + kTilesPerCta);
  if (t_begin >= t_end) return;
  const int n_my = t_end - t_begin;

  // ---- shared memory carve-up (1024-byte aligned for the swizzled tiles) ----
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* base = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  uint8_t* sB = base;
  uint8_t* sA = base + kBTileBytes;
  float* w_s = reinterpret_cast<float*>(sA + kStages * kATileBytes);  // [TOK][HI] holds w / 2
  float2* cd_s = reinterpret_cast<float2*>(w_s + kN);                // [TOK]  (c_t = sum_j w_tj / 2, c_t - shift_t)
  uint64_t* bars = reinterpret_cast<uint64_t*>(cd_s + 64);
  uint64_t* a_full = bars;
  uint64_t* a_empty = bars + kStages;
  uint64_t* b_full = bars + 2 * kStages;
  uint64_t* t_full = b_full + 1;
  uint64_t* t_empty = t_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(t_empty + 2);
  float2* stat_s = reinterpret_cast<float2*>(bars + 32);  // [4 quarters][TOK] per-warp statistic sums
  float* tau_s = reinterpret_cast<float*>(stat_s + 4 * 64);  // [TOK] survivor threshold
  int32_t* scap_s = reinterpret_cast<int32_t*>(tau_s + 64);  // [TOK] room of the token's segment
  uint32_t* cnt_s = reinterpret_cast<uint32_t*>(scap_s + 64);  // [2][4 quarters][TOK] survivors per tile

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    mbar_init(b_full, 1);
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
  if (warp >= 2) {
    for (int i = threadIdx.x - 64; i < kN; i += kThreads - 64) {
      const int t = i / HI, j = i % HI;
      w_s[i] = (t < ntok) ? 0.5f * p.w[(int64_t)(tok0 + t) * HI + j] : 0.f;
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp >= 2) {
    for (int t = threadIdx.x - 64; t < TOK; t += kThreads - 64) {
      float c = 0.f;
#pragma unroll
      for (int j = 0; j < HI; ++j) c += w_s[t * HI + j];
      cd_s[t] = make_float2(c, (p.shift && t < ntok) ? c - p.shift[tok0 + t] : c);
    }
    if constexpr (MODE == kEmit) {
      // the row's threshold: its normal quantile of K14 / n from the sampled statistics (taken
      // relative to the shift); rows that keep every key, or have no sample, take -inf
      for (int t = threadIdx.x - 64; t < TOK; t += kThreads - 64) {
        float tau = -INFINITY;
        int32_t room = 0;
        if (t < ntok) {
          const int64_t pos = p.q_pos0 + tok0 + t;
          int64_t n = p.causal ? min(p.Lkv, pos + 1) : p.Lkv;
          n = n < 0 ? 0 : n;
          room = (int32_t)p.sv.seg_cap(n);
          if (n > p.sv.cap) {
            const double* st = p.samp_stats + (int64_t)(tok0 + t) * 3;
            if (st[2] > 0.0) {
              const double mu = st[0] / st[2];
              const double var = st[1] / st[2] - mu * mu;
              const float sd = (float)sqrt(var > 0.0 ? var : 0.0);
              const float pt = (float)p.sv.K14 / (float)n;
              if (pt < 1.f)
                tau = (p.shift ? p.shift[tok0 + t] : 0.f) + (float)mu + sd * 1.41421356f * erfinvf(1.f - 2.f * pt);
            }
          }
        }
        tau_s[t] = tau;
        scap_s[t] = room;
      }
    }
  }
  __syncthreads();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------ TMA producer ------------------------------------
    if (lane == 0) {
      mbar_arrive_expect_tx(b_full, kBTileBytes);
      tma_load_3d(sB, &tmQ, 0, 0, tok0, b_full);
      for (int i = 0; i < n_my; ++i) {
        const int s = i % kStages;
        if (!mbar_wait(&a_empty[s], ((i / kStages) & 1) ^ 1, p.err)) break;
        mbar_arrive_expect_tx(&a_full[s], kATileBytes);
        tma_load_2d(sA + s * kATileBytes, &tmK, 0, (t_begin + i) * ts * kKeys, &a_full[s]);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------- MMA issuer -------------------------------------
    if (lane == 0) {
      bool ok = mbar_wait(b_full, 0, p.err);
      const uint64_t bdesc0 = sw128_desc(smem_u32(sB));
      for (int i = 0; ok && i < n_my; ++i) {
        const int s = i % kStages, buf = i & 1;
        if (!mbar_wait(&a_full[s], (i / kStages) & 1, p.err)) break;
        if (!mbar_wait(&t_empty[buf], ((i >> 1) & 1) ^ 1, p.err)) break;
        fence_after();
        const uint64_t adesc0 = sw128_desc(smem_u32(sA + s * kATileBytes));
#pragma unroll
        for (int k = 0; k < kDI / 16; ++k)
          umma(tmem + buf * kN, adesc0 + 2 * k, bdesc0 + 2 * k, idesc_bf16(kKeys, kN), k > 0 ? 1u : 0u);
        umma_commit(&a_empty[s]);
        umma_commit(&t_full[buf]);
      }
      // every MMA must have completed before TMEM is released
      if (n_my > 0) mbar_wait(&t_full[(n_my - 1) & 1], ((n_my - 1) >> 1) & 1, p.err);
    }
  } else {
    // -------------------------------------- epilogue --------------------------------------
    const int ew = warp - 2;
    const int quarter = warp & 3;   // TMEM lane quarter this warp may access
    const int sub = ew >> 2;        // which quarter of the block's tokens
    uint64_t hb2[HI / 2];
#pragma unroll
    for (int j = 0; j < HI / 2; ++j) hb2[j] = pack2(0.5f * p.bias[2 * j], 0.5f * p.bias[2 * j + 1]);
    const uint64_t hs2 = pack2(p.half_scale, p.half_scale);
    float s1[TOK_Q], s2[TOK_Q];
#pragma unroll
    for (int t = 0; t < TOK_Q; ++t) s1[t] = s2[t] = 0.f;
    const int64_t pos0 = p.q_pos0 + tok0;

    if constexpr (MODE != kEmit) {
      // kScores / kSample: one tile after the other, scores stored (kScores) or only summed
      float unused = 0.f;
      for (int i = 0; i < n_my; ++i) {
        const int buf = i & 1;
        if (!mbar_wait(&t_full[buf], (i >> 1) & 1, p.err)) break;
        fence_after();
        const int64_t tile_key0 = (int64_t)(t_begin + i) * ts * kKeys;
        const int64_t key = tile_key0 + quarter * 32 + lane;
        const bool key_ok = key < p.Lkv;
        // the whole tile is unmasked for every token of the block?
        const bool tile_full = (tile_key0 + kKeys <= p.Lkv) && (!p.causal || tile_key0 + kKeys - 1 <= pos0) &&
                               ntok == TOK;
        const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16) + buf * kN + sub * (kN / 4);
        static_assert((kN / 4) / 32 == 2, "two 32-column chunks per warp");
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t r[32];
          tmem_ld32(tbase + c * 32, r);
          tmem_wait_ld(r);
          if (c == 1) {
            // every load of this buffer is done: hand it back to the MMA warp
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&t_empty[buf]);
          }
          float* srow = MODE == kScores ? p.scores + (int64_t)(tok0 + sub * TOK_Q + c * TOK_PER_LD) * p.ld + key
                                        : nullptr;
          // (H_I = 4 keeps the one generic loop: eight tokens per load leave no registers for two)
          if (HI == 8 && tile_full) {
#pragma unroll
            for (int tt = 0; tt < TOK_PER_LD; ++tt) {
              const int tl = c * TOK_PER_LD + tt;  // token within this warp's quarter
              const int ti = sub * TOK_Q + tl;     // token within the block
              epi_token<HI, true, MODE>(r + tt * HI, hs2, hb2, w_s + ti * HI, cd_s[ti], true,
                                        srow + tt * p.ld, s1[tl], s2[tl], unused);
            }
          } else {
#pragma unroll
            for (int tt = 0; tt < TOK_PER_LD; ++tt) {
              const int tl = c * TOK_PER_LD + tt;
              const int ti = sub * TOK_Q + tl;
              const bool ok = key_ok && ti < ntok && (!p.causal || key <= pos0 + ti);
              epi_token<HI, false, MODE>(r + tt * HI, hs2, hb2, w_s + ti * HI, cd_s[ti], ok, srow + tt * p.ld,
                                         s1[tl], s2[tl], unused);
            }
          }
        }
      }
    } else {
      float sc[TOK_Q];               // this key's score for each token (-inf: masked)
      uint32_t seg_n[TOK_Q];         // survivors of each token in this range so far
#pragma unroll
      for (int t = 0; t < TOK_Q; ++t) {
        sc[t] = -INFINITY;
        seg_n[t] = 0;
      }
      // after a failed wait the warp keeps its place in every named barrier but stops waiting
      bool alive = true;
      for (int i = 0; i < n_my; ++i) {
        const int buf = i & 1;
        if (alive && !mbar_wait(&t_full[buf], (i >> 1) & 1, p.err)) alive = false;
        const int64_t tile_key0 = (int64_t)(t_begin + i) * kKeys;
        const int64_t key = tile_key0 + quarter * 32 + lane;
        if (alive) {
          fence_after();
          const bool key_ok = key < p.Lkv;
          const bool tile_full = (tile_key0 + kKeys <= p.Lkv) && (!p.causal || tile_key0 + kKeys - 1 <= pos0) &&
                                 ntok == TOK;
          const uint32_t tbase = tmem + ((uint32_t)(quarter * 32) << 16) + buf * kN + sub * (kN / 4);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            uint32_t r[32];
            tmem_ld32(tbase + c * 32, r);
            tmem_wait_ld(r);
            if (c == 1) {
              fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&t_empty[buf]);
            }
            if (tile_full) {
#pragma unroll
              for (int tt = 0; tt < TOK_PER_LD; ++tt) {
                const int tl = c * TOK_PER_LD + tt;
                const int ti = sub * TOK_Q + tl;
                epi_token<HI, true, MODE>(r + tt * HI, hs2, hb2, w_s + ti * HI, cd_s[ti], true, nullptr, s1[tl],
                                          s2[tl], sc[tl]);
              }
            } else {
#pragma unroll
              for (int tt = 0; tt < TOK_PER_LD; ++tt) {
                const int tl = c * TOK_PER_LD + tt;
                const int ti = sub * TOK_Q + tl;
                const bool ok = key_ok && ti < ntok && (!p.causal || key <= pos0 + ti);
                epi_token<HI, false, MODE>(r + tt * HI, hs2, hb2, w_s + ti * HI, cd_s[ti], ok, nullptr, s1[tl],
                                           s2[tl], sc[tl]);
              }
            }
          }
        }
        // This tile's survivors, written to each token's segment in key order: lane quarter q's
        // keys follow quarters 0..q-1 of the same tile.  The four warps of a token group (same
        // sub, quarters 0..3) exchange their per-token counts through shared memory (two
        // buffers, one named barrier per tile).
        uint32_t bal[TOK_Q];
#pragma unroll
        for (int tl = 0; tl < TOK_Q; ++tl) {
          const float v = sc[tl];
          bal[tl] = __ballot_sync(0xffffffffu, alive && v >= tau_s[sub * TOK_Q + tl] && v > -INFINITY);
        }
        uint32_t mine = 0;
#pragma unroll
        for (int tl = 0; tl < TOK_Q; ++tl)
          if (lane == tl) mine = (uint32_t)__popc(bal[tl]);
        uint32_t* cs = cnt_s + buf * (4 * TOK);
        if (lane < TOK_Q) cs[quarter * TOK + sub * TOK_Q + lane] = mine;
        asm volatile("bar.sync %0, 128;" ::"r"(2 + sub) : "memory");
        // lane l = 8 q + t holds quarter q's count of token t; inclusive scan over the quarters
        uint32_t x = cs[(lane >> 3) * TOK + sub * TOK_Q + (lane & 7)];
        uint32_t y = __shfl_up_sync(0xffffffffu, x, 8);
        if (lane >= 8) x += y;
        y = __shfl_up_sync(0xffffffffu, x, 16);
        if (lane >= 16) x += y;
        const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
        for (int tl = 0; tl < TOK_Q; ++tl) {
          const uint32_t tot = __shfl_sync(0xffffffffu, x, 24 + tl);
          const uint32_t below = __shfl_sync(0xffffffffu, x, quarter > 0 ? (quarter - 1) * 8 + tl : tl);
          if ((bal[tl] >> lane) & 1u) {
            const int ti = sub * TOK_Q + tl;
            const uint32_t pos = seg_n[tl] + (quarter > 0 ? below : 0u) + (uint32_t)__popc(bal[tl] & lt);
            const int32_t room = scap_s[ti];
            if (pos < (uint32_t)room) {
              const int64_t o = (int64_t)(tok0 + ti) * p.seg_stride + (int64_t)blockIdx.x * room + pos;
              p.seg_idx[o] = (int32_t)key;
              p.seg_score[o] = sc[tl];
            }
          }
          seg_n[tl] += tot;
        }
      }
      // every survivor of (token, range) counted, also those beyond the segment's room
      if (quarter == 0 && lane < TOK_Q) {
        uint32_t n = 0;
#pragma unroll
        for (int tl = 0; tl < TOK_Q; ++tl)
          if (lane == tl) n = seg_n[tl];
        const int ti = sub * TOK_Q + lane;
        if (ti < ntok) p.seg_cnt[(int64_t)(tok0 + ti) * p.n_ranges + blockIdx.x] = (int32_t)n;
      }
    }
    // row statistics: reduce the 32 keys of this warp; then either one fp64 atomic per token and
    // value, or (deterministic) the four lane quarters summed in a fixed order into this CTA's
    // key-range partial of each token
    if (p.row_stats) {
      const int64_t k_lo = (int64_t)t_begin * kKeys;
      const int64_t k_hi = min((int64_t)t_end * kKeys, p.Lkv);
#pragma unroll
      for (int tl = 0; tl < TOK_Q; ++tl) {
        float a = s1[tl], b = s2[tl];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          a += __shfl_xor_sync(0xffffffffu, a, o);
          b += __shfl_xor_sync(0xffffffffu, b, o);
        }
        const int ti = sub * TOK_Q + tl;
        if (p.stat_part) {
          if (lane == 0) stat_s[quarter * TOK + ti] = make_float2(a, b);
        } else if (lane == 0 && ti < ntok) {
          double* st = p.row_stats + (int64_t)(tok0 + ti) * 3;
          atomicAdd(st + 0, (double)a);
          atomicAdd(st + 1, (double)b);
          if (quarter == 0) {
            int64_t cnt = 0;
            if constexpr (MODE == kSample) {
              // valid keys of the visited tiles (every ts-th tile from t_begin)
              const int64_t lim = p.causal ? min(p.Lkv, pos0 + ti + 1) : p.Lkv;
              for (int t = t_begin; t < t_end; ++t) {
                const int64_t c = lim - (int64_t)t * ts * kKeys;
                cnt += c <= 0 ? 0 : (c > kKeys ? kKeys : c);
              }
            } else {
              const int64_t hi_k = p.causal ? min(k_hi, pos0 + ti + 1) : k_hi;
              cnt = hi_k > k_lo ? hi_k - k_lo : 0;
            }
            atomicAdd(st + 2, (double)cnt);
          }
        }
      }
      if (p.stat_part) {
        asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory");  // the epilogue warps only
        const int ti = threadIdx.x - 64;
        if (ti < ntok) {
          double a = 0.0, b = 0.0;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 v = stat_s[q * TOK + ti];
            a += (double)v.x;
            b += (double)v.y;
          }
          const int64_t hi_k = p.causal ? min(k_hi, pos0 + ti + 1) : k_hi;
          double* pt = p.stat_part + ((int64_t)(tok0 + ti) * p.n_ranges + blockIdx.x) * 3;
          pt[0] = a;
          pt[1] = b;
          pt[2] = (double)(hi_k > k_lo ? hi_k - k_lo : 0);
        }
      }
    }
  }

  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

// Row statistics from the key-range partials, summed in range order (the same order every run):
// row_stats[r] += sum_j part[r][j].  Ranges a causal row never reached hold zeros.
__global__ void stat_reduce_kernel(int64_t rows, int64_t n_ranges, const double* part, double* row_stats) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  double a = 0.0, b = 0.0, c = 0.0;
  const double* pr = part + r * n_ranges * 3;
  for (int64_t j = 0; j < n_ranges; ++j) {
    a += pr[3 * j];
    b += pr[3 * j + 1];
    c += pr[3 * j + 2];
  }
  row_stats[r * 3] += a;
  row_stats[r * 3 + 1] += b;
  row_stats[r * 3 + 2] += c;
}

// ---------------------------------------------------------------------------------------------
// host side: tensor maps and launch
// ---------------------------------------------------------------------------------------------
}  // namespace tc

int64_t indexer_tc_stat_ranges(int64_t Lkv) {
  const int64_t tiles = (Lkv + tc::kKeys - 1) / tc::kKeys;
  return (tiles + tc::kTilesPerCta - 1) / tc::kTilesPerCta;
}

bool indexer_tc_eligible(const IdxArgs& a) {
  const bool hi_ok = a.HI == 8 || a.HI == 4;
  const bool al = (reinterpret_cast<uintptr_t>(a.qI) % 16 == 0) && (reinterpret_cast<uintptr_t>(a.kI) % 16 == 0) &&
                  ((a.qi_ld * 2) % 16 == 0) && ((a.ki_ld * 2) % 16 == 0);
  return a.dtype == GSA_DTYPE_BF16 && a.dI == tc::kDI && hi_ok && a.act == GSA_ACT_SIGMOID && al &&
         !a.write_masked && a.Lq <= 0x7fffffffLL && a.Lkv <= 0x7fffffffLL && tc::encode_fn() != nullptr;
}

namespace tc {
template <int HI, int MODE>
static int launch_mode(dim3 grid, const CUtensorMap& tmK, const CUtensorMap& tmQ, const Params& p,
                       cudaStream_t stream) {
  if (cudaFuncSetAttribute(indexer_tc_kernel<HI, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) !=
      cudaSuccess)
    return GSA_ERR_LAUNCH;
  indexer_tc_kernel<HI, MODE><<<grid, kThreads, kSmemBytes, stream>>>(tmK, tmQ, p);
  return GSA_OK;
}
}  // namespace tc

// One batch row of the indexer on the tensor cores (B = 1 slice of IdxArgs).
int launch_indexer_tc(const IdxArgs& a, int* err, cudaStream_t stream) {
  return launch_indexer_tc_mode(a, kTcScores, TcSurvivorArgs{}, err, stream);
}

int launch_indexer_tc_mode(const IdxArgs& a, int mode, const TcSurvivorArgs& x, int* err, cudaStream_t stream) {
  using namespace tc;
  if ((mode == kTcSample || mode == kTcEmit) && a.HI != 8) return GSA_ERR_UNSUPPORTED;
  if (mode == kTcEmit && (!x.samp_stats || !x.seg_idx || !x.seg_score || !x.seg_cnt || !a.row_stats || !a.stat_part))
    return GSA_ERR_BAD_ARG;
  if (mode == kTcSample && !a.row_stats) return GSA_ERR_BAD_ARG;
  auto enc = encode_fn();
  CUtensorMap tmK, tmQ;
  {
    cuuint64_t dims[2] = {(cuuint64_t)kDI, (cuuint64_t)a.Lkv};
    cuuint64_t strides[1] = {(cuuint64_t)a.ki_ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)kDI, (cuuint32_t)kKeys};
    cuuint32_t es[2] = {1, 1};
    if (enc(&tmK, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(a.kI), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return GSA_ERR_BAD_ARG;
  }
  const int TOK = kN / a.HI;
  {
    cuuint64_t dims[3] = {(cuuint64_t)kDI, (cuuint64_t)a.HI, (cuuint64_t)a.Lq};
    cuuint64_t strides[2] = {(cuuint64_t)kDI * 2, (cuuint64_t)a.qi_ld * 2};
    cuuint32_t box[3] = {(cuuint32_t)kDI, (cuuint32_t)a.HI, (cuuint32_t)TOK};
    cuuint32_t es[3] = {1, 1, 1};
    if (enc(&tmQ, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(a.qI), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return GSA_ERR_BAD_ARG;
  }
  Params p;
  p.n_rows = (int)a.Lq;
  p.Lkv = a.Lkv;
  p.q_pos0 = a.q_pos0;
  p.causal = a.causal;
  p.half_scale = 0.5f * a.scale;
  p.bias = a.bias;
  p.w = a.w;
  p.shift = a.shift;
  p.scores = mode == kTcScores ? a.scores : nullptr;
  p.ld = a.scores_ld;
  p.row_stats = a.row_stats;
  // the sampled statistics only steer the thresholds: fp64 atomics suffice there
  p.stat_part = (a.row_stats && mode != kTcSample) ? a.stat_part : nullptr;
  p.n_ranges = indexer_tc_stat_ranges(a.Lkv);
  p.err = err;
  p.blk_mask = mode == kTcScores ? x.blk_mask : nullptr;
  p.samp_stats = x.samp_stats;
  p.seg_idx = x.seg_idx;
  p.seg_score = x.seg_score;
  p.seg_cnt = x.seg_cnt;
  p.seg_stride = x.seg_stride;
  p.sv = x.sv;
  const int64_t nb = (a.Lq + TOK - 1) / TOK;
  const int64_t key_limit = a.causal ? std::min<int64_t>(a.Lkv, a.q_pos0 + a.Lq) : a.Lkv;
  const int64_t tile_keys = (int64_t)kKeys * (mode == kTcSample ? kSampleStride : 1);
  const int64_t max_tiles = (key_limit + tile_keys - 1) / tile_keys;
  const int64_t ranges = (max_tiles + kTilesPerCta - 1) / kTilesPerCta;
  if (nb == 0 || ranges == 0) return GSA_OK;
  if (nb > 65535 || ranges > 0x7fffffffLL) return GSA_ERR_BAD_ARG;
  dim3 grid((unsigned)ranges, (unsigned)nb);
  if (p.stat_part &&
      cudaMemsetAsync(p.stat_part, 0, (size_t)a.Lq * p.n_ranges * 3 * sizeof(double), stream) != cudaSuccess)
    return GSA_ERR_CUDA;
  int st;
  if (mode == kTcSample)
    st = launch_mode<8, kSample>(grid, tmK, tmQ, p, stream);
  else if (mode == kTcEmit)
    st = launch_mode<8, kEmit>(grid, tmK, tmQ, p, stream);
  else if (a.HI == 8)
    st = launch_mode<8, kScores>(grid, tmK, tmQ, p, stream);
  else
    st = launch_mode<4, kScores>(grid, tmK, tmQ, p, stream);
  if (st) return st;
  if (cudaGetLastError() != cudaSuccess) return GSA_ERR_LAUNCH;
  if (p.stat_part) {
    stat_reduce_kernel<<<(unsigned)((a.Lq + 255) / 256), 256, 0, stream>>>(a.Lq, p.n_ranges, p.stat_part,
                                                                          a.row_stats);
    if (cudaGetLastError() != cudaSuccess) return GSA_ERR_LAUNCH;
  }
  return GSA_OK;
}

}  // namespace gsa
