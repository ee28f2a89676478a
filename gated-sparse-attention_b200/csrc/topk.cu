// Variance-adaptive top-k selection (adaptive_topk.py:68-193), without sorting.
//
// The reference takes torch.topk(scores, k_eff) sorted descending and keeps sorted position
// p iff p < k_t and the score is finite.  The kept set is exactly "the k_t largest finite
// scores"; order inside the set does not matter to the attention that consumes it.  So:
//
//   gsa_topk_candidates  k_eff largest per row by a 3-pass radix select on the fp32 bit
//                        pattern (11 + 11 + 10 bits), ties broken lower column first,
//                        output compacted in ascending column order.  Variance-independent.
//   gsa_row_variance     unbiased per-row variance from fp64 row sums, rounded to the dtype,
//                        and the deterministic layer-wide sum of the rounded variances.
//   gsa_adaptive_k       k_t in the reference's dtype arithmetic (each op rounded).
//   gsa_select_finalize  k_t largest of each row's candidates, same radix select.
//
// One CTA per row.  Histograms use warp-aggregated shared-memory atomics.
#include "kernels.cuh"

namespace gsa {

constexpr int kSelThreads = 512;
constexpr int kBins = 2048;

// Block-wide exclusive scan of one uint32 per thread; returns the exclusive prefix and
// writes the block total to *total.  `ws` needs kSelThreads/32 + 1 words.
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* ws, uint32_t* total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  uint32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) ws[wid] = x;
  __syncthreads();
  if (wid == 0) {
    uint32_t w = lane < nw ? ws[lane] : 0u;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < nw) ws[lane] = w;  // inclusive warp-total prefix
  }
  __syncthreads();
  uint32_t warp_off = wid > 0 ? ws[wid - 1] : 0u;
  *total = ws[nw - 1];
  __syncthreads();
  return warp_off + x - v;
}

// Row source: either a plain fp32 row, or a candidate list (scores + column ids).
struct RowSrc {
  const float* vals;
  int64_t n;
};

__device__ __forceinline__ bool valid_key(float f) { return !(f == -INFINITY) && !(f != f); }

// Adds the histogram of digit (key >> shift) & mask over elements whose key matches
// `prefix` on the bits above (shift + digit width).  Warp-aggregated atomics.
__device__ void histogram_pass(const RowSrc& src, uint32_t* hist, int shift, uint32_t digit_mask,
                               int prefix_shift, uint32_t prefix, bool use_prefix,
                               uint32_t* finite_count) {
  uint32_t my_finite = 0;
  const int lane = threadIdx.x & 31;
  const int64_t n = src.n;
  const int64_t n_iter = (n + blockDim.x - 1) / blockDim.x;
  for (int64_t it = 0; it < n_iter; ++it) {
    int64_t i = it * blockDim.x + threadIdx.x;
    bool act = false;
    uint32_t digit = 0;
    if (i < n) {
      float f = src.vals[i];
      if (valid_key(f)) {
        uint32_t key = float_key(f);
        ++my_finite;
        if (!use_prefix || (key >> prefix_shift) == prefix) {
          act = true;
          digit = (key >> shift) & digit_mask;
        }
      }
    }
    uint32_t active = __ballot_sync(0xffffffffu, act);
    if (act) {
      uint32_t peers = __match_any_sync(active, digit);
      int leader = __ffs(peers) - 1;
      if (lane == leader) atomicAdd(&hist[digit], (uint32_t)__popc(peers));
    }
  }
  if (finite_count) {
    uint32_t wsum = warp_sum(my_finite);
    if (lane == 0) atomicAdd(finite_count, wsum);
  }
}

// Finds the digit d such that count(digits > d) < K <= count(digits >= d), scanning bins from
// the top.  Writes d and count(digits > d) to out[0..1].
__device__ void find_digit(const uint32_t* hist, int nbins, uint32_t K, uint32_t* ws, uint32_t* out) {
  const int per = (nbins + blockDim.x - 1) / blockDim.x;
  // thread i owns bins [nbins-1 - i*per, ..., nbins - (i+1)*per] (descending)
  uint32_t local = 0;
  for (int j = 0; j < per; ++j) {
    int bin = nbins - 1 - (threadIdx.x * per + j);
    if (bin >= 0) local += hist[bin];
  }
  uint32_t total;
  uint32_t before = block_exclusive_scan(local, ws, &total);
  if (before < K && before + local >= K) {
    uint32_t acc = before;
    for (int j = 0; j < per; ++j) {
      int bin = nbins - 1 - (threadIdx.x * per + j);
      if (bin < 0) break;
      uint32_t c = hist[bin];
      if (acc + c >= K) {
        out[0] = (uint32_t)bin;
        out[1] = acc;
        break;
      }
      acc += c;
    }
  }
  __syncthreads();
}

// Computes the selection threshold of the K largest valid values of `src`:
//   sel[0] = threshold key tau, sel[1] = number of values equal to tau to take (in column
//   order), sel[2] = number of finite values, sel[3] = 1 if every finite value is taken.
__device__ void radix_threshold(const RowSrc& src, uint32_t K, uint32_t* hist, uint32_t* ws,
                                uint32_t* sel) {
  for (int i = threadIdx.x; i < kBins; i += blockDim.x) hist[i] = 0;
  if (threadIdx.x == 0) { sel[2] = 0; sel[3] = 0; }
  __syncthreads();
  histogram_pass(src, hist, 21, 0x7FFu, 0, 0, false, &sel[2]);
  __syncthreads();
  const uint32_t finite = sel[2];
  if (finite <= K) {
    if (threadIdx.x == 0) { sel[0] = 0; sel[1] = 0; sel[3] = 1; }
    __syncthreads();
    return;
  }
  uint32_t* dig = ws + 40;  // two words after the scan scratch
  find_digit(hist, kBins, K, ws, dig);
  uint32_t d1 = dig[0], above1 = dig[1];
  uint32_t K2 = K - above1;
  __syncthreads();
  for (int i = threadIdx.x; i < kBins; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  histogram_pass(src, hist, 10, 0x7FFu, 21, d1, true, nullptr);
  __syncthreads();
  find_digit(hist, kBins, K2, ws, dig);
  uint32_t d2 = dig[0], above2 = dig[1];
  uint32_t K3 = K2 - above2;
  __syncthreads();
  for (int i = threadIdx.x; i < 1024; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  histogram_pass(src, hist, 0, 0x3FFu, 10, (d1 << 11) | d2, true, nullptr);
  __syncthreads();
  find_digit(hist, 1024, K3, ws, dig);
  uint32_t d3 = dig[0], above3 = dig[1];
  if (threadIdx.x == 0) {
    sel[0] = (d1 << 21) | (d2 << 10) | d3;
    sel[1] = K3 - above3;
    sel[3] = 0;
  }
  __syncthreads();
}

// Writes the selected elements (key > tau, plus the first `need_eq` with key == tau in column
// order; or every finite element when take_all) in ascending column order.  Returns the count.
// out_col(i) maps a source position to the column written to out_idx.
template <typename ColMap>
__device__ uint32_t collect(const RowSrc& src, uint32_t tau, uint32_t need_eq, bool take_all,
                            int32_t* out_idx, float* out_score, ColMap out_col, uint32_t* ws,
                            uint32_t cap, uint8_t* out_mask = nullptr) {
  const int64_t n = src.n;
  constexpr int PER = 4;
  const int64_t chunk = (int64_t)blockDim.x * PER;
  uint32_t out_base = 0, eq_seen = 0;
  for (int64_t c0 = 0; c0 < n; c0 += chunk) {
    uint32_t gt_cnt = 0, eq_cnt = 0;
    float v[PER];
    uint8_t kind[PER];  // 0 none, 1 gt, 2 eq
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      int64_t i = c0 + (int64_t)threadIdx.x * PER + j;
      kind[j] = 0;
      v[j] = 0.f;
      if (i < n) {
        float f = src.vals[i];
        v[j] = f;
        if (valid_key(f)) {
          uint32_t key = float_key(f);
          if (take_all || key > tau) { kind[j] = 1; ++gt_cnt; }
          else if (key == tau) { kind[j] = 2; ++eq_cnt; }
        }
      }
    }
    uint32_t packed = gt_cnt | (eq_cnt << 16), total;
    uint32_t pre = block_exclusive_scan(packed, ws, &total);
    uint32_t gt_pre = pre & 0xFFFFu, eq_pre = pre >> 16;
    uint32_t remaining = need_eq > eq_seen ? need_eq - eq_seen : 0u;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      if (kind[j] == 0) continue;
      bool take = kind[j] == 1 || eq_pre < remaining;
      if (take && out_base + gt_pre + min(eq_pre, remaining) < cap) {
        uint32_t pos = out_base + gt_pre + min(eq_pre, remaining);
        int64_t i = c0 + (int64_t)threadIdx.x * PER + j;
        out_idx[pos] = out_col(i);
        if (out_score) out_score[pos] = v[j];
        if (out_mask) out_mask[i] = 1;
      }
      if (kind[j] == 1) ++gt_pre; else ++eq_pre;
    }
    uint32_t gt_tot = total & 0xFFFFu, eq_tot = total >> 16;
    out_base += gt_tot + min(eq_tot, remaining);
    eq_seen += eq_tot;
  }
  return min(out_base, cap);
}

struct IdentityCol {
  __device__ int32_t operator()(int64_t i) const { return (int32_t)i; }
};
struct CandCol {
  const int32_t* cols;
  __device__ int32_t operator()(int64_t i) const { return cols[i]; }
};

// ---------------------------------------------------------------------------------------------
// Bounded-range rows: when every finite score of row r lies in [0, 2 c_r] (sigmoid indexer
// scores: I[t,s] <= sum_j w_tj = 2 c_t), a histogram over kBins equal-width bins of that range
// spreads the row over many bins (the fp32 bit pattern does not: the scores share two or three
// binary exponents).  One pass finds the bin b* holding the k-th largest score; a second pass
// compacts every score in bins >= b* (at most kCap of them) into shared memory, in column
// order; the exact radix select then runs on that small set.  The bin map x -> floor(x * kBins
// / 2c) is monotone, so equal scores share a bin and the top-k set lies inside bins >= b*.
// ---------------------------------------------------------------------------------------------
constexpr int kCap = 8192;

// Bin of x in [0, 2c] -> [0, kBins): the saturating float->uint conversion maps negatives,
// NaN and -inf to 0 and +inf to the top, so the map is monotone on every input.
__device__ __forceinline__ uint32_t lin_bin(float x, float scale) {
  return min(__float2uint_rz(x * scale), (uint32_t)(kBins - 1));
}

// Histogram of the first n scores of a 16-byte aligned row (8 per thread per iteration).
__device__ void linear_histogram(const float* row, int64_t n, float scale, uint32_t* hist) {
  const int64_t n8 = n / 8;
  const float4* row4 = reinterpret_cast<const float4*>(row);
  for (int64_t i = threadIdx.x; i < n8; i += blockDim.x) {
    const float4 a = row4[2 * i], b = row4[2 * i + 1];
    const float e[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) atomicAdd(&hist[lin_bin(e[j], scale)], 1u);
  }
  for (int64_t i = n8 * 8 + threadIdx.x; i < n; i += blockDim.x) atomicAdd(&hist[lin_bin(row[i], scale)], 1u);
}

// Ordered compaction of the finite scores that satisfy `keep` into (vals, cols), 8 consecutive
// scores per thread.  Writes at most kCap of them and returns the full count.
template <typename Keep>
__device__ uint32_t compact_row(const float* row, int64_t n, Keep keep, float* vals, int32_t* cols, uint32_t* ws) {
  constexpr int PER = 16;
  const int64_t chunk = (int64_t)blockDim.x * PER;
  uint32_t base = 0;
  for (int64_t c0 = 0; c0 < n; c0 += chunk) {
    float v[PER];
    const int64_t i0 = c0 + (int64_t)threadIdx.x * PER;
    if (i0 + PER <= n) {
#pragma unroll
      for (int q = 0; q < PER / 4; ++q) {
        const float4 a = *reinterpret_cast<const float4*>(row + i0 + 4 * q);
        v[4 * q] = a.x; v[4 * q + 1] = a.y; v[4 * q + 2] = a.z; v[4 * q + 3] = a.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < PER; ++j) v[j] = (i0 + j < n) ? row[i0 + j] : -INFINITY;
    }
    uint32_t flags = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (keep(v[j]) && valid_key(v[j])) flags |= 1u << j;
    uint32_t total;
    uint32_t pos = base + block_exclusive_scan((uint32_t)__popc(flags), ws, &total);
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      if (flags & (1u << j)) {
        if (pos < (uint32_t)kCap) {
          vals[pos] = v[j];
          cols[pos] = (int32_t)(i0 + j);
        }
        ++pos;
      }
    }
    base += total;
  }
  __syncthreads();
  return base;
}

// ---------------------------------------------------------------------------------------------
// Exact top-K of a small shared-memory set (the survivors of a row, or a row's candidates):
// vals[0..m) finite, in column order.  A 2048-bin histogram over [min, max] finds the bin b* of
// the K-th largest; every value above b* is kept; inside b* the values are ranked exactly
// (value descending, then position) -- b* holds few values unless the set is tie-heavy, in
// which case the 3-pass radix select takes over.  Kept positions are flagged in take[m].
// Returns false if the caller must use the radix select.
// ---------------------------------------------------------------------------------------------
constexpr int kRankCap = 1024;

__device__ bool flag_top_smem(const float* vals, uint32_t m, uint32_t K, uint32_t* hist, uint32_t* ws,
                              uint8_t* take, uint32_t* list, float* red) {
  // min / max
  float lo = INFINITY, hi = -INFINITY;
  for (uint32_t i = threadIdx.x; i < m; i += blockDim.x) {
    lo = fminf(lo, vals[i]);
    hi = fmaxf(hi, vals[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if (lane == 0) { red[wid] = lo; red[32 + wid] = hi; }
  for (int i = threadIdx.x; i < kBins; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  lo = red[0];
  hi = red[32];
  for (int w = 1; w < nw; ++w) { lo = fminf(lo, red[w]); hi = fmaxf(hi, red[32 + w]); }
  if (!(hi > lo)) {
    // one value: the first K positions
    for (uint32_t i = threadIdx.x; i < m; i += blockDim.x) take[i] = i < K;
    __syncthreads();
    return true;
  }
  const float scale = (float)kBins / (hi - lo);
  auto bin = [&](float x) { return min(__float2uint_rz((x - lo) * scale), (uint32_t)(kBins - 1)); };
  for (uint32_t i = threadIdx.x; i < m; i += blockDim.x) atomicAdd(&hist[bin(vals[i])], 1u);
  __syncthreads();
  uint32_t* dig = ws + 40;
  find_digit(hist, kBins, K, ws, dig);
  const uint32_t bstar = dig[0];
  const uint32_t need = K - dig[1];
  const uint32_t e = hist[bstar];
  __syncthreads();
  if (e > (uint32_t)kRankCap) return false;
  // flag everything above b*; list the b* members in position order (8 positions per thread)
  uint32_t base = 0;
  for (uint32_t c0 = 0; c0 < m; c0 += blockDim.x * 8) {
    const uint32_t i0 = c0 + threadIdx.x * 8;
    uint32_t in = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t i = i0 + j;
      if (i < m) {
        const uint32_t b = bin(vals[i]);
        take[i] = b > bstar;
        in |= (uint32_t)(b == bstar) << j;
      }
    }
    uint32_t total;
    uint32_t pos = base + block_exclusive_scan((uint32_t)__popc(in), ws, &total);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (in & (1u << j)) list[pos++] = i0 + j;
    base += total;
  }
  __syncthreads();
  // rank inside b*: value descending, then position ascending
  for (uint32_t a = threadIdx.x; a < e; a += blockDim.x) {
    const uint32_t ia = list[a];
    const float va = vals[ia];
    uint32_t rank = 0;
    for (uint32_t b = 0; b < e; ++b) {
      const float vb = vals[list[b]];
      rank += (vb > va) || (vb == va && b < a);
    }
    if (rank < need) take[ia] = 1;
  }
  __syncthreads();
  return true;
}

// Ordered compaction of the flagged positions: writes out_idx (through col map), out_score and
// out_mask (by position); returns the count.
template <typename ColMap>
__device__ uint32_t collect_flagged(const float* vals, uint32_t m, const uint8_t* take, int32_t* out_idx,
                                    float* out_score, ColMap out_col, uint8_t* out_mask, uint32_t cap, uint32_t* ws) {
  uint32_t base = 0;
  for (uint32_t c0 = 0; c0 < m; c0 += blockDim.x * 8) {
    const uint32_t i0 = c0 + threadIdx.x * 8;
    uint32_t t = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (i0 + j < m && take[i0 + j]) t |= 1u << j;
    uint32_t total;
    uint32_t pos = base + block_exclusive_scan((uint32_t)__popc(t), ws, &total);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (t & (1u << j)) {
        const uint32_t i = i0 + j;
        if (pos < cap) {
          out_idx[pos] = out_col(i);
          if (out_score) out_score[pos] = vals[i];
          if (out_mask) out_mask[i] = 1;
        }
        ++pos;
      }
    }
    base += total;
  }
  return base < cap ? base : cap;
}

struct KeepBins {
  float scale;
  uint32_t bstar;
  __device__ bool operator()(float x) const { return lin_bin(x, scale) >= bstar; }
};
struct KeepAbove {
  float tau;
  __device__ bool operator()(float x) const { return x >= tau; }
};

// The k_eff best candidates of row r (one CTA of kSelThreads threads).  topk_dyn: the dynamic
// shared memory of the bounded path ([kCap] vals, [kCap] cols, flags, tie list).
__device__ void topk_row(int64_t r, int64_t Lq, int64_t n_cols, int64_t q_pos0, int causal, const float* scores,
                         int64_t ld, const float* row_center, const double* row_stats, int32_t k_eff,
                         int64_t out_ld, int32_t* cand_idx, float* cand_score, int32_t* cand_count,
                         uint8_t* topk_dyn) {
  __shared__ uint32_t hist[kBins];
  __shared__ uint32_t ws[48];
  __shared__ uint32_t sel[4];
  int64_t n = n_cols;
  if (causal) n = min(n_cols, q_pos0 + (r % Lq) + 1);
  if (n < 0) n = 0;
  const float* row = scores + r * ld;
  int32_t* oidx = cand_idx + r * out_ld;
  float* osc = cand_score + r * out_ld;
  const uint32_t K = (uint32_t)k_eff;
  RowSrc src{row, n};
  uint32_t cnt = 0;
  bool done = false;
  if (row_center) {
    const float hi = 2.f * row_center[r];
    float* cv = reinterpret_cast<float*>(topk_dyn);
    int32_t* cc = reinterpret_cast<int32_t*>(topk_dyn + kCap * sizeof(float));
    int64_t m = -1;  // number of scores compacted into (cv, cc), -1 = none
    if (n <= (int64_t)K) {
      // every finite score is a candidate
      cnt = collect(src, 0u, 0u, true, oidx, osc, IdentityCol{}, ws, K);
      done = true;
    } else {
      if (row_stats && row_stats[r * 3 + 2] > 0.0) {
        // One pass: a threshold from the row's mean and spread (the indexer's statistics,
        // taken relative to row_center) at the normal quantile of 1.5 K / n.  Retried lower or
        // higher if fewer than K or more than kCap scores pass it.
        const double* st = row_stats + r * 3;
        const double mu_y = st[0] / st[2];
        const double var = st[1] / st[2] - mu_y * mu_y;
        const float sd = (float)sqrt(var > 0.0 ? var : 0.0);
        const float mean = row_center[r] + (float)mu_y;
        const float pt = 1.5f * (float)K / (float)n;
        float tau = pt >= 1.f ? -INFINITY : mean + sd * 1.41421356f * erfinvf(1.f - 2.f * pt);
        for (int attempt = 0; attempt < 3; ++attempt) {
          const uint32_t C = compact_row(row, n, KeepAbove{tau}, cv, cc, ws);
          if (C >= K && C <= (uint32_t)kCap) {
            m = C;
            break;
          }
          if (C < K) tau = attempt == 0 ? tau - sd : -INFINITY;
          else tau = tau + 0.25f * sd;
        }
      }
      if (m < 0 && hi > 0.f && hi < 3.0e38f) {
        // two passes: a histogram over the bounded range finds the bin of the K-th score
        const float scale = (float)kBins / hi;
        for (int i = threadIdx.x; i < kBins; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        linear_histogram(row, n, scale, hist);
        __syncthreads();
        uint32_t* dig = ws + 40;
        find_digit(hist, kBins, K, ws, dig);
        const uint32_t bstar = dig[0];
        const uint32_t C = dig[1] + hist[bstar];
        __syncthreads();
        if (C <= (uint32_t)kCap) m = compact_row(row, n, KeepBins{scale, bstar}, cv, cc, ws);
      }
      if (m >= 0 && m <= kCap) {
        uint8_t* take = reinterpret_cast<uint8_t*>(topk_dyn + 2 * kCap * sizeof(float));
        uint32_t* list = reinterpret_cast<uint32_t*>(take + kCap);
        __shared__ float red[64];
        if ((uint32_t)m <= K) {
          RowSrc s2{cv, m};
          cnt = collect(s2, 0u, 0u, true, oidx, osc, CandCol{cc}, ws, K);
        } else if (flag_top_smem(cv, (uint32_t)m, K, hist, ws, take, list, red)) {
          cnt = collect_flagged(cv, (uint32_t)m, take, oidx, osc, CandCol{cc}, nullptr, K, ws);
        } else {
          RowSrc s2{cv, m};
          radix_threshold(s2, K, hist, ws, sel);
          cnt = collect(s2, sel[0], sel[1], sel[3] != 0, oidx, osc, CandCol{cc}, ws, K);
        }
        done = true;
      }
    }
  }
  if (!done) {
    radix_threshold(src, K, hist, ws, sel);
    cnt = collect(src, sel[0], sel[1], sel[3] != 0, oidx, osc, IdentityCol{}, ws, K);
  }
  if (threadIdx.x == 0) cand_count[r] = (int32_t)cnt;
}

__global__ void __launch_bounds__(kSelThreads) topk_candidates_kernel(
    int64_t Lq, int64_t n_cols, int64_t q_pos0, int causal, const float* scores, int64_t ld,
    const float* row_center, const double* row_stats, int32_t k_eff, int32_t* cand_idx, float* cand_score,
    int32_t* cand_count) {
  extern __shared__ __align__(16) uint8_t topk_dyn[];
  topk_row(blockIdx.x, Lq, n_cols, q_pos0, causal, scores, ld, row_center, row_stats, k_eff, k_eff, cand_idx,
           cand_score, cand_count, topk_dyn);
}

__global__ void __launch_bounds__(kSelThreads) select_finalize_kernel(
    int32_t k_eff, const int32_t* cand_idx, const float* cand_score, const int32_t* cand_count,
    const int32_t* k, int32_t* sel_idx, int64_t sel_ld, int32_t* sel_count, uint8_t* sel_mask, int stage) {
  chain_wait();
  chain_release();
  __shared__ uint32_t hist[kBins];
  __shared__ uint32_t ws[48];
  __shared__ uint32_t sel[4];
  extern __shared__ __align__(16) uint8_t fin_dyn[];  // staged candidates: [k_eff] scores, [k_eff] cols
  const int64_t r = blockIdx.x;
  int32_t c = cand_count[r];
  int32_t kr = k[r];
  if (kr < 0) kr = 0;
  if (kr > sel_ld) kr = (int32_t)sel_ld;  // a row of sel holds at most sel_ld keys
  if (c < 0) c = 0;
  if (c > k_eff) c = k_eff;
  const float* vals = cand_score + r * k_eff;
  const int32_t* cols = cand_idx + r * k_eff;
  uint8_t* mrow = sel_mask ? sel_mask + r * k_eff : nullptr;
  if (mrow)
    for (int i = threadIdx.x; i < k_eff; i += blockDim.x) mrow[i] = 0;
  const bool radix = kr > 0 && kr < c;
  if (radix && stage) {
    // the radix passes re-read the candidates: stage them in shared memory once
    float* sv = reinterpret_cast<float*>(fin_dyn);
    int32_t* si = reinterpret_cast<int32_t*>(fin_dyn + (size_t)k_eff * sizeof(float));
    for (int i = threadIdx.x; i < c; i += blockDim.x) {
      sv[i] = vals[i];
      si[i] = cols[i];
    }
    vals = sv;
    cols = si;
  }
  __syncthreads();
  uint32_t cnt;
  if (kr == 0 || c == 0) {
    cnt = 0;
  } else if (kr >= c) {
    // every candidate is kept: copy in order
    for (int i = threadIdx.x; i < c; i += blockDim.x) {
      sel_idx[r * sel_ld + i] = cols[i];
      if (mrow) mrow[i] = 1;
    }
    cnt = (uint32_t)c;
  } else {
    bool flagged = false;
    if (stage) {
      __shared__ float red[64];
      uint8_t* take = fin_dyn + (size_t)k_eff * 8;
      uint32_t* list = reinterpret_cast<uint32_t*>(take + ((k_eff + 15) / 16) * 16);
      flagged = flag_top_smem(vals, (uint32_t)c, (uint32_t)kr, hist, ws, take, list, red);
      if (flagged)
        cnt = collect_flagged(vals, (uint32_t)c, take, sel_idx + r * sel_ld, nullptr, CandCol{cols}, mrow,
                              (uint32_t)kr, ws);
    }
    if (!flagged) {
      RowSrc src{vals, c};
      radix_threshold(src, (uint32_t)kr, hist, ws, sel);
      cnt = collect(src, sel[0], sel[1], sel[3] != 0, sel_idx + r * sel_ld, nullptr, CandCol{cols}, ws,
                    (uint32_t)kr, mrow);
    }
  }
  if (threadIdx.x == 0) sel_count[r] = (int32_t)cnt;
}

// ---------------------------------------------------------------------------------------------
// Streaming threshold compaction (the layer's candidate pass).  Every finite score of row r at
// or above the threshold tau_r -- the row's normal quantile of 1.25 K / n_r from its
// statistics -- is a survivor; rows of n_r <= cap keep every score.  Survivors are written in ascending column order to cand[r, 0..cap).  A row whose
// survivors are fewer than min(K, n_r) or more than cap goes to fail_list and is selected
// exactly by topk_fallback_kernel.  Either way the row's candidates hold its K best scores, in
// ascending column order, which is all the final selection needs.
//
// Persistent CTAs, three per SM: one producer warp streams each row in 16 KiB chunks through a
// 3-stage shared-memory ring with 1-D bulk copies (the rows are contiguous), continuing across
// rows, so the scores arrive at HBM rate while 8 consumer warps compact.  A chunk's survivors are
// compacted into shared memory first and then copied out with consecutive threads writing
// consecutive positions (scattered per-thread stores cost ~9 sectors per request).  Consumers
// synchronise on a named barrier that excludes the producer.  All waits are bounded.
// ---------------------------------------------------------------------------------------------
constexpr int kCmpConsumers = 256;
constexpr int kCmpThreads = kCmpConsumers + 32;
constexpr int kCmpPer = 16;                              // scores per consumer thread per chunk
constexpr int kCmpChunk = kCmpConsumers * kCmpPer;       // 4096 scores = 16 KiB
constexpr int kCmpStages = 3;
constexpr float kSurvivorFactor = 1.25f;                 // survivors aimed at per needed key
constexpr int kCmpSmem = 256 + kCmpStages * kCmpChunk * 4 + kCmpChunk * 6;  // ring + survivor staging

struct CmpArgs {
  int64_t R, Lq, n_cols, q_pos0;
  int causal;
  const float* scores;
  int64_t ld;
  const float* center;
  const double* stats;
  int32_t K, cap;
  int32_t* idx;
  float* score;
  int32_t* count;
  int32_t* fail_list;
  int32_t* fail_count;
  int* err;
};

__device__ __forceinline__ int64_t cmp_row_cols(const CmpArgs& a, int64_t r) {
  int64_t n = a.n_cols;
  if (a.causal) n = min(a.n_cols, a.q_pos0 + (r % a.Lq) + 1);
  return n < 0 ? 0 : n;
}

__device__ __forceinline__ float cmp_threshold(const CmpArgs& a, int64_t r, int64_t n) {
  if (n <= a.cap) return -INFINITY;
  const double* st = a.stats + r * 3;
  if (!(st[2] > 0.0)) return -INFINITY;  // no statistics: overflows cap, selected exactly
  const double mu_y = st[0] / st[2];
  const double var = st[1] / st[2] - mu_y * mu_y;
  const float sd = (float)sqrt(var > 0.0 ? var : 0.0);
  const float mean = a.center[r] + (float)mu_y;
  const float pt = kSurvivorFactor * (float)a.K / (float)n;
  return pt >= 1.f ? -INFINITY : mean + sd * 1.41421356f * erfinvf(1.f - 2.f * pt);
}

__device__ __forceinline__ void cmp_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kCmpConsumers) : "memory"); }

// Exclusive scan over the consumer threads of four 16-bit counts packed in one 64-bit word (no
// field's total exceeds 16 bits); the scratch alternates between two buffers by the caller.
__device__ __forceinline__ unsigned long long cmp_scan4(unsigned long long v, unsigned long long* ws,
                                                        unsigned long long* total) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  unsigned long long x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) ws[wid] = x;
  cmp_bar();
  unsigned long long off = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < kCmpConsumers / 32; ++w) {
    const unsigned long long c = ws[w];
    if (w < wid) off += c;
    tot += c;
  }
  *total = tot;
  return off + x - v;
}

__global__ void __launch_bounds__(kCmpThreads, 3) threshold_compact_kernel(CmpArgs a) {
  extern __shared__ __align__(128) uint8_t cmp_smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(cmp_smem);
  uint64_t* empty = full + kCmpStages;
  unsigned long long* wsb = reinterpret_cast<unsigned long long*>(empty + kCmpStages);  // 2 x 8
  float* stage = reinterpret_cast<float*>(cmp_smem + 256);
  // a chunk's survivors, in column order: their scores and their columns' offsets in the chunk
  // (16 bits: three CTAs of three stages then fit one SM)
  float* keep_val = stage + kCmpStages * kCmpChunk;                                 // [kCmpChunk]
  uint16_t* keep_off = reinterpret_cast<uint16_t*>(keep_val + kCmpChunk);          // [kCmpChunk]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kCmpStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCmpConsumers / 32);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kCmpConsumers / 32) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int64_t r = blockIdx.x; r < a.R && ok; r += gridDim.x) {
        const int64_t n = cmp_row_cols(a, r);
        const float* row = a.scores + r * a.ld;
        for (int64_t c0 = 0; c0 < n; c0 += kCmpChunk, ++it) {
          const int s = it % kCmpStages;
          if (!mbar_wait(&empty[s], ((it / kCmpStages) & 1u) ^ 1u, a.err)) { ok = false; break; }
          const int64_t cnt = min((int64_t)kCmpChunk, n - c0);
          const uint32_t bytes = (uint32_t)((cnt + 3) / 4 * 16);
          mbar_arrive_expect_tx(&full[s], bytes);
          bulk_g2s(stage + s * kCmpChunk, row + c0, bytes, &full[s]);
        }
      }
      // every copy issued must land before the CTA exits
      const uint32_t first = it > (uint32_t)kCmpStages ? it - (uint32_t)kCmpStages : 0u;
      for (uint32_t i = first; i < it; ++i) mbar_wait(&full[i % kCmpStages], (i / kCmpStages) & 1u, a.err);
    }
    return;
  }

  // ------------------------------ consumers ------------------------------
  uint32_t it = 0, parity = 0;
  bool ok = true;
  for (int64_t r = blockIdx.x; r < a.R; r += gridDim.x) {
    const int64_t n = cmp_row_cols(a, r);
    const float tau = cmp_threshold(a, r, n);
    int32_t* oi = a.idx + r * a.cap;
    float* os = a.score + r * a.cap;
    uint32_t base = 0;
    for (int64_t c0 = 0; c0 < n; c0 += kCmpChunk, ++it) {
      const int s = it % kCmpStages;
      // after a failed wait the warp keeps its place in every barrier but stops waiting
      if (ok && !mbar_wait(&full[s], (it / kCmpStages) & 1u, a.err)) ok = false;
      // Group q of the chunk is columns [q * 1024, (q + 1) * 1024); thread t takes columns
      // 4t .. 4t + 3 of each group, so every float4 read of a warp is 512 contiguous bytes
      // (no bank conflicts).  Column order is (group, thread, element).
      const float4* src = reinterpret_cast<const float4*>(stage + s * kCmpChunk);
      float v[kCmpPer];
#pragma unroll
      for (int q = 0; q < kCmpPer / 4; ++q) {
        const float4 f = src[q * kCmpConsumers + threadIdx.x];
        v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
      }
      const int32_t nn = (int32_t)n;
      uint32_t flags = 0;
      unsigned long long counts = 0;
      if (c0 + kCmpChunk <= n && tau > -INFINITY) {
        // a whole chunk under a finite threshold (the common case): x >= tau alone excludes
        // -inf and NaN, and every column is inside the row
#pragma unroll
        for (int q = 0; q < kCmpPer / 4; ++q) {
          const uint32_t fq = (uint32_t)(v[4 * q] >= tau) | ((uint32_t)(v[4 * q + 1] >= tau) << 1) |
                              ((uint32_t)(v[4 * q + 2] >= tau) << 2) | ((uint32_t)(v[4 * q + 3] >= tau) << 3);
          flags |= fq << (4 * q);
          counts |= (unsigned long long)__popc(fq) << (16 * q);
        }
      } else {
#pragma unroll
        for (int q = 0; q < kCmpPer / 4; ++q) {
          const int32_t col0 = (int32_t)c0 + q * 4 * kCmpConsumers + 4 * (int32_t)threadIdx.x;
          uint32_t fq = 0;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float x = v[4 * q + e];
            if (col0 + e < nn && x >= tau && x > -INFINITY) fq |= 1u << e;  // NaN fails both
          }
          flags |= fq << (4 * q);
          counts |= (unsigned long long)__popc(fq) << (16 * q);
        }
      }
      // release the slot only once every lane's loads have returned (the flags consume them):
      // the next bulk copy into it must not overtake a shared-memory read still in flight
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      unsigned long long tot4;
      const unsigned long long pre4 = cmp_scan4(counts, wsb + (parity & 1u) * 8, &tot4);
      parity ^= 1u;
      uint32_t total = 0;
#pragma unroll
      for (int q = 0; q < kCmpPer / 4; ++q) {
        uint32_t pos = total + (uint32_t)((pre4 >> (16 * q)) & 0xffffu);
        const int32_t col0 = (int32_t)c0 + q * 4 * kCmpConsumers + 4 * (int32_t)threadIdx.x;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (flags & (1u << (4 * q + e))) {
            keep_off[pos] = (uint16_t)(col0 + e - (int32_t)c0);
            keep_val[pos] = v[4 * q + e];
            ++pos;
          }
        }
        total += (uint32_t)((tot4 >> (16 * q)) & 0xffffu);
      }
      cmp_bar();
      // the chunk's survivors go to positions base .. base + total of the row (up to cap)
      const uint32_t lim = base >= (uint32_t)a.cap ? 0u : min(total, (uint32_t)a.cap - base);
      if (ok)
        for (uint32_t i = threadIdx.x; i < lim; i += kCmpConsumers) {
          oi[base + i] = (int32_t)c0 + (int32_t)keep_off[i];
          os[base + i] = keep_val[i];
        }
      base += total;
    }
    if (threadIdx.x == 0) {
      const int64_t need = min((int64_t)a.K, n);
      if ((int64_t)base > a.cap || (int64_t)base < need) a.fail_list[atomicAdd(a.fail_count, 1)] = (int32_t)r;
      a.count[r] = (int32_t)min(base, (uint32_t)a.cap);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// The same compaction for few rows (decode: one row per sequence): each row is cut into kFewSegs
// column segments taken by separate CTAs, in two passes over the scores (the second mostly from
// L2): count each segment's survivors, then write them from the segment's offset (the counts of
// the row's earlier segments).  Output identical to threshold_compact_kernel.
// ---------------------------------------------------------------------------------------------
constexpr int kFewThreads = 256;
constexpr int kFewSegsMax = 16;
constexpr int kFewCols = 32;                          // consecutive columns per thread per round
constexpr int kFewRound = kFewThreads * kFewCols;     // 8192 columns

__device__ __forceinline__ void few_segment(const CmpArgs& a, int64_t r, int nseg, int sg, int64_t& n, int64_t& c0,
                                            int64_t& c1) {
  n = cmp_row_cols(a, r);
  // segments of whole 1024-column groups
  const int64_t groups = (n + 1023) / 1024;
  const int64_t per = (groups + nseg - 1) / nseg;
  c0 = min(n, (int64_t)sg * per * 1024);
  c1 = min(n, c0 + per * 1024);
}

// The survivor flags of this thread's kFewCols consecutive columns from c (bit i: column c + i).
__device__ __forceinline__ uint32_t few_flags(const float* row, int64_t c, int64_t c1, float tau, float (&v)[kFewCols]) {
#pragma unroll
  for (int j = 0; j < kFewCols / 4; ++j) {
    float4 f = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    if (c + 4 * j < c1) f = __ldg(reinterpret_cast<const float4*>(row + c + 4 * j));
    v[4 * j] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w;
  }
  uint32_t fl = 0;
#pragma unroll
  for (int i = 0; i < kFewCols; ++i)
    if (c + i < c1 && v[i] >= tau && v[i] > -INFINITY) fl |= 1u << i;  // NaN fails both
  return fl;
}

__global__ void __launch_bounds__(kFewThreads) compact_few_count_kernel(CmpArgs a, int nseg, int32_t* seg_count) {
  chain_wait();
  chain_release();
  const int64_t r = blockIdx.x;
  const int sg = blockIdx.y;
  if (r == 0 && sg == 0 && threadIdx.x == 0) *a.fail_count = 0;
  int64_t n, c0, c1;
  few_segment(a, r, nseg, sg, n, c0, c1);
  const float tau = cmp_threshold(a, r, n);
  const float* row = a.scores + r * a.ld;
  uint32_t cnt = 0;
  for (int64_t g0 = c0; g0 < c1; g0 += kFewRound) {
    float v[kFewCols];
    cnt += __popc(few_flags(row, g0 + (int64_t)kFewCols * threadIdx.x, c1, tau, v));
  }
  __shared__ uint32_t ws[kFewThreads / 32];
  cnt = warp_sum(cnt);
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = cnt;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t t = 0;
    for (int w = 0; w < kFewThreads / 32; ++w) t += ws[w];
    seg_count[r * kFewSegsMax + sg] = (int32_t)t;
  }
}

__global__ void __launch_bounds__(kFewThreads) compact_few_write_kernel(CmpArgs a, int nseg, const int32_t* seg_count) {
  chain_wait();
  chain_release();
  const int64_t r = blockIdx.x;
  const int sg = blockIdx.y;
  int64_t n, c0, c1;
  few_segment(a, r, nseg, sg, n, c0, c1);
  const float tau = cmp_threshold(a, r, n);
  const float* row = a.scores + r * a.ld;
  uint32_t base = 0, total = 0;
  for (int s2 = 0; s2 < nseg; ++s2) {
    const uint32_t c = (uint32_t)seg_count[r * kFewSegsMax + s2];
    if (s2 < sg) base += c;
    total += c;
  }
  int32_t* oi = a.idx + r * a.cap;
  float* os = a.score + r * a.cap;
  __shared__ uint32_t ws[kFewThreads / 32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  for (int64_t g0 = c0; g0 < c1; g0 += kFewRound) {
    const int64_t c = g0 + (int64_t)kFewCols * threadIdx.x;
    float v[kFewCols];
    const uint32_t fl = few_flags(row, c, c1, tau, v);
    // exclusive prefix of the survivor counts in column order (thread order = column order)
    const uint32_t k = __popc(fl);
    uint32_t x = k;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) ws[wid] = x;
    __syncthreads();
    uint32_t off = 0, tot = 0;
#pragma unroll
    for (int w = 0; w < kFewThreads / 32; ++w) {
      const uint32_t cw = ws[w];
      if (w < wid) off += cw;
      tot += cw;
    }
    __syncthreads();
    uint32_t pos = base + off + x - k;
#pragma unroll
    for (int i = 0; i < kFewCols; ++i)
      if (fl & (1u << i)) {
        if (pos < (uint32_t)a.cap) {
          oi[pos] = (int32_t)(c + i);
          os[pos] = v[i];
        }
        ++pos;
      }
    base += tot;
  }
  if (sg == 0 && threadIdx.x == 0) {
    const int64_t need = min((int64_t)a.K, n);
    if ((int64_t)total > a.cap || (int64_t)total < need) a.fail_list[atomicAdd(a.fail_count, 1)] = (int32_t)r;
    a.count[r] = (int32_t)min(total, (uint32_t)a.cap);
  }
}

// Exact selection (topk_row) of the rows the compaction could not settle.
__global__ void __launch_bounds__(kSelThreads) topk_fallback_kernel(CmpArgs a) {
  chain_wait();
  chain_release();
  extern __shared__ __align__(16) uint8_t topk_dyn[];
  const int32_t nf = *a.fail_count;
  for (int32_t i = blockIdx.x; i < nf; i += gridDim.x) {
    const int64_t r = a.fail_list[i];
    topk_row(r, a.Lq, a.n_cols, a.q_pos0, a.causal, a.scores, a.ld, a.center, a.stats, a.K, a.cap, a.idx,
             a.score, a.count, topk_dyn);
    __syncthreads();
  }
}

int launch_threshold_candidates(int64_t R, int64_t Lq, int64_t n_cols, int64_t q_pos0, int causal,
                                const float* scores, int64_t ld, const float* center, const double* stats,
                                int32_t K, int32_t cap, int32_t* cand_idx, float* cand_score, int32_t* cand_count,
                                int32_t* fail_list, int32_t* fail_count, int32_t* seg_count, int num_sms, int* err,
                                cudaStream_t stream) {
  if (R == 0) return GSA_OK;
  if (R > 0x7fffffffLL || ld % 4 != 0 || (reinterpret_cast<uintptr_t>(scores) % 16) != 0) return GSA_ERR_BAD_ARG;
  CmpArgs a{R, Lq, n_cols, q_pos0, causal, scores, ld, center, stats, K, cap, cand_idx, cand_score, cand_count,
            fail_list, fail_count, err};
  if (seg_count && R < num_sms && R <= 65535) {
    // few rows: about four CTAs per SM in all, and segments of at most one 8192-column round
    // where 16 segments allow it
    const int64_t groups = (n_cols + 1023) / 1024;
    int64_t ns = std::max<int64_t>((groups + 7) / 8, (4LL * num_sms + R - 1) / R);
    ns = std::min<int64_t>(std::min<int64_t>(ns, kFewSegsMax), std::max<int64_t>(1, groups));
    const int nseg = (int)ns;
    const dim3 grid((unsigned)R, (unsigned)nseg);
    // the count kernel also clears the failed-row count
    if (launch_chained(compact_few_count_kernel, grid, dim3(kFewThreads), 0, stream, a, nseg, seg_count) !=
            cudaSuccess ||
        launch_chained(compact_few_write_kernel, grid, dim3(kFewThreads), 0, stream, a, nseg,
                       (const int32_t*)seg_count) != cudaSuccess)
      return GSA_ERR_LAUNCH;
  } else {
    if (cudaMemsetAsync(fail_count, 0, sizeof(int32_t), stream) != cudaSuccess) return GSA_ERR_CUDA;
    if (cudaFuncSetAttribute(threshold_compact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kCmpSmem) !=
        cudaSuccess)
      return GSA_ERR_LAUNCH;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, threshold_compact_kernel, kCmpThreads, kCmpSmem) !=
            cudaSuccess ||
        per_sm < 1)
      return GSA_ERR_LAUNCH;
    int64_t grid = (int64_t)num_sms * per_sm;
    if (grid > R) grid = R;
    threshold_compact_kernel<<<(unsigned)grid, kCmpThreads, kCmpSmem, stream>>>(a);
  }
  if (cudaGetLastError() != cudaSuccess) return GSA_ERR_LAUNCH;
  const size_t dyn = 2 * kCap * sizeof(float) + kCap + kRankCap * sizeof(uint32_t);
  if (cudaFuncSetAttribute(topk_fallback_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn) !=
      cudaSuccess)
    return GSA_ERR_LAUNCH;
  return launch_chained(topk_fallback_kernel, dim3((unsigned)num_sms), dim3(kSelThreads), dyn, stream, a) == cudaSuccess
             ? GSA_OK
             : GSA_ERR_LAUNCH;
}

// ---------------------------------------------------------------------------------------------
// Fused survivor pass, last step.  The tensor-core indexer wrote each row's survivors into one
// segment per key range, in ascending key order; this joins a row's segments in range order
// into its candidate row -- the ascending column order the streaming compaction writes.  A row
// whose segments overflowed their room, or whose survivors number more than cap or fewer than
// min(K, n), goes to fail_list and marks its query block for the exact recomputation (the
// scores of the block into the scratch, then topk_fallback_kernel).  One warp per row.
// ---------------------------------------------------------------------------------------------
struct SegArgs {
  int64_t R, Lq, n_cols, q_pos0;
  int causal;
  SurvivorShape sv;
  const int32_t* seg_idx;
  const float* seg_score;
  const int32_t* seg_cnt;
  int64_t seg_stride, n_ranges;
  int32_t* idx;
  float* score;
  int32_t* count;
  int32_t* fail_list;
  int32_t* fail_count;
  int32_t* blk_flag;  // [R / Lq sequences][blks_per_seq] query blocks that hold a failed row
  int32_t blk_rows;
  int64_t blks_per_seq;
};

constexpr int kConcatThreads = 256;

__global__ void __launch_bounds__(kConcatThreads) seg_concat_kernel(SegArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t r = ((int64_t)blockIdx.x * kConcatThreads + threadIdx.x) >> 5;
  if (r >= a.R) return;
  const int64_t t = r % a.Lq;
  int64_t n = a.causal ? min(a.n_cols, a.q_pos0 + t + 1) : a.n_cols;
  n = n < 0 ? 0 : n;
  const int64_t nr = SurvivorShape::ranges(n);
  const int64_t room = a.sv.seg_cap(n);
  const int32_t* cnt = a.seg_cnt + r * a.n_ranges;
  uint32_t total = 0;
  bool over = false;
  for (int64_t j0 = 0; j0 < nr; j0 += 32) {
    const int32_t c = j0 + lane < nr ? cnt[j0 + lane] : 0;
    over |= c < 0 || (int64_t)c > room;
    total += __reduce_add_sync(0xffffffffu, (uint32_t)max(c, 0));
  }
  over = __any_sync(0xffffffffu, over);
  const int64_t need = min((int64_t)a.sv.K, n);
  if (over || (int64_t)total > a.sv.cap || (int64_t)total < need) {
    if (lane == 0) {
      a.fail_list[atomicAdd(a.fail_count, 1)] = (int32_t)r;
      a.blk_flag[(r / a.Lq) * a.blks_per_seq + t / a.blk_rows] = 1;
      a.count[r] = 0;
    }
    return;
  }
  int32_t* oi = a.idx + r * a.sv.cap;
  float* os = a.score + r * a.sv.cap;
  uint32_t base = 0;
  for (int64_t j0 = 0; j0 < nr; j0 += 32) {
    const uint32_t c = j0 + lane < nr ? (uint32_t)cnt[j0 + lane] : 0u;
    uint32_t x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    const uint32_t excl = base + x - c;
    const int jn = (int)min((int64_t)32, nr - j0);
    for (int jj = 0; jj < jn; ++jj) {
      const uint32_t cj = __shfl_sync(0xffffffffu, c, jj);
      const uint32_t oj = __shfl_sync(0xffffffffu, excl, jj);
      const int64_t src = r * a.seg_stride + (j0 + jj) * room;
      for (uint32_t i = lane; i < cj; i += 32) {
        oi[oj + i] = a.seg_idx[src + i];
        os[oj + i] = a.seg_score[src + i];
      }
    }
    base += __shfl_sync(0xffffffffu, x, 31);
  }
  if (lane == 0) a.count[r] = (int32_t)total;
}

int launch_seg_concat(int64_t R, int64_t Lq, int64_t n_cols, int64_t q_pos0, int causal, const SurvivorShape& sv,
                      const int32_t* seg_idx, const float* seg_score, const int32_t* seg_cnt, int64_t seg_stride,
                      int64_t n_ranges, int32_t* cand_idx, float* cand_score, int32_t* cand_count,
                      int32_t* fail_list, int32_t* fail_count, int32_t* blk_flag, int32_t blk_rows,
                      cudaStream_t stream) {
  if (R == 0) return GSA_OK;
  if (R > 0x7fffffffLL || Lq <= 0 || blk_rows <= 0) return GSA_ERR_BAD_ARG;
  SegArgs a{R, Lq, n_cols, q_pos0, causal, sv, seg_idx, seg_score, seg_cnt, seg_stride, n_ranges,
            cand_idx, cand_score, cand_count, fail_list, fail_count, blk_flag, blk_rows,
            (Lq + blk_rows - 1) / blk_rows};
  const int64_t grid = (R * 32 + kConcatThreads - 1) / kConcatThreads;
  seg_concat_kernel<<<(unsigned)grid, kConcatThreads, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

// Exact selection of the rows in fail_list from the scores in the scratch (rows of failed query
// blocks recomputed there).
int launch_survivor_fallback(int64_t R, int64_t Lq, int64_t n_cols, int64_t q_pos0, int causal,
                             const float* scores, int64_t ld, const float* center, const double* stats, int32_t K,
                             int32_t cap, int32_t* cand_idx, float* cand_score, int32_t* cand_count,
                             int32_t* fail_list, int32_t* fail_count, int num_sms, int* err, cudaStream_t stream) {
  if (R == 0) return GSA_OK;
  if (R > 0x7fffffffLL || ld % 4 != 0 || (reinterpret_cast<uintptr_t>(scores) % 16) != 0) return GSA_ERR_BAD_ARG;
  CmpArgs a{R, Lq, n_cols, q_pos0, causal, scores, ld, center, stats, K, cap, cand_idx, cand_score, cand_count,
            fail_list, fail_count, err};
  const size_t dyn = 2 * kCap * sizeof(float) + kCap + kRankCap * sizeof(uint32_t);
  if (cudaFuncSetAttribute(topk_fallback_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn) !=
      cudaSuccess)
    return GSA_ERR_LAUNCH;
  topk_fallback_kernel<<<(unsigned)num_sms, kSelThreads, dyn, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

// ---------------------------------------------------------------------------------------------
// Final selection, one warp per row (used when no selection mask is asked for).  The k_t best
// of a row's m candidates (ascending columns), ties lower column first, written in ascending
// column order:
//   1. min / max of the scores;
//   2. a 1024-bin histogram over [min, max] in the warp's shared memory: the bin b* holding the
//      k_t-th score; every candidate in a higher bin is kept;
//   3. the cut inside b*: the need-th member under (score desc, position asc), as (v_cut, p_cut).
//      Few members (<= kWarpListCap): ranked exactly from a shared list.  Tie-heavy bins: a radix
//      select over the members' fp32 keys (4 x 8 bits) gives v_cut, an ordered pass p_cut;
//   4. one ordered pass keeps bin > b*, or bin == b* and (v > v_cut, or v == v_cut and position
//      <= p_cut), ranks the kept candidates of each 32 by ballot and stores them coalesced.
// Only warp collectives: no block barriers, 32 rows in flight per SM.
// ---------------------------------------------------------------------------------------------
constexpr int kWarpBins = 1024;
constexpr int kWarpListCap = 256;
constexpr int kWarpSelWarps = 8;
constexpr int kWarpSelSmem = kWarpSelWarps * (kWarpBins * 4 + kWarpListCap * 8);
constexpr int kWarpUnroll = 8;  // loads in flight per lane: each pass walks tiles of 8 x 32 scores

__device__ __forceinline__ float key_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Finds, among hist[0..nb) scanned from the top, the bin where the count from the top reaches K
// (count(bins above) < K <= count(bins >= it)); returns it and the count above it.  nb is a
// multiple of 32; every lane gets the result.
__device__ __forceinline__ void warp_find_bin(const uint32_t* hist, int nb, uint32_t K, uint32_t& bin_out,
                                              uint32_t& above_out) {
  const int lane = threadIdx.x & 31;
  const int per = nb / 32;
  const int top = nb - per * lane - 1;
  uint32_t own = 0;
  for (int j = 0; j < per; ++j) own += hist[top - j];
  uint32_t incl = own;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  const uint32_t excl = incl - own;
  const uint32_t crossing = __ballot_sync(0xffffffffu, excl < K && incl >= K);
  const int src = crossing ? __ffs(crossing) - 1 : 31;
  uint32_t b = 0, above = 0;
  if (lane == src) {
    uint32_t acc = excl;
    for (int j = 0; j < per; ++j) {
      const uint32_t c = hist[top - j];
      b = (uint32_t)(top - j);
      above = acc;
      if (acc + c >= K) break;
      acc += c;
    }
  }
  bin_out = __shfl_sync(0xffffffffu, b, src);
  above_out = __shfl_sync(0xffffffffu, above, src);
}

__global__ void __launch_bounds__(kWarpSelWarps * 32) select_finalize_warp_kernel(
    int64_t R, int32_t cand_ld, const int32_t* cand_idx, const float* cand_score, const int32_t* cand_count,
    const int32_t* k, int32_t* sel_idx, int64_t sel_ld, int32_t* sel_count) {
  chain_wait();
  chain_release();
  extern __shared__ __align__(16) uint8_t wsel_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t* hist = reinterpret_cast<uint32_t*>(wsel_smem) + warp * kWarpBins;
  float* lval = reinterpret_cast<float*>(wsel_smem + kWarpSelWarps * kWarpBins * 4) + warp * 2 * kWarpListCap;
  uint32_t* lpos = reinterpret_cast<uint32_t*>(lval + kWarpListCap);
  const uint32_t lt = (1u << lane) - 1u;
  for (int64_t r = (int64_t)blockIdx.x * kWarpSelWarps + warp; r < R; r += (int64_t)gridDim.x * kWarpSelWarps) {
    int32_t m = cand_count[r];
    m = m < 0 ? 0 : (m > cand_ld ? cand_ld : m);
    int32_t K = k[r];
    K = K < 0 ? 0 : K;
    if ((int64_t)K > sel_ld) K = (int32_t)sel_ld;
    const float* vals = cand_score + r * cand_ld;
    const int32_t* cols = cand_idx + r * cand_ld;
    int32_t* out = sel_idx + r * sel_ld;
    if (K == 0 || m == 0) {
      if (lane == 0) sel_count[r] = 0;
      continue;
    }
    if (K >= m) {
      for (int i = lane; i < m; i += 32) out[i] = cols[i];
      if (lane == 0) sel_count[r] = m;
      continue;
    }
    // 1. range
    float lo = INFINITY, hi = -INFINITY;
    for (int i0 = 0; i0 < m; i0 += 32 * kWarpUnroll) {
      float v[kWarpUnroll];
#pragma unroll
      for (int j = 0; j < kWarpUnroll; ++j) {
        const int i = i0 + j * 32 + lane;
        v[j] = i < m ? vals[i] : vals[0];
      }
#pragma unroll
      for (int j = 0; j < kWarpUnroll; ++j) {
        lo = fminf(lo, v[j]);
        hi = fmaxf(hi, v[j]);
      }
    }
    lo = -warp_max(-lo);
    hi = warp_max(hi);
    float scale = (float)kWarpBins / (hi - lo);
    if (!(hi > lo) || !(scale < INFINITY) || !(scale > 0.f)) scale = 0.f;  // one bin: the cut decides
    auto bin = [&](float x) { return min(__float2uint_rz((x - lo) * scale), (uint32_t)(kWarpBins - 1)); };
    // 2. histogram and the bin of the K-th score
    for (int b = lane; b < kWarpBins; b += 32) hist[b] = 0u;
    __syncwarp();
    for (int i0 = 0; i0 < m; i0 += 32 * kWarpUnroll) {
      float v[kWarpUnroll];
#pragma unroll
      for (int j = 0; j < kWarpUnroll; ++j) {
        const int i = i0 + j * 32 + lane;
        v[j] = i < m ? vals[i] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < kWarpUnroll; ++j)
        if (i0 + j * 32 + lane < m) atomicAdd(&hist[bin(v[j])], 1u);
    }
    __syncwarp();
    uint32_t bstar, above;
    warp_find_bin(hist, kWarpBins, (uint32_t)K, bstar, above);
    const uint32_t need = (uint32_t)K - above;  // >= 1
    const uint32_t e = hist[bstar];
    __syncwarp();
    // 3. the cut inside b*
    float vc = 0.f;
    uint32_t pc = 0;
    if (e <= (uint32_t)kWarpListCap) {
      uint32_t nl = 0;
      for (int i0 = 0; i0 < m; i0 += 32 * kWarpUnroll) {
        float v[kWarpUnroll];
#pragma unroll
        for (int j = 0; j < kWarpUnroll; ++j) {
          const int i = i0 + j * 32 + lane;
          v[j] = i < m ? vals[i] : 0.f;
        }
#pragma unroll
        for (int j = 0; j < kWarpUnroll; ++j) {
          const int i = i0 + j * 32 + lane;
          const bool in = i < m && bin(v[j]) == bstar;
          const uint32_t bal = __ballot_sync(0xffffffffu, in);
          if (in) {
            const uint32_t p = nl + (uint32_t)__popc(bal & lt);
            lval[p] = v[j];
            lpos[p] = (uint32_t)i;
          }
          nl += (uint32_t)__popc(bal);
        }
      }
      __syncwarp();
      bool found = false;
      for (uint32_t a = lane; a < nl; a += 32) {
        const float va = lval[a];
        const uint32_t pa = lpos[a];
        uint32_t rank = 0;
        for (uint32_t b = 0; b < nl; ++b) {
          const float vb = lval[b];
          rank += (vb > va) || (vb == va && lpos[b] < pa);
        }
        if (rank == need - 1) {
          vc = va;
          pc = pa;
          found = true;
        }
      }
      const int src = __ffs(__ballot_sync(0xffffffffu, found)) - 1;
      vc = __shfl_sync(0xffffffffu, vc, src < 0 ? 0 : src);
      pc = __shfl_sync(0xffffffffu, pc, src < 0 ? 0 : src);
    } else {
      // radix select over the members' keys: the need-th largest value among them
      uint32_t prefix = 0, want = need;
      for (int shift = 24; shift >= 0; shift -= 8) {
        for (int b = lane; b < 256; b += 32) hist[b] = 0u;
        __syncwarp();
        const uint32_t pmask = shift == 24 ? 0u : (0xffffffffu << (shift + 8));
        for (int i = lane; i < m; i += 32) {
          const float v = vals[i];
          if (bin(v) != bstar) continue;
          const uint32_t key = float_key(v);
          if ((key & pmask) == (prefix & pmask)) atomicAdd(&hist[(key >> shift) & 0xffu], 1u);
        }
        __syncwarp();
        uint32_t d, ab;
        warp_find_bin(hist, 256, want, d, ab);
        prefix |= d << shift;
        want -= ab;
        __syncwarp();
      }
      vc = key_float(prefix);
      // the want-th member equal to v_cut, in position order
      uint32_t seen = 0;
      for (int i0 = 0; i0 < m; i0 += 32) {
        const int i = i0 + lane;
        const bool eq = i < m && vals[i] == vc && bin(vals[i]) == bstar;
        const uint32_t bal = __ballot_sync(0xffffffffu, eq);
        const uint32_t c = (uint32_t)__popc(bal);
        if (seen + c >= want) {
          // the (want - seen)-th set bit of bal
          uint32_t bb = bal;
          for (uint32_t j = 1; j < want - seen; ++j) bb &= bb - 1u;
          pc = (uint32_t)(i0 + __ffs(bb) - 1);
          break;
        }
        seen += c;
      }
    }
    __syncwarp();
    // 4. ordered output (tiles in order, and chunks of 32 in order within a tile)
    uint32_t base = 0;
    for (int i0 = 0; i0 < m; i0 += 32 * kWarpUnroll) {
      float v[kWarpUnroll];
      int32_t c[kWarpUnroll];
#pragma unroll
      for (int j = 0; j < kWarpUnroll; ++j) {
        const int i = i0 + j * 32 + lane;
        v[j] = i < m ? vals[i] : 0.f;
        c[j] = i < m ? cols[i] : 0;
      }
#pragma unroll
      for (int j = 0; j < kWarpUnroll; ++j) {
        const int i = i0 + j * 32 + lane;
        bool keep = false;
        if (i < m) {
          const uint32_t b = bin(v[j]);
          keep = b > bstar || (b == bstar && (v[j] > vc || (v[j] == vc && (uint32_t)i <= pc)));
        }
        const uint32_t bal = __ballot_sync(0xffffffffu, keep);
        if (keep) {
          const uint32_t p = base + (uint32_t)__popc(bal & lt);
          if (p < (uint32_t)K) out[p] = c[j];
        }
        base += (uint32_t)__popc(bal);
      }
    }
    if (lane == 0) sel_count[r] = (int32_t)min(base, (uint32_t)K);
  }
}

int launch_select_finalize_warp(int64_t R, int32_t cand_ld, const int32_t* cand_idx, const float* cand_score,
                                const int32_t* cand_count, const int32_t* k, int32_t* sel_idx, int64_t sel_ld,
                                int32_t* sel_count, int num_sms, cudaStream_t stream) {
  if (R == 0) return GSA_OK;
  if (cudaFuncSetAttribute(select_finalize_warp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kWarpSelSmem) != cudaSuccess)
    return GSA_ERR_LAUNCH;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, select_finalize_warp_kernel, kWarpSelWarps * 32,
                                                    kWarpSelSmem) != cudaSuccess ||
      per_sm < 1)
    return GSA_ERR_LAUNCH;
  int64_t grid = (int64_t)num_sms * per_sm;
  const int64_t need = (R + kWarpSelWarps - 1) / kWarpSelWarps;
  if (grid > need) grid = need;
  return launch_chained(select_finalize_warp_kernel, dim3((unsigned)grid), dim3(kWarpSelWarps * 32),
                        (size_t)kWarpSelSmem, stream, R, cand_ld, cand_idx, cand_score, cand_count, k, sel_idx, sel_ld,
                        sel_count) == cudaSuccess
             ? GSA_OK
             : GSA_ERR_LAUNCH;
}

// Row statistics of a materialised score matrix: sum, sum of squares, finite count (fp64).
__global__ void row_stats_kernel(int64_t n_cols, const float* scores, int64_t ld, double* stats) {
  const int64_t r = blockIdx.x;
  const float* row = scores + r * ld;
  double s1 = 0.0, s2 = 0.0, c = 0.0;
  for (int64_t i = threadIdx.x; i < n_cols; i += blockDim.x) {
    float f = row[i];
    if (valid_key(f)) {
      double d = f;
      s1 += d;
      s2 += d * d;
      c += 1.0;
    }
  }
  __shared__ double red[3][32];
  s1 = warp_sum(s1); s2 = warp_sum(s2); c = warp_sum(c);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) { red[0][wid] = s1; red[1][wid] = s2; red[2][wid] = c; }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0, b = 0, cc = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) { a += red[0][w]; b += red[1][w]; cc += red[2][w]; }
    stats[r * 3 + 0] += a;
    stats[r * 3 + 1] += b;
    stats[r * 3 + 2] += cc;
  }
}

// Per-row statistics of a materialised score matrix for the entropy and learned adaptive-k methods
// (adaptive_topk.py:84-127), each rounded to the activation dtype as torch rounds its result:
//   out[r] = {valid count, mean, std (unbiased), max of the masked scores (masked entries count as
//             0, over all n_cols entries), softmax entropy of the valid entries}
// with valid = (score != -inf) and the entropy -sum_i p_i log(p_i + 1e-10), p = softmax over the
// valid entries (exp(x - max) times the reciprocal of their sum, as torch's CPU softmax), every
// product and log rounded to the dtype and the sum accumulated in fp32.  One CTA per row, three
// passes over it.
constexpr int kSumThreads = 256;

template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, T* red, Op op) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();  // red may still be read from a previous reduction
  if (lane == 0) red[wid] = v;
  __syncthreads();
  T a = red[0];
  for (int w = 1; w < kSumThreads / 32; ++w) a = op(a, red[w]);
  return a;
}

__global__ void __launch_bounds__(kSumThreads) row_summary_kernel(int64_t n_cols, const float* scores, int64_t ld,
                                                                  int dtype, float* out) {
  __shared__ double redd[kSumThreads / 32];
  __shared__ float redf[kSumThreads / 32];
  const int64_t r = blockIdx.x;
  const float* row = scores + r * ld;
  auto add_d = [](double a, double b) { return a + b; };
  auto add_f = [](float a, float b) { return a + b; };
  auto max_f = [](float a, float b) { return fmaxf(a, b); };
  double s1 = 0.0, s2 = 0.0, c = 0.0;
  float mx = -INFINITY;
  for (int64_t i = threadIdx.x; i < n_cols; i += kSumThreads) {
    const float f = row[i];
    if (f != -INFINITY) {
      s1 += (double)f;
      s2 += (double)f * (double)f;
      c += 1.0;
      mx = fmaxf(mx, f);
    }
  }
  s1 = block_reduce(s1, redd, add_d);
  s2 = block_reduce(s2, redd, add_d);
  c = block_reduce(c, redd, add_d);
  mx = block_reduce(mx, redf, max_f);
  const double N = (double)n_cols;
  // softmax over the valid entries, then sum_i p_i log(p_i + 1e-10) in fp32
  float z = 0.f;
  for (int64_t i = threadIdx.x; i < n_cols; i += kSumThreads) {
    const float f = row[i];
    if (f != -INFINITY) z += expf(f - mx);
  }
  z = block_reduce(z, redf, add_f);
  const float inv_z = 1.0f / z;
  float h = 0.f;
  for (int64_t i = threadIdx.x; i < n_cols; i += kSumThreads) {
    const float f = row[i];
    if (f != -INFINITY) {
      const float pr = rnd(expf(f - mx) * inv_z, dtype);
      const float lp = rnd(logf(rnd(pr + 1e-10f, dtype)), dtype);
      h += rnd(pr * lp, dtype);
    }
  }
  h = block_reduce(h, redf, add_f);
  if (threadIdx.x == 0) {
    float* o = out + r * 5;
    o[0] = (float)c;
    o[1] = rnd((float)(s1 / N), dtype);
    const double var = N > 1.0 ? (s2 - s1 * s1 / N) / (N - 1.0) : (double)NAN;
    o[2] = rnd((float)sqrt(var > 0.0 ? var : (var == var ? 0.0 : var)), dtype);
    o[3] = c < N ? fmaxf(mx, 0.f) : mx;
    o[4] = c > 0.0 ? -rnd(h, dtype) : (float)NAN;
  }
}

// Unbiased variance over all N entries (masked ones count as 0), from sums taken relative to
// a per-row shift c.  With y = x - c: the N - n masked entries have y = -c.
__device__ __forceinline__ double row_var(const double* st, double c, double N) {
  double n = st[2];
  double sy = st[0] - (N - n) * c;
  double syy = st[1] + (N - n) * c * c;
  return (syy - sy * sy / N) / (N - 1.0);
}

constexpr int kVarThreads = 256;

__global__ void row_variance_kernel(int64_t R, double N, int dtype, const double* stats,
                                    const float* shift, float* var_out) {
  const int64_t r = (int64_t)blockIdx.x * kVarThreads + threadIdx.x;
  if (r >= R) return;
  double c = shift ? (double)shift[r] : 0.0;
  var_out[r] = rnd((float)row_var(stats + r * 3, c, N), dtype);
}

// Sum of the rounded per-row variances in a fixed order (one CTA), so the layer mean is
// deterministic: total[0] = sum, total[1] = row count.
__global__ void __launch_bounds__(1024) sum_variance_kernel(int64_t R, const float* var, double* total) {
  __shared__ double red[1024];
  double s = 0;
  for (int64_t i = threadIdx.x; i < R; i += blockDim.x) s += (double)var[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = 512; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) { total[0] = red[0]; total[1] = (double)R; }
}

// k_t in the reference's arithmetic: every op of adaptive_topk.py:96-102,133-136 evaluated in
// fp32 and rounded to the activation dtype, then the min with the valid count in fp32 and
// truncation toward zero (.long()).
__global__ void adaptive_k_kernel(int64_t R, int64_t n_cols, int dtype, gsa_topk_params p,
                                  const float* var, const double* var_total,
                                  const double* stats, int32_t* k_out) {
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= R) return;
  if (!p.use_adaptive) {
    k_out[r] = (int32_t)min((int64_t)p.k_base, n_cols);
    return;
  }
  float mean = rnd(__fdiv_rn((float)var_total[0], (float)var_total[1]), dtype);
  float den = rnd(fadd(mean, 1e-8f), dtype);
  float vn = rnd(__fdiv_rn(var[r], den), dtype);
  float vt = rnd(fmul(vn, p.temperature), dtype);
  float ks = rnd(__fdiv_rn(1.0f, rnd(fadd(1.0f, vt), dtype)), dtype);
  float ka = rnd(fmul((float)p.k_base, rnd(fadd(0.5f, ks), dtype)), dtype);
  float lo = rnd((float)p.k_min, dtype), hi = rnd((float)p.k_max, dtype);
  float kc = fminf(fmaxf(ka, lo), hi);
  if (ka != ka) kc = ka;  // clamp keeps NaN
  float valid = (float)stats[r * 3 + 2];
  float km = (kc != kc) ? kc : fminf(kc, valid);
  int32_t kt;
  if (km != km) kt = 0;
  else kt = (int32_t)truncf(km);
  k_out[r] = kt;
}

// Row variances, their sum and k_t in one CTA for R <= 1024 rows (decode): the same arithmetic
// and the same summation order as row_variance_kernel, sum_variance_kernel and adaptive_k_kernel
// (thread t holds row t; the same 1024-entry tree), so the results are identical bit for bit.
__global__ void __launch_bounds__(1024) variance_adaptive_k_kernel(int64_t R, int64_t n_cols, int dtype,
                                                                   gsa_topk_params p, const double* stats,
                                                                   const float* shift, float* var_out,
                                                                   double* total, int32_t* k_out) {
  chain_wait();
  chain_release();
  __shared__ double red[1024];
  const int t = threadIdx.x;
  const double N = (double)n_cols;
  float v = 0.f;
  if (t < R) {
    const double c = shift ? (double)shift[t] : 0.0;
    v = rnd((float)row_var(stats + (int64_t)t * 3, c, N), dtype);
    var_out[t] = v;
  }
  red[t] = t < R ? (double)v : 0.0;
  __syncthreads();
  for (int o = 512; o > 0; o >>= 1) {
    if (t < o) red[t] += red[t + o];
    __syncthreads();
  }
  if (t == 0) {
    total[0] = red[0];
    total[1] = (double)R;
  }
  __syncthreads();
  if (t >= R) return;
  const double tot[2] = {red[0], (double)R};
  float mean = rnd(__fdiv_rn((float)tot[0], (float)tot[1]), dtype);
  float den = rnd(fadd(mean, 1e-8f), dtype);
  float vn = rnd(__fdiv_rn(v, den), dtype);
  float vt = rnd(fmul(vn, p.temperature), dtype);
  float ks = rnd(__fdiv_rn(1.0f, rnd(fadd(1.0f, vt), dtype)), dtype);
  float ka = rnd(fmul((float)p.k_base, rnd(fadd(0.5f, ks), dtype)), dtype);
  float lo = rnd((float)p.k_min, dtype), hi = rnd((float)p.k_max, dtype);
  float kc = fminf(fmaxf(ka, lo), hi);
  if (ka != ka) kc = ka;
  float valid = (float)stats[(int64_t)t * 3 + 2];
  float km = (kc != kc) ? kc : fminf(kc, valid);
  k_out[t] = (km != km) ? 0 : (int32_t)truncf(km);
}

int launch_variance_adaptive_k(int64_t R, int64_t n_cols, int dtype, const gsa_topk_params& p,
                               const double* stats, const float* shift, float* var_out, double* total,
                               int32_t* k_out, cudaStream_t stream) {
  if (R == 0) return GSA_OK;
  if (R > 1024 || !p.use_adaptive) return GSA_ERR_BAD_ARG;
  return launch_chained(variance_adaptive_k_kernel, dim3(1), dim3(1024), 0, stream, R, n_cols, dtype, p, stats, shift,
                        var_out, total, k_out) == cudaSuccess
             ? GSA_OK
             : GSA_ERR_LAUNCH;
}

// ---------------------------------------------------------------------------------------------
int launch_topk_candidates(int64_t R, int64_t Lq, int64_t n_cols, int64_t q_pos0, int causal,
                           const float* scores, int64_t ld, const float* row_center, const double* row_stats,
                           int32_t k_eff, int32_t* cand_idx, float* cand_score, int32_t* cand_count,
                           cudaStream_t stream) {
  if (R == 0) return GSA_OK;
  if (R > 0x7fffffffLL) return GSA_ERR_BAD_ARG;
  size_t dyn = 0;
  if (row_center) {
    // the float4 loads of the bounded path need 16-byte aligned rows
    if ((reinterpret_cast<uintptr_t>(scores) % 16) != 0 || (ld % 4) != 0) return GSA_ERR_BAD_ARG;
    dyn = 2 * kCap * sizeof(float) + kCap + kRankCap * sizeof(uint32_t);
    if (cudaFuncSetAttribute(topk_candidates_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn) !=
        cudaSuccess)
      return GSA_ERR_LAUNCH;
  }
  topk_candidates_kernel<<<(unsigned)R, kSelThreads, dyn, stream>>>(Lq, n_cols, q_pos0, causal, scores, ld,
                                                                   row_center, row_stats, k_eff, cand_idx,
                                                                   cand_score, cand_count);
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

int launch_select_finalize(int64_t R, int32_t k_eff, const int32_t* cand_idx, const float* cand_score,
                           const int32_t* cand_count, const int32_t* k, int32_t* sel_idx, int64_t sel_ld,
                           int32_t* sel_count, uint8_t* sel_mask, cudaStream_t stream) {
  if (R == 0) return GSA_OK;
  const size_t dyn = (size_t)k_eff * 8 + ((size_t)(k_eff + 15) / 16) * 16 + kRankCap * sizeof(uint32_t);
  const int stage = dyn <= 112 * 1024 ? 1 : 0;
  // static + dynamic shared memory exceeds the 48 KiB default: opt in
  if (stage &&
      cudaFuncSetAttribute(select_finalize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn) !=
          cudaSuccess)
    return GSA_ERR_LAUNCH;
  return launch_chained(select_finalize_kernel, dim3((unsigned)R), dim3(kSelThreads), stage ? dyn : 0, stream, k_eff,
                        cand_idx, cand_score, cand_count, k, sel_idx, sel_ld, sel_count, sel_mask, stage) == cudaSuccess
             ? GSA_OK
             : GSA_ERR_LAUNCH;
}

int launch_row_stats(int64_t R, int64_t n_cols, const float* scores, int64_t ld, double* stats,
                     cudaStream_t stream) {
  if (R == 0) return GSA_OK;
  row_stats_kernel<<<(unsigned)R, 256, 0, stream>>>(n_cols, scores, ld, stats);
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

int launch_row_summary(int64_t R, int64_t n_cols, const float* scores, int64_t ld, int dtype, float* out,
                       cudaStream_t stream) {
  if (R == 0) return GSA_OK;
  row_summary_kernel<<<(unsigned)R, kSumThreads, 0, stream>>>(n_cols, scores, ld, dtype, out);
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

int launch_row_variance(int64_t R, int64_t n_cols, int dtype, const double* stats, const float* shift,
                        float* var_out, double* total, cudaStream_t stream) {
  if (R == 0) return GSA_OK;
  row_variance_kernel<<<(unsigned)((R + kVarThreads - 1) / kVarThreads), kVarThreads, 0, stream>>>(
      R, (double)n_cols, dtype, stats, shift, var_out);
  sum_variance_kernel<<<1, 1024, 0, stream>>>(R, var_out, total);
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

int launch_adaptive_k(int64_t R, int64_t n_cols, int dtype, const gsa_topk_params& p, const float* var,
                      const double* var_total, const double* stats, int32_t* k_out, cudaStream_t stream) {
  if (R == 0) return GSA_OK;
  adaptive_k_kernel<<<(unsigned)((R + 255) / 256), 256, 0, stream>>>(R, n_cols, dtype, p, var, var_total,
                                                                    stats, k_out);
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

}  // namespace gsa
