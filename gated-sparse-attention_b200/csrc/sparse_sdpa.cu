// GQA sparse SDPA with the G1 output gate fused into the epilogue
// (gated_sparse_attention.py:234-290, output_gate.py:124-126).
//
// For every row r = (b, t): one set of sel_count[r] key positions is shared by all heads
// (gated_sparse_attention.py:239, 265-266).  A selected key row is the contiguous
// [Hk, D] slice of K (and of V): 2 KiB each at 8 x 128 bf16.  The kernel is HBM-bound on
// those gathers, so it is built around moving whole key rows:
//
//   * producer warps issue 1-D bulk copies (cp.async.bulk, TMA engine) of the selected keys
//     into a shared-memory ring of stages (16 keys per stage), completing on the stage's
//     mbarrier; three groups of two warps take the stages round-robin, each warp issuing half a
//     stage (a single warp's serial per-lane issue was the limit: 1 -> 2 -> 6 warps took the
//     gather from 7.8 to 12.5 TB/s at 128K tokens, most of it served by L2).  With K and V interleaved per key in HBM ([.., Lkv, 2, Hk, D], the layer's
//     layout) a key is ONE contiguous 4 KiB copy: the copy count, not the byte count, is what
//     limits this engine for 2 KiB rows.  A stage slot is [K row | V row | 16 B pad]; the pad
//     makes the ldmatrix reads of 8 consecutive keys conflict free;
//   * one consumer warp per KV group computes S^T = K_g Q_g^T with mma.sync (keys are the M
//     dimension, the n_rep query heads of the group the N dimension), an online softmax in
//     registers, transposes P with movmatrix and accumulates O^T += V_g^T P^T;
//   * the epilogue divides by the softmax sum, multiplies by the G1 gate and stores.
//
// CTAs are persistent (grid = resident CTAs), each walks rows r = blockIdx.x + i * gridDim.x
// and keeps its copy pipeline running across row boundaries.  All waits are bounded.
#include "kernels.cuh"

namespace gsa {

constexpr int kKeysPerStage = 16;
constexpr int kMaxGroups = 3;  // producer groups of two warps
constexpr int kMaxSplits = 8;  // key ranges per row when rows are fewer than CTAs
constexpr int kMaxRowBytes = 16 * 256 * 2;
__device__ __align__(128) uint8_t g_zero_row[2 * kMaxRowBytes];



__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ uint32_t movm_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}
__device__ __forceinline__ void mma_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Key blocks [lo, hi) of split sp of a row with cnt selected keys (blocks of kKeysPerStage).
__device__ __forceinline__ void split_range(int cnt, int sp, int splits, int& lo, int& hi) {
  const int nkb = (cnt + kKeysPerStage - 1) / kKeysPerStage;
  const int per = (nkb + splits - 1) / splits;
  lo = min(nkb, sp * per);
  hi = min(nkb, lo + per);
}

__device__ __forceinline__ int row_count(const SdpaArgs& a, int64_t row) {
  int c = a.sel_count[row];
  if (c < 0) c = 0;
  if (c > a.sel_ld) c = (int)a.sel_ld;
  return c;
}

// One CTA per SM (its copy ring takes the shared memory): telling the compiler so lets it allocate the
// registers for that occupancy (102 instead of 96 at D 128, 14 warps; 81.5 -> 79.5 ms at 128K tokens).
template <int D, int NREP, int MAXW>
__global__ void __launch_bounds__(MAXW * 32, 1) sdpa_tc_kernel(SdpaArgs a) {
  chain_wait();
  chain_release();
  static_assert(D % 16 == 0 && NREP >= 1 && NREP <= 8, "tile shape");
  extern __shared__ __align__(128) uint8_t smem[];
  const int Hk = a.Hk;
  const int row_bytes = Hk * D * 2;
  const int rs = 2 * row_bytes + 16;  // slot: [K row | V row | pad]
  const int stage_bytes = kKeysPerStage * rs;
  const int nst = a.nstages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + nst;
  uint8_t* stages = smem + 256;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t R = a.B * a.Lq;
  const int64_t NW = R * a.splits;  // work items: (row, key range)
  const int H = Hk * NREP;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nst; ++s) {
      mbar_init(&full[s], 2);  // the two producer warps of the stage's group each arrive once
      mbar_init(&empty[s], (uint32_t)Hk);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp >= Hk) {
    // ---------------------------- producer warps ----------------------------
    // a.nprod / 2 producer groups take stages round-robin; the two warps of a group each issue
    // half of a stage's copies.  The bulk-copy issue of one warp (one lane per copy, serially)
    // is what limits a single producer.  Groups <= nstages keeps the parity waits unambiguous:
    // before a group waits on a stage's empty barrier, its own previous wait (groups iterations
    // earlier) guarantees the releases up to 2 * nstages iterations back, so the barrier is at
    // most one phase behind the phase it waits for.
    const int groups = a.nprod / 2;
    const int pw = warp - Hk;
    const int grp = pw >> 1, half = pw & 1;
    uint32_t it = 0;
    bool ok = true;
    for (int64_t wi = blockIdx.x; wi < NW && ok; wi += gridDim.x) {
      const int64_t row = wi / a.splits;
      const int64_t b = row / a.Lq;
      const int cnt = row_count(a, row);
      const int32_t* idx = a.sel_idx + row * a.sel_ld;
      const int64_t kv_row = a.kv_ld * 2;  // bytes between consecutive keys
      const uint8_t* kbase = reinterpret_cast<const uint8_t*>(a.k) + b * a.kv_bstride * 2;
      const uint8_t* vbase = reinterpret_cast<const uint8_t*>(a.v) + b * a.kv_bstride * 2;
      int kb_lo, kb_hi;
      split_range(cnt, (int)(wi % a.splits), a.splits, kb_lo, kb_hi);
      for (int kb = kb_lo; kb < kb_hi; ++kb, ++it) {
        if ((int)(it % groups) != grp) continue;
        const int s = it % nst;
        const uint32_t ph = (it / nst) & 1u;
        // this warp's 8 slots of the stage; with separate K and V, lanes 8-15 copy the V rows.
        // The key index is loaded before the wait for the slot, so that its latency overlaps
        // the wait instead of delaying the refill.
        const int slot = half * 8 + (lane & 7);
        const int key = kb * kKeysPerStage + slot;
        int64_t j = key < cnt ? (int64_t)idx[key] : -1;
        if (!mbar_wait(&empty[s], ph ^ 1u, a.err)) { ok = false; break; }
        if (lane == 0) mbar_arrive_expect_tx(&full[s], (uint32_t)(kKeysPerStage * row_bytes));
        __syncwarp();
        if (key < cnt && (j < 0 || j >= a.Lkv)) {
          set_error(a.err, GSA_ERR_INDEX);
          j = -1;
        }
        uint8_t* dst = stages + s * stage_bytes + slot * rs;
        if (a.interleaved) {
          // one copy per key: K row and V row are adjacent
          if (lane < 8) bulk_g2s(dst, j >= 0 ? kbase + j * kv_row : g_zero_row, (uint32_t)(2 * row_bytes), &full[s]);
        } else if (lane < 8) {
          bulk_g2s(dst, j >= 0 ? kbase + j * kv_row : g_zero_row, (uint32_t)row_bytes, &full[s]);
        } else if (lane < 16) {
          bulk_g2s(dst + row_bytes, j >= 0 ? vbase + j * kv_row : g_zero_row, (uint32_t)row_bytes, &full[s]);
        }
        // few rows (DRAM-latency bound): warm L2 with the keys a.prefetch stages ahead, so that
        // the ring's copies, which hold shared memory until the consumers take them, land sooner
        if (a.prefetch) {
          const int pkey = key + a.prefetch * kKeysPerStage;
          if (pkey < cnt && pkey < kb_hi * kKeysPerStage) {
            const int64_t j2 = idx[pkey];
            if (j2 >= 0 && j2 < a.Lkv) {
              if (a.interleaved) {
                if (lane < 8) bulk_prefetch_l2(kbase + j2 * kv_row, (uint32_t)(2 * row_bytes));
              } else if (lane < 8) {
                bulk_prefetch_l2(kbase + j2 * kv_row, (uint32_t)row_bytes);
              } else if (lane < 16) {
                bulk_prefetch_l2(vbase + j2 * kv_row, (uint32_t)row_bytes);
              }
            }
          }
        }
      }
    }
    // drain: every copy this warp issued must land before the CTA may exit
    const uint32_t first = it > (uint32_t)nst ? it - (uint32_t)nst : 0u;
    for (uint32_t i = first; i < it; ++i)
      if ((int)(i % groups) == grp) mbar_wait(&full[i % nst], (i / nst) & 1u, a.err);
    return;
  }

  // -------------------------------- consumer warps --------------------------------
  const int g = warp;
  const int grp = lane >> 2, tq = lane & 3;
  const int mi = lane >> 3, r8 = lane & 7;
  uint32_t it = 0;
  for (int64_t wi = blockIdx.x; wi < NW; wi += gridDim.x) {
    const int64_t row = wi / a.splits;
    const int cnt = row_count(a, row);
    const __nv_bfloat16* qrow = a.q + (row * H + (int64_t)g * NREP) * D;
    uint32_t qf[D / 16][2];
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      if (grp < NREP) {
        qf[kk][0] = *reinterpret_cast<const uint32_t*>(qrow + grp * D + kk * 16 + tq * 2);
        qf[kk][1] = *reinterpret_cast<const uint32_t*>(qrow + grp * D + kk * 16 + tq * 2 + 8);
      } else {
        qf[kk][0] = 0u;
        qf[kk][1] = 0u;
      }
    }
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    float o[D / 16][4];
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

    int kb_lo, kb_hi;
    split_range(cnt, (int)(wi % a.splits), a.splits, kb_lo, kb_hi);
    bool ok = true;
    for (int kb = kb_lo; kb < kb_hi; ++kb, ++it) {
      const int s = it % nst;
      const uint32_t ph = (it / nst) & 1u;
      if (!mbar_wait(&full[s], ph, a.err)) { ok = false; break; }
      const uint8_t* Ks = stages + s * stage_bytes;
      const uint8_t* Vs = Ks + row_bytes;
      // Stage the group's K and V tiles in registers and hand the slot back at once: the copy
      // ring then keeps (almost) all of its stages in flight while this warp computes.
      uint32_t kf[D / 16][4], vf[D / 16][4];
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int key = r8 + ((mi & 1) ? 8 : 0);
        const int dim = kk * 16 + ((mi & 2) ? 8 : 0);
        ldsm_x4(smem_u32(Ks + key * rs + (g * D + dim) * 2), kf[kk][0], kf[kk][1], kf[kk][2], kf[kk][3]);
      }
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) {
        const int key = r8 + ((mi & 2) ? 8 : 0);
        const int dim = mt * 16 + ((mi & 1) ? 8 : 0);
        ldsm_x4_t(smem_u32(Vs + key * rs + (g * D + dim) * 2), vf[mt][0], vf[mt][1], vf[mt][2], vf[mt][3]);
      }
      // Hand the slot back only after every ldmatrix of this warp has returned its data: the
      // next bulk copy into the slot must not overtake a shared-memory read in flight.  A value
      // built from one register of each load (the four registers of an ldmatrix arrive
      // together) makes the release wait for them.
      uint32_t dep = 0;
#pragma unroll
      for (int i = 0; i < D / 16; ++i) dep ^= kf[i][0] ^ vf[i][0];
      uint32_t zero;
      asm volatile("and.b32 %0, %1, 0;" : "=r"(zero) : "r"(dep));
      __syncwarp();
      if (lane == 0) mbar_arrive(reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(&empty[s]) + zero));
      // S^T = K Q^T with two independent accumulation chains
      float c[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < D / 16; kk += 2) {
        mma_bf16(c, kf[kk][0], kf[kk][1], kf[kk][2], kf[kk][3], qf[kk][0], qf[kk][1]);
        mma_bf16(c2, kf[kk + 1][0], kf[kk + 1][1], kf[kk + 1][2], kf[kk + 1][3], qf[kk + 1][0], qf[kk + 1][1]);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) c[e] += c2[e];
      const int valid = cnt - kb * kKeysPerStage;
      const bool v0 = grp < valid, v1 = grp + 8 < valid;
      float x0 = v0 ? c[0] * a.scale_log2 : -INFINITY;
      float x1 = v0 ? c[1] * a.scale_log2 : -INFINITY;
      float x2 = v1 ? c[2] * a.scale_log2 : -INFINITY;
      float x3 = v1 ? c[3] * a.scale_log2 : -INFINITY;
      float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float corr0 = exp2f(m0 - mn0), corr1 = exp2f(m1 - mn1);
      const float p0 = exp2f(x0 - mn0), p1 = exp2f(x1 - mn1);
      const float p2 = exp2f(x2 - mn0), p3 = exp2f(x3 - mn1);
      l0 = l0 * corr0 + p0 + p2;
      l1 = l1 * corr1 + p1 + p3;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) {
        o[mt][0] *= corr0;
        o[mt][1] *= corr1;
        o[mt][2] *= corr0;
        o[mt][3] *= corr1;
      }
      const uint32_t b0 = movm_t(pack_bf16(p0, p1));
      const uint32_t b1 = movm_t(pack_bf16(p2, p3));
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) mma_bf16(o[mt], vf[mt][0], vf[mt][1], vf[mt][2], vf[mt][3], b0, b1);
    }
    if (!ok) return;
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
    const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
    const int h0 = tq * 2, h1 = tq * 2 + 1;
    if (a.splits > 1) {
      // partial of this key range: o / l in fp32 and log2(sum exp) = m + log2(l) per head
      float* po = a.part + (wi * H + g * NREP) * D;
      float* pl = a.part + NW * H * D + wi * H + g * NREP;
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int dim = mt * 16 + grp + half * 8;
          if (h0 < NREP) po[h0 * D + dim] = o[mt][half * 2 + 0] * inv0;
          if (h1 < NREP) po[h1 * D + dim] = o[mt][half * 2 + 1] * inv1;
        }
      }
      if (grp == 0) {
        if (h0 < NREP) pl[h0] = l0 > 0.f ? m0 + log2f(l0) : -INFINITY;
        if (h1 < NREP) pl[h1] = l1 > 0.f ? m1 + log2f(l1) : -INFINITY;
      }
      continue;
    }
    if (a.lse_out && grp == 0) {
      // natural-log sum-exp of scale * q.k (m is in log2 units of it)
      float* lr = a.lse_out + row * H + g * NREP;
      if (h0 < NREP) lr[h0] = l0 > 0.f ? (m0 + log2f(l0)) * 0.6931471805599453f : -INFINITY;
      if (h1 < NREP) lr[h1] = l1 > 0.f ? (m1 + log2f(l1)) * 0.6931471805599453f : -INFINITY;
    }
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int dim = mt * 16 + grp + half * 8;
        if (h0 < NREP) {
          const int64_t off = (row * H + g * NREP + h0) * D + dim;
          float y = __bfloat162float(__float2bfloat16_rn(o[mt][half * 2 + 0] * inv0));
          if (a.gate) y *= __bfloat162float(a.gate[off]);
          a.out[off] = __float2bfloat16_rn(y);
        }
        if (h1 < NREP) {
          const int64_t off = (row * H + g * NREP + h1) * D + dim;
          float y = __bfloat162float(__float2bfloat16_rn(o[mt][half * 2 + 1] * inv1));
          if (a.gate) y *= __bfloat162float(a.gate[off]);
          a.out[off] = __float2bfloat16_rn(y);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Precise fp32 kernel: one warp per (row, head), exact expf, fp32 accumulation.  Used for the
// layer's fp32 configuration.
// ---------------------------------------------------------------------------------------------


__global__ void sdpa_f32_kernel(SdpaF32Args a) {
  const int64_t row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  const int64_t b = row / a.Lq;
  const int n_rep = a.H / a.Hk;
  int cnt = a.sel_count[row];
  if (cnt < 0) cnt = 0;
  if (cnt > a.sel_ld) cnt = (int)a.sel_ld;
  const int32_t* idx = a.sel_idx + row * a.sel_ld;
  constexpr int kMaxPerLane = 8;  // D <= 256
  for (int h = warp; h < a.H; h += nw) {
    const int g = h / n_rep;
    const float* qh = a.q + (row * a.H + h) * a.D;
    float qv[kMaxPerLane], ov[kMaxPerLane];
    for (int i = 0; i < kMaxPerLane; ++i) {
      int d = lane + 32 * i;
      qv[i] = d < a.D ? qh[d] : 0.f;
      ov[i] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    for (int j = 0; j < cnt; ++j) {
      int s = idx[j];
      if (s < 0 || s >= a.Lkv) { set_error(a.err, GSA_ERR_INDEX); continue; }
      const float* kr = a.k + b * a.kv_bstride + s * a.kv_ld + (int64_t)g * a.D;
      const float* vr = a.v + b * a.kv_bstride + s * a.kv_ld + (int64_t)g * a.D;
      float dot = 0.f;
      for (int i = 0; i < kMaxPerLane; ++i) {
        int d = lane + 32 * i;
        if (d < a.D) dot = fmaf(qv[i], kr[d], dot);
      }
      dot = warp_sum(dot) * a.scale;
      float mn = fmaxf(m, dot);
      float corr = expf(m - mn), p = expf(dot - mn);
      l = l * corr + p;
      for (int i = 0; i < kMaxPerLane; ++i) {
        int d = lane + 32 * i;
        if (d < a.D) ov[i] = ov[i] * corr + p * vr[d];
      }
      m = mn;
    }
    float inv = l > 0.f ? 1.f / l : 0.f;
    if (a.lse_out && lane == 0) a.lse_out[row * a.H + h] = l > 0.f ? m + logf(l) : -INFINITY;
    for (int i = 0; i < kMaxPerLane; ++i) {
      int d = lane + 32 * i;
      if (d < a.D) {
        int64_t off = (row * a.H + h) * a.D + d;
        float y = ov[i] * inv;
        if (a.gate) y = fmul(y, a.gate[off]);
        a.out[off] = y;
      }
    }
  }
}

// Merge the key-range partials of each (row, head): out = bf16(sum_s 2^(lse_s - M) o_s /
// sum_s 2^(lse_s - M)), times the G1 gate (the unsplit epilogue's roundings).  One CTA per
// (row, head), one thread per dimension; the split weights are computed once per CTA.
__global__ void sdpa_combine_kernel(int64_t R, int H, int D, int splits, const float* part,
                                    const __nv_bfloat16* gate, __nv_bfloat16* out) {
  chain_wait();
  chain_release();
  const int64_t row = blockIdx.x;
  const int h = blockIdx.y;
  const int64_t NW = R * splits;
  __shared__ float wsh[16];
  __shared__ float inv_den;
  if (threadIdx.x == 0) {
    const float* lse = part + NW * H * D + row * splits * H + h;
    float M = -INFINITY;
    for (int s = 0; s < splits; ++s) M = fmaxf(M, lse[s * H]);
    float den = 0.f;
    for (int s = 0; s < splits; ++s) {
      const float w = M > -INFINITY ? exp2f(lse[s * H] - M) : 0.f;
      wsh[s] = w;
      den += w;
    }
    inv_den = den > 0.f ? 1.f / den : 0.f;
  }
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float num = 0.f;
    for (int s = 0; s < splits; ++s) num = fmaf(wsh[s], part[((row * splits + s) * H + h) * D + d], num);
    const int64_t off = (row * H + h) * D + d;
    float y = __bfloat162float(__float2bfloat16_rn(num * inv_den));
    if (gate) y *= __bfloat162float(gate[off]);
    out[off] = __float2bfloat16_rn(y);
  }
}

// ---------------------------------------------------------------------------------------------
struct SdpaCfg {
  int nstages;
  size_t smem;
};

template <int D, int NREP, int MAXW>
static int launch_tc_w(SdpaArgs a, int num_sms, cudaStream_t stream) {
  const int row_bytes = a.Hk * D * 2;
  const int stage_bytes = kKeysPerStage * (2 * row_bytes + 16);
  const int max_smem = 227 * 1024;
  int nst = (max_smem - 256) / stage_bytes;
  if (nst > 8) nst = 8;
  if (nst < 2) return GSA_ERR_UNSUPPORTED;
  a.nstages = nst;
  const size_t smem = 256 + (size_t)nst * stage_bytes;
  auto kern = sdpa_tc_kernel<D, NREP, MAXW>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return GSA_ERR_LAUNCH;
  int per_sm = 0;
  a.nprod = 2 * (nst < kMaxGroups ? nst : kMaxGroups);  // groups <= nstages (see the producer loop)
  const int threads = (a.Hk + a.nprod) * 32;
  if (threads > MAXW * 32) return GSA_ERR_UNSUPPORTED;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess || per_sm < 1)
    return GSA_ERR_LAUNCH;
  const int64_t R = a.B * a.Lq;
  const int H = a.Hk * NREP;
  int64_t grid = (int64_t)num_sms * per_sm;
  // fewer rows than resident CTAs: cut each row's keys into ranges (one per CTA, as many as the
  // partials buffer holds) so that every CTA streams keys; finer ranges cost more in per-range
  // set-up and partials than they gain in balance.  Those launches are bound by DRAM latency,
  // so their producers also prefetch into L2 four stages ahead.
  a.splits = 1;
  a.prefetch = 0;
  if (a.part && R < grid && !a.lse_out) {
    int64_t sp = std::min<int64_t>(grid / R, kMaxSplits);
    while (sp > 1 && R * sp * H * (D + 1) > a.part_floats) --sp;
    a.splits = (int)sp;
    a.prefetch = 4;
  }
  const int64_t items = R * a.splits;
  if (grid > items) grid = items;
  if (launch_chained(kern, dim3((unsigned)grid), dim3(threads), smem, stream, a) != cudaSuccess) return GSA_ERR_LAUNCH;
  if (a.splits > 1 &&
      launch_chained(sdpa_combine_kernel, dim3((unsigned)R, (unsigned)H), dim3(D), 0, stream, R, H, D, a.splits,
                     (const float*)a.part, a.gate, a.out) != cudaSuccess)
    return GSA_ERR_LAUNCH;
  return GSA_OK;
}

// The register-staged consumers want more than the 93 registers a 22-warp block leaves, so
// groups of up to 8 KV heads (8 consumer + 6 producer warps) get a 14-warp build.
template <int D, int NREP>
static int launch_tc(SdpaArgs a, int num_sms, cudaStream_t stream) {
  if (a.Hk + 2 * kMaxGroups <= 14) return launch_tc_w<D, NREP, 14>(a, num_sms, stream);
  return launch_tc_w<D, NREP, 22>(a, num_sms, stream);
}

template <int D>
static int dispatch_nrep(SdpaArgs a, int nrep, int num_sms, cudaStream_t stream) {
  switch (nrep) {
    case 1: return launch_tc<D, 1>(a, num_sms, stream);
    case 2: return launch_tc<D, 2>(a, num_sms, stream);
    case 4: return launch_tc<D, 4>(a, num_sms, stream);
    case 8: return launch_tc<D, 8>(a, num_sms, stream);
    default: return GSA_ERR_UNSUPPORTED;
  }
}

int launch_sdpa_bf16(SdpaArgs a, int D, int nrep, int num_sms, cudaStream_t stream) {
  if (a.B * a.Lq == 0) return GSA_OK;
  if (a.Hk < 1 || a.Hk > 16 || a.Hk * D * 2 > kMaxRowBytes) return GSA_ERR_UNSUPPORTED;
  switch (D) {
    case 64: return dispatch_nrep<64>(a, nrep, num_sms, stream);
    case 128: return dispatch_nrep<128>(a, nrep, num_sms, stream);
    default: return GSA_ERR_UNSUPPORTED;
  }
}

int launch_sdpa_f32(const SdpaF32Args& a, cudaStream_t stream) {
  const int64_t R = a.B * a.Lq;
  if (R == 0) return GSA_OK;
  if (a.D > 256) return GSA_ERR_UNSUPPORTED;
  int warps = a.H < 8 ? a.H : 8;
  sdpa_f32_kernel<<<(unsigned)R, warps * 32, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? GSA_OK : GSA_ERR_LAUNCH;
}

}  // namespace gsa
