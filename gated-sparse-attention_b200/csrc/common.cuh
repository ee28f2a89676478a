// Shared device helpers for the GSA sm_100a kernels: bf16 conversion, torch-compatible
// rounding, mbarrier / bulk-copy PTX wrappers with bounded waits, and the error word.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "gsa_b200.h"

namespace gsa {

// ---------------------------------------------------------------------------------------------
// Element access for the two activation dtypes (GSA_DTYPE_F32 / GSA_DTYPE_BF16).
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ float load_elem(const void* p, int64_t i, int dtype) {
  if (dtype == GSA_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_elem(void* p, int64_t i, float v, int dtype) {
  if (dtype == GSA_DTYPE_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

// Typed element conversions (templated kernels over float / __nv_bfloat16).
__device__ __forceinline__ float to_float(float v) { return v; }
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_float(float v);
template <>
__device__ __forceinline__ float from_float<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Round a float to the activation dtype and back.  torch evaluates each bf16 elementwise op
// in fp32 and rounds the result to bf16; calling this after every op reproduces that.
__device__ __forceinline__ float rnd(float v, int dtype) {
  return dtype == GSA_DTYPE_BF16 ? __bfloat162float(__float2bfloat16_rn(v)) : v;
}

// fp32 ops that the compiler may not contract into FMAs (torch evaluates them one by one).
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }

// Logistic sigmoid evaluated as 1 / (1 + e^-x) with the accurate expf; the reciprocal is the
// correctly rounded one, the same value as the IEEE division 1.0f / d.
__device__ __forceinline__ float sigmoid_precise(float x) { return __frcp_rn(1.0f + expf(-x)); }

// Gate activations of the value / output gates (value_gate.py:98-106).
__device__ __forceinline__ float gate_act(float x, int act, int dtype) {
  if (act == GSA_ACT_SIGMOID) return rnd(sigmoid_precise(x), dtype);
  if (act == GSA_ACT_TANH) {
    float t = rnd(tanhf(x), dtype);
    return rnd(rnd(t + 1.0f, dtype) / 2.0f, dtype);
  }
  // silu: x * sigmoid(x), evaluated by torch as one fused op
  return rnd(x / (1.0f + expf(-x)), dtype);
}

// Monotone map of an fp32 bit pattern to an unsigned key: larger float -> larger key.
__device__ __forceinline__ uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---------------------------------------------------------------------------------------------
// Error word.  Kernels never trap: a failed bounded wait or a bad index sets a code here and
// the kernel returns; the host reads it back through gsa_get_device_error().
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void set_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ---------------------------------------------------------------------------------------------
// mbarrier + bulk copy (TMA) wrappers.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records GSA_ERR_TIMEOUT) if the phase never completes.
// Each try_wait suspends for a hardware-chosen interval, so the limit is generous in time.
constexpr uint32_t kWaitLimit = 1u << 22;

__device__ __forceinline__ bool mbar_wait_limit(uint64_t* bar, uint32_t parity, int* err, uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  set_error(err, GSA_ERR_TIMEOUT);
  return false;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  return mbar_wait_limit(bar, parity, err, kWaitLimit);
}

// 1-D bulk copy global -> shared, completing on an mbarrier (both addresses 16-byte aligned,
// size a multiple of 16).
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Prefetch a global range into L2 through the bulk-copy engine (16-byte aligned, multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void* gsrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gsrc), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched by launch_chained may be scheduled while the
// previous kernel of its stream is still running.  Every CTA of such a kernel executes
// chain_wait() before anything else (it returns once the previous grid has completed and its
// memory is visible; a kernel launched the ordinary way passes straight through), so each
// chained kernel completes after its predecessor and the stream keeps its order.  chain_release()
// lets the next chained kernel be scheduled once every CTA of this one has started.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void chain_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void chain_release() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
static inline cudaError_t launch_chained(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                         cudaStream_t stream, Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) (void)cudaGetLastError();  // reported here; not left for the next launch check
  return e;
}

// ---------------------------------------------------------------------------------------------
// Block-wide helpers.
// ---------------------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace gsa
