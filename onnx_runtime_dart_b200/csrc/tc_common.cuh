// Pieces shared by the tcgen05 GEMM kernels: bounded mbarrier waits and the
// driver's tensor-map encoder.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include <atomic>

#include "b2m_internal.cuh"
#include "ptx.cuh"

namespace b2m {

constexpr uint32_t TC_WAIT_LIMIT = 1u << 26;

// Waits for phase `parity` of `bar`. Gives up when another thread of the CTA
// has raised `abort_flag`, or after TC_WAIT_LIMIT polls (then raises the flag
// and records a timeout in the context's device error word).
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                              int32_t *dev_err) {
  for (uint32_t i = 0; i < TC_WAIT_LIMIT; i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023) == 1023 && *abort_flag) return false;
    if (i > 256) __nanosleep(64);
  }
  *abort_flag = 1;
  if (dev_err) set_dev_error(dev_err, B2M_DEVERR_MBAR_TIMEOUT);
  return false;
}

// Lane 0 waits, the warp follows its verdict: every lane then takes the same
// path through the warp-wide (.sync.aligned) tcgen05 instructions.
__device__ __forceinline__ bool warp_wait_or_abort(uint64_t *bar, uint32_t parity, volatile int *abort_flag,
                                                   int32_t *dev_err) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = wait_or_abort(bar, parity, abort_flag, dev_err) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Raises kernel Kern's dynamic shared-memory limit to `bytes` once per device
// (the attribute persists for the process), keeping it off the per-call path.
template <auto Kern>
void set_smem_limit_once(int bytes) {
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  B2M_CUDA(cudaGetDevice(&dev));
  const uint64_t bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return;
  B2M_CUDA(cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.fetch_or(bit, std::memory_order_acq_rel);
}

// x -> (x0, x1) = (rn_bf16(x), rn_bf16(x - x0)), the two-term split of the
// FAST fp32 GEMM's operands. A finite x whose rounding overflows bf16 keeps
// its truncation as x0; a non-finite x passes through x0.
__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16 &h, __nv_bfloat16 &l) {
  h = __float2bfloat16_rn(x);
  float hf = __bfloat162float(h);
  if (isinf(hf) && isfinite(x)) {
    h = __float2bfloat16_rz(x);
    hf = __bfloat162float(h);
  }
  l = __float2bfloat16_rn(isfinite(x) ? x - hf : 0.f);
}

// split_bf16 of two values at once, packed as bf16x2 words (a in the low
// half). Finite values below 3.38e38 in magnitude (every value whose bf16
// rounding stays finite, with margin) take two packed conversions; anything
// else goes through split_bf16, so the results are identical.
__device__ __forceinline__ void split_bf16x2(float a, float b, uint32_t &hi, uint32_t &lo) {
  if (fabsf(a) < 3.38e38f && fabsf(b) < 3.38e38f) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
    return;
  }
  __nv_bfloat16 h0, l0, h1, l1;
  split_bf16(a, h0, l0);
  split_bf16(b, h1, l1);
  hi = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
  lo = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
}

// SM count of the current device, cached.
int device_sm_count();

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda
// link dependency).
EncodeTiledFn tensor_map_encoder();

// f16 copy of the activations for the tensor-core kernels: A[M][K] fp32 ->
// A16[M][K8] (K8 = K rounded up to 8, zero padded); with `perm` k is permuted
// inside each aligned group of four as (k0, k2, k1, k3).
void launch_f32_to_f16(const float *A, __half *A16, int64_t M, int64_t K, int64_t K8, int perm, cudaStream_t s);

}  // namespace b2m
