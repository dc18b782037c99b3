// Exact fp32 GEMM: bitwise identical to the reference's matmulKernel
// (lib/src/gemm_kernel_simd.dart:32-702) and to the epilogues of opGemm
// (lib/src/onnx_ops.dart:2162-2172) and opMatMulNBits (lib/src/onnx_qlinear_ops.dart:
// 194-226).
//
// Per output element the reference accumulates in k order starting from +0,
// either in a float32 SIMD lane (each product and each sum rounded to float32,
// no fused multiply-add) or, for a few tail columns, in double. The kernels
// below keep that exact order per element: the register-tiled kernel uses
// __fmul_rn/__fadd_rn (never contracted into FFMA) and walks k strictly
// ascending; the double kernel handles the columns the reference runs in
// double. Tiling across threads never reorders any single element's sum.
#include "b2m_internal.cuh"

namespace {

constexpr int BM = 64, BN = 64, BK = 16, TM = 4, TN = 4;  // 256 threads, 4x4 outputs each

__device__ __forceinline__ void batch_offsets(const F32GemmArgs &p, int64_t b, int64_t &aoff,
                                              int64_t &boff) {
  aoff = 0;
  boff = 0;
  for (int d = p.nbd - 1; d >= 0; d--) {
    const int64_t dim = p.bdims[d];
    const int64_t c = b % dim;
    b /= dim;
    aoff += c * p.a_bstride[d];
    boff += c * p.b_bstride[d];
  }
}

// Columns the reference accumulates in double: with fewer than four rows, the
// n % 4 tail of each kernel call (_gemvScalar :601-608, _matmulSmallM
// :665-672); every column of MatMulNBits' single-row decode (:197-202).
__device__ __forceinline__ bool column_is_double(const F32GemmArgs &p, int64_t j) {
  if (p.all_double) return true;
  if (p.m_eff >= 4) return false;
  const int64_t jin = j % p.tile_w;
  const int64_t start = j - jin;
  const int64_t width = (p.N - start) < p.tile_w ? (p.N - start) : p.tile_w;
  return jin >= (width & ~(int64_t)3);
}

__device__ __forceinline__ float epilogue_f32(const F32GemmArgs &p, float y, int64_t i, int64_t j) {
  if (p.epi == EPI_GEMM) {
    if (p.has_alpha) y = __fmul_rn(y, p.alpha);
    if (p.C) {
      float cv = p.C[i * p.c_rs + j * p.c_cs];
      if (p.has_beta) cv = __fmul_rn(cv, p.beta);
      y = __fadd_rn(y, cv);
    }
  } else if (p.epi == EPI_NBITS) {
    y = __double2float_rn((double)y + (p.bias ? (double)p.bias[j] : 0.0));
  }
  return y;
}

__global__ void __launch_bounds__(256) f32_exact_gemm_kernel(const F32GemmArgs p) {
  __shared__ __align__(16) float As[BK][BM + 4];
  __shared__ __align__(16) float Bs[BK][BN + 4];
  int64_t aoff, boff;
  batch_offsets(p, blockIdx.z, aoff, boff);
  const float *A = p.A + aoff;
  const float *B = p.B + boff;
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; i++)
#pragma unroll
    for (int j = 0; j < TN; j++) acc[i][j] = 0.f;

  for (int64_t k0 = 0; k0 < p.K; k0 += BK) {
    // Stage a BM x BK slab of A and a BK x BN slab of B (zero outside).
#pragma unroll
    for (int r = 0; r < (BM * BK) / 256; r++) {
      const int e = tid + r * 256;
      const int mm = e % BM, kk = e / BM;
      const int64_t gi = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gi < p.M && gk < p.K) ? A[gi * p.sa_m + gk * p.sa_k] : 0.f;
    }
#pragma unroll
    for (int r = 0; r < (BN * BK) / 256; r++) {
      const int e = tid + r * 256;
      const int nn = e % BN, kk = e / BN;
      const int64_t gj = n0 + nn, gk = k0 + kk;
      Bs[kk][nn] = (gj < p.N && gk < p.K) ? B[gk * p.sb_k + gj * p.sb_n] : 0.f;
    }
    __syncthreads();
    const int kmax = (p.K - k0) < BK ? (int)(p.K - k0) : BK;
    for (int kk = 0; kk < kmax; kk++) {
      const float4 av = *reinterpret_cast<const float4 *>(&As[kk][ty * TM]);
      const float4 bv = *reinterpret_cast<const float4 *>(&Bs[kk][tx * TN]);
      const float a_[4] = {av.x, av.y, av.z, av.w};
      const float b_[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a_[i], b_[j]));
    }
    __syncthreads();
  }

  float *Y = p.Y + (int64_t)blockIdx.z * p.y_bstride;
#pragma unroll
  for (int i = 0; i < TM; i++) {
    const int64_t gi = m0 + ty * TM + i;
    if (gi >= p.M) continue;
#pragma unroll
    for (int j = 0; j < TN; j++) {
      const int64_t gj = n0 + tx * TN + j;
      if (gj >= p.N) continue;
      Y[gi * p.ldy + gj] = epilogue_f32(p, acc[i][j], gi, gj);
    }
  }
}

// Small-tile variant for grids that would underfill the SMs with 64 x 64
// tiles (e.g. 128 x 1536 outputs): 32 x 32 outputs per CTA, 64 threads with
// 4 x 4 outputs each, and the next 32-k slab fetched into registers while the
// current one is consumed. Same per-element k order as above.
constexpr int SBM = 32, SBN = 32, SBK = 32;

__global__ void __launch_bounds__(64) f32_exact_gemm_small_kernel(const F32GemmArgs p) {
  __shared__ __align__(16) float As[SBK][SBM + 4];
  __shared__ __align__(16) float Bs[SBK][SBN + 4];
  int64_t aoff, boff;
  batch_offsets(p, blockIdx.z, aoff, boff);
  const float *A = p.A + aoff;
  const float *B = p.B + boff;
  const int64_t m0 = (int64_t)blockIdx.y * SBM, n0 = (int64_t)blockIdx.x * SBN;
  const int tid = threadIdx.x, tx = tid & 7, ty = tid >> 3;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0.f;
  float ra[16], rb[16];
  // Element e = tid + 64 r of a slab: A is walked k-fastest, B n-fastest, so
  // row-major operands load coalesced.
  auto fetch = [&](int64_t k0) {
#pragma unroll
    for (int r = 0; r < 16; r++) {
      const int e = tid + 64 * r;
      const int kk = e & 31, mm = e >> 5;
      const int64_t gi = m0 + mm, gk = k0 + kk;
      ra[r] = (gi < p.M && gk < p.K) ? __ldg(A + gi * p.sa_m + gk * p.sa_k) : 0.f;
      const int nn = e & 31, kb = e >> 5;
      const int64_t gj = n0 + nn, gkb = k0 + kb;
      rb[r] = (gj < p.N && gkb < p.K) ? __ldg(B + gkb * p.sb_k + gj * p.sb_n) : 0.f;
    }
  };
  fetch(0);
  for (int64_t k0 = 0; k0 < p.K; k0 += SBK) {
#pragma unroll
    for (int r = 0; r < 16; r++) {
      const int e = tid + 64 * r;
      As[e & 31][e >> 5] = ra[r];
      Bs[e >> 5][e & 31] = rb[r];
    }
    __syncthreads();
    if (k0 + SBK < p.K) fetch(k0 + SBK);
    const int kmax = (p.K - k0) < SBK ? (int)(p.K - k0) : SBK;
    if (kmax == SBK) {
#pragma unroll 8
      for (int kk = 0; kk < SBK; kk++) {
        const float4 av = *reinterpret_cast<const float4 *>(&As[kk][ty * 4]);
        const float4 bv = *reinterpret_cast<const float4 *>(&Bs[kk][tx * 4]);
        const float a_[4] = {av.x, av.y, av.z, av.w};
        const float b_[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
          for (int j = 0; j < 4; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a_[i], b_[j]));
      }
    } else {
      for (int kk = 0; kk < kmax; kk++) {
        const float4 av = *reinterpret_cast<const float4 *>(&As[kk][ty * 4]);
        const float4 bv = *reinterpret_cast<const float4 *>(&Bs[kk][tx * 4]);
        const float a_[4] = {av.x, av.y, av.z, av.w};
        const float b_[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
          for (int j = 0; j < 4; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a_[i], b_[j]));
      }
    }
    __syncthreads();
  }
  float *Y = p.Y + (int64_t)blockIdx.z * p.y_bstride;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int64_t gi = m0 + ty * 4 + i;
    if (gi >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int64_t gj = n0 + tx * 4 + j;
      if (gj >= p.N) continue;
      Y[gi * p.ldy + gj] = epilogue_f32(p, acc[i][j], gi, gj);
    }
  }
}

// Double-accumulated columns. One thread per (row, column) of the double set.
__global__ void __launch_bounds__(128) f32_double_cols_kernel(const F32GemmArgs p) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t i = blockIdx.y;
  if (j >= p.N || i >= p.M) return;
  if (!column_is_double(p, j)) return;
  int64_t aoff, boff;
  batch_offsets(p, blockIdx.z, aoff, boff);
  const float *A = p.A + aoff + i * p.sa_m;
  const float *B = p.B + boff + j * p.sb_n;
  double acc = 0.0;
  // Each float x float product is exact in double, so the fused form equals
  // the reference's `acc += a * b` in Dart doubles.
  for (int64_t k = 0; k < p.K; k++) acc = fma((double)A[k * p.sa_k], (double)B[k * p.sb_k], acc);
  float y;
  if (p.epi == EPI_NBITS_M1) {
    y = __double2float_rn(acc + (p.bias ? (double)p.bias[j] : 0.0));
  } else {
    y = epilogue_f32(p, __double2float_rn(acc), i, j);
  }
  p.Y[(int64_t)blockIdx.z * p.y_bstride + i * p.ldy + j] = y;
}

}  // namespace

void launch_f32_exact(const F32GemmArgs &a, cudaStream_t s) {
  if (a.M <= 0 || a.N <= 0 || a.batch <= 0) return;
  B2M_REQUIRE(a.batch <= 65535, B2M_ERR_UNSUPPORTED, "MatMul: more than 65535 batches");
  const bool any_double = a.all_double || a.m_eff < 4;
  if (!a.all_double) {
    dim3 grid((unsigned)((a.N + BN - 1) / BN), (unsigned)((a.M + BM - 1) / BM), (unsigned)a.batch);
    B2M_REQUIRE(grid.y <= 65535, B2M_ERR_UNSUPPORTED, "MatMul: too many rows");
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    if ((int64_t)grid.x * grid.y * grid.z < 2 * (int64_t)sms) {
      dim3 sg((unsigned)((a.N + SBN - 1) / SBN), (unsigned)((a.M + SBM - 1) / SBM), (unsigned)a.batch);
      B2M_REQUIRE(sg.y <= 65535, B2M_ERR_UNSUPPORTED, "MatMul: too many rows");
      f32_exact_gemm_small_kernel<<<sg, 64, 0, s>>>(a);
    } else {
      f32_exact_gemm_kernel<<<grid, 256, 0, s>>>(a);
    }
    B2M_CUDA(cudaGetLastError());
  }
  if (any_double) {
    B2M_REQUIRE(a.M <= 65535, B2M_ERR_UNSUPPORTED, "MatMul: too many rows");
    dim3 grid((unsigned)((a.N + 127) / 128), (unsigned)a.M, (unsigned)a.batch);
    f32_double_cols_kernel<<<grid, 128, 0, s>>>(a);
    B2M_CUDA(cudaGetLastError());
  }
}
