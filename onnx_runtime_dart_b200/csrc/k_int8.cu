// MatMulInteger / QLinearMatMul kernels (reference: opMatMulInteger and
// opQLinearMatMul, lib/src/onnx_qlinear_ops.dart:32-108).
//
// The integer result is exact: raw = sum_k a*b is accumulated with dp4a in
// int32 and the zero points are applied in the epilogue,
//   y = raw - az*colsum(b) - bz*rowsum(a) + K*az*bz,
// in wrapping 32-bit arithmetic (exact whenever the true result fits int32,
// which the host guarantees by rejecting K > 33025). QLinearMatMul then
// requantizes exactly like the reference: f = f32(double(acc) * mult),
// q = roundHalfEven(f) + y_zp, clamped to [lo, hi].
#include "b2m_internal.cuh"

namespace {

template <bool AS, bool BS>
__device__ __forceinline__ int dp4(uint32_t a, uint32_t b, int c) {
  int d;
  if (AS && BS) asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  else if (AS && !BS) asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  else if (!AS && BS) asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  else asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

__device__ __forceinline__ int32_t zp_at(const void *zp, int is_signed, int64_t i) {
  return is_signed ? (int32_t) reinterpret_cast<const int8_t *>(zp)[i]
                   : (int32_t) reinterpret_cast<const uint8_t *>(zp)[i];
}

struct I8Extra {
  int azp_signed, bzp_signed;
};

constexpr int TILE = 64, KT = 32;  // 64x64 outputs per CTA, 32 k per stage

template <bool AS, bool BS>
__global__ void __launch_bounds__(256) i8_gemm_kernel(const I8GemmArgs p, const I8Extra x) {
  __shared__ uint32_t As[TILE][KT / 4 + 1];
  __shared__ uint32_t Bs[TILE][KT / 4 + 1];
  const int64_t bz_ = blockIdx.z;
  const uint8_t *A = reinterpret_cast<const uint8_t *>(p.A) + bz_ * p.a_bstride;
  const int8_t *Bt = p.Bt + bz_ * p.b_bstride;
  const int64_t m0 = (int64_t)blockIdx.y * TILE, n0 = (int64_t)blockIdx.x * TILE;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  int acc[4][4] = {};
  int rs[4] = {0, 0, 0, 0};
  const uint32_t ones = 0x01010101u;
  for (int64_t k0 = 0; k0 < p.K; k0 += KT) {
    for (int e = tid; e < TILE * (KT / 4); e += 256) {
      const int r = e / (KT / 4), w = e % (KT / 4);
      const int64_t gi = m0 + r;
      uint32_t v = 0;
      if (gi < p.M) {
#pragma unroll
        for (int b = 0; b < 4; b++) {
          const int64_t gk = k0 + w * 4 + b;
          if (gk < p.K) v |= (uint32_t)A[gi * p.K + gk] << (8 * b);
        }
      }
      As[r][w] = v;
      // Packed B rows are zero-padded to npad x kpad; a column slice of a
      // packed weight (a convolution group) may end before its last tile, so
      // rows past N read as zero.
      const int64_t gj = n0 + r;
      Bs[r][w] = gj < p.N ? *reinterpret_cast<const uint32_t *>(Bt + gj * p.kpad + k0 + w * 4) : 0u;
    }
    __syncthreads();
#pragma unroll
    for (int w = 0; w < KT / 4; w++) {
      uint32_t av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; i++) av[i] = As[ty * 4 + i][w];
#pragma unroll
      for (int j = 0; j < 4; j++) bv[j] = Bs[tx * 4 + j][w];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        rs[i] = dp4<AS, false>(av[i], ones, rs[i]);
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = dp4<AS, BS>(av[i], bv[j], acc[i][j]);
      }
    }
    __syncthreads();
  }
  const int32_t *colsum = p.colsum + bz_ * p.colsum_bstride;
  const int64_t obase = bz_ * p.M * p.N;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int64_t gi = m0 + ty * 4 + i;
    if (gi >= p.M) continue;
    // Zero-point rules of the reference (:41-44).
    int32_t az = 0;
    if (p.azp) {
      if (p.azp_len == 1) az = zp_at(p.azp, x.azp_signed, 0);
      else if (p.azp_len == p.M && p.M != 1) az = zp_at(p.azp, x.azp_signed, gi);
    }
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int64_t gj = n0 + tx * 4 + j;
      if (gj >= p.N) continue;
      int32_t bz = 0;
      if (p.bzp) {
        if (p.bzp_len == 1) bz = zp_at(p.bzp, x.bzp_signed, 0);
        else if (p.bzp_len == p.N && p.N != 1) bz = zp_at(p.bzp, x.bzp_signed, gj);
      }
      const uint32_t y = (uint32_t)acc[i][j] - (uint32_t)az * (uint32_t)colsum[gj] -
                         (uint32_t)bz * (uint32_t)rs[i] + (uint32_t)p.K * (uint32_t)az * (uint32_t)bz;
      const int32_t yi = (int32_t)y;
      if (!p.requant) {
        p.Y32[obase + gi * p.N + gj] = yi;
      } else {
        const float f = __double2float_rn(__dmul_rn((double)yi, p.mult));
        long long q = __float2ll_rn(f) + (long long)p.y_zp;
        q = q < p.lo ? p.lo : (q > p.hi ? p.hi : q);
        if (p.lo < 0) reinterpret_cast<int8_t *>(p.Yq)[obase + gi * p.N + gj] = (int8_t)q;
        else reinterpret_cast<uint8_t *>(p.Yq)[obase + gi * p.N + gj] = (uint8_t)q;
      }
    }
  }
}

// B[batch][K][N] (row-major bytes) -> Bt[batch][npad][kpad] (K-major, zero
// padded) and colsum[batch][N] = sum_k b (signed per dtype).
__global__ void i8_pack_kernel(const uint8_t *B, int b_signed, int64_t K, int64_t N, int8_t *bt,
                               int64_t kpad, int64_t npad, int32_t *colsum) {
  const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t b = blockIdx.y;
  if (n >= npad) return;
  const uint8_t *src = B + b * K * N;
  int8_t *dst = bt + (b * npad + n) * kpad;
  int32_t s = 0;
  for (int64_t k = 0; k < kpad; k++) {
    uint8_t v = 0;
    if (n < N && k < K) v = src[k * N + n];
    dst[k] = (int8_t)v;
    s += b_signed ? (int32_t)(int8_t)v : (int32_t)v;
  }
  if (n < N) colsum[b * N + n] = s;
}

}  // namespace

void launch_i8_gemm(const I8GemmArgs &a, cudaStream_t s) {
  if (a.M <= 0 || a.N <= 0 || a.batch <= 0) return;
  dim3 grid((unsigned)((a.N + TILE - 1) / TILE), (unsigned)((a.M + TILE - 1) / TILE), (unsigned)a.batch);
  B2M_REQUIRE(grid.y <= 65535 && grid.z <= 65535, B2M_ERR_UNSUPPORTED, "MatMulInteger: shape too large");
  I8Extra x{a.azp_signed, a.bzp_signed};
  if (a.a_signed && a.b_signed) i8_gemm_kernel<true, true><<<grid, 256, 0, s>>>(a, x);
  else if (a.a_signed) i8_gemm_kernel<true, false><<<grid, 256, 0, s>>>(a, x);
  else if (a.b_signed) i8_gemm_kernel<false, true><<<grid, 256, 0, s>>>(a, x);
  else i8_gemm_kernel<false, false><<<grid, 256, 0, s>>>(a, x);
  B2M_CUDA(cudaGetLastError());
}

void launch_i8_pack(const void *B, int b_signed, int64_t batch, int64_t K, int64_t N, int8_t *bt,
                    int64_t kpad, int64_t npad, int32_t *colsum, cudaStream_t s) {
  dim3 grid((unsigned)((npad + 127) / 128), (unsigned)batch);
  i8_pack_kernel<<<grid, 128, 0, s>>>(reinterpret_cast<const uint8_t *>(B), b_signed, K, N, bt, kpad, npad,
                                       colsum);
  B2M_CUDA(cudaGetLastError());
}
