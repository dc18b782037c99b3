// FAST-mode fp32 MatMul / Gemm on the tensor cores: three bf16 products with
// tcgen05 kind::f16 (bf16 x bf16 -> f32). Reference: opMatMul / opGemm,
// lib/src/onnx_ops.dart:1710-1766, 2152-2173 (fp32 GEMM semantics; FAST mode
// is held to the path's tolerance, max|d|/max|ref| <= 1e-3 and cosine >=
// 0.99999, not to bit equality).
//
// Each fp32 operand x is split into two bf16 terms, x0 = rn(x) and
// x1 = rn(x - x0) (x - x0 is exact in fp32), so |x - x0 - x1| <= 2^-16 |x|.
// Then
//   A.B ~= A0.B0 + A0.B1 + A1.B0
// with every product exact and accumulated in fp32 in TMEM; the dropped A1.B1
// term and the split residuals bound the error per product near 3 * 2^-16
// relative (1e-3 is the contract). Two bf16 planes carry the same bytes as
// one fp32 operand, and a bf16 MMA does twice the work of a tf32 one per
// cycle, so this costs half the shared-memory traffic and half the tensor time
// of a three-product tf32 split. The weight's planes are made once at prepack
// (K-major, K padded to 64); the activations are split per call by
// f32_split_rows.
//
// Persistent kernel, one CTA per SM walking 128 x BN output tiles:
//   warp 0      TMA producer: per 64-k chunk, A0 / A1 (128 x 64) and B0 / B1
//               (BN x 64) boxes into 128-byte-swizzled shared memory.
//   warp 1      TMEM allocation; one thread issues the 12 MMAs of a chunk
//               (4 K=16 steps x 3 products) into one of two accumulators.
//   warps 2-5   epilogue of the other accumulator: tcgen05.ld (lane = row),
//               alpha / beta*C, stores; it overlaps the next tile's MMAs.
// Every wait is bounded; a timeout sets the device error word.
#include <cuda.h>
#include <cuda_bf16.h>

#include <algorithm>

#include "b2m_internal.cuh"
#include "ptx.cuh"
#include "tc_common.cuh"

namespace {

using namespace b2m;

constexpr int FT_THREADS = 192;
constexpr int FT_BM = 128;
constexpr int FT_BK = 64;  // bf16 per 128-byte swizzle row

template <int BN, int STAGES>
struct FtLayout {
  static constexpr uint32_t A_CHUNK = FT_BM * 128;  // 128 rows x 64 bf16
  static constexpr uint32_t B_CHUNK = BN * 128;
  static constexpr uint32_t STAGE = 2 * A_CHUNK + 2 * B_CHUNK;  // x0, x1 of each
  static constexpr uint32_t BAR_OFF = STAGES * STAGE;
  // full[S], empty[S], acc_full[2], acc_empty[2], drain
  static constexpr uint32_t SLOT_OFF = BAR_OFF + (2 * STAGES + 5) * 8;
  static constexpr uint32_t FLAG_OFF = SLOT_OFF + 8;
  static constexpr uint32_t BYTES = FLAG_OFF + 8 + 1024;
  static constexpr uint32_t ACC_COLS = BN;
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "column tile");
  static_assert(BYTES <= 232448, "shared memory");
};

struct FtEpi {
  float *Y;
  int64_t ldy;
  int has_alpha;
  float alpha;
  const float *C;  // Gemm addend (broadcast through its strides) or null
  int64_t c_rs, c_cs;
  int has_beta;
  float beta;
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(FT_THREADS, 1)
    f32_tc_kernel(const __grid_constant__ CUtensorMap ta0, const __grid_constant__ CUtensorMap ta1,
                  const __grid_constant__ CUtensorMap tb0, const __grid_constant__ CUtensorMap tb1,
                  const FtEpi e, int M, int N, int nchunks, int mtiles, int ntiles, int32_t *dev_err) {
  using L = FtLayout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
  uint64_t *empty = full + STAGES;
  uint64_t *acc_full = empty + STAGES;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *drain = acc_empty + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::SLOT_OFF);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::FLAG_OFF);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntile_total = mtiles * ntiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // lane 0 of each epilogue warp
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    mbar_fence_init();
    prefetch_tmap(&ta0);
    prefetch_tmap(&ta1);
    prefetch_tmap(&tb0);
    prefetch_tmap(&tb1);
  }
  if (warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      pdl_wait();  // the split activations come from the kernel launched just before
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntile_total && ok; t += gridDim.x) {
        const int m0 = (t / ntiles) * FT_BM, n0 = (t % ntiles) * BN;
        for (int c = 0; c < nchunks; c++, it++) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!wait_or_abort(&empty[s], ph ^ 1u, abort_flag, dev_err)) {
            ok = false;
            break;
          }
          uint8_t *st = smem + s * L::STAGE;
          mbar_arrive_expect_tx(&full[s], L::STAGE);
          tma_load_2d(st, &ta0, c * FT_BK, m0, &full[s]);
          tma_load_2d(st + L::A_CHUNK, &ta1, c * FT_BK, m0, &full[s]);
          tma_load_2d(st + 2 * L::A_CHUNK, &tb0, c * FT_BK, n0, &full[s]);
          tma_load_2d(st + 2 * L::A_CHUNK + L::B_CHUNK, &tb1, c * FT_BK, n0, &full[s]);
        }
      }
      // Loads still in flight after an abort land before the CTA exits.
      for (int j = it - 1; j >= 0 && j >= it - STAGES; j--)
        wait_or_abort(&full[j % STAGES], (uint32_t)(j / STAGES) & 1u, abort_flag, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(FT_BM, BN, 1u, 1u, 1u);  // F32 <- BF16 x BF16, K-major
      int it = 0, local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < ntile_total && ok; t += gridDim.x, local++) {
        const int buf = local & 1;
        const uint32_t use = (uint32_t)(local >> 1);
        if (!wait_or_abort(&acc_empty[buf], (use & 1u) ^ 1u, abort_flag, dev_err)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * L::ACC_COLS);
        for (int c = 0; c < nchunks; c++, it++) {
          const int s = it % STAGES;
          const uint32_t ph = (uint32_t)(it / STAGES) & 1u;
          if (!wait_or_abort(&full[s], ph, abort_flag, dev_err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t base = smem_u32(smem + s * L::STAGE);
          const uint64_t a0 = sw128_kmajor_desc(base), a1 = sw128_kmajor_desc(base + L::A_CHUNK);
          const uint64_t b0 = sw128_kmajor_desc(base + 2 * L::A_CHUNK);
          const uint64_t b1 = sw128_kmajor_desc(base + 2 * L::A_CHUNK + L::B_CHUNK);
#pragma unroll
          for (int kk = 0; kk < 4; kk++) {  // K = 16 bf16 = 32 bytes per MMA
            const uint64_t o = (uint64_t)(2 * kk);
            umma_f16(d, a1 + o, b0 + o, idesc, (c | kk) != 0 ? 1u : 0u);
            umma_f16(d, a0 + o, b1 + o, idesc, 1u);
            umma_f16(d, a0 + o, b0 + o, idesc, 1u);
          }
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[buf]);
      }
      // Every MMA issued has retired before TMEM is released.
      umma_commit(drain);
      wait_or_abort(drain, 0u, abort_flag, nullptr);
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter
    const bool vec = (N & 3) == 0 && (e.ldy & 3) == 0 && (reinterpret_cast<uintptr_t>(e.Y) & 15) == 0;
    pdl_wait();  // Y may still be read by the kernels this one overlaps
    int local = 0;
    for (int t = blockIdx.x; t < ntile_total; t += gridDim.x, local++) {
      const int buf = local & 1;
      const uint32_t use = (uint32_t)(local >> 1);
      if (!warp_wait_or_abort(&acc_full[buf], use & 1u, abort_flag, dev_err)) break;
      tc_fence_after();
      const int m0 = (t / ntiles) * FT_BM, n0 = (t % ntiles) * BN;
      const int row = m0 + q * 32 + lane;
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * L::ACC_COLS);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tbase + (uint32_t)c0, v);
        tmem_ld_wait();
        if (row < M && n0 + c0 < N) {
          float y[16];
#pragma unroll
          for (int j = 0; j < 16; j++) {
            float tv = __uint_as_float(v[j]);
            const int col = n0 + c0 + j;
            if (e.has_alpha) tv = tv * e.alpha;
            if (e.C && col < N) {
              float cv = e.C[(int64_t)row * e.c_rs + (int64_t)col * e.c_cs];
              if (e.has_beta) cv = cv * e.beta;
              tv = tv + cv;
            }
            y[j] = tv;
          }
          float *yr = e.Y + (int64_t)row * e.ldy + n0 + c0;
          if (vec && n0 + c0 + 16 <= N) {
#pragma unroll
            for (int j = 0; j < 16; j += 4)
              *reinterpret_cast<float4 *>(yr + j) = make_float4(y[j], y[j + 1], y[j + 2], y[j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 16; j++)
              if (n0 + c0 + j < N) yr[j] = y[j];
          }
        }
      }
      // This warp's quarter of the accumulator is free for the tile after next.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// x -> (x0, x1) = (rn_bf16(x), rn_bf16(x - x0)). A finite x whose rounding
// overflows bf16 keeps its truncation as x0; a non-finite x passes through x0.
__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16 &h, __nv_bfloat16 &l) {
  h = __float2bfloat16_rn(x);
  float hf = __bfloat162float(h);
  if (isinf(hf) && isfinite(x)) {
    h = __float2bfloat16_rz(x);
    hf = __bfloat162float(h);
  }
  l = __float2bfloat16_rn(isfinite(x) ? x - hf : 0.f);
}

// A[M][K] (row stride lda) -> x0 / x1 bf16 planes [M][Kp] (zero padded to Kp,
// a multiple of 64), eight k per thread and step.
__global__ void __launch_bounds__(256) f32_split_rows(const float *__restrict__ A, int64_t lda, __nv_bfloat16 *p0,
                                                      __nv_bfloat16 *p1, int64_t M, int64_t K, int64_t Kp) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t groups = Kp >> 3, total = M * groups;
  const bool vec = (lda & 3) == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / groups, k = (i % groups) * 8;
    const float *src = A + m * lda + k;
    float x[8];
    if (vec && k + 8 <= K) {
      const float4 u = *reinterpret_cast<const float4 *>(src), w = *reinterpret_cast<const float4 *>(src + 4);
      x[0] = u.x, x[1] = u.y, x[2] = u.z, x[3] = u.w, x[4] = w.x, x[5] = w.y, x[6] = w.z, x[7] = w.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++) x[j] = k + j < K ? src[j] : 0.f;
    }
    __align__(16) __nv_bfloat16 h[8], l[8];
#pragma unroll
    for (int j = 0; j < 8; j++) split_bf16(x[j], h[j], l[j]);
    *reinterpret_cast<uint4 *>(p0 + m * Kp + k) = *reinterpret_cast<const uint4 *>(h);
    *reinterpret_cast<uint4 *>(p1 + m * Kp + k) = *reinterpret_cast<const uint4 *>(l);
  }
}

CUtensorMap make_map(const void *base, int64_t rows, int64_t kp, int box_rows) {
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)kp, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(kp * 2)};
  const cuuint32_t box[2] = {(cuuint32_t)FT_BK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides,
                                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  B2M_REQUIRE(r == CUDA_SUCCESS, B2M_ERR_CUDA, "cuTensorMapEncodeTiled failed for a bf16 operand plane");
  return m;
}

template <int BN, int STAGES>
void launch_ft(const F32GemmArgs &p, const b2m_weight &w, const __nv_bfloat16 *a0, const __nv_bfloat16 *a1,
               int64_t kp, cudaStream_t s) {
  using L = FtLayout<BN, STAGES>;
  const CUtensorMap t0 = make_map(a0, p.M, kp, FT_BM), t1 = make_map(a1, p.M, kp, FT_BM);
  const CUtensorMap u0 = make_map(w.bx_hi, w.n, kp, BN), u1 = make_map(w.bx_lo, w.n, kp, BN);
  FtEpi e;
  e.Y = p.Y;
  e.ldy = p.ldy;
  e.has_alpha = p.epi == EPI_GEMM ? p.has_alpha : 0;
  e.alpha = p.alpha;
  e.C = p.epi == EPI_GEMM ? p.C : nullptr;
  e.c_rs = p.c_rs;
  e.c_cs = p.c_cs;
  e.has_beta = p.has_beta;
  e.beta = p.beta;
  const int mt = (int)((p.M + FT_BM - 1) / FT_BM), nt = (int)((p.N + BN - 1) / BN);
  const int64_t tiles = (int64_t)mt * nt;
  set_smem_limit_once<f32_tc_kernel<BN, STAGES>>((int)L::BYTES);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)std::min<int64_t>(tiles, device_sm_count()));
  cfg.blockDim = dim3(FT_THREADS);
  cfg.dynamicSmemBytes = L::BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2M_CUDA(cudaLaunchKernelEx(&cfg, f32_tc_kernel<BN, STAGES>, t0, t1, u0, u1, e, (int)p.M, (int)p.N,
                              (int)(kp / FT_BK), mt, nt, p.dev_err));
}

}  // namespace

int64_t f32_tc_kp(int64_t K) { return (K + FT_BK - 1) / FT_BK * FT_BK; }

size_t f32_tc_scratch_bytes(int64_t M, int64_t K) { return (size_t)(2 * M * f32_tc_kp(K) * 2); }

bool f32_tc_eligible(const F32GemmArgs &p, const b2m_weight *w) {
  return w && w->bx_hi && p.batch == 1 && p.sa_k == 1 && p.sa_m == p.K && p.M >= 1 && p.N >= 1 &&
         (p.M + FT_BM - 1) / FT_BM * ((p.N + 31) / 32) <= ((int64_t)1 << 31) - 1 && p.K <= ((int64_t)1 << 30) &&
         p.epi != EPI_NBITS && p.epi != EPI_NBITS_M1;
}

void launch_f32_tc(const F32GemmArgs &p, const b2m_weight &w, void *a_split, cudaStream_t s) {
  const int64_t kp = f32_tc_kp(p.K);
  __nv_bfloat16 *a0 = static_cast<__nv_bfloat16 *>(a_split), *a1 = a0 + p.M * kp;
  {
    const int64_t total = p.M * (kp / 8);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>(device_sm_count() * 8, (total + 255) / 256)));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    B2M_CUDA(cudaLaunchKernelEx(&cfg, f32_split_rows, p.A, p.sa_m, a0, a1, p.M, p.K, kp));
  }
  // Column tile: 256 when that still gives every SM a tile, else narrower.
  const int sms = device_sm_count();
  const int64_t mt = (p.M + FT_BM - 1) / FT_BM;
  if (mt * ((p.N + 255) / 256) >= sms) launch_ft<256, 2>(p, w, a0, a1, kp, s);
  else if (mt * ((p.N + 127) / 128) >= sms / 2) launch_ft<128, 3>(p, w, a0, a1, kp, s);
  else if (mt * ((p.N + 63) / 64) >= sms / 2) launch_ft<64, 4>(p, w, a0, a1, kp, s);
  else launch_ft<32, 4>(p, w, a0, a1, kp, s);
}
