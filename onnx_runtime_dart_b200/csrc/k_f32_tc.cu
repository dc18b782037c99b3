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
//   warp 0      TMA producer: per BK-wide k chunk (32 or 64), A0 / A1
//               (128 x BK) and B0 / B1 (BN x BK) boxes into swizzled shared
//               memory (64- or 128-byte rows).
//   warp 1      TMEM allocation; one thread issues the MMAs of a chunk
//               (BK/16 K=16 steps x 3 products) into one of two accumulators.
//   warps 2-5   epilogue of the other accumulator: tcgen05.ld (lane = row),
//               a 32 x 32 transpose through shared memory, alpha / beta*C and
//               row-contiguous stores; it overlaps the next tile's MMAs.
// Every wait is bounded; a timeout sets the device error word.
#include <cuda.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <climits>

#include "b2m_internal.cuh"
#include "ptx.cuh"
#include "tc_common.cuh"

namespace {

using namespace b2m;

constexpr int FT_THREADS = 192;
constexpr int FT_BM = 128;
constexpr int FT_KPAD = 64;  // K padding of the split planes

// K-major shared-memory descriptor for BK-wide bf16 rows: 128-byte swizzle
// for BK = 64, 64-byte swizzle for BK = 32 (8-row core groups, SBO = 8 rows).
template <int BK>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr) {
  if constexpr (BK == 64) {
    return sw128_kmajor_desc(saddr);
  } else {
    static_assert(BK == 32, "chunk width");
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address, 16-byte units
    d |= (uint64_t)1 << 16;                    // leading byte offset (unused when swizzled)
    d |= (uint64_t)(512 >> 4) << 32;           // stride byte offset: 8 rows x 64 B
    d |= (uint64_t)1 << 46;                    // descriptor version (sm_100)
    d |= (uint64_t)4 << 61;                    // swizzle: 64-byte
    return d;
  }
}

template <int BN, int STAGES, int BK>
struct FtLayout {
  static constexpr uint32_t A_CHUNK = FT_BM * BK * 2;  // 128 rows x BK bf16
  static constexpr uint32_t B_CHUNK = BN * BK * 2;
  static constexpr uint32_t STAGE = 2 * A_CHUNK + 2 * B_CHUNK;  // x0, x1 of each
  static constexpr uint32_t BAR_OFF = STAGES * STAGE;
  // full[S], empty[S], acc_full[2], acc_empty[2], drain
  static constexpr uint32_t SLOT_OFF = BAR_OFF + (2 * STAGES + 5) * 8;
  static constexpr uint32_t FLAG_OFF = SLOT_OFF + 8;
  static constexpr uint32_t EPI_OFF = FLAG_OFF + 16;               // 4 warps x 32 x 33 floats
  static constexpr uint32_t BYTES = EPI_OFF + 4 * 32 * 33 * 4 + 1024;
  static constexpr uint32_t ACC_COLS = BN;
  static constexpr uint32_t TMEM_COLS = 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "column tile");
  static_assert(BK == 32 || BK == 64, "chunk width");
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
  // Channel-major output (convolution): when cm_P > 0, row i of the GEMM is
  // pixel i % cm_P of image i / cm_P, and Y(i, j) lands at
  // Y[(i / cm_P) * cm_bs + j * cm_P + i % cm_P], the NC[D]HW layout. Lane =
  // row in TMEM, so each store instruction of a warp writes 32 consecutive
  // pixels of one channel.
  int64_t cm_P, cm_bs;
};

template <int BN, int STAGES, int BK>
__global__ void __launch_bounds__(FT_THREADS, 1)
    f32_tc_kernel(const __grid_constant__ CUtensorMap ta0, const __grid_constant__ CUtensorMap ta1,
                  const __grid_constant__ CUtensorMap tb0, const __grid_constant__ CUtensorMap tb1,
                  const FtEpi e, int M, int N, int nchunks, int mtiles, int ntiles, int32_t *dev_err) {
  using L = FtLayout<BN, STAGES, BK>;
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
          tma_load_2d(st, &ta0, c * BK, m0, &full[s]);
          tma_load_2d(st + L::A_CHUNK, &ta1, c * BK, m0, &full[s]);
          tma_load_2d(st + 2 * L::A_CHUNK, &tb0, c * BK, n0, &full[s]);
          tma_load_2d(st + 2 * L::A_CHUNK + L::B_CHUNK, &tb1, c * BK, n0, &full[s]);
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
          const uint64_t a0 = kmajor_desc<BK>(base), a1 = kmajor_desc<BK>(base + L::A_CHUNK);
          const uint64_t b0 = kmajor_desc<BK>(base + 2 * L::A_CHUNK);
          const uint64_t b1 = kmajor_desc<BK>(base + 2 * L::A_CHUNK + L::B_CHUNK);
#pragma unroll
          for (int kk = 0; kk < BK / 16; kk++) {  // K = 16 bf16 = 32 bytes per MMA
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
    // Per-warp 32 x 33 transpose buffer: the accumulator arrives one row per
    // lane; it leaves one column per lane, so every store instruction writes
    // 128 contiguous bytes of one output row.
    float *tb = reinterpret_cast<float *>(smem + L::EPI_OFF) + (warp - 2) * (32 * 33);
    pdl_wait();  // Y may still be read by the kernels this one overlaps
    int local = 0;
    for (int t = blockIdx.x; t < ntile_total; t += gridDim.x, local++) {
      const int buf = local & 1;
      const uint32_t use = (uint32_t)(local >> 1);
      if (!warp_wait_or_abort(&acc_full[buf], use & 1u, abort_flag, dev_err)) break;
      tc_fence_after();
      const int m0 = (t / ntiles) * FT_BM, n0 = (t % ntiles) * BN;
      const int r0 = m0 + q * 32;
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * L::ACC_COLS);
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        tmem_ld16(tbase + (uint32_t)c0, *reinterpret_cast<uint32_t(*)[16]>(v));
        tmem_ld16(tbase + (uint32_t)c0 + 16u, *reinterpret_cast<uint32_t(*)[16]>(v + 16));
        tmem_ld_wait();
        if (c0 + 32 == BN) {
          // The accumulator is fully read: release it to the MMA warp early.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acc_empty[buf]);
        }
        if (n0 + c0 >= N || r0 >= M) continue;
        if (e.cm_P > 0) {
          const int row = r0 + lane;
          if (row < M) {
            const int64_t img = row / e.cm_P, pix = row - img * e.cm_P;
            float *yb = e.Y + img * e.cm_bs + pix;
#pragma unroll
            for (int j = 0; j < 32; j++) {
              const int col = n0 + c0 + j;
              if (col < N) {
                float tv = __uint_as_float(v[j]);
                if (e.has_alpha) tv = tv * e.alpha;
                if (e.C) {
                  float cv = e.C[(int64_t)col * e.c_cs];
                  if (e.has_beta) cv = cv * e.beta;
                  tv = tv + cv;
                }
                yb[(int64_t)col * e.cm_P] = tv;
              }
            }
          }
          continue;
        }
#pragma unroll
        for (int j = 0; j < 32; j++) tb[lane * 33 + j] = __uint_as_float(v[j]);
        __syncwarp();
        const int col = n0 + c0 + lane;
        if (col < N) {
          float cv_bcast = 0.f;
          const bool bcast = e.C && e.c_rs == 0;
          if (bcast) {
            cv_bcast = e.C[(int64_t)col * e.c_cs];
            if (e.has_beta) cv_bcast = cv_bcast * e.beta;
          }
          const int rows = min(32, M - r0);
          float *yc = e.Y + (int64_t)r0 * e.ldy + col;
#pragma unroll 4
          for (int i = 0; i < rows; i++) {
            float tv = tb[i * 33 + lane];
            if (e.has_alpha) tv = tv * e.alpha;
            if (bcast) {
              tv = tv + cv_bcast;
            } else if (e.C) {
              float cv = e.C[(int64_t)(r0 + i) * e.c_rs + (int64_t)col * e.c_cs];
              if (e.has_beta) cv = cv * e.beta;
              tv = tv + cv;
            }
            yc[(int64_t)i * e.ldy] = tv;
          }
        }
        __syncwarp();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// A[M][K] (row stride lda) -> x0 / x1 bf16 planes [M][Kp] (zero padded to Kp,
// a multiple of 64), eight k per thread and step.
__global__ void __launch_bounds__(256) f32_split_rows(const float *__restrict__ A, int64_t lda, __nv_bfloat16 *p0,
                                                      __nv_bfloat16 *p1, int64_t M, int64_t K, int64_t Kp) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t groups = Kp >> 3, total = M * groups;
  const bool vec = (lda & 3) == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0;
  const bool narrow = total < INT32_MAX;  // 32-bit index division
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t m, k;
    if (narrow) {
      const int q = (int)i / (int)groups;
      m = q;
      k = ((int)i - q * (int)groups) * 8;
    } else {
      m = i / groups;
      k = (i % groups) * 8;
    }
    const float *src = A + m * lda + k;
    float x[8];
    if (vec && k + 8 <= K) {
      const float4 u = *reinterpret_cast<const float4 *>(src), w = *reinterpret_cast<const float4 *>(src + 4);
      x[0] = u.x, x[1] = u.y, x[2] = u.z, x[3] = u.w, x[4] = w.x, x[5] = w.y, x[6] = w.z, x[7] = w.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++) x[j] = k + j < K ? src[j] : 0.f;
    }
    uint4 h, l;
    split_bf16x2(x[0], x[1], h.x, l.x);
    split_bf16x2(x[2], x[3], h.y, l.y);
    split_bf16x2(x[4], x[5], h.z, l.z);
    split_bf16x2(x[6], x[7], h.w, l.w);
    *reinterpret_cast<uint4 *>(p0 + m * Kp + k) = h;
    *reinterpret_cast<uint4 *>(p1 + m * Kp + k) = l;
  }
}

CUtensorMap make_map(const void *base, int64_t rows, int64_t kp, int box_rows, int bk) {
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)kp, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(kp * 2)};
  const cuuint32_t box[2] = {(cuuint32_t)bk, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides,
                                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                    bk == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  B2M_REQUIRE(r == CUDA_SUCCESS, B2M_ERR_CUDA, "cuTensorMapEncodeTiled failed for a bf16 operand plane");
  return m;
}

// B operand planes (K-major bf16 [b_rows][kp]) and the output layout of one
// launch.
struct FtOperandB {
  const void *hi, *lo;
  int64_t rows;
  int64_t cm_P = 0, cm_bs = 0;
};

template <int BN, int STAGES, int BK>
void launch_ft(const F32GemmArgs &p, const FtOperandB &b, const __nv_bfloat16 *a0, const __nv_bfloat16 *a1,
               int64_t kp, cudaStream_t s) {
  using L = FtLayout<BN, STAGES, BK>;
  const CUtensorMap t0 = make_map(a0, p.M, kp, FT_BM, BK), t1 = make_map(a1, p.M, kp, FT_BM, BK);
  const CUtensorMap u0 = make_map(b.hi, b.rows, kp, BN, BK), u1 = make_map(b.lo, b.rows, kp, BN, BK);
  FtEpi e;
  e.cm_P = b.cm_P;
  e.cm_bs = b.cm_bs;
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
  set_smem_limit_once<f32_tc_kernel<BN, STAGES, BK>>((int)L::BYTES);
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
  B2M_CUDA(cudaLaunchKernelEx(&cfg, f32_tc_kernel<BN, STAGES, BK>, t0, t1, u0, u1, e, (int)p.M, (int)p.N,
                              (int)(kp / BK), mt, nt, p.dev_err));
}

}  // namespace

int64_t f32_tc_kp(int64_t K) { return (K + FT_KPAD - 1) / FT_KPAD * FT_KPAD; }

size_t f32_tc_scratch_bytes(int64_t M, int64_t K) { return (size_t)(2 * M * f32_tc_kp(K) * 2); }

bool f32_tc_shape_ok(const F32GemmArgs &p) {
  return p.batch == 1 && p.sa_k == 1 && p.sa_m == p.K && p.M >= 1 && p.N >= 1 &&
         (p.M + FT_BM - 1) / FT_BM * ((p.N + 31) / 32) <= ((int64_t)1 << 31) - 1 && p.K <= ((int64_t)1 << 30) &&
         p.epi != EPI_NBITS && p.epi != EPI_NBITS_M1;
}

bool f32_tc_eligible(const F32GemmArgs &p, const b2m_weight *w) { return w && w->bx_hi && f32_tc_shape_ok(p); }

namespace {

// Column tile by a makespan model: rounds of tiles over the SMs times the
// tile width, over a relative mainloop efficiency per width (narrow tiles
// re-read A more often per flop). 32-k stages keep four or more stages in
// flight at every width.
void launch_ft_any(const F32GemmArgs &p, const FtOperandB &b, const __nv_bfloat16 *a0, const __nv_bfloat16 *a1,
                   int64_t kp, cudaStream_t s) {
  const int sms = device_sm_count();
  const int64_t mt = (p.M + FT_BM - 1) / FT_BM;
  static const int widths[5] = {256, 192, 128, 64, 32};
  static const double eff[5] = {0.9, 0.88, 0.8, 0.6, 0.4};
  int best = 0;
  double best_cost = 0.0;
  for (int i = 0; i < 5; i++) {
    const int64_t tiles = mt * ((p.N + widths[i] - 1) / widths[i]);
    const double cost = (double)((tiles + sms - 1) / sms) * widths[i] / eff[i];
    if (i == 0 || cost < best_cost) {
      best = i;
      best_cost = cost;
    }
  }
  switch (widths[best]) {
    case 256: launch_ft<256, 4, 32>(p, b, a0, a1, kp, s); break;
    case 192: launch_ft<192, 5, 32>(p, b, a0, a1, kp, s); break;
    case 128: launch_ft<128, 6, 32>(p, b, a0, a1, kp, s); break;
    case 64: launch_ft<64, 8, 32>(p, b, a0, a1, kp, s); break;
    default: launch_ft<32, 8, 32>(p, b, a0, a1, kp, s); break;
  }
}

}  // namespace

void launch_f32_tc_planes(const F32GemmArgs &p, const void *b_hi, const void *b_lo, int64_t b_rows,
                          const void *a_planes, int64_t cm_P, int64_t cm_bs, cudaStream_t s) {
  const int64_t kp = f32_tc_kp(p.K);
  const __nv_bfloat16 *a0 = static_cast<const __nv_bfloat16 *>(a_planes), *a1 = a0 + p.M * kp;
  FtOperandB b;
  b.hi = b_hi;
  b.lo = b_lo;
  b.rows = b_rows;
  b.cm_P = cm_P;
  b.cm_bs = cm_bs;
  launch_ft_any(p, b, a0, a1, kp, s);
}

void launch_f32_split(const float *A, int64_t lda, __nv_bfloat16 *p0, __nv_bfloat16 *p1, int64_t M, int64_t K,
                      int64_t kp, cudaStream_t s) {
  const int64_t total = M * (kp / 8);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>(device_sm_count() * 8, (total + 255) / 256)));
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2M_CUDA(cudaLaunchKernelEx(&cfg, f32_split_rows, A, lda, p0, p1, M, K, kp));
}

void launch_f32_tc(const F32GemmArgs &p, const b2m_weight &w, void *a_split, cudaStream_t s) {
  launch_f32_tc_b(p, w.bx_hi, w.bx_lo, w.n, a_split, s);
}

void launch_f32_tc_b(const F32GemmArgs &p, const void *b_hi, const void *b_lo, int64_t b_rows, void *a_split,
                     cudaStream_t s) {
  const int64_t kp = f32_tc_kp(p.K);
  __nv_bfloat16 *a0 = static_cast<__nv_bfloat16 *>(a_split), *a1 = a0 + p.M * kp;
  launch_f32_split(p.A, p.sa_m, a0, a1, p.M, p.K, kp, s);
  FtOperandB b;
  b.hi = b_hi;
  b.lo = b_lo;
  b.rows = b_rows;
  launch_ft_any(p, b, a0, a1, kp, s);
}
