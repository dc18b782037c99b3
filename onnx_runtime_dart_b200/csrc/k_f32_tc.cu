// FAST-mode fp32 MatMul / Gemm on the tensor cores: 3xTF32 with tcgen05
// kind::tf32. Reference: opMatMul / opGemm, lib/src/onnx_ops.dart:1710-1766,
// 2152-2173 (fp32 GEMM semantics; FAST mode is held to the path's tolerance,
// max|d|/max|ref| <= 1e-3 and cosine >= 0.99999, not to bit equality).
//
// Each operand x is split exactly as x = hi + lo with hi = x truncated to a
// tf32 (10 explicit mantissa bits) and lo = x - hi (exact in fp32); then
//   A.B ~= A_hi.B_hi + A_hi.B_lo + A_lo.B_hi
// with all products accumulated in fp32 in TMEM. The dropped A_lo.B_lo term
// and the tf32 rounding of the lo parts are both ~2^-22 relative: fp32-class
// accuracy at tensor-core rate. The weight's hi/lo planes are made once at
// prepack (K-major); the activations are split per call by f32_split_rows.
//
// One CTA computes a 128 x BN tile of Y (rows of A x weight columns):
//   warp 0      TMA producer: per 32-k chunk, A_hi / A_lo (128 x 32) and
//               B_hi / B_lo (BN x 32) boxes into 128-byte-swizzled shared
//               memory, one mbarrier per stage.
//   warp 1      TMEM allocation; one thread issues the three MMAs per K=8
//               step (12 per chunk) and commits each stage.
//   warps 2-5   epilogue: tcgen05.ld (lane = row), alpha / beta*C, stores.
// Every wait is bounded; a timeout sets the device error word.
#include <cuda.h>

#include <algorithm>

#include "b2m_internal.cuh"
#include "ptx.cuh"
#include "tc_common.cuh"

namespace {

using namespace b2m;

constexpr int FT_THREADS = 192;
constexpr int FT_BM = 128;

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accum)
      : "memory");
}

template <int BN, int STAGES>
struct FtLayout {
  static constexpr uint32_t A_CHUNK = FT_BM * 128;  // 128 rows x 32 fp32
  static constexpr uint32_t B_CHUNK = BN * 128;
  static constexpr uint32_t STAGE = 2 * A_CHUNK + 2 * B_CHUNK;  // hi, lo of each
  static constexpr uint32_t BAR_OFF = STAGES * STAGE;
  static constexpr uint32_t SLOT_OFF = BAR_OFF + (2 * STAGES + 1) * 8;
  static constexpr uint32_t FLAG_OFF = SLOT_OFF + 8;
  static constexpr uint32_t BYTES = FLAG_OFF + 8 + 1024;
  static constexpr uint32_t TMEM_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
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
    f32_tc_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                  const __grid_constant__ CUtensorMap tb_hi, const __grid_constant__ CUtensorMap tb_lo,
                  const FtEpi e, int M, int N, int nchunks, int32_t *dev_err) {
  using L = FtLayout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
  uint64_t *empty = full + STAGES;
  uint64_t *accum = empty + STAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::SLOT_OFF);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::FLAG_OFF);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * FT_BM;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    mbar_fence_init();
    prefetch_tmap(&ta_hi);
    prefetch_tmap(&ta_lo);
    prefetch_tmap(&tb_hi);
    prefetch_tmap(&tb_lo);
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
      int issued = 0;
      for (int c = 0; c < nchunks; c++) {
        const int s = c % STAGES;
        const uint32_t ph = (uint32_t)(c / STAGES) & 1u;
        if (!wait_or_abort(&empty[s], ph ^ 1u, abort_flag, dev_err)) break;
        uint8_t *st = smem + s * L::STAGE;
        mbar_arrive_expect_tx(&full[s], L::STAGE);
        tma_load_2d(st, &ta_hi, c * 32, m0, &full[s]);
        tma_load_2d(st + L::A_CHUNK, &ta_lo, c * 32, m0, &full[s]);
        tma_load_2d(st + 2 * L::A_CHUNK, &tb_hi, c * 32, n0, &full[s]);
        tma_load_2d(st + 2 * L::A_CHUNK + L::B_CHUNK, &tb_lo, c * 32, n0, &full[s]);
        issued = c + 1;
      }
      if (issued > 0) {
        const int c = issued - 1;
        wait_or_abort(&full[c % STAGES], (uint32_t)(c / STAGES) & 1u, abort_flag, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(FT_BM, BN, 1u, 2u, 2u);  // F32 <- TF32 x TF32, K-major
      for (int c = 0; c < nchunks; c++) {
        const int s = c % STAGES;
        const uint32_t ph = (uint32_t)(c / STAGES) & 1u;
        if (!wait_or_abort(&full[s], ph, abort_flag, dev_err)) break;
        tc_fence_after();
        const uint32_t base = smem_u32(smem + s * L::STAGE);
        const uint64_t ahi = sw128_kmajor_desc(base), alo = sw128_kmajor_desc(base + L::A_CHUNK);
        const uint64_t bhi = sw128_kmajor_desc(base + 2 * L::A_CHUNK);
        const uint64_t blo = sw128_kmajor_desc(base + 2 * L::A_CHUNK + L::B_CHUNK);
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {  // K = 8 tf32 = 32 bytes per MMA
          const uint64_t o = (uint64_t)(2 * kk);
          umma_tf32(tmem, alo + o, bhi + o, idesc, (c | kk) != 0 ? 1u : 0u);
          umma_tf32(tmem, ahi + o, blo + o, idesc, 1u);
          umma_tf32(tmem, ahi + o, bhi + o, idesc, 1u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter
    const int row = m0 + q * 32 + lane;
    const bool ok = warp_wait_or_abort(accum, 0u, abort_flag, dev_err);
    tc_fence_after();
    pdl_wait();
    int go = ok && !*abort_flag;
    go = __shfl_sync(0xffffffffu, go, 0);
    if (go) {
      const bool vec = (N & 3) == 0 && (e.ldy & 3) == 0 && (reinterpret_cast<uintptr_t>(e.Y) & 15) == 0;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
        tmem_ld_wait();
        if (row < M && n0 + c0 < N) {
          float y[16];
#pragma unroll
          for (int j = 0; j < 16; j++) {
            float t = __uint_as_float(v[j]);
            const int col = n0 + c0 + j;
            if (e.has_alpha) t = t * e.alpha;
            if (e.C && col < N) {
              float cv = e.C[(int64_t)row * e.c_rs + (int64_t)col * e.c_cs];
              if (e.has_beta) cv = cv * e.beta;
              t = t + cv;
            }
            y[j] = t;
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
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// A[M][K] (row stride lda) -> hi / lo planes [M][Kp] (zero padded to Kp, a
// multiple of 32): hi = a with the low 13 mantissa bits cleared, lo = a - hi.
__global__ void __launch_bounds__(256) f32_split_rows(const float *__restrict__ A, int64_t lda, float *hi, float *lo,
                                                      int64_t M, int64_t K, int64_t Kp) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t total = M * (Kp >> 2);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / (Kp >> 2), k = (i % (Kp >> 2)) * 4;
    float x[4];
#pragma unroll
    for (int j = 0; j < 4; j++) x[j] = k + j < K ? A[m * lda + k + j] : 0.f;
    float h[4], l[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      h[j] = __uint_as_float(__float_as_uint(x[j]) & 0xFFFFE000u);
      l[j] = x[j] - h[j];
    }
    *reinterpret_cast<float4 *>(hi + m * Kp + k) = make_float4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<float4 *>(lo + m * Kp + k) = make_float4(l[0], l[1], l[2], l[3]);
  }
}

CUtensorMap make_map(const float *base, int64_t rows, int64_t kp, int box_rows) {
  CUtensorMap m;
  const cuuint64_t dims[2] = {(cuuint64_t)kp, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(kp * 4)};
  const cuuint32_t box[2] = {32u, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides,
                                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  B2M_REQUIRE(r == CUDA_SUCCESS, B2M_ERR_CUDA, "cuTensorMapEncodeTiled failed for an fp32 operand");
  return m;
}

template <int BN, int STAGES>
void launch_ft(const F32GemmArgs &p, const b2m_weight &w, const float *a_hi, const float *a_lo, int64_t kp,
               cudaStream_t s) {
  using L = FtLayout<BN, STAGES>;
  const CUtensorMap tah = make_map(a_hi, p.M, kp, FT_BM), tal = make_map(a_lo, p.M, kp, FT_BM);
  const CUtensorMap tbh = make_map(w.tf_hi, w.n, kp, BN), tbl = make_map(w.tf_lo, w.n, kp, BN);
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
  set_smem_limit_once<f32_tc_kernel<BN, STAGES>>((int)L::BYTES);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((p.N + BN - 1) / BN), (unsigned)((p.M + FT_BM - 1) / FT_BM));
  cfg.blockDim = dim3(FT_THREADS);
  cfg.dynamicSmemBytes = L::BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2M_CUDA(cudaLaunchKernelEx(&cfg, f32_tc_kernel<BN, STAGES>, tah, tal, tbh, tbl, e, (int)p.M, (int)p.N,
                              (int)(kp / 32), p.dev_err));
}

}  // namespace

int64_t f32_tc_kp(int64_t K) { return (K + 31) / 32 * 32; }

bool f32_tc_eligible(const F32GemmArgs &p, const b2m_weight *w) {
  return w && w->tf_hi && p.batch == 1 && p.sa_k == 1 && p.sa_m == p.K && p.M >= 1 && p.N >= 1 &&
         p.M <= (int64_t)65535 * FT_BM && p.K <= ((int64_t)1 << 30) && p.epi != EPI_NBITS && p.epi != EPI_NBITS_M1;
}

void launch_f32_tc(const F32GemmArgs &p, const b2m_weight &w, float *a_split, cudaStream_t s) {
  const int64_t kp = f32_tc_kp(p.K);
  float *a_hi = a_split, *a_lo = a_split + p.M * kp;
  {
    const int64_t total = p.M * (kp / 4);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>(device_sm_count() * 4, (total + 255) / 256)));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    B2M_CUDA(cudaLaunchKernelEx(&cfg, f32_split_rows, p.A, p.sa_m, a_hi, a_lo, p.M, p.K, kp));
  }
  // Column tile: the widest that still gives about one CTA per SM.
  const int sms = device_sm_count();
  const int64_t mt = (p.M + FT_BM - 1) / FT_BM;
  if (mt * ((p.N + 127) / 128) >= sms) launch_ft<128, 3>(p, w, a_hi, a_lo, kp, s);
  else if (mt * ((p.N + 63) / 64) >= sms / 2) launch_ft<64, 4>(p, w, a_hi, a_lo, kp, s);
  else launch_ft<32, 5>(p, w, a_hi, a_lo, kp, s);
}
