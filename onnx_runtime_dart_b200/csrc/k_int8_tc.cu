// MatMulInteger / QLinearMatMul with a prepacked weight on the tensor cores,
// reference: opMatMulInteger / opQLinearMatMul, lib/src/onnx_qlinear_ops.dart:32-108.
//
//   raw[t, n] = sum_k a[t, k] * b[k, n]                      (exact, int32)
//   y = raw - az(t) * colsum(n) - bz(n) * rowsum(t) + K * az(t) * bz(n)
//
// in wrapping 32-bit arithmetic, which equals the reference's
// sum_k (a - az)(b - bz) whenever that fits int32 (the host rejects K > 33025).
// QLinearMatMul requantizes the int32 exactly like the reference.
//
// Prefill (i8_ts_kernel, M > I8_GEMV_MAX_M): one CTA owns 128 weight columns
// x BT tokens. The int8 weight tile is the A operand of tcgen05.mma.kind::i8
// and lives in TMEM: copy warps load each column's bytes from the ts8 layout
// (coalesced 16-byte loads) and write them with tcgen05.st, so the weights
// never pass through shared memory. The uint8/int8 activations are the B
// operand, brought into 128-byte-swizzled shared memory by TMA straight from
// the caller's [M][K] rows. The accumulator is S32 in TMEM (lane = weight
// column, column = token).
//   warp 0      TMA producer
//   warp 1      TMEM allocation; one thread issues the MMAs
//   warps 2-9   two copy groups (alternate 256-k stages), then the epilogue
// The activation row sums that b zero points need come from i8_rowsum_kernel,
// launched just before (summing them from the shared-memory stages inside
// this kernel stalled the tensor core's operand reads).
// Decode (i8_gemv_kernel, M <= I8_GEMV_MAX_M): weight-streaming dp4a GEMV over
// the same ts8 layout, activations in shared memory.
// Every wait is bounded; a timeout sets the device error word.
#include <cuda.h>

#include <algorithm>

#include "b2m_internal.cuh"
#include "ptx.cuh"
#include "tc_common.cuh"

namespace {

using namespace b2m;

constexpr int I8_THREADS = 320;
constexpr uint32_t I8_TMEM_COLS = 512;
constexpr int I8_KSUB = 2;          // 128-k chunks per pipeline stage
constexpr int I8_GEMV_MAX_M = 16;

// Zero points and output of one call, resolved by the host to the reference's
// rules (:37-44): mode 0 = none, 1 = scalar, 2 = per row (a) / per column (b).
struct I8Epi {
  const void *azp;
  int az_mode, az_signed;
  const void *bzp;
  int bz_mode, bz_signed;
  int32_t *Y32;  // MatMulInteger output, or
  void *Yq;      // QLinearMatMul output (uint8 when lo == 0, else int8)
  double mult;
  int32_t y_zp, lo, hi;
};

__device__ __forceinline__ int32_t zp_load(const void *zp, int is_signed, int64_t i) {
  return is_signed ? (int32_t)__ldg(reinterpret_cast<const int8_t *>(zp) + i)
                   : (int32_t)__ldg(reinterpret_cast<const uint8_t *>(zp) + i);
}

__device__ __forceinline__ int32_t az_at(const I8Epi &e, int64_t t) {
  return e.az_mode == 0 ? 0 : zp_load(e.azp, e.az_signed, e.az_mode == 1 ? 0 : t);
}
__device__ __forceinline__ int32_t bz_at(const I8Epi &e, int64_t n) {
  return e.bz_mode == 0 ? 0 : zp_load(e.bzp, e.bz_signed, e.bz_mode == 1 ? 0 : n);
}

template <bool S>
__device__ __forceinline__ int dp4_ones(uint32_t x, int c) {
  int d;
  if (S) asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(x), "r"(0x01010101), "r"(c));
  else asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(x), "r"(0x01010101), "r"(c));
  return d;
}

template <bool AS, bool WS>
__device__ __forceinline__ int dp4(uint32_t a, uint32_t w, int c) {
  int d;
  if (AS && WS) asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(w), "r"(c));
  else if (AS) asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(w), "r"(c));
  else if (WS) asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(w), "r"(c));
  else asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(w), "r"(c));
  return d;
}

// The output conversion of one corrected int32 element.
template <bool REQ>
__device__ __forceinline__ void i8_emit(const I8Epi &e, int64_t idx, int32_t yi) {
  if constexpr (!REQ) {
    e.Y32[idx] = yi;
  } else {
    const float f = __double2float_rn(__dmul_rn((double)yi, e.mult));
    long long q = __float2ll_rn(f) + (long long)e.y_zp;
    q = q < e.lo ? e.lo : (q > e.hi ? e.hi : q);
    if (e.lo < 0) reinterpret_cast<int8_t *>(e.Yq)[idx] = (int8_t)q;
    else reinterpret_cast<uint8_t *>(e.Yq)[idx] = (uint8_t)q;
  }
}

template <int BT, int STAGES>
struct I8Layout {
  static constexpr uint32_t B_CHUNK = (uint32_t)BT * 128;  // 128 k x BT tokens, one byte each
  static constexpr uint32_t B_STAGE = I8_KSUB * B_CHUNK;
  static constexpr uint32_t BAR_OFF = STAGES * B_STAGE;
  static constexpr uint32_t TOK_OFF = BAR_OFF + (2 * STAGES + 1) * 8;  // az[BT], u[BT] int32
  static constexpr uint32_t SLOT_OFF = TOK_OFF + (uint32_t)BT * 8;
  static constexpr uint32_t FLAG_OFF = SLOT_OFF + 8;
  static constexpr uint32_t BYTES = FLAG_OFF + 8 + 1024;  // + alignment slack
  static constexpr uint32_t A_COL0 = (uint32_t)(BT + 31) / 32 * 32;
  static constexpr uint32_t A_STAGE_COLS = I8_KSUB * 32;
  static_assert(BT % 32 == 0 && BT >= 32 && BT <= 256, "token tile");
  static_assert(A_COL0 + STAGES * A_STAGE_COLS <= I8_TMEM_COLS, "accumulator + weight stages exceed TMEM");
  static_assert(BYTES <= 232448, "shared memory");
};

template <int BT, int STAGES, bool AS, bool WS, bool REQ>
__global__ void __launch_bounds__(I8_THREADS, 1)
    i8_ts_kernel(const __grid_constant__ CUtensorMap tmap_a, const uint4 *__restrict__ ts8,
                 const int32_t *__restrict__ colsum, const int32_t *__restrict__ rowsum, const I8Epi e, int M,
                 int N, int K, int nchunks, int32_t *dev_err) {
  using L = I8Layout<BT, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
  uint64_t *empty = full + STAGES;
  uint64_t *accum = empty + STAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::SLOT_OFF);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::FLAG_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int n0 = tile * 128, t0 = blockIdx.y * BT;
  const int nst = (nchunks + I8_KSUB - 1) / I8_KSUB;
  const int krot = (int)(((unsigned)blockIdx.x * 7u) % (unsigned)nst);
  auto stage_of = [&](int st) { return st + krot < nst ? st + krot : st + krot - nst; };
  auto chunks_of = [&](int rt) { return min(I8_KSUB, nchunks - rt * I8_KSUB); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1 + 4);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    mbar_fence_init();
    prefetch_tmap(&tmap_a);
  }
  if (warp == 1) tmem_alloc(tmem_slot, I8_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      pdl_wait();  // the activations may come from the previous kernel
      int issued = 0;
      for (int st = 0; st < nst; st++) {
        const int s = st % STAGES;
        const uint32_t ph = (uint32_t)(st / STAGES) & 1u;
        if (!wait_or_abort(&empty[s], ph ^ 1u, abort_flag, dev_err)) break;
        const int rt = stage_of(st);
        const int cnt = chunks_of(rt);
        mbar_arrive_expect_tx(&full[s], (uint32_t)cnt * L::B_CHUNK);
        for (int c = 0; c < cnt; c++)
          tma_load_2d(smem + s * L::B_STAGE + c * L::B_CHUNK, &tmap_a, (rt * I8_KSUB + c) * 128, t0, &full[s]);
        issued = st + 1;
      }
      if (issued > 0) {
        const int st = issued - 1;
        wait_or_abort(&full[st % STAGES], (uint32_t)(st / STAGES) & 1u, abort_flag, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // A = weights (TMEM), B = activations (shared memory); S32 accumulate.
      constexpr uint32_t idesc = umma_idesc(128, BT, 2u, WS ? 1u : 0u, AS ? 1u : 0u);
      const uint64_t bdesc0 = sw128_kmajor_desc(smem_u32(smem));
      for (int st = 0; st < nst; st++) {
        const int s = st % STAGES;
        const uint32_t ph = (uint32_t)(st / STAGES) & 1u;
        if (!wait_or_abort(&full[s], ph, abort_flag, dev_err)) break;
        tc_fence_after();
        const uint64_t bd = bdesc0 + (uint64_t)(((uint32_t)s * L::B_STAGE) >> 4);
        const uint32_t a_col = tmem + L::A_COL0 + (uint32_t)s * L::A_STAGE_COLS;
        const int cnt = chunks_of(stage_of(st));
        if (cnt == I8_KSUB) {
          umma_i8_ts_stage(tmem, a_col, bd, L::B_CHUNK >> 4, idesc, st != 0 ? 1u : 0u);
        } else {
#pragma unroll
          for (int kk = 0; kk < 4; kk++)
            umma_i8_ts(tmem, a_col + (uint32_t)(kk * 8), bd + (uint64_t)(2 * kk), idesc, (st | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
    }
  } else {
    const int q = warp & 3;
    const int gq = (warp - 2) >> 2;
    const int cl = q * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const uint4 *wcol = ts8 + (size_t)tile * nchunks * 8 * 128 + cl;
    // One stage of raw weights per thread (KSUB chunks x 8 x 16 bytes);
    // chunk c of the group's next stage is requested once chunk c of this
    // one is in TMEM.
    uint4 ring[I8_KSUB][8];
    auto load = [&](int st, int c) {
      int ch = stage_of(st) * I8_KSUB + c;
      if (ch >= nchunks) ch = nchunks - 1;  // K tail: loaded, never used
      const uint4 *src = wcol + (size_t)ch * 8 * 128;
#pragma unroll
      for (int pl = 0; pl < 8; pl++) ring[c][pl] = __ldg(src + pl * 128);
    };
#pragma unroll
    for (int c = 0; c < I8_KSUB; c++)
      if (gq < nst) load(gq, c);
    for (int st = gq; st < nst; st += 2) {
      const int s = st % STAGES;
      const uint32_t ph = (uint32_t)(st / STAGES) & 1u;
      if (!warp_wait_or_abort(&empty[s], ph ^ 1u, abort_flag, dev_err)) break;
      tc_fence_after();
      const int cnt = chunks_of(stage_of(st));
      const bool more = st + 2 < nst;
#pragma unroll
      for (int c = 0; c < I8_KSUB; c++) {
        if (c < cnt) {
          tmem_st32(lane_base + L::A_COL0 + (uint32_t)(s * L::A_STAGE_COLS + c * 32),
                    *reinterpret_cast<const uint32_t(*)[32]>(&ring[c][0]));
          tmem_st_wait();  // the source registers are reloaded next
        }
        if (more) load(st + 2, c);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);
    }
    // Epilogue: group gq covers tokens [gq * BT/2, (gq + 1) * BT/2).
    const bool ok = warp_wait_or_abort(accum, 0u, abort_flag, dev_err);
    tc_fence_after();
    pdl_wait();  // the row sums (and anything Y aliases) come from earlier kernels
    // Per-token terms of the correction, y = raw - az(t) cs(n) - bz(n) u(t)
    // with u(t) = rowsum(t) - K az(t), staged once per CTA in shared memory
    // (read per element from global memory they are reloaded after every
    // store, which may alias them).
    int32_t *tok_az = reinterpret_cast<int32_t *>(smem + L::TOK_OFF);
    int32_t *tok_u = tok_az + BT;
    {
      const int i = threadIdx.x - 64;  // 256 epilogue threads
      for (int r = i; r < BT; r += 256) {
        const int t = t0 + r;
        int32_t az = 0, u = 0;
        if (t < M) {
          az = az_at(e, t);
          const int32_t rs = e.bz_mode != 0 ? __ldg(rowsum + t) : 0;
          u = (int32_t)((uint32_t)rs - (uint32_t)K * (uint32_t)az);
        }
        tok_az[r] = az;
        tok_u[r] = u;
      }
    }
    named_barrier_sync(1, 256);
    int go = ok && !*abort_flag;
    go = __shfl_sync(0xffffffffu, go, 0);
    if (go) {
      const int n = n0 + cl;
      const bool nok = n < N;
      const int32_t cs = nok ? __ldg(colsum + n) : 0;
      const int32_t bz = nok ? bz_at(e, n) : 0;
      constexpr int HALF = BT / 2;
      constexpr int GRP = HALF % 64 == 0 ? 64 : HALF % 48 == 0 ? 48 : HALF % 32 == 0 ? 32 : 16;
      static_assert(HALF % GRP == 0, "epilogue groups must tile the half tile");
#pragma unroll 1
      for (int c0 = gq * HALF; c0 < (gq + 1) * HALF; c0 += GRP) {
        uint32_t v[GRP];
#pragma unroll
        for (int j = 0; j < GRP; j += 16)
          tmem_ld16(lane_base + (uint32_t)(c0 + j), *reinterpret_cast<uint32_t(*)[16]>(&v[j]));
        tmem_ld_wait();
        if (nok) {
          const int lim = M - (t0 + c0);
#pragma unroll
          for (int j = 0; j < GRP; j++) {
            if (j < lim) {
              const uint32_t y = v[j] - (uint32_t)tok_az[c0 + j] * (uint32_t)cs - (uint32_t)bz * (uint32_t)tok_u[c0 + j];
              i8_emit<REQ>(e, (int64_t)(t0 + c0 + j) * N + n, (int32_t)y);
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, I8_TMEM_COLS);
  }
}

// rowsum[m] = sum_k a[m][k] (as signed or unsigned bytes): one warp per row,
// 16-byte loads when rows allow, for the b zero-point correction.
template <bool AS>
__global__ void __launch_bounds__(256) i8_rowsum_kernel(const uint8_t *__restrict__ A, int32_t *__restrict__ rowsum,
                                                        int M, int K) {
  pdl_launch_dependents();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m = blockIdx.x * 8 + warp;
  if (m >= M) return;
  const uint8_t *row = A + (size_t)m * K;
  int acc = 0;
  if ((K & 15) == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0) {
    for (int k = lane * 16; k < K; k += 512) {
      const uint4 v = __ldg(reinterpret_cast<const uint4 *>(row + k));
      acc = dp4_ones<AS>(v.x, acc);
      acc = dp4_ones<AS>(v.y, acc);
      acc = dp4_ones<AS>(v.z, acc);
      acc = dp4_ones<AS>(v.w, acc);
    }
  } else {
    for (int k = lane; k < K; k += 32) acc += AS ? (int)(int8_t)row[k] : (int)row[k];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) rowsum[m] = acc;
}

// GEMV / small-M: one CTA = 32 weight columns (a quarter of a ts8 tile) x
// all of K; warp w takes 128-k chunks w, w+8, ...; lane = column. The M <= 16
// activation rows sit in shared memory (read as broadcast words).
constexpr int GV_THREADS = 256;

// MM: the largest row count this instantiation serves (1 for single-row
// decode, I8_GEMV_MAX_M otherwise), so the per-row loops unroll exactly.
template <bool AS, bool WS, bool REQ, int MM>
__global__ void __launch_bounds__(GV_THREADS)
    i8_gemv_kernel(const uint4 *__restrict__ ts8, const int32_t *__restrict__ colsum, const uint8_t *__restrict__ A,
                   const I8Epi e, int M, int N, int K, int K128, int nchunks, const PrefetchPlan pf) {
  extern __shared__ uint8_t gsm[];
  uint32_t *a_s = reinterpret_cast<uint32_t *>(gsm);                   // [M][K128/4]
  int *part = reinterpret_cast<int *>(gsm + (size_t)M * K128);         // [8 warps][M][32]
  int *rows = part + 8 * M * 32;                                      // [M]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x >> 2, qc = blockIdx.x & 3;
  // The declared next call's weights go to L2 first.
  if (threadIdx.x == 0 && pf.seg[0]) prefetch_share(pf, blockIdx.x);
  // Weight loads do not depend on earlier kernels: issue the first chunk now.
  const uint4 *wcol = ts8 + (size_t)tile * nchunks * 8 * 128 + qc * 32 + lane;
  uint4 wr[8];
  if (warp < nchunks) {
#pragma unroll
    for (int pl = 0; pl < 8; pl++) wr[pl] = __ldg(wcol + (size_t)warp * 8 * 128 + pl * 128);
  }
  // Trigger the next kernel once this warp's weights have arrived (as the int4
  // decode GEMV does; triggering at entry lets later grids crowd the SMs).
  asm volatile("" ::"r"(wr[0].x), "r"(wr[7].w));
  pdl_launch_dependents();
  pdl_wait();
  const int kw = K128 >> 2;
  for (int i = threadIdx.x; i < M * kw; i += GV_THREADS) {
    const int m = i / kw, k = (i % kw) * 4;
    uint32_t v = 0;
    const uint8_t *row = A + (size_t)m * K;
    if ((K & 3) == 0 && k + 4 <= K) {
      v = __ldg(reinterpret_cast<const uint32_t *>(row + k));
    } else {
#pragma unroll
      for (int b = 0; b < 4; b++)
        if (k + b < K) v |= (uint32_t)row[k + b] << (8 * b);
    }
    a_s[i] = v;
  }
  __syncthreads();
  if (e.bz_mode != 0) {
    for (int m = warp; m < M; m += 8) {
      int acc = 0;
      for (int w = lane; w < kw; w += 32) acc = dp4_ones<AS>(a_s[m * kw + w], acc);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) rows[m] = acc;
    }
  }
  int acc[MM];
#pragma unroll
  for (int m = 0; m < MM; m++) acc[m] = 0;
  for (int ch = warp; ch < nchunks; ch += 8) {
    uint4 nx[8];
    const bool more = ch + 8 < nchunks;
    if (more) {
#pragma unroll
      for (int pl = 0; pl < 8; pl++) nx[pl] = __ldg(wcol + (size_t)(ch + 8) * 8 * 128 + pl * 128);
    }
    const uint32_t *wv = reinterpret_cast<const uint32_t *>(wr);
#pragma unroll
    for (int m = 0; m < MM; m++) {
      if (m < M) {
        const uint32_t *ar = a_s + m * kw + ch * 32;
#pragma unroll
        for (int j = 0; j < 32; j++) acc[m] = dp4<AS, WS>(ar[j], wv[j], acc[m]);
      }
    }
    if (more) {
#pragma unroll
      for (int pl = 0; pl < 8; pl++) wr[pl] = nx[pl];
    }
  }
#pragma unroll
  for (int m = 0; m < MM; m++)
    if (m < M) part[(warp * M + m) * 32 + lane] = acc[m];
  __syncthreads();
  for (int i = threadIdx.x; i < M * 32; i += GV_THREADS) {
    const int m = i >> 5, c = i & 31;
    int raw = 0;
#pragma unroll
    for (int w = 0; w < 8; w++) raw += part[(w * M + m) * 32 + c];
    const int n = tile * 128 + qc * 32 + c;
    if (n < N) {
      const int32_t az = az_at(e, m), bz = bz_at(e, n), rs = e.bz_mode != 0 ? rows[m] : 0;
      const uint32_t y = (uint32_t)raw - (uint32_t)az * (uint32_t)__ldg(colsum + n) - (uint32_t)bz * (uint32_t)rs +
                         (uint32_t)K * (uint32_t)az * (uint32_t)bz;
      i8_emit<REQ>(e, (int64_t)m * N + n, (int32_t)y);
    }
  }
}

int i8_pick_bt(int64_t M, int64_t N, int sms) {
  if (M <= 64) return 64;  // up to 64 rows: the smallest tile that covers them
  static const int cand[] = {256, 192, 128, 96};
  const int64_t ntile = (N + 127) / 128;
  int best = 128;
  int64_t best_cost = -1;
  for (int bt : cand) {
    const int64_t ctas = ntile * ((M + bt - 1) / bt);
    const int64_t waves = (ctas + sms - 1) / sms;
    const int64_t cost = waves * (2 * std::max(bt, 128) + bt + 64);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = bt;
    }
  }
  return best;
}

template <int BT, int STAGES, bool AS, bool WS, bool REQ>
void launch_ts(const I8GemmArgs &a, const I8Weight &w, const I8Epi &e, cudaStream_t s) {
  using L = I8Layout<BT, STAGES>;
  CUtensorMap tm;
  const cuuint64_t dims[2] = {(cuuint64_t)a.K, (cuuint64_t)a.M};
  const cuuint64_t strides[1] = {(cuuint64_t)a.K};
  const cuuint32_t box[2] = {128u, (cuuint32_t)BT};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(a.A), dims, strides,
                                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  B2M_REQUIRE(r == CUDA_SUCCESS, B2M_ERR_CUDA, "cuTensorMapEncodeTiled failed for the int8 activations");
  auto kern = i8_ts_kernel<BT, STAGES, AS, WS, REQ>;
  set_smem_limit_once<i8_ts_kernel<BT, STAGES, AS, WS, REQ>>((int)L::BYTES);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(w.npad / 128), (unsigned)((a.M + BT - 1) / BT));
  cfg.blockDim = dim3(I8_THREADS);
  cfg.dynamicSmemBytes = L::BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2M_CUDA(cudaLaunchKernelEx(&cfg, kern, tm, reinterpret_cast<const uint4 *>(w.ts8), (const int32_t *)w.colsum,
                              (const int32_t *)a.rowsum, e, (int)a.M, (int)a.N, (int)a.K, (int)(w.k128 / 128),
                              a.dev_err));
}

template <bool AS, bool WS, bool REQ>
void launch_ts_bt(const I8GemmArgs &a, const I8Weight &w, const I8Epi &e, cudaStream_t s) {
  if (e.bz_mode != 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((a.M + 7) / 8));
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    B2M_CUDA(cudaLaunchKernelEx(&cfg, i8_rowsum_kernel<AS>, reinterpret_cast<const uint8_t *>(a.A), a.rowsum,
                                (int)a.M, (int)a.K));
  }
  const int sms = device_sm_count();
  switch (i8_pick_bt(a.M, a.N, sms)) {
    case 256: launch_ts<256, 3, AS, WS, REQ>(a, w, e, s); break;
    case 192: launch_ts<192, 4, AS, WS, REQ>(a, w, e, s); break;
    case 128: launch_ts<128, 6, AS, WS, REQ>(a, w, e, s); break;
    case 64: launch_ts<64, 6, AS, WS, REQ>(a, w, e, s); break;
    default: launch_ts<96, 6, AS, WS, REQ>(a, w, e, s); break;
  }
}

template <bool AS, bool WS, bool REQ, int MM>
void launch_gemv_m(const I8GemmArgs &a, const I8Weight &w, const I8Epi &e, cudaStream_t s) {
  const size_t smem = (size_t)a.M * w.k128 + (size_t)8 * a.M * 32 * 4 + (size_t)a.M * 4;
  auto kern = i8_gemv_kernel<AS, WS, REQ, MM>;
  set_smem_limit_once<i8_gemv_kernel<AS, WS, REQ, MM>>(232448);
  PrefetchPlan pf = a.pf;
  pf.set_grid(w.npad / 128 * 4);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(w.npad / 128 * 4));
  cfg.blockDim = dim3(GV_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2M_CUDA(cudaLaunchKernelEx(&cfg, kern, reinterpret_cast<const uint4 *>(w.ts8), (const int32_t *)w.colsum,
                              reinterpret_cast<const uint8_t *>(a.A), e, (int)a.M, (int)a.N, (int)a.K, (int)w.k128,
                              (int)(w.k128 / 128), pf));
}

template <bool AS, bool WS, bool REQ>
void launch_gemv(const I8GemmArgs &a, const I8Weight &w, const I8Epi &e, cudaStream_t s) {
  if (a.M == 1)
    launch_gemv_m<AS, WS, REQ, 1>(a, w, e, s);
  else
    launch_gemv_m<AS, WS, REQ, I8_GEMV_MAX_M>(a, w, e, s);
}

template <bool REQ>
void dispatch_signs(const I8GemmArgs &a, const I8Weight &w, const I8Epi &e, bool gemv, cudaStream_t s) {
  const bool as = a.a_signed != 0, ws = a.b_signed != 0;
  if (gemv) {
    if (as && ws) launch_gemv<true, true, REQ>(a, w, e, s);
    else if (as) launch_gemv<true, false, REQ>(a, w, e, s);
    else if (ws) launch_gemv<false, true, REQ>(a, w, e, s);
    else launch_gemv<false, false, REQ>(a, w, e, s);
  } else {
    if (as && ws) launch_ts_bt<true, true, REQ>(a, w, e, s);
    else if (as) launch_ts_bt<true, false, REQ>(a, w, e, s);
    else if (ws) launch_ts_bt<false, true, REQ>(a, w, e, s);
    else launch_ts_bt<false, false, REQ>(a, w, e, s);
  }
}

}  // namespace

bool launch_i8_tc(const I8GemmArgs &a, const I8Weight &w, cudaStream_t s) {
  if (!w.ts8 || a.batch != 1 || a.M <= 0 || a.N <= 0 || a.K <= 0) return false;
  if (a.M > (int64_t)65535 * 96 || a.K > (int64_t)1 << 30) return false;
  const bool gemv = a.M <= I8_GEMV_MAX_M;
  if (gemv && (size_t)a.M * w.k128 > (size_t)160 * 1024) return false;  // activations must fit shared memory
  if (!gemv && (a.K % 16) != 0) return false;  // TMA row pitch must be a multiple of 16 bytes
  if (!gemv && (reinterpret_cast<uintptr_t>(a.A) & 15) != 0) return false;
  I8Epi e;
  e.azp = a.azp;
  e.az_mode = !a.azp ? 0 : a.azp_len == 1 ? 1 : (a.azp_len == a.M && a.M != 1) ? 2 : 0;
  e.az_signed = a.azp_signed;
  e.bzp = a.bzp;
  e.bz_mode = !a.bzp ? 0 : a.bzp_len == 1 ? 1 : (a.bzp_len == a.N && a.N != 1) ? 2 : 0;
  e.bz_signed = a.bzp_signed;
  e.Y32 = a.Y32;
  e.Yq = a.Yq;
  e.mult = a.mult;
  e.y_zp = a.y_zp;
  e.lo = a.lo;
  e.hi = a.hi;
  if (a.requant) dispatch_signs<true>(a, w, e, gemv, s);
  else dispatch_signs<false>(a, w, e, gemv, s);
  return true;
}
