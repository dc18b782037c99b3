// MatMulNBits prefill GEMM on the 5th-generation tensor cores (tcgen05 + TMEM),
// reference: opMatMulNBits m > 1 path, lib/src/onnx_qlinear_ops.dart:208-226.
//
//   Y[M, N] = A[M, K] . dequant(W)[N, K]^T + bias,   f16 operands, fp32 accumulate
//
// One CTA computes a 128 x BN tile of Y with the accumulator in TMEM:
//   warp 0      TMA producer: A (pre-converted to f16) tiles of 128 x 64 into
//               128-byte-swizzled shared memory, one mbarrier per stage.
//   warp 1      allocates TMEM, issues tcgen05.mma.kind::f16 (one thread),
//               commits each stage back to the producers.
//   warps 2-9   dequantize the int4 weights of the stage (fragment-major
//               packed layout, one coalesced 16-byte load per lane per
//               16x64 record, plus a 16-byte f16 scale entry) to f16 (q - zp
//               exact, times the block scale) and store them straight into
//               the swizzled K-major B tile; a register ring prefetches the
//               next four stages' records.
//   warps 2-5   after the main loop: read TMEM (tcgen05.ld), add bias, store.
// Every mbarrier wait is bounded; a timeout sets the context's device error
// word and the CTA exits after releasing its TMEM.
#include <cuda.h>

#include <algorithm>
#include <climits>
#include <type_traits>

#include "b2m_internal.cuh"
#include "ptx.cuh"
#include "tc_common.cuh"

namespace {

using namespace b2m;

constexpr int TC_BM = 128;
constexpr int TC_BK = 64;           // one 128-byte swizzle row of f16

// Shared-memory layout of one CTA: STAGES stages of KS 64-k chunks each, A
// (activation, 128 rows) and B (weight, BN rows) sub-tiles per chunk, all in
// the 128-byte swizzle, then the mbarriers.
template <int BN, int STAGES, int KS>
struct TcLayout {
  static constexpr uint32_t A_CHUNK = TC_BM * TC_BK * 2;  // 16 KB
  static constexpr uint32_t B_CHUNK = BN * TC_BK * 2;
  static constexpr uint32_t A_STAGE = KS * A_CHUNK;
  static constexpr uint32_t B_STAGE = KS * B_CHUNK;
  static constexpr uint32_t A_OFF = 0;
  static constexpr uint32_t B_OFF = A_OFF + STAGES * A_STAGE;
  static constexpr uint32_t BAR_OFF = B_OFF + STAGES * B_STAGE;
  static constexpr uint32_t BARS = 2 * STAGES + 1;
  static constexpr uint32_t SLOT_OFF = BAR_OFF + BARS * 8;
  static constexpr uint32_t FLAG_OFF = SLOT_OFF + 8;
  static constexpr uint32_t BYTES = FLAG_OFF + 8 + 1024;  // + alignment slack
  static constexpr uint32_t TMEM_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
};

// Byte offset of (row, k) inside a 128-byte-swizzled K-major tile of f16.
__device__ __forceinline__ uint32_t sw128_off(int row, int k) {
  return (uint32_t)(row * 128 + ((((k >> 3) ^ (row & 7))) << 4) + ((k & 7) << 1));
}

// One 16-column x 64-k record of packed weights with its scales / zero
// points, as loaded by one lane (fragment-major layout, see k_nbits.cu):
// v = words (group 0, col g), (group 0, col g+8), (group 1, col g),
// (group 1, col g+8); s/z indexed [group][block half][col g / g+8].
template <bool BS16>
struct Rec {
  static constexpr int SPS = BS16 ? 2 : 1;
  uint4 v;
  float s[2][SPS][2];
  float z[2][SPS][2];
};

template <int ZPK, bool BS16>
__device__ __forceinline__ Rec<BS16> load_rec(const NbitsWeight &w, int tile16, int chunk, int lane, int nchunks,
                                              int groups, int nb) {
  Rec<BS16> r;
  const int g = lane >> 2;
  const bool have = tile16 < (int)(w.npad >> 4);
  r.v = make_uint4(0u, 0u, 0u, 0u);
  if (have) r.v = __ldg(reinterpret_cast<const uint4 *>(w.bq + (((size_t)tile16 * nchunks + chunk) * 32 + lane) * 16));
#pragma unroll
  for (int grp = 0; grp < 2; grp++) {
    const int G = 2 * chunk + grp;
#pragma unroll
    for (int hf = 0; hf < Rec<BS16>::SPS; hf++) {
      int blk = BS16 ? (2 * G + hf) : (G * 32) / w.block;
      const bool valid = have && G < groups && blk < nb;
      if (!valid) blk = 0;
#pragma unroll
      for (int hi = 0; hi < 2; hi++) {
        const int col = tile16 * 16 + g + 8 * hi;
        float s = 0.f, z = 8.f;
        if (valid) {
          s = __ldg(w.scales + (size_t)col * nb + blk);
          if (ZPK == 1) {
            const uint8_t zb = __ldg(w.zp_u8 + (size_t)col * w.zstride + (blk >> 1));
            z = (float)((blk & 1) ? (zb >> 4) : (zb & 15));
          } else if (ZPK == 2) {
            z = __ldg(w.zp_f32 + (size_t)col * nb + blk);
          }
        }
        r.s[grp][hf][hi] = s;
        r.z[grp][hf][hi] = z;
      }
    }
  }
  return r;
}

// Dequantize a record into the B stage (rows row0 .. row0+15), natural k
// order: the product (q - zp) * scale is formed in fp32 and rounded once.
template <bool BS16, bool UNUSED>
__device__ __forceinline__ void store_rec(const Rec<BS16> &r, uint8_t *b_stage, int row0, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int grp = 0; grp < 2; grp++) {
#pragma unroll
    for (int hf = 0; hf < 2; hf++) {
      const int sb = BS16 ? hf : 0;
      const int kloc = grp * 32 + hf * 16 + 4 * t;
#pragma unroll
      for (int hi = 0; hi < 2; hi++) {
        const uint32_t x = grp ? (hi ? r.v.w : r.v.z) : (hi ? r.v.y : r.v.x);
        const float s = r.s[grp][sb][hi], z = r.z[grp][sb][hi];
        const uint32_t bytes = x >> (16 * hf);
        const float q0 = (float)(bytes & 15), q1 = (float)((bytes >> 4) & 15);
        const float q2 = (float)((bytes >> 8) & 15), q3 = (float)((bytes >> 12) & 15);
        const uint32_t lo2 = h2_as_u32(__floats2half2_rn((q0 - z) * s, (q1 - z) * s));
        const uint32_t hi2 = h2_as_u32(__floats2half2_rn((q2 - z) * s, (q3 - z) * s));
        const int row = row0 + g + 8 * hi;
        *reinterpret_cast<uint2 *>(b_stage + sw128_off(row, kloc)) = make_uint2(lo2, hi2);
      }
    }
  }
}

// Prefill-friendly record (block >= 32, integer zero points, f16-safe
// scales): the nibbles plus one 16-byte scale entry per MMA row group g,
// eight halves (s, 1024 + zp) for columns g / g+8 of both 32-k groups.
struct RecS {
  uint4 v;
  uint4 e;
};

__device__ __forceinline__ RecS load_recs(const NbitsWeight &w, int tile16, int chunk, int lane, int nchunks) {
  RecS r;
  r.v = make_uint4(0u, 0u, 0u, 0u);
  r.e = make_uint4(0u, 0u, 0u, 0u);
  if (tile16 < (int)(w.npad >> 4)) {
    const size_t rec = (size_t)tile16 * nchunks + chunk;
    r.v = __ldg(reinterpret_cast<const uint4 *>(w.bq + (rec * 32 + lane) * 16));
    r.e = __ldg(reinterpret_cast<const uint4 *>(w.srec + (rec * 8 + (lane >> 2)) * 16));
  }
  return r;
}

// Dequantize into the B stage with k permuted inside every aligned group of
// four as (k0, k2, k1, k3); the activation operand is stored with the same
// permutation, so the MMA's sum over k is unchanged.
__device__ __forceinline__ void store_recs(const RecS &r, uint8_t *b_stage, int row0, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int grp = 0; grp < 2; grp++) {
#pragma unroll
    for (int hi = 0; hi < 2; hi++) {
      const uint32_t sz = grp ? (hi ? r.e.w : r.e.z) : (hi ? r.e.y : r.e.x);  // half2(s, 1024 + zp)
      const __half2 ss = u32_as_h2(prmt(sz, sz, 0x1010u));
      const __half2 zz = u32_as_h2(prmt(sz, sz, 0x3232u));
      const uint32_t x = grp ? (hi ? r.v.w : r.v.z) : (hi ? r.v.y : r.v.x);
      const int row = row0 + g + 8 * hi;
#pragma unroll
      for (int hf = 0; hf < 2; hf++) {
        const uint32_t d = prmt(x, 0u, hf ? 0x4342u : 0x4140u);
        const uint32_t e = (d & 0x000F000Fu) | 0x64006400u;         // 1024 + q(k0), 1024 + q(k2)
        const uint32_t o = ((d >> 4) & 0x000F000Fu) | 0x64006400u;  // 1024 + q(k1), 1024 + q(k3)
        const uint32_t we = h2_as_u32(__hmul2(__hsub2(u32_as_h2(e), zz), ss));
        const uint32_t wo = h2_as_u32(__hmul2(__hsub2(u32_as_h2(o), zz), ss));
        *reinterpret_cast<uint2 *>(b_stage + sw128_off(row, grp * 32 + hf * 16 + 4 * t)) = make_uint2(we, wo);
      }
    }
  }
}

template <int BN, int STAGES, int KS, int ZPK, bool BS16, bool SREC, int DQG, int PF>
__global__ void __launch_bounds__((2 + DQG * (BN / 16)) * 32, 1)
    nbits_tc_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_y,
                    const NbitsWeight w, const float *bias, float *Y, int M, int N, int use_tma_store,
                    int32_t *dev_err) {
  using L = TcLayout<BN, STAGES, KS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  // One "full" barrier per stage completes when the activation TMA bytes have
  // landed AND every dequant thread of the stage has arrived, so the MMA
  // thread waits once per stage: each mbarrier wait stalls that thread for
  // ~150 cycles in which it issues no MMA.
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
  uint64_t *empty = full + STAGES;
  uint64_t *accum = empty + STAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::SLOT_OFF);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::FLAG_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * TC_BM;
  const int nchunks = (int)(w.kp / TC_BK);
  const int nst = (nchunks + KS - 1) / KS;
  const int nb = (int)w.nblocks;
  const int groups = (int)((w.nblocks * w.block + 31) >> 5);
  // CTAs sharing an M tile would otherwise request the same activation k-tile
  // at the same moment; each column tile walks K from its own starting stage
  // (the accumulation order is still fixed per output element, so results
  // stay deterministic).
  const int krot = (int)(((unsigned)blockIdx.x * 7u) % (unsigned)nst);
  auto stage_of = [&](int st) { return st + krot < nst ? st + krot : st + krot - nst; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1 + (BN / 16) * 32);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    mbar_fence_init();
    prefetch_tmap(&tmap_a);
  }
  if (warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // The activation operand is written by the previous kernel (the f16
      // conversion); everything before this point — TMEM, barriers, and the
      // weight prefetch / dequant of the producer warps — overlaps it under
      // programmatic dependent launch.
      pdl_wait();
      int issued = 0;
      for (int st = 0; st < nst; st++) {
        const int s = st % STAGES;
        const uint32_t ph = (uint32_t)(st / STAGES) & 1u;
        if (!wait_or_abort(&empty[s], ph ^ 1u, abort_flag, dev_err)) break;
        const int rt = stage_of(st);
        const int cnt = (rt * KS + KS <= nchunks) ? KS : nchunks - rt * KS;
        mbar_arrive_expect_tx(&full[s], (uint32_t)cnt * L::A_CHUNK);
        for (int c = 0; c < cnt; c++)
          tma_load_2d(smem + L::A_OFF + s * L::A_STAGE + c * L::A_CHUNK, &tmap_a, (rt * KS + c) * TC_BK, m0,
                      &full[s]);
        issued = st + 1;
      }
      // Never leave a copy in flight into shared memory we are about to free.
      if (issued > 0) {
        const int st = issued - 1;
        wait_or_abort(&full[st % STAGES], (uint32_t)(st / STAGES) & 1u, abort_flag, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(TC_BM, BN, 1u, 0u, 0u);  // F32 <- F16 x F16
      for (int st = 0; st < nst; st++) {
        const int s = st % STAGES;
        const uint32_t ph = (uint32_t)(st / STAGES) & 1u;
        if (!wait_or_abort(&full[s], ph, abort_flag, dev_err)) break;
        tc_fence_after();
        const int rt = stage_of(st);
        const int cnt = (rt * KS + KS <= nchunks) ? KS : nchunks - rt * KS;
        const uint32_t a_base = smem_u32(smem + L::A_OFF + s * L::A_STAGE);
        const uint32_t b_base = smem_u32(smem + L::B_OFF + s * L::B_STAGE);
#pragma unroll
        for (int c = 0; c < KS; c++) {
          if (c < cnt) {
#pragma unroll
            for (int kk = 0; kk < TC_BK / 16; kk++)
              umma_f16(tmem, sw128_kmajor_desc(a_base + c * L::A_CHUNK + kk * 32),
                       sw128_kmajor_desc(b_base + c * L::B_CHUNK + kk * 32), idesc, (st | c | kk) != 0 ? 1u : 0u);
          }
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
    }
  } else {
    // Dequant producers: DQG groups of BN/16 warps; group gq handles the
    // stages gq, gq + DQG, ... and warp `rec` of a group owns record `rec`
    // (16 columns x 64 k) of each chunk of its stages. Every warp keeps the
    // raw records of its next PF stages in registers, so global-load latency
    // overlaps the dequantization of earlier stages.
    using RecT = typename std::conditional<SREC, RecS, Rec<BS16>>::type;
    const int dw = warp - 2;
    const int rec = dw % (BN / 16), gq = dw / (BN / 16);
    auto load = [&](int st, int c) -> RecT {
      const int ch = stage_of(st) * KS + c;
      if constexpr (SREC) return load_recs(w, n0 / 16 + rec, ch < nchunks ? ch : 0, lane, nchunks);
      else return load_rec<ZPK, BS16>(w, n0 / 16 + rec, ch < nchunks ? ch : 0, lane, nchunks, groups, nb);
    };
    RecT ring[PF][KS];
#pragma unroll
    for (int j = 0; j < PF; j++)
#pragma unroll
      for (int c = 0; c < KS; c++)
        if (gq + j * DQG < nst) ring[j][c] = load(gq + j * DQG, c);
    bool alive = true;
    for (int i0 = 0; gq + i0 * DQG < nst && alive; i0 += PF) {
#pragma unroll
      for (int j = 0; j < PF; j++) {
        const int st = gq + (i0 + j) * DQG;
        if (st < nst && alive) {
          const int s = st % STAGES;
          const uint32_t ph = (uint32_t)(st / STAGES) & 1u;
          RecT nxt[KS];
          const int sn = st + PF * DQG;
#pragma unroll
          for (int c = 0; c < KS; c++)
            if (sn < nst) nxt[c] = load(sn, c);
          if (!wait_or_abort(&empty[s], ph ^ 1u, abort_flag, dev_err)) {
            alive = false;
          } else {
            const int rt = stage_of(st);
            const int cnt = (rt * KS + KS <= nchunks) ? KS : nchunks - rt * KS;
            uint8_t *b_stage = smem + L::B_OFF + s * L::B_STAGE;
#pragma unroll
            for (int c = 0; c < KS; c++) {
              if (c < cnt) {
                if constexpr (SREC) store_recs(ring[j][c], b_stage + c * L::B_CHUNK, rec * 16, lane);
                else store_rec<BS16, false>(ring[j][c], b_stage + c * L::B_CHUNK, rec * 16, lane);
              }
            }
            fence_proxy_async_smem();
            mbar_arrive(&full[s]);
#pragma unroll
            for (int c = 0; c < KS; c++) ring[j][c] = nxt[c];
          }
        }
      }
    }
    // Epilogue: warps 2..5 cover TMEM lane quarters 2, 3, 0, 1.
    if (warp < 6) {
      const int q = warp & 3;
      const bool ok = wait_or_abort(accum, 0u, abort_flag, dev_err);
      tc_fence_after();
      pdl_wait();  // earlier kernels of the stream are complete before Y is written
      const bool go = ok && !*abort_flag;
      if (use_tma_store) {
        if (go) {
          // Stage 128 x 32 fp32 boxes in shared memory (the pipeline buffers
          // are free once the accumulator is complete) in the 128-byte
          // swizzle — conflict-free for one row per lane — and write each box
          // with one TMA store; rows / columns past M, N are clipped.
          uint8_t *stage_base = smem + L::A_OFF;
#pragma unroll 1
          for (int cb = 0; cb < BN / 32; cb++) {
            uint8_t *box = stage_base + cb * (TC_BM * 128);
            const int r = q * 32 + lane;
#pragma unroll
            for (int h = 0; h < 2; h++) {
              uint32_t v[16];
              tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(cb * 32 + h * 16), v);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 16; j += 4) {
                float4 o = make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                                       __uint_as_float(v[j + 3]));
                const int col = n0 + cb * 32 + h * 16 + j;
                if (bias) {
                  o.x += col + 0 < N ? __ldg(bias + col + 0) : 0.f;
                  o.y += col + 1 < N ? __ldg(bias + col + 1) : 0.f;
                  o.z += col + 2 < N ? __ldg(bias + col + 2) : 0.f;
                  o.w += col + 3 < N ? __ldg(bias + col + 3) : 0.f;
                }
                const int chunk = (h * 16 + j) >> 2;  // 16-byte chunk of the 128-byte row
                *reinterpret_cast<float4 *>(box + r * 128 + ((chunk ^ (r & 7)) << 4)) = o;
              }
            }
          }
        }
        // All four epilogue warps reach this barrier whatever their state.
        fence_proxy_async_smem();
        named_barrier_sync(1, 128);
        if (go && warp == 2 && lane == 0) {
          uint8_t *stage_base = smem + L::A_OFF;
          for (int cb = 0; cb < BN / 32; cb++)
            if (n0 + cb * 32 < N) tma_store_2d(&tmap_y, stage_base + cb * (TC_BM * 128), n0 + cb * 32, m0);
          bulk_commit_group();
          bulk_wait_group0();
        }
      } else if (go) {
        const int row = m0 + q * 32 + lane;
        {
          const bool vec_store = (N & 3) == 0 && ((reinterpret_cast<uintptr_t>(Y) & 15) == 0) &&
                                 (bias == nullptr || (reinterpret_cast<uintptr_t>(bias) & 15) == 0);
#pragma unroll 1
          for (int c = 0; c < BN / 16; c++) {
            uint32_t r[16];
            tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 16), r);
            tmem_ld_wait();
            if (row < M) {
              float *yrow = Y + (size_t)row * N;
              const int cb = n0 + c * 16;
              if (vec_store && cb + 16 <= N) {
#pragma unroll
                for (int j = 0; j < 16; j += 4) {
                  float4 o = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                         __uint_as_float(r[j + 3]));
                  if (bias) {
                    const float4 b = __ldg(reinterpret_cast<const float4 *>(bias + cb + j));
                    o.x += b.x;
                    o.y += b.y;
                    o.z += b.z;
                    o.w += b.w;
                  }
                  *reinterpret_cast<float4 *>(yrow + cb + j) = o;
                }
              } else {
#pragma unroll
                for (int j = 0; j < 16; j++) {
                  const int col = cb + j;
                  if (col < N) yrow[col] = __uint_as_float(r[j]) + (bias ? __ldg(bias + col) : 0.f);
                }
              }
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
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// A[M][K] float32 -> A16[M][K8] f16 (zero padding up to K8, a multiple of 8);
// with `perm`, k is permuted inside each aligned group of four as
// (k0, k2, k1, k3), matching the dequantized weight tiles of store_recs.
__global__ void __launch_bounds__(512) f32_to_f16_rows(const float *A, __half *A16, int64_t M, int64_t K, int64_t K8,
                                                        int perm, int vec) {
  pdl_launch_dependents();  // the GEMM may start its weight-side prologue now
  pdl_wait();               // A (and the scratch we overwrite) are free to use
  const int64_t total = M * K8;
  const bool narrow = total < INT32_MAX;  // 32-bit index division
  for (int64_t idx = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x * 8) {
    int64_t m, k;
    if (narrow) {
      const int q = (int)idx / (int)K8;
      m = q;
      k = (int)idx - q * (int)K8;
    } else {
      m = idx / K8;
      k = idx % K8;
    }
    float f[8];
    const float *row = A + m * K;
    if (vec) {  // rows start 16-byte aligned and K % 4 == 0: two 16-byte loads
      const float4 lo = __ldg(reinterpret_cast<const float4 *>(row + k));
      const float4 hi = k + 4 < K ? __ldg(reinterpret_cast<const float4 *>(row + k + 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
      f[0] = lo.x, f[1] = lo.y, f[2] = lo.z, f[3] = lo.w, f[4] = hi.x, f[5] = hi.y, f[6] = hi.z, f[7] = hi.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++) f[j] = k + j < K ? row[k + j] : 0.f;
    }
    // Two values per conversion (the same round-to-nearest as one at a time).
    __align__(16) __half2 h[4];
    if (perm) {
      h[0] = __floats2half2_rn(f[0], f[2]);
      h[1] = __floats2half2_rn(f[1], f[3]);
      h[2] = __floats2half2_rn(f[4], f[6]);
      h[3] = __floats2half2_rn(f[5], f[7]);
    } else {
#pragma unroll
      for (int j = 0; j < 4; j++) h[j] = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
    }
    *reinterpret_cast<uint4 *>(A16 + idx) = *reinterpret_cast<const uint4 *>(h);
  }
}

template <int BN, int STAGES, int KS, int ZPK, bool BS16, bool SREC, int DQG, int PF>
void launch_tc_t(const CUtensorMap &tm, const CUtensorMap &ty, int use_ty, const NbitsArgs &a, cudaStream_t s) {
  using L = TcLayout<BN, STAGES, KS>;
  auto kern = nbits_tc_kernel<BN, STAGES, KS, ZPK, BS16, SREC, DQG, PF>;
  set_smem_limit_once<nbits_tc_kernel<BN, STAGES, KS, ZPK, BS16, SREC, DQG, PF>>((int)L::BYTES);
  dim3 grid((unsigned)((a.N + BN - 1) / BN), (unsigned)((a.M + TC_BM - 1) / TC_BM));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3((2 + DQG * (BN / 16)) * 32);
  cfg.dynamicSmemBytes = L::BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2M_CUDA(cudaLaunchKernelEx(&cfg, kern, tm, ty, *a.w, a.bias, a.Y, (int)a.M, (int)a.N, use_ty, a.dev_err));
}

template <int BN, int STAGES, int KS, int DQG, int PF>
void launch_tc_bn(const CUtensorMap &tm, const CUtensorMap &ty, int use_ty, const NbitsArgs &a, cudaStream_t s) {
  if (a.w->srec) {
    launch_tc_t<BN, STAGES, KS, 1, false, true, DQG, PF>(tm, ty, use_ty, a, s);
    return;
  }
  // Generic records (fp32 scales, block 16, float zero points) are larger:
  // a one-stage prefetch keeps them in registers.
  const bool bs16 = a.w->block == 16;
  switch (a.w->zp_kind) {
    case 0: bs16 ? launch_tc_t<BN, STAGES, KS, 0, true, false, DQG, 1>(tm, ty, use_ty, a, s) : launch_tc_t<BN, STAGES, KS, 0, false, false, DQG, 1>(tm, ty, use_ty, a, s); break;
    case 1: bs16 ? launch_tc_t<BN, STAGES, KS, 1, true, false, DQG, 1>(tm, ty, use_ty, a, s) : launch_tc_t<BN, STAGES, KS, 1, false, false, DQG, 1>(tm, ty, use_ty, a, s); break;
    default: bs16 ? launch_tc_t<BN, STAGES, KS, 2, true, false, DQG, 1>(tm, ty, use_ty, a, s) : launch_tc_t<BN, STAGES, KS, 2, false, false, DQG, 1>(tm, ty, use_ty, a, s); break;
  }
}

}  // namespace

namespace b2m {

int device_sm_count() {
  static std::atomic<int> cache[64] = {};
  int dev = 0;
  B2M_CUDA(cudaGetDevice(&dev));
  std::atomic<int> &slot = cache[dev & 63];
  int v = slot.load(std::memory_order_relaxed);
  if (v == 0) {
    B2M_CUDA(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev));
    slot.store(v, std::memory_order_relaxed);
  }
  return v;
}

EncodeTiledFn tensor_map_encoder() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    B2M_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    B2M_REQUIRE(p && q == cudaDriverEntryPointSuccess, B2M_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

void launch_f32_to_f16(const float *A, __half *A16, int64_t M, int64_t K, int64_t K8, int perm, cudaStream_t s) {
  // At most one small CTA per SM, so the PDL-launched GEMM's CTAs find room
  // and start their weight prologue while this kernel runs.
  const int64_t total = M * K8 / 8;
  const int sms = device_sm_count();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)std::max<int64_t>(1, std::min<int64_t>(sms, (total + 511) / 512)));
  cfg.blockDim = dim3(512);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int vec = (K % 4) == 0 && (reinterpret_cast<uintptr_t>(A) & 15) == 0;
  B2M_CUDA(cudaLaunchKernelEx(&cfg, f32_to_f16_rows, A, A16, M, K, K8, perm, vec));
}

}  // namespace b2m

int64_t nbits_tc_k8(int64_t K) { return (K + 7) / 8 * 8; }

bool nbits_tc_supported(const NbitsWeight &w, int64_t M, int64_t K, int64_t N) {
  return M >= 1 && M <= (int64_t)65535 * TC_BM && N <= (int64_t)1 << 30 && K <= (int64_t)1 << 30 &&
         w.kp / TC_BK >= 1;
}

void launch_nbits_tc(const NbitsArgs &a, __half *a16, cudaStream_t s) {
  const int64_t K8 = nbits_tc_k8(a.K);
  if (a.w->tsq) {
    launch_f32_to_f16(a.A, a16, a.M, a.K, K8, 0, s);
    launch_nbits_ts(a, a16, K8, s);
    return;
  }
  launch_f32_to_f16(a.A, a16, a.M, a.K, K8, a.w->srec ? 1 : 0, s);
  CUtensorMap tm;
  const cuuint64_t dims[2] = {(cuuint64_t)K8, (cuuint64_t)a.M};
  const cuuint64_t strides[1] = {(cuuint64_t)(K8 * 2)};
  const cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)TC_BM};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a16, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  B2M_REQUIRE(r == CUDA_SUCCESS, B2M_ERR_CUDA, "cuTensorMapEncodeTiled failed for the activation operand");
  // Output tensor map for the TMA-store epilogue (fp32 Y, 32 x 128 boxes,
  // 128-byte swizzle); needs 16-byte aligned rows.
  CUtensorMap ty;
  int use_ty = 0;
  if ((a.N % 4) == 0 && (reinterpret_cast<uintptr_t>(a.Y) & 15) == 0) {
    const cuuint64_t ydims[2] = {(cuuint64_t)a.N, (cuuint64_t)a.M};
    const cuuint64_t ystr[1] = {(cuuint64_t)(a.N * 4)};
    const cuuint32_t ybox[2] = {32, (cuuint32_t)TC_BM};
    CUresult ry = tensor_map_encoder()(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.Y, ydims, ystr, ybox, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    B2M_REQUIRE(ry == CUDA_SUCCESS, B2M_ERR_CUDA, "cuTensorMapEncodeTiled failed for the output");
    use_ty = 1;
  } else {
    ty = tm;  // unused
  }
  launch_tc_bn<128, 3, 2, 2, 2>(tm, ty, use_ty, a, s);
}
