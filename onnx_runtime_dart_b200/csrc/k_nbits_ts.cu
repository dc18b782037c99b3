// MatMulNBits prefill GEMM with the dequantized weights as the TMEM operand,
// reference: opMatMulNBits m > 1 path, lib/src/onnx_qlinear_ops.dart:208-226.
//
//   Y^T[N, M] = dequant(W)[N, K] . A[M, K]^T     (f16 operands, fp32 accumulate)
//
// One CTA owns 128 weight columns x BT tokens. The weight tile is the MMA's A
// operand and lives in tensor memory: dequant warps turn the int4 nibbles into
// f16 in registers and write them with tcgen05.st, so the weights never touch
// shared memory. The activations (converted to f16 by the kernel launched
// before this one) are the B operand, brought into 128-byte-swizzled shared
// memory by TMA. Shared memory then carries only the activation stream (one
// TMA write and one MMA read per byte), half of what a kernel with both
// operands in shared memory moves per MMA cycle.
//
//   warp 0      TMA producer for the activation stages.
//   warp 1      TMEM allocation; one thread issues tcgen05.mma (A from TMEM).
//   warps 2-9   two dequant groups of four warps (one per TMEM lane quarter)
//               taking alternate 128-k stages; each thread owns one weight
//               column. After the main loop they are the epilogue: tcgen05.ld
//               of the accumulator (lane = weight column, column = token), add
//               bias, stage the half tile in shared memory, one TMA store
//               (or, for unaligned outputs, coalesced stores of Y rows).
// SwiGLU epilogue (act / act16 given): the weight's rows are tile-interleaved,
// each 128-column tile holding 64 gate columns and then the 64 matching up
// columns, and the CTA writes act = silu(gate) * up for its 64 columns (fp32
// and / or f16) from the staged tile instead of Y.
// Accumulator in TMEM columns [0, BT); A stages from column A_COL0 on, 64
// columns per 128-k stage (two f16 per 32-bit column, k order).
// Every mbarrier wait is bounded; a timeout sets the context's device error
// word and the CTA exits after releasing its TMEM.
#include <cuda.h>

#include <algorithm>
#include <atomic>

#include "b2m_internal.cuh"
#include "ptx.cuh"
#include "tc_common.cuh"

namespace {

using namespace b2m;

// Thread-block cluster helpers for the split-K reduction through
// distributed shared memory.
__device__ __forceinline__ uint32_t dsmem_map(uint32_t saddr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
  return d;
}
__device__ __forceinline__ float4 dsmem_ld4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

constexpr int TS_THREADS = 320;
constexpr uint32_t TS_TMEM_COLS = 512;

// BT tokens per CTA; a pipeline stage is KSUB chunks of 64 k.
template <int BT, int STAGES, int KSUB>
struct TsLayout {
  static constexpr uint32_t B_CHUNK = (uint32_t)BT * 128;  // 64 k x BT tokens of f16
  static constexpr uint32_t B_STAGE = KSUB * B_CHUNK;
  static constexpr uint32_t BAR_OFF = STAGES * B_STAGE;
  static constexpr uint32_t SLOT_OFF = BAR_OFF + (2 * STAGES + 1) * 8;
  static constexpr uint32_t FLAG_OFF = SLOT_OFF + 8;
  static constexpr uint32_t BYTES = FLAG_OFF + 8 + 1024;  // + alignment slack
  static constexpr uint32_t A_COL0 = (uint32_t)(BT + 31) / 32 * 32;
  static constexpr uint32_t A_STAGE_COLS = KSUB * 32;
  static_assert(BT % 32 == 0 && BT >= 32 && BT <= 256, "token tile: multiple of 32 in [32, 256]");
  static_assert(KSUB == 2 || KSUB == 4, "stage: 128 or 256 k");
  static_assert(A_COL0 + STAGES * A_STAGE_COLS <= TS_TMEM_COLS, "accumulator + weight stages exceed TMEM");
  static_assert(BYTES <= 232448, "shared memory");
  static_assert((uint32_t)BT * 128 * 4 <= STAGES * B_STAGE, "the output tile is staged in the activation stages");
};

// The raw weights of one 64-k chunk for one column: 64 nibbles and the two
// (s, 1024 + zp) pairs of its 32-k groups.
struct TsRec {
  uint4 v0, v1;
  uint2 sz;
};

// Nibble word j holds k 8j .. 8j+7 at bit offsets 0,16,4,20,8,24,12,28, so
// (x >> 4i) & 0x000F000F carries the pair (8j+2i, 8j+2i+1); OR-ing 0x6400
// into each half gives the f16 numbers 1024 + q exactly, 1024 + q - (1024 +
// zp) = q - zp is exact, and the product with the f16 scale rounds once.
__device__ __forceinline__ void ts_dequant(const TsRec &r, uint32_t (&out)[32]) {
  const uint32_t w[8] = {r.v0.x, r.v0.y, r.v0.z, r.v0.w, r.v1.x, r.v1.y, r.v1.z, r.v1.w};
#pragma unroll
  for (int g = 0; g < 2; g++) {
    const uint32_t e = g ? r.sz.y : r.sz.x;
    const __half2 ss = u32_as_h2(prmt(e, e, 0x1010u));
    const __half2 zz = u32_as_h2(prmt(e, e, 0x3232u));
#pragma unroll
    for (int jj = 0; jj < 4; jj++) {
      const uint32_t x = w[g * 4 + jj];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const uint32_t p = ((x >> (4 * i)) & 0x000F000Fu) | 0x64006400u;
        out[(g * 4 + jj) * 4 + i] = h2_as_u32(__hmul2(__hsub2(u32_as_h2(p), zz), ss));
      }
    }
  }
}

// act[i .. i+3] = silu(g) * u (silu_mul_kernel's arithmetic), and / or its
// f16 copy rounded to nearest (i a multiple of 4, 16-byte aligned outputs).
__device__ __forceinline__ void swiglu_store4(float *act, __half *act16, size_t i, float4 g, float4 u) {
  const float4 o = make_float4(silu_times(g.x, u.x), silu_times(g.y, u.y), silu_times(g.z, u.z), silu_times(g.w, u.w));
  if (act) *reinterpret_cast<float4 *>(act + i) = o;
  if (act16) {
    const __half2 a = __floats2half2_rn(o.x, o.y), b = __floats2half2_rn(o.z, o.w);
    uint2 w;
    w.x = h2_as_u32(a);
    w.y = h2_as_u32(b);
    *reinterpret_cast<uint2 *>(act16 + i) = w;
  }
}

template <int BT, int STAGES, int KSUB>
__global__ void __launch_bounds__(TS_THREADS, 1)
    nbits_ts_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_y,
                    int use_tma_y, const uint4 *__restrict__ tsq, const uint2 *__restrict__ tss,
                    const float *__restrict__ bias, float *__restrict__ Y, int M, int N, int nchunks,
                    int32_t *dev_err, const PrefetchPlan pf, float *__restrict__ act, __half *__restrict__ act16) {
  using L = TsLayout<BT, STAGES, KSUB>;
  const bool swiglu = act != nullptr || act16 != nullptr;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  // full[s]: the stage's activation bytes landed (TMA, one arrival + tx) and
  // its weights are in TMEM (one arrival per dequant warp); empty[s]: the MMAs
  // reading the stage completed; accum: the whole accumulator is final.
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + L::BAR_OFF);
  uint64_t *empty = full + STAGES;
  uint64_t *accum = empty + STAGES;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::SLOT_OFF);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::FLAG_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const int n0 = tile * 128, t0 = blockIdx.y * BT;
  // Split-K over a cluster of gridDim.z CTAs: CTA z sums the stages
  // [sbeg, sbeg + nst); the partial tiles are added through distributed
  // shared memory at the end.
  const int nst_all = (nchunks + KSUB - 1) / KSUB;
  const int splits = gridDim.z, zr = blockIdx.z;
  const int sbeg = (int)((int64_t)nst_all * zr / splits);
  const int nst = (int)((int64_t)nst_all * (zr + 1) / splits) - sbeg;
  // The CTAs of one token tile would otherwise request the same activation
  // k-tile at the same moment; each weight tile walks its K range from its own
  // starting stage (the summation order stays fixed per output element).
  const int krot = (int)(((unsigned)blockIdx.x * 7u) % (unsigned)nst);
  auto stage_of = [&](int st) { return sbeg + (st + krot < nst ? st + krot : st + krot - nst); };
  auto chunks_of = [&](int rt) { return min(KSUB, nchunks - rt * KSUB); };

  if (threadIdx.x == 0) {
    // The declared next call's weights go to L2 (this CTA's share).
    if (pf.seg[0]) prefetch_share(pf, blockIdx.x + (int64_t)gridDim.x * (blockIdx.y + (int64_t)gridDim.y * blockIdx.z));
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1 + 4);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    mbar_fence_init();
    prefetch_tmap(&tmap_a);
  }
  if (warp == 1) tmem_alloc(tmem_slot, TS_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Every CTA is resident: the next kernel of the stream may launch and wait
  // for this grid on the SMs' spare room.
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // The activations are written by the conversion kernel launched just
      // before; TMEM, barriers and the first weight stages overlap it.
      pdl_wait();
      int issued = 0;
      for (int st = 0; st < nst; st++) {
        const int s = st % STAGES;
        const uint32_t ph = (uint32_t)(st / STAGES) & 1u;
        if (!wait_or_abort(&empty[s], ph ^ 1u, abort_flag, dev_err)) break;
        const int rt = stage_of(st);
        const int cnt = chunks_of(rt);
        mbar_arrive_expect_tx(&full[s], (uint32_t)cnt * L::B_CHUNK);
        for (int c = 0; c < cnt; c++)
          tma_load_2d(smem + s * L::B_STAGE + c * L::B_CHUNK, &tmap_a, (rt * KSUB + c) * 64, t0, &full[s]);
        issued = st + 1;
      }
      // Never leave a copy in flight into shared memory that is about to be freed.
      if (issued > 0) {
        const int st = issued - 1;
        wait_or_abort(&full[st % STAGES], (uint32_t)(st / STAGES) & 1u, abort_flag, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(128, BT, 1u, 0u, 0u);  // F32 <- F16 x F16, both K-major
      // Descriptors are formed by adding 16-byte offsets to stage 0's (the
      // start-address field cannot overflow below 256 KB of shared memory).
      // Every readiness check in this thread stalls the MMA issue for about
      // one MMA's time, so a stage carries 8 or 16 MMAs per check.
      const uint64_t bdesc0 = sw128_kmajor_desc(smem_u32(smem));
      for (int st = 0; st < nst; st++) {
        const int s = st % STAGES;
        const uint32_t ph = (uint32_t)(st / STAGES) & 1u;
        if (!wait_or_abort(&full[s], ph, abort_flag, dev_err)) break;
        tc_fence_after();
        const uint64_t bd = bdesc0 + (uint64_t)(((uint32_t)s * L::B_STAGE) >> 4);
        const uint32_t a_col = tmem + L::A_COL0 + (uint32_t)s * L::A_STAGE_COLS;
        const int cnt = chunks_of(stage_of(st));
        if (cnt == KSUB) {
#pragma unroll
          for (int h = 0; h < KSUB / 2; h++)
            umma_f16_ts_stage(tmem, a_col + h * 64, bd + h * (2 * L::B_CHUNK >> 4), L::B_CHUNK >> 4, idesc,
                              (st | h) != 0 ? 1u : 0u);
        } else {  // K tail: the last stage holds fewer chunks
          for (int c = 0; c < cnt; c++)
#pragma unroll
            for (int kk = 0; kk < 4; kk++)
              umma_f16_ts(tmem, a_col + (uint32_t)(c * 32 + kk * 8), bd + (uint64_t)(c * (L::B_CHUNK >> 4) + 2 * kk),
                          idesc, (st | c | kk) != 0 ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
    }
  } else {
    const int q = warp & 3;          // TMEM lane quarter this warp may access
    const int gq = (warp - 2) >> 2;  // dequant group: stages gq, gq + 2, ...
    const int cl = q * 32 + lane;    // weight column within the tile
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const uint4 *qcol = tsq + (size_t)tile * nchunks * 256 + cl;
    const uint2 *scol = tss + (size_t)tile * nchunks * 128 + cl;
    auto load = [&](int st, int c) -> TsRec {
      int ch = stage_of(st) * KSUB + c;
      if (ch >= nchunks) ch = nchunks - 1;  // K tail: loaded, never used
      TsRec r;
      r.v0 = __ldg(qcol + (size_t)(2 * ch) * 128);
      r.v1 = __ldg(qcol + (size_t)(2 * ch + 1) * 128);
      r.sz = __ldg(scol + (size_t)ch * 128);
      return r;
    };
    // One stage of raw records per thread; chunk c of the group's next stage
    // is requested as soon as chunk c of this one is dequantized, so every
    // load has about two stages of time to arrive.
    TsRec ring[KSUB];
#pragma unroll
    for (int c = 0; c < KSUB; c++)
      if (gq < nst) ring[c] = load(gq, c);
    for (int st = gq; st < nst; st += 2) {
      const int s = st % STAGES;
      const uint32_t ph = (uint32_t)(st / STAGES) & 1u;
      if (!warp_wait_or_abort(&empty[s], ph ^ 1u, abort_flag, dev_err)) break;
      tc_fence_after();
      const int cnt = chunks_of(stage_of(st));
      const bool more = st + 2 < nst;
#pragma unroll
      for (int c = 0; c < KSUB; c++) {
        if (c < cnt) {
          uint32_t o[32];
          ts_dequant(ring[c], o);
          tmem_st32(lane_base + L::A_COL0 + (uint32_t)(s * L::A_STAGE_COLS + c * 32), o);
        }
        if (more) ring[c] = load(st + 2, c);
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[s]);
    }
    // Epilogue: group gq stores tokens [gq * BT/2, (gq + 1) * BT/2) of the tile.
    const bool ok = warp_wait_or_abort(accum, 0u, abort_flag, dev_err);
    tc_fence_after();
    pdl_wait();  // earlier kernels of the stream are complete before Y is written
    int go = ok && !*abort_flag;
    go = __shfl_sync(0xffffffffu, go, 0);
    if (go) {
      const int col = n0 + cl;
      const bool colok = col < N;
      // With K split, the raw partial tile is staged (no bias) for the
      // cluster reduction below.
      const bool stage = use_tma_y || splits > 1 || swiglu;
      const float b = (bias && colok && splits == 1) ? __ldg(bias + col) : 0.f;
      // All TMEM loads of a group of up to 64 tokens go out before one wait;
      // a wait per 16 columns serializes the load latency.
      constexpr int HALF = BT / 2;
      constexpr int GRP = HALF % 64 == 0 ? 64 : HALF % 48 == 0 ? 48 : HALF % 32 == 0 ? 32 : 16;
      static_assert(HALF % GRP == 0, "epilogue groups must tile the half tile");
      // With an output tensor map the group's half tile goes through shared
      // memory (the activation stages, idle once the accumulator is final:
      // every stage's TMA landed before its MMAs ran) as a row-major
      // [HALF tokens][128 columns] box, written by one TMA store; a lane's
      // direct stores are 4-byte column slices, 48 per token group, and the
      // write burst of a tile took ~2.5 us that way.
      float *stage_out = reinterpret_cast<float *>(smem) + (size_t)gq * HALF * 128;
#pragma unroll 1
      for (int c0 = gq * HALF; c0 < (gq + 1) * HALF; c0 += GRP) {
        uint32_t v[GRP];
#pragma unroll
        for (int j = 0; j < GRP; j += 16)
          tmem_ld16(lane_base + (uint32_t)(c0 + j), *reinterpret_cast<uint32_t(*)[16]>(&v[j]));
        tmem_ld_wait();
        if (stage) {
#pragma unroll
          for (int j = 0; j < GRP; j++) stage_out[(c0 - gq * HALF + j) * 128 + cl] = __uint_as_float(v[j]) + b;
          continue;
        }
        if (colok) {
          float *yc = Y + (size_t)(t0 + c0) * N + col;
          const int lim = M - (t0 + c0);
#pragma unroll
          for (int j = 0; j < GRP; j++)
            if (j < lim) yc[(size_t)j * N] = __uint_as_float(v[j]) + b;
        }
      }
    }
    if (swiglu && splits == 1) {
      // Every epilogue warp takes the group barrier, aborted or not; then the
      // group pairs gate column j with up column 64 + j of its staged rows.
      named_barrier_sync(2 + gq, 128);
      if (go) {
        constexpr int HALF = BT / 2;
        const float *so = reinterpret_cast<const float *>(smem) + (size_t)gq * HALF * 128;
        const int gt = (warp - 2 - 4 * gq) * 32 + lane;
        for (int it = gt; it < HALF * 16; it += 128) {
          const int row = it >> 4, c4 = (it & 15) * 4;
          const int t = t0 + gq * HALF + row;
          if (t >= M) continue;
          const float4 g = *reinterpret_cast<const float4 *>(so + row * 128 + c4);
          const float4 u = *reinterpret_cast<const float4 *>(so + row * 128 + 64 + c4);
          swiglu_store4(act, act16, (size_t)t * (size_t)(N >> 1) + (size_t)tile * 64 + c4, g, u);
        }
      }
    } else if (use_tma_y && splits == 1) {
      // Every epilogue warp takes the group barrier, aborted or not.
      fence_proxy_async_smem();
      named_barrier_sync(2 + gq, 128);
      if (go && warp == 2 + 4 * gq && lane == 0) {
        tma_store_2d(&tmap_y, reinterpret_cast<float *>(smem) + (size_t)gq * (BT / 2) * 128, n0, t0 + gq * (BT / 2));
        bulk_commit_group();
        bulk_wait_group0();
      }
    }
  }
  if (splits > 1) {
    // Every thread of every CTA of the cluster takes both cluster barriers,
    // aborted or not. CTA z adds the staged partial tiles of all ranks, in
    // rank order, for its share of the tile's token rows.
    __syncwarp();
    pdl_wait();  // (returns at once) every thread that writes Y has waited on the prior grid
    cluster_sync_all();
    const int per = (BT + splits - 1) / splits;
    const int rb = zr * per, re = min(BT, rb + per);
    const uint32_t sbase = smem_u32(smem);
    const bool vec = (N & 3) == 0 && (reinterpret_cast<uintptr_t>(Y) & 15) == 0;
    if (!*abort_flag && swiglu) {
      // Gate columns [c4, c4 + 4) and the matching up columns 64 + c4 ..,
      // each summed over the ranks in rank order (the plain path's order).
      for (int it = threadIdx.x; it < (re - rb) * 16; it += TS_THREADS) {
        const int row = rb + (it >> 4), c4 = (it & 15) * 4;
        const int t = t0 + row;
        if (t >= M) continue;
        const uint32_t og = (uint32_t)(row * 128 + c4) * 4u, ou = og + 64u * 4u;
        float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = g;
        for (int rk = 0; rk < splits; rk++) {
          const float4 p = dsmem_ld4(dsmem_map(sbase + og, (uint32_t)rk));
          g.x += p.x, g.y += p.y, g.z += p.z, g.w += p.w;
          const float4 q4 = dsmem_ld4(dsmem_map(sbase + ou, (uint32_t)rk));
          u.x += q4.x, u.y += q4.y, u.z += q4.z, u.w += q4.w;
        }
        if (bias) {
          const int cg = n0 + c4, cu = n0 + 64 + c4;
          g.x = g.x + __ldg(bias + cg), g.y = g.y + __ldg(bias + cg + 1);
          g.z = g.z + __ldg(bias + cg + 2), g.w = g.w + __ldg(bias + cg + 3);
          u.x = u.x + __ldg(bias + cu), u.y = u.y + __ldg(bias + cu + 1);
          u.z = u.z + __ldg(bias + cu + 2), u.w = u.w + __ldg(bias + cu + 3);
        } else {
          g.x = g.x + 0.f, g.y = g.y + 0.f, g.z = g.z + 0.f, g.w = g.w + 0.f;
          u.x = u.x + 0.f, u.y = u.y + 0.f, u.z = u.z + 0.f, u.w = u.w + 0.f;
        }
        swiglu_store4(act, act16, (size_t)t * (size_t)(N >> 1) + (size_t)tile * 64 + c4, g, u);
      }
    } else if (!*abort_flag) {
      for (int it = threadIdx.x; it < (re - rb) * 32; it += TS_THREADS) {
        const int row = rb + (it >> 5), c4 = (it & 31) * 4;
        const int t = t0 + row, col = n0 + c4;
        if (t >= M || col >= N) continue;
        const uint32_t off = (uint32_t)(row * 128 + c4) * 4u;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int rk = 0; rk < splits; rk++) {
          const float4 p = dsmem_ld4(dsmem_map(sbase + off, (uint32_t)rk));
          acc.x += p.x, acc.y += p.y, acc.z += p.z, acc.w += p.w;
        }
        const float o[4] = {acc.x, acc.y, acc.z, acc.w};
        float *yr = Y + (size_t)t * N + col;
        if (vec && col + 4 <= N) {
          float4 w4;
          w4.x = o[0] + (bias ? __ldg(bias + col) : 0.f);
          w4.y = o[1] + (bias ? __ldg(bias + col + 1) : 0.f);
          w4.z = o[2] + (bias ? __ldg(bias + col + 2) : 0.f);
          w4.w = o[3] + (bias ? __ldg(bias + col + 3) : 0.f);
          *reinterpret_cast<float4 *>(yr) = w4;
        } else {
#pragma unroll
          for (int j = 0; j < 4; j++)
            if (col + j < N) yr[j] = o[j] + (bias ? __ldg(bias + col + j) : 0.f);
        }
      }
    }
    cluster_sync_all();  // the peers have read this CTA's partial tile
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TS_TMEM_COLS);
  }
}

template <int BT, int STAGES, int KSUB>
void launch_ts_t(const NbitsArgs &a, const __half *a16, int64_t K8, int splits, cudaStream_t s, float *act,
                 __half *act16) {
  using L = TsLayout<BT, STAGES, KSUB>;
  CUtensorMap tm;
  const cuuint64_t dims[2] = {(cuuint64_t)K8, (cuuint64_t)a.M};
  const cuuint64_t strides[1] = {(cuuint64_t)(K8 * 2)};
  const cuuint32_t box[2] = {64u, (cuuint32_t)BT};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = tensor_map_encoder()(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(a16), dims, strides,
                                    box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  B2M_REQUIRE(r == CUDA_SUCCESS, B2M_ERR_CUDA, "cuTensorMapEncodeTiled failed for the activation operand");
  // Output map for the TMA-store epilogue: [M][N] fp32 rows, boxes of 128
  // columns x BT/2 tokens (needs 16-byte aligned rows; otherwise direct stores).
  CUtensorMap ty = tm;
  int use_ty = 0;
  if (!act && !act16 && (a.N % 4) == 0 && (reinterpret_cast<uintptr_t>(a.Y) & 15) == 0) {
    const cuuint64_t ydims[2] = {(cuuint64_t)a.N, (cuuint64_t)a.M};
    const cuuint64_t ystr[1] = {(cuuint64_t)(a.N * 4)};
    const cuuint32_t ybox[2] = {128u, (cuuint32_t)(BT / 2)};
    CUresult ry = tensor_map_encoder()(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, a.Y, ydims, ystr, ybox, estr,
                                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    B2M_REQUIRE(ry == CUDA_SUCCESS, B2M_ERR_CUDA, "cuTensorMapEncodeTiled failed for the output");
    use_ty = 1;
  }
  auto kern = nbits_ts_kernel<BT, STAGES, KSUB>;
  set_smem_limit_once<nbits_ts_kernel<BT, STAGES, KSUB>>((int)L::BYTES);
  PrefetchPlan pf = a.pf;
  pf.set_grid((a.w->npad / 128) * ((a.M + BT - 1) / BT) * splits);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.w->npad / 128), (unsigned)((a.M + BT - 1) / BT), (unsigned)splits);
  cfg.blockDim = dim3(TS_THREADS);
  cfg.dynamicSmemBytes = L::BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = (unsigned)splits;
  cfg.attrs = attr;
  cfg.numAttrs = splits > 1 ? 2 : 1;
  B2M_CUDA(cudaLaunchKernelEx(&cfg, kern, tm, ty, use_ty, reinterpret_cast<const uint4 *>(a.w->tsq),
                              reinterpret_cast<const uint2 *>(a.w->tss), a.bias, a.Y, (int)a.M, (int)a.N,
                              (int)(a.w->kp / 64), a.dev_err, pf, act, act16));
}

// Token-tile width. Per CTA: MMA time (a readiness check per stage caps the
// issue rate at about one MMA per 64 cycles, so tiles under 128 tokens cost as
// much per k-step as 128), the output burst (BT x 128 fp32, write throughput
// per SM is the limit: about half a column-unit per token) and a fixed cost;
// times the number of waves over the SMs.
int nbits_ts_pick_bt(int64_t M, int64_t N, int sms) {
  // Up to 64 rows (the decoder's decode projections): a 64-token tile,
  // measured 3-12% faster per op than 96 at 64 rows for the four projection
  // shapes of the config-5 decoder.
  if (M <= 64) return 64;
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

}  // namespace

namespace {

// Split-K: only when the output tiles leave three quarters of the SMs idle
// (the decoder's projections at 64 tokens); then the smallest cluster that
// reaches the fewest stages per CTA (<= 8 CTAs, at least one 128/256-k stage
// each) and still fits, checked once per tile width with the occupancy API.
template <int BT, int STAGES, int KSUB>
int ts_splits(const NbitsArgs &a, int sms) {
  const int64_t ctas = (a.w->npad / 128) * ((a.M + BT - 1) / BT);
  if (ctas * 4 > sms) return 1;
  const int64_t nst = (a.w->kp / 64 + KSUB - 1) / KSUB;
  // Each CTA keeps at least two stages: at 64 rows, splitting K = 1024 (four
  // 256-k stages, 32 column tiles) four ways measured 6.9 us per op against
  // 6.4 unsplit or two ways; K = 2048 / 3072 gain from splits down to two
  // stages per CTA and little beyond.
  const int64_t lim = std::min<int64_t>({(int64_t)8, std::max<int64_t>(1, nst / 2), sms / ctas});
  // The fewest CTAs that reach the smallest stage count per CTA.
  const int64_t per = (nst + lim - 1) / lim;
  int want = (int)((nst + per - 1) / per);
  static std::atomic<int> max_ok{0};
  if (max_ok.load() == 0) {
    using L = TsLayout<BT, STAGES, KSUB>;
    set_smem_limit_once<nbits_ts_kernel<BT, STAGES, KSUB>>((int)L::BYTES);
    int best = 1;
    for (int c = 2; c <= 8; c++) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(1, 1, (unsigned)c);
      cfg.blockDim = dim3(TS_THREADS);
      cfg.dynamicSmemBytes = L::BYTES;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = 1;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = (unsigned)c;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, nbits_ts_kernel<BT, STAGES, KSUB>, &cfg) == cudaSuccess && n > 0) best = c;
      else (void)cudaGetLastError();
    }
    max_ok.store(best);
  }
  return std::max(1, std::min(want, max_ok.load()));
}

template <int BT, int STAGES, int KSUB>
void launch_ts_split(const NbitsArgs &a, const __half *a16, int64_t K8, int sms, cudaStream_t s, float *act,
                     __half *act16) {
  launch_ts_t<BT, STAGES, KSUB>(a, a16, K8, ts_splits<BT, STAGES, KSUB>(a, sms), s, act, act16);
}

}  // namespace

void launch_nbits_ts(const NbitsArgs &a, const __half *a16, int64_t K8, cudaStream_t s, float *act, __half *act16) {
  const int sms = device_sm_count();
  switch (nbits_ts_pick_bt(a.M, a.N, sms)) {
    case 256: launch_ts_split<256, 3, 2>(a, a16, K8, sms, s, act, act16); break;
    case 192: launch_ts_split<192, 4, 2>(a, a16, K8, sms, s, act, act16); break;
    case 128: launch_ts_split<128, 3, 4>(a, a16, K8, sms, s, act, act16); break;
    case 64: launch_ts_split<64, 3, 4>(a, a16, K8, sms, s, act, act16); break;
    default: launch_ts_split<96, 3, 4>(a, a16, K8, sms, s, act, act16); break;
  }
}
