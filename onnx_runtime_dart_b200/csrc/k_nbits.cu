// MatMulNBits kernels (reference: opMatMulNBits, lib/src/onnx_qlinear_ops.dart:115-228).
//
//  * nbits_smallm_kernel  FAST mode, M <= 64 (token decode and small batches).
//    HBM-bound GEMV: each CTA owns 32 output columns over all of K, pulls its
//    packed nibbles, scales and zero points into shared memory with 1-D bulk
//    copies issued BEFORE griddepcontrol.wait (weights never depend on the
//    previous kernel, so under programmatic dependent launch the weight fetch
//    of step i+1 overlaps the tail of step i), then runs warp-level
//    m16n8k16 f16 MMAs with the weights as the 16-row operand (exact integers
//    q - zp) and the activations (split into f16 hi + lo parts, so the product
//    keeps ~22 bits of A) as the 8-column operand. The per-(column, block)
//    scale multiplies the fp32 partial of each block, so scales stay fp32.
//  * nbits_simt_kernel    FAST mode fallback for shapes the other kernels do
//    not take: dequantize a tile to fp32 in shared memory, fp32 FMA.
//  * nbits_dequant_f32    EXACT mode: materialise W[N][K] float32 exactly as
//    the reference's weight() (:177-191) does, for the exact fp32 GEMM.
#include "b2m_internal.cuh"
#include "ptx.cuh"

namespace {

using namespace b2m;

constexpr int SM_COLS = 32;    // output columns per CTA (two m16 tiles)
constexpr int SM_WARPS = 8;    // warps split K
constexpr int SM_THREADS = SM_WARPS * 32;

struct SmallmLayout {
  uint32_t wq, sc, zp, red, bar, total;
};

__host__ __device__ inline SmallmLayout smallm_layout(const NbitsWeight &w, int mt) {
  SmallmLayout L;
  L.wq = 0;
  L.sc = L.wq + (uint32_t)(SM_COLS * (w.kp / 2));
  L.zp = L.sc + (uint32_t)(SM_COLS * w.nblocks * 4);
  uint32_t zbytes = 0;
  if (w.zp_kind == 1) zbytes = (uint32_t)(SM_COLS * w.zstride);
  if (w.zp_kind == 2) zbytes = (uint32_t)(SM_COLS * w.nblocks * 4);
  L.red = (L.zp + zbytes + 15u) & ~15u;
  L.bar = L.red + (uint32_t)(SM_WARPS * 2 * mt * 32 * 4 * 4);
  L.total = L.bar + 16;
  return L;
}

// Four activations of row `r`, k = k0..k0+3 (zero outside [0,M) x [0,K)).
__device__ __forceinline__ float4 load_act4(const float *A, int64_t M, int64_t K, int64_t r, int64_t k0,
                                            bool vec_ok) {
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (r >= M) return v;
  const float *row = A + r * K;
  if (vec_ok) {
    if (k0 < K) v = __ldg(reinterpret_cast<const float4 *>(row + k0));
  } else {
    if (k0 + 0 < K) v.x = __ldg(row + k0 + 0);
    if (k0 + 1 < K) v.y = __ldg(row + k0 + 1);
    if (k0 + 2 < K) v.z = __ldg(row + k0 + 2);
    if (k0 + 3 < K) v.w = __ldg(row + k0 + 3);
  }
  return v;
}

// f16 hi + lo split of (x, y): hi = rn16(x), lo = rn16(x - hi).
__device__ __forceinline__ void split_h2(float x, float y, uint32_t &hi, uint32_t &lo) {
  const __half2 h = __floats2half2_rn(x, y);
  const float2 hf = __half22float2(h);
  const __half2 l = __floats2half2_rn(x - hf.x, y - hf.y);
  hi = h2_as_u32(h);
  lo = h2_as_u32(l);
}

template <int ZPK>
__device__ __forceinline__ float zp_value(const uint8_t *zs, int64_t c, int64_t blk, const NbitsWeight &w) {
  if (ZPK == 1) {
    const uint8_t z = reinterpret_cast<const uint8_t *>(zs)[c * w.zstride + (blk >> 1)];
    return (float)((blk & 1) ? (z >> 4) : (z & 15));
  } else if (ZPK == 2) {
    return reinterpret_cast<const float *>(zs)[c * w.nblocks + blk];
  }
  return 8.f;
}

// Weight fragment pair for one MMA step from the reordered 32-bit word:
// selector picks bytes (b0,b1) for step 0 or (b2,b3) for step 1.
// Returns half2(n_{4t}, n_{4t+2}) - zp and half2(n_{4t+1}, n_{4t+3}) - zp.
template <int ZPK>
__device__ __forceinline__ void wfrag(uint32_t x, uint32_t sel, float zp, uint32_t &even, uint32_t &odd) {
  const uint32_t d = prmt(x, 0u, sel);
  const uint32_t e = (d & 0x000F000Fu) | 0x64006400u;         // 1024 + n
  const uint32_t o = ((d >> 4) & 0x000F000Fu) | 0x64006400u;  // 1024 + n
  if (ZPK == 2) {
    const __half2 base = __float2half2_rn(1024.f);
    const __half2 z = __float2half2_rn(zp);
    even = h2_as_u32(__hsub2(__hsub2(u32_as_h2(e), base), z));
    odd = h2_as_u32(__hsub2(__hsub2(u32_as_h2(o), base), z));
  } else {
    const __half2 z = __float2half2_rn(1024.f + zp);  // exact: 1024..1039
    even = h2_as_u32(__hsub2(u32_as_h2(e), z));
    odd = h2_as_u32(__hsub2(u32_as_h2(o), z));
  }
}

template <int MT, int ZPK, bool BS16>
__global__ void __launch_bounds__(SM_THREADS) nbits_smallm_kernel(const NbitsArgs p, const NbitsWeight w) {
  extern __shared__ __align__(128) uint8_t smem[];
  const SmallmLayout L = smallm_layout(w, MT);
  uint8_t *s_wq = smem + L.wq;
  float *s_sc = reinterpret_cast<float *>(smem + L.sc);
  uint8_t *s_zp = smem + L.zp;
  float *s_red = reinterpret_cast<float *>(smem + L.red);
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem + L.bar);

  const int64_t col0 = (int64_t)blockIdx.x * SM_COLS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t row_bytes = w.kp / 2;

  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t wq_bytes = (uint32_t)(SM_COLS * row_bytes);
    const uint32_t sc_bytes = (uint32_t)(SM_COLS * w.nblocks * 4);
    uint32_t zp_bytes = 0;
    if (ZPK == 1) zp_bytes = (uint32_t)(SM_COLS * w.zstride);
    if (ZPK == 2) zp_bytes = (uint32_t)(SM_COLS * w.nblocks * 4);
    mbar_arrive_expect_tx(bar, wq_bytes + sc_bytes + zp_bytes);
    bulk_g2s(s_wq, w.bq + col0 * row_bytes, wq_bytes, bar);
    bulk_g2s(s_sc, w.scales + col0 * w.nblocks, sc_bytes, bar);
    if (ZPK == 1) bulk_g2s(s_zp, w.zp_u8 + col0 * w.zstride, zp_bytes, bar);
    if (ZPK == 2) bulk_g2s(s_zp, w.zp_f32 + col0 * w.nblocks, zp_bytes, bar);
  }
  pdl_launch_dependents();
  pdl_wait();  // activations / output buffer of the previous kernel are ready

  const bool vec_ok = ((p.K & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.A) & 15) == 0);
  const int64_t groups = w.kp / 32;
  const int64_t g_begin = groups * warp / SM_WARPS, g_end = groups * (warp + 1) / SM_WARPS;

  float acc[2][MT][4];
#pragma unroll
  for (int tt = 0; tt < 2; tt++)
#pragma unroll
    for (int mt = 0; mt < MT; mt++)
#pragma unroll
      for (int e = 0; e < 4; e++) acc[tt][mt][e] = 0.f;

  const bool ok = mbar_wait_bounded(bar, 0, 1u << 24);
  if (!ok) {
    if (lane == 0 && p.dev_err) atomicExch(p.dev_err, B2M_DEVERR_MBAR_TIMEOUT);
  } else {
    for (int64_t gi = g_begin; gi < g_end; gi++) {
      const int64_t kb = gi * 32;
      // Activation fragments: both MMA steps, all row groups.
      uint32_t bhi[2][MT][2], blo[2][MT][2];
#pragma unroll
      for (int s = 0; s < 2; s++)
#pragma unroll
        for (int mt = 0; mt < MT; mt++) {
          const float4 v = load_act4(p.A, p.M, p.K, mt * 8 + g, kb + 16 * s + 4 * t, vec_ok);
          split_h2(v.x, v.z, bhi[s][mt][0], blo[s][mt][0]);
          split_h2(v.y, v.w, bhi[s][mt][1], blo[s][mt][1]);
        }
#pragma unroll
      for (int tt = 0; tt < 2; tt++) {
        const int c0 = tt * 16 + g, c1 = c0 + 8;
        const uint32_t x0 = *reinterpret_cast<const uint32_t *>(s_wq + c0 * row_bytes + kb / 2 + 4 * t);
        const uint32_t x1 = *reinterpret_cast<const uint32_t *>(s_wq + c1 * row_bytes + kb / 2 + 4 * t);
        if (BS16) {
#pragma unroll
          for (int s = 0; s < 2; s++) {
            const int64_t blk = kb / 16 + s;
            const float z0 = zp_value<ZPK>(s_zp, c0, blk, w), z1 = zp_value<ZPK>(s_zp, c1, blk, w);
            const float sc0 = s_sc[c0 * w.nblocks + blk], sc1 = s_sc[c1 * w.nblocks + blk];
            const uint32_t sel = s == 0 ? 0x4140u : 0x4342u;
            uint32_t a[4];
            wfrag<ZPK>(x0, sel, z0, a[0], a[2]);
            wfrag<ZPK>(x1, sel, z1, a[1], a[3]);
#pragma unroll
            for (int mt = 0; mt < MT; mt++) {
              float d[4] = {0.f, 0.f, 0.f, 0.f};
              mma_16816(d, a, bhi[s][mt][0], bhi[s][mt][1], d);
              mma_16816(d, a, blo[s][mt][0], blo[s][mt][1], d);
              acc[tt][mt][0] = fmaf(sc0, d[0], acc[tt][mt][0]);
              acc[tt][mt][1] = fmaf(sc0, d[1], acc[tt][mt][1]);
              acc[tt][mt][2] = fmaf(sc1, d[2], acc[tt][mt][2]);
              acc[tt][mt][3] = fmaf(sc1, d[3], acc[tt][mt][3]);
            }
          }
        } else {
          const int64_t blk = kb / w.block;
          const float z0 = zp_value<ZPK>(s_zp, c0, blk, w), z1 = zp_value<ZPK>(s_zp, c1, blk, w);
          const float sc0 = s_sc[c0 * w.nblocks + blk], sc1 = s_sc[c1 * w.nblocks + blk];
          uint32_t a0[4], a1[4];
          wfrag<ZPK>(x0, 0x4140u, z0, a0[0], a0[2]);
          wfrag<ZPK>(x1, 0x4140u, z1, a0[1], a0[3]);
          wfrag<ZPK>(x0, 0x4342u, z0, a1[0], a1[2]);
          wfrag<ZPK>(x1, 0x4342u, z1, a1[1], a1[3]);
#pragma unroll
          for (int mt = 0; mt < MT; mt++) {
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            mma_16816(d, a0, bhi[0][mt][0], bhi[0][mt][1], d);
            mma_16816(d, a0, blo[0][mt][0], blo[0][mt][1], d);
            mma_16816(d, a1, bhi[1][mt][0], bhi[1][mt][1], d);
            mma_16816(d, a1, blo[1][mt][0], blo[1][mt][1], d);
            acc[tt][mt][0] = fmaf(sc0, d[0], acc[tt][mt][0]);
            acc[tt][mt][1] = fmaf(sc0, d[1], acc[tt][mt][1]);
            acc[tt][mt][2] = fmaf(sc1, d[2], acc[tt][mt][2]);
            acc[tt][mt][3] = fmaf(sc1, d[3], acc[tt][mt][3]);
          }
        }
      }
    }
  }

  // Cross-warp reduction over the K split, in fixed warp order.
#pragma unroll
  for (int tt = 0; tt < 2; tt++)
#pragma unroll
    for (int mt = 0; mt < MT; mt++)
      *reinterpret_cast<float4 *>(&s_red[(((warp * 2 + tt) * MT + mt) * 32 + lane) * 4]) =
          make_float4(acc[tt][mt][0], acc[tt][mt][1], acc[tt][mt][2], acc[tt][mt][3]);
  __syncthreads();
  if (!ok) return;
  constexpr int OUTS = 2 * MT * 32 * 4;
  for (int o = threadIdx.x; o < OUTS; o += SM_THREADS) {
    const int e = o & 3, ln = (o >> 2) & 31, mt = (o >> 7) % MT, tt = (o >> 7) / MT;
    float sum = 0.f;
#pragma unroll
    for (int wp = 0; wp < SM_WARPS; wp++) sum += s_red[(((wp * 2 + tt) * MT + mt) * 32 + ln) * 4 + e];
    const int gg = ln >> 2, t4 = ln & 3;
    const int64_t col = col0 + tt * 16 + gg + ((e & 2) ? 8 : 0);
    const int64_t row = mt * 8 + 2 * t4 + (e & 1);
    if (row < p.M && col < p.N) {
      if (p.bias) sum += p.bias[col];
      p.Y[row * p.N + col] = sum;
    }
  }
}

// Nibble of column row `wrow` (reordered layout) at logical k.
__device__ __forceinline__ int nib_at(const uint8_t *wrow, int64_t k) {
  const int64_t grp = k >> 5;
  const int kin = (int)(k & 31);
  const int kk = kin & 15;
  const int byte = 4 * (kk >> 2) + ((kin >> 4) << 1) + ((kk & 3) >> 1);
  const uint8_t b = wrow[grp * 16 + byte];
  return (kk & 1) ? (b >> 4) : (b & 15);
}

// Generic fp32 tile kernel: Y[64 x 64] per CTA, K in steps of 32.
__global__ void __launch_bounds__(256) nbits_simt_kernel(const NbitsArgs p, const NbitsWeight w) {
  __shared__ float As[32][64 + 4];
  __shared__ float Ws[32][64 + 4];
  const int64_t m0 = (int64_t)blockIdx.y * 64, n0 = (int64_t)blockIdx.x * 64;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < p.K; k0 += 32) {
    for (int e = tid; e < 64 * 32; e += 256) {
      const int mm = e % 64, kk = e / 64;
      const int64_t gi = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gi < p.M && gk < p.K) ? p.A[gi * p.K + gk] : 0.f;
      const int64_t gj = n0 + mm;
      float wv = 0.f;
      if (gj < p.N && gk < p.K) {
        const int64_t blk = gk / w.block;
        const int q = nib_at(w.bq + gj * (w.kp / 2), gk);
        float zp = 8.f;
        if (w.zp_kind == 1) {
          const uint8_t z = w.zp_u8[gj * w.zstride + (blk >> 1)];
          zp = (float)((blk & 1) ? (z >> 4) : (z & 15));
        } else if (w.zp_kind == 2) {
          zp = w.zp_f32[gj * w.nblocks + blk];
        }
        wv = ((float)q - zp) * w.scales[gj * w.nblocks + blk];
      }
      Ws[kk][mm] = wv;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; kk++) {
      float a_[4], b_[4];
#pragma unroll
      for (int i = 0; i < 4; i++) a_[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; j++) b_[j] = Ws[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a_[i], b_[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int64_t gi = m0 + ty * 4 + i;
    if (gi >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int64_t gj = n0 + tx * 4 + j;
      if (gj >= p.N) continue;
      p.Y[gi * p.N + gj] = acc[i][j] + (p.bias ? p.bias[gj] : 0.f);
    }
  }
}

// W[n][k] = f32((q - zp) * scale), bit-exact with the reference's weight().
__global__ void nbits_dequant_kernel(const NbitsWeight w, int64_t K, int64_t N, float *out) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= N * K) return;
  const int64_t n = idx / K, k = idx % K;
  const int64_t blk = k / w.block;
  const int q = nib_at(w.bq + n * (w.kp / 2), k);
  const float s = w.scales[n * w.nblocks + blk];
  float v;
  if (w.zp_kind == 2) {
    // (q - zp) and the product in double, then one rounding to float32.
    v = __double2float_rn(__dmul_rn(__dsub_rn((double)q, (double)w.zp_f32[n * w.nblocks + blk]), (double)s));
  } else {
    int zp = 8;
    if (w.zp_kind == 1) {
      const uint8_t z = w.zp_u8[n * w.zstride + (blk >> 1)];
      zp = (blk & 1) ? (z >> 4) : (z & 15);
    }
    // (q - zp) is a small integer: the float32 product is the correctly
    // rounded exact product, as in the reference's double-then-store.
    v = __fmul_rn((float)(q - zp), s);
  }
  out[idx] = v;
}

template <int MT, int ZPK, bool BS16>
void launch_smallm_t(const NbitsArgs &a, cudaStream_t s, bool pdl) {
  const SmallmLayout L = smallm_layout(*a.w, MT);
  auto kern = nbits_smallm_kernel<MT, ZPK, BS16>;
  B2M_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((a.N + SM_COLS - 1) / SM_COLS));
  cfg.blockDim = dim3(SM_THREADS);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2M_CUDA(cudaLaunchKernelEx(&cfg, kern, a, *a.w));
}

template <int MT>
void launch_smallm_mt(const NbitsArgs &a, cudaStream_t s, bool pdl) {
  const bool bs16 = a.w->block == 16;
  switch (a.w->zp_kind) {
    case 0: bs16 ? launch_smallm_t<MT, 0, true>(a, s, pdl) : launch_smallm_t<MT, 0, false>(a, s, pdl); break;
    case 1: bs16 ? launch_smallm_t<MT, 1, true>(a, s, pdl) : launch_smallm_t<MT, 1, false>(a, s, pdl); break;
    default: bs16 ? launch_smallm_t<MT, 2, true>(a, s, pdl) : launch_smallm_t<MT, 2, false>(a, s, pdl); break;
  }
}

}  // namespace

bool nbits_smallm_supported(const NbitsWeight &w, int64_t M) {
  if (M < 1 || M > 64) return false;
  const int mt = M <= 8 ? 1 : M <= 16 ? 2 : M <= 32 ? 4 : 8;
  return smallm_layout(w, mt).total <= 200 * 1024;
}

void launch_nbits_smallm(const NbitsArgs &a, cudaStream_t s, bool pdl) {
  if (a.M <= 8) launch_smallm_mt<1>(a, s, pdl);
  else if (a.M <= 16) launch_smallm_mt<2>(a, s, pdl);
  else if (a.M <= 32) launch_smallm_mt<4>(a, s, pdl);
  else launch_smallm_mt<8>(a, s, pdl);
}

void launch_nbits_simt(const NbitsArgs &a, cudaStream_t s) {
  dim3 grid((unsigned)((a.N + 63) / 64), (unsigned)((a.M + 63) / 64));
  B2M_REQUIRE(grid.y <= 65535, B2M_ERR_UNSUPPORTED, "MatMulNBits: too many rows");
  nbits_simt_kernel<<<grid, 256, 0, s>>>(a, *a.w);
  B2M_CUDA(cudaGetLastError());
}

void launch_nbits_dequant_f32(const NbitsWeight &w, int64_t K, int64_t N, float *out, cudaStream_t s) {
  const int64_t total = N * K;
  nbits_dequant_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(w, K, N, out);
  B2M_CUDA(cudaGetLastError());
}
