// MatMulNBits kernels (reference: opMatMulNBits, lib/src/onnx_qlinear_ops.dart:115-228).
//
//  * nbits_decode_kernel  FAST mode, M <= 32 (token decode and small batches).
//    HBM-bound GEMV over the fragment-major packed layout (below): each lane
//    issues one coalesced 16-byte weight load per 64-k chunk and converts the
//    nibbles to f16 MMA fragments (exact integers q - zp) BEFORE
//    griddepcontrol.wait — the weights never depend on the previous kernel, so
//    under programmatic dependent launch the weight stream of step i+1
//    overlaps step i. After the wait only the activations (split into f16
//    hi + lo, keeping ~22 bits of A) are loaded and fed to warp-level
//    m16n8k16 MMAs; the per-(column, block) scale multiplies each block's
//    fp32 partial, so scales stay fp32.
//  * nbits_simt_kernel    FAST mode fallback for shapes the other kernels do
//    not take: dequantize a tile to fp32 in shared memory, fp32 FMA.
//  * nbits_dequant_f32    EXACT mode: materialise W[N][K] float32 exactly as
//    the reference's weight() (:177-191) does, for the exact fp32 GEMM.
#include "b2m_internal.cuh"
#include "ptx.cuh"
#include "tc_common.cuh"

namespace {

using namespace b2m;

// ---------------------------------------------------------------------------
// Packed layout ("fragment-major", written by the prepack in runtime.cu):
// the weights of 16 output columns (a tile) and 64 consecutive k (a chunk)
// form one 512-byte record; lane L = 4g + t of a warp owns bytes
// [16L, 16L+16): four 32-bit words, (32-k group 0, column g), (group 0,
// column g+8), (group 1, column g), (group 1, column g+8). Inside a word the
// bytes are the column's original packed bytes 2t, 2t+1, 8+2t, 9+2t of that
// 32-k group, i.e. k in [4t, 4t+4) and [16+4t, 16+4t+4). One coalesced 16-byte
// load per lane therefore yields exactly the m16n8k16 A-fragments of two MMA
// steps for two groups.
// ---------------------------------------------------------------------------
__host__ __device__ inline int64_t fm_byte(int64_t kp, int64_t col, int64_t k, int &nib_hi) {
  const int64_t tile = col >> 4;
  const int cc = (int)(col & 15), g = cc & 7, hi = cc >> 3;
  const int64_t chunk = k >> 6;
  const int grp = (int)((k >> 5) & 1);
  const int kin = (int)(k & 31), kk = kin & 15, t = kk >> 2;
  const int b = ((kin >> 4) << 1) + ((kk & 3) >> 1);
  nib_hi = kk & 1;
  return ((tile * (kp >> 6) + chunk) * 32 + (g * 4 + t)) * 16 + 4 * (2 * grp + hi) + b;
}

__device__ __forceinline__ int nib_at(const uint8_t *bq, int64_t kp, int64_t col, int64_t k) {
  int h;
  const uint8_t b = bq[fm_byte(kp, col, k, h)];
  return h ? (b >> 4) : (b & 15);
}

constexpr int DEC_WARPS = 16;  // warps per CTA; each owns 64-k chunks
constexpr bool DEC_LO = true;  // activations as f16 hi + lo (~22 bits)

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
__device__ __forceinline__ float zp_load(const NbitsWeight &w, int64_t col, int64_t blk) {
  if (ZPK == 1) {
    const uint8_t z = __ldg(w.zp_u8 + col * w.zstride + (blk >> 1));
    return (float)((blk & 1) ? (z >> 4) : (z & 15));
  } else if (ZPK == 2) {
    return __ldg(w.zp_f32 + col * w.nblocks + blk);
  }
  return 8.f;
}

// Weight fragment pair for one MMA step from one packed word: selector picks
// bytes (b0,b1) for step 0 or (b2,b3) for step 1. Returns
// half2(n_{4t} - zp, n_{4t+2} - zp) and half2(n_{4t+1} - zp, n_{4t+3} - zp).
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

// Decode GEMV, M <= 8*MT. One CTA = 16 output columns (one m16 tile) over all
// of K; warp w owns 64-k chunks w, w+NW, ... (at most CPW of them). Everything
// that depends only on the weights — the coalesced 16-byte fragment loads,
// nibble -> f16 conversion with the zero point subtracted (exact integers in
// [-15, 15]), the scales — happens before griddepcontrol.wait, so under
// programmatic dependent launch it overlaps the previous kernel. After the
// wait: activation loads (f16 hi, plus the f16 residual lo when LO), MMAs,
// per-block scaling, a fixed-order cross-warp reduction and the store.
template <int MT, int ZPK, bool BS16, int CPW, int NW, bool LO>
__global__ void __launch_bounds__(NW * 32) nbits_decode_kernel(const NbitsArgs p, const NbitsWeight w) {
  extern __shared__ __align__(16) float s_red[];  // [NW][MT][32][4]
  constexpr int SPS = BS16 ? 2 : 1;              // scales per 32-k group
  const int tile = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int nchunks = (int)(w.kp >> 6);
  const int nb = (int)w.nblocks;
  const int groups = (int)((w.nblocks * w.block + 31) >> 5);  // 32-k groups holding real nibbles
  const int c0 = tile * 16 + g, c1 = c0 + 8;

  uint32_t af[CPW][2][2][4];  // [chunk][group][step][a0..a3]
  float sc[CPW][2][SPS][2];   // [chunk][group][block][col g, col g+8]
#pragma unroll
  for (int i = 0; i < CPW; i++) {
    const int c = warp + i * NW;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (c < nchunks)
      v = __ldg(reinterpret_cast<const uint4 *>(w.bq + (((size_t)tile * nchunks + c) * 32 + lane) * 16));
#pragma unroll
    for (int grp = 0; grp < 2; grp++) {
      const int G = 2 * c + grp;
      const uint32_t x0 = grp ? v.z : v.x, x1 = grp ? v.w : v.y;
#pragma unroll
      for (int s = 0; s < 2; s++) {
        const int sb = BS16 ? s : 0;
        int blk = BS16 ? (2 * G + s) : (G * 32) / w.block;
        const bool valid = G < groups && blk < nb;
        if (!valid) blk = 0;
        const float z0 = zp_load<ZPK>(w, c0, blk), z1 = zp_load<ZPK>(w, c1, blk);
        if (BS16 || s == 0) {
          sc[i][grp][sb][0] = valid ? __ldg(w.scales + (size_t)c0 * nb + blk) : 0.f;
          sc[i][grp][sb][1] = valid ? __ldg(w.scales + (size_t)c1 * nb + blk) : 0.f;
        }
        const uint32_t sel = s == 0 ? 0x4140u : 0x4342u;
        wfrag<ZPK>(x0, sel, z0, af[i][grp][s][0], af[i][grp][s][2]);
        wfrag<ZPK>(x1, sel, z1, af[i][grp][s][1], af[i][grp][s][3]);
      }
    }
  }

  // Allow the next kernel in the stream to start its weight-only prologue
  // now that ours is done (triggering earlier lets several future kernels
  // crowd the SMs and measured slower); its griddepcontrol.wait still waits
  // for this whole grid to complete.
  pdl_launch_dependents();
  pdl_wait();  // the previous kernel's results (our activations) are visible

  const bool vec_ok = ((p.K & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.A) & 15) == 0);
  float acc[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; mt++)
#pragma unroll
    for (int e = 0; e < 4; e++) acc[mt][e] = 0.f;

#pragma unroll
  for (int i = 0; i < CPW; i++) {
    const int c = warp + i * NW;
    if (c >= nchunks) break;
    float4 av[2][2][MT];
#pragma unroll
    for (int grp = 0; grp < 2; grp++)
#pragma unroll
      for (int s = 0; s < 2; s++)
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
          av[grp][s][mt] = load_act4(p.A, p.M, p.K, mt * 8 + g, c * 64 + grp * 32 + s * 16 + 4 * t, vec_ok);
#pragma unroll
    for (int grp = 0; grp < 2; grp++) {
#pragma unroll
      for (int mt = 0; mt < MT; mt++) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < 2; s++) {
          const float4 v = av[grp][s][mt];
          uint32_t h0, l0, h1, l1;
          if (LO) {
            split_h2(v.x, v.z, h0, l0);
            split_h2(v.y, v.w, h1, l1);
          } else {
            h0 = h2_as_u32(__floats2half2_rn(v.x, v.z));
            h1 = h2_as_u32(__floats2half2_rn(v.y, v.w));
          }
          if (BS16) {
            float e[4] = {0.f, 0.f, 0.f, 0.f};
            mma_16816(e, af[i][grp][s], h0, h1, e);
            if (LO) mma_16816(e, af[i][grp][s], l0, l1, e);
            acc[mt][0] = fmaf(sc[i][grp][s % SPS][0], e[0], acc[mt][0]);
            acc[mt][1] = fmaf(sc[i][grp][s % SPS][0], e[1], acc[mt][1]);
            acc[mt][2] = fmaf(sc[i][grp][s % SPS][1], e[2], acc[mt][2]);
            acc[mt][3] = fmaf(sc[i][grp][s % SPS][1], e[3], acc[mt][3]);
          } else {
            mma_16816(d, af[i][grp][s], h0, h1, d);
            if (LO) mma_16816(d, af[i][grp][s], l0, l1, d);
          }
        }
        if (!BS16) {
          acc[mt][0] = fmaf(sc[i][grp][0][0], d[0], acc[mt][0]);
          acc[mt][1] = fmaf(sc[i][grp][0][0], d[1], acc[mt][1]);
          acc[mt][2] = fmaf(sc[i][grp][0][1], d[2], acc[mt][2]);
          acc[mt][3] = fmaf(sc[i][grp][0][1], d[3], acc[mt][3]);
        }
      }
    }
  }

  // Cross-warp reduction over the K split, in fixed warp order.
#pragma unroll
  for (int mt = 0; mt < MT; mt++)
    *reinterpret_cast<float4 *>(&s_red[((warp * MT + mt) * 32 + lane) * 4]) =
        make_float4(acc[mt][0], acc[mt][1], acc[mt][2], acc[mt][3]);
  __syncthreads();
  constexpr int OUTS = MT * 32 * 4;
  for (int o = threadIdx.x; o < OUTS; o += NW * 32) {
    const int e = o & 3, ln = (o >> 2) & 31, mt = o >> 7;
    float sum = 0.f;
#pragma unroll
    for (int wp = 0; wp < NW; wp++) sum += s_red[((wp * MT + mt) * 32 + ln) * 4 + e];
    const int col = tile * 16 + (ln >> 2) + ((e & 2) ? 8 : 0);
    const int row = mt * 8 + 2 * (ln & 3) + (e & 1);
    if (row < p.M && col < p.N) {
      if (p.bias) sum += __ldg(p.bias + col);
      p.Y[(size_t)row * p.N + col] = sum;
    }
  }
}

// Decode GEMV over the decode records (NbitsWeight::drec: block >= 32,
// integer or absent zero points), the same arithmetic as nbits_decode_kernel
// with every weight-side load of a chunk reduced to three per lane. The
// post-wait path (activation loads, MMAs, the cross-warp sum) is the chain's
// critical path, so its shape is fixed at compile time: VEC (16-byte aligned
// activation rows, K % 4 == 0) and FIT (the warps' chunks cover exactly the
// padded K, no chunk guard).
// (minBlocks 1 lets ptxas schedule the post-wait path with more registers:
// 52 instead of 42 at MT = CPW = 1, 1.84 instead of 2.02 us per chained
// launch; the occupancy itself measured the same either way.)
template <int MT, int CPW, bool VEC, bool FIT>
__global__ void __launch_bounds__(DEC_WARPS * 32, 1) nbits_decode_rec_kernel(const NbitsArgs p, const uint8_t *drec,
                                                                            int nchunks) {
  constexpr int NW = DEC_WARPS;
  __shared__ __align__(16) float s_red[NW * MT * 32 * 4];
  const int tile = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  // The declared next call's weights go to L2 first, so that its weight
  // prologue (launched when this grid triggers) reads L2 instead of HBM.
  if (threadIdx.x == 0 && p.pf.seg[0]) prefetch_share(p.pf, blockIdx.x);

  uint4 v[CPW];
  float4 s4[CPW];
  uint32_t zw[CPW];
#pragma unroll
  for (int i = 0; i < CPW; i++) {
    const int c = warp + i * NW;
    v[i] = make_uint4(0u, 0u, 0u, 0u);
    s4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    zw[i] = 0x8888u;
    if (FIT || c < nchunks) {
      const uint8_t *r = drec + ((size_t)tile * nchunks + c) * DREC_BYTES;
      v[i] = __ldg(reinterpret_cast<const uint4 *>(r + lane * 16));
      s4[i] = __ldg(reinterpret_cast<const float4 *>(r + 512 + g * 16));
      zw[i] = __ldg(reinterpret_cast<const uint16_t *>(r + 640 + g * 2));
    }
  }
  uint32_t af[CPW][2][2][4];  // [chunk][group][step][a0..a3]
#pragma unroll
  for (int i = 0; i < CPW; i++)
#pragma unroll
    for (int grp = 0; grp < 2; grp++) {
      const float z0 = (float)((zw[i] >> (4 * grp)) & 15u), z1 = (float)((zw[i] >> (8 + 4 * grp)) & 15u);
      const uint32_t x0 = grp ? v[i].z : v[i].x, x1 = grp ? v[i].w : v[i].y;
#pragma unroll
      for (int s = 0; s < 2; s++) {
        const uint32_t sel = s == 0 ? 0x4140u : 0x4342u;
        wfrag<1>(x0, sel, z0, af[i][grp][s][0], af[i][grp][s][2]);
        wfrag<1>(x1, sel, z1, af[i][grp][s][1], af[i][grp][s][3]);
      }
    }

  pdl_launch_dependents();  // after the weight prologue (earlier measured slower)
  pdl_wait();               // the previous kernel's results (our activations) are visible

  float acc[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; mt++)
#pragma unroll
    for (int e = 0; e < 4; e++) acc[mt][e] = 0.f;
#pragma unroll
  for (int i = 0; i < CPW; i++) {
    const int c = warp + i * NW;
    if (!FIT && c >= nchunks) break;
    float4 av[2][2][MT];
#pragma unroll
    for (int grp = 0; grp < 2; grp++)
#pragma unroll
      for (int s = 0; s < 2; s++)
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
          av[grp][s][mt] = load_act4(p.A, p.M, p.K, mt * 8 + g, c * 64 + grp * 32 + s * 16 + 4 * t, VEC);
#pragma unroll
    for (int grp = 0; grp < 2; grp++) {
      const float sa = grp ? s4[i].y : s4[i].x, sb = grp ? s4[i].w : s4[i].z;
#pragma unroll
      for (int mt = 0; mt < MT; mt++) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int s = 0; s < 2; s++) {
          const float4 a4 = av[grp][s][mt];
          uint32_t h0, l0, h1, l1;
          split_h2(a4.x, a4.z, h0, l0);
          split_h2(a4.y, a4.w, h1, l1);
          mma_16816(d, af[i][grp][s], h0, h1, d);
          mma_16816(d, af[i][grp][s], l0, l1, d);
        }
        acc[mt][0] = fmaf(sa, d[0], acc[mt][0]);
        acc[mt][1] = fmaf(sa, d[1], acc[mt][1]);
        acc[mt][2] = fmaf(sb, d[2], acc[mt][2]);
        acc[mt][3] = fmaf(sb, d[3], acc[mt][3]);
      }
    }
  }

  // Cross-warp reduction over the K split, in fixed warp order.
#pragma unroll
  for (int mt = 0; mt < MT; mt++)
    *reinterpret_cast<float4 *>(&s_red[((warp * MT + mt) * 32 + lane) * 4]) =
        make_float4(acc[mt][0], acc[mt][1], acc[mt][2], acc[mt][3]);
  __syncthreads();
  constexpr int OUTS = MT * 32 * 4;
  static_assert(OUTS <= NW * 32, "one output per thread");
  if (threadIdx.x < OUTS) {
    const int o = threadIdx.x;
    const int e = o & 3, ln = (o >> 2) & 31, mt = o >> 7;
    float sum = 0.f;
#pragma unroll
    for (int wp = 0; wp < NW; wp++) sum += s_red[((wp * MT + mt) * 32 + ln) * 4 + e];
    const int col = tile * 16 + (ln >> 2) + ((e & 2) ? 8 : 0);
    const int row = mt * 8 + 2 * (ln & 3) + (e & 1);
    if (row < p.M && col < p.N) {
      if (p.bias) sum += __ldg(p.bias + col);
      p.Y[(size_t)row * p.N + col] = sum;
    }
  }
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
        const int q = nib_at(w.bq, w.kp, gj, gk);
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
  const int q = nib_at(w.bq, w.kp, n, k);
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

// PRECISE-mode weight planes: the exact weight (as nbits_dequant_kernel makes
// it) split into bf16 hi = rn(w), lo = rn(w - hi), K-major [N][kp], zero for
// k >= K. Two consecutive k per thread.
__global__ void nbits_split_planes_kernel(const NbitsWeight w, int64_t K, int64_t N, int64_t kp, uint32_t *hi,
                                          uint32_t *lo) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;  // pair index
  const int64_t half = kp >> 1;
  if (idx >= N * half) return;
  const int64_t n = idx / half, k0 = (idx - n * half) * 2;
  float v[2];
#pragma unroll
  for (int j = 0; j < 2; j++) {
    const int64_t k = k0 + j;
    v[j] = 0.f;
    if (k < K) {
      const int64_t blk = k / w.block;
      const int q = nib_at(w.bq, w.kp, n, k);
      const float sc = w.scales[n * w.nblocks + blk];
      if (w.zp_kind == 2) {
        v[j] = __double2float_rn(__dmul_rn(__dsub_rn((double)q, (double)w.zp_f32[n * w.nblocks + blk]), (double)sc));
      } else {
        int zp = 8;
        if (w.zp_kind == 1) {
          const uint8_t z = w.zp_u8[n * w.zstride + (blk >> 1)];
          zp = (blk & 1) ? (z >> 4) : (z & 15);
        }
        v[j] = __fmul_rn((float)(q - zp), sc);
      }
    }
  }
  uint32_t h, l;
  split_bf16x2(v[0], v[1], h, l);
  hi[idx] = h;
  lo[idx] = l;
}

// Decode records (see NbitsWeight::drec): one warp per (tile, chunk); lanes
// copy the 512-byte fragment record, lanes 0-7 write the scales and
// zero-point word of columns g / g+8. Scales of groups past the real blocks
// are 0 (those nibbles are zero padding), as the bq path treats them.
__global__ void nbits_drec_kernel(const NbitsWeight w, int64_t records) {
  const int64_t rec = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (rec >= records) return;
  const int64_t nchunks = w.kp >> 6;
  const int64_t tile = rec / nchunks, c = rec - tile * nchunks;
  uint8_t *r = w.drec + rec * DREC_BYTES;
  reinterpret_cast<uint4 *>(r)[lane] = reinterpret_cast<const uint4 *>(w.bq + rec * 512)[lane];
  if (lane < 8) {
    const int64_t groups = (w.nblocks * w.block + 31) >> 5;
    float sv[4];
    uint32_t zw = 0;
    for (int j = 0; j < 4; j++) {
      const int64_t col = tile * 16 + lane + ((j & 2) ? 8 : 0);
      const int grp = j & 1;
      const int64_t G = 2 * c + grp;
      const int64_t blk = (G * 32) / w.block;
      const bool valid = G < groups && blk < w.nblocks;
      sv[j] = valid ? w.scales[col * w.nblocks + blk] : 0.f;
      uint32_t z = 8;
      if (valid && w.zp_kind == 1) {
        const uint8_t b = w.zp_u8[col * w.zstride + (blk >> 1)];
        z = (blk & 1) ? (b >> 4) : (b & 15);
      }
      // word layout: (g, grp 0) | (g, grp 1) << 4 | (g+8, grp 0) << 8 | (g+8, grp 1) << 12
      zw |= z << (4 * j);
    }
    float4 s4 = make_float4(sv[0], sv[1], sv[2], sv[3]);
    *reinterpret_cast<float4 *>(r + 512 + lane * 16) = s4;
    *reinterpret_cast<uint16_t *>(r + 640 + lane * 2) = (uint16_t)zw;
  }
}

template <int MT, int ZPK, bool BS16, int CPW>
void launch_decode_t(const NbitsArgs &a, cudaStream_t s, bool pdl) {
  auto kern = nbits_decode_kernel<MT, ZPK, BS16, CPW, DEC_WARPS, DEC_LO>;
  const int smem = DEC_WARPS * MT * 32 * 4 * (int)sizeof(float);
  if (smem > 48 * 1024) B2M_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((a.N + 15) / 16));
  cfg.blockDim = dim3(DEC_WARPS * 32);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2M_CUDA(cudaLaunchKernelEx(&cfg, kern, a, *a.w));
}

template <int MT, int CPW, bool VEC, bool FIT>
void launch_decode_rec_t(const NbitsArgs &a, cudaStream_t s, bool pdl) {
  NbitsArgs p = a;
  const unsigned grid = (unsigned)((a.N + 15) / 16);
  p.pf.set_grid(grid);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(DEC_WARPS * 32);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  B2M_CUDA(cudaLaunchKernelEx(&cfg, nbits_decode_rec_kernel<MT, CPW, VEC, FIT>, p, (const uint8_t *)a.w->drec,
                              (int)(a.w->kp / 64)));
}

template <int MT, int CPW>
void launch_decode_rec(const NbitsArgs &a, cudaStream_t s, bool pdl) {
  const bool vec = (a.K & 3) == 0 && (reinterpret_cast<uintptr_t>(a.A) & 15) == 0;
  const bool fit = a.w->kp / 64 == (int64_t)CPW * DEC_WARPS;
  if (vec) {
    fit ? launch_decode_rec_t<MT, CPW, true, true>(a, s, pdl) : launch_decode_rec_t<MT, CPW, true, false>(a, s, pdl);
  } else {
    fit ? launch_decode_rec_t<MT, CPW, false, true>(a, s, pdl) : launch_decode_rec_t<MT, CPW, false, false>(a, s, pdl);
  }
}

template <int MT, int CPW>
void launch_decode_z(const NbitsArgs &a, cudaStream_t s, bool pdl) {
  if (a.w->drec) {
    launch_decode_rec<MT, CPW>(a, s, pdl);
    return;
  }
  const bool bs16 = a.w->block == 16;
  switch (a.w->zp_kind) {
    case 0: bs16 ? launch_decode_t<MT, 0, true, CPW>(a, s, pdl) : launch_decode_t<MT, 0, false, CPW>(a, s, pdl); break;
    case 1: bs16 ? launch_decode_t<MT, 1, true, CPW>(a, s, pdl) : launch_decode_t<MT, 1, false, CPW>(a, s, pdl); break;
    default: bs16 ? launch_decode_t<MT, 2, true, CPW>(a, s, pdl) : launch_decode_t<MT, 2, false, CPW>(a, s, pdl); break;
  }
}

int decode_cpw(const NbitsWeight &w) {
  const int64_t chunks = w.kp / 64;
  return (int)((chunks + DEC_WARPS - 1) / DEC_WARPS);
}

}  // namespace

// Row groups x chunks per warp that the decode kernel is instantiated for
// (register budget: weights of CPW chunks stay in registers across the wait).
bool nbits_smallm_supported(const NbitsWeight &w, int64_t M) {
  if (M < 1 || M > 32) return false;
  const int cpw = decode_cpw(w);
  const int mt = M <= 8 ? 1 : M <= 16 ? 2 : 4;
  if (cpw <= 1) return true;
  if (cpw <= 2) return mt <= 2;
  if (cpw <= 4) return mt == 1;
  return false;
}

void launch_nbits_smallm(const NbitsArgs &a, cudaStream_t s, bool pdl) {
  const int cpw = decode_cpw(*a.w);
  const int mt = a.M <= 8 ? 1 : a.M <= 16 ? 2 : 4;
  B2M_REQUIRE(nbits_smallm_supported(*a.w, a.M), B2M_ERR_CUDA, "internal: decode kernel shape not instantiated");
  if (cpw <= 1) {
    if (mt == 1) launch_decode_z<1, 1>(a, s, pdl);
    else if (mt == 2) launch_decode_z<2, 1>(a, s, pdl);
    else launch_decode_z<4, 1>(a, s, pdl);
  } else if (cpw <= 2) {
    if (mt == 1) launch_decode_z<1, 2>(a, s, pdl);
    else launch_decode_z<2, 2>(a, s, pdl);
  } else if (cpw == 3 && a.w->drec) {
    launch_decode_rec<1, 3>(a, s, pdl);  // K = 3072: the warps' chunks cover K exactly
  } else {
    launch_decode_z<1, 4>(a, s, pdl);
  }
}

void nbits_build_drec(NbitsWeight &w, cudaStream_t s) {
  if (w.drec || w.block < 32 || w.zp_kind == 2 || !w.bq) return;
  const int64_t records = (w.npad / 16) * (w.kp / 64);
  B2M_CUDA(cudaMalloc(&w.drec, (size_t)(records * DREC_BYTES)));
  nbits_drec_kernel<<<(unsigned)((records + 7) / 8), 256, 0, s>>>(w, records);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaFree(w.drec);
    w.drec = nullptr;
    B2M_CUDA(e);
  }
}

void launch_nbits_simt(const NbitsArgs &a, cudaStream_t s) {
  dim3 grid((unsigned)((a.N + 63) / 64), (unsigned)((a.M + 63) / 64));
  B2M_REQUIRE(grid.y <= 65535, B2M_ERR_UNSUPPORTED, "MatMulNBits: too many rows");
  nbits_simt_kernel<<<grid, 256, 0, s>>>(a, *a.w);
  B2M_CUDA(cudaGetLastError());
}

void launch_nbits_split_planes(const NbitsWeight &w, int64_t K, int64_t N, int64_t kp, uint16_t *hi, uint16_t *lo,
                               cudaStream_t s) {
  const int64_t pairs = N * (kp / 2);
  nbits_split_planes_kernel<<<(unsigned)((pairs + 255) / 256), 256, 0, s>>>(
      w, K, N, kp, reinterpret_cast<uint32_t *>(hi), reinterpret_cast<uint32_t *>(lo));
  B2M_CUDA(cudaGetLastError());
}

void launch_nbits_dequant_f32(const NbitsWeight &w, int64_t K, int64_t N, float *out, cudaStream_t s) {
  const int64_t total = N * K;
  nbits_dequant_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(w, K, N, out);
  B2M_CUDA(cudaGetLastError());
}
