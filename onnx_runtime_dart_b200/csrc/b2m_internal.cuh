// Internal types shared by the runtime (runtime.cu) and the kernel files.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <string>
#include <unordered_map>

#include "../../include/b2m.h"

// ---------------------------------------------------------------------------
// Errors: every ABI entry point converts a thrown B2mError into a status code
// and a thread-local message; nothing escapes the C boundary.
// ---------------------------------------------------------------------------
struct B2mError {
  b2m_status code;
  std::string msg;
};

[[noreturn]] void b2m_throw(b2m_status code, const std::string &msg);
// Sets the message b2m_last_error() returns on this thread.
void b2m_set_last_error(const std::string &msg);

#define B2M_CUDA(expr)                                                                     \
  do {                                                                                     \
    cudaError_t e__ = (expr);                                                              \
    if (e__ != cudaSuccess) {                                                              \
      (void)cudaGetLastError();                                                            \
      b2m_throw(e__ == cudaErrorMemoryAllocation ? B2M_ERR_OUT_OF_MEMORY : B2M_ERR_CUDA,   \
                std::string(#expr) + ": " + cudaGetErrorString(e__));                      \
    }                                                                                      \
  } while (0)

#define B2M_REQUIRE(cond, code, msg) \
  do {                               \
    if (!(cond)) b2m_throw((code), (msg)); \
  } while (0)

// Device-side error codes written by kernels that contain bounded waits.
#define B2M_DEVERR_NONE 0
#define B2M_DEVERR_MBAR_TIMEOUT 1
#define B2M_DEVERR_TMEM_TIMEOUT 2
#define B2M_DEVERR_INDEX 4       // gather id / rotary position outside its table
#define B2M_DEVERR_CACHE_FULL 5  // KV-cache append past its capacity

#define B2M_ATTN_COUNTERS 65536
// Device state block of a context: error word, counters (runtime.cu).
#define B2M_DEV_STATE_BYTES 256

struct b2m_ctx {
  int device = 0;
  int sm_count = 0;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  cudaMemPool_t pool = nullptr;
  const volatile int32_t *cancel_flag = nullptr;
  int64_t byte_budget = 0;
  int64_t live_bytes = 0;
  bool timing = false;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  float last_ms = 0.f;
  bool timing_pending = false;
  // Grow-only device workspace for op temporaries (transposes, converted
  // operands). Stream-ordered: reused by the next op on the same stream.
  void *scratch = nullptr;
  size_t scratch_bytes = 0;
  // The error word that kernels with bounded spin-waits (and index checks)
  // set: mapped pinned host memory, so a synchronising call reads it with a
  // plain load instead of a device-to-host copy. dev_err is its device
  // address, err_host its host address.
  int32_t *dev_err = nullptr;
  int32_t *err_host = nullptr;
  // Self-resetting device counters (zero between calls; B2M_DEV_STATE_BYTES),
  // used by DynamicQuantizeLinear.
  uint32_t *dev_counter = nullptr;
  // Programmatic dependent launch for the decode kernels (env
  // B2M_DISABLE_PDL=1 turns it off, e.g. to compare timelines).
  bool pdl = true;
  // Attention numerics (b2m_set_attention_mode): fp32 CUDA-core kernels and
  // no key splits when set.
  bool attn_exact = false;
  // Split-merge counters of the decode attention (launch_gqa), zeroed at
  // allocation and re-armed by the kernel; B2M_ATTN_COUNTERS words.
  uint32_t *attn_counters = nullptr;
  // Declared successors (b2m_weight_set_next): the weight whose call follows
  // each weight's call; its kernels prefetch the successor into L2.
  std::unordered_map<const b2m_weight *, const b2m_weight *> next_of;
  // Pinned staging for the host-buffer helpers.
  void *pinned = nullptr;
  size_t pinned_bytes = 0;
};

struct b2m_tensor {
  b2m_ctx *ctx = nullptr;
  void *data = nullptr;
  int32_t dtype = 0;
  int32_t rank = 0;
  int64_t shape[B2M_MAX_RANK] = {0};
  int64_t numel = 0;
  bool owned = false;
};

enum WeightKind { W_F32 = 1, W_I8 = 2, W_NBITS = 3 };

// Packed MatMulNBits weights (see prepack in runtime.cu):
//   bq      npad*kp/2 bytes in the fragment-major layout of k_nbits.cu: one
//           512-byte record per (16 columns, 64 k), 16 bytes per MMA lane.
//   scales  [npad][nblocks] float
//   zp_u8   [npad][zstride] packed uint4 (low nibble = even block), or
//   zp_f32  [npad][nblocks] float, or neither (zero point 8).
struct NbitsWeight {
  uint8_t *bq = nullptr;
  float *scales = nullptr;
  uint8_t *zp_u8 = nullptr;
  float *zp_f32 = nullptr;
  int zp_kind = 0;  // 0 none, 1 packed uint4, 2 float
  int block = 0;
  int64_t nblocks = 0;
  int64_t zstride = 0;
  int64_t kp = 0;    // padded K (multiple of 64, >= nblocks*block)
  int64_t npad = 0;  // padded N (multiple of 128)
  float *wdeq = nullptr;  // exact-mode float32 W [N][K], made on first use
  // PRECISE-mode operand of the FAST fp32 GEMM: the exactly dequantized W
  // split into bf16 hi / lo planes [N][f32_tc_kp(K)] (K-major), made on first
  // use.
  uint16_t *px_hi = nullptr, *px_lo = nullptr;
  // All scales are 0 or normal f16 numbers and zero points are integers, so
  // the tensor-core dequant may scale in f16 (one rounding per weight).
  bool f16_scales = false;
  // Prefill scale records (block >= 32, integer zero points, f16-safe
  // scales): [npad/16][kp/64][8] x 16 bytes, eight halves (s, 1024 + zp) for
  // columns g / g+8 of the two 32-k groups of a chunk; null otherwise.
  uint8_t *srec = nullptr;
  // TMEM-operand prefill layout (same eligibility as srec). tsq: per
  // (128-column tile, 64-k chunk) two 128 x 16-byte planes; column c's 32
  // bytes hold its 64 nibbles, word j = k 8j..8j+7 at bit offsets
  // 0,16,4,20,8,24,12,28. tss: per (tile, chunk) 128 x 2 words, half2
  // (s, 1024 + zp) of the chunk's two 32-k groups.
  uint8_t *tsq = nullptr;
  uint32_t *tss = nullptr;
  // Decode records (block >= 32, integer or absent zero points; derived on
  // the device from bq / scales / zero points, not exported): per (16-column
  // tile, 64-k chunk) DREC_BYTES = the 512-byte fragment record of bq, then
  // for each g in 0..7 the fp32 scales s(g, group 0), s(g, group 1),
  // s(g+8, group 0), s(g+8, group 1), then for each g a 16-bit word of the four
  // zero-point nibbles in the same order. One 16-byte load per lane for the
  // nibbles, one for the scales and one 2-byte load for the zero points.
  uint8_t *drec = nullptr;
};
constexpr int DREC_BYTES = 656;

// Packed int8 / uint8 weights: bt[npad][kpad] (K-major), colsum[n] = sum_k b.
// ts8: TMEM-operand / GEMV layout, per (128-column tile, 128-k chunk) eight
// planes of 128 columns x 16 bytes; plane p holds k 16p..16p+15 of the chunk
// for each column (k128 = K rounded up to 128).
struct I8Weight {
  int8_t *bt = nullptr;
  int32_t *colsum = nullptr;
  int32_t dtype = 0;
  int64_t kpad = 0, npad = 0;
  uint8_t *ts8 = nullptr;
  int64_t k128 = 0;
};

// Device buffers of a packed weight, for b2m_weight_export / import.
enum WeightSegment {
  SEG_F32, SEG_BX_HI, SEG_BX_LO, SEG_I8_BT, SEG_I8_COLSUM, SEG_I8_TS8, SEG_NB_BQ, SEG_NB_SCALES, SEG_NB_ZP_U8,
  SEG_NB_ZP_F32, SEG_NB_SREC, SEG_NB_TSQ, SEG_NB_TSS, SEG_COUNT
};

struct b2m_weight {
  b2m_ctx *ctx = nullptr;
  int kind = 0;
  int64_t k = 0, n = 0;
  size_t seg_bytes[SEG_COUNT] = {0};  // allocation size of each device buffer
  float *f32 = nullptr;  // W_F32: [K][N] row-major
  // W_F32 FAST-mode planes: K-major bf16 [N][roundup(K,64)], hi = rn(w),
  // lo = rn(w - hi).
  uint16_t *bx_hi = nullptr, *bx_lo = nullptr;
  I8Weight i8;
  NbitsWeight nb;
};

// ---------------------------------------------------------------------------
// Kernel launchers (implemented in k_*.cu)
// ---------------------------------------------------------------------------

// Epilogue kinds of the exact fp32 GEMM.
enum F32Epi {
  EPI_NONE = 0,
  EPI_GEMM = 1,      // y = acc; y *= alpha (if has_alpha); y += (beta*)C
  EPI_NBITS = 2,     // y = f32((double)acc + bias)   (tile path, :221-224)
  EPI_NBITS_M1 = 3,  // y = f32(sum_double + bias)    (decode path, :203)
};

struct F32GemmArgs {
  const float *A = nullptr;
  const float *B = nullptr;
  float *Y = nullptr;
  int64_t M = 0, N = 0, K = 0;
  int64_t sa_m = 0, sa_k = 0;  // A(i,k) = A[i*sa_m + k*sa_k]
  int64_t sb_k = 0, sb_n = 0;  // B(k,j) = B[k*sb_k + j*sb_n]
  int64_t ldy = 0;
  // Broadcast batches: batch index decomposes over bdims (row-major); the
  // operand offsets use per-dim strides (0 on broadcast dims).
  int nbd = 0;
  int64_t bdims[6] = {0};
  int64_t a_bstride[6] = {0};
  int64_t b_bstride[6] = {0};
  int64_t y_bstride = 0;
  int64_t batch = 1;
  // Reference numerics: which columns accumulate in double.
  int64_t m_eff = 0;   // row count the reference kernel saw (after batch collapse)
  int64_t tile_w = 0;  // column tile width of the reference call (N, or 32 for NBits)
  int all_double = 0;  // MatMulNBits single-row decode: every column in double
  // Epilogue
  int epi = EPI_NONE;
  int has_alpha = 0;
  float alpha = 1.f;
  const float *C = nullptr;
  int64_t c_rs = 0, c_cs = 0;
  int has_beta = 0;
  float beta = 1.f;
  const float *bias = nullptr;
  int32_t *dev_err = nullptr;
};

void launch_f32_exact(const F32GemmArgs &a, cudaStream_t s);
// FAST fp32 GEMM (three bf16 products on tcgen05) for a prepacked weight and
// contiguous A rows; `a_split` is scratch of f32_tc_scratch_bytes(M, K).
int64_t f32_tc_kp(int64_t K);
size_t f32_tc_scratch_bytes(int64_t M, int64_t K);
bool f32_tc_eligible(const F32GemmArgs &p, const b2m_weight *w);
void launch_f32_tc(const F32GemmArgs &p, const b2m_weight &w, void *a_split, cudaStream_t s);
// The same with the B planes given directly ([b_rows][f32_tc_kp(K)] each).
void launch_f32_tc_b(const F32GemmArgs &p, const void *b_hi, const void *b_lo, int64_t b_rows, void *a_split,
                     cudaStream_t s);
bool f32_tc_shape_ok(const F32GemmArgs &p);
// A[M][K] (row stride lda) -> bf16 hi / lo planes [M][kp] (zero padded).
void launch_f32_split(const float *A, int64_t lda, __nv_bfloat16 *p0, __nv_bfloat16 *p1, int64_t M, int64_t K,
                      int64_t kp, cudaStream_t s);
// The same GEMM on operands already split into bf16 planes: A planes (x0 then
// x1, each [M][f32_tc_kp(K)]) and B planes [b_rows][f32_tc_kp(K)]; p.Y, p.ldy
// and the Gemm epilogue fields as above. cm_P > 0 selects the channel-major
// output of a convolution: Y(i, j) at Y[(i / cm_P) * cm_bs + j * cm_P + i % cm_P].
void launch_f32_tc_planes(const F32GemmArgs &p, const void *b_hi, const void *b_lo, int64_t b_rows,
                          const void *a_planes, int64_t cm_P, int64_t cm_bs, cudaStream_t s);

// Convolution (Conv / ConvInteger / QLinearConv) as GEMMs over an im2col
// panel. Geometry with 1-3 spatial dims carried as three (leading unit dims).
struct ConvGeom {
  int64_t n = 0, cin = 0, m = 0, group = 1, cpg = 0, mpg = 0;
  int64_t in[3] = {1, 1, 1};   // D, H, W
  int64_t k[3] = {1, 1, 1};    // kernel D, H, W
  int64_t st[3] = {1, 1, 1};   // strides
  int64_t dil[3] = {1, 1, 1};  // dilations
  int64_t pad[3] = {0, 0, 0};  // leading pads (the trailing ones only shape the output)
  int64_t out[3] = {1, 1, 1};  // output D, H, W
  int64_t K = 0;               // cpg * kernel volume: the GEMM's reduction length
  int64_t P = 0;               // output pixels per image
};
// im2col of group `grp` for images [b0, b0 + nb): fp32 [nb][K][P] (the
// reference's panel, pixels contiguous), zero at padded taps.
void launch_conv_im2col_f32(const float *x, const ConvGeom &g, int64_t grp, int64_t b0, int64_t nb, float *cols,
                            cudaStream_t s);
// The same panel as rows [nb * P][kp] of bf16 split planes (hi, then lo),
// pixel-major, k zero-padded to kp (a multiple of 64): the FAST GEMM's A.
void launch_conv_im2col_planes(const float *x, const ConvGeom &g, int64_t grp, int64_t b0, int64_t nb, int64_t kp,
                               void *hi, void *lo, cudaStream_t s);
// int8 / uint8 rows [nb * P][kg] (kg >= K): padded taps and k >= K hold the
// input zero point (*xzp, or 0), so (x - xzp) vanishes there.
void launch_conv_im2col_i8(const void *x, const ConvGeom &g, int64_t grp, int64_t b0, int64_t nb, int64_t kg,
                           const void *xzp, uint8_t *rows, cudaStream_t s);
// Direct convolution, one output per thread, accumulated in double from the
// bias over the taps in (c, kd, kh, kw) order and rounded once (the
// reference's depthwise and N-D paths). wt: [K][m] (the prepacked layout).
// pad_taps != 0 also adds the zero products of padded taps.
void launch_conv_direct_double(const float *x, const float *wt, const float *bias, const ConvGeom &g, int pad_taps,
                               float *y, cudaStream_t s);
// ConvTranspose geometry (1-3 spatial dims carried as three): input [n][cin]
// [in...], weight [cin][mpg][k...], output [n][m][out...]; pad = leading pads
// (after output_shape has been resolved).
struct ConvTGeom {
  int64_t n = 0, cin = 0, m = 0, group = 1, cpg = 0, mpg = 0;
  int64_t in[3] = {1, 1, 1}, k[3] = {1, 1, 1}, st[3] = {1, 1, 1}, dil[3] = {1, 1, 1}, pad[3] = {0, 0, 0};
  int64_t out[3] = {1, 1, 1};
};
// Overlap-add of one group's GEMM planes prod[mpg * kvol][in_h * in_w] (one
// image, depth 1) into y [m][out_h][out_w]: each output element sums its
// planes in (kh, kw) order in float32, then adds the bias.
void launch_conv_transpose_col2im(const float *prod, const ConvTGeom &g, int64_t grp, const float *bias, float *y,
                                  cudaStream_t s);
// The reference's generic scatter, gathered per output element: over input
// channels of the group, then input positions in ascending order, each
// non-zero input adds x * w in double onto the float32 value; then the bias.
void launch_conv_transpose_scatter(const float *x, const float *w, const float *bias, const ConvTGeom &g, float *y,
                                   cudaStream_t s);

// QLinearConv's requantisation: q = roundEven((z + bias[ch]) * mult) + y_zp
// clamped to [lo, hi], mult = x_scale * w_scale[ch or 0] / y_scale in double.
struct ConvRequant {
  double xs = 0.0, ys = 1.0;
  const float *ws = nullptr;
  int64_t ws_len = 1;
  const int32_t *bias = nullptr;
  int32_t y_zp = 0, lo = 0, hi = 255;
};
// z [nb * P][mpg] int32 -> y[b][grp * mpg + j][p]: int32 (y32), or requantized
// bytes (yq with rq).
void launch_conv_scatter(const int32_t *z, const ConvGeom &g, int64_t grp, int64_t b0, int64_t nb, int32_t *y32,
                         void *yq, const ConvRequant &rq, cudaStream_t s);

// L2 prefetch of the next call's weight (its declared successor): CTA i of a
// launch takes bytes [i * share[j], (i + 1) * share[j]) of segment j (share a
// multiple of 16, set on the host for the launch's grid); empty when seg[0]
// is null.
struct PrefetchPlan {
  const void *seg[2] = {nullptr, nullptr};
  int64_t bytes[2] = {0, 0};
  int64_t share[2] = {0, 0};
  void set_grid(int64_t ctas) {
    for (int j = 0; j < 2; j++) share[j] = seg[j] && ctas > 0 ? ((bytes[j] + ctas - 1) / ctas + 15) / 16 * 16 : 0;
  }
};

// MatMulNBits
struct NbitsArgs {
  const float *A = nullptr;  // [M][K]
  const NbitsWeight *w = nullptr;
  const float *bias = nullptr;  // [N] or null
  float *Y = nullptr;           // [M][N]
  int64_t M = 0, K = 0, N = 0;
  int32_t *dev_err = nullptr;
  PrefetchPlan pf;
};
bool nbits_smallm_supported(const NbitsWeight &w, int64_t M);
// Builds w.drec from bq / scales / zero points when the weight qualifies.
void nbits_build_drec(NbitsWeight &w, cudaStream_t s);
void launch_nbits_smallm(const NbitsArgs &a, cudaStream_t s, bool pdl);
void launch_nbits_simt(const NbitsArgs &a, cudaStream_t s);
void launch_nbits_dequant_f32(const NbitsWeight &w, int64_t K, int64_t N, float *out, cudaStream_t s);
// W dequantized exactly (as nbits_dequant_f32) and split into bf16 hi / lo
// planes [N][kp], zero for k >= K.
void launch_nbits_split_planes(const NbitsWeight &w, int64_t K, int64_t N, int64_t kp, uint16_t *hi, uint16_t *lo,
                               cudaStream_t s);
// tcgen05 prefill GEMM; `a16` is scratch for A converted to f16, M x nbits_tc_k8(K).
int64_t nbits_tc_k8(int64_t K);
bool nbits_tc_supported(const NbitsWeight &w, int64_t M, int64_t K, int64_t N);
void launch_nbits_tc(const NbitsArgs &a, __half *a16, cudaStream_t s);
// The TMEM-operand variant (weights with tsq/tss), called by launch_nbits_tc
// after the activation conversion.
namespace b2m {
// fp32 rows -> f16 rows of K8 columns (zero padded; k permuted in groups of
// four when perm), the conversion in front of the tensor-core GEMMs.
void launch_f32_to_f16(const float *A, __half *A16, int64_t M, int64_t K, int64_t K8, int perm, cudaStream_t s);
}  // namespace b2m
// act / act16 (optional, 16-byte aligned): the SwiGLU epilogue. The weight's
// N = 2I rows are tile-interleaved (rows 128t .. 128t+63 the gate rows 64t ..,
// rows 128t+64 .. the matching up rows; N % 128 == 0) and the kernel writes
// act[M][I] = silu(gate) * up (fp32 and / or f16) instead of Y.
void launch_nbits_ts(const NbitsArgs &a, const __half *a16, int64_t K8, cudaStream_t s, float *act = nullptr,
                     __half *act16 = nullptr);

// Transformer glue (k_glue.cu)
// gamma_rs > 0: row i of a group of `per` rows uses gains gamma + i * gamma_rs
// (per-head gains, e.g. the q and k norms of one packed projection in one
// launch); 0: every row uses gamma. y16 (optional; D % 8 == 0 and per ==
// rows): the output rows also as f16 (round to nearest), the operand a FAST
// MatMulNBits prefill GEMM takes.
void launch_rmsnorm(const float *x, const float *skip, const float *gamma, float *y, float *sum_out, int64_t rows,
                    int D, double eps, int64_t per, int64_t gstride, cudaStream_t s, int64_t gamma_rs = 0,
                    __half *y16 = nullptr);
// p0 / p1 (optional; D % 64 == 0): the output rows also as the bf16 hi / lo
// planes a FAST fp32 Gemm takes as its A operand.
void launch_layernorm(const float *x, const float *skip, const float *gamma, const float *beta, float *y,
                      float *sum_out, int64_t rows, int D, double eps, cudaStream_t s,
                      __nv_bfloat16 *p0 = nullptr, __nv_bfloat16 *p1 = nullptr);
// SwiGLU over a tile-interleaved gate / up output y [rows][2I] (the layout
// of launch_nbits_ts's SwiGLU epilogue): act / act16 [rows][I], either may be
// null; I % 64 == 0, 16-byte aligned buffers.
void launch_silu_mul_tiles(const float *y, int64_t rows, int64_t I, float *act, __half *act16, cudaStream_t s);
void launch_silu_mul(const float *gate, const float *up, int64_t g_rs, int64_t u_rs, float *y, int64_t rows,
                     int64_t D, cudaStream_t s, __half *y16 = nullptr);
void launch_gelu(const float *x, float *y, int64_t n, cudaStream_t s);
// GELU into bf16 hi / lo planes (and y when not null); n % 4 == 0, aligned.
void launch_gelu_split(const float *x, float *y, __nv_bfloat16 *p0, __nv_bfloat16 *p1, int64_t n, cudaStream_t s);
void launch_add(const float *a, const float *b, float *y, int64_t rows, int64_t D, int b_bcast, cudaStream_t s);
void launch_gather_rows(const float *table, const int64_t *ids, float *y, int64_t rows, int64_t V, int64_t D,
                        int32_t *err, cudaStream_t s);
// Row argmax in two passes; pv / pi hold rows x argmax_chunks(rows, V)
// partial results.
int argmax_chunks(int64_t rows, int64_t V);
void launch_argmax(const float *x, int64_t *out, int64_t rows, int64_t V, float *pv, int64_t *pi, cudaStream_t s);
// Decode calls (S == 1) split the cached keys over gqa_decode_splits(...)
// CTAs per (kv head, sequence); split_part holds B*H*nsplit*(2 + D) floats
// (null: no split).
int gqa_decode_splits(int B, int S, int H, int KVH, int D, int CAP);
// Whether launch_gqa (same arguments) writes out16 from the attention kernel
// itself; then `out` may be null (only the f16 output is written).
bool gqa_writes_f16(const float *q, int64_t q_rs, const float *kcache, const float *vcache, const int32_t *past,
                    const float *cos, int rot, int B, int S, int H, int KVH, int D, int CAP, int nsplit, bool exact,
                    bool counters);
void launch_gqa(const float *q, const float *k, const float *v, int64_t q_rs, int64_t kv_rs, float *kcache,
                float *vcache, const int32_t *past, const float *cos, const float *sin, int half, int rot,
                int interleaved, float *out, int B, int S, int H, int KVH, int D, int CAP, float scale, int32_t *err,
                float *split_part, int nsplit, bool exact, uint32_t *counters, cudaStream_t s,
                __half *out16 = nullptr, const float *qk_gain = nullptr, double qk_eps = 0.0);
// `qk_gain` ([H + KVH][D] gain rows, or null): q and k are first RMS-normalised
// per head (eps `qk_eps`), inside the decode kernel for S == 1 (which then
// also appends the token's key and value), else in place by the head-rows
// norm before the append.
// `counters` (B * KVH zeroed words, or null): the last split CTA of each (kv
// head, sequence) merges the key splits itself, instead of a separate
// combine launch; the words are zero again when the call completes.
// `exact`: the fp32 CUDA-core attention kernels only (no bf16-split tensor-core
// kernels); with nsplit = 1 every sequence's result is independent of the batch.
void launch_mha(const float *q, const float *k, const float *v, int64_t q_rs, int64_t kv_rs, const float *mask,
                int64_t mask_bs, int64_t mask_hs, int64_t mask_qs, float *out, int B, int S, int T, int H, int KVH,
                int D, float scale, int causal, int32_t *err, bool exact, cudaStream_t s,
                __nv_bfloat16 *planes = nullptr);
void launch_advance_positions(int32_t *past, int n, int delta, cudaStream_t s);
void launch_rotary(const float *x, int64_t x_rs, const int64_t *pos, int pos_per_batch, const float *cos,
                   const float *sin, int half, int max_pos, float *y, int64_t y_rs, int B, int S, int heads, int D,
                   int rot, int interleaved, int32_t *err, cudaStream_t s);

// DynamicQuantizeLinear (k_quant.cu): y = quantized x, scale / zp written to
// device memory. `partial` holds dql_partial_floats() floats; `counter` is a
// zeroed device word the kernel leaves zeroed.
size_t dql_partial_floats();
void launch_dynamic_quantize(const float *x, int64_t n, uint8_t *y, float *scale, uint8_t *zp, float *partial,
                             uint32_t *counter, cudaStream_t s);

// MatMulInteger / QLinearMatMul
struct I8GemmArgs {
  const void *A = nullptr;  // [batch_a][M][K] uint8 or int8
  int a_signed = 0;
  int64_t a_bstride = 0;    // elements between A batches (0 = broadcast)
  const int8_t *Bt = nullptr;  // [batch_b][npad][kpad] K-major
  int b_signed = 0;
  int64_t b_bstride = 0;
  int64_t kpad = 0;
  const int32_t *colsum = nullptr;  // [batch_b][n] (stride n)
  int64_t colsum_bstride = 0;
  const void *azp = nullptr;  // scalar or [M]; dtype of A
  int64_t azp_len = 0;
  const void *bzp = nullptr;  // scalar or [N]; dtype of B
  int64_t bzp_len = 0;
  int azp_signed = 0, bzp_signed = 0;
  int64_t M = 0, N = 0, K = 0, batch = 1;
  // output
  int32_t *Y32 = nullptr;  // MatMulInteger
  void *Yq = nullptr;      // QLinearMatMul (uint8 or int8)
  int requant = 0;
  double mult = 0.0;
  // L2 prefetch of the declared next call's weight (b2m_weight_set_next).
  PrefetchPlan pf;
  int32_t y_zp = 0, lo = 0, hi = 0;
  int32_t *dev_err = nullptr;
  // Scratch for the tensor-core path's activation row sums (M int32), used
  // when there are b zero points.
  int32_t *rowsum = nullptr;
};
void launch_i8_gemm(const I8GemmArgs &a, cudaStream_t s);
// Tensor-core / GEMV path for a prepacked weight with ts8 (batch 1): true if
// it handled the call. Needs a.rowsum (M int32 of scratch) for M > 16.
bool launch_i8_tc(const I8GemmArgs &a, const I8Weight &w, cudaStream_t s);
void launch_i8_pack(const void *B, int b_signed, int64_t batch, int64_t K, int64_t N, int8_t *bt,
                    int64_t kpad, int64_t npad, int32_t *colsum, cudaStream_t s);
