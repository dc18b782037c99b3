// Thin inline-PTX helpers for sm_100a: mbarriers, 1-D bulk copies (TMA
// engine, no multicast), programmatic dependent launch, warp-level MMA.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

namespace b2m {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after `max_iters` polls (with backoff) and returns
// false, so a kernel never spins forever on a barrier that cannot complete.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint32_t max_iters) {
  for (uint32_t i = 0; i < max_iters; i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i > 64) __nanosleep(i > 4096 ? 1024 : 32);
  }
  return false;
}

// 1-D bulk copy global -> shared through the TMA engine, completing on `bar`.
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue now / wait until the previous kernel's results are visible. Both
// are no-ops when the launch did not enable programmatic serialization.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

__device__ __forceinline__ uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// D = A(16x16 f16, row) * B(16x8 f16, col) + C, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1,
                                          const float c[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}

}  // namespace b2m

// ---------------------------------------------------------------------------
// sm_100a tensor-core (tcgen05 / TMEM) and TMA helpers.
// ---------------------------------------------------------------------------
namespace b2m {

// 2-D tiled TMA load (no multicast) completing on `bar`; coordinates are
// (innermost, outer) in elements.
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 2-D tiled TMA store shared -> global (bulk-group completion); coordinates
// (innermost, outer) in elements. Out-of-range parts of the box are clipped.
__device__ __forceinline__ void tma_store_2d(const void *tmap, const void *src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
// Records `code` in the context's error word, which lives in mapped host
// memory: a plain store, since device atomics on host memory are not
// guaranteed across PCIe (every writer stores a nonzero code; any one of them
// is enough for the host).
__device__ __forceinline__ void set_dev_error(int32_t *err, int32_t code) {
  *reinterpret_cast<volatile int32_t *>(err) = code;
}

// silu(g) * u in float, the arithmetic of the SiLU*Mul glue op; the decode
// GEMV's fused SwiGLU load uses the same function, so both give the same bits.
__device__ __forceinline__ float silu_times(float g, float u) { return g / (1.f + expf(-g)) * u; }

// Hint: bring [src, src + bytes) into L2 (16-byte aligned address, size a
// multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// This CTA's share of the segments of a prefetch plan: CTA `cta` takes bytes
// [cta * share, (cta + 1) * share) of each segment (share a multiple of 16,
// computed on the host), in pieces of at most 16 KB. Segment sizes are
// multiples of 16.
template <typename Plan>
__device__ __forceinline__ void prefetch_share(const Plan &pl, int64_t cta) {
#pragma unroll
  for (int j = 0; j < 2; j++) {
    if (!pl.seg[j] || pl.share[j] <= 0) continue;
    int64_t off = cta * pl.share[j];
    const int64_t end = off + pl.share[j] < pl.bytes[j] ? off + pl.share[j] : pl.bytes[j];
    for (; off < end; off += 16384) {
      const int64_t n = end - off < 16384 ? end - off : 16384;
      bulk_prefetch_l2(static_cast<const uint8_t *>(pl.seg[j]) + off, (uint32_t)n);
    }
  }
}

__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until the bulk stores committed by this thread have completed.
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void *tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// Makes this thread's generic-proxy shared-memory writes visible to the async
// proxy (tcgen05.mma operand reads, TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// TMEM allocation by one full warp; the base address lands in *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Shared-memory matrix descriptor: K-major operand in the 128-byte swizzle
// layout (rows of 128 bytes, 8-row groups 1024 bytes apart). The tile base
// must be 1024-byte aligned; advancing along K inside the 128-byte row adds
// the byte offset to the start address.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address, 16-byte units
  d |= (uint64_t)1 << 16;                    // leading byte offset (unused for this layout)
  d |= (uint64_t)(1024 >> 4) << 32;          // stride byte offset: 8-row group pitch
  d |= (uint64_t)1 << 46;                    // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                    // swizzle: 128-byte
  return d;
}

// Instruction descriptor for kind::f16 / kind::i8 with K-major A and B.
//   c_format [4,6): 1 = F32, 2 = S32; a/b format [7,10) / [10,13);
//   N >> 3 at [17,23); M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t umma_idesc(int m, int n, uint32_t c_fmt, uint32_t a_fmt, uint32_t b_fmt) {
  return (c_fmt << 4) | (a_fmt << 7) | (b_fmt << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accum)
      : "memory");
}

// A operand from TMEM (128 lanes = rows of A, K packed two f16 per 32-bit
// column in k order), B from shared memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                            uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(db), "r"(idesc), "r"(accum)
      : "memory");
}

// Eight TS MMAs of kind::i8 (two 128-byte chunks x four K=32 steps), same
// operand walk as umma_f16_ts_stage (32 bytes of K per MMA either way).
__device__ __forceinline__ void umma_i8_ts_stage(uint32_t tmem_d, uint32_t a, uint64_t bd, uint32_t b_chunk16,
                                                 uint32_t idesc, uint32_t accum) {
  const uint64_t c1 = bd + b_chunk16;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %18, 0;\n\t"
      "setp.eq.b32 q, %17, %17;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %9, %17, p;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%2], %10, %17, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%3], %11, %17, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%4], %12, %17, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%5], %13, %17, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%6], %14, %17, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%7], %15, %17, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%8], %16, %17, q;\n\t"
      "}" ::"r"(tmem_d),
      "r"(a), "r"(a + 8), "r"(a + 16), "r"(a + 24), "r"(a + 32), "r"(a + 40), "r"(a + 48), "r"(a + 56),
      "l"(bd), "l"(bd + 2), "l"(bd + 4), "l"(bd + 6), "l"(c1), "l"(c1 + 2), "l"(c1 + 4), "l"(c1 + 6),
      "r"(idesc), "r"(accum)
      : "memory");
}
__device__ __forceinline__ void umma_i8_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                           uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(db), "r"(idesc), "r"(accum)
      : "memory");
}

// One 128-k stage of TS MMAs (two 64-k chunks x four K=16 steps) as a single
// asm statement: all addresses are formed before the first MMA issues, so the
// eight tcgen05.mma go out back to back. `bd` is the stage's first B
// descriptor; chunk c starts `b_chunk16` 16-byte units further, each K=16
// step 2 units (32 bytes); the A operand advances 32 TMEM columns per chunk
// and 8 per step. `accum` = 0 overwrites D with the first product.
__device__ __forceinline__ void umma_f16_ts_stage(uint32_t tmem_d, uint32_t a, uint64_t bd, uint32_t b_chunk16,
                                                  uint32_t idesc, uint32_t accum) {
  const uint64_t c1 = bd + b_chunk16;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %18, 0;\n\t"
      "setp.eq.b32 q, %17, %17;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %9, %17, p;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %10, %17, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%3], %11, %17, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], %12, %17, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%5], %13, %17, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%6], %14, %17, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%7], %15, %17, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%8], %16, %17, q;\n\t"
      "}" ::"r"(tmem_d),
      "r"(a), "r"(a + 8), "r"(a + 16), "r"(a + 24), "r"(a + 32), "r"(a + 40), "r"(a + 48), "r"(a + 56),
      "l"(bd), "l"(bd + 2), "l"(bd + 4), "l"(bd + 6), "l"(c1), "l"(c1 + 2), "l"(c1 + 4), "l"(c1 + 6),
      "r"(idesc), "r"(accum)
      : "memory");
}

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accum)
      : "memory");
}

// Arrives on `bar` once all previously issued tcgen05.mma of this thread
// have completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 16 consecutive 32-bit TMEM columns -> 16 registers per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
// 32 registers per thread -> 32 lanes x 32 consecutive 32-bit TMEM columns.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
               : "memory");
}
// 8 registers per thread -> 32 lanes x 8 consecutive 32-bit TMEM columns.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace b2m
