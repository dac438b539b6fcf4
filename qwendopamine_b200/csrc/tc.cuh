// tc.cuh -- Blackwell (sm_100a) tensor-memory and async-copy primitives:
// mbarriers with bounded waits, TMA 2-D tile loads, TMEM allocation and
// 32x32b loads/stores, tcgen05.mma (kind::f16, one CTA) with shared-memory
// matrix descriptors for 128-byte-swizzled tiles.
#pragma once

#include <cuda.h>

#include "mma16.cuh"

namespace gdn2 {
namespace tc {

// A wait on one mbarrier phase gives up after this much wall time (a correct
// kernel completes each phase within microseconds) or this many polls.
constexpr uint64_t kWaitLimitNs = 1000000000ull;
constexpr long kMaxPollRounds = 1L << 24;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase with the given parity; false if the time limit ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (long r = 0; r < kMaxPollRounds; ++r) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try(bar, parity)) return true;
    if (global_ns() - t0 > limit_ns) return false;
  }
  return false;
}
// Same, decided for the whole warp: true only if every lane saw the phase.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity,
                                          uint64_t limit_ns = kWaitLimitNs) {
  const bool ok = mbar_wait(bar, parity, limit_ns);
  return __all_sync(0xffffffffu, ok) != 0;
}

// 2-D tiled TMA load (no multicast) completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled TMA load (no multicast) completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// 1-D bulk copy global -> shared (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// ---- TMEM ------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                   smem_u32(dst)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane (warp w reads lanes
// 32*(w%4) .. +31; taddr must carry that lane base in bits 16+).  The values
// are valid only after tmem_wait_ld().
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 16 consecutive fp32 columns of this thread's TMEM lane (same lane rule).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31])));
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}

// ---- UMMA descriptors --------------------------------------------------------
// Shared-memory matrix descriptor (sm_100 format, version 1): start address,
// leading / stride byte offsets (16-byte units), layout type in bits 61-63
// (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t sdesc(const void* p, uint32_t lbo, uint32_t sbo,
                                          uint32_t layout) {
  uint64_t d = (uint64_t)((smem_u32(p) >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)(layout & 7u) << 61;
  return d;
}
constexpr uint32_t kSwizzle128 = 2;
// The same descriptor with its start-address field zero: OR in a shared-
// memory address in 16-byte units (addresses stay below 2^18, so the field's
// 14 bits hold it) -- the layout bits fold to constants and each descriptor
// of a fixed tile costs one add and one OR.
__host__ __device__ constexpr uint64_t sdesc_layout(uint32_t lbo, uint32_t sbo, uint32_t layout) {
  return ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) | ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)(layout & 7u) << 61);
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 accumulation.
// a_mn / b_mn: operand is MN-major (else K-major).
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int a_mn, int b_mn) {
  return (1u << 4)              // D format: f32
         | (1u << 7)            // A format: bf16
         | (1u << 10)           // B format: bf16
         | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D(tmem) (+)= A(smem) * B(smem), issued by the calling thread.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}
// Arrive on `bar` once every previously issued tcgen05.mma of this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                   smem_u32(bar))
               : "memory");
}

}  // namespace tc

// ---- host: TMA tensor maps (tmap.cu) ------------------------------------------
// Whether cuTensorMapEncodeTiled is reachable.
bool tmap_available();
// 2-D bf16 map over `rows` rows of `inner` elements; box = box_x x 64 rows,
// 128-byte swizzle (or none).
bool tmap_2d_bf16(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint32_t box_x,
                  bool swizzle);
// Same with a box of box_x x box_y rows (box_x * 2 = 128 bytes), 128-byte swizzle.
bool tmap_2d_box_bf16(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows,
                      uint32_t box_x, uint32_t box_y);
// 3-D map over token rows [rows][H][D] of 2- or 4-byte elements: box box_x
// columns (128 bytes) x 1 head x 64 rows, 128-byte swizzle.
// Unswizzled 2-D or 3-D map (dims innermost first, strides of the outer
// dimensions in bytes): a box lands in shared memory densely, so a box wider
// than the data it needs gives padded rows; elements outside the tensor read
// as zero.
bool tmap_plain(CUtensorMap* m, const void* base, int rank, const uint64_t* dims,
                const uint64_t* strides_bytes, const uint32_t* box, int elem_bytes);
bool tmap_rows(CUtensorMap* m, const void* base, uint64_t D, uint64_t H, uint64_t rows,
               uint32_t box_x, int elem_bytes);

}  // namespace gdn2
