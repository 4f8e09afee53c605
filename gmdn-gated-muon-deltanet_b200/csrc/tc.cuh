// Blackwell (sm_100a) tensor-core primitives: tcgen05 MMA with TMEM
// accumulators, shared-memory matrix descriptors, TMA tile loads and
// mbarriers with bounded waits.
//
// Layout conventions (bf16 operands, 128-byte swizzle):
//   * A "tile" is R rows x 64 columns of bf16 (128 B per row) stored in the
//     canonical SW128 arrangement: row r at byte r*128, its 16-byte chunk j at
//     position j ^ (r % 8).  Tiles start on 1024-byte boundaries.  A wider
//     matrix (R x 128) is two tiles ("panels") back to back.  This is what a
//     TMA load with CU_TENSOR_MAP_SWIZZLE_128B and a 64-column box writes.
//   * Read with K along the columns, a panel is a K-major operand: SBO = 1024
//     (eight rows), advance 32 bytes per K=16 step inside the 128-byte row.
//   * Read with K along the rows, it is an MN-major operand: LBO = byte
//     distance between the 64-wide panels, SBO = 1024 (eight K rows), advance
//     2048 bytes per K=16 step.
//   * Accumulators: M=128 puts row m in TMEM lane m; M=64 puts row m in lane
//     (m % 16) + 32 * (m / 16) (the first half of each 32-lane subpartition).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace gmdn {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// status word and bounded waits
// ---------------------------------------------------------------------------

// Bits of the per-launch status word a kernel ORs in on failure.
enum : uint32_t {
  kStatusWaitTimeout = 1u,  // an mbarrier wait gave up
  kStatusBadShape = 2u,
};

// Upper bound of one wait: ~2 s of wall time (globaltimer is in ns).
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// One arrival per warp: all 32 lanes call it (converged); lane 0 arrives after
// the warp has synchronised, so the barrier's count is the number of warps.
// Each lane's earlier fences (tcgen05 before_thread_sync, proxy.async) are
// ordered before the arrival by the warp barrier.  An mbarrier arrival is an
// atomic on one shared-memory word: 256 per-thread arrivals serialise on it
// (measured: hand-offs of 150-300 cycles), 8 per-warp arrivals do not.
__device__ __forceinline__ void mbar_arrive_warp(uint64_t* bar) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Same, but the thread may be suspended (not spinning, so it leaves the
// issue slots to the working warps) for up to `hint_ns` while the phase is
// still open.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity,
                                                    uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Gives up after
// limit_ns (kWaitLimitNs in the kernels), ORs kStatusWaitTimeout into *status
// and sets *abort (shared) so that the other warps stop too.  Returns false on
// give-up or if another warp already aborted.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, uint32_t* status,
                                              volatile int* abort_flag, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (*abort_flag) return false;
    if (global_ns() - t0 > limit_ns) {
      *abort_flag = 1;
      atomicOr(status, kStatusWaitTimeout);
      return false;
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status,
                                          volatile int* abort_flag) {
  return mbar_wait_for(bar, parity, status, abort_flag, kWaitLimitNs);
}

// ---------------------------------------------------------------------------
// fences
// ---------------------------------------------------------------------------

// Make generic-proxy shared-memory writes visible to the async proxy (the
// tensor core and TMA), before signalling the thread that issues them.
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMEM allocation (one full warp executes these)
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// ---------------------------------------------------------------------------
// descriptors
// ---------------------------------------------------------------------------

// Shared-memory matrix descriptor, SW128 layout, sm_100 version field.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // version = 1 (sm_100)
  d |= 2ull << 61;  // layout type: SWIZZLE_128B
  return d;
}

// K-major operand: rows = M (or N), K along the 128-byte rows.  `panel0` is
// the first 64-column panel; `panel_stride` the byte distance to the next one
// (K in [64, 128) lives there).  kstep counts K=16 steps.
//
// The descriptor of the panel is built once and the step offset is added to
// its start-address field (bits 0-13, address / 16; no carry for shared
// addresses below 256 KB).  With the panel loop-invariant and the step a
// constant of an unrolled loop this is one add per MMA: the single issuing
// thread otherwise spends ~200 cycles of dependent integer work per MMA and
// becomes the bottleneck (measured: 245 vs 64 cycles per 128x128x16 MMA).
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t panel0, uint32_t panel_stride,
                                                int kstep) {
  const uint32_t k = static_cast<uint32_t>(kstep) * 16u;
  const uint32_t off = (k >> 6) * panel_stride + (k & 63u) * 2u;
  return sw128_desc(panel0, 16u, 1024u) + static_cast<uint64_t>(off >> 4);
}

// MN-major operand: rows = K, M (or N) along the 128-byte rows, 64 per panel.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t panel0, uint32_t panel_stride,
                                                 int kstep) {
  return sw128_desc(panel0, panel_stride, 1024u) +
         static_cast<uint64_t>(static_cast<uint32_t>(kstep) * 128u);
}

// Instruction descriptor, kind::f16 with bf16 A/B and fp32 accumulation.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn, bool b_mn,
                                                  bool neg_a = false) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((neg_a ? 1u : 0u) << 13) |
         ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// tf32 operands (kind::tf32): fp32 containers, 32 per 128-byte row, K = 8 per
// instruction.  K-major: panel = 32 K columns, kstep counts K=8 steps (32 bytes
// along the row).  MN-major: rows = K, 32 M/N elements per row and panel, a
// K=8 step is one 1024-byte swizzle atom.
__device__ __forceinline__ uint64_t desc_kmajor_tf32(uint32_t panel0, uint32_t panel_stride,
                                                     int kstep) {
  const uint32_t k = static_cast<uint32_t>(kstep) * 8u;
  const uint32_t off = (k >> 5) * panel_stride + (k & 31u) * 4u;
  return sw128_desc(panel0, 16u, 1024u) + static_cast<uint64_t>(off >> 4);
}
__device__ __forceinline__ uint64_t desc_mnmajor_tf32(uint32_t panel0, uint32_t panel_stride,
                                                      int kstep) {
  return sw128_desc(panel0, panel_stride, 1024u) +
         static_cast<uint64_t>(static_cast<uint32_t>(kstep) * 64u);
}

// Instruction descriptor, kind::tf32 with fp32 accumulation.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N, bool a_mn, bool b_mn,
                                                  bool neg_a = false) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((neg_a ? 1u : 0u) << 13) |
         ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// fp32 -> tf32 (round to nearest, ties away; low 13 bits cleared), so the
// tensor core reads the operand exactly.
__device__ __forceinline__ float round_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// ---------------------------------------------------------------------------
// MMA issue (one thread) and completion
// ---------------------------------------------------------------------------

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same with the A operand in TMEM: an M x 16 bf16 slab, row m in lane m,
// elements 2i and 2i+1 packed (low, high) in column a_tmem + i.
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// A operand in TMEM: an M x 8 fp32 slab, row m in lane m, element k in column
// a_tmem + k.
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every MMA issued so far by this thread is done.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// TMEM -> registers.  32x32b: thread i of the warp reads lane (base lane + i),
// N consecutive 32-bit columns.  The warp may touch only lanes
// [32 * (warp % 4), 32 * (warp % 4) + 32).
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// registers -> TMEM, same 32x32b shape as tmem_ld16.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint4 r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr),
               "r"(r.x), "r"(r.y), "r"(r.z), "r"(r.w)
               : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t tmem_lane_base(int warp) {
  return static_cast<uint32_t>((warp & 3) * 32) << 16;
}

// ---------------------------------------------------------------------------
// TMA: 2-D tiled bulk tensor load into shared memory, completion counted in
// bytes on an mbarrier.  No multicast.
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// 2-D tiled bulk tensor store shared -> global (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const void* tmap, int x, int y, const void* src) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(tmap),
      "r"(x), "r"(y), "r"(smem_u32(src))
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until committed bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until committed bulk stores are complete.
__device__ __forceinline__ void bulk_wait0() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// ... all but the N most recently committed groups.
template <int N>
__device__ __forceinline__ void bulk_wait_n() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Cross-CTA hand-off of data written by bulk stores and read by TMA loads
// (both async proxy) through a counter in global memory (generic proxy):
// the writer waits for its stores to complete, orders them before the
// counter's release with a proxy fence; the reader acquires the counter and
// orders its later TMA loads after it with the same fence.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Plain 1-D bulk copy global -> shared (16-byte aligned, size multiple of 16).
// shared -> global bulk copy (16-byte aligned, size a multiple of 16), bulk group
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// SW128 tile element addressing for threads that read or write tiles
// ---------------------------------------------------------------------------

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a panel.
__device__ __forceinline__ uint32_t sw128_chunk(int row, int chunk) {
  return static_cast<uint32_t>(row) * 128u +
         (static_cast<uint32_t>(chunk ^ (row & 7)) << 4);
}

// Byte offset of element `col` (0..63) of row `row` inside a panel (bf16).
__device__ __forceinline__ uint32_t sw128_elem(int row, int col) {
  return sw128_chunk(row, col >> 3) + static_cast<uint32_t>(col & 7) * 2u;
}

// Square root and reciprocal from the special-function unit's approximations
// (relative error a few 2^-23).  The IEEE-rounded sqrtf / __frcp_rn are long
// instruction sequences: on the adam reverse chain's per-element pass (three
// of them per element, on the chain, two warps a scheduler) a clock64 trace
// put the pass's arithmetic at ~3.5k cycles per 8 elements against ~0.8k with
// these.  Both are used only where the result feeds the bf16 path.
__device__ __forceinline__ float sqrt_sfu(float x) { return x > 0.f ? x * rsqrtf(x) : 0.f; }
__device__ __forceinline__ float rcp_sfu(float x) { return __fdividef(1.f, x); }

// Element pairs on sm_100's packed fp32x2 FMA / multiply / add: one
// instruction for two elements, each rounded exactly as the scalar one.
__device__ __forceinline__ float2 p2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 p2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {   // a - b, exact as a subtraction
  return __ffma2_rn(b, make_float2(-1.f, -1.f), a);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float bf16_lo(uint32_t x) { return __uint_as_float(x << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t x) { return __uint_as_float(x & 0xFFFF0000u); }

__device__ __forceinline__ uint4 pack8(const float* v) {
  uint4 w;
  w.x = pack_bf16(v[0], v[1]);
  w.y = pack_bf16(v[2], v[3]);
  w.z = pack_bf16(v[4], v[5]);
  w.w = pack_bf16(v[6], v[7]);
  return w;
}

__device__ __forceinline__ void unpack8(uint4 w, float* v) {
  v[0] = bf16_lo(w.x); v[1] = bf16_hi(w.x);
  v[2] = bf16_lo(w.y); v[3] = bf16_hi(w.y);
  v[4] = bf16_lo(w.z); v[5] = bf16_hi(w.z);
  v[6] = bf16_lo(w.w); v[7] = bf16_hi(w.w);
}

// Write 8 floats of row `row`, columns [col8*8, col8*8+8) of a bf16 tile made
// of 64-column panels `panel_stride` bytes apart, as one swizzled 16-byte chunk.
__device__ __forceinline__ void st_row8(uint8_t* tile, uint32_t panel_stride, int row, int col8,
                                        const float* v) {
  uint8_t* p = tile + (col8 >> 3) * panel_stride + sw128_chunk(row, col8 & 7);
  *reinterpret_cast<uint4*>(p) = pack8(v);
}

__device__ __forceinline__ uint4 ld_row8(const uint8_t* tile, uint32_t panel_stride, int row,
                                         int col8) {
  return *reinterpret_cast<const uint4*>(tile + (col8 >> 3) * panel_stride +
                                         sw128_chunk(row, col8 & 7));
}

// 64 x 64 bf16 identity in one SW128 panel (call with all threads of the CTA).
__device__ __forceinline__ void build_identity64(uint8_t* panel, int tid, int nthreads) {
  for (int r = tid; r < 64; r += nthreads) {
    for (int c8 = 0; c8 < 8; ++c8) {
      uint4 w = make_uint4(0, 0, 0, 0);
      if ((r >> 3) == c8) {
        const uint32_t one = 0x3F80u << (16 * (r & 1));
        const int word = (r & 7) >> 1;
        if (word == 0) w.x = one;
        if (word == 1) w.y = one;
        if (word == 2) w.z = one;
        if (word == 3) w.w = one;
      }
      *reinterpret_cast<uint4*>(panel + sw128_chunk(r, c8)) = w;
    }
  }
}

// Phase-parity waits: `use` counts completions of the barrier.  wait_use waits
// for completion `use`; wait_free for completion `use - 1` (immediately true
// for use 0), the producer side of a ring slot.
__device__ __forceinline__ bool wait_use(uint64_t* b, int use, uint32_t* st, volatile int* ab) {
  return mbar_wait(b, static_cast<uint32_t>(use) & 1u, st, ab);
}
__device__ __forceinline__ bool wait_free(uint64_t* b, int use, uint32_t* st, volatile int* ab) {
  return mbar_wait(b, (static_cast<uint32_t>(use) & 1u) ^ 1u, st, ab);
}

// Warp-uniform variants for roles whose warps arrive with mbar_arrive_warp:
// every lane waits and the warp agrees on the outcome, so after a give-up the
// whole warp leaves together and no lane is left behind in a later __syncwarp.
__device__ __forceinline__ bool wait_use_w(uint64_t* b, int use, uint32_t* st, volatile int* ab) {
  return __all_sync(0xffffffffu, wait_use(b, use, st, ab));
}
__device__ __forceinline__ bool wait_free_w(uint64_t* b, int use, uint32_t* st, volatile int* ab) {
  return __all_sync(0xffffffffu, wait_free(b, use, st, ab));
}

// Named barrier among `nthreads` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Per-thread slabs (layouts in fast_path.h, TcBufs): row c, column half `half`.
__device__ __forceinline__ float4* slab_f32(float* base, int bh, int half, int f, int c) {
  return reinterpret_cast<float4*>(base) + ((static_cast<size_t>(bh) * 2 + half) * 16 + f) * 128 + c;
}
__device__ __forceinline__ uint4* slab_bf16(uint16_t* base, size_t m, int half, int g, int c) {
  return reinterpret_cast<uint4*>(base) + ((m * 2 + half) * 8 + g) * 128 + c;
}
__device__ __forceinline__ void ld_f16x4(const float* base4, float* v) {
  // 16 consecutive slab floats of one thread = 4 float4 at a 128-float4 stride
#pragma unroll
  for (int f = 0; f < 4; ++f) {
    const float4 x = reinterpret_cast<const float4*>(base4)[f * 128];
    v[4 * f] = x.x;
    v[4 * f + 1] = x.y;
    v[4 * f + 2] = x.z;
    v[4 * f + 3] = x.w;
  }
}
__device__ __forceinline__ void st_f16x4(float* base4, const float* v) {
#pragma unroll
  for (int f = 0; f < 4; ++f)
    reinterpret_cast<float4*>(base4)[f * 128] = make_float4(v[4 * f], v[4 * f + 1], v[4 * f + 2], v[4 * f + 3]);
}

}  // namespace tc
}  // namespace gmdn
