// Tensor-core state scan at the fast_state_scan boundary (fp32 U, K in HBM),
// dh = 128: the GMDN_PREC_FAST path of gmdn_scan_fwd / gmdn_scan_bwd for the
// delta rule (the reference's default tf32 `tl.dot`, fast_scan.py:196-199, run
// on tcgen05 with more precision than tf32: it meets the 1e-4 fp32 bar).
//
// One CTA per (batch, head) walks the N chunks in order (fast_scan.py:72-95):
//
//   S_out[i] = S_i                        (pre-update state)
//   G_i      = U_i - S_i K_i
//   S_{i+1}  = a_i S_i + G_i
//
// The product S_i K_i is a split-bf16 GEMM on the tensor cores: S = S_hi +
// S_lo and K = K_hi + K_lo (each part bf16, ~16 significant bits together),
// D = S_hi K_hi + S_hi K_lo + S_lo K_hi with fp32 accumulation in TMEM.
//
//   * S (fp32) lives in the registers of the eight state warps: thread (row c
//     = TMEM lane, half h) owns S[c][64h .. 64h+63].  They write S_hi / S_lo
//     as packed bf16 pairs into TMEM, the A operand (128 x 128, K = dk).
//   * K_i and U_i arrive by TMA as fp32 in four 128-byte-swizzled boxes of 32
//     columns x 128 rows each, issued a chunk ahead by one thread.  After the
//     products of chunk i the state warps turn K_{i+1} into the bf16 hi / lo
//     tiles (two 64-column SW128 panels each, rows = dk), the MN-major B
//     operand, next to their own update of S: the raw box and the tiles are
//     read and written in orders where 32 threads hit every bank group once
//     per 8 rows (four wavefronts per 512 bytes).
//   * S_out[i] = S_i goes out through a 32 KB staging area and TMA stores, one
//     half of the columns after the other, while the products of chunk i run.
//     Storing rows straight from the registers (one row per thread) sends a
//     16-byte partial line per thread and instruction to L2 and cost as much
//     as the whole chain.
//
// Warp roles (352 threads): warps 0-7 state, 8 TMA loads, 9 TMA stores,
// 10 TMEM allocation and MMA issue.  Every wait is bounded (tc.cuh).
//
// HBM per chunk-head: U, K in (128 KB), S out (64 KB).

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "fast_path.h"
#include "tc.cuh"

namespace gmdn {
namespace {

using namespace tc;

constexpr int kD = 128;
constexpr int kThreadsScan = 352;   // warps 0-7 state, 8 TMA loads, 9 TMA stores, 10 MMA
constexpr uint32_t P128 = 16384;    // panel stride of a 128-row bf16 tile

// shared memory (bytes from a 1024-aligned base); an fp32 matrix is four
// 128-byte-swizzled TMA boxes of 32 columns x 128 rows (16 KB each)
constexpr uint32_t SC_KR = 0;          // K_i fp32 (64 KB)
constexpr uint32_t SC_KT = 65536;      // K_i bf16 hi (32 KB) + lo (32 KB): the MMA's B operand
constexpr uint32_t SC_U = 131072;      // U_i fp32 (64 KB)
constexpr uint32_t SC_SO = 196608;     // S_i staging for the TMA store: two boxes (32 KB)
constexpr uint32_t SC_BAR = 229376;
constexpr uint32_t SC_SMEM = SC_BAR + 256 + 1024;
static_assert(SC_SMEM <= 232448, "shared memory per block");

// TMEM columns: S hi / lo (packed bf16 pairs, the A operand), the product
constexpr uint32_t TS_SH = 0, TS_SL = 64, TS_G = 128;

struct BarsS {
  uint64_t u_full, u_empty, k_full, k_empty;
  uint64_t so_full[2], so_free[2];   // S staging, [h]: columns 64h .. 64h + 63
  uint64_t s_full, g_full, final_mma;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(BarsS) <= 256, "barrier block");

struct ScanTcArgs {
  const float* a;
  uint32_t* status;
  int N;
};

// 16-byte chunk holding fp32 columns [c, c+4) of row r of a matrix stored as
// four 128-byte-swizzled boxes of 32 columns (what a TMA load with
// CU_TENSOR_MAP_SWIZZLE_128B and a 32 x 128 box writes).  Thirty-two threads
// on consecutive rows reading the same columns hit every bank group once per
// eight rows: four wavefronts for 512 bytes, no conflict.
__device__ __forceinline__ uint32_t box_off(int r, int c) {
  const int j = (c & 31) >> 2;
  return (c >> 5) * 16384 + r * 128 + ((j ^ (r & 7)) << 4);
}

// Forward (REV false): chunks in order, B = K MN-major, G' = S K.
// Reverse (REV true): the delta backward's reverse chain, the same kernel with
// the chunks in reverse order, S := Sbar, U := gS, S_out := dU and B = K
// K-major (C = Sbar K^T): Sbar_i = a_i Sbar_{i+1} + (gS_i - Sbar_{i+1} K_i^T),
// dU_i = Sbar_{i+1} (fast_scan.py:182-186 for delta, where Gbar = Sbar).
template <bool REV>
__global__ void __launch_bounds__(kThreadsScan, 1)
scan_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_u, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_s, ScanTcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  BarsS* bars = reinterpret_cast<BarsS*>(sm + SC_BAR);
  volatile int* ab = &bars->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int N = args.N;
  uint32_t* status = args.status;
  constexpr uint32_t kTmemCols = 256;

  if (threadIdx.x == 0) {
    mbar_init(&bars->u_full, 1);
    mbar_init(&bars->u_empty, 8);
    mbar_init(&bars->k_full, 1);
    mbar_init(&bars->k_empty, 8);
    for (int h = 0; h < 2; ++h) {
      mbar_init(&bars->so_full[h], 4);
      mbar_init(&bars->so_free[h], 1);
    }
    mbar_init(&bars->s_full, 8);
    mbar_init(&bars->g_full, 1);
    mbar_init(&bars->final_mma, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 10) {
    tmem_alloc(&bars->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const size_t mat0 = static_cast<size_t>(bh) * N;   // matrix index of chunk 0
  auto chunk = [&](int i) { return REV ? N - 1 - i : i; };
  auto row0 = [&](int i) { return static_cast<int>((mat0 + chunk(i)) * kD); };

  if (warp == 8) {
    // ------------------------------------------------------------ TMA loads: K_j, U_j
    if (lane == 0) {
      int issued = 0;
      for (int j = 0; j < N; ++j) {
        if (!wait_free(&bars->k_empty, j, status, ab)) break;   // K_{j-1} converted
        mbar_expect_tx(&bars->k_full, 65536);
#pragma unroll
        for (int bx = 0; bx < 4; ++bx)
          tma_load_2d(sm + SC_KR + bx * 16384, &tm_k, bx * 32, row0(j), &bars->k_full);
        if (!wait_free(&bars->u_empty, j, status, ab)) { issued = -(j + 1); break; }
        mbar_expect_tx(&bars->u_full, 65536);
#pragma unroll
        for (int bx = 0; bx < 4; ++bx)
          tma_load_2d(sm + SC_U + bx * 16384, &tm_u, bx * 32, row0(j), &bars->u_full);
        issued = j + 1;
      }
      // no load may still be in flight when the block exits
      int dummy = 0;
      const int nk = issued < 0 ? -issued : issued, nu = issued < 0 ? -issued - 1 : issued;
      if (nk >= 1) mbar_wait(&bars->k_full, (nk - 1) & 1, status, &dummy);
      if (nu >= 1) mbar_wait(&bars->u_full, (nu - 1) & 1, status, &dummy);
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ TMA stores: S_out[i] = S_i
    // Both halves of S_i go through the same two staging boxes, one half
    // after the other: columns 0-63 (state warps 0-3), then 64-127 (4-7).
    if (lane == 0) {
      for (int i = 0; i < N; ++i) {
        bool ok = true;
        for (int h = 0; h < 2 && ok; ++h) {
          if (!wait_use(&bars->so_full[h], i, status, ab)) { ok = false; break; }
          tma_store_2d(&tm_s, 64 * h, row0(i), sm + SC_SO);
          tma_store_2d(&tm_s, 64 * h + 32, row0(i), sm + SC_SO + 16384);
          bulk_commit();
          bulk_wait_read0();
          mbar_arrive(&bars->so_free[h]);
        }
        if (!ok) break;
      }
      bulk_wait0();
    }
  } else if (warp == 10) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      // forward: S (TMEM) x K (MN-major); reverse: Sbar (TMEM) x K^T (K-major)
      constexpr uint32_t ID = idesc_bf16(128, 128, false, !REV);
      auto bdesc = [](uint32_t t, int k) {
        return REV ? desc_kmajor(t, P128, k) : desc_mnmajor(t, P128, k);
      };
      const uint32_t kh = smem_u32(sm + SC_KT), kl = kh + 32768u;
      for (int i = 0; i < N; ++i) {
        if (!wait_use(&bars->s_full, i, status, ab)) break;   // S_i and K_i tiles ready
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(tmem + TS_G, tmem + TS_SH + k * 8, bdesc(kh, k), ID, k > 0);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(tmem + TS_G, tmem + TS_SH + k * 8, bdesc(kl, k), ID, 1);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(tmem + TS_G, tmem + TS_SL + k * 8, bdesc(kh, k), ID, 1);
        mma_commit(&bars->g_full);
      }
      mma_commit(&bars->final_mma);
      int dummy = 0;
      mbar_wait(&bars->final_mma, 0, status, &dummy);
    }
  } else {
    // ------------------------------------------------------------ state rows
    const int c = (warp & 3) * 32 + lane;   // row of S = TMEM lane
    const int h = warp >> 2;                // columns [64 h, 64 h + 64)
    const uint32_t lb = tmem_lane_base(warp);
    float st[64];
#pragma unroll
    for (int e = 0; e < 64; ++e) st[e] = 0.f;

    // K_m fp32 (raw boxes) -> bf16 hi / lo tiles, the MMA's MN-major B
    // operand; unit (row r, 8-column group g), thread t takes units t + 256 b
    // (both sides conflict-free: four wavefronts per 512 bytes)
    auto convert_k = [&]() {
      uint8_t* kt = sm + SC_KT;
      const int t = threadIdx.x;
#pragma unroll 4
      for (int b = 0; b < 8; ++b) {
        const int u = t + 256 * b;
        const int r = u >> 4, g = u & 15;
        const float4 x0 = *reinterpret_cast<const float4*>(sm + SC_KR + box_off(r, 8 * g));
        const float4 x1 = *reinterpret_cast<const float4*>(sm + SC_KR + box_off(r, 8 * g + 4));
        const float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        float hi[8], lo[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          hi[e] = __bfloat162float(__float2bfloat16_rn(v[e]));
          lo[e] = v[e] - hi[e];
        }
        st_row8(kt, P128, r, g, hi);
        st_row8(kt + 32768, P128, r, g, lo);
      }
      fence_async_smem();                   // tiles -> the MMA (async proxy)
      mbar_arrive_warp(&bars->k_empty);     // raw K read: the next K may load
    };

    {
      uint32_t zr[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) zr[e] = 0u;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        tmem_st16(tmem + lb + TS_SH + h * 32 + q * 16, zr);
        tmem_st16(tmem + lb + TS_SL + h * 32 + q * 16, zr);
      }
      tmem_st_wait();
    }
    bool ok = wait_use_w(&bars->k_full, 0, status, ab);
    if (ok) convert_k();
    tc_fence_before();
    mbar_arrive_warp(&bars->s_full);
    for (int i = 0; ok && i < N; ++i) {
      // pre-update state out: this half's 64 columns into the staging boxes
      // (after the other half of S_{i-1}, or this half's, has been read out)
      if (!(h == 0 ? wait_free_w(&bars->so_free[1], i, status, ab)
                   : wait_use_w(&bars->so_free[0], i, status, ab)))
        break;
#pragma unroll
      for (int f = 0; f < 16; ++f)
        *reinterpret_cast<float4*>(sm + SC_SO + box_off(c, 4 * f)) =
            make_float4(st[4 * f], st[4 * f + 1], st[4 * f + 2], st[4 * f + 3]);
      fence_async_smem();
      mbar_arrive_warp(&bars->so_full[h]);
      const float a = __ldg(args.a + mat0 + chunk(i));
      if (!wait_use_w(&bars->u_full, i, status, ab)) break;
      if (!wait_use_w(&bars->g_full, i, status, ab)) break;
      tc_fence_after();
      const bool last = i + 1 == N;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float g[16];
        tmem_ld16(tmem + lb + TS_G + h * 64 + 16 * q, g);
        // U_i (row c, columns 64 h + 16 q ..)
        float u[16];
#pragma unroll
        for (int f = 0; f < 4; ++f) {
          const float4 x =
              *reinterpret_cast<const float4*>(sm + SC_U + box_off(c, h * 64 + 16 * q + 4 * f));
          u[4 * f] = x.x;
          u[4 * f + 1] = x.y;
          u[4 * f + 2] = x.z;
          u[4 * f + 3] = x.w;
        }
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) st[16 * q + e] = fmaf(a, st[16 * q + e], u[e] - g[e]);
      }
      // U_i read: the next U may load (the proxy fence orders these generic
      // reads before the TMA's async-proxy writes into the same boxes)
      fence_async_smem();
      mbar_arrive_warp(&bars->u_empty);
      if (last) break;
      // K_{i+1} into the tiles (the products of chunk i are done: g_full)
      if (!wait_use_w(&bars->k_full, i + 1, status, ab)) break;
      convert_k();
      // S_{i+1} as packed bf16 hi / lo into TMEM (A operand of the next products)
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        uint32_t hh[16], ll[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float x0 = st[32 * q + 2 * e], x1 = st[32 * q + 2 * e + 1];
          hh[e] = pack_bf16(x0, x1);
          ll[e] = pack_bf16(x0 - bf16_lo(hh[e]), x1 - bf16_hi(hh[e]));
        }
        tmem_st16(tmem + lb + TS_SH + h * 32 + q * 16, hh);
        tmem_st16(tmem + lb + TS_SL + h * 32 + q * 16, ll);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive_warp(&bars->s_full);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 10) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Delta backward, the parts off the chain: for every matrix (b, h, i)
//   dK_i = -S_i^T dU_i          (fast_scan.py:185, dU_i = Gbar_i)
//   da_i = <dU_i, S_i>          (fast_scan.py:150; for delta Gbar = Sbar)
// Persistent: one CTA per SM walks the matrices.  Sixteen converter warps
// read S_i and dU_i (fp32) from global memory in row order (a warp reads one
// 512-byte row per load), add the dot products for da_i, and write both as
// split bf16 hi / lo tiles (rows = v, the contracted index); one thread
// issues D = S_hi^T dU_hi + S_hi^T dU_lo + S_lo^T dU_hi (both operands
// MN-major) into one of two TMEM accumulators, which the same warps drain
// into a staging area for the TMA store of dK_i while the next matrix's
// products run.  The next matrix's loads are in flight meanwhile.
// ---------------------------------------------------------------------------

constexpr int kConvWarpsDk = 16;                 // convert and drain, 4 per TMEM lane group
constexpr int kMmaWarpDk = kConvWarpsDk;         // TMEM allocation, MMA issue
constexpr int kStoreWarpDk = kConvWarpsDk + 1;   // TMA stores of dK
constexpr int kThreadsDk = (kConvWarpsDk + 2) * 32;
constexpr uint32_t DK_S = 0;            // S_i hi (32 KB), lo (32 KB)
constexpr uint32_t DK_U = 65536;        // dU_i hi, lo
constexpr uint32_t DK_O = 131072;       // dK_i fp32 staging: four SW128 boxes (64 KB)
constexpr uint32_t DK_BAR = 196608;
constexpr uint32_t DK_SMEM = DK_BAR + 256 + 1024;

struct BarsDk {
  uint64_t tiles_full, done[2], d_free[2], o_full, o_free, final_mma;
  uint32_t tmem_base;
  int abort_flag;
  int red_count[2];
  float red[2][kConvWarpsDk];
};
static_assert(sizeof(BarsDk) <= 256, "barrier block");

struct DkArgs {
  const float *S, *dU;
  float* da;
  uint32_t* status;
  int mats;
};

__global__ void __launch_bounds__(kThreadsDk, 1)
scan_bwd_dk_tc_kernel(const __grid_constant__ CUtensorMap tm_dk, DkArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  BarsDk* bars = reinterpret_cast<BarsDk*>(sm + DK_BAR);
  volatile int* ab = &bars->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t* status = args.status;
  const int G = gridDim.x;

  if (threadIdx.x == 0) {
    mbar_init(&bars->tiles_full, kConvWarpsDk);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->done[b], 1);
      mbar_init(&bars->d_free[b], kConvWarpsDk);
      bars->red_count[b] = 0;
    }
    mbar_init(&bars->o_full, kConvWarpsDk);
    mbar_init(&bars->o_free, 1);
    mbar_init(&bars->final_mma, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarpDk) {
    tmem_alloc(&bars->tmem_base, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == kMmaWarpDk) {
    if (lane == 0) {
      // D[m][n] = -sum_v S[v][m] dU[v][n]: A = S^T and B = dU, both MN-major
      constexpr uint32_t ID = idesc_bf16(128, 128, true, true, true);
      const uint32_t sh = smem_u32(sm + DK_S), sl = sh + 32768u;
      const uint32_t uh = smem_u32(sm + DK_U), ul = uh + 32768u;
      int it = 0;
      for (int m = blockIdx.x; m < args.mats; m += G, ++it) {
        const int b = it & 1;
        if (!wait_use(&bars->tiles_full, it, status, ab)) break;
        if (!wait_free(&bars->d_free[b], it >> 1, status, ab)) break;
        tc_fence_after();
        const uint32_t d = tmem + b * 128;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(d, desc_mnmajor(sh, P128, k), desc_mnmajor(uh, P128, k), ID, k > 0);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(d, desc_mnmajor(sh, P128, k), desc_mnmajor(ul, P128, k), ID, 1);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(d, desc_mnmajor(sl, P128, k), desc_mnmajor(uh, P128, k), ID, 1);
        mma_commit(&bars->done[b]);   // D ready and both tiles free
      }
      mma_commit(&bars->final_mma);
      int dummy = 0;
      mbar_wait(&bars->final_mma, 0, status, &dummy);
    }
  } else if (warp == kStoreWarpDk) {
    if (lane == 0) {
      int it = 0;
      for (int m = blockIdx.x; m < args.mats; m += G, ++it) {
        if (!wait_use(&bars->o_full, it, status, ab)) break;
#pragma unroll
        for (int bx = 0; bx < 4; ++bx)
          tma_store_2d(&tm_dk, bx * 32, m * kD, sm + DK_O + bx * 16384);
        bulk_commit();
        bulk_wait_read0();
        mbar_arrive(&bars->o_free);
      }
      bulk_wait0();
    }
  } else {
    const int t = threadIdx.x;              // 0 .. 511
    const int r = (warp & 3) * 32 + lane;   // TMEM lane m (drain)
    const int qc = warp >> 2;               // drain columns [32 qc, 32 qc + 32)
    const uint32_t lb = tmem_lane_base(warp);
    // dK_i: TMEM -> the staging boxes (box qc, row r: conflict-free) -> TMA store
    auto drain = [&](int itp) -> bool {
      const int b = itp & 1;
      if (!wait_use_w(&bars->done[b], itp >> 1, status, ab)) return false;
      if (!wait_free_w(&bars->o_free, itp, status, ab)) return false;   // last store read out
      tc_fence_after();
      uint8_t* ob = sm + DK_O + qc * 16384 + r * 128;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        float x[16];
        tmem_ld16(tmem + lb + b * 128 + qc * 32 + 16 * q, x);
        tmem_ld_wait();
#pragma unroll
        for (int f = 0; f < 4; ++f)
          *reinterpret_cast<float4*>(ob + (((4 * q + f) ^ (r & 7)) << 4)) =
              make_float4(x[4 * f], x[4 * f + 1], x[4 * f + 2], x[4 * f + 3]);
      }
      tc_fence_before();
      mbar_arrive_warp(&bars->d_free[b]);
      fence_async_smem();
      mbar_arrive_warp(&bars->o_full);
      return true;
    };
    // S_i and dU_i in coalesced order: float4 j = t + 512 f is row j >> 5,
    // columns 4 (j & 31) .. + 3, so a warp reads one 512-byte row per load.
    // The next matrix's loads go out as soon as this one's tiles are written,
    // so they are in flight while its products run and the previous dK drains.
    float4 sv4[8], uv4[8];
    auto load_mat = [&](int mm) {
      const float4* sp = reinterpret_cast<const float4*>(args.S + static_cast<size_t>(mm) * kD * kD);
      const float4* up = reinterpret_cast<const float4*>(args.dU + static_cast<size_t>(mm) * kD * kD);
#pragma unroll
      for (int f = 0; f < 8; ++f) {
        sv4[f] = __ldg(sp + t + 512 * f);
        uv4[f] = __ldg(up + t + 512 * f);
      }
    };
    // four fp32 -> bf16 hi / lo at (row, columns 4 c4 ..): 8 bytes into the
    // MN-major SW128 tile (panel c4 / 16, 16-byte chunk (c4 % 16) / 2, half c4 % 2)
    auto put4 = [&](uint8_t* tile, int row, int c4, float4 x) {
      const float v[4] = {x.x, x.y, x.z, x.w};
      float hi[4], lo[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        hi[e] = __bfloat162float(__float2bfloat16_rn(v[e]));
        lo[e] = v[e] - hi[e];
      }
      const uint32_t off = (c4 >> 4) * P128 + sw128_chunk(row, (c4 & 15) >> 1) + (c4 & 1) * 8;
      *reinterpret_cast<uint2*>(tile + off) = make_uint2(pack_bf16(hi[0], hi[1]), pack_bf16(hi[2], hi[3]));
      *reinterpret_cast<uint2*>(tile + 32768 + off) =
          make_uint2(pack_bf16(lo[0], lo[1]), pack_bf16(lo[2], lo[3]));
    };
    if (static_cast<int>(blockIdx.x) < args.mats) load_mat(blockIdx.x);
    int it = 0;
    bool ok = true;
    for (int m = blockIdx.x; m < args.mats; m += G, ++it) {
      // the tiles are free once the products of the previous matrix are done
      if (it >= 1 && !wait_use_w(&bars->done[(it - 1) & 1], (it - 1) >> 1, status, ab)) {
        ok = false;
        break;
      }
      float part = 0.f;
#pragma unroll
      for (int f = 0; f < 8; ++f) {
        const int j = t + 512 * f;
        const int row = j >> 5, c4 = j & 31;
        part = fmaf(sv4[f].x, uv4[f].x, part);
        part = fmaf(sv4[f].y, uv4[f].y, part);
        part = fmaf(sv4[f].z, uv4[f].z, part);
        part = fmaf(sv4[f].w, uv4[f].w, part);
        put4(sm + DK_S, row, c4, sv4[f]);
        put4(sm + DK_U, row, c4, uv4[f]);
      }
      fence_async_smem();
      mbar_arrive_warp(&bars->tiles_full);
      if (m + G < args.mats) load_mat(m + G);
      // da_i = <S_i, dU_i>: per-warp partials, summed in warp order by the
      // last warp to arrive (no block-wide barrier, so no unbounded wait)
      part = warp_sum(part);
      if (lane == 0) {
        const int slot = it & 1;
        bars->red[slot][warp] = part;
        __threadfence_block();
        if (atomicAdd(&bars->red_count[slot], 1) == kConvWarpsDk - 1) {
          __threadfence_block();
          float tot = 0.f;
#pragma unroll
          for (int w = 0; w < kConvWarpsDk; ++w) tot += bars->red[slot][w];
          args.da[m] = tot;
          bars->red_count[slot] = 0;
        }
      }
      // the previous matrix's dK while this one's products run
      if (it >= 1 && !drain(it - 1)) {
        ok = false;
        break;
      }
    }
    if (ok && it >= 1 && !*ab) drain(it - 1);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarpDk) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// rows x 128 fp32 matrix as a TMA map with 32 x 128 boxes and 128-byte swizzle.
cudaError_t make_tmap_f32_rows128(CUtensorMap* map, const void* base, uint64_t rows) {
  using Fn = PFN_cuTensorMapEncodeTiled_v12000;
  static Fn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return cudaErrorNotSupported;
    fn = reinterpret_cast<Fn>(p);
  }
  cuuint64_t dims[2] = {128, rows};
  cuuint64_t strides[1] = {512};
  cuuint32_t box[2] = {32, 128};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides,
                  box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <bool REV>
cudaError_t launch_scan_fwd_tc(const float* U, const float* K, float* S, const ScanTcArgs& a,
                               int BH, cudaStream_t st) {
  const uint64_t rows = static_cast<uint64_t>(BH) * a.N * kD;
  CUtensorMap mu, mk, ms;
  cudaError_t e;
  if ((e = make_tmap_f32_rows128(&mu, U, rows)) != cudaSuccess) return e;
  if ((e = make_tmap_f32_rows128(&mk, K, rows)) != cudaSuccess) return e;
  if ((e = make_tmap_f32_rows128(&ms, S, rows)) != cudaSuccess) return e;
  e = cudaFuncSetAttribute(scan_fwd_tc_kernel<REV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           SC_SMEM);
  if (e != cudaSuccess) return e;
  scan_fwd_tc_kernel<REV><<<BH, kThreadsScan, SC_SMEM, st>>>(mu, mk, ms, a);
  return cudaGetLastError();
}

}  // namespace

// Delta only.  Adam's update M / (sqrt(V) + 1e-6) turns sign-like where
// V ~ 0 (chunk 0, small nu), so product errors of ~2^-17 move its states by
// ~1e-3 and its K cotangent by ~1e-1: adam stays on the exact-fp32 kernels at
// both precisions.  The kernels move U, K, S, gS, dU and dK as 16-byte
// vectors (TMA or float4), so every such pointer must be 16-byte aligned;
// others take the exact kernels.
static bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

bool scan_fwd_tc_supported(const ScanArgs& p) {
  return p.rule == 0 && p.dh == kD && p.N >= 1 && tma_encode_available() && al16(p.U) &&
         al16(p.K) && al16(p.S);
}

cudaError_t scan_fwd_tc(const ScanArgs& p, uint32_t* status, cudaStream_t st) {
  if (p.rule != 0) return cudaErrorInvalidValue;
  ScanTcArgs a{};
  a.a = p.a;
  a.status = status;
  a.N = p.N;
  return launch_scan_fwd_tc<false>(p.U, p.K, p.S, a, p.BH, st);
}

bool scan_bwd_tc_supported(const ScanArgs& p) {
  return p.rule == 0 && p.dh == kD && p.N >= 1 && tma_encode_available() && al16(p.K) &&
         al16(p.S) && al16(p.gS) && al16(p.dU) && al16(p.dK);
}

cudaError_t scan_bwd_chain_tc(const ScanArgs& p, uint32_t* status, cudaStream_t st) {
  if (p.rule != 0) return cudaErrorInvalidValue;
  // reverse chain: U := gS, dU_i = Sbar_{i+1}
  ScanTcArgs a{};
  a.a = p.a;
  a.status = status;
  a.N = p.N;
  return launch_scan_fwd_tc<true>(p.gS, p.K, p.dU, a, p.BH, st);
}

cudaError_t scan_bwd_dk_tc(const ScanArgs& p, uint32_t* status, cudaStream_t st) {
  if (p.rule != 0) return cudaErrorInvalidValue;
  // delta reads no b, mu, nu
  const size_t sc = static_cast<size_t>(p.BH) * p.N * sizeof(float);
  cudaError_t e;
  if ((e = cudaMemsetAsync(p.db, 0, sc, st)) != cudaSuccess) return e;
  if ((e = cudaMemsetAsync(p.dm, 0, sc, st)) != cudaSuccess) return e;
  if ((e = cudaMemsetAsync(p.dn, 0, sc, st)) != cudaSuccess) return e;
  e = cudaFuncSetAttribute(scan_bwd_dk_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           DK_SMEM);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
    return e;
  DkArgs d{};
  d.S = p.S;
  d.dU = p.dU;
  d.da = p.da;
  d.status = status;
  d.mats = p.BH * p.N;
  CUtensorMap mdk;
  if ((e = make_tmap_f32_rows128(&mdk, p.dK, static_cast<uint64_t>(d.mats) * kD)) != cudaSuccess)
    return e;
  const int grid = sms < d.mats ? sms : d.mats;
  scan_bwd_dk_tc_kernel<<<grid, kThreadsDk, DK_SMEM, st>>>(mdk, d);
  return cudaGetLastError();
}

}  // namespace gmdn
