// Fused tensor-core forward of the mixer core, muon rule, dh = 128 (or 64,
// as a dh-128 head with zero upper features, see fwd_tc.cu), C = 64.
//
// Same residual form of the chunk as the delta kernel (fwd_tc.cu): with
// E_j = v_j - k_j S_j^T and token weights w_s = prod_{t>s} mu_t
// (train_ablation.py:151-158),
//
//   G_j     = E_j^T (w k_j)                              (train_ablation.py:164-165)
//             (E^T and w k both as bf16 hi + lo: hi.hi + lo.hi + hi.lo)
//   o_j     = q_j S_j^T + A_j E_j                        (train_ablation.py:166-167, 186)
//   M_{j+1} = mu_c M_j + G_j
//   X       = msign(M_{j+1}): X_0 = M / (|M|_F + 1e-7), then ns quintic
//             Newton-Schulz steps X <- c0 X + (c1 Gram + c2 Gram^2) X, Gram = X X^T
//   S_{j+1} = a_c S_j + b_c X                            (fast_scan.py:63-69, 86-89)
//
// The Newton-Schulz products run on the tensor cores with split bf16
// operands (x = hi + lo, three MMAs per product: hi.hi + hi.lo + lo.hi), so
// each product carries about 16 significant bits, and accumulate in fp32:
//
//   Gram  = X X^T          A = X, B = X (both K-major)          -> A1
//   Gram2 = Gram Gram      A = B = Gram (symmetric, K-major)     -> A2
//   X'    = P' X           A = P' from TMEM, B = X (MN-major)    -> A2
//   with P' = c0 I + c1 Gram + c2 Gram2 formed by the state warps.
//
// The first step takes X_0 = M unnormalised and folds 1/den into the Gram
// drain (1/den^2) and into P' (1/den).
//
// For the backward the kernel keeps S_j (bf16 hi and lo), M_{j+1} (fp32 slab) and the
// Newton-Schulz inputs X_0 (= M_{j+1} unnormalised), X_1 .. X_{ns-1} as the
// split bf16 tiles the MMAs read, copied out with bulk stores while the
// products run.
//
// Shared memory is time-shared: the chunk phase (E^T hi/lo, w*k, o staging)
// and the Newton-Schulz Gram tiles occupy the same 64 KB, and the S history
// staging reuses the X tiles after the last step.
//
// Warp roles (448 threads): warps 0-7 own the fp32 state (row c of S,
// 64 columns each), update M in a per-thread slab (the M history the backward
// reads) and drain every Newton-Schulz accumulator; warps 8-11 drain E, build
// w*k and A, and stage o; warp 12 issues TMA loads; warp 13 issues every MMA.

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "fast_path.h"
#include "tc.cuh"

namespace gmdn {
namespace {

using namespace tc;

constexpr int kC = 64;
constexpr int kD = 128;
constexpr int kThreadsM = 448;

constexpr uint32_t P64 = 8192;    // panel stride of a 64-row bf16 tile
constexpr uint32_t P128 = 16384;  // panel stride of a 128-row bf16 tile

// shared-memory map (bytes from a 1024-aligned base)
constexpr uint32_t M_Q = 0;          // q, k, v: one stage, 16 KB each
constexpr uint32_t M_K = 16384;
constexpr uint32_t M_V = 32768;
constexpr uint32_t M_AS = 49152;     // A_j bf16, 1 panel x 64 rows
constexpr uint32_t M_I = 57344;      // 64 x 64 identity
constexpr uint32_t M_XH = 65536;     // X hi, 2 panels x 128 rows (also S history staging)
constexpr uint32_t M_XL = 98304;     // X lo
constexpr uint32_t M_GH = 131072;    // Gram hi  | chunk phase: E^T hi (16 KB), E^T lo (16 KB)
constexpr uint32_t M_GL = 163840;    // Gram lo  | chunk phase: w*k (16 KB), o staging (16 KB)
constexpr uint32_t M_EH = 131072;
constexpr uint32_t M_EL = 147456;
constexpr uint32_t M_WK = 163840;
constexpr uint32_t M_OS = 180224;
constexpr uint32_t M_WKL = 196608;   // w*k bf16 remainder (16 KB), outside the Gram tiles
constexpr uint32_t M_GATE = 212992;  // beta[64], mu[64], w[64]
constexpr uint32_t M_RED = 213760;   // per-warp partial sums [8]
constexpr uint32_t M_BAR = 214016;
constexpr uint32_t M_SMEM = M_BAR + 256 + 1024;

// TMEM columns
constexpr uint32_t TM_EP = 0;    // E(j) (128 x 64) and P(j+1) (64 x 64), one at a time
constexpr uint32_t TM_O = 64;    // o^T
constexpr uint32_t TM_A1 = 128;  // G(j), then Gram
constexpr uint32_t TM_A2 = 256;  // Gram^2, then X'
constexpr uint32_t TM_SH = 384;  // S hi | P' hi (packed bf16 pairs)
constexpr uint32_t TM_SL = 448;  // S lo | P' lo

struct BarsM {
  uint64_t ld_full, ld_empty;
  uint64_t p_full, as_full, wk_full, e_full, e_smem, g_full, o_full, o_empty, os_free, s_full;
  uint64_t x_ready, gram_full, gram_smem, g2_full, p_ready, x_full;
  uint64_t final_mma;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(BarsM) <= 256, "barrier block");

struct MuonArgs {
  const float *alpha, *beta, *mu;
  uint16_t* S_hist;
  uint16_t* S_lo_hist;   // S_j - bf16(S_j), bf16
  float* M_hist;      // fp32 slab per chunk: M_{j+1}
  uint8_t* X_hist;    // per chunk ns slots of 64 KB: X_k hi tile, X_k lo tile
  uint32_t* status;
  int N, T, ns;
  int store_hi;   // dh 128: store o's upper 64 columns (dh 64: they are the zero padding)
};

// Split x into bf16 hi + lo and store 8 values of row `row` at column group
// col8 (of 16 per 128-column row) into the hi and lo K-major tiles.
__device__ __forceinline__ void st_split8(uint8_t* th, uint8_t* tl, int row, int col8,
                                          const float* x) {
  float hi[8], lo[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    hi[i] = __bfloat162float(__float2bfloat16_rn(x[i]));
    lo[i] = x[i] - hi[i];
  }
  st_row8(th, P128, row, col8, hi);
  st_row8(tl, P128, row, col8, lo);
}

// 16 consecutive values of row c -> packed bf16 hi / lo pairs in TMEM (8 columns each).
__device__ __forceinline__ void tmem_split16(uint32_t th, uint32_t tl, const float* x) {
  uint32_t hh[8], ll[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    hh[t] = pack_bf16(x[2 * t], x[2 * t + 1]);
    ll[t] = pack_bf16(x[2 * t] - bf16_lo(hh[t]), x[2 * t + 1] - bf16_hi(hh[t]));
  }
  tmem_st8(th, hh);
  tmem_st8(tl, ll);
}

__global__ void __launch_bounds__(kThreadsM, 1)
chunk_fwd_tc_muon(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                  const __grid_constant__ CUtensorMap tm_sh, const __grid_constant__ CUtensorMap tm_sl,
                  MuonArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  BarsM* bars = reinterpret_cast<BarsM*>(sm + M_BAR);
  float* gate_beta = reinterpret_cast<float*>(sm + M_GATE);
  float* gate_mu = gate_beta + 64;
  float* gate_w = gate_beta + 128;
  float* red = reinterpret_cast<float*>(sm + M_RED);
  volatile int* ab = &bars->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int N = args.N, ns = args.ns;
  uint32_t* status = args.status;

  if (threadIdx.x == 0) {
    mbar_init(&bars->ld_full, 1);
    mbar_init(&bars->ld_empty, 1 + 128);
    mbar_init(&bars->p_full, 1);
    mbar_init(&bars->as_full, 128);
    mbar_init(&bars->wk_full, 128);
    mbar_init(&bars->e_full, 1);
    mbar_init(&bars->e_smem, 128);
    mbar_init(&bars->g_full, 1);
    mbar_init(&bars->o_full, 1);
    mbar_init(&bars->o_empty, 128);
    mbar_init(&bars->os_free, 1);
    mbar_init(&bars->s_full, 256);
    mbar_init(&bars->x_ready, 256);
    mbar_init(&bars->gram_full, 1);
    mbar_init(&bars->gram_smem, 256);
    mbar_init(&bars->g2_full, 1);
    mbar_init(&bars->p_ready, 256);
    mbar_init(&bars->x_full, 1);
    mbar_init(&bars->final_mma, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  build_identity64(sm + M_I, threadIdx.x, kThreadsM);
  if (warp == 13) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const size_t tok0 = static_cast<size_t>(bh) * args.T;

  if (warp == 12) {
    // ------------------------------------------------------------ TMA loads (one stage)
    if (lane == 0) {
      int issued = 0;
      for (int j = 0; j < N; ++j) {
        const int row = static_cast<int>(tok0) + j * kC;
        if (!wait_free(&bars->ld_empty, j, status, ab)) break;   // chunks 0..j-1 consumed
        mbar_expect_tx(&bars->ld_full, 6 * 8192 + 512);
        tma_load_2d(sm + M_Q, &tm_q, 0, row, &bars->ld_full);
        tma_load_2d(sm + M_Q + P64, &tm_q, 64, row, &bars->ld_full);
        tma_load_2d(sm + M_K, &tm_k, 0, row, &bars->ld_full);
        tma_load_2d(sm + M_K + P64, &tm_k, 64, row, &bars->ld_full);
        tma_load_2d(sm + M_V, &tm_v, 0, row, &bars->ld_full);
        tma_load_2d(sm + M_V + P64, &tm_v, 64, row, &bars->ld_full);
        bulk_load(gate_beta, args.beta + tok0 + j * kC, 256, &bars->ld_full);
        bulk_load(gate_mu, args.mu + tok0 + j * kC, 256, &bars->ld_full);
        issued = j + 1;
      }
      int dummy = 0;
      if (issued >= 1) mbar_wait(&bars->ld_full, (issued - 1) & 1, status, &dummy);
    }
  } else if (warp == 13) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      const uint32_t q_s = smem_u32(sm + M_Q), k_s = smem_u32(sm + M_K), v_s = smem_u32(sm + M_V);
      const uint32_t wk_s = smem_u32(sm + M_WK), as_s = smem_u32(sm + M_AS);
      const uint32_t wkl_s = smem_u32(sm + M_WKL);
      const uint32_t eh_s = smem_u32(sm + M_EH), el_s = smem_u32(sm + M_EL);
      const uint32_t id_s = smem_u32(sm + M_I);
      const uint32_t xh_s = smem_u32(sm + M_XH), xl_s = smem_u32(sm + M_XL);
      const uint32_t gh_s = smem_u32(sm + M_GH), gl_s = smem_u32(sm + M_GL);
      constexpr uint32_t ID_P = idesc_bf16(64, 64, false, false);
      constexpr uint32_t ID_EV = idesc_bf16(128, 64, true, false, true);   // -v^T I
      constexpr uint32_t ID_ES = idesc_bf16(128, 64, false, false);        // S k^T (A in TMEM)
      constexpr uint32_t ID_G = idesc_bf16(128, 128, false, true);         // E^T (wk)
      constexpr uint32_t ID_O2 = idesc_bf16(128, 64, false, false);        // E^T A^T
      constexpr uint32_t ID_KK = idesc_bf16(128, 128, false, false);       // X X^T, Gram Gram
      constexpr uint32_t ID_PX = idesc_bf16(128, 128, false, true);        // P' X (A in TMEM)
      auto issue_P = [&](int j) -> bool {
        if (!wait_use(&bars->ld_full, j, status, ab)) return false;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(tmem + TM_EP, desc_kmajor(q_s, P64, k), desc_kmajor(k_s, P64, k), ID_P, k > 0);
        mma_commit(&bars->p_full);
        return true;
      };
      // D = A B^T with A, B K-major 128 x 128 split tiles (hi.hi + hi.lo + lo.hi)
      auto mm_kk = [&](uint32_t d, uint32_t ah, uint32_t al, uint32_t bh_, uint32_t bl) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(d, desc_kmajor(ah, P128, k), desc_kmajor(bh_, P128, k), ID_KK, k > 0);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(d, desc_kmajor(ah, P128, k), desc_kmajor(bl, P128, k), ID_KK, 1);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(d, desc_kmajor(al, P128, k), desc_kmajor(bh_, P128, k), ID_KK, 1);
      };
      bool ok = N > 0 && issue_P(0);
      for (int j = 0; ok && j < N; ++j) {
        // E(j): D = -v^T I + S_hi k^T + S_lo k^T = -E^T  (EP must be free: A(j) built)
        if (!wait_use(&bars->as_full, j, status, ab)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + TM_EP, desc_mnmajor(v_s, P64, k), desc_kmajor(id_s, P64, k), ID_EV, k > 0);
        if (!wait_use(&bars->s_full, j, status, ab)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(tmem + TM_EP, tmem + TM_SH + k * 8, desc_kmajor(k_s, P64, k), ID_ES, 1);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(tmem + TM_EP, tmem + TM_SL + k * 8, desc_kmajor(k_s, P64, k), ID_ES, 1);
        mma_commit(&bars->e_full);
        // o1(j): o^T = S_hi q^T
        if (!wait_free(&bars->o_empty, j, status, ab)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(tmem + TM_O, tmem + TM_SH + k * 8, desc_kmajor(q_s, P64, k), ID_ES, k > 0);
        // G(j) = E^T_hi wk_hi + E^T_lo wk_hi + E^T_hi wk_lo -> A1
        if (!wait_use(&bars->e_smem, j, status, ab)) break;
        if (!wait_use(&bars->wk_full, j, status, ab)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + TM_A1, desc_kmajor(eh_s, P128, k), desc_mnmajor(wk_s, P64, k), ID_G, k > 0);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + TM_A1, desc_kmajor(el_s, P128, k), desc_mnmajor(wk_s, P64, k), ID_G, 1);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + TM_A1, desc_kmajor(eh_s, P128, k), desc_mnmajor(wkl_s, P64, k), ID_G, 1);
        mma_commit(&bars->g_full);
        // o2(j): o^T += E^T_hi A^T
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + TM_O, desc_kmajor(eh_s, P128, k), desc_kmajor(as_s, P64, k), ID_O2, 1);
        mma_commit(&bars->o_full);
        mma_commit(&bars->ld_empty);
        // Newton-Schulz steps of chunk j
        for (int k = 0; ok && k < ns; ++k) {
          const int u = j * ns + k;
          if (!wait_use(&bars->x_ready, u, status, ab)) { ok = false; break; }
          tc_fence_after();
          mm_kk(tmem + TM_A1, xh_s, xl_s, xh_s, xl_s);              // Gram = X X^T
          mma_commit(&bars->gram_full);
          if (!wait_use(&bars->gram_smem, u, status, ab)) { ok = false; break; }
          tc_fence_after();
          mm_kk(tmem + TM_A2, gh_s, gl_s, gh_s, gl_s);              // Gram^2
          mma_commit(&bars->g2_full);
          if (!wait_use(&bars->p_ready, u, status, ab)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)                            // X' = P' X
            mma_bf16_ts(tmem + TM_A2, tmem + TM_SH + kk * 8, desc_mnmajor(xh_s, P128, kk), ID_PX, kk > 0);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_bf16_ts(tmem + TM_A2, tmem + TM_SH + kk * 8, desc_mnmajor(xl_s, P128, kk), ID_PX, 1);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma_bf16_ts(tmem + TM_A2, tmem + TM_SL + kk * 8, desc_mnmajor(xh_s, P128, kk), ID_PX, 1);
          mma_commit(&bars->x_full);
        }
        if (!ok) break;
        if (j + 1 < N && !issue_P(j + 1)) break;
      }
      mma_commit(&bars->final_mma);
      int dummy = 0;
      mbar_wait(&bars->final_mma, 0, status, &dummy);
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ state rows
    const int c = (warp & 3) * 32 + lane;   // row of S, M, X = TMEM lane
    const int half = warp >> 2;             // columns [64 half, 64 half + 64)
    const uint32_t lb = tmem_lane_base(warp);
    const int tid = threadIdx.x;            // 0..255
    float st[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) st[i] = 0.f;
    {
      uint32_t zr[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) zr[i] = 0u;
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        tmem_st16(tmem + lb + TM_SH + half * 32 + b * 16, zr);
        tmem_st16(tmem + lb + TM_SL + half * 32 + b * 16, zr);
      }
      tmem_st_wait();
      const size_t s0 = (static_cast<size_t>(bh) * N) * kD * kD + static_cast<size_t>(c) * kD + half * 64;
      uint4* g = reinterpret_cast<uint4*>(args.S_hist + s0);
      uint4* gl = reinterpret_cast<uint4*>(args.S_lo_hist + s0);
      const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int i = 0; i < 8; ++i) g[i] = gl[i] = z;
    }
    tc_fence_before();
    mbar_arrive(&bars->s_full);
    // sum over the 256 state threads (every state thread gets the total)
    auto block_sum256 = [&](float v) -> float {
      v = warp_sum(v);
      named_sync(2, 256);  // previous readers of red are done
      if (lane == 0) red[warp] = v;
      named_sync(2, 256);
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) t += red[w];
      return t;
    };
    // S_{j+1} = a S_j + b X with X in TMEM (fp32) or, ns = 0, X = M / den from the slab
    auto state_update = [&](int j, float a, float b, uint32_t xcol, bool from_slab, float inv) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float x[16];
        if (from_slab) {
          ld_f16x4(reinterpret_cast<float*>(slab_f32(args.M_hist, bh * N + j, half, 4 * q, c)), x);
#pragma unroll
          for (int t = 0; t < 16; ++t) x[t] *= inv;
        } else {
          tmem_ld16(tmem + lb + xcol + half * 64 + 16 * q, x);
          tmem_ld_wait();
        }
#pragma unroll
        for (int t = 0; t < 16; ++t) st[16 * q + t] = fmaf(a, st[16 * q + t], b * x[t]);
      }
      tc_fence_before();
#pragma unroll
      for (int q = 0; q < 4; ++q)
        tmem_split16(tmem + lb + TM_SH + half * 32 + q * 8, tmem + lb + TM_SL + half * 32 + q * 8,
                     st + 16 * q);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bars->s_full);
      // history for the backward: S_{j+1} hi through the (now free) X tile
      if (j + 1 < N) {
        if (tid == 0) bulk_wait_read0();   // X tile copies out have read the tile
        named_sync(2, 256);
        // and its bf16 remainder through the X lo tile: the alpha cotangent
        // <Sb_{j+1}, S_j> is a cancelling sum that bf16 S alone moves by ~2e-2
        uint8_t* panel = sm + M_XH + half * P128;
        uint8_t* panel_lo = sm + M_XL + half * P128;
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4) {
          const float* v = st + 8 * q4;
          const uint4 hi4 = pack8(v);
          float lo8[8];
          unpack8(hi4, lo8);
#pragma unroll
          for (int t = 0; t < 8; ++t) lo8[t] = v[t] - lo8[t];
          *reinterpret_cast<uint4*>(panel + sw128_chunk(c, q4)) = hi4;
          *reinterpret_cast<uint4*>(panel_lo + sw128_chunk(c, q4)) = pack8(lo8);
        }
        fence_async_smem();
        named_sync(2, 256);
        if (tid == 0) {
          const int srow = (bh * N + j + 1) * kD;
          tma_store_2d(&tm_sh, 0, srow, sm + M_XH);
          tma_store_2d(&tm_sh, 64, srow, sm + M_XH + P128);
          tma_store_2d(&tm_sl, 0, srow, sm + M_XL);
          tma_store_2d(&tm_sl, 64, srow, sm + M_XL + P128);
          bulk_commit();
        }
      }
    };
    for (int j = 0; j < N; ++j) {
      const float* al = args.alpha + tok0 + j * kC;
      const float* be = args.beta + tok0 + j * kC;
      const float* mu = args.mu + tok0 + j * kC;
      const float a = expf(warp_sum(logf(fmaxf(__ldg(al + lane), kGateFloor)) +
                                    logf(fmaxf(__ldg(al + lane + 32), kGateFloor))));
      const float b = warp_sum(__ldg(be + lane) + __ldg(be + lane + 32)) * (1.f / kC);
      const float mc = expf(warp_sum(logf(fmaxf(__ldg(mu + lane), kGateFloor)) +
                                     logf(fmaxf(__ldg(mu + lane + 32), kGateFloor))));
      if (!wait_use(&bars->g_full, j, status, ab)) break;
      tc_fence_after();
      // the previous S history store has left the X tile
      if (tid == 0) bulk_wait_read0();
      named_sync(2, 256);
      // pass 1: M_{j+1} = mu_c M_j + G_j -> slab, and X_0 := M (hi / lo, unnormalised)
      float sq = 0.f;
      const size_t mj = static_cast<size_t>(bh) * N + j;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float m[16], g[16];
        if (j > 0)
          ld_f16x4(reinterpret_cast<float*>(slab_f32(args.M_hist, mj - 1, half, 4 * q, c)), m);
        else
#pragma unroll
          for (int t = 0; t < 16; ++t) m[t] = 0.f;
        tmem_ld16(tmem + lb + TM_A1 + half * 64 + 16 * q, g);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          m[t] = fmaf(mc, m[t], g[t]);
          sq = fmaf(m[t], m[t], sq);
        }
        st_f16x4(reinterpret_cast<float*>(slab_f32(args.M_hist, mj, half, 4 * q, c)), m);
        st_split8(sm + M_XH, sm + M_XL, c, half * 8 + 2 * q, m);
        st_split8(sm + M_XH, sm + M_XL, c, half * 8 + 2 * q + 1, m + 8);
      }
      const float den = sqrtf(block_sum256(sq)) + kEpsNorm;
      const float inv = 1.f / den;
      if (ns == 0) {
        state_update(j, a, b, 0, true, inv);
        continue;
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->x_ready);
      uint8_t* xslot = args.X_hist + (static_cast<size_t>(bh) * N + j) * ns * 65536u;
      auto store_x = [&](int k) {   // X_k tiles -> history slot k
        named_sync(2, 256);
        if (tid == 0) {
          bulk_store(xslot + k * 65536u, sm + M_XH, 32768u);
          bulk_store(xslot + k * 65536u + 32768u, sm + M_XL, 32768u);
          bulk_commit();
        }
      };
      store_x(0);
      bool ok = true;
      for (int k = 0; k < ns; ++k) {
        const int u = j * ns + k;
        const float gs = k == 0 ? inv * inv : 1.f;   // Gram scale (first step: X_0 = M / den)
        // Gram -> hi / lo tiles (they alias the chunk phase's E^T / w*k / o staging)
        if (!wait_use(&bars->gram_full, u, status, ab)) { ok = false; break; }
        if (k == 0 && !wait_use(&bars->os_free, j, status, ab)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float g[16];
          tmem_ld16(tmem + lb + TM_A1 + half * 64 + 16 * q, g);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 16; ++t) g[t] *= gs;
          st_split8(sm + M_GH, sm + M_GL, c, half * 8 + 2 * q, g);
          st_split8(sm + M_GH, sm + M_GL, c, half * 8 + 2 * q + 1, g + 8);
        }
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(&bars->gram_smem);
        // P' = c0 I + c1 Gram + c2 Gram^2 (first step: times 1/den) -> TMEM (S hi / lo columns)
        if (!wait_use(&bars->g2_full, u, status, ab)) { ok = false; break; }
        tc_fence_after();
        const float ps = k == 0 ? inv : 1.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float g[16], g2[16];
          const int col = half * 64 + 16 * q;
          tmem_ld16(tmem + lb + TM_A1 + col, g);
          tmem_ld16(tmem + lb + TM_A2 + col, g2);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            float v = fmaf(kNsC1, g[t] * gs, kNsC2 * g2[t]);
            if (col + t == c) v += kNsC0;
            g[t] = v * ps;
          }
          tmem_split16(tmem + lb + TM_SH + half * 32 + q * 8, tmem + lb + TM_SL + half * 32 + q * 8, g);
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&bars->p_ready);
        // X' -> hi / lo tiles for the next step, or the state update after the last
        if (!wait_use(&bars->x_full, u, status, ab)) { ok = false; break; }
        tc_fence_after();
        if (k + 1 < ns) {
          if (tid == 0) bulk_wait_read0();   // slot k copy has read the tile
          named_sync(2, 256);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float x[16];
            tmem_ld16(tmem + lb + TM_A2 + half * 64 + 16 * q, x);
            tmem_ld_wait();
            st_split8(sm + M_XH, sm + M_XL, c, half * 8 + 2 * q, x);
            st_split8(sm + M_XH, sm + M_XL, c, half * 8 + 2 * q + 1, x + 8);
          }
          fence_async_smem();
          tc_fence_before();
          mbar_arrive(&bars->x_ready);
          store_x(k + 1);
        } else {
          state_update(j, a, b, TM_A2, false, 1.f);
        }
      }
      if (!ok) break;
    }
    // shared memory must outlive the reads of the bulk stores; grid completion
    // makes their global writes visible to the next kernel
    if (tid == 0) bulk_wait_read0();
  } else {
    // ------------------------------------------------------------ chunk-local (warps 8-11)
    const int tb = threadIdx.x - 256;          // 0..127
    const int sp = warp - 8;                   // TMEM subpartition
    const uint32_t lb = tmem_lane_base(warp);
    const int row = sp * 32 + lane;            // TMEM lane of this thread
    const int t16 = sp * 16 + (lane & 15);     // M=64 row of lanes 0-15
    // w_s = prod_{t>s} clamp(mu_t) (log-space suffix sum), then w * k
    auto build_wk = [&](int j) -> bool {
      if (!wait_use(&bars->ld_full, j, status, ab)) return false;
      if (warp == 8) {
        const float l0 = logf(fmaxf(gate_mu[2 * lane], kGateFloor));
        const float l1 = logf(fmaxf(gate_mu[2 * lane + 1], kGateFloor));
        // inclusive suffix sum over lanes of (l0 + l1)
        float s = l0 + l1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_down_sync(0xffffffffu, s, o);
          if (lane + o < 32) s += y;
        }
        // s = sum over tokens >= 2 lane; w_{2l} = exp(s - l0), w_{2l+1} = exp(s - l0 - l1)
        gate_w[2 * lane] = expf(s - l0);
        gate_w[2 * lane + 1] = expf(s - l0 - l1);
      }
      named_sync(1, 128);
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int id = tb + 128 * m;            // 16-byte chunk id, 0..1023
        const uint32_t off = static_cast<uint32_t>(id) * 16u;
        const float w = gate_w[(id & 511) >> 3];
        const uint4 x = *reinterpret_cast<const uint4*>(sm + M_K + off);
        // w k as bf16 hi + lo: the muon weights are long products of gates,
        // and a single bf16 rounding of w k in G perturbs the state enough to
        // move the mu cotangent (a cancelling sum over the chunk) by ~3e-2
        const uint32_t xs[4] = {x.x, x.y, x.z, x.w};
        uint32_t yh[4], yl[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = bf16_lo(xs[e]) * w, p1 = bf16_hi(xs[e]) * w;
          yh[e] = pack_bf16(p0, p1);
          yl[e] = pack_bf16(p0 - bf16_lo(yh[e]), p1 - bf16_hi(yh[e]));
        }
        *reinterpret_cast<uint4*>(sm + M_WK + off) = make_uint4(yh[0], yh[1], yh[2], yh[3]);
        *reinterpret_cast<uint4*>(sm + M_WKL + off) = make_uint4(yl[0], yl[1], yl[2], yl[3]);
      }
      fence_async_smem();
      mbar_arrive(&bars->wk_full);
      mbar_arrive(&bars->ld_empty);
      return true;
    };
    // P -> A = tril(P) * beta (bf16); A must be free (o2(j-1) done)
    auto build_as = [&](int j) -> bool {
      if (!wait_use(&bars->p_full, j, status, ab)) return false;
      if (j >= 1 && !wait_use(&bars->o_full, j - 1, status, ab)) return false;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < 4; cc += 2) {
        float p0[16], p1[16];
        tmem_ld16(tmem + lb + TM_EP + cc * 16, p0);
        tmem_ld16(tmem + lb + TM_EP + cc * 16 + 16, p1);
        tmem_ld_wait();
        if (lane < 16) {
          float v8[8];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const float* src = h < 2 ? p0 + h * 8 : p1 + (h - 2) * 8;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int sc = cc * 16 + h * 8 + i;
              v8[i] = (sc <= t16) ? src[i] * gate_beta[sc] : 0.f;
            }
            st_row8(sm + M_AS, P64, t16, cc * 2 + h, v8);
          }
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->as_full);
      return true;
    };
    bool ok = N > 0 && build_as(0);
    for (int j = 0; ok && j < N; ++j) {
      // E3: -E^T -> E^T hi / lo (the Gram tiles of chunk j-1 are done: E(j) needed S_j)
      if (!wait_use(&bars->e_full, j, status, ab)) break;
      tc_fence_after();
      {
        float x0[16], x1[16], x2[16], x3[16];
        tmem_ld16(tmem + lb + TM_EP, x0);
        tmem_ld16(tmem + lb + TM_EP + 16, x1);
        tmem_ld16(tmem + lb + TM_EP + 32, x2);
        tmem_ld16(tmem + lb + TM_EP + 48, x3);
        tmem_ld_wait();
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          const float* src = (h < 2 ? x0 : h < 4 ? x1 : h < 6 ? x2 : x3) + (h & 1) * 8;
          float hi[8], lo[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float e = -src[i];
            hi[i] = __bfloat162float(__float2bfloat16_rn(e));
            lo[i] = e - hi[i];
          }
          st_row8(sm + M_EH, P128, row, h, hi);
          st_row8(sm + M_EL, P128, row, h, lo);
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->e_smem);
      if (!build_wk(j)) break;
      // o epilogue: o^T (lanes = value column c) -> staged o[t][c] -> TMA store
      if (!wait_use(&bars->o_full, j, status, ab)) break;
      tc_fence_after();
      named_sync(1, 128);
      {
        uint8_t* os = sm + M_OS + (row >> 6) * P64;
        const int ccol = row & 63;
        float x0[16], x1[16], x2[16], x3[16];
        tmem_ld16(tmem + lb + TM_O, x0);
        tmem_ld16(tmem + lb + TM_O + 16, x1);
        tmem_ld16(tmem + lb + TM_O + 32, x2);
        tmem_ld16(tmem + lb + TM_O + 48, x3);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive(&bars->o_empty);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          *reinterpret_cast<__nv_bfloat16*>(os + sw128_elem(i, ccol)) = __float2bfloat16_rn(x0[i]);
          *reinterpret_cast<__nv_bfloat16*>(os + sw128_elem(16 + i, ccol)) = __float2bfloat16_rn(x1[i]);
          *reinterpret_cast<__nv_bfloat16*>(os + sw128_elem(32 + i, ccol)) = __float2bfloat16_rn(x2[i]);
          *reinterpret_cast<__nv_bfloat16*>(os + sw128_elem(48 + i, ccol)) = __float2bfloat16_rn(x3[i]);
        }
      }
      fence_async_smem();
      named_sync(1, 128);
      if (tb == 0) {
        const int orow = static_cast<int>(tok0) + j * kC;
        tma_store_2d(&tm_o, 0, orow, sm + M_OS);
        if (args.store_hi) tma_store_2d(&tm_o, 64, orow, sm + M_OS + P64);
        bulk_commit();
        bulk_wait_read0();          // the staging tile is free for the Gram tiles
        mbar_arrive(&bars->os_free);
      }
      if (j + 1 < N && !build_as(j + 1)) break;
    }
    // shared memory must outlive the reads of the bulk stores; grid completion
    // makes their global writes visible to the next kernel
    if (tb == 0) bulk_wait_read0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

bool chunk_fwd_muon_tc_supported(const ChunkArgs& p) {
  return p.rule == 1 && (p.dh == kD || p.dh == 64) && p.C == kC && !p.io_f32 && p.N >= 1 &&
         tma_encode_available();
}

cudaError_t chunk_fwd_muon_tc(const ChunkArgs& p, const TcBufs& b, int ns, cudaStream_t st) {
  if (!b.M_hist || (ns > 0 && !b.X_hist)) return cudaErrorInvalidValue;
  if (!b.S_lo_hist) return cudaErrorInvalidValue;
  CUtensorMap mq, mk, mv, mo, msh, msl;
  const uint64_t rows = static_cast<uint64_t>(p.BH) * p.T;
  cudaError_t e;
  if ((e = make_tmap_rows128(&msh, b.S_hist, static_cast<uint64_t>(p.BH) * p.N * kD, 128)) !=
      cudaSuccess)
    return e;
  if ((e = make_tmap_rows128(&msl, b.S_lo_hist, static_cast<uint64_t>(p.BH) * p.N * kD, 128)) !=
      cudaSuccess)
    return e;
  const uint32_t w = static_cast<uint32_t>(p.dh);
  if ((e = make_tmap_rows128(&mq, p.q, rows, 64, w)) != cudaSuccess) return e;
  if ((e = make_tmap_rows128(&mk, p.k, rows, 64, w)) != cudaSuccess) return e;
  if ((e = make_tmap_rows128(&mv, p.v, rows, 64, w)) != cudaSuccess) return e;
  if ((e = make_tmap_rows128(&mo, p.o, rows, 64, w)) != cudaSuccess) return e;
  MuonArgs a{};
  a.store_hi = p.dh == kD;
  a.alpha = p.alpha;
  a.beta = p.beta;
  a.mu = p.mu;
  a.S_hist = b.S_hist;
  a.S_lo_hist = b.S_lo_hist;
  a.M_hist = b.M_hist;
  a.X_hist = b.X_hist;
  a.status = b.status;
  a.N = p.N;
  a.T = p.T;
  a.ns = ns;
  e = cudaFuncSetAttribute(chunk_fwd_tc_muon, cudaFuncAttributeMaxDynamicSharedMemorySize, M_SMEM);
  if (e != cudaSuccess) return e;
  chunk_fwd_tc_muon<<<p.BH, kThreadsM, M_SMEM, st>>>(mq, mk, mv, mo, msh, msl, a);
  return cudaGetLastError();
}

}  // namespace gmdn
