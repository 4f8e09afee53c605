// Reverse chain of the muon mixer core on the tensor cores, dh = 128, C = 64.
//
// One CTA per (b, h) walks the chunks in reverse.  With the state cotangent
// Sb_{j+1} (fp32, registers of the state warps) and the moment cotangent
// Mb_{j+1} (fp32 slab), chunk j takes two phases:
//
// Phase B, the msign VJP (fast_scan.py:107-131, 158-163), for
// Mi = M_{j+1} (the forward's M history) and Y = b_c Sb_{j+1}:
//   for k = ns-1 .. 0, with X_k from the forward's history tiles:
//     G  = X_k X_k^T,  P' = c0 I + c1 G + c2 G^2
//     Ps = Y X_k^T + X_k Y^T
//     Gs = c1 Ps + c2 (Ps G + G Ps)
//     Y <- P' Y + Gs X_k                        (the cotangent of X_k)
//   dM  = Y / den - <Y, Mi> / den^2 * Mi / |Mi|,   den = |Mi| + 1e-7
//   Gb_j = Mb_{j+1} + dM,   Mb_j = mu_c Gb_j
//   da_c = <Sb_{j+1}, S_j>,  db_c = <Sb_{j+1}, X_ns>,  dmu_c = <Gb_j, M_j>
// (X_ns = P'_{ns-1} X_{ns-1} is formed in the first step.)  Every product is
// a split bf16 GEMM (hi.hi + hi.lo + lo.hi, fp32 accumulation).  The stored
// X_0 is M unnormalised; the k = 0 step scales G by 1/den^2, Ps by 1/den and
// Gs by 1/den.
//
// Phase A, the chain step (as the delta kernel, with Gb_j for Sb_{j+1}):
//   dE_j^T = (Gb_j k_j^T + dO_j^T A'_j) diag(w),  A' = A / w (w applied in the drain)
//   Sb_j   = a_c Sb_{j+1} + dO_j^T q_j - dE_j^T k_j
// and Gb_j (bf16) goes to the history for the token-gradient kernel.
//
// Shared memory: three 64 KB split tiles X, Y, Z for phase B; phase A's q,
// k, dO tiles live in Z, its w*k, A and dE^T tiles in X, the Gb history
// staging in Y.  TMEM: R1 (G | chain accumulator C), R2 (G^2 | X_ns | the
// new Y | dE^T and P), R3 (P' | Ps | Gs | Gb as packed bf16 hi / lo A
// operands), R4 (Ps, then Ps c1/c2 + Ps G + G Ps).

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
constexpr int kThreadsMB = 448;
// Token weights w_s = prod_{t>s} mu_t can underflow; A' = A / w and the dE^T
// drain both use max(w, kMuonWFloor) (the error, (w_eff - w) Gb k^T, is below
// 1e-28 |Gb k^T|).
constexpr float kMuonWFloor = 1e-30f;
constexpr uint32_t P64 = 8192;
constexpr uint32_t P128 = 16384;

// shared memory
constexpr uint32_t U_X = 0;          // X_k hi (32 KB), lo (32 KB)
constexpr uint32_t U_Y = 65536;      // Y hi, lo
constexpr uint32_t U_Z = 131072;     // G hi, lo
constexpr uint32_t A_WK = 0;         // phase A, in X: unused (16 KB)
constexpr uint32_t A_AS = 16384;     //                A (8 KB)
constexpr uint32_t A_DEH = 32768;    //                dE^T hi (16 KB)
constexpr uint32_t A_DEL = 49152;    //                dE^T lo (16 KB)
constexpr uint32_t A_SS = 65536;     // phase B end, in Y: Gb hi staging (32 KB), lo (32 KB)
constexpr uint32_t A_Q = 131072;     // phase A, in Z: q, k, dO (16 KB each)
constexpr uint32_t A_K = 147456;
constexpr uint32_t A_G = 163840;
constexpr uint32_t U_GATE = 196608;  // beta[64], mu[64], w[64]
constexpr uint32_t U_RED = 197376;   // [4][8] partial sums
constexpr uint32_t U_BAR = 197632;
constexpr uint32_t U_SMEM = U_BAR + 256 + 1024;

// TMEM
constexpr uint32_t R1 = 0, R2 = 128, R3 = 256, R4 = 384;
constexpr uint32_t R2_E = 128, R2_P = 192;   // phase A: dE^T (128 x 64), P (64 x 64)

struct BarsMB {
  uint64_t ld_full, p_full, as_full, wk_full, de_full, de_smem, c_full, gb_ready;
  uint64_t y_ready, x_loaded, gram_full, gram_smem, g2_full, p_ready, xn_full, xn_done;
  uint64_t ps_full, ps_ready, h_full, gs_ready, xb_full, final_mma;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(BarsMB) <= 256, "barrier block");

struct MuonBwArgs {
  const float *alpha, *beta, *mu;
  const uint16_t* S_hist;
  const uint16_t* S_lo_hist;
  const float* M_hist;
  const uint8_t* X_hist;
  float* Mb_ws;
  float *dac, *dbc, *dmc, *dnc;
  uint32_t* status;
  int N, T, ns;
};

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

__device__ __forceinline__ void tmem_st16f(uint32_t taddr, const float* x) {
  uint32_t r[16];
#pragma unroll
  for (int t = 0; t < 16; ++t) r[t] = __float_as_uint(x[t]);
  tmem_st16(taddr, r);
}

__global__ void __launch_bounds__(kThreadsMB, 1)
chunk_bwd1_tc_muon(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_g, const __grid_constant__ CUtensorMap tm_gb,
                   const __grid_constant__ CUtensorMap tm_gbl, MuonBwArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  BarsMB* bars = reinterpret_cast<BarsMB*>(sm + U_BAR);
  float* gate_beta = reinterpret_cast<float*>(sm + U_GATE);
  float* gate_mu = gate_beta + 64;
  float* gate_w = gate_beta + 128;
  float* red = reinterpret_cast<float*>(sm + U_RED);
  volatile int* ab = &bars->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int N = args.N, ns = args.ns;
  uint32_t* status = args.status;

  if (threadIdx.x == 0) {
    uint64_t* b = &bars->ld_full;
    const int counts[22] = {1, 1, 128, 128, 1, 128, 1, 256, 256, 1, 1, 256, 1, 256, 1, 256,
                            1, 256, 1, 256, 1, 1};
    for (int i = 0; i < 22; ++i) mbar_init(b + i, counts[i]);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 13) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const size_t tok0 = static_cast<size_t>(bh) * args.T;

  if (warp == 12) {
    // ------------------------------------------------------------ TMA: phase A tiles, reverse order
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < N; ++i) {
        const int j = N - 1 - i;
        const int row = static_cast<int>(tok0) + j * kC;
        // Z (and the gate area) are free once phase B of this chunk is done
        if (!wait_use(&bars->gb_ready, i, status, ab)) break;
        mbar_expect_tx(&bars->ld_full, 6 * 8192 + 512);
        tma_load_2d(sm + A_Q, &tm_q, 0, row, &bars->ld_full);
        tma_load_2d(sm + A_Q + P64, &tm_q, 64, row, &bars->ld_full);
        tma_load_2d(sm + A_K, &tm_k, 0, row, &bars->ld_full);
        tma_load_2d(sm + A_K + P64, &tm_k, 64, row, &bars->ld_full);
        tma_load_2d(sm + A_G, &tm_g, 0, row, &bars->ld_full);
        tma_load_2d(sm + A_G + P64, &tm_g, 64, row, &bars->ld_full);
        bulk_load(gate_beta, args.beta + tok0 + j * kC, 256, &bars->ld_full);
        bulk_load(gate_mu, args.mu + tok0 + j * kC, 256, &bars->ld_full);
        issued = i + 1;
      }
      int dummy = 0;
      if (issued >= 1) mbar_wait(&bars->ld_full, (issued - 1) & 1, status, &dummy);
    }
  } else if (warp == 13) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      const uint32_t x_h = smem_u32(sm + U_X), x_l = x_h + 32768;
      const uint32_t y_h = smem_u32(sm + U_Y), y_l = y_h + 32768;
      const uint32_t z_h = smem_u32(sm + U_Z), z_l = z_h + 32768;
      const uint32_t q_s = smem_u32(sm + A_Q), k_s = smem_u32(sm + A_K), g_s = smem_u32(sm + A_G);
      const uint32_t as_s = smem_u32(sm + A_AS);
      const uint32_t deh_s = smem_u32(sm + A_DEH), del_s = smem_u32(sm + A_DEL);
      constexpr uint32_t ID_KK = idesc_bf16(128, 128, false, false);
      constexpr uint32_t ID_KM = idesc_bf16(128, 128, false, true);
      constexpr uint32_t ID_P = idesc_bf16(64, 64, false, false);
      constexpr uint32_t ID_Z = idesc_bf16(128, 128, true, true);
      constexpr uint32_t ID_X = idesc_bf16(128, 64, true, true);
      constexpr uint32_t ID_Y = idesc_bf16(128, 64, false, false);
      constexpr uint32_t ID_W = idesc_bf16(128, 128, false, true, true);
      // D (+)= A B^T, split K-major 128 x 128 tiles
      auto mm_kk = [&](uint32_t d, uint32_t ah, uint32_t al, uint32_t bh_, uint32_t bl, bool acc) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(d, desc_kmajor(ah, P128, k), desc_kmajor(bh_, P128, k), ID_KK, (acc || k > 0) ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(d, desc_kmajor(ah, P128, k), desc_kmajor(bl, P128, k), ID_KK, 1);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(d, desc_kmajor(al, P128, k), desc_kmajor(bh_, P128, k), ID_KK, 1);
      };
      // D (+)= A B with A split in TMEM (hi at a, lo at a + 64) and B split MN-major
      auto mm_tm = [&](uint32_t d, uint32_t a, uint32_t bh_, uint32_t bl, bool acc) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(d, a + k * 8, desc_mnmajor(bh_, P128, k), ID_KM, (acc || k > 0) ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(d, a + k * 8, desc_mnmajor(bl, P128, k), ID_KM, 1);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(d, a + 64 + k * 8, desc_mnmajor(bh_, P128, k), ID_KM, 1);
      };
      // D (+)= A B^T with A split in TMEM and B split K-major
      auto mm_tk = [&](uint32_t d, uint32_t a, uint32_t bh_, uint32_t bl, bool acc) {
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(d, a + k * 8, desc_kmajor(bh_, P128, k), ID_KK, (acc || k > 0) ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(d, a + k * 8, desc_kmajor(bl, P128, k), ID_KK, 1);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(d, a + 64 + k * 8, desc_kmajor(bh_, P128, k), ID_KK, 1);
      };
      bool ok = true;
      for (int i = 0; ok && i < N; ++i) {
        // ---- phase B
        for (int kk = 0; kk < ns; ++kk) {
          const int u = i * ns + kk;
          if (!wait_use(&bars->x_loaded, u, status, ab) || !wait_use(&bars->y_ready, u, status, ab)) {
            ok = false;
            break;
          }
          tc_fence_after();
          mm_kk(tmem + R1, x_h, x_l, x_h, x_l, false);            // G = X X^T
          mma_commit(&bars->gram_full);
          if (!wait_use(&bars->gram_smem, u, status, ab)) { ok = false; break; }
          tc_fence_after();
          mm_kk(tmem + R2, z_h, z_l, z_h, z_l, false);            // G^2
          mma_commit(&bars->g2_full);
          if (!wait_use(&bars->p_ready, u, status, ab)) { ok = false; break; }
          tc_fence_after();
          if (kk == 0) {                                          // X_ns = P' X_{ns-1}
            mm_tm(tmem + R2, tmem + R3, x_h, x_l, false);
            mma_commit(&bars->xn_full);
            if (!wait_use(&bars->xn_done, i, status, ab)) { ok = false; break; }
            tc_fence_after();
          }
          mm_tm(tmem + R2, tmem + R3, y_h, y_l, false);           // P' Y
          mm_kk(tmem + R4, y_h, y_l, x_h, x_l, false);            // Ps = Y X^T
          mm_kk(tmem + R4, x_h, x_l, y_h, y_l, true);             //    + X Y^T
          mma_commit(&bars->ps_full);
          if (!wait_use(&bars->ps_ready, u, status, ab)) { ok = false; break; }
          tc_fence_after();
          mm_tk(tmem + R4, tmem + R3, z_h, z_l, true);            // += Ps G
          mm_kk(tmem + R4, z_h, z_l, y_h, y_l, true);             // += G Ps
          mma_commit(&bars->h_full);
          if (!wait_use(&bars->gs_ready, u, status, ab)) { ok = false; break; }
          tc_fence_after();
          mm_tm(tmem + R2, tmem + R3, x_h, x_l, true);            // += Gs X
          mma_commit(&bars->xb_full);
        }
        if (!ok) break;
        // ---- phase A
        if (!wait_use(&bars->ld_full, i, status, ab)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(tmem + R2_P, desc_kmajor(q_s, P64, k), desc_kmajor(k_s, P64, k), ID_P, k > 0);
        mma_commit(&bars->p_full);
        if (!wait_use(&bars->gb_ready, i, status, ab)) break;
        if (!wait_use(&bars->wk_full, i, status, ab)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(tmem + R2_E, tmem + R3 + k * 8, desc_kmajor(k_s, P64, k), ID_Y, k > 0);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(tmem + R2_E, tmem + R3 + 64 + k * 8, desc_kmajor(k_s, P64, k), ID_Y, 1);
        if (!wait_use(&bars->as_full, i, status, ab)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + R2_E, desc_mnmajor(g_s, P64, k), desc_mnmajor(as_s, P64, k), ID_X, 1);
        mma_commit(&bars->de_full);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + R1, desc_mnmajor(g_s, P64, k), desc_mnmajor(q_s, P64, k), ID_Z, k > 0);
        if (!wait_use(&bars->de_smem, i, status, ab)) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + R1, desc_kmajor(deh_s, P128, k), desc_mnmajor(k_s, P64, k), ID_W, 1);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + R1, desc_kmajor(del_s, P128, k), desc_mnmajor(k_s, P64, k), ID_W, 1);
        mma_commit(&bars->c_full);
      }
      mma_commit(&bars->final_mma);
      int dummy = 0;
      mbar_wait(&bars->final_mma, 0, status, &dummy);
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ state warps
    const int c = (warp & 3) * 32 + lane;
    const int half = warp >> 2;
    const uint32_t lb = tmem_lane_base(warp);
    const int tid = threadIdx.x;
    float sb[64];
#pragma unroll
    for (int t = 0; t < 64; ++t) sb[t] = 0.f;
    // sum over the 256 state threads, up to four values at once
    auto block_sum4 = [&](float* v, int n) {
#pragma unroll
      for (int x = 0; x < 4; ++x)
        if (x < n) v[x] = warp_sum(v[x]);
      named_sync(2, 256);
      if (lane == 0)
        for (int x = 0; x < n; ++x) red[x * 8 + warp] = v[x];
      named_sync(2, 256);
      for (int x = 0; x < n; ++x) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) t += red[x * 8 + w];
        v[x] = t;
      }
    };
    uint64_t* xl_bar = &bars->x_loaded;
    auto load_x = [&](int j, int k) {   // X_k tiles of chunk j -> X (tid 0)
      const uint8_t* src = args.X_hist + ((static_cast<size_t>(bh) * N + j) * ns + k) * 65536u;
      mbar_expect_tx(xl_bar, 65536u);
      bulk_load(sm + U_X, src, 32768u, xl_bar);
      bulk_load(sm + U_X + 32768u, src + 32768u, 32768u, xl_bar);
    };
    bool ok = true;
    for (int i = 0; ok && i < N; ++i) {
      const int j = N - 1 - i;
      const size_t mj = static_cast<size_t>(bh) * N + j;
      const float* be = args.beta + tok0 + j * kC;
      const float* mu = args.mu + tok0 + j * kC;
      const float* al = args.alpha + tok0 + j * kC;
      const float b = warp_sum(__ldg(be + lane) + __ldg(be + lane + 32)) * (1.f / kC);
      const float mc = expf(warp_sum(logf(fmaxf(__ldg(mu + lane), kGateFloor)) +
                                     logf(fmaxf(__ldg(mu + lane + 32), kGateFloor))));
      const float a = expf(warp_sum(logf(fmaxf(__ldg(al + lane), kGateFloor)) +
                                    logf(fmaxf(__ldg(al + lane + 32), kGateFloor))));
      // ================= phase B
      // previous Gb staging store has left Y; phase A of chunk j+1 is done with X (c_full)
      if (tid == 0) bulk_wait_read0();
      named_sync(2, 256);
      if (tid == 0 && ns > 0) load_x(j, ns - 1);
      // |Mi|, da = <Sb, S_j>, and Y = b Sb -> split tiles
      float red4[4] = {0.f, 0.f, 0.f, 0.f};   // |Mi|^2, da
      {
        const float* mi = args.M_hist;
        const uint4* srow = reinterpret_cast<const uint4*>(args.S_hist + (mj * kD + c) * kD + half * 64);
        const uint4* slrow =
            reinterpret_cast<const uint4*>(args.S_lo_hist + (mj * kD + c) * kD + half * 64);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float m[16], s8[16], sl8[16];
          ld_f16x4(reinterpret_cast<const float*>(slab_f32(const_cast<float*>(mi), static_cast<int>(mj), half, 4 * q, c)), m);
          unpack8(srow[2 * q], s8);
          unpack8(srow[2 * q + 1], s8 + 8);
          unpack8(slrow[2 * q], sl8);
          unpack8(slrow[2 * q + 1], sl8 + 8);
#pragma unroll
          for (int t = 0; t < 16; ++t) s8[t] += sl8[t];   // S_j to ~16 bits
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            red4[0] = fmaf(m[t], m[t], red4[0]);
            red4[1] = fmaf(sb[16 * q + t], s8[t], red4[1]);
          }
          if (ns > 0) {
            float y[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) y[t] = b * sb[16 * q + t];
            st_split8(sm + U_Y, sm + U_Y + 32768, c, half * 8 + 2 * q, y);
            st_split8(sm + U_Y, sm + U_Y + 32768, c, half * 8 + 2 * q + 1, y + 8);
          }
        }
      }
      block_sum4(red4, 2);
      const float fro = sqrtf(red4[0]);
      const float den = fro + kEpsNorm;
      const float inv = 1.f / den;
      const float dsum = red4[1];
      float db_sum = 0.f;
      if (ns > 0) {
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(&bars->y_ready);
      }
      for (int kk = 0; kk < ns; ++kk) {
        const int k = ns - 1 - kk;
        const int u = i * ns + kk;
        const float xs = k == 0 ? inv : 1.f;   // the stored X_0 is M unnormalised
        // G -> split Z tiles
        if (!wait_use(&bars->gram_full, u, status, ab)) { ok = false; break; }
        tc_fence_after();
        const float gs = xs * xs;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float g[16];
          tmem_ld16(tmem + lb + R1 + half * 64 + 16 * q, g);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 16; ++t) g[t] *= gs;
          st_split8(sm + U_Z, sm + U_Z + 32768, c, half * 8 + 2 * q, g);
          st_split8(sm + U_Z, sm + U_Z + 32768, c, half * 8 + 2 * q + 1, g + 8);
        }
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(&bars->gram_smem);
        // P' -> R3
        if (!wait_use(&bars->g2_full, u, status, ab)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float g[16], g2[16];
          const int col = half * 64 + 16 * q;
          tmem_ld16(tmem + lb + R1 + col, g);
          tmem_ld16(tmem + lb + R2 + col, g2);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            float v = fmaf(kNsC1, g[t] * gs, kNsC2 * g2[t]);
            if (col + t == c) v += kNsC0;
            g[t] = v;
          }
          tmem_split16(tmem + lb + R3 + half * 32 + q * 8, tmem + lb + R3 + 64 + half * 32 + q * 8, g);
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&bars->p_ready);
        if (kk == 0) {   // db = <Sb, X_ns>
          if (!wait_use(&bars->xn_full, i, status, ab)) { ok = false; break; }
          tc_fence_after();
          float part = 0.f;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float x[16];
            tmem_ld16(tmem + lb + R2 + half * 64 + 16 * q, x);
            tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < 16; ++t) part = fmaf(sb[16 * q + t], x[t] * xs, part);
          }
          db_sum = part;
          tc_fence_before();
          mbar_arrive(&bars->xn_done);
        }
        // Ps -> R3 (A operand), Y tiles (B operand), R4 <- (c1 / c2) Ps
        if (!wait_use(&bars->ps_full, u, status, ab)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float p[16];
          const int col = half * 64 + 16 * q;
          tmem_ld16(tmem + lb + R4 + col, p);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 16; ++t) p[t] *= xs;
          tmem_split16(tmem + lb + R3 + half * 32 + q * 8, tmem + lb + R3 + 64 + half * 32 + q * 8, p);
          st_split8(sm + U_Y, sm + U_Y + 32768, c, half * 8 + 2 * q, p);
          st_split8(sm + U_Y, sm + U_Y + 32768, c, half * 8 + 2 * q + 1, p + 8);
#pragma unroll
          for (int t = 0; t < 16; ++t) p[t] *= kNsC1 / kNsC2;
          tmem_st16f(tmem + lb + R4 + col, p);
        }
        tmem_st_wait();
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(&bars->ps_ready);
        // Gs = c2 R4 (k = 0: / den) -> R3
        if (!wait_use(&bars->h_full, u, status, ab)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float h[16];
          tmem_ld16(tmem + lb + R4 + half * 64 + 16 * q, h);
          tmem_ld_wait();
#pragma unroll
          for (int t = 0; t < 16; ++t) h[t] *= kNsC2 * xs;
          tmem_split16(tmem + lb + R3 + half * 32 + q * 8, tmem + lb + R3 + 64 + half * 32 + q * 8, h);
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&bars->gs_ready);
        // the new Y (cotangent of X_k)
        if (!wait_use(&bars->xb_full, u, status, ab)) { ok = false; break; }
        tc_fence_after();
        if (k > 0) {
          if (tid == 0) load_x(j, k - 1);   // X is free: its last reader (Gs X) is done
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float y[16];
            tmem_ld16(tmem + lb + R2 + half * 64 + 16 * q, y);
            tmem_ld_wait();
            st_split8(sm + U_Y, sm + U_Y + 32768, c, half * 8 + 2 * q, y);
            st_split8(sm + U_Y, sm + U_Y + 32768, c, half * 8 + 2 * q + 1, y + 8);
          }
          fence_async_smem();
          tc_fence_before();
          mbar_arrive(&bars->y_ready);
        }
      }
      if (!ok) break;
      // ---- msign VJP finish: dM = Y / den - <Y, Mi> / den^2 * Mi / |Mi|
      // (ns = 0: X = M / den, Y = b Sb, db = <Sb, M> / den)
      auto ybar = [&](int q, float (&y)[16]) {
        if (ns > 0) {
          tmem_ld16(tmem + lb + R2 + half * 64 + 16 * q, y);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int t = 0; t < 16; ++t) y[t] = b * sb[16 * q + t];
        }
      };
      float r3[4] = {0.f, 0.f, 0.f, 0.f};   // inner, db (ns = 0)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float y[16], m[16];
        ybar(q, y);
        ld_f16x4(reinterpret_cast<const float*>(slab_f32(const_cast<float*>(args.M_hist), static_cast<int>(mj), half, 4 * q, c)), m);
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          r3[0] = fmaf(y[t], m[t], r3[0]);
          if (ns == 0) r3[1] = fmaf(sb[16 * q + t], m[t] * inv, r3[1]);
        }
      }
      if (ns == 0) db_sum = r3[1];
      r3[1] = db_sum;
      block_sum4(r3, 2);
      const float inner = r3[0];
      const float dbsum = r3[1];
      const float cm = inner * inv * inv / fmaxf(fro, 1e-12f);
      float dm_part = 0.f;
      // Gb = Mb + dM -> R3 (A operand of phase A), staging (history), Mb <- mu_c Gb
      uint8_t* stage = sm + A_SS + half * P128;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float y[16], m[16], gb[16];
        ybar(q, y);
        ld_f16x4(reinterpret_cast<const float*>(slab_f32(const_cast<float*>(args.M_hist), static_cast<int>(mj), half, 4 * q, c)), m);
        float* mbp = reinterpret_cast<float*>(slab_f32(args.Mb_ws, bh, half, 4 * q, c));
        if (j + 1 < N) ld_f16x4(mbp, gb);
        else
#pragma unroll
          for (int t = 0; t < 16; ++t) gb[t] = 0.f;
#pragma unroll
        for (int t = 0; t < 16; ++t) gb[t] += y[t] * inv - cm * m[t];
        if (j > 0) {
          float mp[16];
          ld_f16x4(reinterpret_cast<const float*>(slab_f32(const_cast<float*>(args.M_hist), static_cast<int>(mj - 1), half, 4 * q, c)), mp);
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            dm_part = fmaf(gb[t], mp[t], dm_part);
            mp[t] = mc * gb[t];
          }
          st_f16x4(mbp, mp);
        }
        tmem_split16(tmem + lb + R3 + half * 32 + q * 8, tmem + lb + R3 + 64 + half * 32 + q * 8, gb);
#pragma unroll
        for (int h8 = 0; h8 < 2; ++h8) {
          const uint4 hi4 = pack8(gb + 8 * h8);
          float lo8[8];
          unpack8(hi4, lo8);
#pragma unroll
          for (int t = 0; t < 8; ++t) lo8[t] = gb[8 * h8 + t] - lo8[t];
          *reinterpret_cast<uint4*>(stage + sw128_chunk(c, 2 * q + h8)) = hi4;
          *reinterpret_cast<uint4*>(stage + 32768 + sw128_chunk(c, 2 * q + h8)) = pack8(lo8);
        }
      }
      tmem_st_wait();
      fence_async_smem();
      float r1[4] = {dm_part, 0.f, 0.f, 0.f};
      block_sum4(r1, 1);
      if (tid == 0) {
        const int hrow = (bh * N + j) * kD;
        tma_store_2d(&tm_gb, 0, hrow, sm + A_SS);
        tma_store_2d(&tm_gb, 64, hrow, sm + A_SS + P128);
        tma_store_2d(&tm_gbl, 0, hrow, sm + A_SS + 32768);
        tma_store_2d(&tm_gbl, 64, hrow, sm + A_SS + 32768 + P128);
        bulk_commit();
        args.dac[mj] = dsum;
        args.dbc[mj] = dbsum;
        args.dmc[mj] = r1[0];
        args.dnc[mj] = 0.f;
      }
      tc_fence_before();
      fence_async_smem();   // tile and gate reads before the next loads (async proxy)
      mbar_arrive(&bars->gb_ready);
      // ================= phase A: Sb_j = a_c Sb_{j+1} + C
      if (!wait_use(&bars->c_full, i, status, ab)) break;
      tc_fence_after();
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float cc[16];
        tmem_ld16(tmem + lb + R1 + half * 64 + 16 * q, cc);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 16; ++t) sb[16 * q + t] = fmaf(a, sb[16 * q + t], cc[t]);
      }
      tc_fence_before();
    }
    // shared memory must outlive the reads of the bulk stores; grid completion
    // makes their global writes visible to the next kernel
    if (tid == 0) bulk_wait_read0();
  } else {
    // ------------------------------------------------------------ chunk-local (warps 8-11)
    const int tb = threadIdx.x - 256;
    const int sp = warp - 8;
    const uint32_t lb = tmem_lane_base(warp);
    const int row = sp * 32 + lane;
    const int t16 = sp * 16 + (lane & 15);
    for (int i = 0; i < N; ++i) {
      // w * k (w_s = prod_{t>s} mu_t); X is free once phase B of this chunk is done
      if (!wait_use(&bars->ld_full, i, status, ab)) break;
      if (!wait_use(&bars->gb_ready, i, status, ab)) break;
      if (warp == 8) {
        const float l0 = logf(fmaxf(gate_mu[2 * lane], kGateFloor));
        const float l1 = logf(fmaxf(gate_mu[2 * lane + 1], kGateFloor));
        float s = l0 + l1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_down_sync(0xffffffffu, s, o);
          if (lane + o < 32) s += y;
        }
        gate_w[2 * lane] = expf(s - l0);
        gate_w[2 * lane + 1] = expf(s - l0 - l1);
      }
      named_sync(1, 128);
      // w is applied to the columns of dE^T in its drain (dE^T = (Gb k^T +
      // dO^T A') diag(w), A' = A / w) instead of being multiplied into k: w k
      // rounded to bf16 would break the cancellation in Gb (w k)^T against the
      // forward's G, whose w k keeps ~16 bits
      mbar_arrive(&bars->wk_full);
      // A = tril(P) * beta
      if (!wait_use(&bars->p_full, i, status, ab)) break;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < 4; cc += 2) {
        float p0[16], p1[16];
        tmem_ld16(tmem + lb + R2_P + cc * 16, p0);
        tmem_ld16(tmem + lb + R2_P + cc * 16 + 16, p1);
        tmem_ld_wait();
        if (lane < 16) {
          float v8[8];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const float* src = h < 2 ? p0 + h * 8 : p1 + (h - 2) * 8;
#pragma unroll
            for (int x = 0; x < 8; ++x) {
              const int sc = cc * 16 + h * 8 + x;
              // SFU reciprocal: A' goes to bf16, and IEEE divisions here held
              // up the chain's X product (tc.cuh)
              v8[x] = (sc <= t16)
                          ? src[x] * gate_beta[sc] * rcp_sfu(fmaxf(gate_w[sc], kMuonWFloor))
                          : 0.f;
            }
            st_row8(sm + A_AS, P64, t16, cc * 2 + h, v8);
          }
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->as_full);
      // dE^T -> hi / lo
      if (!wait_use(&bars->de_full, i, status, ab)) break;
      tc_fence_after();
      {
        float x0[16], x1[16], x2[16], x3[16];
        tmem_ld16(tmem + lb + R2_E, x0);
        tmem_ld16(tmem + lb + R2_E + 16, x1);
        tmem_ld16(tmem + lb + R2_E + 32, x2);
        tmem_ld16(tmem + lb + R2_E + 48, x3);
        tmem_ld_wait();
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          const float* src = (h < 2 ? x0 : h < 4 ? x1 : h < 6 ? x2 : x3) + (h & 1) * 8;
          float hi[8], lo[8];
#pragma unroll
          for (int x = 0; x < 8; ++x) {
            const float d = src[x] * fmaxf(gate_w[h * 8 + x], kMuonWFloor);
            hi[x] = __bfloat162float(__float2bfloat16_rn(d));
            lo[x] = d - hi[x];
          }
          st_row8(sm + A_DEH, P128, row, h, hi);
          st_row8(sm + A_DEL, P128, row, h, lo);
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->de_smem);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

cudaError_t chunk_bwd1_muon_tc(const ChunkArgs& p, const TcBufs& b, int ns, cudaStream_t st) {
  if (!b.M_hist || (ns > 0 && !b.X_hist) || !b.M_ws || !b.dac || !b.dbc || !b.dmc || !b.dnc ||
      !b.Gbar_lo_hist || !b.S_lo_hist)
    return cudaErrorInvalidValue;
  CUtensorMap mq, mk, mg, mgb, mgbl;
  const uint64_t rows = static_cast<uint64_t>(p.BH) * p.T;
  cudaError_t e;
  const uint32_t w = static_cast<uint32_t>(p.dh);
  if ((e = make_tmap_rows128(&mq, p.q, rows, 64, w)) != cudaSuccess) return e;
  if ((e = make_tmap_rows128(&mk, p.k, rows, 64, w)) != cudaSuccess) return e;
  if ((e = make_tmap_rows128(&mg, p.dO, rows, 64, w)) != cudaSuccess) return e;
  if ((e = make_tmap_rows128(&mgb, b.Gbar_hist, static_cast<uint64_t>(p.BH) * p.N * kD, 128)) !=
      cudaSuccess)
    return e;
  if ((e = make_tmap_rows128(&mgbl, b.Gbar_lo_hist, static_cast<uint64_t>(p.BH) * p.N * kD, 128)) !=
      cudaSuccess)
    return e;
  MuonBwArgs a{};
  a.alpha = p.alpha;
  a.beta = p.beta;
  a.mu = p.mu;
  a.S_hist = b.S_hist;
  a.S_lo_hist = b.S_lo_hist;
  a.M_hist = b.M_hist;
  a.X_hist = b.X_hist;
  a.Mb_ws = b.M_ws;
  a.dac = b.dac;
  a.dbc = b.dbc;
  a.dmc = b.dmc;
  a.dnc = b.dnc;
  a.status = b.status;
  a.N = p.N;
  a.T = p.T;
  a.ns = ns;
  e = cudaFuncSetAttribute(chunk_bwd1_tc_muon, cudaFuncAttributeMaxDynamicSharedMemorySize, U_SMEM);
  if (e != cudaSuccess) return e;
  chunk_bwd1_tc_muon<<<p.BH, kThreadsMB, U_SMEM, st>>>(mq, mk, mg, mgb, mgbl, a);
  return cudaGetLastError();
}

}  // namespace gmdn
