// Fused tensor-core forward of the mixer core, delta rule, dh = 128, C = 64.
//
// One CTA per (batch, head) walks the N chunks in order.  Per chunk j
// (train_ablation.py:142-187 with the scan of fast_scan.py:72-95):
//
//   A(j)  Kw_j = k^T (w k)      M128 N128 K64   -> TMEM RK
//         Uv_j = v^T (w k)      M128 N128 K64   -> TMEM RU[j%2]
//         P_j  = q k^T          M64  N64  K128  -> TMEM RX, lanes 0-15
//   B(j)  Qt_j = I q - A_j k    M64  N128 K64   -> TMEM RX, lanes 0-15
//         (A_j = tril(P_j) * beta_col, bf16 in shared memory)
//   C(j)  G_j = Uv_j - S_j Kw_j (S_j = hi + lo, two bf16 passes) -> RU[j%2]
//   D(j)  o_j = Qt_j S_j^T + A_j v_j   M64 N128 -> TMEM RX, lanes 16-31
//   state S_{j+1} = a_j S_j + G_j  (fp32, in registers of warps 0-3)
//
// The MMA thread issues C(j), D(j), A(j+1), B(j+1) per step, so the next
// chunk's loads and products overlap the sequential state update.
//
// Warp roles (320 threads): warps 0-3 own the fp32 state (one row of S per
// thread), run the sequential update and store o; warps 4-7 drain the
// chunk-local accumulators (Kw, P -> A, Qt) and build w*k; warp 8 issues TMA
// loads; warp 9 allocates TMEM and issues every MMA from one thread.  All
// hand-offs are mbarriers; every wait is bounded (tc.cuh) and a timeout sets
// the status word and unwinds all roles.
//
// Bytes per chunk-head: q, k, v in (48 KB), o out (16 KB), S_j bf16 out for
// the backward (32 KB).  Tensor work per chunk-head: 2*2*C*d^2 (Kw, Uv) +
// 2*C^2*d (P) + 2*C^2*d (Qt) + 2*2*d^3 (state, hi+lo) + 2*(C*d^2 + C^2*d) (o).

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
constexpr int kThreadsTc = 320;

// shared-memory map (bytes from a 1024-aligned base)
constexpr uint32_t OFF_Q = 0;             // q_j: 2 panels x 64 rows
constexpr uint32_t OFF_K = 16384;         // k: 2 stages x 16 KB
constexpr uint32_t OFF_V = 49152;         // v: 2 stages x 16 KB
constexpr uint32_t OFF_WK = 81920;        // w * k_j
constexpr uint32_t OFF_AS = 98304;        // A_j bf16, 1 panel x 64 rows
constexpr uint32_t OFF_QT = 106496;       // Qt_j bf16, 2 panels x 64 rows
constexpr uint32_t OFF_I = 122880;        // 64 x 64 identity
constexpr uint32_t OFF_SH = 131072;       // S_j hi, 2 panels x 128 rows
constexpr uint32_t OFF_SL = 163840;       // S_j lo
constexpr uint32_t OFF_KW = 196608;       // Kw_j bf16, 2 panels x 128 rows
constexpr uint32_t OFF_GATE = 229376;     // beta: 2 stages x 64 floats
constexpr uint32_t OFF_BAR = 229888;      // mbarriers and flags
constexpr uint32_t SMEM_BYTES = OFF_BAR + 256 + 1024;

constexpr uint32_t P64 = 8192;    // panel stride of a 64-row tile
constexpr uint32_t P128 = 16384;  // panel stride of a 128-row tile

// TMEM columns.  RX holds two M=64 accumulators side by side: lanes 0-15 of
// every subpartition for P / Qt, lanes 16-31 for o.
constexpr uint32_t TM_U0 = 0, TM_U1 = 128, TM_K = 256, TM_X = 384;
constexpr uint32_t TM_HI16 = 16u << 16;  // lane offset of the upper half

struct Bars {
  uint64_t q_full, q_empty;
  uint64_t kv_full[2], kv_empty[2];
  uint64_t wk_full, wk_empty;
  uint64_t kwp_full, kw_smem;
  uint64_t as_full, qt_full, qt_smem;
  uint64_t g_full[2], g_empty[2];
  uint64_t s_full, o_full, o_empty;
  uint64_t final_mma;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Bars) <= 256, "barrier block");

struct FwdArgs {
  const float* beta;
  const float* alpha;
  uint16_t* o;
  uint16_t* S_hist;
  uint32_t* status;
  int N, T;
};

__device__ __forceinline__ bool wait_full(uint64_t* b, int use, uint32_t* st, Bars* B) {
  return mbar_wait(b, static_cast<uint32_t>(use) & 1u, st, &B->abort_flag);
}
__device__ __forceinline__ bool wait_empty(uint64_t* b, int use, uint32_t* st, Bars* B) {
  return mbar_wait(b, (static_cast<uint32_t>(use) & 1u) ^ 1u, st, &B->abort_flag);
}

__global__ void __launch_bounds__(kThreadsTc, 1)
chunk_fwd_tc_delta(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, FwdArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  Bars* bars = reinterpret_cast<Bars*>(sm + OFF_BAR);
  float* gate_beta = reinterpret_cast<float*>(sm + OFF_GATE);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int N = args.N;
  uint32_t* status = args.status;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_empty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1 + 128);
      mbar_init(&bars->g_full[s], 1);
      mbar_init(&bars->g_empty[s], 128);
    }
    mbar_init(&bars->wk_full, 128);
    mbar_init(&bars->wk_empty, 1);
    mbar_init(&bars->kwp_full, 1);
    mbar_init(&bars->kw_smem, 128);
    mbar_init(&bars->as_full, 128);
    mbar_init(&bars->qt_full, 1);
    mbar_init(&bars->qt_smem, 128);
    mbar_init(&bars->s_full, 128);
    mbar_init(&bars->o_full, 1);
    mbar_init(&bars->o_empty, 128);
    mbar_init(&bars->final_mma, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  build_identity64(sm + OFF_I, threadIdx.x, kThreadsTc);
  if (warp == 9) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const size_t tok0 = static_cast<size_t>(bh) * args.T;

  if (warp == 8) {
    // ------------------------------------------------------------ TMA
    if (lane == 0) {
      int kv_issued = 0, q_issued = 0;
      for (int j = 0; j < N; ++j) {
        const int s = j & 1;
        const int row = static_cast<int>(tok0) + j * kC;
        if (!wait_empty(&bars->kv_empty[s], j >> 1, status, bars)) break;
        mbar_expect_tx(&bars->kv_full[s], 4 * 8192 + 256);
        tma_load_2d(sm + OFF_K + s * 16384, &tm_k, 0, row, &bars->kv_full[s]);
        tma_load_2d(sm + OFF_K + s * 16384 + P64, &tm_k, 64, row, &bars->kv_full[s]);
        tma_load_2d(sm + OFF_V + s * 16384, &tm_v, 0, row, &bars->kv_full[s]);
        tma_load_2d(sm + OFF_V + s * 16384 + P64, &tm_v, 64, row, &bars->kv_full[s]);
        bulk_load(gate_beta + s * 64, args.beta + tok0 + j * kC, 256, &bars->kv_full[s]);
        kv_issued = j + 1;
        if (!wait_empty(&bars->q_empty, j, status, bars)) break;
        mbar_expect_tx(&bars->q_full, 2 * 8192);
        tma_load_2d(sm + OFF_Q, &tm_q, 0, row, &bars->q_full);
        tma_load_2d(sm + OFF_Q + P64, &tm_q, 64, row, &bars->q_full);
        q_issued = j + 1;
      }
      // Never leave with copies in flight (matters only after an abort).
      int dummy = 0;
      for (int j = kv_issued - 2; j < kv_issued; ++j) {
        if (j < 0) continue;
        mbar_wait(&bars->kv_full[j & 1], (j >> 1) & 1, status, &dummy);
      }
      if (q_issued > 0) mbar_wait(&bars->q_full, (q_issued - 1) & 1, status, &dummy);
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      const uint32_t q_s = smem_u32(sm + OFF_Q);
      const uint32_t wk_s = smem_u32(sm + OFF_WK);
      const uint32_t as_s = smem_u32(sm + OFF_AS);
      const uint32_t qt_s = smem_u32(sm + OFF_QT);
      const uint32_t id_s = smem_u32(sm + OFF_I);
      const uint32_t sh_s = smem_u32(sm + OFF_SH);
      const uint32_t sl_s = smem_u32(sm + OFF_SL);
      const uint32_t kw_s = smem_u32(sm + OFF_KW);
      constexpr uint32_t ID_KW = idesc_bf16(128, 128, true, true);
      constexpr uint32_t ID_P = idesc_bf16(64, 64, false, false);
      constexpr uint32_t ID_QT = idesc_bf16(64, 128, false, true);
      constexpr uint32_t ID_QTN = idesc_bf16(64, 128, false, true, true);
      constexpr uint32_t ID_SC = idesc_bf16(128, 128, false, true, true);
      constexpr uint32_t ID_O1 = idesc_bf16(64, 128, false, false);
      constexpr uint32_t ID_O2 = idesc_bf16(64, 128, false, true);
      // A(jj): Kw, Uv, P of chunk jj
      auto issue_A = [&](int jj) -> bool {
        const int s = jj & 1;
        const uint32_t k_s = smem_u32(sm + OFF_K + s * 16384);
        const uint32_t v_s = smem_u32(sm + OFF_V + s * 16384);
        if (!wait_full(&bars->kv_full[s], jj >> 1, status, bars)) return false;
        if (!wait_full(&bars->q_full, jj, status, bars)) return false;
        if (!wait_full(&bars->wk_full, jj, status, bars)) return false;
        if (jj >= 2 && !wait_full(&bars->g_empty[s], (jj >> 1) - 1, status, bars)) return false;
        tc_fence_after();
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + TM_K, desc_mnmajor(k_s, P64, k), desc_mnmajor(wk_s, P64, k), ID_KW, k > 0);
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + (s ? TM_U1 : TM_U0), desc_mnmajor(v_s, P64, k),
                   desc_mnmajor(wk_s, P64, k), ID_KW, k > 0);
        for (int k = 0; k < 8; ++k)
          mma_bf16(tmem + TM_X, desc_kmajor(q_s, P64, k), desc_kmajor(k_s, P64, k), ID_P, k > 0);
        mma_commit(&bars->kwp_full);
        mma_commit(&bars->wk_empty);
        return true;
      };
      // B(jj): Qt = I q - A k
      auto issue_B = [&](int jj) -> bool {
        const uint32_t k_s = smem_u32(sm + OFF_K + (jj & 1) * 16384);
        if (!wait_full(&bars->as_full, jj, status, bars)) return false;
        tc_fence_after();
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + TM_X, desc_kmajor(id_s, P64, k), desc_mnmajor(q_s, P64, k), ID_QT, k > 0);
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + TM_X, desc_kmajor(as_s, P64, k), desc_mnmajor(k_s, P64, k), ID_QTN, 1);
        mma_commit(&bars->qt_full);
        mma_commit(&bars->q_empty);
        return true;
      };
      bool ok = N > 0 && issue_A(0) && issue_B(0);
      for (int j = 0; ok && j < N; ++j) {
        const int s = j & 1;
        const uint32_t v_s = smem_u32(sm + OFF_V + s * 16384);
        const uint32_t ru = tmem + (s ? TM_U1 : TM_U0);
        // C(j): G = Uv - S_hi Kw - S_lo Kw  (Kw read MN-major: B[a][b] = Kw[a][b])
        if (!wait_full(&bars->kw_smem, j, status, bars)) break;
        if (!wait_full(&bars->s_full, j, status, bars)) break;
        tc_fence_after();
        for (int k = 0; k < 8; ++k)
          mma_bf16(ru, desc_kmajor(sh_s, P128, k), desc_mnmajor(kw_s, P128, k), ID_SC, 1);
        for (int k = 0; k < 8; ++k)
          mma_bf16(ru, desc_kmajor(sl_s, P128, k), desc_mnmajor(kw_s, P128, k), ID_SC, 1);
        mma_commit(&bars->g_full[s]);
        // D(j): o = Qt S_hi^T + A v  (lanes 16-31 of RX)
        if (!wait_full(&bars->qt_smem, j, status, bars)) break;
        if (!wait_empty(&bars->o_empty, j, status, bars)) break;
        tc_fence_after();
        for (int k = 0; k < 8; ++k)
          mma_bf16(tmem + TM_HI16 + TM_X, desc_kmajor(qt_s, P64, k), desc_kmajor(sh_s, P128, k),
                   ID_O1, k > 0);
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + TM_HI16 + TM_X, desc_kmajor(as_s, P64, k), desc_mnmajor(v_s, P64, k),
                   ID_O2, 1);
        mma_commit(&bars->o_full);
        mma_commit(&bars->kv_empty[s]);
        if (j + 1 < N && !(issue_A(j + 1) && issue_B(j + 1))) break;
      }
      // every MMA issued so far has completed before TMEM is released
      mma_commit(&bars->final_mma);
      int dummy = 0;
      mbar_wait(&bars->final_mma, 0, status, &dummy);
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------ state rows, o store
    const int c = warp * 32 + lane;  // row of S = TMEM lane
    const uint32_t lb = tmem_lane_base(warp);
    uint8_t* Sh = sm + OFF_SH;
    uint8_t* Sl = sm + OFF_SL;
    float st[kD];
#pragma unroll
    for (int i = 0; i < kD; ++i) st[i] = 0.f;
    {
      const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int c8 = 0; c8 < 16; ++c8) {
        *reinterpret_cast<uint4*>(Sh + (c8 >> 3) * P128 + sw128_chunk(c, c8 & 7)) = z;
        *reinterpret_cast<uint4*>(Sl + (c8 >> 3) * P128 + sw128_chunk(c, c8 & 7)) = z;
      }
      uint4* g = reinterpret_cast<uint4*>(args.S_hist + (static_cast<size_t>(bh) * N) * kD * kD +
                                          static_cast<size_t>(c) * kD);
#pragma unroll
      for (int i = 0; i < 16; ++i) g[i] = z;
    }
    fence_async_smem();
    mbar_arrive(&bars->s_full);
    for (int j = 0; j < N; ++j) {
      const int s = j & 1;
      const float* al = args.alpha + tok0 + j * kC;
      float la = logf(fmaxf(__ldg(al + lane), kGateFloor)) +
                 logf(fmaxf(__ldg(al + lane + 32), kGateFloor));
      const float a = expf(warp_sum(la));
      if (!wait_full(&bars->g_full[s], j >> 1, status, bars)) break;
      tc_fence_after();
      const uint32_t ru = tmem + lb + (s ? TM_U1 : TM_U0);
#pragma unroll
      for (int cc = 0; cc < 8; cc += 2) {
        float g0[16], g1[16];
        tmem_ld16(ru + cc * 16, g0);
        tmem_ld16(ru + cc * 16 + 16, g1);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          st[cc * 16 + i] = fmaf(a, st[cc * 16 + i], g0[i]);
          st[cc * 16 + 16 + i] = fmaf(a, st[cc * 16 + 16 + i], g1[i]);
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->g_empty[s]);
      if (!wait_full(&bars->o_full, j, status, bars)) break;
      // S_{j+1} = hi + lo into shared memory; hi also to the history
      uint4* gdst = nullptr;
      if (j + 1 < N)
        gdst = reinterpret_cast<uint4*>(args.S_hist +
                                        (static_cast<size_t>(bh) * N + j + 1) * kD * kD +
                                        static_cast<size_t>(c) * kD);
#pragma unroll
      for (int c8 = 0; c8 < 16; ++c8) {
        float hi[8], lo[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float x = st[c8 * 8 + i];
          hi[i] = __bfloat162float(__float2bfloat16_rn(x));
          lo[i] = x - hi[i];
        }
        const uint4 wh = pack8(hi);
        *reinterpret_cast<uint4*>(Sh + (c8 >> 3) * P128 + sw128_chunk(c, c8 & 7)) = wh;
        *reinterpret_cast<uint4*>(Sl + (c8 >> 3) * P128 + sw128_chunk(c, c8 & 7)) = pack8(lo);
        if (gdst) gdst[c8] = wh;
      }
      fence_async_smem();
      mbar_arrive(&bars->s_full);
      // o rows: lanes 16-31 of each subpartition hold row 16*warp + lane - 16
      tc_fence_after();
      {
        const int t = warp * 16 + (lane & 15);
        uint4* odst = reinterpret_cast<uint4*>(args.o) +
                      ((tok0 + static_cast<size_t>(j) * kC + t) * kD) / 8;
#pragma unroll
        for (int cc = 0; cc < 8; cc += 2) {
          float x0[16], x1[16];
          tmem_ld16(tmem + lb + TM_X + cc * 16, x0);
          tmem_ld16(tmem + lb + TM_X + cc * 16 + 16, x1);
          tmem_ld_wait();
          if (lane >= 16) {
            odst[cc * 2 + 0] = pack8(x0);
            odst[cc * 2 + 1] = pack8(x0 + 8);
            odst[cc * 2 + 2] = pack8(x1);
            odst[cc * 2 + 3] = pack8(x1 + 8);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->o_empty);
    }
  } else {
    // ------------------------------------------------------------ chunk-local (warps 4-7)
    const int tb = threadIdx.x - 128;          // 0..127
    const int sp = warp - 4;                   // TMEM subpartition
    const uint32_t lb = tmem_lane_base(warp);
    const int row = sp * 32 + lane;            // TMEM lane of this thread
    const int t16 = sp * 16 + (lane & 15);     // M=64 row of lanes 0-15
    // E1: w * k for chunk jj (delta: w = beta)
    auto build_wk = [&](int jj) -> bool {
      const int s = jj & 1;
      if (!wait_full(&bars->kv_full[s], jj >> 1, status, bars)) return false;
      if (!wait_empty(&bars->wk_empty, jj, status, bars)) return false;
      const uint8_t* ks = sm + OFF_K + s * 16384;
      uint8_t* wk = sm + OFF_WK;
      const float* bs = gate_beta + s * 64;
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int id = tb + 128 * m;            // 16-byte chunk id, 0..1023
        const uint32_t off = static_cast<uint32_t>(id) * 16u;
        const float w = bs[(id & 511) >> 3];    // row inside the panel
        const uint4 x = *reinterpret_cast<const uint4*>(ks + off);
        uint4 y;
        y.x = pack_bf16(bf16_lo(x.x) * w, bf16_hi(x.x) * w);
        y.y = pack_bf16(bf16_lo(x.y) * w, bf16_hi(x.y) * w);
        y.z = pack_bf16(bf16_lo(x.z) * w, bf16_hi(x.z) * w);
        y.w = pack_bf16(bf16_lo(x.w) * w, bf16_hi(x.w) * w);
        *reinterpret_cast<uint4*>(wk + off) = y;
      }
      fence_async_smem();
      mbar_arrive(&bars->wk_full);
      mbar_arrive(&bars->kv_empty[s]);
      return true;
    };
    // E2: P -> A = tril(P) * beta (bf16)
    auto build_as = [&](int jj) -> bool {
      const float* bs = gate_beta + (jj & 1) * 64;
      if (!wait_full(&bars->kwp_full, jj, status, bars)) return false;
      if (jj >= 1 && !wait_full(&bars->o_full, jj - 1, status, bars)) return false;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < 4; cc += 2) {
        float p0[16], p1[16];
        tmem_ld16(tmem + lb + TM_X + cc * 16, p0);
        tmem_ld16(tmem + lb + TM_X + cc * 16 + 16, p1);
        tmem_ld_wait();
        if (lane < 16) {
          float v8[8];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const float* src = h < 2 ? p0 + h * 8 : p1 + (h - 2) * 8;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int sc = cc * 16 + h * 8 + i;
              v8[i] = (sc <= t16) ? src[i] * bs[sc] : 0.f;
            }
            st_row8(sm + OFF_AS, P64, t16, cc * 2 + h, v8);
          }
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->as_full);
      return true;
    };
    bool ok = N > 0 && build_wk(0) && build_as(0);
    for (int j = 0; ok && j < N; ++j) {
      // E0: Kw -> bf16 shared (row a = lane row, all 128 columns)
      if (!wait_full(&bars->kwp_full, j, status, bars)) break;
      if (j >= 1 && !wait_full(&bars->g_full[(j - 1) & 1], (j - 1) >> 1, status, bars)) break;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < 8; cc += 2) {
        float x0[16], x1[16];
        tmem_ld16(tmem + lb + TM_K + cc * 16, x0);
        tmem_ld16(tmem + lb + TM_K + cc * 16 + 16, x1);
        tmem_ld_wait();
        st_row8(sm + OFF_KW, P128, row, cc * 2, x0);
        st_row8(sm + OFF_KW, P128, row, cc * 2 + 1, x0 + 8);
        st_row8(sm + OFF_KW, P128, row, cc * 2 + 2, x1);
        st_row8(sm + OFF_KW, P128, row, cc * 2 + 3, x1 + 8);
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->kw_smem);
      // E3: Qt (lanes 0-15, row t, 128 columns) -> bf16 shared
      if (!wait_full(&bars->qt_full, j, status, bars)) break;
      if (j >= 1 && !wait_full(&bars->o_full, j - 1, status, bars)) break;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < 8; cc += 2) {
        float x0[16], x1[16];
        tmem_ld16(tmem + lb + TM_X + cc * 16, x0);
        tmem_ld16(tmem + lb + TM_X + cc * 16 + 16, x1);
        tmem_ld_wait();
        if (lane < 16) {
          st_row8(sm + OFF_QT, P64, t16, cc * 2, x0);
          st_row8(sm + OFF_QT, P64, t16, cc * 2 + 1, x0 + 8);
          st_row8(sm + OFF_QT, P64, t16, cc * 2 + 2, x1);
          st_row8(sm + OFF_QT, P64, t16, cc * 2 + 3, x1 + 8);
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->qt_smem);
      if (j + 1 < N && !(build_wk(j + 1) && build_as(j + 1))) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace

namespace {

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

}  // namespace

// rows x 128 bf16 matrix, 64 x 64 boxes, 128-byte swizzle.
cudaError_t make_tmap_rows128(CUtensorMap* map, const void* base, uint64_t rows,
                              uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  cuuint64_t dims[2] = {128, rows};
  cuuint64_t strides[1] = {256};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                  strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

bool chunk_fwd_tc_supported(const ChunkArgs& p) {
  return p.rule == 0 && p.dh == kD && p.C == kC && !p.io_f32 && p.N >= 1 && encode_fn();
}

size_t chunk_fwd_tc_saved_bytes(int BH, int N) {
  return static_cast<size_t>(BH) * N * kD * kD * sizeof(uint16_t);
}

cudaError_t chunk_fwd_tc(const ChunkArgs& p, uint16_t* S_hist, uint32_t* status,
                         cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  const uint64_t rows = static_cast<uint64_t>(p.BH) * p.T;
  cudaError_t e;
  if ((e = make_tmap_rows128(&mq, p.q, rows, 64)) != cudaSuccess) return e;
  if ((e = make_tmap_rows128(&mk, p.k, rows, 64)) != cudaSuccess) return e;
  if ((e = make_tmap_rows128(&mv, p.v, rows, 64)) != cudaSuccess) return e;
  FwdArgs a;
  a.beta = p.beta;
  a.alpha = p.alpha;
  a.o = static_cast<uint16_t*>(p.o);
  a.S_hist = S_hist;
  a.status = status;
  a.N = p.N;
  a.T = p.T;
  e = cudaFuncSetAttribute(chunk_fwd_tc_delta, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           SMEM_BYTES);
  if (e != cudaSuccess) return e;
  chunk_fwd_tc_delta<<<p.BH, kThreadsTc, SMEM_BYTES, st>>>(mq, mk, mv, a);
  return cudaGetLastError();
}

}  // namespace gmdn
