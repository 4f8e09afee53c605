// Fused tensor-core forward of the mixer core, delta rule, dh = 128, C = 64.
//
// One CTA per (batch, head) walks the N chunks in order.  Per chunk j
// (train_ablation.py:142-187 with the scan of fast_scan.py:72-95):
//
//   A(j)  Kw_j = k^T (w k)      M128 N128 K64   -> TMEM RK
//         Uv_j = v^T (w k)      M128 N128 K64   -> TMEM RU[j%2]
//         P_j  = q k^T          M64  N64  K128  -> TMEM RPQ
//   B(j)  Qt_j^T = q^T I - k^T A_j^T            -> TMEM RPQ  (A_j = tril(P_j) * beta)
//   C(j)  G_j = Uv_j - S_j Kw_j  (S_j = hi + lo, two bf16 passes)   -> RU[j%2]
//   D(j)  o_j^T = S_j Qt_j^T + v^T A_j^T        -> TMEM RO
//   state S_{j+1} = a_j S_j + G_j  (fp32, in registers of warps 0-3)
//
// Warp roles (320 threads): warps 0-3 own the fp32 state (one row of S per
// thread) and run the sequential update; warps 4-7 drain the chunk-local
// accumulators (Kw, P -> A, Qt, o) and build w*k; warp 8 issues TMA loads;
// warp 9 allocates TMEM and issues every MMA from one thread.  All
// hand-offs are mbarriers; every wait is bounded (tc.cuh) and a timeout
// sets the status word and unwinds all roles.
//
// Bytes per chunk-head: q, k, v in (48 KB), o out (16 KB), S_j bf16 out for
// the backward (32 KB).  Tensor work per chunk-head: 2*2*C*d^2 (Kw, Uv) +
// 2*C^2*d (P) + 2*(C*d*C) (Qt) + 2*2*d^3 (state, hi+lo) + 2*(C*d^2 + C^2*d) (o).

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

// TMEM columns
constexpr uint32_t TM_U0 = 0, TM_U1 = 128, TM_K = 256, TM_PQ = 384, TM_O = 448;

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

// Write 8 floats of row `row`, columns [col8*8, col8*8+8) of a 2-panel bf16
// tile (64 columns per panel) as one 16-byte swizzled chunk.
__device__ __forceinline__ void st_row8(uint8_t* tile, uint32_t panel_stride, int row, int col8,
                                        const float* v) {
  uint4 w;
  w.x = pack_bf16(v[0], v[1]);
  w.y = pack_bf16(v[2], v[3]);
  w.z = pack_bf16(v[4], v[5]);
  w.w = pack_bf16(v[6], v[7]);
  uint8_t* p = tile + (col8 >> 3) * panel_stride + sw128_chunk(row, col8 & 7);
  *reinterpret_cast<uint4*>(p) = w;
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
  // 64 x 64 identity (bf16 1.0 = 0x3F80) in the SW128 layout
  for (int r = threadIdx.x; r < 64; r += kThreadsTc) {
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
      *reinterpret_cast<uint4*>(sm + OFF_I + sw128_chunk(r, c8)) = w;
    }
  }
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
      constexpr uint32_t ID_QT = idesc_bf16(128, 64, true, false);
      constexpr uint32_t ID_QTN = idesc_bf16(128, 64, true, false, true);
      constexpr uint32_t ID_SC = idesc_bf16(128, 128, false, true, true);
      constexpr uint32_t ID_O1 = idesc_bf16(128, 64, false, false);
      constexpr uint32_t ID_O2 = idesc_bf16(128, 64, true, false);
      for (int j = 0; j < N; ++j) {
        const int s = j & 1;
        const uint32_t k_s = smem_u32(sm + OFF_K + s * 16384);
        const uint32_t v_s = smem_u32(sm + OFF_V + s * 16384);
        const uint32_t ru = tmem + (s ? TM_U1 : TM_U0);
        // A(j)
        if (!wait_full(&bars->kv_full[s], j >> 1, status, bars)) break;
        if (!wait_full(&bars->q_full, j, status, bars)) break;
        if (!wait_full(&bars->wk_full, j, status, bars)) break;
        if (j >= 2 && !wait_full(&bars->g_empty[s], (j >> 1) - 1, status, bars)) break;
        if (j >= 1 && !wait_full(&bars->kw_smem, j - 1, status, bars)) break;
        if (j >= 1 && !wait_full(&bars->qt_smem, j - 1, status, bars)) break;
        tc_fence_after();
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + TM_K, desc_mnmajor(k_s, P64, k), desc_mnmajor(wk_s, P64, k), ID_KW, k > 0);
        for (int k = 0; k < 4; ++k)
          mma_bf16(ru, desc_mnmajor(v_s, P64, k), desc_mnmajor(wk_s, P64, k), ID_KW, k > 0);
        for (int k = 0; k < 8; ++k)
          mma_bf16(tmem + TM_PQ, desc_kmajor(q_s, P64, k), desc_kmajor(k_s, P64, k), ID_P, k > 0);
        mma_commit(&bars->kwp_full);
        mma_commit(&bars->wk_empty);
        // B(j): Qt^T = q^T I - k^T A^T
        if (!wait_full(&bars->as_full, j, status, bars)) break;
        tc_fence_after();
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + TM_PQ, desc_mnmajor(q_s, P64, k), desc_kmajor(id_s, P64, k), ID_QT, k > 0);
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + TM_PQ, desc_mnmajor(k_s, P64, k), desc_kmajor(as_s, P64, k), ID_QTN, 1);
        mma_commit(&bars->qt_full);
        mma_commit(&bars->q_empty);
        // C(j): G = Uv - S_hi Kw - S_lo Kw (Kw read MN-major: B[a][b] = Kw[a][b])
        if (!wait_full(&bars->kw_smem, j, status, bars)) break;
        if (!wait_full(&bars->s_full, j, status, bars)) break;
        tc_fence_after();
        for (int k = 0; k < 8; ++k)
          mma_bf16(ru, desc_kmajor(sh_s, P128, k), desc_mnmajor(kw_s, P128, k), ID_SC, 1);
        for (int k = 0; k < 8; ++k)
          mma_bf16(ru, desc_kmajor(sl_s, P128, k), desc_mnmajor(kw_s, P128, k), ID_SC, 1);
        mma_commit(&bars->g_full[s]);
        // D(j): o^T = S_hi Qt^T + v^T A^T
        if (!wait_full(&bars->qt_smem, j, status, bars)) break;
        if (!wait_empty(&bars->o_empty, j, status, bars)) break;
        tc_fence_after();
        for (int k = 0; k < 8; ++k)
          mma_bf16(tmem + TM_O, desc_kmajor(sh_s, P128, k), desc_kmajor(qt_s, P64, k), ID_O1, k > 0);
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + TM_O, desc_mnmajor(v_s, P64, k), desc_kmajor(as_s, P64, k), ID_O2, 1);
        mma_commit(&bars->o_full);
        mma_commit(&bars->kv_empty[s]);
      }
      // every MMA issued so far has completed before TMEM is released
      mma_commit(&bars->final_mma);
      int dummy = 0;
      mbar_wait(&bars->final_mma, 0, status, &dummy);
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------ state (rows of S)
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
      for (int cc = 0; cc < 8; ++cc) {
        float g[16];
        tmem_ld16(ru + cc * 16, g);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i) st[cc * 16 + i] = fmaf(a, st[cc * 16 + i], g[i]);
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
        st_row8(Sh, P128, c, c8, hi);
        st_row8(Sl, P128, c, c8, lo);
        if (gdst) {
          uint4 w;
          w.x = pack_bf16(hi[0], hi[1]);
          w.y = pack_bf16(hi[2], hi[3]);
          w.z = pack_bf16(hi[4], hi[5]);
          w.w = pack_bf16(hi[6], hi[7]);
          gdst[c8] = w;
        }
      }
      fence_async_smem();
      mbar_arrive(&bars->s_full);
    }
  } else {
    // ------------------------------------------------------------ chunk-local (warps 4-7)
    const int tb = threadIdx.x - 128;          // 0..127
    const int sp = warp - 4;                   // TMEM subpartition
    const uint32_t lb = tmem_lane_base(warp);
    const int row = sp * 32 + lane;            // TMEM lane of this thread
    bool ok = true;
    // w * k for chunk jj (delta: w = beta)
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
        const int r = (id & 511) >> 3;          // row inside the panel
        const float w = bs[r];
        uint4 x = *reinterpret_cast<const uint4*>(ks + off);
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
    if (N > 0) ok = build_wk(0);
    for (int j = 0; ok && j < N; ++j) {
      const int s = j & 1;
      const float* bs = gate_beta + s * 64;
      // E2: P -> A = tril(P) * beta (bf16)
      if (!wait_full(&bars->kwp_full, j, status, bars)) break;
      if (j >= 1 && !wait_full(&bars->o_full, j - 1, status, bars)) break;
      tc_fence_after();
      {
        const int t = sp * 16 + (lane & 15);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          float p[16];
          tmem_ld16(tmem + lb + TM_PQ + cc * 16, p);
          tmem_ld_wait();
          if (lane < 16) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              float v8[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int sc = cc * 16 + h * 8 + i;
                v8[i] = (sc <= t) ? p[h * 8 + i] * bs[sc] : 0.f;
              }
              st_row8(sm + OFF_AS, P64, t, cc * 2 + h, v8);
            }
          }
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->as_full);
      // E0: Kw -> bf16 shared (row a = lane row, all 128 columns)
      if (j >= 1 && !wait_full(&bars->g_full[(j - 1) & 1], (j - 1) >> 1, status, bars)) break;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        float x[16];
        tmem_ld16(tmem + lb + TM_K + cc * 16, x);
        tmem_ld_wait();
        st_row8(sm + OFF_KW, P128, row, cc * 2, x);
        st_row8(sm + OFF_KW, P128, row, cc * 2 + 1, x + 8);
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->kw_smem);
      // E3: Qt^T (lane = d, columns = t) -> Qt[t][d] bf16
      if (!wait_full(&bars->qt_full, j, status, bars)) break;
      tc_fence_after();
      {
        uint8_t* qt = sm + OFF_QT + (row >> 6) * P64;
        const int dcol = row & 63;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          float x[16];
          tmem_ld16(tmem + lb + TM_PQ + cc * 16, x);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i)
            *reinterpret_cast<__nv_bfloat16*>(qt + sw128_elem(cc * 16 + i, dcol)) =
                __float2bfloat16_rn(x[i]);
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&bars->qt_smem);
      // E1 for the next chunk
      if (j + 1 < N && !build_wk(j + 1)) break;
      // E5: o^T (lane = c, columns = t) -> o[t][c]
      if (!wait_full(&bars->o_full, j, status, bars)) break;
      tc_fence_after();
      {
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(args.o) +
                           (tok0 + static_cast<size_t>(j) * kC) * kD + row;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          float x[16];
          tmem_ld16(tmem + lb + TM_O + cc * 16, x);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[static_cast<size_t>(cc * 16 + i) * kD] = __float2bfloat16_rn(x[i]);
        }
      }
      tc_fence_before();
      mbar_arrive(&bars->o_empty);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

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
