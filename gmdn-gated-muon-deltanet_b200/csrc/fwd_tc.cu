// Fused tensor-core forward of the mixer core, delta and adam rules,
// dh = 128 (or 64), C = 64.  A dh-64 head runs as a dh-128 one whose upper 64
// features are zero: its TMA maps are 64 columns wide, so the load of the
// upper panel fills shared memory with zeros, and the store of o's upper panel
// is skipped.  The state then stays zero outside its leading 64 x 64 block.
//
// One CTA per (batch, head) walks the N chunks in order.  The chunk update
// of the reference (fast_scan.py:82-85 on the products of
// train_ablation.py:160-167) is evaluated in residual form: with the errors
// of chunk j against the frozen state, E_j = v_j - k_j S_j^T,
//
//   G_j = Uv_j - S_j Kw_j = E_j^T (w k_j)
//   o_j = Qt_j S_j^T + A_j v_j = q_j S_j^T + A_j E_j,  A_j = tril(q k^T) * beta
//   S_{j+1} = a_j S_j + G_j                                   (delta, w = beta)
//   M' = mu_c M + (1 - mu_c) G_j,  V' = nu_c V + (1 - nu_c) G_j^2,
//   S_{j+1} = a_j S_j + b_c M' / (sqrt(V') + 1e-6)             (adam, w = 1)
//
// (fast_scan.py:82-94; chunk scalars train_ablation.py:169-175).  Adam keeps
// the fp32 moments in a per-thread slab of global memory (128 KB per head, L2
// resident) and writes G_j and the pre-update moments as bf16 for the
// backward.
//
// Per chunk the MMA thread issues (M x N x K):
//   E(j)   -E_j^T = -v_j^T I + S_j k_j^T   128 x 64 x 64, 128 x 64 x 128 (S hi, lo)
//   o1(j)  o_j^T  = S_j q_j^T              128 x 64 x 128 (S hi)
//   G(j)   G_j    = (w E_j)^T k_j          128 x 128 x 64 (w E hi, lo)
//   o2(j)  o_j^T += (w E_j)^T A'_j^T       128 x 64 x 64,  A' = tril(q k^T) beta / w
//   P(j+1) P      = q k^T                  64 x 64 x 128
// S_j hi/lo (packed bf16) live in TMEM as the A operand of E and o1, and the
// token weights are folded into E: the drain writes w E as packed bf16 hi/lo
// back into TMEM, where it is the A operand of G and o2.  Besides the
// operands TMA brings in, the chain never touches shared memory (shared-memory
// bandwidth, not the tensor core, bounded the chain when E and w k went
// through it).
//
// Warp roles (448 threads): warps 0-7 own the fp32 state (row c of S,
// 64 columns each) and run S_{j+1} = a_j S_j + G_j; warps 8-11 drain E,
// build A, and stage o for a TMA store; warp 12 issues TMA loads;
// warp 13 allocates TMEM and issues every MMA from one thread.  All hand-offs
// are mbarriers with bounded waits (tc.cuh).
//
// HBM per chunk-head: q, k, v in (48 KB), o out (16 KB), S_j bf16 out for the
// backward (32 KB); adam adds G_j, M_j, V_j bf16 out (96 KB).

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
constexpr int kThreadsTc = 448;

// shared-memory map (bytes from a 1024-aligned base)
constexpr uint32_t OFF_Q = 0;             // q: 2 stages x 16 KB
constexpr uint32_t OFF_K = 32768;         // k: 2 stages
constexpr uint32_t OFF_V = 65536;         // v: 2 stages
constexpr uint32_t OFF_AS = 98304;        // A_j bf16, 1 panel x 64 rows
constexpr uint32_t OFF_I = 106496;        // 64 x 64 identity
constexpr uint32_t OFF_OS = 114688;       // o_j staging for the TMA store, 2 panels x 64 rows
constexpr uint32_t OFF_SS = 131072;       // S_{j+1} hi staging for the TMA store, 2 panels x 128 rows
constexpr uint32_t OFF_GATE = 163840;     // beta, alpha, mu, nu: 2 stages x 64 floats each
constexpr uint32_t OFF_BAR = 165888;      // mbarriers and flags
constexpr uint32_t SMEM_BYTES = OFF_BAR + 256 + 1024;

constexpr uint32_t P64 = 8192;    // panel stride of a 64-row tile
constexpr uint32_t P128 = 16384;  // panel stride of a 128-row tile

// TMEM columns
constexpr uint32_t TM_E = 0, TM_G = 64, TM_O = 192, TM_P = 256, TM_SH = 384, TM_SL = 448;
constexpr uint32_t TM_WEH = 320, TM_WEL = 352;   // w E^T hi / lo, packed bf16 pairs (64 tokens)

// Who drains E: delta, the eight state warps (idle between packing S and G;
// two warps per TMEM subpartition); adam, the four chunk-local warps (its
// state warps carry the moment update).
template <int RULE>
constexpr int kEWarps = RULE == 0 ? 8 : 4;

struct Bars {
  uint64_t ld_full[2], ld_empty[2];
  uint64_t p_full, as_full, wk_full, e_full, e_smem, g_full, s_full, o_full, o_empty;
  uint64_t final_mma;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Bars) <= 256, "barrier block");

struct FwdArgs {
  const float* beta;
  const float* alpha;
  const float *mu, *nu;
  uint16_t* S_hist;
  uint16_t *G_hist, *Mp_hist, *Vp_hist;  // adam
  float *M_ws, *V_ws;                    // adam
  uint32_t* status;
  int N, T;
  int store_hi;   // dh 128: store o's upper 64 columns (dh 64: they are the zero padding)
};

template <int RULE>
__global__ void __launch_bounds__(kThreadsTc, 1)
chunk_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                   const __grid_constant__ CUtensorMap tm_sh, FwdArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  Bars* bars = reinterpret_cast<Bars*>(sm + OFF_BAR);
  float* gate_beta = reinterpret_cast<float*>(sm + OFF_GATE);   // [2][64]
  float* gate_alpha = gate_beta + 128;                           // [2][64]
  float* gate_mu = gate_beta + 256;                              // adam: [2][64]
  float* gate_nu = gate_beta + 384;                              // adam: [2][64]
  volatile int* ab = &bars->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x;
  const int N = args.N;
  uint32_t* status = args.status;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->ld_full[s], 1);
      // MMA commit, the E-draining warps (adam: and the state warps, which read
      // the stage's gates for their chunk scalars)
      mbar_init(&bars->ld_empty[s], 1 + kEWarps<RULE> + (RULE == 2 ? 8 : 0));
    }
    mbar_init(&bars->p_full, 1);
    mbar_init(&bars->as_full, 4);
    mbar_init(&bars->e_full, 1);
    mbar_init(&bars->e_smem, kEWarps<RULE>);
    mbar_init(&bars->g_full, 1);
    mbar_init(&bars->s_full, 8);
    mbar_init(&bars->o_full, 1);
    mbar_init(&bars->o_empty, 4);
    mbar_init(&bars->final_mma, 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  build_identity64(sm + OFF_I, threadIdx.x, kThreadsTc);
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
    // ------------------------------------------------------------ TMA loads
    if (lane == 0) {
      int issued = 0;
      for (int j = 0; j < N; ++j) {
        const int s = j & 1;
        const int row = static_cast<int>(tok0) + j * kC;
        if (!wait_free(&bars->ld_empty[s], j >> 1, status, ab)) break;
        mbar_expect_tx(&bars->ld_full[s], 6 * 8192 + 512 + (RULE == 2 ? 512 : 0));
        tma_load_2d(sm + OFF_Q + s * 16384, &tm_q, 0, row, &bars->ld_full[s]);
        tma_load_2d(sm + OFF_Q + s * 16384 + P64, &tm_q, 64, row, &bars->ld_full[s]);
        tma_load_2d(sm + OFF_K + s * 16384, &tm_k, 0, row, &bars->ld_full[s]);
        tma_load_2d(sm + OFF_K + s * 16384 + P64, &tm_k, 64, row, &bars->ld_full[s]);
        tma_load_2d(sm + OFF_V + s * 16384, &tm_v, 0, row, &bars->ld_full[s]);
        tma_load_2d(sm + OFF_V + s * 16384 + P64, &tm_v, 64, row, &bars->ld_full[s]);
        bulk_load(gate_beta + s * 64, args.beta + tok0 + j * kC, 256, &bars->ld_full[s]);
        bulk_load(gate_alpha + s * 64, args.alpha + tok0 + j * kC, 256, &bars->ld_full[s]);
        if (RULE == 2) {
          bulk_load(gate_mu + s * 64, args.mu + tok0 + j * kC, 256, &bars->ld_full[s]);
          bulk_load(gate_nu + s * 64, args.nu + tok0 + j * kC, 256, &bars->ld_full[s]);
        }
        issued = j + 1;
      }
      // Never leave with copies in flight (matters only after an abort).
      int dummy = 0;
      for (int j = issued - 2; j < issued; ++j)
        if (j >= 0) mbar_wait(&bars->ld_full[j & 1], (j >> 1) & 1, status, &dummy);
    }
  } else if (warp == 13) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      const uint32_t as_s = smem_u32(sm + OFF_AS);
      const uint32_t id_s = smem_u32(sm + OFF_I);
      constexpr uint32_t ID_P = idesc_bf16(64, 64, false, false);
      constexpr uint32_t ID_EV = idesc_bf16(128, 64, true, false, true);   // -v^T I
      constexpr uint32_t ID_ES = idesc_bf16(128, 64, false, false);        // S k^T (A in TMEM)
      constexpr uint32_t ID_G = idesc_bf16(128, 128, false, true);         // (w E)^T k (A in TMEM)
      constexpr uint32_t ID_O2 = idesc_bf16(128, 64, false, false);        // (w E)^T A'^T (A in TMEM)
      auto stage = [&](uint32_t base, int j) { return smem_u32(sm + base + (j & 1) * 16384); };
      auto issue_P = [&](int j) -> bool {
        if (!wait_use(&bars->ld_full[j & 1], j >> 1, status, ab)) return false;
        tc_fence_after();
        #pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(tmem + TM_P, desc_kmajor(stage(OFF_Q, j), P64, k),
                   desc_kmajor(stage(OFF_K, j), P64, k), ID_P, k > 0);
        mma_commit(&bars->p_full);
        return true;
      };
      // -v_j^T I into the E accumulator (it must be free: E(j-1) drained); v_j
      // must have landed in its stage
      auto issue_E1 = [&](int j) -> bool {
        if (!wait_use(&bars->ld_full[j & 1], j >> 1, status, ab)) return false;
        tc_fence_after();
        const uint32_t v_s = stage(OFF_V, j);
        #pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + TM_E, desc_mnmajor(v_s, P64, k), desc_kmajor(id_s, P64, k), ID_EV, k > 0);
        return true;
      };
      // Issue order per chunk: E(j); o1(j) (runs while E(j) is drained); G(j) as
      // soon as the drain ends; then o2(j), -v^T I and P of the next chunk, which
      // run while the state is updated.
      bool ok = N > 0 && issue_P(0);
      ok = ok && issue_E1(0);
      for (int j = 0; ok && j < N; ++j) {
        const uint32_t q_s = stage(OFF_Q, j), k_s = stage(OFF_K, j);
        // E(j): D = -v^T I + S_hi k^T + S_lo k^T = -E^T
        if (!wait_use(&bars->s_full, j, status, ab)) break;
        tc_fence_after();
        #pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(tmem + TM_E, tmem + TM_SH + k * 8, desc_kmajor(k_s, P64, k), ID_ES, 1);
        #pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(tmem + TM_E, tmem + TM_SL + k * 8, desc_kmajor(k_s, P64, k), ID_ES, 1);
        mma_commit(&bars->e_full);
        // o1(j): o^T = S_hi q^T
        if (!wait_free(&bars->o_empty, j, status, ab)) break;
        tc_fence_after();
        #pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(tmem + TM_O, tmem + TM_SH + k * 8, desc_kmajor(q_s, P64, k), ID_ES, k > 0);
        // G(j) = (w E)^T_hi k + (w E)^T_lo k   (A from TMEM)
        if (!wait_use(&bars->e_smem, j, status, ab)) break;
        tc_fence_after();
        #pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16_ts(tmem + TM_G, tmem + TM_WEH + k * 8, desc_mnmajor(k_s, P64, k), ID_G, k > 0);
        #pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16_ts(tmem + TM_G, tmem + TM_WEL + k * 8, desc_mnmajor(k_s, P64, k), ID_G, 1);
        mma_commit(&bars->g_full);
        // G(j) is the stage's last reader (o2 reads A' and TMEM only): release it
        // now, so the load of chunk j+2 starts an o2 earlier
        mma_commit(&bars->ld_empty[j & 1]);
        // o2(j): o^T += (w E)^T_hi A'^T, once A'(j) is built
        if (!wait_use(&bars->as_full, j, status, ab)) break;
        tc_fence_after();
        #pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16_ts(tmem + TM_O, tmem + TM_WEH + k * 8, desc_kmajor(as_s, P64, k), ID_O2, 1);
        mma_commit(&bars->o_full);
        if (j + 1 < N && !issue_E1(j + 1)) break;   // E(j) has been drained (e_smem)
        // P(j+1) last: A'(j) has read P(j) (as_full), and an issue blocks this
        // thread while the pipe is busy, so between o1 and G it kept the thread
        // from seeing the end of the E drain (~1,000 cycles per chunk)
        if (j + 1 < N && !issue_P(j + 1)) break;
      }
      // every MMA issued so far has completed before TMEM is released
      mma_commit(&bars->final_mma);
      int dummy = 0;
      mbar_wait(&bars->final_mma, 0, status, &dummy);
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ state rows
    const int c = (warp & 3) * 32 + lane;   // row of S = TMEM lane
    const int half = warp >> 2;             // columns [64 half, 64 half + 64)
    const uint32_t lb = tmem_lane_base(warp);
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
      uint4* g = reinterpret_cast<uint4*>(args.S_hist + (static_cast<size_t>(bh) * N) * kD * kD +
                                          static_cast<size_t>(c) * kD + half * 64);
      const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
      for (int i = 0; i < 8; ++i) g[i] = z;
    }
    tc_fence_before();
    mbar_arrive_warp(&bars->s_full);
    for (int j = 0; j < N; ++j) {
      // chunk scalars from the gates the TMA brought into this chunk's stage (a
      // global load here stalled the E drain behind it)
      if (!wait_use_w(&bars->ld_full[j & 1], j >> 1, status, ab)) break;
      const float* ga = gate_alpha + (j & 1) * 64;
      const float a = expf(warp_sum(logf(fmaxf(ga[lane], kGateFloor)) +
                                    logf(fmaxf(ga[lane + 32], kGateFloor))));
      if constexpr (kEWarps<RULE> == 8) {
        // -E^T (lanes = value row c, this warp's 32 token columns) -> w E^T hi / lo,
        // packed bf16 pairs into TMEM, the A operand of G and o2
        if (!wait_use_w(&bars->e_full, j, status, ab)) break;
        tc_fence_after();
        const float* ws = gate_beta + (j & 1) * 64 + half * 32;   // delta: w = beta
        float x0[16], x1[16];
        tmem_ld16(tmem + lb + TM_E + half * 32, x0);
        tmem_ld16(tmem + lb + TM_E + half * 32 + 16, x1);
        tmem_ld_wait();
        uint32_t hh[16], ll[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const float y0 = t < 8 ? x0[2 * t] : x1[2 * t - 16];
          const float y1 = t < 8 ? x0[2 * t + 1] : x1[2 * t - 15];
          const float e0 = -y0 * ws[2 * t], e1 = -y1 * ws[2 * t + 1];
          hh[t] = pack_bf16(e0, e1);
          ll[t] = pack_bf16(e0 - bf16_lo(hh[t]), e1 - bf16_hi(hh[t]));
        }
        tmem_st16(tmem + lb + TM_WEH + half * 16, hh);
        tmem_st16(tmem + lb + TM_WEL + half * 16, ll);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive_warp(&bars->e_smem);
        fence_async_smem();   // gate reads before the stage's reload (async proxy)
        mbar_arrive_warp(&bars->ld_empty[j & 1]);   // done with this stage's gates
      }
      if constexpr (RULE == 2) {
        const float* be = gate_beta + (j & 1) * 64;
        const float* mu = gate_mu + (j & 1) * 64;
        const float* nu = gate_nu + (j & 1) * 64;
        const float b = warp_sum(be[lane] + be[lane + 32]) * (1.f / kC);
        const float mc = expf(warp_sum(logf(fmaxf(mu[lane], kGateFloor)) +
                                       logf(fmaxf(mu[lane + 32], kGateFloor))));
        const float nc = expf(warp_sum(logf(fmaxf(nu[lane], kGateFloor)) +
                                       logf(fmaxf(nu[lane + 32], kGateFloor))));
        fence_async_smem();   // gate reads before the stage's reload (async proxy)
        mbar_arrive_warp(&bars->ld_empty[j & 1]);   // done with this stage's gates
        // M_j, V_j (fp32, L2-resident slabs) in 8-column groups, the next
        // group's loaded while this one computes; group 0's go out before the
        // wait for G, so no slab round trip sits between G and the update
        const size_t mj = static_cast<size_t>(bh) * N + j;
        float4 nm0 = make_float4(0.f, 0.f, 0.f, 0.f), nm1 = nm0, nv0 = nm0, nv1 = nm0;
        if (j > 0) {
          const float4* m0p = slab_f32(args.M_ws, bh, half, 0, c);
          const float4* v0p = slab_f32(args.V_ws, bh, half, 0, c);
          nm0 = m0p[0];
          nm1 = m0p[128];
          nv0 = v0p[0];
          nv1 = v0p[128];
        }
        if (!wait_use_w(&bars->g_full, j, status, ab)) break;
        tc_fence_after();
        const uint32_t rg = tmem + lb + TM_G + half * 64;
#pragma unroll
        for (int g8 = 0; g8 < 8; ++g8) {
          float4* mp = slab_f32(args.M_ws, bh, half, 2 * g8, c);
          float4* vp = slab_f32(args.V_ws, bh, half, 2 * g8, c);
          float mv[8] = {nm0.x, nm0.y, nm0.z, nm0.w, nm1.x, nm1.y, nm1.z, nm1.w};
          float vv[8] = {nv0.x, nv0.y, nv0.z, nv0.w, nv1.x, nv1.y, nv1.z, nv1.w};
          if (j > 0 && g8 + 1 < 8) {
            nm0 = mp[256];   // group g8 + 1: float4 rows 2 g8 + 2, 2 g8 + 3
            nm1 = mp[384];
            nv0 = vp[256];
            nv1 = vp[384];
          }
          float g[8];
          tmem_ld8(rg + 8 * g8, g);
          tmem_ld_wait();
          // pre-update G_j, M_j, V_j for the backward
          *slab_bf16(args.G_hist, mj, half, g8, c) = pack8(g);
          *slab_bf16(args.Mp_hist, mj, half, g8, c) = pack8(mv);
          *slab_bf16(args.Vp_hist, mj, half, g8, c) = pack8(vv);
          // element pairs on the packed fp32x2 instructions, SFU square root
          // and reciprocal (the update is on the chain; tc.cuh)
#pragma unroll
          for (int t = 0; t < 8; t += 2) {
            const float2 G = p2(g[t], g[t + 1]);
            const float2 m1 = fma2(p2(mc), p2(mv[t], mv[t + 1]), mul2(p2(1.f - mc), G));
            const float2 v1 = fma2(p2(nc), p2(vv[t], vv[t + 1]), mul2(p2(1.f - nc), mul2(G, G)));
            mv[t] = m1.x;
            mv[t + 1] = m1.y;
            vv[t] = v1.x;
            vv[t + 1] = v1.y;
            const float2 rden = p2(rcp_sfu(sqrt_sfu(v1.x) + kEpsAdam),
                                   rcp_sfu(sqrt_sfu(v1.y) + kEpsAdam));
            const float2 sn = fma2(p2(a), p2(st[8 * g8 + t], st[8 * g8 + t + 1]),
                                   mul2(mul2(p2(b), m1), rden));
            st[8 * g8 + t] = sn.x;
            st[8 * g8 + t + 1] = sn.y;
          }
          if (j + 1 < N) {
            mp[0] = make_float4(mv[0], mv[1], mv[2], mv[3]);
            mp[128] = make_float4(mv[4], mv[5], mv[6], mv[7]);
            vp[0] = make_float4(vv[0], vv[1], vv[2], vv[3]);
            vp[128] = make_float4(vv[4], vv[5], vv[6], vv[7]);
          }
        }
      } else {
      if (!wait_use_w(&bars->g_full, j, status, ab)) break;
      tc_fence_after();
      {
        const uint32_t rg = tmem + lb + TM_G + half * 64;
        float g0[16], g1[16], g2[16], g3[16];
        tmem_ld16(rg, g0);
        tmem_ld16(rg + 16, g1);
        tmem_ld16(rg + 32, g2);
        tmem_ld16(rg + 48, g3);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          st[t] = fmaf(a, st[t], g0[t]);
          st[16 + t] = fmaf(a, st[16 + t], g1[t]);
          st[32 + t] = fmaf(a, st[32 + t], g2[t]);
          st[48 + t] = fmaf(a, st[48 + t], g3[t]);
        }
      }
      }
      // S_{j+1} as packed bf16 hi / lo into TMEM (A operand of E and o1)
      uint32_t ph[32];
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        uint32_t pl[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const float x0 = st[b * 32 + 2 * t], x1 = st[b * 32 + 2 * t + 1];
          ph[b * 16 + t] = pack_bf16(x0, x1);
          pl[t] = pack_bf16(x0 - bf16_lo(ph[b * 16 + t]), x1 - bf16_hi(ph[b * 16 + t]));
        }
        uint32_t hh[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) hh[t] = ph[b * 16 + t];
        tmem_st16(tmem + lb + TM_SH + half * 32 + b * 16, hh);
        tmem_st16(tmem + lb + TM_SL + half * 32 + b * 16, pl);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive_warp(&bars->s_full);
      // history for the backward: S_{j+1} hi through a staging tile and one
      // TMA store (row-per-thread global stores would be 32 partial sectors
      // per instruction)
      if (j + 1 < N) {
        if (threadIdx.x == 0) bulk_wait_read0();
        named_sync(2, 256);
        uint8_t* panel = sm + OFF_SS + half * P128;
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4)
          *reinterpret_cast<uint4*>(panel + sw128_chunk(c, q4)) =
              make_uint4(ph[4 * q4], ph[4 * q4 + 1], ph[4 * q4 + 2], ph[4 * q4 + 3]);
        fence_async_smem();
        named_sync(2, 256);
        if (threadIdx.x == 0) {
          const int srow = (bh * N + j + 1) * kD;
          tma_store_2d(&tm_sh, 0, srow, sm + OFF_SS);
          tma_store_2d(&tm_sh, 64, srow, sm + OFF_SS + P128);
          bulk_commit();
        }
      }
    }
    // shared memory must outlive the reads of the bulk stores; grid completion
    // makes their global writes visible to the next kernel
    if (threadIdx.x == 0) bulk_wait_read0();
  } else {
    // ------------------------------------------------------------ chunk-local (warps 8-11)
    const int tb = threadIdx.x - 256;          // 0..127
    const int sp = warp - 8;                   // TMEM subpartition
    const uint32_t lb = tmem_lane_base(warp);
    const int row = sp * 32 + lane;            // TMEM lane of this thread
    const int t16 = sp * 16 + (lane & 15);     // M=64 row of lanes 0-15
    // P -> A' = tril(P) * beta / w (bf16): delta (w = beta) tril(P), adam (w = 1)
    // tril(P) * beta; A' must be free (o2(jj-1) done)
    auto build_as = [&](int jj) -> bool {
      const float* bs = gate_beta + (jj & 1) * 64;
      if (!wait_use_w(&bars->p_full, jj, status, ab)) return false;
      if (jj >= 1 && !wait_use_w(&bars->o_full, jj - 1, status, ab)) return false;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < 4; cc += 2) {
        float p0[16], p1[16];
        tmem_ld16(tmem + lb + TM_P + cc * 16, p0);
        tmem_ld16(tmem + lb + TM_P + cc * 16 + 16, p1);
        tmem_ld_wait();
        if (lane < 16) {
          float v8[8];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const float* src = h < 2 ? p0 + h * 8 : p1 + (h - 2) * 8;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int sc = cc * 16 + h * 8 + i;
              v8[i] = (sc <= t16) ? (RULE == 0 ? src[i] : src[i] * bs[sc]) : 0.f;
            }
            st_row8(sm + OFF_AS, P64, t16, cc * 2 + h, v8);
          }
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive_warp(&bars->as_full);
      return true;
    };
    bool ok = N > 0 && build_as(0);
    for (int j = 0; ok && j < N; ++j) {
      // E3: -E^T (lanes = value row c, 64 token columns) -> w E^T hi / lo, packed
      // bf16 pairs back into TMEM (the A operand of G and o2)
      if (!wait_use_w(&bars->e_full, j, status, ab)) break;
      if constexpr (kEWarps<RULE> == 4) {
      tc_fence_after();
      {
        const float* ws = gate_beta + (j & 1) * 64;   // delta: w = beta; adam: w = 1
        float x0[16], x1[16], x2[16], x3[16];
        tmem_ld16(tmem + lb + TM_E, x0);
        tmem_ld16(tmem + lb + TM_E + 16, x1);
        tmem_ld16(tmem + lb + TM_E + 32, x2);
        tmem_ld16(tmem + lb + TM_E + 48, x3);
        tmem_ld_wait();
        auto x = [&](int i) { return i < 16 ? x0[i] : i < 32 ? x1[i - 16] : i < 48 ? x2[i - 32] : x3[i - 48]; };
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          uint32_t hh[16], ll[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            const int s0 = b * 32 + 2 * t;
            const float e0 = RULE == 0 ? -x(s0) * ws[s0] : -x(s0);
            const float e1 = RULE == 0 ? -x(s0 + 1) * ws[s0 + 1] : -x(s0 + 1);
            hh[t] = pack_bf16(e0, e1);
            ll[t] = pack_bf16(e0 - bf16_lo(hh[t]), e1 - bf16_hi(hh[t]));
          }
          tmem_st16(tmem + lb + TM_WEH + b * 16, hh);
          tmem_st16(tmem + lb + TM_WEL + b * 16, ll);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      mbar_arrive_warp(&bars->e_smem);
      fence_async_smem();   // gate reads before the stage's reload (async proxy)
      mbar_arrive_warp(&bars->ld_empty[j & 1]);   // done with this stage's gates
      }
      if (j + 1 < N && !build_as(j + 1)) break;
      // E5: o^T (lanes = value column c, 64 token columns) -> staged o[t][c] -> TMA store
      if (!wait_use_w(&bars->o_full, j, status, ab)) break;
      tc_fence_after();
      if (tb == 0) bulk_wait_read0();        // previous store has left the staging tile
      named_sync(1, 128);
      {
        uint8_t* os = sm + OFF_OS + (row >> 6) * P64;
        const int ccol = row & 63;
        float x0[16], x1[16], x2[16], x3[16];
        tmem_ld16(tmem + lb + TM_O, x0);
        tmem_ld16(tmem + lb + TM_O + 16, x1);
        tmem_ld16(tmem + lb + TM_O + 32, x2);
        tmem_ld16(tmem + lb + TM_O + 48, x3);
        tmem_ld_wait();
        tc_fence_before();
        mbar_arrive_warp(&bars->o_empty);
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
        tma_store_2d(&tm_o, 0, orow, sm + OFF_OS);
        if (args.store_hi) tma_store_2d(&tm_o, 64, orow, sm + OFF_OS + P64);
        bulk_commit();
      }
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

// rows x width bf16 matrix, 64 x box_rows boxes, 128-byte swizzle.
cudaError_t make_tmap_rows128(CUtensorMap* map, const void* base, uint64_t rows,
                              uint32_t box_rows, uint32_t width) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  if (width != 64 && width != 128) return cudaErrorInvalidValue;
  cuuint64_t dims[2] = {width, rows};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(width) * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                  strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

bool tma_encode_available() { return encode_fn() != nullptr; }

bool chunk_fwd_tc_supported(const ChunkArgs& p) {
  return (p.rule == 0 || p.rule == 2) && (p.dh == kD || p.dh == 64) && p.C == kC && !p.io_f32 &&
         p.N >= 1 && encode_fn();
}

template <int RULE>
cudaError_t launch_fwd_tc(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                          const CUtensorMap& mo, const CUtensorMap& msh, const FwdArgs& a,
                          int grid, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(chunk_fwd_tc_kernel<RULE>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return e;
  chunk_fwd_tc_kernel<RULE><<<grid, kThreadsTc, SMEM_BYTES, st>>>(mq, mk, mv, mo, msh, a);
  return cudaGetLastError();
}

cudaError_t chunk_fwd_tc(const ChunkArgs& p, const TcBufs& b, cudaStream_t st) {
  CUtensorMap mq, mk, mv, mo, msh;
  const uint64_t rows = static_cast<uint64_t>(p.BH) * p.T;
  cudaError_t e;
  if ((e = make_tmap_rows128(&msh, b.S_hist, static_cast<uint64_t>(p.BH) * p.N * kD, 128)) !=
      cudaSuccess)
    return e;
  const uint32_t w = static_cast<uint32_t>(p.dh);
  if ((e = make_tmap_rows128(&mq, p.q, rows, 64, w)) != cudaSuccess) return e;
  if ((e = make_tmap_rows128(&mk, p.k, rows, 64, w)) != cudaSuccess) return e;
  if ((e = make_tmap_rows128(&mv, p.v, rows, 64, w)) != cudaSuccess) return e;
  if ((e = make_tmap_rows128(&mo, p.o, rows, 64, w)) != cudaSuccess) return e;
  FwdArgs a{};
  a.store_hi = p.dh == kD;
  a.beta = p.beta;
  a.alpha = p.alpha;
  a.mu = p.mu;
  a.nu = p.nu;
  a.S_hist = b.S_hist;
  a.G_hist = b.G_hist;
  a.Mp_hist = b.Mp_hist;
  a.Vp_hist = b.Vp_hist;
  a.M_ws = b.M_ws;
  a.V_ws = b.V_ws;
  a.status = b.status;
  a.N = p.N;
  a.T = p.T;
  if (p.rule == 2) {
    if (!p.nu || !b.G_hist || !b.Mp_hist || !b.Vp_hist || !b.M_ws || !b.V_ws)
      return cudaErrorInvalidValue;
    return launch_fwd_tc<2>(mq, mk, mv, mo, msh, a, p.BH, st);
  }
  return launch_fwd_tc<0>(mq, mk, mv, mo, msh, a, p.BH, st);
}

}  // namespace gmdn
