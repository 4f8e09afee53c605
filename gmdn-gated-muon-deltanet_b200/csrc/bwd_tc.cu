// Tensor-core backward of the mixer core, delta and adam rules, dh = 128, C = 64.
//
// The backward is written in the residual form of the chunk update: with
// E_j = v_j - k_j S_j^T (the errors of chunk j against the frozen state) the
// reference's G_j = Uv_j - S_j Kw_j (fast_scan.py:82, train_ablation.py:
// 164-165) equals E_j^T (w k_j), and o_j = Qt_j S_j^T + A_j v_j
// (train_ablation.py:166-167, 186) equals q_j S_j^T + A_j E_j.  Its chain
// rule gives, for the state cotangent Sb_{j+1} = dL/dS_{j+1}:
//
//   dE_j     = A_j^T dO_j + (w k_j) Sb_{j+1}^T
//   Sb_j     = a_j Sb_{j+1} + dO_j^T q_j - dE_j^T k_j
//   dv_j     = dE_j
//   dq_j     = dO_j S_j + dP_j k_j,            dP = tril(dO E^T) * beta_col
//   dk_j     = -dE_j S_j + w * (E_j Sb_{j+1}) + dP_j^T q_j
//   dbeta_s  = sum_t tril(dO E^T)[t][s] P[t][s] + k_s . (E_j Sb_{j+1})_s
//            = <E_j[s], dE_j[s]> / beta_s         (delta: both terms regroup)
//   dalpha_s = <Sb_{j+1}, S_j> a_j / alpha_s
//
// (identical to the reference's autograd of train_ablation.py:142-187 with
// fast_scan.py:72-95; checked against it in tests/).
//
// Adam (w = 1) replaces Sb_{j+1} in dE_j and dk_j by Gb_j, the cotangent of
// G_j, which the reverse chain forms per element from Sb_{j+1}, the moment
// cotangents Mb, Vb and the forward's G_j, M_j, V_j (fast_scan.py:168-182):
//
//   Mi = mu M_j + (1 - mu) G,  Vi = nu V_j + (1 - nu) G^2,  den = sqrt(Vi) + 1e-6
//   Mt = Mb + b Sb / den,      Vt = Vb - b Sb Mi / den^2 / (2 max(sqrt(Vi), 1e-12))
//   Gb = (1 - mu) Mt + 2 (1 - nu) G Vt,   Mb <- mu Mt,   Vb <- nu Vt
//   da_c = <Sb, S_j>, db_c = <Sb, Mi / den>, dmu_c = <Mt, M_j - G>, dnu_c = <Vt, V_j - G^2>
//
// bw1: one CTA per (b, h) walks the chunks in reverse and produces Gb_j
//      (= Sb_{j+1} for delta) for every chunk (bf16, for bw2).  The chain products use split bf16
//      (hi + lo) operands for Sb and dE; Sb hi/lo live in TMEM as the A
//      operand of their product, so the recurrence never touches shared
//      memory.
// bw2: persistent, one CTA per SM walking the (b, h, chunk) tiles; each tile's
//      token and gate gradients come from q, k, v, dO, S_j and Gb_j.

#include <cuda.h>

#include "common.cuh"
#include "fast_path.h"
#include "tc.cuh"

namespace gmdn {
namespace {

using namespace tc;

constexpr int kC = 64;
constexpr int kD = 128;
constexpr uint32_t P64 = 8192;
constexpr uint32_t P128 = 16384;
constexpr uint32_t HI16 = 16u << 16;

struct BwArgs {
  const float* beta;
  const float* alpha;
  const float *mu, *nu;
  uint16_t* Gbar_hist;
  const uint16_t* S_hist;
  const uint16_t *G_hist, *Mp_hist, *Vp_hist;  // adam
  float *M_ws, *V_ws;                          // adam: Mb, Vb slabs
  float *dac, *dbc, *dmc, *dnc;                // adam: chunk-scalar cotangents
  uint16_t *dq, *dk, *dv;
  float *dalpha, *dbeta, *dmu, *dnu;
  uint32_t* status;
  uint32_t* progress;   // fused backward: per (b, h), chunks (from the last) whose Gb_j is stored
  int N, T;
  int tiles;      // bw2: B * H * N
  int store_hi;   // dh 128: store the upper 64 columns of dq, dk, dv (dh 64: zero padding)
};

// ===========================================================================
// bw1: reverse chain
// ===========================================================================

// Fused backward: the chain publishes the Gb_j it has stored kPubLag steps
// after the store (waiting on the store's completion) and every kPubEvery
// steps: each publication is a proxy fence and a gpu-scope release on the
// chain's storing thread, ~0.6 us of the chain's time (publishing every step
// took the chains of 64 sequences from 0.18 to 0.22 ms; every 4 or 8 steps
// measured best).
constexpr int kPubLag = 1;
constexpr int kPubEvery = 8;

constexpr int kThreads1 = 448;  // warps 0-7 state, 8-11 chunk-local, 12 TMA + P, Z, 13 chain MMAs
// adam adds warp 14, which streams the forward's G, M, V history into a ring,
// and warp 15, which loads the S_j history tile of each adam pass
template <int RULE>
constexpr int kThreads1R = RULE == 2 ? kThreads1 + 64 : kThreads1;
constexpr int kStagesMax = 3;

// Shared-memory map of the reverse chain (bytes from a 1024-aligned base).
// q, k, dO come through a ring of kSt stages: delta's ~2.5 us step wants the
// load of step i+3 issued after step i (three stages).  Adam's step is ~10x
// longer, so two stages hide that load, and the space goes to what its adam
// pass reads per element: the S_j history tile (32 KB, SW128 panels like the
// Gb staging, loaded by TMA for each pass) and a ring of four 12 KB slots for
// the G, M, V history (one slot = one 8-column group: 3 arrays x 2 halves x
// 128 rows x 16 bytes).
template <int RULE>
struct L1 {
  static constexpr int kSt = RULE == 2 ? 2 : 3;
  static constexpr uint32_t Q = 0;                        // q: kSt stages x 16 KB
  static constexpr uint32_t K = Q + kSt * 16384;          // k
  static constexpr uint32_t G = K + kSt * 16384;          // dO
  static constexpr uint32_t AS = G + kSt * 16384;         // A' (bf16), 1 panel x 64 rows
  static constexpr uint32_t SS = AS + 8192;               // Gb hi staging, 2 panels x 128 rows
  static constexpr uint32_t GATE = SS + 32768;            // beta, alpha, mu, nu: kSt x 64 floats
  static constexpr uint32_t RED = GATE + kSt * 4 * 256;   // adam: per-warp partials [8][4]
  static constexpr uint32_t SH = (RED + 128 + 1023) / 1024 * 1024;   // adam: S_j tile
  static constexpr uint32_t HIST = SH + (RULE == 2 ? 32768 : 0);     // adam: the history ring
  static constexpr int kHist = RULE == 2 ? 4 : 0;
  static constexpr uint32_t HSLOT = 12288;
  static constexpr uint32_t BAR = HIST + kHist * HSLOT;
  static constexpr uint32_t SMEM = BAR + 512 + 1024;   // barrier block, alignment slack
  static_assert(SMEM <= 232448, "shared memory per block");
};

// TMEM: chain accumulator C, dE^T hi / lo (packed bf16 pairs, the A operand of
// C -= dE^T k), D = Gb k^T + dO^T A' (dE^T = D diag(w)), P (lanes 0-15), Gb hi
// and lo packed bf16 pairs (64 columns each = 128 values per lane).  The token
// weights are applied in the drain of D (A' = A / w), so no w k tile exists and
// the chain's operands other than the TMA-loaded tiles stay in TMEM.
constexpr uint32_t T1_C = 0, T1_DEH = 128, T1_DEL = 160, T1_E = 256, T1_P = 320, T1_SH = 384,
                   T1_SL = 448;
// adam: Sb_{j+1} (fp32, 128 values a lane) parked in columns 128-255 during
// the adam pass (dE^T hi / lo are dead from W's completion to the next dE
// drain, 192-255 are unused), so its 64 registers a thread are free for the
// pass's temporaries instead of spilling
constexpr uint32_t T1_STASH = 128;

// Who drains dE: the eight state warps (idle between packing Sb and W; two
// warps per TMEM subpartition drain in about half the time of one).  Delta's
// state warps stage the Gb history after the drain, from Sb hi in TMEM, so it
// overlaps W instead of delaying the drain.
template <int RULE>
constexpr int kDeWarps1 = 8;

struct Bars1 {
  uint64_t ld_full[kStagesMax], ld_empty[kStagesMax];
  uint64_t wk_full, p_full, as_full, de_full, de_smem;
  uint64_t c_full[2], c_empty[2];
  uint64_t s_full, final_mma, z_full, final_tma;
  uint64_t hist_full[4], hist_empty[4];   // adam
  uint64_t sh_full, sh_free;              // adam
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Bars1) <= 512, "barrier block");

// The reverse chain of sequence bh.  kPub (the fused backward, below): after
// each Gb_j store has completed, publish in args.progress[bh] how many chunks,
// counted from the last, have their Gb_j in memory (one step behind the
// stores, so the storing thread never waits on the one it just issued).
template <int RULE, bool kPub>
__device__ __forceinline__ void bw1_body(const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                                         const CUtensorMap& tm_g, const CUtensorMap& tm_sb,
                                         const CUtensorMap& tm_sh, const BwArgs& args, int bh) {
  using Lay = L1<RULE>;
  constexpr int kStages1 = Lay::kSt;
  constexpr uint32_t B1_Q = Lay::Q, B1_K = Lay::K, B1_G = Lay::G, B1_AS = Lay::AS, B1_SS = Lay::SS,
                     B1_GATE = Lay::GATE, B1_RED = Lay::RED, B1_BAR = Lay::BAR;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  Bars1* bars = reinterpret_cast<Bars1*>(sm + B1_BAR);
  float* gate_beta = reinterpret_cast<float*>(sm + B1_GATE);   // [kStages1][64] by ring stage
  float* gate_alpha = gate_beta + kStages1 * 64;
  float* gate_mu = gate_beta + 2 * kStages1 * 64;   // adam
  float* gate_nu = gate_beta + 3 * kStages1 * 64;   // adam
  volatile int* ab = &bars->abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = args.N;
  uint32_t* status = args.status;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages1; ++s) {
      mbar_init(&bars->ld_full[s], 1);
      // MMA commit after W, the warps that drain dE (and read the stage's gates)
      mbar_init(&bars->ld_empty[s], 1 + kDeWarps1<RULE>);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->c_full[s], 1);
      mbar_init(&bars->c_empty[s], 8);
    }
    mbar_init(&bars->p_full, 1);
    mbar_init(&bars->as_full, 4);
    mbar_init(&bars->de_full, 1);
    mbar_init(&bars->de_smem, kDeWarps1<RULE>);
    mbar_init(&bars->s_full, 8);
    mbar_init(&bars->final_mma, 1);
    mbar_init(&bars->z_full, 1);
    mbar_init(&bars->final_tma, 1);
    for (int s = 0; s < Lay::kHist; ++s) {
      mbar_init(&bars->hist_full[s], 1);
      mbar_init(&bars->hist_empty[s], 8);
    }
    mbar_init(&bars->sh_full, 1);
    mbar_init(&bars->sh_free, 8);
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

  constexpr uint32_t ID_P = idesc_bf16(64, 64, false, false);
  constexpr uint32_t ID_Z = idesc_bf16(128, 128, true, true);
  auto stage = [&](uint32_t base, int i) { return smem_u32(sm + base + (i % kStages1) * 16384); };
  if (warp == 12) {
    // ------------------------------------------------------------ TMA (reverse chunk order)
    // and the off-chain products P(i) = q k^T and Z(i): C = dO^T q.  An MMA issue
    // blocks its thread while the tensor pipe is busy, so these go from this
    // thread, each into a window where the pipe is otherwise idle (P(i+1) while
    // dE(i) is drained, Z(i+1) while Sb_j is packed), and the MMA thread issues
    // only the chain's products.
    if (lane == 0) {
      int issued = 0;
      auto load = [&](int i) -> bool {
        const int j = N - 1 - i, s = i % kStages1;
        const int row = static_cast<int>(tok0) + j * kC;
        if (!wait_free(&bars->ld_empty[s], i / kStages1, status, ab)) return false;
        mbar_expect_tx(&bars->ld_full[s], 6 * 8192 + 512 + (RULE == 2 ? 512 : 0));
        tma_load_2d(sm + B1_Q + s * 16384, &tm_q, 0, row, &bars->ld_full[s]);
        tma_load_2d(sm + B1_Q + s * 16384 + P64, &tm_q, 64, row, &bars->ld_full[s]);
        tma_load_2d(sm + B1_K + s * 16384, &tm_k, 0, row, &bars->ld_full[s]);
        tma_load_2d(sm + B1_K + s * 16384 + P64, &tm_k, 64, row, &bars->ld_full[s]);
        tma_load_2d(sm + B1_G + s * 16384, &tm_g, 0, row, &bars->ld_full[s]);
        tma_load_2d(sm + B1_G + s * 16384 + P64, &tm_g, 64, row, &bars->ld_full[s]);
        bulk_load(gate_beta + s * 64, args.beta + tok0 + j * kC, 256, &bars->ld_full[s]);
        bulk_load(gate_alpha + s * 64, args.alpha + tok0 + j * kC, 256, &bars->ld_full[s]);
        if (RULE == 2) {
          bulk_load(gate_mu + s * 64, args.mu + tok0 + j * kC, 256, &bars->ld_full[s]);
          bulk_load(gate_nu + s * 64, args.nu + tok0 + j * kC, 256, &bars->ld_full[s]);
        }
        issued = i + 1;
        return true;
      };
      auto issue_P = [&](int i) -> bool {
        if (!wait_use(&bars->ld_full[i % kStages1], i / kStages1, status, ab)) return false;
        tc_fence_after();
        #pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(tmem + T1_P, desc_kmajor(stage(B1_Q, i), P64, k),
                   desc_kmajor(stage(B1_K, i), P64, k), ID_P, k > 0);
        mma_commit(&bars->p_full);
        return true;
      };
      // C must have been drained (step i-1); ld_full(i) was waited for by issue_P(i)
      auto issue_Z = [&](int i) -> bool {
        if (i >= 1 && !wait_use(&bars->c_empty[0], i - 1, status, ab)) return false;
        tc_fence_after();
        #pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + T1_C, desc_mnmajor(stage(B1_G, i), P64, k),
                   desc_mnmajor(stage(B1_Q, i), P64, k), ID_Z, k > 0);
        mma_commit(&bars->z_full);
        return true;
      };
      // Per step i, in the order the inputs are released: P(i+1) once A'(i) has
      // been built from P(i) and X(i) has left the pipe, Z(i+1) once C(i) has
      // been drained (it runs while Sb is packed), then the load of step i+3
      // (its stage is free since W(i)).  Issuing the load first held Z(i+1)
      // back ~1,000 cycles, into the next step's chain products.
      bool ok = true;
      for (int i = 0; ok && i < kStages1 && i < N; ++i) ok = load(i);
      ok = ok && N > 0 && issue_P(0) && issue_Z(0);
      for (int i = 0; ok && i + 1 < N; ++i) {
        if (!wait_use(&bars->as_full, i, status, ab) || !wait_use(&bars->de_full, i, status, ab) ||
            !issue_P(i + 1))
          break;
        if (!issue_Z(i + 1)) break;
        if (i + kStages1 < N && !load(i + kStages1)) break;
      }
      // no MMA or copy of this thread may still be in flight when the CTA exits
      mma_commit(&bars->final_tma);
      int dummy = 0;
      mbar_wait(&bars->final_tma, 0, status, &dummy);
      for (int i = issued - kStages1; i < issued; ++i)
        if (i >= 0) mbar_wait(&bars->ld_full[i % kStages1], (i / kStages1) & 1, status, &dummy);
    }
  } else if (warp == 13) {
    // ------------------------------------------------------------ chain MMAs
    if (lane == 0) {
      const uint32_t as_s = smem_u32(sm + B1_AS);
      constexpr uint32_t ID_X = idesc_bf16(128, 64, true, true);
      constexpr uint32_t ID_Y = idesc_bf16(128, 64, false, false);
      constexpr uint32_t ID_W = idesc_bf16(128, 128, false, true, true);
      for (int i = 0; i < N; ++i) {
        const uint32_t k_s = stage(B1_K, i);
        // Y(i): D = Gb_hi k^T + Gb_lo k^T  (Gb from TMEM);  X(i): D += dO^T A'
        if (!wait_use(&bars->ld_full[i % kStages1], i / kStages1, status, ab) ||
            !wait_use(&bars->s_full, i, status, ab))
          break;
        tc_fence_after();
        #pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(tmem + T1_E, tmem + T1_SH + k * 8, desc_kmajor(k_s, P64, k), ID_Y, k > 0);
        #pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16_ts(tmem + T1_E, tmem + T1_SL + k * 8, desc_kmajor(k_s, P64, k), ID_Y, 1);
        if (!wait_use(&bars->as_full, i, status, ab)) break;
        tc_fence_after();
        #pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + T1_E, desc_mnmajor(stage(B1_G, i), P64, k),
                   desc_mnmajor(as_s, P64, k), ID_X, 1);
        mma_commit(&bars->de_full);
        // W(i): C -= dE^T_hi k + dE^T_lo k   (dE^T from TMEM; C = dO^T q from Z(i))
        if (!wait_use(&bars->de_smem, i, status, ab) || !wait_use(&bars->z_full, i, status, ab))
          break;
        tc_fence_after();
        #pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16_ts(tmem + T1_C, tmem + T1_DEH + k * 8, desc_mnmajor(k_s, P64, k), ID_W, 1);
        #pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16_ts(tmem + T1_C, tmem + T1_DEL + k * 8, desc_mnmajor(k_s, P64, k), ID_W, 1);
        mma_commit(&bars->c_full[0]);
        mma_commit(&bars->ld_empty[i % kStages1]);
      }
      mma_commit(&bars->final_mma);
      int dummy = 0;
      mbar_wait(&bars->final_mma, 0, status, &dummy);
    }
  } else if (warp == 14) {
    // ------------------------------------------------------------ adam: history ring
    // The state warps' adam pass of step i reads, per 8-column group, the
    // forward's G, M, V of chunk N - 2 - i; element loads from global memory
    // there put a DRAM round trip per group on the chain (~0.7 ms of a 1.9 ms
    // chain at config 3).  This thread bulk-copies the groups, in the order
    // the passes read them, into a ring of four slots, running half a pass
    // ahead while the chain does the rest of its step.
    if constexpr (RULE == 2) {
      if (lane == 0) {
        constexpr int kH = Lay::kHist;
        int n = 0;   // groups issued
        bool ok = true;
        for (int i = 0; ok && i + 1 < N; ++i) {
          const size_t mm = static_cast<size_t>(bh) * N + (N - 2 - i);
          for (int g = 0; g < 8; ++g, ++n) {
            const int slot = n % kH;
            if (!wait_free(&bars->hist_empty[slot], n / kH, status, ab)) {
              ok = false;
              break;
            }
            mbar_expect_tx(&bars->hist_full[slot], Lay::HSLOT);
            uint8_t* dst = sm + Lay::HIST + slot * Lay::HSLOT;
            const uint16_t* src[3] = {args.G_hist, args.Mp_hist, args.Vp_hist};
#pragma unroll
            for (int arr = 0; arr < 3; ++arr)
#pragma unroll
              for (int h = 0; h < 2; ++h)
                bulk_load(dst + arr * 4096 + h * 2048,
                          slab_bf16(const_cast<uint16_t*>(src[arr]), mm, h, g, 0), 2048,
                          &bars->hist_full[slot]);
          }
        }
        // no copy may still be in flight when the block exits
        int dummy = 0;
        for (int k = n - kH; k < n; ++k)
          if (k >= 0) mbar_wait(&bars->hist_full[k % kH], (k / kH) & 1, status, &dummy);
      }
    }
  } else if (warp == 15) {
    // ------------------------------------------------------------ adam: S_j history tile
    // The pass of step i reads <Sb_{j+1}, S_j> for chunk jm = N - 2 - i; row-
    // per-thread loads of S_j put a DRAM round trip per group on the chain.
    // The tile of pass i goes in as soon as pass i - 1 is done with it.
    if constexpr (RULE == 2) {
      if (lane == 0) {
        int n = 0;
        for (int i = 0; i + 1 < N; ++i, ++n) {
          if (!wait_free(&bars->sh_free, i, status, ab)) break;
          const int row = static_cast<int>((static_cast<size_t>(bh) * N + (N - 2 - i)) * kD);
          mbar_expect_tx(&bars->sh_full, 32768);
          tma_load_2d(sm + Lay::SH, &tm_sh, 0, row, &bars->sh_full);
          tma_load_2d(sm + Lay::SH + P128, &tm_sh, 64, row, &bars->sh_full);
        }
        int dummy = 0;
        if (n >= 1) mbar_wait(&bars->sh_full, (n - 1) & 1, status, &dummy);
      }
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ state cotangent rows
    const int c = (warp & 3) * 32 + lane;   // row of Sb = TMEM lane
    const int half = warp >> 2;             // columns [64 half, 64 half + 64)
    const uint32_t lb = tmem_lane_base(warp);
    float sb[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) sb[i] = 0.f;
    {
      uint32_t zr[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) zr[i] = 0u;
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        tmem_st16(tmem + lb + T1_SH + half * 32 + b * 16, zr);
        tmem_st16(tmem + lb + T1_SL + half * 32 + b * 16, zr);
      }
      tmem_st_wait();
      if (N > 0) {
        uint4* g = reinterpret_cast<uint4*>(
            args.Gbar_hist + (static_cast<size_t>(bh) * N + N - 1) * kD * kD +
            static_cast<size_t>(c) * kD + half * 64);
        const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int i = 0; i < 8; ++i) g[i] = z;
        if (RULE == 2 && threadIdx.x == 0) {
          const size_t last = static_cast<size_t>(bh) * N + N - 1;
          args.dac[last] = args.dbc[last] = args.dmc[last] = args.dnc[last] = 0.f;
        }
      }
    }
    tc_fence_before();
    mbar_arrive_warp(&bars->s_full);
    // Adam: Gb_jm, Mb, Vb and the chunk-scalar cotangents of chunk jm from
    // sb = Sb_{jm+1}; Gb_jm hi / lo go to TMEM for the next chain product and
    // Gb_jm hi to the history.  Works in 8-column groups to stay in registers.
    // (chunk jm = N - 1 - (i + 1) is step i + 1's: its gates are in that step's
    // ring stage, which these warps release only after step i + 1's dE drain)
    auto adam_pass = [&](int jm) -> bool {
      const size_t mm = static_cast<size_t>(bh) * N + jm;
      const int in = N - 1 - jm;
      if (!wait_use_w(&bars->ld_full[in % kStages1], in / kStages1, status, ab)) return false;
      const float* be = gate_beta + (in % kStages1) * 64;
      const float* mu = gate_mu + (in % kStages1) * 64;
      const float* nu = gate_nu + (in % kStages1) * 64;
      const float b = warp_sum(be[lane] + be[lane + 32]) * (1.f / kC);
      const float mc = expf(warp_sum(logf(fmaxf(mu[lane], kGateFloor)) +
                                     logf(fmaxf(mu[lane + 32], kGateFloor))));
      const float nc = expf(warp_sum(logf(fmaxf(nu[lane], kGateFloor)) +
                                     logf(fmaxf(nu[lane + 32], kGateFloor))));
      const bool have_bar = jm + 2 < N;   // Mb, Vb of chunk jm + 1 exist (else zero)
      const int pass = N - 2 - jm;
      if (!wait_use_w(&bars->sh_full, pass, status, ab)) return false;
      const uint8_t* stile = sm + Lay::SH + half * P128;   // S_j, row c, this half's panel
      float2 pda2 = p2(0.f), pdb2 = p2(0.f), pdm2 = p2(0.f), pdn2 = p2(0.f);
      // Mb, Vb of the next group load while this one computes (L2 round trips
      // one group ahead instead of on the chain)
      float4 nm0 = make_float4(0.f, 0.f, 0.f, 0.f), nm1 = nm0, nv0 = nm0, nv1 = nm0;
      if (have_bar) {
        const float4* mp0 = slab_f32(args.M_ws, bh, half, 0, c);
        const float4* vp0 = slab_f32(args.V_ws, bh, half, 0, c);
        nm0 = mp0[0];
        nm1 = mp0[128];
        nv0 = vp0[0];
        nv1 = vp0[128];
      }
      if (threadIdx.x == 0) bulk_wait_read0();
      named_sync(2, 256);
      uint8_t* panel = sm + B1_SS + half * P128;
#pragma unroll
      for (int g8 = 0; g8 < 8; ++g8) {
        float g[8], mp[8], vp[8], sv[8], mb[8], vb[8], gb[8];
        {
          // G, M, V of this group from the history ring (pass N - 2 - jm)
          constexpr int kH = Lay::kHist > 0 ? Lay::kHist : 1;
          const int n = (N - 2 - jm) * 8 + g8, slot = n % kH;
          if (!wait_use_w(&bars->hist_full[slot], n / kH, status, ab)) return false;
          const uint8_t* hb = sm + Lay::HIST + slot * Lay::HSLOT + half * 2048 + c * 16;
          unpack8(*reinterpret_cast<const uint4*>(hb), g);
          unpack8(*reinterpret_cast<const uint4*>(hb + 4096), mp);
          unpack8(*reinterpret_cast<const uint4*>(hb + 8192), vp);
          // the slot's next bulk copy (async proxy) must not overtake these reads
          fence_async_smem();
          mbar_arrive_warp(&bars->hist_empty[slot]);
        }
        unpack8(*reinterpret_cast<const uint4*>(stile + sw128_chunk(c, g8)), sv);
        if (g8 == 7) {   // S_j read out: the next pass's tile may load
          fence_async_smem();
          mbar_arrive_warp(&bars->sh_free);
        }
        float sbv[8];   // Sb_{j+1} of this group, from the TMEM stash
        tmem_ld8(tmem + lb + T1_STASH + half * 64 + 8 * g8, sbv);
        tmem_ld_wait();
        float4* mbp = slab_f32(args.M_ws, bh, half, 2 * g8, c);
        float4* vbp = slab_f32(args.V_ws, bh, half, 2 * g8, c);
        mb[0] = nm0.x; mb[1] = nm0.y; mb[2] = nm0.z; mb[3] = nm0.w;
        mb[4] = nm1.x; mb[5] = nm1.y; mb[6] = nm1.z; mb[7] = nm1.w;
        vb[0] = nv0.x; vb[1] = nv0.y; vb[2] = nv0.z; vb[3] = nv0.w;
        vb[4] = nv1.x; vb[5] = nv1.y; vb[6] = nv1.z; vb[7] = nv1.w;
        if (have_bar && g8 + 1 < 8) {
          nm0 = mbp[256];   // group g8 + 1: f = 2 g8 + 2 (two float4 rows on)
          nm1 = mbp[384];
          nv0 = vbp[256];
          nv1 = vbp[384];
        }
        // element pairs (tc.cuh p2 / fma2 / mul2): the pass is on the chain.
        // One reciprocal square root serves both sqrt(Vi) and 1 / max(sqrt(Vi),
        // 1e-12), one reciprocal 1 / (sqrt(Vi) + eps): two special-function ops
        // an element instead of an IEEE square root and four IEEE divisions.
#pragma unroll
        for (int t = 0; t < 8; t += 2) {
          const float2 sbar = p2(sbv[t], sbv[t + 1]);
          const float2 G = p2(g[t], g[t + 1]), Mp = p2(mp[t], mp[t + 1]), Vp = p2(vp[t], vp[t + 1]);
          const float2 GG = mul2(G, G);
          const float2 mi = fma2(p2(mc), Mp, mul2(p2(1.f - mc), G));
          const float2 vi = fma2(p2(nc), Vp, mul2(p2(1.f - nc), GG));
          const float rs0 = rsqrtf(vi.x), rs1 = rsqrtf(vi.y);   // +inf at 0
          const float2 root = p2(vi.x > 0.f ? vi.x * rs0 : 0.f, vi.y > 0.f ? vi.y * rs1 : 0.f);
          const float2 rden = p2(rcp_sfu(root.x + kEpsAdam), rcp_sfu(root.y + kEpsAdam));
          const float2 hr = mul2(p2(0.5f), p2(fminf(rs0, 1e12f), fminf(rs1, 1e12f)));
          const float2 mr = mul2(mi, rden);   // Mi / den
          pda2 = fma2(sbar, p2(sv[t], sv[t + 1]), pda2);
          pdb2 = fma2(sbar, mr, pdb2);
          const float2 ub = mul2(p2(b), sbar);
          const float2 mt = fma2(ub, rden, p2(mb[t], mb[t + 1]));
          const float2 vt = sub2(p2(vb[t], vb[t + 1]), mul2(mul2(mul2(ub, mr), rden), hr));
          pdm2 = fma2(mt, sub2(Mp, G), pdm2);
          pdn2 = fma2(vt, sub2(Vp, GG), pdn2);
          const float2 mbn = mul2(p2(mc), mt), vbn = mul2(p2(nc), vt);
          const float2 gbn = fma2(p2(1.f - mc), mt, mul2(mul2(p2(2.f * (1.f - nc)), G), vt));
          mb[t] = mbn.x;
          mb[t + 1] = mbn.y;
          vb[t] = vbn.x;
          vb[t + 1] = vbn.y;
          gb[t] = gbn.x;
          gb[t + 1] = gbn.y;
        }
        if (jm >= 1) {
          mbp[0] = make_float4(mb[0], mb[1], mb[2], mb[3]);
          mbp[128] = make_float4(mb[4], mb[5], mb[6], mb[7]);
          vbp[0] = make_float4(vb[0], vb[1], vb[2], vb[3]);
          vbp[128] = make_float4(vb[4], vb[5], vb[6], vb[7]);
        }
        const uint4 hh = pack8(gb);
        uint4 pl;
        pl.x = pack_bf16(gb[0] - bf16_lo(hh.x), gb[1] - bf16_hi(hh.x));
        pl.y = pack_bf16(gb[2] - bf16_lo(hh.y), gb[3] - bf16_hi(hh.y));
        pl.z = pack_bf16(gb[4] - bf16_lo(hh.z), gb[5] - bf16_hi(hh.z));
        pl.w = pack_bf16(gb[6] - bf16_lo(hh.w), gb[7] - bf16_hi(hh.w));
        tmem_st4(tmem + lb + T1_SH + half * 32 + g8 * 4, hh);
        tmem_st4(tmem + lb + T1_SL + half * 32 + g8 * 4, pl);
        *reinterpret_cast<uint4*>(panel + sw128_chunk(c, g8)) = hh;
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive_warp(&bars->s_full);
      float* red = reinterpret_cast<float*>(sm + B1_RED);
      const float pda = warp_sum(pda2.x + pda2.y);
      const float pdb = warp_sum(pdb2.x + pdb2.y);
      const float pdm = warp_sum(pdm2.x + pdm2.y);
      const float pdn = warp_sum(pdn2.x + pdn2.y);
      if (lane == 0) {
        red[warp * 4 + 0] = pda;
        red[warp * 4 + 1] = pdb;
        red[warp * 4 + 2] = pdm;
        red[warp * 4 + 3] = pdn;
      }
      fence_async_smem();
      named_sync(2, 256);
      if (threadIdx.x == 0) {
        const int hrow = (bh * N + jm) * kD;
        tma_store_2d(&tm_sb, 0, hrow, sm + B1_SS);
        tma_store_2d(&tm_sb, 64, hrow, sm + B1_SS + P128);
        bulk_commit();
        float t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          t0 += red[w * 4 + 0];
          t1 += red[w * 4 + 1];
          t2 += red[w * 4 + 2];
          t3 += red[w * 4 + 3];
        }
        args.dac[mm] = t0;
        args.dbc[mm] = t1;
        args.dmc[mm] = t2;
        args.dnc[mm] = t3;
      }
      return true;
    };
    for (int i = 0; i < N; ++i) {
      const int j = N - 1 - i;
      // chunk scalar a_j from the gates the TMA brought into this step's stage (a
      // global load here stalled the dE drain behind it)
      if (!wait_use_w(&bars->ld_full[i % kStages1], i / kStages1, status, ab)) break;
      const float* ga = gate_alpha + (i % kStages1) * 64;
      const float a = expf(warp_sum(logf(fmaxf(ga[lane], kGateFloor)) +
                                    logf(fmaxf(ga[lane + 32], kGateFloor))));
      if constexpr (kDeWarps1<RULE> == 8) {
        // dE^T = D diag(w) (delta: w = beta; adam: w = 1; lanes = value row c, this
        // warp's 32 token columns) -> packed bf16 hi / lo pairs into TMEM, the A
        // operand of C -= dE^T k
        if (!wait_use_w(&bars->de_full, i, status, ab)) break;
        tc_fence_after();
        const float* ws = gate_beta + (i % kStages1) * 64 + half * 32;
        float x0[16], x1[16];
        tmem_ld16(tmem + lb + T1_E + half * 32, x0);
        tmem_ld16(tmem + lb + T1_E + half * 32 + 16, x1);
        tmem_ld_wait();
        uint32_t hh[16], ll[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const float y0 = t < 8 ? x0[2 * t] : x1[2 * t - 16];
          const float y1 = t < 8 ? x0[2 * t + 1] : x1[2 * t - 15];
          const float e0 = RULE == 0 ? y0 * ws[2 * t] : y0;
          const float e1 = RULE == 0 ? y1 * ws[2 * t + 1] : y1;
          hh[t] = pack_bf16(e0, e1);
          ll[t] = pack_bf16(e0 - bf16_lo(hh[t]), e1 - bf16_hi(hh[t]));
        }
        tmem_st16(tmem + lb + T1_DEH + half * 16, hh);
        tmem_st16(tmem + lb + T1_DEL + half * 16, ll);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive_warp(&bars->de_smem);
        fence_async_smem();   // gate reads before the stage's reload (async proxy)
        mbar_arrive_warp(&bars->ld_empty[i % kStages1]);   // done with this stage
      }
      if constexpr (RULE == 0) {
        // history for bw2: Gb_j = Sb_{j+1} hi, packed in TMEM since the previous
        // step, through a staging tile and one TMA store (row N-1 is zero)
        if (i >= 1) {
          float f0[16], f1[16];
          tmem_ld16(tmem + lb + T1_SH + half * 32, f0);
          tmem_ld16(tmem + lb + T1_SH + half * 32 + 16, f1);
          tmem_ld_wait();
          if (threadIdx.x == 0) bulk_wait_read0();
          named_sync(2, 256);
          uint8_t* panel = sm + B1_SS + half * P128;
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) {
            const float* f = q4 < 4 ? f0 + 4 * q4 : f1 + 4 * (q4 - 4);
            *reinterpret_cast<uint4*>(panel + sw128_chunk(c, q4)) =
                make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                           __float_as_uint(f[3]));
          }
          fence_async_smem();
          named_sync(2, 256);
          if (threadIdx.x == 0) {
            const int srow = (bh * N + j) * kD;
            tma_store_2d(&tm_sb, 0, srow, sm + B1_SS);
            tma_store_2d(&tm_sb, 64, srow, sm + B1_SS + P128);
            bulk_commit();
            if constexpr (kPub) {
              // kPubLag steps behind: the stores of steps 1 .. i-kPubLag (chunks
              // N-2 .. N-1-i+kPubLag) are complete, and row N-1 was written before
              // the state warps' barriers above
              if (i >= kPubLag && i % kPubEvery == 0) {
                bulk_wait_n<kPubLag>();
                fence_proxy_async_global();
                st_release_gpu(args.progress + bh, static_cast<uint32_t>(i + 1 - kPubLag));
              }
            }
          }
        }
      }
      if (!wait_use_w(&bars->c_full[0], i, status, ab)) break;
      tc_fence_after();
      const uint32_t rc = tmem + lb + T1_C + half * 64;
      {
        float g0[16], g1[16], g2[16], g3[16];
        tmem_ld16(rc, g0);
        tmem_ld16(rc + 16, g1);
        tmem_ld16(rc + 32, g2);
        tmem_ld16(rc + 48, g3);
        tmem_ld_wait();
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          sb[t] = fmaf(a, sb[t], g0[t]);
          sb[16 + t] = fmaf(a, sb[16 + t], g1[t]);
          sb[32 + t] = fmaf(a, sb[32 + t], g2[t]);
          sb[48 + t] = fmaf(a, sb[48 + t], g3[t]);
        }
      }
      tc_fence_before();
      mbar_arrive_warp(&bars->c_empty[0]);
      if constexpr (RULE == 2) {
        if (j >= 1) {
          // park Sb_{j+1} in TMEM for the pass, take it back after
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t r[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) r[t] = __float_as_uint(sb[16 * q + t]);
            tmem_st16(tmem + lb + T1_STASH + half * 64 + 16 * q, r);
          }
          tmem_st_wait();
          if (!adam_pass(j - 1)) break;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float x[16];
            tmem_ld16(tmem + lb + T1_STASH + half * 64 + 16 * q, x);
            tmem_ld_wait();
#pragma unroll
            for (int t = 0; t < 16; ++t) sb[16 * q + t] = x[t];
          }
        }
      } else {
      // Sb_j as packed bf16 hi / lo pairs into TMEM (A operand of the next
      // chain product)
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        uint32_t pl[16], hh[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const float x0 = sb[b * 32 + 2 * t], x1 = sb[b * 32 + 2 * t + 1];
          hh[t] = pack_bf16(x0, x1);
          pl[t] = pack_bf16(x0 - bf16_lo(hh[t]), x1 - bf16_hi(hh[t]));
        }
        tmem_st16(tmem + lb + T1_SH + half * 32 + b * 16, hh);
        tmem_st16(tmem + lb + T1_SL + half * 32 + b * 16, pl);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive_warp(&bars->s_full);
      }
    }
    // shared memory must outlive the reads of the bulk stores; grid completion
    // makes their global writes visible to the next kernel
    if (threadIdx.x == 0) {
      if constexpr (kPub) {
        bulk_wait0();
        if (!*ab) {   // every Gb_j stored (an aborted chain publishes nothing more, so
                      // its readers give up on their bounded waits)
          fence_proxy_async_global();
          st_release_gpu(args.progress + bh, static_cast<uint32_t>(N));
        }
      } else {
        bulk_wait_read0();
      }
    }
  } else {
    // ------------------------------------------------------------ chunk-local (warps 8-11)
    const int sp = warp - 8;
    const uint32_t lb = tmem_lane_base(warp);
    const int t16 = sp * 16 + (lane & 15);
    auto build_as = [&](int i) -> bool {
      const float* bs = gate_beta + (i % kStages1) * 64;
      if (!wait_use_w(&bars->p_full, i, status, ab)) return false;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < 4; cc += 2) {
        float p0[16], p1[16];
        tmem_ld16(tmem + lb + T1_P + cc * 16, p0);
        tmem_ld16(tmem + lb + T1_P + cc * 16 + 16, p1);
        tmem_ld_wait();
        if (lane < 16) {
          float v8[8];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const float* src = h < 2 ? p0 + h * 8 : p1 + (h - 2) * 8;
#pragma unroll
            for (int x = 0; x < 8; ++x) {
              const int sc = cc * 16 + h * 8 + x;
              // A' = tril(P) beta / w: delta (w = beta) tril(P), adam tril(P) beta
              v8[x] = (sc <= t16) ? (RULE == 0 ? src[x] : src[x] * bs[sc]) : 0.f;
            }
            st_row8(sm + B1_AS, P64, t16, cc * 2 + h, v8);
          }
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive_warp(&bars->as_full);
      return true;
    };
    bool ok = N > 0 && build_as(0);
    for (int i = 0; ok && i < N; ++i) {
      // dE^T = D diag(w) (lanes = value row c, 64 token columns) -> packed bf16
      // hi / lo pairs into TMEM (the A operand of C -= dE^T k); adam's state
      // warps drain it instead, and A'(i+1) waits only for X(i)
      if (!wait_use_w(&bars->de_full, i, status, ab)) break;
      if constexpr (kDeWarps1<RULE> == 4) {
      tc_fence_after();
      {
        const float* ws = gate_beta + (i % kStages1) * 64;   // delta: w = beta; adam: w = 1
        float x0[16], x1[16], x2[16], x3[16];
        tmem_ld16(tmem + lb + T1_E, x0);
        tmem_ld16(tmem + lb + T1_E + 16, x1);
        tmem_ld16(tmem + lb + T1_E + 32, x2);
        tmem_ld16(tmem + lb + T1_E + 48, x3);
        tmem_ld_wait();
        auto x = [&](int t) { return t < 16 ? x0[t] : t < 32 ? x1[t - 16] : t < 48 ? x2[t - 32] : x3[t - 48]; };
#pragma unroll
        for (int b = 0; b < 2; ++b) {
          uint32_t hh[16], ll[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            const int s0 = b * 32 + 2 * t;
            const float e0 = RULE == 0 ? x(s0) * ws[s0] : x(s0);
            const float e1 = RULE == 0 ? x(s0 + 1) * ws[s0 + 1] : x(s0 + 1);
            hh[t] = pack_bf16(e0, e1);
            ll[t] = pack_bf16(e0 - bf16_lo(hh[t]), e1 - bf16_hi(hh[t]));
          }
          tmem_st16(tmem + lb + T1_DEH + b * 16, hh);
          tmem_st16(tmem + lb + T1_DEL + b * 16, ll);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      mbar_arrive_warp(&bars->de_smem);
      fence_async_smem();   // gate reads before the stage's reload (async proxy)
      mbar_arrive_warp(&bars->ld_empty[i % kStages1]);   // done with this stage's gates
      }
      if (i + 1 < N && !build_as(i + 1)) break;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int RULE>
__global__ void __launch_bounds__(kThreads1R<RULE>, 1)
chunk_bwd1_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_g, const __grid_constant__ CUtensorMap tm_sb,
                    const __grid_constant__ CUtensorMap tm_sh, BwArgs args) {
  bw1_body<RULE, false>(tm_q, tm_k, tm_g, tm_sb, tm_sh, args, static_cast<int>(blockIdx.x));
}

// ===========================================================================
// bw2: token and gate gradients of one chunk
// ===========================================================================
//
// Warps 0-7 drain accumulators (warp w reads TMEM subpartition w % 4; warps
// w and w + 4 split the columns), warp 8 issues the MMAs, warp 9 the TMA loads.
// Accumulators: E^T (M=128) feeds dA and dWk through MN-major descriptors;
// the outputs dq, dk, dv and the small C x C products are M=64 (row-major),
// paired two per TMEM column range (lanes 0-15 / 16-31).

constexpr int kThreads2 = 320;
// The fused backward runs where at least this many SMs are left beside the
// chains.  Measured (delta, T 4096, steps of one B200): 16, 32 and 64
// sequences 0.358 / 0.371 / 0.462 ms against 0.394 / 0.438 / 0.516 ms with
// the two plain launches; at 128 sequences (20 spare SMs) the fused launch
// was 3 % slower (the chains' publications cost more than 20 SMs return).
constexpr int kFusedMinWorkers = 32;
// a worker's share: kFusedNum / kFusedDen tiles per chain step (the best of
// 0.3 ... 0.6 at 64 sequences; larger shares outlast the chains)
constexpr int kFusedNum = 3, kFusedDen = 10;
// Muon token weights w_s = prod_{t>s} mu_t can underflow; A' = A / w uses
// max(w, kMuonWFloor), and the drain multiplies by the same value, so dE is
// exact up to (w_eff - w) k Gb^T, below 1e-28 |k Gb^T|.
constexpr float kMuonWFloor = 1e-30f;
constexpr uint32_t B2_Q = 0, B2_K = 16384, B2_V = 32768, B2_G = 49152;
constexpr uint32_t B2_ST0 = 65536;    // S_j and Gb_j, 2 panels x 128 rows each, in
constexpr uint32_t B2_ST1 = 98304;    // these two tiles with roles swapped every tile
constexpr uint32_t B2_AS = 131072;    // A bf16 [t][s]; then dk staging, panel 0
constexpr uint32_t B2_E = 139264;     // E^T bf16 [c][s], 1 panel x 128 rows; then dq staging
constexpr uint32_t B2_WK = 155648;    // delta, adam: q of odd local tiles (muon: unused)
constexpr uint32_t B2_DE = 172032;    // dE bf16 [s][c] (= dv, stored from here)
constexpr uint32_t B2_DP = 188416;    // dP bf16 [t][s]; then dk staging, panel 1
constexpr uint32_t B2_I = 196608;     // identity
constexpr uint32_t B2_RED = 204800;   // muon: Gb lo, panel 1; delta, adam: k of odd local tiles
constexpr uint32_t B2_GATE = 221440;  // 2 x {beta, alpha, mu, w}[64], 2 x dw[2][64], 2 x column-sum
                                      // partials [4][64] (by local tile parity), muon prefix sums [64]
constexpr uint32_t B2_BAR = 226816;
constexpr uint32_t B2_SMEM = B2_BAR + 256 + 1024;

// TMEM: X0 P | dA, XE E^T, X2 dE | dWk, and two regions D[0], D[1] holding dK
// (lanes 0-15) | dQ (lanes 16-31) of alternate tiles, so the next tile's phase 1
// can run while epilogue 3 still reads this tile's dq and dK.
constexpr uint32_t T2_X0 = 0, T2_XE = 64, T2_X2 = 128, T2_D0 = 256;

struct Bars2 {
  uint64_t ld_a, ld_v, ld_b[2], ld_sb, ph1a, ph1, ep1, wk_full, da_done, ph2, de_ready, ep2, s_free, ph3,
      x2_free, d_free[2], k_free, lo_full, tail_done, final_mma;
  uint32_t tmem_base;
  int abort_flag;
  float da[2];                 // by local tile parity: a tile's gate gradients are
  float a_c[2], m_c[2], n_c[2];   // written while the next tile runs
};
static_assert(sizeof(Bars2) <= 256, "barrier block");

// Persistent: CTA b handles tiles b, b + G, b + 2G, ... (tile = bh * N + chunk).
// Warp 9 issues every load, each input group of the next tile as soon as the
// current tile is done with the tiles it goes into: v once phase 1a has read
// it (delta, adam; muon keeps E^T lo in the v tile until phase 2 and loads v
// with dO), dO and S_j after phase 2 (and delta's da), Gb_j after -dE S.
// S_j and Gb_j swap their two tiles every tile, so the next S_j (needed first,
// by phase 1) goes into the current Gb_j tile a phase earlier than S_j's own
// tile frees.  q and k are double-buffered for delta and adam (the w k tile
// and the reduction array are not needed there), so the q, k of local tile
// i+2 load once tile i is done with its buffer; muon loads the next tile's q,
// k after phase 3.  Phase 1 runs the products that need no S_j (P, v^T I)
// first, so A is built while S_j arrives.  dq is staged in the E^T tile, dk in
// the A and dP tiles (one 64-column panel each) and dv is stored from the dE
// tile, so no input tile holds an output; the next tile's epilogue waits for
// the stores' reads only before it writes A and E^T.
// Delta and adam apply the token weight w to the rows of dE in its drain
// (delta: A = tril(P), dE = diag(beta) (A^T dO + k Gb^T); adam: w = 1), so
// k Gb^T is issued with phase 1 and runs while epilogue 1 drains; muon builds
// w * k (w_s = prod_{t>s} mu_t can underflow, so beta / w is no option).
// dbeta: delta takes it whole as the row product <E_s, dE_s / beta_s>; muon
// and adam reduce the column sums of tril(dA) * P across lanes with shuffles.
// Which tiles a bw2 CTA takes: entries e0 + w, e0 + w + W, ... below e1, w
// the CTA's index among the W workers (CTAs from worker0 on).  order 0: entry
// = tile (bh * N + j); order 1: the order in which the reverse chains finish
// Gb_j (chunk N-1 of every sequence, then N-2, ...).  progress (fused
// backward): a worker waits until the chain of a tile's sequence has
// published its Gb_j before loading it.
struct Sched2 {
  int e0, e1, worker0, BH, N, order;
  const uint32_t* progress;
  __device__ __forceinline__ int list_tile(int e) const {
    const int r = e / BH;   // r-th chunk from the last
    return (e - r * BH) * N + (N - 1 - r);
  }
};

// kMode (compile time, so the plain kernel carries none of the schedule):
// 0 every tile, entry = tile, CTA b takes b, b + grid, ...; 1 the entries
// sc.e0 .. sc.e1 - 1 in the chains' order (what the fused backward left);
// 2 a worker of the fused backward (waits for each tile's Gb_j).
template <int RULE, int kMode>
__device__ __forceinline__ void bw2_body(const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                                         const CUtensorMap& tm_v, const CUtensorMap& tm_g,
                                         const CUtensorMap& tm_s, const CUtensorMap& tm_sb,
                                         const CUtensorMap& tm_sbl, const CUtensorMap& tm_dq,
                                         const CUtensorMap& tm_dk, const CUtensorMap& tm_dv,
                                         const BwArgs& args, const Sched2& sc) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  Bars2* bars = reinterpret_cast<Bars2*>(sm + B2_BAR);
  float* gate0 = reinterpret_cast<float*>(sm + B2_GATE);   // [2][4][64]
  float* gdw0 = gate0 + 512;     // [2 tiles][2][64]: partial k.dWk of each column half
  float* gpart0 = gdw0 + 256;    // [2 tiles][4][64]: column sums of tril(dA) * P, 16-row groups
  float* gpre = gpart0 + 512;    // [64]: muon, sum_{u<s} dw_u w_u
  volatile int* ab = &bars->abort_flag;
  // q, k buffers: two for delta and adam (local tile i uses buffer i & 1)
  constexpr int kQK = RULE == 1 ? 1 : 2;
  auto qk_buf = [&](int i) { return kQK == 2 ? (i & 1) : 0; };
  auto qk_use = [&](int i) { return kQK == 2 ? (i >> 1) : i; };   // uses of that buffer before
  auto q_off = [&](int i) { return qk_buf(i) ? B2_WK : B2_Q; };
  auto k_off = [&](int i) { return qk_buf(i) ? B2_RED : B2_K; };
  // S_j and Gb_j of local tile i; tile i+1's S_j goes where tile i's Gb_j was
  // (free after phase 2) and its Gb_j where tile i's S_j was (free after -dE S)
  auto s_off = [&](int i) { return (i & 1) ? B2_ST1 : B2_ST0; };
  auto sb_off = [&](int i) { return (i & 1) ? B2_ST0 : B2_ST1; };
  auto d_tm = [&](int i) { return T2_D0 + static_cast<uint32_t>(i & 1) * 128u; };
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = args.N;
  // this CTA's entries: ew, ew + G, ... below `tiles` (tile_at maps them to tiles)
  const int tiles = kMode == 0 ? args.tiles : sc.e1;
  const int G = kMode == 2 ? static_cast<int>(gridDim.x) - sc.worker0 : static_cast<int>(gridDim.x);
  const int ew = kMode == 0 ? static_cast<int>(blockIdx.x)
                            : sc.e0 + static_cast<int>(blockIdx.x) - (kMode == 2 ? sc.worker0 : 0);
  auto tile_at = [&](int e) {
    if constexpr (kMode == 0) {
      return e;
    } else {
      return sc.list_tile(e);
    }
  };
  uint32_t* status = args.status;
  // gate buffer of local tile i: beta, alpha, mu, w
  auto gates = [&](int i) { return gate0 + (i & 1) * 256; };

  if (threadIdx.x == 0) {
    mbar_init(&bars->ld_a, 1);
    mbar_init(&bars->ld_v, 1);
    mbar_init(&bars->ld_b[0], 1);
    mbar_init(&bars->ld_b[1], 1);
    mbar_init(&bars->ld_sb, 1);
    mbar_init(&bars->ph1a, 1);
    mbar_init(&bars->ph1, 1);
    mbar_init(&bars->ep1, 8);
    mbar_init(&bars->wk_full, 8);
    mbar_init(&bars->ph2, 1);
    mbar_init(&bars->de_ready, 8);
    mbar_init(&bars->ep2, 8);
    mbar_init(&bars->s_free, 1);
    mbar_init(&bars->ph3, 1);
    mbar_init(&bars->k_free, 8);
    mbar_init(&bars->da_done, 8);
    mbar_init(&bars->x2_free, 8);
    mbar_init(&bars->d_free[0], 8);
    mbar_init(&bars->d_free[1], 8);
    mbar_init(&bars->lo_full, 1);
    mbar_init(&bars->tail_done, 1);
    mbar_init(&bars->final_mma, 1);
    bars->abort_flag = 0;
    bars->da[0] = bars->da[1] = 0.f;
    fence_mbar_init();
  }
  build_identity64(sm + B2_I, threadIdx.x, blockDim.x);
  if (warp == 8) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 9) {
    // ------------------------------------------------------------ TMA loads (one thread)
    // Each input group of the next tile is issued as soon as the current tile
    // releases the tiles it goes into, off the MMA thread (a copy issue blocks
    // its thread for a while, and on the MMA thread that delayed the chain).
    if (lane == 0) {
      // group a: dO, S_j and the gates (into tiles the previous tile's phase 2
      // has done with); muon also v (its v tile holds E^T lo until phase 2)
      auto issue_a = [&](int i, int tile) {
        const int bh = tile / N, j = tile % N;
        const int tok = bh * args.T + j * kC;
        const int srow = (bh * N + j) * kD;
        float* gt = gates(i);
        mbar_expect_tx(&bars->ld_a, (RULE == 1 ? 4 : 2) * 8192 + 2 * 16384 + 512 +
                                        (RULE == 1 ? 256 : 0));
        if (RULE == 1) {
          tma_load_2d(sm + B2_V, &tm_v, 0, tok, &bars->ld_a);
          tma_load_2d(sm + B2_V + P64, &tm_v, 64, tok, &bars->ld_a);
        }
        tma_load_2d(sm + B2_G, &tm_g, 0, tok, &bars->ld_a);
        tma_load_2d(sm + B2_G + P64, &tm_g, 64, tok, &bars->ld_a);
        tma_load_2d(sm + s_off(i), &tm_s, 0, srow, &bars->ld_a);
        tma_load_2d(sm + s_off(i) + P128, &tm_s, 64, srow, &bars->ld_a);
        bulk_load(gt, args.beta + tok, 256, &bars->ld_a);
        bulk_load(gt + 64, args.alpha + tok, 256, &bars->ld_a);
        if (RULE == 1) bulk_load(gt + 128, args.mu + tok, 256, &bars->ld_a);
      };
      // delta, adam: v alone, as soon as the previous tile's phase 1a has read it
      auto issue_v = [&](int tile) {
        const int bh = tile / N, j = tile % N;
        const int tok = bh * args.T + j * kC;
        mbar_expect_tx(&bars->ld_v, 2 * 8192);
        tma_load_2d(sm + B2_V, &tm_v, 0, tok, &bars->ld_v);
        tma_load_2d(sm + B2_V + P64, &tm_v, 64, tok, &bars->ld_v);
      };
      // group sb: Gb_j (into the tile the previous tile's -dE S has done with;
      // first read by k Gb^T after phase 1)
      auto issue_sb = [&](int i, int tile) {
        const int srow = tile * kD;   // tile = bh * N + j
        mbar_expect_tx(&bars->ld_sb, 2 * 16384);
        tma_load_2d(sm + sb_off(i), &tm_sb, 0, srow, &bars->ld_sb);
        tma_load_2d(sm + sb_off(i) + P128, &tm_sb, 64, srow, &bars->ld_sb);
      };
      // group b: q, k of local tile i into its buffer (read by phases 1 and 3; k also
      // by epilogue 2)
      auto issue_b = [&](int i, int tile) {
        const int bh = tile / N, j = tile % N;
        const int tok = bh * args.T + j * kC;
        uint64_t* bar = &bars->ld_b[qk_buf(i)];
        mbar_expect_tx(bar, 4 * 8192);
        tma_load_2d(sm + q_off(i), &tm_q, 0, tok, bar);
        tma_load_2d(sm + q_off(i) + P64, &tm_q, 64, tok, bar);
        tma_load_2d(sm + k_off(i), &tm_k, 0, tok, bar);
        tma_load_2d(sm + k_off(i) + P64, &tm_k, 64, tok, bar);
      };
      // muon: lo half of Gb_j into the dE tile and the reduction array (free
      // until epilogue 2 of the same tile)
      auto issue_lo = [&](int tile) {
        const int srow = tile * kD;   // tile = bh * N + j
        mbar_expect_tx(&bars->lo_full, 2 * 16384);
        tma_load_2d(sm + B2_DE, &tm_sbl, 0, srow, &bars->lo_full);
        tma_load_2d(sm + B2_RED, &tm_sbl, 64, srow, &bars->lo_full);
      };
      // local tile of a load group in flight, not yet waited on
      int pa = -1, ps = -1, pl = -1, pv = -1, pb[2] = {-1, -1};
      // fused backward: Gb_j of a tile is loaded only once its chain has published it
      auto ready = [&](int tile) -> bool {
        if constexpr (kMode != 2) return true;
        const uint32_t* pr = sc.progress + tile / N;
        const uint32_t need = static_cast<uint32_t>(N - tile % N);
        if (ld_acquire_gpu(pr) < need) {
          const uint64_t t0 = global_ns();
          while (ld_acquire_gpu(pr) < need) {
            if (*ab) return false;
            if (global_ns() - t0 > kWaitLimitNs) {
              *ab = 1;
              atomicOr(status, kStatusWaitTimeout);
              return false;
            }
            __nanosleep(200);
          }
        }
        fence_proxy_async_global();   // the TMA loads that follow read what was published
        return true;
      };
      bool started = false;
      if (ew < tiles) {
        const int t0 = tile_at(ew);
        if (RULE != 1) {
          issue_v(t0);
          pv = 0;
        }
        issue_a(0, t0);
        issue_b(0, t0);
        pa = pb[0] = 0;
        if (kQK == 2 && ew + G < tiles) {
          issue_b(1, tile_at(ew + G));
          pb[1] = 1;
        }
        if (ready(t0)) {
          issue_sb(0, t0);
          ps = 0;
          started = true;
        }
        if (RULE == 1) {
          issue_lo(t0);
          pl = 0;
        }
      }
      int i = 0;
      for (int e = ew; started && e < tiles; e += G, ++i) {
        const int ne = e + G;
        const int next = ne < tiles ? tile_at(ne) : 0;
        if (RULE != 1 && ne < tiles) {   // phase 1a has read v: the next tile's
          if (!wait_use(&bars->ph1a, i, status, ab)) break;
          issue_v(next);
          pv = i + 1;
        }
        if (ne < tiles) {
          // dO and Gb_j have been read (Gb_j also by da): the next tile's dO and S_j
          if (!wait_use(&bars->ph2, i, status, ab) || !wait_use(&bars->da_done, i, status, ab)) break;
          issue_a(i + 1, next);
          pa = i + 1;
          // S_j has been read by -dE S: the next tile's Gb_j into its tile
          if (!wait_use(&bars->s_free, i, status, ab) || !ready(next)) break;
          issue_sb(i + 1, next);
          ps = i + 1;
        }
        // q and k have been read (k also by epilogue 2): the q, k of the tile that
        // uses this buffer next
        const int nbe = e + kQK * G;
        if (nbe < tiles) {
          if (!wait_use(&bars->ph3, i, status, ab) || !wait_use(&bars->k_free, i, status, ab)) break;
          issue_b(i + kQK, tile_at(nbe));
          pb[qk_buf(i)] = i + kQK;
        }
        if (RULE == 1 && ne < tiles) {
          if (!wait_use(&bars->tail_done, i, status, ab)) break;
          issue_lo(next);
          pl = i + 1;
        }
      }
      // no copy of ours may still be in flight when the CTA exits
      int dummy = 0;
      if (pa >= 0) mbar_wait(&bars->ld_a, pa & 1, status, &dummy);
      if (pv >= 0) mbar_wait(&bars->ld_v, pv & 1, status, &dummy);
      for (int b = 0; b < 2; ++b)
        if (pb[b] >= 0) mbar_wait(&bars->ld_b[b], qk_use(pb[b]) & 1, status, &dummy);
      if (ps >= 0) mbar_wait(&bars->ld_sb, ps & 1, status, &dummy);
      if (pl >= 0) mbar_wait(&bars->lo_full, pl & 1, status, &dummy);
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ MMAs (one thread)
    if (lane == 0) {
      const uint32_t v_s = smem_u32(sm + B2_V), g_s = smem_u32(sm + B2_G);
      const uint32_t as_s = smem_u32(sm + B2_AS), e_s = smem_u32(sm + B2_E);
      const uint32_t de_s = smem_u32(sm + B2_DE);
      const uint32_t dp_s = smem_u32(sm + B2_DP), id_s = smem_u32(sm + B2_I);
      constexpr uint32_t ID_P = idesc_bf16(64, 64, false, false);
      constexpr uint32_t ID_KM = idesc_bf16(64, 128, false, true);        // A K-major, B MN-major
      constexpr uint32_t ID_KK = idesc_bf16(64, 128, false, false);       // both K-major
      constexpr uint32_t ID_KMN = idesc_bf16(64, 128, false, true, true);
      constexpr uint32_t ID_MM = idesc_bf16(64, 128, true, true);         // both MN-major
      constexpr uint32_t ID_EV = idesc_bf16(128, 64, true, false);        // E^T: v^T I
      constexpr uint32_t ID_EK = idesc_bf16(128, 64, false, false, true); // E^T: -S k^T
      constexpr uint32_t ID_DA = idesc_bf16(64, 64, false, true);         // dO E^T
      int i = 0;
      for (int e = ew; e < tiles; e += G, ++i) {
        const uint32_t q_s = smem_u32(sm + q_off(i)), k_s = smem_u32(sm + k_off(i));
        const uint32_t s_s = smem_u32(sm + s_off(i)), sb_s = smem_u32(sm + sb_off(i));
        if (RULE == 1 && !wait_use(&bars->ld_a, i, status, ab)) break;
        if (!wait_use(&bars->ld_b[qk_buf(i)], qk_use(i), status, ab)) break;
        // P overwrites X0: muon and adam read tile i-1's P and dA there for the
        // dbeta column sums until epilogue 2 arrives on k_free (delta's dbeta
        // needs no P)
        if (RULE != 0 && i >= 1 && !wait_use(&bars->k_free, i - 1, status, ab)) break;
        tc_fence_after();
        // phase 1a (no S_j): P = q k^T; E^T = v^T
        #pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(tmem + T2_X0, desc_kmajor(q_s, P64, k), desc_kmajor(k_s, P64, k), ID_P, k > 0);
        if (RULE != 1) {
          if (!wait_use(&bars->ld_v, i, status, ab)) break;
          tc_fence_after();
        }
        #pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + T2_XE, desc_mnmajor(v_s, P64, k), desc_kmajor(id_s, P64, k), ID_EV, k > 0);
        mma_commit(&bars->ph1a);
        // phase 1b: E^T -= S k^T; dQ = dO S into D[i & 1] (epilogue 3 of tile i-2 has
        // read it)
        if (RULE != 1 && !wait_use(&bars->ld_a, i, status, ab)) break;
        if (i >= 2 && !wait_use(&bars->d_free[i & 1], (i >> 1) - 1, status, ab)) break;
        tc_fence_after();
        #pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(tmem + T2_XE, desc_kmajor(s_s, P128, k), desc_kmajor(k_s, P64, k), ID_EK, 1);
        #pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(tmem + HI16 + d_tm(i), desc_kmajor(g_s, P64, k), desc_mnmajor(s_s, P128, k),
                   ID_KM, k > 0);
        mma_commit(&bars->ph1);
        if (!wait_use(&bars->ld_sb, i, status, ab)) break;
        // X2 (dE | dWk) is written next: epilogue 3 of tile i-1 has read dWk
        if (i >= 1 && !wait_use(&bars->x2_free, i - 1, status, ab)) break;
        tc_fence_after();
        if constexpr (RULE != 1) {
          // delta, adam: the k Gb^T part of dE needs no epilogue output (w is applied
          // to the rows of dE in its drain), so it runs while epilogue 1 drains
          #pragma unroll
          for (int k = 0; k < 8; ++k)
            mma_bf16(tmem + T2_X2, desc_kmajor(k_s, P64, k), desc_kmajor(sb_s, P128, k), ID_KK, k > 0);
        }
        if (!wait_use(&bars->ep1, i, status, ab)) break;
        if (RULE == 1 && i >= 1 && !wait_use(&bars->x2_free, i - 1, status, ab)) break;
        if (RULE == 1 && !wait_use(&bars->wk_full, i, status, ab)) break;
        if (RULE == 1 && !wait_use(&bars->lo_full, i, status, ab)) break;
        tc_fence_after();
        // phase 2: dE = diag(w) (A'^T dO + k Gb^T);  dA = dO E^T;  dWk = E Gb
        #pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + T2_X2, desc_mnmajor(as_s, P64, k), desc_mnmajor(g_s, P64, k), ID_MM,
                   RULE != 1 || k > 0);
        if constexpr (RULE == 1) {
          const uint32_t sbl_s = smem_u32(sm + B2_DE);   // panels 32 KB apart (dE tile, B2_RED)
          #pragma unroll
          for (int k = 0; k < 8; ++k)
            mma_bf16(tmem + T2_X2, desc_kmajor(k_s, P64, k), desc_kmajor(sb_s, P128, k), ID_KK, 1);
          #pragma unroll
          for (int k = 0; k < 8; ++k)
            mma_bf16(tmem + T2_X2, desc_kmajor(k_s, P64, k), desc_kmajor(sbl_s, B2_RED - B2_DE, k),
                     ID_KK, 1);
        }
        #pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(tmem + HI16 + T2_X0, desc_kmajor(g_s, P64, k), desc_mnmajor(e_s, P128, k), ID_DA,
                   k > 0);
        #pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(tmem + HI16 + T2_X2, desc_mnmajor(e_s, P128, k), desc_mnmajor(sb_s, P128, k),
                   ID_MM, k > 0);
        if constexpr (RULE == 1) {
          const uint32_t sbl_s = smem_u32(sm + B2_DE);
          const uint32_t el_s = smem_u32(sm + B2_V);
          #pragma unroll
          for (int k = 0; k < 8; ++k)
            mma_bf16(tmem + HI16 + T2_X2, desc_mnmajor(e_s, P128, k),
                     desc_mnmajor(sbl_s, B2_RED - B2_DE, k), ID_MM, 1);
          #pragma unroll
          for (int k = 0; k < 8; ++k)
            mma_bf16(tmem + HI16 + T2_X2, desc_mnmajor(el_s, P128, k), desc_mnmajor(sb_s, P128, k),
                     ID_MM, 1);
        }
        mma_commit(&bars->ph2);
        if (!wait_use(&bars->de_ready, i, status, ab)) break;
        tc_fence_after();
        // phase 3: dK = -dE S (S_j's last reader, as soon as dE is in shared memory)
        // + dP^T q;  dq += dP k
        #pragma unroll
        for (int k = 0; k < 8; ++k)
          mma_bf16(tmem + d_tm(i), desc_kmajor(de_s, P64, k), desc_mnmajor(s_s, P128, k), ID_KMN,
                   k > 0);
        mma_commit(&bars->s_free);
        if (!wait_use(&bars->ep2, i, status, ab)) break;
        tc_fence_after();
        #pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + d_tm(i), desc_mnmajor(dp_s, P64, k), desc_mnmajor(q_s, P64, k), ID_MM, 1);
        #pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16(tmem + HI16 + d_tm(i), desc_kmajor(dp_s, P64, k), desc_mnmajor(k_s, P64, k), ID_KM,
                   1);
        mma_commit(&bars->ph3);
      }
      // every MMA issued has completed before TMEM is released
      mma_commit(&bars->final_mma);
      int dummy = 0;
      mbar_wait(&bars->final_mma, 0, status, &dummy);
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ epilogue warps 0-7
    const int tid = threadIdx.x;               // 0..255
    const int sp = warp & 3, half = warp >> 2; // subpartition, column half
    const uint32_t lb = tmem_lane_base(warp);
    const bool hi = lane >= 16;
    const int r16 = sp * 16 + (lane & 15);     // M=64 row of this lane's accumulator
    const int c128 = sp * 32 + lane;           // M=128 row (TMEM lane)
    // Gate gradients of local tile li (tile tl), run while the next tile's phase 2
    // is in the pipe (the epilogue is idle then): its gate loads, column sums, dw
    // and chunk scalars are kept by tile parity until the next tile's da_done.
    auto gate_stage = [&](int li, int tl) {
      const int bh = tl / N, j = tl % N;
      const size_t tok = static_cast<size_t>(bh) * args.T + static_cast<size_t>(j) * kC;
      const float* gbeta = gates(li);
      const float* galpha = gbeta + 64;
      const float* gmu = gbeta + 128;
      const float* gw = gbeta + 192;
      const float* gdw = gdw0 + (li & 1) * 128;
      const float* gpart = gpart0 + (li & 1) * 256;
      (void)gbeta;
      (void)gmu;
      (void)gw;
      // muon: exclusive prefix sums of dw_u w_u by one warp
      {
        if constexpr (RULE == 1) {
          if (warp == 0) {
            const float x0 = (gdw[2 * lane] + gdw[64 + 2 * lane]) * gw[2 * lane];
            const float x1 = (gdw[2 * lane + 1] + gdw[65 + 2 * lane]) * gw[2 * lane + 1];
            float incl = x0 + x1;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const float y = __shfl_up_sync(0xffffffffu, incl, o);
              if (lane >= o) incl += y;
            }
            const float excl = incl - x0 - x1;   // tokens < 2 lane
            gpre[2 * lane] = excl;
            gpre[2 * lane + 1] = excl + x0;
          }
        }
      }
      named_sync(1, 256);
      if (tid < kC) {
        const int s = tid;
        // column sums of tril(dA) * P (muon, adam; delta's whole dbeta is in gdw)
        const float db =
            RULE == 0 ? 0.f : gpart[s] + gpart[64 + s] + gpart[128 + s] + gpart[192 + s];
        const float al = galpha[s];
        const size_t g = tok + s;
        if constexpr (RULE == 1) {
          // b_c = mean(beta); a_c, mu_c products; w_u = prod_{t>u} mu_t adds
          // dmu_s += sum_{u<s} dw_u w_u / mu_s
          const size_t gi = static_cast<size_t>(bh) * N + j;
          args.dbeta[g] = db + args.dbc[gi] * (1.f / kC);
          args.dalpha[g] =
              (al >= kGateFloor) ? args.dac[gi] * bars->a_c[li & 1] / fmaxf(al, kGateFloor) : 0.f;
          const float mu = gmu[s];
          float dmu = 0.f;
          if (mu >= kGateFloor) dmu = (args.dmc[gi] * bars->m_c[li & 1] + gpre[s]) / fmaxf(mu, kGateFloor);
          args.dmu[g] = dmu;
          if (args.dnu) args.dnu[g] = 0.f;
        } else if constexpr (RULE == 2) {
          // chunk scalars: b_c = mean(beta), a_c / mu_c / nu_c = prod of the clamped gates
          const size_t gi = static_cast<size_t>(bh) * N + j;
          args.dbeta[g] = db + args.dbc[gi] * (1.f / kC);
          args.dalpha[g] =
              (al >= kGateFloor) ? args.dac[gi] * bars->a_c[li & 1] / fmaxf(al, kGateFloor) : 0.f;
          const float mu = __ldg(args.mu + g), nu = __ldg(args.nu + g);
          args.dmu[g] = (mu >= kGateFloor) ? args.dmc[gi] * bars->m_c[li & 1] / fmaxf(mu, kGateFloor) : 0.f;
          args.dnu[g] = (nu >= kGateFloor) ? args.dnc[gi] * bars->n_c[li & 1] / fmaxf(nu, kGateFloor) : 0.f;
        } else {
          args.dbeta[g] = db + gdw[s] + gdw[64 + s];
          args.dalpha[g] =
              (al >= kGateFloor) ? bars->da[li & 1] * bars->a_c[li & 1] / fmaxf(al, kGateFloor) : 0.f;
          args.dmu[g] = 0.f;
          if (args.dnu) args.dnu[g] = 0.f;
        }
      }
    };
    int i = 0;
    for (int e = ew; e < tiles; e += G, ++i) {
      const int tile = tile_at(e);
      const int bh = tile / N, j = tile % N;
      const size_t tok = static_cast<size_t>(bh) * args.T + static_cast<size_t>(j) * kC;
      float* gbeta = gates(i);
      float* galpha = gbeta + 64;
      float* gmu = gbeta + 128;
      float* gw = gbeta + 192;
      float* gdw = gdw0 + (i & 1) * 128;
      float* gpart = gpart0 + (i & 1) * 256;
      const uint32_t k_tile = k_off(i);
      // the gate gradients of two tiles back are done with this parity's da
      named_sync(1, 256);
      if (tid == 0) bars->da[i & 1] = 0.f;
      named_sync(1, 256);
      if (!wait_use_w(&bars->ld_a, i, status, ab) ||
          !wait_use_w(&bars->ld_b[qk_buf(i)], qk_use(i), status, ab))
        break;
      if constexpr (RULE == 1) {  // w_s = exp(sum_{t>s} log clamp(mu_t)), log-space suffix sums
        if (warp == 0) {
          const float l0 = logf(fmaxf(gmu[2 * lane], kGateFloor));
          const float l1 = logf(fmaxf(gmu[2 * lane + 1], kGateFloor));
          float sfx = l0 + l1;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_down_sync(0xffffffffu, sfx, o);
            if (lane + o < 32) sfx += y;
          }
          gw[2 * lane] = expf(sfx - l0);
          gw[2 * lane + 1] = expf(sfx - l0 - l1);
        }
        named_sync(1, 256);
      }
      if constexpr (RULE == 1) {
        // w is ready for epilogues 1 and 2 (every rule applies w to the rows of dE
        // in its drain instead of multiplying it into k: w k rounded to bf16 would
        // break the cancellation in w k Gb^T, |Gb| ~ 50 against ~0.1)
        mbar_arrive_warp(&bars->wk_full);
      }
      if (warp == 0) {  // chunk decay product a_c = prod clamp(alpha)
        const float la = logf(fmaxf(galpha[lane], kGateFloor)) +
                         logf(fmaxf(galpha[lane + 32], kGateFloor));
        const float sum = warp_sum(la);
        if (lane == 0) bars->a_c[i & 1] = expf(sum);
      }
      if ((RULE == 2 && (warp == 1 || warp == 2)) || (RULE == 1 && warp == 1)) {  // mu_c, nu_c
        const float* gsrc = (warp == 1 ? args.mu : args.nu) + tok;
        const float lg = logf(fmaxf(__ldg(gsrc + lane), kGateFloor)) +
                         logf(fmaxf(__ldg(gsrc + lane + 32), kGateFloor));
        const float sum = warp_sum(lg);
        if (lane == 0) (warp == 1 ? bars->m_c : bars->n_c)[i & 1] = expf(sum);
      }
      // ---- epilogue 1: A = tril(P) (delta) or tril(P) beta (lanes 0-15) once P is
      // done, then E^T -> bf16 (all lanes)
      if (!wait_use_w(&bars->ph1a, i, status, ab)) break;
      // the previous tile's stores have read their staging (E^T, A, dP, dE tiles)
      if (tid == 0) bulk_wait_read0();
      named_sync(1, 256);
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c0 = half * 32 + cc * 16;
        float p[16];
        tmem_ld16(tmem + lb + T2_X0 + c0, p);
        tmem_ld_wait();
        if (!hi) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float v8[8];
#pragma unroll
            for (int x = 0; x < 8; ++x) {
              const int sc = c0 + h * 8 + x;
              // A' = tril(P) beta / w: delta (w = beta) tril(P); muon tril(P) beta / w
              // (w floored, see kMuonWFloor); adam (w = 1) tril(P) beta
              v8[x] = (sc <= r16) ? (RULE == 0   ? p[h * 8 + x]
                                     : RULE == 1 ? p[h * 8 + x] * gbeta[sc] *
                                                       rcp_sfu(fmaxf(gw[sc], kMuonWFloor))
                                                 : p[h * 8 + x] * gbeta[sc])
                                  : 0.f;
            }
            st_row8(sm + B2_AS, P64, r16, (c0 >> 3) + h, v8);
          }
        }
      }
      if (!wait_use_w(&bars->ph1, i, status, ab)) break;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c0 = half * 32 + cc * 16;
        float e[16];
        tmem_ld16(tmem + lb + T2_XE + c0, e);
        tmem_ld_wait();
        st_row8(sm + B2_E, P128, c128, c0 >> 3, e);
        st_row8(sm + B2_E, P128, c128, (c0 >> 3) + 1, e + 8);
        if constexpr (RULE == 1) {
          // muon: E^T lo into the v tile (v's last reader was phase 1), so E Gb
          // keeps ~16 bits against a large Gb
          float lo[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) lo[t] = e[t] - __bfloat162float(__float2bfloat16_rn(e[t]));
          st_row8(sm + B2_V, P128, c128, c0 >> 3, lo);
          st_row8(sm + B2_V, P128, c128, (c0 >> 3) + 1, lo + 8);
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive_warp(&bars->ep1);
      if (i >= 1) gate_stage(i - 1, tile_at(e - G));
      if constexpr (RULE == 0) {
        if (!wait_use_w(&bars->ld_sb, i, status, ab)) break;
        // da = <Sb_{j+1}, S_j> while phase 2 runs (phase 1 is bound by shared-memory
        // reads): row c128, column half `half` (adam, muon: from the chain)
        float part = 0.f;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          float a8[8], b8[8];
          unpack8(ld_row8(sm + s_off(i), P128, c128, half * 8 + c8), a8);
          unpack8(ld_row8(sm + sb_off(i), P128, c128, half * 8 + c8), b8);
#pragma unroll
          for (int x = 0; x < 8; ++x) part = fmaf(a8[x], b8[x], part);
        }
        part = warp_sum(part);
        if (lane == 0) atomicAdd(&bars->da[i & 1], part);
      }
      fence_async_smem();   // Gb_j, gate reads before the group's reload (async proxy)
      mbar_arrive_warp(&bars->da_done);
      // ---- epilogue 2: dE -> bf16 (also dv), then dP = tril(dA) beta; dbeta pieces; dw
      if (!wait_use_w(&bars->ph2, i, status, ab)) break;
      tc_fence_after();
      // X2: dE (lanes 0-15; delta: times beta_s, muon: times w_s), row s = r16,
      // 64 columns
      const float wde = RULE == 0 ? gbeta[r16] : RULE == 1 ? fmaxf(gw[r16], kMuonWFloor) : 1.f;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int c0 = half * 64 + cc * 16;
        float x[16];
        tmem_ld16(tmem + lb + T2_X2 + c0, x);
        tmem_ld_wait();
        if (!hi) {
          if constexpr (RULE != 2) {
#pragma unroll
            for (int y = 0; y < 16; ++y) x[y] *= wde;
          }
          st_row8(sm + B2_DE, P64, r16, c0 >> 3, x);
          st_row8(sm + B2_DE, P64, r16, (c0 >> 3) + 1, x + 8);
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive_warp(&bars->de_ready);   // -dE S may start (S_j's last reader)
      // X0: P (lanes 0-15) and dA (lanes 16-31) of the same row t = r16
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c0 = half * 32 + cc * 16;
        float x[16];
        tmem_ld16(tmem + lb + T2_X0 + c0, x);
        tmem_ld_wait();
        if (hi) {  // x = dA row t
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float v8[8];
#pragma unroll
            for (int y = 0; y < 8; ++y) {
              const int sc = c0 + h * 8 + y;
              v8[y] = (sc <= r16) ? x[h * 8 + y] * gbeta[sc] : 0.f;
            }
            st_row8(sm + B2_DP, P64, r16, (c0 >> 3) + h, v8);
          }
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive_warp(&bars->ep2);
      named_sync(1, 256);
      if (tid == 0) {   // dv = dE, straight from the dE tile
        tma_store_2d(&tm_dv, 0, static_cast<int>(tok), sm + B2_DE);
        if (args.store_hi) tma_store_2d(&tm_dv, 64, static_cast<int>(tok), sm + B2_DE + P64);
        bulk_commit();
      }
      // dbeta's A part: column sums over t of tril(dA) * P, off the critical path
      // (phase 3 runs).  Lanes 16-31 hold dA row t = r16 (P row t from lane - 16);
      // the 16 rows of a warp are summed by a butterfly over lanes 16-31 that
      // leaves each lane two of the warp's 32 column sums.  X0 stays valid until
      // the next tile's phase 1.
      if constexpr (RULE == 0) {
        // Delta: X2 (lanes 0-15) = A^T dO + k Gb^T before the beta scaling, and
        // dbeta_s = sum_t tril(dA)[t,s] P[t,s] + k_s . (E Gb)_s = <E_s, X2_s>: both
        // pieces regroup into that row product (E^T from shared memory).  X2 is
        // intact until epilogue 3 releases it.
        float dbp = 0.f;
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          const int c0 = half * 64 + cc * 16;
          float x[16];
          tmem_ld16(tmem + lb + T2_X2 + c0, x);
          tmem_ld_wait();
          if (!hi) {
#pragma unroll
            for (int y = 0; y < 16; ++y) {
              const float e = __bfloat162float(
                  *reinterpret_cast<const __nv_bfloat16*>(sm + B2_E + sw128_elem(c0 + y, r16)));
              dbp = fmaf(e, x[y], dbp);
            }
          }
        }
        if (!hi) gdw[half * 64 + r16] = dbp;
        // epilogue 3 stages dq in the E^T tile: every warp is done reading E^T first
        named_sync(1, 256);
      } else {
        float v[32];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int c0 = half * 32 + cc * 16;
          float x[16];
          tmem_ld16(tmem + lb + T2_X0 + c0, x);
          tmem_ld_wait();
#pragma unroll
          for (int y = 0; y < 16; ++y) {
            const float other = __shfl_xor_sync(0xffffffffu, x[y], 16);
            v[cc * 16 + y] = (hi && c0 + y <= r16) ? x[y] * other : 0.f;
          }
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int m = 8 >> r, n = 16 >> r;   // lane bit exchanged, values kept
          const bool up = (lane & m) != 0;
#pragma unroll
          for (int k = 0; k < n; ++k) {
            const float send = up ? v[k] : v[n + k];
            const float keep = up ? v[n + k] : v[k];
            v[k] = keep + __shfl_xor_sync(0xffffffffu, send, m);
          }
        }
        if (hi) {
          const int col = half * 32 + ((lane & 8) ? 16 : 0) + ((lane & 4) ? 8 : 0) +
                          ((lane & 2) ? 4 : 0) + ((lane & 1) ? 2 : 0);
          gpart[sp * 64 + col] = v[0];
          gpart[sp * 64 + col + 1] = v[1];
        }
      }
      if constexpr (RULE == 1) {
        // dw_s = k_s . dWk_s (lanes 16-31 of X2, row s = r16), read before k is reloaded
        float dw = 0.f;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int c0 = half * 64 + cc * 16;
          float x[16];
          tmem_ld16(tmem + lb + T2_X2 + c0, x);
          tmem_ld_wait();
          if (hi) {
            float k8[8];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              unpack8(ld_row8(sm + k_tile, P64, r16, (c0 >> 3) + h), k8);
#pragma unroll
              for (int y = 0; y < 8; ++y) dw = fmaf(k8[y], x[h * 8 + y], dw);
            }
          }
        }
        if (hi) gdw[half * 64 + r16] = dw;
      }
      fence_async_smem();   // k reads before the buffer's reload (async proxy)
      mbar_arrive_warp(&bars->k_free);
      // ---- epilogue 3: dq (staged in the E^T tile), dk (A and dP tiles), gate gradients
      if (!wait_use_w(&bars->ph3, i, status, ab)) break;
      tc_fence_after();
      const float w = RULE == 0 ? gbeta[r16] : RULE == 1 ? gw[r16] : 1.f;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        const int c0 = half * 64 + cc * 16;
        float x13[16], x2[16];
        tmem_ld16(tmem + lb + d_tm(i) + c0, x13);   // dq at lanes 16-31, dK part at lanes 0-15
        tmem_ld16(tmem + lb + T2_X2 + c0, x2);      // dWk at lanes 16-31
        tmem_ld_wait();
        if (cc == 3) {   // later tiles' products may overwrite X2 and D[i & 1] now
          tc_fence_before();
          mbar_arrive_warp(&bars->x2_free);
          mbar_arrive_warp(&bars->d_free[i & 1]);
        }
        float dwk[16];
#pragma unroll
        for (int y = 0; y < 16; ++y) dwk[y] = __shfl_xor_sync(0xffffffffu, x2[y], 16);
        if (hi) {
          st_row8(sm + B2_E, P64, r16, c0 >> 3, x13);
          st_row8(sm + B2_E, P64, r16, (c0 >> 3) + 1, x13 + 8);
        } else {
#pragma unroll
          for (int y = 0; y < 16; ++y) x13[y] = fmaf(w, dwk[y], x13[y]);
          st_row8(sm + B2_AS, B2_DP - B2_AS, r16, c0 >> 3, x13);
          st_row8(sm + B2_AS, B2_DP - B2_AS, r16, (c0 >> 3) + 1, x13 + 8);
        }
      }
      fence_async_smem();
      named_sync(1, 256);
      if (tid == 0) {
        tma_store_2d(&tm_dq, 0, static_cast<int>(tok), sm + B2_E);
        if (args.store_hi) tma_store_2d(&tm_dq, 64, static_cast<int>(tok), sm + B2_E + P64);
        tma_store_2d(&tm_dk, 0, static_cast<int>(tok), sm + B2_AS);
        if (args.store_hi) tma_store_2d(&tm_dk, 64, static_cast<int>(tok), sm + B2_DP);
        bulk_commit();
      }
      if constexpr (RULE == 1) {
        // the dE tile (read by the dv store) is free for the next Gb lo
        fence_async_smem();
        named_sync(1, 256);
        if (tid == 0) {
          bulk_wait_read0();
          mbar_arrive(&bars->tail_done);
        }
      }
    }
    if (i >= 1 && !*ab) gate_stage(i - 1, tile_at(ew + (i - 1) * G));
    // shared memory must outlive the reads of the bulk stores; grid completion
    // makes their global writes visible to the next kernel
    if (tid == 0) bulk_wait_read0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int RULE, int kMode>
__global__ void __launch_bounds__(kThreads2, 1)
chunk_bwd2_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_g,
                    const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_sb,
                    const __grid_constant__ CUtensorMap tm_sbl,
                    const __grid_constant__ CUtensorMap tm_dq, const __grid_constant__ CUtensorMap tm_dk,
                    const __grid_constant__ CUtensorMap tm_dv, BwArgs args, Sched2 sc) {
  bw2_body<RULE, kMode>(tm_q, tm_k, tm_v, tm_g, tm_s, tm_sb, tm_sbl, tm_dq, tm_dk, tm_dv, args,
                        sc);
}

// Fused backward (delta): CTAs 0 .. BH-1 run the reverse chains, publishing
// how far each has stored Gb_j; the other CTAs compute the token gradients of
// the chunks the chains have finished, in the order they finish, each waiting
// (bounded) for its tile's Gb_j.  With fewer sequences than SMs the chains
// leave SMs idle, and this puts the token gradients there while the chains
// run; a plain bw2 launch takes the tiles left after it.  A cooperative
// launch: all CTAs are resident at once, so no worker waits on a chain that
// has not been scheduled.  The chain's maps are the token kernel's q, k, dO,
// Gb and S maps.
template <int RULE>
__global__ void __launch_bounds__(kThreads1R<RULE>, 1)
chunk_bwd_fused_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                          const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v,
                          const __grid_constant__ CUtensorMap tm_g,
                          const __grid_constant__ CUtensorMap tm_s,
                          const __grid_constant__ CUtensorMap tm_sb,
                          const __grid_constant__ CUtensorMap tm_sbl,
                          const __grid_constant__ CUtensorMap tm_dq,
                          const __grid_constant__ CUtensorMap tm_dk,
                          const __grid_constant__ CUtensorMap tm_dv, BwArgs args, Sched2 sc) {
  if (static_cast<int>(blockIdx.x) < sc.worker0)
    bw1_body<RULE, true>(tm_q, tm_k, tm_g, tm_sb, tm_s, args, static_cast<int>(blockIdx.x));
  else
    bw2_body<RULE, 2>(tm_q, tm_k, tm_v, tm_g, tm_s, tm_sb, tm_sbl, tm_dq, tm_dk, tm_dv, args, sc);
}

}  // namespace

bool chunk_bwd_tc_supported(const ChunkArgs& p) { return chunk_fwd_tc_supported(p); }

namespace {

BwArgs bw_args(const ChunkArgs& p, const TcBufs& b) {
  BwArgs a{};
  a.beta = p.beta;
  a.alpha = p.alpha;
  a.mu = p.mu;
  a.nu = p.nu;
  a.Gbar_hist = b.Gbar_hist;
  a.S_hist = b.S_hist;
  a.G_hist = b.G_hist;
  a.Mp_hist = b.Mp_hist;
  a.Vp_hist = b.Vp_hist;
  a.M_ws = b.M_ws;
  a.V_ws = b.V_ws;
  a.dac = b.dac;
  a.dbc = b.dbc;
  a.dmc = b.dmc;
  a.dnc = b.dnc;
  a.dq = static_cast<uint16_t*>(p.dq);
  a.dk = static_cast<uint16_t*>(p.dk);
  a.dv = static_cast<uint16_t*>(p.dv);
  a.dalpha = p.dalpha;
  a.dbeta = p.dbeta;
  a.dmu = p.dmu;
  a.dnu = p.dnu;
  a.status = b.status;
  a.progress = b.progress;
  a.N = p.N;
  a.T = p.T;
  a.store_hi = p.dh == kD;
  return a;
}

bool adam_bufs_ok(const ChunkArgs& p, const TcBufs& b) {
  return p.nu && b.G_hist && b.Mp_hist && b.Vp_hist && b.M_ws && b.V_ws && b.dac && b.dbc &&
         b.dmc && b.dnc;
}

template <int RULE>
cudaError_t launch_bw1(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mg,
                       const CUtensorMap& msb, const CUtensorMap& msh, const BwArgs& a, int grid,
                       cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(chunk_bwd1_tc_kernel<RULE>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, L1<RULE>::SMEM);
  if (e != cudaSuccess) return e;
  chunk_bwd1_tc_kernel<RULE><<<grid, kThreads1R<RULE>, L1<RULE>::SMEM, st>>>(mq, mk, mg, msb, msh,
                                                                               a);
  return cudaGetLastError();
}

cudaError_t sm_count(int* sms) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev);
  return e;
}

// bw2 is persistent: one CTA per SM (it needs all of the SM's shared memory)
// walks its entries with a stride of the grid size.  first > 0: the entries
// left by the fused backward (readiness order from `first` on).
template <int RULE, int kMode>
cudaError_t launch_bw2_mode(const CUtensorMap* m, BwArgs a, int BH, int N, int first,
                            cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(chunk_bwd2_tc_kernel<RULE, kMode>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, B2_SMEM);
  if (e != cudaSuccess) return e;
  int sms = 0;
  if ((e = sm_count(&sms)) != cudaSuccess) return e;
  const int tiles = BH * N;
  a.tiles = tiles;
  const Sched2 sc{first, tiles, 0, BH, N, first > 0 ? 1 : 0, nullptr};
  const int left = tiles - first;
  if (left <= 0) return cudaSuccess;
  const int grid = sms < left ? sms : left;
  chunk_bwd2_tc_kernel<RULE, kMode><<<grid, kThreads2, B2_SMEM, st>>>(
      m[0], m[1], m[2], m[3], m[4], m[5], m[6], m[7], m[8], m[9], a, sc);
  return cudaGetLastError();
}

template <int RULE>
cudaError_t launch_bw2(const CUtensorMap* m, BwArgs a, int BH, int N, int first, cudaStream_t st) {
  return first > 0 ? launch_bw2_mode<RULE, 1>(m, a, BH, N, first, st)
                   : launch_bw2_mode<RULE, 0>(m, a, BH, N, first, st);
}

// The token maps of bw2 (and the fused backward): q, k, v, dO, S_j, Gb_j,
// Gb_j lo (muon; else Gb_j again), dq, dk, dv
cudaError_t bw2_maps(const ChunkArgs& p, const TcBufs& b, CUtensorMap* m) {
  const uint64_t rows = static_cast<uint64_t>(p.BH) * p.T;
  const uint64_t srows = static_cast<uint64_t>(p.BH) * p.N * kD;
  const void* lo = (p.rule == 1 && b.Gbar_lo_hist) ? b.Gbar_lo_hist : b.Gbar_hist;
  const void* base[10] = {p.q, p.k, p.v, p.dO, b.S_hist, b.Gbar_hist, lo, p.dq, p.dk, p.dv};
  for (int i = 0; i < 10; ++i) {
    const bool hist = i >= 4 && i <= 6;
    cudaError_t e = make_tmap_rows128(&m[i], base[i], hist ? srows : rows, hist ? 128 : 64,
                                      hist ? 128u : static_cast<uint32_t>(p.dh));
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

cudaError_t chunk_bwd1_tc(const ChunkArgs& p, const TcBufs& b, cudaStream_t st) {
  CUtensorMap mq, mk, mg, msb, msh;
  const uint64_t rows = static_cast<uint64_t>(p.BH) * p.T;
  const uint64_t srows = static_cast<uint64_t>(p.BH) * p.N * kD;
  cudaError_t e;
  const uint32_t w = static_cast<uint32_t>(p.dh);
  if ((e = make_tmap_rows128(&mq, p.q, rows, 64, w)) != cudaSuccess) return e;
  if ((e = make_tmap_rows128(&mk, p.k, rows, 64, w)) != cudaSuccess) return e;
  if ((e = make_tmap_rows128(&mg, p.dO, rows, 64, w)) != cudaSuccess) return e;
  if ((e = make_tmap_rows128(&msb, b.Gbar_hist, srows, 128)) != cudaSuccess) return e;
  if ((e = make_tmap_rows128(&msh, b.S_hist, srows, 128)) != cudaSuccess) return e;   // adam's pass
  const BwArgs a = bw_args(p, b);
  if (p.rule == 2) {
    if (!adam_bufs_ok(p, b)) return cudaErrorInvalidValue;
    return launch_bw1<2>(mq, mk, mg, msb, msh, a, p.BH, st);
  }
  return launch_bw1<0>(mq, mk, mg, msb, msh, a, p.BH, st);
}

cudaError_t chunk_bwd2_tc(const ChunkArgs& p, const TcBufs& b, cudaStream_t st, int first) {
  CUtensorMap m[10];
  cudaError_t e = bw2_maps(p, b, m);
  if (e != cudaSuccess) return e;
  const BwArgs a = bw_args(p, b);
  if (p.rule == 2) {
    if (!adam_bufs_ok(p, b) || !p.dnu) return cudaErrorInvalidValue;
    return launch_bw2<2>(m, a, p.BH, p.N, first, st);
  }
  if (p.rule == 1) {
    if (!b.dac || !b.dbc || !b.dmc || !b.Gbar_lo_hist) return cudaErrorInvalidValue;
    return launch_bw2<1>(m, a, p.BH, p.N, first, st);
  }
  return launch_bw2<0>(m, a, p.BH, p.N, first, st);
}

int chunk_bwd_fused_tiles(const ChunkArgs& p) {
  int sms = 0;
  if (p.rule != 0 || p.N <= 0 || sm_count(&sms) != cudaSuccess) return 0;
  const int workers = sms - p.BH;
  if (workers < kFusedMinWorkers) return 0;
  const int per_worker = (p.N * kFusedNum + kFusedDen - 1) / kFusedDen;
  const long long n = static_cast<long long>(workers) * per_worker;
  const long long tiles = static_cast<long long>(p.BH) * p.N;
  return static_cast<int>(n < tiles ? n : tiles);
}

cudaError_t chunk_bwd_fused_tc(const ChunkArgs& p, const TcBufs& b, int n_fused,
                               cudaStream_t st) {
  if (p.rule != 0 || !b.progress || n_fused <= 0) return cudaErrorInvalidValue;
  CUtensorMap m[10];
  cudaError_t e = bw2_maps(p, b, m);
  if (e != cudaSuccess) return e;
  int sms = 0;
  if ((e = sm_count(&sms)) != cudaSuccess) return e;
  const uint32_t smem = L1<0>::SMEM > B2_SMEM ? L1<0>::SMEM : B2_SMEM;
  e = cudaFuncSetAttribute(chunk_bwd_fused_tc_kernel<0>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  if ((e = cudaMemsetAsync(b.progress, 0, sizeof(uint32_t) * p.BH, st)) != cudaSuccess) return e;
  BwArgs a = bw_args(p, b);
  a.tiles = p.BH * p.N;
  const Sched2 sc{0, n_fused, p.BH, p.BH, p.N, 1, b.progress};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(sms));
  cfg.blockDim = dim3(kThreads1R<0>);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, chunk_bwd_fused_tc_kernel<0>, m[0], m[1], m[2], m[3], m[4], m[5],
                         m[6], m[7], m[8], m[9], a, sc);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace gmdn
