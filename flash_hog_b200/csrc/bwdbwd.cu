// Attention double backward (vjp of the attention vjp) on sm_100a.
//
// Two launches, no atomics, no (Nq, Nk) intermediate in global memory:
//
//  * query-tiled pass (`bwdbwd_q_kernel`): one CTA per 128 query rows of one
//    (batch, head). It streams the key side (K, V, ddK, ddV) twice. The first
//    sweep forms the row statistics
//        dD = rowsum(ddS o P),  r1 = rowsum(dO ddV^T o P),  r2 = rowsum(dP o P),
//        r3 = rowsum(dP o ddS o P),  B = r1 - dD r2 - D dD + r3,
//    the second forms dS, dS2, ddP and P and accumulates
//        dQ' = dS ddK + dS2 K,   ddO = ddP V + P ddV.
//    dD and B are written to caller-provided scratch for the second pass.
//    (Stats sweep merged as in flash_hog/csrc/tk_bwdbwd/stage1.cuh:187-195,231-237;
//    per-element formulas of flash_hog/jax/_pallas_gpu_kernel.py:149-278.)
//  * key-tiled pass (`bwdbwd_k_kernel`): one CTA per 128 key rows. It works on
//    transposed scores (S^T = K Q^T, as flash_hog/csrc/tk_bwdbwd/stage2.cuh:172-178)
//    so each thread owns a key row, streams the query side with its per-query
//    statistics (L, D, dD, B) and accumulates
//        dK' = dS^T ddQ + dS2^T Q,   dV' = ddP^T dO
//    (flash_hog/jax/_pallas_gpu_kernel.py:309-416).
//
// Per kept (q, k) pair the two passes issue 14 + 8 = 22 bf16 GEMM-equivalents on
// the tensor cores (tcgen05.mma, fp32 accumulation in TMEM).

#include <cuda_runtime.h>

#include <cmath>

#include "kernels.h"
#include "ws_common.cuh"

namespace fh {
namespace {

struct BBArgs {
  AttnShape sh;
  const float* lse;
  const float* delta;  // D = rowsum(dO o): read by both passes
  float* delta_out;    // non-null: the query pass computes D from o and writes it here (= delta)
  float* dd;
  float* bv;
  __nv_bfloat16* dq2;
  __nv_bfloat16* ddo;
  __nv_bfloat16* dk2;
  __nv_bfloat16* dv2;
  int* status;
  int grp_q;  // query pass: (query head, batch) pairs per locality group (grouped_order)
  int grp_k;  // key pass: (key head, batch) pairs per locality group
};

// ----------------------------------------------------------------------------------
// query-tiled pass
// ----------------------------------------------------------------------------------

template <int HD>
struct QPass {
  // Key rows per streamed tile and ring depth: 64 x 4 at head_dim 64; 32 x 3 at
  // 128, where accumulators of 2 x 128 columns leave TMEM room for 32-key scores.
  static constexpr int BN = HD == 64 ? 64 : 32;
  static constexpr int ST = HD == 64 ? 4 : 3;
  static constexpr int CW = BN / 2;                // columns of a tile per elementwise thread
  static constexpr int RES = kBM * HD * 2;         // one resident bf16 tile (panels of 128 rows)
  static constexpr int RES_PANEL = kBM * 128;
  static constexpr int STR = BN * HD * 2;          // one streamed bf16 tile
  static constexpr int PAIR = 2 * STR;             // two streamed tiles as pair panels
  static constexpr int PAIR_PANEL = 2 * BN * 128;
  static constexpr int SLOT = 2 * PAIR;            // (K | ddK) pair, (V | ddV) pair
  static constexpr int SMEM = 1024 + 3 * RES + ST * SLOT;  // Q, dO, ddQ, ring (O borrows the last slot)
  // TMEM: score buffer 0 [0, 256); accumulators dQ', ddO; bf16 operands dS,
  // dS2, ddP, P (BN/2 packed columns each). During the stats sweep the
  // accumulator and operand columns hold score buffer 1.
  static constexpr int C_S = 0, C_DDS = BN, C_DP = 2 * BN, C_DPA = 3 * BN, SCORE_COLS = 4 * BN;
  static constexpr int C_DQ = SCORE_COLS, C_DDO = SCORE_COLS + HD, C_OPS = SCORE_COLS + 2 * HD;
  static constexpr int OPS_COLS = BN / 2;
  // head_dim 128: ddQ as packed bf16 in TMEM (HD/2 columns after the operands), the A
  // operand of ddS += ddQ K^T as a TS product that reads only K from shared memory (the
  // SS form with 32-key tiles is bound by shared-memory reads: 40 cycles a k-step
  // against 16 of math).
  static constexpr bool DDQ_T = HD == 128;
  static constexpr int C_DDQ = C_OPS + 4 * OPS_COLS;
  static constexpr int TMEM_COLS = 512;
  static_assert(C_DDQ + (DDQ_T ? HD / 2 : 0) <= TMEM_COLS, "TMEM budget");
  static_assert(2 * SCORE_COLS <= (DDQ_T ? C_DDQ : TMEM_COLS), "stats sweep double-buffers the scores");
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(CW % 16 == 0 && HD % 64 == 0, "tile shapes");
};

// Stats sweep: row partial sums over this thread's CW columns. dD and r3 are
// accumulated without the softmax scale of ddS (applied once per row after the
// sweep): dD/scale += P ddS', r1 += P dPa, r2 += P dP, r3/scale += P ddS' dP.
// The arithmetic runs on column pairs with the packed fp32x2 instructions
// (fma/mul/add.rn.f32x2: per lane the same IEEE results as the scalar forms, one
// issue slot for two), so the sums are kept as (even, odd) column pairs.
template <int CW, bool MASK>
__device__ __forceinline__ void q_stats(const uint32_t (&vs)[CW], const uint32_t (&vdds)[CW],
                                        const uint32_t (&vdp)[CW], const uint32_t (&vdpa)[CW], int kc, int klo,
                                        int khi, float sc2, float lg, float2& dD, float2& r1, float2& r2,
                                        float2& r3) {
  const float2 m = make_float2(sc2, sc2), nl = make_float2(-lg, -lg);
#pragma unroll
  for (int i = 0; i < CW; i += 2) {
    float2 s = __ffma2_rn(f2(vs[i], vs[i + 1]), m, nl);
    if (MASK) {
      if (kc + i > khi || kc + i < klo) s.x = -INFINITY;
      if (kc + i + 1 > khi || kc + i + 1 < klo) s.y = -INFINITY;
    }
    const float2 p = make_float2(ex2(s.x), ex2(s.y));
    const float2 dp = f2(vdp[i], vdp[i + 1]);
    const float2 t = __fmul2_rn(f2(vdds[i], vdds[i + 1]), p);
    dD = __fadd2_rn(dD, t);
    r3 = __ffma2_rn(t, dp, r3);
    r1 = __ffma2_rn(f2(vdpa[i], vdpa[i + 1]), p, r1);
    r2 = __ffma2_rn(dp, p, r2);
  }
}

// Second sweep: packed bf16 pairs of dS/scale, dS2/scale, ddP and P for this
// thread's CW columns (the softmax scale of dS and dS2 is applied to dQ' in
// the epilogue instead of per element). With u = ddS - dD and c = dD D + B,
//   ddP = P u,  dS/scale = P (dP - D),
//   dS2/scale = P (dPa + dP u - ddS D - B) = P (dPa - c) + ddP (dP - D).
// Column pairs go through the packed fp32x2 instructions, as in q_stats.
template <int CW, bool MASK>
__device__ __forceinline__ void q_ops(const uint32_t (&vs)[CW], const uint32_t (&vdds)[CW],
                                      const uint32_t (&vdp)[CW], const uint32_t (&vdpa)[CW], int kc, int klo, int khi,
                                      float sc, float sc2, float lg, float dv, float dD, float cq,
                                      uint32_t (&o_ds)[CW / 2], uint32_t (&o_ds2)[CW / 2], uint32_t (&o_ddp)[CW / 2],
                                      uint32_t (&o_p)[CW / 2]) {
  const float2 m = make_float2(sc2, sc2), nl = make_float2(-lg, -lg), msc = make_float2(sc, sc);
  const float2 ndd = make_float2(-dD, -dD), ndv = make_float2(-dv, -dv), ncq = make_float2(-cq, -cq);
#pragma unroll
  for (int i = 0; i < CW; i += 2) {
    float2 s = __ffma2_rn(f2(vs[i], vs[i + 1]), m, nl);
    if (MASK) {
      if (kc + i > khi || kc + i < klo) s.x = -INFINITY;
      if (kc + i + 1 > khi || kc + i + 1 < klo) s.y = -INFINITY;
    }
    const float2 p = make_float2(ex2(s.x), ex2(s.y));
    const float2 u = __ffma2_rn(f2(vdds[i], vdds[i + 1]), msc, ndd);  // ddS - dD
    const float2 dpd = __fadd2_rn(f2(vdp[i], vdp[i + 1]), ndv);       // dP - D
    const float2 ddp = __fmul2_rn(p, u);
    const float2 ds = __fmul2_rn(p, dpd);
    const float2 ds2 = __ffma2_rn(ddp, dpd, __fmul2_rn(p, __fadd2_rn(f2(vdpa[i], vdpa[i + 1]), ncq)));
    o_p[i / 2] = pack_bf16(p.x, p.y);
    o_ddp[i / 2] = pack_bf16(ddp.x, ddp.y);
    o_ds[i / 2] = pack_bf16(ds.x, ds.y);
    o_ds2[i / 2] = pack_bf16(ds2.x, ds2.y);
  }
}

// Forward-tangent forms (dO = 0): the stats sweep needs only dD/scale += P ddS', and
// the second sweep only P and ddP = P (ddS - dD).
template <int CW, bool MASK>
__device__ __forceinline__ void q_stats_tj(const uint32_t (&vs)[CW], const uint32_t (&vdds)[CW], int kc, int klo,
                                           int khi, float sc2, float lg, float2& dD) {
  const float2 m = make_float2(sc2, sc2), nl = make_float2(-lg, -lg);
#pragma unroll
  for (int i = 0; i < CW; i += 2) {
    float2 s = __ffma2_rn(f2(vs[i], vs[i + 1]), m, nl);
    if (MASK) {
      if (kc + i > khi || kc + i < klo) s.x = -INFINITY;
      if (kc + i + 1 > khi || kc + i + 1 < klo) s.y = -INFINITY;
    }
    dD = __fadd2_rn(dD, __fmul2_rn(f2(vdds[i], vdds[i + 1]), make_float2(ex2(s.x), ex2(s.y))));
  }
}

template <int CW, bool MASK>
__device__ __forceinline__ void q_ops_tj(const uint32_t (&vs)[CW], const uint32_t (&vdds)[CW], int kc, int klo,
                                         int khi, float sc, float sc2, float lg, float dD,
                                         uint32_t (&o_ddp)[CW / 2], uint32_t (&o_p)[CW / 2]) {
  const float2 m = make_float2(sc2, sc2), nl = make_float2(-lg, -lg), msc = make_float2(sc, sc);
  const float2 ndd = make_float2(-dD, -dD);
#pragma unroll
  for (int i = 0; i < CW; i += 2) {
    float2 s = __ffma2_rn(f2(vs[i], vs[i + 1]), m, nl);
    if (MASK) {
      if (kc + i > khi || kc + i < klo) s.x = -INFINITY;
      if (kc + i + 1 > khi || kc + i + 1 < klo) s.y = -INFINITY;
    }
    const float2 p = make_float2(ex2(s.x), ex2(s.y));
    const float2 ddp = __fmul2_rn(p, __ffma2_rn(f2(vdds[i], vdds[i + 1]), msc, ndd));
    o_p[i / 2] = pack_bf16(p.x, p.y);
    o_ddp[i / 2] = pack_bf16(ddp.x, ddp.y);
  }
}

// TJ (forward tangent): dO = 0 and (ddQ, ddK, ddV) = (tQ, tK, tV). Then dP = dPa = 0,
// D = B = 0, dS = dS2 = 0 and dQ' = 0, and the pass reduces to the jvp of the forward:
// ddO = ddP V + P ddV = tO and dD = rowsum(P ddS) = tL. It skips the dO products, the
// dQ' products and dO's tile: 8 of the 14 GEMM-equivalents per pair remain.
template <int HD, bool VL, bool TJ, bool GRP>
__global__ void __launch_bounds__(kBBThreads, 1)
    bwdbwd_q_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_ddq, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_ddk,
                    const __grid_constant__ CUtensorMap tm_ddv, const __grid_constant__ CUtensorMap tm_o,
                    const BBArgs a) {
  using G = QPass<HD>;
  constexpr int BN = G::BN, ST = G::ST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* s_q = sm;
  uint8_t* s_do = s_q + G::RES;
  uint8_t* s_ddq = s_do + G::RES;
  uint8_t* s_ring = s_ddq + G::RES;
  // When D is computed here, O is staged in the last ring slot, which the
  // first ST-1 key tiles do not use; the producer refills that slot only once
  // every elementwise warp has read O (bar_ofree).
  uint8_t* s_o = s_ring + (ST - 1) * G::SLOT;
  static_assert(G::RES <= G::SLOT, "O fits in one ring slot");
  __shared__ uint64_t bar_res, bar_full[ST], bar_empty[ST];
  __shared__ uint64_t bar_sc_full[2], bar_sc_empty[2], bar_ops_full, bar_ops_empty, bar_acc, bar_red, bar_ofree;
  __shared__ uint64_t bar_tres;  // head_dim 128: ddQ copied into TMEM
  __shared__ float red[4][2][kBM];  // stats-sweep partial sums: statistic, warpgroup, row
  __shared__ float dred[2][kBM];    // partial rowsum(dO o): warpgroup, row
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Grid (H, B, query tiles), longest causal rows first; GRP: a 1-D grid in the
  // locality-grouped order.
  int h = blockIdx.x, b = blockIdx.y, qt = gridDim.z - 1 - blockIdx.z;
  if constexpr (GRP) {
    const int nq = (a.sh.Tq + kBM - 1) / kBM;
    int qi, hb;
    grouped_order(blockIdx.x, nq, a.sh.H * a.sh.B, a.grp_q, &qi, &hb);
    h = hb % a.sh.H, b = hb / a.sh.H, qt = nq - 1 - qi;
  }
  SeqRange sr;
  const AttnShape sh = seq_shape<VL>(a.sh, b, &sr);  // this sequence's lengths and mask; sr: where its rows start
  const int q0 = qt * kBM;
  int j0;
  const int n = key_tiles(sh, q0, kBM, BN, &j0);  // key tiles j0, j0 + 1, ... per sweep (0: no row sees a key)
  const int total = 2 * n;
  // Score buffer of tile `it` and how many earlier tiles used that buffer:
  // the stats sweep alternates buffers 0 and 1, the second sweep uses buffer 0.
  auto buf_of = [n](int it) { return it < n ? (it & 1) : 0; };
  auto use_of = [n](int it) { return it < n ? (it >> 1) : ((n + 1) >> 1) + (it - n); };

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar_res, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_sc_full[i], 1);
      mbar_init(&bar_sc_empty[i], kBBEwWarps);
    }
    mbar_init(&bar_ops_full, kBBEwWarps);
    mbar_init(&bar_ops_empty, 1);
    mbar_init(&bar_acc, 1);
    mbar_init(&bar_red, kBBEwWarps);
    mbar_init(&bar_ofree, kBBEwWarps);
    mbar_init(&bar_tres, kBBEwWarps);
    mbar_fence_init();
  }
  if (warp == kBBWarpMma) tmem_alloc(&tmem_base, G::TMEM_COLS);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == kBBWarpProducer) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      const bool fuse_d = !TJ && a.delta_out != nullptr;
      mbar_arrive_expect_tx(&bar_res, (fuse_d ? 4 : TJ ? 2 : 3) * G::RES);
      tma_rows<HD>(s_q, &tm_q, &bar_res, sr.q0 + q0, kBM, h, sr.bc);
      if (!TJ) tma_rows<HD>(s_do, &tm_do, &bar_res, sr.q0 + q0, kBM, h, sr.bc);
      tma_rows<HD>(s_ddq, &tm_ddq, &bar_res, sr.q0 + q0, kBM, h, sr.bc);
      if (fuse_d) tma_rows<HD>(s_o, &tm_o, &bar_res, sr.q0 + q0, kBM, h, sr.bc);
      int issued = 0;
      for (int it = 0; it < total; ++it) {
        const int s = it % ST;
        if (it >= ST && !mbar_wait(&bar_empty[s], ((it / ST) - 1) & 1, &abort_flag)) {
          raise_error(a.status, &abort_flag, kDevTimeoutSlotEmpty);
          break;
        }
        if (fuse_d && it == ST - 1 && !mbar_wait(&bar_ofree, 0, &abort_flag)) {
          raise_error(a.status, &abort_flag, kDevTimeoutSlotEmpty);
          break;
        }
        const int k0 = (j0 + it % n) * BN;
        uint8_t* slot = s_ring + s * G::SLOT;
        mbar_arrive_expect_tx(&bar_full[s], G::SLOT);
        tma_pair<HD>(slot, &tm_k, &tm_ddk, &bar_full[s], sr.k0 + k0, BN, h / sh.G, sr.bc);
        tma_pair<HD>(slot + G::PAIR, &tm_v, &tm_ddv, &bar_full[s], sr.k0 + k0, BN, h / sh.G, sr.bc);
        issued = it + 1;
      }
      // Every issued copy must land before this CTA's shared memory is released.
      bool drained = mbar_wait(&bar_res, 0, nullptr);
      for (int it = issued > ST ? issued - ST : 0; it < issued; ++it)
        drained &= mbar_wait(&bar_full[it % ST], (it / ST) & 1, nullptr);
      if (!drained) raise_error(a.status, &abort_flag, kDevTimeoutDrain);
    }
  } else if (warp == kBBWarpMma) {
    // ------------------------------ score MMA issuer ------------------------------
    // Products sharing an A operand are one N=128 MMA:
    //   [S | Q ddK^T] = Q [K ; ddK]^T,  ddS += ddQ K^T,  [dP | dPa] = dO [V ; ddV]^T
    {
      constexpr int KS = HD / 16;
      const uint32_t id128 = idesc_bf16_f32(kBM, 2 * BN, false, false);
      const uint32_t id64 = idesc_bf16_f32(kBM, BN, false, false);
      const uint64_t a_q = kdesc(s_q), a_do = kdesc(s_do);
      [[maybe_unused]] const uint64_t a_ddq = kdesc(s_ddq);  // head_dim 64 (SS form)
      const uint64_t b_ring = kdesc(s_ring);  // pair (K | ddK) of slot 0, K-major
      constexpr uint64_t kSlot = G::SLOT >> 4, kPair = G::PAIR >> 4;
      bool ok = mbar_wait_warp(&bar_res, 0, &abort_flag);
      if (!ok && lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutTmaFull);
      if (G::DDQ_T && ok) {  // ddQ in TMEM (copied by the elementwise warps)
        ok = mbar_wait_warp(&bar_tres, 0, &abort_flag);
        if (!ok && lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutEpilogue);
      }
      for (int it = 0; ok && it < total; ++it) {
        const int s = it % ST, sb = buf_of(it), u = use_of(it);
        if (!mbar_wait_warp(&bar_full[s], (it / ST) & 1, &abort_flag)) {
          if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutTmaFull);
          break;
        }
        if (u > 0 && !mbar_wait_warp(&bar_sc_empty[sb], (u - 1) & 1, &abort_flag)) {
          if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutEpilogue);
          break;
        }
        tc_fence_after();
        const uint64_t bk = b_ring + s * kSlot;
        const uint32_t tb = tmem + sb * G::SCORE_COLS;
        umma_chain_w<KS, G::RES_PANEL, G::PAIR_PANEL, false>(tb + G::C_S, a_q, bk, id128, false);
        if constexpr (G::DDQ_T) {
          umma_chain_tsk_w<KS, G::PAIR_PANEL>(tb + G::C_DDS, tmem + G::C_DDQ, bk, id64, true);
        } else {
          umma_chain_w<KS, G::RES_PANEL, G::PAIR_PANEL, false>(tb + G::C_DDS, a_ddq, bk, id64, true);
        }
        if constexpr (!TJ)
          umma_chain_w<KS, G::RES_PANEL, G::PAIR_PANEL, false>(tb + G::C_DP, a_do, bk + kPair, id128, false);
        umma_commit_w(&bar_sc_full[sb]);
        if (it < n) umma_commit_w(&bar_empty[s]);  // stats sweep: slot free once scored
      }
    }
  } else if (warp == kBBWarpMmaOut) {
    // ----------------------------- operand MMA issuer -----------------------------
    // Second-sweep tile j, A in TMEM:  dQ'/scale += dS ddK + dS2 K,  ddO += ddP V + P ddV
    {
      constexpr int KO = BN / 16, OC = G::OPS_COLS;
      const uint32_t id_out = idesc_bf16_f32(kBM, HD, false, true);
      const uint64_t mn_ring = mndesc(s_ring, G::PAIR_PANEL);  // K of slot 0, MN-major
      constexpr uint64_t kSlot = G::SLOT >> 4, kPair = G::PAIR >> 4, kHalf = (BN * 128) >> 4;
      const uint32_t t_ops = tmem + G::C_OPS;
      bool ok = true;
      for (int j = 0; j < n; ++j) {
        if (!mbar_wait_warp(&bar_ops_full, j & 1, &abort_flag)) {
          if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutEpilogue);
          ok = false;
          break;
        }
        tc_fence_after();
        const int sp = (n + j) % ST;
        const uint64_t mk = mn_ring + sp * kSlot;  // K; ddK = +kHalf; V = +kPair; ddV = +kPair+kHalf
        const bool acc = j > 0;
        if constexpr (!TJ) {
          umma_chain_ts_w<KO>(tmem + G::C_DQ, t_ops, mk + kHalf, id_out, acc);
          umma_chain_ts_w<KO>(tmem + G::C_DQ, t_ops + OC, mk, id_out, true);
        }
        umma_chain_ts_w<KO>(tmem + G::C_DDO, t_ops + 2 * OC, mk + kPair, id_out, acc);
        umma_chain_ts_w<KO>(tmem + G::C_DDO, t_ops + 3 * OC, mk + kPair + kHalf, id_out, true);
        umma_commit_w(&bar_ops_empty);
        umma_commit_w(&bar_empty[sp]);
      }
      if (ok) umma_commit_w(&bar_acc);
    }
  } else {
    // --------------------------- elementwise warps ----------------------------
    const int wg = (warp - kBBFirstEwWarp) >> 2;  // column half of every tile
    const int r = (warp & 3) * 32 + lane;         // TMEM lane = query row inside the tile
    constexpr int CW = G::CW;
    const int cb = wg * CW;
    const int row = q0 + r;
    const bool row_ok = row < sh.Tq;
    const size_t vi = q_stat(sh, sr, row_ok ? row : 0, h);
    const float lse = row_ok ? a.lse[vi] : 0.f;
    const float lg = lse > -INFINITY ? lse * kLog2e : 0.f;  // -inf: the row sees no key (all masked)
    const int khi = key_hi(sh, row), klo = key_lo(sh, row);
    const float sc = sh.scale, sc2 = sh.scale * kLog2e;
    float dD = 0.f, Bv = 0.f, cq = 0.f;
    bool ok = true;
    float dv = 0.f;
    if constexpr (G::DDQ_T) {
      // head_dim 128: this CTA's ddQ rows into TMEM, each warpgroup half of the head_dim
      // columns, for the TS form of ddS += ddQ K^T (the score issuer waits for it before
      // the first ddS product).
      ok = mbar_wait_warp(&bar_res, 0, &abort_flag);
      if (ok) {
        row_to_tmem<HD / 2>(s_ddq, r, wg * (HD / 2), tmem + tmem_lane_base(warp & 3) + G::C_DDQ);
        tmem_wait_st();
        warp_arrive(&bar_tres);
      }
    }
    if constexpr (TJ) {
      dv = 0.f;  // dO = 0
    } else if (a.delta_out == nullptr) {
      dv = row_ok ? a.delta[vi] : 0.f;
    } else {
      // D = rowsum(dO o) of this row from the resident tiles, while the first
      // scores are computed: each warpgroup sums half of the head_dim columns.
      if (ok) ok = mbar_wait_warp(&bar_res, 0, &abort_flag);
      dv = ok ? rowdot_share<HD>(s_o, s_do, r, wg) : 0.f;
      dred[wg][r] = dv;
      warp_arrive(&bar_ofree);  // O has been read: its ring slot may be refilled
      named_bar_sync(1, kBBEwWarps * 32);
      dv = dred[0][r] + dred[1][r];
      if (wg == 0 && row_ok) a.delta_out[vi] = dv;
    }
    // Waits for streamed tile `it`'s scores and loads this thread's share of them into
    // registers, then releases the score buffer to the tensor core.
    auto load_scores = [&](int it, uint32_t (&vs)[CW], uint32_t (&vdds)[CW], uint32_t (&vdp)[CW],
                           uint32_t (&vdpa)[CW]) {
      const int sb = buf_of(it);
      if (!mbar_wait_warp(&bar_sc_full[sb], use_of(it) & 1, &abort_flag)) return false;
      tc_fence_after();
      const uint32_t tb = tmem + sb * G::SCORE_COLS;
      tmem_share<CW>(tb, warp, G::C_S + cb, vs);
      tmem_share<CW>(tb, warp, G::C_DDS + cb, vdds);
      if constexpr (!TJ) {
        tmem_share<CW>(tb, warp, G::C_DP + cb, vdp);
        tmem_share<CW>(tb, warp, G::C_DPA + cb, vdpa);
      }
      tmem_wait_ld();
      reg_fence(vs);
      reg_fence(vdds);
      if constexpr (!TJ) {
        reg_fence(vdp);
        reg_fence(vdpa);
      }
      warp_arrive(&bar_sc_empty[sb]);  // the tensor core may reuse this score buffer now
      return true;
    };
    // Sweep 1: the row statistics. Its partial sums live only in this loop.
    if (ok && n > 0) {
      float2 pdD = make_float2(0.f, 0.f), pr1 = pdD, pr2 = pdD, pr3 = pdD;  // (even, odd) column partial sums
      for (int j = 0; ok && j < n; ++j) {
        const int kc = (j0 + j) * BN + cb;  // first key of this thread's columns
        uint32_t vs[CW], vdds[CW], vdp[CW], vdpa[CW];
        ok = load_scores(j, vs, vdds, vdp, vdpa);
        if (!ok) break;
        if constexpr (TJ) {
          if (kc + CW - 1 > khi || kc < klo)
            q_stats_tj<CW, true>(vs, vdds, kc, klo, khi, sc2, lg, pdD);
          else
            q_stats_tj<CW, false>(vs, vdds, kc, klo, khi, sc2, lg, pdD);
        } else {
          if (kc + CW - 1 > khi || kc < klo)
            q_stats<CW, true>(vs, vdds, vdp, vdpa, kc, klo, khi, sc2, lg, pdD, pr1, pr2, pr3);
          else
            q_stats<CW, false>(vs, vdds, vdp, vdpa, kc, klo, khi, sc2, lg, pdD, pr1, pr2, pr3);
        }
      }
      if (ok) {
        // Combine the column pairs, then the two warpgroups' column halves (same
        // order on both sides).
        red[0][wg][r] = pdD.x + pdD.y;
        red[1][wg][r] = pr1.x + pr1.y;
        red[2][wg][r] = pr2.x + pr2.y;
        red[3][wg][r] = pr3.x + pr3.y;
        warp_arrive(&bar_red);
        ok = mbar_wait_warp(&bar_red, 0, &abort_flag);
      }
      if (ok) {
        dD = (red[0][0][r] + red[0][1][r]) * sc;
        const float r1 = red[1][0][r] + red[1][1][r];
        const float r2 = red[2][0][r] + red[2][1][r];
        const float r3 = (red[3][0][r] + red[3][1][r]) * sc;
        Bv = r1 - dD * r2 - dv * dD + r3;
        cq = r1 - dD * r2 + r3;  // dD D + B
      }
    }
    // Sweep 2: the bf16 operands of the accumulating MMAs.
    for (int j = 0; ok && j < n; ++j) {
      const int kc = (j0 + j) * BN + cb;
      uint32_t vs[CW], vdds[CW], vdp[CW], vdpa[CW];
      ok = load_scores(n + j, vs, vdds, vdp, vdpa);
      if (!ok) break;
      uint32_t o_ds[CW / 2], o_ds2[CW / 2], o_ddp[CW / 2], o_p[CW / 2];
      if constexpr (TJ) {
        if (kc + CW - 1 > khi || kc < klo)
          q_ops_tj<CW, true>(vs, vdds, kc, klo, khi, sc, sc2, lg, dD, o_ddp, o_p);
        else
          q_ops_tj<CW, false>(vs, vdds, kc, klo, khi, sc, sc2, lg, dD, o_ddp, o_p);
      } else {
        if (kc + CW - 1 > khi || kc < klo)
          q_ops<CW, true>(vs, vdds, vdp, vdpa, kc, klo, khi, sc, sc2, lg, dv, dD, cq, o_ds, o_ds2, o_ddp, o_p);
        else
          q_ops<CW, false>(vs, vdds, vdp, vdpa, kc, klo, khi, sc, sc2, lg, dv, dD, cq, o_ds, o_ds2, o_ddp, o_p);
      }
      if (j > 0) ok = mbar_wait_warp(&bar_ops_empty, (j - 1) & 1, &abort_flag);
      if (!ok) break;
      tc_fence_after();
      // This warpgroup's CW keys are packed columns [CW/2 wg, CW/2 wg + CW/2) of each operand.
      const uint32_t to = tmem + tmem_lane_base(warp & 3) + G::C_OPS + (CW / 2) * wg;
      if constexpr (!TJ) {
        tmem_st_ops(to, o_ds);
        tmem_st_ops(to + G::OPS_COLS, o_ds2);
      }
      tmem_st_ops(to + 2 * G::OPS_COLS, o_ddp);
      tmem_st_ops(to + 3 * G::OPS_COLS, o_p);
      tmem_wait_st();
      warp_arrive(&bar_ops_full);
    }
    if (ok && n == 0) {
      // No key tile: every output of these rows is zero.
      if (row_ok) {
        if (!TJ || wg == 1) zero_row_global<HD>((wg == 0 ? a.dq2 : a.ddo) + q_row(sh, sr, row, h));
        if (wg == 0) {
          a.dd[vi] = 0.f;
          if (!TJ) a.bv[vi] = 0.f;
        }
      }
    } else if (ok) {
      ok = mbar_wait_warp(&bar_acc, 0, &abort_flag);
    }
    if (ok && n > 0) {
      tc_fence_after();
      const int srow = row_ok ? row : 0;
      if (wg == 0) {
        if constexpr (!TJ) tmem_row_to_global<HD>(tmem, warp, G::C_DQ, a.dq2 + q_row(sh, sr, srow, h), row_ok, sc);
        if (row_ok) {
          a.dd[vi] = dD;
          if (!TJ) a.bv[vi] = Bv;
        }
      } else {
        tmem_row_to_global<HD>(tmem, warp, G::C_DDO, a.ddo + q_row(sh, sr, srow, h), row_ok);
      }
    } else if (!ok && threadIdx.x == kBBFirstEwWarp * 32) {
      raise_error(a.status, &abort_flag, kDevTimeoutMma);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kBBWarpMma) tmem_dealloc(tmem, G::TMEM_COLS);
}

// ----------------------------------------------------------------------------------
// key-tiled pass
// ----------------------------------------------------------------------------------

template <int HD>
struct KPass {
  // Query rows per streamed tile and ring depth: 64 x 4 at head_dim 64; 32 x 3 at
  // 128 (four 32 KB resident key-side tiles leave room for three 28 KB slots).
  static constexpr int BN = HD == 64 ? 64 : 32;
  static constexpr int ST = HD == 64 ? 4 : 3;
  static constexpr int CW = BN / 2;
  static constexpr int RES = kBM * HD * 2;
  static constexpr int RES_PANEL = kBM * 128;
  static constexpr int STR = BN * HD * 2;
  static constexpr int PAIR = 2 * STR;
  static constexpr int PAIR_PANEL = 2 * BN * 128;
  // Per-query biases of the four score products as a K = 16 bf16 operand
  // (32-byte rows, 32B swizzle): rows [BN m, BN m + BN) hold product m's bias
  // for each streamed query as a (hi, lo) bf16 pair in columns 0-1, zeros after.
  static constexpr int BIAS_ROW = 32;
  static constexpr int BIAS = 4 * BN * BIAS_ROW;
  static constexpr int ONES = kBM * BIAS_ROW;      // resident A operand: (1, 1, 0, ...) per key row
  static constexpr int SLOT = PAIR + STR + BIAS;   // (Q | ddQ) pair, dO, biases
  static constexpr int SMEM = 1024 + 4 * RES + ONES + ST * SLOT;
  // TMEM: scores, accumulators dK', dV', bf16 operands dS^T, dS2^T, ddP^T (A of the MMAs).
  static constexpr int C_S = 0, C_DDS = BN, C_DP = 2 * BN, C_DPA = 3 * BN;
  static constexpr int C_DK = 4 * BN, C_DV = 4 * BN + HD, C_OPS = 4 * BN + 2 * HD;
  // head_dim 128: ddV as packed bf16 in TMEM (HD/2 columns), the A operand of
  // dPa^T = ddV dO^T as a TS product that reads only dO from shared memory (with 32-query
  // tiles the SS form is shared-memory bound at 40 cycles per k-step against 16 of math).
  // At head_dim 64 the per-item copy costs more than the 64-query chain saves.
  static constexpr bool DDV_T = HD == 128;
  static constexpr int C_DDV = C_OPS + 3 * (BN / 2);
  static constexpr int OPS_COLS = BN / 2;
  static constexpr int TMEM_COLS = 512;
  static_assert(SLOT % 1024 == 0 && (4 * RES + ONES) % 1024 == 0, "slots must keep panels 1024-byte aligned");
  static_assert(C_DDV + (DDV_T ? HD / 2 : 0) <= TMEM_COLS, "TMEM budget");
  static_assert(C_DDS == C_S + BN && C_DP == C_S + 2 * BN && C_DPA == C_S + 3 * BN, "one bias MMA covers 4 products");
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(CW % 16 == 0 && BN % 32 == 0, "tile shapes");
};

// Packed bf16 pairs of dS^T/scale, dS2^T/scale and ddP^T for this thread's CW
// query columns (the scale of dS, dS2 is applied to dK' in the epilogue), by
// the same identities as the query pass. The per-query statistics arrive
// already folded into the score products by the bias MMA:
//   vs = S - L/scale,  vdds = ddS/scale - dD/scale,  vdp = dP - D,  vdpa = dPa - c.
// Column pairs go through the packed fp32x2 instructions.
template <int CW, bool MASK>
__device__ __forceinline__ void k_ops(const uint32_t (&vs)[CW], const uint32_t (&vdds)[CW],
                                      const uint32_t (&vdp)[CW], const uint32_t (&vdpa)[CW], int qc, int qlo, int qhi,
                                      float sc, float sc2, uint32_t (&o_ds)[CW / 2],
                                      uint32_t (&o_ds2)[CW / 2], uint32_t (&o_ddp)[CW / 2]) {
  const float2 m = make_float2(sc2, sc2), msc = make_float2(sc, sc);
#pragma unroll
  for (int i = 0; i < CW; i += 2) {
    float2 s = __fmul2_rn(f2(vs[i], vs[i + 1]), m);
    if (MASK) {
      if (qc + i > qhi || qc + i < qlo) s.x = -INFINITY;
      if (qc + i + 1 > qhi || qc + i + 1 < qlo) s.y = -INFINITY;
    }
    const float2 p = make_float2(ex2(s.x), ex2(s.y));
    const float2 u = __fmul2_rn(f2(vdds[i], vdds[i + 1]), msc);  // ddS - dD
    const float2 dpd = f2(vdp[i], vdp[i + 1]);                     // dP - D
    const float2 ddp = __fmul2_rn(p, u);
    const float2 ds = __fmul2_rn(p, dpd);
    const float2 ds2 = __ffma2_rn(ddp, dpd, __fmul2_rn(p, f2(vdpa[i], vdpa[i + 1])));
    o_ddp[i / 2] = pack_bf16(ddp.x, ddp.y);
    o_ds[i / 2] = pack_bf16(ds.x, ds.y);
    o_ds2[i / 2] = pack_bf16(ds2.x, ds2.y);
  }
}


// A unit of key-pass work: one 128-row key tile of one (key head, batch).
// `l` is the item's sequence (its lengths and mask), `r` where that sequence's rows start.
struct KItem {
  int hk, b, k0, qt_begin, n, total;  // n query tiles per query head; total = n * G streamed tiles
  AttnShape l;
  SeqRange r;
};

// Work item w in heaviest-first order (key tile 0 first: the most causal query
// tiles), key heads fastest; GRP: in locality groups of g (key head, batch) pairs.
template <bool VL, bool GRP>
__device__ __forceinline__ KItem k_item(const AttnShape& sh, int w, int bn, int g) {
  int kt, hb;
  if constexpr (GRP) {
    grouped_order(w, (sh.Tk + kBM - 1) / kBM, sh.Hk * sh.B, g, &kt, &hb);
  } else {
    const int per_kt = sh.Hk * sh.B;
    kt = w / per_kt;
    hb = w - kt * per_kt;
  }
  KItem it;
  it.hk = hb % sh.Hk;
  it.b = hb / sh.Hk;
  it.k0 = kt * kBM;
  it.l = seq_shape<VL>(sh, it.b, &it.r);
  it.n = query_tiles(it.l, it.k0, kBM, bn, &it.qt_begin);  // query tiles that see any of these keys
  it.total = it.n * sh.G;
  return it;
}


// Persistent key-tiled pass: gridDim.x CTAs (one per SM) each run a sequence of
// work items. The ring and the per-tile barriers run on one tile counter (gt)
// across items; per item the producer reloads the resident tiles once the score
// MMAs of the previous item are done (bar_res_empty), so the reload overlaps the
// previous item's last tile and epilogue, and the operand MMAs of an item start
// only once the previous item's accumulators were read out (bar_acc_empty).
template <int HD, bool VL, bool GRP>
__global__ void __launch_bounds__(kBBThreads, 1)
    bwdbwd_k_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ CUtensorMap tm_ddk, const __grid_constant__ CUtensorMap tm_ddv,
                    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_ddq, const BBArgs a) {
  using G = KPass<HD>;
  constexpr int BN = G::BN, ST = G::ST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* s_k = sm;
  uint8_t* s_v = s_k + G::RES;
  uint8_t* s_ddk = s_v + G::RES;
  uint8_t* s_ddv = s_ddk + G::RES;
  uint8_t* s_ones = s_ddv + G::RES;
  uint8_t* s_ring = s_ones + G::ONES;
  __shared__ uint64_t bar_res, bar_res_empty, bar_full[ST], bar_empty[ST];
  __shared__ uint64_t bar_sc_full, bar_sc_empty, bar_ops_full, bar_ops_empty, bar_acc, bar_acc_empty, bar_tres;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const AttnShape& sh = a.sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = sh.Hk * sh.B * ((sh.Tk + kBM - 1) / kBM);
  const int P = gridDim.x, c = blockIdx.x;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar_res, 1);
    mbar_init(&bar_res_empty, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    mbar_init(&bar_sc_full, 1);
    mbar_init(&bar_sc_empty, kBBEwWarps);
    mbar_init(&bar_ops_full, kBBEwWarps);
    mbar_init(&bar_ops_empty, 1);
    mbar_init(&bar_acc, 1);
    mbar_init(&bar_acc_empty, kBBEwWarps);
    mbar_init(&bar_tres, kBBEwWarps);
    mbar_fence_init();
  }
  if (threadIdx.x < kBM) {
    // The resident ones operand: row r = (1, 1, 0, ..., 0), so ones x biases^T
    // adds hi + lo of each query's bias to every key row.
    const uint32_t t = smem_u32(s_ones);
    st_shared_v4(t + sw32_offset(threadIdx.x, 0), 0x3F803F80u, 0u, 0u, 0u);
    st_shared_v4(t + sw32_offset(threadIdx.x, 1), 0u, 0u, 0u, 0u);
    fence_async_smem();
  }
  if (warp == kBBWarpMma) tmem_alloc(&tmem_base, G::TMEM_COLS);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == kBBWarpProducer) {
    // ---------------------- TMA producer (whole warp) -----------------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_q);
    }
    const float inv_scale = 1.f / sh.scale;
    constexpr int RPL = BN / 32;
    // Per-query statistics of streamed tile `it` of item `w`, into registers.
    auto load_stats = [&](const KItem& w, int it, float (&raw)[RPL][4]) {
      const int q0 = (w.qt_begin + it % w.n) * BN;
      const int h = w.hk * sh.G + it / w.n;
#pragma unroll
      for (int k = 0; k < RPL; ++k) {
        const int q = q0 + lane + 32 * k;
        const size_t idx = q_stat(w.l, w.r, q < w.l.Tq ? q : 0, h);
        raw[k][0] = a.lse[idx];
        raw[k][1] = a.delta[idx];
        raw[k][2] = a.dd[idx];
        raw[k][3] = a.bv[idx];
      }
    };
    int gt = 0, ai = 0;  // tiles and active items issued so far
    bool ok = true;
    for (int j = 0; ok; ++j) {
      const int wi = snake_item(j, c, P);
      if (wi >= n_items) break;
      const KItem w = k_item<VL, GRP>(sh, wi, BN, a.grp_k);
      if (w.total == 0) continue;
      // The previous item's score MMAs no longer read the resident tiles.
      if (ai > 0 && !mbar_wait_warp(&bar_res_empty, (ai - 1) & 1, &abort_flag)) {
        if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutSlotEmpty);
        break;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(&bar_res, 4 * G::RES);
        tma_rows<HD>(s_k, &tm_k, &bar_res, w.r.k0 + w.k0, kBM, w.hk, w.r.bc);
        tma_rows<HD>(s_v, &tm_v, &bar_res, w.r.k0 + w.k0, kBM, w.hk, w.r.bc);
        tma_rows<HD>(s_ddk, &tm_ddk, &bar_res, w.r.k0 + w.k0, kBM, w.hk, w.r.bc);
        tma_rows<HD>(s_ddv, &tm_ddv, &bar_res, w.r.k0 + w.k0, kBM, w.hk, w.r.bc);
      }
      ++ai;
      float raw_next[RPL][4];
      load_stats(w, 0, raw_next);
      for (int it = 0; it < w.total; ++it, ++gt) {
        const int s = gt % ST;
        const int q0 = (w.qt_begin + it % w.n) * BN;
        const int h = w.hk * sh.G + it / w.n;  // query head of this tile
        if (gt >= ST && !mbar_wait_warp(&bar_empty[s], ((gt / ST) - 1) & 1, &abort_flag)) {
          if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutSlotEmpty);
          ok = false;
          break;
        }
        uint8_t* slot = s_ring + s * G::SLOT;
        // Copies first (their bytes are expected without arriving), then the
        // biases; the single arrive after the biases completes the slot's phase
        // together with the copies.
        if (lane == 0) {
          mbar_expect_tx(&bar_full[s], G::PAIR + G::STR);
          tma_pair<HD>(slot, &tm_q, &tm_ddq, &bar_full[s], w.r.q0 + q0, BN, h, w.r.bc);
          tma_rows<HD>(slot + G::PAIR, &tm_do, &bar_full[s], w.r.q0 + q0, BN, h, w.r.bc);
        }
        float raw[RPL][4];  // first use of this tile's statistics: after its copies are issued
#pragma unroll
        for (int k = 0; k < RPL; ++k)
#pragma unroll
          for (int m = 0; m < 4; ++m) raw[k][m] = raw_next[k][m];
        const uint32_t bias = smem_u32(slot + G::PAIR + G::STR);
#pragma unroll
        for (int k = 0; k < RPL; ++k) {
          const bool v = q0 + lane + 32 * k < w.l.Tq;
          const float lse = raw[k][0], dl = raw[k][1], ddl = raw[k][2];
          const int r = lane + 32 * k;
          // L = -inf: the query sees no key and all its elements are masked.
          store_bias_row(bias, r, (v && lse > -INFINITY) ? -lse * inv_scale : 0.f);  // S - L/scale
          store_bias_row(bias, BN + r, v ? -ddl * inv_scale : 0.f);              // ddS/scale - dD/scale
          store_bias_row(bias, 2 * BN + r, v ? -dl : 0.f);                       // dP - D
          store_bias_row(bias, 3 * BN + r, v ? -fmaf(ddl, dl, raw[k][3]) : 0.f); // dPa - c, c = dD D + B
        }
        fence_async_smem();  // the tensor core reads the biases through the async proxy
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar_full[s]);
        // Next tile's statistics: issued after the proxy fence, which would
        // otherwise wait for these loads too.
        if (it + 1 < w.total) load_stats(w, it + 1, raw_next);
      }
    }
    if (lane == 0) {
      // Every issued copy must land before this CTA's shared memory is released.
      bool drained = ai == 0 || mbar_wait(&bar_res, (ai - 1) & 1, nullptr);
      for (int t = gt > ST ? gt - ST : 0; t < gt; ++t) drained &= mbar_wait(&bar_full[t % ST], (t / ST) & 1, nullptr);
      if (!drained) raise_error(a.status, &abort_flag, kDevTimeoutDrain);
    }
  } else if (warp == kBBWarpMma) {
    // ------------------------------ score MMA issuer ------------------------------
    //   [S^T | K ddQ^T] = K [Q ; ddQ]^T,  ddS^T += ddK Q^T,  dP^T = V dO^T,  dPa^T = ddV dO^T
    constexpr int KS = HD / 16;
    const uint32_t id128 = idesc_bf16_f32(kBM, 2 * BN, false, false);
    const uint32_t id64 = idesc_bf16_f32(kBM, BN, false, false);
    const uint64_t a_k = kdesc(s_k), a_v = kdesc(s_v), a_ddk = kdesc(s_ddk), a_ddv = kdesc(s_ddv);
    const uint64_t b_ring = kdesc(s_ring);          // pair (Q | ddQ) of slot 0
    const uint64_t b_do = kdesc(s_ring + G::PAIR);  // dO of slot 0
    const uint32_t id_bias = idesc_bf16_f32(kBM, 4 * BN, false, false);
    const uint64_t a_ones = smem_desc(smem_u32(s_ones), 16, 8 * G::BIAS_ROW, kSwizzle32B);
    const uint64_t b_bias = smem_desc(smem_u32(s_ring + G::PAIR + G::STR), 16, 8 * G::BIAS_ROW, kSwizzle32B);
    constexpr uint64_t kSlot = G::SLOT >> 4;
    int gt = 0, ai = 0;
    bool ok = true;
    for (int j = 0; ok; ++j) {
      const int wi = snake_item(j, c, P);
      if (wi >= n_items) break;
      const KItem w = k_item<VL, GRP>(sh, wi, BN, a.grp_k);
      if (w.total == 0) continue;
      if (!mbar_wait_warp(&bar_res, ai & 1, &abort_flag)) {
        if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutTmaFull);
        break;
      }
      // This item's ddV in TMEM (copied by the elementwise warps once the residents landed).
      if (G::DDV_T && !mbar_wait_warp(&bar_tres, ai & 1, &abort_flag)) {
        if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutEpilogue);
        break;
      }
      for (int it = 0; it < w.total; ++it, ++gt) {
        const int s = gt % ST;
        if (!mbar_wait_warp(&bar_full[s], (gt / ST) & 1, &abort_flag)) {
          if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutTmaFull);
          ok = false;
          break;
        }
        if (gt > 0 && !mbar_wait_warp(&bar_sc_empty, (gt - 1) & 1, &abort_flag)) {
          if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutEpilogue);
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t bq = b_ring + s * kSlot, bo = b_do + s * kSlot;
        // Biases first (one N = 4 BN MMA over all four products), then the products accumulate.
        umma_bf16_w(tmem + G::C_S, a_ones, b_bias + s * kSlot, id_bias, 0u);
        umma_chain_w<KS, G::RES_PANEL, G::PAIR_PANEL, false>(tmem + G::C_S, a_k, bq, id128, true);
        umma_chain_w<KS, G::RES_PANEL, G::PAIR_PANEL, false>(tmem + G::C_DDS, a_ddk, bq, id64, true);
        umma_chain_w<KS, G::RES_PANEL, BN * 128, false>(tmem + G::C_DP, a_v, bo, id64, true);
        if constexpr (G::DDV_T)
          umma_chain_tsk_w<KS, BN * 128>(tmem + G::C_DPA, tmem + G::C_DDV, bo, id64, true);
        else
          umma_chain_w<KS, G::RES_PANEL, BN * 128, false>(tmem + G::C_DPA, a_ddv, bo, id64, true);
        umma_commit_w(&bar_sc_full);
      }
      if (!ok) break;
      umma_commit_w(&bar_res_empty);  // once these MMAs finish, the residents may be reloaded
      ++ai;
    }
  } else if (warp == kBBWarpMmaOut) {
    // ----------------------------- operand MMA issuer -----------------------------
    //   dK'/scale += dS^T ddQ + dS2^T Q,  dV' += ddP^T dO   (A in TMEM)
    constexpr int KO = BN / 16, OC = G::OPS_COLS;
    const uint32_t id_out = idesc_bf16_f32(kBM, HD, false, true);
    const uint64_t mn_ring = mndesc(s_ring, G::PAIR_PANEL);     // Q of slot 0, MN-major
    const uint64_t mn_do = mndesc(s_ring + G::PAIR, BN * 128);  // dO of slot 0, MN-major
    constexpr uint64_t kSlot = G::SLOT >> 4, kHalf = (BN * 128) >> 4;
    const uint32_t t_ops = tmem + G::C_OPS;
    int gt = 0, ai = 0;
    bool ok = true;
    for (int j = 0; ok; ++j) {
      const int wi = snake_item(j, c, P);
      if (wi >= n_items) break;
      const KItem w = k_item<VL, GRP>(sh, wi, BN, a.grp_k);
      if (w.total == 0) continue;
      for (int it = 0; it < w.total; ++it, ++gt) {
        if (!mbar_wait_warp(&bar_ops_full, gt & 1, &abort_flag)) {
          if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutEpilogue);
          ok = false;
          break;
        }
        // The first product of an item overwrites the accumulators: the previous
        // item's epilogue must have read them.
        if (it == 0 && ai > 0 && !mbar_wait_warp(&bar_acc_empty, (ai - 1) & 1, &abort_flag)) {
          if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutEpilogue);
          ok = false;
          break;
        }
        tc_fence_after();
        const int sp = gt % ST;
        const uint64_t mq = mn_ring + sp * kSlot, mo = mn_do + sp * kSlot;
        const bool acc = it > 0;
        umma_chain_ts_w<KO>(tmem + G::C_DK, t_ops, mq + kHalf, id_out, acc);
        umma_chain_ts_w<KO>(tmem + G::C_DK, t_ops + OC, mq, id_out, true);
        umma_chain_ts_w<KO>(tmem + G::C_DV, t_ops + 2 * OC, mo, id_out, acc);
        umma_commit_w(&bar_ops_empty);
        umma_commit_w(&bar_empty[sp]);
      }
      if (!ok) break;
      umma_commit_w(&bar_acc);
      ++ai;
    }
  } else {
    // --------------------------- elementwise warps ----------------------------
    const int wg = (warp - kBBFirstEwWarp) >> 2;
    const int r = (warp & 3) * 32 + lane;  // TMEM lane = key row inside the tile
    constexpr int CW = G::CW;
    const int cb = wg * CW;
    const float sc = sh.scale, sc2 = sh.scale * kLog2e;
    int gt = 0, ai = 0;
    bool ok = true;
    for (int j = 0; ok; ++j) {
      const int wi = snake_item(j, c, P);
      if (wi >= n_items) break;
      const KItem w = k_item<VL, GRP>(sh, wi, BN, a.grp_k);
      const int key = w.k0 + r;
      const bool key_ok = key < w.l.Tk;
      const int qhi = query_hi(w.l, key), qlo = query_lo(w.l, key);  // queries that see this key
      const int skey = key_ok ? key : 0;
      __nv_bfloat16* dst = (wg == 0 ? a.dk2 : a.dv2) + k_row(w.l, w.r, skey, w.hk);
      if (w.total == 0) {
        // No query sees these keys (causal with Tk > Tq): the gradients are zero.
        if (key_ok) zero_row_global<HD>(dst);
        continue;
      }
      // head_dim 128: this item's ddV rows into TMEM, each warpgroup half of the head_dim columns, once
      // the residents landed (which also means the previous item's score MMAs, the last
      // readers of the TMEM copy, are done).
      if constexpr (G::DDV_T) {
        ok = mbar_wait_warp(&bar_res, ai & 1, &abort_flag);
        if (!ok) break;
        row_to_tmem<HD / 2>(s_ddv, r, wg * (HD / 2), tmem + tmem_lane_base(warp & 3) + G::C_DDV);
        tmem_wait_st();
        warp_arrive(&bar_tres);
      }
      for (int it = 0; it < w.total; ++it, ++gt) {
        const int qc = (w.qt_begin + it % w.n) * BN + cb;  // first query of this thread's columns
        ok = mbar_wait_warp(&bar_sc_full, gt & 1, &abort_flag);
        if (!ok) break;
        tc_fence_after();
        uint32_t vs[CW], vdds[CW], vdp[CW], vdpa[CW];
        tmem_share<CW>(tmem, warp, G::C_S + cb, vs);
        tmem_share<CW>(tmem, warp, G::C_DDS + cb, vdds);
        tmem_share<CW>(tmem, warp, G::C_DP + cb, vdp);
        tmem_share<CW>(tmem, warp, G::C_DPA + cb, vdpa);
        tmem_wait_ld();
        reg_fence(vs);
        reg_fence(vdds);
        reg_fence(vdp);
        reg_fence(vdpa);
        warp_arrive(&bar_sc_empty);
        const bool need_mask = qc + CW - 1 > qhi || qc < qlo;
        uint32_t o_ds[CW / 2], o_ds2[CW / 2], o_ddp[CW / 2];
        if (need_mask)
          k_ops<CW, true>(vs, vdds, vdp, vdpa, qc, qlo, qhi, sc, sc2, o_ds, o_ds2, o_ddp);
        else
          k_ops<CW, false>(vs, vdds, vdp, vdpa, qc, qlo, qhi, sc, sc2, o_ds, o_ds2, o_ddp);
        if (gt > 0) ok = mbar_wait_warp(&bar_ops_empty, (gt - 1) & 1, &abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t to = tmem + tmem_lane_base(warp & 3) + G::C_OPS + (CW / 2) * wg;
        tmem_st_ops(to, o_ds);
        tmem_st_ops(to + G::OPS_COLS, o_ds2);
        tmem_st_ops(to + 2 * G::OPS_COLS, o_ddp);
        tmem_wait_st();
        warp_arrive(&bar_ops_full);
      }
      if (ok) ok = mbar_wait_warp(&bar_acc, ai & 1, &abort_flag);
      if (!ok) {
        if (threadIdx.x == kBBFirstEwWarp * 32) raise_error(a.status, &abort_flag, kDevTimeoutMma);
        break;
      }
      tc_fence_after();
      tmem_row_to_global<HD>(tmem, warp, wg == 0 ? G::C_DK : G::C_DV, dst, key_ok, wg == 0 ? sc : 1.f);
      warp_arrive(&bar_acc_empty);  // the accumulators may be overwritten by the next item
      ++ai;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kBBWarpMma) tmem_dealloc(tmem, G::TMEM_COLS);
}

template <int HD, bool VL>
int launch_bwdbwd_hd(const AttnShape& s, const BwdBwdPtrs& p, int passes, int* status, cudaStream_t stream) {
  using GQ = QPass<HD>;
  using GK = KPass<HD>;
  CUtensorMap mq[8], mk[7];
  // Query-tiled pass: 128-row query tiles, 64-row key tiles.
  // dO and O are only read by the passes that need them (the forward-tangent pass reads
  // neither); a stand-in base keeps their maps valid when they are absent.
  bool ok = make_seq_map(&mq[0], p.q, HD, s.total_q, s.H, map_batch(s), s.sq, kBM) &&
            make_seq_map(&mq[1], p.dO ? p.dO : p.q, HD, s.total_q, s.H, map_batch(s), s.sq, kBM) &&
            make_seq_map(&mq[2], p.ddq, HD, s.total_q, s.H, map_batch(s), s.sq, kBM) &&
            make_seq_map(&mq[3], p.k, HD, s.total_k, s.Hk, map_batch(s), s.sk, GQ::BN) &&
            make_seq_map(&mq[4], p.v, HD, s.total_k, s.Hk, map_batch(s), s.sk, GQ::BN) &&
            make_seq_map(&mq[5], p.ddk, HD, s.total_k, s.Hk, map_batch(s), s.sk, GQ::BN) &&
            make_seq_map(&mq[6], p.ddv, HD, s.total_k, s.Hk, map_batch(s), s.sk, GQ::BN) &&
            make_seq_map(&mq[7], p.o ? p.o : p.q, HD, s.total_q, s.H, map_batch(s), s.sq, kBM);  // O: only read when D is fused
  // Key-tiled pass: 128-row key tiles, 64-row query tiles.
  ok = ok && make_seq_map(&mk[0], p.k, HD, s.total_k, s.Hk, map_batch(s), s.sk, kBM) &&
       make_seq_map(&mk[1], p.v, HD, s.total_k, s.Hk, map_batch(s), s.sk, kBM) &&
       make_seq_map(&mk[2], p.ddk, HD, s.total_k, s.Hk, map_batch(s), s.sk, kBM) &&
       make_seq_map(&mk[3], p.ddv, HD, s.total_k, s.Hk, map_batch(s), s.sk, kBM) &&
       make_seq_map(&mk[4], p.q, HD, s.total_q, s.H, map_batch(s), s.sq, GK::BN) &&
       make_seq_map(&mk[5], p.dO ? p.dO : p.q, HD, s.total_q, s.H, map_batch(s), s.sq, GK::BN) &&
       make_seq_map(&mk[6], p.ddq, HD, s.total_q, s.H, map_batch(s), s.sq, GK::BN);
  if (!ok) return kInvalidArgument;
  if (ensure_smem_limit(reinterpret_cast<const void*>(&bwdbwd_q_kernel<HD, VL, false, false>), GQ::SMEM) != kOk ||
      ensure_smem_limit(reinterpret_cast<const void*>(&bwdbwd_q_kernel<HD, VL, true, false>), GQ::SMEM) != kOk ||
      ensure_smem_limit(reinterpret_cast<const void*>(&bwdbwd_k_kernel<HD, VL, false>), GK::SMEM) != kOk)
    return kLaunchFailed;
  if constexpr (!VL) {
    if (ensure_smem_limit(reinterpret_cast<const void*>(&bwdbwd_q_kernel<HD, false, false, true>), GQ::SMEM) != kOk ||
        ensure_smem_limit(reinterpret_cast<const void*>(&bwdbwd_q_kernel<HD, false, true, true>), GQ::SMEM) != kOk ||
        ensure_smem_limit(reinterpret_cast<const void*>(&bwdbwd_k_kernel<HD, false, true>), GK::SMEM) != kOk)
      return kLaunchFailed;
  }
  // With `o`, the query pass computes D into delta_out and the key pass reads it there.
  BBArgs args{s,
              p.lse,
              p.o ? p.delta_out : p.delta,
              p.o ? p.delta_out : nullptr,
              p.dd,
              p.bv,
              static_cast<__nv_bfloat16*>(p.dq2),
              static_cast<__nv_bfloat16*>(p.ddo),
              static_cast<__nv_bfloat16*>(p.dk2),
              static_cast<__nv_bfloat16*>(p.dv2),
              status};
  // Shared streamed tiles per head: K, V, ddK, ddV of a key head for the query pass;
  // Q, ddQ and dO of its query heads for the key pass.
  const int G = s.H / s.Hk;
  args.grp_q = locality_group(s.H * s.B, G, 4ll * s.Tk * HD * 2);
  args.grp_k = locality_group(s.Hk * s.B, 1, 3ll * G * s.Tq * HD * 2);
  // The grouped kernels only where the groups split the pairs (packed ragged batches
  // keep the plain order). The persistent key pass groups only equal-weight items (no
  // causal mask): its static snake balances work only over a heaviest-first sequence,
  // which a grouped causal order is not (measured: key pass 2.24 -> 3.00 ms at causal
  // B1 H32 S8192 D128), while the query pass is balanced by the block scheduler.
  const bool grp_q = !VL && args.grp_q < s.H * s.B, grp_k = !VL && !s.causal && args.grp_k < s.Hk * s.B;
  const int nq = (s.Tq + kBM - 1) / kBM;
  const dim3 gq(s.H, s.B, nq), gq_grouped(s.H * s.B * nq);
  if (passes & (kPassFwdTangent | kPassQuery)) {
    const bool tj = (passes & kPassFwdTangent) != 0;
#define FH_Q_LAUNCH(TJ_, GRP_, GRID)                                                                       \
  bwdbwd_q_kernel<HD, GRP_ ? false : VL, TJ_, GRP_><<<GRID, kBBThreads, GQ::SMEM, stream>>>(                 \
      mq[0], mq[1], mq[2], mq[3], mq[4], mq[5], mq[6], mq[7], args)
    if (grp_q) {
      if (tj) FH_Q_LAUNCH(true, true, gq_grouped);
      else FH_Q_LAUNCH(false, true, gq_grouped);
    } else if (tj) {
      FH_Q_LAUNCH(true, false, gq);
    } else {
      FH_Q_LAUNCH(false, false, gq);
    }
#undef FH_Q_LAUNCH
    if (after_launch() != kOk) return kLaunchFailed;
  }
  if (passes & kPassKey) {
    // Persistent: one CTA per SM (at most one per work item).
    const int items = s.Hk * s.B * ((s.Tk + kBM - 1) / kBM);
    const dim3 gk(static_cast<unsigned>(items < sm_count() ? items : sm_count()));
    if (grp_k)
      bwdbwd_k_kernel<HD, false, true><<<gk, kBBThreads, GK::SMEM, stream>>>(mk[0], mk[1], mk[2], mk[3], mk[4], mk[5],
                                                                             mk[6], args);
    else
      bwdbwd_k_kernel<HD, VL, false><<<gk, kBBThreads, GK::SMEM, stream>>>(mk[0], mk[1], mk[2], mk[3], mk[4], mk[5],
                                                                            mk[6], args);
    if (after_launch() != kOk) return kLaunchFailed;
  }
  return kOk;
}

}  // namespace

int launch_bwdbwd(const AttnShape& s, int hd, const BwdBwdPtrs& p, int passes, int* status, cudaStream_t stream) {
  if (hd == 64) return s.cu_q ? launch_bwdbwd_hd<64, true>(s, p, passes, status, stream) : launch_bwdbwd_hd<64, false>(s, p, passes, status, stream);
  if (hd == 128) return s.cu_q ? launch_bwdbwd_hd<128, true>(s, p, passes, status, stream) : launch_bwdbwd_hd<128, false>(s, p, passes, status, stream);
  return kUnsupported;
}

}  // namespace fh
