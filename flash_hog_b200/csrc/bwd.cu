// First-order attention backward on sm_100a: dQ, dK, dV from (Q, K, V, O, dO, L),
// the rule the reference delegates to cuDNN
// (flash_hog/jax/_attention_impl.py:242-261; formulas of
// flash_hog/_jax_refs/jax_impl.py:142-191).
//
// Two launches, no atomics, no (Nq, Nk) intermediate in global memory:
//  * `bwd_dq_kernel`, query-tiled: one CTA per 128 query rows. It computes
//    D = rowsum(dO o O) for its rows (written out for the second launch), then
//    streams 64-key tiles of K, V:  S = Q K^T, dP = dO V^T,
//    dS/scale = P o (dP - D), dQ/scale += dS K;
//  * `bwd_dkdv_kernel`, key-tiled on transposed scores: one CTA per 128 key
//    rows; it streams 64-query tiles of Q, dO with their L and D:
//    S^T = K Q^T, dP^T = V dO^T, dV += P^T dO, dK/scale += dS^T Q.
//
// Both use the 11-warp layout of the double backward (two MMA issuers, a TMA
// producer, two elementwise warpgroups). The resident operand of every score
// product (Q and dO, or K and V) is copied into TMEM once per CTA, so the score
// MMAs read only the streamed tile from shared memory and run at the tensor
// core's math rate; the key-tiled pass folds -L/scale and -D into its score
// accumulators with one bias MMA per tile, so its elementwise warps read no
// per-query statistics.

#include <cuda_runtime.h>

#include <cmath>

#include "kernels.h"
#include "ws_common.cuh"

namespace fh {
namespace {

struct BwdArgs {
  AttnShape sh;
  const float* lse;
  float* delta;  // D = rowsum(dO o O): written by the query-tiled pass, read by the key-tiled pass
  __nv_bfloat16* dq;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  const __nv_bfloat16* dq_acc;  // optional addends of dq, dk, dv (may alias them)
  const __nv_bfloat16* dk_acc;
  const __nv_bfloat16* dv_acc;
  int* status;
  int grp_q;  // dQ pass: (query head, batch) pairs per locality group (grouped_order)
  int grp_k;  // dK/dV pass: (key head, batch) pairs per locality group
};

// ----------------------------------------------------------------------------------
// query-tiled pass: dQ (and D)
// ----------------------------------------------------------------------------------

template <int HD>
struct DqPass {
  static constexpr int BN = 64;  // keys per streamed tile
  static constexpr int ST = 4;   // ring depth
  static constexpr int RES = kBM * HD * 2;
  static constexpr int RES_PANEL = kBM * 128;
  static constexpr int STR = BN * HD * 2;
  static constexpr int STR_PANEL = BN * 128;
  static constexpr int SLOT = 2 * STR;                     // K, V
  static constexpr int SMEM = 1024 + 2 * RES + ST * SLOT;  // Q, dO, ring (O borrows the last slot)
  // Two layouts, both latency-bound loops made to overlap:
  //  * head_dim 64 -- two CTAs per SM: one score buffer [S | dP] and one bf16 dS
  //    operand shared by both elementwise warpgroups (each takes half the
  //    columns of every tile), score MMAs from shared memory; 224 TMEM columns
  //    and at most 93 registers a thread, so the two CTAs' tile loops (and one's
  //    prologue and the other's tiles) hide each other's waits;
  //  * head_dim 128 -- one CTA per SM: each warpgroup takes alternate key tiles
  //    with its own score buffer and dS operand ("ping-pong"), so one computes
  //    while the other waits; Q in TMEM as the A operand of S = Q K^T.
  // TMEM: score buffers, the dQ accumulator, the dS operands (BN/2 packed
  // columns each), then (ping-pong) Q as packed bf16.
  static constexpr bool PP = HD == 128;
  static constexpr int CTAS = PP ? 1 : 2;  // resident CTAs per SM
  static constexpr int NBUF = PP ? 2 : 1;  // score buffers and dS operands
  static constexpr int CW = PP ? BN : BN / 2;  // columns of a tile per elementwise thread
  static constexpr int ARRIVALS = PP ? kBBEwWarps / 2 : kBBEwWarps;  // warps consuming one buffer
  static constexpr int C_S = 0, C_DP = BN, SCORE_COLS = 2 * BN, OPS_COLS = BN / 2;
  static constexpr int C_DQ = NBUF * SCORE_COLS, C_OPS = C_DQ + HD, C_QT = C_OPS + NBUF * OPS_COLS;
  static constexpr int TMEM_COLS = PP ? 512 : 256;
  static_assert(C_QT + (PP ? HD / 2 : 0) <= TMEM_COLS, "TMEM budget");
  static_assert(CTAS * SMEM <= 228 * 1024 - CTAS * 2048, "shared memory of the resident CTAs");
  static_assert(RES <= SLOT, "O fits in one ring slot");
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(HD % 64 == 0 && RES_PANEL == kBM * 128, "tile shapes");
};

// Packed bf16 pairs of dS/scale = P (dP - D) for this thread's CW key columns
// (column pairs through the packed fp32x2 instructions).
template <int CW, bool MASK>
__device__ __forceinline__ void dq_ops(const uint32_t (&vs)[CW], const uint32_t (&vdp)[CW], int kc, int klo, int khi,
                                       float sc2, float lg, float dv, uint32_t (&o_ds)[CW / 2]) {
  const float2 m = make_float2(sc2, sc2), nl = make_float2(-lg, -lg), ndv = make_float2(-dv, -dv);
#pragma unroll
  for (int i = 0; i < CW; i += 2) {
    float2 s = __ffma2_rn(f2(vs[i], vs[i + 1]), m, nl);
    if (MASK) {
      if (kc + i > khi || kc + i < klo) s.x = -INFINITY;
      if (kc + i + 1 > khi || kc + i + 1 < klo) s.y = -INFINITY;
    }
    const float2 ds = __fmul2_rn(make_float2(ex2(s.x), ex2(s.y)), __fadd2_rn(f2(vdp[i], vdp[i + 1]), ndv));
    o_ds[i / 2] = pack_bf16(ds.x, ds.y);
  }
}

template <int HD, bool VL, bool GRP>
__global__ void __launch_bounds__(kBBThreads, DqPass<HD>::CTAS)
    bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                  const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                  const __grid_constant__ CUtensorMap tm_o, const BwdArgs a) {
  using G = DqPass<HD>;
  constexpr int BN = G::BN, ST = G::ST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* s_q = sm;
  uint8_t* s_do = s_q + G::RES;
  uint8_t* s_ring = s_do + G::RES;
  // O is staged in the last ring slot, which the first ST-1 key tiles do not
  // use; the producer refills it only once every elementwise warp has read O.
  uint8_t* s_o = s_ring + (ST - 1) * G::SLOT;
  __shared__ uint64_t bar_res, bar_tres, bar_ofree, bar_dred, bar_full[ST], bar_empty[ST];
  // Ping-pong: score buffer and dS operand w belong to elementwise warpgroup w,
  // which takes key tiles w, w + 2, ... Otherwise only index 0 is used.
  __shared__ uint64_t bar_sc_full[2], bar_sc_empty[2], bar_ops_full[2], bar_ops_empty[2], bar_acc;
  __shared__ float dred[2][kBM];  // partial rowsum(dO o O): warpgroup, row
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
  const int n = key_tiles(sh, q0, kBM, BN, &j0);  // key tiles j0, j0 + 1, ... (0: no row sees a key)

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar_res, 1);
    mbar_init(&bar_tres, kBBEwWarps);
    mbar_init(&bar_ofree, kBBEwWarps);
    mbar_init(&bar_dred, kBBEwWarps);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_sc_full[i], 1);
      mbar_init(&bar_sc_empty[i], G::ARRIVALS);
      mbar_init(&bar_ops_full[i], G::ARRIVALS);
      mbar_init(&bar_ops_empty[i], 1);
    }
    mbar_init(&bar_acc, 1);
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
      mbar_arrive_expect_tx(&bar_res, 3 * G::RES);
      tma_rows<HD>(s_q, &tm_q, &bar_res, sr.q0 + q0, kBM, h, sr.bc);
      tma_rows<HD>(s_do, &tm_do, &bar_res, sr.q0 + q0, kBM, h, sr.bc);
      tma_rows<HD>(s_o, &tm_o, &bar_res, sr.q0 + q0, kBM, h, sr.bc);
      int issued = 0;
      for (int it = 0; it < n; ++it) {
        const int s = it % ST;
        if (it >= ST && !mbar_wait(&bar_empty[s], ((it / ST) - 1) & 1, &abort_flag)) {
          raise_error(a.status, &abort_flag, kDevTimeoutSlotEmpty);
          break;
        }
        if (it == ST - 1 && !mbar_wait(&bar_ofree, 0, &abort_flag)) {
          raise_error(a.status, &abort_flag, kDevTimeoutSlotEmpty);
          break;
        }
        uint8_t* slot = s_ring + s * G::SLOT;
        mbar_arrive_expect_tx(&bar_full[s], G::SLOT);
        tma_rows<HD>(slot, &tm_k, &bar_full[s], sr.k0 + (j0 + it) * BN, BN, h / sh.G, sr.bc);
        tma_rows<HD>(slot + G::STR, &tm_v, &bar_full[s], sr.k0 + (j0 + it) * BN, BN, h / sh.G, sr.bc);
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
    //   S = Q K^T,  dP = dO V^T   (K, V K-major in the ring; Q from TMEM when ping-ponging)
    constexpr int KS = HD / 16;
    const uint32_t id_s = idesc_bf16_f32(kBM, BN, false, false);
    const uint64_t b_ring = kdesc(s_ring);  // K of slot 0
    const uint64_t a_q = kdesc(s_q), a_do = kdesc(s_do);
    constexpr uint64_t kSlot = G::SLOT >> 4, kStr = G::STR >> 4;
    bool ok = mbar_wait_warp(&bar_res, 0, &abort_flag) && mbar_wait_warp(&bar_tres, 0, &abort_flag);
    if (!ok && lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutTmaFull);
    for (int it = 0; ok && it < n; ++it) {
      const int s = it % ST, sb = G::PP ? (it & 1) : 0, u = G::PP ? (it >> 1) : it;
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
      if constexpr (G::PP)
        umma_chain_tsk_w<KS, G::STR_PANEL>(tb + G::C_S, tmem + G::C_QT, bk, id_s, false);
      else
        umma_chain_w<KS, G::RES_PANEL, G::STR_PANEL, false>(tb + G::C_S, a_q, bk, id_s, false);
      umma_chain_w<KS, G::RES_PANEL, G::STR_PANEL, false>(tb + G::C_DP, a_do, bk + kStr, id_s, false);
      umma_commit_w(&bar_sc_full[sb]);
    }
  } else if (warp == kBBWarpMmaOut) {
    // ----------------------------- operand MMA issuer -----------------------------
    //   dQ/scale += dS K   (dS in TMEM, K MN-major in the ring), tiles in order
    const uint32_t id_dq = idesc_bf16_f32(kBM, HD, false, true);
    const uint64_t mn_ring = mndesc(s_ring, G::STR_PANEL);
    constexpr uint64_t kSlot = G::SLOT >> 4;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int w = G::PP ? (j & 1) : 0;
      if (!mbar_wait_warp(&bar_ops_full[w], (G::PP ? (j >> 1) : j) & 1, &abort_flag)) {
        if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutEpilogue);
        ok = false;
        break;
      }
      tc_fence_after();
      const int s = j % ST;
      umma_chain_ts_w<BN / 16>(tmem + G::C_DQ, tmem + G::C_OPS + w * G::OPS_COLS, mn_ring + s * kSlot, id_dq, j > 0);
      umma_commit_w(&bar_ops_empty[w]);
      umma_commit_w(&bar_empty[s]);
    }
    if (ok) umma_commit_w(&bar_acc);
  } else {
    // --------------------------- elementwise warps ----------------------------
    const int wg = (warp - kBBFirstEwWarp) >> 2;  // takes key tiles wg, wg + 2, ...
    const int r = (warp & 3) * 32 + lane;         // TMEM lane = query row inside the tile
    const uint32_t lane_t = tmem + tmem_lane_base(warp & 3);
    const int row = q0 + r;
    const bool row_ok = row < sh.Tq;
    const size_t vi = q_stat(sh, sr, row_ok ? row : 0, h);
    const float lse = row_ok ? a.lse[vi] : 0.f;
    const float lg = lse > -INFINITY ? lse * kLog2e : 0.f;  // -inf: the row sees no key (all masked)
    const int khi = key_hi(sh, row), klo = key_lo(sh, row);
    const float sc2 = sh.scale * kLog2e;
    bool ok = mbar_wait_warp(&bar_res, 0, &abort_flag);
    float dv = 0.f;
    if (ok) {
      if constexpr (G::PP) {  // this warpgroup's half of the head_dim columns of Q into TMEM
        row_to_tmem<HD / 2>(s_q, r, wg * (HD / 2), lane_t + G::C_QT);
        tmem_wait_st();
      }
      warp_arrive(&bar_tres);
      // D = rowsum(dO o O) of this row: each warpgroup sums half the columns.
      dred[wg][r] = rowdot_share<HD>(s_o, s_do, r, wg);
      warp_arrive(&bar_ofree);  // O has been read: its ring slot may be refilled
      warp_arrive(&bar_dred);
      ok = mbar_wait_warp(&bar_dred, 0, &abort_flag);
      dv = dred[0][r] + dred[1][r];
      if (ok && wg == 0 && row_ok) a.delta[vi] = dv;
    }
    if constexpr (G::PP) {
      const uint32_t tb = tmem + wg * G::SCORE_COLS;
      const uint32_t to = lane_t + G::C_OPS + wg * G::OPS_COLS;
      for (int j = wg; ok && j < n; j += 2) {
        const int u = j >> 1;  // earlier tiles of this warpgroup
        ok = mbar_wait_warp(&bar_sc_full[wg], u & 1, &abort_flag);
        if (!ok) break;
        tc_fence_after();
        uint32_t vs[BN], vdp[BN];
        tmem_share<BN>(tb, warp, G::C_S, vs);
        tmem_share<BN>(tb, warp, G::C_DP, vdp);
        tmem_wait_ld();
        reg_fence(vs);
        reg_fence(vdp);
        warp_arrive(&bar_sc_empty[wg]);  // the tensor core may reuse this score buffer now
        const int kc = (j0 + j) * BN;
        const bool need_mask = kc + BN - 1 > khi || kc < klo;
        uint32_t o_ds[BN / 2];
        if (need_mask)
          dq_ops<BN, true>(vs, vdp, kc, klo, khi, sc2, lg, dv, o_ds);
        else
          dq_ops<BN, false>(vs, vdp, kc, klo, khi, sc2, lg, dv, o_ds);
        if (u > 0) ok = mbar_wait_warp(&bar_ops_empty[wg], (u - 1) & 1, &abort_flag);
        if (!ok) break;
        tc_fence_after();
        tmem_st16(to, *reinterpret_cast<const uint32_t(*)[16]>(&o_ds[0]));
        tmem_st16(to + 16, *reinterpret_cast<const uint32_t(*)[16]>(&o_ds[16]));
        tmem_wait_st();
        warp_arrive(&bar_ops_full[wg]);
      }
    } else {
      // Shared tiles: warpgroup wg takes columns [CW wg, CW wg + CW) of every tile.
      constexpr int CW = G::CW;
      const int cb = wg * CW;
      for (int j = 0; ok && j < n; ++j) {
        ok = mbar_wait_warp(&bar_sc_full[0], j & 1, &abort_flag);
        if (!ok) break;
        tc_fence_after();
        uint32_t vs[CW], vdp[CW];
        tmem_share<CW>(tmem, warp, G::C_S + cb, vs);
        tmem_share<CW>(tmem, warp, G::C_DP + cb, vdp);
        tmem_wait_ld();
        reg_fence(vs);
        reg_fence(vdp);
        warp_arrive(&bar_sc_empty[0]);
        const int kc = (j0 + j) * BN + cb;  // first key of this thread's columns
        const bool need_mask = kc + CW - 1 > khi || kc < klo;
        uint32_t o_ds[CW / 2];
        if (need_mask)
          dq_ops<CW, true>(vs, vdp, kc, klo, khi, sc2, lg, dv, o_ds);
        else
          dq_ops<CW, false>(vs, vdp, kc, klo, khi, sc2, lg, dv, o_ds);
        if (j > 0) ok = mbar_wait_warp(&bar_ops_empty[0], (j - 1) & 1, &abort_flag);
        if (!ok) break;
        tc_fence_after();
        tmem_st_ops(lane_t + G::C_OPS + (CW / 2) * wg, o_ds);
        tmem_wait_st();
        warp_arrive(&bar_ops_full[0]);
      }
    }
    if (ok && n == 0) {
      // No key tile: dQ = 0 (plus the addend).
      const size_t off = q_row(sh, sr, row_ok ? row : 0, h) + wg * (HD / 2);
      for (int c = 0; row_ok && c < HD / 2; c += 8)
        reinterpret_cast<uint4*>(a.dq + off + c)[0] =
            a.dq_acc ? reinterpret_cast<const uint4*>(a.dq_acc + off + c)[0] : make_uint4(0, 0, 0, 0);
    } else if (ok) {
      ok = mbar_wait_warp(&bar_acc, 0, &abort_flag);
    }
    if (ok && n > 0) {
      tc_fence_after();
      const int srow = row_ok ? row : 0;
      const size_t off = q_row(sh, sr, srow, h) + wg * (HD / 2);
      tmem_row_to_global<HD / 2>(tmem, warp, G::C_DQ + wg * (HD / 2), a.dq + off, row_ok, sh.scale,
                                 a.dq_acc ? a.dq_acc + off : nullptr);
    } else if (!ok && threadIdx.x == kBBFirstEwWarp * 32) {
      raise_error(a.status, &abort_flag, kDevTimeoutMma);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kBBWarpMma) tmem_dealloc(tmem, G::TMEM_COLS);
}

// ----------------------------------------------------------------------------------
// key-tiled pass: dK, dV
// ----------------------------------------------------------------------------------

template <int HD>
struct DkvPass {
  // Two layouts:
  //  * head_dim 64 -- two CTAs per SM: one score buffer [S^T | dP^T] into which
  //    the elementwise warps write the bf16 operands P^T and dS^T back once both
  //    warpgroups have read their scores; K and V stay in shared memory; 256 TMEM
  //    columns. One warp issues every MMA, so each tile's operand products are
  //    ordered before the next tile's bias MMA overwrites the buffer. The two
  //    CTAs hide each other's waits;
  //  * head_dim 128 -- one CTA per SM: separate operand columns, K in TMEM as the
  //    A operand of S^T = K Q^T.
  static constexpr bool TWO = HD == 64;
  static constexpr int CTAS = TWO ? 2 : 1;
  static constexpr int BN = 64;  // queries per streamed tile
  static constexpr int ST = TWO ? 3 : 4;
  static constexpr int CW = BN / 2;
  static constexpr int RES = kBM * HD * 2;
  static constexpr int RES_PANEL = kBM * 128;
  static constexpr int STR = BN * HD * 2;
  static constexpr int STR_PANEL = BN * 128;
  // Per-query biases of the two score products as a K = 16 bf16 operand (32-byte
  // rows, 32B swizzle): rows [0, BN) hold -L/scale, rows [BN, 2 BN) hold -D, each
  // a (hi, lo) bf16 pair in columns 0-1, zeros after.
  static constexpr int BIAS_ROW = 32;
  static constexpr int BIAS = 2 * BN * BIAS_ROW;
  static constexpr int ONES = kBM * BIAS_ROW;  // resident A operand: (1, 1, 0, ...) per key row
  static constexpr int SLOT = 2 * STR + BIAS;  // Q, dO, biases
  static constexpr int SMEM = 1024 + 2 * RES + ONES + ST * SLOT;
  // TMEM: the score buffer [S^T | dP^T], the dK and dV accumulators, the bf16
  // operands P^T and dS^T (over the scores, or after the accumulators), then
  // (one CTA per SM) K as packed bf16.
  static constexpr int C_S = 0, C_DP = BN, SCORE_COLS = 2 * BN, OPS_COLS = BN / 2;
  static constexpr int C_DK = SCORE_COLS, C_DV = C_DK + HD;
  static constexpr int C_P = TWO ? C_S : C_DV + HD, C_DS = TWO ? C_DP : C_P + OPS_COLS;
  static constexpr int C_KT = C_DV + HD + 2 * OPS_COLS;
  static constexpr int TMEM_COLS = TWO ? 256 : 512;
  static_assert(TWO ? C_DV + HD <= TMEM_COLS : C_KT + HD / 2 <= TMEM_COLS, "TMEM budget");
  static_assert(CTAS * SMEM <= 228 * 1024 - CTAS * 2048, "shared memory of the resident CTAs");
  static_assert(C_DP == C_S + BN, "one bias MMA covers both products");
  static_assert(SLOT % 1024 == 0 && (2 * RES + ONES) % 1024 == 0, "slots must keep panels 1024-byte aligned");
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(CW % 16 == 0 && HD % 64 == 0 && RES_PANEL == kBM * 128, "tile shapes");
};

// Packed bf16 pairs of P^T and dS^T/scale = P^T (dP^T - D) for this thread's CW
// query columns; the statistics arrive folded into the scores by the bias MMA:
//   vs = S - L/scale,  vdp = dP - D.
template <int CW, bool MASK>
__device__ __forceinline__ void dkv_ops(const uint32_t (&vs)[CW], const uint32_t (&vdp)[CW], int qc, int qlo, int qhi,
                                        float sc2, uint32_t (&o_p)[CW / 2], uint32_t (&o_ds)[CW / 2]) {
  const float2 m = make_float2(sc2, sc2);
#pragma unroll
  for (int i = 0; i < CW; i += 2) {
    float2 s = __fmul2_rn(f2(vs[i], vs[i + 1]), m);
    if (MASK) {
      if (qc + i > qhi || qc + i < qlo) s.x = -INFINITY;
      if (qc + i + 1 > qhi || qc + i + 1 < qlo) s.y = -INFINITY;
    }
    const float2 p = make_float2(ex2(s.x), ex2(s.y));
    const float2 ds = __fmul2_rn(p, f2(vdp[i], vdp[i + 1]));
    o_p[i / 2] = pack_bf16(p.x, p.y);
    o_ds[i / 2] = pack_bf16(ds.x, ds.y);
  }
}

template <int HD, bool VL, bool GRP>
__global__ void __launch_bounds__(kBBThreads, DkvPass<HD>::CTAS)
    bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                    const BwdArgs a) {
  using G = DkvPass<HD>;
  constexpr int BN = G::BN, ST = G::ST, CW = G::CW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* s_k = sm;
  uint8_t* s_v = s_k + G::RES;
  uint8_t* s_ones = s_v + G::RES;
  uint8_t* s_ring = s_ones + G::ONES;
  __shared__ uint64_t bar_res, bar_tres, bar_full[ST], bar_empty[ST];
  __shared__ uint64_t bar_sc_full, bar_sc_empty, bar_ops_full, bar_ops_empty, bar_acc;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Grid (Hk, B, key tiles), key tile 0 first (the most causal query tiles); GRP: a
  // 1-D grid in the locality-grouped order.
  int hk = blockIdx.x, b = blockIdx.y, kt = blockIdx.z;
  if constexpr (GRP) {
    int hb;
    grouped_order(blockIdx.x, (a.sh.Tk + kBM - 1) / kBM, a.sh.Hk * a.sh.B, a.grp_k, &kt, &hb);
    hk = hb % a.sh.Hk, b = hb / a.sh.Hk;
  }
  SeqRange sr;
  const AttnShape sh = seq_shape<VL>(a.sh, b, &sr);
  const int k0 = kt * kBM;
  int qt_begin;
  const int n = query_tiles(sh, k0, kBM, BN, &qt_begin);  // query tiles that see any of these keys
  const int total = n * sh.G;  // streamed tiles: n per query head of the group

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar_res, 1);
    mbar_init(&bar_tres, kBBEwWarps);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    mbar_init(&bar_sc_full, 1);
    mbar_init(&bar_sc_empty, kBBEwWarps);  // both layouts: every score share has been read
    mbar_init(&bar_ops_full, kBBEwWarps);
    mbar_init(&bar_ops_empty, 1);
    mbar_init(&bar_acc, 1);
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

  if (total == 0) {
    // No query sees these keys (causal with Tk > Tq): the gradients are zero.
    if (warp >= kBBFirstEwWarp) {
      const int wg = (warp - kBBFirstEwWarp) >> 2;
      const int key = k0 + (warp & 3) * 32 + lane;
      const size_t off = k_row(sh, sr, key < sh.Tk ? key : 0, hk);
      const __nv_bfloat16* add = wg == 0 ? a.dk_acc : a.dv_acc;
      __nv_bfloat16* dst = (wg == 0 ? a.dk : a.dv) + off;
      if (key < sh.Tk) {
        if (add) {  // the outputs are the addends
          for (int c = 0; c < HD; c += 8)
            reinterpret_cast<uint4*>(dst + c)[0] = reinterpret_cast<const uint4*>(add + off + c)[0];
        } else {
          zero_row_global<HD>(dst);
        }
      }
    }
  } else if (warp == kBBWarpProducer) {
    // ---------------------- TMA producer (whole warp) -----------------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_q);
      mbar_arrive_expect_tx(&bar_res, 2 * G::RES);
      tma_rows<HD>(s_k, &tm_k, &bar_res, sr.k0 + k0, kBM, hk, sr.bc);
      tma_rows<HD>(s_v, &tm_v, &bar_res, sr.k0 + k0, kBM, hk, sr.bc);
    }
    const float inv_scale = 1.f / sh.scale;
    constexpr int RPL = BN / 32;
    // L and D of the queries of streamed tile `it`, into registers.
    auto load_stats = [&](int it, float (&raw)[RPL][2]) {
      const int q0 = (qt_begin + it % n) * BN;
      const int h = hk * sh.G + it / n;
#pragma unroll
      for (int k = 0; k < RPL; ++k) {
        const int q = q0 + lane + 32 * k;
        const size_t idx = q_stat(sh, sr, q < sh.Tq ? q : 0, h);
        raw[k][0] = a.lse[idx];
        raw[k][1] = a.delta[idx];
      }
    };
    float raw_next[RPL][2];
    load_stats(0, raw_next);
    int issued = 0;
    for (int it = 0; it < total; ++it) {
      const int s = it % ST;
      const int q0 = (qt_begin + it % n) * BN;
      const int h = hk * sh.G + it / n;  // query head of this tile
      if (it >= ST && !mbar_wait_warp(&bar_empty[s], ((it / ST) - 1) & 1, &abort_flag)) {
        if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutSlotEmpty);
        break;
      }
      uint8_t* slot = s_ring + s * G::SLOT;
      // Copies first (their bytes are expected without arriving), then the
      // biases; the single arrive after the biases completes the slot's phase
      // together with the copies.
      if (lane == 0) {
        mbar_expect_tx(&bar_full[s], 2 * G::STR);
        tma_rows<HD>(slot, &tm_q, &bar_full[s], sr.q0 + q0, BN, h, sr.bc);
        tma_rows<HD>(slot + G::STR, &tm_do, &bar_full[s], sr.q0 + q0, BN, h, sr.bc);
      }
      float raw[RPL][2];
#pragma unroll
      for (int k = 0; k < RPL; ++k) {
        raw[k][0] = raw_next[k][0];
        raw[k][1] = raw_next[k][1];
      }
      const uint32_t bias = smem_u32(slot + 2 * G::STR);
#pragma unroll
      for (int k = 0; k < RPL; ++k) {
        // Queries past the end, or with L = -inf (no visible key: every element of
        // theirs is masked), get a zero bias.
        const bool v = q0 + lane + 32 * k < sh.Tq && raw[k][0] > -INFINITY;
        const int r = lane + 32 * k;
        store_bias_row(bias, r, v ? -raw[k][0] * inv_scale : 0.f);  // S - L/scale
        store_bias_row(bias, BN + r, v ? -raw[k][1] : 0.f);         // dP - D
      }
      fence_async_smem();  // the tensor core reads the biases through the async proxy
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_full[s]);
      issued = it + 1;
      if (it + 1 < total) load_stats(it + 1, raw_next);
    }
    if (lane == 0) {
      // Every issued copy must land before this CTA's shared memory is released.
      bool drained = mbar_wait(&bar_res, 0, nullptr);
      for (int t = issued > ST ? issued - ST : 0; t < issued; ++t)
        drained &= mbar_wait(&bar_full[t % ST], (t / ST) & 1, nullptr);
      if (!drained) raise_error(a.status, &abort_flag, kDevTimeoutDrain);
    }
  } else if (warp == kBBWarpMma) {
    // ------------------------------ score MMA issuer ------------------------------
    //   [S^T | dP^T] = ones [-L/scale ; -D]^T,  S^T += K Q^T,  dP^T += V dO^T
    constexpr int KS = HD / 16;
    const uint32_t id_s = idesc_bf16_f32(kBM, BN, false, false);
    const uint32_t id_bias = idesc_bf16_f32(kBM, 2 * BN, false, false);
    const uint64_t b_q = kdesc(s_ring);  // Q of slot 0; dO follows at +STR
    const uint64_t a_k = kdesc(s_k), a_v = kdesc(s_v);
    constexpr int KO = BN / 16;
    const uint32_t id_o = idesc_bf16_f32(kBM, HD, false, true);
    const uint64_t mn_q = mndesc(s_ring, G::STR_PANEL);
    const uint64_t mn_do = mndesc(s_ring + G::STR, G::STR_PANEL);
    const uint64_t a_ones = smem_desc(smem_u32(s_ones), 16, 8 * G::BIAS_ROW, kSwizzle32B);
    const uint64_t b_bias = smem_desc(smem_u32(s_ring + 2 * G::STR), 16, 8 * G::BIAS_ROW, kSwizzle32B);
    constexpr uint64_t kSlot = G::SLOT >> 4, kStr = G::STR >> 4;
    bool ok = mbar_wait_warp(&bar_res, 0, &abort_flag) && mbar_wait_warp(&bar_tres, 0, &abort_flag);
    if (!ok && lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutTmaFull);
    for (int it = 0; ok && it < total; ++it) {
      const int s = it % ST;
      if (!mbar_wait_warp(&bar_full[s], (it / ST) & 1, &abort_flag)) {
        if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutTmaFull);
        break;
      }
      // One CTA per SM: the score buffer is free once its scores were read.
      if (!G::TWO && it > 0 && !mbar_wait_warp(&bar_sc_empty, (it - 1) & 1, &abort_flag)) {
        if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      const uint64_t bq = b_q + s * kSlot;
      umma_bf16_w(tmem + G::C_S, a_ones, b_bias + s * kSlot, id_bias, 0u);
      if constexpr (G::TWO)
        umma_chain_w<KS, G::RES_PANEL, G::STR_PANEL, false>(tmem + G::C_S, a_k, bq, id_s, true);
      else
        umma_chain_tsk_w<KS, G::STR_PANEL>(tmem + G::C_S, tmem + G::C_KT, bq, id_s, true);
      umma_chain_w<KS, G::RES_PANEL, G::STR_PANEL, false>(tmem + G::C_DP, a_v, bq + kStr, id_s, true);
      umma_commit_w(&bar_sc_full);
      if constexpr (G::TWO) {
        // The operand products of this tile, issued before the next tile's bias
        // MMA overwrites the operands (the tensor core runs in issue order).
        if (!mbar_wait_warp(&bar_ops_full, it & 1, &abort_flag)) {
          if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutEpilogue);
          ok = false;
          break;
        }
        tc_fence_after();
        umma_chain_ts_w<KO>(tmem + G::C_DV, tmem + G::C_P, mn_do + s * kSlot, id_o, it > 0);
        umma_chain_ts_w<KO>(tmem + G::C_DK, tmem + G::C_DS, mn_q + s * kSlot, id_o, it > 0);
        umma_commit_w(&bar_empty[s]);
      }
    }
    if (G::TWO && ok) umma_commit_w(&bar_acc);
  } else if (warp == kBBWarpMmaOut) {
    // ----------------------- operand MMA issuer (one CTA per SM) -----------------------
    //   dV += P^T dO,  dK/scale += dS^T Q   (A in TMEM, B MN-major in the ring)
    constexpr int KO = BN / 16;
    const uint32_t id_o = idesc_bf16_f32(kBM, HD, false, true);
    const uint64_t mn_q = mndesc(s_ring, G::STR_PANEL);
    const uint64_t mn_do = mndesc(s_ring + G::STR, G::STR_PANEL);
    constexpr uint64_t kSlot = G::SLOT >> 4;
    bool ok = true;
    for (int it = 0; !G::TWO && it < total; ++it) {
      if (!mbar_wait_warp(&bar_ops_full, it & 1, &abort_flag)) {
        if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutEpilogue);
        ok = false;
        break;
      }
      tc_fence_after();
      const int s = it % ST;
      umma_chain_ts_w<KO>(tmem + G::C_DV, tmem + G::C_P, mn_do + s * kSlot, id_o, it > 0);
      umma_chain_ts_w<KO>(tmem + G::C_DK, tmem + G::C_DS, mn_q + s * kSlot, id_o, it > 0);
      umma_commit_w(&bar_ops_empty);
      umma_commit_w(&bar_empty[s]);
    }
    if (!G::TWO && ok) umma_commit_w(&bar_acc);
  } else {
    // --------------------------- elementwise warps ----------------------------
    const int wg = (warp - kBBFirstEwWarp) >> 2;
    const int r = (warp & 3) * 32 + lane;  // TMEM lane = key row inside the tile
    const uint32_t lane_t = tmem + tmem_lane_base(warp & 3);
    const int cb = wg * CW;
    const int key = k0 + r;
    const bool key_ok = key < sh.Tk;
    const int qhi = query_hi(sh, key), qlo = query_lo(sh, key);  // queries that see this key
    const float sc2 = sh.scale * kLog2e;
    bool ok = mbar_wait_warp(&bar_res, 0, &abort_flag);
    if (ok) {
      if constexpr (!G::TWO) {  // this warpgroup's half of the head_dim columns of K into TMEM
        row_to_tmem<HD / 2>(s_k, r, wg * (HD / 2), lane_t + G::C_KT);
        tmem_wait_st();
      }
      warp_arrive(&bar_tres);
    }
    for (int it = 0; ok && it < total; ++it) {
      ok = mbar_wait_warp(&bar_sc_full, it & 1, &abort_flag);
      if (!ok) break;
      tc_fence_after();
      const int qc = (qt_begin + it % n) * BN + cb;  // first query of this thread's columns
      // Two CTAs per SM (80 registers a thread): the share in two halves of CW/2
      // columns, so half the scores are live at a time.
      constexpr int HW = G::TWO ? CW / 2 : CW, NH = CW / HW;
      uint32_t o_p[NH][HW / 2], o_ds[NH][HW / 2];
#pragma unroll
      for (int hf = 0; hf < NH; ++hf) {
        uint32_t vs[HW], vdp[HW];
        tmem_share<HW>(tmem, warp, G::C_S + cb + hf * HW, vs);
        tmem_share<HW>(tmem, warp, G::C_DP + cb + hf * HW, vdp);
        tmem_wait_ld();
        reg_fence(vs);
        reg_fence(vdp);
        if (hf == NH - 1) warp_arrive(&bar_sc_empty);  // this warp has read all its scores
        const int qh = qc + hf * HW;
        if (qh + HW - 1 > qhi || qh < qlo)
          dkv_ops<HW, true>(vs, vdp, qh, qlo, qhi, sc2, o_p[hf], o_ds[hf]);
        else
          dkv_ops<HW, false>(vs, vdp, qh, qlo, qhi, sc2, o_p[hf], o_ds[hf]);
      }
      // Two CTAs per SM: the operands overwrite score columns that the other
      // warpgroup reads, so wait until both have read theirs. One CTA per SM:
      // wait until the previous operands have been consumed.
      if constexpr (G::TWO)
        ok = mbar_wait_warp(&bar_sc_empty, it & 1, &abort_flag);
      else if (it > 0)
        ok = mbar_wait_warp(&bar_ops_empty, (it - 1) & 1, &abort_flag);
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int hf = 0; hf < NH; ++hf) {
        tmem_st_ops(lane_t + G::C_P + (CW / 2) * wg + hf * (HW / 2), o_p[hf]);
        tmem_st_ops(lane_t + G::C_DS + (CW / 2) * wg + hf * (HW / 2), o_ds[hf]);
      }
      tmem_wait_st();
      warp_arrive(&bar_ops_full);
    }
    if (ok) ok = mbar_wait_warp(&bar_acc, 0, &abort_flag);
    if (ok) {
      tc_fence_after();
      const size_t off = k_row(sh, sr, key_ok ? key : 0, hk);
      const __nv_bfloat16* add = wg == 0 ? a.dk_acc : a.dv_acc;
      tmem_row_to_global<HD>(tmem, warp, wg == 0 ? G::C_DK : G::C_DV, (wg == 0 ? a.dk : a.dv) + off, key_ok,
                             wg == 0 ? sh.scale : 1.f, add ? add + off : nullptr);
    } else if (threadIdx.x == kBBFirstEwWarp * 32) {
      raise_error(a.status, &abort_flag, kDevTimeoutMma);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kBBWarpMma) tmem_dealloc(tmem, G::TMEM_COLS);
}

template <int HD, bool VL>
int launch_bwd_hd(const AttnShape& s, const BwdPtrs& p, int* status, cudaStream_t stream) {
  using GQ = DqPass<HD>;
  using GK = DkvPass<HD>;
  CUtensorMap mq[5], mk[4];
  bool ok = make_seq_map(&mq[0], p.q, HD, s.total_q, s.H, map_batch(s), s.sq, kBM) &&
            make_seq_map(&mq[1], p.dO, HD, s.total_q, s.H, map_batch(s), s.sq, kBM) &&
            make_seq_map(&mq[2], p.k, HD, s.total_k, s.Hk, map_batch(s), s.sk, GQ::BN) &&
            make_seq_map(&mq[3], p.v, HD, s.total_k, s.Hk, map_batch(s), s.sk, GQ::BN) &&
            make_seq_map(&mq[4], p.o, HD, s.total_q, s.H, map_batch(s), s.sq, kBM) &&
            make_seq_map(&mk[0], p.k, HD, s.total_k, s.Hk, map_batch(s), s.sk, kBM) &&
            make_seq_map(&mk[1], p.v, HD, s.total_k, s.Hk, map_batch(s), s.sk, kBM) &&
            make_seq_map(&mk[2], p.q, HD, s.total_q, s.H, map_batch(s), s.sq, GK::BN) &&
            make_seq_map(&mk[3], p.dO, HD, s.total_q, s.H, map_batch(s), s.sq, GK::BN);
  if (!ok) return kInvalidArgument;
  if (ensure_smem_limit(reinterpret_cast<const void*>(&bwd_dq_kernel<HD, VL, false>), GQ::SMEM) != kOk ||
      ensure_smem_limit(reinterpret_cast<const void*>(&bwd_dkdv_kernel<HD, VL, false>), GK::SMEM) != kOk)
    return kLaunchFailed;
  if constexpr (!VL) {
    if (ensure_smem_limit(reinterpret_cast<const void*>(&bwd_dq_kernel<HD, false, true>), GQ::SMEM) != kOk ||
        ensure_smem_limit(reinterpret_cast<const void*>(&bwd_dkdv_kernel<HD, false, true>), GK::SMEM) != kOk)
      return kLaunchFailed;
  }
  BwdArgs args{s,
               p.lse,
               p.delta,
               static_cast<__nv_bfloat16*>(p.dq),
               static_cast<__nv_bfloat16*>(p.dk),
               static_cast<__nv_bfloat16*>(p.dv),
               static_cast<const __nv_bfloat16*>(p.dq_acc),
               static_cast<const __nv_bfloat16*>(p.dk_acc),
               static_cast<const __nv_bfloat16*>(p.dv_acc),
               status,
               // Shared streamed tiles per head: K and V of a key head (dQ pass); Q and
               // dO of its query heads (dK/dV pass).
               locality_group(s.H * s.B, s.H / s.Hk, 2ll * s.Tk * HD * 2),
               locality_group(s.Hk * s.B, 1, 2ll * (s.H / s.Hk) * s.Tq * HD * 2)};
  // The grouped kernels only where the groups split the pairs.
  const int nq = (s.Tq + kBM - 1) / kBM, nk = (s.Tk + kBM - 1) / kBM;
  if (!VL && args.grp_q < s.H * s.B)
    bwd_dq_kernel<HD, false, true><<<dim3(s.H * s.B * nq), kBBThreads, GQ::SMEM, stream>>>(mq[0], mq[1], mq[2], mq[3],
                                                                                         mq[4], args);
  else
    bwd_dq_kernel<HD, VL, false><<<dim3(s.H, s.B, nq), kBBThreads, GQ::SMEM, stream>>>(mq[0], mq[1], mq[2], mq[3],
                                                                                     mq[4], args);
  if (after_launch() != kOk) return kLaunchFailed;
  if (!VL && args.grp_k < s.Hk * s.B)
    bwd_dkdv_kernel<HD, false, true><<<dim3(s.Hk * s.B * nk), kBBThreads, GK::SMEM, stream>>>(mk[0], mk[1], mk[2],
                                                                                            mk[3], args);
  else
    bwd_dkdv_kernel<HD, VL, false><<<dim3(s.Hk, s.B, nk), kBBThreads, GK::SMEM, stream>>>(mk[0], mk[1], mk[2], mk[3],
                                                                                        args);
  return after_launch();
}

}  // namespace

int launch_bwd(const AttnShape& s, int hd, const BwdPtrs& p, int* status, cudaStream_t stream) {
  if (hd == 64) return s.cu_q ? launch_bwd_hd<64, true>(s, p, status, stream) : launch_bwd_hd<64, false>(s, p, status, stream);
  if (hd == 128) return s.cu_q ? launch_bwd_hd<128, true>(s, p, status, stream) : launch_bwd_hd<128, false>(s, p, status, stream);
  return kUnsupported;
}

}  // namespace fh
