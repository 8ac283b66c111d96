// First-order attention backward on sm_100a: dQ, dK, dV from (Q, K, V, O, dO, L),
// the rule the reference delegates to cuDNN
// (flash_hog/jax/_attention_impl.py:242-261; formulas of
// flash_hog/_jax_refs/jax_impl.py:142-191).
//
// Atomic-free split into two launches after the D = rowsum(dO o O) pre-pass:
//  * `bwd_dq_kernel`, query-tiled: S = Q K^T, dP = dO V^T,
//    dS = scale P o (dP - D), dQ += dS K;
//  * `bwd_dkdv_kernel`, key-tiled on transposed scores: S^T = K Q^T,
//    dP^T = V dO^T, dV += P^T dO, dK += dS^T Q.

#include <cuda_runtime.h>

#include <cmath>

#include "kernels.h"

namespace fh {
namespace {

struct BwdArgs {
  AttnShape sh;
  const float* lse;
  const float* delta;
  __nv_bfloat16* dq;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  int* status;
};

constexpr int round_up_1024(int x) { return (x + 1023) / 1024 * 1024; }

template <int HD>
struct DqPass {
  static constexpr int BN = 64, ST = 3;
  static constexpr int RES = kBM * HD * 2;
  static constexpr int STR = BN * HD * 2;
  static constexpr int SLOT = 2 * STR;  // K | V
  static constexpr int OPS = kBM * BN * 2;
  static constexpr int SMEM = 1024 + 2 * RES + ST * SLOT + OPS;
  static constexpr int C_S = 0, C_DP = BN, C_DQ = 2 * BN;
  static constexpr int TMEM_COLS = 256;
  static_assert(C_DQ + HD <= TMEM_COLS, "TMEM budget");
};

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                  const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                  const BwdArgs a) {
  using G = DqPass<HD>;
  constexpr int BN = G::BN, ST = G::ST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* s_q = sm;
  uint8_t* s_do = s_q + G::RES;
  uint8_t* s_ring = s_do + G::RES;
  uint8_t* s_ops = s_ring + ST * G::SLOT;
  __shared__ uint64_t bar_res, bar_full[ST], bar_empty[ST];
  __shared__ uint64_t bar_sc_full, bar_sc_empty, bar_ops_full, bar_ops_empty, bar_acc;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const AttnShape& sh = a.sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x, b = blockIdx.y;
  const int qt = gridDim.z - 1 - blockIdx.z;
  const int q0 = qt * kBM;
  const int kv_end = sh.causal ? min(sh.Tk, q0 + kBM) : sh.Tk;
  const int n = (kv_end + BN - 1) / BN;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar_res, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    mbar_init(&bar_sc_full, 1);
    mbar_init(&bar_sc_empty, kEwThreads);
    mbar_init(&bar_ops_full, kEwThreads);
    mbar_init(&bar_ops_empty, 1);
    mbar_init(&bar_acc, 1);
    mbar_fence_init();
  }
  if (warp == kWarpMma) tmem_alloc(&tmem_base, G::TMEM_COLS);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == kWarpProducer) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      mbar_arrive_expect_tx(&bar_res, 2 * G::RES);
      tma_rows<HD>(s_q, &tm_q, &bar_res, q0, kBM, h, b);
      tma_rows<HD>(s_do, &tm_do, &bar_res, q0, kBM, h, b);
      int issued = 0;
      for (int it = 0; it < n; ++it) {
        const int s = it % ST;
        if (it >= ST && !mbar_wait(&bar_empty[s], ((it / ST) - 1) & 1, &abort_flag)) {
          raise_error(a.status, &abort_flag, kDevTimeoutSlotEmpty);
          break;
        }
        uint8_t* slot = s_ring + s * G::SLOT;
        mbar_arrive_expect_tx(&bar_full[s], G::SLOT);
        tma_rows<HD>(slot, &tm_k, &bar_full[s], it * BN, BN, h / sh.G, b);
        tma_rows<HD>(slot + G::STR, &tm_v, &bar_full[s], it * BN, BN, h / sh.G, b);
        issued = it + 1;
      }
      bool drained = mbar_wait(&bar_res, 0, nullptr);
      for (int it = issued > ST ? issued - ST : 0; it < issued; ++it)
        drained &= mbar_wait(&bar_full[it % ST], (it / ST) & 1, nullptr);
      if (!drained) raise_error(a.status, &abort_flag, kDevTimeoutDrain);
    }
  } else if (warp == kWarpMma) {
    if (lane == 0) {
      const uint32_t id_sc = idesc_bf16_f32(kBM, BN, false, false);
      const uint32_t id_out = idesc_bf16_f32(kBM, HD, false, true);
      bool ok = mbar_wait(&bar_res, 0, &abort_flag);
      if (!ok) raise_error(a.status, &abort_flag, kDevTimeoutTmaFull);
      for (int it = 0; ok && it <= n; ++it) {
        if (it < n) {
          const int s = it % ST;
          if (!mbar_wait(&bar_full[s], (it / ST) & 1, &abort_flag) ||
              (it > 0 && !mbar_wait(&bar_sc_empty, (it - 1) & 1, &abort_flag))) {
            raise_error(a.status, &abort_flag, kDevTimeoutTmaFull);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* slot = s_ring + s * G::SLOT;
          gemm_abt(tmem + G::C_S, s_q, slot, BN, HD / 16, id_sc, false);              // S  = Q K^T
          gemm_abt(tmem + G::C_DP, s_do, slot + G::STR, BN, HD / 16, id_sc, false);   // dP = dO V^T
          umma_commit(&bar_sc_full);
        }
        const int t = it - 1;
        if (t >= 0) {
          if (!mbar_wait(&bar_ops_full, t & 1, &abort_flag)) {
            raise_error(a.status, &abort_flag, kDevTimeoutEpilogue);
            ok = false;
            break;
          }
          tc_fence_after();
          const int sp = t % ST;
          gemm_ab(tmem + G::C_DQ, s_ops, s_ring + sp * G::SLOT, BN, BN / 16, id_out, t > 0);  // dQ += dS K
          umma_commit(&bar_ops_empty);
          umma_commit(&bar_empty[sp]);
        }
      }
      if (ok) umma_commit(&bar_acc);
    }
  } else {
    const int r = threadIdx.x;
    const int row = q0 + r;
    const bool row_ok = row < sh.Tq;
    const size_t vi = stat_index(b, h, row_ok ? row : 0, sh.H, sh.Tq);
    const float lg = row_ok ? a.lse[vi] * kLog2e : 0.f;
    const float dv = row_ok ? a.delta[vi] : 0.f;
    const float sc = sh.scale, sc2 = sh.scale * kLog2e;
    bool ok = true;
    for (int it = 0; it < n; ++it) {
      const int k0 = it * BN;
      ok = __all_sync(0xffffffffu, mbar_wait(&bar_sc_full, it & 1, &abort_flag));
      if (ok && it > 0) ok = __all_sync(0xffffffffu, mbar_wait(&bar_ops_empty, (it - 1) & 1, &abort_flag));
      if (!ok) break;
      tc_fence_after();
      const bool need_mask = (k0 + BN > sh.Tk) || (sh.causal && k0 + BN - 1 > q0);
#pragma unroll 1
      for (int c = 0; c < BN / 16; ++c) {
        uint32_t vs[16], vdp[16];
        tmem_row16(tmem, warp, G::C_S + c * 16, vs);
        tmem_row16(tmem, warp, G::C_DP + c * 16, vdp);
        tmem_wait_ld();
        reg_fence16(vs);
        reg_fence16(vdp);
        float o_ds[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int key = k0 + c * 16 + i;
          float s = fmaf(__uint_as_float(vs[i]), sc2, -lg);
          if (need_mask && (key >= sh.Tk || (sh.causal && key > row))) s = -INFINITY;
          const float p = ex2(s);
          o_ds[i] = p * sc * (__uint_as_float(vdp[i]) - dv);
        }
        stage_bf16x16(s_ops, r, c, o_ds);
      }
      tc_fence_before();
      mbar_arrive(&bar_sc_empty);
      fence_async_smem();
      mbar_arrive(&bar_ops_full);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bar_acc, 0, &abort_flag));
    if (ok) {
      tc_fence_after();
      tmem_row_to_global<HD>(tmem, warp, G::C_DQ, a.dq + row_offset(sh.sq, b, row_ok ? row : 0, h), row_ok);
    } else if (threadIdx.x == 0) {
      raise_error(a.status, &abort_flag, kDevTimeoutMma);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) tmem_dealloc(tmem, G::TMEM_COLS);
}

template <int HD>
struct DkvPass {
  static constexpr int BN = 64, ST = 3;
  static constexpr int RES = kBM * HD * 2;
  static constexpr int STR = BN * HD * 2;
  static constexpr int VEC = BN * 4;
  static constexpr int SLOT = round_up_1024(2 * STR + 2 * VEC);  // Q | dO | L, D
  static constexpr int OPS = kBM * BN * 2;
  static constexpr int SMEM = 1024 + 2 * RES + ST * SLOT + 2 * OPS;
  static constexpr int C_S = 0, C_DP = BN, C_DK = 2 * BN, C_DV = 2 * BN + HD;
  static constexpr int TMEM_COLS = C_DV + HD <= 256 ? 256 : 512;
  static_assert(C_DV + HD <= TMEM_COLS, "TMEM budget");
};

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
                    const BwdArgs a) {
  using G = DkvPass<HD>;
  constexpr int BN = G::BN, ST = G::ST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* s_k = sm;
  uint8_t* s_v = s_k + G::RES;
  uint8_t* s_ring = s_v + G::RES;
  uint8_t* s_ops = s_ring + ST * G::SLOT;  // P^T | dS^T
  __shared__ uint64_t bar_res, bar_full[ST], bar_empty[ST];
  __shared__ uint64_t bar_sc_full, bar_sc_empty, bar_ops_full, bar_ops_empty, bar_acc;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const AttnShape& sh = a.sh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hk = blockIdx.x, b = blockIdx.y;  // key/value head
  const int kt = blockIdx.z;
  const int k0 = kt * kBM;
  const int nq_tiles = (sh.Tq + BN - 1) / BN;
  const int qt_begin = sh.causal ? k0 / BN : 0;
  const int n = nq_tiles > qt_begin ? nq_tiles - qt_begin : 0;  // query tiles per query head
  // Streamed tile `it` is query tile qt_begin + it % n of query head hk*G + it / n:
  // the G query heads sharing this key head accumulate into the same dK, dV.
  const int total = n * sh.G;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar_res, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    mbar_init(&bar_sc_full, 1);
    mbar_init(&bar_sc_empty, kEwThreads);
    mbar_init(&bar_ops_full, kEwThreads);
    mbar_init(&bar_ops_empty, 1);
    mbar_init(&bar_acc, 1);
    mbar_fence_init();
  }
  if (warp == kWarpMma) tmem_alloc(&tmem_base, G::TMEM_COLS);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == kWarpProducer) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_q);
      mbar_arrive_expect_tx(&bar_res, 2 * G::RES);
      tma_rows<HD>(s_k, &tm_k, &bar_res, k0, kBM, hk, b);
      tma_rows<HD>(s_v, &tm_v, &bar_res, k0, kBM, hk, b);
    }
    int issued = 0;
    for (int it = 0; it < total; ++it) {
      const int s = it % ST;
      const int q0 = (qt_begin + it % n) * BN;
      const int h = hk * sh.G + it / n;
      float st[2][2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int q = q0 + lane + 32 * k;
        const bool v = q < sh.Tq;
        const size_t idx = stat_index(b, h, v ? q : 0, sh.H, sh.Tq);
        st[k][0] = v ? a.lse[idx] : 0.f;
        st[k][1] = v ? a.delta[idx] : 0.f;
      }
      bool ok = true;
      if (it >= ST) ok = mbar_wait(&bar_empty[s], ((it / ST) - 1) & 1, &abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        if (lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutSlotEmpty);
        break;
      }
      uint8_t* slot = s_ring + s * G::SLOT;
      float* sv = reinterpret_cast<float*>(slot + 2 * G::STR);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        sv[lane + 32 * k] = st[k][0];
        sv[BN + lane + 32 * k] = st[k][1];
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_expect_tx(&bar_full[s], 2 * G::STR);
        tma_rows<HD>(slot, &tm_q, &bar_full[s], q0, BN, h, b);
        tma_rows<HD>(slot + G::STR, &tm_do, &bar_full[s], q0, BN, h, b);
      }
      __syncwarp();
      issued = it + 1;
    }
    if (lane == 0) {
      bool drained = mbar_wait(&bar_res, 0, nullptr);
      for (int it = issued > ST ? issued - ST : 0; it < issued; ++it)
        drained &= mbar_wait(&bar_full[it % ST], (it / ST) & 1, nullptr);
      if (!drained) raise_error(a.status, &abort_flag, kDevTimeoutDrain);
    }
  } else if (warp == kWarpMma) {
    if (lane == 0 && n > 0) {
      const uint32_t id_sc = idesc_bf16_f32(kBM, BN, false, false);
      const uint32_t id_out = idesc_bf16_f32(kBM, HD, false, true);
      bool ok = mbar_wait(&bar_res, 0, &abort_flag);
      if (!ok) raise_error(a.status, &abort_flag, kDevTimeoutTmaFull);
      for (int it = 0; ok && it <= total; ++it) {
        if (it < total) {
          const int s = it % ST;
          if (!mbar_wait(&bar_full[s], (it / ST) & 1, &abort_flag) ||
              (it > 0 && !mbar_wait(&bar_sc_empty, (it - 1) & 1, &abort_flag))) {
            raise_error(a.status, &abort_flag, kDevTimeoutTmaFull);
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* slot = s_ring + s * G::SLOT;
          gemm_abt(tmem + G::C_S, s_k, slot, BN, HD / 16, id_sc, false);             // S^T  = K Q^T
          gemm_abt(tmem + G::C_DP, s_v, slot + G::STR, BN, HD / 16, id_sc, false);   // dP^T = V dO^T
          umma_commit(&bar_sc_full);
        }
        const int t = it - 1;
        if (t >= 0) {
          if (!mbar_wait(&bar_ops_full, t & 1, &abort_flag)) {
            raise_error(a.status, &abort_flag, kDevTimeoutEpilogue);
            ok = false;
            break;
          }
          tc_fence_after();
          const int sp = t % ST;
          const uint8_t* slot = s_ring + sp * G::SLOT;
          gemm_ab(tmem + G::C_DV, s_ops, slot + G::STR, BN, BN / 16, id_out, t > 0);   // dV += P^T dO
          gemm_ab(tmem + G::C_DK, s_ops + G::OPS, slot, BN, BN / 16, id_out, t > 0);   // dK += dS^T Q
          umma_commit(&bar_ops_empty);
          umma_commit(&bar_empty[sp]);
        }
      }
      if (ok) umma_commit(&bar_acc);
    }
  } else {
    const int r = threadIdx.x;
    const int key = k0 + r;
    const bool key_ok = key < sh.Tk;
    const float sc = sh.scale, sc2 = sh.scale * kLog2e;
    bool ok = true;
    for (int it = 0; it < total; ++it) {
      const int s = it % ST;
      const int q0 = (qt_begin + it % n) * BN;
      ok = __all_sync(0xffffffffu, mbar_wait(&bar_sc_full, it & 1, &abort_flag));
      if (ok && it > 0) ok = __all_sync(0xffffffffu, mbar_wait(&bar_ops_empty, (it - 1) & 1, &abort_flag));
      if (!ok) break;
      tc_fence_after();
      const float* sv = reinterpret_cast<const float*>(s_ring + s * G::SLOT + 2 * G::STR);
      const bool need_mask = (q0 + BN > sh.Tq) || (sh.causal && q0 < k0 + kBM - 1);
#pragma unroll 1
      for (int c = 0; c < BN / 16; ++c) {
        uint32_t vs[16], vdp[16];
        tmem_row16(tmem, warp, G::C_S + c * 16, vs);
        tmem_row16(tmem, warp, G::C_DP + c * 16, vdp);
        tmem_wait_ld();
        reg_fence16(vs);
        reg_fence16(vdp);
        float o_p[16], o_ds[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int col = c * 16 + i;
          const int q = q0 + col;
          float s = fmaf(__uint_as_float(vs[i]), sc2, -sv[col] * kLog2e);
          if (need_mask && (q >= sh.Tq || (sh.causal && q < key))) s = -INFINITY;
          const float p = ex2(s);
          o_p[i] = p;
          o_ds[i] = p * sc * (__uint_as_float(vdp[i]) - sv[BN + col]);
        }
        stage_bf16x16(s_ops, r, c, o_p);
        stage_bf16x16(s_ops + G::OPS, r, c, o_ds);
      }
      tc_fence_before();
      mbar_arrive(&bar_sc_empty);
      fence_async_smem();
      mbar_arrive(&bar_ops_full);
    }
    const int skey = key_ok ? key : 0;
    __nv_bfloat16* dk_row = a.dk + row_offset(sh.sk, b, skey, hk);
    __nv_bfloat16* dv_row = a.dv + row_offset(sh.sk, b, skey, hk);
    if (n == 0) {
      if (key_ok) {
        zero_row_global<HD>(dk_row);
        zero_row_global<HD>(dv_row);
      }
    } else {
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bar_acc, 0, &abort_flag));
      if (ok) {
        tc_fence_after();
        tmem_row_to_global<HD>(tmem, warp, G::C_DK, dk_row, key_ok);
        tmem_row_to_global<HD>(tmem, warp, G::C_DV, dv_row, key_ok);
      } else if (threadIdx.x == 0) {
        raise_error(a.status, &abort_flag, kDevTimeoutMma);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) tmem_dealloc(tmem, G::TMEM_COLS);
}

template <int HD>
int launch_bwd_hd(const AttnShape& s, const BwdPtrs& p, int* status, cudaStream_t stream) {
  using GQ = DqPass<HD>;
  using GK = DkvPass<HD>;
  CUtensorMap mq[4], mk[4];
  bool ok = make_seq_map(&mq[0], p.q, HD, s.Tq, s.H, s.B, s.sq, kBM) &&
            make_seq_map(&mq[1], p.dO, HD, s.Tq, s.H, s.B, s.sq, kBM) &&
            make_seq_map(&mq[2], p.k, HD, s.Tk, s.Hk, s.B, s.sk, GQ::BN) &&
            make_seq_map(&mq[3], p.v, HD, s.Tk, s.Hk, s.B, s.sk, GQ::BN) &&
            make_seq_map(&mk[0], p.k, HD, s.Tk, s.Hk, s.B, s.sk, kBM) &&
            make_seq_map(&mk[1], p.v, HD, s.Tk, s.Hk, s.B, s.sk, kBM) &&
            make_seq_map(&mk[2], p.q, HD, s.Tq, s.H, s.B, s.sq, GK::BN) &&
            make_seq_map(&mk[3], p.dO, HD, s.Tq, s.H, s.B, s.sq, GK::BN);
  if (!ok) return kInvalidArgument;
  if (ensure_smem_limit(reinterpret_cast<const void*>(&bwd_dq_kernel<HD>), GQ::SMEM) != kOk ||
      ensure_smem_limit(reinterpret_cast<const void*>(&bwd_dkdv_kernel<HD>), GK::SMEM) != kOk)
    return kLaunchFailed;
  int rc = launch_rowdot(s, HD, p.o, p.dO, p.delta, stream);
  if (rc != kOk) return rc;
  BwdArgs args{s, p.lse, p.delta, static_cast<__nv_bfloat16*>(p.dq), static_cast<__nv_bfloat16*>(p.dk),
               static_cast<__nv_bfloat16*>(p.dv), status};
  bwd_dq_kernel<HD><<<dim3(s.H, s.B, (s.Tq + kBM - 1) / kBM), kThreads, GQ::SMEM, stream>>>(mq[0], mq[1], mq[2],
                                                                                          mq[3], args);
  if (after_launch() != kOk) return kLaunchFailed;
  bwd_dkdv_kernel<HD><<<dim3(s.Hk, s.B, (s.Tk + kBM - 1) / kBM), kThreads, GK::SMEM, stream>>>(mk[0], mk[1], mk[2],
                                                                                            mk[3], args);
  return after_launch();
}

}  // namespace

int launch_bwd(const AttnShape& s, int hd, const BwdPtrs& p, int* status, cudaStream_t stream) {
  if (hd == 64) return launch_bwd_hd<64>(s, p, status, stream);
  if (hd == 128) return launch_bwd_hd<128>(s, p, status, stream);
  return kUnsupported;
}

}  // namespace fh
