// Attention forward on sm_100a: O = softmax(scale Q K^T + mask) V and the
// natural-log log-sum-exp L, the residuals the reference's forward rule saves
// (flash_hog/jax/_attention_impl.py:224-239 -- there produced by cuDNN).
//
// One CTA per 128 query rows of one (batch, head). Key/value tiles of 128 rows
// stream through a TMA ring. S = Q K^T is double-buffered in TMEM so the tensor
// core scores tile j+1 while the elementwise warps run the online softmax of
// tile j. Each tile's P V product lands in its own TMEM buffer and is folded
// into a register accumulator with the running rescale factor, so the
// accumulator is never read-modify-written in TMEM.

#include <cuda_runtime.h>

#include <cmath>

#include "kernels.h"

namespace fh {
namespace {

struct FwdArgs {
  AttnShape sh;
  __nv_bfloat16* o;
  float* lse;
  int* status;
};

template <int HD>
struct FPass {
  static constexpr int BN = 128;
  static constexpr int ST = HD == 128 ? 2 : 3;  // K|V slots: 64 KB each at head_dim 128
  static constexpr int RES = kBM * HD * 2;
  static constexpr int STR = BN * HD * 2;
  static constexpr int SLOT = 2 * STR;       // K | V
  static constexpr int OPS = kBM * BN * 2;   // P (two 64-column panels)
  static constexpr int SMEM = 1024 + RES + ST * SLOT + OPS;
  static constexpr int C_S0 = 0, C_S1 = BN, C_O0 = 2 * BN, C_O1 = 2 * BN + HD;
  static constexpr int TMEM_COLS = 512;
  static_assert(C_O1 + HD <= TMEM_COLS, "TMEM budget");
  static_assert(SMEM <= 232448, "shared memory budget");
};

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const FwdArgs a) {
  using G = FPass<HD>;
  constexpr int BN = G::BN, ST = G::ST;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* s_q = sm;
  uint8_t* s_ring = s_q + G::RES;
  uint8_t* s_p = s_ring + ST * G::SLOT;
  __shared__ uint64_t bar_res, bar_full[ST], bar_empty[ST];
  __shared__ uint64_t bar_s_full[2], bar_s_free[2], bar_o_full[2], bar_o_free[2], bar_p_full, bar_p_empty;
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
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar_s_full[i], 1);
      mbar_init(&bar_s_free[i], kEwThreads);
      mbar_init(&bar_o_full[i], 1);
      mbar_init(&bar_o_free[i], kEwThreads);
    }
    mbar_init(&bar_p_full, kEwThreads);
    mbar_init(&bar_p_empty, 1);
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
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(&bar_res, G::RES);
      tma_rows<HD>(s_q, &tm_q, &bar_res, q0, kBM, h, b);
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
      const uint32_t id_s = idesc_bf16_f32(kBM, BN, false, false);
      const uint32_t id_o = idesc_bf16_f32(kBM, HD, false, true);
      bool ok = mbar_wait(&bar_res, 0, &abort_flag);
      if (!ok) raise_error(a.status, &abort_flag, kDevTimeoutTmaFull);
      for (int it = 0; ok && it <= n; ++it) {
        if (it < n) {
          const int s = it % ST;
          if (!mbar_wait(&bar_full[s], (it / ST) & 1, &abort_flag) ||
              (it >= 2 && !mbar_wait(&bar_s_free[it & 1], ((it >> 1) - 1) & 1, &abort_flag))) {
            raise_error(a.status, &abort_flag, kDevTimeoutTmaFull);
            ok = false;
            break;
          }
          tc_fence_after();
          gemm_abt(tmem + ((it & 1) ? G::C_S1 : G::C_S0), s_q, s_ring + s * G::SLOT, BN, HD / 16, id_s, false);
          umma_commit(&bar_s_full[it & 1]);
        }
        const int t = it - 1;  // tile whose P is due
        if (t >= 0) {
          if (!mbar_wait(&bar_p_full, t & 1, &abort_flag) ||
              (t >= 2 && !mbar_wait(&bar_o_free[t & 1], ((t >> 1) - 1) & 1, &abort_flag))) {
            raise_error(a.status, &abort_flag, kDevTimeoutEpilogue);
            ok = false;
            break;
          }
          tc_fence_after();
          const int sp = t % ST;
          gemm_ab(tmem + ((t & 1) ? G::C_O1 : G::C_O0), s_p, s_ring + sp * G::SLOT + G::STR, BN, BN / 16, id_o,
                  false);  // O_t = P_t V_t
          umma_commit(&bar_o_full[t & 1]);
          umma_commit(&bar_p_empty);
          umma_commit(&bar_empty[sp]);
        }
      }
    }
  } else {
    const int r = threadIdx.x;
    const int row = q0 + r;
    const bool row_ok = row < sh.Tq;
    const float sc2 = sh.scale * kLog2e;
    float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
    float acc[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) acc[i] = 0.f;
    bool ok = true;

    // Folds O_t (TMEM buffer t&1) into the register accumulator: acc = acc * alpha + O_t.
    auto fold = [&](int t, float alpha) -> bool {
      if (!__all_sync(0xffffffffu, mbar_wait(&bar_o_full[t & 1], (t >> 1) & 1, &abort_flag))) return false;
      tc_fence_after();
      const int col = (t & 1) ? G::C_O1 : G::C_O0;
#pragma unroll
      for (int c = 0; c < HD; c += 16) {
        uint32_t v[16];
        tmem_row16(tmem, warp, col + c, v);
        tmem_wait_ld();
        reg_fence16(v);
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[c + i] = fmaf(acc[c + i], alpha, __uint_as_float(v[i]));
      }
      tc_fence_before();
      mbar_arrive(&bar_o_free[t & 1]);
      return true;
    };

    for (int it = 0; it < n; ++it) {
      const int k0 = it * BN;
      if (!__all_sync(0xffffffffu, mbar_wait(&bar_s_full[it & 1], (it >> 1) & 1, &abort_flag))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int cs = (it & 1) ? G::C_S1 : G::C_S0;
      const bool need_mask = (k0 + BN > sh.Tk) || (sh.causal && k0 + BN - 1 > q0);
      // pass 1: row maximum of this tile (log2 domain)
      float tmax = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t v[16];
        tmem_row16(tmem, warp, cs + c, v);
        tmem_wait_ld();
        reg_fence16(v);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int key = k0 + c + i;
          float s = __uint_as_float(v[i]) * sc2;
          if (need_mask && (key >= sh.Tk || (sh.causal && key > row))) s = -INFINITY;
          tmax = fmaxf(tmax, s);
        }
      }
      const float m_new = fmaxf(m, tmax);
      const float base = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = ex2(m - base);
      // P of the previous tile must be consumed before this tile's P is written.
      if (it > 0 && !__all_sync(0xffffffffu, mbar_wait(&bar_p_empty, (it - 1) & 1, &abort_flag))) {
        ok = false;
        break;
      }
      // pass 2: P = exp2(s - m_new), row sum, bf16 operand panels
      float psum = 0.f;
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t v[16];
        tmem_row16(tmem, warp, cs + c, v);
        tmem_wait_ld();
        reg_fence16(v);
        float p[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int key = k0 + c + i;
          float s = __uint_as_float(v[i]) * sc2;
          if (need_mask && (key >= sh.Tk || (sh.causal && key > row))) s = -INFINITY;
          p[i] = ex2(s - base);
          psum += p[i];
        }
        stage_bf16x16(s_p + (c / 64) * (kBM * 128), r, (c % 64) / 16, p);
      }
      tc_fence_before();
      mbar_arrive(&bar_s_free[it & 1]);
      fence_async_smem();
      mbar_arrive(&bar_p_full);
      l = l * alpha + psum;
      m = m_new;
      if (it > 0 && !fold(it - 1, alpha_prev)) {
        ok = false;
        break;
      }
      alpha_prev = alpha;
    }
    if (ok) ok = fold(n - 1, alpha_prev);
    if (ok) {
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      if (row_ok) {
        __nv_bfloat16* dst = a.o + row_offset(sh.sq, b, row, h);
#pragma unroll
        for (int c = 0; c < HD; c += 16) {
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = acc[c + i] * inv;
          store_bf16x16(dst + c, v);
        }
        a.lse[stat_index(b, h, row, sh.H, sh.Tq)] = (m + log2f(l)) * kLn2;
      }
    } else if (threadIdx.x == 0) {
      raise_error(a.status, &abort_flag, kDevTimeoutMma);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kWarpMma) tmem_dealloc(tmem, G::TMEM_COLS);
}

template <int HD>
int launch_fwd_hd(const AttnShape& s, const FwdPtrs& p, int* status, cudaStream_t stream) {
  using G = FPass<HD>;
  CUtensorMap mq, mk, mv;
  if (!make_seq_map(&mq, p.q, HD, s.Tq, s.H, s.B, s.sq, kBM) ||
      !make_seq_map(&mk, p.k, HD, s.Tk, s.Hk, s.B, s.sk, G::BN) ||
      !make_seq_map(&mv, p.v, HD, s.Tk, s.Hk, s.B, s.sk, G::BN))
    return kInvalidArgument;
  if (ensure_smem_limit(reinterpret_cast<const void*>(&fwd_kernel<HD>), G::SMEM) != kOk) return kLaunchFailed;
  FwdArgs args{s, static_cast<__nv_bfloat16*>(p.o), p.lse, status};
  const dim3 grid(s.H, s.B, (s.Tq + kBM - 1) / kBM);
  fwd_kernel<HD><<<grid, kThreads, G::SMEM, stream>>>(mq, mk, mv, args);
  return after_launch();
}

}  // namespace

int launch_fwd(const AttnShape& s, int hd, const FwdPtrs& p, int* status, cudaStream_t stream) {
  if (hd == 64) return launch_fwd_hd<64>(s, p, status, stream);
  if (hd == 128) return launch_fwd_hd<128>(s, p, status, stream);
  return kUnsupported;
}

}  // namespace fh
