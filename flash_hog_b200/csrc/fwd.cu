// Attention forward on sm_100a: O = softmax(scale Q K^T + mask) V and the
// natural-log log-sum-exp L, the residuals the reference's forward rule saves
// (flash_hog/jax/_attention_impl.py:224-239 -- there produced by cuDNN).
//
// A CTA owns T 128-row query tiles of one (batch, head) -- T = 1 at head_dim
// 64 (two CTAs per SM), T = 2 at 128 -- that share every streamed 128-row K|V
// tile of a TMA ring. Warp 0 allocates TMEM and issues every MMA
// (warp-convergent, one elected lane), warp 1 is the TMA producer, and each
// query tile has a softmax warpgroup (warps 2-5, then 6-9): thread (warp, lane)
// owns TMEM lane 32*(warp%4)+lane, one query row.
//
// TMEM per tile: a score buffer S (128 columns) and the output accumulator O,
// and at head_dim 64 a separate bf16 buffer for P (64 columns). The softmax
// warps turn S(j) into P(j); O += P(j) V_j reads P from TMEM (A operand) and V
// from shared memory.
//  * head_dim 64: the softmax warps release S as soon as they have loaded it, so
//    S(j+1) is computed while they exponentiate tile j; P(j) goes to its own
//    buffer once the previous product has read it. S, P and O take 256 TMEM
//    columns, so two CTAs share an SM and hide each other's waits.
//  * head_dim 128 (TMEM holds no extra P buffers): P(j) is written back over the
//    first half of S(j), and S(j+1) is issued right behind O += P(j) V_j into the
//    same buffer (the tensor core runs in issue order). The two tiles of a CTA
//    share the exponential units; each warpgroup computes while the other waits.
// At both head dims a quarter of the exponentials go to a polynomial on the FMA
// pipe, which shortens the softmax step that lies on each tile's critical path.
// K and V of a ring slot land and are released on their own barriers: a slot's K is
// free once the score products of its key tile are done, so the next K load starts
// about one key tile earlier than it could if K and V were released together.
// Online softmax with lazy rescaling: P = exp2(s - m) against a running maximum
// m that is only raised -- and O, l rescaled in TMEM -- when a row's maximum
// grows by more than 2^8, so P stays below 2^8 and most tiles need no rescale.

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
  int grp;  // (query head, batch) pairs per locality group (grouped_order)
};


constexpr int kFwdWarpMma = 0;
constexpr int kFwdWarpProducer = 1;
constexpr int kFwdFirstEwWarp = 2;
constexpr int kFwdEwWarps = 4;       // per query tile
constexpr float kRescaleLog2 = 8.f;  // P < 2^8 between rescales

template <int HD>
struct FPass {
  // Query tiles per CTA: one at head_dim 64, where S, a separate P buffer and O
  // take 256 TMEM columns and two CTAs share an SM; two at 128 (one CTA per SM).
  static constexpr int T = HD == 64 ? 1 : 2;
  static constexpr int CTAS = T == 1 ? 2 : 1;
  static constexpr int THREADS = 64 + 128 * T;
  static constexpr int ROWS = kBM * T;           // query rows per CTA
  static constexpr int BN = 128;                 // key rows per streamed tile
  static constexpr int ST = 2;                   // K|V slots: 32 KB at head_dim 64, 64 KB at 128
  static constexpr int RES = kBM * HD * 2;       // one 128-row query tile
  static constexpr int STR = BN * HD * 2;
  static constexpr int SLOT = 2 * STR;  // K | V
  static constexpr int SMEM = 1024 + T * RES + ST * SLOT;
  // TMEM: S of tile t at t*BN; with separate P buffers (head_dim 64), P of tile
  // t at 2*BN + t*BN/2; O of tile t at C_O + t*HD.
  static constexpr bool SEP_P = HD == 64;
  static constexpr int C_P = T * BN;
  static constexpr int C_O = SEP_P ? T * BN + T * BN / 2 : T * BN;
  static constexpr int TMEM_COLS = CTAS == 2 ? 256 : 512;
  static_assert(C_O + T * HD <= TMEM_COLS, "TMEM budget");
  static_assert(CTAS * SMEM <= 228 * 1024 - CTAS * 2048, "shared memory of the resident CTAs");
  static_assert(SMEM <= 232448, "shared memory budget");
  // The issuer waits for K of key tile j+1 (S(j+1)) before it releases tile j's V:
  // with one slot that wait could never end.
  static_assert(ST >= 2, "the ring must hold the next key tile while the current one is in use");
};

// 2^x for a pair of floats on the FMA and integer pipes instead of the MUFU unit:
// x = j + f with j = round(x) (adding 1.5 * 2^23 rounds to an integer) and f in
// [-0.5, 0.5]; 2^f by a degree-3 polynomial whose coefficients were fitted for this
// library by a Lawson (iteratively reweighted least-squares) minimax iteration on the
// relative error over [-0.5, 0.5] (max 7.5e-5, far below the bf16 rounding of P); j
// is added to the result's exponent field. x < -126, including a masked -inf, gives 0.
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
  const float2 big = make_float2(12582912.f, 12582912.f);
  const float2 t = __fadd2_rn(x, big);
  const float2 j = __fadd2_rn(t, make_float2(-12582912.f, -12582912.f));
  const float2 f = __ffma2_rn(j, make_float2(-1.f, -1.f), x);
  float2 p = __ffma2_rn(f, make_float2(0.055171342699099686f, 0.055171342699099686f),
                        make_float2(0.24261034141576007f, 0.24261034141576007f));
  p = __ffma2_rn(p, f, make_float2(0.6932609672206897f, 0.6932609672206897f));
  p = __ffma2_rn(p, f, make_float2(0.9999281213111199f, 0.9999281213111199f));
  float2 r;
  r.x = __int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23));
  r.y = __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23));
  r.x = x.x < -126.f ? 0.f : r.x;
  r.y = x.y < -126.f ? 0.f : r.y;
  return r;
}

// All lanes of the warp have finished their TMEM accesses; one lane arrives.
__device__ __forceinline__ void fwd_warp_arrive(uint64_t* bar) {
  tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

template <int HD, bool VL, bool GRP>
__global__ void __launch_bounds__(FPass<HD>::THREADS, FPass<HD>::CTAS)
    fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const FwdArgs a) {
  using G = FPass<HD>;
  constexpr int BN = G::BN, ST = G::ST, T = G::T;
  constexpr bool SEP_P = G::SEP_P;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* s_q = sm;  // tile A, then tile B
  uint8_t* s_ring = s_q + T * G::RES;
  // Per query tile t: scores ready, scores loaded (separate P only), P written,
  // P read by its product (separate P only), last O update done.
  // K and V of a ring slot land and are released separately: a slot's K is free once
  // the score products of its key tile are done, long before its V has been used.
  __shared__ uint64_t bar_q, bar_kfull[ST], bar_vfull[ST], bar_kempty[ST], bar_vempty[ST], bar_s_full[2],
      bar_s_empty[2], bar_p_full[2], bar_p_free[2], bar_o_done[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Grid (H, B, query tiles), longest causal rows first; GRP: a 1-D grid in the
  // locality-grouped order.
  int h = blockIdx.x, b = blockIdx.y, qt = gridDim.z - 1 - blockIdx.z;
  if constexpr (GRP) {
    const int nq = (a.sh.Tq + G::ROWS - 1) / G::ROWS;
    int qi, hb;
    grouped_order(blockIdx.x, nq, a.sh.H * a.sh.B, a.grp, &qi, &hb);
    h = hb % a.sh.H, b = hb / a.sh.H, qt = nq - 1 - qi;
  }
  SeqRange sr;
  const AttnShape sh = seq_shape<VL>(a.sh, b, &sr);  // this sequence's lengths and mask; sr: where its rows start
  const int q0 = qt * G::ROWS;
  // Key tiles of each query tile: nt[t] tiles from key tile jt[t] (0 when the
  // tile lies past the last query row or sees no key). The ring streams the
  // union [jlo, jlo + n); tile t joins at ring position at[t].
  int nt[2] = {0, 0}, jt[2] = {0, 0}, at[2] = {0, 0};
#pragma unroll
  for (int t = 0; t < T; ++t) nt[t] = key_tiles(sh, q0 + t * kBM, kBM, BN, &jt[t]);
  const int jlo = nt[0] > 0 ? (nt[1] > 0 ? min(jt[0], jt[1]) : jt[0]) : jt[1];
  int jhi = jlo;
#pragma unroll
  for (int t = 0; t < T; ++t) {
    if (nt[t] > 0) jhi = max(jhi, jt[t] + nt[t]);
    at[t] = jt[t] - jlo;
  }
  const int n = jhi - jlo;  // key tiles streamed (0 if no row sees a key)

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bar_q, 1);
    for (int s = 0; s < ST; ++s) {
      mbar_init(&bar_kfull[s], 1);
      mbar_init(&bar_vfull[s], 1);
      mbar_init(&bar_kempty[s], 1);
      mbar_init(&bar_vempty[s], 1);
    }
    for (int t = 0; t < T; ++t) {
      mbar_init(&bar_s_full[t], 1);
      mbar_init(&bar_s_empty[t], kFwdEwWarps);
      mbar_init(&bar_p_full[t], kFwdEwWarps);
      mbar_init(&bar_p_free[t], 1);
      mbar_init(&bar_o_done[t], 1);
    }
    mbar_fence_init();
  }
  if (warp == kFwdWarpMma) tmem_alloc(&tmem_base, G::TMEM_COLS);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (warp == kFwdWarpProducer) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(&bar_q, T * G::RES);
      for (int t = 0; t < T; ++t) tma_rows<HD>(s_q + t * G::RES, &tm_q, &bar_q, sr.q0 + q0 + t * kBM, kBM, h, sr.bc);
      int k_issued = 0, v_issued = 0;
      for (int j = 0; j < n; ++j) {
        const int s = j % ST;
        const uint32_t ph = ((j / ST) - 1) & 1;
        uint8_t* slot = s_ring + s * G::SLOT;
        if (j >= ST && !mbar_wait(&bar_kempty[s], ph, &abort_flag)) {
          raise_error(a.status, &abort_flag, kDevTimeoutSlotEmpty);
          break;
        }
        mbar_arrive_expect_tx(&bar_kfull[s], G::STR);
        tma_rows<HD>(slot, &tm_k, &bar_kfull[s], sr.k0 + (jlo + j) * BN, BN, h / sh.G, sr.bc);
        k_issued = j + 1;
        if (j >= ST && !mbar_wait(&bar_vempty[s], ph, &abort_flag)) {
          raise_error(a.status, &abort_flag, kDevTimeoutSlotEmpty);
          break;
        }
        mbar_arrive_expect_tx(&bar_vfull[s], G::STR);
        tma_rows<HD>(slot + G::STR, &tm_v, &bar_vfull[s], sr.k0 + (jlo + j) * BN, BN, h / sh.G, sr.bc);
        v_issued = j + 1;
      }
      // Every issued copy must land before this CTA's shared memory is released.
      bool drained = mbar_wait(&bar_q, 0, nullptr);
      for (int j = k_issued > ST ? k_issued - ST : 0; j < k_issued; ++j)
        drained &= mbar_wait(&bar_kfull[j % ST], (j / ST) & 1, nullptr);
      for (int j = v_issued > ST ? v_issued - ST : 0; j < v_issued; ++j)
        drained &= mbar_wait(&bar_vfull[j % ST], (j / ST) & 1, nullptr);
      if (!drained) raise_error(a.status, &abort_flag, kDevTimeoutDrain);
    }
  } else if (warp == kFwdWarpMma) {
    // -------------------------------- MMA issuer --------------------------------
    // Per key tile j and query tile t: O_t += P_t(j) V_j, then S_t(j+1) = Q_t K_{j+1}^T
    // into the same TMEM columns (issue order keeps the product's reads first).
    constexpr int KS = HD / 16, KO = BN / 16;
    const uint32_t id_s = idesc_bf16_f32(kBM, BN, false, false);
    const uint32_t id_o = idesc_bf16_f32(kBM, HD, false, true);
    const uint64_t a_q = kdesc(s_q);
    constexpr uint64_t kRes = G::RES >> 4;
    const uint64_t b_k = kdesc(s_ring);                      // K of slot 0, K-major
    const uint64_t b_v = mndesc(s_ring + G::STR, BN * 128);  // V of slot 0, MN-major
    constexpr uint64_t kSlot = G::SLOT >> 4;
    auto issue_s = [&](int t, int j) -> bool {
      const int s = j % ST;
      if (!mbar_wait_warp(&bar_kfull[s], (j / ST) & 1, &abort_flag)) return false;
      tc_fence_after();
      umma_chain_w<KS, kBM * 128, BN * 128, false>(tmem + t * BN, a_q + t * kRes, b_k + s * kSlot, id_s, false);
      umma_commit_w(&bar_s_full[t]);
      return true;
    };
    // Ring position j holds key tile jlo + j; tile t's own step is u = j - at[t].
    // Every score product of ring position j is issued before iteration j (position 0
    // before the loop), so K of position j + 1 is released at the end of iteration j;
    // V of position j once iteration j's products are done.
    auto wait_v = [&](int j) -> bool {
      if (!mbar_wait_warp(&bar_vfull[j % ST], (j / ST) & 1, &abort_flag)) return false;
      tc_fence_after();
      return true;
    };
    bool ok = mbar_wait_warp(&bar_q, 0, &abort_flag);
    for (int t = 0; ok && t < T; ++t)
      if (nt[t] > 0 && at[t] == 0) ok = issue_s(t, 0);
    if (ok && n > 0) umma_commit_w(&bar_kempty[0]);
    for (int j = 0; ok && SEP_P && j < n; ++j) {
      // Separate P: S(u+1) as soon as S(u) has been loaded, then the products.
#pragma unroll
      for (int t = 0; ok && t < T; ++t) {
        const int u = j - at[t];
        if (u + 1 < 0 || u + 1 >= nt[t]) continue;
        if (u >= 0) ok = mbar_wait_warp(&bar_s_empty[t], u & 1, &abort_flag);
        ok = ok && issue_s(t, j + 1);
      }
      if (ok && j + 1 < n) umma_commit_w(&bar_kempty[(j + 1) % ST]);
      ok = ok && wait_v(j);
#pragma unroll
      for (int t = 0; ok && t < T; ++t) {
        const int u = j - at[t];
        if (u < 0 || u >= nt[t]) continue;
        if (!mbar_wait_warp(&bar_p_full[t], u & 1, &abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        umma_chain_ts_w<KO>(tmem + G::C_O + t * HD, tmem + G::C_P + t * (BN / 2), b_v + (j % ST) * kSlot, id_o,
                            u > 0);
        umma_commit_w(&bar_p_free[t]);
        if (u + 1 == nt[t]) umma_commit_w(&bar_o_done[t]);
      }
      if (ok) umma_commit_w(&bar_vempty[j % ST]);
    }
    for (int j = 0; ok && !SEP_P && j < n; ++j) {
      ok = wait_v(j);
#pragma unroll
      for (int t = 0; ok && t < T; ++t) {
        const int u = j - at[t];
        if (u == -1 && nt[t] > 0) {  // the tile's first key tile is the next one
          ok = issue_s(t, j + 1);
          continue;
        }
        if (u < 0 || u >= nt[t]) continue;
        if (!mbar_wait_warp(&bar_p_full[t], u & 1, &abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        umma_chain_ts_w<KO>(tmem + G::C_O + t * HD, tmem + t * BN, b_v + (j % ST) * kSlot, id_o, u > 0);
        if (u + 1 < nt[t]) {
          ok = issue_s(t, j + 1);
        } else {
          umma_commit_w(&bar_o_done[t]);
        }
      }
      if (ok && j + 1 < n) umma_commit_w(&bar_kempty[(j + 1) % ST]);
      if (ok) umma_commit_w(&bar_vempty[j % ST]);
    }
    if (!ok && lane == 0) raise_error(a.status, &abort_flag, kDevTimeoutTmaFull);
  } else {
    // ------------------------------ softmax warpgroups ------------------------------
    const int t = (warp - kFwdFirstEwWarp) >> 2;  // query tile of this warpgroup
    const int r = (warp & 3) * 32 + lane;         // TMEM lane = query row inside the tile
    const int row = q0 + t * kBM + r;
    const bool row_ok = row < sh.Tq;
    int jt0;  // first key tile of this warpgroup's query tile
    const int nj = key_tiles(sh, q0 + t * kBM, kBM, BN, &jt0);
    const int khi = key_hi(sh, row), klo = key_lo(sh, row);  // this row's visible keys
    const float sc2 = sh.scale * kLog2e;
    const uint32_t lane_base = tmem + tmem_lane_base(warp & 3);
    const uint32_t tcol = lane_base + t * BN;
    const uint32_t ocol = lane_base + G::C_O + t * HD;
    float m_used = -INFINITY, l = 0.f;  // running maximum (log2 domain) and the sum against it
    bool ok = true;
    for (int j = 0; j < nj; ++j) {
      const int k0 = (jt0 + j) * BN;
      ok = mbar_wait_warp(&bar_s_full[t], j & 1, &abort_flag);
      if (!ok) break;
      tc_fence_after();
      uint32_t v[BN];
#pragma unroll
      for (int c = 0; c < BN; c += 16) tmem_ld16(tcol + c, *reinterpret_cast<uint32_t(*)[16]>(&v[c]));
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < BN; ++i) asm volatile("" : "+r"(v[i])::"memory");
      if constexpr (G::SEP_P) fwd_warp_arrive(&bar_s_empty[t]);  // S(j+1) may be computed now
      if (k0 + BN - 1 > khi || k0 < klo) {
#pragma unroll
        for (int i = 0; i < BN; ++i)
          if (k0 + i > khi || k0 + i < klo) v[i] = __float_as_uint(-INFINITY);
      }
      // Row maximum of the raw scores (the scale is positive), eight independent chains.
      float mx[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) mx[c] = __uint_as_float(v[c]);
#pragma unroll
      for (int i = 8; i < BN; ++i) mx[i & 7] = fmaxf(mx[i & 7], __uint_as_float(v[i]));
#pragma unroll
      for (int c = 4; c > 0; c >>= 1)
#pragma unroll
        for (int k = 0; k < c; ++k) mx[k] = fmaxf(mx[k], mx[k + c]);
      const float tmax = mx[0] * sc2;  // log2 domain
      const float m_new = fmaxf(m_used, tmax);
      float f = 1.f;  // rescale factor of O and l, applied before this tile's P is added
      if (j == 0) {
        m_used = m_new;
      } else if (m_new > m_used + kRescaleLog2) {
        f = ex2(m_used - m_new);
        m_used = m_new;
      }
      auto rescale_o = [&]() {
#pragma unroll
        for (int c = 0; c < HD; c += 16) {
          uint32_t o[16];
          tmem_ld16(ocol + c, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
          tmem_st16(ocol + c, o);
        }
        tmem_wait_st();
      };
      // P over S: O is stable now -- S(j) was issued after O += P(j-1) V_{j-1}, so
      // its completion (just waited for) implies that update's.
      // The TMEM loads and stores of a rescale are warp-collective: the warp rescales
      // together when any of its rows needs it (the others multiply by f = 1).
      const bool warp_rescale = __any_sync(0xffffffffu, f != 1.f);
      if (!G::SEP_P && warp_rescale) rescale_o();
      const float base = (m_used == -INFINITY) ? 0.f : m_used;
      uint32_t pk[BN / 2];
      // Column pairs through the packed fp32x2 instructions; the row sum in two
      // (even, odd) pair accumulators.
      float2 ps2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      const float2 m2 = make_float2(sc2, sc2), nb2 = make_float2(-base, -base);
#pragma unroll
      for (int i = 0; i < BN; i += 2) {
        const float2 s = __ffma2_rn(make_float2(__uint_as_float(v[i]), __uint_as_float(v[i + 1])), m2, nb2);
        // A quarter of the column pairs take 2^x on the FMA pipe (exp2_fma2).
        const float2 p = ((i >> 1) & 7) < 2 ? exp2_fma2(s) : make_float2(ex2(s.x), ex2(s.y));
        ps2[(i >> 1) & 1] = __fadd2_rn(ps2[(i >> 1) & 1], p);
        pk[i / 2] = pack_bf16(p.x, p.y);
      }
      const float ps[4] = {ps2[0].x, ps2[0].y, ps2[1].x, ps2[1].y};
      uint32_t pcol = tcol;
      if constexpr (G::SEP_P) {
        // The P buffer and O are free once the previous product is done.
        if (j > 0) {
          ok = mbar_wait_warp(&bar_p_free[t], (j - 1) & 1, &abort_flag);
          if (!ok) break;
          tc_fence_after();
          if (warp_rescale) rescale_o();
        }
        pcol = lane_base + G::C_P + t * (BN / 2);
      }
      l = l * f + ((ps[0] + ps[1]) + (ps[2] + ps[3]));
#pragma unroll
      for (int c = 0; c < BN / 2; c += 16) tmem_st16(pcol + c, *reinterpret_cast<const uint32_t(*)[16]>(&pk[c]));
      tmem_wait_st();
      fwd_warp_arrive(&bar_p_full[t]);  // P(j) is in TMEM
    }
    if (ok && nj > 0) ok = mbar_wait_warp(&bar_o_done[t], 0, &abort_flag);
    if (ok && nj > 0) {
      tc_fence_after();
      const float inv = (l > 0.f) ? 1.f / l : 0.f;
      __nv_bfloat16* dst = a.o + q_row(sh, sr, row_ok ? row : 0, h);
#pragma unroll
      for (int c = 0; c < HD; c += 16) {
        uint32_t o[16];
        tmem_ld16(ocol + c, o);
        tmem_wait_ld();
        float x[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) x[i] = __uint_as_float(o[i]) * inv;
        if (row_ok) store_bf16x16(dst + c, x);
      }
      if (row_ok) a.lse[q_stat(sh, sr, row, h)] = (m_used + log2f(l)) * kLn2;
    } else if (ok && row_ok) {
      // No key tile for these rows: O = 0 and L = -inf (no visible key).
      zero_row_global<HD>(a.o + q_row(sh, sr, row, h));
      a.lse[q_stat(sh, sr, row, h)] = -INFINITY;
    } else if (!ok && (threadIdx.x & 127) == 0) {
      raise_error(a.status, &abort_flag, kDevTimeoutMma);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kFwdWarpMma) tmem_dealloc(tmem, G::TMEM_COLS);
}

template <int HD, bool VL>
int launch_fwd_hd(const AttnShape& s, const FwdPtrs& p, int* status, cudaStream_t stream) {
  using G = FPass<HD>;
  CUtensorMap mq, mk, mv;
  if (!make_seq_map(&mq, p.q, HD, s.total_q, s.H, map_batch(s), s.sq, kBM) ||
      !make_seq_map(&mk, p.k, HD, s.total_k, s.Hk, map_batch(s), s.sk, G::BN) ||
      !make_seq_map(&mv, p.v, HD, s.total_k, s.Hk, map_batch(s), s.sk, G::BN))
    return kInvalidArgument;
  if (ensure_smem_limit(reinterpret_cast<const void*>(&fwd_kernel<HD, VL, false>), G::SMEM) != kOk) return kLaunchFailed;
  if constexpr (!VL) {
    if (ensure_smem_limit(reinterpret_cast<const void*>(&fwd_kernel<HD, false, true>), G::SMEM) != kOk)
      return kLaunchFailed;
  }
  // K and V of a key head are the tiles the query tiles of its heads share.
  FwdArgs args{s, static_cast<__nv_bfloat16*>(p.o), p.lse, status,
               locality_group(s.H * s.B, s.H / s.Hk, 2ll * s.Tk * HD * 2)};
  const int nq = (s.Tq + G::ROWS - 1) / G::ROWS;
  if (!VL && args.grp < s.H * s.B)  // grouped only where the groups split the pairs
    fwd_kernel<HD, false, true><<<dim3(s.H * s.B * nq), G::THREADS, G::SMEM, stream>>>(mq, mk, mv, args);
  else
    fwd_kernel<HD, VL, false><<<dim3(s.H, s.B, nq), G::THREADS, G::SMEM, stream>>>(mq, mk, mv, args);
  return after_launch();
}

}  // namespace

int launch_fwd(const AttnShape& s, int hd, const FwdPtrs& p, int* status, cudaStream_t stream) {
  if (hd == 64) return s.cu_q ? launch_fwd_hd<64, true>(s, p, status, stream) : launch_fwd_hd<64, false>(s, p, status, stream);
  if (hd == 128) return s.cu_q ? launch_fwd_hd<128, true>(s, p, status, stream) : launch_fwd_hd<128, false>(s, p, status, stream);
  return kUnsupported;
}

}  // namespace fh
