// fp32 attention: forward, first-order backward and double backward with fp32
// operands, on the CUDA cores.
//
// The tensor-core kernels (fwd.cu, bwd.cu, bwdbwd.cu) take bf16 operands. The
// reference also accepts fp32 inputs and then computes in fp32: its Pallas
// double backward keeps the operand dtype in every product
// (flash_hog/jax/_pallas_gpu_kernel.py:236-256, the casts are to the operand
// dtype) and its XLA reference differentiates fp32 attention twice
// (flash_hog/_jax_refs/jax_impl.py:194-247). Results must then agree with that
// reference to 1e-3, which bf16 (8-bit mantissa) operands cannot meet; tf32
// (10-bit) is not enough either once the double backward chains four products.
// These kernels keep every product in fp32 (fmaf), with the same multi-pass
// schedule, masks, GQA mapping and strided BTNH layout as the bf16 path.
//
// Every kernel has one shape: a CTA of 256 threads owns kRes = 64 "resident"
// rows (queries for the query-side passes, keys for the key-side ones), keeps
// their operands in shared memory, and streams BN-row tiles of the other side.
// Thread (rg, cg) = (tid / 16, tid % 16) owns resident rows 4 rg .. 4 rg + 3;
// of a score tile it owns columns cg + 16 j, of an output tile the 4-column
// chunks cg + 16 m. A row's 16 owners are one half-warp, so row reductions are
// 4 xor-shuffles. Where shared memory allows a second buffer (the forward; both
// double-backward passes at head_dim 64) the next streamed tile is fetched with
// cp.async while the current one is used. No kernel spins: the only waits are
// __syncthreads and cp.async.wait_group on the CTA's own copies.

#include <cuda_runtime.h>

#include <cmath>

#include "kernels.h"

namespace fh {
namespace f32 {

constexpr int kThreads = 256;
constexpr int kRes = 64;  // resident rows per CTA

template <int HD>
struct Geo {
  static_assert(HD == 64 || HD == 128, "head_dim 64 or 128");
  static constexpr int BN = HD == 64 ? 64 : 32;  // streamed rows per tile
  static constexpr int SP = HD + 4;              // padded row stride (floats) of an operand tile
  static constexpr int SC = BN + 4;              // padded row stride of a score tile
  static constexpr int NC = BN / 16;             // score columns per thread
  static constexpr int NO = HD / 16;             // output columns per thread
  static constexpr int RES = kRes * SP;          // floats of a resident operand tile
  static constexpr int STR = BN * SP;            // floats of a streamed operand tile
  static constexpr int SCORE = kRes * SC;        // floats of a score tile
};

__device__ __forceinline__ float sum16(float x) {
#pragma unroll
  for (int o = 8; o; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__device__ __forceinline__ float max16(float x) {
#pragma unroll
  for (int o = 8; o; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

__device__ __forceinline__ bool visible(const AttnShape& s, int i, int j) {
  return i < s.Tq && j < s.Tk && j >= key_lo(s, i) && j <= key_hi(s, i);
}

// rows [row0, row0 + ROWS) of head h of batch b (zeros past `len`) into a
// padded [ROWS][HD + 4] tile. Pointers are 16-byte aligned and strides are
// multiples of 8 elements (checked by the C ABI), so rows load as float4.
template <int HD, int ROWS>
__device__ __forceinline__ void load_rows(float* dst, const float* __restrict__ src, const Strides3& st, int b, int h,
                                          int row0, int len) {
  constexpr int CH = HD / 4;
  const float* base = src + static_cast<long long>(b) * st.b + static_cast<long long>(h) * st.h;
  for (int idx = threadIdx.x; idx < ROWS * CH; idx += kThreads) {
    const int r = idx / CH, c = idx - r * CH;
    const int t = row0 + r;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (t < len) v = __ldg(reinterpret_cast<const float4*>(base + static_cast<long long>(t) * st.t) + c);
    *reinterpret_cast<float4*>(dst + r * (HD + 4) + 4 * c) = v;
  }
}

// load_rows with cp.async (16-byte copies, zero-filled past `len`): the copies
// land in shared memory without passing through registers and complete at the
// next cp_async_wait, so a tile can be fetched while the previous one is used.
template <int HD, int ROWS>
__device__ __forceinline__ void load_rows_async(float* dst, const float* __restrict__ src, const Strides3& st, int b,
                                                int h, int row0, int len) {
  constexpr int CH = HD / 4;
  const float* base = src + static_cast<long long>(b) * st.b + static_cast<long long>(h) * st.h;
  for (int idx = threadIdx.x; idx < ROWS * CH; idx += kThreads) {
    const int r = idx / CH, c = idx - r * CH;
    const int t = row0 + r;
    const bool ok = t < len;
    const float* g = ok ? base + static_cast<long long>(t) * st.t + 4 * c : base;  // no bytes read when !ok
    const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(dst + r * (HD + 4) + 4 * c));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sa), "l"(g), "r"(ok ? 16 : 0) : "memory");
  }
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}

// Waits until at most N of this thread's committed cp.async groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// load_stats with 4-byte cp.async copies (zero past Tq); not committed here: the
// caller's next load_rows_async commits them with its rows.
__device__ __forceinline__ void stats_async(float* dst, const float* __restrict__ src, const AttnShape& s, int b,
                                            int h, int q0, int n) {
  for (int r = threadIdx.x; r < n; r += kThreads) {
    const int t = q0 + r;
    const bool ok = t < s.Tq;
    const float* g = ok ? src + (static_cast<long long>(b) * s.H + h) * s.Tq + t : src;
    const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(dst + r));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(sa), "l"(g), "r"(ok ? 4 : 0) : "memory");
  }
}

// Key-tile buffers of the double backward's query pass: two where shared memory
// allows (head_dim 64: 221 KB per CTA), else one.
template <int HD>
struct QueryPassBuffers {
  using G = Geo<HD>;
  static constexpr int bytes(int n) { return (3 * G::RES + n * 4 * G::STR + 2 * G::SCORE) * 4; }
  static constexpr int N = bytes(2) <= 232448 ? 2 : 1;
};

// Streamed-tile buffers of the double backward's key pass: two where shared memory
// allows (head_dim 64: 223 KB per CTA), else one.
template <int HD>
struct KeyPassBuffers {
  using G = Geo<HD>;
  static constexpr int bytes(int n) { return (4 * G::RES + n * (3 * G::STR + 4 * G::BN) + 3 * G::SCORE) * 4; }
  static constexpr int N = bytes(2) <= 232448 ? 2 : 1;
};

// Per-query statistics of a streamed query tile: dst[r] = src[(b H + h) Tq + q0 + r] (0 past Tq).
__device__ __forceinline__ void load_stats(float* dst, const float* __restrict__ src, const AttnShape& s, int b, int h,
                                           int q0, int n) {
  for (int r = threadIdx.x; r < n; r += kThreads) {
    const int t = q0 + r;
    dst[r] = t < s.Tq ? src[(static_cast<long long>(b) * s.H + h) * s.Tq + t] : 0.f;
  }
}

// acc[i][j] += sum_d A[4 rg + i][d] * B[cg + 16 j][d]  (A: resident tile, B: streamed tile)
// The products run on the packed fp32x2 FMA (one issue slot for two IEEE fmas):
// each dot product keeps (even, odd) head_dim partial sums, added at the end.
template <int HD, int NR, int NC>
__device__ __forceinline__ void score_acc(float (&acc)[4][NC], const float* A, const float* B, int rg, int cg) {
  constexpr int SP = HD + 4;
  const float* a0 = A + rg * 4 * SP;
  const float* b0 = B + cg * SP;
  float2 acc2[4][NC];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < NC; ++j) acc2[i][j] = make_float2(acc[i][j], 0.f);
#pragma unroll 4
  for (int d = 0; d < HD; d += 4) {
    float4 a[4], bb[NC];
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = *reinterpret_cast<const float4*>(a0 + i * SP + d);
#pragma unroll
    for (int j = 0; j < NC; ++j) bb[j] = *reinterpret_cast<const float4*>(b0 + j * 16 * SP + d);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < NC; ++j) {
        acc2[i][j] = __ffma2_rn(make_float2(a[i].x, a[i].y), make_float2(bb[j].x, bb[j].y), acc2[i][j]);
        acc2[i][j] = __ffma2_rn(make_float2(a[i].z, a[i].w), make_float2(bb[j].z, bb[j].w), acc2[i][j]);
      }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < NC; ++j) acc[i][j] = acc2[i][j].x + acc2[i][j].y;
}

template <int C>
__device__ __forceinline__ float lane4(const float4& v) {
  return C == 0 ? v.x : C == 1 ? v.y : C == 2 ? v.z : v.w;
}

// acc columns (4 m, 4 m + 1) and (4 m + 2, 4 m + 3) as fp32x2 pairs: two packed fmas per 4 columns.
template <int C, int M>
__device__ __forceinline__ void out_step(float2 (&acc)[4][2 * M], const float4 (&p)[4], const float* brow, int cg) {
#pragma unroll
  for (int m = 0; m < M; ++m) {
    const float4 b = *reinterpret_cast<const float4*>(brow + (cg + 16 * m) * 4);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float pv = lane4<C>(p[i]);
      acc[i][2 * m] = __ffma2_rn(make_float2(pv, pv), make_float2(b.x, b.y), acc[i][2 * m]);
      acc[i][2 * m + 1] = __ffma2_rn(make_float2(pv, pv), make_float2(b.z, b.w), acc[i][2 * m + 1]);
    }
  }
}

// acc[i][4 m + c] += sum_n P[4 rg + i][n] * B[n][4 (cg + 16 m) + c]  (P: score tile, B: streamed tile)
template <int HD, int BN>
__device__ __forceinline__ void out_acc(float (&acc)[4][HD / 16], const float* P, const float* B, int rg, int cg) {
  constexpr int SP = HD + 4, SC = BN + 4, M = HD / 64;
  const float* p0 = P + rg * 4 * SC;
  float2 acc2[4][2 * M];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 2 * M; ++j) acc2[i][j] = make_float2(acc[i][2 * j], acc[i][2 * j + 1]);
#pragma unroll 2
  for (int n = 0; n < BN; n += 4) {
    float4 p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = *reinterpret_cast<const float4*>(p0 + i * SC + n);
    out_step<0, M>(acc2, p, B + (n + 0) * SP, cg);
    out_step<1, M>(acc2, p, B + (n + 1) * SP, cg);
    out_step<2, M>(acc2, p, B + (n + 2) * SP, cg);
    out_step<3, M>(acc2, p, B + (n + 3) * SP, cg);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 2 * M; ++j) {
      acc[i][2 * j] = acc2[i][j].x;
      acc[i][2 * j + 1] = acc2[i][j].y;
    }
}

// out rows (4 rg + i) of the resident tile = mult * acc (+ add, same layout as out).
template <int HD>
__device__ __forceinline__ void store_rows(float* __restrict__ out, const float* add, const Strides3& st, int b, int h,
                                           int row0, int len, const float (&acc)[4][HD / 16], const float (&mult)[4],
                                           int rg, int cg) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int t = row0 + rg * 4 + i;
    if (t >= len) continue;
    const long long off = static_cast<long long>(b) * st.b + static_cast<long long>(t) * st.t +
                          static_cast<long long>(h) * st.h;
#pragma unroll
    for (int m = 0; m < HD / 64; ++m) {
      const int col = (cg + 16 * m) * 4;
      float4 v = make_float4(acc[i][4 * m] * mult[i], acc[i][4 * m + 1] * mult[i], acc[i][4 * m + 2] * mult[i],
                             acc[i][4 * m + 3] * mult[i]);
      if (add) {
        const float4 a = *reinterpret_cast<const float4*>(add + off + col);
        v.x += a.x;
        v.y += a.y;
        v.z += a.z;
        v.w += a.w;
      }
      *reinterpret_cast<float4*>(out + off + col) = v;
    }
  }
}

template <int N, int M>
__device__ __forceinline__ void zero(float (&a)[N][M]) {
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int j = 0; j < M; ++j) a[i][j] = 0.f;
}

__device__ __forceinline__ long long stat_index(const AttnShape& s, int b, int h, int t) {
  return (static_cast<long long>(b) * s.H + h) * s.Tq + t;
}

// ------------------------------------------------------------------------------------
// Forward: O = softmax(scale Q K^T) V, L = log-sum-exp (natural log), online over key
// tiles (flash_hog/jax/_attention_impl.py:224-239 computes these with cuDNN).
// ------------------------------------------------------------------------------------
// Two CTAs per SM where shared memory allows (forward and first-order backward; the
// double-backward passes need 171-209 KB per CTA): twice the resident warps to hide
// shared-memory and global-load latency, at <= 128 registers per thread.
template <int HD>
constexpr int kFwdCtas = 2;
template <int HD>
constexpr int kDkdvCtas = HD == 64 ? 2 : 1;

template <int HD>
__global__ void __launch_bounds__(kThreads, kFwdCtas<HD>)
    fwd_kernel(AttnShape s, const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
               float* __restrict__ o, float* __restrict__ lse) {
  using G = Geo<HD>;
  extern __shared__ float4 smem_f4[];
  // K and V tiles are double-buffered: buffer it & 1 holds tile it, and tile it + 1
  // is fetched (cp.async) while tile it is used.
  float* sQ = reinterpret_cast<float*>(smem_f4);
  float* sKV = sQ + G::RES;  // [2][K | V]
  float* sP = sKV + 4 * G::STR;
  const int r0 = blockIdx.x * kRes, h = blockIdx.y, b = blockIdx.z, hk = h / s.G;
  const int rg = threadIdx.x >> 4, cg = threadIdx.x & 15;
  load_rows<HD, kRes>(sQ, q, s.sq, b, h, r0, s.Tq);
  float m[4], l[4], acc[4][G::NO];
#pragma unroll
  for (int i = 0; i < 4; ++i) m[i] = -INFINITY, l[i] = 0.f;
  zero(acc);
  int first;
  const int nt = key_tiles(s, r0, kRes, G::BN, &first);
  auto fetch = [&](int t) {
    float* buf = sKV + (t & 1) * 2 * G::STR;
    load_rows_async<HD, G::BN>(buf, k, s.sk, b, hk, (first + t) * G::BN, s.Tk);
    load_rows_async<HD, G::BN>(buf + G::STR, v, s.sk, b, hk, (first + t) * G::BN, s.Tk);
  };
  if (nt > 0) fetch(0);
  for (int it = 0; it < nt; ++it) {
    const int c0 = (first + it) * G::BN;
    // Buffer (it + 1) & 1 was last read in iteration it - 1, which ended with a barrier.
    if (it + 1 < nt) {
      fetch(it + 1);
      cp_async_wait<2>();  // tile it's two groups have landed; tile it + 1's may be pending
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float* sK = sKV + (it & 1) * 2 * G::STR;
    const float* sV = sK + G::STR;
    float sc[4][G::NC];
    zero(sc);
    score_acc<HD, kRes, G::NC>(sc, sQ, sK, rg, cg);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = r0 + rg * 4 + i;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < G::NC; ++j) {
        sc[i][j] = visible(s, row, c0 + cg + 16 * j) ? sc[i][j] * s.scale : -INFINITY;
        mx = fmaxf(mx, sc[i][j]);
      }
      const float mn = fmaxf(m[i], max16(mx));
      const float base = mn == -INFINITY ? 0.f : mn;
      const float alpha = expf(m[i] - base);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < G::NC; ++j) {
        const float p = expf(sc[i][j] - base);
        sP[(rg * 4 + i) * G::SC + cg + 16 * j] = p;
        rs += p;
      }
      l[i] = l[i] * alpha + sum16(rs);
      m[i] = mn;
#pragma unroll
      for (int n = 0; n < G::NO; ++n) acc[i][n] *= alpha;
    }
    __syncthreads();
    out_acc<HD, G::BN>(acc, sP, sV, rg, cg);
    __syncthreads();  // sP and this tile's buffer are free for the next iteration
  }
  float inv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    inv[i] = l[i] > 0.f ? 1.f / l[i] : 0.f;
    const int row = r0 + rg * 4 + i;
    if (cg == 0 && row < s.Tq) lse[stat_index(s, b, h, row)] = l[i] > 0.f ? m[i] + logf(l[i]) : -INFINITY;
  }
  store_rows<HD>(o, nullptr, s.sq, b, h, r0, s.Tq, acc, inv, rg, cg);
}

// D = rowsum(dO o O), one warp per query row (flash_hog/jax/_tk_gpu.py:93).
template <int HD>
__global__ void __launch_bounds__(kThreads)
    rowdot_kernel(AttnShape s, const float* __restrict__ o, const float* __restrict__ dO, float* __restrict__ delta) {
  const long long row = static_cast<long long>(blockIdx.x) * (kThreads / 32) + (threadIdx.x >> 5);
  const long long rows = static_cast<long long>(s.B) * s.H * s.Tq;
  if (row >= rows) return;  // whole warps leave together
  const int lane = threadIdx.x & 31;
  const int t = static_cast<int>(row % s.Tq);
  const long long bh = row / s.Tq;
  const int h = static_cast<int>(bh % s.H), b = static_cast<int>(bh / s.H);
  const long long off = static_cast<long long>(b) * s.sq.b + static_cast<long long>(t) * s.sq.t +
                        static_cast<long long>(h) * s.sq.h;
  float acc = 0.f;
  for (int e = lane; e < HD; e += 32) acc = fmaf(o[off + e], dO[off + e], acc);
#pragma unroll
  for (int w = 16; w; w >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, w);
  if (lane == 0) delta[row] = acc;
}

// ------------------------------------------------------------------------------------
// First-order backward (flash_hog/jax/_attention_impl.py:242-261 computes these with
// cuDNN): P = exp(scale S - L), dS = scale P o (dO V^T - D);
//   query side: dQ = dS K;   key side: dV = P^T dO, dK = dS^T Q.
// ------------------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(kThreads, kFwdCtas<HD>)
    dq_kernel(AttnShape s, const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
              const float* __restrict__ dO, const float* __restrict__ lse, const float* __restrict__ delta,
              float* __restrict__ dq, const float* dq_acc) {
  using G = Geo<HD>;
  extern __shared__ float4 smem_f4[];
  float* sQ = reinterpret_cast<float*>(smem_f4);
  float* sdO = sQ + G::RES;
  float* sK = sdO + G::RES;
  float* sV = sK + G::STR;
  float* sS = sV + G::STR;
  const int r0 = blockIdx.x * kRes, h = blockIdx.y, b = blockIdx.z, hk = h / s.G;
  const int rg = threadIdx.x >> 4, cg = threadIdx.x & 15;
  load_rows<HD, kRes>(sQ, q, s.sq, b, h, r0, s.Tq);
  load_rows<HD, kRes>(sdO, dO, s.sq, b, h, r0, s.Tq);
  float L[4], D[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = r0 + rg * 4 + i;
    L[i] = row < s.Tq ? lse[stat_index(s, b, h, row)] : 0.f;
    D[i] = row < s.Tq ? delta[stat_index(s, b, h, row)] : 0.f;
  }
  float acc[4][G::NO];
  zero(acc);
  int first;
  const int nt = key_tiles(s, r0, kRes, G::BN, &first);
  for (int it = 0; it < nt; ++it) {
    const int c0 = (first + it) * G::BN;
    __syncthreads();
    load_rows<HD, G::BN>(sK, k, s.sk, b, hk, c0, s.Tk);
    load_rows<HD, G::BN>(sV, v, s.sk, b, hk, c0, s.Tk);
    __syncthreads();
    float sc[4][G::NC], dp[4][G::NC];
    zero(sc);
    zero(dp);
    score_acc<HD, kRes, G::NC>(sc, sQ, sK, rg, cg);
    score_acc<HD, kRes, G::NC>(dp, sdO, sV, rg, cg);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < G::NC; ++j) {
        const bool vis = visible(s, r0 + rg * 4 + i, c0 + cg + 16 * j);
        const float p = vis ? expf(sc[i][j] * s.scale - L[i]) : 0.f;
        sS[(rg * 4 + i) * G::SC + cg + 16 * j] = s.scale * p * (dp[i][j] - D[i]);
      }
    __syncthreads();
    out_acc<HD, G::BN>(acc, sS, sK, rg, cg);
  }
  const float one[4] = {1.f, 1.f, 1.f, 1.f};
  store_rows<HD>(dq, dq_acc, s.sq, b, h, r0, s.Tq, acc, one, rg, cg);
}

template <int HD>
__global__ void __launch_bounds__(kThreads, kDkdvCtas<HD>)
    dkdv_kernel(AttnShape s, const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                const float* __restrict__ dO, const float* __restrict__ lse, const float* __restrict__ delta,
                float* __restrict__ dk, float* __restrict__ dv, const float* dk_acc, const float* dv_acc) {
  using G = Geo<HD>;
  extern __shared__ float4 smem_f4[];
  float* sK = reinterpret_cast<float*>(smem_f4);
  float* sV = sK + G::RES;
  float* sQ = sV + G::RES;
  float* sdO = sQ + G::STR;
  float* sP = sdO + G::STR;
  float* sS = sP + G::SCORE;
  float* sL = sS + G::SCORE;
  float* sD = sL + G::BN;
  const int k0 = blockIdx.x * kRes, hk = blockIdx.y, b = blockIdx.z;
  const int rg = threadIdx.x >> 4, cg = threadIdx.x & 15;
  load_rows<HD, kRes>(sK, k, s.sk, b, hk, k0, s.Tk);
  load_rows<HD, kRes>(sV, v, s.sk, b, hk, k0, s.Tk);
  float adk[4][G::NO], adv[4][G::NO];
  zero(adk);
  zero(adv);
  int first;
  const int nt = query_tiles(s, k0, kRes, G::BN, &first);
  for (int g = 0; g < s.G; ++g) {
    const int h = hk * s.G + g;
    for (int it = 0; it < nt; ++it) {
      const int q0 = (first + it) * G::BN;
      __syncthreads();
      load_rows<HD, G::BN>(sQ, q, s.sq, b, h, q0, s.Tq);
      load_rows<HD, G::BN>(sdO, dO, s.sq, b, h, q0, s.Tq);
      load_stats(sL, lse, s, b, h, q0, G::BN);
      load_stats(sD, delta, s, b, h, q0, G::BN);
      __syncthreads();
      float st[4][G::NC], dpt[4][G::NC];
      zero(st);
      zero(dpt);
      score_acc<HD, kRes, G::NC>(st, sK, sQ, rg, cg);
      score_acc<HD, kRes, G::NC>(dpt, sV, sdO, rg, cg);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < G::NC; ++j) {
          const int c = cg + 16 * j;
          const bool vis = visible(s, q0 + c, k0 + rg * 4 + i);
          const float p = vis ? expf(st[i][j] * s.scale - sL[c]) : 0.f;
          sP[(rg * 4 + i) * G::SC + c] = p;
          sS[(rg * 4 + i) * G::SC + c] = s.scale * p * (dpt[i][j] - sD[c]);
        }
      __syncthreads();
      out_acc<HD, G::BN>(adv, sP, sdO, rg, cg);
      out_acc<HD, G::BN>(adk, sS, sQ, rg, cg);
    }
  }
  const float one[4] = {1.f, 1.f, 1.f, 1.f};
  store_rows<HD>(dk, dk_acc, s.sk, b, hk, k0, s.Tk, adk, one, rg, cg);
  store_rows<HD>(dv, dv_acc, s.sk, b, hk, k0, s.Tk, adv, one, rg, cg);
}

// ------------------------------------------------------------------------------------
// Double backward (flash_hog/_jax_refs/jax_impl.py:273-336,
// flash_hog/jax/_pallas_gpu_kernel.py:149-278,333-369), per (query i, key j):
//   P = exp(scale S - L)   dP = dO V^T   ddS = scale (ddQ K^T + Q ddK^T)   X = dO ddV^T
//   dD = rowsum(P o ddS)   dP2 = X - dP dD - ddS D + dP o ddS   B = rowsum(P o dP2)
//   dS = scale P (dP - D)  dS2 = scale P (dP2 - B)  ddP = P (ddS - dD)
//   dQ' = dS ddK + dS2 K   ddO = ddP V + P ddV     dK' = dS^T ddQ + dS2^T Q   dV' = ddP^T dO
// The query pass needs dD before dP2 exists; expanding B's rowsum,
//   B = rowsum(P o X) - dD rowsum(P o dP) - D dD + rowsum(P o dP o ddS),
// so one sweep gathers all row statistics and a second sweep produces dQ' and ddO.
// ------------------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    bbq_kernel(AttnShape s, const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
               const float* __restrict__ dO, const float* __restrict__ ddq, const float* __restrict__ ddk,
               const float* __restrict__ ddv, const float* __restrict__ lse, const float* __restrict__ delta,
               float* __restrict__ dq2, float* __restrict__ ddo, float* __restrict__ dd_out,
               float* __restrict__ b_out) {
  using G = Geo<HD>;
  constexpr int NBUF = QueryPassBuffers<HD>::N;
  constexpr int BUF = 4 * G::STR;  // K | V | ddK | ddV of one key tile
  extern __shared__ float4 smem_f4[];
  float* sQ = reinterpret_cast<float*>(smem_f4);
  float* sdO = sQ + G::RES;
  float* sddQ = sdO + G::RES;
  float* kbuf = sddQ + G::RES;  // [NBUF][BUF]
  float* tA = kbuf + NBUF * BUF;
  float* tB = tA + G::SCORE;
  const int r0 = blockIdx.x * kRes, h = blockIdx.y, b = blockIdx.z, hk = h / s.G;
  const int rg = threadIdx.x >> 4, cg = threadIdx.x & 15;
  load_rows<HD, kRes>(sQ, q, s.sq, b, h, r0, s.Tq);
  load_rows<HD, kRes>(sdO, dO, s.sq, b, h, r0, s.Tq);
  load_rows<HD, kRes>(sddQ, ddq, s.sq, b, h, r0, s.Tq);
  float L[4], D[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = r0 + rg * 4 + i;
    L[i] = row < s.Tq ? lse[stat_index(s, b, h, row)] : 0.f;
    D[i] = row < s.Tq ? delta[stat_index(s, b, h, row)] : 0.f;
  }
  int first;
  const int nt = key_tiles(s, r0, kRes, G::BN, &first);

  // Items u = 0 .. 2 nt - 1: sweep 1 (row statistics) over the key tiles, then sweep 2
  // (dQ', ddO) over the same tiles. With two buffers, item u + 1's tile is fetched
  // (cp.async) while item u's is used, across the sweep boundary too.
  const int total = 2 * nt;
  auto fetch = [&](int u) {
    const int c0 = (first + u % nt) * G::BN;
    float* buf = kbuf + (u % NBUF) * BUF;
    load_rows_async<HD, G::BN>(buf, k, s.sk, b, hk, c0, s.Tk);
    load_rows_async<HD, G::BN>(buf + G::STR, v, s.sk, b, hk, c0, s.Tk);
    load_rows_async<HD, G::BN>(buf + 2 * G::STR, ddk, s.sk, b, hk, c0, s.Tk);
    load_rows_async<HD, G::BN>(buf + 3 * G::STR, ddv, s.sk, b, hk, c0, s.Tk);
  };

  float sdd[4] = {0.f, 0.f, 0.f, 0.f}, sy[4] = {0.f, 0.f, 0.f, 0.f}, sx[4] = {0.f, 0.f, 0.f, 0.f},
        sz[4] = {0.f, 0.f, 0.f, 0.f};
  float dD[4], Bv[4];
  auto finish_stats = [&]() {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      dD[i] = sum16(sdd[i]);
      Bv[i] = sum16(sx[i]) - dD[i] * sum16(sy[i]) - D[i] * dD[i] + sum16(sz[i]);
      const int row = r0 + rg * 4 + i;
      if (cg == 0 && row < s.Tq) {
        dd_out[stat_index(s, b, h, row)] = dD[i];
        b_out[stat_index(s, b, h, row)] = Bv[i];
      }
    }
  };
  float aq[4][G::NO], ao[4][G::NO];
  zero(aq);
  zero(ao);

  if (NBUF == 2 && total > 0) fetch(0);
  for (int u = 0; u < total; ++u) {
    const int c0 = (first + u % nt) * G::BN;
    if (NBUF == 2) {
      // Buffer (u + 1) % 2 was last read in item u - 1, which ended with a barrier.
      if (u + 1 < total) {
        fetch(u + 1);
        cp_async_wait<4>();  // item u's four groups have landed
      } else {
        cp_async_wait<0>();
      }
    } else {
      fetch(u);  // the previous item ended with a barrier
      cp_async_wait<0>();
    }
    __syncthreads();
    const float* sK = kbuf + (u % NBUF) * BUF;
    const float* sV = sK + G::STR;
    const float* sddK = sV + G::STR;
    const float* sddV = sddK + G::STR;
    // The tile's four score-like products: S, dP, ddS (unscaled) and X.
    float sc[4][G::NC], dp[4][G::NC], dds[4][G::NC], x[4][G::NC];
    zero(sc);
    zero(dp);
    zero(dds);
    zero(x);
    score_acc<HD, kRes, G::NC>(sc, sQ, sK, rg, cg);
    score_acc<HD, kRes, G::NC>(dp, sdO, sV, rg, cg);
    score_acc<HD, kRes, G::NC>(dds, sddQ, sK, rg, cg);
    score_acc<HD, kRes, G::NC>(dds, sQ, sddK, rg, cg);
    score_acc<HD, kRes, G::NC>(x, sdO, sddV, rg, cg);
    if (u < nt) {  // sweep 1 (block-uniform branch)
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < G::NC; ++j) {
          if (!visible(s, r0 + rg * 4 + i, c0 + cg + 16 * j)) continue;
          const float p = expf(sc[i][j] * s.scale - L[i]);
          const float d2 = dds[i][j] * s.scale;
          sdd[i] = fmaf(p, d2, sdd[i]);
          sy[i] = fmaf(p, dp[i][j], sy[i]);
          sx[i] = fmaf(p, x[i][j], sx[i]);
          sz[i] = fmaf(p * dp[i][j], d2, sz[i]);
        }
      if (u == nt - 1) finish_stats();
    } else {  // sweep 2, in two halves over the two score tiles
      float ds2[4][G::NC], pp[4][G::NC];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < G::NC; ++j) {
          const int at = (rg * 4 + i) * G::SC + cg + 16 * j;
          float p = 0.f, ds = 0.f, d2s = 0.f, ddp = 0.f;
          if (visible(s, r0 + rg * 4 + i, c0 + cg + 16 * j)) {
            p = expf(sc[i][j] * s.scale - L[i]);
            const float d2 = dds[i][j] * s.scale;
            const float dp2 = x[i][j] - dp[i][j] * dD[i] - d2 * D[i] + dp[i][j] * d2;
            ds = s.scale * p * (dp[i][j] - D[i]);
            d2s = s.scale * p * (dp2 - Bv[i]);
            ddp = p * (d2 - dD[i]);
          }
          tA[at] = ds;
          tB[at] = ddp;
          ds2[i][j] = d2s;
          pp[i][j] = p;
        }
      __syncthreads();
      out_acc<HD, G::BN>(aq, tA, sddK, rg, cg);  // dQ' += dS ddK
      out_acc<HD, G::BN>(ao, tB, sV, rg, cg);    // ddO += ddP V
      __syncthreads();
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < G::NC; ++j) {
          const int at = (rg * 4 + i) * G::SC + cg + 16 * j;
          tA[at] = ds2[i][j];
          tB[at] = pp[i][j];
        }
      __syncthreads();
      out_acc<HD, G::BN>(aq, tA, sK, rg, cg);    // dQ' += dS2 K
      out_acc<HD, G::BN>(ao, tB, sddV, rg, cg);  // ddO += P ddV
    }
    __syncthreads();  // this item's buffer and the score tiles are free
  }
  if (nt == 0) finish_stats();  // rows that see no key: dD = B = 0
  const float one[4] = {1.f, 1.f, 1.f, 1.f};
  if (dq2) store_rows<HD>(dq2, nullptr, s.sq, b, h, r0, s.Tq, aq, one, rg, cg);
  store_rows<HD>(ddo, nullptr, s.sq, b, h, r0, s.Tq, ao, one, rg, cg);
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    bbk_kernel(AttnShape s, const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
               const float* __restrict__ dO, const float* __restrict__ ddq, const float* __restrict__ ddk,
               const float* __restrict__ ddv, const float* __restrict__ lse, const float* __restrict__ delta,
               const float* __restrict__ dd, const float* __restrict__ bvec, float* __restrict__ dk2,
               float* __restrict__ dv2) {
  using G = Geo<HD>;
  extern __shared__ float4 smem_f4[];
  constexpr int NBUF = KeyPassBuffers<HD>::N;
  constexpr int BUF = 3 * G::STR + 4 * G::BN;  // Q | dO | ddQ | L | D | dD | B of one query tile
  float* sK = reinterpret_cast<float*>(smem_f4);
  float* sV = sK + G::RES;
  float* sddK = sV + G::RES;
  float* sddV = sddK + G::RES;
  float* sbuf = sddV + G::RES;  // [NBUF][BUF]
  float* tDS = sbuf + NBUF * BUF;
  float* tDS2 = tDS + G::SCORE;
  float* tDDP = tDS2 + G::SCORE;
  const int k0 = blockIdx.x * kRes, hk = blockIdx.y, b = blockIdx.z;
  const int rg = threadIdx.x >> 4, cg = threadIdx.x & 15;
  load_rows<HD, kRes>(sK, k, s.sk, b, hk, k0, s.Tk);
  load_rows<HD, kRes>(sV, v, s.sk, b, hk, k0, s.Tk);
  load_rows<HD, kRes>(sddK, ddk, s.sk, b, hk, k0, s.Tk);
  load_rows<HD, kRes>(sddV, ddv, s.sk, b, hk, k0, s.Tk);
  float ak[4][G::NO], av[4][G::NO];
  zero(ak);
  zero(av);
  int first;
  const int nt = query_tiles(s, k0, kRes, G::BN, &first);
  // Items u = (query head g of the group, query tile it) in order; with two buffers,
  // item u + 1 is fetched (cp.async) while item u is used.
  const int total = s.G * nt;
  auto fetch = [&](int u) {
    const int h = hk * s.G + u / nt, q0 = (first + u % nt) * G::BN;
    float* buf = sbuf + (u % NBUF) * BUF;
    float* st = buf + 3 * G::STR;
    stats_async(st, lse, s, b, h, q0, G::BN);
    stats_async(st + G::BN, delta, s, b, h, q0, G::BN);
    stats_async(st + 2 * G::BN, dd, s, b, h, q0, G::BN);
    stats_async(st + 3 * G::BN, bvec, s, b, h, q0, G::BN);
    load_rows_async<HD, G::BN>(buf, q, s.sq, b, h, q0, s.Tq);  // commits the statistics too
    load_rows_async<HD, G::BN>(buf + G::STR, dO, s.sq, b, h, q0, s.Tq);
    load_rows_async<HD, G::BN>(buf + 2 * G::STR, ddq, s.sq, b, h, q0, s.Tq);
  };
  if (NBUF == 2 && total > 0) fetch(0);
  for (int u = 0; u < total; ++u) {
    const int q0 = (first + u % nt) * G::BN;
    if (NBUF == 2) {
      // Buffer (u + 1) % 2 was last read in item u - 1, which ended with a barrier.
      if (u + 1 < total) {
        fetch(u + 1);
        cp_async_wait<3>();  // item u's three groups have landed
      } else {
        cp_async_wait<0>();
      }
    } else {
      fetch(u);  // the previous item ended with a barrier
      cp_async_wait<0>();
    }
    __syncthreads();
    const float* sQ = sbuf + (u % NBUF) * BUF;
    const float* sdO = sQ + G::STR;
    const float* sddQ = sdO + G::STR;
    const float* sL = sddQ + G::STR;
    const float* sD = sL + G::BN;
    const float* sdD = sD + G::BN;
    const float* sB = sdD + G::BN;
    {
      // Transposed products: rows are keys, columns queries.
      float st[4][G::NC], dpt[4][G::NC], ddst[4][G::NC], xt[4][G::NC];
      zero(st);
      zero(dpt);
      zero(ddst);
      zero(xt);
      score_acc<HD, kRes, G::NC>(st, sK, sQ, rg, cg);
      score_acc<HD, kRes, G::NC>(dpt, sV, sdO, rg, cg);
      score_acc<HD, kRes, G::NC>(ddst, sK, sddQ, rg, cg);
      score_acc<HD, kRes, G::NC>(ddst, sddK, sQ, rg, cg);
      score_acc<HD, kRes, G::NC>(xt, sddV, sdO, rg, cg);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < G::NC; ++j) {
          const int c = cg + 16 * j;
          const int at = (rg * 4 + i) * G::SC + c;
          float ds = 0.f, ds2 = 0.f, ddp = 0.f;
          if (visible(s, q0 + c, k0 + rg * 4 + i)) {
            const float p = expf(st[i][j] * s.scale - sL[c]);
            const float d2 = ddst[i][j] * s.scale;
            const float dp2 = xt[i][j] - dpt[i][j] * sdD[c] - d2 * sD[c] + dpt[i][j] * d2;
            ds = s.scale * p * (dpt[i][j] - sD[c]);
            ds2 = s.scale * p * (dp2 - sB[c]);
            ddp = p * (d2 - sdD[c]);
          }
          tDS[at] = ds;
          tDS2[at] = ds2;
          tDDP[at] = ddp;
        }
      __syncthreads();
      out_acc<HD, G::BN>(ak, tDS, sddQ, rg, cg);
      out_acc<HD, G::BN>(ak, tDS2, sQ, rg, cg);
      out_acc<HD, G::BN>(av, tDDP, sdO, rg, cg);
    }
    __syncthreads();  // this item's buffer and the score tiles are free
  }
  const float one[4] = {1.f, 1.f, 1.f, 1.f};
  store_rows<HD>(dk2, nullptr, s.sk, b, hk, k0, s.Tk, ak, one, rg, cg);
  store_rows<HD>(dv2, nullptr, s.sk, b, hk, k0, s.Tk, av, one, rg, cg);
}

template <int HD>
constexpr int smem_fwd() {
  using G = Geo<HD>;
  return (G::RES + 4 * G::STR + G::SCORE) * 4;
}
static_assert(2 * (smem_fwd<64>() + 1024) <= 233472 && 2 * (smem_fwd<128>() + 1024) <= 233472,
              "two forward CTAs per SM");
template <int HD>
constexpr int smem_dq() {
  using G = Geo<HD>;
  return (2 * G::RES + 2 * G::STR + G::SCORE) * 4;
}
template <int HD>
constexpr int smem_dkdv() {
  using G = Geo<HD>;
  return (2 * G::RES + 2 * G::STR + 2 * G::SCORE + 2 * G::BN) * 4;
}
template <int HD>
constexpr int smem_bbq() {
  return QueryPassBuffers<HD>::bytes(QueryPassBuffers<HD>::N);
}
static_assert(QueryPassBuffers<64>::N == 2 && QueryPassBuffers<128>::N == 1, "query-pass buffering");
template <int HD>
constexpr int smem_bbk() {
  return KeyPassBuffers<HD>::bytes(KeyPassBuffers<HD>::N);
}
static_assert(KeyPassBuffers<64>::N == 2 && KeyPassBuffers<128>::N == 1, "key-pass buffering");
static_assert(smem_bbq<64>() <= 232448 && smem_bbk<64>() <= 232448, "shared memory per CTA");
static_assert(smem_bbq<128>() <= 232448 && smem_bbk<128>() <= 232448, "shared memory per CTA");

inline dim3 query_grid(const AttnShape& s) { return dim3((s.Tq + kRes - 1) / kRes, s.H, s.B); }
inline dim3 key_grid(const AttnShape& s) { return dim3((s.Tk + kRes - 1) / kRes, s.Hk, s.B); }

template <int HD>
int fwd(const AttnShape& s, const F32FwdPtrs& p, cudaStream_t st) {
  constexpr int sm = smem_fwd<HD>();
  if (ensure_smem_limit(reinterpret_cast<const void*>(&fwd_kernel<HD>), sm) != kOk) return kLaunchFailed;
  fwd_kernel<HD><<<query_grid(s), kThreads, sm, st>>>(s, p.q, p.k, p.v, p.o, p.lse);
  return after_launch();
}

template <int HD>
int rowdot(const AttnShape& s, const float* o, const float* dO, float* delta, cudaStream_t st) {
  const long long rows = static_cast<long long>(s.B) * s.H * s.Tq;
  const long long blocks = (rows + kThreads / 32 - 1) / (kThreads / 32);
  if (blocks > 0x7fffffffLL) return kUnsupported;
  rowdot_kernel<HD><<<static_cast<unsigned>(blocks), kThreads, 0, st>>>(s, o, dO, delta);
  return after_launch();
}

template <int HD>
int bwd(const AttnShape& s, const F32BwdPtrs& p, cudaStream_t st) {
  int rc = rowdot<HD>(s, p.o, p.dO, p.delta, st);
  if (rc != kOk) return rc;
  constexpr int sq = smem_dq<HD>(), sk = smem_dkdv<HD>();
  if (ensure_smem_limit(reinterpret_cast<const void*>(&dq_kernel<HD>), sq) != kOk) return kLaunchFailed;
  if (ensure_smem_limit(reinterpret_cast<const void*>(&dkdv_kernel<HD>), sk) != kOk) return kLaunchFailed;
  dq_kernel<HD><<<query_grid(s), kThreads, sq, st>>>(s, p.q, p.k, p.v, p.dO, p.lse, p.delta, p.dq, p.dq_acc);
  if ((rc = after_launch()) != kOk) return rc;
  dkdv_kernel<HD><<<key_grid(s), kThreads, sk, st>>>(s, p.q, p.k, p.v, p.dO, p.lse, p.delta, p.dk, p.dv, p.dk_acc,
                                                      p.dv_acc);
  return after_launch();
}

template <int HD>
int bwdbwd(const AttnShape& s, const F32BwdBwdPtrs& p, int passes, cudaStream_t st) {
  int rc = kOk;
  if (passes & kPassQuery) {
    if ((rc = rowdot<HD>(s, p.o, p.dO, p.delta, st)) != kOk) return rc;
    constexpr int sm = smem_bbq<HD>();
    if (ensure_smem_limit(reinterpret_cast<const void*>(&bbq_kernel<HD>), sm) != kOk) return kLaunchFailed;
    bbq_kernel<HD><<<query_grid(s), kThreads, sm, st>>>(s, p.q, p.k, p.v, p.dO, p.ddq, p.ddk, p.ddv, p.lse, p.delta,
                                                         p.dq2, p.ddo, p.dd, p.bv);
    if ((rc = after_launch()) != kOk) return rc;
  }
  if (passes & kPassKey) {
    constexpr int sm = smem_bbk<HD>();
    if (ensure_smem_limit(reinterpret_cast<const void*>(&bbk_kernel<HD>), sm) != kOk) return kLaunchFailed;
    bbk_kernel<HD><<<key_grid(s), kThreads, sm, st>>>(s, p.q, p.k, p.v, p.dO, p.ddq, p.ddk, p.ddv, p.lse, p.delta,
                                                       p.dd, p.bv, p.dk2, p.dv2);
    rc = after_launch();
  }
  return rc;
}

}  // namespace f32

int launch_fwd_f32(const AttnShape& s, int hd, const F32FwdPtrs& p, cudaStream_t stream) {
  return hd == 64 ? f32::fwd<64>(s, p, stream) : f32::fwd<128>(s, p, stream);
}

int launch_bwd_f32(const AttnShape& s, int hd, const F32BwdPtrs& p, cudaStream_t stream) {
  return hd == 64 ? f32::bwd<64>(s, p, stream) : f32::bwd<128>(s, p, stream);
}

int launch_bwdbwd_f32(const AttnShape& s, int hd, const F32BwdBwdPtrs& p, int passes, cudaStream_t stream) {
  return hd == 64 ? f32::bwdbwd<64>(s, p, passes, stream) : f32::bwdbwd<128>(s, p, passes, stream);
}

}  // namespace fh
