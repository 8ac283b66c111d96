// Cross entropy of the grad-norm-penalty step's language-model head: forward,
// backward and the backward's backward, one kernel each, one CTA per row.
//
// For logits z (rows x vocab, fp32 or bf16) and targets t:
//   forward        lse_r = log sum_v exp(z_rv),  loss_r = lse_r - z_r,t_r
//   backward       dz = g s (p - onehot(t)),  p = exp(z - lse) (softmax), g the
//                  upstream scalar (device memory), s a host scale (1/rows for a mean)
//   backward's backward, given the cotangent u of dz:
//                  gz = g s p (u - <p, u>_row)           (w.r.t. z)
//                  gg_r = s (<p_r, u_r> - u_r,t_r)       (w.r.t. g, summed over rows by the caller)
// A target outside [0, vocab) contributes no one-hot term (and a NaN loss).
// The model computes these from a (rows, vocab) tensor that is read once per pass
// (twice in the backward's backward, the second time from L2); a framework's
// composition of log_softmax, nll and their gradients writes fp32 copies of the
// logits and several intermediates of the same size.

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "kernels.h"

namespace fh {
namespace {

constexpr int kXentThreads = 256;
constexpr float kXLog2e = 1.4426950408889634f;

__device__ __forceinline__ float x2f(float v) { return v; }
__device__ __forceinline__ float x2f(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T f2x(float v);
template <>
__device__ __forceinline__ float f2x<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 f2x<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

__device__ __forceinline__ float xex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Block-wide sum (all threads receive it); `red` holds one float per warp.
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // `red` may still be read by a previous call
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kXentThreads / 32; ++w) t += red[w];
  return t;
}

// Row r's elements in 16-byte vectors of E = 16 / sizeof(T) (when `vec`), then a
// scalar tail; f(index, value) for each element this thread owns.
template <typename T, typename F>
__device__ __forceinline__ void for_row(const T* __restrict__ row, int vocab, bool vec, F&& f) {
  constexpr int E = 16 / sizeof(T);
  const int nvec = vec ? vocab / E : 0;
  for (int i = threadIdx.x; i < nvec; i += kXentThreads) {
    const uint4 x = reinterpret_cast<const uint4*>(row)[i];
    const T* e = reinterpret_cast<const T*>(&x);
#pragma unroll
    for (int k = 0; k < E; ++k) f(i * E + k, x2f(e[k]));
  }
  for (int i = nvec * E + threadIdx.x; i < vocab; i += kXentThreads) f(i, x2f(row[i]));
}

template <typename T>
__global__ void __launch_bounds__(kXentThreads) xent_fwd_kernel(int vocab, long long ld, bool vec,
                                                                 const T* __restrict__ z,
                                                                 const long long* __restrict__ t,
                                                                 float* __restrict__ lse, float* __restrict__ loss) {
  __shared__ float red[kXentThreads / 32];
  const int r = blockIdx.x;
  const T* row = z + static_cast<long long>(r) * ld;
  // Online: running maximum m and the sum s of exp(z - m) over this thread's elements.
  float m = -INFINITY, s = 0.f;
  for_row(row, vocab, vec, [&](int, float x) {
    if (x > m) {
      s = s * xex2((m - x) * kXLog2e);
      m = x;
    }
    s += xex2((x - m) * kXLog2e);
  });
  // Block maximum, then the sums rescaled to it.
  float bm = m;
#pragma unroll
  for (int o = 16; o; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
  __shared__ float redm[kXentThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) redm[warp] = bm;
  __syncthreads();
  bm = redm[0];
#pragma unroll
  for (int w = 1; w < kXentThreads / 32; ++w) bm = fmaxf(bm, redm[w]);
  const float part = m == -INFINITY ? 0.f : s * xex2((m - bm) * kXLog2e);
  const float total = block_sum(part, red);
  if (threadIdx.x == 0) {
    const float l = bm + logf(total);
    lse[r] = l;
    const long long tr = t[r];  // a target outside [0, vocab) gives a NaN loss (no element is read)
    loss[r] = (tr >= 0 && tr < vocab) ? l - x2f(row[tr]) : __int_as_float(0x7fc00000);
  }
}

template <typename T>
__global__ void __launch_bounds__(kXentThreads) xent_bwd_kernel(int vocab, long long ld, bool vec,
                                                                 const T* __restrict__ z,
                                                                 const long long* __restrict__ t,
                                                                 const float* __restrict__ lse,
                                                                 const float* __restrict__ g, float s,
                                                                 T* __restrict__ dz) {
  const int r = blockIdx.x;
  const T* row = z + static_cast<long long>(r) * ld;
  T* out = dz + static_cast<long long>(r) * vocab;
  const float l = lse[r], gs = g[0] * s;
  const long long tr = t[r];
  constexpr int E = 16 / sizeof(T);
  const int nvec = vec ? vocab / E : 0;
  for (int i = threadIdx.x; i < nvec; i += kXentThreads) {
    const uint4 x = reinterpret_cast<const uint4*>(row)[i];
    const T* e = reinterpret_cast<const T*>(&x);
    uint4 o;
    T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int k = 0; k < E; ++k) {
      const float p = xex2((x2f(e[k]) - l) * kXLog2e);
      oe[k] = f2x<T>(gs * (p - (i * E + k == tr ? 1.f : 0.f)));
    }
    reinterpret_cast<uint4*>(out)[i] = o;
  }
  for (int i = nvec * E + threadIdx.x; i < vocab; i += kXentThreads) {
    const float p = xex2((x2f(row[i]) - l) * kXLog2e);
    out[i] = f2x<T>(gs * (p - (i == tr ? 1.f : 0.f)));
  }
}

template <typename T>
__global__ void __launch_bounds__(kXentThreads) xent_bwd_bwd_kernel(int vocab, long long ld, bool vec,
                                                                     const T* __restrict__ z,
                                                                     const long long* __restrict__ t,
                                                                     const float* __restrict__ lse,
                                                                     const float* __restrict__ g, float s,
                                                                     const T* __restrict__ u, T* __restrict__ gz,
                                                                     float* __restrict__ gg) {
  __shared__ float red[kXentThreads / 32];
  const int r = blockIdx.x;
  const T* row = z + static_cast<long long>(r) * ld;
  const T* urow = u + static_cast<long long>(r) * vocab;
  T* out = gz + static_cast<long long>(r) * vocab;
  const float l = lse[r], gs = g[0] * s;
  constexpr int E = 16 / sizeof(T);
  const int nvec = vec ? vocab / E : 0;
  // <p, u> over the row.
  float dot = 0.f;
  for (int i = threadIdx.x; i < nvec; i += kXentThreads) {
    const uint4 x = reinterpret_cast<const uint4*>(row)[i], y = reinterpret_cast<const uint4*>(urow)[i];
    const T* e = reinterpret_cast<const T*>(&x);
    const T* ue = reinterpret_cast<const T*>(&y);
#pragma unroll
    for (int k = 0; k < E; ++k) dot = fmaf(xex2((x2f(e[k]) - l) * kXLog2e), x2f(ue[k]), dot);
  }
  for (int i = nvec * E + threadIdx.x; i < vocab; i += kXentThreads)
    dot = fmaf(xex2((x2f(row[i]) - l) * kXLog2e), x2f(urow[i]), dot);
  dot = block_sum(dot, red);
  // gz = g s p (u - dot).
  for (int i = threadIdx.x; i < nvec; i += kXentThreads) {
    const uint4 x = reinterpret_cast<const uint4*>(row)[i], y = reinterpret_cast<const uint4*>(urow)[i];
    const T* e = reinterpret_cast<const T*>(&x);
    const T* ue = reinterpret_cast<const T*>(&y);
    uint4 o;
    T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int k = 0; k < E; ++k) oe[k] = f2x<T>(gs * xex2((x2f(e[k]) - l) * kXLog2e) * (x2f(ue[k]) - dot));
    reinterpret_cast<uint4*>(out)[i] = o;
  }
  for (int i = nvec * E + threadIdx.x; i < vocab; i += kXentThreads)
    out[i] = f2x<T>(gs * xex2((x2f(row[i]) - l) * kXLog2e) * (x2f(urow[i]) - dot));
  if (threadIdx.x == 0) {
    const long long tr = t[r];
    gg[r] = s * (dot - ((tr >= 0 && tr < vocab) ? x2f(urow[tr]) : 0.f));
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int launch_xent(int op, bool bf16, int rows, int vocab, long long ld, const void* z, const long long* t, float* lse,
                float* loss, const float* g, float s, const void* u, void* out, float* gg, cudaStream_t stream) {
  const int e = bf16 ? 8 : 4;  // elements per 16-byte vector
  const bool vec = aligned16(z) && ld % e == 0 && vocab % e == 0 && aligned16(u) && aligned16(out);
#define FH_XENT(T)                                                                                                  \
  do {                                                                                                              \
    const T* zz = static_cast<const T*>(z);                                                                         \
    if (op == 0)                                                                                                    \
      xent_fwd_kernel<T><<<rows, kXentThreads, 0, stream>>>(vocab, ld, vec, zz, t, lse, loss);                      \
    else if (op == 1)                                                                                               \
      xent_bwd_kernel<T><<<rows, kXentThreads, 0, stream>>>(vocab, ld, vec, zz, t, lse, g, s, static_cast<T*>(out)); \
    else                                                                                                            \
      xent_bwd_bwd_kernel<T><<<rows, kXentThreads, 0, stream>>>(vocab, ld, vec, zz, t, lse, g, s,                   \
                                                                 static_cast<const T*>(u), static_cast<T*>(out), gg); \
  } while (0)
  if (bf16) FH_XENT(__nv_bfloat16);
  else FH_XENT(float);
#undef FH_XENT
  return after_launch();
}

}  // namespace fh
