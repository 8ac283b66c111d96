// Fused LayerNorm and GELU kernels with their first- and second-order backward,
// for the grad-norm-penalty training step (L + lam ||dL/dtheta||^2), whose gradient
// differentiates every layer's backward once more.
//
// No counterpart in the reference, which has no model code; in a framework these
// ops' double backward is a composite of many elementwise and reduction kernels.
// Here each pass is one kernel over the rows (plus one small column reduction for
// the LayerNorm weight gradients), HBM-bound: every tensor is read or written once.
//
// LayerNorm over the last dimension (N = cols), per row, with r = 1/sqrt(var + eps):
//   forward     xh = (x - mean) r,  y = xh w + b
//   backward    g = dy w,  dx = r (g - mean(g) - xh mean(g xh)),  dw = sum_rows dy xh,  db = sum_rows dy
//   double bwd  given cotangents (u, vb, cb) of (dx, dw, db):
//     t    = r (u - mean(u) - xh mean(u xh))
//     gdy  = w t + vb xh + cb,          gw = sum_rows dy t
//     G    = -(r/N) (Sux g + Sgx u) + vb dy                      (partial in xh at fixed r)
//     gx   = r (G - mean(G) - xh mean(G xh)) - (r^2/N) xh Phi_r,  Phi_r = <u, dx> / r
//   with Su = sum u, Sux = sum u xh, Sg = sum g, Sgx = sum g xh.
// GELU (the exact form, x Phi(x)):
//   h = x Phi(x);  gelu'(x) = Phi(x) + x phi(x);  gelu''(x) = phi(x) (2 - x^2).
//
// Layout: LayerNorm tensors are fp32 (rows, cols) row-major, cols a multiple of 4
// and at most 1024; one warp per row, each lane holding cols/128 float4 chunks.
// Column sums go to a per-block partial buffer and a second kernel adds the
// partials in a fixed order (deterministic, no atomics).

#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <cmath>
#include <cstdint>

#include "kernels.h"

namespace fh {
namespace {

constexpr int kLnWarps = 8;             // rows in flight per block
constexpr int kLnMaxChunks = 8;         // float4 chunks per lane: cols <= 32 * 4 * 8 = 1024

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ float4 ld4_or0(const float* p, bool ok) {
  return ok ? ld4(p) : make_float4(0.f, 0.f, 0.f, 0.f);
}
__device__ __forceinline__ float at(const float4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }
__device__ __forceinline__ void set(float4& v, int i, float x) {
  if (i == 0) v.x = x; else if (i == 1) v.y = x; else if (i == 2) v.z = x; else v.w = x;
}

// Row statistics of x for one warp: mean and 1/sqrt(var + eps) (two passes over registers).
template <int C>
__device__ __forceinline__ void row_stats(const float4 (&x)[C], int nch, int cols, float eps, float* mean, float* rstd) {
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < C; ++c)
    if (c < nch) s += (x[c].x + x[c].y) + (x[c].z + x[c].w);
  const float mu = warp_sum(s) / cols;
  float q = 0.f;
#pragma unroll
  for (int c = 0; c < C; ++c)
    if (c < nch)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float d = at(x[c], i) - mu;
        q = fmaf(d, d, q);
      }
  *mean = mu;
  *rstd = rsqrtf(warp_sum(q) / cols + eps);
}

template <int C>
__global__ void __launch_bounds__(32 * kLnWarps) ln_fwd_kernel(int rows, int cols, const float* __restrict__ x,
                                                                const float* __restrict__ w,
                                                                const float* __restrict__ b, float eps,
                                                                float* __restrict__ y, float* __restrict__ mean,
                                                                float* __restrict__ rstd) {
  const int lane = threadIdx.x & 31, nch = cols / 128 + ((cols & 127) > lane * 4 ? 1 : 0);
  for (int row = blockIdx.x * kLnWarps + (threadIdx.x >> 5); row < rows; row += gridDim.x * kLnWarps) {
    const float* xr = x + static_cast<size_t>(row) * cols;
    float4 xv[C];
#pragma unroll
    for (int c = 0; c < C; ++c) xv[c] = ld4_or0(xr + c * 128 + lane * 4, c < nch);
    float mu, r;
    row_stats<C>(xv, nch, cols, eps, &mu, &r);
    float* yr = y + static_cast<size_t>(row) * cols;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      if (c >= nch) continue;
      const int col = c * 128 + lane * 4;
      const float4 wv = ld4(w + col), bv = ld4(b + col);
      float4 o;
      o.x = fmaf((xv[c].x - mu) * r, wv.x, bv.x);
      o.y = fmaf((xv[c].y - mu) * r, wv.y, bv.y);
      o.z = fmaf((xv[c].z - mu) * r, wv.z, bv.z);
      o.w = fmaf((xv[c].w - mu) * r, wv.w, bv.w);
      st4(yr + col, o);
    }
    if (lane == 0) {
      mean[row] = mu;
      rstd[row] = r;
    }
  }
}

// Adds this block's per-warp column partials (acc0, acc1 per lane) into
// part[blockIdx.x][2][cols] through shared memory, in a fixed warp order.
template <int C>
__device__ __forceinline__ void block_column_partials(const float4 (&acc0)[C], const float4 (&acc1)[C], int nch,
                                                      int cols, float* __restrict__ part, float* smem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // smem: [kLnWarps][2][cols]
#pragma unroll
  for (int c = 0; c < C; ++c) {
    if (c >= nch) continue;
    const int col = c * 128 + lane * 4;
    st4(smem + (warp * 2 + 0) * cols + col, acc0[c]);
    st4(smem + (warp * 2 + 1) * cols + col, acc1[c]);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * cols; i += blockDim.x) {
    const int k = i / cols, col = i - k * cols;
    float s = 0.f;
    for (int wi = 0; wi < kLnWarps; ++wi) s += smem[(wi * 2 + k) * cols + col];
    part[(static_cast<size_t>(blockIdx.x) * 2 + k) * cols + col] = s;
  }
}

template <int C>
__global__ void __launch_bounds__(32 * kLnWarps, 2) ln_bwd_kernel(int rows, int cols, const float* __restrict__ x,
                                                                const float* __restrict__ w,
                                                                const float* __restrict__ mean,
                                                                const float* __restrict__ rstd,
                                                                const float* __restrict__ dy, float* __restrict__ dx,
                                                                float* __restrict__ part) {
  extern __shared__ float smem[];
  const int lane = threadIdx.x & 31, nch = cols / 128 + ((cols & 127) > lane * 4 ? 1 : 0);
  float4 adw[C], adb[C];
#pragma unroll
  for (int c = 0; c < C; ++c) adw[c] = adb[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  const float inv_n = 1.f / cols;
  for (int row = blockIdx.x * kLnWarps + (threadIdx.x >> 5); row < rows; row += gridDim.x * kLnWarps) {
    const size_t off = static_cast<size_t>(row) * cols;
    const float mu = mean[row], r = rstd[row];
    // Two passes over the row; the second re-reads x, w, dy (from L1) instead of
    // keeping them in registers, which leaves room for two blocks per SM.
    float sg = 0.f, sgx = 0.f;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const bool ok = c < nch;
      const int col = c * 128 + lane * 4;
      const float4 xv = ld4_or0(x + off + col, ok), wv = ld4_or0(w + col, ok), dyv = ld4_or0(dy + off + col, ok);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float xhi = ok ? (at(xv, i) - mu) * r : 0.f;
        const float gi = at(dyv, i) * at(wv, i);
        sg += gi;
        sgx = fmaf(gi, xhi, sgx);
        set(adw[c], i, fmaf(at(dyv, i), xhi, at(adw[c], i)));
        set(adb[c], i, at(adb[c], i) + at(dyv, i));
      }
    }
    const float a = warp_sum(sg) * inv_n, be = warp_sum(sgx) * inv_n;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      if (c >= nch) continue;
      const int col = c * 128 + lane * 4;
      const float4 xv = ld4(x + off + col), wv = ld4(w + col), dyv = ld4(dy + off + col);
      float4 o;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        set(o, i, r * (at(dyv, i) * at(wv, i) - a - (at(xv, i) - mu) * r * be));
      st4(dx + off + col, o);
    }
  }
  block_column_partials<C>(adw, adb, nch, cols, part, smem);
}

// Second-order backward. u, vb, cb may be null (zero cotangents).
template <int C>
__global__ void __launch_bounds__(32 * kLnWarps, 2) ln_bwd_bwd_kernel(
    int rows, int cols, const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ mean,
    const float* __restrict__ rstd, const float* __restrict__ dy, const float* __restrict__ u,
    const float* __restrict__ vb, const float* __restrict__ cb, float* __restrict__ gx, float* __restrict__ gdy,
    float* __restrict__ part) {
  extern __shared__ float smem[];
  const int lane = threadIdx.x & 31, nch = cols / 128 + ((cols & 127) > lane * 4 ? 1 : 0);
  float4 agw[C], unused[C];
#pragma unroll
  for (int c = 0; c < C; ++c) agw[c] = unused[c] = make_float4(0.f, 0.f, 0.f, 0.f);
  const float n = static_cast<float>(cols), inv_n = 1.f / n;
  for (int row = blockIdx.x * kLnWarps + (threadIdx.x >> 5); row < rows; row += gridDim.x * kLnWarps) {
    const size_t off = static_cast<size_t>(row) * cols;
    const float mu = mean[row], r = rstd[row];
    // Two passes over the row; the second re-reads x, dy, u (from L1) instead of
    // keeping them in registers, which leaves room for two blocks per SM.
    float su = 0.f, sux = 0.f, sg = 0.f, sgx = 0.f, sug = 0.f, svd = 0.f, svdx = 0.f;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const bool ok = c < nch;
      const int col = c * 128 + lane * 4;
      const float4 xv = ld4_or0(x + off + col, ok), wv = ld4_or0(w + col, ok);
      const float4 vv = ld4_or0(vb + col, ok && vb);
      const float4 dyv = ld4_or0(dy + off + col, ok), uv = ld4_or0(u + off + col, ok && u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float xhi = ok ? (at(xv, i) - mu) * r : 0.f;
        const float gi = at(dyv, i) * at(wv, i), ui = at(uv, i), vd = at(vv, i) * at(dyv, i);
        su += ui;
        sux = fmaf(ui, xhi, sux);
        sg += gi;
        sgx = fmaf(gi, xhi, sgx);
        sug = fmaf(ui, gi, sug);
        svd += vd;
        svdx = fmaf(vd, xhi, svdx);
      }
    }
    su = warp_sum(su);
    sux = warp_sum(sux);
    sg = warp_sum(sg);
    sgx = warp_sum(sgx);
    sug = warp_sum(sug);
    svd = warp_sum(svd);
    svdx = warp_sum(svdx);
    const float mu_u = su * inv_n, mu_ux = sux * inv_n;
    const float mean_g = -r * inv_n * inv_n * (sux * sg + sgx * su) + svd * inv_n;   // mean(G)
    const float mean_gx = -2.f * r * sux * sgx * inv_n * inv_n + svdx * inv_n;       // mean(G xh)
    const float phi_r = sug - sg * su * inv_n - sgx * sux * inv_n;                    // <u, dx> / r
    const float kx = r * r * inv_n * phi_r;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      if (c >= nch) continue;
      const int col = c * 128 + lane * 4;
      const float4 wv = ld4(w + col);
      const float4 vv = vb ? ld4(vb + col) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 cv = cb ? ld4(cb + col) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 xv = ld4(x + off + col), dyv = ld4(dy + off + col);
      const float4 uv = u ? ld4(u + off + col) : make_float4(0.f, 0.f, 0.f, 0.f);
      float4 ox, od;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float xhi = (at(xv, i) - mu) * r, ui = at(uv, i), dyi = at(dyv, i);
        const float t = r * (ui - mu_u - xhi * mu_ux);
        set(od, i, fmaf(at(wv, i), t, fmaf(at(vv, i), xhi, at(cv, i))));
        set(agw[c], i, fmaf(dyi, t, at(agw[c], i)));
        const float gi = dyi * at(wv, i);
        const float G = -r * inv_n * (sux * gi + sgx * ui) + at(vv, i) * dyi;
        set(ox, i, r * (G - mean_g - xhi * mean_gx) - kx * xhi);
      }
      st4(gx + off + col, ox);
      st4(gdy + off + col, od);
    }
  }
  block_column_partials<C>(agw, unused, nch, cols, part, smem);
}

// out0[col] = sum_p part[p][0][col], out1 likewise, in a fixed order: the parts are
// split into kSumGroups runs of consecutive parts, each run summed in order by one
// warp of the block (32 columns per block), then the run sums added in run order.
constexpr int kSumGroups = 16;
__global__ void __launch_bounds__(32 * kSumGroups) column_sum_kernel(int nparts, int cols,
                                                                     const float* __restrict__ part,
                                                                     float* __restrict__ out0,
                                                                     float* __restrict__ out1) {
  __shared__ float runs[kSumGroups][32];
  const int cx = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int i = blockIdx.x * 32 + cx;  // (k, col) flattened over 2 * cols
  const bool valid = i < 2 * cols;
  const int k = valid ? i / cols : 0, col = valid ? i - k * cols : 0;
  const int per = (nparts + kSumGroups - 1) / kSumGroups;
  const int p0 = g * per, p1 = min(nparts, p0 + per);
  float s = 0.f;
  if (valid) {
#pragma unroll 8
    for (int p = p0; p < p1; ++p) s += part[(static_cast<size_t>(p) * 2 + k) * cols + col];
  }
  runs[g][cx] = s;
  __syncthreads();
  if (g == 0 && valid) {
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < kSumGroups; ++q) t += runs[q][cx];
    float* out = k == 0 ? out0 : out1;
    if (out) out[col] = t;
  }
}

// ---------------------------------------------------------------------------------
// GELU (exact), elementwise, T = float or __nv_bfloat16, fp32 arithmetic
// ---------------------------------------------------------------------------------

constexpr float kInvSqrt2 = 0.70710678118654752f;
constexpr float kInvSqrt2Pi = 0.39894228040143268f;

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// mode 0: out0 = gelu(a)
// mode 1: out0 = dh gelu'(a)
// mode 2: out0 = c gelu'(a) (cotangent of dh), out1 = c dh gelu''(a) (cotangent of a); dh may be null (zero)
// One element: the outputs of `mode` from a (and dh, c where the mode reads them).
template <int MODE>
__device__ __forceinline__ void gelu_elem(float x, float dhv, float cv, bool has_dh, float& o0, float& o1) {
  const float cdf = 0.5f * (1.f + erff(x * kInvSqrt2));
  if constexpr (MODE == 0) {
    o0 = x * cdf;
  } else {
    const float pdf = kInvSqrt2Pi * expf(-0.5f * x * x);
    const float d1 = fmaf(x, pdf, cdf);
    if constexpr (MODE == 1) {
      o0 = dhv * d1;
    } else {
      o0 = cv * d1;
      o1 = has_dh ? cv * dhv * pdf * (2.f - x * x) : 0.f;
    }
  }
}

template <typename T, int MODE>
__global__ void gelu_kernel(long long n, const T* __restrict__ a, const T* __restrict__ dh, const T* __restrict__ c,
                            T* __restrict__ out0, T* __restrict__ out1) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float o0 = 0.f, o1 = 0.f;
    gelu_elem<MODE>(to_f(a[i]), MODE == 1 || (MODE == 2 && dh) ? to_f(dh[i]) : 0.f, MODE == 2 ? to_f(c[i]) : 0.f,
                    dh != nullptr, o0, o1);
    out0[i] = from_f<T>(o0);
    if (MODE == 2 && out1) out1[i] = from_f<T>(o1);
  }
}

// 16-byte vectors of E = 16 / sizeof(T) elements (all pointers 16-byte aligned); the
// last n % E elements by the first threads of block 0. Same per-element math.
template <typename T, int MODE>
__global__ void gelu_vec_kernel(long long n, const T* __restrict__ a, const T* __restrict__ dh,
                                const T* __restrict__ c, T* __restrict__ out0, T* __restrict__ out1) {
  constexpr int E = 16 / sizeof(T);
  const long long nvec = n / E;
  const bool has_dh = dh != nullptr;
  for (long long v = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; v < nvec;
       v += static_cast<long long>(gridDim.x) * blockDim.x) {
    uint4 av = reinterpret_cast<const uint4*>(a)[v], dv = make_uint4(0u, 0u, 0u, 0u), cvv = dv;
    if (MODE == 1 || (MODE == 2 && has_dh)) dv = reinterpret_cast<const uint4*>(dh)[v];
    if (MODE == 2) cvv = reinterpret_cast<const uint4*>(c)[v];
    const T* ae = reinterpret_cast<const T*>(&av);
    const T* de = reinterpret_cast<const T*>(&dv);
    const T* ce = reinterpret_cast<const T*>(&cvv);
    uint4 r0, r1;
    T* e0 = reinterpret_cast<T*>(&r0);
    T* e1 = reinterpret_cast<T*>(&r1);
#pragma unroll
    for (int e = 0; e < E; ++e) {
      float o0 = 0.f, o1 = 0.f;
      gelu_elem<MODE>(to_f(ae[e]), to_f(de[e]), to_f(ce[e]), has_dh, o0, o1);
      e0[e] = from_f<T>(o0);
      e1[e] = from_f<T>(o1);
    }
    reinterpret_cast<uint4*>(out0)[v] = r0;
    if (MODE == 2 && out1) reinterpret_cast<uint4*>(out1)[v] = r1;
  }
  if (blockIdx.x == 0 && threadIdx.x < n - nvec * E) {
    const long long i = nvec * E + threadIdx.x;
    float o0 = 0.f, o1 = 0.f;
    gelu_elem<MODE>(to_f(a[i]), MODE == 1 || (MODE == 2 && has_dh) ? to_f(dh[i]) : 0.f,
                    MODE == 2 ? to_f(c[i]) : 0.f, has_dh, o0, o1);
    out0[i] = from_f<T>(o0);
    if (MODE == 2 && out1) out1[i] = from_f<T>(o1);
  }
}

int ln_grid(int rows) {
  const int blocks = (rows + kLnWarps - 1) / kLnWarps;
  const int cap = 4 * sm_count();
  return blocks < cap ? blocks : cap;
}

template <int C>
int ln_launch(int op, int rows, int cols, const float* x, const float* w, const float* b, const float* mean,
              const float* rstd, const float* dy, const float* u, const float* vb, const float* cb, float eps,
              float* out0, float* out1, float* out2, float* out3, float* part, cudaStream_t stream) {
  const int grid = ln_grid(rows);
  const size_t smem = static_cast<size_t>(kLnWarps) * 2 * cols * sizeof(float);
  if (op == 0) {
    ln_fwd_kernel<C><<<grid, 32 * kLnWarps, 0, stream>>>(rows, cols, x, w, b, eps, out0, out1, out2);
    return after_launch();
  }
  if (smem > 48 * 1024) {
    const void* f = op == 1 ? reinterpret_cast<const void*>(&ln_bwd_kernel<C>)
                            : reinterpret_cast<const void*>(&ln_bwd_bwd_kernel<C>);
    if (ensure_smem_limit(f, static_cast<int>(smem)) != kOk) return kLaunchFailed;
  }
  if (op == 1) {
    // out0 = dx, out1 = dw, out2 = db
    ln_bwd_kernel<C><<<grid, 32 * kLnWarps, smem, stream>>>(rows, cols, x, w, mean, rstd, dy, out0, part);
  } else {
    // out0 = gx, out1 = gdy, out2 = gw
    ln_bwd_bwd_kernel<C><<<grid, 32 * kLnWarps, smem, stream>>>(rows, cols, x, w, mean, rstd, dy, u, vb, cb, out0,
                                                                 out1, part);
  }
  if (after_launch() != kOk) return kLaunchFailed;
  float* c0 = op == 1 ? out1 : out2;
  float* c1 = op == 1 ? out2 : nullptr;
  column_sum_kernel<<<(2 * cols + 31) / 32, 32 * kSumGroups, 0, stream>>>(grid, cols, part, c0, c1);
  return after_launch();
}

}  // namespace

int ln_partials_rows(int rows) { return ln_grid(rows); }

int launch_layernorm(int op, int rows, int cols, const float* x, const float* w, const float* b, const float* mean,
                     const float* rstd, const float* dy, const float* u, const float* vb, const float* cb, float eps,
                     float* out0, float* out1, float* out2, float* part, cudaStream_t stream) {
  const int chunks = (cols + 127) / 128;
  if (chunks <= 2) return ln_launch<2>(op, rows, cols, x, w, b, mean, rstd, dy, u, vb, cb, eps, out0, out1, out2, nullptr, part, stream);
  if (chunks <= 4) return ln_launch<4>(op, rows, cols, x, w, b, mean, rstd, dy, u, vb, cb, eps, out0, out1, out2, nullptr, part, stream);
  if (chunks <= 6) return ln_launch<6>(op, rows, cols, x, w, b, mean, rstd, dy, u, vb, cb, eps, out0, out1, out2, nullptr, part, stream);
  if (chunks <= kLnMaxChunks)
    return ln_launch<kLnMaxChunks>(op, rows, cols, x, w, b, mean, rstd, dy, u, vb, cb, eps, out0, out1, out2, nullptr,
                                   part, stream);
  return kUnsupported;
}

int launch_gelu(int mode, bool bf16, long long n, const void* a, const void* dh, const void* c, void* out0, void* out1,
                cudaStream_t stream) {
  const int block = 256;
  // 16-byte vectors when every pointer allows them (torch allocations do).
  auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool vec = aligned(a) && aligned(dh) && aligned(c) && aligned(out0) && aligned(out1);
  const long long per_thread = vec ? (bf16 ? 8 : 4) : 1;
  long long blocks = (n / per_thread + block - 1) / block;
  const long long cap = 8LL * sm_count();
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const unsigned g = static_cast<unsigned>(blocks);
#define FH_GELU(T, K)                                                                                                \
  do {                                                                                                               \
    const T *pa = static_cast<const T*>(a), *pdh = static_cast<const T*>(dh), *pc = static_cast<const T*>(c);       \
    T *p0 = static_cast<T*>(out0), *p1 = static_cast<T*>(out1);                                                      \
    if (mode == 0) K<T, 0><<<g, block, 0, stream>>>(n, pa, pdh, pc, p0, p1);                                         \
    else if (mode == 1) K<T, 1><<<g, block, 0, stream>>>(n, pa, pdh, pc, p0, p1);                                    \
    else K<T, 2><<<g, block, 0, stream>>>(n, pa, pdh, pc, p0, p1);                                                   \
  } while (0)
  if (bf16 && vec) FH_GELU(__nv_bfloat16, gelu_vec_kernel);
  else if (bf16) FH_GELU(__nv_bfloat16, gelu_kernel);
  else if (vec) FH_GELU(float, gelu_vec_kernel);
  else FH_GELU(float, gelu_kernel);
#undef FH_GELU
  return after_launch();
}

}  // namespace fh
