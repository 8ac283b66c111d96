// D = rowsum(dO o O) per query row, fp32, written as (B, H, Tq).
//
// The reference computes this vector in XLA before its double-backward
// kernels (flash_hog/jax/_pallas_gpu_kernel.py:110, flash_hog/jax/_tk_gpu.py:93);
// the first-order backward uses the same vector. Memory-bound: each row is read
// once with 16-byte loads, HD/8 lanes per row, reduced with warp shuffles.

#include <cuda_runtime.h>

#include "kernels.h"

namespace fh {
namespace {

template <int HD>
__global__ void __launch_bounds__(256) rowdot_kernel(const __nv_bfloat16* __restrict__ o,
                                                     const __nv_bfloat16* __restrict__ dO, float* __restrict__ delta,
                                                     AttnShape sh) {
  constexpr int LANES = HD / 8;  // lanes per row, 8 bf16 each
  const long long gid = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long row = gid / LANES;  // (b, h, t) in statistics order
  const int part = static_cast<int>(gid % LANES);
  const long long nrows = static_cast<long long>(sh.B) * sh.H * sh.Tq;
  float acc = 0.f;
  if (row < nrows) {
    const int t = static_cast<int>(row % sh.Tq);
    const int h = static_cast<int>((row / sh.Tq) % sh.H);
    const int b = static_cast<int>(row / (static_cast<long long>(sh.Tq) * sh.H));
    const size_t off = row_offset(sh.sq, b, t, h) + part * 8;
    const uint4 x = *reinterpret_cast<const uint4*>(o + off);
    const uint4 y = *reinterpret_cast<const uint4*>(dO + off);
    const __nv_bfloat162* xa = reinterpret_cast<const __nv_bfloat162*>(&x);
    const __nv_bfloat162* ya = reinterpret_cast<const __nv_bfloat162*>(&y);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 xf = __bfloat1622float2(xa[i]);
      const float2 yf = __bfloat1622float2(ya[i]);
      acc = fmaf(xf.x, yf.x, acc);
      acc = fmaf(xf.y, yf.y, acc);
    }
  }
#pragma unroll
  for (int off = LANES / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (row < nrows && part == 0) delta[row] = acc;
}

template <int HD>
int launch_rowdot_hd(const AttnShape& s, const void* o, const void* dO, float* delta, cudaStream_t stream) {
  const long long threads = static_cast<long long>(s.B) * s.H * s.Tq * (HD / 8);
  const int block = 256;
  const long long grid = (threads + block - 1) / block;
  if (grid > 0x7fffffffLL) return kInvalidArgument;
  rowdot_kernel<HD><<<static_cast<unsigned>(grid), block, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(o), static_cast<const __nv_bfloat16*>(dO), delta, s);
  return after_launch();
}

}  // namespace

int launch_rowdot(const AttnShape& shape, int hd, const void* o, const void* dO, float* delta, cudaStream_t stream) {
  // D is per query row: a packed variable-length batch is one batch entry of total_q rows.
  AttnShape s = shape;
  if (s.cu_q) {
    s.B = 1;
    s.Tq = s.total_q;
  }
  if (hd == 64) return launch_rowdot_hd<64>(s, o, dO, delta, stream);
  if (hd == 128) return launch_rowdot_hd<128>(s, o, dO, delta, stream);
  return kUnsupported;
}

}  // namespace fh
