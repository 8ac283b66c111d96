// Pieces shared by the warp-specialised attention kernels (double backward and
// first-order backward): the 11-warp CTA layout, TMEM operand shares, bias
// operands for the tensor core, and the persistent work-item order.

#pragma once

#include "attn_common.cuh"

namespace fh {

// ----------------------------------------------------------------------------------
// CTA layout shared by the warp-specialised kernels
// ----------------------------------------------------------------------------------
//
// 11 warps. Warp 0 allocates TMEM and issues the score MMAs, warp 1 issues the
// accumulating (operand) MMAs, warp 2 is the TMA producer, warps 3-10 are two
// elementwise warpgroups: thread (warp, lane) owns TMEM lane 32*(warp%4)+lane
// (one resident row) and warpgroup w = (warp-3)/4 owns columns [CW w, CW w + CW)
// of every BN-row streamed tile (CW = BN/2: 32 at head_dim 64, 16 at 128). TMEM lane quadrants pin the elementwise warps
// to all four schedulers, and their arithmetic starves a co-resident issuing
// thread; two issuers on different schedulers halve that exposure and let the
// score MMAs of the next tile and the operand MMAs of this tile be issued
// independently, each as soon as its inputs are ready.
// Each elementwise thread loads its CW-column share of all four score tiles
// into registers and releases the score buffer at once. The bf16 operands it
// produces (dS, dS2, ddP, P) go back to TMEM with tcgen05.st and are read there
// as the A operand of the accumulating MMAs.
constexpr int kBBThreads = 352;
constexpr int kBBEwWarps = 8;  // elementwise arrivals are one per warp
constexpr int kBBWarpMma = 0;      // score MMAs; TMEM allocation
constexpr int kBBWarpMmaOut = 1;   // operand (accumulating) MMAs
constexpr int kBBWarpProducer = 2;
constexpr int kBBFirstEwWarp = 3;

// All lanes of the warp have finished their TMEM / shared-memory accesses; one lane arrives.
__device__ __forceinline__ void warp_arrive(uint64_t* bar) {
  tc_fence_before();
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
}

// This thread's CW-column share of a score tile (x16 loads).
template <int CW>
__device__ __forceinline__ void tmem_share(uint32_t tmem, int warp, int col, uint32_t (&r)[CW]) {
  static_assert(CW % 16 == 0, "shares are whole x16 loads");
#pragma unroll
  for (int c = 0; c < CW; c += 16)
    tmem_ld16(tmem + tmem_lane_base(warp & 3) + col + c, *reinterpret_cast<uint32_t(*)[16]>(&r[c]));
}

// Two raw fp32 register values as an fp32x2 operand of the packed instructions.
__device__ __forceinline__ float2 f2(uint32_t a, uint32_t b) { return make_float2(__uint_as_float(a), __uint_as_float(b)); }

template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i])::"memory");
}

// Stores a thread's N packed bf16 operand columns (N = 16 or 8) to TMEM.
template <int N>
__device__ __forceinline__ void tmem_st_ops(uint32_t taddr, const uint32_t (&r)[N]) {
  static_assert(N == 16 || N == 8, "operand shares are 16 or 8 packed columns");
  if constexpr (N == 16) tmem_st16(taddr, r);
  else tmem_st8(taddr, r);
}

// One 16-byte chunk of a 32B-swizzled K = 16 bf16 operand row (tiles 256-byte aligned).
__device__ __forceinline__ uint32_t sw32_offset(int r, int c) {
  return static_cast<uint32_t>(r * 32 + ((c ^ ((r >> 2) & 1)) << 4));
}

// Writes (hi, lo) with hi + lo = x to within 2^-16 |x| as row r of a bias operand.
__device__ __forceinline__ void store_bias_row(uint32_t tile, int r, float x) {
  const __nv_bfloat16 hi = __float2bfloat16_rn(x);
  const __nv_bfloat16 lo = __float2bfloat16_rn(x - __bfloat162float(hi));
  const uint32_t pair = static_cast<uint32_t>(__bfloat16_as_ushort(hi)) |
                        (static_cast<uint32_t>(__bfloat16_as_ushort(lo)) << 16);
  st_shared_v4(tile + sw32_offset(r, 0), pair, 0u, 0u, 0u);
  st_shared_v4(tile + sw32_offset(r, 1), 0u, 0u, 0u, 0u);
}

// Partial rowsum(dO o) over head_dim columns [HD/2 wg, HD/2 wg + HD/2) of row r of two
// resident 128-row tiles (128B-swizzled 64-column panels, as loaded by TMA).
template <int HD>
__device__ __forceinline__ float rowdot_share(const uint8_t* s_o, const uint8_t* s_do, int r, int wg) {
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < HD / 16; ++c) {  // 16-byte chunks: HD/8 per row, half of them per warpgroup
    const int chunk = wg * (HD / 16) + c;
    const int panel = chunk >> 3;
    const uint32_t off = panel * kBM * 128 + sw128_offset(r, chunk & 7);
    const uint4 x = *reinterpret_cast<const uint4*>(s_o + off);
    const uint4 y = *reinterpret_cast<const uint4*>(s_do + off);
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
  return acc;
}

// Copies bf16 columns [c0, c0 + NC) of row r of a resident 128-row tile
// (128B-swizzled 64-column panels, as loaded by TMA) into this thread's TMEM
// lane as packed pairs -- the layout of a TMEM A operand: column j holds
// elements 2j (low half) and 2j + 1 -- starting at TMEM address `t` + c0/2.
template <int NC>
__device__ __forceinline__ void row_to_tmem(const uint8_t* tile, int r, int c0, uint32_t t) {
  static_assert(NC % 32 == 0, "whole x16 stores");
#pragma unroll
  for (int c = 0; c < NC; c += 32) {
    uint32_t v[16];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int chunk = (c0 + c) / 8 + k;  // 16-byte chunk of the row
      const uint4 x =
          *reinterpret_cast<const uint4*>(tile + (chunk >> 3) * kBM * 128 + sw128_offset(r, chunk & 7));
      v[4 * k] = x.x;
      v[4 * k + 1] = x.y;
      v[4 * k + 2] = x.z;
      v[4 * k + 3] = x.w;
    }
    tmem_st16(t + (c0 + c) / 2, v);
  }
}

// The j-th item of persistent CTA c out of P: a "snake" over the heaviest-first
// order (c, then 2P-1-c, ...), which balances the causal work to within a few
// percent without a global counter.
__device__ __forceinline__ int snake_item(int j, int c, int P) { return j * P + ((j & 1) ? P - 1 - c : c); }

}  // namespace fh
