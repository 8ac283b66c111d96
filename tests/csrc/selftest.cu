// Unit test of the tcgen05 building blocks (not part of the attention API), plus
// host entry points for the launch-order helpers of attn_common.cuh (grouped_order,
// locality_group), which the CPU tests drive directly.
//
// One CTA computes C[128][N] = A[128][K] * B in fp32 through TMA-loaded,
// 128B-swizzled panels and tcgen05.mma, then reads the accumulator back from
// TMEM. It checks, on the GPU, the conventions every attention kernel relies
// on: the K-major and MN-major shared-memory descriptors (including panel
// strides), the instruction descriptor, the TMEM lane/column layout seen by
// tcgen05.ld, and the swizzled st.shared writes used for thread-built operands.

#include <cuda_runtime.h>

#include "attn_common.cuh"
#include "tc05.cuh"
#include "tmap.h"

namespace {

constexpr int kThreads = 128;

struct SelftestArgs {
  const __nv_bfloat16* A;  // [128][K] row-major
  float* C;                // [128][N] row-major
  int N, K, b_mn, a_threads;
  int* status;
};

__global__ void __launch_bounds__(kThreads, 1)
    umma_selftest_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         SelftestArgs p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_s = smem;               // K/64 panels x 16 KB
  uint8_t* b_s = smem + 2 * 16384;   // up to 64 KB
  __shared__ uint64_t bar_load, bar_mma;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid / 32;
  const int N = p.N, K = p.K;
  const int a_panels = K / 64;
  const uint32_t a_bytes = a_panels * 16384u;
  const uint32_t b_bytes = static_cast<uint32_t>(N) * K * 2u;

  if (tid == 0) {
    abort_flag = 0;
    fh::mbar_init(&bar_load, 1);
    fh::mbar_init(&bar_mma, 1);
    fh::mbar_fence_init();
  }
  if (warp == 0) fh::tmem_alloc(&tmem_base, 256);
  __syncthreads();
  fh::tc_fence_after();
  const uint32_t tmem = tmem_base;

  if (p.a_threads) {
    // Each thread writes its row of A into the swizzled panels.
    const __nv_bfloat16* row = p.A + static_cast<size_t>(tid) * K;
    for (int pnl = 0; pnl < a_panels; ++pnl)
      for (int c = 0; c < 8; ++c) {
        uint4 v = *reinterpret_cast<const uint4*>(row + pnl * 64 + c * 8);
        fh::st_shared_v4(fh::smem_u32(a_s + pnl * 16384) + fh::sw128_offset(tid, c), v.x, v.y, v.z, v.w);
      }
    fh::fence_async_smem();
  }
  __syncthreads();

  bool ok = true;
  if (tid == 0) {
    fh::mbar_arrive_expect_tx(&bar_load, (p.a_threads ? 0u : a_bytes) + b_bytes);
    if (!p.a_threads)
      for (int pnl = 0; pnl < a_panels; ++pnl) fh::tma_load_2d(a_s + pnl * 16384, &tmA, &bar_load, pnl * 64, 0);
    if (!p.b_mn) {
      // Bt[N][K]: panels of N rows x 64 K-columns.
      for (int pnl = 0; pnl < a_panels; ++pnl) fh::tma_load_2d(b_s + pnl * N * 128, &tmB, &bar_load, pnl * 64, 0);
    } else {
      // B[K][N]: panels of K rows x 64 N-columns.
      for (int pnl = 0; pnl < N / 64; ++pnl) fh::tma_load_2d(b_s + pnl * K * 128, &tmB, &bar_load, pnl * 64, 0);
    }
    ok = fh::mbar_wait(&bar_load, 0, &abort_flag);
    if (ok) {
      fh::tc_fence_after();
      const uint32_t idesc = fh::idesc_bf16_f32(128, N, false, p.b_mn != 0);
      for (int ks = 0; ks < K / 16; ++ks) {
        const uint32_t a_addr = fh::smem_u32(a_s) + (ks / 4) * 16384 + (ks % 4) * 32;
        const uint64_t adesc = fh::smem_desc(a_addr, 16, 1024, fh::kSwizzle128B);
        uint64_t bdesc;
        if (!p.b_mn) {
          const uint32_t b_addr = fh::smem_u32(b_s) + (ks / 4) * N * 128 + (ks % 4) * 32;
          bdesc = fh::smem_desc(b_addr, 16, 1024, fh::kSwizzle128B);
        } else {
          const uint32_t b_addr = fh::smem_u32(b_s) + ks * 16 * 128;
          bdesc = fh::smem_desc(b_addr, K * 128, 1024, fh::kSwizzle128B);
        }
        fh::umma_bf16(tmem, adesc, bdesc, idesc, ks > 0 ? 1u : 0u);
      }
      fh::umma_commit(&bar_mma);
    } else {
      abort_flag = 1;
      atomicExch(p.status, fh::kDevTimeoutTmaFull);
    }
  }
  __syncwarp();
  ok = fh::mbar_wait(&bar_mma, 0, &abort_flag);
  if (ok) {
    fh::tc_fence_after();
    const int row = warp * 32 + (tid % 32);
    for (int c0 = 0; c0 < N; c0 += 16) {
      uint32_t r[16];
      fh::tmem_ld16(tmem + fh::tmem_lane_base(warp) + c0, r);
      fh::tmem_wait_ld();
      fh::reg_fence16(r);
      for (int j = 0; j < 16; ++j) p.C[static_cast<size_t>(row) * N + c0 + j] = __uint_as_float(r[j]);
    }
  } else if (tid == 0) {
    atomicExch(p.status, fh::kDevTimeoutMma);
  }
  fh::tc_fence_before();
  __syncthreads();
  if (warp == 0) fh::tmem_dealloc(tmem, 256);
}

}  // namespace

// C ABI used only by tests/test_gpu_primitives.py.
extern "C" int fh_selftest_umma(const void* A, const void* B, float* C, int N, int K, int b_mn, int a_threads,
                                int* status, void* stream) {
  if (K != 64 && K != 128) return 1;
  if (N < 64 || N > 256 || N % 64 != 0) return 1;
  CUtensorMap tmA, tmB;
  {
    uint64_t dims[2] = {static_cast<uint64_t>(K), 128};
    uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    uint32_t box[2] = {64, 128};
    if (!fh::make_tmap_bf16(&tmA, A, 2, dims, strides, box)) return 2;
  }
  if (!b_mn) {
    uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    uint32_t box[2] = {64, static_cast<uint32_t>(N)};
    if (!fh::make_tmap_bf16(&tmB, B, 2, dims, strides, box)) return 2;
  } else {
    uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(K)};
    uint64_t strides[1] = {static_cast<uint64_t>(N) * 2};
    uint32_t box[2] = {64, static_cast<uint32_t>(K)};
    if (!fh::make_tmap_bf16(&tmB, B, 2, dims, strides, box)) return 2;
  }
  const int smem = 1024 + 2 * 16384 + 65536;
  cudaFuncSetAttribute(umma_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  SelftestArgs args{static_cast<const __nv_bfloat16*>(A), C, N, K, b_mn, a_threads, status};
  umma_selftest_kernel<<<1, kThreads, smem, static_cast<cudaStream_t>(stream)>>>(tmA, tmB, args);
  return cudaGetLastError() == cudaSuccess ? 0 : 3;
}

// Host wrappers of the attention kernels' launch-order helpers (CPU-testable).
extern "C" void fh_selftest_grouped_order(int w, int tiles, int pairs, int g, int* ti, int* pair) {
  fh::grouped_order(w, tiles, pairs, g, ti, pair);
}

extern "C" int fh_selftest_locality_group(int pairs, int shared, long long bytes_per_head) {
  return fh::locality_group(pairs, shared, bytes_per_head);
}
