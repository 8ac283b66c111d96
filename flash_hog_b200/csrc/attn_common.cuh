// Shared pieces of the attention kernels: problem description, tile geometry,
// operand-descriptor helpers and the role layout of a CTA.
//
// Every attention kernel here has the same shape:
//   * a CTA owns BM = 128 "resident" rows (query rows for the query-tiled
//     kernels, key rows for the key-tiled ones) -- these are the TMEM lanes;
//   * it streams BN-row tiles of the other side through a TMA ring;
//   * warp 4 is the TMA producer, warp 5 allocates TMEM and issues tcgen05.mma
//     from one thread, warps 0-3 (one warpgroup, thread = TMEM lane = row) do
//     the elementwise math and the epilogue;
//   * score-like products land in TMEM, the elementwise warps turn them into
//     bf16 operand panels in shared memory, and accumulating products read
//     those panels.

#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "tc05.cuh"

namespace fh {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

constexpr int kBM = 128;            // resident rows per CTA (= TMEM lanes)
constexpr int kThreads = 192;       // 6 warps
constexpr int kWarpProducer = 4;
constexpr int kWarpMma = 5;
constexpr int kEwThreads = 128;     // warps 0-3

// Strides (in elements) of a (batch, seq, head, head_dim) tensor; head_dim stride is 1.
struct Strides3 {
  long long b, t, h;
};

// The mask is a band: with `causal`, query i sees key j iff j <= i + diag and,
// when window > 0, j > i + diag - window (diag = 0: top-left causal; diag =
// Tk - Tq: bottom-right; window: sliding-window length). Without `causal` every
// key is visible.
//
// Packed variable-length batches: with cu_q/cu_k set, sequence b is rows
// [cu_q[b], cu_q[b+1]) of the packed query-side tensors (batch 1, total_q rows)
// and rows [cu_k[b], cu_k[b+1]) of the key-side ones; Tq/Tk are then the longest
// sequence lengths (grid sizes) and each sequence is masked on its own (its own
// lengths and, with `br`, its own bottom-right diagonal). seq_shape() gives a
// kernel the shape of one sequence and where its rows start.
struct AttnShape {
  int B, H, Tq, Tk;  // H: query heads; B: sequences
  int Hk, G;         // key/value heads and the group size H / Hk (query head h uses key head h / G)
  Strides3 sq;   // query-side tensors
  Strides3 sk;   // key-side tensors
  float scale;
  int causal;
  int diag;
  int window;
  int br;                     // bottom-right alignment: diag = Tk - Tq of each sequence
  const int* cu_q;            // varlen sequence starts (B + 1 entries), or null (dense)
  const int* cu_k;
  int total_q, total_k;       // rows of the packed tensors (varlen); Tq, Tk (dense)
};

// Where sequence b's rows start: the batch coordinate of its tensors' views and
// its first query and key row (0, 0 for a dense batch).
struct SeqRange {
  int bc, q0, k0;
};

// The shape of sequence b alone and, in *r, where its rows start. Dense batches
// return `s` itself. Varlen offsets are clamped to the packed tensors, so even
// inconsistent cu_seqlens never address a row outside them.
// Kernels are instantiated for dense (VL = false: `s` itself, no varlen arithmetic)
// and packed (VL = true) batches.
template <bool VL>
__device__ __forceinline__ AttnShape seq_shape(const AttnShape& s, int b, SeqRange* r) {
  if constexpr (!VL) {
    *r = SeqRange{b, 0, 0};
    return s;
  }
  AttnShape l = s;
  const int q0 = max(0, min(s.cu_q[b], s.total_q)), q1 = max(q0, min(s.cu_q[b + 1], s.total_q));
  const int k0 = max(0, min(s.cu_k[b], s.total_k)), k1 = max(k0, min(s.cu_k[b + 1], s.total_k));
  l.Tq = min(q1 - q0, s.Tq);
  l.Tk = min(k1 - k0, s.Tk);
  l.diag = s.br ? l.Tk - l.Tq : 0;
  *r = SeqRange{0, q0, k0};
  return l;
}

// Visible keys [key_lo, key_hi] of query row i (empty when key_hi < key_lo).
__host__ __device__ __forceinline__ int key_hi(const AttnShape& s, int i) {
  return s.causal ? min(s.Tk - 1, i + s.diag) : s.Tk - 1;
}
__host__ __device__ __forceinline__ int key_lo(const AttnShape& s, int i) {
  return (s.causal && s.window > 0) ? max(0, i + s.diag - s.window + 1) : 0;
}
// Queries [query_lo, query_hi] that see key j (empty when query_hi < query_lo).
__host__ __device__ __forceinline__ int query_lo(const AttnShape& s, int j) {
  return s.causal ? max(0, j - s.diag) : 0;
}
__host__ __device__ __forceinline__ int query_hi(const AttnShape& s, int j) {
  return (s.causal && s.window > 0) ? min(s.Tq - 1, j - s.diag + s.window - 1) : s.Tq - 1;
}

// Streamed tiles of `bn` rows that query rows [r0, r0 + rows) need: tiles
// [*first, *first + return value) of the key sequence (0 tiles if none).
__host__ __device__ __forceinline__ int key_tiles(const AttnShape& s, int r0, int rows, int bn, int* first) {
  const int r1 = min(r0 + rows, s.Tq) - 1;
  *first = 0;
  if (r1 < r0) return 0;
  const int lo = key_lo(s, r0), hi = key_hi(s, r1);
  if (hi < lo) return 0;
  *first = lo / bn;
  return hi / bn + 1 - *first;
}
// Streamed tiles of `bn` query rows that key rows [k0, k0 + rows) need.
__host__ __device__ __forceinline__ int query_tiles(const AttnShape& s, int k0, int rows, int bn, int* first) {
  const int k1 = min(k0 + rows, s.Tk) - 1;
  *first = 0;
  if (k1 < k0) return 0;
  const int lo = query_lo(s, k0), hi = query_hi(s, k1);
  if (hi < lo) return 0;
  *first = lo / bn;
  return hi / bn + 1 - *first;
}

// Launch order with L2 locality. A grid of `pairs` (head, batch) pairs x `tiles` tiles
// runs in groups of g pairs: each group's tiles heaviest first (ti = 0) with the group's
// pairs fastest. The CTAs in flight at once then stream the per-head tiles they share
// (K and V for query tiles, Q and dO for key tiles) of a few heads, which stay in L2,
// instead of one or two tiles of every head. w in [0, pairs * tiles).
__host__ __device__ __forceinline__ void grouped_order(int w, int tiles, int pairs, int g, int* ti, int* pair) {
  const int span = g * tiles;
  const int grp = w / span, rem = w - grp * span;
  const int gs = min(g, pairs - grp * g);
  *ti = rem / gs;
  *pair = grp * g + rem % gs;
}

// Group size for grouped_order: every pair in one group (the plain heaviest-first order,
// which balances causal work best) while the shared tiles of all pairs fit in L2
// together, else groups whose shared tiles take about 32 MB. `bytes_per_head` is what
// the CTAs of one head stream in common, `shared` how many consecutive pairs read it
// (the query heads of one key head under GQA, else 1); the result is a multiple of it.
inline int locality_group(int pairs, int shared, long long bytes_per_head) {
  constexpr long long kFitsInL2 = 96ll << 20, kGroupBytes = 32ll << 20;
  if (static_cast<long long>(pairs / shared) * bytes_per_head <= kFitsInL2) return pairs;
  long long g = kGroupBytes / (bytes_per_head > 0 ? bytes_per_head : 1);
  g = (g < 1 ? 1 : g) * shared;
  return g < pairs ? static_cast<int>(g) : pairs;
}

__device__ __forceinline__ size_t row_offset(const Strides3& s, int b, int t, int h) {
  return static_cast<size_t>(b) * s.b + static_cast<size_t>(t) * s.t + static_cast<size_t>(h) * s.h;
}

// Index into a (B, H, T) fp32 statistics vector.
__device__ __forceinline__ size_t stat_index(int b, int h, int t, int H, int T) {
  return (static_cast<size_t>(b) * H + h) * T + t;
}

// Offset of query row t (of its sequence) of head h: query-side tensors and statistics.
__device__ __forceinline__ size_t q_row(const AttnShape& s, const SeqRange& r, int t, int h) {
  return row_offset(s.sq, r.bc, r.q0 + t, h);
}
__device__ __forceinline__ size_t k_row(const AttnShape& s, const SeqRange& r, int t, int h) {
  return row_offset(s.sk, r.bc, r.k0 + t, h);
}
__device__ __forceinline__ size_t q_stat(const AttnShape& s, const SeqRange& r, int t, int h) {
  return stat_index(r.bc, h, r.q0 + t, s.H, s.total_q);
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Loads `rows` rows x HD columns starting at sequence row `row0` of head (b, h)
// into HD/64 consecutive 128B-swizzled panels at `dst` (panel stride rows*128).
template <int HD>
__device__ __forceinline__ void tma_rows(uint8_t* dst, const CUtensorMap* map, uint64_t* bar, int row0, int rows,
                                         int h, int b) {
#pragma unroll
  for (int pnl = 0; pnl < HD / 64; ++pnl) tma_load_4d(dst + pnl * rows * 128, map, bar, pnl * 64, row0, h, b);
}

// Descriptor for k-step `ks` (16 bf16 along K) of a K-major operand whose K
// extent is spread over 64-column panels of `rows` rows.
__device__ __forceinline__ uint64_t desc_k(const uint8_t* base, int rows, int ks) {
  const uint32_t a = smem_u32(base) + (ks >> 2) * rows * 128 + (ks & 3) * 32;
  return smem_desc(a, 16, 1024, kSwizzle128B);
}

// Descriptor for k-step `ks` (16 rows along K) of an MN-major operand stored as
// panels of `rows` K-rows x 64 MN-columns (panel stride rows*128).
__device__ __forceinline__ uint64_t desc_mn(const uint8_t* base, int rows, int ks) {
  const uint32_t a = smem_u32(base) + ks * 16 * 128;
  return smem_desc(a, rows * 128, 1024, kSwizzle128B);
}

// D (+)= A * B^T, A = [128 x K] K-major panels (a_rows = 128), B = [N x K]
// K-major panels (b_rows = N); K = 16 * ksteps.
__device__ __forceinline__ void gemm_abt(uint32_t d, const uint8_t* a, const uint8_t* bm, int b_rows, int ksteps,
                                         uint32_t idesc, bool acc) {
  for (int ks = 0; ks < ksteps; ++ks)
    umma_bf16(d, desc_k(a, kBM, ks), desc_k(bm, b_rows, ks), idesc, (acc || ks > 0) ? 1u : 0u);
}

// D (+)= A * B, A = [128 x K] K-major panels, B = [K x N] MN-major panels of
// K rows (b_rows = K); K = 16 * ksteps.
__device__ __forceinline__ void gemm_ab(uint32_t d, const uint8_t* a, const uint8_t* bm, int b_rows, int ksteps,
                                        uint32_t idesc, bool acc) {
  for (int ks = 0; ks < ksteps; ++ks)
    umma_bf16(d, desc_k(a, kBM, ks), desc_mn(bm, b_rows, ks), idesc, (acc || ks > 0) ? 1u : 0u);
}

// ---- precomputed descriptors ----------------------------------------------------
// A descriptor's low 14 bits hold (shared address >> 4); every operand of a
// k-step chain differs from the chain's first descriptor by a compile-time
// offset in those bits, so the issuing thread adds an immediate per k-step.

// Base descriptor of a K-major operand (128B swizzle, 8-row groups 1024 B apart).
__device__ __forceinline__ uint64_t kdesc(const void* p) { return smem_desc(smem_u32(p), 16, 1024, kSwizzle128B); }

// Base descriptor of an MN-major operand whose 64-column panels are
// `panel_bytes` apart.
__device__ __forceinline__ uint64_t mndesc(const void* p, uint32_t panel_bytes) {
  return smem_desc(smem_u32(p), panel_bytes, 1024, kSwizzle128B);
}

// Descriptor offset of k-step ks of a K-major operand whose 64-column K panels
// are PANEL bytes apart: 32 bytes per k-step inside a panel.
template <int PANEL>
__device__ __forceinline__ constexpr uint64_t koff(int ks) {
  return static_cast<uint64_t>((ks >> 2) * (PANEL >> 4) + (ks & 3) * 2);
}

// Descriptor offset of k-step ks of an MN-major operand: 16 rows of 128 bytes.
__device__ __forceinline__ constexpr uint64_t mnoff(int ks) { return static_cast<uint64_t>(ks * 128); }

// KSTEPS chained tcgen05.mma into d: A K-major (panels A_PANEL bytes apart);
// B K-major (panels B_PANEL apart) or MN-major. The first k-step overwrites d
// unless `acc`.
template <int KSTEPS, int A_PANEL, int B_PANEL, bool B_MN>
__device__ __forceinline__ void umma_chain(uint32_t d, uint64_t a0, uint64_t b0, uint32_t idesc, bool acc) {
#pragma unroll
  for (int ks = 0; ks < KSTEPS; ++ks)
    umma_bf16(d, a0 + koff<A_PANEL>(ks), b0 + (B_MN ? mnoff(ks) : koff<B_PANEL>(ks)), idesc,
              (acc || ks > 0) ? 1u : 0u);
}

// KSTEPS chained tcgen05.mma with A in TMEM (8 columns per k-step from a_tmem)
// and B an MN-major shared-memory operand.
template <int KSTEPS>
__device__ __forceinline__ void umma_chain_ts(uint32_t d, uint32_t a_tmem, uint64_t b0, uint32_t idesc, bool acc) {
#pragma unroll
  for (int ks = 0; ks < KSTEPS; ++ks)
    umma_bf16_ts(d, a_tmem + 8 * ks, b0 + mnoff(ks), idesc, (acc || ks > 0) ? 1u : 0u);
}

// Warp-convergent forms of the two chains (the whole warp calls them), issued
// four k-steps per elected asm block.
template <int KSTEPS, int A_PANEL, int B_PANEL, bool B_MN>
__device__ __forceinline__ void umma_chain_w(uint32_t d, uint64_t a0, uint64_t b0, uint32_t idesc, bool acc) {
  static_assert(KSTEPS % 4 == 0, "chains are issued four k-steps at a time");
#pragma unroll
  for (int ks = 0; ks < KSTEPS; ks += 4) {
    auto bo = [&](int k) { return b0 + (B_MN ? mnoff(k) : koff<B_PANEL>(k)); };
    umma_bf16_x4_w(d, a0 + koff<A_PANEL>(ks), a0 + koff<A_PANEL>(ks + 1), a0 + koff<A_PANEL>(ks + 2),
                   a0 + koff<A_PANEL>(ks + 3), bo(ks), bo(ks + 1), bo(ks + 2), bo(ks + 3), idesc,
                   (acc || ks > 0) ? 1u : 0u);
  }
}

template <int KSTEPS>
__device__ __forceinline__ void umma_chain_ts_w(uint32_t d, uint32_t a_tmem, uint64_t b0, uint32_t idesc, bool acc) {
  static_assert(KSTEPS % 4 == 0 || KSTEPS == 2, "chains are issued four (or two) k-steps at a time");
  if constexpr (KSTEPS == 2) {
    umma_bf16_ts_x2_w(d, a_tmem, b0 + mnoff(0), b0 + mnoff(1), idesc, acc ? 1u : 0u);
  } else {
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ks += 4)
      umma_bf16_ts_x4_w(d, a_tmem + 8 * ks, b0 + mnoff(ks), b0 + mnoff(ks + 1), b0 + mnoff(ks + 2),
                        b0 + mnoff(ks + 3), idesc, (acc || ks > 0) ? 1u : 0u);
  }
}

// KSTEPS chained tcgen05.mma with A in TMEM and B a K-major shared-memory
// operand whose 64-column K panels are B_PANEL bytes apart.
template <int KSTEPS, int B_PANEL>
__device__ __forceinline__ void umma_chain_tsk_w(uint32_t d, uint32_t a_tmem, uint64_t b0, uint32_t idesc, bool acc) {
  static_assert(KSTEPS % 4 == 0, "chains are issued four k-steps at a time");
#pragma unroll
  for (int ks = 0; ks < KSTEPS; ks += 4)
    umma_bf16_ts_x4_w(d, a_tmem + 8 * ks, b0 + koff<B_PANEL>(ks), b0 + koff<B_PANEL>(ks + 1),
                      b0 + koff<B_PANEL>(ks + 2), b0 + koff<B_PANEL>(ks + 3), idesc, (acc || ks > 0) ? 1u : 0u);
}

// Loads a pair of BN-row tiles (X then Y) of HD columns into "pair" panels:
// panel p holds X's rows then Y's rows (2*BN rows of 128 bytes), so the pair is
// one 2*BN-row K-major operand and each half is an MN-major operand with panel
// stride 2*BN*128.
template <int HD>
__device__ __forceinline__ void tma_pair(uint8_t* dst, const CUtensorMap* mx, const CUtensorMap* my, uint64_t* bar,
                                         int row0, int bn, int h, int b) {
#pragma unroll
  for (int pnl = 0; pnl < HD / 64; ++pnl) {
    tma_load_4d(dst + pnl * 2 * bn * 128, mx, bar, pnl * 64, row0, h, b);
    tma_load_4d(dst + pnl * 2 * bn * 128 + bn * 128, my, bar, pnl * 64, row0, h, b);
  }
}

// Records the first device-side error of a launch and raises the CTA's abort flag.
__device__ __forceinline__ void raise_error(int* status, volatile int* abort_flag, int code) {
  *abort_flag = 1;
  if (status) atomicCAS(status, 0, code);
}

// Loads 16 TMEM columns starting at `col` for this thread's lane. A warp may
// only reach the 32 lanes of its sub-partition: lanes 32*(warp % 4) ... +31.
__device__ __forceinline__ void tmem_row16(uint32_t tmem, int warp, int col, uint32_t (&r)[16]) {
  tmem_ld16(tmem + tmem_lane_base(warp & 3) + col, r);
}

// Writes 16 floats as bf16 (32 contiguous bytes) to global memory.
__device__ __forceinline__ void store_bf16x16(__nv_bfloat16* dst, const float (&v)[16]) {
  uint4 a, c;
  a.x = pack_bf16(v[0], v[1]);
  a.y = pack_bf16(v[2], v[3]);
  a.z = pack_bf16(v[4], v[5]);
  a.w = pack_bf16(v[6], v[7]);
  c.x = pack_bf16(v[8], v[9]);
  c.y = pack_bf16(v[10], v[11]);
  c.z = pack_bf16(v[12], v[13]);
  c.w = pack_bf16(v[14], v[15]);
  reinterpret_cast<uint4*>(dst)[0] = a;
  reinterpret_cast<uint4*>(dst)[1] = c;
}

// Writes 16 floats as bf16 into chunks (2*c16, 2*c16+1) of row r of a
// 128B-swizzled panel.
__device__ __forceinline__ void stage_bf16x16(uint8_t* panel, int r, int c16, const float (&v)[16]) {
  const uint32_t base = smem_u32(panel);
  st_shared_v4(base + sw128_offset(r, 2 * c16), pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]),
               pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
  st_shared_v4(base + sw128_offset(r, 2 * c16 + 1), pack_bf16(v[8], v[9]), pack_bf16(v[10], v[11]),
               pack_bf16(v[12], v[13]), pack_bf16(v[14], v[15]));
}

// Drains the TMEM accumulator columns [col, col+HD) of this thread's lane,
// times `mult`, plus the bf16 row `add` when it is not null (it may alias
// `dst`: each element is read before it is written), to a bf16 row in global memory.
template <int HD>
__device__ __forceinline__ void tmem_row_to_global(uint32_t tmem, int warp, int col, __nv_bfloat16* dst,
                                                   bool write, float mult = 1.f, const __nv_bfloat16* add = nullptr) {
#pragma unroll
  for (int c = 0; c < HD; c += 16) {
    uint32_t r[16];
    tmem_row16(tmem, warp, col + c, r);
    tmem_wait_ld();
    reg_fence16(r);
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]) * mult;
    if (write && add) {
      uint4 a[2];
      a[0] = reinterpret_cast<const uint4*>(add + c)[0];
      a[1] = reinterpret_cast<const uint4*>(add + c)[1];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(a);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 f = __bfloat1622float2(h[i]);
        v[2 * i] += f.x;
        v[2 * i + 1] += f.y;
      }
    }
    if (write) store_bf16x16(dst + c, v);
  }
}

template <int HD>
__device__ __forceinline__ void zero_row_global(__nv_bfloat16* dst) {
#pragma unroll
  for (int c = 0; c < HD; c += 8) reinterpret_cast<uint4*>(dst + c)[0] = make_uint4(0, 0, 0, 0);
}

}  // namespace fh
