/*
 * flash_hog_b200 -- C ABI of the B200 (sm_100a) attention hot path of Flash Hog:
 * forward, first-order backward and double backward (vjp of the vjp).
 *
 * The reference reaches its native double backward through one XLA FFI handler,
 * `TkBwdBwd` (flash_hog/csrc/tk_bwdbwd/ffi.cu:79-98), registered with
 * `jax.ffi.register_ffi_target("tk_bwdbwd", ...)` (flash_hog/jax/_tk_gpu.py:57)
 * and called through `jax.ffi.ffi_call` (flash_hog/jax/_tk_gpu.py:96-100). Its
 * forward and first-order backward are cuDNN custom calls
 * (flash_hog/jax/_attention_impl.py:224-261). The entry points below replace
 * those three call sites with plain C functions: raw device pointers, sizes,
 * strides, a stream, an int status. No torch or XLA types cross this boundary.
 *
 * Conventions shared by all entry points
 *  - Every tensor operand (bf16; fp32 for the _f32 entry points) is addressed
 *    as (batch, seq, head, head_dim) with the
 *    element strides given in fh_attn_dims (head_dim stride 1). BTNH, the layout
 *    of the reference API (flash_hog/jax/attention.py:19-49), and BHTD, the
 *    layout of the reference's native kernels (ffi.cu:7-10), are both strided
 *    views of this form. Strides must be multiples of 8 elements and base
 *    pointers 16-byte aligned (TMA requirements).
 *  - Per-query fp32 vectors (lse, delta, dd, bvec) are (batch, head, seq_q)
 *    contiguous, the layout of the cuDNN log-sum-exp the reference saves
 *    (flash_hog/jax/_attention_impl.py:114-139). lse is the natural-log
 *    log-sum-exp of the scaled, masked scores.
 *  - causal = 1 applies the top-left mask (query i sees keys j <= i), the mask
 *    of flash_hog/jax/_pallas_gpu_kernel.py:37-41; causal = 2 the bottom-right
 *    one (query i sees keys j <= i + seq_k - seq_q), the alignment of the
 *    reference's JAX statements (flash_hog/_jax_refs/jax_impl.py:104-109), which
 *    also take a sliding window: fh_attn_dims.window = W > 0 further limits
 *    query i to the W keys ending at its diagonal. causal = 0: no mask (window
 *    must be 0). A query that sees no key at all (bottom-right with seq_q >
 *    seq_k) gets o = 0, lse = -inf and zero gradients.
 *  - head_dim is 64 or 128; seq_q, seq_k >= 1 (no divisibility requirement:
 *    ragged edges are masked); heads a multiple of kv_heads (grouped-query
 *    attention; key-side tensors and dk, dv, dk2, dv2 have kv_heads heads).
 *  - Calls are asynchronous on `stream` (a cudaStream_t, may be NULL for the
 *    legacy default stream) and never allocate device memory except a 4-byte
 *    status word per device on first use. Scratch buffers are the caller's, as
 *    XLA owns the scratch outputs of TkBwdBwd.
 *  - A returned FH_OK means the work was enqueued. Device-side failures (a
 *    bounded wait that expired) are reported by fh_device_status().
 *  - Re-entrant: the per-device one-time set-up is guarded by a mutex (the
 *    reference handler uses an unsynchronised static flag, ffi.cu:41-46).
 */
#ifndef FLASH_HOG_B200_H_
#define FLASH_HOG_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. 1 and 3 correspond to ffi::Error::InvalidArgument and
 * ffi::Error::Internal of the reference handler (ffi.cu:36-39, 74-76). */
enum fh_status {
  FH_OK = 0,
  FH_ERR_INVALID_ARGUMENT = 1,
  FH_ERR_UNSUPPORTED = 2,
  FH_ERR_LAUNCH = 3,
  FH_ERR_DEVICE = 4,
  FH_ERR_INJECTED = 5,
  FH_ERR_NO_DEVICE = 6
};

/* Element strides of a (batch, seq, head, head_dim) tensor; head_dim stride is 1. */
typedef struct fh_strides {
  int64_t batch;
  int64_t seq;
  int64_t head;
} fh_strides;

typedef struct fh_attn_dims {
  int32_t batch;
  int32_t heads;
  int32_t seq_q;
  int32_t seq_k;
  int32_t head_dim;
  fh_strides q; /* Q, O, dO, ddQ and the query-side outputs dQ, dQ', ddO */
  fh_strides k; /* K, V, ddK, ddV and the key-side outputs dK, dV, dK', dV' */
  /* Key/value heads for grouped-query attention: 0 (= heads) or a divisor of
   * heads; query head n attends with key/value head n / (heads / kv_heads), the
   * reference's "(kv_heads group)" grouping (flash_hog/jax/_pallas_gpu_kernel.py:106-107). */
  int32_t kv_heads;
  /* Sliding-window length of a causal mask (0 = unlimited): query i sees keys j
   * with diag_i - W < j <= diag_i, where diag_i = i (causal = 1) or
   * i + seq_k - seq_q (causal = 2) -- get_mask_bottom_right's
   * (qi >= kj) & (qi - kj < sliding_window_length), flash_hog/_jax_refs/jax_impl.py:104-109. */
  int32_t window;
  /* Packed variable-length batches (bf16 entry points; NULL = a dense batch).
   * With cu_seqlens_q and cu_seqlens_k set (device arrays of batch + 1
   * non-decreasing int32 offsets, first 0), sequence b is query rows
   * [cu_seqlens_q[b], cu_seqlens_q[b+1]) and key rows [cu_seqlens_k[b],
   * cu_seqlens_k[b+1]) of packed tensors with one batch entry:
   *  - seq_q / seq_k are the packed row counts (total tokens) and the strides'
   *    batch members are ignored;
   *  - max_seqlen_q / max_seqlen_k bound every sequence's lengths (they size
   *    the grids; rows of a longer sequence past them are not written);
   *  - per-query vectors (lse, delta, dd, bvec) are (heads, seq_q), i.e. (1,
   *    heads, total rows);
   *  - each sequence is masked on its own: causal = 2 aligns each sequence's
   *    diagonal bottom-right (query i sees keys j <= i + Tk_b - Tq_b), the
   *    window applies per sequence, and a sequence with no keys gets o = 0,
   *    lse = -inf and zero gradients.
   * The reference's JAX statements give each (qs, ks) pair its own bottom-right
   * mask (flash_hog/_jax_refs/jax_impl.py:104-130); this packs such pairs into
   * one call. The fp32 entry points reject packed batches. */
  const int32_t* cu_seqlens_q;
  const int32_t* cu_seqlens_k;
  int32_t max_seqlen_q;
  int32_t max_seqlen_k;
} fh_attn_dims;

/* Forward: o = softmax(scale * q k^T + mask) v, lse = logsumexp(scale * q k^T + mask).
 * Replaces the cuDNN forward with residuals, flash_hog/jax/_attention_impl.py:224-239
 * (`cuda_dot_product_attention(..., return_residual=True)`). */
int fh_attn_fwd(void* stream, const fh_attn_dims* dims, const void* q, const void* k, const void* v, void* o,
                float* lse, float scale, int causal);

/* D = rowsum(dO * o) per query row, fp32 (batch, head, seq_q).
 * Replaces the XLA einsum of flash_hog/jax/_tk_gpu.py:93 and
 * flash_hog/jax/_pallas_gpu_kernel.py:110. */
int fh_attn_rowdot(void* stream, const fh_attn_dims* dims, const void* o, const void* dO, float* delta);

/* First-order backward: dq, dk, dv from (q, k, v, o, dO, lse). `delta` is
 * caller scratch of batch*heads*seq_q floats (receives rowsum(dO * o)).
 * Replaces the cuDNN backward, flash_hog/jax/_attention_impl.py:242-261. */
int fh_attn_bwd(void* stream, const fh_attn_dims* dims, const void* q, const void* k, const void* v, const void* o,
                const void* dO, const float* lse, void* dq, void* dk, void* dv, float* delta, float scale,
                int causal);

/* Double backward: given the first-order residuals (q, k, v, dO, lse, delta) and
 * the cotangents (ddq, ddk, ddv) of (dq, dk, dv), computes
 *   dq2 = d<(dq,dk,dv),(ddq,ddk,ddv)>/dq, dk2 (/dk), dv2 (/dv), ddo (/dO).
 * `delta` = rowsum(dO * o) (fh_attn_rowdot). `dd` and `bvec` are caller
 * scratch of batch*heads*seq_q floats each; on return they hold the row
 * statistics dD = rowsum(ddS * P) and B = rowsum(dP2 * P).
 * Same buffers, order and meaning as TkBwdBwd (flash_hog/csrc/tk_bwdbwd/ffi.cu:79-98:
 * Q,K,V,dO,ddQ,ddK,ddV,L,D -> dQ2,ddO,dK2,dV2,dD,B; attribute scale), plus the
 * mask flag and the non-causal, cross-length and strided cases of the Pallas
 * rule flash_hog/jax/_pallas_gpu_kernel.py:49-422. */
int fh_attn_bwdbwd(void* stream, const fh_attn_dims* dims, const void* q, const void* k, const void* v,
                   const void* dO, const void* ddq, const void* ddk, const void* ddv, const float* lse,
                   const float* delta, void* dq2, void* ddo, void* dk2, void* dv2, float* dd, float* bvec,
                   float scale, int causal);

/* One pass of fh_attn_bwdbwd, same arguments plus `pass`:
 *   FH_PASS_QUERY (1): the query-tiled pass -- writes dq2, ddo, dd, bvec
 *                      (dk2, dv2 unused, may be NULL);
 *   FH_PASS_KEY   (2): the key-tiled pass -- reads dd, bvec, writes dk2, dv2
 *                      (dq2, ddo unused, may be NULL);
 *   3: both, identical to fh_attn_bwdbwd.
 * The reference runs the same two stages as separate kernels and times them
 * separately (flash_hog/csrc/tk_bwdbwd/ffi.cu:71-73, BENCHMARKS.md:45-46); this
 * entry lets a caller schedule or time them one at a time. */
enum fh_bwdbwd_pass { FH_PASS_QUERY = 1, FH_PASS_KEY = 2, FH_PASS_FWD_TANGENT = 4 };
int fh_attn_bwdbwd_pass(void* stream, const fh_attn_dims* dims, const void* q, const void* k, const void* v,
                        const void* dO, const void* ddq, const void* ddk, const void* ddv, const float* lse,
                        const float* delta, void* dq2, void* ddo, void* dk2, void* dv2, float* dd, float* bvec,
                        float scale, int causal, int pass);

/* Double backward from the forward output o instead of a precomputed delta:
 * the query-tiled pass computes D = rowsum(dO * o) for its rows itself and
 * writes it to `delta` (caller scratch of batch*heads*seq_q floats), which the
 * key-tiled pass reads -- one kernel launch fewer than fh_attn_rowdot followed
 * by fh_attn_bwdbwd, same results up to the summation order of D.
 * Replaces the reference's flash_bwdbwd (flash_hog/jax/_tk_gpu.py:83-103, which
 * computes D with an XLA einsum at _tk_gpu.py:93 before calling TkBwdBwd;
 * the Pallas rule does the same at _pallas_gpu_kernel.py:110).
 * `passes`: FH_PASS_QUERY, FH_PASS_KEY (after a query pass on the same
 * buffers) or both (3).
 * Forward tangent: `passes` = FH_PASS_FWD_TANGENT with (ddq, ddk, ddv) =
 * (tq, tk, tv) runs the query pass for dO = 0 and writes the jvp of the forward,
 * to = d O into `ddo` and tlse = d lse into `dd`. It skips the products that vanish
 * at dO = 0 (8 of the pass's 14 GEMM-equivalents per pair remain); o, dO, dq2,
 * delta and bvec are neither read nor written (may be NULL). FH_PASS_QUERY with a
 * zero-filled dO gives the same result to within rounding. */
int fh_attn_bwdbwd_o(void* stream, const fh_attn_dims* dims, const void* q, const void* k, const void* v,
                     const void* o, const void* dO, const void* ddq, const void* ddk, const void* ddv,
                     const float* lse, void* dq2, void* ddo, void* dk2, void* dv2, float* delta, float* dd,
                     float* bvec, float scale, int causal, int passes);

/* Forward-mode derivative (jvp) of the first-order backward. No counterpart in
 * the reference, which differentiates the backward in reverse mode only
 * (flash_hog/jax/attention.py:100-130); this is the forward-over-reverse path
 * of Hessian-vector products. The backward (dq, dk, dv) = grad_{q,k,v} <O, dO>
 * is the gradient of phi = <O(q, k, v), dO>, so its jvp with tangents
 * (tq, tk, tv, tdO) is
 *   (tdq, tdk, tdv) = Hess(phi) (tq, tk, tv) + J_O^T tdO:
 * the double backward with (ddq, ddk, ddv) = (tq, tk, tv) (a Hessian is
 * symmetric, so its vjp is its jvp) plus the first-order backward of tdO, whose
 * kernels add their results in place. The double backward's ddO output is the
 * forward tangent of the attention output, returned in `to`.
 *  - Inputs as for fh_attn_bwdbwd_o (q, k, v, o, dO, lse) plus the tangents
 *    tq (query side), tk, tv (key side) and tdO (query side; NULL = zero).
 *  - Outputs tdq, tdk, tdv, to. Scratch delta, dd, bvec: batch*heads*seq_q floats each.
 *  - Two kernel launches, four with tdO. */
int fh_attn_jvp_bwd(void* stream, const fh_attn_dims* dims, const void* q, const void* k, const void* v,
                    const void* o, const void* dO, const float* lse, const void* tq, const void* tk, const void* tv,
                    const void* tdO, void* tdq, void* tdk, void* tdv, void* to, float* delta, float* dd, float* bvec,
                    float scale, int causal);

/* Allocation-free double backward. No counterpart in the reference: it exists
 * for callers that cannot allocate device memory while they run -- an XLA FFI
 * handler only gets the buffers XLA assigned up front (and JAX reserves most of
 * the GPU for its own pool), and servers that reserve their whole memory budget
 * at start-up never allocate per request. Such a caller still passes the inputs
 * (q, k, v, o, dO, ddq, ddk, ddv, lse) and outputs (dq2, ddo, dk2, dv2) as for
 * fh_attn_bwdbwd_o, but no scratch: D = rowsum(dO * o), dD and B live in a
 * 6 MiB static device array inside the library (3 x 2^19 floats). Two kernel
 * launches, the same kernels as fh_attn_bwdbwd_o, and bit-identical results.
 *  - Limit: batch * heads * seq_q <= 524288 query rows; larger problems get
 *    FH_ERR_INVALID_ARGUMENT (see fh_last_error()) -- use fh_attn_bwdbwd_o.
 *  - It never calls cudaMalloc/cudaFree or any allocating routine. The first
 *    call on each device looks up the array's device address
 *    (cudaGetSymbolAddress, once per device); make that first call before any
 *    stream capture.
 *  - Memory still appears once per device: with CUDA's lazy module loading (the
 *    default), the first call on a device makes the driver load this library's
 *    module there, which reserves the 6 MiB array and the kernel code at that
 *    moment. A caller whose device memory is spoken for later (a JAX process
 *    before it reserves its pool) should make one small call at start-up.
 *  - Every call shares the one array and leaves its contents behind. Nothing in
 *    it needs to start at zero (each call writes all it reads before reading
 *    it), but calls whose GPU work overlaps (different streams, no ordering
 *    between them) race on it.
 *  - The array is held by every GPU on which the library's module is loaded,
 *    until the process exits.
 *  - device_status: optional (may be NULL) caller-owned, zeroed device int in
 *    which the kernels record a device-side error code (fh_device_status() reads
 *    the library's own word, which this entry point does not use). */
int fh_attn_bwdbwd_noalloc(void* stream, const fh_attn_dims* dims, const void* q, const void* k, const void* v,
                           const void* o, const void* dO, const void* ddq, const void* ddk, const void* ddv,
                           const float* lse, void* dq2, void* ddo, void* dk2, void* dv2, float scale, int causal,
                           int* device_status);

/* fp32 operands. The entry points above take bf16 tensors and compute their
 * products on the tensor cores with bf16 operands. The reference also accepts
 * fp32 inputs and then keeps them in fp32: its Pallas double backward casts
 * each score-like operand to the dtype of the tensor it multiplies
 * (flash_hog/jax/_pallas_gpu_kernel.py:251-256), and its XLA reference
 * differentiates fp32 attention twice (flash_hog/_jax_refs/jax_impl.py:194-247).
 * These four entry points do the same with fp32 products and fp32 accumulation
 * on the CUDA cores, for results within 1e-3 of an fp32/fp64 reference. Same
 * dims, masks, GQA mapping, strides, scratch and outputs as their bf16
 * counterparts; all tensors are fp32. There are no device-side waits, so
 * fh_device_status() has nothing to report for them.
 *  - fh_attn_fwd_f32: as fh_attn_fwd.
 *  - fh_attn_bwd_f32: as fh_attn_bwd (delta receives rowsum(dO * o)).
 *  - fh_attn_bwdbwd_f32: as fh_attn_bwdbwd_o, including `passes` and the
 *    forward-tangent use; dq2 may be NULL for a query pass.
 *  - fh_attn_jvp_bwd_f32: as fh_attn_jvp_bwd. */
int fh_attn_fwd_f32(void* stream, const fh_attn_dims* dims, const float* q, const float* k, const float* v,
                    float* o, float* lse, float scale, int causal);
int fh_attn_bwd_f32(void* stream, const fh_attn_dims* dims, const float* q, const float* k, const float* v,
                    const float* o, const float* dO, const float* lse, float* dq, float* dk, float* dv, float* delta,
                    float scale, int causal);
int fh_attn_bwdbwd_f32(void* stream, const fh_attn_dims* dims, const float* q, const float* k, const float* v,
                       const float* o, const float* dO, const float* ddq, const float* ddk, const float* ddv,
                       const float* lse, float* dq2, float* ddo, float* dk2, float* dv2, float* delta, float* dd,
                       float* bvec, float scale, int causal, int passes);
int fh_attn_jvp_bwd_f32(void* stream, const fh_attn_dims* dims, const float* q, const float* k, const float* v,
                        const float* o, const float* dO, const float* lse, const float* tq, const float* tk,
                        const float* tv, const float* tdO, float* tdq, float* tdk, float* tdv, float* to,
                        float* delta, float* dd, float* bvec, float scale, int causal);

/* LayerNorm and GELU of the grad-norm-penalty training step (the model step of
 * configuration 5: L + lam ||dL/dtheta||^2 differentiates every layer's backward).
 * No counterpart in the reference, which has no model code (its hot path is the
 * attention op alone). Each pass is one kernel over the rows (LayerNorm weight
 * gradients add one deterministic column reduction), so a second-order step does
 * not run the dozens of elementwise kernels a framework composes these gradients
 * from.
 *  - LayerNorm over the last dimension of a (rows, cols) fp32 row-major tensor,
 *    cols a multiple of 4 in [4, 1024]; eps inside the square root.
 *    fh_layernorm_fwd: y = (x - mean) rstd w + b; mean, rstd per row (rows floats).
 *    fh_layernorm_bwd: dx, dw = sum_rows dy xhat, db = sum_rows dy.
 *    fh_layernorm_bwd_bwd: the gradient of <ddx, dx> + <ddw, dw> + <ddb, db>
 *      w.r.t. x (gx), w (gw) and dy (gdy); ddx, ddw, ddb may be NULL (zero).
 *    `scratch`: fh_layernorm_scratch_floats(rows, cols) floats (per-block column
 *    partials of the weight gradients), on the current device.
 *  - fh_gelu: exact GELU x Phi(x) over n elements, dtype 0 = fp32, 1 = bf16
 *    (fp32 arithmetic either way). mode 0: out0 = gelu(a); mode 1: out0 =
 *    dh gelu'(a); mode 2 (the backward's backward, given the cotangent c of its
 *    output): out0 = c gelu'(a) (w.r.t. dh), out1 = c dh gelu''(a) (w.r.t. a;
 *    dh NULL = zero, out1 NULL = not computed). */
long long fh_layernorm_scratch_floats(int rows, int cols);
int fh_layernorm_fwd(void* stream, int rows, int cols, const float* x, const float* w, const float* b, float eps,
                     float* y, float* mean, float* rstd);
int fh_layernorm_bwd(void* stream, int rows, int cols, const float* x, const float* w, const float* mean,
                     const float* rstd, const float* dy, float* dx, float* dw, float* db, float* scratch);
int fh_layernorm_bwd_bwd(void* stream, int rows, int cols, const float* x, const float* w, const float* mean,
                         const float* rstd, const float* dy, const float* ddx, const float* ddw, const float* ddb,
                         float* gx, float* gw, float* gdy, float* scratch);
int fh_gelu(void* stream, int mode, int dtype, long long n, const void* a, const void* dh, const void* c, void* out0,
            void* out1);

/* Cross entropy of the same step's language-model head (no counterpart in the
 * reference either). Logits z are `rows` rows of `vocab` elements, dtype 0 = fp32,
 * 1 = bf16, row stride `ld` elements (>= vocab); targets t are int64 in [0, vocab)
 * (one outside gives a NaN loss and no one-hot term). One kernel per pass, one CTA
 * per row; all outputs are contiguous, fp32 vectors have `rows` entries.
 *  - fh_xent_fwd: lse[r] = log sum_v exp(z[r,v]), loss[r] = lse[r] - z[r,t[r]].
 *  - fh_xent_bwd: dz = g s (softmax(z) - onehot(t)), in z's dtype; g points to the
 *    fp32 upstream scalar (device memory), s is a host scale (1/rows for a mean).
 *  - fh_xent_bwd_bwd: given the cotangent u of dz (z's dtype, contiguous):
 *    gz = g s p (u - <p, u>_row) with p = softmax(z) (z's dtype), and
 *    gg[r] = s (<p_r, u_r> - u[r,t[r]]), whose sum is the cotangent of g. */
int fh_xent_fwd(void* stream, int dtype, int rows, int vocab, long long ld, const void* z, const long long* t,
                float* lse, float* loss);
int fh_xent_bwd(void* stream, int dtype, int rows, int vocab, long long ld, const void* z, const long long* t,
                const float* lse, const float* g, float s, void* dz);
int fh_xent_bwd_bwd(void* stream, int dtype, int rows, int vocab, long long ld, const void* z, const long long* t,
                    const float* lse, const float* g, float s, const void* u, void* gz, float* gg);

/* Synchronises `stream`, then reads and clears the status word the kernels of
 * the current device record device-side failures in. *code receives 0 or one
 * of the device error codes (1..5: which bounded wait expired). Returns FH_OK,
 * or FH_ERR_DEVICE when *code != 0. */
int fh_device_status(void* stream, int* code);

/* Detail message of the last non-FH_OK status returned on this thread by an
 * entry point (empty if none). The reference handler carries such text in
 * ffi::Error (ffi.cu:36-39, 74-76). */
const char* fh_last_error(void);

/* Human-readable name of an fh_status value. */
const char* fh_status_string(int status);

/* ABI version of this header (bumped on any signature change). */
int fh_abi_version(void);

/* Number of kernels this library has launched in the process so far (all
 * devices, every entry point). No counterpart in the reference; a benchmark
 * reads it before and after a timed region to report its kernel launches. */
unsigned long long fh_launch_count(void);

#define FH_ABI_VERSION 8

#ifdef __cplusplus
}
#endif

#endif /* FLASH_HOG_B200_H_ */
