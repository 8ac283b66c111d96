// Internal launch interface between the C ABI (capi.cu) and the kernels.

#pragma once

#include <cuda_runtime.h>

#include "attn_common.cuh"

namespace fh {

// Return codes shared with include/flash_hog_b200.h.
enum HostStatus : int {
  kOk = 0,
  kInvalidArgument = 1,
  kUnsupported = 2,
  kLaunchFailed = 3,
  kDeviceError = 4,
  kInjected = 5,
  kNoDevice = 6,
};

struct FwdPtrs {
  const void *q, *k, *v;
  void* o;
  float* lse;
};

struct BwdPtrs {
  const void *q, *k, *v, *o, *dO;
  const float* lse;
  void *dq, *dk, *dv;
  float* delta;  // scratch: rowsum(dO * O), written by the first kernel
  // Optional addends (same layout as dq, dk, dv; may alias them): the outputs
  // become dq_acc + dQ, ... -- how the forward-mode derivative of the backward
  // adds its first-order term to the double-backward term.
  const void* dq_acc = nullptr;
  const void* dk_acc = nullptr;
  const void* dv_acc = nullptr;
};

struct BwdBwdPtrs {
  const void *q, *k, *v, *dO, *ddq, *ddk, *ddv;
  const float *lse, *delta;
  void *dq2, *ddo, *dk2, *dv2;
  float *dd, *bv;  // scratch written by the query-tiled pass, read by the key-tiled pass
  // Optional: with `o` set, D = rowsum(dO o) is computed by the query-tiled pass
  // into `delta_out` (which the key-tiled pass then reads) and `delta` is unused.
  const void* o = nullptr;
  float* delta_out = nullptr;
};

int launch_fwd(const AttnShape& s, int hd, const FwdPtrs& p, int* status, cudaStream_t stream);
int launch_rowdot(const AttnShape& s, int hd, const void* o, const void* dO, float* delta, cudaStream_t stream);
int launch_bwd(const AttnShape& s, int hd, const BwdPtrs& p, int* status, cudaStream_t stream);
// passes: bitmask of kPassQuery (query-tiled: dQ', ddO, dD, B) and kPassKey (key-tiled: dK', dV'),
// or kPassFwdTangent alone: the query-tiled pass for dO = 0 (ddO = the forward's tangent,
// dD = the log-sum-exp's tangent; dO, O, delta, dq2 and bv are neither read nor written).
enum BwdBwdPass : int { kPassQuery = 1, kPassKey = 2, kPassFwdTangent = 4 };
int launch_bwdbwd(const AttnShape& s, int hd, const BwdBwdPtrs& p, int passes, int* status, cudaStream_t stream);

// fp32 operands on the CUDA cores (f32.cu): same passes, masks, GQA mapping and
// layouts as the bf16 kernels; `delta` is written by a rowdot kernel (forward
// output `o` and `dO`) whenever a pass needs D. No device waits, so no status word.
struct F32FwdPtrs {
  const float *q, *k, *v;
  float *o, *lse;
};

struct F32BwdPtrs {
  const float *q, *k, *v, *o, *dO, *lse;
  float *dq, *dk, *dv, *delta;
  const float* dq_acc = nullptr;  // optional addends, as in BwdPtrs
  const float* dk_acc = nullptr;
  const float* dv_acc = nullptr;
};

struct F32BwdBwdPtrs {
  const float *q, *k, *v, *o, *dO, *ddq, *ddk, *ddv, *lse;
  float *delta;               // written by the query pass, read by the key pass
  float *dq2, *ddo, *dk2, *dv2;  // dq2 may be null (query pass: ddO only)
  float *dd, *bv;
};

int launch_fwd_f32(const AttnShape& s, int hd, const F32FwdPtrs& p, cudaStream_t stream);
int launch_bwd_f32(const AttnShape& s, int hd, const F32BwdPtrs& p, cudaStream_t stream);
int launch_bwdbwd_f32(const AttnShape& s, int hd, const F32BwdBwdPtrs& p, int passes, cudaStream_t stream);

// LayerNorm over rows of `cols` fp32 values and its backward / double backward
// (ln_gelu.cu). op 0: forward (out0 = y, out1 = mean, out2 = rstd); op 1: backward
// (out0 = dx, out1 = dw, out2 = db); op 2: double backward with cotangents u, vb, cb
// of (dx, dw, db), any of them null = zero (out0 = grad x, out1 = grad dy,
// out2 = grad w). `part` is scratch of ln_partials_rows(rows) * 2 * cols floats
// (ops 1 and 2).
int launch_layernorm(int op, int rows, int cols, const float* x, const float* w, const float* b, const float* mean,
                     const float* rstd, const float* dy, const float* u, const float* vb, const float* cb, float eps,
                     float* out0, float* out1, float* out2, float* part, cudaStream_t stream);
int ln_partials_rows(int rows);
// Exact GELU over n elements (fp32 or bf16): mode 0 out0 = gelu(a); mode 1 out0 =
// dh gelu'(a); mode 2 out0 = c gelu'(a), out1 = c dh gelu''(a) (dh null = zero).
int launch_gelu(int mode, bool bf16, long long n, const void* a, const void* dh, const void* c, void* out0, void* out1,
                cudaStream_t stream);
// Cross entropy over (rows, vocab) logits: op 0 forward (lse, loss), 1 backward
// (out = dz), 2 backward's backward (u = cotangent of dz; out = gz, gg per row).
// `lse` is written by op 0 and read by ops 1 and 2.
int launch_xent(int op, bool bf16, int rows, int vocab, long long ld, const void* z, const long long* t, float* lse,
                float* loss, const float* g, float s, const void* u, void* out, float* gg, cudaStream_t stream);

// Checks the kernel launch just made (cudaGetLastError) and, if it was queued,
// counts it for fh_launch_count(). Returns kOk or kLaunchFailed.
int after_launch();

// Streaming multiprocessors of the current device (cached per device): the
// grid size of the persistent kernels.
int sm_count();

// Sets the dynamic shared memory limit of `func` on the current device once.
int ensure_smem_limit(const void* func, int bytes);

// Batch extent of the tensors' TMA maps: the batch for dense inputs, 1 for packed
// variable-length ones (whose sequences are row ranges of one batch entry).
inline int map_batch(const AttnShape& s) { return s.cu_q ? 1 : s.B; }

// 4-D (head_dim, seq, head, batch) bf16 map with a {64, rows, 1, 1} box.
bool make_seq_map(CUtensorMap* map, const void* base, int hd, int seq, int heads, int batch, const Strides3& st,
                  int rows);

}  // namespace fh
