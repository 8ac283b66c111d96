// C ABI entry points (include/flash_hog_b200.h): argument validation, device
// selection from the stream, per-device one-time set-up, host-side fault
// injection, and dispatch to the kernel launchers.

#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

#include "flash_hog_b200.h"
#include "kernels.h"
#include "tmap.h"

namespace fh {

namespace {

constexpr int kMaxDevices = 64;

std::mutex g_mutex;
thread_local char g_last_error[256] = "";

// Records a detail message for fh_last_error() and returns `code`.
int fail(int code, const char* what) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", what);
  return code;
}
int* g_status_word[kMaxDevices] = {nullptr};
std::set<std::pair<int, const void*>> g_smem_done;

int current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

// Makes the stream's device current *and* binds its primary context to the
// calling thread. Callers such as autograd worker threads may have a current
// device in their own CUDA runtime without a driver context bound to the
// thread; TMA descriptor encoding needs one (else CUDA_ERROR_INVALID_CONTEXT).
// A stream that is being captured into a CUDA graph is not queried (a query can
// invalidate the capture); it belongs to the current device, as during capture
// the capturing thread has that device current.
int select_stream_device(cudaStream_t stream) {
  int dev = current_device();
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  bool query = stream != nullptr;
  if (query && cudaStreamIsCapturing(stream, &capture) != cudaSuccess) {
    cudaGetLastError();  // not a launch failure: leave no error for after_launch() to find
    query = false;
  }
  if (query && capture == cudaStreamCaptureStatusNone) {
    int sdev = -1;
    if (cudaStreamGetDevice(stream, &sdev) == cudaSuccess) {
      dev = sdev;
    } else {
      // Follow the CUDA convention that the stream belongs to the current device.
      cudaGetLastError();
    }
  }
  if (dev < 0) return fail(kNoDevice, "no current CUDA device");
  if (cudaSetDevice(dev) != cudaSuccess) return fail(kNoDevice, "cudaSetDevice failed");
  return kOk;
}

// Per-device status word (allocated once, zeroed).
int* status_word() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_status_word[dev]) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return nullptr;
    g_status_word[dev] = p;
  }
  return g_status_word[dev];
}

// FLASH_HOG_B200_INJECT_ERROR=<entry>[,<entry>...] or "all": the named entry
// points return FH_ERR_INJECTED without launching anything. Host-side fault
// injection for the callers' error paths; nothing reaches the GPU.
bool injected(const char* entry) {
  const char* env = std::getenv("FLASH_HOG_B200_INJECT_ERROR");
  if (!env || !*env) return false;
  if (std::strcmp(env, "all") == 0) return true;
  const size_t n = std::strlen(entry);
  for (const char* p = env; *p;) {
    const char* e = std::strchr(p, ',');
    const size_t len = e ? static_cast<size_t>(e - p) : std::strlen(p);
    if (len == n && std::strncmp(p, entry, n) == 0) return true;
    if (!e) break;
    p = e + 1;
  }
  return false;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool strides_ok(const fh_strides& s) {
  return s.batch >= 0 && s.seq > 0 && s.head >= 0 && s.batch % 8 == 0 && s.seq % 8 == 0 && s.head % 8 == 0;
}

int validate(const fh_attn_dims* d, AttnShape* out, float scale, int causal, bool allow_varlen = true) {
  g_last_error[0] = 0;
  if (!d) return fail(kInvalidArgument, "dims is NULL");
  const bool varlen = d->cu_seqlens_q != nullptr || d->cu_seqlens_k != nullptr;
  if (varlen && !allow_varlen) return fail(kUnsupported, "packed variable-length batches need the bf16 entry points");
  if (varlen && (!d->cu_seqlens_q || !d->cu_seqlens_k))
    return fail(kInvalidArgument, "a packed batch needs both cu_seqlens_q and cu_seqlens_k");
  if (varlen && ((reinterpret_cast<uintptr_t>(d->cu_seqlens_q) | reinterpret_cast<uintptr_t>(d->cu_seqlens_k)) & 3u))
    return fail(kInvalidArgument, "cu_seqlens arrays must be 4-byte aligned");
  if (varlen && (d->max_seqlen_q < 1 || d->max_seqlen_k < 1 || d->max_seqlen_q > d->seq_q ||
                 d->max_seqlen_k > d->seq_k))
    return fail(kInvalidArgument, "max_seqlen_q/k must be in [1, seq_q/k] (seq_q/k: packed rows)");
  if (d->batch < 1 || d->heads < 1 || d->seq_q < 1 || d->seq_k < 1)
    return fail(kInvalidArgument, "batch, heads, seq_q and seq_k must be >= 1");
  if (d->head_dim != 64 && d->head_dim != 128) return fail(kUnsupported, "head_dim must be 64 or 128");
  if (!strides_ok(d->q) || !strides_ok(d->k))
    return fail(kInvalidArgument, "strides must be non-negative multiples of 8 elements (seq stride > 0)");
  if (!(scale == scale)) return fail(kInvalidArgument, "scale is NaN");
  const int kv = d->kv_heads ? d->kv_heads : d->heads;
  if (kv < 1 || d->heads % kv != 0) return fail(kInvalidArgument, "heads must be a multiple of kv_heads");
  out->B = d->batch;
  out->H = d->heads;
  out->Hk = kv;
  out->G = d->heads / kv;
  out->Tq = d->seq_q;
  out->Tk = d->seq_k;
  out->sq = Strides3{varlen ? 0 : d->q.batch, d->q.seq, d->q.head};
  out->sk = Strides3{varlen ? 0 : d->k.batch, d->k.seq, d->k.head};
  if (causal < 0 || causal > 2)
    return fail(kInvalidArgument, "causal must be 0 (no mask), 1 (top-left) or 2 (bottom-right)");
  if (d->window < 0) return fail(kInvalidArgument, "window must be >= 0");
  if (d->window > 0 && !causal) return fail(kInvalidArgument, "a sliding window needs a causal mask");
  out->scale = scale;
  out->causal = causal ? 1 : 0;
  out->br = causal == 2 ? 1 : 0;
  out->window = d->window;
  out->total_q = d->seq_q;
  out->total_k = d->seq_k;
  if (varlen) {
    // Sequences are row ranges of one batch entry; each kernel derives its
    // sequence's lengths and diagonal (seq_shape). Tq/Tk size the grids.
    out->cu_q = d->cu_seqlens_q;
    out->cu_k = d->cu_seqlens_k;
    out->Tq = d->max_seqlen_q;
    out->Tk = d->max_seqlen_k;
    out->diag = 0;
  } else {
    out->cu_q = out->cu_k = nullptr;
    out->diag = causal == 2 ? d->seq_k - d->seq_q : 0;
  }
  return kOk;
}

constexpr const char* kAlignMsg = "a tensor pointer is NULL or not 16-byte aligned";

template <typename... P>
bool all_aligned(P... ptrs) {
  return (... && (ptrs != nullptr && aligned16(ptrs)));
}

}  // namespace

std::atomic<unsigned long long> g_launches{0};
std::atomic<int> g_sm_count[kMaxDevices];

int sm_count() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 1;
  int n = g_sm_count[dev].load(std::memory_order_relaxed);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 1;
    g_sm_count[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

int after_launch() {
  if (cudaGetLastError() != cudaSuccess) return kLaunchFailed;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return kOk;
}

int ensure_smem_limit(const void* func, int bytes) {
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(g_mutex);
  auto key = std::make_pair(dev, func);
  if (g_smem_done.count(key)) return kOk;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
    return fail(kLaunchFailed, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize) failed");
  g_smem_done.insert(key);
  return kOk;
}

bool make_seq_map(CUtensorMap* map, const void* base, int hd, int seq, int heads, int batch, const Strides3& st,
                  int rows) {
  const uint64_t dims[4] = {static_cast<uint64_t>(hd), static_cast<uint64_t>(seq), static_cast<uint64_t>(heads),
                            static_cast<uint64_t>(batch)};
  // Size-1 dimensions may carry any stride; give them a legal one.
  const uint64_t sb = st.b > 0 ? st.b : 8, sh = st.h > 0 ? st.h : 8;
  const uint64_t strides[3] = {static_cast<uint64_t>(st.t) * 2, sh * 2, sb * 2};
  const uint32_t box[4] = {64, static_cast<uint32_t>(rows), 1, 1};
  int cu = 0;
  if (make_tmap_bf16(map, base, 4, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, &cu)) return true;
  char msg[240];
  std::snprintf(msg, sizeof(msg),
                "cuTensorMapEncodeTiled failed (CUresult %d) for base %p dims {%llu,%llu,%llu,%llu} "
                "strides {%llu,%llu,%llu} box rows %d",
                cu, base, (unsigned long long)dims[0], (unsigned long long)dims[1], (unsigned long long)dims[2],
                (unsigned long long)dims[3], (unsigned long long)strides[0], (unsigned long long)strides[1],
                (unsigned long long)strides[2], rows);
  fail(kInvalidArgument, msg);
  return false;
}

}  // namespace fh

using namespace fh;

extern "C" {

int fh_abi_version(void) { return FH_ABI_VERSION; }

unsigned long long fh_launch_count(void) { return fh::g_launches.load(std::memory_order_relaxed); }

const char* fh_last_error(void) { return g_last_error; }

const char* fh_status_string(int status) {
  switch (status) {
    case FH_OK: return "ok";
    case FH_ERR_INVALID_ARGUMENT: return "invalid argument";
    case FH_ERR_UNSUPPORTED: return "unsupported configuration";
    case FH_ERR_LAUNCH: return "kernel launch failed";
    case FH_ERR_DEVICE: return "device-side error (bounded wait expired)";
    case FH_ERR_INJECTED: return "injected error";
    case FH_ERR_NO_DEVICE: return "no CUDA device";
    default: return "unknown status";
  }
}

int fh_attn_fwd(void* stream, const fh_attn_dims* dims, const void* q, const void* k, const void* v, void* o,
                float* lse, float scale, int causal) {
  if (injected("fh_attn_fwd")) return FH_ERR_INJECTED;
  AttnShape s;
  int rc = validate(dims, &s, scale, causal);
  if (rc != kOk) return rc;
  if (!all_aligned(q, k, v, o) || !lse) return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = select_stream_device(st)) != kOk) return rc;
  int* status = status_word();
  if (!status) return FH_ERR_NO_DEVICE;
  return launch_fwd(s, dims->head_dim, FwdPtrs{q, k, v, o, lse}, status, st);
}

int fh_attn_rowdot(void* stream, const fh_attn_dims* dims, const void* o, const void* dO, float* delta) {
  if (injected("fh_attn_rowdot")) return FH_ERR_INJECTED;
  AttnShape s;
  int rc = validate(dims, &s, 1.f, 0);
  if (rc != kOk) return rc;
  if (!all_aligned(o, dO) || !delta) return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = select_stream_device(st)) != kOk) return rc;
  return launch_rowdot(s, dims->head_dim, o, dO, delta, st);
}

int fh_attn_bwd(void* stream, const fh_attn_dims* dims, const void* q, const void* k, const void* v, const void* o,
                const void* dO, const float* lse, void* dq, void* dk, void* dv, float* delta, float scale,
                int causal) {
  if (injected("fh_attn_bwd")) return FH_ERR_INJECTED;
  AttnShape s;
  int rc = validate(dims, &s, scale, causal);
  if (rc != kOk) return rc;
  if (!all_aligned(q, k, v, o, dO, dq, dk, dv) || !lse || !delta) return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = select_stream_device(st)) != kOk) return rc;
  int* status = status_word();
  if (!status) return FH_ERR_NO_DEVICE;
  return launch_bwd(s, dims->head_dim, BwdPtrs{q, k, v, o, dO, lse, dq, dk, dv, delta}, status, st);
}

// `o` null: `delta` is an input. `o` set: the query pass computes D into
// `delta_out`, which the key pass reads.
static int bwdbwd_entry(const char* entry, void* stream, const fh_attn_dims* dims, const void* q, const void* k,
                        const void* v, const void* o, const void* dO, const void* ddq, const void* ddk,
                        const void* ddv, const float* lse, const float* delta, float* delta_out, void* dq2, void* ddo,
                        void* dk2, void* dv2, float* dd, float* bvec, float scale, int causal, int passes) {
  if (injected(entry)) return FH_ERR_INJECTED;
  AttnShape s;
  int rc = validate(dims, &s, scale, causal);
  if (rc != kOk) return rc;
  if (passes == kPassFwdTangent) {
    // dO = 0: only q, k, v, the tangents (ddq, ddk, ddv), lse and the outputs ddo, dd are used.
    if (!all_aligned(q, k, v, ddq, ddk, ddv, ddo) || !lse || !dd) return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((rc = select_stream_device(st)) != kOk) return rc;
    int* status = status_word();
    if (!status) return FH_ERR_NO_DEVICE;
    return launch_bwdbwd(
        s, dims->head_dim,
        BwdBwdPtrs{q, k, v, nullptr, ddq, ddk, ddv, lse, nullptr, nullptr, ddo, nullptr, nullptr, dd, nullptr},
        kPassFwdTangent, status, st);
  }
  if (passes < 1 || passes > 3) return fail(FH_ERR_INVALID_ARGUMENT, "pass must be 1, 2, 3 or 4 (forward tangent)");
  if (!all_aligned(q, k, v, dO, ddq, ddk, ddv) || !lse || !dd || !bvec)
    return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  if (o ? (!all_aligned(o) || !delta_out) : !delta) return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  if ((passes & kPassQuery) && !all_aligned(dq2, ddo)) return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  if ((passes & kPassKey) && !all_aligned(dk2, dv2)) return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = select_stream_device(st)) != kOk) return rc;
  int* status = status_word();
  if (!status) return FH_ERR_NO_DEVICE;
  return launch_bwdbwd(
      s, dims->head_dim,
      BwdBwdPtrs{q, k, v, dO, ddq, ddk, ddv, lse, delta, dq2, ddo, dk2, dv2, dd, bvec, o, delta_out}, passes,
      status, st);
}

int fh_attn_bwdbwd(void* stream, const fh_attn_dims* dims, const void* q, const void* k, const void* v,
                   const void* dO, const void* ddq, const void* ddk, const void* ddv, const float* lse,
                   const float* delta, void* dq2, void* ddo, void* dk2, void* dv2, float* dd, float* bvec,
                   float scale, int causal) {
  return bwdbwd_entry("fh_attn_bwdbwd", stream, dims, q, k, v, nullptr, dO, ddq, ddk, ddv, lse, delta, nullptr, dq2,
                      ddo, dk2, dv2, dd, bvec, scale, causal, kPassQuery | kPassKey);
}

int fh_attn_bwdbwd_pass(void* stream, const fh_attn_dims* dims, const void* q, const void* k, const void* v,
                        const void* dO, const void* ddq, const void* ddk, const void* ddv, const float* lse,
                        const float* delta, void* dq2, void* ddo, void* dk2, void* dv2, float* dd, float* bvec,
                        float scale, int causal, int pass) {
  return bwdbwd_entry("fh_attn_bwdbwd_pass", stream, dims, q, k, v, nullptr, dO, ddq, ddk, ddv, lse, delta, nullptr,
                      dq2, ddo, dk2, dv2, dd, bvec, scale, causal, pass);
}

int fh_attn_bwdbwd_o(void* stream, const fh_attn_dims* dims, const void* q, const void* k, const void* v,
                     const void* o, const void* dO, const void* ddq, const void* ddk, const void* ddv,
                     const float* lse, void* dq2, void* ddo, void* dk2, void* dv2, float* delta, float* dd,
                     float* bvec, float scale, int causal, int passes) {
  return bwdbwd_entry("fh_attn_bwdbwd_o", stream, dims, q, k, v, o, dO, ddq, ddk, ddv, lse, nullptr, delta, dq2, ddo,
                      dk2, dv2, dd, bvec, scale, causal, passes);
}

int fh_attn_jvp_bwd(void* stream, const fh_attn_dims* dims, const void* q, const void* k, const void* v,
                    const void* o, const void* dO, const float* lse, const void* tq, const void* tk, const void* tv,
                    const void* tdO, void* tdq, void* tdk, void* tdv, void* to, float* delta, float* dd, float* bvec,
                    float scale, int causal) {
  if (injected("fh_attn_jvp_bwd")) return FH_ERR_INJECTED;
  AttnShape s;
  int rc = validate(dims, &s, scale, causal);
  if (rc != kOk) return rc;
  if (!all_aligned(q, k, v, o, dO, tq, tk, tv, tdq, tdk, tdv, to) || !lse || !delta || !dd || !bvec)
    return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  if (tdO && !all_aligned(tdO)) return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = select_stream_device(st)) != kOk) return rc;
  int* status = status_word();
  if (!status) return FH_ERR_NO_DEVICE;
  // Hessian term: the double backward with (ddq, ddk, ddv) = (tq, tk, tv).
  rc = launch_bwdbwd(s, dims->head_dim,
                     BwdBwdPtrs{q, k, v, dO, tq, tk, tv, lse, nullptr, tdq, to, tdk, tdv, dd, bvec, o, delta},
                     kPassQuery | kPassKey, status, st);
  if (rc != kOk || !tdO) return rc;
  // Plus the first-order backward of the cotangent tangent tdO, added in place.
  BwdPtrs p{q, k, v, o, tdO, lse, tdq, tdk, tdv, delta};
  p.dq_acc = tdq;
  p.dk_acc = tdk;
  p.dv_acc = tdv;
  return launch_bwd(s, dims->head_dim, p, status, st);
}

int fh_attn_fwd_f32(void* stream, const fh_attn_dims* dims, const float* q, const float* k, const float* v,
                    float* o, float* lse, float scale, int causal) {
  if (injected("fh_attn_fwd_f32")) return FH_ERR_INJECTED;
  AttnShape s;
  int rc = validate(dims, &s, scale, causal, false);
  if (rc != kOk) return rc;
  if (!all_aligned(q, k, v, o) || !lse) return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = select_stream_device(st)) != kOk) return rc;
  return launch_fwd_f32(s, dims->head_dim, F32FwdPtrs{q, k, v, o, lse}, st);
}

int fh_attn_bwd_f32(void* stream, const fh_attn_dims* dims, const float* q, const float* k, const float* v,
                    const float* o, const float* dO, const float* lse, float* dq, float* dk, float* dv, float* delta,
                    float scale, int causal) {
  if (injected("fh_attn_bwd_f32")) return FH_ERR_INJECTED;
  AttnShape s;
  int rc = validate(dims, &s, scale, causal, false);
  if (rc != kOk) return rc;
  if (!all_aligned(q, k, v, o, dO, dq, dk, dv) || !lse || !delta) return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = select_stream_device(st)) != kOk) return rc;
  return launch_bwd_f32(s, dims->head_dim, F32BwdPtrs{q, k, v, o, dO, lse, dq, dk, dv, delta}, st);
}

int fh_attn_bwdbwd_f32(void* stream, const fh_attn_dims* dims, const float* q, const float* k, const float* v,
                       const float* o, const float* dO, const float* ddq, const float* ddk, const float* ddv,
                       const float* lse, float* dq2, float* ddo, float* dk2, float* dv2, float* delta, float* dd,
                       float* bvec, float scale, int causal, int passes) {
  if (injected("fh_attn_bwdbwd_f32")) return FH_ERR_INJECTED;
  AttnShape s;
  int rc = validate(dims, &s, scale, causal, false);
  if (rc != kOk) return rc;
  if (passes < 1 || passes > 3) return fail(FH_ERR_INVALID_ARGUMENT, "pass must be 1, 2 or 3");
  if (!all_aligned(q, k, v, dO, ddq, ddk, ddv) || !lse || !delta || !dd || !bvec)
    return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  if ((passes & kPassQuery) && (!all_aligned(o, ddo) || (dq2 && !aligned16(dq2))))
    return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  if ((passes & kPassKey) && !all_aligned(dk2, dv2)) return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = select_stream_device(st)) != kOk) return rc;
  return launch_bwdbwd_f32(s, dims->head_dim,
                           F32BwdBwdPtrs{q, k, v, o, dO, ddq, ddk, ddv, lse, delta, dq2, ddo, dk2, dv2, dd, bvec},
                           passes, st);
}

int fh_attn_jvp_bwd_f32(void* stream, const fh_attn_dims* dims, const float* q, const float* k, const float* v,
                        const float* o, const float* dO, const float* lse, const float* tq, const float* tk,
                        const float* tv, const float* tdO, float* tdq, float* tdk, float* tdv, float* to,
                        float* delta, float* dd, float* bvec, float scale, int causal) {
  if (injected("fh_attn_jvp_bwd_f32")) return FH_ERR_INJECTED;
  AttnShape s;
  int rc = validate(dims, &s, scale, causal, false);
  if (rc != kOk) return rc;
  if (!all_aligned(q, k, v, o, dO, tq, tk, tv, tdq, tdk, tdv, to) || !lse || !delta || !dd || !bvec)
    return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  if (tdO && !all_aligned(tdO)) return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = select_stream_device(st)) != kOk) return rc;
  rc = launch_bwdbwd_f32(s, dims->head_dim,
                         F32BwdBwdPtrs{q, k, v, o, dO, tq, tk, tv, lse, delta, tdq, to, tdk, tdv, dd, bvec},
                         kPassQuery | kPassKey, st);
  if (rc != kOk || !tdO) return rc;
  // The first-order backward of tdO reuses `delta` for rowsum(tdO * o).
  F32BwdPtrs p{q, k, v, o, tdO, lse, tdq, tdk, tdv, delta};
  p.dq_acc = tdq;
  p.dk_acc = tdk;
  p.dv_acc = tdv;
  return launch_bwd_f32(s, dims->head_dim, p, st);
}

// ------------------------------------------------------------------------------------
// LayerNorm and GELU of the grad-norm-penalty model step
// ------------------------------------------------------------------------------------

static int ln_check(int rows, int cols) {
  g_last_error[0] = 0;
  if (rows < 1 || cols < 4 || cols % 4 != 0 || cols > 1024)
    return fail(FH_ERR_UNSUPPORTED, "layernorm needs rows >= 1 and cols a multiple of 4 in [4, 1024]");
  return kOk;
}

long long fh_layernorm_scratch_floats(int rows, int cols) {
  if (ln_check(rows, cols) != kOk) return -1;
  return static_cast<long long>(ln_partials_rows(rows)) * 2 * cols;
}

int fh_layernorm_fwd(void* stream, int rows, int cols, const float* x, const float* w, const float* b, float eps,
                     float* y, float* mean, float* rstd) {
  if (injected("fh_layernorm_fwd")) return FH_ERR_INJECTED;
  int rc = ln_check(rows, cols);
  if (rc != kOk) return rc;
  if (!all_aligned(x, w, b, y) || !mean || !rstd) return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = select_stream_device(st)) != kOk) return rc;
  return launch_layernorm(0, rows, cols, x, w, b, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, eps, y, mean,
                          rstd, nullptr, st);
}

int fh_layernorm_bwd(void* stream, int rows, int cols, const float* x, const float* w, const float* mean,
                     const float* rstd, const float* dy, float* dx, float* dw, float* db, float* scratch) {
  if (injected("fh_layernorm_bwd")) return FH_ERR_INJECTED;
  int rc = ln_check(rows, cols);
  if (rc != kOk) return rc;
  if (!all_aligned(x, w, dy, dx, dw, db, scratch) || !mean || !rstd) return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = select_stream_device(st)) != kOk) return rc;
  return launch_layernorm(1, rows, cols, x, w, nullptr, mean, rstd, dy, nullptr, nullptr, nullptr, 0.f, dx, dw, db,
                          scratch, st);
}

int fh_layernorm_bwd_bwd(void* stream, int rows, int cols, const float* x, const float* w, const float* mean,
                         const float* rstd, const float* dy, const float* ddx, const float* ddw, const float* ddb,
                         float* gx, float* gw, float* gdy, float* scratch) {
  if (injected("fh_layernorm_bwd_bwd")) return FH_ERR_INJECTED;
  int rc = ln_check(rows, cols);
  if (rc != kOk) return rc;
  if (!all_aligned(x, w, dy, gx, gw, gdy, scratch) || !mean || !rstd) return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  if ((ddx && !aligned16(ddx)) || (ddw && !aligned16(ddw)) || (ddb && !aligned16(ddb)))
    return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = select_stream_device(st)) != kOk) return rc;
  return launch_layernorm(2, rows, cols, x, w, nullptr, mean, rstd, dy, ddx, ddw, ddb, 0.f, gx, gdy, gw, scratch, st);
}

int fh_gelu(void* stream, int mode, int dtype, long long n, const void* a, const void* dh, const void* c, void* out0,
            void* out1) {
  if (injected("fh_gelu")) return FH_ERR_INJECTED;
  g_last_error[0] = 0;
  if (mode < 0 || mode > 2 || (dtype != 0 && dtype != 1) || n < 0)
    return fail(FH_ERR_INVALID_ARGUMENT, "gelu: mode 0..2, dtype 0 (fp32) or 1 (bf16), n >= 0");
  if (!a || !out0 || (mode == 1 && !dh) || (mode == 2 && !c)) return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  if (n == 0) return FH_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = select_stream_device(st);
  if (rc != kOk) return rc;
  return launch_gelu(mode, dtype == 1, n, a, dh, c, out0, out1, st);
}

static int xent_check(int rows, int vocab, long long ld, int dtype, const void* z, const long long* t) {
  g_last_error[0] = 0;
  if (rows < 1 || vocab < 1 || ld < vocab || (dtype != 0 && dtype != 1) || !z || !t)
    return fail(FH_ERR_INVALID_ARGUMENT, "xent: rows >= 1, vocab >= 1, ld >= vocab, dtype 0 (fp32) or 1 (bf16)");
  return kOk;
}

int fh_xent_fwd(void* stream, int dtype, int rows, int vocab, long long ld, const void* z, const long long* t,
                float* lse, float* loss) {
  if (injected("fh_xent_fwd")) return FH_ERR_INJECTED;
  int rc = xent_check(rows, vocab, ld, dtype, z, t);
  if (rc != kOk) return rc;
  if (!lse || !loss) return fail(FH_ERR_INVALID_ARGUMENT, "xent: lse and loss are required");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = select_stream_device(st)) != kOk) return rc;
  return launch_xent(0, dtype == 1, rows, vocab, ld, z, t, lse, loss, nullptr, 0.f, nullptr, nullptr, nullptr, st);
}

int fh_xent_bwd(void* stream, int dtype, int rows, int vocab, long long ld, const void* z, const long long* t,
                const float* lse, const float* g, float s, void* dz) {
  if (injected("fh_xent_bwd")) return FH_ERR_INJECTED;
  int rc = xent_check(rows, vocab, ld, dtype, z, t);
  if (rc != kOk) return rc;
  if (!lse || !g || !dz) return fail(FH_ERR_INVALID_ARGUMENT, "xent: lse, g and dz are required");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = select_stream_device(st)) != kOk) return rc;
  return launch_xent(1, dtype == 1, rows, vocab, ld, z, t, const_cast<float*>(lse), nullptr, g, s, nullptr, dz,
                     nullptr, st);
}

int fh_xent_bwd_bwd(void* stream, int dtype, int rows, int vocab, long long ld, const void* z, const long long* t,
                    const float* lse, const float* g, float s, const void* u, void* gz, float* gg) {
  if (injected("fh_xent_bwd_bwd")) return FH_ERR_INJECTED;
  int rc = xent_check(rows, vocab, ld, dtype, z, t);
  if (rc != kOk) return rc;
  if (!lse || !g || !u || !gz || !gg) return fail(FH_ERR_INVALID_ARGUMENT, "xent: lse, g, u, gz and gg are required");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = select_stream_device(st)) != kOk) return rc;
  return launch_xent(2, dtype == 1, rows, vocab, ld, z, t, const_cast<float*>(lse), nullptr, g, s, u, gz, gg, st);
}

int fh_device_status(void* stream, int* code) {
  if (!code) return FH_ERR_INVALID_ARGUMENT;
  *code = 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = select_stream_device(st);
  if (rc != kOk) return rc;
  int* word = status_word();
  if (!word) return FH_ERR_NO_DEVICE;
  if (cudaStreamSynchronize(st) != cudaSuccess) return FH_ERR_LAUNCH;
  int host = 0;
  if (cudaMemcpy(&host, word, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return FH_ERR_LAUNCH;
  if (host != 0 && cudaMemset(word, 0, sizeof(int)) != cudaSuccess) return FH_ERR_LAUNCH;
  *code = host;
  return host == 0 ? FH_OK : FH_ERR_DEVICE;
}

}  // extern "C"

// ------------------------------------------------------------------------------------
// Allocation-free double backward
// ------------------------------------------------------------------------------------
//
// Some callers of this library cannot allocate device memory on the call path:
// an XLA FFI handler only receives the buffers XLA assigned before the
// computation started, and JAX reserves most of the GPU for its own pool up
// front, so a handler that calls cudaMalloc competes for (or fails to get) the
// remainder; inference servers that reserve their whole memory budget at start
// and never allocate per request are in the same position. They still own the
// inputs and outputs, but have nowhere to put the double backward's per-query
// scratch (D, dD, B). For them the scratch lives in a fixed file-scope device
// array instead.

namespace fh {
namespace {

// Capacity of the static scratch in query rows (batch * heads * seq_q).
constexpr long long kNoAllocMaxRows = 1LL << 19;

// D | dD | B for up to kNoAllocMaxRows query rows: 3 x 2 MiB = 6 MiB, held by
// every GPU on which this library's module is loaded until the process exits.
static __device__ __align__(256) float g_noalloc_scratch[3 * kNoAllocMaxRows];

float* g_noalloc_ptr[kMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device. Host code cannot
// use the array's name as a device address (it names a host-side shadow), so
// the address is looked up once per device, with that device current.
int noalloc_scratch(float** out) {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return fail(kNoDevice, "no current CUDA device");
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      char msg[200];
      std::snprintf(msg, sizeof(msg), "cudaGetSymbolAddress of the static scratch failed: %s",
                    cudaGetErrorString(e));
      return fail(kLaunchFailed, msg);
    }
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return kOk;
}

}  // namespace
}  // namespace fh

extern "C" int fh_attn_bwdbwd_noalloc(void* stream, const fh_attn_dims* dims, const void* q, const void* k,
                                      const void* v, const void* o, const void* dO, const void* ddq,
                                      const void* ddk, const void* ddv, const float* lse, void* dq2, void* ddo,
                                      void* dk2, void* dv2, float scale, int causal, int* device_status) {
  if (injected("fh_attn_bwdbwd_noalloc")) return FH_ERR_INJECTED;
  AttnShape s;
  int rc = validate(dims, &s, scale, causal);
  if (rc != kOk) return rc;
  const long long rows = static_cast<long long>(s.cu_q ? 1 : s.B) * s.H * s.total_q;
  if (rows > kNoAllocMaxRows) {
    char msg[240];
    std::snprintf(msg, sizeof(msg),
                  "batch*heads*seq_q = %lld exceeds the %lld query rows of fh_attn_bwdbwd_noalloc's static "
                  "scratch; use fh_attn_bwdbwd with caller-provided scratch",
                  rows, kNoAllocMaxRows);
    return fail(FH_ERR_INVALID_ARGUMENT, msg);
  }
  if (!all_aligned(q, k, v, o, dO, ddq, ddk, ddv, dq2, ddo, dk2, dv2) || !lse)
    return fail(FH_ERR_INVALID_ARGUMENT, kAlignMsg);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((rc = select_stream_device(st)) != kOk) return rc;
  float* scratch = nullptr;
  if ((rc = noalloc_scratch(&scratch)) != kOk) return rc;
  // Two launches, as fh_attn_bwdbwd_o: the query-tiled pass computes D from o
  // for its rows and writes D, dD and B; the key-tiled pass reads them. Every
  // element the key pass reads is written earlier in the same call, so nothing
  // needs clearing and a previous call's leftovers are never read.
  float* delta = scratch;
  float* dd = scratch + kNoAllocMaxRows;
  float* bv = scratch + 2 * kNoAllocMaxRows;
  return launch_bwdbwd(
      s, dims->head_dim,
      BwdBwdPtrs{q, k, v, dO, ddq, ddk, ddv, lse, nullptr, dq2, ddo, dk2, dv2, dd, bv, o, delta},
      kPassQuery | kPassKey, device_status, st);
}
