// XLA FFI handlers around the C ABI, for a JAX binding of this library.
//
// NOT BUILT ON THIS IMAGE: it needs jaxlib's FFI headers (`jax.ffi.include_dir()`),
// and jax/jaxlib are not installed here. `flash_hog_b200.build.build_xla_ffi()`
// compiles it into `libfh_xla_ffi.so` wherever those headers exist and skips it
// otherwise.
//
// The handlers replace the reference's native plugin and its cuDNN calls at their
// call sites:
//   * FhBwdBwd   -- `TkBwdBwd` (flash_hog/csrc/tk_bwdbwd/ffi.cu:79-98): the same nine
//                   buffers Q, K, V, dO, ddQ, ddK, ddV, L, D, the attribute `scale`, and
//                   the same six results dQ2, ddO, dK2, dV2 and the scratch dD, B; plus
//                   the attributes `causal` (0, 1 top-left, 2 bottom-right) and `window`;
//   * FhBwdBwdO  -- the whole `flash_bwdbwd` of flash_hog/jax/_tk_gpu.py:83-103: O in
//                   place of D (computed inside the query-tiled pass), D returned as a
//                   seventh (scratch) result;
//   * FhAttnFwd  -- the cuDNN forward with residuals (flash_hog/jax/_attention_impl.py:224-239):
//                   results O and the natural-log log-sum-exp L;
//   * FhAttnBwd  -- the cuDNN backward (flash_hog/jax/_attention_impl.py:242-261):
//                   results dQ, dK, dV and the scratch D.
// Register each with jax.ffi.register_ffi_target(name, jax.ffi.pycapsule(lib.<Handler>),
// platform="CUDA"), as flash_hog/jax/_tk_gpu.py:57 does for TkBwdBwd.
//
// Layout: query-side tensors are (B, Tq, N, H) and key-side (B, Tk, Nkv, H), both
// contiguous -- the reference API's BTNH, so no transpose is needed (the kernels
// build their TMA descriptors from the strides). With the attribute `bhtd` = 1 the
// buffers are (B, N, T, H) instead, TkBwdBwd's layout (ffi.cu:7-10). Statistics
// vectors (L, D, dD, B) are (B, N, Tq) fp32. Nkv < N is grouped-query attention.
//
// Errors: argument problems map to ffi::Error::InvalidArgument, launch or device
// failures to ffi::Error::Internal, each with fh_last_error()'s message -- the
// reference handler's two error kinds (ffi.cu:36-39, 74-76). Nothing is allocated:
// XLA owns every buffer, scratch included, as it does for TkBwdBwd. The one-time
// per-device set-up inside the library is mutex-guarded (ffi.cu:41-46 uses an
// unsynchronised static flag).

#include <cstdint>
#include <string>

#include "flash_hog_b200.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

// fh_attn_dims of a query-side and a key-side buffer (rank 4, contiguous).
bool make_dims(const ffi::AnyBuffer& q, const ffi::AnyBuffer& k, bool bhtd, int32_t window, fh_attn_dims* d,
               std::string* why) {
  *d = fh_attn_dims{};  // dense batch: no cu_seqlens
  auto qd = q.dimensions();
  auto kd = k.dimensions();
  if (qd.size() != 4 || kd.size() != 4) {
    *why = "expected rank-4 query and key tensors";
    return false;
  }
  // (B, T, N, H) or, with bhtd, (B, N, T, H).
  const int64_t qt = bhtd ? qd[2] : qd[1], qn = bhtd ? qd[1] : qd[2];
  const int64_t kt = bhtd ? kd[2] : kd[1], kn = bhtd ? kd[1] : kd[2];
  if (qd[0] != kd[0] || qd[3] != kd[3]) {
    *why = "query and key tensors disagree on batch or head_dim";
    return false;
  }
  d->batch = static_cast<int32_t>(qd[0]);
  d->heads = static_cast<int32_t>(qn);
  d->seq_q = static_cast<int32_t>(qt);
  d->seq_k = static_cast<int32_t>(kt);
  d->head_dim = static_cast<int32_t>(qd[3]);
  const int64_t h = qd[3];
  d->q = bhtd ? fh_strides{qn * qt * h, h, qt * h} : fh_strides{qt * qn * h, qn * h, h};
  d->k = bhtd ? fh_strides{kn * kt * h, h, kt * h} : fh_strides{kt * kn * h, kn * h, h};
  d->kv_heads = static_cast<int32_t>(kn);
  d->window = window;
  return true;
}

ffi::Error status_to_error(int rc) {
  if (rc == FH_OK) return ffi::Error::Success();
  const std::string msg = std::string(fh_status_string(rc)) + ": " + fh_last_error();
  if (rc == FH_ERR_INVALID_ARGUMENT || rc == FH_ERR_UNSUPPORTED) return ffi::Error::InvalidArgument(msg);
  return ffi::Error::Internal(msg);
}

bool all_bf16(std::initializer_list<const ffi::AnyBuffer*> xs) {
  for (const ffi::AnyBuffer* x : xs)
    if (x->element_type() != ffi::DataType::BF16) return false;
  return true;
}

template <typename T>
T* out(ffi::Result<ffi::AnyBuffer>& r) {
  return static_cast<T*>(r->untyped_data());
}

template <typename T>
const T* in(const ffi::AnyBuffer& x) {
  return static_cast<const T*>(x.untyped_data());
}

ffi::Error FhAttnFwdImpl(cudaStream_t stream, ffi::AnyBuffer q, ffi::AnyBuffer k, ffi::AnyBuffer v, float scale,
                         int32_t causal, int32_t window, int32_t bhtd, ffi::Result<ffi::AnyBuffer> o,
                         ffi::Result<ffi::AnyBuffer> lse) {
  fh_attn_dims d;
  std::string why;
  if (!make_dims(q, k, bhtd != 0, window, &d, &why)) return ffi::Error::InvalidArgument(why);
  if (!all_bf16({&q, &k, &v})) return ffi::Error::InvalidArgument("q, k, v must be bf16");
  return status_to_error(fh_attn_fwd(stream, &d, q.untyped_data(), k.untyped_data(), v.untyped_data(),
                                     o->untyped_data(), out<float>(lse), scale, causal));
}

ffi::Error FhAttnBwdImpl(cudaStream_t stream, ffi::AnyBuffer q, ffi::AnyBuffer k, ffi::AnyBuffer v, ffi::AnyBuffer o,
                         ffi::AnyBuffer dO, ffi::AnyBuffer lse, float scale, int32_t causal, int32_t window,
                         int32_t bhtd, ffi::Result<ffi::AnyBuffer> dq, ffi::Result<ffi::AnyBuffer> dk,
                         ffi::Result<ffi::AnyBuffer> dv, ffi::Result<ffi::AnyBuffer> delta) {
  fh_attn_dims d;
  std::string why;
  if (!make_dims(q, k, bhtd != 0, window, &d, &why)) return ffi::Error::InvalidArgument(why);
  if (!all_bf16({&q, &k, &v, &o, &dO})) return ffi::Error::InvalidArgument("q, k, v, o, dO must be bf16");
  return status_to_error(fh_attn_bwd(stream, &d, q.untyped_data(), k.untyped_data(), v.untyped_data(),
                                     o.untyped_data(), dO.untyped_data(), in<float>(lse), dq->untyped_data(),
                                     dk->untyped_data(), dv->untyped_data(), out<float>(delta), scale, causal));
}

ffi::Error FhBwdBwdImpl(cudaStream_t stream, ffi::AnyBuffer q, ffi::AnyBuffer k, ffi::AnyBuffer v, ffi::AnyBuffer dO,
                        ffi::AnyBuffer ddq, ffi::AnyBuffer ddk, ffi::AnyBuffer ddv, ffi::AnyBuffer lse,
                        ffi::AnyBuffer delta, float scale, int32_t causal, int32_t window, int32_t bhtd,
                        ffi::Result<ffi::AnyBuffer> dq2, ffi::Result<ffi::AnyBuffer> ddo,
                        ffi::Result<ffi::AnyBuffer> dk2, ffi::Result<ffi::AnyBuffer> dv2,
                        ffi::Result<ffi::AnyBuffer> dd, ffi::Result<ffi::AnyBuffer> b) {
  fh_attn_dims d;
  std::string why;
  if (!make_dims(q, k, bhtd != 0, window, &d, &why)) return ffi::Error::InvalidArgument(why);
  if (!all_bf16({&q, &k, &v, &dO, &ddq, &ddk, &ddv})) return ffi::Error::InvalidArgument("tensors must be bf16");
  return status_to_error(fh_attn_bwdbwd(stream, &d, q.untyped_data(), k.untyped_data(), v.untyped_data(),
                                        dO.untyped_data(), ddq.untyped_data(), ddk.untyped_data(), ddv.untyped_data(),
                                        in<float>(lse), in<float>(delta), dq2->untyped_data(), ddo->untyped_data(),
                                        dk2->untyped_data(), dv2->untyped_data(), out<float>(dd), out<float>(b),
                                        scale, causal));
}

ffi::Error FhBwdBwdOImpl(cudaStream_t stream, ffi::AnyBuffer q, ffi::AnyBuffer k, ffi::AnyBuffer v, ffi::AnyBuffer o,
                         ffi::AnyBuffer dO, ffi::AnyBuffer ddq, ffi::AnyBuffer ddk, ffi::AnyBuffer ddv,
                         ffi::AnyBuffer lse, float scale, int32_t causal, int32_t window, int32_t bhtd,
                         ffi::Result<ffi::AnyBuffer> dq2, ffi::Result<ffi::AnyBuffer> ddo,
                         ffi::Result<ffi::AnyBuffer> dk2, ffi::Result<ffi::AnyBuffer> dv2,
                         ffi::Result<ffi::AnyBuffer> delta, ffi::Result<ffi::AnyBuffer> dd,
                         ffi::Result<ffi::AnyBuffer> b) {
  fh_attn_dims d;
  std::string why;
  if (!make_dims(q, k, bhtd != 0, window, &d, &why)) return ffi::Error::InvalidArgument(why);
  if (!all_bf16({&q, &k, &v, &o, &dO, &ddq, &ddk, &ddv})) return ffi::Error::InvalidArgument("tensors must be bf16");
  return status_to_error(fh_attn_bwdbwd_o(stream, &d, q.untyped_data(), k.untyped_data(), v.untyped_data(),
                                          o.untyped_data(), dO.untyped_data(), ddq.untyped_data(), ddk.untyped_data(),
                                          ddv.untyped_data(), in<float>(lse), dq2->untyped_data(), ddo->untyped_data(),
                                          dk2->untyped_data(), dv2->untyped_data(), out<float>(delta),
                                          out<float>(dd), out<float>(b), scale, causal, FH_PASS_QUERY | FH_PASS_KEY));
}

}  // namespace

XLA_FFI_DEFINE_HANDLER_SYMBOL(FhAttnFwd, FhAttnFwdImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()  // Q
                                  .Arg<ffi::AnyBuffer>()  // K
                                  .Arg<ffi::AnyBuffer>()  // V
                                  .Attr<float>("scale")
                                  .Attr<int32_t>("causal")
                                  .Attr<int32_t>("window")
                                  .Attr<int32_t>("bhtd")
                                  .Ret<ffi::AnyBuffer>()    // O
                                  .Ret<ffi::AnyBuffer>());  // L

XLA_FFI_DEFINE_HANDLER_SYMBOL(FhAttnBwd, FhAttnBwdImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()  // Q
                                  .Arg<ffi::AnyBuffer>()  // K
                                  .Arg<ffi::AnyBuffer>()  // V
                                  .Arg<ffi::AnyBuffer>()  // O
                                  .Arg<ffi::AnyBuffer>()  // dO
                                  .Arg<ffi::AnyBuffer>()  // L
                                  .Attr<float>("scale")
                                  .Attr<int32_t>("causal")
                                  .Attr<int32_t>("window")
                                  .Attr<int32_t>("bhtd")
                                  .Ret<ffi::AnyBuffer>()    // dQ
                                  .Ret<ffi::AnyBuffer>()    // dK
                                  .Ret<ffi::AnyBuffer>()    // dV
                                  .Ret<ffi::AnyBuffer>());  // D (scratch)

XLA_FFI_DEFINE_HANDLER_SYMBOL(FhBwdBwd, FhBwdBwdImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()  // Q
                                  .Arg<ffi::AnyBuffer>()  // K
                                  .Arg<ffi::AnyBuffer>()  // V
                                  .Arg<ffi::AnyBuffer>()  // dO
                                  .Arg<ffi::AnyBuffer>()  // ddQ
                                  .Arg<ffi::AnyBuffer>()  // ddK
                                  .Arg<ffi::AnyBuffer>()  // ddV
                                  .Arg<ffi::AnyBuffer>()  // L
                                  .Arg<ffi::AnyBuffer>()  // D
                                  .Attr<float>("scale")
                                  .Attr<int32_t>("causal")
                                  .Attr<int32_t>("window")
                                  .Attr<int32_t>("bhtd")
                                  .Ret<ffi::AnyBuffer>()    // dQ2
                                  .Ret<ffi::AnyBuffer>()    // ddO
                                  .Ret<ffi::AnyBuffer>()    // dK2
                                  .Ret<ffi::AnyBuffer>()    // dV2
                                  .Ret<ffi::AnyBuffer>()    // dD (scratch)
                                  .Ret<ffi::AnyBuffer>());  // B (scratch)

XLA_FFI_DEFINE_HANDLER_SYMBOL(FhBwdBwdO, FhBwdBwdOImpl,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::AnyBuffer>()  // Q
                                  .Arg<ffi::AnyBuffer>()  // K
                                  .Arg<ffi::AnyBuffer>()  // V
                                  .Arg<ffi::AnyBuffer>()  // O
                                  .Arg<ffi::AnyBuffer>()  // dO
                                  .Arg<ffi::AnyBuffer>()  // ddQ
                                  .Arg<ffi::AnyBuffer>()  // ddK
                                  .Arg<ffi::AnyBuffer>()  // ddV
                                  .Arg<ffi::AnyBuffer>()  // L
                                  .Attr<float>("scale")
                                  .Attr<int32_t>("causal")
                                  .Attr<int32_t>("window")
                                  .Attr<int32_t>("bhtd")
                                  .Ret<ffi::AnyBuffer>()    // dQ2
                                  .Ret<ffi::AnyBuffer>()    // ddO
                                  .Ret<ffi::AnyBuffer>()    // dK2
                                  .Ret<ffi::AnyBuffer>()    // dV2
                                  .Ret<ffi::AnyBuffer>()    // D (scratch)
                                  .Ret<ffi::AnyBuffer>()    // dD (scratch)
                                  .Ret<ffi::AnyBuffer>());  // B (scratch)
