// Python glue for the per-token decode entry points.
//
// A decode step is a few microseconds of GPU time, so building nine ctypes descriptors
// in Python (about 4 us each) would dominate it. This module fills the bd_tensor
// descriptors from torch tensors in C++ and calls the C ABI of libbdecode.so directly,
// on the tensors' current CUDA stream. It links nothing of its own: the bd_* symbols
// resolve against libbdecode.so, which the Python package loads with RTLD_GLOBAL
// before importing this module. Every function returns the C ABI status code; the
// caller maps non-zero codes to exceptions (bd_last_error holds the message).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <cmath>
#include <stdexcept>
#include <tuple>

#include "bdecode.h"

namespace {

bd_tensor desc(const at::Tensor& t, int device) {
  if (!t.is_cuda()) throw std::invalid_argument("bytes_b200: expected CUDA tensors (there is no CPU path)");
  if (t.get_device() != device) throw std::invalid_argument("bytes_b200: tensors are on different devices");
  if (t.dim() > 6) throw std::invalid_argument("bytes_b200: too many dimensions");
  bd_tensor d{};
  switch (t.scalar_type()) {
    case at::kFloat: d.dtype = BD_F32; break;
    case at::kHalf: d.dtype = BD_F16; break;
    case at::kBFloat16: d.dtype = BD_BF16; break;
    case at::kFloat8_e4m3fn: d.dtype = BD_F8E4M3; break;
    case at::kByte: d.dtype = BD_U8; break;
    case at::kChar: d.dtype = BD_I8; break;
    case at::kInt: d.dtype = BD_I32; break;
    case at::kLong: d.dtype = BD_I64; break;
    default: throw std::invalid_argument("bytes_b200: unsupported dtype");
  }
  d.data = t.numel() > 0 ? t.data_ptr() : nullptr;
  d.ndim = int(t.dim());
  for (int i = 0; i < d.ndim; ++i) {
    d.shape[i] = t.size(i);
    d.stride[i] = t.stride(i);
  }
  return d;
}

at::Tensor workspace(size_t bytes, const at::Tensor& like) {
  return at::empty({int64_t(bytes > 0 ? bytes : 1)}, like.options().dtype(at::kByte));
}

// bd_kivi_decode_attn_stages on the current stream, workspace from the caching allocator.
int64_t kivi_decode(const at::Tensor& Q3, const at::Tensor& Kq, const at::Tensor& Ks, const at::Tensor& Km,
                    const at::Tensor& Kr, const at::Tensor& Vq, const at::Tensor& Vs, const at::Tensor& Vm,
                    const at::Tensor& Vr, int64_t bits, int64_t group_size, double scaling, const at::Tensor& out,
                    int64_t stages) {
  const int dev = Q3.get_device();
  const bd_tensor dq = desc(Q3, dev), dkq = desc(Kq, dev), dks = desc(Ks, dev), dkm = desc(Km, dev),
                  dkr = desc(Kr, dev), dvq = desc(Vq, dev), dvs = desc(Vs, dev), dvm = desc(Vm, dev),
                  dvr = desc(Vr, dev), dout = desc(out, dev);
  const c10::cuda::CUDAGuard guard(Q3.device());
  const size_t nws = bd_kivi_decode_attn_workspace(&dq, &dkq, &dkr, int(bits));
  const at::Tensor ws = workspace(nws, Q3);
  return bd_kivi_decode_attn_stages(&dq, &dkq, &dks, &dkm, &dkr, &dvq, &dvs, &dvm, &dvr, int(bits), int(group_size),
                                    float(scaling), &dout, ws.data_ptr(), nws, int(stages),
                                    at::cuda::getCurrentCUDAStream(dev).stream());
}

// bd_decode_attn (bf16 / fp8 dense cache) on the current stream.
int64_t decode_attn(const at::Tensor& q3, const at::Tensor& k, const at::Tensor& v, const at::Tensor& out,
                    double scaling) {
  const int dev = q3.get_device();
  const bd_tensor dq = desc(q3, dev), dk = desc(k, dev), dv = desc(v, dev), dout = desc(out, dev);
  const c10::cuda::CUDAGuard guard(q3.device());
  const size_t nws = bd_decode_attn_workspace(&dq, &dk);
  const at::Tensor ws = workspace(nws, q3);
  return bd_decode_attn(&dq, &dk, &dv, &dout, float(scaling), ws.data_ptr(), nws,
                        at::cuda::getCurrentCUDAStream(dev).stream());
}

// Descriptor of a [B, H, 1, D] tensor viewed as [B, H, D] (the reference's decode query and
// output layout), without creating the view.
bd_tensor desc_drop2(const at::Tensor& t, int device) {
  bd_tensor d = desc(t, device);
  d.ndim = 3;
  d.shape[2] = t.size(3);
  d.stride[2] = t.stride(3);
  return d;
}

// kivi_decode_attn(Q [B,Hq,1,D], packed caches, bits, group_size) -> (status, out [B,Hq,1,D]).
// The whole drop-in call in C++: output allocation, descriptors, workspace and the two
// launches. A non-zero status leaves the caller to take its general path (re-laid-out
// copies, or the error).
std::tuple<int64_t, at::Tensor> kivi_decode_attn(const at::Tensor& Q, const at::Tensor& Kq, const at::Tensor& Ks,
                                                 const at::Tensor& Km, const at::Tensor& Kr, const at::Tensor& Vq,
                                                 const at::Tensor& Vs, const at::Tensor& Vm, const at::Tensor& Vr,
                                                 int64_t bits, int64_t group_size) {
  if (Q.dim() != 4 || Q.size(2) != 1 || Kr.scalar_type() != at::kBFloat16 || Vr.scalar_type() != at::kBFloat16 ||
      Ks.scalar_type() != at::kHalf || Km.scalar_type() != at::kHalf || Vs.scalar_type() != at::kHalf ||
      Vm.scalar_type() != at::kHalf || (Q.scalar_type() != at::kBFloat16 && Kr.size(2) > 0))
    return {BD_ERR_DTYPE, at::Tensor()};
  const int dev = Q.get_device();
  at::Tensor out = at::empty({Q.size(0), Q.size(1), 1, Q.size(3)}, Q.options());
  const bd_tensor dq = desc_drop2(Q, dev), dkq = desc(Kq, dev), dks = desc(Ks, dev), dkm = desc(Km, dev),
                  dkr = desc(Kr, dev), dvq = desc(Vq, dev), dvs = desc(Vs, dev), dvm = desc(Vm, dev),
                  dvr = desc(Vr, dev), dout = desc_drop2(out, dev);
  const c10::cuda::CUDAGuard guard(Q.device());
  const size_t nws = bd_kivi_decode_attn_workspace(&dq, &dkq, &dkr, int(bits));
  const at::Tensor ws = workspace(nws, Q);
  const int rc = bd_kivi_decode_attn_stages(&dq, &dkq, &dks, &dkm, &dkr, &dvq, &dvs, &dvm, &dvr, int(bits),
                                            int(group_size), float(1.0 / std::sqrt(double(Q.size(3)))), &dout,
                                            ws.data_ptr(), nws, 7, at::cuda::getCurrentCUDAStream(dev).stream());
  return {rc, out};
}

// decode_attn_bf16 / decode_attn_fp8 (no scale) -> (status, out [B,Hq,1,D] in q's dtype).
std::tuple<int64_t, at::Tensor> decode_attn_nq(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v) {
  if (q.dim() != 4 || q.size(2) != 1) return {BD_ERR_SHAPE, at::Tensor()};
  if (k.scalar_type() == at::kBFloat16 && q.scalar_type() != at::kBFloat16) return {BD_ERR_DTYPE, at::Tensor()};
  const int dev = q.get_device();
  at::Tensor out = at::empty({q.size(0), q.size(1), 1, q.size(3)}, q.options());
  const bd_tensor dq = desc_drop2(q, dev), dk = desc(k, dev), dv = desc(v, dev), dout = desc_drop2(out, dev);
  const c10::cuda::CUDAGuard guard(q.device());
  const size_t nws = bd_decode_attn_workspace(&dq, &dk);
  const at::Tensor ws = workspace(nws, q);
  const int rc = bd_decode_attn(&dq, &dk, &dv, &dout, 1.0f, ws.data_ptr(), nws,
                                at::cuda::getCurrentCUDAStream(dev).stream());
  return {rc, out};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "C++ descriptor glue for the bytes_b200 decode entry points";
  m.def("kivi_decode", &kivi_decode, "bd_kivi_decode_attn_stages on the current CUDA stream");
  m.def("decode_attn", &decode_attn, "bd_decode_attn on the current CUDA stream");
  m.def("kivi_decode_attn", &kivi_decode_attn, "the drop-in KIVI decode step: (status, out [B,Hq,1,D])");
  m.def("decode_attn_nq", &decode_attn_nq, "decode_attn_bf16 / decode_attn_fp8: (status, out [B,Hq,1,D])");
}
